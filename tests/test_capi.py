"""The per-op C ABI (include/vc4b200.h) as the reference's layer loop drives it.

tests/capi/forward_gpu_hidden.cpp restates Session::forward_gpu_hidden
(engine/src/session.cpp:1459-1584) call for call against the header.  It is
compiled here with g++ against the header and the built library (no CUDA
headers: the ABI is plain C), and on a GPU it must give vc4_step's logits and
greedy tokens bit for bit.
"""
import os
import subprocess

import numpy as np
import pytest

import vc4b200
from conftest import ROOT, full_model_path
from vc4b200 import mmcf_writer, synth

SRC = os.path.join(ROOT, "tests", "capi", "forward_gpu_hidden.cpp")
LIBDIR = os.path.dirname(vc4b200.engine.LIB_PATH)


def build_driver(out_dir: str) -> str:
    exe = os.path.join(out_dir, "forward_gpu_hidden")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I" + os.path.join(ROOT, "include"), SRC,
                    "-L" + LIBDIR, "-lvc4b200", "-Wl,-rpath," + LIBDIR, "-o", exe], check=True)
    return exe


def test_driver_compiles_and_links(tmp_path):
    assert os.access(build_driver(str(tmp_path)), os.X_OK)


def _fnv(lg):
    h = 1469598103934665603
    for v in np.rint(lg * 256.0).astype(np.int64):
        q = int(v) & 0xFFFFFFFF
        for b in range(4):
            h = ((h ^ ((q >> (8 * b)) & 0xFF)) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return "%016x" % h


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["tiny_q8", "tiny_moe_q4", "tiny_t3", "c1", "c2"])
def test_layer_loop_over_the_per_op_abi_equals_step(tmp_path, key):
    cfg = dict(synth.TINY_CONFIGS, **synth.CONFIGS)[key]
    if key in synth.CONFIGS:
        path = full_model_path(key)
    else:
        path = str(tmp_path / "m.mmcf")
        mmcf_writer.write_config(cfg, path)
    prompt = synth.prompt_tokens(cfg)[:6]
    steps = 4
    exe = build_driver(str(tmp_path))
    r = subprocess.run([exe, path, str(cfg.seq), str(cfg.kv_bits), str(len(prompt)), str(steps)] +
                       [str(t) for t in prompt], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = [l.split() for l in r.stdout.strip().splitlines()]
    assert len(lines) == len(prompt) + steps
    gpu = vc4b200.GPU(0)
    model = vc4b200.Model(gpu, path)
    sess = vc4b200.Session(model, slots=1, seq=cfg.seq, kv={16: "q16", 8: "q8"}[cfg.kv_bits])
    tok = prompt[0]
    for pos, (p, nxt, dig) in enumerate(lines):
        lg = sess.step(tok, pos)
        assert int(p) == pos
        assert _fnv(lg) == dig, "%s position %d: per-op logits differ from vc4_step" % (key, pos)
        assert int(nxt) == int(np.argmax(lg))
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else int(nxt)
