"""CUDA path vs the CPU oracle on the tiny parity models (every code path of
the five benchmark configurations at a size the oracle runs in seconds).

Tolerance (the north star's): max |dlogit| <= 1e-2 with greedy agreement.  The
canonical arithmetic is shared, so the expected difference is zero; the KV
bytes are compared bit for bit.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
import vc4b200
from vc4b200 import synth

TOL = 1e-2
KV = {16: "q16", 8: "q8"}


@pytest.fixture(scope="module")
def gpu():
    return vc4b200.GPU(0)


def _teacher_forced(sess, om_sess, toks):
    """Logits at every position for a fixed token sequence, engine and oracle."""
    a, b = [], []
    for pos, t in enumerate(toks):
        a.append(sess.step(t, pos))
        b.append(om_sess.step(t, pos))
    return np.stack(a), np.stack(b)


@pytest.mark.gpu
@pytest.mark.parametrize("key", list(synth.TINY_CONFIGS))
def test_decode_matches_oracle(gpu, tiny_paths, key):
    cfg = synth.TINY_CONFIGS[key]
    path = tiny_paths[key]
    prompt = synth.prompt_tokens(cfg)
    om = oracle.Model(path)
    # 1. teacher forced over the random prompt: logits at every position
    model = vc4b200.Model(gpu, path)
    sess = vc4b200.Session(model, slots=1, seq=cfg.seq, kv=KV[cfg.kv_bits])
    osess = oracle.Session(om, cfg.kv_bits)
    got, ref = _teacher_forced(sess, osess, prompt)
    d = np.abs(got - ref)
    assert d.max() <= TOL, "max |dlogit| %g at %s" % (d.max(), np.unravel_index(d.argmax(), d.shape))
    assert (got.argmax(1) == ref.argmax(1)).all()
    exact = int((d == 0).all(axis=1).sum())
    print("%s: %d/%d positions bit-exact" % (key, exact, len(prompt)))
    # 2. the packed KV rows are the oracle's bytes
    for layer in range(om.info.layers):
        assert sess.kv_rows(layer, len(prompt)) == osess.kv_rows(layer, len(prompt)), "KV bytes differ at layer %d" % layer
    # 3. free-running greedy decode through the prefill path
    sess2 = vc4b200.Session(model, slots=1, seq=cfg.seq, kv=KV[cfg.kv_bits])
    toks, logs = vc4b200.generate(sess2, prompt, cfg.steps)
    rtoks, rlogs, _ = oracle.generate(om, cfg.kv_bits, prompt, cfg.steps)
    assert toks == rtoks
    assert np.abs(logs - rlogs).max() <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["tiny_q8", "tiny_q4", "tiny_t3", "tiny_moe_q4"])
def test_matvec_s_matches_oracle(gpu, tiny_paths, key):
    """GPU::matvec_s through the device layout equals the oracle's exact
    integers for every matrix kind (the dequantisation is bit-exact)."""
    path = tiny_paths[key]
    om = oracle.Model(path)
    model = vc4b200.Model(gpu, path)
    info = model.info
    rng = np.random.default_rng(5)
    E = info.experts
    cases = [("qkv", 0, 0), ("wo", 1, 0), ("w1", 0, 1 if E else 0), ("w3", 1, 2 if E else 0), ("logits", 0, 0)]
    if E:
        cases.append(("router", 1, 0))
    for name, layer, expert in cases:
        which = vc4b200.MATS[name]
        rows, cols, _, _ = om.mat_shape(which, layer if name != "logits" else 0, expert)
        x = (rng.integers(-2000, 2000, size=cols) / 256.0).astype(np.float32)
        got = model.matvec_s(name, x, layer=layer, expert=expert)
        xq = np.empty(cols, np.int16)
        k = oracle.lib().orc_scale_input(x.ctypes.data_as(oracle.C.c_void_p), cols, xq.ctypes.data_as(oracle.C.c_void_p))
        if name == "logits":
            ref = np.concatenate([om.matvec(6, t, 0, xq) for t in range(om.info.n_logit_tiles)])
        else:
            ref = om.matvec(which, layer, expert, xq)
        ref = (ref.astype(np.float32) / 256.0) * np.float32(2.0 ** -k)
        assert np.array_equal(got, ref), "%s: %d rows differ" % (name, int((got != ref).sum()))


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["tiny_q8", "tiny_moe_q4", "tiny_t3"])
@pytest.mark.parametrize("n", [6, 10, 33, 64, 300])
def test_batched_equals_serial(gpu, tiny_paths, key, n):
    """Several sequences in one pass give each sequence's serial result: 6
    runs the one-sequence kernels four inputs at a time, 10 the many-sequence
    (prep + matmat) kernels, 33 their tensor-core (tcgen05) form for q8, 64
    also the one-CTA-per-head attention for many sequences, 300 more
    16-sequence units than SMs (tensor-core ranges run in several rounds
    under the balanced split)."""
    cfg = synth.TINY_CONFIGS[key]
    model = vc4b200.Model(gpu, tiny_paths[key])
    prompts = [synth.prompt_tokens(cfg, i)[:10] for i in range(n)]
    bs = vc4b200.Session(model, slots=n, seq=cfg.seq, kv=KV[cfg.kv_bits])
    logs_b = []
    for pos in range(10):
        nxt, lg = bs.step_batch(list(range(n)), [p[pos] for p in prompts], [pos] * n, want_logits=True)
        logs_b.append(lg)
    for i in range(n):
        ss = vc4b200.Session(model, slots=1, seq=cfg.seq, kv=KV[cfg.kv_bits])
        for pos in range(10):
            lg = ss.step(prompts[i][pos], pos)
            assert np.array_equal(lg, logs_b[pos][i]), "sequence %d position %d" % (i, pos)


@pytest.mark.gpu
@pytest.mark.parametrize("split", ["aligned", "balanced"])
def test_tensor_core_splits(split):
    """Both work splits of the tensor-core matmats give the serial results:
    groups of sequences inside a tile, one CTA each, and equal ranges of
    16-sequence units per SM run in rounds.  A process fixes its split once
    (VC4_TC_SPLIT), so the batched tests run again in a child process."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, VC4_TC_SPLIT=split)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.abspath(__file__) + "::test_batched_equals_serial", "-k", "tiny_q8 or tiny_t3"],
                       env=env, cwd=root, capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-2000:])


@pytest.mark.gpu
def test_prefix_cache_roundtrip(gpu, tiny_paths, tmp_path):
    """MMKV1 save, restore into another session, continue: identical decode."""
    cfg = synth.TINY_CONFIGS["tiny_q8"]
    model = vc4b200.Model(gpu, tiny_paths["tiny_q8"])
    prompt = synth.prompt_tokens(cfg)
    a = vc4b200.Session(model, slots=1, seq=cfg.seq, kv="q16")
    a.prefill(prompt, 0, want_logits=False)
    path = str(tmp_path / "p.mmkv")
    a.save_prefix_cache(path, prompt)
    b = vc4b200.Session(model, slots=2, seq=cfg.seq, kv="q16")
    assert b.load_prefix_cache(path, slot=1) == list(prompt)
    for layer in range(model.info.layers):
        assert b.kv_rows(layer, len(prompt), slot=1) == a.kv_rows(layer, len(prompt))
    la = a.step(7, len(prompt))
    lb = b.step(7, len(prompt), slot=1)
    assert np.array_equal(la, lb)


@pytest.mark.gpu
@pytest.mark.parametrize("wtype,rows,cols", [(0, 4100, 1024), (1, 4100, 2048), (2, 4100, 4096), (0, 16384, 2048)])
def test_streaming_matvec_equals_block_kernel(gpu, wtype, rows, cols):
    """matvec_s streams large matrices with persistent warps (lane = row,
    whole 32-row blocks per warp); on the same synthetic matrix its output
    equals the one-CTA-per-block kernel's (checked against the oracle above)
    bit for bit, ragged last block included."""
    import ctypes as C
    digests = []
    for path in (1, 2):
        ms, byt, dig = C.c_double(), C.c_double(), C.c_uint64()
        rc = vc4b200.lib().vc4_matvec_probe(0, wtype, rows, cols, path, 1, 0, C.byref(ms), C.byref(byt), C.byref(dig))
        assert rc == 0, vc4b200.lib().vc4_last_error().decode()
        digests.append(dig.value)
    assert digests[0] == digests[1]
