"""Pin the CPU oracle and the MMCF writer to the reference itself (no GPU).

* The writer reproduces the reference packer's bytes (sha256 recorded by
  tests/golden/make_golden.py, which ran engine/tools/mmcf_pack.py unchanged)
  for the tiny parity models and the five benchmark configurations.
* The oracle's decode of every tensor equals what the reference's own loader
  (engine/src/model.cpp, built into oracle/_ref) decoded from the same file.
* The q16 quantiser reproduces the x_pack byte vectors of
  engine/tests/test_xformat.cpp (I16_1, I16_2: the activation format).
"""
import hashlib
import struct

import numpy as np
import pytest

import oracle
from vc4b200 import mmcf_writer, synth

FULL = ["c0", "c0r", "c1", "c2", "c3", "c4"]


def _container(key):
    cfg = dict(synth.CONFIGS, **synth.TINY_CONFIGS)[key]
    return cfg, mmcf_writer.pack_config(cfg)


@pytest.mark.parametrize("key", list(synth.TINY_CONFIGS) + FULL)
def test_writer_matches_reference_packer(golden, key):
    _, data = _container(key)
    want = golden["containers"][key]
    assert len(data) == want["bytes"]
    assert hashlib.sha256(data).hexdigest() == want["sha256"]


def test_xformat_vectors(golden):
    cases = [c for c in golden["xformat"] if c["format"] in ("I16_1", "I16_2")]
    assert len(cases) == 2
    for c in cases:
        q = [oracle.lib().orc_q16(v) for v in c["values"]]
        out = []
        if c["format"] == "I16_1":
            for v in q:
                u = v & 0xFFFF
                out += [u >> 8, u & 0xFF, 0, 255]
        else:
            q = q + [0] * (len(q) % 2)
            for a, b in zip(q[0::2], q[1::2]):
                out += [(a & 0xFFFF) >> 8, a & 0xFF, (b & 0xFFFF) >> 8, b & 0xFF]
        assert out == c["bytes"], c


def _f32bits(x):
    return "%08x" % struct.unpack("<I", struct.pack("<f", x))[0]


def _check_mat(om, ref, which, layer, expert, name):
    rows, cols, wtype, scale = om.mat_shape(which, layer, expert)
    assert (rows, cols) == (ref["rows"], ref["cols"]), name
    lev = om.mat_levels(which, layer, expert).astype(np.int32)
    if wtype == 2:       # t3: the reference expanded the 2-bit levels to +-127 (T3_EXPAND)
        assert ref["type"] == "q8"
        lev = lev * 127
        assert _f32bits(np.float32(struct.unpack("<f", bytes.fromhex(ref["scale"])[::-1])[0]) * np.float32(127.0)) \
            == _f32bits(scale), name
    else:
        assert ref["type"] == {0: "q8", 1: "q4", 3: "i16"}[wtype], name
        assert ref["scale"] == _f32bits(scale), name
    assert oracle.fnv64(lev) == ref["levels"], name
    if wtype == 1:
        s16, m16 = om.mat_q4params(which, layer, expert)
        assert oracle.fnv64(s16.astype(np.int32)) == ref["s16"], name
        assert oracle.fnv64(m16.astype(np.int32)) == ref["m16"], name
    plane = om.mat_plane(which, layer, expert)
    if "row_scale" in ref:
        assert plane is not None and oracle.fnv64(plane) == ref["row_scale"]["fnv"], name
    else:
        assert plane is None, name


@pytest.mark.parametrize("key", list(synth.TINY_CONFIGS) + FULL)
def test_oracle_loader_matches_reference_loader(golden, tmp_path, key):
    _, data = _container(key)
    path = str(tmp_path / "m.mmcf")
    with open(path, "wb") as f:
        f.write(data)
    ref = golden["containers"][key]["reference_load"]
    om = oracle.Model(path)
    inf = om.info
    for k in ("dim", "hidden", "layers", "heads", "kv_heads", "vocab", "head_dim", "kv_dim", "experts",
              "moe_hidden", "rope_half", "qk_norm"):
        assert getattr(inf, k) == ref[k], k
    assert _f32bits(inf.rope_theta) == ref["rope_theta"]
    assert _f32bits(inf.rms_eps) == ref["rms_eps"]
    assert oracle.fnv64(om.emb().astype(np.int32)) == ref["emb"]["fnv"]
    for i, name in enumerate(["emb_scale", "rms_att", "rms_ffn", "rms_final", "q_norm", "k_norm"]):
        v = om.vec(i)
        assert len(v) == ref[name]["n"] and oracle.fnv64(v) == ref[name]["fnv"], name
    for layer in range(inf.layers):
        _check_mat(om, ref["qkv"][layer], 0, layer, 0, "qkv%d" % layer)
        _check_mat(om, ref["wo"][layer], 1, layer, 0, "wo%d" % layer)
        if inf.experts:
            _check_mat(om, ref["router"][layer], 5, layer, 0, "router%d" % layer)
            for e in range(inf.experts):
                x = ref["experts_w"][layer][e]
                for which, nm in ((2, "w1"), (3, "w3"), (4, "w2")):
                    _check_mat(om, x[nm], which, layer, e, "%s%d.%d" % (nm, layer, e))
        else:
            for which, nm in ((2, "w1"), (3, "w3"), (4, "w2")):
                _check_mat(om, ref[nm][layer], which, layer, 0, "%s%d" % (nm, layer))
    assert len(ref["logits"]) == inf.n_logit_tiles
    for t in range(inf.n_logit_tiles):
        _check_mat(om, ref["logits"][t], 6, t, 0, "logits%d" % t)


def test_expf_error_bound():
    """orc_expf (Cody-Waite + degree-7 Taylor) stays within 2 ulp of exp over
    the softmax and SiLU ranges; the kernels evaluate the same operations."""
    xs = np.concatenate([np.linspace(-87.0, 0.0, 4001), np.linspace(-20.0, 20.0, 4001),
                         np.array([0.0, -1e-7, 1e-7, -0.3465736, 0.3465736])]).astype(np.float32)
    worst = 0.0
    for x in xs:
        got = np.float32(oracle.expf(float(x)))
        want = np.exp(np.float64(x))
        ulp = np.spacing(np.float32(want))
        worst = max(worst, abs(float(got) - want) / float(ulp))
    assert worst <= 2.0, worst
    assert oracle.expf(100.0) == float("inf") and oracle.expf(-200.0) == 0.0


@pytest.mark.parametrize("key", list(synth.TINY_CONFIGS))
def test_canonical_vs_literal_reference_order(tiny_paths, key):
    """The canonical arithmetic (exact integer dots, double position sums, the
    portable exp) against the reference's literal float orders (sequential
    fp32 sums, libm expf, fp32 shader accumulation): logits within the 1e-2
    tolerance and the same greedy tokens."""
    cfg = synth.TINY_CONFIGS[key]
    om = oracle.Model(tiny_paths[key])
    prompt = synth.prompt_tokens(cfg)
    a, la, _ = oracle.generate(om, cfg.kv_bits, prompt, cfg.steps)
    b, lb, _ = oracle.generate(om, cfg.kv_bits, prompt, cfg.steps, literal=True)
    assert a == b
    assert np.abs(la - lb).max() <= 1e-2


def test_kv_codec_rails_and_ties():
    """encKV (shaders_attn.cpp:141-159): floor(v*scale+0.5) clamped; ties go up."""
    q16, q8 = oracle.lib().orc_kv_q16, oracle.lib().orc_kv_q8
    assert q16(0.5 / 2048) == 1 and q16(-0.5 / 2048) == 0 and q16(-1.5 / 2048) == -1
    assert q16(16.0) == 32767 and q16(-16.0) == -32768 and q16(-100.0) == -32768
    assert q8(0.5 / 16) == 1 and q8(-0.5 / 16) == 0 and q8(7.9375) == 127 and q8(8.0) == 127
    assert q8(-8.0) == -128 and q8(-9.0) == -128


def test_rope_tables_match_between_library_and_oracle():
    """The engine's host helper builds the same cos/sin bits as the oracle
    (both restate session.cpp:188-202)."""
    import vc4b200
    c1, s1 = vc4b200.rope_tables(1e6, 96, 64)
    half = 48
    c2 = np.empty(64 * half, np.float32)
    s2 = np.empty(64 * half, np.float32)
    oracle.lib().orc_rope_tables(1e6, 96, 64, None, c2.ctypes.data_as(oracle.C.c_void_p),
                                 s2.ctypes.data_as(oracle.C.c_void_p))
    assert np.array_equal(c1.ravel(), c2) and np.array_equal(s1.ravel(), s2)
