"""CUDA path vs the CPU oracle at the positions the benchmark configurations
decode at (SEQ up to 1024), without running the long prompts.

The same seeded KV rows (random cache levels, a few on the rails) are written
into the engine's cache (vc4_kv_write_rows) and the oracle's, then one
teacher-forced step at position `pos` is compared: logits within 1e-2 with
greedy agreement (the north star's tolerance), and the cache row the step
appends byte for byte in every layer.  The batch-1 cases run the cluster
attention kernel over up to 1024 positions split across its 8 CTAs; the
batched cases (>= 128 units of sequence x KV head x q-head pair) run the
many-sequence kernel, whose K/V tiles of 128 positions stream through a
three-stage ring that wraps several times at these lengths.  The device KV
codec is also checked on its own against the oracle's at the rails, at every
rounding tie and at signed zero (shaders_attn.cpp:141-159).
"""
import numpy as np
import pytest

import oracle
import vc4b200
from conftest import full_model_path
from vc4b200 import synth

TOL = 1e-2
KV = {16: "q16", 8: "q8"}


@pytest.fixture(scope="module")
def gpu():
    return vc4b200.GPU(0)


def random_rows(rng, n: int, kv_dim: int, kv_bits: int) -> bytes:
    """n packed cache rows (K then V, kv_dim values each) of random levels:
    q16 big-endian on the 1/2048 grid, q8 on the 1/16 grid; 1% on the rails."""
    if kv_bits == 16:
        lv = np.clip(np.rint(rng.normal(0.0, 1200.0, size=(n, 2 * kv_dim))), -32768, 32767)
        rail = rng.random(lv.shape) < 0.01
        lv[rail] = np.where(rng.random(int(rail.sum())) < 0.5, -32768, 32767)
        return lv.astype(">i2").tobytes()
    lv = np.clip(np.rint(rng.normal(0.0, 12.0, size=(n, 2 * kv_dim))), -128, 127)
    rail = rng.random(lv.shape) < 0.01
    lv[rail] = np.where(rng.random(int(rail.sum())) < 0.5, -128, 127)
    return lv.astype(np.int8).tobytes()


def _check(got, ref, what):
    d = float(np.abs(got - ref).max())
    assert d <= TOL, "%s: max |dlogit| %g" % (what, d)
    assert int(np.argmax(got)) == int(np.argmax(ref)), "%s: greedy token differs" % what


@pytest.mark.gpu
@pytest.mark.parametrize("key,positions", [("c0", [127, 128, 129, 255]), ("c0r", [128, 255]),
                                           ("c1", [127, 128, 129, 255]),
                                           ("c4b1", [511, 512, 767]), ("c3", [1023])])
def test_one_sequence_at_benchmark_positions(gpu, key, positions):
    cfg = synth.CONFIGS[key]
    path = full_model_path(key)
    om = oracle.Model(path)
    model = vc4b200.Model(gpu, path)
    info = model.info
    for pos in positions:
        rng = np.random.default_rng(1000 + pos)
        sess = vc4b200.Session(model, slots=1, seq=cfg.seq, kv=KV[cfg.kv_bits])
        osess = oracle.Session(om, cfg.kv_bits)
        for l in range(info.layers):
            rows = random_rows(rng, pos, info.kv_dim, cfg.kv_bits)
            sess.kv_write(l, pos, rows)
            osess.kv_write(l, pos, rows)
        tok = int(rng.integers(0, info.vocab))
        _check(sess.step(tok, pos), osess.step(tok, pos), "%s pos %d" % (key, pos))
        rb = sess.kv_row_bytes()
        for l in range(info.layers):
            assert sess.kv_rows(l, pos + 1)[pos * rb:] == osess.kv_rows(l, pos + 1)[pos * rb:], \
                "%s pos %d: appended KV row of layer %d differs" % (key, pos, l)
        sess.close()
        osess.close()


@pytest.mark.gpu
@pytest.mark.parametrize("key,n,positions", [
    ("c4", 40, [511, 512, 767, 600, 700, 640, 128, 255]),
    ("c2", 64, [383, 384, 385, 511]),
    ("c3b32", 32, [1023, 1000, 777, 512]),
])
def test_many_sequences_at_benchmark_positions(gpu, key, n, positions):
    """The configured batch (c2: 64 sequences, c3b32: 32) or one above the
    many-sequence threshold (c4), each sequence at its own position."""
    cfg = synth.CONFIGS[key]
    path = full_model_path(key)
    om = oracle.Model(path)
    model = vc4b200.Model(gpu, path)
    info = model.info
    sess = vc4b200.Session(model, slots=n, seq=cfg.seq, kv=KV[cfg.kv_bits])
    rng = np.random.default_rng(77)
    pos = [positions[i % len(positions)] for i in range(n)]
    toks = [int(t) for t in rng.integers(0, info.vocab, size=n)]
    rows = []
    for i in range(n):
        r = [random_rows(rng, pos[i], info.kv_dim, cfg.kv_bits) for _ in range(info.layers)]
        for l in range(info.layers):
            sess.kv_write(l, pos[i], r[l], slot=i)
        rows.append(r)
    nxt, lg = sess.step_batch(list(range(n)), toks, pos, want_logits=True)
    rb = sess.kv_row_bytes()
    for i in range(n):
        osess = oracle.Session(om, cfg.kv_bits)
        for l in range(info.layers):
            osess.kv_write(l, pos[i], rows[i][l])
        ref = osess.step(toks[i], pos[i])
        _check(lg[i], ref, "%s sequence %d pos %d" % (key, i, pos[i]))
        assert int(nxt[i]) == int(np.argmax(ref))
        for l in range(info.layers):
            assert sess.kv_rows(l, pos[i] + 1, slot=i)[pos[i] * rb:] == osess.kv_rows(l, pos[i] + 1)[pos[i] * rb:], \
                "%s sequence %d: appended KV row of layer %d differs" % (key, i, l)
        osess.close()


def _codec_inputs(kv_bits: int) -> np.ndarray:
    """Rails, values past them, signed zero, every rounding tie (n + 0.5)/grid
    near zero and near the rails with its two float neighbours, and a dense
    random sweep of the whole range."""
    grid = 2048.0 if kv_bits == 16 else 16.0
    lo, hi = (-32768, 32767) if kv_bits == 16 else (-128, 127)
    rail = (hi + 1) / grid
    v = [0.0, -0.0, rail, -rail, rail / 2, -rail / 2, hi / grid, lo / grid, 2 * rail, -2 * rail, 1e30, -1e30,
         np.inf, -np.inf, 16.0, -16.0, 8.0, -8.0]
    if kv_bits == 16:
        ns = np.concatenate([np.arange(-600, 600), np.arange(lo - 80, lo + 600), np.arange(hi - 600, hi + 80)])
    else:
        ns = np.arange(lo - 20, hi + 20)
    ties = ((ns + 0.5) / grid).astype(np.float32)
    v = np.concatenate([np.array(v, np.float32), ties, np.nextafter(ties, np.float32(np.inf)),
                        np.nextafter(ties, np.float32(-np.inf)), (ns / grid).astype(np.float32)])
    rng = np.random.default_rng(3)
    sweep = rng.uniform(-1.25 * rail, 1.25 * rail, size=200000).astype(np.float32)
    tiny = (rng.uniform(-1, 1, size=20000) * 10.0 ** rng.uniform(-12, 0, size=20000)).astype(np.float32)
    return np.concatenate([v, sweep, tiny]).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("kv_bits", [16, 8])
def test_device_kv_codec_matches_oracle(kv_bits):
    import ctypes as C
    x = _codec_inputs(kv_bits)
    kvb = kv_bits // 8
    out = np.empty(x.size * kvb, np.uint8)
    rc = vc4b200.lib().vc4_kv_codec_probe(0, kv_bits, x.ctypes.data_as(C.c_void_p), x.size,
                                          out.ctypes.data_as(C.c_void_p))
    assert rc == 0, vc4b200.lib().vc4_last_error().decode()
    L = oracle.lib()
    if kv_bits == 16:
        got = out.view(">i2").astype(np.int64)
        ref = np.array([L.orc_kv_q16(float(v)) for v in x], np.int64)
    else:
        got = out.view(np.int8).astype(np.int64)
        ref = np.array([L.orc_kv_q8(float(v)) for v in x], np.int64)
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, "%d values differ, first %r: device %d oracle %d" % (
        bad.size, float(x[bad[0]]), got[bad[0]], ref[bad[0]])
