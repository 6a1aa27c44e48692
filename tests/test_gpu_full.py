"""CUDA path vs the CPU oracle at the five benchmark configurations' full
shapes, on shortened workloads the oracle finishes in seconds.

Tolerance: max |dlogit| <= 1e-2 with greedy agreement (the north star's); the
KV rows are compared bit for bit.
"""
import numpy as np
import pytest

import oracle
import vc4b200
from conftest import full_model_path
from vc4b200 import synth

TOL = 1e-2
KV = {16: "q16", 8: "q8"}


def _path(key):
    return full_model_path(key)


@pytest.fixture(scope="module")
def gpu():
    return vc4b200.GPU(0)


@pytest.mark.gpu
@pytest.mark.parametrize("key,prompt_len,steps", [("c0", 24, 8), ("c0r", 24, 8), ("c1", 24, 8), ("c3", 12, 4)])
def test_single_stream_full_shape(gpu, key, prompt_len, steps):
    cfg = synth.CONFIGS[key]
    path = _path(key)
    om = oracle.Model(path)
    model = vc4b200.Model(gpu, path)
    prompt = synth.prompt_tokens(cfg)[:prompt_len]
    sess = vc4b200.Session(model, slots=1, seq=cfg.seq, kv=KV[cfg.kv_bits])
    osess = oracle.Session(om, cfg.kv_bits)
    exact = 0
    for pos, t in enumerate(prompt):
        a = sess.step(t, pos)
        b = osess.step(t, pos)
        d = np.abs(a - b).max()
        assert d <= TOL, "%s position %d: max |dlogit| %g" % (key, pos, d)
        assert int(np.argmax(a)) == int(np.argmax(b))
        exact += int(d == 0)
    print("%s: %d/%d positions bit-exact" % (key, exact, len(prompt)))
    for layer in (0, om.info.layers - 1):
        assert sess.kv_rows(layer, len(prompt)) == osess.kv_rows(layer, len(prompt))
    sess2 = vc4b200.Session(model, slots=1, seq=cfg.seq, kv=KV[cfg.kv_bits])
    toks, logs = vc4b200.generate(sess2, prompt, steps)
    rtoks, rlogs, _ = oracle.generate(om, cfg.kv_bits, prompt, steps)
    assert toks == rtoks
    assert np.abs(logs - rlogs).max() <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n", [6, 10])
def test_moe_batch_full_shape(gpu, n):
    """c2: MoE q4, KV q8, several sequences per pass routed to different
    experts (10: the many-sequence kernels)."""
    cfg = synth.CONFIGS["c2"]
    path = _path("c2")
    om = oracle.Model(path)
    model = vc4b200.Model(gpu, path)
    P = 10
    prompts = [synth.prompt_tokens(cfg, i)[:P] for i in range(n)]
    sess = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    got = []
    for pos in range(P):
        _, lg = sess.step_batch(list(range(n)), [p[pos] for p in prompts], [pos] * n, want_logits=True)
        got.append(lg)
    routes = set()
    for i in range(n):
        os_ = oracle.Session(om, 8)
        for pos in range(P):
            ref = os_.step(prompts[i][pos], pos)
            d = np.abs(got[pos][i] - ref).max()
            assert d <= TOL, "sequence %d position %d: %g" % (i, pos, d)
            assert int(np.argmax(got[pos][i])) == int(np.argmax(ref))
            routes.update(os_.route(l) for l in range(om.info.layers))
        assert sess.kv_rows(3, P, slot=i) == os_.kv_rows(3, P)
    assert len(routes) >= 2, "the batch exercised only one expert"


@pytest.mark.gpu
@pytest.mark.parametrize("n", [4, 9, 33])
def test_prefix_restore_batch_full_shape(gpu, tmp_path, n):
    """c4: one prefix prefilled once, saved as MMKV1, restored into every slot
    of a batch, then greedy decode of all slots in one pass (KV q8; 9 runs the
    many-sequence kernels, 33 their tcgen05 tensor-core form)."""
    cfg = synth.CONFIGS["c4"]
    path = _path("c4")
    om = oracle.Model(path)
    model = vc4b200.Model(gpu, path)
    prefix = synth.prompt_tokens(cfg)[:32]
    first = vc4b200.Session(model, slots=1, seq=cfg.seq, kv="q8")
    first.prefill(prefix, 0, want_logits=False)
    mmkv = str(tmp_path / "prefix.mmkv")
    first.save_prefix_cache(mmkv, prefix)
    steps = 6
    batch = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    for s in range(n):
        assert batch.load_prefix_cache(mmkv, slot=s) == prefix
    # each slot continues from the prefix with a different next token
    nxt = [prefix[-1] if s == 0 else (prefix[-1] + 97 * s) % cfg.shape.vocab for s in range(n)]
    outs = []
    # the cache holds rows 0..P-1, so decode starts at position P with a
    # different token per slot
    pos = len(prefix)
    toks = list(nxt)
    for _ in range(steps):
        nx, lg = batch.step_batch(list(range(n)), toks, [pos] * n, want_logits=True)
        outs.append(lg)
        toks = [int(t) for t in nx]
        pos += 1
    rows = first.kv_rows(0, len(prefix))
    ref_pre = oracle.Session(om, 8)                 # the prefix's rows are the oracle's bytes
    for p, t in enumerate(prefix):
        ref_pre.step(t, p, want_logits=False)
    for l in range(om.info.layers):
        assert ref_pre.kv_rows(l, len(prefix)) == first.kv_rows(l, len(prefix)), "prefix layer %d" % l
    for s in range(n):
        os_ = oracle.Session(om, 8)
        for l in range(om.info.layers):
            os_.kv_write(l, len(prefix), first.kv_rows(l, len(prefix)))
        t, p = nxt[s], len(prefix)
        for k in range(steps):
            ref = os_.step(t, p)
            d = np.abs(outs[k][s] - ref).max()
            assert d <= TOL, "slot %d step %d: %g" % (s, k, d)
            t, p = int(np.argmax(ref)), p + 1
            assert t == int(np.argmax(outs[k][s]))
    assert rows == batch.kv_rows(0, len(prefix), slot=2)[: len(rows)]


@pytest.mark.gpu
def test_batch_1024_equals_serial(gpu, tmp_path):
    """c4 at the bench's 1024 sequences per pass: the tensor-core matmats run
    their largest sequence groups (64-128 per CTA, all 512 TMEM columns for
    w1/w3), two CTAs per SM with two-stage copy rings for the logits and
    19-stage rings for w2; each sampled sequence gets its one-sequence result
    bit for bit."""
    cfg = synth.CONFIGS["c4"]
    model = vc4b200.Model(gpu, _path("c4"))
    prefix = synth.prompt_tokens(cfg)[:32]
    first = vc4b200.Session(model, slots=1, seq=cfg.seq, kv="q8")
    first.prefill(prefix, 0, want_logits=False)
    mmkv = str(tmp_path / "prefix.mmkv")
    first.save_prefix_cache(mmkv, prefix)
    n, steps = 1024, 3
    batch = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    for s in range(n):
        batch.load_prefix_cache(mmkv, slot=s)
    toks = [(prefix[-1] + 97 * s) % cfg.shape.vocab for s in range(n)]
    fed, outs = [], []
    pos = len(prefix)
    for _ in range(steps):
        fed.append(list(toks))
        nx, lg = batch.step_batch(list(range(n)), toks, [pos] * n, want_logits=True)
        outs.append(lg)
        toks = [int(t) for t in nx]
        pos += 1
    for s in (0, 1, 63, 64, 127, 128, 511, 777, 1000, 1023):
        one = vc4b200.Session(model, slots=1, seq=cfg.seq, kv="q8")
        one.load_prefix_cache(mmkv)
        for k in range(steps):
            lg = one.step(fed[k][s], len(prefix) + k)
            assert np.array_equal(lg, outs[k][s]), "sequence %d step %d" % (s, k)
