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
@pytest.mark.parametrize("shared", [False, True])
def test_batch_1024_equals_serial(gpu, tmp_path, shared):
    """c4 at the bench's 1024 sequences per pass: the tensor-core matmats run
    their largest sequence groups (64-128 per CTA, all 512 TMEM columns for
    w1/w3), two CTAs per SM with two-stage copy rings for the logits and
    19-stage rings for w2; each sampled sequence gets its one-sequence result
    bit for bit.  With the 300-row prefix held once (shared), every sequence
    reads its three prefix tiles from the session's one copy."""
    cfg = synth.CONFIGS["c4"]
    model = vc4b200.Model(gpu, _path("c4"))
    prefix = synth.prompt_tokens(cfg)[:300]
    first = vc4b200.Session(model, slots=1, seq=cfg.seq, kv="q8")
    first.prefill(prefix, 0, want_logits=False)
    mmkv = str(tmp_path / "prefix.mmkv")
    first.save_prefix_cache(mmkv, prefix)
    n, steps = 1024, 3
    batch = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    if shared:
        batch.load_prefix_cache_shared(mmkv, list(range(n)))
    else:
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


# the sidecar's field set (prefix_cache.cpp:104-128)
SIDECAR_KEYS = {"format", "version", "source_size", "source_mtime", "dim", "hidden", "layers", "heads", "kv_heads",
                "vocab", "seq", "head_dim", "rope_theta", "kv_bits", "act_fmt", "hybrid", "kv_scale", "kv_width",
                "vstep", "n_tokens", "tokens_fnv64", "system_fnv64", "tools_fnv64", "template"}


@pytest.mark.gpu
def test_build_prefix_cache(gpu, tmp_path):
    """`--build-prefix-cache` for a tokenised prompt (prefix_build.cpp:22-83):
    the file equals a serial prefill plus save_prefix_cache byte for byte, its
    rows are the oracle's, the sidecar carries the reference's field set with
    the container's template name and the FNV-1a hashes, and an empty or too
    long prompt is refused."""
    import json
    from vc4b200.engine import fnv64
    cfg = synth.CONFIGS["c4"]
    path = _path("c4")
    model = vc4b200.Model(gpu, path)
    prefix = synth.prompt_tokens(cfg)[:40]
    built = str(tmp_path / "built.mmkv")
    s = vc4b200.Session(model, slots=2, seq=cfg.seq, kv="q8")
    system = "You are a helpful assistant."
    s.build_prefix_cache(built, prefix, slot=1, system=system, tools="[]")
    saved = str(tmp_path / "saved.mmkv")
    ref = vc4b200.Session(model, slots=1, seq=cfg.seq, kv="q8")
    ref.prefill(prefix, 0, want_logits=False)
    ref.save_prefix_cache(saved, prefix, system_fnv=fnv64(system.encode()), tools_fnv=fnv64(b"[]"))
    assert open(built, "rb").read() == open(saved, "rb").read()
    om = oracle.Model(path)
    os_ = oracle.Session(om, 8)
    for p, t in enumerate(prefix):
        os_.step(t, p, want_logits=False)
    for l in range(om.info.layers):
        assert s.kv_rows(l, len(prefix), slot=1) == os_.kv_rows(l, len(prefix)), "layer %d" % l
    meta = json.load(open(built + ".json"))
    assert set(meta) == SIDECAR_KEYS
    assert meta["template"] == "plain" and meta["n_tokens"] == len(prefix) and meta["kv_bits"] == 8
    tok_fnv = fnv64(b"".join(int(t).to_bytes(4, "little") for t in prefix))
    assert meta["tokens_fnv64"] == "%016x" % tok_fnv
    assert meta["system_fnv64"] == "%016x" % fnv64(system.encode())
    assert meta["tools_fnv64"] == "%016x" % fnv64(b"[]")
    assert json.load(open(saved + ".json")) == meta
    for bad in ([], list(range(cfg.seq + 1))):
        with pytest.raises(vc4b200.EngineError):
            s.build_prefix_cache(str(tmp_path / "bad.mmkv"), bad)


@pytest.mark.gpu
def test_shared_and_private_prefixes_in_one_batch(gpu, tmp_path):
    """Slots that read the shared prefix next to slots restored into their own
    rows in one many-sequence pass (slots 32-63 alternate shared and private
    restores, slots 48-63 run at scattered positions): every sequence equals
    the same restore in a session without a shared prefix, bit for bit."""
    cfg = synth.CONFIGS["c4"]
    model = vc4b200.Model(gpu, _path("c4"))
    prefix = synth.prompt_tokens(cfg)[:200]
    first = vc4b200.Session(model, slots=16, seq=cfg.seq, kv="q8")
    first.prefill(prefix, 0, want_logits=False, batched=True)
    mmkv = str(tmp_path / "prefix.mmkv")
    first.save_prefix_cache(mmkv, prefix)
    n = 64
    priv = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    mix = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    for s in range(n):
        priv.load_prefix_cache(mmkv, slot=s)
    sharing = [s for s in range(n) if s < 32 or s % 2 == 0]
    mix.load_prefix_cache_shared(mmkv, sharing)
    for s in range(n):
        if s not in sharing:
            mix.load_prefix_cache(mmkv, slot=s)
    P = len(prefix)
    toks = [(prefix[-1] + 31 * s) % cfg.shape.vocab for s in range(n)]
    pos = [P + (s % 5 if s >= 48 else 0) for s in range(n)]
    for _ in range(3):
        na, la = priv.step_batch(list(range(n)), toks, pos, want_logits=True)
        nb, lb = mix.step_batch(list(range(n)), toks, pos, want_logits=True)
        assert np.array_equal(la, lb) and list(na) == list(nb)
        toks = [int(t) for t in na]
        pos = [p + 1 for p in pos]
    for s in (0, 33, 50, 63):
        assert mix.kv_rows(3, pos[s], slot=s) == priv.kv_rows(3, pos[s], slot=s)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [9, 33])
def test_shared_prefix_equals_private_restore(gpu, tmp_path, n):
    """c4 with the prefix held once (vc4_load_prefix_cache_shared) against the
    same prefix restored into every slot's own rows: logits, greedy tokens
    and KV rows equal bit for bit (9 slots: cluster attention; 33: the
    many-sequence kernel, whose 300-row prefix spans three K/V tiles).  Then
    copy on write: a row write, a host-array step inside the prefix and a
    prefill over it each give only that slot its own rows; a device-array
    step inside the prefix is refused through the session's check word."""
    cfg = synth.CONFIGS["c4"]
    model = vc4b200.Model(gpu, _path("c4"))
    prefix = synth.prompt_tokens(cfg)[:300]
    first = vc4b200.Session(model, slots=64, seq=cfg.seq, kv="q8")
    first.prefill(prefix, 0, want_logits=False, batched=True)
    mmkv = str(tmp_path / "prefix.mmkv")
    first.save_prefix_cache(mmkv, prefix)
    priv = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    shar = vc4b200.Session(model, slots=n, seq=cfg.seq, kv="q8")
    for s in range(n):
        assert priv.load_prefix_cache(mmkv, slot=s) == prefix
    assert shar.load_prefix_cache_shared(mmkv, list(range(n))) == prefix
    P = len(prefix)
    toks = [(prefix[-1] + 97 * s) % cfg.shape.vocab for s in range(n)]
    pos = P
    for _ in range(4):
        na, la = priv.step_batch(list(range(n)), toks, [pos] * n, want_logits=True)
        nb, lb = shar.step_batch(list(range(n)), toks, [pos] * n, want_logits=True)
        assert np.array_equal(la, lb) and list(na) == list(nb)
        toks = [int(t) for t in na]
        pos += 1
    L = model.info.layers
    for s in (0, n - 1):
        for l in (0, L - 1):
            assert shar.kv_rows(l, pos, slot=s) == priv.kv_rows(l, pos, slot=s)
    # a row write into slot 1's prefix: slot 1 alone sees it
    rb = shar.kv_row_bytes()
    rows = bytearray(shar.kv_rows(0, 2, slot=1))
    rows[:rb] = bytes((b + 1) & 0xFF for b in rows[:rb])
    shar.kv_write(0, 2, bytes(rows), slot=1)
    assert shar.kv_rows(0, 2, slot=1) == bytes(rows)
    assert shar.kv_rows(0, P, slot=2) == priv.kv_rows(0, P, slot=2)
    assert shar.kv_rows(1, pos, slot=1) == priv.kv_rows(1, pos, slot=1)
    # a host-array step inside slot 2's prefix: the same as in a private slot
    la = priv.step(prefix[100], 100, slot=2)
    lb = shar.step(prefix[100], 100, slot=2)
    assert np.array_equal(la, lb)
    assert shar.kv_rows(0, P, slot=3) == priv.kv_rows(0, P, slot=3)
    # a prefill over slot 3's prefix
    la = priv.prefill(prefix[50:80], 50, slot=3)
    lb = shar.prefill(prefix[50:80], 50, slot=3)
    assert np.array_equal(la, lb)
    for l in (0, L - 1):
        assert shar.kv_rows(l, pos, slot=3) == priv.kv_rows(l, pos, slot=3)
    # a device-array step inside slot 4's prefix is refused, its row unwritten
    import torch
    d_slots = torch.tensor([4], dtype=torch.int32, device="cuda")
    d_tok = torch.tensor([prefix[10]], dtype=torch.int32, device="cuda")
    d_pos = torch.tensor([10], dtype=torch.int32, device="cuda")
    d_next = torch.zeros(1, dtype=torch.int32, device="cuda")
    before = shar.kv_rows(0, P, slot=4)
    with pytest.raises(vc4b200.EngineError, match="shared prefix"):
        # the first pass of a shape checks the word itself; a replay would at check()
        shar.step_batch_device(1, d_slots.data_ptr(), d_tok.data_ptr(), d_pos.data_ptr(), d_next.data_ptr(), False)
        shar.check()
    assert shar.kv_rows(0, P, slot=4) == before
