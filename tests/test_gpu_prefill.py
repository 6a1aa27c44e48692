"""Batched prefill (vc4_prefill_batch) against the serial prompt loop.

The reference batches prefill with step_pair and PREFILL_BATCH
(session.cpp:1598-1795) and accepts either only when it is byte-identical to
the serial loop.  The same bar holds here: a prompt run as batches of the
many-sequence path (tensor-core matmats for q8 from 32 positions, t3 from 64)
must give the serial loop's last-position logits and every K/V row bit for
bit.  The chunking follows the session's slot count, so the cases cover one
chunk, several chunks, and a tail short enough to take the serial loop.
"""
import numpy as np
import pytest

import vc4b200
from conftest import full_model_path
from vc4b200 import synth

KV = {16: "q16", 8: "q8"}


@pytest.fixture(scope="module")
def gpu():
    return vc4b200.GPU(0)


@pytest.mark.gpu
@pytest.mark.parametrize("key,n,slots", [
    ("c1", 128, 128),    # q4, KV q16: one chunk of 128 (CUDA-core matmats)
    ("c4", 512, 512),    # q8, KV q8: one chunk of 512 (tensor-core matmats), the bench's prefix
    ("c0", 128, 48),     # q8: chunks 48, 48, then 32 (tensor cores from 32)
    ("c2", 200, 64),     # MoE q4: chunks 64, 64, 64, then 8 positions through the serial loop
    ("c3", 160, 80),     # t3, head size 64, SEQ 1024: chunks 80, 80 (tensor cores from 64)
])
def test_prefill_batch_equals_serial(gpu, key, n, slots):
    cfg = synth.CONFIGS[key]
    model = vc4b200.Model(gpu, full_model_path(key))
    prompt = (synth.prompt_tokens(cfg) * 4)[:n]
    kv = KV[cfg.kv_bits]
    ser = vc4b200.Session(model, slots=1, seq=cfg.seq, kv=kv)
    want = ser.prefill(prompt, 0)
    bat = vc4b200.Session(model, slots=slots, seq=cfg.seq, kv=kv)
    slot = slots - 1                       # a slot other than 0: the chunk's entries all name it
    got = bat.prefill(prompt, 0, slot=slot, batched=True)
    assert np.array_equal(got, want), "max |d| %g" % np.abs(got - want).max()
    for l in range(model.info.layers):
        assert bat.kv_rows(l, n, slot=slot) == ser.kv_rows(l, n), "layer %d" % l
    # decoding on from the batched prefix continues exactly as from the serial one
    t = int(np.argmax(want))
    a = ser.step(t, n)
    b = bat.step(t, n, slot=slot)
    assert np.array_equal(a, b)


@pytest.mark.gpu
def test_prefill_batch_from_a_later_position(gpu):
    """A prompt appended after existing rows (pos0 > 0), as a chat turn does."""
    cfg = synth.CONFIGS["c4"]
    model = vc4b200.Model(gpu, full_model_path("c4"))
    prompt = synth.prompt_tokens(cfg)[:300]
    ser = vc4b200.Session(model, slots=1, seq=cfg.seq, kv="q8")
    bat = vc4b200.Session(model, slots=128, seq=cfg.seq, kv="q8")
    ser.prefill(prompt[:100], 0, want_logits=False)
    bat.prefill(prompt[:100], 0, want_logits=False, batched=True)
    want = ser.prefill(prompt[100:], 100)
    got = bat.prefill(prompt[100:], 100, batched=True)
    assert np.array_equal(got, want)
    for l in (0, model.info.layers - 1):
        assert bat.kv_rows(l, 300) == ser.kv_rows(l, 300)


@pytest.mark.gpu
@pytest.mark.parametrize("key,stride", [("tiny_q8", -1), ("tiny_moe_q4", -1), ("tiny_t3", 0)])
def test_perplexity_windows_match_the_oracle(tiny_paths, key, stride):
    """`--ppl` windows (ppl.cpp:23-88) over 150 tokens of a tiny model (span =
    SEQ 64): context positions prefilled in batches, the scored positions'
    logits from one batched pass, against the oracle stepping every position
    of every window; stride -1 is the default span/2, 0 cold windows."""
    import oracle
    cfg = synth.TINY_CONFIGS[key]
    toks = sum((synth.prompt_tokens(cfg, i) for i in range(8)), [])[:150]
    model = vc4b200.Model(vc4b200.GPU(0), tiny_paths[key])
    sess = vc4b200.Session(model, slots=64, seq=cfg.seq, kv=KV[cfg.kv_bits])
    got = vc4b200.perplexity(sess, toks, stride=stride)
    om = oracle.Model(tiny_paths[key])

    def scorer(win, first):
        s = oracle.Session(om, cfg.kv_bits)
        out = [s.step(t, j, want_logits=j >= first) for j, t in enumerate(win)]
        s.close()
        return out[first:]
    want = vc4b200.perplexity(None, toks, span=cfg.seq, stride=stride, scorer=scorer)
    assert (got["tokens"], got["windows"], got["span"], got["stride"]) == \
        (want["tokens"], want["windows"], want["span"], want["stride"]) and got["tokens"] == 149
    assert abs(got["nll"] - want["nll"]) <= 1e-4, (got, want)
