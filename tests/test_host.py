"""Host-side logic, no GPU: the C ABI's exports, the container reader's
refusals (Model::probe, model.cpp:152 refuse()), and the data-parallel
plumbing bench.py runs under torchrun, exercised as 2-rank gloo groups."""
import os
import re
import struct
import zlib

import numpy as np
import pytest

import oracle
import vc4b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "vc4b200.h")).read()
    return sorted(set(re.findall(r"VC4_API\s+[\w\s\*]*?\b(vc4_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = _declared()
    assert len(names) >= 27
    L = vc4b200.lib()
    for n in names:
        assert hasattr(L, n), n
    assert set(names) <= set(vc4b200.engine._PROTOS), "python binding misses %s" % (set(names) - set(vc4b200.engine._PROTOS))


def test_no_gpu_is_a_loud_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(vc4b200.EngineError) as e:
        vc4b200.GPU(0)
    assert "vc4b200 error" in str(e.value)


@pytest.mark.parametrize("key", ["tiny_q8", "tiny_q4", "tiny_moe_q4", "tiny_t3", "tiny_flat_q8"])
def test_probe_matches_oracle(tiny_paths, key):
    info = vc4b200.probe(tiny_paths[key])
    om = oracle.Model(tiny_paths[key])
    for k in ("dim", "hidden", "layers", "heads", "kv_heads", "vocab", "seq", "head_dim", "kv_dim", "experts",
              "moe_hidden", "ffn_width", "ffn_chunked", "ffn_chunk", "qk_norm", "rope_half", "wtype"):
        assert getattr(info, k) == getattr(om.info, k), k
    assert info.head_dedup == (key == "tiny_t3")


def _mutants(data: bytes):
    """(name, bytes) of damaged containers both readers must refuse."""
    b = bytearray(data)
    out = [("truncated", bytes(b[:40])), ("bad magic", b"XMCF" + bytes(b[4:]))]
    v = bytearray(b); v[4:6] = struct.pack("<H", 9); out.append(("version", bytes(v)))
    c = bytearray(b); c[8] ^= 1; out.append(("header crc", bytes(c)))        # n_tensors changed, crc stale
    s = bytearray(b) + b"\0" * 16; out.append(("size field", bytes(s)))
    # drop the embedding: rewrite its record's id to an unknown kind (with a fresh header crc)
    t = bytearray(b)
    meta_off, meta_size = struct.unpack_from("<II", t, 16)
    data_off, = struct.unpack_from("<Q", t, 24)
    n, = struct.unpack_from("<I", t, 8)
    ver, = struct.unpack_from("<H", t, 4)
    rs = 64 if ver >= 3 else 48
    table = data_off - n * rs
    for i in range(n):
        if struct.unpack_from("<H", t, table + i * rs)[0] == 1:
            struct.pack_into("<H", t, table + i * rs, 0x3F)
    out.append(("no embedding", bytes(t)))
    return out


@pytest.mark.parametrize("key", ["tiny_q8", "tiny_t3"])
def test_damaged_containers_are_refused(tiny_paths, tmp_path, key):
    data = open(tiny_paths[key], "rb").read()
    for name, blob in _mutants(data):
        p = str(tmp_path / (name.replace(" ", "_") + ".mmcf"))
        with open(p, "wb") as f:
            f.write(blob)
        with pytest.raises(vc4b200.EngineError):
            vc4b200.probe(p)
        with pytest.raises(RuntimeError):
            oracle.Model(p)
    with pytest.raises(vc4b200.EngineError) as e:
        vc4b200.probe(str(tmp_path / "missing.mmcf"))
    assert "cannot open" in str(e.value)


# ---------------------------------------------------------------------------
# data-parallel plumbing: 2 gloo ranks on the CPU
# ---------------------------------------------------------------------------

def _rank_main(rank, world, port, mode, path, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vc4-gles2-inference_b200"), os.path.join(ROOT, "oracle")]
    import bench
    from vc4b200 import synth
    try:
        dist = bench.Dist(backend="gloo", timeout_s=20)
        cfg = synth.TINY_CONFIGS["tiny_q8"]
        ids = bench.sequence_ids(dist.rank, 2)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the timed region")
        import oracle as orc
        om = orc.Model(path)
        toks = 0
        for i in ids:
            t, _, _ = orc.generate(om, cfg.kv_bits, synth.prompt_tokens(cfg, i)[:6], 3)
            toks += len(t)
        dist.barrier()
        total = dist.sum(toks)
        slowest = dist.max(float(rank + 1))
        q.put((rank, ids, total, slowest, None))
        dist.close()
    except Exception as e:  # the surviving rank reports what it saw
        q.put((rank, None, None, None, type(e).__name__ + ": " + str(e)[:200]))


def _run_ranks(mode, path, timeout=90):
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, mode, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=timeout)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


def test_gloo_two_ranks_shard_sequences_and_reduce(tiny_paths):
    res = _run_ranks("ok", tiny_paths["tiny_q8"])
    assert res[0][1] == [0, 1] and res[1][1] == [2, 3]      # disjoint sequences per rank
    assert res[0][2] == res[1][2] == 2 * 2 * 3               # tokens summed over ranks
    assert res[0][3] == res[1][3] == 2.0                     # time = max over ranks


def test_gloo_rank_failure_is_detected_not_hung(tiny_paths):
    """A rank that raises before the timed region: the other rank's next
    collective ends with an error inside the process-group timeout."""
    res = _run_ranks("fail", tiny_paths["tiny_q8"])
    assert res[1][4] and "rank 1 fails" in res[1][4]
    assert res[0][4] is not None                              # rank 0 saw an error, not a hang


@pytest.mark.parametrize("stride", [-1, 0, 10])
def test_perplexity_windows_follow_the_reference_loop(tiny_paths, stride):
    """vc4b200.perplexity's windowing against a literal restatement of
    run_ppl's loop (ppl.cpp:23-88: a fresh session per window, every position
    stepped, a token scored once), both scoring through the CPU oracle."""
    import oracle
    from vc4b200 import perplexity, synth
    from vc4b200.engine import log_prob
    cfg = synth.TINY_CONFIGS["tiny_q8"]
    toks = sum((synth.prompt_tokens(cfg, i) for i in range(8)), [])[:150]
    om = oracle.Model(tiny_paths["tiny_q8"])
    span = cfg.seq

    def scorer(win, first):
        s = oracle.Session(om, cfg.kv_bits)
        out = [s.step(t, j, want_logits=j >= first) for j, t in enumerate(win)]
        s.close()
        return out[first:]
    got = perplexity(None, toks, span=span, stride=stride, scorer=scorer)
    st = span // 2 if stride < 0 else stride
    st = min(st or span - 1, span - 1)
    warm, n, nxt, windows, nll, cnt = span - st, len(toks), 1, 0, 0.0, 0
    while nxt < n:
        a = 0 if windows == 0 else nxt - warm
        ln = min(span, n - a)
        if ln < 2 or a < 0:
            break
        s = oracle.Session(om, cfg.kv_bits)
        for j in range(ln - 1):
            t = a + j + 1
            lg = s.step(toks[a + j], j, want_logits=t >= nxt)
            if t < nxt:
                continue
            nll += -log_prob(lg, toks[t])
            cnt += 1
            nxt = t + 1
        s.close()
        windows += 1
    assert (got["tokens"], got["windows"], got["stride"]) == (cnt, windows, st)
    assert got["nll"] == nll / cnt


def test_fnv64_matches_the_reference_constants():
    """The sidecar's FNV-1a-64 as the reference computes it (common.cpp:63-67,
    prefix_cache.cpp:94-104): offset basis 1469598103934665603 (the reference's
    constant; the published FNV basis has one more digit,
    14695981039346656037, and the sidecar must carry the reference's value),
    prime 1099511628211, tokens hashed as four little-endian bytes each."""
    from vc4b200.engine import fnv64
    basis, prime = 1469598103934665603, 1099511628211
    assert fnv64(b"") == basis
    h = basis
    for b in b"foobar":
        h = ((h ^ b) * prime) & 0xFFFFFFFFFFFFFFFF
    assert fnv64(b"foobar") == h == 0x88FAD7C0A8FF07F2
    toks = [1, 258, 70000]
    h = basis
    for t in toks:
        for k in range(4):
            h = ((h ^ ((t >> (8 * k)) & 0xFF)) * prime) & 0xFFFFFFFFFFFFFFFF
    assert fnv64(b"".join(t.to_bytes(4, "little") for t in toks)) == h
