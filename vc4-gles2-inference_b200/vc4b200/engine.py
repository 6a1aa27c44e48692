"""ctypes binding of the engine's C ABI (include/vc4b200.h) and the host-side
mirror of the reference's session interface.

`Session` mirrors engine/src/session.h: step (Session::step,
session.cpp:1797-1821), step_greedy (1827-1842), save_prefix_cache /
load_prefix_cache (prefix_cache.cpp:25-207), plus the multi-sequence calls this
tier adds.  Errors raise `EngineError` carrying the library's message.  There
is no fallback: without the built library on a CUDA device every call fails.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# VC4B200_LIB names another build of the library (a measurement variant)
LIB_PATH = os.environ.get("VC4B200_LIB") or os.path.join(_HERE, "_lib", "libvc4b200.so")

WQ8, WQ4, WT3 = 0, 1, 2
MATS = {"qkv": 0, "wo": 1, "w1": 2, "w3": 3, "w2": 4, "router": 5, "logits": 6}


class EngineError(RuntimeError):
    pass


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "dim", "hidden", "layers", "heads", "kv_heads", "vocab", "seq", "head_dim", "kv_dim",
        "experts", "moe_hidden", "ffn_width", "ffn_chunked", "ffn_chunk",
        "qk_norm", "rope_half", "head_dedup", "wtype")] + [
        ("rope_theta", C.c_float), ("rms_eps", C.c_float),
        ("weight_bytes", C.c_uint64), ("source_size", C.c_uint64), ("source_mtime", C.c_uint64)]


_lib = None

# name -> (restype, argtypes); every symbol include/vc4b200.h declares
_PROTOS = {
    "vc4_last_error": (C.c_char_p, []),
    "vc4_gpu_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "vc4_gpu_destroy": (None, [C.c_void_p]),
    "vc4_gpu_sync": (C.c_int, [C.c_void_p]),
    "vc4_model_load": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
    "vc4_model_load_bytes": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
    "vc4_model_info_get": (C.c_int, [C.c_void_p, C.POINTER(ModelInfo)]),
    "vc4_model_free": (None, [C.c_void_p]),
    "vc4_model_probe": (C.c_int, [C.c_char_p, C.POINTER(ModelInfo)]),
    "vc4_profile_op": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_int, C.c_int, C.POINTER(C.c_double)]),
    "vc4_op_bytes": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_double)]),
    "vc4_matvec_probe": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "vc4_kv_codec_probe": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
    "vc4_session_create": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                     C.POINTER(C.c_void_p)]),
    "vc4_session_destroy": (None, [C.c_void_p]),
    "vc4_rope_tables": (None, [C.c_float, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "vc4_step": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "vc4_step_greedy": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "vc4_step_batch": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "vc4_step_batch_device": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_int]),
    "vc4_session_stream": (C.c_void_p, [C.c_void_p]),
    "vc4_session_check": (C.c_int, [C.c_void_p]),
    "vc4_prefill": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "vc4_prefill_batch": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "vc4_prefill_logits": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "vc4_kv_row_bytes": (C.c_int, [C.c_void_p]),
    "vc4_kv_read_rows": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "vc4_kv_write_rows": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "vc4_save_prefix_cache": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_void_p, C.c_int, C.c_uint64,
                                        C.c_uint64]),
    "vc4_load_prefix_cache": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_void_p, C.c_int,
                                        C.POINTER(C.c_int)]),
    "vc4_load_prefix_cache_shared": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                               C.POINTER(C.c_int)]),
    "vc4_build_prefix_cache": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_char_p, C.c_uint64,
                                         C.c_uint64]),
    "vc4_matvec_s": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "vc4_matvec_s_noalloc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p]),
    "vc4_embedding": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "vc4_upload_hidden": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int]),
    "vc4_rmsnorm": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "vc4_attention_block": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "vc4_matvec_add": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "vc4_matvec_from": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "vc4_ffn_split": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "vc4_logits_from": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "vc4_logits_argmax_from": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "vc4_read_buffer": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "vc4_counters": (C.c_int, [C.c_void_p, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]),
    "vc4_launches_per_step": (C.c_int, [C.c_void_p, C.c_int]),
}


def lib():
    """Load the in-tree library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise EngineError("libvc4b200.so is not built (%s); run __graft_entry__.build()" % LIB_PATH)
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _PROTOS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise EngineError("vc4b200 error %d: %s" % (rc, lib().vc4_last_error().decode(errors="replace")))


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def rope_tables(theta: float, head_dim: int, seq: int, factors=None):
    """cos, sin tables (seq x head_dim/2) as Session::reset builds them."""
    half = head_dim // 2
    c = np.empty(seq * half, np.float32)
    s = np.empty(seq * half, np.float32)
    f = None if factors is None else np.ascontiguousarray(factors, np.float32)
    lib().vc4_rope_tables(theta, head_dim, seq, _p(f) if f is not None else None, _p(c), _p(s))
    return c.reshape(seq, half), s.reshape(seq, half)


def probe(path: str) -> ModelInfo:
    """Model::probe: validate a container on the host (no GPU needed)."""
    info = ModelInfo()
    _check(lib().vc4_model_probe(path.encode(), C.byref(info)))
    return info


class GPU:
    """The device context (class GPU's constructor, gpu.cpp:31-42)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().vc4_gpu_create(device, C.byref(h)))
        self._h = h

    def sync(self):
        _check(lib().vc4_gpu_sync(self._h))

    def close(self):
        if self._h:
            lib().vc4_gpu_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """An uploaded container (Model::load + GPU::upload)."""

    def __init__(self, gpu: GPU, path: str = None, data: bytes = None):
        h = C.c_void_p()
        if data is not None:
            buf = C.create_string_buffer(data, len(data))
            _check(lib().vc4_model_load_bytes(gpu._h, buf, len(data), C.byref(h)))
        else:
            _check(lib().vc4_model_load(gpu._h, path.encode(), C.byref(h)))
        self._h = h
        self.gpu = gpu
        self.info = ModelInfo()
        _check(lib().vc4_model_info_get(h, C.byref(self.info)))

    def matvec_s(self, which, x, layer: int = 0, expert: int = 0):
        """GPU::matvec_s (gpu_conv.cpp:271-287) of one model matrix."""
        w = MATS[which] if isinstance(which, str) else int(which)
        x = np.ascontiguousarray(x, np.float32)
        rows = {0: self.info.dim + 2 * self.info.kv_dim, 1: self.info.dim, 2: self.info.ffn_width,
                3: self.info.ffn_width, 4: self.info.dim, 5: self.info.experts, 6: self.info.vocab}[w]
        out = np.empty(rows, np.float32)
        _check(lib().vc4_matvec_s(self._h, w, layer, expert, _p(x), _p(out)))
        return out

    def close(self):
        if self._h:
            lib().vc4_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """Decode state for `slots` independent sequences over one model."""

    def __init__(self, model: Model, slots: int = 1, seq: int = 0, kv: str = "q16", rope=None):
        kv_bits = {"q16": 16, "q8": 8, 16: 16, 8: 8}[kv]
        h = C.c_void_p()
        if rope is not None:
            c = np.ascontiguousarray(rope[0], np.float32)
            s = np.ascontiguousarray(rope[1], np.float32)
            _check(lib().vc4_session_create(model._h, slots, seq, kv_bits, _p(c), _p(s), C.byref(h)))
        else:
            _check(lib().vc4_session_create(model._h, slots, seq, kv_bits, None, None, C.byref(h)))
        self._h = h
        self.model = model
        self.slots = slots
        self.kv_bits = kv_bits
        self.vocab = model.info.vocab
        self.seq = seq or model.info.seq

    # -- the reference's per-token calls ------------------------------------
    def step(self, token: int, pos: int, want_logits: bool = True, slot: int = 0):
        out = np.empty(self.vocab, np.float32) if want_logits else None
        _check(lib().vc4_step(self._h, slot, int(token), int(pos), _p(out) if want_logits else None))
        return out

    def step_greedy(self, token: int, pos: int, slot: int = 0) -> int:
        t = C.c_int()
        _check(lib().vc4_step_greedy(self._h, slot, int(token), int(pos), C.byref(t)))
        return t.value

    def step_batch(self, slots, tokens, pos, want_logits: bool = False):
        slots = np.ascontiguousarray(slots, np.int32)
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        n = len(slots)
        nxt = np.empty(n, np.int32)
        lg = np.empty((n, self.vocab), np.float32) if want_logits else None
        _check(lib().vc4_step_batch(self._h, n, _p(slots), _p(tokens), _p(pos), _p(nxt),
                                    _p(lg) if want_logits else None))
        return (nxt, lg) if want_logits else nxt

    def step_batch_device(self, n: int, d_slots: int, d_tokens: int, d_pos: int, d_next: int, advance: bool):
        """Enqueue one pass over device arrays (raw device pointers as ints)."""
        _check(lib().vc4_step_batch_device(self._h, n, C.c_void_p(d_slots), C.c_void_p(d_tokens),
                                           C.c_void_p(d_pos), C.c_void_p(d_next), 1 if advance else 0))

    def stream(self) -> int:
        return lib().vc4_session_stream(self._h) or 0

    def check(self) -> None:
        """Raise if a device-resident pass failed a kernel self-check."""
        _check(lib().vc4_session_check(self._h))

    def prefill(self, tokens, pos0: int = 0, slot: int = 0, want_logits: bool = True, batched: bool = False):
        """The prompt's positions pos0.. on `slot`; returns the last
        position's logits.  batched=True runs them as batches of the
        many-sequence path (vc4_prefill_batch), with the serial loop's results."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.vocab, np.float32) if want_logits else None
        fn = lib().vc4_prefill_batch if batched else lib().vc4_prefill
        _check(fn(self._h, slot, _p(t), len(t), pos0, _p(out) if want_logits else None))
        return out

    def prefill_logits(self, tokens, pos0: int = 0, slot: int = 0):
        """Batched prefill returning every position's logits (len x vocab)."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((len(t), self.vocab), np.float32)
        _check(lib().vc4_prefill_logits(self._h, slot, _p(t), len(t), pos0, _p(out)))
        return out

    # -- KV rows and the MMKV1 prefix cache ---------------------------------
    def kv_row_bytes(self) -> int:
        return lib().vc4_kv_row_bytes(self._h)

    def kv_rows(self, layer: int, n: int, slot: int = 0) -> bytes:
        buf = np.empty(n * self.kv_row_bytes(), np.uint8)
        _check(lib().vc4_kv_read_rows(self._h, slot, layer, n, _p(buf)))
        return buf.tobytes()

    def kv_write(self, layer: int, n: int, data: bytes, slot: int = 0) -> None:
        buf = np.frombuffer(data, np.uint8).copy()
        _check(lib().vc4_kv_write_rows(self._h, slot, layer, n, _p(buf)))

    def save_prefix_cache(self, path: str, toks, slot: int = 0, system_fnv: int = 0, tools_fnv: int = 0):
        t = np.ascontiguousarray(toks, np.int32)
        _check(lib().vc4_save_prefix_cache(self._h, slot, path.encode(), _p(t), len(t), system_fnv, tools_fnv))

    def build_prefix_cache(self, path: str, toks, slot: int = 0, system: str = None, tools: str = None):
        """`--build-prefix-cache` (prefix_build.cpp:22-83) for a tokenised
        prompt: prefill `toks` on `slot` from position 0, then write the
        MMKV1 file and its sidecar.  `system` / `tools` are the raw texts
        whose FNV-1a-64 the sidecar records (0 when absent, as for a prompt
        file)."""
        t = np.ascontiguousarray(toks, np.int32)
        sf = fnv64(system.encode()) if system is not None else 0
        tf = fnv64(tools.encode()) if tools is not None else 0
        _check(lib().vc4_build_prefix_cache(self._h, slot, _p(t), len(t), path.encode(), sf, tf))

    def load_prefix_cache(self, path: str, slot: int = 0):
        buf = np.empty(self.seq, np.int32)
        n = C.c_int()
        _check(lib().vc4_load_prefix_cache(self._h, slot, path.encode(), _p(buf), len(buf), C.byref(n)))
        return [int(v) for v in buf[:n.value]]

    def load_prefix_cache_shared(self, path: str, slots):
        """Restore one MMKV1 prefix into every slot of `slots`, held once on
        the device (vc4_load_prefix_cache_shared); returns its tokens."""
        sl = np.ascontiguousarray(slots, np.int32)
        buf = np.empty(self.seq, np.int32)
        n = C.c_int()
        _check(lib().vc4_load_prefix_cache_shared(self._h, path.encode(), _p(sl), len(sl), _p(buf), len(buf),
                                                  C.byref(n)))
        return [int(v) for v in buf[:n.value]]

    def counters(self):
        a, b = C.c_longlong(), C.c_longlong()
        _check(lib().vc4_counters(self._h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def launches_per_step(self, n: int = 1) -> int:
        return lib().vc4_launches_per_step(self._h, n)

    def close(self):
        if self._h:
            lib().vc4_session_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def log_prob(logits, token: int) -> float:
    """log softmax(logits)[token] in double, as run_ppl sums it
    (ppl.cpp:66-71): max, sum of exp(v - max), (l[token] - max) - log(sum)."""
    v = np.asarray(logits, np.float64)
    mx = float(v.max())
    return (float(v[token]) - mx) - float(np.log(np.exp(v - mx).sum()))


def perplexity(session: "Session", tokens, span: int = 0, stride: int = -1, slot: int = 0,
               scorer=None) -> dict:
    """`--ppl` (ppl.cpp:23-88): windows of `span` positions (the session's
    sequence length by default) advancing by `stride` (span/2 by default; 0:
    cold windows of span-1), each window restarted at position 0 with
    span - stride tokens of context.  Context positions are prefilled in
    batches; every scored position's logits come from one batched pass
    (vc4_prefill_logits), which equals Session::step position by position.
    `scorer(window_tokens, first_scored)` replaces the session (for a CPU
    check); it returns the logits of positions first_scored.. of the window."""
    tokens = [int(t) for t in tokens]
    if len(tokens) < 4:
        raise EngineError("not enough tokens")
    span = span or session.seq
    stride = span // 2 if stride < 0 else stride
    stride = max(stride, 0) or span - 1
    stride = min(stride, span - 1)
    warm = span - stride
    n, nxt, windows, nll, cnt = len(tokens), 1, 0, 0.0, 0
    while nxt < n:
        a = 0 if windows == 0 else nxt - warm
        ln = min(span, n - a)
        if ln < 2 or a < 0:
            break
        win = tokens[a:a + ln]
        first = max(0, nxt - a - 1)          # positions before this one predict tokens already scored
        if scorer is not None:
            lg = scorer(win[:ln - 1], first)
        else:
            if first:
                session.prefill(win[:first], 0, slot=slot, want_logits=False, batched=True)
            lg = session.prefill_logits(win[first:ln - 1], first, slot=slot)
        for j in range(first, ln - 1):
            t = a + j + 1
            nll += -log_prob(lg[j - first], tokens[t])
            cnt += 1
            nxt = t + 1
        windows += 1
    if not cnt:
        raise EngineError("no tokens scored")
    return {"ppl": float(np.exp(nll / cnt)), "nll": nll / cnt, "tokens": cnt, "windows": windows,
            "span": span, "stride": stride}


def fnv64(data: bytes) -> int:
    """FNV-1a-64 over bytes (common.cpp:63-67): the sidecar's system_fnv64
    and tools_fnv64."""
    h = 1469598103934665603
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def generate(session: Session, prompt, steps: int, slot: int = 0):
    """Prompt positions through vc4_prefill, then greedy decode; returns
    (tokens, logits per decode step), logits[i] having produced tokens[i]."""
    pos = len(prompt) - 1
    if len(prompt) > 1:
        session.prefill(prompt[:-1], 0, slot=slot, want_logits=False)
    tok = prompt[-1]
    toks, logs = [], []
    for _ in range(steps):
        lg = session.step(tok, pos, slot=slot)
        pos += 1
        tok = int(np.argmax(lg))
        toks.append(tok)
        logs.append(lg)
    return toks, np.stack(logs)
