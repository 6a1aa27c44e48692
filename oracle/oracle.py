"""ctypes wrapper over the CPU oracle (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; it is the checker, never the product path.  See vc4_oracle.h for
the arithmetic it restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_loader.so")


class Info(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "dim", "hidden", "layers", "heads", "kv_heads", "vocab", "seq", "head_dim", "kv_dim",
        "qk_norm", "rope_half", "experts", "moe_hidden", "ffn_width", "ffn_chunked", "ffn_chunk",
        "n_logit_tiles", "wtype", "version")] + [("rope_theta", C.c_float), ("rms_eps", C.c_float)]


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, ip = C.c_void_p, C.c_int
        L.orc_model_load.argtypes = [C.c_char_p, C.POINTER(vp), C.c_char_p, ip]
        L.orc_model_free.argtypes = [vp]
        L.orc_model_info.argtypes = [vp, C.POINTER(Info)]
        L.orc_session_new.restype = vp
        L.orc_session_new.argtypes = [vp, ip, ip]
        L.orc_session_free.argtypes = [vp]
        L.orc_step.argtypes = [vp, ip, ip, vp]
        L.orc_argmax.argtypes = [vp, ip]
        L.orc_kv_row_bytes.argtypes = [vp]
        L.orc_kv_read.argtypes = [vp, ip, ip, vp]
        L.orc_kv_write.argtypes = [vp, ip, ip, vp]
        L.orc_last_route.argtypes = [vp, ip]
        L.orc_expf.restype = C.c_float
        L.orc_expf.argtypes = [C.c_float]
        L.orc_set_threads.restype = None
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_q16.restype = C.c_int16
        L.orc_q16.argtypes = [C.c_float]
        L.orc_kv_q16.restype = C.c_int16
        L.orc_kv_q16.argtypes = [C.c_float]
        L.orc_kv_q8.restype = C.c_int8
        L.orc_kv_q8.argtypes = [C.c_float]
        L.orc_scale_input.argtypes = [vp, ip, vp]
        L.orc_rope_tables.argtypes = [C.c_float, ip, ip, vp, vp, vp]
        L.orc_model_matvec.argtypes = [vp, ip, ip, ip, vp, ip, vp]
        L.orc_model_mat_shape.argtypes = [vp, ip, ip, ip, C.POINTER(ip), C.POINTER(ip), C.POINTER(ip),
                                          C.POINTER(C.c_float)]
        L.orc_model_mat_levels.argtypes = [vp, ip, ip, ip, vp]
        L.orc_model_mat_rowscale16.argtypes = [vp, ip, ip, ip, vp]
        L.orc_model_mat_q4params.argtypes = [vp, ip, ip, ip, vp, vp]
        L.orc_model_mat_plane.argtypes = [vp, ip, ip, ip, vp]
        L.orc_model_emb.argtypes = [vp, vp]
        L.orc_model_vec.argtypes = [vp, ip, vp]
        L.orc_fnv1a64.restype = C.c_uint64
        L.orc_fnv1a64.argtypes = [vp, C.c_uint64]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Model:
    def __init__(self, path: str):
        self._h = C.c_void_p()
        err = C.create_string_buffer(256)
        rc = lib().orc_model_load(path.encode(), C.byref(self._h), err, 256)
        if rc != 0:
            raise RuntimeError("oracle load failed (%d): %s" % (rc, err.value.decode()))
        self.info = Info()
        lib().orc_model_info(self._h, C.byref(self.info))

    def close(self):
        if self._h:
            lib().orc_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def mat_shape(self, which, layer=0, expert=0):
        r, c, t, s = C.c_int(), C.c_int(), C.c_int(), C.c_float()
        if lib().orc_model_mat_shape(self._h, which, layer, expert, C.byref(r), C.byref(c), C.byref(t), C.byref(s)):
            raise KeyError((which, layer, expert))
        return r.value, c.value, t.value, s.value

    def mat_levels(self, which, layer=0, expert=0):
        r, c, _, _ = self.mat_shape(which, layer, expert)
        out = np.empty(r * c, np.int32)
        lib().orc_model_mat_levels(self._h, which, layer, expert, _ptr(out))
        return out.reshape(r, c)

    def mat_rowscale16(self, which, layer=0, expert=0):
        r, _, _, _ = self.mat_shape(which, layer, expert)
        out = np.empty(r, np.uint16)
        return out if lib().orc_model_mat_rowscale16(self._h, which, layer, expert, _ptr(out)) == 1 else None

    def mat_q4params(self, which, layer=0, expert=0):
        r, c, _, _ = self.mat_shape(which, layer, expert)
        s16 = np.empty(r * (c // 32), np.int16)
        m16 = np.empty(r * (c // 32), np.int16)
        lib().orc_model_mat_q4params(self._h, which, layer, expert, _ptr(s16), _ptr(m16))
        return s16.reshape(r, -1), m16.reshape(r, -1)

    def mat_plane(self, which, layer=0, expert=0):
        r, _, _, _ = self.mat_shape(which, layer, expert)
        out = np.empty(r, np.float32)
        return out if lib().orc_model_mat_plane(self._h, which, layer, expert, _ptr(out)) == 1 else None

    def emb(self):
        n = lib().orc_model_emb(self._h, None)
        out = np.empty(n, np.int8)
        lib().orc_model_emb(self._h, _ptr(out))
        return out

    def vec(self, which: int):
        n = lib().orc_model_vec(self._h, which, None)
        out = np.empty(max(n, 0), np.float32)
        if n > 0:
            lib().orc_model_vec(self._h, which, _ptr(out))
        return out

    def matvec(self, which, layer, expert, xq: np.ndarray):
        r, _, _, _ = self.mat_shape(which, layer, expert)
        xq = np.ascontiguousarray(xq, np.int16)
        out = np.empty(r, np.int32)
        lib().orc_model_matvec(self._h, which, layer, expert, _ptr(xq), 0, _ptr(out))
        return out


class Session:
    def __init__(self, model: Model, kv_bits: int, literal: bool = False):
        self.model = model
        self._h = lib().orc_session_new(model._h, kv_bits, 1 if literal else 0)
        if not self._h:
            raise RuntimeError("oracle session refused (kv_bits=%d)" % kv_bits)
        self.vocab = model.info.vocab

    def close(self):
        if self._h:
            lib().orc_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def step(self, token: int, pos: int, want_logits: bool = True):
        out = np.empty(self.vocab, np.float32) if want_logits else None
        rc = lib().orc_step(self._h, int(token), int(pos), _ptr(out) if want_logits else None)
        if rc != 0:
            raise RuntimeError("oracle step failed (%d)" % rc)
        return out

    def kv_rows(self, layer: int, n: int) -> bytes:
        rb = lib().orc_kv_row_bytes(self._h)
        buf = np.empty(rb * n, np.uint8)
        lib().orc_kv_read(self._h, layer, n, _ptr(buf))
        return buf.tobytes()

    def kv_write(self, layer: int, n: int, data: bytes) -> None:
        buf = np.frombuffer(data, np.uint8).copy()
        lib().orc_kv_write(self._h, layer, n, _ptr(buf))

    def route(self, layer: int) -> int:
        return lib().orc_last_route(self._h, layer)


def argmax(logits: np.ndarray) -> int:
    """First maximum (sampling.cpp:160-162)."""
    return int(np.argmax(logits))


def generate(model: Model, kv_bits: int, prompt, steps: int, literal: bool = False):
    """Prompt positions serially, then greedy decode; returns (tokens, logits per
    decode step) where logits[i] produced tokens[i]."""
    s = Session(model, kv_bits, literal)
    pos = 0
    for t in prompt[:-1]:
        s.step(t, pos, want_logits=False)
        pos += 1
    tok = prompt[-1]
    toks, logs = [], []
    for _ in range(steps):
        lg = s.step(tok, pos)
        pos += 1
        tok = argmax(lg)
        toks.append(tok)
        logs.append(lg)
    return toks, np.stack(logs), s


def fnv64(a: np.ndarray) -> str:
    """FNV-1a/64 of an array's bytes, as 16 hex digits."""
    a = np.ascontiguousarray(a)
    return "%016x" % lib().orc_fnv1a64(_ptr(a), a.nbytes)


def expf(x: float) -> float:
    return lib().orc_expf(x)


def ref_summary(path: str):
    """The reference loader's decode summary (needs oracle/_ref built here)."""
    import json
    L = C.CDLL(REF_LIB_PATH)
    L.ref_load_summary.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
    cap = 1 << 22
    buf = C.create_string_buffer(cap)
    rc = L.ref_load_summary(path.encode(), buf, cap)
    if rc != 0:
        raise RuntimeError("reference loader failed (%d)" % rc)
    return json.loads(buf.value.decode())


def set_threads(n: int) -> None:
    """Host threads the oracle's row-parallel matvecs use (the launcher's
    OMP_NUM_THREADS otherwise, which torchrun sets to 1)."""
    lib().orc_set_threads(int(n))
