"""MMCF container writer for the synthetic models (the benchmark's input producer).

The reference packs containers with engine/tools/mmcf_pack.py; that script is
not available on the GPU host, so this module writes the same byte layout from
the same float tensors.  What has to be alike is alike by necessity -- the
container format (docs/checkpoint-container.md), the quantisers' arithmetic
(mmcf_hf.py qmat/q8mat/q4mat/t3mat, lines 51-165) and the record order
(mmcf_hf.py tensors_from_hf, lines 1658-2013; mmcf_pack.py build, 284-432) --
and tests/test_oracle_pins.py::test_writer_matches_reference_packer checks
the output against the reference packer's bytes (sha256 recorded by
tests/golden/make_golden.py).  The q4 quantiser follows mmcf_hf.py q4mat
expression for expression: the byte contract leaves no freedom there.

The rail calibration pass the reference packer runs (metadata key 15, written
only when a model's SwiGLU hidden exceeds the q16 rail) is not restated: the
synthetic models never reach the rail, which the recorded digests confirm.
"""
from __future__ import annotations

import struct
import zlib

import numpy as np

from . import synth

MAGIC = b"MMCF"
HEADER_SIZE = 64
ALIGN = 16
LOGITS_GRID = 1536

DT_F32, DT_I16, DT_Q8U8, DT_Q8I8, DT_Q4, DT_T3 = 0, 1, 2, 3, 4, 7
K_EMB, K_EMB_SCALE, K_RMS_ATT, K_RMS_FFN, K_RMS_FINAL, K_QN, K_KN = 1, 2, 3, 4, 5, 6, 7
K_QKV, K_WO, K_W1, K_W3, K_W2, K_ROUTER, K_LOGITS = 0x10, 0x11, 0x12, 0x13, 0x15, 0x16, 0x20


# ---- quantisers --------------------------------------------------------------
# numpy 2 promotes a Python float against a float32 array to float32, so every
# "array / scale" below runs in float32 exactly as the reference's expressions do.

def _i16(w):
    w = np.asarray(w, np.float32)
    mx = float(np.abs(w).max())
    if mx == 0:
        mx = 1.0
    s = mx / 32767.0
    return np.clip(np.rint(w / s), -32767, 32767).astype(np.int16), s


def _q8(w):
    w = np.asarray(w, np.float32)
    mx = float(np.abs(w).max())
    if mx == 0:
        mx = 1.0
    s = mx / 127.0
    return np.clip(np.rint(w / s), -127, 127).astype(np.int8), s


def _q8_via_i16(w):
    q, s = _i16(w)
    return _q8(q.astype(np.float32) * s)


def _q8_rows(w, via_i16):
    """Per-row q8 of an embedding: one (levels, scale) per row, row by row."""
    w = np.asarray(w, np.float32)
    lev = np.empty(w.shape, np.int8)
    sc = np.empty(w.shape[0], np.float32)
    for i in range(w.shape[0]):
        lev[i], sc[i] = _q8_via_i16(w[i]) if via_i16 else _q8(w[i])
    return lev, sc


def _q8_per_row(w):
    """--q8-row-scale: one scale per output row (max|w|/127, zero rows 1),
    levels rint(w/s) clipped to +-127; the record carries the largest row
    scale and part 3 the row scales relative to it (mmcf_hf.py q8_per_row)."""
    w = np.asarray(w, np.float32)
    s = np.abs(w).max(axis=1, keepdims=True) / np.float32(127.0)
    s[s == 0] = 1.0
    q = np.clip(np.rint(w / s), -127, 127).astype(np.int8)
    unit = float(s.max())
    return q, unit, (s[:, 0] / np.float32(unit)).astype(np.float32)


def _q4(w):
    w = np.asarray(w, np.float32)
    rows, cols = w.shape
    if cols % 32:
        raise ValueError("q4 needs cols divisible by 32: %dx%d" % (rows, cols))
    groups = cols // 32
    z = w.reshape(rows, groups, 32)
    lo = z.min(axis=2, keepdims=True)
    hi = z.max(axis=2, keepdims=True)
    sc = (hi - lo) / 15.0
    sc[sc == 0] = 1.0
    nib = np.clip(np.rint((z - lo) / sc), 0, 15).astype(np.uint8).reshape(rows, cols)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    gsc, glo = sc[:, :, 0], lo[:, :, 0]
    ps = float(max(np.abs(gsc).max(), np.abs(glo).max(), 1e-12) / 32767.0)
    s16 = np.clip(np.rint(gsc / ps), -32767, 32767).astype("<i2")
    m16 = np.clip(np.rint(glo / ps), -32767, 32767).astype("<i2")
    return packed, s16, m16, ps, groups


def _t3(w):
    """Per-row ternary to the 2-bit texel grid: texel (c, t) holds rows 2t, 2t+1
    by columns 8c..8c+7, bit 0 magnitude, bit 1 sign."""
    w = np.asarray(w, np.float32)
    rows, cols = w.shape
    a = np.abs(w)
    mx = a.max(axis=1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        rel = np.abs(a - mx) / np.maximum(mx, 1e-30)
    if not ((a == 0) | (rel <= 1e-3)).all():
        raise ValueError("matrix is not per-row ternary")
    s = a.max(axis=1) / 127.0
    s[s == 0] = 1.0
    lev = np.rint(w / (s[:, None] * 127.0))
    code = (np.abs(lev) > 0.5).astype(np.uint8) | ((lev < -0.5).astype(np.uint8) << 1)
    code = np.pad(code, ((0, rows % 2), (0, (-cols) % 8)))
    r2, c2 = code.shape
    q = code.reshape(r2 // 2, 2, c2 // 8, 2, 4)
    b = q[..., 0] | (q[..., 1] << 2) | (q[..., 2] << 4) | (q[..., 3] << 6)
    body = b.transpose(0, 2, 1, 3).reshape(r2 // 2, -1).astype(np.uint8)
    unit = float(s.max())
    return body.tobytes(), unit, (s / unit).astype(np.float32)


# ---- records ----------------------------------------------------------------

class _Records:
    def __init__(self, scheme, q8_row=False):
        self.scheme = scheme
        self.q8_row = q8_row
        self.items = []      # (id, dtype, rows, cols, group, payload, scale, aux)

    def add(self, tid, dt, rows, cols, group, payload, scale, aux=0):
        self.items.append((tid, dt, rows, cols, group, payload, float(scale), aux))

    def matrix(self, kind, layer, w, aux=0):
        w = np.asarray(w, np.float32)
        rows, cols = w.shape
        base = kind | (layer << 8)
        if self.scheme == "q8" and self.q8_row:
            q, unit, plane = _q8_per_row(w)
            self.add(base, DT_Q8I8, rows, cols, 0, q.tobytes(), unit, aux)
            self.add(base | (3 << 14), DT_F32, rows, 1, 0, (plane / np.float32(1.0)).astype("<f4").tobytes(), 0.0, aux)
        elif self.scheme == "q8":
            q, s = _q8_via_i16(w)
            self.add(base, DT_Q8I8, rows, cols, 0, q.tobytes(), s, aux)
        elif self.scheme == "t3":
            body, unit, plane = _t3(w)
            self.add(base, DT_T3, rows, cols, 0, body, unit, aux)
            self.add(base | (3 << 14), DT_F32, rows, 1, 0, plane.astype("<f4").tobytes(), 0.0, aux)
        elif self.scheme == "q4":
            packed, s16, m16, ps, groups = _q4(w)
            self.add(base, DT_Q4, rows, cols, 32, packed.tobytes(), ps, aux)
            self.add(base | (1 << 14), DT_I16, rows, groups, 0, s16.tobytes(), 0.0, aux)
            self.add(base | (2 << 14), DT_I16, rows, groups, 0, m16.tobytes(), 0.0, aux)
        else:
            raise ValueError("scheme " + self.scheme)


def _tlv(key, payload):
    return struct.pack("<HHI", key, 1, len(payload)) + payload


def pack(shape: synth.Shape, tensors: dict, scheme: str, seq: int, *,
         head_dedup: bool = False, rms_eps: float = 1e-6, q8_row: bool = False) -> bytes:
    """Build the container bytes the reference packer writes for
    `mmcf_pack.py --in DIR --quant SCHEME --seq SEQ --rms-eps 1e-6
    --template plain [--head-dedup] [--q8-row-scale]`."""
    f32 = lambda name: np.asarray(tensors[name], np.float32)   # noqa: E731
    s = shape
    moe = s.experts > 0
    ffn_w = s.moe_hidden if moe else s.hidden
    split = 1 if (moe or 2 * ffn_w > 2048) else 0
    if not split:
        raise ValueError("fused-W13 containers are not produced by this writer")
    recs = _Records(scheme, q8_row=q8_row)
    emb = f32("model.embed_tokens.weight")
    lev, es = _q8_rows(emb, via_i16=(scheme == "q8"))
    recs.add(K_EMB, DT_Q8I8, s.vocab, s.dim, 0, lev.tobytes(), 0.0)
    recs.add(K_EMB_SCALE, DT_F32, s.vocab, 1, 0, es.tobytes(), 0.0)
    stack = lambda fmt: np.stack([f32(fmt % l) for l in range(s.layers)])   # noqa: E731
    recs.add(K_RMS_ATT, DT_F32, s.layers, s.dim, 0, stack("model.layers.%d.input_layernorm.weight").tobytes(), 0.0)
    recs.add(K_RMS_FFN, DT_F32, s.layers, s.dim, 0, stack("model.layers.%d.post_attention_layernorm.weight").tobytes(), 0.0)
    recs.add(K_RMS_FINAL, DT_F32, 1, s.dim, 0, f32("model.norm.weight").tobytes(), 0.0)
    if s.qk_norm:
        recs.add(K_QN, DT_F32, s.layers, s.head_dim, 0, stack("model.layers.%d.self_attn.q_norm.weight").tobytes(), 0.0)
        recs.add(K_KN, DT_F32, s.layers, s.head_dim, 0, stack("model.layers.%d.self_attn.k_norm.weight").tobytes(), 0.0)
    for l in range(s.layers):
        p = "model.layers.%d." % l
        qkv = np.concatenate([f32(p + "self_attn.q_proj.weight"), f32(p + "self_attn.k_proj.weight"),
                              f32(p + "self_attn.v_proj.weight")], axis=0)
        recs.matrix(K_QKV, l, qkv)
        recs.matrix(K_WO, l, f32(p + "self_attn.o_proj.weight"))
        if moe:
            q, sc = _i16(f32(p + "mlp.gate.weight"))
            recs.add(K_ROUTER | (l << 8), DT_I16, s.experts, s.dim, 0, q.astype("<i2").tobytes(), sc)
            for e in range(s.experts):
                x = p + "mlp.experts.%d." % e
                recs.matrix(K_W1, l, f32(x + "gate_proj.weight"), aux=e)
                recs.matrix(K_W3, l, f32(x + "up_proj.weight"), aux=e)
                recs.matrix(K_W2, l, f32(x + "down_proj.weight"), aux=e)
        else:
            recs.matrix(K_W1, l, f32(p + "mlp.gate_proj.weight"))
            recs.matrix(K_W3, l, f32(p + "mlp.up_proj.weight"))
            recs.matrix(K_W2, l, f32(p + "mlp.down_proj.weight"))
    if not head_dedup:
        for i, st in enumerate(range(0, s.vocab, LOGITS_GRID)):
            w = emb[st:st + LOGITS_GRID]
            if scheme == "q4":
                q, sc = _q8(w)
                recs.add(K_LOGITS | (i << 8), DT_Q8I8, w.shape[0], w.shape[1], 0, q.tobytes(), sc)
            else:
                recs.matrix(K_LOGITS, i, w)

    model = struct.pack("<7i", s.dim, s.hidden, s.layers, s.heads, s.kv_heads, s.vocab, seq)
    rope = struct.pack("<fBBH", float(s.theta), 1, 1 if s.qk_norm else 0, 0)
    quant = struct.pack("<BBBB", {"q8": 1, "q4": 2, "t3": 3}[scheme], 32 if scheme == "q4" else 0, 1, split)
    template = bytes([0]) + b"You are a helpful assistant.\0plain\0"
    md = (_tlv(1, model) + _tlv(2, rope) + _tlv(3, quant) + _tlv(4, template) +
          _tlv(5, struct.pack("<I", 0)) + _tlv(6, b"model\0"))
    md += _tlv(11, struct.pack("<f", rms_eps))
    if moe:
        md += _tlv(13, struct.pack("<4i", s.experts, 1, s.moe_hidden, 1))

    version = 3 if moe else 2
    rsize = 64 if version >= 3 else 48
    table_off = HEADER_SIZE + len(md)
    table_off = (table_off + ALIGN - 1) // ALIGN * ALIGN
    data_off = table_off + len(recs.items) * rsize
    table, data = bytearray(), bytearray()
    for tid, dt, rows, cols, group, payload, scale, aux in recs.items:
        if dt == DT_Q8I8 and (tid & 0xFF) != K_EMB:      # texture tensors are stored +128
            payload = (np.frombuffer(payload, np.uint8) ^ 0x80).tobytes()
            dt = DT_Q8U8
        data += b"\0" * ((-(data_off + len(data))) % ALIGN)
        off = len(data)
        data += payload
        rec = struct.pack("<HBBBB", tid, dt, 0, group, 0) + struct.pack("<II", rows, cols)
        rec += struct.pack("<QQ", off, len(payload)) + struct.pack("<I", zlib.crc32(payload) & 0xFFFFFFFF)
        rec += struct.pack("<f", scale) + struct.pack("<H", aux)
        table += rec[:rsize] + b"\0" * max(0, rsize - len(rec))
    file_size = data_off + len(data)
    body = MAGIC + struct.pack("<HHIIIIQQ", version, HEADER_SIZE, len(recs.items), 0,
                               HEADER_SIZE, len(md), data_off, file_size)
    head = (body + struct.pack("<I", zlib.crc32(body) & 0xFFFFFFFF)).ljust(HEADER_SIZE, b"\0")
    out = bytearray(head) + md
    out += b"\0" * (table_off - len(out))
    out += table
    out += data
    return bytes(out)


def pack_config(cfg: synth.Config) -> bytes:
    return pack(cfg.shape, synth.hf_tensors(cfg.shape, cfg.seed), cfg.quant, cfg.seq,
                head_dedup=cfg.head_dedup, q8_row=bool(cfg.extra.get("q8_row")))


def write_config(cfg: synth.Config, path: str) -> str:
    data = pack_config(cfg)
    with open(path, "wb") as f:
        f.write(data)
    return path
