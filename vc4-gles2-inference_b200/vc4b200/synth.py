"""Seeded synthetic models for the five benchmark configurations and the tiny
parity models.

No checkpoint or dataset is available here, so every model is random-init with
the architecture of the configuration it stands for: MiniMind3-64M (dense and
MoE) with N(0, 0.02) weights and unit norms, and a BitCPM-shaped ternary
decoder whose linear weights are U{-1, 0, +1} times a per-row scale from
U(0.01, 0.05).  Tensors use the HuggingFace names and float16 storage, which
is what the reference packer (engine/tools/mmcf_hf.py load_minimind, lines
907-1044) reads from a model directory.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class Shape:
    name: str
    dim: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    vocab: int
    theta: float
    qk_norm: bool
    experts: int = 0
    moe_hidden: int = 0
    ternary: bool = False

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads


MM3 = Shape("minimind3-64m", 768, 2432, 8, 8, 4, 6400, 1e6, True)
MM3_MOE = Shape("minimind3-moe", 768, 2432, 8, 8, 4, 6400, 1e6, True, experts=4, moe_hidden=2432)
BITCPM = Shape("bitcpm-0.5b", 1024, 4096, 24, 16, 2, 73448, 10000.0, False, ternary=True)

# Parity models: the same code paths (split FFN, two chunks above 2048 rows,
# several logits tiles, GQA, qk-norm) at a size the oracle runs in seconds.
TINY = Shape("tiny", 64, 2112, 2, 4, 2, 1600, 1e6, True)
TINY_FLAT = Shape("tiny-unchunked", 64, 1056, 2, 4, 2, 1600, 1e6, True)
TINY_MOE = Shape("tiny-moe", 64, 2112, 2, 4, 2, 1600, 1e6, True, experts=4, moe_hidden=2112)
TINY_T3 = Shape("tiny-t3", 64, 2112, 2, 4, 1, 3100, 10000.0, False, ternary=True)


@dataclass
class Config:
    """One benchmark or parity configuration: model + quantisation + workload."""
    key: str
    shape: Shape
    quant: str            # q8 | q4 | t3
    kv_bits: int          # 16 | 8
    seq: int
    prompt: int
    steps: int
    batch: int = 1
    head_dedup: bool = False
    seed: int = 1234
    extra: dict = field(default_factory=dict)


CONFIGS = {
    "c0": Config("c0", MM3, "q8", 16, 256, 128, 64),
    "c1": Config("c1", MM3, "q4", 16, 256, 128, 64),
    # config 0 with one q8 scale per output row (the packer's --q8-row-scale,
    # BASELINE's "per-row symmetric int8 + f32 scale" wording)
    "c0r": Config("c0r", MM3, "q8", 16, 256, 128, 64, extra={"q8_row": True}),
    "c2": Config("c2", MM3_MOE, "q4", 8, 512, 256, 128, batch=64),
    "c3": Config("c3", BITCPM, "t3", 16, 1024, 512, 128, head_dedup=True),
    "c3b32": Config("c3b32", BITCPM, "t3", 16, 1024, 512, 128, batch=32, head_dedup=True),
    # config 4: one 512-token prefix prefilled once and restored into every
    # sequence slot (MMKV1), swept over the sequences per GPU
    "c4": Config("c4", MM3, "q8", 8, 768, 512, 256, batch=16, extra={"prefix_restore": True}),
    "c4b1": Config("c4b1", MM3, "q8", 8, 768, 512, 256, batch=1, extra={"model": "c4", "prefix_restore": True}),
    "c4b128": Config("c4b128", MM3, "q8", 8, 768, 512, 256, batch=128, extra={"model": "c4", "prefix_restore": True}),
    "c4b1024": Config("c4b1024", MM3, "q8", 8, 768, 512, 256, batch=1024,
                      extra={"model": "c4", "prefix_restore": True}),
}

TINY_CONFIGS = {
    "tiny_q8": Config("tiny_q8", TINY, "q8", 16, 64, 24, 16, seed=7),
    "tiny_q4": Config("tiny_q4", TINY, "q4", 16, 64, 24, 16, seed=8),
    "tiny_flat_q8": Config("tiny_flat_q8", TINY_FLAT, "q8", 8, 64, 24, 16, seed=9),
    "tiny_moe_q4": Config("tiny_moe_q4", TINY_MOE, "q4", 8, 64, 24, 16, seed=10),
    "tiny_t3": Config("tiny_t3", TINY_T3, "t3", 16, 64, 24, 16, head_dedup=True, seed=11),
}


def hf_config(s: Shape, seq: int) -> dict:
    """config.json for the synthetic model (a Qwen3 / Qwen3-MoE / Llama block)."""
    cfg = {
        "architectures": ["Qwen3ForCausalLM"],
        "model_type": "qwen3",
        "hidden_size": s.dim,
        "intermediate_size": s.hidden,
        "num_hidden_layers": s.layers,
        "num_attention_heads": s.heads,
        "num_key_value_heads": s.kv_heads,
        "head_dim": s.head_dim,
        "vocab_size": s.vocab,
        "rope_theta": s.theta,
        "rms_norm_eps": 1e-6,
        "hidden_act": "silu",
        "tie_word_embeddings": True,
        "max_position_embeddings": max(seq, 2048),
    }
    if s.experts:
        cfg.update({"architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
                    "num_experts": s.experts, "num_experts_per_tok": 1,
                    "norm_topk_prob": True, "moe_intermediate_size": s.moe_hidden,
                    "decoder_sparse_step": 1, "mlp_only_layers": []})
    if s.ternary:
        cfg.update({"architectures": ["LlamaForCausalLM"], "model_type": "llama"})
    return cfg


def _ternary(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    lev = rng.integers(-1, 2, size=(rows, cols), dtype=np.int8)
    scale = rng.uniform(0.01, 0.05, size=rows).astype(np.float16)
    return lev.astype(np.float16) * scale[:, None]


def hf_tensors(s: Shape, seed: int) -> dict:
    """name -> float16 array, drawn in a fixed order from one seeded generator."""
    rng = np.random.default_rng(seed)
    hd, kvd = s.head_dim, s.kv_heads * s.head_dim

    def mat(rows, cols):
        if s.ternary:
            return _ternary(rng, rows, cols)
        return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)).astype(np.float16)

    t = {"model.embed_tokens.weight": mat(s.vocab, s.dim)}
    ones = np.ones(s.dim, np.float16)
    for l in range(s.layers):
        p = f"model.layers.{l}."
        t[p + "self_attn.q_proj.weight"] = mat(s.dim, s.dim)
        t[p + "self_attn.k_proj.weight"] = mat(kvd, s.dim)
        t[p + "self_attn.v_proj.weight"] = mat(kvd, s.dim)
        t[p + "self_attn.o_proj.weight"] = mat(s.dim, s.dim)
        if s.qk_norm:
            t[p + "self_attn.q_norm.weight"] = np.ones(hd, np.float16)
            t[p + "self_attn.k_norm.weight"] = np.ones(hd, np.float16)
        if s.experts:
            t[p + "mlp.gate.weight"] = mat(s.experts, s.dim)
            for e in range(s.experts):
                q = p + f"mlp.experts.{e}."
                t[q + "gate_proj.weight"] = mat(s.moe_hidden, s.dim)
                t[q + "up_proj.weight"] = mat(s.moe_hidden, s.dim)
                t[q + "down_proj.weight"] = mat(s.dim, s.moe_hidden)
        else:
            t[p + "mlp.gate_proj.weight"] = mat(s.hidden, s.dim)
            t[p + "mlp.up_proj.weight"] = mat(s.hidden, s.dim)
            t[p + "mlp.down_proj.weight"] = mat(s.dim, s.hidden)
        t[p + "input_layernorm.weight"] = ones.copy()
        t[p + "post_attention_layernorm.weight"] = ones.copy()
    t["model.norm.weight"] = ones.copy()
    return t


def write_safetensors(path: str, tensors: dict) -> None:
    """A plain safetensors file (8-byte header length, JSON header, data)."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": "F16", "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def write_hf_dir(path: str, cfg: Config) -> None:
    import os
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config(cfg.shape, cfg.seq), f, indent=1)
    write_safetensors(os.path.join(path, "model.safetensors"), hf_tensors(cfg.shape, cfg.seed))


def prompt_tokens(cfg: Config, seq_index: int = 0) -> list:
    """The seeded prompt of one sequence: ids uniform in [0, vocab)."""
    rng = np.random.default_rng(cfg.seed * 1000003 + 17 + seq_index)
    return [int(v) for v in rng.integers(0, cfg.shape.vocab, size=cfg.prompt)]
