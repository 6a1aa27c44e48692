"""vc4b200: the B200-native quantized decode path of the vc4-gles2-inference
engine (q8/q4/t3 matvecs with fused dequantisation, GQA attention over the
packed q16/q8 KV cache, RMSNorm/QK-norm/RoPE/SwiGLU/top-1 MoE glue), behind
the C ABI in include/vc4b200.h.
"""
from .engine import (EngineError, GPU, Model, ModelInfo, Session, generate, lib, perplexity, probe,  # noqa: F401
                     rope_tables, LIB_PATH, MATS)
from . import synth, mmcf_writer  # noqa: F401
