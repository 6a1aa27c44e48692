/*
 * vc4_oracle.h -- CPU oracle for the quantized decode path (TEST INFRASTRUCTURE).
 *
 * This is the checker, not the product.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load it.  It restates, in plain C, the
 * arithmetic of the reference engine's CPU layer loop (engine/src/session.cpp
 * Session::forward, lines 373-556 and the helpers at 1932-2080) with the
 * shader arithmetic the loop draws through (engine/src/shaders.cpp,
 * engine/src/gpu_conv.cpp:227-287, engine/src/gpu_ffn.cpp:67-132) and the
 * packed KV cache codec the GPU path writes (engine/src/shaders_attn.cpp:141-159,
 * grids from engine/src/gpu_attn.cpp:89-92).
 *
 * Canonical arithmetic (both this oracle and the CUDA kernels follow it):
 *   - every weight x activation dot product is an exact integer (int64);
 *     the reference shaders accumulate the same integers in fp32;
 *   - the scale epilogue of a matvec is floor(double(S) * double(scale) + 0.5)
 *     clamped to the q16 rail (the shaders' floor(s*ws+0.5));
 *   - float loops are written out op by op with no fused multiply-add unless
 *     fmaf() is spelled out;
 *   - a query head is put on a power-of-two integer grid (orc_q_grid_exp)
 *     and its score with a cached key is the exact integer dot with the
 *     cache levels, rounded once to float, times the head's constant
 *     fl(2^-F / cache grid / sqrt(head_dim)); the reference sums q*k
 *     sequentially in fp32;
 *   - attention weights are integers E_t = rint(exp(s_t - max) * 2^k) on a grid
 *     fine enough for k to keep every sum of E_t and E_t x (cache level) an
 *     exact integer in double (orc_attn_weight_exp), so the softmax
 *     denominator and P x V are exact and independent of summation order; the
 *     output is rint(float(num / den * c)) on the q16 grid (ties to even);
 *   - exp() is orc_expf(), a Cody-Waite range reduction with a degree-7
 *     Taylor polynomial (see vc4_oracle.c), identical op for op in the kernels.
 * ORC_LITERAL selects the reference's literal float orders instead (sequential
 * fp32 sums, libm expf, fp32 shader accumulation) for the documented
 * comparison between the two.
 */
#ifndef VC4_ORACLE_H
#define VC4_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_OK = 0, ORC_EIO = 1, ORC_EFORMAT = 2, ORC_EUNSUPPORTED = 3, ORC_EARG = 4 };
enum { ORC_W_Q8 = 0, ORC_W_Q4 = 1, ORC_W_T3 = 2, ORC_W_I16 = 3 };

typedef struct orc_model orc_model;
typedef struct orc_session orc_session;

/* Model description (filled by orc_model_info). */
typedef struct {
    int dim, hidden, layers, heads, kv_heads, vocab, seq, head_dim, kv_dim;
    int qk_norm, rope_half, experts, moe_hidden, ffn_width, ffn_chunked, ffn_chunk;
    int n_logit_tiles, wtype, version;
    float rope_theta, rms_eps;
} orc_info;

int orc_model_load(const char* path, orc_model** out, char* err, int errlen);
void orc_model_free(orc_model* m);
int orc_model_info(const orc_model* m, orc_info* info);

/* Rope tables exactly as Session::reset builds them (session.cpp:188-202). */
void orc_rope_tables(float theta, int head_dim, int seq, const float* factors,
                     float* cos_out, float* sin_out);

/* A decode session.  kv_bits is 16 or 8 (the KV axis).  literal: 0 the
   canonical arithmetic, ORC_LITERAL the reference's literal float orders with
   the packed KV cache, ORC_LITERAL_FLOAT_KV the literal orders with the
   reference CPU path's float K/V cache (session.cpp:446-447; the packed rows
   are then not kept). */
enum { ORC_CANONICAL = 0, ORC_LITERAL = 1, ORC_LITERAL_FLOAT_KV = 2 };
orc_session* orc_session_new(const orc_model* m, int kv_bits, int literal);
void orc_session_free(orc_session* s);
/* One position through the layer loop.  logits (vocab floats, q16 grid) may be
   NULL when the caller needs no logits (prompt positions). Returns ORC_OK. */
int orc_step(orc_session* s, int token, int pos, float* logits);
/* Greedy argmax with the first-maximum rule (sampling.cpp:160-162). */
int orc_argmax(const float* logits, int n);
/* Bytes of one packed KV row (K then V) of one layer: the MMKV1 texel row. */
int orc_kv_row_bytes(const orc_session* s);
int orc_kv_read(const orc_session* s, int layer, int n, uint8_t* out);
int orc_kv_write(orc_session* s, int layer, int n, const uint8_t* in);
/* Per-layer MoE routes of the last step (experts == 0: returns -1). */
int orc_last_route(const orc_session* s, int layer);

/* ---- primitives, for kernel unit tests ---- */
float orc_expf(float x);
/* Host threads of the row-parallel matvecs (OpenMP); <= 0 leaves the default. */
void orc_set_threads(int n);
/* matvec_s input scaling (gpu_conv.cpp:271-287): returns k, fills xq. */
int orc_scale_input(const float* x, int n, int16_t* xq);
/* q16 host quantisation (common.h:188-193). */
int16_t orc_q16(float v);
/* KV codec: q16 grid 1/2048 big-endian, q8 grid 1/16. */
int16_t orc_kv_q16(float v);
int8_t orc_kv_q8(float v);
/* Exponent F of a query head's integer grid for max|q| = qmax: 22 - e with
   qmax = f * 2^e, f in [0.5, 1), clamped to [-100, 100]. */
int orc_q_grid_exp(float qmax);
/* Exponent k of the attention weights' grid for len positions and the cache
   width: 53 - (7 for q8, 15 for q16) - ceil(log2 len). */
int orc_attn_weight_exp(int len, int kv_bits);
/* One matvec of a model matrix over q16 ints.  k is the power-of-two input
   scale already applied to xq (folded into the epilogue as 2^k); out receives
   the clamped q16 integers.  which: 0 qkv, 1 wo, 2 w1, 3 w3, 4 w2, 5 router,
   6 logits tile (layer = tile index), expert selects an MoE expert. */
int orc_model_matvec(const orc_model* m, int which, int layer, int expert,
                     const int16_t* xq, int k, int32_t* out);
/* The shader matvec of one model matrix over columns [c0, c1) (xq holds
   c1 - c0 q16 ints; no input scaling), every row: out receives the clamped
   q16 ints.  literal selects the shaders' fp32 accumulation for q8 / t3
   (the i16 router is exact in both). */
int orc_model_mv(const orc_model* m, int which, int layer, int expert, int c0, int c1,
                 const int16_t* xq, int literal, int32_t* out);
/* The GPU FFN gate kernel the CPU path draws (gpu_ffn.cpp:17-132): gate/up
   matvecs of the q16 input xq (dim values), SiLU(g)*u (times 2^-hs for a
   key-15 layer), stored as q16 ints in hq (ffn_width values). */
int orc_ffn_hidden(const orc_model* m, int layer, int expert, const int16_t* xq, int literal, int16_t* hq);
/* Decoded weight level of one entry (for dequant parity). */
int orc_model_mat_shape(const orc_model* m, int which, int layer, int expert,
                        int* rows, int* cols, int* wtype, float* scale);
int orc_model_mat_levels(const orc_model* m, int which, int layer, int expert,
                         int32_t* levels /* rows*cols */);
int orc_model_mat_rowscale16(const orc_model* m, int which, int layer, int expert,
                             uint16_t* p16 /* rows, or returns 0 if none */);
int orc_model_mat_q4params(const orc_model* m, int which, int layer, int expert,
                           int16_t* s16, int16_t* m16);
/* The container's f32 row plane of a matrix (returns 1, or 0 if it has none). */
int orc_model_mat_plane(const orc_model* m, int which, int layer, int expert, float* plane);
/* Embedding levels (vocab*dim) and the model's f32 vectors:
   which 0 emb_scale, 1 rms_att, 2 rms_ffn, 3 rms_final, 4 q_norm, 5 k_norm.
   Returns the element count (out may be NULL to query it). */
int orc_model_emb(const orc_model* m, int8_t* out);
int orc_model_vec(const orc_model* m, int which, float* out);
/* 64-bit FNV-1a of a byte string (the digest the golden summaries carry). */
uint64_t orc_fnv1a64(const uint8_t* p, uint64_t n);

#ifdef __cplusplus
}
#endif
#endif
