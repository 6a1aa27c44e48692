// kernels.cu -- sm_100a kernels of the quantized decode step.
//
// One decode step of one layer is five kernels:
//   qkv    embedding (layer 0) + RMSNorm + matvec_s(qkv)             -> qkv floats
//   attn   qk-norm + RoPE + packed KV append + attention over the cache -> att (q16)
//   wo     matvec_s(wo) + residual add                               -> x1 (q16)
//   gate   RMSNorm + [MoE router] + w1/w3 matvecs + SwiGLU            -> h (q16)
//   down   w2 (one or two column chunks) + residual add              -> x (q16)
// and after the last layer `logits` (RMSNorm + logits matvec + first-max
// argmax).  The arithmetic is the reference CPU layer loop's
// (engine/src/session.cpp:373-556) with the shader arithmetic of the
// matrices it draws; every weight x activation product is an exact integer
// (dp4a on the 8-bit weights and the split lo/hi bytes of the q16 input), and
// each float step is an explicitly rounded IEEE operation so the CPU oracle
// reproduces it bit for bit.  Build with --fmad=false.
#include "vc4b200_internal.h"

#include <cstdio>
#include <map>
#include <utility>

namespace vc4 {
namespace {

constexpr int kThreads = kWarps * 32;

// ---------------------------------------------------------------------------
// Exact arithmetic helpers (each mirrors one step of the oracle)
// ---------------------------------------------------------------------------

__device__ __forceinline__ int dp4a_su(int a, unsigned b, int c) {
    int d; asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d; asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int dp4a_uu(unsigned a, unsigned b, int c) {
    int d; asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d; asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}

// q16 host quantisation: lrintf(v*256) clamped (common.h:188-193).
__device__ __forceinline__ int q16h(float v) {
    const int q = __float2int_rn(__fmul_rn(v, 256.0f));
    return q < -32768 ? -32768 : q > 32767 ? 32767 : q;
}
// q16 shader store: clamp(floor(v*256+0.5)) (xformat.cpp x_st2).
__device__ __forceinline__ int q16s(float v) {
    float f = floorf(__fadd_rn(__fmul_rn(v, 256.0f), 0.5f));
    f = f < -32768.0f ? -32768.0f : f > 32767.0f ? 32767.0f : f;
    return (int)f;
}
// Matvec epilogue: floor(S*sc + 0.5) clamped to the q16 rail.
__device__ __forceinline__ int mv_epi(long long S, float sc) {
    double v = floor(__dadd_rn(__dmul_rn(__ll2double_rn(S), (double)sc), 0.5));
    v = v < -32768.0 ? -32768.0 : v > 32767.0 ? 32767.0 : v;
    return (int)v;
}
// Portable exp: Cody-Waite reduction + degree-7 Taylor (same ops as orc_expf).
__device__ __forceinline__ float vexp(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.97208404541016f) return 0.0f;
    const float k = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = __fmaf_rn(-k, 0.693145751953125f, x);
    r = __fmaf_rn(-k, 1.428606765330187045037746429443359375e-06f, r);
    float p = 1.98412698412698412698e-4f;
    p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ki = (int)k;
    if (ki > 127) { p = __fmul_rn(p, 2.0f); ki -= 1; }
    if (ki < -126) return __fmul_rn(__fmul_rn(p, __int_as_float((ki + 64 + 127) << 23)), __int_as_float((-64 + 127) << 23));
    return __fmul_rn(p, __int_as_float((ki + 127) << 23));
}
// SiLU(g)*u in the shaders' order.
__device__ __forceinline__ float swiglu1(float g, float u) {
    const float den = __fadd_rn(1.0f, vexp(-g));
    return __fmul_rn(__fdiv_rn(g, den), u);
}

// ---------------------------------------------------------------------------
// Block reductions (256 threads)
// ---------------------------------------------------------------------------

struct Red {
    long long i64[kWarps];
    double f64[kWarps];
    float f32[kWarps];
    int i32[kWarps];
};

__device__ long long block_sum_i64(long long v, Red& r) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) r.i64[threadIdx.x >> 5] = v;
    __syncthreads();
    long long t = 0;
    for (int w = 0; w < kWarps; ++w) t += r.i64[w];
    return t;
}
__device__ int block_max_i32(int v, Red& r) {
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) r.i32[threadIdx.x >> 5] = v;
    __syncthreads();
    int t = r.i32[0];
    for (int w = 1; w < kWarps; ++w) t = max(t, r.i32[w]);
    return t;
}
__device__ float block_max_f32(float v, Red& r) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) r.f32[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = r.f32[0];
    for (int w = 1; w < kWarps; ++w) t = fmaxf(t, r.f32[w]);
    return t;
}
__device__ double block_sum_f64(double v, Red& r) {
    for (int o = 16; o; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) r.f64[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < kWarps; ++w) t = __dadd_rn(t, r.f64[w]);
    return t;
}

// ---------------------------------------------------------------------------
// Input staging: q16 ints -> (optionally 2^k scaled) ints split into lo/hi bytes
// ---------------------------------------------------------------------------

struct XStage {
    uint8_t* lo;       // [nb][stride]
    int8_t* hi;        // [nb][stride]
    int stride;        // padded column count
    int* gsum;         // q4: [nb][stride/32] group sums; t3: [nb] totals (in gsum[b*gstride])
    int gstride;
    int k[8];          // per input: power-of-two input scale (matvec_s)
};

// matvec_s scaling exponent of a q16 vector (gpu_conv.cpp:271-287):
// max|x| = f*2^e with f in [0.5, 1) gives k = 6 - e.
__device__ int scale_exponent(const int16_t* v, int n, Red& r) {
    int mx = 0;
    for (int c = threadIdx.x; c < n; c += blockDim.x) mx = max(mx, abs((int)v[c]));
    mx = block_max_i32(mx, r);
    if (mx == 0) return 0;
    int e = 0;
    frexpf(__fmul_rn((float)mx, 1.0f / 256.0f), &e);
    return 6 - e;
}

// Stage one input: x'[c] = v[c]*2^k (k >= 0: exact shift; k < 0: x_pack's
// round-half-even), zero-padded to `stride`; group sums for q4 / total for t3.
template <int WT>
__device__ void stage_one(XStage& xs, int b, const int16_t* v, int n, int k, Red& r) {
    uint8_t* lo = xs.lo + (size_t)b * xs.stride;
    int8_t* hi = xs.hi + (size_t)b * xs.stride;
    const float sk = ldexpf(1.0f, k);
    int tot = 0;
    for (int c = threadIdx.x; c < xs.stride; c += blockDim.x) {
        int q = 0;
        if (c < n) {
            const int a = v[c];
            q = k >= 0 ? (a << k) : __float2int_rn(__fmul_rn((float)a, sk));
        }
        lo[c] = (uint8_t)(q & 0xFF);
        hi[c] = (int8_t)(q >> 8);
        tot += q;
    }
    if (WT == W_T3) {
        const long long t = block_sum_i64(tot, r);
        if (threadIdx.x == 0) xs.gsum[b * xs.gstride] = (int)t;
    }
    __syncthreads();
    if (WT == W_Q4) {
        const int ng = xs.stride / 32;
        for (int g = threadIdx.x; g < ng; g += blockDim.x) {
            int s = 0;
            for (int j = 0; j < 32; ++j) s += (int)lo[g * 32 + j] + 256 * (int)hi[g * 32 + j];
            xs.gsum[b * xs.gstride + g] = s;
        }
    }
    __syncthreads();
}

// RMSNorm of a q16 vector into q16 ints (session.cpp:1932-1948 with the exact
// integer sum of squares rounded once).
__device__ void rmsnorm_q16(const int16_t* x, const float* w, int D, float eps, int16_t* out, Red& r) {
    long long ss = 0;
    for (int c = threadIdx.x; c < D; c += blockDim.x) { const long long a = x[c]; ss += a * a; }
    ss = block_sum_i64(ss, r);
    const float s1 = __fmul_rn(__ll2float_rn(ss), 1.0f / 65536.0f);
    const float s2 = __fdiv_rn(s1, (float)D);
    const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s2, eps)));
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        const float xv = __fmul_rn((float)x[c], 1.0f / 256.0f);
        out[c] = (int16_t)q16h(__fmul_rn(w[c], __fmul_rn(rr, xv)));
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Matvec core: one 32-row block of one matrix over nb staged inputs.
// Warp w takes chunks w, w+8, ...; each lane owns one row.  Returns the
// warp's partial exact sums.
// ---------------------------------------------------------------------------

template <int WT, int NB>
__device__ __forceinline__ void mv_block(const DMat& W, int blk, const XStage& xs, int nb, long long (&S)[NB]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nch = W.nchunks;
    int alo[NB], ahi[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) { alo[b] = 0; ahi[b] = 0; S[b] = 0; }
    const int4* body = reinterpret_cast<const int4*>(W.body) + (size_t)blk * nch * 32 + lane;
    for (int j = warp; j < nch; j += kWarps) {
        const int4 w = __ldg(body + (size_t)j * 32);
        if (WT == W_Q8) {
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb) break;
                const uint4 L = *reinterpret_cast<const uint4*>(xs.lo + (size_t)b * xs.stride + j * 16);
                const uint4 H = *reinterpret_cast<const uint4*>(xs.hi + (size_t)b * xs.stride + j * 16);
                alo[b] = dp4a_su(w.x, L.x, alo[b]); alo[b] = dp4a_su(w.y, L.y, alo[b]);
                alo[b] = dp4a_su(w.z, L.z, alo[b]); alo[b] = dp4a_su(w.w, L.w, alo[b]);
                ahi[b] = dp4a_ss(w.x, (int)H.x, ahi[b]); ahi[b] = dp4a_ss(w.y, (int)H.y, ahi[b]);
                ahi[b] = dp4a_ss(w.z, (int)H.z, ahi[b]); ahi[b] = dp4a_ss(w.w, (int)H.w, ahi[b]);
            }
        } else if (WT == W_T3) {
            const unsigned wd[4] = {(unsigned)w.x, (unsigned)w.y, (unsigned)w.z, (unsigned)w.w};
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb) break;
                const uint4* L4 = reinterpret_cast<const uint4*>(xs.lo + (size_t)b * xs.stride + j * 64);
                const uint4* H4 = reinterpret_cast<const uint4*>(xs.hi + (size_t)b * xs.stride + j * 64);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 L = L4[q], H = H4[q];
                    const unsigned e0 = wd[q] & 0x03030303u, e1 = (wd[q] >> 2) & 0x03030303u;
                    const unsigned e2 = (wd[q] >> 4) & 0x03030303u, e3 = (wd[q] >> 6) & 0x03030303u;
                    alo[b] = dp4a_uu(e0, L.x, alo[b]); alo[b] = dp4a_uu(e1, L.y, alo[b]);
                    alo[b] = dp4a_uu(e2, L.z, alo[b]); alo[b] = dp4a_uu(e3, L.w, alo[b]);
                    ahi[b] = dp4a_us(e0, (int)H.x, ahi[b]); ahi[b] = dp4a_us(e1, (int)H.y, ahi[b]);
                    ahi[b] = dp4a_us(e2, (int)H.z, ahi[b]); ahi[b] = dp4a_us(e3, (int)H.w, ahi[b]);
                }
            }
        } else {  // W_Q4: chunk j is scale group j
            const int sp = __ldg(W.q4p + ((size_t)blk * nch + j) * 32 + lane);
            const long long s16 = (short)(sp & 0xFFFF), m16 = (short)(sp >> 16);
            const unsigned wd[4] = {(unsigned)w.x, (unsigned)w.y, (unsigned)w.z, (unsigned)w.w};
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb) break;
                const uint4* L4 = reinterpret_cast<const uint4*>(xs.lo + (size_t)b * xs.stride + j * 32);
                const uint4* H4 = reinterpret_cast<const uint4*>(xs.hi + (size_t)b * xs.stride + j * 32);
                const uint4 L0 = L4[0], L1 = L4[1], H0 = H4[0], H1 = H4[1];
                const unsigned l[8] = {L0.x, L0.y, L0.z, L0.w, L1.x, L1.y, L1.z, L1.w};
                const unsigned h[8] = {H0.x, H0.y, H0.z, H0.w, H1.x, H1.y, H1.z, H1.w};
                int nlo = 0, nhi = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const unsigned n0 = wd[q] & 0x0F0F0F0Fu, n1 = (wd[q] >> 4) & 0x0F0F0F0Fu;
                    nlo = dp4a_uu(n0, l[2 * q], nlo); nlo = dp4a_uu(n1, l[2 * q + 1], nlo);
                    nhi = dp4a_us(n0, (int)h[2 * q], nhi); nhi = dp4a_us(n1, (int)h[2 * q + 1], nhi);
                }
                const long long N = (long long)nlo + 256LL * nhi;
                S[b] += s16 * N + m16 * (long long)xs.gsum[b * xs.gstride + j];
            }
        }
    }
    if (WT != W_Q4) {
#pragma unroll
        for (int b = 0; b < NB; ++b) S[b] = (long long)alo[b] + 256LL * (long long)ahi[b];
    }
}

// Cross-warp sum of the per-warp partials: on return every thread with
// warp index b < nb holds the full sum of row (lane) for input b.
template <int NB>
__device__ __forceinline__ long long reduce_warps(const long long (&S)[NB], int nb, long long* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int b = 0; b < NB; ++b) red[(warp * NB + b) * 32 + lane] = S[b];
    __syncthreads();
    long long t = 0;
    if (warp < nb)
        for (int w = 0; w < kWarps; ++w) t += red[(w * NB + warp) * 32 + lane];
    __syncthreads();
    return t;
}

struct SmemLayout {
    // dynamic shared memory: [Red][red i64 kWarps*NB*32][gsum][lo][hi][scratch int16]
    static __device__ char* base() { extern __shared__ __align__(16) char smem[]; return smem; }
};

template <int NB>
__device__ void carve(int stride, int gstride, XStage& xs, Red*& red, long long*& part, int16_t*& tmp, int tmp_n) {
    char* p = SmemLayout::base();
    red = reinterpret_cast<Red*>(p); p += (sizeof(Red) + 15) / 16 * 16;
    part = reinterpret_cast<long long*>(p); p += sizeof(long long) * kWarps * NB * 32;
    xs.gsum = reinterpret_cast<int*>(p); p += (sizeof(int) * NB * gstride + 15) / 16 * 16;
    xs.lo = reinterpret_cast<uint8_t*>(p); p += (size_t)NB * stride;
    xs.hi = reinterpret_cast<int8_t*>(p); p += (size_t)NB * stride;
    tmp = reinterpret_cast<int16_t*>(p);
    (void)tmp_n;
    xs.stride = stride; xs.gstride = gstride;
}

__host__ size_t smem_bytes(int nb, int stride, int gstride, int tmp_n) {
    return (sizeof(Red) + 15) / 16 * 16 + sizeof(long long) * kWarps * nb * 32 +
           (sizeof(int) * nb * gstride + 15) / 16 * 16 + 2 * (size_t)nb * stride + sizeof(int16_t) * (size_t)tmp_n;
}

__host__ __device__ inline int cpc_of(int wt) { return wt == W_Q8 ? 16 : wt == W_Q4 ? 32 : 64; }
__host__ __device__ inline int x_stride(const DMat& W) { return W.nchunks * cpc_of(W.wtype); }
__host__ __device__ inline int g_stride(const DMat& W) { return W.wtype == W_Q4 ? W.nchunks : 1; }

// ---------------------------------------------------------------------------
// Kernel parameter blocks
// ---------------------------------------------------------------------------

struct Dims {
    int dim, kv_dim, heads, kv_heads, head_dim, layers, vocab, ffn, chunk, experts, seq, row_bytes, kv_bits;
    int rope_half, qk_norm;
    float eps;
};

Dims dims_of(const DModel& m, const State& s) {
    Dims d;
    d.dim = m.h.dim; d.kv_dim = m.h.kv_dim; d.heads = m.h.heads; d.kv_heads = m.h.kv_heads;
    d.head_dim = m.h.head_dim; d.layers = m.h.layers; d.vocab = m.h.vocab; d.ffn = m.ffn_width;
    d.chunk = m.ffn_chunk; d.experts = m.h.experts; d.seq = s.seq; d.row_bytes = s.row_bytes;
    d.kv_bits = s.kv_bits; d.rope_half = m.h.rope_half; d.qk_norm = m.h.qk_norm; d.eps = m.h.rms_eps;
    return d;
}

// ---------------------------------------------------------------------------
// qkv: [embedding] + RMSNorm + matvec_s(qkv)
// ---------------------------------------------------------------------------

template <int WT, int NB>
__global__ void __launch_bounds__(kThreads) k_qkv(DMat W, DMat E, const float* emb_scale, const float* rms_w,
                                                  State s, Batch bt, Dims d, int layer, int b0) {
    XStage xs; Red* red; long long* part; int16_t* tmp;
    carve<NB>(x_stride(W), g_stride(W), xs, red, part, tmp, NB * d.dim);
    const int nb = min(NB, bt.n - b0);
    for (int b = 0; b < nb; ++b) {
        const int slot = bt.slot[b0 + b];
        int16_t* x = s.x + (size_t)slot * d.dim;
        int16_t* xin = tmp + (size_t)b * d.dim;
        if (layer == 0) {
            // embedding (session.cpp:342-371): q16(level * row scale); rows are
            // read from the blocked q8 layout of the embedding matrix.
            const int tok = bt.token[b0 + b];
            const float es = emb_scale[tok];
            const int8_t* eb = reinterpret_cast<const int8_t*>(E.body) + ((size_t)(tok / 32) * E.nchunks * 32 + (tok % 32)) * 16;
            for (int c = threadIdx.x; c < d.dim; c += blockDim.x) {
                const int lv = eb[(size_t)(c / 16) * 512 + (c % 16)];
                const int16_t q = (int16_t)q16h(__fmul_rn((float)lv, es));
                xin[c] = q;
                if (blockIdx.x == 0) x[c] = q;
            }
            if (blockIdx.x == 0 && threadIdx.x == 0) s.best[slot] = 0ull;
        } else {
            for (int c = threadIdx.x; c < d.dim; c += blockDim.x) xin[c] = x[c];
        }
        __syncthreads();
        rmsnorm_q16(xin, rms_w, d.dim, d.eps, xin, *red);
        xs.k[b] = scale_exponent(xin, d.dim, *red);
        stage_one<WT>(xs, b, xin, d.dim, xs.k[b], *red);
    }
    long long S[NB];
    mv_block<WT, NB>(W, blockIdx.x, xs, nb, S);
    const long long tot = reduce_warps<NB>(S, nb, part);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        if (row < W.rows) {
            const long long St = WT == W_T3 ? tot - xs.gsum[warp * xs.gstride] : tot;
            const int v = mv_epi(St, W.rscale[row]);
            const float out = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), ldexpf(1.0f, -xs.k[warp]));
            s.qkv[(size_t)bt.slot[b0 + warp] * (d.dim + 2 * d.kv_dim) + row] = out;
        }
    }
}

// ---------------------------------------------------------------------------
// wo: matvec_s(wo, att) + add_q16 residual -> x1
// ---------------------------------------------------------------------------

template <int WT, int NB>
__global__ void __launch_bounds__(kThreads) k_wo(DMat W, State s, Batch bt, Dims d, int b0) {
    XStage xs; Red* red; long long* part; int16_t* tmp;
    carve<NB>(x_stride(W), g_stride(W), xs, red, part, tmp, 0);
    const int nb = min(NB, bt.n - b0);
    for (int b = 0; b < nb; ++b) {
        const int16_t* a = s.att + (size_t)bt.slot[b0 + b] * d.dim;
        xs.k[b] = scale_exponent(a, d.dim, *red);
        stage_one<WT>(xs, b, a, d.dim, xs.k[b], *red);
    }
    long long S[NB];
    mv_block<WT, NB>(W, blockIdx.x, xs, nb, S);
    const long long tot = reduce_warps<NB>(S, nb, part);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        if (row < W.rows) {
            const int slot = bt.slot[b0 + warp];
            const long long St = WT == W_T3 ? tot - xs.gsum[warp * xs.gstride] : tot;
            const int v = mv_epi(St, W.rscale[row]);
            const float wo = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), ldexpf(1.0f, -xs.k[warp]));
            const float xr = __fmul_rn((float)s.x[(size_t)slot * d.dim + row], 1.0f / 256.0f);
            s.x1[(size_t)slot * d.dim + row] = (int16_t)q16h(__fadd_rn(xr, wo));
        }
    }
}

// ---------------------------------------------------------------------------
// gate: RMSNorm(x1) + [router] + w1/w3 + SwiGLU -> h
// ---------------------------------------------------------------------------

// MoE route of one q16 input (session.cpp:1523-1536 + pick_expert 110-115):
// matvec_s over the i16 router, first maximum.
__device__ int route_of(const int16_t* xbf, const DMat& R, int D, int experts, Red& r, int* scratch) {
    const int k = scale_exponent(xbf, D, r);
    const float sk = ldexpf(1.0f, k);
    int best = 0;
    float bestv = 0.0f;
    for (int e = 0; e < experts; ++e) {
        long long acc = 0;
        for (int c = threadIdx.x; c < D; c += blockDim.x) {
            const int a = xbf[c];
            const int q = k >= 0 ? (a << k) : __float2int_rn(__fmul_rn((float)a, sk));
            acc += (long long)R.w16[(size_t)e * D + c] * q;
        }
        acc = block_sum_i64(acc, r);
        const int v = mv_epi(acc, R.rscale[e]);
        const float g = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), ldexpf(1.0f, -k));
        if (e == 0 || g > bestv) { best = e; bestv = g; }
    }
    (void)scratch;
    return best;
}

template <int WT, int NB>
__global__ void __launch_bounds__(kThreads) k_gate(const DMat* mats, int i_w1, int i_w3, int i_router, int e_base,
                                                   const float* rms_w, State s, Batch bt, Dims d, int layer, int b0,
                                                   int hs) {
    // MoE: blockIdx.y is the expert; the CTA serves the inputs routed to it.
    const int expert = blockIdx.y;
    const DMat& W1 = mats[d.experts ? e_base + expert * 4 + 0 : i_w1];
    const DMat& W3 = mats[d.experts ? e_base + expert * 4 + 1 : i_w3];
    XStage xs; Red* red; long long* part; int16_t* tmp;
    carve<NB>(x_stride(W1), g_stride(W1), xs, red, part, tmp, (NB + 1) * d.dim);
    int* members = reinterpret_cast<int*>(tmp + (size_t)(NB + 1) * d.dim);   // batch indices served
    const int n_all = min(NB, bt.n - b0);
    int nb = 0;
    for (int b = 0; b < n_all; ++b) {
        const int slot = bt.slot[b0 + b];
        int16_t* xin = tmp + (size_t)nb * d.dim;
        rmsnorm_q16(s.x1 + (size_t)slot * d.dim, rms_w, d.dim, d.eps, xin, *red);
        if (d.experts) {
            const int e = route_of(xin, mats[i_router], d.dim, d.experts, *red, nullptr);
            if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) s.route[(size_t)slot * d.layers + layer] = e;
            __syncthreads();
            if (e != expert) continue;
        }
        if (threadIdx.x == 0) members[nb] = b;
        xs.k[nb] = 0;
        stage_one<WT>(xs, nb, xin, d.dim, 0, *red);
        ++nb;
    }
    if (nb == 0) return;
    long long S1[NB], S3[NB];
    mv_block<WT, NB>(W1, blockIdx.x, xs, nb, S1);
    const long long t1 = reduce_warps<NB>(S1, nb, part);
    mv_block<WT, NB>(W3, blockIdx.x, xs, nb, S3);
    const long long t3 = reduce_warps<NB>(S3, nb, part);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        if (row < W1.rows) {
            const int slot = bt.slot[b0 + members[warp]];
            const int corr = WT == W_T3 ? xs.gsum[warp * xs.gstride] : 0;
            const int g = mv_epi(t1 - corr, W1.rscale[row]);
            const int u = mv_epi(t3 - corr, W3.rscale[row]);
            float y = swiglu1(__fmul_rn((float)g, 1.0f / 256.0f), __fmul_rn((float)u, 1.0f / 256.0f));
            if (hs > 0) y = __fmul_rn(y, ldexpf(1.0f, -hs));     // metadata key 15 store scale
            s.h[(size_t)slot * d.ffn + row] = (int16_t)q16s(y);
        }
    }
}

// ---------------------------------------------------------------------------
// down: w2 (one or two column chunks) + residual -> x
// ---------------------------------------------------------------------------

template <int WT, int NB>
__global__ void __launch_bounds__(kThreads) k_down(const DMat* mats, int i_w2a, int i_w2b, int e_base,
                                                   State s, Batch bt, Dims d, int layer, int b0) {
    const int expert = blockIdx.y;
    const DMat& Wa = mats[d.experts ? e_base + expert * 4 + 2 : i_w2a];
    const bool two = d.chunk < d.ffn;
    const DMat& Wb = mats[d.experts ? e_base + expert * 4 + 3 : (two ? i_w2b : i_w2a)];
    XStage xa, xb; Red* red; long long* part; int16_t* tmp;
    // stage A in the carved buffers, stage B right after them
    carve<NB>(x_stride(Wa), g_stride(Wa), xa, red, part, tmp, 0);
    xb = xa;
    const int sb = two ? x_stride(Wb) : 0;
    xb.stride = sb > 0 ? sb : 1;
    xb.gstride = g_stride(Wb);
    xb.gsum = reinterpret_cast<int*>(tmp);
    xb.lo = reinterpret_cast<uint8_t*>(xb.gsum + NB * xb.gstride + 4);
    xb.lo = reinterpret_cast<uint8_t*>(((uintptr_t)xb.lo + 15) & ~(uintptr_t)15);
    xb.hi = reinterpret_cast<int8_t*>(xb.lo + (size_t)NB * xb.stride);
    int* members = reinterpret_cast<int*>(xb.hi + (size_t)NB * xb.stride);
    const int n_all = min(NB, bt.n - b0);
    int nb = 0;
    for (int b = 0; b < n_all; ++b) {
        const int slot = bt.slot[b0 + b];
        if (d.experts && s.route[(size_t)slot * d.layers + layer] != expert) continue;
        const int16_t* h = s.h + (size_t)slot * d.ffn;
        if (threadIdx.x == 0) members[nb] = b;
        stage_one<WT>(xa, nb, h, d.chunk, 0, *red);
        if (two) stage_one<WT>(xb, nb, h + d.chunk, d.ffn - d.chunk, 0, *red);
        ++nb;
    }
    __syncthreads();
    if (nb == 0) return;
    long long Sa[NB], Sb[NB];
    mv_block<WT, NB>(Wa, blockIdx.x, xa, nb, Sa);
    const long long ta = reduce_warps<NB>(Sa, nb, part);
    long long tb = 0;
    if (two) {
        mv_block<WT, NB>(Wb, blockIdx.x, xb, nb, Sb);
        tb = reduce_warps<NB>(Sb, nb, part);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        if (row < Wa.rows) {
            const int slot = bt.slot[b0 + members[warp]];
            const int va = mv_epi(WT == W_T3 ? ta - xa.gsum[warp * xa.gstride] : ta, Wa.rscale[row]);
            float o2 = __fmul_rn((float)va, 1.0f / 256.0f);
            if (two) {
                const int vb = mv_epi(WT == W_T3 ? tb - xb.gsum[warp * xb.gstride] : tb, Wb.rscale[row]);
                // add_q16 of the two chunk outputs (session.cpp:2052-2067)
                o2 = __fmul_rn((float)q16h(__fadd_rn(o2, __fmul_rn((float)vb, 1.0f / 256.0f))), 1.0f / 256.0f);
            }
            const float x1 = __fmul_rn((float)s.x1[(size_t)slot * d.dim + row], 1.0f / 256.0f);
            s.x[(size_t)slot * d.dim + row] = (int16_t)q16h(__fadd_rn(x1, o2));
        }
    }
}

// ---------------------------------------------------------------------------
// logits: RMSNorm(x) + logits matvec + first-max argmax
// ---------------------------------------------------------------------------

template <int WT, int NB>
__global__ void __launch_bounds__(kThreads) k_logits(DMat W, const float* rms_w, State s, Batch bt, Dims d, int b0) {
    XStage xs; Red* red; long long* part; int16_t* tmp;
    carve<NB>(x_stride(W), g_stride(W), xs, red, part, tmp, NB * d.dim);
    const int nb = min(NB, bt.n - b0);
    for (int b = 0; b < nb; ++b) {
        int16_t* xin = tmp + (size_t)b * d.dim;
        rmsnorm_q16(s.x + (size_t)bt.slot[b0 + b] * d.dim, rms_w, d.dim, d.eps, xin, *red);
        xs.k[b] = 0;
        stage_one<WT>(xs, b, xin, d.dim, 0, *red);
    }
    long long S[NB];
    mv_block<WT, NB>(W, blockIdx.x, xs, nb, S);
    const long long tot = reduce_warps<NB>(S, nb, part);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        const int slot = bt.slot[b0 + warp];
        unsigned long long key = 0ull;
        if (row < W.rows) {
            const int v = mv_epi(tot, W.rscale[row]);
            s.logits[(size_t)slot * d.vocab + row] = v;
            key = ((unsigned long long)(unsigned)(v + 32768) << 32) | (unsigned)(0xFFFFFFFFu - (unsigned)row);
        }
        for (int o = 16; o; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
            key = k2 > key ? k2 : key;
        }
        if (lane == 0 && key) atomicMax(&s.best[slot], key);
    }
}

// ---------------------------------------------------------------------------
// attention: qk-norm + RoPE + KV append (packed codec) + attention
// ---------------------------------------------------------------------------

constexpr int kTile = 128;   // positions per staged K/V tile
constexpr int kRedBytes = (int)((sizeof(Red) + 15) / 16 * 16);

__device__ __forceinline__ float kv_decode(const uint8_t* row, int i, int kv_bits) {
    if (kv_bits == 16) {
        const int q = (int)(short)(((unsigned)row[2 * i] << 8) | row[2 * i + 1]);
        return __fdiv_rn((float)q, 2048.0f);
    }
    return __fdiv_rn((float)(signed char)row[i], 16.0f);
}

__global__ void __launch_bounds__(kThreads) k_attn(const float* q_norm, const float* k_norm, State s, Batch bt, Dims d, int layer) {
    extern __shared__ __align__(16) char smem[];
    const int g = blockIdx.x, b = blockIdx.y;
    const int slot = bt.slot[b], pos = bt.pos[b];
    const int hd = d.head_dim, group = d.heads / d.kv_heads, half = hd / 2;
    const int hp = hd + 1;                     // padded tile stride (floats)
    Red* red = reinterpret_cast<Red*>(smem);
    float* qv = reinterpret_cast<float*>(smem + kRedBytes);    // group*hd
    float* kvv = qv + group * hd;                                // 2*hd (k, v)
    float* tile = kvv + 2 * hd;                                  // kTile*hp
    float* sc = tile + kTile * hp;                               // group*seq
    double* pv = reinterpret_cast<double*>(((uintptr_t)(sc + (size_t)group * d.seq) + 15) & ~(uintptr_t)15);
    const float* qkv = s.qkv + (size_t)slot * (d.dim + 2 * d.kv_dim);
    for (int i = threadIdx.x; i < group * hd; i += blockDim.x) qv[i] = qkv[g * group * hd + i];
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        kvv[i] = qkv[d.dim + g * hd + i];
        kvv[hd + i] = qkv[d.dim + d.kv_dim + g * hd + i];
    }
    __syncthreads();
    // qk-norm (session.cpp:1950-1961): the squares of one head share a
    // power-of-two grid, so the double sum is exact in any order.
    if (d.qk_norm) {
        for (int hh = 0; hh <= group; ++hh) {
            float* v = hh < group ? qv + hh * hd : kvv;
            const float* w = (hh < group ? q_norm : k_norm) + (size_t)layer * hd;
            double acc = 0.0;
            for (int i = threadIdx.x; i < hd; i += blockDim.x) acc = __dadd_rn(acc, __dmul_rn((double)v[i], (double)v[i]));
            acc = block_sum_f64(acc, *red);
            const float ss = __double2float_rn(acc);
            const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), 1e-6f)));
            __syncthreads();
            for (int i = threadIdx.x; i < hd; i += blockDim.x) v[i] = __fmul_rn(w[i], __fmul_rn(r, v[i]));
            __syncthreads();
        }
    }
    // RoPE (session.cpp:1963-1987) with the host-built cos/sin tables.
    {
        const float* cs = s.rope_cos + (size_t)pos * half;
        const float* sn = s.rope_sin + (size_t)pos * half;
        for (int t = threadIdx.x; t < (group + 1) * half; t += blockDim.x) {
            const int hh = t / half, i = t % half;
            float* o = hh < group ? qv + hh * hd : kvv;
            const int ia = d.rope_half ? i : 2 * i, ib = d.rope_half ? i + half : 2 * i + 1;
            const float a = o[ia], bb = o[ib], c = cs[i], sv = sn[i];
            o[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, sv));
            o[ib] = __fadd_rn(__fmul_rn(a, sv), __fmul_rn(bb, c));
        }
    }
    __syncthreads();
    // KV append: the packed codec (shaders_attn.cpp:141-159), this head's slice.
    uint8_t* kvbase = s.kv + ((size_t)slot * d.layers + layer) * d.seq * d.row_bytes;
    {
        uint8_t* row = kvbase + (size_t)pos * d.row_bytes;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            const int c = g * hd + i;
            for (int w = 0; w < 2; ++w) {
                const float v = kvv[w * hd + i];
                if (d.kv_bits == 16) {
                    float q = floorf(__fadd_rn(__fmul_rn(v, 2048.0f), 0.5f));
                    q = q < -32768.0f ? -32768.0f : q > 32767.0f ? 32767.0f : q;
                    const unsigned u = (unsigned)(int)q & 0xFFFFu;
                    uint8_t* p = row + (size_t)w * 2 * d.kv_dim + 2 * c;
                    p[0] = (uint8_t)(u >> 8); p[1] = (uint8_t)u;
                } else {
                    float q = floorf(__fadd_rn(__fmul_rn(v, 16.0f), 0.5f));
                    q = q < -128.0f ? -128.0f : q > 127.0f ? 127.0f : q;
                    row[(size_t)w * d.kv_dim + c] = (uint8_t)(int)q;
                }
            }
        }
    }
    __syncthreads();
    const int vofs = d.kv_bits == 16 ? 2 * d.kv_dim : d.kv_dim;   // V starts here in a row
    const float sq = __fsqrt_rn((float)hd);
    // scores: one thread per position, sequential fp32 dot (session.cpp:2031-2036)
    for (int t0 = 0; t0 <= pos; t0 += kTile) {
        const int nt = min(kTile, pos + 1 - t0);
        for (int e = threadIdx.x; e < nt * hd; e += blockDim.x) {
            const int t = e / hd, i = e % hd;
            tile[t * hp + i] = kv_decode(kvbase + (size_t)(t0 + t) * d.row_bytes, g * hd + i, d.kv_bits);
        }
        __syncthreads();
        for (int t = threadIdx.x; t < nt; t += blockDim.x) {
            const float* kr = tile + t * hp;
            for (int hh = 0; hh < group; ++hh) {
                const float* q = qv + hh * hd;
                float acc = 0.0f;
                for (int i = 0; i < hd; ++i) acc = __fadd_rn(acc, __fmul_rn(q[i], kr[i]));
                acc = __fdiv_rn(acc, sq);
                sc[(size_t)hh * d.seq + t0 + t] = acc;
            }
        }
        __syncthreads();
    }
    // softmax per head: max, exp, double sum, divide (session.cpp:2037-2040)
    for (int hh = 0; hh < group; ++hh) {
        float* S = sc + (size_t)hh * d.seq;
        float m = -1e30f;
        for (int t = threadIdx.x; t <= pos; t += blockDim.x) m = fmaxf(m, S[t]);
        m = block_max_f32(m, *red);
        double sum = 0.0;
        for (int t = threadIdx.x; t <= pos; t += blockDim.x) {
            const float e = vexp(__fsub_rn(S[t], m));
            S[t] = e;
            sum = __dadd_rn(sum, (double)e);
        }
        sum = block_sum_f64(sum, *red);
        const float fs = __double2float_rn(sum);
        for (int t = threadIdx.x; t <= pos; t += blockDim.x) S[t] = __fdiv_rn(S[t], fs);
        __syncthreads();
    }
    // P.V in double: warp w takes positions w, w+8, ..; lanes take dims.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nd = (hd + 31) / 32;
    double acc[8 * 4];   // group <= 8, hd <= 128
    for (int a = 0; a < group * nd; ++a) acc[a] = 0.0;
    for (int t0 = 0; t0 <= pos; t0 += kTile) {
        const int nt = min(kTile, pos + 1 - t0);
        __syncthreads();
        for (int e = threadIdx.x; e < nt * hd; e += blockDim.x) {
            const int t = e / hd, i = e % hd;
            tile[t * hp + i] = kv_decode(kvbase + (size_t)(t0 + t) * d.row_bytes + vofs - (d.kv_bits == 16 ? 0 : 0),
                                         g * hd + i, d.kv_bits);
        }
        __syncthreads();
        for (int t = warp; t < nt; t += kWarps) {
            const float* vr = tile + t * hp;
            for (int hh = 0; hh < group; ++hh) {
                const double p = (double)sc[(size_t)hh * d.seq + t0 + t];
                for (int m = 0; m < nd; ++m) {
                    const int i = lane + 32 * m;
                    if (i < hd) acc[hh * nd + m] = __dadd_rn(acc[hh * nd + m], __dmul_rn(p, (double)vr[i]));
                }
            }
        }
    }
    __syncthreads();
    for (int hh = 0; hh < group; ++hh)
        for (int m = 0; m < nd; ++m) {
            const int i = lane + 32 * m;
            if (i < hd) pv[((size_t)warp * group + hh) * hd + i] = acc[hh * nd + m];
        }
    __syncthreads();
    for (int e = threadIdx.x; e < group * hd; e += blockDim.x) {
        double t = 0.0;
        for (int w = 0; w < kWarps; ++w) t = __dadd_rn(t, pv[(size_t)w * group * hd + e]);
        const float o = __double2float_rn(t);
        s.att[(size_t)slot * d.dim + g * group * hd + e] = (int16_t)q16h(o);
    }
}

// ---------------------------------------------------------------------------
// bare matvec (CPU-path entry)
// ---------------------------------------------------------------------------

template <int WT>
__global__ void __launch_bounds__(kThreads) k_raw(DMat W, const int16_t* xq, int n, int32_t* out) {
    XStage xs; Red* red; long long* part; int16_t* tmp;
    carve<1>(x_stride(W), g_stride(W), xs, red, part, tmp, 0);
    xs.k[0] = 0;
    stage_one<WT>(xs, 0, xq, n, 0, *red);
    long long S[1];
    mv_block<WT, 1>(W, blockIdx.x, xs, 1, S);
    const long long tot = reduce_warps<1>(S, 1, part);
    if (threadIdx.x < 32) {
        const int row = blockIdx.x * 32 + threadIdx.x;
        if (row < W.rows) out[row] = mv_epi(WT == W_T3 ? tot - xs.gsum[0] : tot, W.rscale[row]);
    }
}

// i16 matrix (the MoE router, shaders.cpp:1216-1230): one block per row.
__global__ void __launch_bounds__(kThreads) k_raw_i16(DMat W, const int16_t* xq, int n, int32_t* out) {
    __shared__ Red red;
    const int row = blockIdx.x;
    long long acc = 0;
    for (int c = threadIdx.x; c < n; c += blockDim.x) acc += (long long)W.w16[(size_t)row * n + c] * xq[c];
    acc = block_sum_i64(acc, red);
    if (threadIdx.x == 0) out[row] = mv_epi(acc, W.rscale[row]);
}

// Greedy token of each sequence from its packed argmax key; optionally
// advance the sequence (next token, position + 1).
__global__ void k_finalize(State s, Batch bt, int* next, int* tokens, int* pos, int advance, const int* forced) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= bt.n) return;
    const unsigned long long key = s.best[bt.slot[b]];
    const int tok = (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
    next[b] = tok;
    if (advance) {
        const int p = pos[b] + 1;
        tokens[b] = forced ? forced[p < s.seq ? p : s.seq - 1] : tok;
        pos[b] = p;
    }
}

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------

// Raise a kernel's dynamic shared memory limit once per size; repeated calls
// (and calls during graph capture) are no-ops.
template <typename K>
void set_smem(K kernel, size_t bytes) {
    static std::map<std::pair<const void*, int>, size_t> done;
    int dev = 0;
    cudaGetDevice(&dev);
    size_t& have = done[{(const void*)kernel, dev}];
    if (bytes <= 48 * 1024 || bytes <= have) return;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    have = bytes;
}

constexpr int kNB = 4;   // inputs per CTA for the batched matvecs

template <int WT>
void qkv_t(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
    const DMat& W = m.mats[m.qkv[layer]];
    const DMat& E = m.mats[m.emb_mat];
    Dims d = dims_of(m, s);
    const size_t sm = smem_bytes(kNB, x_stride(W), g_stride(W), kNB * d.dim);
    set_smem(k_qkv<WT, kNB>, sm);
    for (int b0 = 0; b0 < bt.n; b0 += kNB)
        k_qkv<WT, kNB><<<W.rblocks, kThreads, sm, st>>>(W, E, m.d_emb_scale, m.d_rms_att + (size_t)layer * d.dim, s, bt, d, layer, b0);
}

template <int WT>
void wo_t(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
    const DMat& W = m.mats[m.wo[layer]];
    Dims d = dims_of(m, s);
    const size_t sm = smem_bytes(kNB, x_stride(W), g_stride(W), 0);
    set_smem(k_wo<WT, kNB>, sm);
    for (int b0 = 0; b0 < bt.n; b0 += kNB) k_wo<WT, kNB><<<W.rblocks, kThreads, sm, st>>>(W, s, bt, d, b0);
}

template <int WT>
void gate_t(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
    Dims d = dims_of(m, s);
    const int ebase = d.experts ? m.e_w1[(size_t)layer * d.experts] : 0;
    const DMat& W1 = m.mats[d.experts ? ebase : m.w1[layer]];
    const size_t sm = smem_bytes(kNB, x_stride(W1), g_stride(W1), (kNB + 1) * d.dim) + 64;
    set_smem(k_gate<WT, kNB>, sm);
    dim3 grid(W1.rblocks, d.experts ? d.experts : 1);
    for (int b0 = 0; b0 < bt.n; b0 += kNB)
        k_gate<WT, kNB><<<grid, kThreads, sm, st>>>(m.d_mats, d.experts ? 0 : m.w1[layer], d.experts ? 0 : m.w3[layer],
                                                     d.experts ? m.router[layer] : 0, ebase,
                                                     m.d_rms_ffn + (size_t)layer * d.dim, s, bt, d, layer, b0,
                                                     layer < (int)m.h.hid_scale.size() ? (int)m.h.hid_scale[layer] : 0);
}

template <int WT>
void down_t(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
    Dims d = dims_of(m, s);
    const int ebase = d.experts ? m.e_w1[(size_t)layer * d.experts] : 0;
    const DMat& Wa = m.mats[d.experts ? ebase + 2 : m.w2a[layer]];
    const bool two = m.ffn_chunked;
    const DMat& Wb = m.mats[d.experts ? ebase + 3 : (two ? m.w2b[layer] : m.w2a[layer])];
    const size_t sm = smem_bytes(kNB, x_stride(Wa), g_stride(Wa), 0) +
                      (two ? 2 * (size_t)kNB * x_stride(Wb) + sizeof(int) * kNB * g_stride(Wb) : 16) + 256;
    set_smem(k_down<WT, kNB>, sm);
    dim3 grid(Wa.rblocks, d.experts ? d.experts : 1);
    for (int b0 = 0; b0 < bt.n; b0 += kNB)
        k_down<WT, kNB><<<grid, kThreads, sm, st>>>(m.d_mats, d.experts ? 0 : m.w2a[layer],
                                                     d.experts ? 0 : (two ? m.w2b[layer] : m.w2a[layer]), ebase, s, bt, d,
                                                     layer, b0);
}

template <int WT>
void logits_t(const DModel& m, const State& s, const Batch& bt, cudaStream_t st) {
    const DMat& W = m.mats[m.logits_mat];
    Dims d = dims_of(m, s);
    const size_t sm = smem_bytes(kNB, x_stride(W), g_stride(W), kNB * d.dim);
    set_smem(k_logits<WT, kNB>, sm);
    for (int b0 = 0; b0 < bt.n; b0 += kNB)
        k_logits<WT, kNB><<<W.rblocks, kThreads, sm, st>>>(W, m.d_rms_final, s, bt, d, b0);
}

}  // namespace

#define VC4_DISPATCH(WT, FN, ...)                          \
    do {                                                   \
        if ((WT) == W_Q8) FN<W_Q8>(__VA_ARGS__);           \
        else if ((WT) == W_Q4) FN<W_Q4>(__VA_ARGS__);      \
        else FN<W_T3>(__VA_ARGS__);                        \
    } while (0)

void launch_embed_qkv(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    VC4_DISPATCH(m.mats[m.qkv[layer]].wtype, qkv_t, m, s, b, layer, st);
}
void launch_wo(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    VC4_DISPATCH(m.mats[m.wo[layer]].wtype, wo_t, m, s, b, layer, st);
}
void launch_ffn_gate(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    const int wt = m.h.experts ? m.mats[m.e_w1[(size_t)layer * m.h.experts]].wtype : m.mats[m.w1[layer]].wtype;
    VC4_DISPATCH(wt, gate_t, m, s, b, layer, st);
}
void launch_ffn_down(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    const int wt = m.h.experts ? m.mats[m.e_w1[(size_t)layer * m.h.experts] + 2].wtype : m.mats[m.w2a[layer]].wtype;
    VC4_DISPATCH(wt, down_t, m, s, b, layer, st);
}
void launch_logits(const DModel& m, const State& s, const Batch& b, cudaStream_t st) {
    logits_t<W_Q8>(m, s, b, st);
}

void launch_attention(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    Dims d = dims_of(m, s);
    const int group = d.heads / d.kv_heads, hd = d.head_dim;
    const size_t sm = kRedBytes + sizeof(float) * ((size_t)group * hd + 2 * hd + (size_t)kTile * (hd + 1) +
                                             (size_t)group * d.seq) +
                      16 + sizeof(double) * (size_t)kWarps * group * hd;
    set_smem(k_attn, sm);
    k_attn<<<dim3(d.kv_heads, b.n), kThreads, sm, st>>>(m.d_q_norm, m.d_k_norm, s, b, d, layer);
}

void launch_matvec_raw(const DModel& m, int mat, const int16_t* xq, int n, int32_t* out, cudaStream_t st) {
    const DMat& W = m.mats[mat];
    if (W.wtype == W_I16) { k_raw_i16<<<W.rows, kThreads, 0, st>>>(W, xq, n, out); return; }
    const size_t sm = smem_bytes(1, x_stride(W), g_stride(W), 0);
    if (W.wtype == W_Q8) { set_smem(k_raw<W_Q8>, sm); k_raw<W_Q8><<<W.rblocks, kThreads, sm, st>>>(W, xq, n, out); }
    else if (W.wtype == W_Q4) { set_smem(k_raw<W_Q4>, sm); k_raw<W_Q4><<<W.rblocks, kThreads, sm, st>>>(W, xq, n, out); }
    else { set_smem(k_raw<W_T3>, sm); k_raw<W_T3><<<W.rblocks, kThreads, sm, st>>>(W, xq, n, out); }
}

void launch_finalize(const State& s, const Batch& b, int* next, int* tokens, int* pos, int advance,
                     const int* forced, cudaStream_t st) {
    k_finalize<<<(b.n + 127) / 128, 128, 0, st>>>(s, b, next, tokens, pos, advance, forced);
}

int kernel_launches_per_step(const DModel& m, int n) {
    const int g = (n + kNB - 1) / kNB;
    return m.h.layers * (4 * g + 1) + g + 1;
}

}  // namespace vc4
