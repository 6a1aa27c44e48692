// kernels.cuh -- sm_100a kernels of the quantized decode step (shared by the
// translation units: kernels.cu holds the weight-type independent kernels and
// the launch entry points, ops_q8.cu / ops_q4.cu / ops_t3.cu instantiate the
// matvec kernels of one weight type each, so the three compile in parallel).
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
#pragma once
#include "vc4b200_internal.h"

#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

namespace vc4 {
namespace {

constexpr int kThreads = kWarps * 32;
constexpr size_t kMaxDynSmem = 227 * 1024;   // opt-in dynamic shared memory per CTA on sm_100
__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

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

// Exact conversions on the integer and FMA pipes instead of the conversion
// (XU) pipe, which bounds the instruction-heavy epilogues.  1.5 * 2^23 has a
// unit ulp: adding it to |v| < 2^22 rounds v to the nearest integer (ties to
// even, the rounding of cvt.rni and of lrintf) and leaves that integer in the
// low mantissa bits.
constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
constexpr int kMagicBits = 0x4B400000;
__device__ __forceinline__ float i2f_small(int i) {   // (float)i, |i| < 2^22
    return __fsub_rn(__int_as_float(kMagicBits + i), kMagic);
}
__device__ __forceinline__ int f2i_rn_small(float v) {   // __float2int_rn(v), |v| < 2^22
    return __float_as_int(__fadd_rn(v, kMagic)) - kMagicBits;
}
__device__ __forceinline__ float rint_small(float v) {   // rintf(v) up to the sign of a zero, |v| < 2^22
    return __fsub_rn(__fadd_rn(v, kMagic), kMagic);
}

// q16 host quantisation: lrintf(v*256) clamped (common.h:188-193).  Values
// beyond +-2^22 clamp to the rail either way; NaN gives 0 (cvt.rni's value).
__device__ __forceinline__ int q16h(float v) {
    const float t = fminf(fmaxf(__fmul_rn(v, 256.0f), -4194304.0f), 4194303.0f);
    const int q = f2i_rn_small(t);
    return v != v ? 0 : q < -32768 ? -32768 : q > 32767 ? 32767 : q;
}
// q16 shader store: clamp(floor(v*256+0.5)) (xformat.cpp x_st2).
__device__ __forceinline__ int q16s(float v) {
    float f = floorf(__fadd_rn(__fmul_rn(v, 256.0f), 0.5f));
    f = f < -32768.0f ? -32768.0f : f > 32767.0f ? 32767.0f : f;
    return (int)f;
}
// Matvec epilogue: floor(S*sc + 0.5) clamped to the q16 rail, in double.
__device__ __forceinline__ int mv_epi(long long S, float sc) {
    double v = floor(__dadd_rn(__dmul_rn(__ll2double_rn(S), (double)sc), 0.5));
    v = v < -32768.0 ? -32768.0 : v > 32767.0 ? 32767.0 : v;
    return (int)v;
}
__device__ __noinline__ int mv_epi_dbl(long long S, float sc) { return mv_epi(S, sc); }
// A row scale as sc = m * 2^-sh with an integer mantissa m (carrying the
// sign; zero is m = 0, sh = 1).  sh = 0 marks a scale (subnormal, inf, NaN)
// that only the double path takes.
struct RowScale {
    int m, sh;
    float sc;
};
__device__ __forceinline__ RowScale row_scale(float sc) {
    const unsigned u = __float_as_uint(sc);
    const int e = (int)((u >> 23) & 0xFFu);
    RowScale r;
    r.sc = sc;
    if (e == 0 && (u & 0x7FFFFFu) == 0) {
        r.m = 0;
        r.sh = 1;
    } else if (e == 0 || e == 0xFF) {
        r.m = 0;
        r.sh = 0;
    } else {
        const int mant = (int)((u & 0x7FFFFFu) | 0x800000u);
        r.m = (u >> 31) ? -mant : mant;
        r.sh = 150 - e;
    }
    return r;
}
// The same value without the conversion pipe.  For |S| < 2^28 and
// 1 <= sh <= 53, |S*m| < 2^52 and |S*m| + 2^(sh-1) < 2^53, so the double
// path's product and its +0.5 are exact and its floor is the integer
// (S*m + 2^(sh-1)) >> sh (an arithmetic shift floors).  Other inputs take the
// double path.
// The integer form, without branches; `ok` is false where the double path
// must be taken instead (the caller fixes those up outside its chains).
__device__ __forceinline__ int mv_epi_int(long long S, const RowScale& r, bool& ok) {
    ok = r.sh >= 1 && r.sh <= 53 && S > -(1LL << 28) && S < (1LL << 28);
    const int sh = min(max(r.sh, 1), 53);
    const long long v = ((long long)(int)S * r.m + (1LL << (sh - 1))) >> sh;
    return v < -32768 ? -32768 : v > 32767 ? 32767 : (int)v;
}
__device__ __forceinline__ int mv_epi(long long S, const RowScale& r) {
    bool ok;
    const int v = mv_epi_int(S, r, ok);
    return ok ? v : mv_epi_dbl(S, r.sc);
}
// 2^k for -126 <= k <= 127, built in the exponent field (exact).
__device__ __forceinline__ float pow2f(int k) { return __int_as_float((127 + k) << 23); }

// Portable exp: Cody-Waite reduction + degree-7 Taylor (same ops as orc_expf).
// Written without branches, so that the many independent exps of an epilogue
// interleave: the reduction runs on x clamped to the finite range, the
// scaling p * 2^k is (p * 2^a) * 2^b with a + b = k and both factors normal
// (a = 1 for k = 128, as p*2 then 2^(k-1); a = k + 64, b = -64 below 2^-126;
// b = 0 otherwise, an exact multiply by one), and the out-of-range and NaN
// inputs are selected at the end.
__device__ __forceinline__ float vexp(float x) {
    const float xc = fminf(fmaxf(x, -103.97208404541016f), 88.72283935546875f);
    const float k = rint_small(__fmul_rn(xc, 1.44269502162933349609375f));   // |k| <= 150
    float r = __fmaf_rn(-k, 0.693145751953125f, xc);
    r = __fmaf_rn(-k, 1.428606765330187045037746429443359375e-06f, r);
    float p = 1.98412698412698412698e-4f;
    p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ki = f2i_rn_small(k);
    const int ea = ki > 127 ? 1 : ki < -126 ? ki + 64 : ki;
    const int eb = ki - ea;
    float y = __fmul_rn(__fmul_rn(p, __int_as_float((ea + 127) << 23)), __int_as_float((eb + 127) << 23));
    y = x > 88.72283935546875f ? __int_as_float(0x7f800000) : y;
    y = x < -103.97208404541016f ? 0.0f : y;
    return x != x ? x : y;
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
// ---------------------------------------------------------------------------
// Input staging: q16 ints -> (optionally 2^k scaled) ints split into lo/hi bytes
// ---------------------------------------------------------------------------

constexpr int kPer = 16;   // vector elements per thread: inputs of up to 16*256 = 4096 columns

struct XStage {
    uint8_t* lo;       // [nb][stride]
    int8_t* hi;        // [nb][stride]
    int stride;        // padded column count
    int* gsum;         // q4: [nb][stride/32] group sums; t3: [nb] totals (in gsum[b*gstride])
    int gstride;
    int k[8];          // per input: power-of-two input scale (matvec_s)
};

// Copy n int16 from global to shared memory with every load issued before the
// first store (one DRAM round trip); 16-byte vectors when aligned.
__device__ __forceinline__ void load_vec(const int16_t* __restrict__ g, int n, int16_t* sm) {
    if ((n & 7) == 0 && (((uintptr_t)g | (uintptr_t)sm) & 15) == 0) {
        const int nv = n >> 3;
        uint4 t[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int v = threadIdx.x + i * blockDim.x;
            if (v < nv) t[i] = __ldcg(reinterpret_cast<const uint4*>(g) + v);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int v = threadIdx.x + i * blockDim.x;
            if (v < nv) reinterpret_cast<uint4*>(sm)[v] = t[i];
        }
        return;
    }
    int16_t t[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        t[i] = c < n ? __ldcg(g + c) : (int16_t)0;
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < n) sm[c] = t[i];
    }
}

// This thread's elements c = threadIdx.x + i*blockDim.x of a float vector,
// loaded into registers (the per-layer norm weights, prefetched early).
__device__ __forceinline__ void load_f32_regs(const float* __restrict__ g, int n, float (&r)[kPer]) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        r[i] = c < n ? __ldg(g + c) : 0.0f;
    }
}

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
// round-half-even), zero-padded to `stride`; q4 group sums by warp shuffles
// (a warp covers one 32-column group per iteration), the t3 total by a block
// reduction.  v is in shared memory.  Ends with a barrier.
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
        if (WT == W_Q4) {
            int g = q;
            for (int o = 16; o; o >>= 1) g += __shfl_xor_sync(0xffffffffu, g, o);
            if ((threadIdx.x & 31) == 0) xs.gsum[b * xs.gstride + (c >> 5)] = g;
        }
        tot += q;
    }
    if (WT == W_T3) {
        const long long t = block_sum_i64(tot, r);
        if (threadIdx.x == 0) xs.gsum[b * xs.gstride] = (int)t;
    }
    __syncthreads();
}

// RMSNorm of a q16 vector into q16 ints (session.cpp:1932-1948 with the exact
// integer sum of squares rounded once).  x and out are shared memory; w holds
// this thread's norm weights (load_f32_regs).
__device__ void rmsnorm_q16(const int16_t* x, const float (&w)[kPer], int D, float eps, int16_t* out, Red& r) {
    long long ss = 0;
    for (int c = threadIdx.x; c < D; c += blockDim.x) { const long long a = x[c]; ss += a * a; }
    ss = block_sum_i64(ss, r);
    const float s1 = __fmul_rn(__ll2float_rn(ss), 1.0f / 65536.0f);
    const float s2 = __fdiv_rn(s1, (float)D);
    const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s2, eps)));
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < D) {
            const float xv = __fmul_rn((float)x[c], 1.0f / 256.0f);
            out[c] = (int16_t)q16h(__fmul_rn(w[i], __fmul_rn(rr, xv)));
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Matvec core: one 32-row block of one matrix over nb staged inputs.
// Warp w owns chunks w, w+8, w+16, ...; each lane owns one row.  The chunks a
// warp needs are loaded into registers first (mv_prefetch), before the kernel
// waits on its predecessor, so the DRAM latency of the weights overlaps the
// previous kernel; mv_compute then returns the warp's exact partial sums.
// ---------------------------------------------------------------------------

// Programmatic dependent launch: let the next kernel start its weight
// prefetch now; wait for the previous kernel's results before touching them.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ int4 ld_weights(const int4* p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}


// ---------------------------------------------------------------------------
// Bulk copies (cp.async.bulk, the 1-D TMA) into shared memory, completed on
// mbarriers.  Waits are bounded by the global timer.
// ---------------------------------------------------------------------------

__device__ __forceinline__ unsigned smem_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
// Makes mbarrier initialisation visible to the asynchronous (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses before
// later bulk copies into the same memory.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// global -> shared, `bytes` a multiple of 16, both addresses 16-byte aligned.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned long long* bar, unsigned parity) {
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Waits for phase `parity` of `bar`; false if it has not completed within
// `limit_ns` (the caller then reports an error instead of waiting for ever).
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity,
                                          unsigned long long limit_ns = 100000000ull) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try(bar, parity))
        if (global_ns() - t0 > limit_ns) return false;
    return true;
}

// cp.async: 16- or 4-byte global -> shared copies, completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Error word values besides shared-memory shortfalls (which record the bytes needed).
constexpr int kErrCopyTimeout = -2;
constexpr int kErrRingShape = -3;   // a tensor-core matmat launched with a ring or box plan it cannot run
constexpr int kStreamStages = 4;   // ring depth of the streaming kernels

template <int MAXC>
struct WRegs {
    int4 w[MAXC];
    int sp[MAXC];   // q4: packed (s16 | m16 << 16) of the chunk's scale group
    float rs;       // the epilogue scale of this lane's row
};

template <int WT, int MAXC>
__device__ __forceinline__ void mv_prefetch(const DMat& W, int blk, WRegs<MAXC>& R) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nch = W.nchunks;
    const int4* body = reinterpret_cast<const int4*>(W.body) + (size_t)blk * nch * 32 + lane;
#pragma unroll
    for (int k = 0; k < MAXC; ++k) {
        const int j = warp + k * kWarps;
        if (j < nch) {
            R.w[k] = ld_weights(body + (size_t)j * 32);
            if (WT == W_Q4) R.sp[k] = __ldg(W.q4p + ((size_t)blk * nch + j) * 32 + lane);
        }
    }
    R.rs = __ldg(W.rscale + (size_t)blk * 32 + lane);
}

// OWN: the staged input holds only this warp's chunks, slot k for chunk j.
template <int WT, int NB, int MAXC, bool OWN = false>
__device__ __forceinline__ void mv_compute(const DMat& W, const WRegs<MAXC>& R, const XStage& xs, int nb,
                                           long long (&S)[NB]) {
    const int warp = threadIdx.x >> 5, nch = W.nchunks;
    int alo[NB], ahi[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) { alo[b] = 0; ahi[b] = 0; S[b] = 0; }
#pragma unroll
    for (int k = 0; k < MAXC; ++k) {
        const int j = warp + k * kWarps;
        if (j >= nch) break;
        const int4 w = R.w[k];
        const int xi = OWN ? k : j;   // staged chunk index
        if (WT == W_Q8) {
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb) break;
                const uint4 L = *reinterpret_cast<const uint4*>(xs.lo + (size_t)b * xs.stride + xi * 16);
                const uint4 H = *reinterpret_cast<const uint4*>(xs.hi + (size_t)b * xs.stride + xi * 16);
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
                const uint4* L4 = reinterpret_cast<const uint4*>(xs.lo + (size_t)b * xs.stride + xi * 64);
                const uint4* H4 = reinterpret_cast<const uint4*>(xs.hi + (size_t)b * xs.stride + xi * 64);
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
            const long long s16 = (short)(R.sp[k] & 0xFFFF), m16 = (short)(R.sp[k] >> 16);
            const unsigned wd[4] = {(unsigned)w.x, (unsigned)w.y, (unsigned)w.z, (unsigned)w.w};
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb) break;
                const uint4* L4 = reinterpret_cast<const uint4*>(xs.lo + (size_t)b * xs.stride + xi * 32);
                const uint4* H4 = reinterpret_cast<const uint4*>(xs.hi + (size_t)b * xs.stride + xi * 32);
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
                S[b] += s16 * N + m16 * (long long)xs.gsum[b * xs.gstride + xi];
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
    static __device__ char* base() { extern __shared__ __align__(16) char smem[]; return smem; }
};

// Self-check before any shared-memory use: the launch must have reserved at
// least `need` bytes of dynamic shared memory.  A short launch records the
// shortfall in the session's error word and the block returns without
// touching shared memory (the host turns the word into an error).
__device__ __forceinline__ bool smem_ok(size_t need, int* err) {
    unsigned have;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(have));
    if ((size_t)have >= need) return true;
    if (threadIdx.x == 0) atomicMax(err, (int)need);
    return false;
}

// dynamic shared memory: [Red][partials kWarps*NB*32][gsum][lo][hi][scratch]
template <int NB>
__device__ void carve(int stride, int gstride, XStage& xs, Red*& red, long long*& part, int16_t*& tmp) {
    char* p = SmemLayout::base();
    red = reinterpret_cast<Red*>(p); p += (sizeof(Red) + 15) / 16 * 16;
    part = reinterpret_cast<long long*>(p); p += sizeof(long long) * kWarps * NB * 32;
    xs.gsum = reinterpret_cast<int*>(p); p += (sizeof(int) * NB * gstride + 15) / 16 * 16;
    xs.lo = reinterpret_cast<uint8_t*>(p); p += (size_t)NB * stride;
    xs.hi = reinterpret_cast<int8_t*>(p); p += (size_t)NB * stride;
    tmp = reinterpret_cast<int16_t*>(p);
    xs.stride = stride; xs.gstride = gstride;
}

__host__ __device__ size_t smem_bytes(int nb, int stride, int gstride, int tmp_n) {
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
    int hostffn;     // dense FFN in two chunks: the CPU layer loop's host FFN (see ffn_host below)
    float eps;
};

// The cache rows of (slot, layer): a position below the slot's shared-prefix
// length is a row of the session's shared prefix, any other its own row.
struct KvRows {
    uint8_t* own;
    const uint8_t* shared;
    int plen;
    __device__ __forceinline__ const uint8_t* at(int t, int row_bytes) const {
        return (t < plen ? shared : own) + (size_t)t * row_bytes;
    }
};
__device__ __forceinline__ KvRows kv_rows_of(const State& s, int slot, int layer, int layers, int seq, int row_bytes) {
    KvRows r;
    r.own = s.kv + ((size_t)slot * layers + layer) * seq * row_bytes;
    r.plen = s.plen ? __ldg(s.plen + slot) : 0;
    r.shared = s.pkv ? s.pkv + (size_t)layer * s.pcap * row_bytes : r.own;
    return r;
}
// An append at a position the shared prefix serves: recorded in the error
// word (the host reports it) and not written.
constexpr int kErrSharedAppend = -5;

Dims dims_of(const DModel& m, const State& s) {
    Dims d;
    d.dim = m.h.dim; d.kv_dim = m.h.kv_dim; d.heads = m.h.heads; d.kv_heads = m.h.kv_heads;
    d.head_dim = m.h.head_dim; d.layers = m.h.layers; d.vocab = m.h.vocab; d.ffn = m.ffn_width;
    d.chunk = m.ffn_chunk; d.experts = m.h.experts; d.seq = s.seq; d.row_bytes = s.row_bytes;
    d.kv_bits = s.kv_bits; d.rope_half = m.h.rope_half; d.qk_norm = m.h.qk_norm; d.eps = m.h.rms_eps;
    d.hostffn = (!m.h.experts && m.ffn_chunked) ? 1 : 0;
    return d;
}

// ---------------------------------------------------------------------------
// The two FFN forms of the reference CPU layer loop (session.cpp:475-551).
//  - GPU FFN (MoE, or a dense FFN of at most 2048 rows): the gate kernel
//    reads the q16 input as uploaded, stores SiLU(g)*u*2^-hs with the
//    shaders' floor(v*256 + 0.5), and w2 reads that q16 hidden vector as is
//    (gpu_ffn.cpp:17-132, gpu_matvec.cpp:32-55).
//  - Host FFN (a dense FFN split into two chunks): Model::split_ffn
//    (model.cpp:217-270, run by App::prepare_model) leaves w1 empty, so the
//    loop runs matvec_s on the gate/up halves (2^k input scale), the host
//    SwiGLU rounded with quantize_act (lrintf), times 2^-hs, then matvec_s of
//    each w2 half with its own 2^k (session.cpp:499-524, 2069-2080).  With
//    q = the q16 hidden ints of a half and max|q|/256 = f*2^e, that half's w2
//    input is rint(q * 2^(6-e)) and its output (v/256) * 2^-(6-e+hs).  For
//    6-e >= 0 the input is q shifted, so the exact dot is the unscaled one
//    times 2^(6-e): the w2 partial sums and records stay unscaled and the
//    epilogue applies the exponent from the half's maximum (State::hmax).
//    6-e < 0 (a hidden value of 64 or more) would round the input; the
//    kernels report it (kErrHiddenRange) rather than return other numbers.
// ---------------------------------------------------------------------------
constexpr int kErrHiddenRange = -4;

__host__ __device__ inline size_t hmax_at(int layer, int b, int half, int slots) {
    return (((size_t)layer * slots + b) * 2 + half);
}
// The w2 input exponent of one hidden half from its max |q16| (matvec_s: 6 - e).
__device__ __forceinline__ int hidden_exp(const State& s, int layer, int b, int half) {
    int e = 0;
    const int mx = __ldcg(s.hmax + hmax_at(layer, b, half, s.slots));
    if (mx == 0) return 0;
    frexpf(__fmul_rn((float)mx, 1.0f / 256.0f), &e);
    return 6 - e;
}
// One w2 half of the host FFN: (floor(S * 2^k * ws + 0.5) clamped)/256 * 2^-(k + hs).
// k >= 0 (the caller has refused negative exponents).
__device__ __forceinline__ float host_w2_out(long long S, const RowScale& ws, int k, int hs) {
    const float v = __fmul_rn(i2f_small(mv_epi(S * (1LL << k), ws)), 1.0f / 256.0f);
    return __fmul_rn(v, pow2f(-(k + hs)));
}
__device__ __forceinline__ float host_w2_out(long long S, float ws, int k, int hs) {
    const float v = __fmul_rn((float)mv_epi(S * (1LL << k), ws), 1.0f / 256.0f);
    return __fmul_rn(v, pow2f(-(k + hs)));
}
__device__ __forceinline__ float host_w2_out(long long S, float ws, int k, int hs, int* err) {
    if (k < 0) {
        atomicExch(err, kErrHiddenRange);
        k = 0;
    }
    return host_w2_out(S, ws, k, hs);
}
// The host FFN's gate value: the hidden q16 int of SiLU(g)*u with g, u the
// matvec_s outputs of a 2^k scaled input (quantize_act: lrintf).
__device__ __forceinline__ int host_hidden(int g, int u, int k) {
    const float sk = pow2f(-k);
    const float gf = __fmul_rn(__fmul_rn(i2f_small(g), 1.0f / 256.0f), sk);
    const float uf = __fmul_rn(__fmul_rn(i2f_small(u), 1.0f / 256.0f), sk);
    return q16h(swiglu1(gf, uf));
}

// ---------------------------------------------------------------------------
// Per-pass activations are indexed by the batch position b; only the KV cache
// is indexed by the sequence's slot.  Every kernel issues its weight, scale
// and norm-weight loads before griddepcontrol.wait and needs one dependent
// round trip for its activations afterwards.
// ---------------------------------------------------------------------------

// Two matrices a kernel reads by value, per expert for MoE (blockIdx.y).
struct MatSet {
    DMat a[8];
    DMat b[8];
    DMat router;
};

// ---------------------------------------------------------------------------
// Warp-staged matvec kernels.  Warp w of a CTA computes the dot products of
// the column chunks j = w, w + kWarps, ... (its slots k = 0, 1, ...), so it
// only reads the input bytes of those chunks.  Every warp prepares them
// itself from the whole input vector in shared memory: the RMSNorm sum of
// squares, the power-of-two input scale (from the maximum over all columns)
// and the t3 column total are warp reductions, identical in every warp, and
// the bytes of x' = x*2^k for the warp's own chunks go to its own slice.  A
// kernel therefore has two block barriers: after its inputs land in shared
// memory, and for the cross-warp sum of the dot products.
// ---------------------------------------------------------------------------

struct WStage {     // one warp's slice of staged input bytes
    uint8_t* lo;    // [nb][wst]
    int8_t* hi;     // [nb][wst]
    int* gsum;      // q4: [nb][gst] chunk sums; t3: [nb] totals (gsum[b*gst])
    int wst, gst;
};

__host__ __device__ inline int own_slots(int nch) { return (nch + kWarps - 1) / kWarps; }
__host__ __device__ inline size_t wstage_bytes(const DMat& W, int nb) {
    const int own = own_slots(W.nchunks), cpc = cpc_of(W.wtype), gst = W.wtype == W_Q4 ? own : 1;
    return align16((size_t)2 * nb * own * cpc) + align16(sizeof(int) * (size_t)nb * gst);
}
__device__ __forceinline__ WStage wstage_at(const DMat& W, int nb, char* base) {
    WStage w;
    const int own = own_slots(W.nchunks);
    char* p = base + (size_t)(threadIdx.x >> 5) * wstage_bytes(W, nb);
    w.wst = own * cpc_of(W.wtype);
    w.gst = W.wtype == W_Q4 ? own : 1;
    w.lo = reinterpret_cast<uint8_t*>(p);
    w.hi = reinterpret_cast<int8_t*>(p + (size_t)nb * w.wst);
    w.gsum = reinterpret_cast<int*>(p + align16((size_t)2 * nb * w.wst));
    return w;
}
__device__ __forceinline__ XStage xstage_of(const WStage& w) {
    XStage x;
    x.lo = w.lo; x.hi = w.hi; x.stride = w.wst; x.gsum = w.gsum; x.gstride = w.gst;
    return x;
}

// Dynamic shared memory of the warp-staged kernels.
struct MvLayout {
    size_t part, x, nw, ws, extra, total;
};
__host__ __device__ inline MvLayout mv_layout(size_t ws_per_warp, int nb, int nvals, int nnw, size_t extra) {
    MvLayout L;
    size_t o = 0;
    L.part = o;  o = align16(o + sizeof(long long) * 2 * kWarps * (size_t)nb * 32);
    L.x = o;     o = align16(o + sizeof(int16_t) * (size_t)nvals);
    L.nw = o;    o = align16(o + sizeof(float) * (size_t)nnw);
    L.ws = o;    o = align16(o + kWarps * ws_per_warp);
    L.extra = o; o = align16(o + extra);
    L.total = o;
    return L;
}

__device__ __forceinline__ long long warp_sum_i64(long long v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// matvec_s input scale: k = 6 - e for max|x| = f*2^e (gpu_conv.cpp:271-287), 0 for a zero vector.
__device__ __forceinline__ int exp_from_max(int mx) {
    if (mx == 0) return 0;
    int e = 0;
    frexpf(__fmul_rn((float)mx, 1.0f / 256.0f), &e);
    return 6 - e;
}
// 1/sqrt(mean(x^2) + eps) of a q16 vector from its exact integer sum of squares
// (session.cpp:1932-1948, the sum rounded once).
__device__ __forceinline__ float rms_rr(long long ss, int D, float eps) {
    const float s1 = __fmul_rn(__ll2float_rn(ss), 1.0f / 65536.0f);
    const float s2 = __fdiv_rn(s1, (float)D);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s2, eps)));
}
__device__ __forceinline__ int xnorm(int a, float w, float rr) {
    return q16h(__fmul_rn(w, __fmul_rn(rr, __fmul_rn((float)a, 1.0f / 256.0f))));
}
__device__ __forceinline__ int xscale(int a, int k, float sk) {
    return k >= 0 ? (a << k) : __float2int_rn(__fmul_rn((float)a, sk));
}
__device__ __forceinline__ long long warp_sumsq(const int16_t* x, int D) {
    long long ss = 0;
#pragma unroll 8
    for (int c = (threadIdx.x & 31); c < D; c += 32) { const int a = x[c]; ss += a * a; }
    return warp_sum_i64(ss);
}

// x'[c] = value(c)*2^k into the warp's slice for the columns of its own
// chunks (zero past D); q4: the sum of each chunk; t3: the total over all D
// columns.  Ends with the slice written by this warp (caller: __syncwarp).
template <int WT, typename F>
__device__ __forceinline__ void warp_stage(const WStage& ws, int b, int nch, int D, int k, F value) {
    constexpr int cpc = WT == W_Q8 ? 16 : WT == W_Q4 ? 32 : 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float sk = ldexpf(1.0f, k);
    uint8_t* lo = ws.lo + (size_t)b * ws.wst;
    int8_t* hi = ws.hi + (size_t)b * ws.wst;
#pragma unroll 4
    for (int e = lane; e < ws.wst; e += 32) {
        const int slot = e / cpc, j = warp + slot * kWarps, c = j * cpc + e % cpc;
        const int q = (j < nch && c < D) ? xscale(value(c), k, sk) : 0;
        lo[e] = (uint8_t)(q & 0xFF);
        hi[e] = (int8_t)(q >> 8);
        if (WT == W_Q4) {   // wst is a multiple of 32: every lane is here, one chunk per pass
            const int gs = __reduce_add_sync(0xffffffffu, q);
            if (lane == 0) ws.gsum[b * ws.gst + slot] = gs;
        }
    }
    if (WT == W_T3) {
        int t = 0;
#pragma unroll 8
        for (int c = lane; c < D; c += 32) t += xscale(value(c), k, sk);
        t = __reduce_add_sync(0xffffffffu, t);
        if (lane == 0) ws.gsum[b * ws.gst] = t;
    }
}

// Cross-warp sum of V partial dot products per (input, row) with one block
// barrier; on return warps b < nb hold the totals of input b, row `lane`.
// The partial buffer is not reused afterwards.
template <int NB, int V>
__device__ __forceinline__ void reduce_once(const long long (&S)[V][NB], int nb, long long* red,
                                            long long (&out)[V]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
        for (int b = 0; b < NB; ++b) red[((warp * V + v) * NB + b) * 32 + lane] = S[v][b];
    __syncthreads();
#pragma unroll
    for (int v = 0; v < V; ++v) {
        long long t = 0;
        if (warp < nb)
            for (int w = 0; w < kWarps; ++w) t += red[((w * V + v) * NB + warp) * 32 + lane];
        out[v] = t;
    }
}

// ---------------------------------------------------------------------------
// FFN output by partial sums.  The w2 matvec takes the q16 hidden vector
// without input scaling, so its exact integer dot product is the sum over any
// split of the columns.  Each gate CTA multiplies its own 32 hidden values by
// the matching 32 columns of w2 and adds the per-row partial sums into
// State::sdown (int64, so the order of the additions does not matter); the
// consumer of the layer's output (the next layer's qkv kernel, or logits)
// applies the w2 row scales and the residual add.  A chunked w2 (hidden width
// above the chunk) keeps one sum per column half, each rounded to q16 before
// add_q16, as the chunked FFN does (gpu_ffn.cpp:67-132, session.cpp:2052-2067).
// ---------------------------------------------------------------------------

__host__ __device__ inline size_t sdown_at(int layer, int b, int half, int dim, int slots) {
    return (((size_t)layer * slots + b) * 2 + half) * dim;
}

// Where the consumer finds the w2 row scales of the layer it rebuilds.
struct DownSrc {
    int layer;            // the layer whose FFN output is rebuilt; -1: none (layer 0 input is the embedding)
    int two;              // chunked w2
    int hs;               // that layer's key-15 hidden shift (host FFN output scale)
    const float* ra;      // dense model: row scales of the two w2 halves
    const float* rb;
    const DMat* dm;       // MoE: the device matrix table, expert e's halves at dm[ia + 4e], dm[ib + 4e]
    int ia, ib;
};

// One chunk of one row: the same integer arithmetic as mv_compute for input
// bytes lo/hi of the chunk's columns; q4: gsum = the chunk's input sum.
template <int WT>
__device__ __forceinline__ long long chunk_dot(const int4 w, int sp, const uint8_t* lo, const int8_t* hi, int gsum) {
    if (WT == W_Q8) {
        const uint4 L = *reinterpret_cast<const uint4*>(lo), H = *reinterpret_cast<const uint4*>(hi);
        int a = 0, c = 0;
        a = dp4a_su(w.x, L.x, a); a = dp4a_su(w.y, L.y, a); a = dp4a_su(w.z, L.z, a); a = dp4a_su(w.w, L.w, a);
        c = dp4a_ss(w.x, (int)H.x, c); c = dp4a_ss(w.y, (int)H.y, c); c = dp4a_ss(w.z, (int)H.z, c); c = dp4a_ss(w.w, (int)H.w, c);
        return (long long)a + 256LL * c;
    } else if (WT == W_T3) {
        const unsigned wd[4] = {(unsigned)w.x, (unsigned)w.y, (unsigned)w.z, (unsigned)w.w};
        const uint4* L4 = reinterpret_cast<const uint4*>(lo);
        const uint4* H4 = reinterpret_cast<const uint4*>(hi);
        int a = 0, c = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 L = L4[q], H = H4[q];
            const unsigned e0 = wd[q] & 0x03030303u, e1 = (wd[q] >> 2) & 0x03030303u;
            const unsigned e2 = (wd[q] >> 4) & 0x03030303u, e3 = (wd[q] >> 6) & 0x03030303u;
            a = dp4a_uu(e0, L.x, a); a = dp4a_uu(e1, L.y, a); a = dp4a_uu(e2, L.z, a); a = dp4a_uu(e3, L.w, a);
            c = dp4a_us(e0, (int)H.x, c); c = dp4a_us(e1, (int)H.y, c); c = dp4a_us(e2, (int)H.z, c); c = dp4a_us(e3, (int)H.w, c);
        }
        return (long long)a + 256LL * c;
    } else {
        const long long s16 = (short)(sp & 0xFFFF), m16 = (short)(sp >> 16);
        const unsigned wd[4] = {(unsigned)w.x, (unsigned)w.y, (unsigned)w.z, (unsigned)w.w};
        const uint4* L4 = reinterpret_cast<const uint4*>(lo);
        const uint4* H4 = reinterpret_cast<const uint4*>(hi);
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
        return s16 * ((long long)nlo + 256LL * nhi) + m16 * (long long)gsum;
    }
}

// x = add_q16(x1, FFN output) of input bi (its batch position) from the
// layer's partial sums, block-wide into xout; `write` also stores it to s.x.
__device__ __forceinline__ void rebuild_x(const State& s, const Dims& d, const DownSrc& ds, int bi, int16_t* xout,
                                          bool write) {
    const float* ra = ds.ra;
    const float* rb = ds.rb;
    if (d.experts) {
        const int e = __ldcg(s.route + (size_t)bi * d.layers + ds.layer);
        ra = ds.dm[ds.ia + 4 * e].rscale;
        if (ds.two) rb = ds.dm[ds.ib + 4 * e].rscale;
    }
    const long long* S = s.sdown + sdown_at(ds.layer, bi, 0, d.dim, s.slots);
    const int16_t* x1 = s.x1 + (size_t)bi * d.dim;
    // the host FFN's w2 input exponents: their loads go out with the first
    // round's, the exponents are taken after
    const int ma = d.hostffn ? __ldcg(s.hmax + hmax_at(ds.layer, bi, 0, s.slots)) : 0;
    const int mb = d.hostffn ? __ldcg(s.hmax + hmax_at(ds.layer, bi, 1, s.slots)) : 0;
    int ka = 0, kb = 0;
    // kU rows per thread per round: every load of a round is issued before the first use
    constexpr int kU = 4;
    for (int base = 0; base < d.dim; base += kU * kThreads) {
        long long sa[kU], sb[kU];
        float fa[kU], fb[kU];
        int xv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int r = base + u * kThreads + threadIdx.x;
            sa[u] = sb[u] = 0;
            fa[u] = fb[u] = 0.0f;
            xv[u] = 0;
            if (r < d.dim) {
                sa[u] = __ldcg(S + r);
                fa[u] = __ldg(ra + r);
                if (ds.two) { sb[u] = __ldcg(S + d.dim + r); fb[u] = __ldg(rb + r); }
                xv[u] = __ldcg(x1 + r);
            }
        }
        if (d.hostffn && base == 0) {
            ka = exp_from_max(ma);
            kb = exp_from_max(mb);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int r = base + u * kThreads + threadIdx.x;
            if (r >= d.dim) continue;
            float o2;
            if (d.hostffn) {
                const float oa = host_w2_out(sa[u], fa[u], ka, ds.hs, s.err);
                const float ob = host_w2_out(sb[u], fb[u], kb, ds.hs, s.err);
                o2 = __fmul_rn((float)q16h(__fadd_rn(oa, ob)), 1.0f / 256.0f);
            } else {
                o2 = __fmul_rn((float)mv_epi(sa[u], fa[u]), 1.0f / 256.0f);
                if (ds.two) {
                    const int vb = mv_epi(sb[u], fb[u]);
                    o2 = __fmul_rn((float)q16h(__fadd_rn(o2, __fmul_rn((float)vb, 1.0f / 256.0f))), 1.0f / 256.0f);
                }
            }
            const int16_t x = (int16_t)q16h(__fadd_rn(__fmul_rn((float)xv[u], 1.0f / 256.0f), o2));
            xout[r] = x;
            if (write) s.x[(size_t)bi * d.dim + r] = x;
        }
    }
}

// Zeroes the partial sums of `layer` for every batch position, split over the grid.
__device__ __forceinline__ void zero_sdown(const State& s, const Dims& d, int layer) {
    const size_t n = (size_t)s.slots * 2 * d.dim;                  // int64 values, a multiple of 2
    uint4* p = reinterpret_cast<uint4*>(s.sdown + sdown_at(layer, 0, 0, d.dim, s.slots));
    const size_t nv = n / 2, per = (nv + gridDim.x - 1) / gridDim.x;
    const size_t v0 = (size_t)blockIdx.x * per, v1 = v0 + per < nv ? v0 + per : nv;
    for (size_t v = v0 + threadIdx.x; v < v1; v += kThreads) p[v] = make_uint4(0u, 0u, 0u, 0u);
}

// ---------------------------------------------------------------------------
// qkv: embedding (layer 0) or x, RMSNorm, matvec_s(qkv) -> fp32 qkv
// ---------------------------------------------------------------------------

template <int WT, int NB, int MAXC>
__global__ void __launch_bounds__(kThreads) k_qkv(DMat W, DMat E, const float* emb_scale, const float* rms_w,
                                                  State s, Batch bt, Dims d, int layer, int b0, DownSrc ds) {
    const MvLayout L = mv_layout(wstage_bytes(W, NB), NB, NB * d.dim, d.dim, 0);
    if (!smem_ok(L.total, s.err)) return;
    char* sm = SmemLayout::base();
    WRegs<MAXC> R;
    mv_prefetch<WT, MAXC>(W, blockIdx.x, R);
    float* nws = reinterpret_cast<float*>(sm + L.nw);
    for (int c = threadIdx.x; c < d.dim; c += kThreads) nws[c] = __ldg(rms_w + c);
    pdl_launch_dependents();
    pdl_wait();
    int16_t* xv = reinterpret_cast<int16_t*>(sm + L.x);
    const int nb = min(NB, bt.n - b0);
    // the host FFN maxima this layer's gate kernel accumulates start from zero
    if (d.hostffn && blockIdx.x == 0 && threadIdx.x < 2 * nb)
        s.hmax[hmax_at(layer, b0 + threadIdx.x / 2, threadIdx.x % 2, s.slots)] = 0;
    for (int b = 0; b < nb; ++b) {
        const int bi = b0 + b;
        int16_t* xin = xv + (size_t)b * d.dim;
        if (layer == 0) {
            // embedding (session.cpp:342-371): q16(level * row scale); the row
            // is read from the blocked q8 layout of the embedding matrix.
            const int tok = bt.token[bi];
            const float es = emb_scale[tok];
            const int8_t* eb = reinterpret_cast<const int8_t*>(E.body) + ((size_t)(tok / 32) * E.nchunks * 32 + (tok % 32)) * 16;
            int16_t* x = s.x + (size_t)bi * d.dim;
#pragma unroll 4
            for (int c = threadIdx.x; c < d.dim; c += kThreads) {
                const int16_t q = (int16_t)q16h(__fmul_rn((float)eb[(size_t)(c / 16) * 512 + (c % 16)], es));
                xin[c] = q;
                if (blockIdx.x == 0) x[c] = q;
            }
            if (blockIdx.x == 0 && threadIdx.x == 0) s.best[bi] = 0ull;
        } else {
            rebuild_x(s, d, ds, bi, xin, blockIdx.x == 0);
        }
    }
    // the logits of the previous pass have consumed the last layer's sums
    if (layer == 0 && b0 == 0) zero_sdown(s, d, d.layers - 1);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const WStage ws = wstage_at(W, NB, sm + L.ws);
    int kw = 0;   // input scale of input `warp` (its epilogue)
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= nb) break;
        const int16_t* x = xv + (size_t)b * d.dim;
        const float rr = rms_rr(warp_sumsq(x, d.dim), d.dim, d.eps);
        int mx = 0;
#pragma unroll 8
        for (int c = lane; c < d.dim; c += 32) mx = max(mx, abs(xnorm(x[c], nws[c], rr)));
        const int k = exp_from_max(__reduce_max_sync(0xffffffffu, mx));
        if (b == warp) kw = k;
        warp_stage<WT>(ws, b, W.nchunks, d.dim, k, [&](int c) { return xnorm(x[c], nws[c], rr); });
    }
    __syncwarp();
    long long S[1][NB], tot[1];
    mv_compute<WT, NB, MAXC, true>(W, R, xstage_of(ws), nb, S[0]);
    reduce_once<NB, 1>(S, nb, reinterpret_cast<long long*>(sm + L.part), tot);
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        if (row < W.rows) {
            const long long St = WT == W_T3 ? tot[0] - ws.gsum[warp * ws.gst] : tot[0];
            const int v = mv_epi(St, R.rs);
            const float out = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), pow2f(-kw));
            s.qkv[(size_t)(b0 + warp) * (d.dim + 2 * d.kv_dim) + row] = out;
        }
    }
}

// ---------------------------------------------------------------------------
// wo: matvec_s(wo, att) + add_q16 residual -> x1
// ---------------------------------------------------------------------------

template <int WT, int NB, int MAXC>
__global__ void __launch_bounds__(kThreads) k_wo(DMat W, State s, Batch bt, Dims d, int layer, int b0) {
    const MvLayout L = mv_layout(wstage_bytes(W, NB), NB, NB * d.dim, 0, 0);
    if (!smem_ok(L.total, s.err)) return;
    char* sm = SmemLayout::base();
    WRegs<MAXC> R;
    mv_prefetch<WT, MAXC>(W, blockIdx.x, R);
    pdl_launch_dependents();
    pdl_wait();
    const int nb = min(NB, bt.n - b0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 32 + lane;
    // the residual this thread's epilogue adds, fetched with the inputs
    const int xres = (warp < nb && row < W.rows) ? (int)__ldcg(s.x + (size_t)(b0 + warp) * d.dim + row) : 0;
    if (layer > 0 && b0 == 0) zero_sdown(s, d, layer - 1);   // this layer's qkv has consumed them
    int16_t* av = reinterpret_cast<int16_t*>(sm + L.x);
    for (int b = 0; b < nb; ++b) load_vec(s.att + (size_t)(b0 + b) * d.dim, d.dim, av + (size_t)b * d.dim);
    __syncthreads();
    const WStage ws = wstage_at(W, NB, sm + L.ws);
    int kw = 0;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= nb) break;
        const int16_t* a = av + (size_t)b * d.dim;
        int mx = 0;
#pragma unroll 8
        for (int c = lane; c < d.dim; c += 32) mx = max(mx, abs((int)a[c]));
        const int k = exp_from_max(__reduce_max_sync(0xffffffffu, mx));
        if (b == warp) kw = k;
        warp_stage<WT>(ws, b, W.nchunks, d.dim, k, [&](int c) { return (int)a[c]; });
    }
    __syncwarp();
    long long S[1][NB], tot[1];
    mv_compute<WT, NB, MAXC, true>(W, R, xstage_of(ws), nb, S[0]);
    reduce_once<NB, 1>(S, nb, reinterpret_cast<long long*>(sm + L.part), tot);
    if (warp < nb && row < W.rows) {
        const long long St = WT == W_T3 ? tot[0] - ws.gsum[warp * ws.gst] : tot[0];
        const int v = mv_epi(St, R.rs);
        const float wo = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), pow2f(-kw));
        const float xr = __fmul_rn((float)xres, 1.0f / 256.0f);
        s.x1[(size_t)(b0 + warp) * d.dim + row] = (int16_t)q16h(__fadd_rn(xr, wo));
    }
}

// ---------------------------------------------------------------------------
// ffn: RMSNorm(x1), optional MoE routing (top-1, shaders.cpp:1216-1230 and
// session.cpp:110-115), w1/w3 matvecs and SwiGLU (q16 pair rounding,
// shaders.cpp:116-136) for this CTA's 32 hidden rows, then their share of w2:
// the rows' q16 values times the matching 32 columns of w2, added into the
// layer's partial sums (the GPU FFN path the CPU session draws).
// ---------------------------------------------------------------------------

constexpr int kFfnRB = 4;   // w2 row blocks per warp fetched before the dependency wait

template <int WT>
__host__ __device__ inline size_t ffn_down_bytes(int nb) {
    constexpr int span = WT == W_T3 ? 64 : 32;
    return align16((size_t)2 * nb * span) + align16(sizeof(int) * (size_t)nb * 33);
}

template <int WT, int NB, int MAXC>
__global__ void __launch_bounds__(kThreads) k_gate(MatSet M, MatSet M2, const float* rms_w, State s, Batch bt, Dims d,
                                                   int layer, int b0, int hs, int early) {
    constexpr int cpc = WT == W_Q8 ? 16 : WT == W_Q4 ? 32 : 64;
    constexpr int span = WT == W_T3 ? 64 : 32;       // staged w2 input columns: the chunk(s) holding the 32 rows
    const int expert = blockIdx.y;
    const DMat& W1 = M.a[expert];
    const DMat& W3 = M.b[expert];
    // this CTA's hidden rows [32*bx, 32*bx + 32) are columns [c0, c0 + 32) of w2 half `half`
    const bool two = d.chunk < d.ffn;
    const int half = (two && 32 * (int)blockIdx.x >= d.chunk) ? 1 : 0;
    const DMat& W2 = half ? M2.b[expert] : M2.a[expert];
    const int c0 = 32 * (int)blockIdx.x - (half ? d.chunk : 0);
    const int j0 = c0 / cpc, off = c0 % cpc, nch2 = W2.nchunks;
    const size_t rbytes = d.experts ? sizeof(int16_t) * (size_t)d.experts * d.dim : 0;
    const MvLayout L = mv_layout(wstage_bytes(W1, NB), NB, NB * d.dim, d.dim, align16(rbytes + 64) + ffn_down_bytes<WT>(NB));
    if (!smem_ok(L.total, s.err)) return;
    char* sm = SmemLayout::base();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    WRegs<MAXC> R1, R3;
    int4 w2a[kFfnRB], w2b[kFfnRB];
    int w2p[kFfnRB];
    auto fetch_w2 = [&](int i, int4& wa, int4& wb, int& sp) {
        const int rb = warp + i * kWarps;
        const int4* body = reinterpret_cast<const int4*>(W2.body) + lane;
        wa = ld_weights(body + ((size_t)rb * nch2 + j0) * 32);
        if (WT == W_Q8 && j0 + 1 < nch2) wb = ld_weights(body + ((size_t)rb * nch2 + j0 + 1) * 32);
        if (WT == W_Q4) sp = __ldg(W2.q4p + ((size_t)rb * nch2 + j0) * 32 + lane);
    };
    auto prefetch = [&]() {
        mv_prefetch<WT, MAXC>(W1, blockIdx.x, R1);
        mv_prefetch<WT, MAXC>(W3, blockIdx.x, R3);
#pragma unroll
        for (int i = 0; i < kFfnRB; ++i)
            if (warp + i * kWarps < W2.rblocks) fetch_w2(i, w2a[i], w2b[i], w2p[i]);
    };
    if (early) prefetch();
    float* nws = reinterpret_cast<float*>(sm + L.nw);
    for (int c = threadIdx.x; c < d.dim; c += kThreads) nws[c] = __ldg(rms_w + c);
    int16_t* rw = reinterpret_cast<int16_t*>(sm + L.extra);             // router rows
    int* members = reinterpret_cast<int*>(sm + L.extra + align16(rbytes));
    uint8_t* dlo = reinterpret_cast<uint8_t*>(sm + L.extra + align16(rbytes + 64));
    int8_t* dhi = reinterpret_cast<int8_t*>(dlo + (size_t)NB * span);
    int* dsum = reinterpret_cast<int*>(sm + L.extra + align16(rbytes + 64) + align16((size_t)2 * NB * span));
    int* hq = dsum + NB;                                                  // [NB][32] q16 hidden values
    for (int i = threadIdx.x; i < d.experts * d.dim; i += kThreads) rw[i] = M.router.w16[i];
    pdl_launch_dependents();
    pdl_wait();
    int16_t* xv = reinterpret_cast<int16_t*>(sm + L.x);
    const int n_all = min(NB, bt.n - b0);
    for (int b = 0; b < n_all; ++b) load_vec(s.x1 + (size_t)(b0 + b) * d.dim, d.dim, xv + (size_t)b * d.dim);
    __syncthreads();
    const WStage ws = wstage_at(W1, NB, sm + L.ws);
    int nb = 0;
    int kx_own = 0;   // the input exponent of member `warp` (the warp's epilogue input)
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= n_all) break;
        const int16_t* x = xv + (size_t)b * d.dim;
        const float rr = rms_rr(warp_sumsq(x, d.dim), d.dim, d.eps);
        if (d.experts) {
            // router: matvec_s over the normalised input, first maximum wins
            int mx = 0;
    #pragma unroll 8
        for (int c = lane; c < d.dim; c += 32) mx = max(mx, abs(xnorm(x[c], nws[c], rr)));
            const int k = exp_from_max(__reduce_max_sync(0xffffffffu, mx));
            const float sk = ldexpf(1.0f, k);
            int best = 0;
            float bestv = 0.0f;
            for (int e = 0; e < d.experts; ++e) {
                long long acc = 0;
#pragma unroll 8
                for (int c = lane; c < d.dim; c += 32)
                    acc += (long long)rw[(size_t)e * d.dim + c] * xscale(xnorm(x[c], nws[c], rr), k, sk);
                const int v = mv_epi(warp_sum_i64(acc), M.router.rscale[e]);
                const float gv = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), ldexpf(1.0f, -k));
                if (e == 0 || gv > bestv) { best = e; bestv = gv; }
            }
            if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
                s.route[(size_t)(b0 + b) * d.layers + layer] = best;
            if (best != expert) continue;
        }
        if (threadIdx.x == 0) members[nb] = b;
        int kx = 0;
        if (d.hostffn) {   // matvec_s of the normalised input (gpu_conv.cpp:271-287)
            int mx = 0;
#pragma unroll 8
            for (int c = lane; c < d.dim; c += 32) mx = max(mx, abs(xnorm(x[c], nws[c], rr)));
            kx = exp_from_max(__reduce_max_sync(0xffffffffu, mx));
        }
        if (warp == nb) kx_own = kx;
        warp_stage<WT>(ws, nb, W1.nchunks, d.dim, kx, [&](int c) { return xnorm(x[c], nws[c], rr); });
        ++nb;
    }
    if (nb == 0) return;   // the same in every warp: no input routed to this expert
    if (!early) prefetch();
    __syncwarp();
    long long S[2][NB], tot[2];
    const XStage xs = xstage_of(ws);
    mv_compute<WT, NB, MAXC, true>(W1, R1, xs, nb, S[0]);
    mv_compute<WT, NB, MAXC, true>(W3, R3, xs, nb, S[1]);
    reduce_once<NB, 2>(S, nb, reinterpret_cast<long long*>(sm + L.part), tot);
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        int q = 0;
        if (row < W1.rows) {
            const int corr = WT == W_T3 ? ws.gsum[warp * ws.gst] : 0;
            const int g = mv_epi(tot[0] - corr, R1.rs);
            const int u = mv_epi(tot[1] - corr, R3.rs);
            if (d.hostffn) {
                q = host_hidden(g, u, kx_own);
            } else {
                float y = swiglu1(__fmul_rn((float)g, 1.0f / 256.0f), __fmul_rn((float)u, 1.0f / 256.0f));
                if (hs > 0) y = __fmul_rn(y, ldexpf(1.0f, -hs));     // metadata key 15 store scale
                q = q16s(y);
            }
        }
        hq[warp * 32 + lane] = q;
        const int sum = __reduce_add_sync(0xffffffffu, q);
        if (lane == 0) dsum[warp] = sum;
        if (d.hostffn) {
            const int mq = __reduce_max_sync(0xffffffffu, abs(q));
            if (lane == 0 && mq) atomicMax(s.hmax + hmax_at(layer, b0 + members[warp], half, s.slots), mq);
        }
    }
    __syncthreads();
    // the w2 input bytes of this CTA's columns (zero for the rest of the chunk)
    for (int t = threadIdx.x; t < nb * span; t += kThreads) {
        const int m = t / span, col = t % span;
        const int v = (col >= off && col < off + 32) ? hq[m * 32 + col - off] : 0;
        dlo[m * span + col] = (uint8_t)(v & 0xFF);
        dhi[m * span + col] = (int8_t)(v >> 8);
    }
    __syncthreads();
    // w2 rows: warp w takes row blocks w, w + kWarps, ...; lanes are rows
    for (int i = 0; warp + i * kWarps < W2.rblocks; ++i) {
        const int rb = warp + i * kWarps, row = rb * 32 + lane;
        int4 wa = make_int4(0, 0, 0, 0), wb = make_int4(0, 0, 0, 0);
        int sp = 0;
        if (i < kFfnRB) {
#pragma unroll
            for (int u = 0; u < kFfnRB; ++u)
                if (u == i) { wa = w2a[u]; wb = w2b[u]; sp = w2p[u]; }
        } else {
            fetch_w2(i, wa, wb, sp);
        }
        for (int m = 0; m < nb; ++m) {
            const uint8_t* lo = dlo + m * span;
            const int8_t* hi = dhi + m * span;
            long long S2;
            if (WT == W_Q8) {
                S2 = chunk_dot<W_Q8>(wa, 0, lo, hi, 0);
                if (j0 + 1 < nch2) S2 += chunk_dot<W_Q8>(wb, 0, lo + 16, hi + 16, 0);
            } else if (WT == W_Q4) {
                S2 = chunk_dot<W_Q4>(wa, sp, lo, hi, dsum[m]);
            } else {
                S2 = chunk_dot<W_T3>(wa, 0, lo, hi, 0) - dsum[m];   // codes are w + 1
            }
            if (row < W2.rows)
                atomicAdd(reinterpret_cast<unsigned long long*>(
                              s.sdown + sdown_at(layer, b0 + members[m], half, d.dim, s.slots) + row),
                          (unsigned long long)S2);
        }
    }
}


// ---------------------------------------------------------------------------
// logits: RMSNorm(x) + logits matvec + first-max argmax; the last CTA of the
// launch turns the packed keys into greedy tokens (and advances the sequences)
// ---------------------------------------------------------------------------

struct Finalize {
    int* next;          // greedy token per batch position
    int* tokens;        // advance: becomes the greedy (or forced) token
    int* pos;           // advance: + 1
    const int* forced;  // prefill: token at each position
    int advance;
};

// Logits and the greedy token.  The greedy token is the first maximum
// (sampling.cpp:160-162), found by a packed-key atomicMax over all rows; the
// last CTA to finish writes the next token (and advances position and token
// for the device-resident decode loop).  Two kernels share that tail:
//  - k_logits: one CTA per 32-row block, the columns split over the warps,
//    for heads of up to a few hundred blocks (latency: every SM busy at once);
//  - k_logits_wide: one warp per 32-row block (lanes are rows, each warp walks
//    all column chunks, no cross-warp reduction), grid-stride over the blocks,
//    several CTAs per SM, for heads of thousands of blocks (HBM streaming).
__device__ __forceinline__ unsigned long long logit_key(int v, int row) {
    return ((unsigned long long)(unsigned)(v + 32768) << 32) | (unsigned)(0xFFFFFFFFu - (unsigned)row);
}

__device__ __forceinline__ void logits_finish(State& s, int b0, int nb, const Finalize& fz) {
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(s.done, 1) == (int)(gridDim.x * gridDim.y * gridDim.z) - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
        const int bi = b0 + i;
        const unsigned long long key = __ldcg(&s.best[bi]);
        const int tok = (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
        fz.next[bi] = tok;
        if (fz.advance) {
            const int p = fz.pos[bi] + 1;
            fz.tokens[bi] = fz.forced ? fz.forced[p < s.seq ? p : s.seq - 1] : tok;
            fz.pos[bi] = p;
        }
    }
    if (threadIdx.x == 0) *s.done = 0;
}

template <int NB>
__device__ __forceinline__ void logits_stage_inputs(const DMat& W, const float (&nw)[kPer], State& s, const Dims& d,
                                                    const DownSrc& ds, int b0, int nb, XStage& xs, Red*& red,
                                                    int16_t*& tmp) {
    long long* part;
    carve<NB>(x_stride(W), g_stride(W), xs, red, part, tmp);
    for (int b = 0; b < nb; ++b) rebuild_x(s, d, ds, b0 + b, tmp + (size_t)b * d.dim, false);
    __syncthreads();
    for (int b = 0; b < nb; ++b) {
        int16_t* xin = tmp + (size_t)b * d.dim;
        rmsnorm_q16(xin, nw, d.dim, d.eps, xin, *red);
        xs.k[b] = 0;
        stage_one<W_Q8>(xs, b, xin, d.dim, 0, *red);
    }
}

template <int NB, int MAXC>
__global__ void __launch_bounds__(kThreads) k_logits(DMat W, const float* rms_w, State s, Batch bt, Dims d, int b0,
                                                     Finalize fz, DownSrc ds) {
    const MvLayout L = mv_layout(wstage_bytes(W, NB), NB, NB * d.dim, d.dim, 0);
    if (!smem_ok(L.total, s.err)) return;
    char* sm = SmemLayout::base();
    WRegs<MAXC> R;
    mv_prefetch<W_Q8, MAXC>(W, blockIdx.x, R);
    float* nws = reinterpret_cast<float*>(sm + L.nw);
    for (int c = threadIdx.x; c < d.dim; c += kThreads) nws[c] = __ldg(rms_w + c);
    pdl_launch_dependents();
    pdl_wait();
    int16_t* xv = reinterpret_cast<int16_t*>(sm + L.x);
    const int nb = min(NB, bt.n - b0);
    for (int b = 0; b < nb; ++b) rebuild_x(s, d, ds, b0 + b, xv + (size_t)b * d.dim, false);
    __syncthreads();
    const WStage ws = wstage_at(W, NB, sm + L.ws);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= nb) break;
        const int16_t* x = xv + (size_t)b * d.dim;
        const float rr = rms_rr(warp_sumsq(x, d.dim), d.dim, d.eps);
        warp_stage<W_Q8>(ws, b, W.nchunks, d.dim, 0, [&](int c) { return xnorm(x[c], nws[c], rr); });
    }
    __syncwarp();
    long long S[1][NB], tot[1];
    mv_compute<W_Q8, NB, MAXC, true>(W, R, xstage_of(ws), nb, S[0]);
    reduce_once<NB, 1>(S, nb, reinterpret_cast<long long*>(sm + L.part), tot);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < nb) {
        const int row = blockIdx.x * 32 + lane;
        const int bi = b0 + warp;
        unsigned long long key = 0ull;
        if (row < W.rows) {
            const int v = mv_epi(tot[0], R.rs);
            s.logits[(size_t)bi * d.vocab + row] = v;
            key = logit_key(v, row);
        }
        for (int o = 16; o; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
            key = k2 > key ? k2 : key;
        }
        if (lane == 0 && key) { atomicMax(&s.best[bi], key); __threadfence(); }
    }
    logits_finish(s, b0, nb, fz);
}

// One warp per 32-row block: lanes are rows, the warp walks every column
// chunk of its blocks.  Each warp streams its weights through its own ring of
// shared-memory stages filled by bulk copies (pieces of up to kWidePiece
// 16-column chunks, 512 contiguous bytes per chunk), so the copies in flight
// cost no registers; the first pieces are requested before the grid-dependency
// wait.  Blocks are dealt to warps round-robin over the whole grid.
constexpr int kWidePiece = 16;

__host__ __device__ inline size_t wide_base(const DMat& W, int nb, int dim) {
    return (smem_bytes(nb, x_stride(W), g_stride(W), nb * dim) + 127) & ~(size_t)127;
}
// Ring stages per warp that fit next to the input staging (0: none fit).
__host__ __device__ inline int wide_stages(const DMat& W, int nb, int dim) {
    const size_t base = wide_base(W, nb, dim);
    if (base >= kMaxDynSmem) return 0;
    const size_t per_warp = (kMaxDynSmem - base) / kWarps;
    const size_t stage = (size_t)kWidePiece * 512 + 8;
    const int st = (int)(per_warp / stage);
    return st > 4 ? 4 : st;
}
__host__ __device__ inline size_t wide_smem(const DMat& W, int nb, int dim, int stages) {
    return wide_base(W, nb, dim) + (size_t)kWarps * stages * ((size_t)kWidePiece * 512 + 8);
}

template <int NB>
__global__ void __launch_bounds__(kThreads) k_logits_wide(DMat W, const float* rms_w, State s, Batch bt, Dims d,
                                                         int b0, Finalize fz, int stages, DownSrc ds) {
    if (!smem_ok(wide_smem(W, NB, d.dim, stages), s.err)) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nch = W.nchunks;
    char* ring = SmemLayout::base() + wide_base(W, NB, d.dim) + (size_t)warp * stages * kWidePiece * 512;
    unsigned long long* bar = reinterpret_cast<unsigned long long*>(
        SmemLayout::base() + wide_base(W, NB, d.dim) + (size_t)kWarps * stages * kWidePiece * 512) + warp * stages;
    const int ppb = (nch + kWidePiece - 1) / kWidePiece;             // pieces per block
    const int stride = gridDim.x * kWarps;
    const int first = blockIdx.x * kWarps + warp;
    const int nblk = first < W.rblocks ? (W.rblocks - first + stride - 1) / stride : 0;
    const int npieces = nblk * ppb;
    auto issue = [&](int p) {
        const int blk = first + (p / ppb) * stride, j0 = (p % ppb) * kWidePiece;
        const unsigned bytes = (unsigned)min(kWidePiece, nch - j0) * 512u;
        unsigned long long* b = &bar[p % stages];
        mbar_expect_tx(b, bytes);
        bulk_g2s(ring + (size_t)(p % stages) * kWidePiece * 512, W.body + ((size_t)blk * nch + j0) * 512, bytes, b);
    };
    if (lane == 0) {
        for (int i = 0; i < stages; ++i) mbar_init(&bar[i], 1);
        mbar_fence_init();
        for (int p = 0; p < min(stages, npieces); ++p) issue(p);
    }
    float nw[kPer];
    load_f32_regs(rms_w, d.dim, nw);
    pdl_launch_dependents();
    pdl_wait();
    XStage xs; Red* red; int16_t* tmp;
    const int nb = min(NB, bt.n - b0);
    logits_stage_inputs<NB>(W, nw, s, d, ds, b0, nb, xs, red, tmp);   // block-wide; publishes the mbarriers
    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) best[b] = 0ull;
    int alo[NB], ahi[NB];
    float rs = 0.0f;
    bool failed = false;
    for (int p = 0; p < npieces; ++p) {
        const int blk = first + (p / ppb) * stride, j0 = (p % ppb) * kWidePiece;
        if (j0 == 0) {
            rs = __ldg(W.rscale + (size_t)blk * 32 + lane);
#pragma unroll
            for (int b = 0; b < NB; ++b) { alo[b] = 0; ahi[b] = 0; }
        }
        if (!mbar_wait(&bar[p % stages], (unsigned)(p / stages) & 1u)) { failed = true; break; }
        const int4* buf = reinterpret_cast<const int4*>(ring + (size_t)(p % stages) * kWidePiece * 512) + lane;
        const int nu = min(kWidePiece, nch - j0);
#pragma unroll 4
        for (int u = 0; u < nu; ++u) {
            const int4 w = buf[u * 32];
            const int j = j0 + u;
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
        }
        __syncwarp();
        if (lane == 0 && p + stages < npieces) {
            fence_proxy_async();
            issue(p + stages);
        }
        if (j0 + kWidePiece >= nch) {
            const int row = blk * 32 + lane;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb || row >= W.rows) continue;
                const int v = mv_epi((long long)alo[b] + 256LL * (long long)ahi[b], rs);
                s.logits[(size_t)(b0 + b) * d.vocab + row] = v;
                const unsigned long long key = logit_key(v, row);
                best[b] = key > best[b] ? key : best[b];
            }
        }
    }
    if (failed) {
        // a copy did not land in time: report it and wait (bounded) for this
        // warp's copies still in flight before the shared memory is released
        if (lane == 0) {
            atomicExch(s.err, kErrCopyTimeout);
            for (int p = 0; p < npieces; ++p) mbar_wait(&bar[p % stages], (unsigned)(p / stages) & 1u, 10000000ull);
        }
        __syncwarp();
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= nb) break;
        unsigned long long kk = best[b];
        for (int o = 16; o; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, kk, o);
            kk = k2 > kk ? k2 : kk;
        }
        if (lane == 0 && kk) atomicMax(&s.best[b0 + b], kk);
    }
    logits_finish(s, b0, nb, fz);
}

#ifdef VC4_COMMON_TU
// Attention for one (KV head, sequence) runs on group/hq clusters of kAttnCtas
// CTAs, each cluster serving hq of the KV head's query heads, with a single
// cluster barrier:
//  - before the grid-dependency wait every CTA stages the cache rows it needs
//    (cp.async) and decodes them to fp32 in shared memory: the K rows of its
//    contiguous share of positions 0..pos, and a slice of V columns for every
//    position;
//  - after the wait each CTA rebuilds the normalised, rotated q heads and the
//    new k (identical in every CTA), encodes the new cache row (written by the
//    CTA whose share holds `pos`), computes the scores of its positions and
//    stores them into every CTA of the cluster (distributed shared memory);
//  - after the barrier each CTA holds all scores, runs the softmax for all
//    positions itself (the same order in every CTA) and computes P.V for its
//    own V columns, so no partial results cross CTAs.
// The arithmetic is the reference's (session.cpp:1989-2050): sequential fp32
// q.k per position, global max, exp(s - max), out = sum_t (e_t / sum e) v_t,
// with e_t on a 2^-k grid (attn_weights) so that every sum is exact.
constexpr int kAttnCtas = 8;

__host__ __device__ inline int attn_vs(int hd) { return (((hd + kAttnCtas - 1) / kAttnCtas) + 3) & ~3; }
__host__ __device__ inline int attn_rows(int seq) { return (seq + kAttnCtas - 1) / kAttnCtas; }

struct AttnSmem {
    uint8_t* kraw;   // attn_rows(seq) x hbytes: K rows of this CTA's positions (cache bytes)
    uint8_t* vraw;   // seq x vs*kvb: this CTA's V columns of every position (cache bytes)
    double* pv;      // max(kThreads, group*vs): P.V partials
    double* redd;    // kWarps: softmax sums per warp
    double* den;     // group: sums of the attention weights
    float* kt;       // attn_rows(seq) x (hd + 4): decoded K rows
    float* vt;       // seq x vs: decoded V columns
    float* q;        // (group + 1) x hd: q heads, then the new k
    float* vn;       // hd: the new v
    float* rc;       // hd/2: RoPE cos at pos
    float* rsn;      // hd/2: RoPE sin at pos
    float* wq;       // hd: q_norm weights of the layer
    float* wk;       // hd: k_norm weights of the layer
    float* redf;     // kWarps: softmax maxima per warp
    float* sc;       // group x seq: scores, then probabilities (cluster-written)
    int* qi;         // group x hd: the q heads on their integer grids
    float* gsc;      // group: each q head's score constant (warp_q_grid)
};

__host__ __device__ inline size_t attn_carve(int group, int hd, int seq, int kv_bits, char* base, AttnSmem* sm) {
    const int kvb = kv_bits / 8, vs = attn_vs(hd), rows = attn_rows(seq);
    const int npv = group * vs > kThreads ? group * vs : kThreads;
    size_t o = 0;
    const size_t kraw = o; o = align16(o + (size_t)rows * hd * kvb);
    const size_t vraw = o; o = align16(o + (size_t)seq * vs * kvb);
    const size_t pv = o;   o = align16(o + sizeof(double) * npv);
    const size_t redd = o; o = align16(o + sizeof(double) * kWarps);
    const size_t den = o;  o = align16(o + sizeof(double) * group);
    const size_t kt = o;   o = align16(o + sizeof(float) * (size_t)rows * (hd + 4));
    const size_t vt = o;   o = align16(o + sizeof(float) * (size_t)seq * vs);
    const size_t q = o;    o = align16(o + sizeof(float) * (size_t)(group + 1) * hd);
    const size_t vn = o;   o += sizeof(float) * hd;
    const size_t rc = o;   o += sizeof(float) * (hd / 2);
    const size_t rsn = o;  o += sizeof(float) * (hd / 2);
    const size_t wq = o;   o += sizeof(float) * hd;
    const size_t wk = o;   o += sizeof(float) * hd;
    const size_t redf = o; o += sizeof(float) * kWarps;
    const size_t sc = o;   o += sizeof(float) * (size_t)group * seq;
    o = align16(o);
    const size_t qi = o;   o += sizeof(int) * (size_t)group * hd;
    const size_t gsc = o;  o += sizeof(float) * (size_t)group;
    if (sm) {
        sm->qi = reinterpret_cast<int*>(base + qi);
        sm->gsc = reinterpret_cast<float*>(base + gsc);
        sm->kraw = reinterpret_cast<uint8_t*>(base + kraw);
        sm->vraw = reinterpret_cast<uint8_t*>(base + vraw);
        sm->pv = reinterpret_cast<double*>(base + pv);
        sm->redd = reinterpret_cast<double*>(base + redd);
        sm->den = reinterpret_cast<double*>(base + den);
        sm->kt = reinterpret_cast<float*>(base + kt);
        sm->vt = reinterpret_cast<float*>(base + vt);
        sm->q = reinterpret_cast<float*>(base + q);
        sm->vn = reinterpret_cast<float*>(base + vn);
        sm->rc = reinterpret_cast<float*>(base + rc);
        sm->rsn = reinterpret_cast<float*>(base + rsn);
        sm->wq = reinterpret_cast<float*>(base + wq);
        sm->wk = reinterpret_cast<float*>(base + wk);
        sm->redf = reinterpret_cast<float*>(base + redf);
        sm->sc = reinterpret_cast<float*>(base + sc);
    }
    return align16(o);
}
__host__ __device__ inline size_t attn_smem_bytes(int group, int hd, int seq, int kv_bits) {
    return attn_carve(group, hd, seq, kv_bits, nullptr, nullptr);
}



// The values of one 32-bit word of a packed cache row: two q16 big-endian
// values on the 1/2048 grid, or four q8 two's-complement values on the 1/16
// grid (shaders_attn.cpp:141-159).  Returns the number of values.
__device__ __forceinline__ int kv_word(unsigned w, int kvb, float* out) {
    if (kvb == 2) {
        out[0] = __fmul_rn((float)(short)(((w & 0xFFu) << 8) | ((w >> 8) & 0xFFu)), 1.0f / 2048.0f);
        out[1] = __fmul_rn((float)(short)((((w >> 16) & 0xFFu) << 8) | (w >> 24)), 1.0f / 2048.0f);
        return 2;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = __fmul_rn((float)(signed char)((w >> (8 * j)) & 0xFFu), 1.0f / 16.0f);
    return 4;
}
// The integer levels of one 32-bit word of a packed cache row (kv_word
// without the grid), as floats.
__device__ __forceinline__ int kv_codes(unsigned w, int kvb, float* out) {
    if (kvb == 2) {
        out[0] = (float)(short)(((w & 0xFFu) << 8) | ((w >> 8) & 0xFFu));
        out[1] = (float)(short)((((w >> 16) & 0xFFu) << 8) | (w >> 24));
        return 2;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = (float)(signed char)((w >> (8 * j)) & 0xFFu);
    return 4;
}
// The packed bytes of one value (the inverse of kv_word), as the low bits of a word.
__device__ __forceinline__ unsigned kv_encode(float x, int kvb, float* dec) {
    if (kvb == 2) {
        float q = floorf(__fadd_rn(__fmul_rn(x, 2048.0f), 0.5f));
        q = q < -32768.0f ? -32768.0f : q > 32767.0f ? 32767.0f : q;
        *dec = __fmul_rn(q, 1.0f / 2048.0f);
        const unsigned u = (unsigned)(int)q & 0xFFFFu;
        return (u >> 8) | ((u & 0xFFu) << 8);           // big-endian byte order in memory
    }
    float q = floorf(__fadd_rn(__fmul_rn(x, 16.0f), 0.5f));
    q = q < -128.0f ? -128.0f : q > 127.0f ? 127.0f : q;
    *dec = __fmul_rn(q, 1.0f / 16.0f);
    return (unsigned)(int)q & 0xFFu;
}

// Attention weights of hq heads over positions 0..len-1 (sc[hh*seq + t]), in
// place: kWarps / hq warps per head (one when there are more heads than
// warps) take the maximum, then E_t = rint(exp(s_t - max) * 2^k), an integer
// stored as a float, and den[hh] = sum_t E_t.  k = 53 - (7 for q8 levels, 15
// for q16) - ceil(log2 len) keeps every |E_t * level| at most 2^53 / len, so
// the double sums here and in P.V are exact integers and their order is free:
// any kernel layout gives the same bits.
__host__ __device__ inline int attn_weight_exp(int len, int kvb) {
    int lg = 0;
    while ((1 << lg) < len) ++lg;
    return 53 - (kvb == 2 ? 15 : 7) - lg;
}

// Exponent F of a query head's integer grid: with max|q| = f * 2^e (f in
// [0.5, 1)), F = 22 - e, so every |rint(q * 2^F)| <= 2^22 splits into three
// balanced signed bytes; clamped to [-100, 100].  A score is the exact
// integer dot of rint(q * 2^F) with the cache levels, rounded once to float,
// times 2^-F / grid (exact), divided by sqrt(hd).
__device__ __forceinline__ int q_grid_exp(float qmax) {
    if (!(qmax > 0.0f)) return 0;
    int e = 0;
    frexpf(qmax, &e);
    const int F = 22 - e;
    return F > 100 ? 100 : F < -100 ? -100 : F;
}

// One warp puts q head v (hd floats) on its integer grid: qi[i] = rint(v[i]
// * 2^F); returns the head's score constant fl(2^-F / grid / sqrt(hd)) (kvb 2:
// grid 2048, 1: grid 16), so a score is float(S) * constant.
__device__ __forceinline__ float warp_q_grid(const float* v, int hd, int kvb, int* qi) {
    const int lane = threadIdx.x & 31;
    float m = 0.0f;
    for (int i = lane; i < hd; i += 32) m = fmaxf(m, fabsf(v[i]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int F = q_grid_exp(m);
    const float sF = pow2f(F);
    for (int i = lane; i < hd; i += 32) qi[i] = __float2int_rn(__fmul_rn(v[i], sF));
    return __fdiv_rn(pow2f(-F - (kvb == 2 ? 11 : 4)), __fsqrt_rn((float)hd));
}

__device__ void attn_weights(float* scores, int seq, int len, int hq, int kvb, float* redf, double* redd,
                             double* den) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float wscale = __int_as_float((127 + attn_weight_exp(len, kvb)) << 23);   // 2^k, exact
    const int wph = hq >= kWarps ? 1 : kWarps / hq;
    const int hpr = kWarps / wph;                 // heads per round
    const int hw = warp / wph, sub = warp % wph, step = wph * 32;
    for (int r0 = 0; r0 < hq; r0 += hpr) {
        const int hh = r0 + hw;
        const bool act = hw < hpr && hh < hq;
        float* p = scores + (act ? hh : 0) * seq;
        float m = -1e30f;
        if (act)
            for (int t = sub * 32 + lane; t < len; t += step) m = fmaxf(m, p[t]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) redf[warp] = m;
        __syncthreads();
        double a = 0.0;
        if (act) {
            m = redf[hw * wph];
            for (int k = 1; k < wph; ++k) m = fmaxf(m, redf[hw * wph + k]);
#pragma unroll 4
            for (int t = sub * 32 + lane; t < len; t += step) {
                const float e = rintf(__fmul_rn(vexp(__fsub_rn(p[t], m)), wscale));
                p[t] = e;
                a = __dadd_rn(a, (double)e);
            }
        }
        for (int o = 16; o; o >>= 1) a = __dadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) redd[warp] = a;
        __syncthreads();
        if (act && sub == 0 && lane == 0) {
            double tot = 0.0;
            for (int k = 0; k < wph; ++k) tot = __dadd_rn(tot, redd[hw * wph + k]);
            den[hh] = tot;
        }
        __syncthreads();
    }
}

// One attention output on the q16 grid: the float num / den * c rounded to
// the nearest integer, ties to even (the host's lrintf, common.h:188-193),
// clamped; num = sum E_t * code_t, c = 256 * the cache grid (16 for q8, 1/8
// for q16).
__device__ __forceinline__ int16_t att_q16(double num, double den, int kvb) {
    const float y = __double2float_rn(__dmul_rn(__ddiv_rn(num, den), kvb == 2 ? 0.125 : 16.0));
    const int q = __float2int_rn(y);
    return (int16_t)(q < -32768 ? -32768 : q > 32767 ? 32767 : q);
}

// HD > 0: the head size fixed at compile time (the loops unroll).
template <int HD>
__global__ void __cluster_dims__(kAttnCtas, 1, 1) __launch_bounds__(kThreads)
k_attn(const float* q_norm, const float* k_norm, State s, Batch bt, Dims d, int layer, int hq) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) char smem[];
    const int hd = HD ? HD : d.head_dim, group = d.heads / d.kv_heads, half = hd / 2, hp = hd + 4;
    if (!smem_ok(attn_smem_bytes(hq, hd, d.seq, d.kv_bits), s.err)) return;
    AttnSmem sm;
    attn_carve(hq, hd, d.seq, d.kv_bits, smem, &sm);
    const int rank = (int)cluster.block_rank();
    // cluster (g, split) serves q heads split*hq .. split*hq + hq - 1 of KV head g
    const int qsplit = group / hq, g = blockIdx.x / kAttnCtas / qsplit, split = blockIdx.x / kAttnCtas % qsplit;
    const int h0 = split * hq, b = blockIdx.y;
    const int slot = bt.slot[b], pos = bt.pos[b], len = pos + 1;
    const int per = (len + kAttnCtas - 1) / kAttnCtas;
    const int t0 = min(len, rank * per), t1 = min(len, t0 + per), nt = t1 - t0;
    const int kvb = d.kv_bits / 8, hbytes = hd * kvb, vofs = d.kv_dim * kvb;
    const int vs = attn_vs(hd), c0 = min(hd, rank * vs), c1 = min(hd, c0 + vs), nc = c1 - c0;
    const int vrow = vs * kvb;                    // staged bytes per position of the V slice
    const int vpw = 4 / kvb;                      // values per 32-bit word
    const KvRows kr = kv_rows_of(s, slot, layer, d.layers, d.seq, d.row_bytes);

    // 1. stage and decode the cached rows (every position but `pos`, which
    //    this step writes), the RoPE row and the norm weights
    const int kvec = hbytes / 16;
    for (int v = threadIdx.x; v < nt * kvec; v += kThreads) {
        const int r = v / kvec, c = v % kvec, t = t0 + r;
        if (t != pos) cp_async16(sm.kraw + r * hbytes + c * 16, kr.at(t, d.row_bytes) + g * hbytes + c * 16);
    }
    const int vw = nc * kvb / 4;                  // words per position of the V slice
    for (int v = threadIdx.x; v < pos * vw; v += kThreads) {
        const int t = v / vw, c = v % vw;
        cp_async4(sm.vraw + (size_t)t * vrow + c * 4, kr.at(t, d.row_bytes) + vofs + g * hbytes + c0 * kvb + c * 4);
    }
    for (int i = threadIdx.x; i < half; i += kThreads) {
        sm.rc[i] = s.rope_cos[(size_t)pos * half + i];
        sm.rsn[i] = s.rope_sin[(size_t)pos * half + i];
    }
    if (d.qk_norm)
        for (int i = threadIdx.x; i < hd; i += kThreads) {
            sm.wq[i] = q_norm[(size_t)layer * hd + i];
            sm.wk[i] = k_norm[(size_t)layer * hd + i];
        }
    cp_async_wait_all();
    __syncthreads();
    const int kw = hbytes / 4;
    for (int v = threadIdx.x; v < nt * kw; v += kThreads) {
        const int r = v / kw, c = v % kw;
        if (t0 + r == pos) continue;
        float f[4];
        const int n = kv_codes(reinterpret_cast<const unsigned*>(sm.kraw + r * hbytes)[c], kvb, f);
        for (int j = 0; j < n; ++j) sm.kt[r * hp + c * n + j] = f[j];
    }
    for (int v = threadIdx.x; v < pos * vw; v += kThreads) {
        const int t = v / vw, c = v % vw;
        float f[4];
        const int n = kv_codes(reinterpret_cast<const unsigned*>(sm.vraw + (size_t)t * vrow)[c], kvb, f);
        for (int j = 0; j < n; ++j) sm.vt[(size_t)t * vs + c * n + j] = f[j];
    }
    pdl_launch_dependents();
    pdl_wait();

    // 2. q heads, new k, new v from the qkv matvec; qk-norm (exact double sum
    //    of squares) and RoPE, one warp per vector
    const float* qkv = s.qkv + (size_t)b * (d.dim + 2 * d.kv_dim);
    for (int i = threadIdx.x; i < hq * hd; i += kThreads) sm.q[i] = qkv[(g * group + h0) * hd + i];
    for (int i = threadIdx.x; i < hd; i += kThreads) {
        sm.q[hq * hd + i] = qkv[d.dim + g * hd + i];
        sm.vn[i] = qkv[d.dim + d.kv_dim + g * hd + i];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int hh = warp; hh <= hq; hh += kWarps) {
        float* v = sm.q + hh * hd;
        if (d.qk_norm) {
            double acc = 0.0;
            for (int i = lane; i < hd; i += 32) acc = __dadd_rn(acc, __dmul_rn((double)v[i], (double)v[i]));
            for (int o = 16; o; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
            const float ss = __double2float_rn(acc);
            const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), 1e-6f)));
            const float* w = hh < hq ? sm.wq : sm.wk;
            for (int i = lane; i < hd; i += 32) v[i] = __fmul_rn(w[i], __fmul_rn(r, v[i]));
            __syncwarp();
        }
        for (int i = lane; i < half; i += 32) {
            const int ia = d.rope_half ? i : 2 * i, ib = d.rope_half ? i + half : 2 * i + 1;
            const float a = v[ia], bb = v[ib], c = sm.rc[i], sv = sm.rsn[i];
            v[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, sv));
            v[ib] = __fadd_rn(__fmul_rn(a, sv), __fmul_rn(bb, c));
        }
    }
    __syncthreads();
    for (int hh = warp; hh < hq; hh += kWarps) {
        const float g = warp_q_grid(sm.q + hh * hd, hd, kvb, sm.qi + hh * hd);
        if (lane == 0) sm.gsc[hh] = g;
    }

    // 3. encode the new row one 32-bit word at a time (shaders_attn.cpp:141-159);
    //    every CTA encodes it identically, the one whose share holds `pos`
    //    writes it to the cache (the first split of the KV head)
    const bool owner = pos >= t0 && pos < t1;
    const bool writer = owner && split == 0 && pos >= kr.plen;
    if (owner && split == 0 && pos < kr.plen && threadIdx.x == 0) atomicMin(s.err, kErrSharedAppend);
    uint8_t* row = kr.own + (size_t)pos * d.row_bytes;
    for (int e = threadIdx.x; e < 2 * kw; e += kThreads) {
        const int w = e / kw, c = e % kw, i0 = c * vpw;
        const float* src = w ? sm.vn : sm.q + hq * hd;
        unsigned word = 0;
        float dec[4];
        for (int j = 0; j < vpw; ++j) word |= kv_encode(src[i0 + j], kvb, &dec[j]) << (8 * kvb * j);
        if (writer) *reinterpret_cast<unsigned*>(row + (w ? vofs : 0) + g * hbytes + c * 4) = word;
        for (int j = 0; j < vpw; ++j) {
            const int i = i0 + j;
            if (!w && owner) sm.kt[(pos - t0) * hp + i] = __fmul_rn(dec[j], kvb == 2 ? 2048.0f : 16.0f);
            if (w && i >= c0 && i < c1) sm.vt[(size_t)pos * vs + i - c0] = __fmul_rn(dec[j], kvb == 2 ? 2048.0f : 16.0f);
        }
    }
    __syncthreads();

    // 4. scores of this CTA's positions: the exact integer dot of the q head
    //    on its grid with the cache levels, one rounding to float, times the
    //    head's constant; stored into every CTA of the cluster
    for (int e = threadIdx.x; e < nt * hq; e += kThreads) {
        const int r = e / hq, hh = e % hq;
        const float4* kr = reinterpret_cast<const float4*>(sm.kt + r * hp);
        const int4* qh = reinterpret_cast<const int4*>(sm.qi + hh * hd);
        long long S = 0;
#pragma unroll 4
        for (int i = 0; i < hd / 4; ++i) {
            const float4 k4 = kr[i];
            const int4 q4 = qh[i];
            S += (long long)q4.x * (int)k4.x + (long long)q4.y * (int)k4.y + (long long)q4.z * (int)k4.z +
                 (long long)q4.w * (int)k4.w;
        }
        const float acc = __fmul_rn(__ll2float_rn(S), sm.gsc[hh]);
        float* dst = sm.sc + hh * d.seq + t0 + r;
#pragma unroll
        for (int c = 0; c < kAttnCtas; ++c) *cluster.map_shared_rank(dst, c) = acc;
    }
    cluster.sync();   // the last access to another CTA's shared memory

    // 5. integer weights over all positions (every CTA computes them all)
    attn_weights(sm.sc, d.seq, len, hq, kvb, sm.redf, sm.redd, sm.den);

    // 6. P.V for this CTA's V columns: each output's positions split into ks
    //    contiguous ranges; the sums of E_t * code are exact
    const int nout = hq * nc;
    if (nout == 0) return;
    const int ks = nout >= kThreads ? 1 : min(32, kThreads / nout);
    const int chunk = (len + ks - 1) / ks;
    for (int e = threadIdx.x; e < nout * ks; e += kThreads) {
        const int o = e / ks, j = e % ks, hh = o / nc, i = o % nc;
        const int ta = min(len, j * chunk), tb = min(len, ta + chunk);
        const float* p = sm.sc + hh * d.seq;
        const float* vc = sm.vt + i;
        double a = 0.0;
#pragma unroll 4
        for (int t = ta; t < tb; ++t) a = __fma_rn((double)p[t], (double)vc[(size_t)t * vs], a);
        sm.pv[e] = a;
    }
    __syncthreads();
    for (int o = threadIdx.x; o < nout; o += kThreads) {
        double a = 0.0;
        for (int j = 0; j < ks; ++j) a = __dadd_rn(a, sm.pv[o * ks + j]);
        const int hh = o / nc, i = o % nc;
        s.att[(size_t)b * d.dim + (size_t)(g * group + h0 + hh) * hd + c0 + i] = att_q16(a, sm.den[hh], kvb);
    }
}


// Attention for many sequences at once: one CTA (no cluster) per (sequence,
// KV head, q heads of the CTA), both contractions on the tensor cores as exact
// integer MMAs (mma.sync m16n8k32 with 8-bit operands and int32
// accumulators):
//  - K rows and then V rows stream through a ring of kAbStages shared-memory
//    tiles of kAbRows positions (cp.async), rows padded to an odd number of
//    16-byte units so ldmatrix reads hit distinct banks;
//  - scores: each q head on its integer grid (warp_q_grid) is split into
//    three balanced signed bytes, the B operand (column 4*head + limb, so a
//    lane and its neighbour hold a head's limbs and one shuffle combines
//    them); the A operand is a K tile: q8 levels as they are, q16 levels as
//    a signed high-byte and an unsigned low-byte plane; S = sum_limb
//    256^limb (256 D_hi + D_lo) is the exact integer dot, and the score is
//    float(S) times one per-head constant;
//  - weights: at the last K tile one pass takes the maximum, E_t (integers
//    < 2^47), their exact double sum and E_t's byte limbs;
//  - P.V: E_t split into unsigned byte limbs is the A operand (row h*NL +
//    limb), a V tile read with ldmatrix.trans the B operand (q8: even and odd
//    columns; q16: high and low byte planes); every limb product and their
//    combination into num = sum_t E_t * level_t are exact integers.  Each
//    warp keeps its position block's limb products in its int32 MMA
//    accumulators across the V tiles (at most seq/4 * 255 * 255 < 2^31) and
//    writes them once, as int64, into the freed ring; the blocks and limbs
//    are combined at the end (no atomics).
// A sequence's output is therefore the cluster kernel's, bit for bit.
// Positions inside a 32-wide MMA k block are taken in the order ldmatrix of
// 16-bit pairs delivers them (attnb_k_of); the weight limbs are stored in it.
constexpr int kAbRows = 128;
constexpr int kAbStages = 2;
static_assert(kAbStages >= 2, "the tile loop keeps kAbStages - 1 tiles in flight");
constexpr int kAbMaxLimbs = 6;      // E_t < 2^47: six bytes

__host__ __device__ inline int attnb_pitch(int hbytes) { return (hbytes / 16) % 2 ? hbytes : hbytes + 16; }
// bytes of one row of the weight-limb matrix: whole tiles of positions,
// padded to an odd number of 16-byte units
__host__ __device__ inline int attnb_epitch(int seq) {
    const int p = (seq + kAbRows - 1) / kAbRows * kAbRows;
    return (p / 16) % 2 ? p : p + 16;
}
// The k index (0..31 inside a 32-wide MMA block) that holds element p of the
// block when the operand rows were read as 16-bit pairs and split by
// byte_perm: k = 4q + r holds element 16*(k/16) + {2q, 2q+1, 8+2q, 9+2q}[r].
__host__ __device__ inline int attnb_k_of(int p) {
    const int b = p >> 4, r = p & 15;
    return 16 * b + (r < 8 ? 4 * (r >> 1) + (r & 1) : 4 * ((r - 8) >> 1) + 2 + (r & 1));
}

struct AbSmem {
    uint8_t* ring;   // kAbStages x kAbRows x pitch cache bytes; at the end (with newrow and ea) the P.V partial sums
    uint8_t* newrow; // 2 x hbytes: this step's K and V row
    uint8_t* ea;     // 16 x epitch: weight limbs, row h*NL + limb, positions in MMA k order
    uint8_t* qb;     // 8 x hd: q limbs, column 4*head + limb, dims in MMA k order
    double* redd;    // kWarps x 2: per-warp sums of the weights
    double* den;     // hq
    float* q;        // (hq + 1) x hd: q heads, then the new k
    float* vn;       // hd: the new v
    float* rc;
    float* rsn;
    float* wq;
    float* wk;
    float* redf;     // kWarps x 2: per-warp score maxima
    float* gsc;      // hq: each q head's score constant (warp_q_grid)
    float* sc;       // hq x seq: scores, then E_t
    int* qi;         // hq x hd: the q heads on their integer grids
};

__host__ __device__ inline size_t attnb_carve(int hq, int hd, int seq, int kv_bits, char* base, AbSmem* sm) {
    const int hbytes = hd * (kv_bits / 8);
    size_t o = 0;
    // ring, newrow and ea are dead once the last V tile is multiplied; the
    // P.V partial sums (4 position blocks x hq*NL rows x hd int64) take their
    // place, so the three together are at least that large
    const size_t part = (size_t)4 * hq * kAbMaxLimbs * hd * sizeof(long long);
    const size_t rows = align16((size_t)kAbStages * kAbRows * attnb_pitch(hbytes));
    const size_t rest = align16(2 * (size_t)hbytes) + align16(16 * (size_t)attnb_epitch(seq));
    const size_t ring = o; o = rows + rest >= part ? rows : align16(part - rest);
    const size_t nr = o;   o = align16(o + 2 * (size_t)hbytes);
    const size_t ea = o;   o = align16(o + 16 * (size_t)attnb_epitch(seq));
    const size_t qb = o;   o = align16(o + 8 * (size_t)hd);
    const size_t redd = o; o = align16(o + sizeof(double) * kWarps * 2);
    const size_t den = o;  o = align16(o + sizeof(double) * hq);
    const size_t q = o;    o = align16(o + sizeof(float) * (size_t)(hq + 1) * hd);
    const size_t vn = o;   o += sizeof(float) * hd;
    const size_t rc = o;   o += sizeof(float) * (hd / 2);
    const size_t rsn = o;  o += sizeof(float) * (hd / 2);
    const size_t wq = o;   o += sizeof(float) * hd;
    const size_t wk = o;   o += sizeof(float) * hd;
    const size_t redf = o; o += sizeof(float) * kWarps * 2;
    const size_t gsc = o;  o += sizeof(float) * hq;
    const size_t sc = o;   o += sizeof(float) * (size_t)hq * seq;
    const size_t qi = o;   o += sizeof(int) * (size_t)hq * hd;
    if (sm) {
        sm->ring = reinterpret_cast<uint8_t*>(base + ring);
        sm->newrow = reinterpret_cast<uint8_t*>(base + nr);
        sm->ea = reinterpret_cast<uint8_t*>(base + ea);
        sm->qb = reinterpret_cast<uint8_t*>(base + qb);
        sm->redd = reinterpret_cast<double*>(base + redd);
        sm->den = reinterpret_cast<double*>(base + den);
        sm->q = reinterpret_cast<float*>(base + q);
        sm->vn = reinterpret_cast<float*>(base + vn);
        sm->rc = reinterpret_cast<float*>(base + rc);
        sm->rsn = reinterpret_cast<float*>(base + rsn);
        sm->wq = reinterpret_cast<float*>(base + wq);
        sm->wk = reinterpret_cast<float*>(base + wk);
        sm->redf = reinterpret_cast<float*>(base + redf);
        sm->gsc = reinterpret_cast<float*>(base + gsc);
        sm->sc = reinterpret_cast<float*>(base + sc);
        sm->qi = reinterpret_cast<int*>(base + qi);
    }
    return align16(o);
}
__host__ __device__ inline size_t attnb_smem_bytes(int hq, int hd, int seq, int kv_bits) {
    return attnb_carve(hq, hd, seq, kv_bits, nullptr, nullptr);
}

// ldmatrix of four 8x8 16-bit matrices (row addresses from lanes 0-7, 8-15,
// 16-23, 24-31), plain and transposed.
__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(unsigned addr, unsigned (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// D += A (16x32, 8-bit, row) * B (32x8, 8-bit, col), int32 accumulators;
// AU / BU select unsigned operands.
template <bool AU, bool BU>
__device__ __forceinline__ void mma_i8(int (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    if (!AU && !BU)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else if (AU && !BU)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else if (AU && BU)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// HD: the head size (a multiple of 32, at most 128); HQ: q heads per CTA (1 or 2).
// mode 0 (decode): append this step's K/V row, then attend.  A batched prefill
// holds several positions of one sequence in one pass, where a CTA's cache
// reads would race with the rows the other positions' CTAs append; it runs
// the kernel twice: mode 1 appends every row and returns, mode 2 (the next
// launch, so every row is in the cache) attends without writing.
template <int KVB, int HQ, int HD>
__global__ void __launch_bounds__(kThreads, KVB == 1 && HD <= 96 ? 4 : 2)
k_attn_b(const float* q_norm, const float* k_norm, State s, Batch bt, Dims d, int layer, int mode) {
    static_assert(HD % 32 == 0 && HD <= 128 && (HQ == 1 || HQ == 2), "k_attn_b shape");
    extern __shared__ __align__(16) char smem[];
    constexpr int hq = HQ, hd = HD, half = HD / 2, hbytes = HD * KVB, kw = hbytes / 4, kvec = hbytes / 16;
    constexpr int KS = HD / 32;                        // MMA k blocks per head
    const int group = d.heads / d.kv_heads;
    if (!smem_ok(attnb_smem_bytes(hq, hd, d.seq, KVB * 8), s.err)) return;
    AbSmem sm;
    attnb_carve(hq, hd, d.seq, KVB * 8, smem, &sm);
    const int qsplit = group / hq, g = blockIdx.x / qsplit, split = blockIdx.x % qsplit;
    const int h0 = split * hq, b = blockIdx.y;
    const int slot = bt.slot[b], pos = bt.pos[b], len = pos + 1;
    const int vofs = d.kv_dim * KVB, pitch = attnb_pitch(hbytes), epitch = attnb_epitch(d.seq);
    const int ntile = mode == 1 ? 0 : (len + kAbRows - 1) / kAbRows;   // an append launch reads no tile
    const KvRows kr = kv_rows_of(s, slot, layer, d.layers, d.seq, d.row_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
    // tile u < ntile: K rows of positions [u*R, ...); ntile <= u < 2*ntile: V rows.
    // Thread (row r0, 16-byte column cc) copies rows r0, r0 + rpp, ...
    const int rpp = kThreads / kvec, cc = threadIdx.x % kvec, r0 = threadIdx.x / kvec;
    auto issue = [&](int u) {
        if (u < 2 * ntile && r0 < rpp) {
            const int kind = u >= ntile, t0 = (kind ? u - ntile : u) * kAbRows, nt = min(kAbRows, len - t0);
            uint8_t* dst = sm.ring + (size_t)(u % kAbStages) * kAbRows * pitch + cc * 16 + r0 * pitch;
            const int cofs = (kind ? vofs : 0) + g * hbytes + cc * 16;
            for (int r = r0; r < nt; r += rpp, dst += rpp * pitch)
                if (t0 + r != pos) cp_async16(dst, kr.at(t0 + r, d.row_bytes) + cofs);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // the first tiles' copies go out before the grid-dependency wait, except
    // in an attend launch, whose rows the append launch just before it wrote
    if (mode != 2) {
#pragma unroll
        for (int u = 0; u < kAbStages - 1; ++u) issue(u);
    }
    for (int i = threadIdx.x; i < half; i += kThreads) {
        sm.rc[i] = s.rope_cos[(size_t)pos * half + i];
        sm.rsn[i] = s.rope_sin[(size_t)pos * half + i];
    }
    if (d.qk_norm)
        for (int i = threadIdx.x; i < hd; i += kThreads) {
            sm.wq[i] = q_norm[(size_t)layer * hd + i];
            sm.wk[i] = k_norm[(size_t)layer * hd + i];
        }
    // zero the limb matrices and the P.V sums (absent heads, limbs and
    // positions past the sequence multiply as zero)
    for (int i = threadIdx.x; i < 16 * epitch / 16; i += kThreads) reinterpret_cast<int4*>(sm.ea)[i] = make_int4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < 8 * hd / 16; i += kThreads) reinterpret_cast<int4*>(sm.qb)[i] = make_int4(0, 0, 0, 0);
    pdl_launch_dependents();
    pdl_wait();
    if (mode == 2) {
#pragma unroll
        for (int u = 0; u < kAbStages - 1; ++u) issue(u);
    }

    // q heads, new k and v, qk-norm and RoPE (as the cluster kernel)
    const float* qkv = s.qkv + (size_t)b * (d.dim + 2 * d.kv_dim);
    for (int i = threadIdx.x; i < hq * hd; i += kThreads) sm.q[i] = qkv[(g * group + h0) * hd + i];
    for (int i = threadIdx.x; i < hd; i += kThreads) {
        sm.q[hq * hd + i] = qkv[d.dim + g * hd + i];
        sm.vn[i] = qkv[d.dim + d.kv_dim + g * hd + i];
    }
    __syncthreads();
    for (int hh = warp; hh <= hq; hh += kWarps) {
        float* v = sm.q + hh * hd;
        if (d.qk_norm) {
            double acc = 0.0;
            for (int i = lane; i < hd; i += 32) acc = __dadd_rn(acc, __dmul_rn((double)v[i], (double)v[i]));
            for (int o = 16; o; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
            const float ss = __double2float_rn(acc);
            const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), 1e-6f)));
            const float* w = hh < hq ? sm.wq : sm.wk;
            for (int i = lane; i < hd; i += 32) v[i] = __fmul_rn(w[i], __fmul_rn(r, v[i]));
            __syncwarp();
        }
        for (int i = lane; i < half; i += 32) {
            const int ia = d.rope_half ? i : 2 * i, ib = d.rope_half ? i + half : 2 * i + 1;
            const float a = v[ia], bb = v[ib], c = sm.rc[i], sv = sm.rsn[i];
            v[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, sv));
            v[ib] = __fadd_rn(__fmul_rn(a, sv), __fmul_rn(bb, c));
        }
    }
    __syncthreads();
    // encode the new row; the first q-head split's CTA writes it to the cache,
    // every CTA keeps its bytes for position `pos`
    uint8_t* row = kr.own + (size_t)pos * d.row_bytes + g * hbytes;
    const bool writer = split == 0 && mode != 2 && pos >= kr.plen;
    if (split == 0 && mode != 2 && pos < kr.plen && threadIdx.x == 0) atomicMin(s.err, kErrSharedAppend);
    for (int e = threadIdx.x; e < 2 * kw; e += kThreads) {
        const int w = e / kw, c = e % kw, i0 = c * (4 / KVB);
        const float* src = w ? sm.vn : sm.q + hq * hd;
        unsigned word = 0;
        float dec;
        for (int j = 0; j < 4 / KVB; ++j) word |= kv_encode(src[i0 + j], KVB, &dec) << (8 * KVB * j);
        if (writer) *reinterpret_cast<unsigned*>(row + (w ? vofs : 0) + c * 4) = word;
        *reinterpret_cast<unsigned*>(sm.newrow + w * hbytes + c * 4) = word;
    }
    if (mode == 1) return;   // the copies of an append launch are empty groups
    // each q head on its integer grid, split into balanced signed bytes: the
    // score MMAs' B operand, column 4*head + limb (limb 3 zero), dims in MMA k order
    if (warp < hq) {
        const float gs = warp_q_grid(sm.q + warp * hd, hd, KVB, sm.qi + warp * hd);
        if (lane == 0) sm.gsc[warp] = gs;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < hq * hd; e += kThreads) {
        const int hh = e / hd, i = e % hd;
        int v = sm.qi[e];
        const int l0 = ((v + 128) & 255) - 128;
        v = (v - l0) >> 8;
        const int l1 = ((v + 128) & 255) - 128;
        const int l2 = (v - l1) >> 8;
        const int k = KVB == 2 ? (i & ~31) + attnb_k_of(i & 31) : i;
        sm.qb[(4 * hh + 0) * hd + k] = (uint8_t)l0;
        sm.qb[(4 * hh + 1) * hd + k] = (uint8_t)l1;
        sm.qb[(4 * hh + 2) * hd + k] = (uint8_t)l2;
    }
    __syncthreads();
    // B fragments of the q limbs for every k block (column n = lane/4 = 4*head + limb)
    unsigned bq[KS][2];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        bq[ks][0] = *reinterpret_cast<const unsigned*>(sm.qb + gq * hd + ks * 32 + 4 * tq);
        bq[ks][1] = *reinterpret_cast<const unsigned*>(sm.qb + gq * hd + ks * 32 + 16 + 4 * tq);
    }

    // P.V work of a warp: position block pb (32 of a tile's 128 rows) and half
    // of the V columns; q8 blocks of 16 columns (even and odd MMAs), q16
    // blocks of 8 (high and low byte MMAs)
    constexpr int kDB = KVB == 1 ? HD / 16 : HD / 8;   // column blocks
    constexpr int kDBW = kDB / 2;                       // per warp
    const int pb = warp & 3, dh = warp >> 2;
    int acc[kDBW][2][4];
#pragma unroll
    for (int i = 0; i < kDBW; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[i][j][k] = 0;
    int nl = 0;                                         // weight limbs
    const unsigned ea_base = smem_addr(sm.ea);

    // One barrier per tile: it makes tile u visible and retires tile u-1, whose
    // slot the copy of tile u + stages - 1 then refills during tile u's work.
    for (int u = 0; u < 2 * ntile; ++u) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kAbStages - 2) : "memory");
        __syncthreads();
        issue(u + kAbStages - 1);
        uint8_t* tile = sm.ring + (size_t)(u % kAbStages) * kAbRows * pitch;
        const int kind = u >= ntile, t0 = (kind ? u - ntile : u) * kAbRows, nt = min(kAbRows, len - t0);
        if (pos >= t0 && pos < t0 + nt) {
            // this step's row, which the copies skipped
            for (int i = threadIdx.x; i < hbytes / 4; i += kThreads)
                reinterpret_cast<unsigned*>(tile + (pos - t0) * pitch)[i] =
                    reinterpret_cast<const unsigned*>(sm.newrow + kind * hbytes)[i];
            __syncthreads();
        }
        const unsigned tb = smem_addr(tile);
        if (!kind) {
            // scores of this K tile: warp w takes rows 16w .. 16w+15
            const int rb = warp * 16;
            if (rb < nt) {
                const int lr = rb + (lane & 7) + 8 * ((lane >> 3) & 1);   // ldmatrix row of this lane
                int dlo[4] = {0, 0, 0, 0}, dhi[4] = {0, 0, 0, 0};
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    if (KVB == 1) {
                        unsigned a[4];
                        ldsm_x4(tb + lr * pitch + ks * 32 + 16 * (lane >> 4), a);
                        mma_i8<false, false>(dhi, a, bq[ks][0], bq[ks][1]);
                    } else {
                        unsigned m[4], n[4], ah[4], al[4];
                        ldsm_x4(tb + lr * pitch + ks * 64 + 16 * (lane >> 4), m);
                        ldsm_x4(tb + lr * pitch + ks * 64 + 32 + 16 * (lane >> 4), n);
                        ah[0] = __byte_perm(m[0], m[2], 0x6420); al[0] = __byte_perm(m[0], m[2], 0x7531);
                        ah[1] = __byte_perm(m[1], m[3], 0x6420); al[1] = __byte_perm(m[1], m[3], 0x7531);
                        ah[2] = __byte_perm(n[0], n[2], 0x6420); al[2] = __byte_perm(n[0], n[2], 0x7531);
                        ah[3] = __byte_perm(n[1], n[3], 0x6420); al[3] = __byte_perm(n[1], n[3], 0x7531);
                        mma_i8<false, false>(dhi, ah, bq[ks][0], bq[ks][1]);
                        mma_i8<true, false>(dlo, al, bq[ks][0], bq[ks][1]);
                    }
                }
                // column 4*head + limb: lane tq holds (head tq/2, limbs 0 and 1) for
                // tq even, (head tq/2, limb 2) for tq odd; one shuffle per row
                // brings limb 2 to the even lane
                int v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) v[j] = KVB == 1 ? dhi[j] : dhi[j] * 256 + dlo[j];
                const int l2a = __shfl_down_sync(0xffffffffu, v[0], 1);
                const int l2b = __shfl_down_sync(0xffffffffu, v[2], 1);
                const int hh = tq >> 1;
                if (!(tq & 1) && hh < hq) {
                    const float ch = sm.gsc[hh];
                    const long long Sa = (long long)v[0] + 256LL * v[1] + 65536LL * l2a;
                    const long long Sb = (long long)v[2] + 256LL * v[3] + 65536LL * l2b;
                    const int ra = rb + gq, rbb = rb + gq + 8;
                    if (ra < nt) sm.sc[hh * d.seq + t0 + ra] = __fmul_rn(__ll2float_rn(Sa), ch);
                    if (rbb < nt) sm.sc[hh * d.seq + t0 + rbb] = __fmul_rn(__ll2float_rn(Sb), ch);
                }
            }
        } else {
            if (u == ntile) {
                // the weights E_t = rint(exp(s_t - max) * 2^k) of every position,
                // their exact sum, and their limbs: row h*NL + limb, position t at
                // column 32*(t/32) + attnb_k_of(t%32)
                const int kexp = attn_weight_exp(len, KVB);
                const float wscale = __int_as_float((127 + kexp) << 23);   // 2^k, exact
                nl = (kexp + 8) / 8;
                float mx[HQ];
#pragma unroll
                for (int hh = 0; hh < HQ; ++hh) mx[hh] = -1e30f;
                for (int t = threadIdx.x; t < len; t += kThreads)
#pragma unroll
                    for (int hh = 0; hh < HQ; ++hh) mx[hh] = fmaxf(mx[hh], sm.sc[hh * d.seq + t]);
#pragma unroll
                for (int hh = 0; hh < HQ; ++hh) {
                    for (int o = 16; o; o >>= 1) mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], o));
                    if (lane == 0) sm.redf[warp * HQ + hh] = mx[hh];
                }
                __syncthreads();
#pragma unroll
                for (int hh = 0; hh < HQ; ++hh) {
                    mx[hh] = sm.redf[hh];
                    for (int w = 1; w < kWarps; ++w) mx[hh] = fmaxf(mx[hh], sm.redf[w * HQ + hh]);
                }
                double dn[HQ];
#pragma unroll
                for (int hh = 0; hh < HQ; ++hh) dn[hh] = 0.0;
                for (int t = threadIdx.x; t < len; t += kThreads) {
                    uint8_t* col = sm.ea + (t & ~31) + attnb_k_of(t & 31);
#pragma unroll
                    for (int hh = 0; hh < HQ; ++hh) {
                        const float e = rintf(__fmul_rn(vexp(__fsub_rn(sm.sc[hh * d.seq + t], mx[hh])), wscale));
                        dn[hh] = __dadd_rn(dn[hh], (double)e);
                        // E < 2^47: bytes 0-3 from the low word, 4-5 from the high one
                        const unsigned long long E = (unsigned long long)e;
                        const unsigned lo = (unsigned)E, hi = (unsigned)(E >> 32);
                        uint8_t* c = col + (size_t)hh * nl * epitch;
#pragma unroll
                        for (int l = 0; l < kAbMaxLimbs; ++l)
                            if (l < nl) c[l * epitch] = (uint8_t)((l < 4 ? lo : hi) >> (8 * (l & 3)));
                    }
                }
#pragma unroll
                for (int hh = 0; hh < HQ; ++hh) {
                    for (int o = 16; o; o >>= 1) dn[hh] = __dadd_rn(dn[hh], __shfl_xor_sync(0xffffffffu, dn[hh], o));
                    if (lane == 0) sm.redd[warp * HQ + hh] = dn[hh];
                }
                __syncthreads();
                if (threadIdx.x < HQ) {
                    double tot = 0.0;
                    for (int w = 0; w < kWarps; ++w) tot = __dadd_rn(tot, sm.redd[w * HQ + threadIdx.x]);
                    sm.den[threadIdx.x] = tot;
                }
            }
            // P.V of this V tile
            const int pr = pb * 32;
            if (pr < nt) {
                unsigned a[4];
                ldsm_x4(ea_base + ((lane & 7) + 8 * ((lane >> 3) & 1)) * epitch + t0 + pr + 16 * (lane >> 4), a);
                const unsigned vrow = tb + (pr + (lane & 7) + 8 * (lane >> 3)) * pitch;
#pragma unroll
                for (int i = 0; i < kDBW; ++i) {
                    const int db = dh * kDBW + i;
                    unsigned m[4];
                    ldsm_x4_t(vrow + db * 16, m);
                    const unsigned b00 = __byte_perm(m[0], m[1], 0x6420), b01 = __byte_perm(m[2], m[3], 0x6420);
                    const unsigned b10 = __byte_perm(m[0], m[1], 0x7531), b11 = __byte_perm(m[2], m[3], 0x7531);
                    if (KVB == 1) {
                        mma_i8<true, false>(acc[i][0], a, b00, b01);   // even columns
                        mma_i8<true, false>(acc[i][1], a, b10, b11);   // odd columns
                    } else {
                        mma_i8<true, false>(acc[i][0], a, b00, b01);   // high bytes (signed)
                        mma_i8<true, true>(acc[i][1], a, b10, b11);    // low bytes (unsigned)
                    }
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();   // the ring is free: it takes the partial sums
    // each warp's exact limb products of its position block: part[pb][m][column]
    // (int64) for the rows m = h*NL + limb that exist
    long long* part = reinterpret_cast<long long*>(sm.ring);
    const int rows = hq * nl;
#pragma unroll
    for (int i = 0; i < kDBW; ++i) {
        const int db = dh * kDBW + i;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = gq + 8 * (j >> 1), col = 2 * tq + (j & 1);
            if (m >= rows) continue;
            long long* pm = part + ((size_t)pb * rows + m) * hd;
            if (KVB == 1) {
                pm[db * 16 + 2 * col] = acc[i][0][j];
                pm[db * 16 + 2 * col + 1] = acc[i][1][j];
            } else {
                pm[db * 8 + col] = (long long)acc[i][0][j] * 256 + acc[i][1][j];
            }
        }
    }
    __syncthreads();
    for (int o = threadIdx.x; o < hq * hd; o += kThreads) {
        const int hh = o / hd, i = o % hd;
        long long num = 0;
        for (int q = 0; q < 4; ++q)
            for (int l = 0; l < nl; ++l) num += part[((size_t)q * rows + hh * nl + l) * hd + i] * (1LL << (8 * l));
        s.att[(size_t)b * d.dim + (size_t)(g * group + h0 + hh) * hd + i] = att_q16((double)num, sm.den[hh], KVB);
    }
}

#endif  // VC4_COMMON_TU

// ---------------------------------------------------------------------------
// bare matvec (CPU-path entry)
// ---------------------------------------------------------------------------

template <int WT, int MAXC>
__global__ void __launch_bounds__(kThreads) k_raw(DMat W, const int16_t* xq, int n, int32_t* out) {
    WRegs<MAXC> R;
    mv_prefetch<WT, MAXC>(W, blockIdx.x, R);
    XStage xs; Red* red; long long* part; int16_t* tmp;
    carve<1>(x_stride(W), g_stride(W), xs, red, part, tmp);
    xs.k[0] = 0;
    stage_one<WT>(xs, 0, xq, n, 0, *red);
    long long S[1];
    mv_compute<WT, 1, MAXC>(W, R, xs, 1, S);
    const long long tot = reduce_warps<1>(S, 1, part);
    if (threadIdx.x < 32) {
        const int row = blockIdx.x * 32 + threadIdx.x;
        if (row < W.rows) out[row] = mv_epi(WT == W_T3 ? tot - xs.gsum[0] : tot, W.rscale[row]);
    }
}

// matvec_s for large matrices: persistent CTAs (two per SM) stage the input
// once, then each warp streams whole 32-row blocks, lane = row, with
// kStreamUnroll 16-byte loads per lane (512 contiguous bytes per warp) in
// flight while it multiplies the previous batch; no partial sum crosses warps
// and no barrier sits in the stream.  k_raw pays a CTA launch, the input
// staging and a cross-warp reduction for every block.  The integer
// arithmetic is k_raw's (exact dp4a dots, the same epilogue), so the outputs
// are equal.
constexpr int kStreamUnroll = 8;
constexpr int kStreamMinBlocks = 512;   // row blocks from which matvec_s streams

template <int WT>
__global__ void __launch_bounds__(kThreads, 2) k_raw_stream(DMat W, const int16_t* xq, int n, int32_t* out) {
    constexpr int U = kStreamUnroll;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nch = W.nchunks;
    const int nbat = (nch + U - 1) / U;
    const int stride = gridDim.x * kWarps, first = blockIdx.x * kWarps + warp;
    const int nblk = first < W.rblocks ? (W.rblocks - first + stride - 1) / stride : 0;
    const int items = nblk * nbat;   // (block, batch of U chunks) pairs of this warp
    int4 wn[U];
    int spn[U];
    auto load = [&](int t, int4 (&w)[U], int (&sp)[U]) {
        const int blk = first + (t / nbat) * stride, j0 = (t % nbat) * U;
        const int4* body = reinterpret_cast<const int4*>(W.body) + (size_t)blk * nch * 32 + lane;
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (j0 + u < nch) {
                w[u] = ld_weights(body + (size_t)(j0 + u) * 32);
                if (WT == W_Q4) sp[u] = __ldg(W.q4p + ((size_t)blk * nch + j0 + u) * 32 + lane);
            }
    };
    if (items > 0) load(0, wn, spn);   // the first weights before the input staging
    XStage xs; Red* red; long long* part; int16_t* tmp;
    carve<1>(x_stride(W), g_stride(W), xs, red, part, tmp);
    xs.k[0] = 0;
    stage_one<WT>(xs, 0, xq, n, 0, *red);
    int alo = 0, ahi = 0;
    long long S = 0;
    for (int t = 0; t < items; ++t) {
        int4 w[U];
        int sp[U];
#pragma unroll
        for (int u = 0; u < U; ++u) { w[u] = wn[u]; sp[u] = spn[u]; }
        if (t + 1 < items) load(t + 1, wn, spn);
        const int blk = first + (t / nbat) * stride, j0 = (t % nbat) * U;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u;
            if (j >= nch) break;
            if (WT == W_Q8) {
                const uint4 L = *reinterpret_cast<const uint4*>(xs.lo + j * 16);
                const uint4 H = *reinterpret_cast<const uint4*>(xs.hi + j * 16);
                alo = dp4a_su(w[u].x, L.x, alo); alo = dp4a_su(w[u].y, L.y, alo);
                alo = dp4a_su(w[u].z, L.z, alo); alo = dp4a_su(w[u].w, L.w, alo);
                ahi = dp4a_ss(w[u].x, (int)H.x, ahi); ahi = dp4a_ss(w[u].y, (int)H.y, ahi);
                ahi = dp4a_ss(w[u].z, (int)H.z, ahi); ahi = dp4a_ss(w[u].w, (int)H.w, ahi);
            } else if (WT == W_T3) {
                const unsigned wd[4] = {(unsigned)w[u].x, (unsigned)w[u].y, (unsigned)w[u].z, (unsigned)w[u].w};
                const uint4* L4 = reinterpret_cast<const uint4*>(xs.lo + j * 64);
                const uint4* H4 = reinterpret_cast<const uint4*>(xs.hi + j * 64);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 L = L4[q], H = H4[q];
                    const unsigned e0 = wd[q] & 0x03030303u, e1 = (wd[q] >> 2) & 0x03030303u;
                    const unsigned e2 = (wd[q] >> 4) & 0x03030303u, e3 = (wd[q] >> 6) & 0x03030303u;
                    alo = dp4a_uu(e0, L.x, alo); alo = dp4a_uu(e1, L.y, alo);
                    alo = dp4a_uu(e2, L.z, alo); alo = dp4a_uu(e3, L.w, alo);
                    ahi = dp4a_us(e0, (int)H.x, ahi); ahi = dp4a_us(e1, (int)H.y, ahi);
                    ahi = dp4a_us(e2, (int)H.z, ahi); ahi = dp4a_us(e3, (int)H.w, ahi);
                }
            } else {
                S += chunk_dot<W_Q4>(w[u], sp[u], xs.lo + j * 32, xs.hi + j * 32, xs.gsum[j]);
            }
        }
        if (j0 + U >= nch) {   // the block's last batch: epilogue of this lane's row
            const long long tot = WT == W_Q4 ? S : (long long)alo + 256LL * (long long)ahi;
            const int row = blk * 32 + lane;
            if (row < W.rows) out[row] = mv_epi(WT == W_T3 ? tot - xs.gsum[0] : tot, __ldg(W.rscale + row));
            alo = ahi = 0;
            S = 0;
        }
    }
}

#ifdef VC4_COMMON_TU
// i16 matrix (the MoE router, shaders.cpp:1216-1230): one block per row.
__global__ void __launch_bounds__(kThreads) k_raw_i16(DMat W, const int16_t* xq, int n, int32_t* out) {
    __shared__ Red red;
    const int row = blockIdx.x;
    long long acc = 0;
    for (int c = threadIdx.x; c < n; c += blockDim.x) acc += (long long)W.w16[(size_t)row * n + c] * xq[c];
    acc = block_sum_i64(acc, red);
    if (threadIdx.x == 0) out[row] = mv_epi(acc, W.rscale[row]);
}
#endif  // VC4_COMMON_TU

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------

// Raise a kernel's dynamic shared memory limit once per size; repeated calls
// (and calls during graph capture) are no-ops.
template <typename K>
void set_smem(K kernel, size_t bytes) {
    static std::map<std::pair<const void*, int>, size_t> done;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    size_t& have = done[{(const void*)kernel, dev}];
    if (bytes <= 48 * 1024 || bytes <= have) return;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    have = bytes;
}

// Every decode kernel is launched as a programmatic dependent of the one
// before it (griddepcontrol in the kernels), inside the captured graph too.
template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, size_t smem, cudaStream_t st, Args... args) {
    set_smem(kernel, smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// launch_pdl with a block size other than kThreads.
template <typename... KArgs, typename... Args>
void launch_pdl_block(void (*kernel)(KArgs...), dim3 grid, int block, size_t smem, cudaStream_t st, Args... args) {
    set_smem(kernel, smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

#include "batch.cuh"

constexpr int kNB = 4;   // inputs per CTA for the batched matvecs

// Registers per warp for a matrix: the smallest of 4/8/12/20 chunks that
// covers nchunks/8 (upload refuses a matrix above 160 chunks).
inline int maxc_for(int nch) {
    const int per = (nch + kWarps - 1) / kWarps;
    return per <= 4 ? 4 : per <= 8 ? 8 : per <= 12 ? 12 : 20;
}

#define VC4_MAXC(M, F, ...)                                          \
    do {                                                             \
        if ((M) == 4) F<4>(__VA_ARGS__);                             \
        else if ((M) == 8) F<8>(__VA_ARGS__);                        \
        else if ((M) == 12) F<12>(__VA_ARGS__);                      \
        else F<20>(__VA_ARGS__);                                     \
    } while (0)

// The w2 row scales the consumer of `layer`'s FFN output needs.
inline DownSrc down_src(const DModel& m, int layer) {
    DownSrc ds{};
    ds.layer = layer;
    ds.two = m.ffn_chunked ? 1 : 0;
    if (layer < 0) return ds;
    ds.hs = layer < (int)m.h.hid_scale.size() ? (int)m.h.hid_scale[layer] : 0;
    if (m.h.experts) {
        const int eb = m.e_w1[(size_t)layer * m.h.experts];
        ds.dm = m.d_mats;
        ds.ia = eb + 2;
        ds.ib = eb + 3;
    } else {
        ds.ra = m.mats[m.w2a[layer]].rscale;
        ds.rb = ds.two ? m.mats[m.w2b[layer]].rscale : nullptr;
    }
    return ds;
}

template <int WT>
struct Ops {
    template <int NB, int MAXC>
    static void qkv_nb(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        const DMat& W = m.mats[m.qkv[layer]];
        const DMat& E = m.mats[m.emb_mat];
        Dims d = dims_of(m, s);
        const size_t sm = mv_layout(wstage_bytes(W, NB), NB, NB * d.dim, d.dim, 0).total;
        const DownSrc ds = down_src(m, layer - 1);
        for (int b0 = 0; b0 < bt.n; b0 += NB)
            launch_pdl(k_qkv<WT, NB, MAXC>, dim3(W.rblocks), sm, st, W, E, m.d_emb_scale,
                       (const float*)(m.d_rms_att + (size_t)layer * d.dim), s, bt, d, layer, b0, ds);
    }
    template <int NB, int MAXC>
    static void wo_nb(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        const DMat& W = m.mats[m.wo[layer]];
        Dims d = dims_of(m, s);
        const size_t sm = mv_layout(wstage_bytes(W, NB), NB, NB * d.dim, 0, 0).total;
        for (int b0 = 0; b0 < bt.n; b0 += NB)
            launch_pdl(k_wo<WT, NB, MAXC>, dim3(W.rblocks), sm, st, W, s, bt, d, layer, b0);
    }
    template <int NB, int MAXC>
    static void gate_nb(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        Dims d = dims_of(m, s);
        MatSet M, M2;
        const bool two = m.ffn_chunked;
        if (d.experts) {
            const int eb = m.e_w1[(size_t)layer * d.experts];
            for (int e = 0; e < d.experts; ++e) {
                M.a[e] = m.mats[eb + 4 * e];
                M.b[e] = m.mats[eb + 4 * e + 1];
                M2.a[e] = m.mats[eb + 4 * e + 2];
                M2.b[e] = two ? m.mats[eb + 4 * e + 3] : m.mats[eb + 4 * e + 2];
            }
            M.router = m.mats[m.router[layer]];
        } else {
            M.a[0] = m.mats[m.w1[layer]];
            M.b[0] = m.mats[m.w3[layer]];
            M2.a[0] = m.mats[m.w2a[layer]];
            M2.b[0] = two ? m.mats[m.w2b[layer]] : m.mats[m.w2a[layer]];
        }
        const DMat& W1 = M.a[0];
        const size_t rbytes = d.experts ? sizeof(int16_t) * (size_t)d.experts * d.dim : 0;
        const size_t sm =
            mv_layout(wstage_bytes(W1, NB), NB, NB * d.dim, d.dim, align16(rbytes + 64) + ffn_down_bytes<WT>(NB)).total;
        const dim3 grid(W1.rblocks, d.experts ? d.experts : 1);
        const int hs = layer < (int)m.h.hid_scale.size() ? (int)m.h.hid_scale[layer] : 0;
        const int early = d.experts == 0 || bt.n >= 2 * d.experts;
        for (int b0 = 0; b0 < bt.n; b0 += NB)
            launch_pdl(k_gate<WT, NB, MAXC>, grid, sm, st, M, M2, (const float*)(m.d_rms_ffn + (size_t)layer * d.dim),
                       s, bt, d, layer, b0, hs, early);
    }
    template <int NB, int MAXC>
    static void logits_nb(const DModel& m, const State& s, const Batch& bt, const Finalize& fz, cudaStream_t st) {
        const DMat& W = m.mats[m.logits_mat];
        Dims d = dims_of(m, s);
        const int nsm = std::max(1, m.num_sms);
        const int stages = wide_stages(W, NB, d.dim);
        if (W.rblocks > 2 * nsm && stages >= 2) {
            const int grid = std::min((W.rblocks + kWarps - 1) / kWarps, nsm);
            const size_t wsm = wide_smem(W, NB, d.dim, stages);
            for (int b0 = 0; b0 < bt.n; b0 += NB)
                launch_pdl(k_logits_wide<NB>, dim3(grid), wsm, st, W, (const float*)m.d_rms_final, s, bt, d, b0, fz,
                           stages, down_src(m, m.h.layers - 1));
        } else {
            const size_t csm = mv_layout(wstage_bytes(W, NB), NB, NB * d.dim, d.dim, 0).total;
            for (int b0 = 0; b0 < bt.n; b0 += NB)
                launch_pdl(k_logits<NB, MAXC>, dim3(W.rblocks), csm, st, W, (const float*)m.d_rms_final, s, bt, d, b0,
                           fz, down_src(m, m.h.layers - 1));
        }
    }
    template <int MAXC>
    static void qkv(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        if (bt.n == 1) qkv_nb<1, MAXC>(m, s, bt, layer, st);
        else qkv_nb<kNB, MAXC>(m, s, bt, layer, st);
    }
    template <int MAXC>
    static void wo(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        if (bt.n == 1) wo_nb<1, MAXC>(m, s, bt, layer, st);
        else wo_nb<kNB, MAXC>(m, s, bt, layer, st);
    }
    template <int MAXC>
    static void gate(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        if (bt.n == 1) gate_nb<1, MAXC>(m, s, bt, layer, st);
        else gate_nb<kNB, MAXC>(m, s, bt, layer, st);
    }
    template <int MAXC>
    static void logits(const DModel& m, const State& s, const Batch& bt, const Finalize& fz, cudaStream_t st) {
        if (bt.n == 1) logits_nb<1, MAXC>(m, s, bt, fz, st);
        else logits_nb<kNB, MAXC>(m, s, bt, fz, st);
    }
    template <int MAXC>
    static void raw(const DMat& W, const int16_t* xq, int n, int32_t* out, cudaStream_t st) {
        const size_t sm = smem_bytes(1, x_stride(W), g_stride(W), 0);
        set_smem(k_raw<WT, MAXC>, sm);
        k_raw<WT, MAXC><<<W.rblocks, kThreads, sm, st>>>(W, xq, n, out);
    }
    static void raw_stream(const DMat& W, const int16_t* xq, int n, int32_t* out, cudaStream_t st) {
        const size_t sm = smem_bytes(1, x_stride(W), g_stride(W), 0);
        set_smem(k_raw_stream<WT>, sm);
        int dev = 0, nsm = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        const int grid = std::max(1, std::min(2 * nsm, (W.rblocks + kWarps - 1) / kWarps));
        k_raw_stream<WT><<<grid, kThreads, sm, st>>>(W, xq, n, out);
    }
};

// Launchers of the many-sequence path (batch.cuh).
constexpr int kMmGroupMax = 32;   // staged records per CTA at a time (two CTAs fit an SM)

// Grid z of a matmat launch: split the sequences so that about two CTAs per
// SM exist, each keeping at least `min_seqs` sequences (the expected count per
// expert for MoE); a CTA's warps serve kMmNI sequences each per sweep.
inline int mm_splits(const DModel& m, int ctas, int seqs, int min_seqs) {
    const int target = 2 * std::max(1, m.num_sms);
    int z = (target + ctas - 1) / ctas;
    z = std::min(z, std::max(1, seqs / min_seqs));
    return std::max(1, z);
}

// Tensor-core matmat launch (q8 or t3 weights, sequences not split by expert);
// false when the shapes do not fit, the caller then runs k_mm.
// Below kTcMinSeqs sequences a 128-row tile leaves most SMs idle and the CUDA-
// core kernel is faster; the logits head (many tiles) uses the tensor cores
// from kBatchMin.
constexpr int kTcMinSeqs = 32;
// t3 weights read as int8 levels move 4x the bytes of the packed 2-bit codes,
// so the CUDA-core matmat stays faster up to more sequences (c3 at 32: 13.8k
// vs 10.6k tokens/s)
constexpr int kTcMinSeqsT3 = 64;
constexpr size_t kSmemPerSm = 228 * 1024;   // shared memory of one SM (sm_100)

// TMA descriptors of the tensor-core matmat, encoded on the host through the
// runtime's driver entry point (the library does not link libcuda).
inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}
// A q8 or t3 matrix's row-major int8 copy, rows of x_stride bytes; one box is 64 rows x
// 128 bytes in the 128-byte swizzle layout (half of a weight tile's stage).
inline bool tmap_weights(CUtensorMap* map, const DMat& W) {
    const auto enc = tmap_encode_fn();
    if (!enc || !W.rm) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)x_stride(W), (cuuint64_t)W.rblocks * 32};
    const cuuint64_t strides[1] = {(cuuint64_t)x_stride(W)};
    const cuuint32_t box[2] = {128, 64}, es[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, W.rm, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// n staged records of rec_bytes (a multiple of 16); one box is N/2 records x
// 128 bytes in the 128-byte swizzle layout (half of a stage of one input plane).
inline bool tmap_records(CUtensorMap* map, const char* recs, int rec_bytes, int n, int N) {
    const auto enc = tmap_encode_fn();
    if (!enc || rec_bytes % 16) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)rec_bytes, (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)rec_bytes};
    const cuuint32_t box[2] = {128, (cuuint32_t)(N / 2)}, es[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<char*>(recs), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// VC4_TC_SPLIT=aligned|balanced pins the tensor-core matmats' work split
// (measurement sweeps); unset, the launch estimates which is shorter.
inline int tc_split_override() {
    static const int v = [] {
        const char* e = getenv("VC4_TC_SPLIT");
        return !e ? 0 : !strcmp(e, "aligned") ? 1 : !strcmp(e, "balanced") ? 2 : 0;
    }();
    return v;
}

template <int OP>
inline bool tc_launch(const DModel& m, const State& s, const Batch& bt, int layer, const DMat& W0, const DMat* W1,
                      int rec_bytes, int from_hrec, int lo0, int hi0, int lo1, int hi1, int hs, const DownRec& dr,
                      const Finalize& fz, cudaStream_t st) {
    if (OP != kOpLogits && bt.n < (W0.wtype == W_T3 ? kTcMinSeqsT3 : kTcMinSeqs)) return false;
    if ((W0.wtype != W_Q8 && W0.wtype != W_T3) || (W1 && (W1->wtype != W0.wtype || W1->rblocks != W0.rblocks)))
        return false;
    TcArgs a{};
    a.p[0] = TcPass{W0, lo0, hi0};
    a.npass = W1 ? 2 : 1;
    a.p[1] = W1 ? TcPass{*W1, lo1, hi1} : a.p[0];
    a.nin = (W1 && (lo1 != lo0 || hi1 != hi0)) ? 2 : 1;
    if (W1 && a.nin == 1 && W1->nchunks != W0.nchunks) return false;
    a.rec_bytes = rec_bytes;
    a.from_hrec = from_hrec;
    a.hs = hs;
    a.dr = dr;
    a.kc = std::max(tc_kchunks(W0), W1 ? tc_kchunks(*W1) : 0);
    a.t3 = W0.wtype == W_T3;
    const int tiles = (W0.rows + 127) / 128;
    const int nsm = std::max(1, m.num_sms);
    a.tiles = tiles;
    // The work is (tile, 16-sequence unit) pairs.  Aligned split: groups of N
    // sequences inside a tile, one CTA each, N chosen for the fewest bytes
    // streamed into the busiest SM (the tile's weights once per CTA, the
    // group's inputs once per tile).  Balanced split: one CTA per SM, equal
    // ranges of units, run in rounds of at most N sequences.  The epilogue is
    // done in pieces of 16 sequences per warp quarter, so a CTA's time is its
    // pieces per warp; the balanced split pays when the aligned one would
    // leave a second wave.
    static const int max_res = [] {   // the register file: 64K registers per SM
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, k_tmm<OP>) != cudaSuccess || fa.numRegs <= 0) return 1;
        return std::max(1, std::min(2, 65536 / (kTcThreads * fa.numRegs)));
    }();
    const int units_pt = (bt.n + 15) / 16;
    const long long units = (long long)tiles * units_pt;
    // TMEM: 2 * npass * N columns per CTA, shared by the CTAs of an SM
    const int cap = std::min(256, 512 / max_res / (2 * a.npass)) & ~15;
    const int nmax = (bt.n + 15) & ~15;
    const int slots = nsm * max_res;   // CTAs resident at once
    int Na = 0, ctas_a = 0;
    {
        double best = 0.0;
        for (int c = 16; c <= cap; c *= 2) {
            if (c > 16 && c / 2 >= nmax) break;
            if ((size_t)a.npass * kTcTileA * 2 + (size_t)a.nin * 2 * c * 128 * 2 > kMaxDynSmem) continue;   // two stages
            const int k = tiles * ((bt.n + c - 1) / c);
            const double per = (double)a.npass * a.kc * 2048 + (double)a.nin * a.kc * std::min(c, nmax) * 32;
            const double load = (double)((k + slots - 1) / slots) * per;
            if (Na == 0 || load <= best) { Na = c; ctas_a = k; best = load; }
        }
    }
    const int ctas_b = (int)std::min<long long>(units, slots);
    const int per_b = (int)((units + ctas_b - 1) / ctas_b);
    const int Nb = 16 * std::min(per_b, cap / 16);
    // pieces per warp of the busiest slot (4 warp quarters share a round's pieces)
    const int pieces_a = ((ctas_a + slots - 1) / slots) * ((Na / 16 + 3) / 4);
    // a range cut by a tile boundary or by N costs at most one partial piece more
    const int pieces_b = (per_b + 3) / 4 + (per_b > 1 ? 1 : 0);
    const int split = tc_split_override();   // 1 aligned, 2 balanced, 0 by the estimate
    // an aligned split that leaves a few CTAs for a second wave pays a whole
    // round for them (w1+w3 at 1024 sequences: 304 CTAs on 296 slots, 59.4 us
    // against 55.6 us balanced, measured)
    const bool spill = ctas_a > slots && ctas_a % slots <= slots / 8;
    const bool balanced = split == 2 || (split == 0 && Na > 0 && (pieces_b < pieces_a || spill));
    if (!balanced && Na == 0) return false;
    a.group = balanced ? Nb : Na;
    a.groups = balanced ? 0 : (bt.n + Na - 1) / Na;
    const int ctas = balanced ? ctas_b : ctas_a;
    const int resident = std::max(1, std::min(std::min((ctas + nsm - 1) / nsm, 4), max_res));
    int cols = 32;
    while (cols < 2 * a.npass * a.group) cols *= 2;
    a.tmem_cols = cols;
    // ring depth: the shared memory of the CTAs that share an SM
    const size_t budget = std::min(kMaxDynSmem, kSmemPerSm / std::min(resident, 512 / cols) - 1024);
    a.stages = 0;
    const size_t fixed = tc_smem(a), per_stage = tc_stage_bytes(a) + 16;   // ring stage + its two mbarriers
    a.stages = budget > fixed ? (int)std::min<size_t>(kTcMaxStages, (budget - fixed) / per_stage) : 0;
    if (a.stages < 2 || 2 * a.npass + 4 * a.nin > kTcThreads / 32 - 1) return false;
    const int N = a.group;
    TcMaps maps;
    if (!tmap_weights(&maps.a[0], W0) || !tmap_weights(&maps.a[1], W1 ? *W1 : W0) ||
        !tmap_records(&maps.b, from_hrec ? s.hrec : s.xrec, rec_bytes, bt.n, N))
        return false;
    Dims d = dims_of(m, s);
    launch_pdl_block(k_tmm<OP>, dim3(ctas), kTcThreads, tc_smem(a), st, maps, a, s, bt, d, layer, fz);
    return true;
}

template <int WT>
struct BOps {
    static void prep(const DModel& m, const State& s, const Batch& bt, int layer, int op, const DMat& W,
                     cudaStream_t st, DownRec dr = DownRec{}) {
        Dims d = dims_of(m, s);
        const float* rw = op == kOpWo ? m.d_rms_att
                        : op == kOpQkv ? m.d_rms_att + (size_t)layer * d.dim
                        : op == kOpGate ? m.d_rms_ffn + (size_t)layer * d.dim
                        : m.d_rms_final;
        DMat router{};
        if (op == kOpGate && d.experts) router = m.mats[m.router[layer]];
        launch_pdl(k_prep<WT>, dim3(bt.n), sizeof(int16_t) * (size_t)d.dim, st, W, m.mats[m.emb_mat], m.d_emb_scale,
                   rw, router, s, bt, d, layer, op, dr);
    }
    template <int OP>
    static void mm(const DModel& m, const State& s, const Batch& bt, int layer, const MatSet& M, int experts, int hs,
                   const Finalize& fz, cudaStream_t st, DownRec dr = DownRec{}) {
        Dims d = dims_of(m, s);
        const DMat& W = M.a[0];
        const int nm = OP == kOpGate ? 2 : 1;
        const int ctas = W.rblocks * (experts ? experts : 1);
        const int splits = mm_splits(m, ctas, bt.n / (experts ? experts : 1), 4);
        const size_t fixed = mm_smem(W, nm, 0, bt.n);
        const int want = (bt.n + splits - 1) / splits;
        const int group = std::max(1, std::min(std::min(want, kMmGroupMax), (int)((kMaxDynSmem - fixed) / xrec_bytes(W))));
        launch_pdl(k_mm<WT, OP>, dim3(W.rblocks, experts ? experts : 1, splits), mm_smem(W, nm, group, bt.n), st, M, s,
                   bt, d, layer, group, hs, fz, dr);
    }
    static void qkv(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        MatSet M;
        M.a[0] = M.b[0] = m.mats[m.qkv[layer]];
        prep(m, s, bt, layer, kOpQkv, M.a[0], st);
        const DMat& W = M.a[0];
        if (!tc_launch<kOpQkv>(m, s, bt, layer, W, nullptr, (int)xrec_bytes(W), 0, 0, x_stride(W), 0, 0, 0, DownRec{},
                               Finalize{}, st))
            mm<kOpQkv>(m, s, bt, layer, M, 0, 0, Finalize{}, st);
    }
    static void wo(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        MatSet M;
        M.a[0] = M.b[0] = m.mats[m.wo[layer]];
        prep(m, s, bt, layer, kOpWo, M.a[0], st);
        const DMat& W = M.a[0];
        if (!tc_launch<kOpWo>(m, s, bt, layer, W, nullptr, (int)xrec_bytes(W), 0, 0, x_stride(W), 0, 0, 0, DownRec{},
                              Finalize{}, st))
            mm<kOpWo>(m, s, bt, layer, M, 0, 0, Finalize{}, st);
    }
    static void ffn(const DModel& m, const State& s, const Batch& bt, int layer, cudaStream_t st) {
        Dims d = dims_of(m, s);
        MatSet M, M2;
        const bool two = m.ffn_chunked;
        if (d.experts) {
            const int eb = m.e_w1[(size_t)layer * d.experts];
            for (int e = 0; e < d.experts; ++e) {
                M.a[e] = m.mats[eb + 4 * e];
                M.b[e] = m.mats[eb + 4 * e + 1];
                M2.a[e] = m.mats[eb + 4 * e + 2];
                M2.b[e] = two ? m.mats[eb + 4 * e + 3] : m.mats[eb + 4 * e + 2];
            }
        } else {
            M.a[0] = m.mats[m.w1[layer]];
            M.b[0] = m.mats[m.w3[layer]];
            M2.a[0] = m.mats[m.w2a[layer]];
            M2.b[0] = two ? m.mats[m.w2b[layer]] : m.mats[m.w2a[layer]];
        }
        const int hs = layer < (int)m.h.hid_scale.size() ? (int)m.h.hid_scale[layer] : 0;
        const DMat& Wa = M2.a[0];
        const DMat& Wb = M2.b[0];
        const DownRec dr = down_rec(Wa, Wb, two);
        prep(m, s, bt, layer, kOpGate, M.a[0], st, dr);
        const DMat& W1 = M.a[0];
        const bool tc = d.experts == 0 &&
                        tc_launch<kOpGate>(m, s, bt, layer, W1, &M.b[0], (int)xrec_bytes(W1), 0, 0, x_stride(W1), 0,
                                           x_stride(W1), hs, dr, Finalize{}, st);
        if (!tc) mm<kOpGate>(m, s, bt, layer, M, d.experts, hs, Finalize{}, st, dr);
        if (tc && tc_launch<kOpDown>(m, s, bt, layer, Wa, two ? &Wb : nullptr, (int)dr.bytes, 1, (int)dr.lo_a,
                                     (int)dr.hi_a, (int)dr.lo_b, (int)dr.hi_b, hs, dr, Finalize{}, st))
            return;
        const int e = d.experts ? d.experts : 1;
        // dense: as few as four sequences per CTA (c4 at 16: ffn 55.4 -> 51.7 us,
        // c3b32 57.5 -> 56.4 us); MoE keeps whole sweeps of the expert's
        // sequences (c2 took 85 -> 102 us split finer)
        const int splits = mm_splits(m, Wa.rblocks * e, bt.n / e, d.experts ? kWarps * kMmNI : 2 * kMmNI);
        const size_t fixed = mmdown_smem(Wa, Wb, two, 0, bt.n);
        const int want = (bt.n + splits - 1) / splits;
        const int group =
            std::max(1, std::min(std::min(want, kMmGroupMax), (int)((kMaxDynSmem - fixed) / down_rec(Wa, Wb, two).bytes)));
        launch_pdl(k_mmdown<WT>, dim3(Wa.rblocks, e, splits), mmdown_smem(Wa, Wb, two, group, bt.n), st, M2, s, bt, d,
                   layer, group, hs);
    }
};

}  // namespace

// Per-weight-type launch entry points (ops_q8.cu, ops_q4.cu, ops_t3.cu).
#define VC4_OPS_DECL(SUF)                                                                       \
    void qkv_##SUF(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);  \
    void wo_##SUF(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);   \
    void gate_##SUF(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st); \
    void raw_##SUF(const DMat& W, const int16_t* xq, int n, int32_t* out, cudaStream_t st, int path = 0); \
    void bqkv_##SUF(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);    \
    void bwo_##SUF(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);     \
    void bffn_##SUF(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);
VC4_OPS_DECL(q8)
VC4_OPS_DECL(q4)
VC4_OPS_DECL(t3)

}  // namespace vc4
