// ops.cu -- the per-op boundary: the calls the reference's fused GPU layer
// loop (Session::forward_gpu_hidden, session.cpp:1459-1584) makes on class GPU
// (gpu.h:84-175, 256-264), one C function each, over per-slot device buffers
// instead of GL textures.  A layer loop written against these calls gives the
// token vc4_step gives: their arithmetic is the decode pass's (the reference
// CPU path's quantisation points, exact integer dots), which the fused kernels
// of engine.cu compute in fewer launches.  Buffers are q16 ints, one row per
// (buffer, slot); work is queued on the session stream.
#include "kernels.cuh"
#include "../../include/vc4b200.h"

#include <cstring>
#include <string>
#include <vector>

namespace vc4 {

namespace {

constexpr int kNumBufs = 9;    // VC4_BUF_HIDDEN .. VC4_BUF_TMP

// The per-op buffers of one session, made on its first per-op call.
struct OpBufs {
    int width = 0;             // max(dim, ffn width): the longest row
    int16_t* buf = nullptr;    // [kNumBufs][slots][width] q16 ints
    float* pend = nullptr;     // [slots][dim]: the first w2 half's output, waiting for the second
    int16_t* xq = nullptr;     // [width]: a staged matvec input
    int* kexp = nullptr;       // [2]: the staged input's 2^k exponent, and scratch
    int* call = nullptr;       // [3]: slot, token, position of an attention call
    int32_t* out = nullptr;    // [2 * rows_max]: matvec outputs (gate and up side by side)
    int rows_max = 0;
    std::vector<char> pending; // [slots]: TMP carries a first w2 half
};

int fail(int code, const std::string& msg) { return set_error(code, msg.c_str()); }

#define OPCK(call)                                                                                   \
    do {                                                                                             \
        const cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess) return fail(VC4_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

int16_t* buf_row(const OpBufs& o, int b, int slot, int slots) {
    return o.buf + ((size_t)b * slots + slot) * o.width;
}

// ---- kernels ------------------------------------------------------------------

// Stage a q16 row for a matvec: x' = x * 2^k, k from max|x| as matvec_s picks it
// (gpu_conv.cpp:271-287) when `scaled`, else 0 (an uploaded texture, read as is).
__global__ void k_op_stage(const int16_t* src, int n, int scaled, int16_t* xq, int* kout) {
    __shared__ Red red;
    int mx = 0;
    for (int c = threadIdx.x; c < n; c += blockDim.x) mx = max(mx, abs((int)src[c]));
    mx = block_max_i32(mx, red);
    const int k = scaled ? exp_from_max(mx) : 0;
    const float sk = ldexpf(1.0f, k);
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
        const int q = xscale(src[c], k, sk);
        xq[c] = (int16_t)(q < -32768 ? -32768 : q > 32767 ? 32767 : q);
    }
    if (threadIdx.x == 0) *kout = k;
}

// RMSNorm of one q16 row (session.cpp:1932-1948, the exact integer sum).
__global__ void k_op_rmsnorm(const int16_t* src, const float* w, int D, float eps, int16_t* dst) {
    __shared__ Red red;
    extern __shared__ __align__(16) char smem[];
    int16_t* x = reinterpret_cast<int16_t*>(smem);
    float nw[kPer];
    load_f32_regs(w, D, nw);
    for (int c = threadIdx.x; c < D; c += blockDim.x) x[c] = src[c];
    __syncthreads();
    rmsnorm_q16(x, nw, D, eps, x, red);
    for (int c = threadIdx.x; c < D; c += blockDim.x) dst[c] = x[c];
}

// matvec_s output as floats: (v/256) * 2^-k (the qkv vector attention reads).
__global__ void k_op_floats(const int32_t* v, int n, const int* k, float* out) {
    const float sk = ldexpf(1.0f, -*k);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = __fmul_rn(__fmul_rn((float)v[i], 1.0f / 256.0f), sk);
}

// dst = add_q16(res, (v/256) * 2^-k) (the attention output's residual add).
__global__ void k_op_add(const int16_t* res, const int32_t* v, const int* k, int n, int16_t* dst) {
    const float sk = ldexpf(1.0f, -*k);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float o = __fmul_rn(__fmul_rn((float)v[i], 1.0f / 256.0f), sk);
        dst[i] = (int16_t)q16h(__fadd_rn(__fmul_rn((float)res[i], 1.0f / 256.0f), o));
    }
}

// The FFN hidden row from gate g and up u (both matvec outputs of the staged
// input): the host FFN's quantize_act(SiLU(g)*u) with g, u read back *2^-k, or
// the GPU FFN's floor(SiLU(g)*u*2^-hs*256 + 0.5).
__global__ void k_op_gate(const int32_t* g, const int32_t* u, const int* k, int host, int hs, int F, int16_t* h) {
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < F; r += gridDim.x * blockDim.x) {
        int q;
        if (host) {
            q = host_hidden(g[r], u[r], *k);
        } else {
            float y = swiglu1(__fmul_rn((float)g[r], 1.0f / 256.0f), __fmul_rn((float)u[r], 1.0f / 256.0f));
            if (hs > 0) y = __fmul_rn(y, ldexpf(1.0f, -hs));
            q = q16s(y);
        }
        h[r] = (int16_t)q;
    }
}

// One w2 matvec's output o, then by `mode`: 0 a whole w2 (dst = add_q16(res, o)),
// 1 the first half (kept in pend; dst = res), 2 the second half (dst =
// add_q16(res, add_q16(pend, o))).  Host FFN: o = (v/256) * 2^-(k+hs); GPU FFN:
// o = v/256.
__global__ void k_op_w2(const int32_t* v, const int* k, int host, int hs, const int16_t* res, float* pend, int mode,
                        int D, int16_t* dst) {
    const float sk = host ? ldexpf(1.0f, -(*k + hs)) : 1.0f;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x) {
        float o = __fmul_rn((float)v[i], 1.0f / 256.0f);
        if (host) o = __fmul_rn(o, sk);
        const float x1 = __fmul_rn((float)res[i], 1.0f / 256.0f);
        if (mode == 1) {
            pend[i] = o;
            dst[i] = res[i];
        } else {
            if (mode == 2) o = __fmul_rn((float)q16h(__fadd_rn(pend[i], o)), 1.0f / 256.0f);
            dst[i] = (int16_t)q16h(__fadd_rn(x1, o));
        }
    }
}

__global__ void k_op_set_call(int* call, int slot, int token, int pos) {
    call[0] = slot;
    call[1] = token;
    call[2] = pos;
}

// Session::embedding (session.cpp:342-371): q16(level * row scale) of one token,
// read from the blocked q8 layout of the embedding matrix.
__global__ void k_op_embed(DMat E, const float* emb_scale, int tok, int D, int16_t* dst) {
    const float es = emb_scale[tok];
    const int8_t* eb = reinterpret_cast<const int8_t*>(E.body) + ((size_t)(tok / 32) * E.nchunks * 32 + (tok % 32)) * 16;
    for (int c = threadIdx.x; c < D; c += blockDim.x)
        dst[c] = (int16_t)q16h(__fmul_rn((float)eb[(size_t)(c / 16) * 512 + (c % 16)], es));
}

// ---- host helpers --------------------------------------------------------------

int ensure(vc4_session* s, OpBufs** out) {
    const SessionView v = session_view(s);
    if (*v.ops) {
        *out = static_cast<OpBufs*>(*v.ops);
        return VC4_OK;
    }
    const DModel& m = *v.m;
    OpBufs* o = new OpBufs();
    o->width = std::max(m.h.dim, m.ffn_width);
    int rows = m.h.dim + 2 * m.h.kv_dim;
    for (const DMat& w : m.mats) rows = std::max(rows, w.rows);
    o->rows_max = rows;
    o->pending.assign(v.slots, 0);
    const bool ok = cudaMalloc(&o->buf, sizeof(int16_t) * kNumBufs * (size_t)v.slots * o->width) == cudaSuccess &&
                    cudaMalloc(&o->pend, sizeof(float) * (size_t)v.slots * m.h.dim) == cudaSuccess &&
                    cudaMalloc(&o->xq, sizeof(int16_t) * (size_t)o->width) == cudaSuccess &&
                    cudaMalloc(&o->kexp, sizeof(int) * 4) == cudaSuccess &&
                    cudaMalloc(&o->call, sizeof(int) * 4) == cudaSuccess &&
                    cudaMalloc(&o->out, sizeof(int32_t) * 2 * (size_t)rows) == cudaSuccess;
    if (!ok) {
        free_op_buffers(o);
        return fail(VC4_ECUDA, "per-op buffer allocation failed");
    }
    cudaMemsetAsync(o->buf, 0, sizeof(int16_t) * kNumBufs * (size_t)v.slots * o->width, v.stream);
    *v.ops = o;
    *out = o;
    return VC4_OK;
}

int check_args(vc4_session* s, int slot, std::initializer_list<int> bufs) {
    const SessionView v = session_view(s);
    if (slot < 0 || slot >= v.slots) return fail(VC4_EINVAL, "slot out of range");
    for (int b : bufs)
        if (b < 0 || b >= kNumBufs) return fail(VC4_EINVAL, "no such per-op buffer");
    return VC4_OK;
}

// matvec of model matrix `mat` over a buffer row (n values): staged, then the
// bare matvec kernel; the clamped q16 results land in o->out + off.
void matvec(const SessionView& v, OpBufs* o, int mat, const int16_t* src, int n, int scaled, size_t off) {
    k_op_stage<<<1, kThreads, 0, v.stream>>>(src, n, scaled, o->xq, o->kexp);
    launch_matvec_raw(*v.m, mat, o->xq, n, o->out + off, v.stream);
    *v.launches += 2;
}

int grid_of(int n) { return std::max(1, std::min((n + 255) / 256, 1184)); }

}  // namespace

void free_op_buffers(void* p) {
    OpBufs* o = static_cast<OpBufs*>(p);
    if (!o) return;
    for (void* d : {(void*)o->buf, (void*)o->pend, (void*)o->xq, (void*)o->kexp, (void*)o->call, (void*)o->out})
        if (d) cudaFree(d);
    delete o;
}

}  // namespace vc4

using namespace vc4;

extern "C" {

int vc4_embedding(vc4_session* s, int slot, int token, int dst) {
    if (int e = check_args(s, slot, {dst})) return e;
    const SessionView v = session_view(s);
    const DModel& m = *v.m;
    if (token < 0 || token >= m.h.vocab) return fail(VC4_EINVAL, "token id out of range");
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(m.device));
    if (int e = ensure(s, &o)) return e;
    k_op_embed<<<1, kThreads, 0, v.stream>>>(m.mats[m.emb_mat], m.d_emb_scale, token, m.h.dim,
                                             buf_row(*o, dst, slot, v.slots));
    *v.launches += 1;
    o->pending[slot] &= dst != VC4_BUF_TMP;
    OPCK(cudaGetLastError());
    return VC4_OK;
}

int vc4_upload_hidden(vc4_session* s, int slot, const float* x, int dst) {
    if (int e = check_args(s, slot, {dst})) return e;
    const SessionView v = session_view(s);
    const int D = v.m->h.dim;
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(v.m->device));
    if (int e = ensure(s, &o)) return e;
    std::vector<int16_t> q(D);
    for (int i = 0; i < D; ++i) {
        const long r = lrintf(x[i] * 256.0f);   // quantize_act (common.h:188-193)
        q[i] = (int16_t)(r < -32768 ? -32768 : r > 32767 ? 32767 : r);
    }
    OPCK(cudaMemcpyAsync(buf_row(*o, dst, slot, v.slots), q.data(), sizeof(int16_t) * D, cudaMemcpyHostToDevice,
                         v.stream));
    OPCK(cudaStreamSynchronize(v.stream));   // q is a host temporary
    *v.syncs += 1;
    if (dst == VC4_BUF_TMP) o->pending[slot] = 0;
    return VC4_OK;
}

int vc4_rmsnorm(vc4_session* s, int slot, int src, int weights, int layer, int dst) {
    if (int e = check_args(s, slot, {src, dst})) return e;
    const SessionView v = session_view(s);
    const DModel& m = *v.m;
    const int D = m.h.dim;
    if (weights < 0 || weights > 2 || (weights < 2 && (layer < 0 || layer >= m.h.layers)))
        return fail(VC4_EINVAL, "rmsnorm: weights 0 (attention), 1 (ffn) or 2 (final) of a valid layer");
    const float* w = weights == 0 ? m.d_rms_att + (size_t)layer * D
                   : weights == 1 ? m.d_rms_ffn + (size_t)layer * D
                   : m.d_rms_final;
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(m.device));
    if (int e = ensure(s, &o)) return e;
    k_op_rmsnorm<<<1, kThreads, sizeof(int16_t) * D, v.stream>>>(buf_row(*o, src, slot, v.slots), w, D, m.h.rms_eps,
                                                               buf_row(*o, dst, slot, v.slots));
    *v.launches += 1;
    OPCK(cudaGetLastError());
    return VC4_OK;
}

int vc4_attention_block(vc4_session* s, int slot, int layer, int pos, int src, int dst) {
    if (int e = check_args(s, slot, {src, dst})) return e;
    const SessionView v = session_view(s);
    const DModel& m = *v.m;
    const State& st = *v.st;
    if (layer < 0 || layer >= m.h.layers) return fail(VC4_EINVAL, "layer out of range");
    if (pos < 0 || pos >= st.seq) return fail(VC4_EINVAL, "position out of range");
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(m.device));
    if (int e = ensure(s, &o)) return e;
    const int D = m.h.dim, Q = D + 2 * m.h.kv_dim;
    // qkv = matvec_s(qkv, xb) into batch position 0 of the pass buffers, then the
    // attention kernel for (slot, pos): qk-norm, RoPE, the packed KV append,
    // attention.  The attention kernel reads its (slot, pos) before its
    // grid-dependency wait, so they are written ahead of the matvec, not by the
    // kernel right before it.
    if (int e = session_unshare(s, slot, pos)) return e;   // the append below writes row pos
    k_op_set_call<<<1, 1, 0, v.stream>>>(o->call, slot, 0, pos);
    matvec(v, o, m.qkv[layer], buf_row(*o, src, slot, v.slots), D, 1, 0);
    k_op_floats<<<grid_of(Q), 256, 0, v.stream>>>(o->out, Q, o->kexp, st.qkv);
    Batch b;
    b.n = 1;
    b.slot = o->call;
    b.token = o->call + 1;
    b.pos = o->call + 2;
    launch_attention(m, st, b, layer, v.stream);
    OPCK(cudaMemcpyAsync(buf_row(*o, dst, slot, v.slots), st.att, sizeof(int16_t) * D, cudaMemcpyDeviceToDevice,
                         v.stream));
    *v.launches += 3;
    OPCK(cudaGetLastError());
    return VC4_OK;
}

int vc4_matvec_add(vc4_session* s, int slot, int which, int layer, int expert, int src, int residual, int dst) {
    if (int e = check_args(s, slot, {src, residual, dst})) return e;
    const SessionView v = session_view(s);
    const DModel& m = *v.m;
    const int D = m.h.dim;
    const bool host = !m.h.experts && m.ffn_chunked;
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(m.device));
    if (int e = ensure(s, &o)) return e;
    int16_t* dptr = buf_row(*o, dst, slot, v.slots);
    const int16_t* rptr = buf_row(*o, residual, slot, v.slots);
    if (which == 1) {   // wo: add_q16(x, matvec_s(wo, att))
        if (layer < 0 || layer >= m.h.layers) return fail(VC4_EINVAL, "layer out of range");
        matvec(v, o, m.wo[layer], buf_row(*o, src, slot, v.slots), D, 1, 0);
        k_op_add<<<grid_of(D), 256, 0, v.stream>>>(rptr, o->out, o->kexp, D, dptr);
        *v.launches += 1;
        OPCK(cudaGetLastError());
        return VC4_OK;
    }
    if (which != 4 && which != 7) return fail(VC4_EINVAL, "matvec_add: which is 1 (wo), 4 (w2 or its first half) or 7 (second half)");
    if (layer < 0 || layer >= m.h.layers) return fail(VC4_EINVAL, "layer out of range");
    if (m.h.experts && (expert < 0 || expert >= m.h.experts)) return fail(VC4_EINVAL, "expert out of range");
    const int eb = m.h.experts ? m.e_w1[(size_t)layer * m.h.experts + expert] : -1;
    const int wa = eb >= 0 ? eb + 2 : m.w2a[layer];
    const int wb = eb >= 0 ? eb + 3 : m.w2b[layer];
    if (which == 7 && !m.ffn_chunked) return fail(VC4_EINVAL, "matvec_add: this FFN has one w2");
    const int mat = which == 4 ? wa : wb;
    const int n = m.mats[mat].cols;
    int mode = 0;
    if (m.ffn_chunked) {
        if (which == 4) {
            mode = 1;
            if (dst != VC4_BUF_TMP) return fail(VC4_EINVAL, "matvec_add: the first w2 half goes to VC4_BUF_TMP");
        } else {
            if (residual != VC4_BUF_TMP || !o->pending[slot])
                return fail(VC4_ESTATE, "matvec_add: the second w2 half needs the first half's VC4_BUF_TMP");
            mode = 2;
        }
    }
    const int hs = layer < (int)m.h.hid_scale.size() ? (int)m.h.hid_scale[layer] : 0;
    matvec(v, o, mat, buf_row(*o, src, slot, v.slots), n, host ? 1 : 0, 0);
    k_op_w2<<<grid_of(D), 256, 0, v.stream>>>(o->out, o->kexp, host ? 1 : 0, hs, rptr,
                                              o->pend + (size_t)slot * D, mode, D, dptr);
    *v.launches += 1;
    o->pending[slot] = mode == 1 ? 1 : (dst == VC4_BUF_TMP ? 0 : o->pending[slot]);
    OPCK(cudaGetLastError());
    return VC4_OK;
}

int vc4_matvec_from(vc4_session* s, int slot, int which, int layer, int expert, int src, int input_scale,
                    float* out) {
    if (int e = check_args(s, slot, {src})) return e;
    const SessionView v = session_view(s);
    const DModel& m = *v.m;
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(m.device));
    if (int e = ensure(s, &o)) return e;
    int mat = -1;
    if (which == 5) {
        if (!m.h.experts || layer < 0 || layer >= m.h.layers) return fail(VC4_EINVAL, "matvec_from: no router");
        mat = m.router[layer];
    } else if (which == 0 || which == 1) {
        if (layer < 0 || layer >= m.h.layers) return fail(VC4_EINVAL, "layer out of range");
        mat = which == 0 ? m.qkv[layer] : m.wo[layer];
    } else {
        return fail(VC4_EINVAL, "matvec_from: which is 0 (qkv), 1 (wo) or 5 (router)");
    }
    (void)expert;
    const DMat& W = m.mats[mat];
    matvec(v, o, mat, buf_row(*o, src, slot, v.slots), W.cols, input_scale ? 1 : 0, 0);
    std::vector<int32_t> r(W.rows);
    int k = 0;
    OPCK(cudaMemcpyAsync(r.data(), o->out, sizeof(int32_t) * W.rows, cudaMemcpyDeviceToHost, v.stream));
    OPCK(cudaMemcpyAsync(&k, o->kexp, sizeof(int), cudaMemcpyDeviceToHost, v.stream));
    OPCK(cudaStreamSynchronize(v.stream));
    *v.syncs += 1;
    const float inv = ldexpf(1.0f, -k);
    for (int i = 0; i < W.rows; ++i) out[i] = ((float)r[i] / 256.0f) * inv;
    return VC4_OK;
}

int vc4_ffn_split(vc4_session* s, int slot, int layer, int expert, int src, int dst_a, int dst_b) {
    if (int e = check_args(s, slot, {src, dst_a, dst_b})) return e;
    const SessionView v = session_view(s);
    const DModel& m = *v.m;
    const int D = m.h.dim, F = m.ffn_width;
    const bool host = !m.h.experts && m.ffn_chunked;
    if (layer < 0 || layer >= m.h.layers) return fail(VC4_EINVAL, "layer out of range");
    if (m.h.experts && (expert < 0 || expert >= m.h.experts)) return fail(VC4_EINVAL, "expert out of range");
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(m.device));
    if (int e = ensure(s, &o)) return e;
    const int eb = m.h.experts ? m.e_w1[(size_t)layer * m.h.experts + expert] : -1;
    const int w1 = eb >= 0 ? eb : m.w1[layer], w3 = eb >= 0 ? eb + 1 : m.w3[layer];
    const int16_t* x = buf_row(*o, src, slot, v.slots);
    // gate and up over the same staged input (one stage, two bare matvecs)
    k_op_stage<<<1, kThreads, 0, v.stream>>>(x, D, host ? 1 : 0, o->xq, o->kexp);
    launch_matvec_raw(m, w1, o->xq, D, o->out, v.stream);
    launch_matvec_raw(m, w3, o->xq, D, o->out + o->rows_max, v.stream);
    int16_t* h = o->xq;   // the hidden row, then split into the two chunk buffers
    const int hs = layer < (int)m.h.hid_scale.size() ? (int)m.h.hid_scale[layer] : 0;
    k_op_gate<<<grid_of(F), 256, 0, v.stream>>>(o->out, o->out + o->rows_max, o->kexp, host ? 1 : 0, hs, F, h);
    const int ca = m.ffn_chunked ? m.ffn_chunk : F;
    OPCK(cudaMemcpyAsync(buf_row(*o, dst_a, slot, v.slots), h, sizeof(int16_t) * ca, cudaMemcpyDeviceToDevice,
                         v.stream));
    if (m.ffn_chunked)
        OPCK(cudaMemcpyAsync(buf_row(*o, dst_b, slot, v.slots), h + ca, sizeof(int16_t) * (F - ca),
                             cudaMemcpyDeviceToDevice, v.stream));
    *v.launches += 4;
    OPCK(cudaGetLastError());
    return VC4_OK;
}

int vc4_logits_from(vc4_session* s, int slot, int src, float* logits) {
    if (int e = check_args(s, slot, {src})) return e;
    const SessionView v = session_view(s);
    const DModel& m = *v.m;
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(m.device));
    if (int e = ensure(s, &o)) return e;
    const int V = m.h.vocab;
    matvec(v, o, m.logits_mat, buf_row(*o, src, slot, v.slots), m.h.dim, 0, 0);
    std::vector<int32_t> r(V);
    OPCK(cudaMemcpyAsync(r.data(), o->out, sizeof(int32_t) * V, cudaMemcpyDeviceToHost, v.stream));
    OPCK(cudaStreamSynchronize(v.stream));
    *v.syncs += 1;
    if (int e = kernel_check(s)) return e;
    for (int i = 0; i < V; ++i) logits[i] = (float)r[i] / 256.0f;
    return VC4_OK;
}

int vc4_logits_argmax_from(vc4_session* s, int slot, int src, int* token) {
    const SessionView v = session_view(s);
    std::vector<float> lg(v.m->h.vocab);
    if (int e = vc4_logits_from(s, slot, src, lg.data())) return e;
    int best = 0;   // the first maximum (sampling.cpp:160-162)
    for (int i = 1; i < (int)lg.size(); ++i)
        if (lg[i] > lg[best]) best = i;
    *token = best;
    return VC4_OK;
}

int vc4_read_buffer(vc4_session* s, int slot, int buf, int n, float* out) {
    if (int e = check_args(s, slot, {buf})) return e;
    const SessionView v = session_view(s);
    OpBufs* o = nullptr;
    OPCK(cudaSetDevice(v.m->device));
    if (int e = ensure(s, &o)) return e;
    if (n < 0 || n > o->width) return fail(VC4_EINVAL, "read_buffer: n out of range");
    std::vector<int16_t> q(n);
    OPCK(cudaMemcpyAsync(q.data(), buf_row(*o, buf, slot, v.slots), sizeof(int16_t) * n, cudaMemcpyDeviceToHost,
                         v.stream));
    OPCK(cudaStreamSynchronize(v.stream));
    *v.syncs += 1;
    for (int i = 0; i < n; ++i) out[i] = (float)q[i] / 256.0f;
    return VC4_OK;
}

}  // extern "C"
