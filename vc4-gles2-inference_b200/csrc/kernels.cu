// kernels.cu -- launch entry points of the decode step; the weight-type
// independent kernels (attention, logits, the i16 router matvec) are
// instantiated here, the matvec kernels of each weight type in ops_*.cu.
#define VC4_COMMON_TU
#include "kernels.cuh"

namespace vc4 {
namespace {
using LogitsOps = Ops<W_Q8>;
}  // namespace

// Calls FN_q8 / FN_q4 / FN_t3 by weight type.
#define VC4_BY_TYPE(WT, FN, ...)                  \
    do {                                          \
        if ((WT) == W_Q8) FN##_q8(__VA_ARGS__);   \
        else if ((WT) == W_Q4) FN##_q4(__VA_ARGS__); \
        else FN##_t3(__VA_ARGS__);                \
    } while (0)

// The many-sequence kernels serve a pass of at least kBatchMin sequences
// when every weight block fits shared memory next to one staged input.
static bool batched(const State& s, const Batch& b) { return s.batch_ok && b.n >= kBatchMin; }

void launch_embed_qkv(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    const DMat& W = m.mats[m.qkv[layer]];
    if (batched(s, b)) VC4_BY_TYPE(W.wtype, bqkv, m, s, b, layer, st);
    else VC4_BY_TYPE(W.wtype, qkv, m, s, b, layer, st);
}
void launch_wo(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    const DMat& W = m.mats[m.wo[layer]];
    if (batched(s, b)) VC4_BY_TYPE(W.wtype, bwo, m, s, b, layer, st);
    else VC4_BY_TYPE(W.wtype, wo, m, s, b, layer, st);
}
void launch_ffn_gate(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    const DMat& W = m.h.experts ? m.mats[m.e_w1[(size_t)layer * m.h.experts]] : m.mats[m.w1[layer]];
    if (batched(s, b)) VC4_BY_TYPE(W.wtype, bffn, m, s, b, layer, st);
    else VC4_BY_TYPE(W.wtype, gate, m, s, b, layer, st);
}
void launch_logits(const DModel& m, const State& s, const Batch& b, int* next, int* tokens, int* pos, int advance,
                   const int* forced, cudaStream_t st) {
    const DMat& W = m.mats[m.logits_mat];
    Finalize fz{next, tokens, pos, forced, advance};
    if (batched(s, b)) {
        MatSet M;
        M.a[0] = M.b[0] = W;
        BOps<W_Q8>::prep(m, s, b, m.h.layers - 1, kOpLogits, W, st);
        if (!tc_launch<kOpLogits>(m, s, b, m.h.layers - 1, W, nullptr, (int)xrec_bytes(W), 0, 0, x_stride(W), 0, 0, 0,
                                  DownRec{}, fz, st))
            BOps<W_Q8>::mm<kOpLogits>(m, s, b, m.h.layers - 1, M, 0, 0, fz, st);
        return;
    }
    VC4_MAXC(maxc_for(W.nchunks), LogitsOps::logits, m, s, b, fz, st);
}

// Bytes of one staged input record of the many-sequence path (the largest over
// the matrices a prep kernel stages for) and whether every weight block of
// the model fits the matmat kernels' shared memory.
size_t batch_record_bytes(const DModel& m) {
    const DMat& w1 = m.h.experts ? m.mats[m.e_w1[0]] : m.mats[m.w1[0]];
    return std::max(std::max(xrec_bytes(m.mats[m.qkv[0]]), xrec_bytes(m.mats[m.wo[0]])),
                    std::max(xrec_bytes(w1), xrec_bytes(m.mats[m.logits_mat])));
}
size_t batch_hidden_bytes(const DModel& m) {
    const DMat& wa = m.h.experts ? m.mats[m.e_w1[0] + 2] : m.mats[m.w2a[0]];
    const DMat& wb = m.ffn_chunked ? (m.h.experts ? m.mats[m.e_w1[0] + 3] : m.mats[m.w2b[0]]) : wa;
    return down_rec(wa, wb, m.ffn_chunked).bytes;
}
bool batch_path_fits(const DModel& m, int slots) {
    for (int l = 0; l < m.h.layers; ++l) {
        const int eb = m.h.experts ? m.e_w1[(size_t)l * m.h.experts] : -1;
        const DMat& w1 = eb >= 0 ? m.mats[eb] : m.mats[m.w1[l]];
        const DMat& wa = eb >= 0 ? m.mats[eb + 2] : m.mats[m.w2a[l]];
        const DMat& wb = m.ffn_chunked ? (eb >= 0 ? m.mats[eb + 3] : m.mats[m.w2b[l]]) : wa;
        if (mm_smem(m.mats[m.qkv[l]], 1, 1, slots) > kMaxDynSmem || mm_smem(m.mats[m.wo[l]], 1, 1, slots) > kMaxDynSmem ||
            mm_smem(w1, 2, 1, slots) > kMaxDynSmem || mmdown_smem(wa, wb, m.ffn_chunked, 1, slots) > kMaxDynSmem)
            return false;
    }
    return mm_smem(m.mats[m.logits_mat], 1, 1, slots) <= kMaxDynSmem;
}

// q heads per cluster: two when the group divides by two, else one
int attn_heads_per_cluster(int group) { return group % 2 == 0 ? 2 : 1; }

// From this many (sequence, KV head, q-head pair) units the one-CTA-per-unit
// kernel beats the clusters (whose per-CTA softmax is redundant work): at 16
// c4 sequences (64 units) 22.1 us per layer against the clusters' 35.9 us.
constexpr int kAttnBatchUnits = 32;

template <int KVB, int HQ>
static void launch_attn_b(const DModel& m, const State& s, const Batch& b, const Dims& d, int layer, size_t smb,
                          int mode, cudaStream_t st) {
    const int group = d.heads / d.kv_heads;
    const dim3 grid(d.kv_heads * (group / HQ), b.n);
    const float *qn = m.d_q_norm, *kn = m.d_k_norm;
    if (d.head_dim == 96) launch_pdl(k_attn_b<KVB, HQ, 96>, grid, smb, st, qn, kn, s, b, d, layer, mode);
    else if (d.head_dim == 64) launch_pdl(k_attn_b<KVB, HQ, 64>, grid, smb, st, qn, kn, s, b, d, layer, mode);
    else launch_pdl(k_attn_b<KVB, HQ, 128>, grid, smb, st, qn, kn, s, b, d, layer, mode);
}

bool prefill_attention_fits(const DModel& m, const State& s) {
    const int group = m.h.heads / m.h.kv_heads;
    const bool hd_ok = m.h.head_dim == 64 || m.h.head_dim == 96 || m.h.head_dim == 128;
    return hd_ok && attnb_smem_bytes(attn_heads_per_cluster(group), m.h.head_dim, s.seq, s.kv_bits) <= kMaxDynSmem;
}

void launch_attention(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st, int mode) {
    Dims d = dims_of(m, s);
    const int group = d.heads / d.kv_heads, hq = attn_heads_per_cluster(group);
    const int units = b.n * d.kv_heads * (group / hq);
    const size_t smb = attnb_smem_bytes(hq, d.head_dim, d.seq, d.kv_bits);
    // the many-sequence kernel is instantiated for head sizes 64, 96 and 128;
    // a prefill's append / attend launches (mode 1, 2) always take it (the
    // caller checked prefill_attention_fits)
    const bool hd_ok = d.head_dim == 64 || d.head_dim == 96 || d.head_dim == 128;
    if ((units >= kAttnBatchUnits || mode) && smb <= kMaxDynSmem && hd_ok) {
        if (d.kv_bits == 8) {
            if (hq == 2) launch_attn_b<1, 2>(m, s, b, d, layer, smb, mode, st);
            else launch_attn_b<1, 1>(m, s, b, d, layer, smb, mode, st);
        } else {
            if (hq == 2) launch_attn_b<2, 2>(m, s, b, d, layer, smb, mode, st);
            else launch_attn_b<2, 1>(m, s, b, d, layer, smb, mode, st);
        }
        return;
    }
    const size_t sm = attn_smem_bytes(hq, d.head_dim, d.seq, d.kv_bits);
    if (d.head_dim == 96) launch_pdl(k_attn<96>, dim3(d.kv_heads * (group / hq) * kAttnCtas, b.n), sm, st, (const float*)m.d_q_norm,
               (const float*)m.d_k_norm, s, b, d, layer, hq);
    else if (d.head_dim == 64) launch_pdl(k_attn<64>, dim3(d.kv_heads * (group / hq) * kAttnCtas, b.n), sm, st, (const float*)m.d_q_norm,
               (const float*)m.d_k_norm, s, b, d, layer, hq);
    else launch_pdl(k_attn<0>, dim3(d.kv_heads * (group / hq) * kAttnCtas, b.n), sm, st, (const float*)m.d_q_norm,
               (const float*)m.d_k_norm, s, b, d, layer, hq);
}

void launch_matvec_raw(const DModel& m, int mat, const int16_t* xq, int n, int32_t* out, cudaStream_t st) {
    const DMat& W = m.mats[mat];
    if (W.wtype == W_I16) { k_raw_i16<<<W.rows, kThreads, 0, st>>>(W, xq, n, out); return; }
    VC4_BY_TYPE(W.wtype, raw, W, xq, n, out, st);
}

int kernel_launches_per_step(const DModel& m, const State& s, int n) {
    Batch b;
    b.n = n;
    if (batched(s, b)) return m.h.layers * 8 + 2;   // prep + matmat per op, w2, attention; prep + logits
    const int g = n == 1 ? 1 : (n + kNB - 1) / kNB;
    return m.h.layers * (3 * g + 1) + g;
}

int max_input_cols() { return kPer * kThreads; }

bool attention_fits(int seq, int head_dim, int kv_bits, int kv_dim, int group) {
    const int hbytes = head_dim * (kv_bits / 8);
    if (hbytes % 16 || kv_dim % 16 || head_dim % 4) return false;
    // the attention weights' exact sums: 2^23 * 2^15 * seq < 2^53
    if (seq > 32768) return false;
    return attn_smem_bytes(attn_heads_per_cluster(group), head_dim, seq, kv_bits) <= kMaxDynSmem;
}

int matvec_max_chunks() { return 20 * kWarps; }

namespace {
// Reads n 16-byte words; stores only if their xor is a value no fill produces,
// so the loads stay and nothing is written.
__global__ void k_read_all(const int4* __restrict__ p, size_t n, int* sink) {
    int acc = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int4 v = __ldcs(p + i);
        acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    if (acc == 0x5A5A5A5B) *sink = acc;
}
}  // namespace

void l2_flush(void* buf, size_t bytes, int val, cudaStream_t st) {
    cudaMemsetAsync(buf, val & 0x7F, bytes, st);   // a uniform fill: every word's xor is 0, the sink is never written
    k_read_all<<<1184, 512, 0, st>>>(static_cast<const int4*>(buf), bytes / 16, static_cast<int*>(buf));
}

}  // namespace vc4

// ---------------------------------------------------------------------------
// Matvec roofline probe: the matvec_s kernel on a synthetic matrix in HBM
// ---------------------------------------------------------------------------

#include "vc4b200.h"

#include <vector>

namespace vc4 {
namespace {
__global__ void k_fill_bytes(uint8_t* p, size_t n, uint32_t seed) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t h = (uint32_t)i * 2654435761u ^ seed;
        h ^= h >> 15;
        h *= 2246822519u;
        h ^= h >> 13;
        p[i] = (uint8_t)h;
    }
}
}  // namespace
}  // namespace vc4

namespace vc4 {
namespace {
// The cache codec of the attention kernels (kv_encode) on arbitrary inputs:
// value i's packed bytes, as the cache row holds them (q16: two bytes,
// big-endian; q8: one two's-complement byte).
__global__ void k_kv_codec(const float* __restrict__ x, int n, int kvb, uint8_t* __restrict__ out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float dec;
        const unsigned w = kv_encode(x[i], kvb, &dec);
        out[(size_t)i * kvb] = (uint8_t)w;
        if (kvb == 2) out[(size_t)i * 2 + 1] = (uint8_t)(w >> 8);
    }
}
}  // namespace
}  // namespace vc4

extern "C" VC4_API int vc4_kv_codec_probe(int device, int kv_bits, const float* x, int n, void* out) {
    using namespace vc4;
    if ((kv_bits != 16 && kv_bits != 8) || n <= 0 || !x || !out) return set_error(VC4_EINVAL, "kv_codec_probe: bad arguments");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(VC4_ECUDA, "kv_codec_probe: cudaSetDevice failed");
    const int kvb = kv_bits / 8;
    float* dx = nullptr;
    uint8_t* dy = nullptr;
    if (cudaMalloc(&dx, (size_t)n * 4) != cudaSuccess) return set_error(VC4_ECUDA, "kv_codec_probe: cudaMalloc failed");
    if (cudaMalloc(&dy, (size_t)n * kvb) != cudaSuccess) {
        cudaFree(dx);
        return set_error(VC4_ECUDA, "kv_codec_probe: cudaMalloc failed");
    }
    cudaError_t e = cudaMemcpy(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        k_kv_codec<<<(n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184, 256>>>(dx, n, kvb, dy);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(out, dy, (size_t)n * kvb, cudaMemcpyDeviceToHost);
    cudaFree(dx);
    cudaFree(dy);
    if (e != cudaSuccess) return set_error(VC4_ECUDA, "kv_codec_probe: a CUDA call failed");
    return VC4_OK;
}

extern "C" VC4_API int vc4_matvec_probe(int device, int wtype, int rows, int cols, int path, int reps, int flush,
                                        double* ms_avg, double* bytes, unsigned long long* digest) {
    using namespace vc4;
    if (wtype < W_Q8 || wtype > W_T3 || rows <= 0 || cols <= 0 || path < 0 || path > 2 || reps <= 0 || !ms_avg ||
        !bytes || !digest)
        return set_error(VC4_EINVAL, "matvec_probe: bad arguments");
    if (wtype == W_Q4 && cols % 32) return set_error(VC4_EINVAL, "matvec_probe: q4 columns must be whole groups of 32");
    const int cpc = cols_per_chunk(wtype);
    DMat W;
    W.rows = rows; W.cols = cols; W.wtype = wtype;
    W.rblocks = (rows + kRowBlock - 1) / kRowBlock;
    W.nchunks = (cols + cpc - 1) / cpc;
    if (W.nchunks > matvec_max_chunks() || W.nchunks * cpc > max_input_cols())
        return set_error(VC4_EINVAL, "matvec_probe: matrix too wide for the matvec kernel");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(VC4_ECUDA, "matvec_probe: cudaSetDevice failed");
    const size_t nbody = (size_t)W.rblocks * W.nchunks * 512, nq4 = wtype == W_Q4 ? (size_t)W.rblocks * W.nchunks * 128 : 0;
    const size_t kFlush = flush ? (size_t)256 << 20 : 0;
    void *body = nullptr, *q4p = nullptr, *rs = nullptr, *xq = nullptr, *out = nullptr, *fl = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = VC4_OK;
    auto done = [&](int code, const char* msg) {
        if (code != VC4_OK) rc = set_error(code, msg);
        if (st) cudaStreamSynchronize(st);
        for (void* p : {body, q4p, rs, xq, out, fl}) if (p) cudaFree(p);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        if (st) cudaStreamDestroy(st);
        return rc;
    };
    if (cudaMalloc(&body, nbody) != cudaSuccess || (nq4 && cudaMalloc(&q4p, nq4) != cudaSuccess) ||
        cudaMalloc(&rs, (size_t)W.rblocks * kRowBlock * 4) != cudaSuccess || cudaMalloc(&xq, (size_t)cols * 2) != cudaSuccess ||
        cudaMalloc(&out, (size_t)rows * 4) != cudaSuccess || (kFlush && cudaMalloc(&fl, kFlush) != cudaSuccess))
        return done(VC4_ECUDA, "matvec_probe: cudaMalloc failed");
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess || cudaEventCreate(&e0) != cudaSuccess ||
        cudaEventCreate(&e1) != cudaSuccess)
        return done(VC4_ECUDA, "matvec_probe: stream or event creation failed");
    W.body = static_cast<uint8_t*>(body);
    W.q4p = static_cast<int32_t*>(q4p);
    W.rscale = static_cast<float*>(rs);
    k_fill_bytes<<<1184, 256, 0, st>>>(W.body, nbody, 0x1234u);
    if (nq4) k_fill_bytes<<<1184, 256, 0, st>>>(reinterpret_cast<uint8_t*>(q4p), nq4, 0x5678u);
    k_fill_bytes<<<64, 256, 0, st>>>(static_cast<uint8_t*>(xq), (size_t)cols * 2, 0x9abcu);
    cudaMemsetAsync(rs, 0x3A, (size_t)W.rblocks * kRowBlock * 4, st);   // row scales near 7e-4
    VC4_BY_TYPE(wtype, raw, W, static_cast<const int16_t*>(xq), cols, static_cast<int32_t*>(out), st, path);   // warm-up
    double total = 0.0;
    for (int r = 0; r < reps; ++r) {
        if (kFlush) l2_flush(fl, kFlush, r, st);
        cudaEventRecord(e0, st);
        VC4_BY_TYPE(wtype, raw, W, static_cast<const int16_t*>(xq), cols, static_cast<int32_t*>(out), st, path);
        cudaEventRecord(e1, st);
        if (cudaEventSynchronize(e1) != cudaSuccess) return done(VC4_ECUDA, "matvec_probe: a launch failed");
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e0, e1);
        total += ms;
    }
    if (cudaGetLastError() != cudaSuccess) return done(VC4_ECUDA, "matvec_probe: a launch failed");
    const double per = wtype == W_Q8 ? 1.0 : wtype == W_Q4 ? 0.5 : 0.25;
    *bytes = per * rows * cols + (wtype == W_Q4 ? 4.0 * rows * (cols / 32) : 0.0) + 4.0 * rows + 2.0 * cols + 4.0 * rows;
    *ms_avg = total / reps;
    std::vector<int32_t> h(rows);
    if (cudaMemcpyAsync(h.data(), out, (size_t)rows * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return done(VC4_ECUDA, "matvec_probe: reading the output failed");
    unsigned long long f = 1469598103934665603ull;   // FNV-1a over the output bytes
    for (int32_t v : h)
        for (int b = 0; b < 4; ++b) f = (f ^ (((uint32_t)v >> (8 * b)) & 0xFFu)) * 1099511628211ull;
    *digest = f;
    return done(VC4_OK, "");
}
