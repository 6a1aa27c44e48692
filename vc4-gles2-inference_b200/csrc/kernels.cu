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
// kernel beats the clusters (whose per-CTA softmax is redundant work).
constexpr int kAttnBatchUnits = 128;

template <int KVB, int HQ>
static void launch_attn_b(const DModel& m, const State& s, const Batch& b, const Dims& d, int layer, size_t smb,
                          cudaStream_t st) {
    const int group = d.heads / d.kv_heads;
    launch_pdl(k_attn_b<KVB, HQ>, dim3(d.kv_heads * (group / HQ), b.n), smb, st, (const float*)m.d_q_norm,
               (const float*)m.d_k_norm, s, b, d, layer);
}

void launch_attention(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st) {
    Dims d = dims_of(m, s);
    const int group = d.heads / d.kv_heads, hq = attn_heads_per_cluster(group);
    const int units = b.n * d.kv_heads * (group / hq);
    const size_t smb = attnb_smem_bytes(hq, d.head_dim, d.seq, d.kv_bits);
    if (units >= kAttnBatchUnits && smb <= kMaxDynSmem && d.head_dim <= 4 * kThreads) {
        if (d.kv_bits == 8) {
            if (hq == 2) launch_attn_b<1, 2>(m, s, b, d, layer, smb, st);
            else launch_attn_b<1, 1>(m, s, b, d, layer, smb, st);
        } else {
            if (hq == 2) launch_attn_b<2, 2>(m, s, b, d, layer, smb, st);
            else launch_attn_b<2, 1>(m, s, b, d, layer, smb, st);
        }
        return;
    }
    const size_t sm = attn_smem_bytes(hq, d.head_dim, d.seq, d.kv_bits);
    launch_pdl(k_attn, dim3(d.kv_heads * (group / hq) * kAttnCtas, b.n), sm, st, (const float*)m.d_q_norm,
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

}  // namespace vc4
