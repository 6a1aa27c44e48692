// vc4b200_internal.h -- shared definitions of the B200 decode engine.
//
// Device data layout (HBM):
//   * A weight matrix is stored in 32-row blocks.  Inside a block the rows are
//     interleaved at 16-byte granularity: chunk j of row (32*b + l) lives at
//     byte ((b*nchunks + j)*32 + l)*16.  One warp-wide 16-byte load therefore
//     reads 512 contiguous bytes, lane l getting its own row's chunk j.  A chunk
//     is 16 q8 weights, 32 q4 weights (one scale group) or 64 t3 weights.
//   * q8 weights are signed levels (the container's +128 bias removed).
//   * q4 nibbles are re-paired so byte k of a 4-byte word holds column k in its
//     low nibble and column k+4 in its high nibble; the group's int16 scale and
//     min travel as one int32 per (row, group) in the same 32-row interleave.
//   * t3 weights are 2-bit offset codes e = w + 1 in {0,1,2}; byte b of a
//     32-bit word holds the codes of columns b, b+4, b+8, b+12 of a 16-column
//     group at bits 0, 2, 4, 6, so (word >> 2i) & 0x03030303 is four
//     consecutive columns as bytes.  The dot product subtracts sum(x) once.
//   * q8 and t3 matrices also keep a plain row-major int8 copy of their
//     levels (rows of nchunks*cols_per_chunk bytes) that the tensor-core
//     matmat loads as 128-byte-wide TMA boxes.
//   * Every matrix carries one float epilogue scale per row (the reference's
//     `ws`, or (p16*ws)/65536 for a row-scaled matrix) and is padded to whole
//     blocks and chunks with zero weights.
//   * The KV cache keeps the reference's packed texel rows (K then V per
//     position, q16 big-endian or q8 bytes), so MMKV1 save/restore is a copy.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include <cuda_runtime.h>

namespace vc4 {

enum WType : int { W_Q8 = 0, W_Q4 = 1, W_T3 = 2, W_I16 = 3 };

constexpr int kRowBlock = 32;      // rows per block (one per lane)
constexpr int kChunkBytes = 16;    // bytes per chunk per row
constexpr int kWarps = 8;          // warps per matvec CTA (split the chunks)
constexpr int kLogitsGrid = 1536;  // logits tile height (logits_grid.h)

inline int cols_per_chunk(int wt) { return wt == W_Q8 ? 16 : wt == W_Q4 ? 32 : 64; }

// ---- host-side model (parsed container, reference semantics) -----------------

struct HMat {
    int rows = 0, cols = 0, wtype = W_Q8;
    float scale = 1.0f;              // q8/i16 ws; t3 record scale*127; q4 ps
    std::vector<int8_t> lev;         // q8 / t3 signed levels, rows*cols
    std::vector<uint8_t> nib;        // q4 nibble values, rows*cols
    std::vector<int16_t> s16, m16;   // q4 group planes, rows*groups
    std::vector<int16_t> w16;        // i16
    std::vector<uint16_t> p16;       // 16-bit row plane (empty: per-matrix scale)
    std::vector<float> plane;        // container f32 plane
    int groups() const { return cols / 32; }
};

struct HModel {
    int version = 0, dim = 0, hidden = 0, layers = 0, heads = 0, kv_heads = 0, vocab = 0, seq = 0;
    int head_dim = 0, kv_dim = 0, experts = 0, moe_hidden = 0;
    bool qk_norm = false, rope_half = false, head_dedup = false;
    float rope_theta = 10000.0f, rms_eps = 1e-5f;
    std::vector<float> rope_factors;
    std::vector<uint8_t> hid_scale;
    uint64_t source_size = 0, source_mtime = 0;
    std::string template_name;        // metadata key 4: the chat template's name (MMKV1 sidecar)
    std::vector<int8_t> emb;          // vocab*dim signed levels
    std::vector<float> emb_scale;     // vocab
    std::vector<float> rms_att, rms_ffn, rms_final, q_norm, k_norm;
    std::vector<HMat> qkv, wo, w1, w3, w2, router;
    std::vector<HMat> moe;            // [layer*experts + e]*3: w1, w3, w2
    std::vector<HMat> tiles;
    int ffn_width() const { return experts ? moe_hidden : hidden; }
};

// Parse an MMCF v2/v3 container (returns "" or an error message).
std::string load_mmcf(const std::string& path, HModel& m);
std::string load_mmcf_bytes(const uint8_t* data, size_t size, HModel& m);

// ---- device-side model ------------------------------------------------------

struct DMat {
    int rows = 0, cols = 0, wtype = W_Q8;
    int rblocks = 0, nchunks = 0;    // padded geometry
    uint8_t* body = nullptr;         // rblocks*nchunks*32*16 bytes
    float* rscale = nullptr;         // rblocks*32 epilogue scales
    int32_t* q4p = nullptr;          // q4: rblocks*nchunks*32 packed (s16 | m16<<16)
    int16_t* w16 = nullptr;          // i16 router, row-major
    int8_t* rm = nullptr;            // q8 / t3: the levels row-major, [rblocks*32][nchunks*cols_per_chunk] (tensor-core matmat)
    size_t bytes() const { return (size_t)rblocks * nchunks * 512 + (q4p ? (size_t)rblocks * nchunks * 128 : 0); }
};

struct DModel {
    HModel h;                        // dims and host copies of small tensors (weights dropped)
    int ffn_width = 0, ffn_chunk = 0;
    bool ffn_chunked = false;
    int wtype = W_Q8;
    std::vector<DMat> mats;          // every matrix, owning
    std::vector<int> qkv, wo, w1, w3, w2a, w2b, router;   // per layer: index into mats
    std::vector<int> e_w1, e_w3, e_w2a, e_w2b;            // [layer*experts + e]; the four
                                                          // matrices of an expert are consecutive
    int emb_mat = -1, logits_mat = -1;
    float* d_emb_scale = nullptr;
    float *d_rms_att = nullptr, *d_rms_ffn = nullptr, *d_rms_final = nullptr;
    float *d_q_norm = nullptr, *d_k_norm = nullptr;
    DMat* d_mats = nullptr;          // device array mirror of `mats` (for kernels that pick experts)
    size_t weight_bytes = 0;
    int device = 0;
    int num_sms = 0;                 // streaming multiprocessors of `device`
    std::vector<void*> allocs;     // every device allocation of the model
};

std::string upload_model(HModel&& h, DModel& d);
void free_model(DModel& d);

// ---- per-launch parameter blocks -------------------------------------------------

// The step's batch: n sequences, each with its slot (KV cache / state index),
// token id and position.  All arrays live on the device.
struct Batch {
    int n = 0;
    const int* slot = nullptr;
    const int* token = nullptr;
    const int* pos = nullptr;
};

struct State {                      // per-slot activations, [slot][...]
    // Activations are transient within a pass and indexed by batch position;
    // the KV cache is indexed by the sequence's slot.
    int16_t* x = nullptr;            // residual, q16 ints [slots][dim]
    int16_t* x1 = nullptr;           // residual after attention
    float* qkv = nullptr;            // matvec_s output [slots][dim+2kv]
    int16_t* att = nullptr;          // attention output, q16 [slots][dim]
    int16_t* h = nullptr;            // SwiGLU hidden, q16 [slots][ffn]
    int32_t* logits = nullptr;       // q16 ints [slots][vocab]
    unsigned long long* best = nullptr;   // packed argmax key [slots]
    int* next = nullptr;             // greedy token [slots]
    int* route = nullptr;            // MoE expert [slots][layers]
    uint8_t* kv = nullptr;           // [slots][layers][seq][row_bytes]
    // Shared prefix: one MMKV1 prefix held once for many slots.  Slot s reads
    // its positions t < plen[s] from pkv (row t of layer l at
    // pkv + (l*pcap + t)*row_bytes) and every other position from kv; those
    // rows are read-only (an append below plen is refused).
    uint8_t* pkv = nullptr;          // [layers][pcap][row_bytes]
    int* plen = nullptr;             // [slots], 0: the slot holds all its rows
    int pcap = 0;
    int kv_bits = 16, row_bytes = 0, seq = 0, slots = 0;
    float* rope_cos = nullptr;       // [seq][head_dim/2]
    float* rope_sin = nullptr;
    int* done = nullptr;             // CTA arrival counter of the logits kernel (reset by its last CTA)
    int* err = nullptr;              // kernel self-check word: nonzero = a launch reserved too little shared memory
    long long* sdown = nullptr;      // w2 partial sums [layers][slots][2][dim] (int64, zero between uses)
    int* hmax = nullptr;             // host FFN: max |q16 hidden| per [layers][slots][2 halves] (w2 input scale)
    char* xrec = nullptr;            // many-sequence path: staged matvec inputs [slots][record]
    char* hrec = nullptr;            // many-sequence path: staged w2 inputs [slots][record]
    int batch_ok = 0;                // the many-sequence kernels fit this model
};

// Kernel launchers (kernels.cu).  All enqueue on `st`; none synchronises.
void launch_embed_qkv(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);
// mode 0: decode; 1 / 2: the append and attend launches of a batched prefill
// (several positions of one sequence in one pass; see k_attn_b).
void launch_attention(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st, int mode = 0);
// Whether the many-sequence attention kernel, which a batched prefill needs,
// holds this session's sequence length and head shape.
bool prefill_attention_fits(const DModel& m, const State& s);
void launch_wo(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);
void launch_ffn_gate(const DModel& m, const State& s, const Batch& b, int layer, cudaStream_t st);
// Logits + first-max argmax; the launch's last CTA writes the greedy tokens to
// `next` and, with `advance`, moves each sequence on (token, position + 1);
// `forced` (indexed by position) replaces the greedy token during a prefill.
void launch_logits(const DModel& m, const State& s, const Batch& b, int* next, int* tokens, int* pos, int advance,
                   const int* forced, cudaStream_t st);
// A bare matvec of one model matrix over q16 inputs (the CPU-path entry,
// GPU::matvec_s): xq are already scaled ints, out receives clamped q16 ints.
void launch_matvec_raw(const DModel& m, int mat, const int16_t* xq, int n, int32_t* out, cudaStream_t st);
// Cold-L2 preparation between timed launches: writes `bytes` (more than L2)
// of `buf`, then reads them back, so the lines the write left dirty are
// written back before the timed launch instead of during it.
void l2_flush(void* buf, size_t bytes, int val, cudaStream_t st);
int kernel_launches_per_step(const DModel& m, const State& s, int n);
size_t batch_record_bytes(const DModel& m);
size_t batch_hidden_bytes(const DModel& m);
bool batch_path_fits(const DModel& m, int slots);
// Shape limits of the kernels (checked at upload / session creation).
bool attention_fits(int seq, int head_dim, int kv_bits, int kv_dim, int group);
int matvec_max_chunks();
int max_input_cols();

// Accessors engine.cu gives the library's other translation units.
}  // namespace vc4
struct vc4_model;
struct vc4_session;
namespace vc4 {
int set_error(int code, const char* msg);
const DModel& model_of(const vc4_model* m);
// What the per-op calls (ops.cu) need of a session.
struct SessionView {
    State* st;
    const DModel* m;
    cudaStream_t stream;
    int slots;
    void** ops;                      // the per-op buffers (owned through free_op_buffers)
    long long* launches;
    long long* syncs;
};
SessionView session_view(vc4_session* s);
// Before a write at `pos` of `slot`: a slot whose shared prefix covers pos gets
// its own copy of the prefix rows first (copy on write).
int session_unshare(vc4_session* s, int slot, int pos);
void free_op_buffers(void* ops);
int kernel_check(vc4_session* s);    // the kernels' self-check word (synchronises)
cudaStream_t model_stream(const vc4_model* m);
int lookup_matrix(const vc4_model* m, int which, int layer, int expert, int* idx);
}  // namespace vc4
