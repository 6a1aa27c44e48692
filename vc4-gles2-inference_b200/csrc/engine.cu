// engine.cu -- host side of the B200 decode engine and its C ABI.
//
// Upload (the reference's GPU::upload, gpu_upload.cpp:20-192) re-lays every
// quantised matrix into the 32-row interleaved layout described in
// vc4b200_internal.h.  A decode pass (Session::forward semantics,
// session.cpp:373-556) is 5 kernels per layer plus the logits and a finalize
// kernel; each distinct batch shape is captured once into a CUDA graph and
// replayed, so the host issues one graph launch per step.
#include "vc4b200_internal.h"
#include "../../include/vc4b200.h"

#include <sys/stat.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

using namespace vc4;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------

static thread_local std::string g_err;

static int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

#define CK(call)                                                                          \
    do {                                                                                  \
        cudaError_t e_ = (call);                                                          \
        if (e_ != cudaSuccess) return fail(VC4_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

extern "C" const char* vc4_last_error(void) { return g_err.c_str(); }

// ---------------------------------------------------------------------------
// handles
// ---------------------------------------------------------------------------

struct vc4_gpu {
    int device = 0;
    cudaStream_t stream = nullptr;
};

struct vc4_model {
    vc4_gpu* g = nullptr;
    DModel d;
};

// One decode pass's device arguments; a captured graph is keyed by them.
struct PassArgs {
    int n; const int* slots; int* tokens; int* pos; int* next; int advance; const int* forced;
    int prefill = 0;   // the entries are positions of one sequence: attention appends, then attends
    bool operator<(const PassArgs& o) const {
        return std::tie(n, slots, tokens, pos, next, advance, forced, prefill) <
               std::tie(o.n, o.slots, o.tokens, o.pos, o.next, o.advance, o.forced, o.prefill);
    }
};

struct vc4_session {
    vc4_model* m = nullptr;
    State st;
    int slots = 0;
    int *d_slot = nullptr, *d_tok = nullptr, *d_pos = nullptr, *d_next = nullptr;
    int* h_pin = nullptr;                     // pinned staging: slot, tok, pos, next, error word (5*slots + 16)
    int32_t* h_logits = nullptr;              // pinned logits staging (slots*vocab)
    std::map<PassArgs, cudaGraphExec_t> graphs;
    long long launches = 0, syncs = 0;
    cudaStream_t stream = nullptr;
    void* ops = nullptr;                      // buffers of the per-op calls (ops.cu), made on first use
    std::vector<int> plen;                    // host mirror of st.plen (shared-prefix rows per slot)
};

// ---------------------------------------------------------------------------
// upload: re-lay one matrix (or a column slice of it) into the device layout
// ---------------------------------------------------------------------------

namespace {

float row_epilogue_scale(const HMat& h, int r) {
    if (h.p16.empty()) return h.scale;
    const float a = (float)h.p16[r] * h.scale;          // (p16*ws)*(1/65536), shaders.cpp:339-372
    return a * (1.0f / 65536.0f);
}

std::string relay(const HMat& h, int c0, int c1, DMat& d, std::vector<void*>& allocs) {
    d = DMat();
    d.rows = h.rows; d.cols = c1 - c0; d.wtype = h.wtype;
    d.rblocks = (h.rows + kRowBlock - 1) / kRowBlock;
    const int R = d.rblocks * kRowBlock;
    auto dev = [&](const void* src, size_t bytes, void** dst) -> std::string {
        if (cudaMalloc(dst, bytes) != cudaSuccess) return "cudaMalloc failed for " + std::to_string(bytes) + " bytes";
        allocs.push_back(*dst);
        if (cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return "cudaMemcpy failed";
        return "";
    };
    std::vector<float> rs(R, 0.0f);
    for (int r = 0; r < h.rows; ++r) rs[r] = row_epilogue_scale(h, r);
    if (h.wtype == W_I16) {
        d.nchunks = 0;
        std::string e = dev(h.w16.data(), h.w16.size() * 2, (void**)&d.w16);
        if (e.empty()) e = dev(rs.data(), rs.size() * 4, (void**)&d.rscale);
        return e;
    }
    const int cpc = cols_per_chunk(h.wtype);
    const int ncols = c1 - c0;
    if (h.wtype == W_Q4 && (c0 % 32 || ncols % 32)) return "q4 slice is not group aligned";
    d.nchunks = (ncols + cpc - 1) / cpc;
    if (d.nchunks > matvec_max_chunks() || d.nchunks * cpc > max_input_cols())
        return "matrix too wide for the matvec kernel (" + std::to_string(ncols) + " columns)";
    const size_t nbody = (size_t)d.rblocks * d.nchunks * 32 * 16;
    std::vector<uint8_t> body(nbody, 0);
    std::vector<int32_t> q4p;
    if (h.wtype == W_Q4) q4p.assign((size_t)d.rblocks * d.nchunks * 32, 0);
    for (int r = 0; r < h.rows; ++r) {
        const int blk = r / 32, l = r % 32;
        for (int j = 0; j < d.nchunks; ++j) {
            uint8_t* out = body.data() + (((size_t)blk * d.nchunks + j) * 32 + l) * 16;
            if (h.wtype == W_Q8) {
                for (int k = 0; k < 16; ++k) {
                    const int c = j * 16 + k;
                    out[k] = c < ncols ? (uint8_t)h.lev[(size_t)r * h.cols + c0 + c] : 0;
                }
            } else if (h.wtype == W_T3) {
                for (int q = 0; q < 4; ++q) {
                    uint32_t word = 0;
                    for (int b = 0; b < 4; ++b)
                        for (int i = 0; i < 4; ++i) {
                            const int c = j * 64 + q * 16 + 4 * i + b;
                            const int e = c < ncols ? h.lev[(size_t)r * h.cols + c0 + c] + 1 : 1;
                            word |= (uint32_t)e << (8 * b + 2 * i);
                        }
                    memcpy(out + 4 * q, &word, 4);
                }
            } else {   // q4: chunk j is group c0/32 + j
                const int g = c0 / 32 + j;
                for (int q = 0; q < 4; ++q)
                    for (int b = 0; b < 4; ++b) {
                        const size_t base = (size_t)r * h.cols + (size_t)g * 32 + q * 8;
                        out[4 * q + b] = (uint8_t)(h.nib[base + b] | (h.nib[base + 4 + b] << 4));
                    }
                const size_t gi = (size_t)r * h.groups() + g;
                q4p[((size_t)blk * d.nchunks + j) * 32 + l] =
                    (int32_t)((uint32_t)(uint16_t)h.s16[gi] | ((uint32_t)(uint16_t)h.m16[gi] << 16));
            }
        }
    }
    std::string e = dev(body.data(), body.size(), (void**)&d.body);
    if (e.empty()) e = dev(rs.data(), rs.size() * 4, (void**)&d.rscale);
    if (e.empty() && !q4p.empty()) e = dev(q4p.data(), q4p.size() * 4, (void**)&d.q4p);
    if (e.empty() && (h.wtype == W_Q8 || h.wtype == W_T3)) {
        // row-major copy for the tensor-core matmat: row r's signed levels
        // (q8, or the ternary -1/0/+1) at r*K, K the padded column count
        const size_t K = (size_t)d.nchunks * cpc;
        std::vector<int8_t> rm((size_t)R * K, 0);
        for (int r = 0; r < h.rows; ++r)
            for (int c = 0; c < ncols; ++c) rm[(size_t)r * K + c] = h.lev[(size_t)r * h.cols + c0 + c];
        e = dev(rm.data(), rm.size(), (void**)&d.rm);
    }
    return e;
}

}  // namespace

namespace vc4 {

std::string upload_model(HModel&& h, DModel& d) {
    d.ffn_width = h.ffn_width();
    d.ffn_chunked = d.ffn_width > 2048;                       // model.cpp:217-277
    d.ffn_chunk = d.ffn_chunked ? (d.ffn_width + 1) / 2 : d.ffn_width;
    // the FFN kernel's 32-row tiles of the hidden vector must not straddle the w2 halves
    if (d.ffn_chunked && d.ffn_chunk % 32) return "chunked FFN with a chunk width that is not a multiple of 32";
    std::vector<void*>& al = d.allocs;
    auto add = [&](const HMat& m, int c0, int c1) -> int {
        DMat x;
        std::string e = relay(m, c0, c1, x, al);
        if (!e.empty()) throw std::runtime_error(e);
        d.mats.push_back(x);
        d.weight_bytes += x.bytes();
        return (int)d.mats.size() - 1;
    };
    const int L = h.layers, E = h.experts, F = d.ffn_width, c = d.ffn_chunk;
    try {
        // logits: the tiles stacked into one vocab-row matrix with per-row scales
        HMat lg;
        lg.rows = h.vocab; lg.cols = h.dim; lg.wtype = W_Q8;
        lg.lev.reserve((size_t)h.vocab * h.dim);
        std::vector<float> rsc;
        for (const HMat& t : h.tiles) {
            lg.lev.insert(lg.lev.end(), t.lev.begin(), t.lev.end());
            for (int r = 0; r < t.rows; ++r) rsc.push_back(row_epilogue_scale(t, r));
        }
        // The stacked matrix carries its scales directly: encode them as a
        // plane-free matrix whose per-row scale is patched after the relay.
        lg.scale = 1.0f;
        d.logits_mat = add(lg, 0, h.dim);
        {
            std::vector<float> rs((size_t)d.mats[d.logits_mat].rblocks * 32, 0.0f);
            for (int r = 0; r < h.vocab; ++r) rs[r] = rsc[r];
            cudaMemcpy(d.mats[d.logits_mat].rscale, rs.data(), rs.size() * 4, cudaMemcpyHostToDevice);
        }
        if (h.head_dedup) {
            d.emb_mat = d.logits_mat;                          // the head is the embedding
        } else {
            HMat em;
            em.rows = h.vocab; em.cols = h.dim; em.wtype = W_Q8; em.scale = 1.0f; em.lev = h.emb;
            d.emb_mat = add(em, 0, h.dim);
            d.weight_bytes -= d.mats[d.emb_mat].bytes();         // a lookup reads one row
        }
        for (int l = 0; l < L; ++l) {
            d.qkv.push_back(add(h.qkv[l], 0, h.dim));
            d.wo.push_back(add(h.wo[l], 0, h.dim));
            if (E) {
                d.router.push_back(add(h.router[l], 0, h.dim));
                for (int e = 0; e < E; ++e) {
                    const HMat* x = &h.moe[((size_t)l * E + e) * 3];
                    d.e_w1.push_back(add(x[0], 0, h.dim));
                    d.e_w3.push_back(add(x[1], 0, h.dim));
                    d.e_w2a.push_back(add(x[2], 0, c));
                    if (d.ffn_chunked) d.e_w2b.push_back(add(x[2], c, F));
                    else { d.mats.push_back(DMat()); d.e_w2b.push_back((int)d.mats.size() - 1); }
                }
                d.w1.push_back(-1); d.w3.push_back(-1); d.w2a.push_back(-1); d.w2b.push_back(-1);
            } else {
                d.router.push_back(-1);
                d.w1.push_back(add(h.w1[l], 0, h.dim));
                d.w3.push_back(add(h.w3[l], 0, h.dim));
                d.w2a.push_back(add(h.w2[l], 0, c));
                d.w2b.push_back(d.ffn_chunked ? add(h.w2[l], c, F) : -1);
            }
        }
    } catch (const std::exception& ex) {
        return ex.what();
    }
    d.wtype = h.wo[0].wtype;
    auto upf = [&](const std::vector<float>& v, float** dst) -> bool {
        if (v.empty()) { *dst = nullptr; return true; }
        if (cudaMalloc((void**)dst, v.size() * 4) != cudaSuccess) return false;
        al.push_back(*dst);
        return cudaMemcpy(*dst, v.data(), v.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    };
    if (!upf(h.emb_scale, &d.d_emb_scale) || !upf(h.rms_att, &d.d_rms_att) || !upf(h.rms_ffn, &d.d_rms_ffn) ||
        !upf(h.rms_final, &d.d_rms_final) || !upf(h.q_norm, &d.d_q_norm) || !upf(h.k_norm, &d.d_k_norm))
        return "device allocation of the norm vectors failed";
    if (cudaMalloc((void**)&d.d_mats, sizeof(DMat) * d.mats.size()) != cudaSuccess) return "cudaMalloc(mats)";
    al.push_back(d.d_mats);
    cudaMemcpy(d.d_mats, d.mats.data(), sizeof(DMat) * d.mats.size(), cudaMemcpyHostToDevice);
    // drop the host copies of the weights: the device holds them now
    h.emb.clear(); h.emb.shrink_to_fit();
    h.qkv.clear(); h.wo.clear(); h.w1.clear(); h.w3.clear(); h.w2.clear();
    h.moe.clear(); h.tiles.clear(); h.router.clear();
    d.h = std::move(h);
    return "";
}

void free_model(DModel& d) {
    for (void* p : d.allocs) cudaFree(p);
    d.allocs.clear();
    d.mats.clear();
}

}  // namespace vc4

// ---------------------------------------------------------------------------
// session
// ---------------------------------------------------------------------------

namespace {

void enqueue_pass(vc4_session* s, const PassArgs& a, cudaStream_t st) {
    const DModel& m = s->m->d;
    Batch b;
    b.n = a.n; b.slot = a.slots; b.token = a.tokens; b.pos = a.pos;
    for (int l = 0; l < m.h.layers; ++l) {
        launch_embed_qkv(m, s->st, b, l, st);
        if (a.prefill) {
            launch_attention(m, s->st, b, l, st, 1);   // every position's K/V row first,
            launch_attention(m, s->st, b, l, st, 2);   // then attention over the whole prefix
        } else {
            launch_attention(m, s->st, b, l, st);
        }
        launch_wo(m, s->st, b, l, st);
        launch_ffn_gate(m, s->st, b, l, st);   // gate/up, SwiGLU and the w2 partial sums
    }
    launch_logits(m, s->st, b, a.next, a.tokens, a.pos, a.advance, a.forced, st);
}

}  // namespace

// The kernels' self-check word (shared-memory reservation), read after the
// eager first run of every pass shape.
static int check_kernel_word(vc4_session* s) {
    int w = 0;
    CK(cudaStreamSynchronize(s->stream));
    CK(cudaMemcpy(&w, s->st.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (w > 0) return fail(VC4_ECUDA, "a kernel found its shared-memory reservation too small (needs " + std::to_string(w) + " bytes)");
    if (w == -2) return fail(VC4_ECUDA, "a kernel's bulk copy did not complete within its time limit");
    if (w == -3) return fail(VC4_ECUDA, "a tensor-core matmat was launched with a copy ring or box plan it cannot run");
    if (w == -5)
        return fail(VC4_ESTATE, "a decode step appended at a position the slot's shared prefix serves (those rows are "
                                "read-only; the row was not written)");
    if (w == -4)
        return fail(VC4_ERANGE, "an FFN hidden value reached 64 or more: the w2 input scale of the host FFN would "
                                "round its input, which this engine does not compute (the session's results are void)");
    if (w) return fail(VC4_ECUDA, "kernel self-check failed (code " + std::to_string(w) + ")");
    return VC4_OK;
}

// One decode pass: the first call of a shape runs eagerly (kernel attributes
// are set, errors surface) and captures a graph; later calls replay it.
static int run_pass(vc4_session* s, const PassArgs& a) {
    if (a.n <= 0 || a.n > s->slots) return fail(VC4_EINVAL, "batch size out of range");
    auto& tab = s->graphs;
    auto it = tab.find(a);
    if (it != tab.end()) {
        CK(cudaGraphLaunch(it->second, s->stream));
    } else {
        enqueue_pass(s, a, s->stream);
        CK(cudaGetLastError());
        if (int e = check_kernel_word(s)) return e;
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
        enqueue_pass(s, a, s->stream);
        CK(cudaStreamEndCapture(s->stream, &g));
        cudaGraphExec_t ex = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return fail(VC4_ECUDA, std::string("cudaGraphInstantiate: ") + cudaGetErrorString(e));
        tab[a] = ex;
    }
    s->launches += kernel_launches_per_step(s->m->d, s->st, a.n) + (a.prefill ? s->m->d.h.layers : 0);
    return VC4_OK;
}

extern "C" {

int vc4_gpu_create(int device, vc4_gpu** out) {
    *out = nullptr;
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(VC4_EINVAL, "no CUDA device " + std::to_string(device));
    CK(cudaSetDevice(device));
    vc4_gpu* g = new vc4_gpu();
    g->device = device;
    if (cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete g;
        return fail(VC4_ECUDA, "cudaStreamCreate failed");
    }
    *out = g;
    return VC4_OK;
}

void vc4_gpu_destroy(vc4_gpu* g) {
    if (!g) return;
    cudaSetDevice(g->device);
    cudaStreamDestroy(g->stream);
    delete g;
}

int vc4_gpu_sync(vc4_gpu* g) {
    CK(cudaSetDevice(g->device));
    CK(cudaStreamSynchronize(g->stream));
    return VC4_OK;
}

static int finish_load(vc4_gpu* g, HModel&& h, vc4_model** out) {
    CK(cudaSetDevice(g->device));
    vc4_model* m = new vc4_model();
    m->g = g;
    m->d.device = g->device;
    cudaDeviceGetAttribute(&m->d.num_sms, cudaDevAttrMultiProcessorCount, g->device);
    const std::string e = upload_model(std::move(h), m->d);
    if (!e.empty()) {
        free_model(m->d);
        delete m;
        return fail(VC4_ECUDA, "upload: " + e);
    }
    *out = m;
    return VC4_OK;
}

int vc4_model_load(vc4_gpu* g, const char* path, vc4_model** out) {
    *out = nullptr;
    HModel h;
    const std::string e = load_mmcf(path, h);
    if (!e.empty()) return fail(e.rfind("cannot", 0) == 0 || e.rfind("short", 0) == 0 ? VC4_EIO : VC4_EFORMAT, e);
    return finish_load(g, std::move(h), out);
}

int vc4_model_load_bytes(vc4_gpu* g, const void* data, size_t size, vc4_model** out) {
    *out = nullptr;
    HModel h;
    const std::string e = load_mmcf_bytes((const uint8_t*)data, size, h);
    if (!e.empty()) return fail(VC4_EFORMAT, e);
    h.source_size = size;
    return finish_load(g, std::move(h), out);
}

int vc4_model_info_get(const vc4_model* m, vc4_model_info* o) {
    const HModel& h = m->d.h;
    memset(o, 0, sizeof(*o));
    o->dim = h.dim; o->hidden = h.hidden; o->layers = h.layers; o->heads = h.heads; o->kv_heads = h.kv_heads;
    o->vocab = h.vocab; o->seq = h.seq; o->head_dim = h.head_dim; o->kv_dim = h.kv_dim;
    o->experts = h.experts; o->moe_hidden = h.moe_hidden; o->ffn_width = m->d.ffn_width;
    o->ffn_chunked = m->d.ffn_chunked; o->ffn_chunk = m->d.ffn_chunk; o->qk_norm = h.qk_norm;
    o->rope_half = h.rope_half; o->head_dedup = h.head_dedup; o->wtype = m->d.wtype;
    o->rope_theta = h.rope_theta; o->rms_eps = h.rms_eps; o->weight_bytes = m->d.weight_bytes;
    o->source_size = h.source_size; o->source_mtime = h.source_mtime;
    return VC4_OK;
}

int vc4_model_probe(const char* path, vc4_model_info* o) {
    HModel h;
    const std::string e = load_mmcf(path, h);
    if (!e.empty()) return fail(e.rfind("cannot", 0) == 0 || e.rfind("short", 0) == 0 ? VC4_EIO : VC4_EFORMAT, e);
    memset(o, 0, sizeof(*o));
    o->dim = h.dim; o->hidden = h.hidden; o->layers = h.layers; o->heads = h.heads; o->kv_heads = h.kv_heads;
    o->vocab = h.vocab; o->seq = h.seq; o->head_dim = h.head_dim; o->kv_dim = h.kv_dim;
    o->experts = h.experts; o->moe_hidden = h.moe_hidden; o->ffn_width = h.ffn_width();
    o->ffn_chunked = o->ffn_width > 2048; o->ffn_chunk = o->ffn_chunked ? (o->ffn_width + 1) / 2 : o->ffn_width;
    o->qk_norm = h.qk_norm; o->rope_half = h.rope_half; o->head_dedup = h.head_dedup; o->wtype = h.wo[0].wtype;
    o->rope_theta = h.rope_theta; o->rms_eps = h.rms_eps;
    o->source_size = h.source_size; o->source_mtime = h.source_mtime;
    return VC4_OK;
}

void vc4_model_free(vc4_model* m) {
    if (!m) return;
    cudaSetDevice(m->d.device);
    free_model(m->d);
    delete m;
}

void vc4_rope_tables(float theta, int head_dim, int seq, const float* factors, float* cos_out, float* sin_out) {
    // session.cpp:188-202
    const int half = head_dim / 2;
    for (int p = 0; p < seq; ++p)
        for (int i = 0; i < half; ++i) {
            float freq = 1.0f / powf(theta, (2.0f * i) / head_dim);
            if (factors) freq /= factors[i];
            const float a = p * freq;
            cos_out[(size_t)p * half + i] = cosf(a);
            sin_out[(size_t)p * half + i] = sinf(a);
        }
}

int vc4_session_create(vc4_model* m, int slots, int seq, int kv_bits, const float* rcos, const float* rsin,
                       vc4_session** out) {
    *out = nullptr;
    const HModel& h = m->d.h;
    if (slots <= 0) return fail(VC4_EINVAL, "slots must be positive");
    if (seq <= 0) seq = h.seq;
    if (kv_bits != 16 && kv_bits != 8) return fail(VC4_EINVAL, "kv_bits must be 16 (q16) or 8 (q8)");
    if (kv_bits == 8 && (h.kv_dim % 4 || h.head_dim % 4)) return fail(VC4_EINVAL, "q8 KV needs kv_dim and head_dim divisible by 4");
    if (h.heads / h.kv_heads > 8 || h.head_dim > 128) return fail(VC4_EINVAL, "attention group above 8 or head_dim above 128");
    if (h.dim > max_input_cols() || m->d.ffn_width > max_input_cols())
        return fail(VC4_EINVAL, "model width beyond the kernels' staging limit");
    if (!attention_fits(seq, h.head_dim, kv_bits, h.kv_dim, h.heads / h.kv_heads))
        return fail(VC4_EINVAL, "sequence length / head shape beyond the attention kernel's staging limits");
    CK(cudaSetDevice(m->d.device));
    vc4_session* s = new vc4_session();
    s->m = m; s->slots = slots; s->stream = m->g->stream;
    State& st = s->st;
    st.kv_bits = kv_bits; st.seq = seq; st.slots = slots;
    st.row_bytes = kv_bits == 16 ? h.kv_dim * 4 : h.kv_dim * 2;           // gpu_attn.cpp:89-92
    const size_t D = h.dim, Q = h.dim + 2 * h.kv_dim, F = m->d.ffn_width, V = h.vocab, L = h.layers;
    auto alloc = [&](void** p, size_t bytes) -> bool {
        if (cudaMalloc(p, bytes) != cudaSuccess) return false;
        return cudaMemset(*p, 0, bytes) == cudaSuccess;
    };
    bool ok = alloc((void**)&st.x, slots * D * 2) && alloc((void**)&st.x1, slots * D * 2) &&
              alloc((void**)&st.qkv, slots * Q * 4) && alloc((void**)&st.att, slots * D * 2) &&
              alloc((void**)&st.h, slots * F * 2) && alloc((void**)&st.logits, slots * V * 4) &&
              alloc((void**)&st.best, slots * 8) && alloc((void**)&st.next, slots * 4) &&
              alloc((void**)&st.route, slots * L * 4) &&
              alloc((void**)&st.kv, (size_t)slots * L * seq * st.row_bytes) &&
              alloc((void**)&st.rope_cos, (size_t)seq * (h.head_dim / 2) * 4) &&
              alloc((void**)&st.rope_sin, (size_t)seq * (h.head_dim / 2) * 4) &&
              alloc((void**)&s->d_slot, (size_t)(3 * slots + 1) * 4) && alloc((void**)&s->d_next, (size_t)slots * 4) &&
              alloc((void**)&s->d_pos, (size_t)seq * 4 + 16) && alloc((void**)&st.done, 16) && alloc((void**)&st.err, 16) &&
              alloc((void**)&st.sdown, (size_t)L * slots * 2 * D * 8) &&
              alloc((void**)&st.hmax, (size_t)L * slots * 2 * 4) &&
              alloc((void**)&st.plen, (size_t)slots * 4) &&
              alloc((void**)&st.xrec, (size_t)slots * batch_record_bytes(m->d)) &&
              alloc((void**)&st.hrec, (size_t)slots * batch_hidden_bytes(m->d));
    st.batch_ok = batch_path_fits(m->d, slots) ? 1 : 0;
    s->plen.assign(slots, 0);
    if (!ok) { vc4_session_destroy(s); return fail(VC4_ECUDA, "session allocation failed (slots*seq too large?)"); }
    s->d_tok = s->d_slot + slots;
    if (cudaMallocHost((void**)&s->h_pin, (size_t)(5 * slots + 16) * 4) != cudaSuccess ||
        cudaMallocHost((void**)&s->h_logits, (size_t)slots * V * 4) != cudaSuccess) {
        vc4_session_destroy(s);
        return fail(VC4_ECUDA, "pinned staging allocation failed");
    }
    std::vector<float> c((size_t)seq * (h.head_dim / 2)), sn(c.size());
    if (rcos && rsin) {
        memcpy(c.data(), rcos, c.size() * 4);
        memcpy(sn.data(), rsin, sn.size() * 4);
    } else {
        vc4_rope_tables(h.rope_theta, h.head_dim, seq, h.rope_factors.empty() ? nullptr : h.rope_factors.data(),
                        c.data(), sn.data());
    }
    if (cudaMemcpy(st.rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(st.rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        vc4_session_destroy(s);
        return fail(VC4_ECUDA, "rope table upload failed");
    }
    *out = s;
    return VC4_OK;
}

void vc4_session_destroy(vc4_session* s) {
    if (!s) return;
    cudaSetDevice(s->m->d.device);
    cudaStreamSynchronize(s->stream);
    free_op_buffers(s->ops);
    s->ops = nullptr;
    for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second);
    s->graphs.clear();
    State& st = s->st;
    for (void* p : {(void*)st.x, (void*)st.x1, (void*)st.qkv, (void*)st.att, (void*)st.h, (void*)st.logits,
                    (void*)st.best, (void*)st.next, (void*)st.route, (void*)st.kv, (void*)st.rope_cos,
                    (void*)st.rope_sin, (void*)s->d_slot, (void*)s->d_next, (void*)s->d_pos, (void*)st.done, (void*)st.err,
                    (void*)st.sdown, (void*)st.hmax, (void*)st.xrec, (void*)st.hrec, (void*)st.plen, (void*)st.pkv})
        if (p) cudaFree(p);
    if (s->h_pin) cudaFreeHost(s->h_pin);
    if (s->h_logits) cudaFreeHost(s->h_logits);
    delete s;
}

void* vc4_session_stream(vc4_session* s) { return (void*)s->stream; }

int vc4_session_check(vc4_session* s) {
    CK(cudaSetDevice(s->m->d.device));
    return check_kernel_word(s);
}

static int check_slot_pos(const vc4_session* s, int slot, int pos) {
    if (slot < 0 || slot >= s->slots) return fail(VC4_EINVAL, "slot out of range");
    if (pos < 0 || pos >= s->st.seq) return fail(VC4_EINVAL, "position out of range");
    return VC4_OK;
}

// Host-array batch step: stage (slot, token, pos) through pinned memory, run
// the pass, read the greedy tokens and optionally the logits back.
static int host_step(vc4_session* s, int n, const int* slots, const int* tokens, const int* pos, int* next,
                     float* logits) {
    if (n <= 0 || n > s->slots) return fail(VC4_EINVAL, "batch size out of range");
    const int V = s->m->d.h.vocab;
    std::vector<char> seen(s->slots, 0);
    for (int i = 0; i < n; ++i) {
        if (int e = check_slot_pos(s, slots[i], pos[i])) return e;
        if (tokens[i] < 0 || tokens[i] >= V) return fail(VC4_EINVAL, "token id out of range");
        if (seen[slots[i]]++) return fail(VC4_EINVAL, "a slot appears twice in one batch");
    }
    CK(cudaSetDevice(s->m->d.device));
    for (int i = 0; i < n; ++i)
        if (int e = session_unshare(s, slots[i], pos[i])) return e;
    int* hp = s->h_pin;
    for (int i = 0; i < n; ++i) { hp[i] = slots[i]; hp[n + i] = tokens[i]; hp[2 * n + i] = pos[i]; }
    int* dcall = s->d_slot;   // [slots | tokens | pos] for this n
    CK(cudaMemcpyAsync(dcall, hp, sizeof(int) * 3 * n, cudaMemcpyHostToDevice, s->stream));
    PassArgs a{n, dcall, dcall + n, dcall + 2 * n, s->d_next, 0, nullptr};
    if (int e = run_pass(s, a)) return e;
    CK(cudaMemcpyAsync(hp + 3 * n, s->d_next, sizeof(int) * n, cudaMemcpyDeviceToHost, s->stream));
    CK(cudaMemcpyAsync(hp + 4 * n, s->st.err, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
    if (logits)
        for (int i = 0; i < n; ++i)
            CK(cudaMemcpyAsync(s->h_logits + (size_t)i * V, s->st.logits + (size_t)i * V, sizeof(int32_t) * V,
                               cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    s->syncs++;
    if (hp[4 * n]) return check_kernel_word(s);
    if (next) for (int i = 0; i < n; ++i) next[i] = hp[3 * n + i];
    if (logits)
        for (size_t i = 0; i < (size_t)n * V; ++i) logits[i] = (float)s->h_logits[i] / 256.0f;
    return VC4_OK;
}

int vc4_step(vc4_session* s, int slot, int token, int pos, float* logits) {
    return host_step(s, 1, &slot, &token, &pos, nullptr, logits);
}

int vc4_step_greedy(vc4_session* s, int slot, int token, int pos, int* next_token) {
    return host_step(s, 1, &slot, &token, &pos, next_token, nullptr);
}

int vc4_step_batch(vc4_session* s, int n, const int* slots, const int* tokens, const int* pos, int* next_tokens,
                   float* logits) {
    return host_step(s, n, slots, tokens, pos, next_tokens, logits);
}

int vc4_step_batch_device(vc4_session* s, int n, const int* d_slots, int* d_tokens, int* d_pos, int* d_next,
                          int advance) {
    CK(cudaSetDevice(s->m->d.device));
    PassArgs a{n, d_slots, d_tokens, d_pos, d_next, advance ? 1 : 0, nullptr};
    return run_pass(s, a);
}

int vc4_prefill(vc4_session* s, int slot, const int* tokens, int n, int pos0, float* logits) {
    if (n <= 0) return fail(VC4_EINVAL, "empty prompt");
    if (int e = check_slot_pos(s, slot, pos0)) return e;
    if (pos0 + n > s->st.seq) return fail(VC4_EINVAL, "prompt runs past the sequence length");
    const int V = s->m->d.h.vocab;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= V) return fail(VC4_EINVAL, "token id out of range");
    CK(cudaSetDevice(s->m->d.device));
    if (int e = session_unshare(s, slot, pos0)) return e;
    // prompt[p] at absolute position p; the pass replays with `forced` so each
    // replay moves to the next prompt token on the device.
    std::vector<int> prompt(s->st.seq + 1, 0);
    for (int i = 0; i < n; ++i) prompt[pos0 + i] = tokens[i];
    int* dprompt = s->d_pos;
    int* hp = s->h_pin;
    CK(cudaMemcpyAsync(dprompt, prompt.data(), sizeof(int) * s->st.seq, cudaMemcpyHostToDevice, s->stream));
    int* dcall = s->d_slot + 3 * s->slots - 3;   // a private 3-int call block at the end
    hp[0] = slot; hp[1] = tokens[0]; hp[2] = pos0;
    CK(cudaMemcpyAsync(dcall, hp, sizeof(int) * 3, cudaMemcpyHostToDevice, s->stream));
    CK(cudaStreamSynchronize(s->stream));   // the staging buffers are reused below
    PassArgs a{1, dcall, dcall + 1, dcall + 2, s->d_next, 1, dprompt};
    for (int i = 0; i < n; ++i)
        if (int e = run_pass(s, a)) return e;
    if (logits) CK(cudaMemcpyAsync(s->h_logits, s->st.logits, sizeof(int32_t) * V,
                                   cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    s->syncs++;
    if (logits) for (int i = 0; i < V; ++i) logits[i] = (float)s->h_logits[i] / 256.0f;
    return VC4_OK;
}

// Batched prefill: up to `slots` positions of the prompt per pass, as one
// batch of the many-sequence path (tensor-core matmats for q8 and t3) whose
// entries are (slot, prompt[i], pos0 + i).  Every sum of the pass is exact,
// so each position's results, and the K/V rows it appends, are the serial
// loop's bit for bit.  A chunk too small for the many-sequence kernels runs
// through the serial loop.
constexpr int kPrefillBatchMin = 16;

// The batched prefill; with `all` set, every position's logits go to
// all[i*vocab ..] (positions of a serial tail are stepped one at a time).
static int prefill_batched(vc4_session* s, int slot, const int* tokens, int n, int pos0, float* logits, float* all) {
    if (n <= 0) return fail(VC4_EINVAL, "empty prompt");
    if (int e = check_slot_pos(s, slot, pos0)) return e;
    if (pos0 + n > s->st.seq) return fail(VC4_EINVAL, "prompt runs past the sequence length");
    const DModel& m = s->m->d;
    const int V = m.h.vocab;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= V) return fail(VC4_EINVAL, "token id out of range");
    CK(cudaSetDevice(m.device));
    if (int e = session_unshare(s, slot, pos0)) return e;
    const bool can = s->st.batch_ok && prefill_attention_fits(m, s->st);
    int done = 0, last = 0;   // last: the batch size of the pass that held the final position (0: serial)
    while (done < n) {
        const int c = std::min(n - done, s->slots);
        if (!can || c < kPrefillBatchMin) {
            if (all) {
                for (int i = done; i < n; ++i) {
                    const int p = pos0 + i;
                    if (int e = host_step(s, 1, &slot, tokens + i, &p, nullptr, all + (size_t)i * V)) return e;
                }
                if (logits) memcpy(logits, all + (size_t)(n - 1) * V, sizeof(float) * V);
                return VC4_OK;
            }
            if (int e = vc4_prefill(s, slot, tokens + done, n - done, pos0 + done, nullptr)) return e;
            last = 0;
            break;
        }
        int* hp = s->h_pin;
        for (int i = 0; i < c; ++i) { hp[i] = slot; hp[c + i] = tokens[done + i]; hp[2 * c + i] = pos0 + done + i; }
        int* dcall = s->d_slot;   // [slots | tokens | pos] of this chunk
        CK(cudaMemcpyAsync(dcall, hp, sizeof(int) * 3 * c, cudaMemcpyHostToDevice, s->stream));
        PassArgs a{c, dcall, dcall + c, dcall + 2 * c, s->d_next, 0, nullptr, 1};
        if (int e = run_pass(s, a)) return e;
        if (all) {
            int32_t* hl = s->h_logits;   // pinned, slots x vocab
            CK(cudaMemcpyAsync(hl, s->st.logits, sizeof(int32_t) * (size_t)c * V, cudaMemcpyDeviceToHost, s->stream));
            CK(cudaStreamSynchronize(s->stream));
            if (int e = check_kernel_word(s)) return e;
            for (size_t i = 0; i < (size_t)c * V; ++i) all[(size_t)done * V + i] = (float)hl[i] / 256.0f;
        }
        CK(cudaStreamSynchronize(s->stream));   // the pinned staging is reused by the next chunk
        s->syncs++;
        done += c;
        last = c;
    }
    const int32_t* src = last ? s->st.logits + (size_t)(last - 1) * V : s->st.logits;
    if (logits) CK(cudaMemcpyAsync(s->h_logits, src, sizeof(int32_t) * V, cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    if (int e = check_kernel_word(s)) return e;
    if (logits) for (int i = 0; i < V; ++i) logits[i] = (float)s->h_logits[i] / 256.0f;
    return VC4_OK;
}

int vc4_prefill_batch(vc4_session* s, int slot, const int* tokens, int n, int pos0, float* logits) {
    return prefill_batched(s, slot, tokens, n, pos0, logits, nullptr);
}

int vc4_prefill_logits(vc4_session* s, int slot, const int* tokens, int n, int pos0, float* logits_all) {
    if (!logits_all) return fail(VC4_EINVAL, "logits_all is required");
    return prefill_batched(s, slot, tokens, n, pos0, nullptr, logits_all);
}

int vc4_kv_row_bytes(const vc4_session* s) { return s->st.row_bytes; }

static uint8_t* kv_rows_ptr(vc4_session* s, int slot, int layer) {
    return s->st.kv + ((size_t)slot * s->m->d.h.layers + layer) * s->st.seq * s->st.row_bytes;
}

static uint8_t* prefix_rows_ptr(vc4_session* s, int layer) {
    return s->st.pkv + (size_t)layer * s->st.pcap * s->st.row_bytes;
}

int vc4_kv_read_rows(vc4_session* s, int slot, int layer, int n, void* out) {
    if (slot < 0 || slot >= s->slots || layer < 0 || layer >= s->m->d.h.layers || n < 0 || n > s->st.seq)
        return fail(VC4_EINVAL, "kv read out of range");
    CK(cudaSetDevice(s->m->d.device));
    CK(cudaStreamSynchronize(s->stream));
    // rows below the slot's shared-prefix length come from the shared prefix
    const size_t rb = s->st.row_bytes, shared = (size_t)std::min(n, s->plen[slot]);
    if (shared) CK(cudaMemcpy(out, prefix_rows_ptr(s, layer), shared * rb, cudaMemcpyDeviceToHost));
    if ((size_t)n > shared)
        CK(cudaMemcpy((uint8_t*)out + shared * rb, kv_rows_ptr(s, slot, layer) + shared * rb, (n - shared) * rb,
                      cudaMemcpyDeviceToHost));
    s->syncs++;
    return VC4_OK;
}

int vc4_kv_write_rows(vc4_session* s, int slot, int layer, int n, const void* in) {
    if (slot < 0 || slot >= s->slots || layer < 0 || layer >= s->m->d.h.layers || n < 0 || n > s->st.seq)
        return fail(VC4_EINVAL, "kv write out of range");
    CK(cudaSetDevice(s->m->d.device));
    if (n > 0)
        if (int e = session_unshare(s, slot, 0)) return e;
    CK(cudaStreamSynchronize(s->stream));
    CK(cudaMemcpy(kv_rows_ptr(s, slot, layer), in, (size_t)n * s->st.row_bytes, cudaMemcpyHostToDevice));
    s->syncs++;
    return VC4_OK;
}

int vc4_counters(const vc4_session* s, long long* launches, long long* syncs) {
    if (launches) *launches = s->launches;
    if (syncs) *syncs = s->syncs;
    return VC4_OK;
}

int vc4_launches_per_step(const vc4_session* s, int n) { return kernel_launches_per_step(s->m->d, s->st, n); }

int vc4_matvec_s(vc4_model* m, int which, int layer, int expert, const float* x, float* out) {
    const DModel& d = m->d;
    const HModel& h = d.h;
    if (layer < 0 || layer >= h.layers) { if (which != 6) return fail(VC4_EINVAL, "layer out of range"); }
    int idx = -1;
    const bool moe = h.experts > 0;
    if (moe && (which == 2 || which == 3 || which == 4)) {
        if (expert < 0 || expert >= h.experts) return fail(VC4_EINVAL, "expert out of range");
        idx = d.e_w1[(size_t)layer * h.experts + expert] + (which == 2 ? 0 : which == 3 ? 1 : 2);
    } else {
        switch (which) {
            case 0: idx = d.qkv[layer]; break;
            case 1: idx = d.wo[layer]; break;
            case 2: idx = d.w1[layer]; break;
            case 3: idx = d.w3[layer]; break;
            case 4: idx = d.w2a[layer]; break;
            case 5: idx = moe ? d.router[layer] : -1; break;
            case 6: idx = d.logits_mat; break;
            default: break;
        }
    }
    if (idx < 0) return fail(VC4_EINVAL, "no such matrix");
    if (which == 4 && d.ffn_chunked) return fail(VC4_EINVAL, "w2 of a chunked FFN is two matrices; the CPU path never draws it whole");
    const DMat& W = d.mats[idx];
    const int n = W.cols;
    // matvec_s input scaling (gpu_conv.cpp:271-287)
    float mx = 0.0f;
    for (int i = 0; i < n; ++i) mx = std::max(mx, fabsf(x[i]));
    int k = 0;
    if (mx > 0.0f) { int e = 0; frexpf(mx, &e); k = 6 - e; }
    const float sk = ldexpf(1.0f, k);
    std::vector<int16_t> xq(n);
    for (int i = 0; i < n; ++i) {
        const long q = lrintf((x[i] * sk) * 256.0f);
        xq[i] = (int16_t)(q < -32768 ? -32768 : q > 32767 ? 32767 : q);
    }
    CK(cudaSetDevice(d.device));
    int16_t* dx = nullptr; int32_t* dy = nullptr;
    CK(cudaMalloc(&dx, n * 2));
    if (cudaMalloc(&dy, (size_t)W.rows * 4) != cudaSuccess) { cudaFree(dx); return fail(VC4_ECUDA, "cudaMalloc"); }
    std::vector<int32_t> v(W.rows);
    cudaError_t e = cudaMemcpyAsync(dx, xq.data(), n * 2, cudaMemcpyHostToDevice, m->g->stream);
    if (e == cudaSuccess) { launch_matvec_raw(d, idx, dx, n, dy, m->g->stream); e = cudaGetLastError(); }
    if (e == cudaSuccess) e = cudaMemcpyAsync(v.data(), dy, (size_t)W.rows * 4, cudaMemcpyDeviceToHost, m->g->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->g->stream);
    cudaFree(dx); cudaFree(dy);
    if (e != cudaSuccess) return fail(VC4_ECUDA, std::string("matvec_s: ") + cudaGetErrorString(e));
    const float inv = ldexpf(1.0f, -k);
    for (int r = 0; r < W.rows; ++r) out[r] = ((float)v[r] / 256.0f) * inv;
    return VC4_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// MMKV1 prefix cache (prefix_cache.cpp:25-207)
// ---------------------------------------------------------------------------

namespace {

uint32_t mmkv_flags(const vc4_session* s) {
    const HModel& h = s->m->d.h;
    return (h.qk_norm ? 1u : 0u) | (h.rope_half ? 2u : 0u) | (s->st.kv_bits == 16 ? 4u : 8u);
}
float kv_scale_of(const vc4_session* s) { return s->st.kv_bits == 16 ? 2048.0f : 16.0f; }
// A JSON string body: quote, backslash and control bytes escaped; other bytes
// (UTF-8 included) pass through.
std::string json_escape(const std::string& t) {
    std::string o;
    for (unsigned char c : t) {
        if (c == '"' || c == '\\') { o += '\\'; o += (char)c; }
        else if (c == '\n') o += "\\n";
        else if (c < 0x20) { char b[8]; snprintf(b, sizeof(b), "\\u%04x", c); o += b; }
        else o += (char)c;
    }
    return o;
}
uint32_t kv_width_of(const vc4_session* s) {
    const HModel& h = s->m->d.h;
    return (uint32_t)(s->st.kv_bits == 16 ? h.kv_dim : h.kv_dim / 2);
}

}  // namespace

extern "C" int vc4_save_prefix_cache(vc4_session* s, int slot, const char* path, const int* toks, int n,
                                     uint64_t system_fnv, uint64_t tools_fnv) {
    const HModel& h = s->m->d.h;
    if (slot < 0 || slot >= s->slots) return fail(VC4_EINVAL, "slot out of range");
    if (n <= 0 || n > s->st.seq) return fail(VC4_EINVAL, "token count out of range");
    FILE* f = fopen(path, "wb");
    if (!f) return fail(VC4_EIO, std::string("cannot write ") + path);
    std::vector<uint8_t> buf;
    auto put = [&](const void* p, size_t k) { const uint8_t* b = (const uint8_t*)p; buf.insert(buf.end(), b, b + k); };
    auto u32 = [&](uint32_t v) { put(&v, 4); };
    auto u64 = [&](uint64_t v) { put(&v, 8); };
    put("MMKV1\0\0\0", 8);
    u32(2);
    u64(h.source_size); u64(h.source_mtime);
    u32(h.dim); u32(h.hidden); u32(h.layers); u32(h.heads); u32(h.kv_heads); u32(h.vocab);
    u32((uint32_t)s->st.seq); u32(h.head_dim);
    put(&h.rope_theta, 4);
    u32(mmkv_flags(s));
    u32((uint32_t)n);
    u32(kv_width_of(s));
    const float ks = kv_scale_of(s);
    put(&ks, 4);
    for (int i = 0; i < n; ++i) u32((uint32_t)toks[i]);
    std::vector<uint8_t> rows((size_t)n * s->st.row_bytes);
    for (int l = 0; l < h.layers; ++l) {
        if (int e = vc4_kv_read_rows(s, slot, l, n, rows.data())) { fclose(f); return e; }
        buf.insert(buf.end(), rows.begin(), rows.end());
    }
    const bool ok = fwrite(buf.data(), 1, buf.size(), f) == buf.size();
    fclose(f);
    if (!ok) return fail(VC4_EIO, std::string("short write to ") + path);
    // The sidecar (prefix_cache.cpp:88-131): tokens_fnv64 is FNV-1a over the
    // little-endian u32 token ids.
    uint64_t fnv = 1469598103934665603ull;
    for (int i = 0; i < n; ++i)
        for (int b = 0; b < 4; ++b) { fnv ^= (uint8_t)((uint32_t)toks[i] >> (8 * b)); fnv *= 1099511628211ull; }
    FILE* j = fopen((std::string(path) + ".json").c_str(), "w");
    if (j) {
        fprintf(j,
                "{\"format\":\"mmkv\",\"version\":2,\"source_size\":%llu,\"source_mtime\":%llu,\"dim\":%d,"
                "\"hidden\":%d,\"layers\":%d,\"heads\":%d,\"kv_heads\":%d,\"vocab\":%d,\"seq\":%d,\"head_dim\":%d,"
                "\"rope_theta\":%.9g,\"kv_bits\":%d,\"act_fmt\":\"x16_2\",\"hybrid\":false,\"kv_scale\":%.9g,"
                "\"kv_width\":%u,\"vstep\":0,\"n_tokens\":%d,\"tokens_fnv64\":\"%016llx\",\"system_fnv64\":\"%016llx\","
                "\"tools_fnv64\":\"%016llx\",\"template\":\"%s\"}\n",
                (unsigned long long)h.source_size, (unsigned long long)h.source_mtime, h.dim, h.hidden, h.layers,
                h.heads, h.kv_heads, h.vocab, s->st.seq, h.head_dim, (double)h.rope_theta, s->st.kv_bits, (double)ks,
                kv_width_of(s), n, (unsigned long long)fnv, (unsigned long long)system_fnv,
                (unsigned long long)tools_fnv, json_escape(h.template_name).c_str());
        fclose(j);
    }
    return VC4_OK;
}

static int read_mmkv(vc4_session* s, const char* path, std::vector<uint32_t>& toks, std::vector<uint8_t>& all);

// Copy on write: a slot whose shared prefix covers `pos` gets the prefix rows
// in its own cache rows (every layer) and stops reading the shared copy.
int vc4::session_unshare(vc4_session* s, int slot, int pos) {
    const int pl = s->plen[slot];
    if (pl == 0 || pos >= pl) return VC4_OK;
    const size_t rb = s->st.row_bytes;
    for (int l = 0; l < s->m->d.h.layers; ++l)
        CK(cudaMemcpyAsync(kv_rows_ptr(s, slot, l), prefix_rows_ptr(s, l), (size_t)pl * rb, cudaMemcpyDeviceToDevice,
                           s->stream));
    CK(cudaMemsetAsync(s->st.plen + slot, 0, sizeof(int), s->stream));
    s->plen[slot] = 0;
    return VC4_OK;
}

extern "C" int vc4_load_prefix_cache_shared(vc4_session* s, const char* path, const int* slots, int count,
                                            int* toks_out, int cap, int* n_out) {
    const HModel& h = s->m->d.h;
    if (count <= 0 || count > s->slots) return fail(VC4_EINVAL, "slot count out of range");
    std::vector<char> listed(s->slots, 0);
    for (int i = 0; i < count; ++i) {
        if (slots[i] < 0 || slots[i] >= s->slots) return fail(VC4_EINVAL, "slot out of range");
        if (listed[slots[i]]++) return fail(VC4_EINVAL, "a slot appears twice");
    }
    std::vector<uint32_t> toks;
    std::vector<uint8_t> rows;
    if (int e = read_mmkv(s, path, toks, rows)) return e;
    const int n = (int)toks.size();
    if (n > cap) return fail(VC4_EINVAL, "token buffer too small for the cache");
    CK(cudaSetDevice(s->m->d.device));
    // slots still reading the previous shared prefix keep it as their own rows
    for (int i = 0; i < s->slots; ++i)
        if (s->plen[i] && !listed[i])
            if (int e = session_unshare(s, i, 0)) return e;
    CK(cudaStreamSynchronize(s->stream));
    if (s->st.pcap < n) {
        // the kernels of captured passes hold the State by value: drop them
        for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second);
        s->graphs.clear();
        if (s->st.pkv) cudaFree(s->st.pkv);
        s->st.pkv = nullptr;
        s->st.pcap = 0;
        CK(cudaMalloc((void**)&s->st.pkv, (size_t)h.layers * s->st.seq * s->st.row_bytes));
        s->st.pcap = s->st.seq;
    }
    const size_t lb = (size_t)n * s->st.row_bytes;
    for (int l = 0; l < h.layers; ++l)
        CK(cudaMemcpy(prefix_rows_ptr(s, l), rows.data() + l * lb, lb, cudaMemcpyHostToDevice));
    std::vector<int> pl(s->plen);
    for (int i = 0; i < count; ++i) pl[slots[i]] = n;
    CK(cudaMemcpy(s->st.plen, pl.data(), sizeof(int) * s->slots, cudaMemcpyHostToDevice));
    s->plen = pl;
    for (int i = 0; i < n; ++i) toks_out[i] = (int)toks[i];
    *n_out = n;
    return VC4_OK;
}

extern "C" int vc4_build_prefix_cache(vc4_session* s, int slot, const int* toks, int n, const char* path,
                                      uint64_t system_fnv, uint64_t tools_fnv) {
    // prefix_build.cpp:66-83: refuse an empty or too long prompt, prefill it
    // from position 0 with the serial loop, then write the file and sidecar
    if (n <= 0 || n > s->st.seq) return fail(VC4_EINVAL, "cache prompt empty or too long (" + std::to_string(n) + ")");
    if (int e = vc4_prefill(s, slot, toks, n, 0, nullptr)) return e;
    return vc4_save_prefix_cache(s, slot, path, toks, n, system_fnv, tools_fnv);
}

// Read and validate an MMKV1 file (prefix_cache.cpp:135-207): the token list
// and every layer's rows, layer after layer.
static int read_mmkv(vc4_session* s, const char* path, std::vector<uint32_t>& toks, std::vector<uint8_t>& all) {
    const HModel& h = s->m->d.h;
    FILE* f = fopen(path, "rb");
    if (!f) return fail(VC4_EIO, std::string("cannot read ") + path);
    auto rd = [&](void* p, size_t k) { return fread(p, 1, k, f) == k; };
    char magic[8] = {};
    uint32_t version = 0, dim = 0, hidden = 0, layers = 0, heads = 0, kv_heads = 0, vocab = 0, seq = 0, hd = 0;
    uint32_t flags = 0, n = 0, width = 0, vsw = 0;
    uint64_t size = 0, mtime = 0;
    float theta = 0, ks = 0;
    bool ok = rd(magic, 8) && memcmp(magic, "MMKV1", 5) == 0 && rd(&version, 4) && rd(&size, 8) && rd(&mtime, 8) &&
              rd(&dim, 4) && rd(&hidden, 4) && rd(&layers, 4) && rd(&heads, 4) && rd(&kv_heads, 4) && rd(&vocab, 4) &&
              rd(&seq, 4) && rd(&hd, 4) && rd(&theta, 4) && rd(&flags, 4) && rd(&n, 4) && rd(&width, 4);
    if (ok && version >= 3) ok = rd(&vsw, 4);
    ok = ok && rd(&ks, 4);
    const float want_ks = kv_scale_of(s);
    if (!ok || (version != 2 && version != 3) || dim != (uint32_t)h.dim || hidden != (uint32_t)h.hidden ||
        layers != (uint32_t)h.layers || heads != (uint32_t)h.heads || kv_heads != (uint32_t)h.kv_heads ||
        vocab != (uint32_t)h.vocab || seq != (uint32_t)s->st.seq || hd != (uint32_t)h.head_dim ||
        size != h.source_size || mtime != h.source_mtime || theta != h.rope_theta || width != kv_width_of(s) ||
        vsw != 0 || n == 0 || n > (uint32_t)s->st.seq || flags != mmkv_flags(s) || memcmp(&ks, &want_ks, 4) != 0) {
        fclose(f);
        return fail(VC4_ESTATE, "prefix cache does not match this model, sequence length or KV axis");
    }
    toks.assign(n, 0);
    all.assign((size_t)h.layers * n * s->st.row_bytes, 0);
    const bool got = rd(toks.data(), 4 * (size_t)n) && rd(all.data(), all.size());
    fclose(f);
    if (!got) return fail(VC4_EIO, "truncated prefix cache");
    return VC4_OK;
}

extern "C" int vc4_load_prefix_cache(vc4_session* s, int slot, const char* path, int* toks_out, int cap, int* n_out) {
    if (slot < 0 || slot >= s->slots) return fail(VC4_EINVAL, "slot out of range");
    std::vector<uint32_t> t;
    std::vector<uint8_t> rows;
    if (int e = read_mmkv(s, path, t, rows)) return e;
    const int n = (int)t.size();
    if (n > cap) return fail(VC4_EINVAL, "token buffer too small for the cache");
    const size_t lb = (size_t)n * s->st.row_bytes;
    for (int l = 0; l < s->m->d.h.layers; ++l)
        if (int e = vc4_kv_write_rows(s, slot, l, n, rows.data() + l * lb)) return e;
    for (int i = 0; i < n; ++i) toks_out[i] = (int)t[i];
    *n_out = n;
    return VC4_OK;
}

// ---------------------------------------------------------------------------
// replay probe
// ---------------------------------------------------------------------------

namespace {

void launch_op(vc4_session* s, int op, int layer, const Batch& b, cudaStream_t st) {
    const DModel& m = s->m->d;
    switch (op) {
        case 0: launch_embed_qkv(m, s->st, b, layer, st); break;
        case 1: launch_attention(m, s->st, b, layer, st); break;
        case 2: launch_wo(m, s->st, b, layer, st); break;
        case 3: launch_ffn_gate(m, s->st, b, layer, st); break;
        default: launch_logits(m, s->st, b, s->d_next, nullptr, nullptr, 0, nullptr, st); break;
    }
}

}  // namespace

extern "C" int vc4_profile_op(vc4_session* s, int op, int layer, int n, const int* slots, const int* tokens,
                              const int* pos, int reps, int flush, double* avg_ms) {
    if (op < 0 || op > 5 || layer < 0 || layer >= s->m->d.h.layers || n <= 0 || n > s->slots || reps <= 0)
        return fail(VC4_EINVAL, "profile_op: bad arguments");
    if (op == 4) return fail(VC4_EINVAL, "profile_op: w2 runs inside op 3 (the FFN kernel)");
    for (int i = 0; i < n; ++i)
        if (int e = check_slot_pos(s, slots[i], pos[i])) return e;
    CK(cudaSetDevice(s->m->d.device));
    static thread_local void* scratch = nullptr;
    const size_t kFlush = (size_t)256 << 20;
    if (flush && !scratch) CK(cudaMalloc(&scratch, kFlush));
    int* hp = s->h_pin;
    for (int i = 0; i < n; ++i) { hp[i] = slots[i]; hp[n + i] = tokens[i]; hp[2 * n + i] = pos[i]; }
    int* dcall = s->d_slot;
    CK(cudaMemcpyAsync(dcall, hp, sizeof(int) * 3 * n, cudaMemcpyHostToDevice, s->stream));
    Batch b;
    b.n = n; b.slot = dcall; b.token = dcall + n; b.pos = dcall + 2 * n;
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    double total = 0.0;
    launch_op(s, op, layer, b, s->stream);   // warm: attributes, instruction cache
    for (int r = 0; r < reps; ++r) {
        if (flush) l2_flush(scratch, kFlush, r, s->stream);
        CK(cudaEventRecord(e0, s->stream));
        launch_op(s, op, layer, b, s->stream);
        CK(cudaEventRecord(e1, s->stream));
        CK(cudaEventSynchronize(e1));
        float ms = 0.0f;
        CK(cudaEventElapsedTime(&ms, e0, e1));
        total += ms;
    }
    CK(cudaGetLastError());
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    // replays of the FFN op add their w2 partial sums again: restore the
    // all-zero state every pass starts from
    const HModel& hm = s->m->d.h;
    CK(cudaMemsetAsync(s->st.sdown, 0, (size_t)hm.layers * s->slots * 2 * hm.dim * 8, s->stream));
    if (int e = check_kernel_word(s)) return e;
    *avg_ms = total / reps;
    return VC4_OK;
}

extern "C" int vc4_op_bytes(const vc4_session* s, int op, int layer, int n, const int* pos, double* bytes) {
    const DModel& m = s->m->d;
    const HModel& h = m.h;
    if (op < 0 || op > 5 || layer < 0 || layer >= h.layers || n <= 0) return fail(VC4_EINVAL, "op_bytes: bad arguments");
    if (op == 4) return fail(VC4_EINVAL, "op_bytes: w2 runs inside op 3 (the FFN kernel)");
    auto wbytes = [&](int idx) -> double {
        if (idx < 0) return 0.0;
        const DMat& w = m.mats[idx];
        if (w.wtype == W_I16) return 2.0 * w.rows * w.cols;
        const double per = w.wtype == W_Q8 ? 1.0 : w.wtype == W_Q4 ? 0.5 : 0.25;
        return per * w.rows * w.cols + (w.wtype == W_Q4 ? 4.0 * w.rows * (w.cols / 32) : 0.0) + 4.0 * w.rows;
    };
    const double D = h.dim, Q = h.dim + 2 * h.kv_dim, F = m.ffn_width;
    double b = 0.0;
    switch (op) {
        case 0: b = wbytes(m.qkv[layer]) + n * (2 * D + 4 * Q); break;
        case 1: {
            // distinct cache rows read: a shared prefix counts once
            double kv = 0.0;
            int shared = 0;
            for (int i = 0; i < n; ++i) {
                const int pl = std::min(s->plen[std::min(i, s->slots - 1)], pos[i] + 1);
                kv += (double)(pos[i] + 1 - pl) * s->st.row_bytes;
                shared = std::max(shared, pl);
            }
            kv += (double)shared * s->st.row_bytes;
            b = kv + n * (4 * Q + 2 * D + s->st.row_bytes);
            break;
        }
        case 2: b = wbytes(m.wo[layer]) + n * (2 * D + 2 * D + 2 * D); break;
        case 3: {
            // gate/up of every expert the batch touches (at most min(n, E)), the router, and their w2
            if (h.experts) {
                const int touched = std::min(n, h.experts);
                const int e0 = m.e_w1[(size_t)layer * h.experts];
                b = touched * (wbytes(e0) + wbytes(e0 + 1) + wbytes(e0 + 2) + (m.ffn_chunked ? wbytes(e0 + 3) : 0.0)) +
                    wbytes(m.router[layer]);
            } else {
                b = wbytes(m.w1[layer]) + wbytes(m.w3[layer]) + wbytes(m.w2a[layer]) +
                    (m.ffn_chunked ? wbytes(m.w2b[layer]) : 0.0);
            }
            b += n * (2 * D + 8.0 * 2 * D);   // x1 in, int64 partial sums out
            break;
        }
        default: b = wbytes(m.logits_mat) + n * (2 * D + 4.0 * h.vocab); break;
    }
    *bytes = b;
    return VC4_OK;
}

// ---------------------------------------------------------------------------
// internal accessors for other translation units of the library
// ---------------------------------------------------------------------------

namespace vc4 {

int set_error(int code, const char* msg) { return fail(code, msg); }

const DModel& model_of(const vc4_model* m) { return m->d; }

SessionView session_view(vc4_session* s) {
    SessionView v;
    v.st = &s->st;
    v.m = &s->m->d;
    v.stream = s->stream;
    v.slots = s->slots;
    v.ops = &s->ops;
    v.launches = &s->launches;
    v.syncs = &s->syncs;
    return v;
}

int kernel_check(vc4_session* s) { return check_kernel_word(s); }

cudaStream_t model_stream(const vc4_model* m) { return m->g->stream; }

// The device matrix `which` of `layer` (and `expert`) names, as vc4_matvec_s
// resolves it; returns VC4_OK and the index into DModel::mats.
int lookup_matrix(const vc4_model* m, int which, int layer, int expert, int* idx) {
    const DModel& d = m->d;
    const HModel& h = d.h;
    *idx = -1;
    if (which != 6 && (layer < 0 || layer >= h.layers)) return fail(VC4_EINVAL, "layer out of range");
    const bool moe = h.experts > 0;
    if (moe && (which == 2 || which == 3 || which == 4)) {
        if (expert < 0 || expert >= h.experts) return fail(VC4_EINVAL, "expert out of range");
        *idx = d.e_w1[(size_t)layer * h.experts + expert] + (which == 2 ? 0 : which == 3 ? 1 : 2);
    } else {
        switch (which) {
            case 0: *idx = d.qkv[layer]; break;
            case 1: *idx = d.wo[layer]; break;
            case 2: *idx = d.w1[layer]; break;
            case 3: *idx = d.w3[layer]; break;
            case 4: *idx = d.w2a[layer]; break;
            case 5: *idx = moe ? d.router[layer] : -1; break;
            case 6: *idx = d.logits_mat; break;
            default: break;
        }
    }
    if (*idx < 0) return fail(VC4_EINVAL, "no such matrix");
    if (which == 4 && d.ffn_chunked) return fail(VC4_EINVAL, "w2 of a chunked FFN is two matrices; the CPU path never draws it whole");
    return VC4_OK;
}

}  // namespace vc4
