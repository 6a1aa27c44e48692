// ref_session.cpp -- TEST INFRASTRUCTURE (the checker's checker; never on the
// product path).
//
// Runs the reference's own CPU layer loop -- engine/src/session.cpp:
// Session::Session (rope tables, session.cpp:127-313), Session::step
// (1797-1821), forward (373-556), embedding (342-371), rms_norm (1932-1948),
// head_rms_norm (1950-1961), rope (1963-1987), attention (1989-2050, with its
// KV8_SIM read-time quantiser, 51-69), add_q16 (2052-2067) -- compiled from
// the reference sources where they lie (oracle/Makefile `ref`), against a
// stand-in for class GPU (engine/src/gpu.h:41-633).  No GL function exists in
// this build.  The stand-in's shader calls -- matvec_s (gpu_conv.cpp:271-287),
// matvec (gpu_conv.cpp:227-262), upload_input, ffn_split / ffn_split_chunked
// (gpu_ffn.cpp:17-132), matvec_from (gpu_matvec.cpp:32-55) and logits
// (gpu_matvec.cpp:84-90) -- are the oracle's restatement of the shader
// arithmetic (vc4_oracle.c); every member only the GL path reaches aborts.
// The weights are the reference loader's own (Model::load, model.cpp,
// prepared as App::prepare_model does) for the session, and the oracle's load
// of the same file for the shaders; a Mat is matched to its oracle matrix by
// its place in the Model.
//
//   ref_session CONTAINER MATVEC_MODE OUT N_OUT TOK...
//
// teacher-forces TOK[i] at position i and writes the logits (vocab float32)
// of the last N_OUT positions to OUT.  MATVEC_MODE 1 uses the shaders' fp32
// accumulation (ORC_LITERAL), 0 the exact integer dot.  KV8_SIM=1 in the
// environment selects the reference's q8 read-time cache quantiser.
#include "session.h"
#include "sampling.h"
#include "vc4_oracle.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace {

const Model* g_model = nullptr;
orc_model* g_om = nullptr;
int g_literal = 1;
std::map<GLuint, std::vector<int16_t>> g_tex;   // uploaded q16 activations by handle
GLuint g_next = 1;

[[noreturn]] void gl_only(const char* what) {
    fprintf(stderr, "ref_session: %s belongs to the GL path, which this build does not have\n", what);
    abort();
}

// Where a Mat sits in the reference Model, as an oracle matrix: which (0 qkv,
// 1 wo, 2 w1, 3 w3, 4 w2, 5 router, 6 logits tile), layer (tile index for 6),
// expert, its row range and column range in the whole matrix.
struct Id {
    int which = -1, layer = 0, expert = 0, r0 = 0, r1 = 0, c0 = 0, c1 = 0;
};

Id ident(const Mat& m) {
    const Model& M = *g_model;
    Id id;
    auto hit = [&](const Mat& c, int which, int layer, int expert, int r0, int c0) {
        if (&c != &m) return false;
        id.which = which; id.layer = layer; id.expert = expert;
        id.r0 = r0; id.r1 = r0 + m.rows; id.c0 = c0; id.c1 = c0 + m.cols;
        return true;
    };
    const int ch = M.ffn_chunk;
    for (size_t t = 0; t < M.logits_tiles.size(); ++t)
        if (hit(M.logits_tiles[t], 6, (int)t, 0, 0, 0)) return id;
    for (int l = 0; l < M.layers; ++l) {
        if (hit(M.qkv[l], 0, l, 0, 0, 0) || hit(M.wo[l], 1, l, 0, 0, 0)) return id;
        if (!M.router.empty() && hit(M.router[l], 5, l, 0, 0, 0)) return id;
        if (!M.w1.empty() && (hit(M.w1[l], 2, l, 0, 0, 0) || hit(M.w3[l], 3, l, 0, 0, 0))) return id;
        if (!M.w2.empty() && hit(M.w2[l], 4, l, 0, 0, 0)) return id;
        if (!M.w1a.empty() &&
            (hit(M.w1a[l], 2, l, 0, 0, 0) || hit(M.w1b[l], 2, l, 0, ch, 0) || hit(M.w3a[l], 3, l, 0, 0, 0) ||
             hit(M.w3b[l], 3, l, 0, ch, 0) || hit(M.w2a[l], 4, l, 0, 0, 0) || hit(M.w2b[l], 4, l, 0, 0, ch)))
            return id;
        if (M.is_moe())
            for (int e = 0; e < M.experts; ++e) {
                const Model::MoeExpert& x = M.moe[l][e];
                if (hit(x.w1, 2, l, e, 0, 0) || hit(x.w3, 3, l, e, 0, 0) || hit(x.w2, 4, l, e, 0, 0) ||
                    hit(x.w1a, 2, l, e, 0, 0) || hit(x.w1b, 2, l, e, ch, 0) || hit(x.w3a, 3, l, e, 0, 0) ||
                    hit(x.w3b, 3, l, e, ch, 0) || hit(x.w2a, 4, l, e, 0, 0) || hit(x.w2b, 4, l, e, 0, ch))
                    return id;
            }
    }
    fprintf(stderr, "ref_session: a matrix the layer loop drew is not in the model\n");
    abort();
}

int full_rows(const Id& id) {
    int r = 0, c = 0, t = 0;
    float s = 0.0f;
    if (orc_model_mat_shape(g_om, id.which, id.layer, id.expert, &r, &c, &t, &s) != ORC_OK) {
        fprintf(stderr, "ref_session: the oracle has no matrix %d/%d/%d\n", id.which, id.layer, id.expert);
        abort();
    }
    return r;
}

// One shader matvec over q16 ints: the clamped q16 results of rows r0..r1.
std::vector<int32_t> shader_mv(const Id& id, const int16_t* xq) {
    std::vector<int32_t> out(full_rows(id));
    if (orc_model_mv(g_om, id.which, id.layer, id.expert, id.c0, id.c1, xq, g_literal, out.data()) != ORC_OK) {
        fprintf(stderr, "ref_session: oracle matvec refused %d/%d/%d\n", id.which, id.layer, id.expert);
        abort();
    }
    return std::vector<int32_t>(out.begin() + id.r0, out.begin() + id.r1);
}

GLuint keep(std::vector<int16_t>&& v) {
    g_tex[g_next] = std::move(v);
    return g_next++;
}

const std::vector<int16_t>& tex(GLuint h) {
    auto it = g_tex.find(h);
    if (it == g_tex.end()) {
        fprintf(stderr, "ref_session: unknown activation handle %u\n", h);
        abort();
    }
    return it->second;
}

std::vector<int16_t> q16_of(const std::vector<float>& x) {
    std::vector<int16_t> q(x.size());
    for (size_t i = 0; i < x.size(); ++i) q[i] = orc_q16(x[i]);
    return q;
}

// The FFN gate kernel's q16 hidden (every row of the layer's gate/up).
std::vector<int16_t> hidden_of(const Mat& w1, GLuint x) {
    const Id id = ident(w1);
    std::vector<int16_t> h(g_model->ffn_width());
    if (orc_ffn_hidden(g_om, id.layer, id.expert, tex(x).data(), g_literal, h.data()) != ORC_OK) {
        fprintf(stderr, "ref_session: oracle FFN refused layer %d\n", id.layer);
        abort();
    }
    return h;
}

}  // namespace

// ---- the stand-in for class GPU (declarations: engine/src/gpu.h) ----------

bool gpu_es3_ok() { return false; }

GPU::GPU() {}
GPU::~GPU() {}

void GPU::reset_format_plan() {}
bool GPU::gpu_layer_enabled() const { return false; }
bool GPU::gpu_attn_enabled() const { return false; }
bool GPU::needs_finish() const { return false; }
void GPU::sync() {}

vector<float> GPU::matvec(const Mat& m, const vector<float>& x) {
    const std::vector<int16_t> xq = q16_of(x);
    const std::vector<int32_t> v = shader_mv(ident(m), xq.data());
    vector<float> out(v.size());
    for (size_t i = 0; i < v.size(); ++i) out[i] = (float)v[i] / ACT_SCALE;
    return out;
}

vector<float> GPU::matvec_s(const Mat& m, const vector<float>& x) {
    std::vector<int16_t> xq(x.size());
    const int k = orc_scale_input(x.data(), (int)x.size(), xq.data());
    const std::vector<int32_t> v = shader_mv(ident(m), xq.data());
    const float inv = ldexpf(1.0f, -k);
    vector<float> out(v.size());
    for (size_t i = 0; i < v.size(); ++i) out[i] = ((float)v[i] / ACT_SCALE) * inv;
    return out;
}

GLuint GPU::upload_input(const vector<float>& x) { return keep(q16_of(x)); }

vector<float> GPU::matvec_from(const Mat& m, GLuint x) {
    const Id id = ident(m);
    const std::vector<int16_t>& xq = tex(x);
    if ((int)xq.size() != id.c1 - id.c0) {
        fprintf(stderr, "ref_session: matvec_from input width mismatch\n");
        abort();
    }
    const std::vector<int32_t> v = shader_mv(id, xq.data());
    vector<float> out(v.size());
    for (size_t i = 0; i < v.size(); ++i) out[i] = (float)v[i] / ACT_SCALE;
    return out;
}

GLuint GPU::ffn_split(const Mat& w1, const Mat& w3, GLuint x, int hidden, int hs) {
    (void)w3; (void)hs;   // the oracle reads the layer's w3 and key-15 shift itself
    std::vector<int16_t> h = hidden_of(w1, x);
    h.resize(hidden);
    return keep(std::move(h));
}

void GPU::ffn_split_chunked(const Mat& w1a, const Mat& w3a, const Mat& w1b, const Mat& w3b, GLuint x, int n1,
                            int n2, GLuint& ha, GLuint& hb, int hs) {
    (void)w3a; (void)w1b; (void)w3b; (void)hs;
    const std::vector<int16_t> h = hidden_of(w1a, x);
    ha = keep(std::vector<int16_t>(h.begin(), h.begin() + n1));
    hb = keep(std::vector<int16_t>(h.begin() + n1, h.begin() + n1 + n2));
}

vector<float> GPU::logits(const vector<Mat>& tiles, const vector<float>& x) {
    const std::vector<int16_t> xq = q16_of(x);
    vector<float> out;
    for (const Mat& t : tiles) {
        const std::vector<int32_t> v = shader_mv(ident(t), xq.data());
        for (int32_t q : v) out.push_back((float)q / ACT_SCALE);
    }
    return out;
}

// members only the fused GL path, prefill grouping, conv, RWKV or diagnostics reach
GLuint GPU::ffn_fused(const Mat&, GLuint, int, int) { gl_only("ffn_fused"); }
GLuint GPU::ffn_pair_swiglu_chunk2_p2(const Mat&, const Mat&, GLuint, int, Target&) { gl_only("ffn_pair_swiglu_chunk2_p2"); }
GLuint GPU::rmsnorm_pair2(GLuint, GLuint, GLuint, Target&) { gl_only("rmsnorm_pair2"); }
void GPU::matvec_p2_add_p2(const Mat&, GLuint, GLuint, Target&) { gl_only("matvec_p2_add_p2"); }
void GPU::matvec_p2_add(const Mat&, GLuint, GLuint, GLuint, Target&) { gl_only("matvec_p2_add"); }
void GPU::p2_split(GLuint, Target&, int) { gl_only("p2_split"); }
CandidateResult GPU::logits_candidates(const vector<Mat>&, const vector<float>&, int, float, float) {
    gl_only("logits_candidates");
}
CandidateResult GPU::logits_candidates_from(const vector<Mat>&, GLuint, int, float, float) {
    gl_only("logits_candidates_from");
}
void GPU::init_attention(int, int, int, int, int, int, bool, bool, int, const vector<float>&, const vector<float>&,
                         const vector<float>&, const vector<float>&, bool, bool, const std::vector<uint8_t>*) {
    gl_only("init_attention");
}
GLuint GPU::attention_block(const Mat&, GLuint, int, int) { gl_only("attention_block"); }
void GPU::att_stage(const Mat&, GLuint, int, int, int, int) { gl_only("att_stage"); }
void GPU::att_scores_batch(int, int, int) { gl_only("att_scores_batch"); }
void GPU::att_stats_row(int, int, int) { gl_only("att_stats_row"); }
void GPU::att_v_row(int, int, int, int) { gl_only("att_v_row"); }
GLuint GPU::upload_hidden_grp(const vector<float>&, int, int) { gl_only("upload_hidden_grp"); }
Target& GPU::grp_h(int, int) { gl_only("grp_h"); }
Target& GPU::grp_tmp() { gl_only("grp_tmp"); }
Target& GPU::grp_w2a() { gl_only("grp_w2a"); }
void GPU::init_persistent(int, int, const vector<float>&, const vector<float>&, const vector<float>&) {
    gl_only("init_persistent");
}
GLuint GPU::upload_hidden(const vector<float>&) { gl_only("upload_hidden"); }
GLuint GPU::upload_hidden_b(const vector<float>&) { gl_only("upload_hidden_b"); }
GLuint GPU::rmsnorm(GLuint, GLuint, Target&) { gl_only("rmsnorm"); }
void GPU::matvec_add(const Mat&, GLuint, GLuint, Target&, XFormat) { gl_only("matvec_add"); }
void GPU::init_conv(int, int) { gl_only("init_conv"); }
void GPU::set_conv_kernel(int, const float*, int, int) { gl_only("set_conv_kernel"); }
void GPU::clear_conv_state() { gl_only("clear_conv_state"); }
GLuint GPU::conv_copy(GLuint, Target&) { gl_only("conv_copy"); }
GLuint GPU::conv_block(const Mat&, const Mat&, const Mat&, const Mat&, GLuint, GLuint, int, Target&) {
    gl_only("conv_block");
}
void GPU::init_rwkv(const Model&) { gl_only("init_rwkv"); }
GLuint GPU::rwkv_block(int, const Model&, GLuint, float*) { gl_only("rwkv_block"); }
vector<vector<float>> GPU::matvec_rows(const vector<MvRow>&, int, int) { gl_only("matvec_rows"); }
vector<vector<vector<float>>> GPU::matvec_batch_group(const vector<MvBatch>&) { gl_only("matvec_batch_group"); }
void GPU::rwkv_prof_fused_summary() { gl_only("rwkv_prof_fused_summary"); }
std::vector<float> GPU::rwkv_read_residual(GLuint) { gl_only("rwkv_read_residual"); }
GLuint GPU::rwkv_upload_x0(const std::vector<float>&) { gl_only("rwkv_upload_x0"); }
vector<float> GPU::logits_from(const vector<Mat>&, GLuint) { gl_only("logits_from"); }
bool GPU::logits_argmax_ok(const vector<Mat>&) const { return false; }
int GPU::logits_argmax_from(const vector<Mat>&, GLuint) { gl_only("logits_argmax_from"); }
void GPU::logits_pass_only(const vector<Mat>&, GLuint) { gl_only("logits_pass_only"); }
vector<uint8_t> GPU::read_bytes(Target&, int, int) { gl_only("read_bytes"); }
vector<float> GPU::read_logits_full(const vector<Mat>&) { gl_only("read_logits_full"); }
void GPU::dump_target(const Target&, const char*, int) { gl_only("dump_target"); }
void GPU::dump_cpu_row(const vector<float>&, XFormat, const char*, int) { gl_only("dump_cpu_row"); }

// ---- driver ------------------------------------------------------------------

int main(int argc, char** argv) {
    if (argc < 6) {
        fprintf(stderr, "usage: ref_session CONTAINER MATVEC_MODE OUT N_OUT TOK...\n");
        return 2;
    }
    const std::string path = argv[1];
    g_literal = atoi(argv[2]);
    const char* out_path = argv[3];
    const int n_out = atoi(argv[4]);
    std::vector<int> toks;
    for (int i = 5; i < argc; ++i) toks.push_back(atoi(argv[i]));
    static Model model;
    if (!model.load(path)) {
        fprintf(stderr, "ref_session: the reference loader refused %s\n", path.c_str());
        return 3;
    }
    char err[256] = {0};
    if (orc_model_load(path.c_str(), &g_om, err, sizeof err) != ORC_OK) {
        fprintf(stderr, "ref_session: the oracle refused %s: %s\n", path.c_str(), err);
        return 3;
    }
    // the model preparation of App::prepare_model (app.cpp:14-26) on a
    // desktop GL driver, whose target limit (16384) leaves a hidden above 2048
    // in two FFN chunks (Model::split_ffn, model.cpp:217-270)
    model.split_ffn(16384);
    model.split_rwkv(16384);
    model.apply_q4_fmt();
    model.apply_hidden_scale();
    g_model = &model;
    static GPU gpu;
    Session session(model, gpu);
    FILE* f = fopen(out_path, "wb");
    if (!f) return 4;
    const int n = (int)toks.size();
    for (int p = 0; p < n; ++p) {
        const bool want = p >= n - n_out;
        vector<float> lg = session.step(toks[p], p, want);
        if (want && fwrite(lg.data(), sizeof(float), lg.size(), f) != lg.size()) return 4;
        g_tex.clear();
    }
    fclose(f);
    orc_model_free(g_om);
    return 0;
}
