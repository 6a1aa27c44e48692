// forward_gpu_hidden.cpp -- Session::forward_gpu_hidden (engine/src/session.cpp:
// 1459-1584) and Session::step_greedy (1827-1842) restated call for call over the
// per-op C ABI of include/vc4b200.h, as the reference's Session would drive a
// CUDA-backed class GPU.  Compiled and run by tests/test_capi.py.
//
//   forward_gpu_hidden CONTAINER SEQ KV_BITS N_PROMPT N_STEPS TOK...
//
// prints one line per position: "pos token logit_digest" (FNV-1a over the q16
// logits), the prompt teacher-forced, then greedy steps.
#include "vc4b200.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#define CHECK(x)                                                                    \
    do {                                                                            \
        if (int rc_ = (x)) {                                                        \
            fprintf(stderr, "%s failed (%d): %s\n", #x, rc_, vc4_last_error());      \
            exit(1);                                                                \
        }                                                                           \
    } while (0)

namespace {

vc4_session* g_s = nullptr;
vc4_model_info g_info;

// pick_expert (session.cpp:110-115): the first maximum.
int pick_expert(const std::vector<float>& gate) {
    int best = 0;
    for (size_t i = 1; i < gate.size(); ++i)
        if (gate[i] > gate[best]) best = (int)i;
    return best;
}

// One position through the layer loop; the final rmsnorm lands in VC4_BUF_XF.
void forward_gpu_hidden(int token, int pos) {
    const int slot = 0;
    CHECK(vc4_embedding(g_s, slot, token, VC4_BUF_HIDDEN));                   // h = upload_hidden(embedding(token))
    for (int l = 0; l < g_info.layers; ++l) {
        CHECK(vc4_rmsnorm(g_s, slot, VC4_BUF_HIDDEN, 0, l, VC4_BUF_XB));         // xb = rmsnorm(h, rms_att[l])
        CHECK(vc4_attention_block(g_s, slot, l, pos, VC4_BUF_XB, VC4_BUF_ATT)); // att = attention_block(qkv[l], xb, l, pos)
        CHECK(vc4_matvec_add(g_s, slot, 1, l, 0, VC4_BUF_ATT, VC4_BUF_HIDDEN, VC4_BUF_X1));   // x1 = h + wo[l] att
        CHECK(vc4_rmsnorm(g_s, slot, VC4_BUF_X1, 1, l, VC4_BUF_XBF));          // xbf = rmsnorm(x1, rms_ffn[l])
        int expert = 0;
        if (g_info.experts > 0) {                                                // gate = matvec_from(router[l], xbf)
            std::vector<float> gate(g_info.experts);
            CHECK(vc4_matvec_from(g_s, slot, 5, l, 0, VC4_BUF_XBF, 1, gate.data()));
            expert = pick_expert(gate);
        }
        if (g_info.ffn_chunked) {                                                // ffn_split_chunked + two matvec_adds
            CHECK(vc4_ffn_split(g_s, slot, l, expert, VC4_BUF_XBF, VC4_BUF_HA, VC4_BUF_HB));
            CHECK(vc4_matvec_add(g_s, slot, 4, l, expert, VC4_BUF_HA, VC4_BUF_X1, VC4_BUF_TMP));
            CHECK(vc4_matvec_add(g_s, slot, 7, l, expert, VC4_BUF_HB, VC4_BUF_TMP, VC4_BUF_HIDDEN));
        } else {                                                                 // ffn_split + matvec_add
            CHECK(vc4_ffn_split(g_s, slot, l, expert, VC4_BUF_XBF, VC4_BUF_HA, VC4_BUF_HB));
            CHECK(vc4_matvec_add(g_s, slot, 4, l, expert, VC4_BUF_HA, VC4_BUF_X1, VC4_BUF_HIDDEN));
        }
    }
    CHECK(vc4_rmsnorm(g_s, slot, VC4_BUF_HIDDEN, 2, 0, VC4_BUF_XF));             // xf = rmsnorm(h, rms_final)
}

unsigned long long fnv(const std::vector<float>& lg) {
    unsigned long long h = 1469598103934665603ull;
    for (float v : lg) {
        const int q = (int)lrintf(v * 256.0f);
        for (int b = 0; b < 4; ++b) h = (h ^ ((unsigned)q >> (8 * b) & 0xFFu)) * 1099511628211ull;
    }
    return h;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 6) {
        fprintf(stderr, "usage: forward_gpu_hidden CONTAINER SEQ KV_BITS N_PROMPT N_STEPS TOK...\n");
        return 2;
    }
    const int seq = atoi(argv[2]), kv = atoi(argv[3]), np = atoi(argv[4]), ns = atoi(argv[5]);
    std::vector<int> prompt;
    for (int i = 6; i < argc; ++i) prompt.push_back(atoi(argv[i]));
    if ((int)prompt.size() != np || np < 1) return 2;
    vc4_gpu* g = nullptr;
    vc4_model* m = nullptr;
    CHECK(vc4_gpu_create(0, &g));
    CHECK(vc4_model_load(g, argv[1], &m));
    CHECK(vc4_model_info_get(m, &g_info));
    CHECK(vc4_session_create(m, 1, seq, kv, nullptr, nullptr, &g_s));
    std::vector<float> lg(g_info.vocab);
    int tok = prompt[0];
    for (int pos = 0; pos < np + ns; ++pos) {                                    // step / step_greedy per position
        forward_gpu_hidden(tok, pos);
        CHECK(vc4_logits_from(g_s, 0, VC4_BUF_XF, lg.data()));                   // logits_from(tiles, xf)
        int next = 0;
        CHECK(vc4_logits_argmax_from(g_s, 0, VC4_BUF_XF, &next));                // logits_argmax_from(tiles, xf)
        printf("%d %d %016llx\n", pos, next, fnv(lg));
        tok = pos + 1 < np ? prompt[pos + 1] : next;
    }
    vc4_session_destroy(g_s);
    vc4_model_free(m);
    vc4_gpu_destroy(g);
    return 0;
}
