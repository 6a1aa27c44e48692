// ref_shim.cpp -- TEST INFRASTRUCTURE: a C entry point over the reference
// engine's own MMCF loader, used to pin the oracle's loader.
//
// Built by oracle/Makefile together with the reference's host sources
// (engine/src/model.cpp, common.cpp, switches.cpp, xformat.cpp, compiled where
// they lie, against the typedef-only gles2_stub) into oracle/_ref/.  It calls
// Model::load (model.cpp:23) with T3_EXPAND=1 so a 2-bit body comes back as
// q8 levels (model.cpp:934-970), and reports every decoded tensor as a JSON
// summary: shape, type, scale bits and an FNV-1a/64 digest of the values as
// little-endian int32 (or float bits).  tests/golden/make_golden.py records
// these summaries; tests compare the oracle's own decode against them.
#include "model.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

namespace {

struct Fnv {
    uint64_t h = 1469598103934665603ull;
    void byte(uint8_t b) { h ^= b; h *= 1099511628211ull; }
    void i32(int32_t v) { for (int k = 0; k < 4; ++k) byte((uint8_t)((uint32_t)v >> (8 * k))); }
    void f32(float f) { uint32_t u; memcpy(&u, &f, 4); i32((int32_t)u); }
};

std::string hex64(uint64_t v) { char b[32]; snprintf(b, sizeof b, "%016llx", (unsigned long long)v); return b; }
std::string fbits(float f) { uint32_t u; memcpy(&u, &f, 4); char b[16]; snprintf(b, sizeof b, "%08x", u); return b; }

std::string floats(const std::vector<float>& v) {
    Fnv f; for (float x : v) f.f32(x);
    return "{\"n\":" + std::to_string(v.size()) + ",\"fnv\":\"" + hex64(f.h) + "\"}";
}

std::string mat(const Mat& m) {
    std::string s = "{\"rows\":" + std::to_string(m.rows) + ",\"cols\":" + std::to_string(m.cols);
    Fnv lv;
    const size_t n = (size_t)m.rows * m.cols;
    const char* type = "?";
    float scale = m.scale;
    std::string extra;
    if (m.type == WeightType::INT8) {
        type = "q8";
        const int8_t* p = m.w8();
        for (size_t i = 0; i < n; ++i)
            lv.i32(m.prebiased ? (int32_t)(uint8_t)p[i] - 128 : (int32_t)p[i]);
    } else if (m.type == WeightType::INT16) {
        type = "i16";
        const int16_t* p = m.w16();
        for (size_t i = 0; i < n; ++i) lv.i32(p[i]);
    } else if (m.type == WeightType::INT4) {
        type = "q4";
        const uint8_t* p = m.w4();
        for (size_t i = 0; i < n; ++i) lv.i32((i & 1) ? (p[i / 2] >> 4) : (p[i / 2] & 15));
        scale = m.q4_param_scale;
        Fnv a, b;
        const size_t ng = (size_t)m.rows * m.groups;
        for (size_t i = 0; i < ng; ++i) { a.i32(m.s4()[i]); b.i32(m.m4()[i]); }
        extra = ",\"s16\":\"" + hex64(a.h) + "\",\"m16\":\"" + hex64(b.h) + "\"";
    }
    s += std::string(",\"type\":\"") + type + "\",\"scale\":\"" + fbits(scale) + "\",\"levels\":\"" + hex64(lv.h) + "\"";
    if (!m.row_scale.empty()) s += ",\"row_scale\":" + floats(m.row_scale);
    return s + extra + "}";
}

}  // namespace

extern "C" int ref_load_summary(const char* path, char* out, int cap) {
    setenv("T3_EXPAND", "1", 1);
    Model m;
    if (!m.load(path)) return -1;
    std::string j = "{";
    j += "\"dim\":" + std::to_string(m.dim) + ",\"hidden\":" + std::to_string(m.hidden) +
         ",\"layers\":" + std::to_string(m.layers) + ",\"heads\":" + std::to_string(m.heads) +
         ",\"kv_heads\":" + std::to_string(m.kv_heads) + ",\"vocab\":" + std::to_string(m.vocab) +
         ",\"seq\":" + std::to_string(m.seq) + ",\"head_dim\":" + std::to_string(m.head_dim) +
         ",\"kv_dim\":" + std::to_string(m.kv_dim) + ",\"experts\":" + std::to_string(m.experts) +
         ",\"moe_hidden\":" + std::to_string(m.moe_hidden) +
         ",\"rope_theta\":\"" + fbits(m.rope_theta) + "\",\"rope_half\":" + (m.rope_half ? "1" : "0") +
         ",\"qk_norm\":" + (m.qk_norm ? "1" : "0") + ",\"rms_eps\":\"" + fbits(m.rms_eps) + "\"";
    {
        Fnv f; for (int8_t v : m.emb_q8) f.i32(v);
        j += ",\"emb\":{\"n\":" + std::to_string(m.emb_q8.size()) + ",\"fnv\":\"" + hex64(f.h) + "\"}";
    }
    j += ",\"emb_scale\":" + floats(m.emb_scale) + ",\"rms_att\":" + floats(m.rms_att) +
         ",\"rms_ffn\":" + floats(m.rms_ffn) + ",\"rms_final\":" + floats(m.rms_final) +
         ",\"q_norm\":" + floats(m.q_norm) + ",\"k_norm\":" + floats(m.k_norm);
    auto list = [&](const char* name, const std::vector<Mat>& v) {
        j += std::string(",\"") + name + "\":[";
        for (size_t i = 0; i < v.size(); ++i) j += (i ? "," : "") + mat(v[i]);
        j += "]";
    };
    list("qkv", m.qkv); list("wo", m.wo); list("w1", m.w1); list("w3", m.w3); list("w2", m.w2);
    list("router", m.router); list("logits", m.logits_tiles);
    j += ",\"experts_w\":[";
    for (size_t l = 0; l < m.moe.size(); ++l) {
        j += (l ? "," : "") + std::string("[");
        for (size_t e = 0; e < m.moe[l].size(); ++e)
            j += (e ? "," : "") + std::string("{\"w1\":") + mat(m.moe[l][e].w1) + ",\"w3\":" +
                 mat(m.moe[l][e].w3) + ",\"w2\":" + mat(m.moe[l][e].w2) + "}";
        j += "]";
    }
    j += "]}";
    if ((int)j.size() + 1 > cap) return (int)j.size() + 1;
    memcpy(out, j.c_str(), j.size() + 1);
    return 0;
}
