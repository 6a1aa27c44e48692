// mmcf.cpp -- MMCF container reader of the B200 engine.
//
// Follows the reference reader's contract (engine/src/model.cpp: header
// 614-660, metadata TLVs 662-760, tensor table 873-1560) for the subset the
// decode path needs: dense v2 and top-1 MoE v3 containers with q8 (dtype 2/3),
// q4 (dtype 4 + planes), t3 (dtype 7 + row plane), i16 router and q8
// embeddings, including the head-dedup logits (model.cpp:1565-1590).  Refusals
// mirror the reference: a file this build cannot run is an error, never a
// half-loaded model.
#include "vc4b200_internal.h"

#include <sys/stat.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>

namespace vc4 {
namespace {

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }
float rdf(const uint8_t* p) { float f; uint32_t u = rd32(p); memcpy(&f, &u, 4); return f; }

uint32_t crc32_40(const uint8_t* h) {
    uint32_t crc = 0xFFFFFFFFu;
    for (int i = 0; i < 40; ++i) {
        crc ^= h[i];
        for (int k = 0; k < 8; ++k) crc = (crc & 1) ? 0xEDB88320u ^ (crc >> 1) : (crc >> 1);
    }
    return crc ^ 0xFFFFFFFFu;
}

struct Rec {
    uint16_t id = 0; uint8_t dtype = 0, group = 0; uint32_t rows = 0, cols = 0;
    const uint8_t* data = nullptr; uint64_t bytes = 0; float scale = 0; uint16_t aux = 0;
    uint32_t key() const { return ((uint32_t)aux << 16) | (uint32_t)(id & 0x3FFF); }
};

// The 16-bit row plane the reference uploads (gpu_upload.cpp:32-58).
std::vector<uint16_t> plane16(const std::vector<float>& plane) {
    std::vector<uint16_t> p(plane.size());
    for (size_t r = 0; r < plane.size(); ++r) {
        long q = lrint((double)plane[r] * 65536.0);
        p[r] = (uint16_t)(q < 0 ? 0 : q > 65535 ? 65535 : q);
    }
    return p;
}

std::string read_mat(const Rec& r, const Rec* p1, const Rec* p2, const Rec* p3, HMat& o) {
    o = HMat();
    o.rows = (int)r.rows; o.cols = (int)r.cols;
    const size_t n = (size_t)r.rows * r.cols;
    if (r.dtype == 2 || r.dtype == 3) {                       // as_q8, model.cpp:902-911
        if (r.bytes < n) return "q8 tensor too short";
        o.wtype = W_Q8; o.scale = r.scale;
        o.lev.resize(n);
        for (size_t i = 0; i < n; ++i)
            o.lev[i] = r.dtype == 2 ? (int8_t)((int)r.data[i] - 128) : (int8_t)r.data[i];
    } else if (r.dtype == 1) {                                // as_i16
        if (r.bytes < 2 * n) return "i16 tensor too short";
        o.wtype = W_I16; o.scale = r.scale;
        o.w16.resize(n);
        for (size_t i = 0; i < n; ++i) o.w16[i] = (int16_t)rd16(r.data + 2 * i);
    } else if (r.dtype == 7) {                                // as_t3, model.cpp:925-975
        const size_t stride = (size_t)((r.cols + 7) / 8) * 4;
        if (r.bytes < (size_t)((r.rows + 1) / 2) * stride) return "t3 tensor too short";
        o.wtype = W_T3;
        o.scale = r.scale * 127.0f;
        o.lev.resize(n);
        for (uint32_t y = 0; y < (r.rows + 1) / 2; ++y) {
            const uint8_t* band = r.data + (size_t)y * stride;
            for (uint32_t half = 0; half < 2; ++half) {
                const uint32_t row = 2 * y + half;
                if (row >= r.rows) break;
                for (uint32_t x = 0; x < r.cols; ++x) {
                    const uint8_t byte = band[(size_t)(x >> 3) * 4 + half * 2 + ((x >> 2) & 1)];
                    const unsigned code = (byte >> (2 * (x & 3))) & 3u;
                    o.lev[(size_t)row * r.cols + x] = (code & 1u) ? ((code & 2u) ? -1 : 1) : 0;
                }
            }
        }
    } else if (r.dtype == 4) {                                // q4 body + parts 1/2
        if (!p1 || !p2) return "q4 matrix without its scale/min planes";
        if (r.cols % 32) return "q4 columns are not a multiple of 32";
        if (r.bytes < n / 2) return "q4 tensor too short";
        o.wtype = W_Q4; o.scale = r.scale;
        const size_t ng = (size_t)r.rows * (r.cols / 32);
        if (p1->rows != r.rows || p1->cols != r.cols / 32 || p1->bytes < 2 * ng ||
            p2->rows != r.rows || p2->cols != r.cols / 32 || p2->bytes < 2 * ng)
            return "q4 plane shape mismatch";
        o.nib.resize(n);
        for (size_t i = 0; i < n; ++i) o.nib[i] = (i & 1) ? (r.data[i / 2] >> 4) : (r.data[i / 2] & 15);
        o.s16.resize(ng); o.m16.resize(ng);
        for (size_t i = 0; i < ng; ++i) { o.s16[i] = (int16_t)rd16(p1->data + 2 * i); o.m16[i] = (int16_t)rd16(p2->data + 2 * i); }
    } else {
        return "unsupported matrix dtype " + std::to_string(r.dtype);
    }
    if (p3) {                                                 // part 3 row plane
        if (p3->rows != r.rows || p3->bytes != (uint64_t)r.rows * 4) return "row plane shape mismatch";
        o.plane.resize(r.rows);
        for (uint32_t i = 0; i < r.rows; ++i) o.plane[i] = rdf(p3->data + 4 * i);
        o.p16 = plane16(o.plane);
    }
    return "";
}

std::vector<float> f32s(const Rec& r, size_t count, std::string& err) {
    std::vector<float> v;
    if (r.dtype != 0 || r.bytes < count * 4) { err = "f32 tensor shape"; return v; }
    v.resize(count);
    for (size_t i = 0; i < count; ++i) v[i] = rdf(r.data + 4 * i);
    return v;
}

}  // namespace

std::string load_mmcf_bytes(const uint8_t* h, size_t sz, HModel& m) {
    m = HModel();
    if (sz < 64) return "mmcf: truncated header";
    if (memcmp(h, "MMCF", 4) != 0) return "not an MMCF container";
    m.version = rd16(h + 4);
    if (m.version == 4) return "mmcf: RWKV-7 containers are not supported by this engine";
    if (m.version != 2 && m.version != 3) return "mmcf: unsupported version " + std::to_string(m.version);
    if (rd16(h + 6) != 64) return "mmcf: bad header size";
    const uint32_t ntens = rd32(h + 8), meta_off = rd32(h + 16), meta_size = rd32(h + 20);
    const uint64_t data_off = rd64(h + 24), file_size = rd64(h + 32);
    const int rsize = m.version >= 3 ? 64 : 48;
    if (file_size != (uint64_t)sz) return "mmcf: size field does not match the file";
    const uint32_t stored = rd32(h + 40);
    if (stored && stored != crc32_40(h)) return "mmcf: header crc mismatch";
    if ((uint64_t)meta_off + meta_size > sz || data_off > sz || data_off < (uint64_t)ntens * rsize)
        return "mmcf: bad section offsets";
    const uint64_t table_off = data_off - (uint64_t)ntens * rsize;
    if (table_off < (uint64_t)meta_off + meta_size || table_off % 16) return "mmcf: tensor table does not follow the metadata block";

    bool have_model = false;
    int split = 0;
    for (uint64_t p = meta_off; p + 8 <= (uint64_t)meta_off + meta_size;) {
        const uint16_t key = rd16(h + p), type = rd16(h + p + 2);
        const uint32_t len = rd32(h + p + 4);
        const uint8_t* pl = h + p + 8;
        if (p + 8 + len > (uint64_t)meta_off + meta_size) return "mmcf: TLV overruns the block";
        if (type == 1) {
            if (key == 1 && len >= 28) {
                m.dim = (int)rd32(pl); m.hidden = (int)rd32(pl + 4); m.layers = (int)rd32(pl + 8);
                m.heads = (int)rd32(pl + 12); m.kv_heads = (int)rd32(pl + 16);
                m.vocab = (int)rd32(pl + 20); m.seq = (int)rd32(pl + 24);
                have_model = true;
            } else if (key == 2 && len >= 8) {
                m.rope_theta = rdf(pl); m.rope_half = pl[4] != 0; m.qk_norm = pl[5] != 0;
            } else if (key == 3 && len >= 4) {
                split = pl[3];
            } else if (key == 4 && len >= 3) {
                // template kind byte, default system prompt NUL, template name NUL
                // (model.cpp:684-695); only the name is kept, for the MMKV1 sidecar
                const char* c = (const char*)pl + 1;
                const char* e = (const char*)pl + len;
                const char* nul = (const char*)memchr(c, 0, (size_t)(e - c));
                if (nul) {
                    const char* nul2 = (const char*)memchr(nul + 1, 0, (size_t)(e - nul - 1));
                    if (nul2) m.template_name.assign(nul + 1, (size_t)(nul2 - nul - 1));
                }
            } else if (key == 11 && len >= 4) {
                const float e = rdf(pl);
                if (e > 0.0f) m.rms_eps = e;
            } else if (key == 12 && len >= 1) {
                if (pl[0] == 1) return "mmcf: q24-residual containers are not supported by this engine";
            } else if (key == 13 && len >= 16) {
                m.experts = (int)rd32(pl); m.moe_hidden = (int)rd32(pl + 8);
                if ((int)rd32(pl + 4) != 1) return "mmcf: only top-1 MoE is supported";
                if (!(rd32(pl + 12) & 1)) return "mmcf: MoE without a normalised top-k gate";
            } else if (key == 14) {
                return "mmcf: hybrid (conv) containers are not supported by this engine";
            } else if (key == 15) {
                m.hid_scale.assign(pl, pl + len);
            } else if (key == 16) {
                return "mmcf: RWKV-7 containers are not supported by this engine";
            } else if (key == 17 && len >= 1 && pl[0]) {
                return "mmcf: a logit-shift (key 17) container is not supported by this engine";
            } else if (key == 18 && len >= 4 && len % 4 == 0) {
                m.rope_factors.resize(len / 4);
                for (uint32_t i = 0; i < len / 4; ++i) m.rope_factors[i] = rdf(pl + 4 * i);
            }
        }
        p += 8 + len;
    }
    if (!have_model || m.dim <= 0 || m.heads <= 0 || m.kv_heads <= 0 || m.layers <= 0 || m.vocab <= 0 ||
        m.heads % m.kv_heads || m.dim % m.heads)
        return "mmcf: missing or inconsistent model metadata";
    m.head_dim = m.dim / m.heads;                               // model.cpp:791-792
    m.kv_dim = m.kv_heads * m.head_dim;
    if (m.head_dim % 2) return "mmcf: odd head_dim";
    if (!split) return "mmcf: fused-W13 containers (the CPU FFN path) are not supported by this engine";
    if (!m.rope_factors.empty() && (int)m.rope_factors.size() != m.head_dim / 2) return "mmcf: rope factor count";

    std::vector<Rec> recs(ntens);
    for (uint32_t i = 0; i < ntens; ++i) {
        const uint8_t* r = h + table_off + (uint64_t)i * rsize;
        Rec& o = recs[i];
        o.id = rd16(r); o.dtype = r[2]; o.group = r[4];
        o.rows = rd32(r + 6); o.cols = rd32(r + 10);
        const uint64_t off = rd64(r + 14);
        o.bytes = rd64(r + 22);
        o.scale = rdf(r + 34);
        o.aux = m.version >= 3 ? rd16(r + 38) : 0;
        if (data_off + off + o.bytes > sz) return "mmcf: tensor " + std::to_string(i) + " overruns the file";
        o.data = h + data_off + off;
    }
    std::map<uint32_t, const Rec*> parts[4];
    for (const Rec& r : recs) parts[r.id >> 14][r.key() & ~(3u << 14)] = &r;
    auto part = [&](const Rec& r, int k) -> const Rec* {
        auto it = parts[k].find(r.key() & ~(3u << 14));
        return it == parts[k].end() ? nullptr : it->second;
    };
    const int L = m.layers, E = m.experts, D = m.dim, hd = m.head_dim;
    m.qkv.resize(L); m.wo.resize(L); m.w1.resize(L); m.w3.resize(L); m.w2.resize(L); m.router.resize(L);
    if (E) m.moe.resize((size_t)L * E * 3);
    std::map<int, HMat> tiles;
    std::string err;
    for (const Rec& r : recs) {
        const int kind = r.id & 0xFF, layer = (r.id >> 8) & 0x3F, prt = r.id >> 14;
        if (prt) continue;
        HMat* dst = nullptr;
        switch (kind) {
            case 1:
                if (r.dtype != 3 || (int)r.cols != D) return "mmcf: only q8 embeddings are supported by this engine";
                m.vocab = (int)r.rows;
                m.emb.assign((const int8_t*)r.data, (const int8_t*)r.data + (size_t)r.rows * D);
                continue;
            case 2: m.emb_scale = f32s(r, r.rows, err); break;
            case 3: m.rms_att = f32s(r, (size_t)L * D, err); break;
            case 4: m.rms_ffn = f32s(r, (size_t)L * D, err); break;
            case 5: m.rms_final = f32s(r, (size_t)D, err); break;
            case 6: m.q_norm = f32s(r, (size_t)L * hd, err); break;
            case 7: m.k_norm = f32s(r, (size_t)L * hd, err); break;
            case 8: return "mmcf: i16 embeddings are not supported by this engine";
            case 0x14: return "mmcf: fused W13 is not supported by this engine";
            default: break;
        }
        if (!err.empty()) return "mmcf: " + err;
        if (kind < 0x10) continue;
        const bool is_expert = E > 0 && (kind == 0x12 || kind == 0x13 || kind == 0x15);
        if (kind == 0x20) dst = &tiles[layer];
        else if (layer >= L) continue;
        else if (is_expert) {
            if (r.aux >= E) return "mmcf: expert index out of range";
            dst = &m.moe[((size_t)layer * E + r.aux) * 3 + (kind == 0x12 ? 0 : kind == 0x13 ? 1 : 2)];
        } else if (kind == 0x10) dst = &m.qkv[layer];
        else if (kind == 0x11) dst = &m.wo[layer];
        else if (kind == 0x12) dst = &m.w1[layer];
        else if (kind == 0x13) dst = &m.w3[layer];
        else if (kind == 0x15) dst = &m.w2[layer];
        else if (kind == 0x16) dst = &m.router[layer];
        else continue;
        err = read_mat(r, part(r, 1), part(r, 2), part(r, 3), *dst);
        if (!err.empty()) return "mmcf: " + err;
    }
    if (m.emb.empty() || m.emb_scale.size() != (size_t)m.vocab || m.rms_att.empty() || m.rms_ffn.empty() ||
        m.rms_final.empty())
        return "mmcf: missing required tensors";
    if (m.qk_norm && (m.q_norm.empty() || m.k_norm.empty())) return "mmcf: qk-norm weights missing";
    if (!tiles.empty()) {
        for (int t = 0; t < (int)tiles.size(); ++t) {
            if (!tiles.count(t)) return "mmcf: logits tiles are not contiguous";
            m.tiles.push_back(std::move(tiles[t]));
        }
    } else {                                                  // head dedup, model.cpp:1565-1590
        float unit = 0.0f;
        for (float s : m.emb_scale) if (s > unit) unit = s;
        if (!(unit > 0.0f)) return "mmcf: a dedup head needs embedding scales";
        m.head_dedup = true;
        for (int st = 0; st < m.vocab; st += kLogitsGrid) {
            HMat t;
            t.rows = std::min(kLogitsGrid, m.vocab - st); t.cols = D; t.wtype = W_Q8; t.scale = unit;
            t.lev.assign(m.emb.begin() + (size_t)st * D, m.emb.begin() + (size_t)(st + t.rows) * D);
            t.plane.resize(t.rows);
            for (int r = 0; r < t.rows; ++r) t.plane[r] = m.emb_scale[st + r] / unit;
            t.p16 = plane16(t.plane);
            m.tiles.push_back(std::move(t));
        }
    }
    int vt = 0;
    for (const HMat& t : m.tiles) {
        if (t.cols != D || t.wtype != W_Q8) return "mmcf: logits tiles must be q8 rows of the model width";
        vt += t.rows;
    }
    if (vt != m.vocab) return "mmcf: logits tiles do not cover the vocabulary";
    for (int l = 0; l < L; ++l) {
        if (m.qkv[l].rows != D + 2 * m.kv_dim || m.qkv[l].cols != D || m.wo[l].rows != D || m.wo[l].cols != D)
            return "mmcf: attention matrix shape at layer " + std::to_string(l);
        if (m.qkv[l].wtype == W_I16 || m.wo[l].wtype != m.qkv[l].wtype) return "mmcf: unsupported attention weight type";
        if (E) {
            if (m.router[l].wtype != W_I16 || m.router[l].rows != E || m.router[l].cols != D) return "mmcf: router shape";
            for (int e = 0; e < E; ++e) {
                const HMat* x = &m.moe[((size_t)l * E + e) * 3];
                if (x[0].rows != m.moe_hidden || x[1].rows != m.moe_hidden || x[2].cols != m.moe_hidden ||
                    x[0].cols != D || x[2].rows != D)
                    return "mmcf: expert shape";
            }
        } else if (m.w1[l].rows != m.hidden || m.w3[l].rows != m.hidden || m.w2[l].cols != m.hidden ||
                   m.w1[l].cols != D || m.w2[l].rows != D) {
            return "mmcf: ffn shape at layer " + std::to_string(l);
        }
    }
    // Metadata key 15: fold 2^hs into every w2 (model.cpp:407-429).
    for (int l = 0; l < L && l < (int)m.hid_scale.size(); ++l) {
        const int k = m.hid_scale[l];
        if (k <= 0) continue;
        if (k > 5) return "mmcf: hidden scale exponent above 5";
        const float s = (float)(1u << k);
        if (E) for (int e = 0; e < E; ++e) m.moe[((size_t)l * E + e) * 3 + 2].scale *= s;
        else m.w2[l].scale *= s;
    }
    return "";
}

std::string load_mmcf(const std::string& path, HModel& m) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return "cannot open model: " + path;
    struct stat st {};
    if (fstat(fileno(f), &st) != 0) { fclose(f); return "cannot stat model: " + path; }
    std::vector<uint8_t> buf((size_t)st.st_size);
    if (fread(buf.data(), 1, buf.size(), f) != buf.size()) { fclose(f); return "short read: " + path; }
    fclose(f);
    std::string e = load_mmcf_bytes(buf.data(), buf.size(), m);
    m.source_size = (uint64_t)st.st_size;
    m.source_mtime = (uint64_t)st.st_mtime;
    return e;
}

}  // namespace vc4
