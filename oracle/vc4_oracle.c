/*
 * vc4_oracle.c -- CPU oracle for the quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against and
 * the CPU baseline bench.py times.  Nothing in the product links or calls it.
 *
 * Each function cites the reference file:line whose behaviour it restates
 * (paths are relative to the reference project's root).  The canonical
 * arithmetic is described in vc4_oracle.h.  Build with -ffp-contract=off:
 * every float expression here is meant to round after each operation.
 */
#include "vc4_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* Small helpers                                                              */
/* ------------------------------------------------------------------------- */

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }
static float rdf(const uint8_t* p) { float f; uint32_t u = rd32(p); memcpy(&f, &u, 4); return f; }

static uint32_t crc32_buf(const uint8_t* p, size_t n) {
    static uint32_t table[256];
    static int init = 0;
    if (!init) {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : (c >> 1);
            table[i] = c;
        }
        init = 1;
    }
    uint32_t crc = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; ++i) crc = table[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
    return crc ^ 0xFFFFFFFFu;
}

/* q16 host quantisation: lrintf(v*256) clamped to int16 (common.h:188-193). */
int16_t orc_q16(float v) {
    float s = v * 256.0f;
    long q = lrintf(s);
    if (q < -32768) q = -32768;
    if (q > 32767) q = 32767;
    return (int16_t)q;
}
static float q16f(float v) { return (float)orc_q16(v) / 256.0f; }

/* q16 shader store: clamp(floor(v*256+0.5)) (xformat.cpp x_q16enc / x_st2). */
static int32_t q16s(float v) {
    float s = v * 256.0f;
    float f = floorf(s + 0.5f);
    if (f < -32768.0f) f = -32768.0f;
    if (f > 32767.0f) f = 32767.0f;
    return (int32_t)f;
}

/*
 * Portable exp: Cody & Waite (1980) range reduction x = k*ln2 + r with ln2
 * split into a 16-bit-mantissa high part and a low correction, then the
 * degree-7 Taylor series of e^r on |r| <= ln2/2 in Horner form with fused
 * multiply-adds, and the exact scaling by 2^k through the exponent field.
 * The CUDA kernels evaluate the identical sequence of IEEE operations, so
 * both sides produce the same bits.  (The reference's own portable exp,
 * shaders.cpp:95-103, is a degree-6 Taylor on the same reduction.)
 */
static float pow2i(int k) { /* 2^k for -126 <= k <= 127 */
    uint32_t u = (uint32_t)(k + 127) << 23;
    float f; memcpy(&f, &u, 4); return f;
}
void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

float orc_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541016f) return 0.0f;
    const float k = rintf(x * 1.44269502162933349609375f);           /* x / ln2 */
    float r = fmaf(-k, 0.693145751953125f, x);                        /* ln2 high */
    r = fmaf(-k, 1.428606765330187045037746429443359375e-06f, r);     /* ln2 low  */
    float p = 1.98412698412698412698e-4f;                             /* 1/7! */
    p = fmaf(p, r, 1.38888888888888888889e-3f);                       /* 1/6! */
    p = fmaf(p, r, 8.33333333333333333333e-3f);                       /* 1/5! */
    p = fmaf(p, r, 4.16666666666666666667e-2f);                       /* 1/4! */
    p = fmaf(p, r, 1.66666666666666666667e-1f);                       /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)k;
    if (ki > 127) { p = p * 2.0f; ki -= 1; }
    if (ki < -126) return (p * pow2i(ki + 64)) * pow2i(-64);
    return p * pow2i(ki);
}

/* ------------------------------------------------------------------------- */
/* Model                                                                      */
/* ------------------------------------------------------------------------- */

typedef struct {
    int rows, cols, wtype, groups;
    float scale;      /* q8/i16: ws; t3: record scale*127; q4: ps */
    int8_t* lev;      /* q8 and t3 signed levels, rows*cols */
    uint8_t* nib;     /* q4 nibble values, rows*cols */
    int16_t* s16;     /* q4 group scale, rows*groups */
    int16_t* m16;     /* q4 group min, rows*groups */
    int16_t* w16;     /* i16 */
    uint16_t* p16;    /* row plane quantised to 16 bits, or NULL */
    float* plane;     /* the container's f32 plane, or NULL */
} omat;

typedef struct { omat w1, w3, w2; } oexpert;

struct orc_model {
    orc_info in;
    uint8_t* file;
    size_t fsize;
    int8_t* emb;          /* vocab*dim signed levels */
    float* emb_scale;     /* vocab */
    float *rms_att, *rms_ffn, *rms_final, *q_norm, *k_norm, *rope_factors;
    int n_rope_factors;
    uint8_t hid_scale[64];
    omat *qkv, *wo, *w1, *w3, *w2, *router;  /* per layer */
    oexpert* moe;                             /* layers*experts */
    omat* tiles;
    int n_tiles;
};

static void mat_free(omat* m) {
    free(m->lev); free(m->nib); free(m->s16); free(m->m16); free(m->w16);
    free(m->p16); free(m->plane);
    memset(m, 0, sizeof(*m));
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    int L = m->in.layers;
    if (m->qkv) for (int l = 0; l < L; ++l) {
        mat_free(&m->qkv[l]); mat_free(&m->wo[l]); mat_free(&m->w1[l]);
        mat_free(&m->w3[l]); mat_free(&m->w2[l]); mat_free(&m->router[l]);
    }
    if (m->moe) for (int i = 0; i < L * m->in.experts; ++i) {
        mat_free(&m->moe[i].w1); mat_free(&m->moe[i].w3); mat_free(&m->moe[i].w2);
    }
    for (int t = 0; t < m->n_tiles; ++t) mat_free(&m->tiles[t]);
    free(m->qkv); free(m->wo); free(m->w1); free(m->w3); free(m->w2); free(m->router);
    free(m->moe); free(m->tiles);
    free(m->emb); free(m->emb_scale); free(m->rms_att); free(m->rms_ffn);
    free(m->rms_final); free(m->q_norm); free(m->k_norm); free(m->rope_factors);
    free(m->file);
    free(m);
}

typedef struct {
    uint16_t id; uint8_t dtype, group; uint32_t rows, cols; uint64_t off, bytes;
    float scale; uint16_t aux;
} orec;

static int fail(char* err, int errlen, const char* msg) {
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", msg);
    return ORC_EFORMAT;
}

/* Row plane to 16 bits, two rows a texel in the reference (gpu_upload.cpp:32-58):
   q = clamp(lrint(plane*65536), 0, 65535). */
static uint16_t* plane16(const float* plane, int rows) {
    uint16_t* p = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)rows);
    for (int r = 0; r < rows; ++r) {
        long q = lrint((double)plane[r] * 65536.0);
        if (q < 0) q = 0;
        if (q > 65535) q = 65535;
        p[r] = (uint16_t)q;
    }
    return p;
}

/* A matrix record into an omat (model.cpp:894-975 as_i16/as_q8/as_t3, and the
   q4 parts map at model.cpp:976-1056). */
static int load_mat(orc_model* m, const orec* r, const orec* p1, const orec* p2,
                    const orec* p3, omat* o, char* err, int errlen) {
    const uint8_t* d = m->file + 0; /* data pointers are resolved by caller */
    (void)d;
    memset(o, 0, sizeof(*o));
    o->rows = (int)r->rows; o->cols = (int)r->cols;
    const size_t n = (size_t)r->rows * r->cols;
    const uint8_t* body = (const uint8_t*)(uintptr_t)r->off;   /* resolved absolute */
    if (r->dtype == 2 || r->dtype == 3) {            /* q8u8 pre-biased / q8i8 */
        if (r->bytes < n) return fail(err, errlen, "q8 tensor too short");
        o->wtype = ORC_W_Q8; o->scale = r->scale;
        o->lev = (int8_t*)malloc(n);
        for (size_t i = 0; i < n; ++i)
            o->lev[i] = r->dtype == 2 ? (int8_t)((int)body[i] - 128) : (int8_t)body[i];
    } else if (r->dtype == 1) {                      /* i16 */
        if (r->bytes < n * 2) return fail(err, errlen, "i16 tensor too short");
        o->wtype = ORC_W_I16; o->scale = r->scale;
        o->w16 = (int16_t*)malloc(n * 2);
        for (size_t i = 0; i < n; ++i) o->w16[i] = (int16_t)rd16(body + 2 * i);
    } else if (r->dtype == 7) {                      /* t3 */
        const size_t stride = (size_t)((r->cols + 7) / 8) * 4;
        if (r->bytes < (size_t)((r->rows + 1) / 2) * stride) return fail(err, errlen, "t3 tensor too short");
        o->wtype = ORC_W_T3;
        o->scale = r->scale * 127.0f;                /* model.cpp:925-932 */
        o->lev = (int8_t*)malloc(n);
        for (uint32_t y = 0; y < (r->rows + 1) / 2; ++y) {
            const uint8_t* band = body + (size_t)y * stride;
            for (int half = 0; half < 2; ++half) {
                const uint32_t row = 2 * y + (uint32_t)half;
                if (row >= r->rows) break;
                for (uint32_t x = 0; x < r->cols; ++x) {
                    const uint8_t byte = band[(size_t)(x >> 3) * 4 + (size_t)half * 2 + ((x >> 2) & 1)];
                    const unsigned code = (byte >> (2 * (x & 3))) & 3u;
                    o->lev[(size_t)row * r->cols + x] = (code & 1u) ? ((code & 2u) ? -1 : 1) : 0;
                }
            }
        }
    } else if (r->dtype == 4) {                      /* q4 body + parts 1, 2 */
        if (!p1 || !p2) return fail(err, errlen, "q4 matrix without scale/min planes");
        if (r->cols % 32) return fail(err, errlen, "q4 cols not a multiple of 32");
        if (r->bytes < n / 2) return fail(err, errlen, "q4 tensor too short");
        o->wtype = ORC_W_Q4; o->scale = r->scale; o->groups = (int)(r->cols / 32);
        const size_t ng = (size_t)r->rows * o->groups;
        if (p1->rows != r->rows || p1->cols != (uint32_t)o->groups || p1->bytes < ng * 2 ||
            p2->rows != r->rows || p2->cols != (uint32_t)o->groups || p2->bytes < ng * 2)
            return fail(err, errlen, "q4 plane shape mismatch");
        o->nib = (uint8_t*)malloc(n);
        for (size_t i = 0; i < n; ++i) {
            const uint8_t b = body[i / 2];
            o->nib[i] = (i & 1) ? (b >> 4) : (b & 15);   /* low nibble = even column */
        }
        const uint8_t* ps = (const uint8_t*)(uintptr_t)p1->off;
        const uint8_t* pm = (const uint8_t*)(uintptr_t)p2->off;
        o->s16 = (int16_t*)malloc(ng * 2); o->m16 = (int16_t*)malloc(ng * 2);
        for (size_t i = 0; i < ng; ++i) { o->s16[i] = (int16_t)rd16(ps + 2 * i); o->m16[i] = (int16_t)rd16(pm + 2 * i); }
    } else {
        char msg[96]; snprintf(msg, sizeof msg, "unsupported matrix dtype %d", r->dtype);
        return fail(err, errlen, msg);
    }
    if (p3) {                                         /* per-row plane (part 3) */
        if (p3->rows != r->rows || p3->bytes != (uint64_t)r->rows * 4)
            return fail(err, errlen, "row plane shape mismatch");
        const uint8_t* pp = (const uint8_t*)(uintptr_t)p3->off;
        o->plane = (float*)malloc(sizeof(float) * r->rows);
        for (uint32_t i = 0; i < r->rows; ++i) o->plane[i] = rdf(pp + 4 * i);
        o->p16 = plane16(o->plane, (int)r->rows);
    }
    return ORC_OK;
}

static const orec* find_part(const orec* recs, int n, const orec* base, int part) {
    const uint32_t want = ((uint32_t)base->aux << 16) | (uint32_t)((base->id & 0x3FFF) | (part << 14));
    for (int i = 0; i < n; ++i) {
        const uint32_t key = ((uint32_t)recs[i].aux << 16) | (uint32_t)recs[i].id;
        if (key == want) return &recs[i];
    }
    return NULL;
}

static float* f32_copy(const orec* r, size_t count) {
    if (r->dtype != 0 || r->bytes < count * 4) return NULL;
    float* v = (float*)malloc(count * 4);
    const uint8_t* p = (const uint8_t*)(uintptr_t)r->off;
    for (size_t i = 0; i < count; ++i) v[i] = rdf(p + 4 * i);
    return v;
}

/* MMCF v2/v3 reader: header (model.cpp:614-660), metadata TLVs
   (model.cpp:662-760), tensor table (model.cpp:873-1560). */
int orc_model_load(const char* path, orc_model** out, char* err, int errlen) {
    *out = NULL;
    FILE* f = fopen(path, "rb");
    if (!f) { if (err) snprintf(err, (size_t)errlen, "cannot open %s", path); return ORC_EIO; }
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz < 64) { fclose(f); return fail(err, errlen, "mmcf: truncated header"); }
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->file = (uint8_t*)malloc((size_t)sz);
    m->fsize = (size_t)sz;
    if (fread(m->file, 1, (size_t)sz, f) != (size_t)sz) { fclose(f); orc_model_free(m); return ORC_EIO; }
    fclose(f);
    const uint8_t* h = m->file;
    int rc = ORC_EFORMAT;
    if (memcmp(h, "MMCF", 4) != 0) { fail(err, errlen, "not an MMCF container"); goto bad; }
    const int version = rd16(h + 4);
    if (version != 2 && version != 3) { fail(err, errlen, "mmcf: unsupported version"); goto bad; }
    if (rd16(h + 6) != 64) { fail(err, errlen, "mmcf: bad header size"); goto bad; }
    const uint32_t ntens = rd32(h + 8), meta_off = rd32(h + 16), meta_size = rd32(h + 20);
    const uint64_t data_off = rd64(h + 24), file_size = rd64(h + 32);
    const int rsize = version >= 3 ? 64 : 48;
    if (file_size != (uint64_t)sz) { fail(err, errlen, "mmcf: size field does not match the file"); goto bad; }
    { const uint32_t stored = rd32(h + 40);
      if (stored && stored != crc32_buf(h, 40)) { fail(err, errlen, "mmcf: header crc mismatch"); goto bad; } }
    if ((uint64_t)meta_off + meta_size > (uint64_t)sz || data_off > (uint64_t)sz ||
        data_off < (uint64_t)ntens * rsize) { fail(err, errlen, "mmcf: bad section offsets"); goto bad; }
    const uint64_t table_off = data_off - (uint64_t)ntens * rsize;
    if (table_off < (uint64_t)meta_off + meta_size || (table_off % 16) != 0) {
        fail(err, errlen, "mmcf: tensor table does not follow the metadata block"); goto bad; }

    orc_info* in = &m->in;
    in->version = version;
    in->rms_eps = 1e-5f;
    int have_model = 0, split = 0;
    for (uint64_t p = meta_off; p + 8 <= (uint64_t)meta_off + meta_size;) {
        const uint16_t key = rd16(h + p), type = rd16(h + p + 2);
        const uint32_t len = rd32(h + p + 4);
        const uint8_t* pl = h + p + 8;
        if (p + 8 + len > (uint64_t)meta_off + meta_size) { fail(err, errlen, "mmcf: TLV overruns the block"); goto bad; }
        if (key == 1 && type == 1 && len >= 28) {
            in->dim = (int)rd32(pl); in->hidden = (int)rd32(pl + 4); in->layers = (int)rd32(pl + 8);
            in->heads = (int)rd32(pl + 12); in->kv_heads = (int)rd32(pl + 16);
            in->vocab = (int)rd32(pl + 20); in->seq = (int)rd32(pl + 24);
            have_model = 1;
        } else if (key == 2 && type == 1 && len >= 8) {
            in->rope_theta = rdf(pl); in->rope_half = pl[4] != 0; in->qk_norm = pl[5] != 0;
        } else if (key == 3 && type == 1 && len >= 4) {
            split = pl[3];
        } else if (key == 11 && type == 1 && len >= 4) {
            float e = rdf(pl); if (e > 0.0f) in->rms_eps = e;
        } else if (key == 12 && type == 1 && len >= 1) {
            if (pl[0] == 1) { fail(err, errlen, "q24 residual containers are not supported"); rc = ORC_EUNSUPPORTED; goto bad; }
        } else if (key == 13 && type == 1 && len >= 16) {
            in->experts = (int)rd32(pl); in->moe_hidden = (int)rd32(pl + 8);
            if ((int)rd32(pl + 4) != 1) { fail(err, errlen, "only top-1 MoE is supported"); rc = ORC_EUNSUPPORTED; goto bad; }
        } else if (key == 14 && type == 1) {
            fail(err, errlen, "hybrid (conv) containers are not supported"); rc = ORC_EUNSUPPORTED; goto bad;
        } else if (key == 15 && type == 1 && len >= 1) {
            for (uint32_t i = 0; i < len && i < 64; ++i) m->hid_scale[i] = pl[i];
        } else if (key == 16) {
            fail(err, errlen, "RWKV containers are not supported"); rc = ORC_EUNSUPPORTED; goto bad;
        } else if (key == 18 && type == 1 && len >= 4 && (len % 4) == 0) {
            m->n_rope_factors = (int)(len / 4);
            m->rope_factors = (float*)malloc(len);
            for (uint32_t i = 0; i < len / 4; ++i) m->rope_factors[i] = rdf(pl + 4 * i);
        }
        p += 8 + len;
    }
    if (!have_model || in->dim <= 0 || in->heads <= 0 || in->kv_heads <= 0 || in->layers <= 0 ||
        in->layers > 64 || in->vocab <= 0) { fail(err, errlen, "mmcf: missing or bad model metadata"); goto bad; }
    in->head_dim = in->dim / in->heads;                         /* model.cpp:791-792 */
    in->kv_dim = in->kv_heads * in->head_dim;
    if (!split) { fail(err, errlen, "fused-W13 containers (CPU FFN path) are not supported"); rc = ORC_EUNSUPPORTED; goto bad; }
    if (m->n_rope_factors && m->n_rope_factors != in->head_dim / 2) { fail(err, errlen, "rope factor count"); goto bad; }

    orec* recs = (orec*)calloc(ntens ? ntens : 1, sizeof(orec));
    for (uint32_t i = 0; i < ntens; ++i) {
        const uint8_t* r = h + table_off + (uint64_t)i * rsize;
        orec* o = &recs[i];
        o->id = rd16(r); o->dtype = r[2]; o->group = r[4];
        o->rows = rd32(r + 6); o->cols = rd32(r + 10);
        o->off = rd64(r + 14); o->bytes = rd64(r + 22);
        o->scale = rdf(r + 34);
        o->aux = version >= 3 ? rd16(r + 38) : 0;
        if (data_off + o->off + o->bytes > (uint64_t)sz) { free(recs); fail(err, errlen, "mmcf: tensor overruns the file"); goto bad; }
        o->off = (uint64_t)(uintptr_t)(h + data_off + o->off);   /* absolute address */
    }
    const int L = in->layers, E = in->experts, D = in->dim, hd = in->head_dim;
    m->qkv = (omat*)calloc((size_t)L, sizeof(omat)); m->wo = (omat*)calloc((size_t)L, sizeof(omat));
    m->w1 = (omat*)calloc((size_t)L, sizeof(omat)); m->w3 = (omat*)calloc((size_t)L, sizeof(omat));
    m->w2 = (omat*)calloc((size_t)L, sizeof(omat)); m->router = (omat*)calloc((size_t)L, sizeof(omat));
    if (E > 0) m->moe = (oexpert*)calloc((size_t)L * E, sizeof(oexpert));
    omat tiles[256];
    memset(tiles, 0, sizeof tiles);
    int max_tile = -1;
    for (uint32_t i = 0; i < ntens; ++i) {
        const orec* r = &recs[i];
        const int kind = r->id & 0xFF, layer = (r->id >> 8) & 0x3F, part = r->id >> 14;
        if (part != 0) continue;
        omat* dst = NULL;
        const int e = r->aux;
        if (kind == 1) {
            if (r->dtype != 3 || r->cols != (uint32_t)D) { free(recs); fail(err, errlen, "only q8 embeddings are supported"); rc = ORC_EUNSUPPORTED; goto bad; }
            in->vocab = (int)r->rows;
            m->emb = (int8_t*)malloc((size_t)r->rows * D);
            memcpy(m->emb, (const void*)(uintptr_t)r->off, (size_t)r->rows * D);
            continue;
        }
        if (kind == 2) { m->emb_scale = f32_copy(r, r->rows); continue; }
        if (kind == 3) { m->rms_att = f32_copy(r, (size_t)L * D); continue; }
        if (kind == 4) { m->rms_ffn = f32_copy(r, (size_t)L * D); continue; }
        if (kind == 5) { m->rms_final = f32_copy(r, (size_t)D); continue; }
        if (kind == 6) { m->q_norm = f32_copy(r, (size_t)L * hd); continue; }
        if (kind == 7) { m->k_norm = f32_copy(r, (size_t)L * hd); continue; }
        if (kind == 8) { free(recs); fail(err, errlen, "i16 embeddings are not supported"); rc = ORC_EUNSUPPORTED; goto bad; }
        if (kind == 0x14) { free(recs); fail(err, errlen, "fused W13 is not supported"); rc = ORC_EUNSUPPORTED; goto bad; }
        if (layer >= L && kind != 0x20) continue;
        const int is_expert = E > 0 && (kind == 0x12 || kind == 0x13 || kind == 0x15);
        if (is_expert) {
            if (e >= E) { free(recs); fail(err, errlen, "expert index out of range"); goto bad; }
            oexpert* x = &m->moe[(size_t)layer * E + e];
            dst = kind == 0x12 ? &x->w1 : kind == 0x13 ? &x->w3 : &x->w2;
        } else if (kind == 0x10) dst = &m->qkv[layer];
        else if (kind == 0x11) dst = &m->wo[layer];
        else if (kind == 0x12) dst = &m->w1[layer];
        else if (kind == 0x13) dst = &m->w3[layer];
        else if (kind == 0x15) dst = &m->w2[layer];
        else if (kind == 0x16) dst = &m->router[layer];
        else if (kind == 0x20) {
            if (layer >= 256) continue;
            dst = &tiles[layer];
            if (layer > max_tile) max_tile = layer;
        } else continue;
        const orec* p1 = find_part(recs, (int)ntens, r, 1);
        const orec* p2 = find_part(recs, (int)ntens, r, 2);
        const orec* p3 = find_part(recs, (int)ntens, r, 3);
        int lrc = load_mat(m, r, p1, p2, p3, dst, err, errlen);
        if (lrc != ORC_OK) { free(recs); rc = lrc; goto bad; }
    }
    free(recs);
    if (!m->emb || !m->emb_scale || !m->rms_att || !m->rms_ffn || !m->rms_final) {
        fail(err, errlen, "mmcf: missing required tensors"); goto bad; }
    if (in->qk_norm && (!m->q_norm || !m->k_norm)) { fail(err, errlen, "mmcf: qk_norm without norms"); goto bad; }
    /* Logits tiles, or the dedup head built from the embedding rows
       (model.cpp:1565-1590): plane = emb_scale / unit, unit = max scale. */
    if (max_tile >= 0) {
        m->n_tiles = max_tile + 1;
        m->tiles = (omat*)calloc((size_t)m->n_tiles, sizeof(omat));
        memcpy(m->tiles, tiles, sizeof(omat) * (size_t)m->n_tiles);
    } else {
        float unit = 0.0f;
        for (int v = 0; v < in->vocab; ++v) if (m->emb_scale[v] > unit) unit = m->emb_scale[v];
        if (unit <= 0.0f) { fail(err, errlen, "mmcf: a dedup head needs embedding scales"); goto bad; }
        m->n_tiles = (in->vocab + 1535) / 1536;
        m->tiles = (omat*)calloc((size_t)m->n_tiles, sizeof(omat));
        for (int t = 0; t < m->n_tiles; ++t) {
            const int st = t * 1536, rows = in->vocab - st < 1536 ? in->vocab - st : 1536;
            omat* o = &m->tiles[t];
            o->rows = rows; o->cols = D; o->wtype = ORC_W_Q8; o->scale = unit;
            o->lev = (int8_t*)malloc((size_t)rows * D);
            memcpy(o->lev, m->emb + (size_t)st * D, (size_t)rows * D);
            o->plane = (float*)malloc(sizeof(float) * rows);
            for (int r2 = 0; r2 < rows; ++r2) o->plane[r2] = m->emb_scale[st + r2] / unit;
            o->p16 = plane16(o->plane, rows);
        }
    }
    for (int t = 0; t < m->n_tiles; ++t)
        if (m->tiles[t].rows <= 0 || m->tiles[t].cols != D) { fail(err, errlen, "mmcf: logits tile shape"); goto bad; }
    /* Shape checks the layer loop relies on. */
    for (int l = 0; l < L; ++l) {
        if (m->qkv[l].rows != D + 2 * in->kv_dim || m->qkv[l].cols != D ||
            m->wo[l].rows != D || m->wo[l].cols != D) { fail(err, errlen, "mmcf: attention matrix shape"); goto bad; }
        if (E > 0) {
            if (m->router[l].wtype != ORC_W_I16 || m->router[l].rows != E) { fail(err, errlen, "mmcf: router"); goto bad; }
            for (int x = 0; x < E; ++x) {
                oexpert* ex = &m->moe[(size_t)l * E + x];
                if (ex->w1.rows != in->moe_hidden || ex->w3.rows != in->moe_hidden || ex->w2.cols != in->moe_hidden ||
                    ex->w2.rows != D) { fail(err, errlen, "mmcf: expert shape"); goto bad; }
            }
        } else if (m->w1[l].rows != in->hidden || m->w3[l].rows != in->hidden ||
                   m->w2[l].cols != in->hidden || m->w2[l].rows != D) { fail(err, errlen, "mmcf: ffn shape"); goto bad; }
    }
    in->ffn_width = E > 0 ? in->moe_hidden : in->hidden;
    in->wtype = m->wo[0].wtype;
    /* FFN chunking: a width above 2048 runs as two halves (model.cpp:217-277). */
    in->ffn_chunked = in->ffn_width > 2048;
    in->ffn_chunk = in->ffn_chunked ? (in->ffn_width + 1) / 2 : in->ffn_width;
    if (in->ffn_chunked && in->wtype == ORC_W_Q4 && (in->ffn_chunk % 32)) { fail(err, errlen, "q4 chunk not group aligned"); goto bad; }
    /* Metadata key 15: fold 2^hs into every w2 (model.cpp:407-429). */
    for (int l = 0; l < L; ++l) {
        const int k = m->hid_scale[l];
        if (k <= 0) continue;
        const float s = (float)(1u << k);
        if (E > 0) for (int x = 0; x < E; ++x) m->moe[(size_t)l * E + x].w2.scale *= s;
        else m->w2[l].scale *= s;
    }
    in->n_logit_tiles = m->n_tiles;
    *out = m;
    return ORC_OK;
bad:
    orc_model_free(m);
    return rc;
}

int orc_model_info(const orc_model* m, orc_info* info) { *info = m->in; return ORC_OK; }

void orc_rope_tables(float theta, int head_dim, int seq, const float* factors,
                     float* cos_out, float* sin_out) {
    /* session.cpp:188-202 */
    const int half = head_dim / 2;
    for (int p = 0; p < seq; ++p) {
        for (int i = 0; i < half; ++i) {
            float freq = 1.0f / powf(theta, (2.0f * i) / head_dim);
            if (factors) freq /= factors[i];
            float a = p * freq;
            cos_out[(size_t)p * half + i] = cosf(a);
            sin_out[(size_t)p * half + i] = sinf(a);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Matvec family                                                              */
/* ------------------------------------------------------------------------- */

/* The per-row scale the shaders multiply by: `ws`, or the 16-bit row plane
   times the unit, (p16*ws)*(1/65536) (shaders.cpp:339-372 wsr). */
static float row_scale(const omat* w, int r) {
    if (w->p16) {
        float a = (float)w->p16[r] * w->scale;
        return a * (1.0f / 65536.0f);
    }
    return w->scale;
}

/* Epilogue of every matvec: floor(S*sc + 0.5) clamped to the q16 rail. */
static int32_t mv_epilogue(int64_t S, double sc) {
    double p = (double)S * sc;
    double v = floor(p + 0.5);
    if (v < -32768.0) v = -32768.0;
    if (v > 32767.0) v = 32767.0;
    return (int32_t)v;
}

/* Exact integer dot of row r over columns [c0, c1) with xq[0 .. c1-c0).
   q8 / t3: sum lev*x; i16: sum w*x; q4: sum_g s16*N_g + m16*X_g with
   N_g = sum nib*x, X_g = sum x (shaders.cpp:1249-1274 regrouped exactly). */
static int64_t row_dot(const omat* w, int r, int c0, int c1, const int16_t* xq) {
    const size_t base = (size_t)r * w->cols;
    int64_t S = 0;
    if (w->wtype == ORC_W_Q8 || w->wtype == ORC_W_T3) {
        const int8_t* lv = w->lev + base + c0;
        const int n = c1 - c0;
        for (int b = 0; b < n; b += 256) {
            const int e = b + 256 < n ? b + 256 : n;
            int32_t acc = 0;
            for (int c = b; c < e; ++c) acc += (int32_t)lv[c] * (int32_t)xq[c];
            S += acc;
        }
    } else if (w->wtype == ORC_W_I16) {
        const int16_t* wv = w->w16 + base + c0;
        for (int c = 0; c < c1 - c0; ++c) S += (int64_t)wv[c] * xq[c];
    } else {
        const uint8_t* nb = w->nib + base;
        for (int g = c0 / 32; g < c1 / 32; ++g) {
            int32_t N = 0, X = 0;
            for (int j = 0; j < 32; ++j) {
                const int c = g * 32 + j;
                N += (int32_t)nb[c] * xq[c - c0];
                X += xq[c - c0];
            }
            S += (int64_t)w->s16[(size_t)r * w->groups + g] * N + (int64_t)w->m16[(size_t)r * w->groups + g] * X;
        }
    }
    return S;
}

/* The reference shaders' own fp32 accumulation, four columns a step
   (shaders.cpp:375-417, 468-525), for ORC_LITERAL.  q4 and i16 stay exact. */
static int32_t row_literal(const omat* w, int r, int c0, int c1, const int16_t* xq) {
    if (w->wtype != ORC_W_Q8 && w->wtype != ORC_W_T3)
        return mv_epilogue(row_dot(w, r, c0, c1, xq), w->wtype == ORC_W_Q4 ? (double)w->scale : (double)row_scale(w, r));
    const int8_t* lv = w->lev + (size_t)r * w->cols + c0;
    float s = 0.0f;
    for (int c = 0; c + 3 < c1 - c0; c += 4) {
        float t = (float)lv[c] * (float)xq[c];
        t = t + (float)lv[c + 1] * (float)xq[c + 1];
        t = t + (float)lv[c + 2] * (float)xq[c + 2];
        t = t + (float)lv[c + 3] * (float)xq[c + 3];
        s = s + t;
    }
    float v = floorf(s * row_scale(w, r) + 0.5f);
    if (v < -32768.0f) v = -32768.0f;
    if (v > 32767.0f) v = 32767.0f;
    return (int32_t)v;
}

static void mv_range(const omat* w, int c0, int c1, const int16_t* xq, int32_t* out, int literal) {
    const int par = (int64_t)w->rows * (c1 - c0) >= (1 << 20);
    #pragma omp parallel for schedule(static) if (par)
    for (int r = 0; r < w->rows; ++r) {
        if (literal) { out[r] = row_literal(w, r, c0, c1, xq); continue; }
        const int64_t S = row_dot(w, r, c0, c1, xq);
        const double sc = w->wtype == ORC_W_Q4 ? (double)w->scale : (double)row_scale(w, r);
        out[r] = mv_epilogue(S, sc);
    }
}

/* matvec_s input scaling (gpu_conv.cpp:271-287): k = 6 - e with max|x| = f*2^e,
   x*2^k then x_pack I16_2 (quantize_act, lrintf). */
int orc_scale_input(const float* x, int n, int16_t* xq) {
    float mx = 0.0f;
    for (int i = 0; i < n; ++i) { float a = fabsf(x[i]); if (a > mx) mx = a; }
    int k = 0;
    if (mx > 0.0f) {
        int e = 0;
        frexpf(mx, &e);
        k = 6 - e;
    }
    const float s = ldexpf(1.0f, k);
    for (int i = 0; i < n; ++i) xq[i] = orc_q16(x[i] * s);
    return k;
}

/* ------------------------------------------------------------------------- */
/* Session (the CPU layer loop, session.cpp:373-556)                          */
/* ------------------------------------------------------------------------- */

struct orc_session {
    const orc_model* m;
    int kv_bits, literal, row_bytes;
    float *rope_cos, *rope_sin;
    uint8_t** kv;        /* per layer: seq * row_bytes packed */
    float** kdec;        /* per layer: seq * kv_dim decoded K */
    float** vdec;
    int routes[64];
    /* scratch */
    float *x, *xb, *x1, *xbf, *qkv, *q, *k, *v, *att, *o2, *gate, *h, *scores;
    double* pv;
    int32_t* qi;         /* one query head on its integer grid */
    int16_t* xq;
    int32_t *iv, *iv2, *g, *u;
};

void orc_session_free(orc_session* s) {
    if (!s) return;
    for (int l = 0; l < s->m->in.layers; ++l) { free(s->kv[l]); free(s->kdec[l]); free(s->vdec[l]); }
    free(s->kv); free(s->kdec); free(s->vdec); free(s->rope_cos); free(s->rope_sin);
    free(s->x); free(s->xb); free(s->x1); free(s->xbf); free(s->qkv); free(s->q); free(s->k);
    free(s->v); free(s->att); free(s->o2); free(s->gate); free(s->h); free(s->scores); free(s->pv);
    free(s->qi); free(s->xq); free(s->iv); free(s->iv2); free(s->g); free(s->u);
    free(s);
}

orc_session* orc_session_new(const orc_model* m, int kv_bits, int literal) {
    if (kv_bits != 16 && kv_bits != 8) return NULL;
    const orc_info* in = &m->in;
    if (kv_bits == 8 && (in->kv_dim % 4 || in->head_dim % 4)) return NULL;
    orc_session* s = (orc_session*)calloc(1, sizeof(orc_session));
    s->m = m; s->kv_bits = kv_bits; s->literal = literal;
    s->row_bytes = kv_bits == 16 ? in->kv_dim * 4 : in->kv_dim * 2;   /* gpu_attn.cpp:89-92 */
    const int half = in->head_dim / 2, L = in->layers, S = in->seq;
    s->rope_cos = (float*)malloc(sizeof(float) * (size_t)S * half);
    s->rope_sin = (float*)malloc(sizeof(float) * (size_t)S * half);
    orc_rope_tables(in->rope_theta, in->head_dim, S, m->rope_factors, s->rope_cos, s->rope_sin);
    s->kv = (uint8_t**)calloc((size_t)L, sizeof(void*));
    s->kdec = (float**)calloc((size_t)L, sizeof(void*));
    s->vdec = (float**)calloc((size_t)L, sizeof(void*));
    for (int l = 0; l < L; ++l) {
        s->kv[l] = (uint8_t*)calloc((size_t)S, (size_t)s->row_bytes);
        s->kdec[l] = (float*)calloc((size_t)S * in->kv_dim, sizeof(float));
        s->vdec[l] = (float*)calloc((size_t)S * in->kv_dim, sizeof(float));
    }
    const int D = in->dim, QKV = D + 2 * in->kv_dim;
    int big = in->ffn_width > QKV ? in->ffn_width : QKV;
    if (in->vocab > big) big = in->vocab;
    s->x = (float*)malloc(sizeof(float) * D); s->xb = (float*)malloc(sizeof(float) * D);
    s->x1 = (float*)malloc(sizeof(float) * D); s->xbf = (float*)malloc(sizeof(float) * D);
    s->qkv = (float*)malloc(sizeof(float) * QKV); s->q = (float*)malloc(sizeof(float) * D);
    s->k = (float*)malloc(sizeof(float) * in->kv_dim); s->v = (float*)malloc(sizeof(float) * in->kv_dim);
    s->att = (float*)malloc(sizeof(float) * D); s->o2 = (float*)malloc(sizeof(float) * D);
    s->gate = (float*)malloc(sizeof(float) * 64);
    s->h = (float*)malloc(sizeof(float) * in->ffn_width);
    s->scores = (float*)malloc(sizeof(float) * S);
    s->pv = (double*)malloc(sizeof(double) * in->head_dim);
    s->qi = (int32_t*)malloc(sizeof(int32_t) * in->head_dim);
    s->xq = (int16_t*)malloc(sizeof(int16_t) * big);
    s->iv = (int32_t*)malloc(sizeof(int32_t) * big); s->iv2 = (int32_t*)malloc(sizeof(int32_t) * big);
    s->g = (int32_t*)malloc(sizeof(int32_t) * in->ffn_width); s->u = (int32_t*)malloc(sizeof(int32_t) * in->ffn_width);
    for (int i = 0; i < 64; ++i) s->routes[i] = -1;
    return s;
}

/* rms_norm (session.cpp:1932-1948).  Canonical: the sum of squares of the q16
   integers is exact and rounded once; literal: sequential fp32. */
static void rms_norm(const orc_session* s, const float* x, const float* w, float* o) {
    const int D = s->m->in.dim;
    float ss;
    if (s->literal) {
        ss = 0.0f;
        for (int i = 0; i < D; ++i) ss = ss + x[i] * x[i];
    } else {
        int64_t acc = 0;
        for (int i = 0; i < D; ++i) { const int64_t n = (int64_t)lrintf(x[i] * 256.0f); acc += n * n; }
        ss = (float)acc * (1.0f / 65536.0f);
    }
    ss = ss / (float)D;
    const float r = 1.0f / sqrtf(ss + s->m->in.rms_eps);
    for (int i = 0; i < D; ++i) o[i] = q16f(w[i] * (r * x[i]));
}

/* head_rms_norm (session.cpp:1950-1961).  Canonical: the inputs share one
   power-of-two grid, so the double sum of squares is exact. */
static void head_rms_norm(const orc_session* s, float* v, int n_heads, const float* w) {
    const int hd = s->m->in.head_dim;
    for (int h = 0; h < n_heads; ++h) {
        float* p = v + (size_t)h * hd;
        float ss;
        if (s->literal) {
            ss = 0.0f;
            for (int i = 0; i < hd; ++i) ss = ss + p[i] * p[i];
        } else {
            double acc = 0.0;
            for (int i = 0; i < hd; ++i) acc += (double)p[i] * (double)p[i];
            ss = (float)acc;
        }
        const float r = 1.0f / sqrtf(ss / (float)hd + 1e-6f);
        for (int i = 0; i < hd; ++i) p[i] = w[i] * (r * p[i]);
    }
}

/* rope (session.cpp:1963-1987). */
static void rope(const orc_session* s, float* v, int n_heads, int pos) {
    const int hd = s->m->in.head_dim, half = hd / 2;
    const float* cs = s->rope_cos + (size_t)pos * half;
    const float* sn = s->rope_sin + (size_t)pos * half;
    for (int h = 0; h < n_heads; ++h) {
        float* o = v + (size_t)h * hd;
        for (int i = 0; i < half; ++i) {
            const int ia = s->m->in.rope_half ? i : 2 * i;
            const int ib = s->m->in.rope_half ? i + half : 2 * i + 1;
            const float a = o[ia], b = o[ib], c = cs[i], sv = sn[i];
            const float ac = a * c, bs = b * sv, as = a * sv, bc = b * c;
            o[ia] = ac - bs;
            o[ib] = as + bc;
        }
    }
}

/* KV codec (shaders_attn.cpp:141-159): floor(v*KVSCALE+0.5) clamped. */
int16_t orc_kv_q16(float v) {
    float t = v * 2048.0f;
    float q = floorf(t + 0.5f);
    if (q < -32768.0f) q = -32768.0f;
    if (q > 32767.0f) q = 32767.0f;
    return (int16_t)q;
}
int8_t orc_kv_q8(float v) {
    float t = v * 16.0f;
    float q = floorf(t + 0.5f);
    if (q < -128.0f) q = -128.0f;
    if (q > 127.0f) q = 127.0f;
    return (int8_t)q;
}

static void kv_store(orc_session* s, int layer, int pos, const float* k, const float* v) {
    const int KD = s->m->in.kv_dim;
    uint8_t* row = s->kv[layer] + (size_t)pos * s->row_bytes;
    float* kd = s->kdec[layer] + (size_t)pos * KD;
    float* vd = s->vdec[layer] + (size_t)pos * KD;
    if (s->literal == ORC_LITERAL_FLOAT_KV) {
        /* the reference CPU path's own cache: the float K and V as computed
           (session.cpp:446-447); the packed row is not kept */
        memcpy(kd, k, sizeof(float) * KD);
        memcpy(vd, v, sizeof(float) * KD);
        return;
    }
    for (int i = 0; i < KD; ++i) {
        if (s->kv_bits == 16) {
            const int16_t qk = orc_kv_q16(k[i]), qv = orc_kv_q16(v[i]);
            row[2 * i] = (uint8_t)((uint16_t)qk >> 8); row[2 * i + 1] = (uint8_t)qk;
            row[2 * KD + 2 * i] = (uint8_t)((uint16_t)qv >> 8); row[2 * KD + 2 * i + 1] = (uint8_t)qv;
            kd[i] = (float)qk / 2048.0f; vd[i] = (float)qv / 2048.0f;
        } else {
            const int8_t qk = orc_kv_q8(k[i]), qv = orc_kv_q8(v[i]);
            row[i] = (uint8_t)qk; row[KD + i] = (uint8_t)qv;
            kd[i] = (float)qk / 16.0f; vd[i] = (float)qv / 16.0f;
        }
    }
}

static void kv_decode_row(orc_session* s, int layer, int pos) {
    const int KD = s->m->in.kv_dim;
    const uint8_t* row = s->kv[layer] + (size_t)pos * s->row_bytes;
    float* kd = s->kdec[layer] + (size_t)pos * KD;
    float* vd = s->vdec[layer] + (size_t)pos * KD;
    for (int i = 0; i < KD; ++i) {
        if (s->kv_bits == 16) {
            const int16_t qk = (int16_t)((row[2 * i] << 8) | row[2 * i + 1]);
            const int16_t qv = (int16_t)((row[2 * KD + 2 * i] << 8) | row[2 * KD + 2 * i + 1]);
            kd[i] = (float)qk / 2048.0f; vd[i] = (float)qv / 2048.0f;
        } else {
            kd[i] = (float)(int8_t)row[i] / 16.0f; vd[i] = (float)(int8_t)row[KD + i] / 16.0f;
        }
    }
}

/* Exponent k of the canonical attention weights' grid for len positions:
   53 - (bits of the largest |cache level|: 7 for q8, 15 for q16) -
   ceil(log2 len). */
int orc_attn_weight_exp(int len, int kv_bits) {
    int lg = 0;
    while ((1L << lg) < (long)len) ++lg;
    return 53 - (kv_bits == 16 ? 15 : 7) - lg;
}

/* Exponent F of a query head's integer grid: with max|q| = f * 2^e (f in
   [0.5, 1)), F = 22 - e, so every |q * 2^F| < 2^22 and rint(q * 2^F) splits
   into three balanced signed bytes; clamped to [-100, 100]. */
int orc_q_grid_exp(float qmax) {
    if (!(qmax > 0.0f)) return 0;
    int e = 0;
    frexpf(qmax, &e);
    int F = 22 - e;
    return F > 100 ? 100 : F < -100 ? -100 : F;
}

/* attention (session.cpp:1989-2050) over the decoded cache. */
static void attention(orc_session* s, int layer, int pos) {
    const orc_info* in = &s->m->in;
    const int hd = in->head_dim, KD = in->kv_dim, group = in->heads / in->kv_heads;
    const float sq = sqrtf((float)hd);
    for (int h = 0; h < in->heads; ++h) {
        const int kvh = h / group;
        const float* kb = s->kdec[layer] + (size_t)kvh * hd;
        const float* vb = s->vdec[layer] + (size_t)kvh * hd;
        const float* qh = s->q + (size_t)h * hd;
        float mx = -1e30f;
        if (s->literal) {
            for (int t = 0; t <= pos; ++t) {
                float acc = 0.0f;
                for (int i = 0; i < hd; ++i) acc = acc + qh[i] * kb[(size_t)t * KD + i];
                acc = acc / sq;
                s->scores[t] = acc;
                if (acc > mx) mx = acc;
            }
        } else {
            /* Canonical: q on a per-head power-of-two grid (orc_q_grid_exp),
               an exact integer dot with the cache levels, one rounding to
               float, times the head's constant c = fl(2^-F / grid / sqrt(hd)). */
            float qm = 0.0f;
            for (int i = 0; i < hd; ++i) { const float a = fabsf(qh[i]); if (a > qm) qm = a; }
            const int F = orc_q_grid_exp(qm);
            const float sF = ldexpf(1.0f, F);
            for (int i = 0; i < hd; ++i) s->qi[i] = (int32_t)rintf(qh[i] * sF);
            const float gscale = ldexpf(1.0f, -F - (s->kv_bits == 16 ? 11 : 4));
            const float ch = gscale / sq;               /* one rounding, once per head */
            const float vgrid = s->kv_bits == 16 ? 2048.0f : 16.0f;
            for (int t = 0; t <= pos; ++t) {
                const float* kr = kb + (size_t)t * KD;
                int64_t S = 0;
                for (int i = 0; i < hd; ++i) S += (int64_t)s->qi[i] * (int64_t)(kr[i] * vgrid);
                const float acc = (float)S * ch;
                s->scores[t] = acc;
                if (acc > mx) mx = acc;
            }
        }
        if (s->literal) {
            float sum = 0.0f;
            for (int t = 0; t <= pos; ++t) { s->scores[t] = expf(s->scores[t] - mx); sum = sum + s->scores[t]; }
            for (int t = 0; t <= pos; ++t) s->scores[t] = s->scores[t] / sum;
            for (int i = 0; i < hd; ++i) {
                float a = 0.0f;
                for (int t = 0; t <= pos; ++t) a = a + s->scores[t] * vb[(size_t)t * KD + i];
                s->att[(size_t)h * hd + i] = a;
            }
        } else {
            /* Canonical: integer weights E_t = rint(exp(s_t - max) * 2^k)
               with k = orc_attn_weight_exp(len, kv_bits), then the exact sums
               den = sum E_t and num_i = sum E_t * code_t,i (code = the cache's
               integer level; |E_t * code| <= 2^(53 - ceil(log2 len)), so every
               partial sum is an integer below 2^53 and any summation order
               gives these bits), and att_i = rint(float(num_i / den * c)) (ties to
               even, as the host's lrintf) on the q16 grid, c = 256 * the
               cache grid.  The ratio is the
               reference's sum_t (e_t / sum e) * v_t with e_t on a 2^-k grid. */
            const float vscale = s->kv_bits == 16 ? 2048.0f : 16.0f;
            const double c = s->kv_bits == 16 ? 0.125 : 16.0;
            const int kexp = orc_attn_weight_exp(pos + 1, s->kv_bits);
            double den = 0.0;
            for (int t = 0; t <= pos; ++t) {
                s->scores[t] = rintf(ldexpf(orc_expf(s->scores[t] - mx), kexp));
                den += (double)s->scores[t];
            }
            for (int i = 0; i < hd; ++i) s->pv[i] = 0.0;
            for (int t = 0; t <= pos; ++t) {
                const double e = (double)s->scores[t];
                const float* vr = vb + (size_t)t * KD;
                for (int i = 0; i < hd; ++i) s->pv[i] += e * (double)(vr[i] * vscale);
            }
            for (int i = 0; i < hd; ++i) {
                /* the float output, then the host's lrintf rounding (ties to even) */
                float q = rintf((float)(s->pv[i] / den * c));
                q = q < -32768.0f ? -32768.0f : q > 32767.0f ? 32767.0f : q;
                s->att[(size_t)h * hd + i] = q / 256.0f;
            }
        }
    }
}

/* SiLU(g)*u with the shaders' fp32 order (shaders.cpp:116-136, 1850-1922). */
static float swiglu_lit(int literal, float g, float u) {
    const float e = literal ? expf(-g) : orc_expf(-g);
    const float den = 1.0f + e;
    const float a = g / den;
    return a * u;
}

/* The GPU FFN the CPU path draws for split containers and MoE
   (session.cpp:491-551, gpu_ffn.cpp:67-132): gate/up matvecs rounded to q16,
   SiLU(gate)*up stored as q16 pairs, w2 per chunk rounded to q16, the two
   chunk outputs added with add_q16. */
/* The FFN gate kernel: gate/up matvecs of the q16 input, SiLU(g)*u (times
   2^-hs for a key-15 layer) stored on the q16 grid (the shaders' floor(v+0.5)
   store); g, u and hq hold F values. */
static void ffn_gate(const orc_model* m, int layer, const omat* w1, const omat* w3, const int16_t* xq,
                     int literal, int32_t* g, int32_t* u, int16_t* hq) {
    const int D = m->in.dim, F = m->in.ffn_width;
    const int hs = m->hid_scale[layer];
    const float hsm = hs > 0 ? ldexpf(1.0f, -hs) : 1.0f;
    mv_range(w1, 0, D, xq, g, literal);
    mv_range(w3, 0, D, xq, u, literal);
    for (int r = 0; r < F; ++r) {
        const float gf = (float)g[r] / 256.0f, uf = (float)u[r] / 256.0f;
        float y = swiglu_lit(literal, gf, uf);
        if (hs > 0) y = y * hsm;
        hq[r] = (int16_t)q16s(y);
    }
}

static void ffn(orc_session* s, int layer, const omat* w1, const omat* w3, const omat* w2, float* o2) {
    const orc_info* in = &s->m->in;
    const int D = in->dim, F = in->ffn_width;
    for (int i = 0; i < D; ++i) s->xq[i] = orc_q16(s->xbf[i]);
    int16_t* hq = (int16_t*)malloc(sizeof(int16_t) * F);
    ffn_gate(s->m, layer, w1, w3, s->xq, s->literal, s->g, s->u, hq);
    if (!in->ffn_chunked) {
        mv_range(w2, 0, F, hq, s->iv, s->literal);
        for (int i = 0; i < D; ++i) o2[i] = (float)s->iv[i] / 256.0f;
    } else {
        const int c = in->ffn_chunk;
        mv_range(w2, 0, c, hq, s->iv, s->literal);
        mv_range(w2, c, F, hq + c, s->iv2, s->literal);
        for (int i = 0; i < D; ++i) {
            const float a = (float)s->iv[i] / 256.0f, b = (float)s->iv2[i] / 256.0f;
            o2[i] = q16f(a + b);                               /* add_q16 */
        }
    }
    free(hq);
}

/* The dense FFN of a model whose hidden width is split into two chunks
   (Model::split_ffn, model.cpp:217-270, as App::prepare_model runs it): the
   split leaves w1 empty, so the CPU layer loop takes its host FFN
   (session.cpp:499-524), not the GPU FFN kernels: matvec_s of the gate and
   up halves (2^k input scaling, gpu_conv.cpp:271-287), the host SwiGLU
   rounded with quantize_act (session.cpp:2069-2080), times 2^-hs for a
   key-15 layer, matvec_s of each w2 column half with its own 2^k, and
   add_q16 of the two halves.  The a/b halves of w1 and w3 are row slices,
   so one matvec over all rows gives both. */
static void ffn_host(orc_session* s, int layer, const omat* w1, const omat* w3, const omat* w2, float* o2) {
    const orc_info* in = &s->m->in;
    const int D = in->dim, F = in->ffn_width, c = in->ffn_chunk;
    const int hs = s->m->hid_scale[layer];
    const float hsm = hs > 0 ? ldexpf(1.0f, -hs) : 1.0f;
    const int k = orc_scale_input(s->xbf, D, s->xq);
    mv_range(w1, 0, D, s->xq, s->g, s->literal);
    mv_range(w3, 0, D, s->xq, s->u, s->literal);
    const float inv = ldexpf(1.0f, -k);
    for (int r = 0; r < F; ++r) {
        const float g = ((float)s->g[r] / 256.0f) * inv, u = ((float)s->u[r] / 256.0f) * inv;
        float h = q16f(swiglu_lit(s->literal, g, u));
        if (hs > 0) h = h * hsm;
        s->h[r] = h;
    }
    int16_t* hq = (int16_t*)malloc(sizeof(int16_t) * F);
    const int ka = orc_scale_input(s->h, c, hq);
    mv_range(w2, 0, c, hq, s->iv, s->literal);
    const int kb = orc_scale_input(s->h + c, F - c, hq + c);
    mv_range(w2, c, F, hq + c, s->iv2, s->literal);
    const float ia = ldexpf(1.0f, -ka), ib = ldexpf(1.0f, -kb);
    for (int i = 0; i < D; ++i) {
        const float a = ((float)s->iv[i] / 256.0f) * ia, b = ((float)s->iv2[i] / 256.0f) * ib;
        o2[i] = q16f(a + b);                                   /* add_q16 */
    }
    free(hq);
}

int orc_step(orc_session* s, int token, int pos, float* logits) {
    const orc_model* m = s->m;
    const orc_info* in = &m->in;
    const int D = in->dim, KD = in->kv_dim, hd = in->head_dim, L = in->layers;
    if (token < 0 || token >= in->vocab || pos < 0 || pos >= in->seq) return ORC_EARG;
    /* embedding (session.cpp:342-371): q16(level * row scale) */
    const float es = m->emb_scale[token];
    for (int i = 0; i < D; ++i) s->x[i] = q16f((float)m->emb[(size_t)token * D + i] * es);
    for (int l = 0; l < L; ++l) {
        rms_norm(s, s->x, m->rms_att + (size_t)l * D, s->xb);
        /* qkv = matvec_s(qkv, xb) */
        int k = orc_scale_input(s->xb, D, s->xq);
        mv_range(&m->qkv[l], 0, D, s->xq, s->iv, s->literal);
        const float inv = ldexpf(1.0f, -k);
        for (int r = 0; r < D + 2 * KD; ++r) s->qkv[r] = ((float)s->iv[r] / 256.0f) * inv;
        memcpy(s->q, s->qkv, sizeof(float) * D);
        memcpy(s->k, s->qkv + D, sizeof(float) * KD);
        memcpy(s->v, s->qkv + D + KD, sizeof(float) * KD);
        if (in->qk_norm) {
            head_rms_norm(s, s->q, in->heads, m->q_norm + (size_t)l * hd);
            head_rms_norm(s, s->k, in->kv_heads, m->k_norm + (size_t)l * hd);
        }
        rope(s, s->q, in->heads, pos);
        rope(s, s->k, in->kv_heads, pos);
        kv_store(s, l, pos, s->k, s->v);
        attention(s, l, pos);
        for (int i = 0; i < D; ++i) s->att[i] = q16f(s->att[i]);
        k = orc_scale_input(s->att, D, s->xq);
        mv_range(&m->wo[l], 0, D, s->xq, s->iv, s->literal);
        const float inv2 = ldexpf(1.0f, -k);
        for (int i = 0; i < D; ++i) {
            const float wo = ((float)s->iv[i] / 256.0f) * inv2;
            s->x1[i] = q16f(s->x[i] + wo);                    /* add_q16 */
        }
        rms_norm(s, s->x1, m->rms_ffn + (size_t)l * D, s->xbf);
        int expert = -1;
        if (in->experts > 0) {
            k = orc_scale_input(s->xbf, D, s->xq);
            mv_range(&m->router[l], 0, D, s->xq, s->iv, 0);
            const float inv3 = ldexpf(1.0f, -k);
            for (int e = 0; e < in->experts; ++e) s->gate[e] = ((float)s->iv[e] / 256.0f) * inv3;
            expert = 0;                                        /* pick_expert, session.cpp:110-115 */
            for (int e = 1; e < in->experts; ++e) if (s->gate[e] > s->gate[expert]) expert = e;
            s->routes[l] = expert;
        }
        if (expert >= 0) {
            const oexpert* ex = &m->moe[(size_t)l * in->experts + expert];
            ffn(s, l, &ex->w1, &ex->w3, &ex->w2, s->o2);
        } else if (in->ffn_chunked) {
            ffn_host(s, l, &m->w1[l], &m->w3[l], &m->w2[l], s->o2);
        } else {
            ffn(s, l, &m->w1[l], &m->w3[l], &m->w2[l], s->o2);
        }
        for (int i = 0; i < D; ++i) s->x[i] = q16f(s->x1[i] + s->o2[i]);
    }
    if (!logits) return ORC_OK;
    rms_norm(s, s->x, m->rms_final, s->xb);
    for (int i = 0; i < D; ++i) s->xq[i] = orc_q16(s->xb[i]);
    int v0 = 0;
    for (int t = 0; t < m->n_tiles; ++t) {                     /* gpu_matvec.cpp:56-90 */
        mv_range(&m->tiles[t], 0, D, s->xq, s->iv, s->literal);
        for (int r = 0; r < m->tiles[t].rows; ++r) logits[v0 + r] = (float)s->iv[r] / 256.0f;
        v0 += m->tiles[t].rows;
    }
    return ORC_OK;
}

int orc_argmax(const float* logits, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i) if (logits[i] > logits[best]) best = i;
    return best;
}

int orc_kv_row_bytes(const orc_session* s) { return s->row_bytes; }

int orc_kv_read(const orc_session* s, int layer, int n, uint8_t* out) {
    if (layer < 0 || layer >= s->m->in.layers || n < 0 || n > s->m->in.seq) return ORC_EARG;
    memcpy(out, s->kv[layer], (size_t)n * s->row_bytes);
    return ORC_OK;
}

int orc_kv_write(orc_session* s, int layer, int n, const uint8_t* in) {
    if (layer < 0 || layer >= s->m->in.layers || n < 0 || n > s->m->in.seq) return ORC_EARG;
    memcpy(s->kv[layer], in, (size_t)n * s->row_bytes);
    for (int p = 0; p < n; ++p) kv_decode_row(s, layer, p);
    return ORC_OK;
}

int orc_last_route(const orc_session* s, int layer) {
    if (layer < 0 || layer >= 64) return -1;
    return s->routes[layer];
}

/* ------------------------------------------------------------------------- */
/* Primitive access for the kernel unit tests                                 */
/* ------------------------------------------------------------------------- */

static const omat* pick(const orc_model* m, int which, int layer, int expert) {
    const orc_info* in = &m->in;
    if (which == 6) return (layer >= 0 && layer < m->n_tiles) ? &m->tiles[layer] : NULL;
    if (layer < 0 || layer >= in->layers) return NULL;
    if (in->experts > 0 && (which == 2 || which == 3 || which == 4)) {
        if (expert < 0 || expert >= in->experts) return NULL;
        const oexpert* e = &m->moe[(size_t)layer * in->experts + expert];
        return which == 2 ? &e->w1 : which == 3 ? &e->w3 : &e->w2;
    }
    switch (which) {
        case 0: return &m->qkv[layer];
        case 1: return &m->wo[layer];
        case 2: return &m->w1[layer];
        case 3: return &m->w3[layer];
        case 4: return &m->w2[layer];
        case 5: return in->experts > 0 ? &m->router[layer] : NULL;
        default: return NULL;
    }
}

int orc_model_matvec(const orc_model* m, int which, int layer, int expert,
                     const int16_t* xq, int k, int32_t* out) {
    (void)k;
    const omat* w = pick(m, which, layer, expert);
    if (!w) return ORC_EARG;
    mv_range(w, 0, w->cols, xq, out, 0);
    return ORC_OK;
}

int orc_model_mv(const orc_model* m, int which, int layer, int expert, int c0, int c1,
                 const int16_t* xq, int literal, int32_t* out) {
    const omat* w = pick(m, which, layer, expert);
    if (!w || w->wtype == -1 || c0 < 0 || c1 > w->cols || c0 >= c1) return ORC_EARG;
    if (w->wtype == ORC_W_Q4 && (c0 % 32 || c1 % 32)) return ORC_EARG;
    mv_range(w, c0, c1, xq, out, which == 5 ? 0 : literal);
    return ORC_OK;
}

int orc_ffn_hidden(const orc_model* m, int layer, int expert, const int16_t* xq, int literal, int16_t* hq) {
    const orc_info* in = &m->in;
    if (layer < 0 || layer >= in->layers) return ORC_EARG;
    const omat *w1, *w3;
    if (in->experts > 0) {
        if (expert < 0 || expert >= in->experts) return ORC_EARG;
        const oexpert* e = &m->moe[(size_t)layer * in->experts + expert];
        w1 = &e->w1; w3 = &e->w3;
    } else {
        w1 = &m->w1[layer]; w3 = &m->w3[layer];
    }
    const int F = in->ffn_width;
    int32_t* g = (int32_t*)malloc(sizeof(int32_t) * F);
    int32_t* u = (int32_t*)malloc(sizeof(int32_t) * F);
    ffn_gate(m, layer, w1, w3, xq, literal, g, u, hq);
    free(g); free(u);
    return ORC_OK;
}

int orc_model_mat_shape(const orc_model* m, int which, int layer, int expert,
                        int* rows, int* cols, int* wtype, float* scale) {
    const omat* w = pick(m, which, layer, expert);
    if (!w) return ORC_EARG;
    *rows = w->rows; *cols = w->cols; *wtype = w->wtype; *scale = w->scale;
    return ORC_OK;
}

int orc_model_mat_levels(const orc_model* m, int which, int layer, int expert, int32_t* levels) {
    const omat* w = pick(m, which, layer, expert);
    if (!w) return ORC_EARG;
    const size_t n = (size_t)w->rows * w->cols;
    for (size_t i = 0; i < n; ++i)
        levels[i] = w->lev ? w->lev[i] : w->nib ? w->nib[i] : w->w16[i];
    return ORC_OK;
}

int orc_model_mat_rowscale16(const orc_model* m, int which, int layer, int expert, uint16_t* p16) {
    const omat* w = pick(m, which, layer, expert);
    if (!w) return ORC_EARG;
    if (!w->p16) return 0;
    memcpy(p16, w->p16, sizeof(uint16_t) * (size_t)w->rows);
    return 1;
}

int orc_model_mat_q4params(const orc_model* m, int which, int layer, int expert, int16_t* s16, int16_t* m16) {
    const omat* w = pick(m, which, layer, expert);
    if (!w || w->wtype != ORC_W_Q4) return ORC_EARG;
    memcpy(s16, w->s16, sizeof(int16_t) * (size_t)w->rows * w->groups);
    memcpy(m16, w->m16, sizeof(int16_t) * (size_t)w->rows * w->groups);
    return ORC_OK;
}

int orc_model_mat_plane(const orc_model* m, int which, int layer, int expert, float* plane) {
    const omat* w = pick(m, which, layer, expert);
    if (!w || !w->plane) return 0;
    memcpy(plane, w->plane, sizeof(float) * (size_t)w->rows);
    return 1;
}

int orc_model_emb(const orc_model* m, int8_t* out) {
    const int n = m->in.vocab * m->in.dim;
    if (out) memcpy(out, m->emb, (size_t)n);
    return n;
}

int orc_model_vec(const orc_model* m, int which, float* out) {
    const orc_info* in = &m->in;
    const float* src = NULL;
    int n = 0;
    switch (which) {
        case 0: src = m->emb_scale; n = in->vocab; break;
        case 1: src = m->rms_att; n = in->layers * in->dim; break;
        case 2: src = m->rms_ffn; n = in->layers * in->dim; break;
        case 3: src = m->rms_final; n = in->dim; break;
        case 4: src = m->q_norm; n = m->q_norm ? in->layers * in->head_dim : 0; break;
        case 5: src = m->k_norm; n = m->k_norm ? in->layers * in->head_dim : 0; break;
        default: return -1;
    }
    if (out && src) memcpy(out, src, sizeof(float) * (size_t)n);
    return n;
}

uint64_t orc_fnv1a64(const uint8_t* p, uint64_t n) {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t i = 0; i < n; ++i) { h ^= p[i]; h *= 1099511628211ull; }
    return h;
}
