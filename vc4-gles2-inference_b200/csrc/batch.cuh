// batch.cuh -- the decode pass for many sequences at once (included by
// kernels.cuh inside vc4::(anonymous)).
//
// At kBatchMin or more sequences per pass every matvec op becomes
//   prep:   one CTA per sequence: the op's input vector (embedding, x, att or
//           x1), RMSNorm, the top-1 MoE route, the matvec_s input scale k and
//           the byte staging of x' = x*2^k for the consuming matrix, written
//           once to State::xrec (lo bytes | hi bytes | q4 chunk or t3 total
//           sums | k);
//   matmat: one CTA per 32-row block: the block's weights, q4 parameters and
//           row scales land in shared memory by bulk copies issued before the
//           grid-dependency wait, the sequences' records follow in groups,
//           and each warp serves its own sequences over all column chunks
//           (lanes are rows), so no partial sum crosses warps.
// w2 reads the hidden vectors directly (no input scale) and writes the
// residual sum x itself.  The integer arithmetic is that of the one-sequence
// kernels (exact dp4a products, the same epilogues), so a sequence's result
// does not depend on the batch it runs in.

constexpr int kBatchMin = 8;
constexpr int kMmNI = 2;      // sequences a warp carries through one sweep of the chunks

enum { kOpQkv = 0, kOpWo = 1, kOpGate = 2, kOpLogits = 3 };

__host__ __device__ inline size_t align128(size_t x) { return (x + 127) & ~(size_t)127; }

// One staged input: lo[stride] | hi[stride] | gsum[gst] | k
__host__ __device__ inline size_t xrec_bytes(const DMat& W) {
    return 2 * (size_t)x_stride(W) + align16(sizeof(int) * (size_t)(g_stride(W) + 1));
}

// The block's weights, q4 parameters and row scales, as copied to shared memory.
__host__ __device__ inline size_t mm_wbytes(const DMat& W) {
    return (size_t)W.nchunks * 512 + (W.wtype == W_Q4 ? (size_t)W.nchunks * 128 : 0) + 128;
}

// The w2 input of one sequence, written by the gate matmat as it produces the
// hidden values (x' = h: no input scale): lo | hi | chunk sums (q4) or total
// (t3) of column half a, then the same for half b of a chunked w2.
struct DownRec {   // byte offsets inside one staged hidden vector
    size_t lo_a, hi_a, g_a, lo_b, hi_b, g_b, bytes;
};
__host__ __device__ inline DownRec down_rec(const DMat& Wa, const DMat& Wb, bool two) {
    DownRec r;
    const size_t sa = x_stride(Wa), sb = two ? x_stride(Wb) : 0;
    r.lo_a = 0; r.hi_a = sa; r.g_a = 2 * sa;
    r.lo_b = r.g_a + align16(sizeof(int) * (g_stride(Wa) + 1));
    r.hi_b = r.lo_b + sb; r.g_b = r.hi_b + sb;
    r.bytes = r.g_b + (two ? align16(sizeof(int) * (g_stride(Wb) + 1)) : 0);
    return r;
}
// Top-1 MoE route of a normalised input (block-wide; the first maximum wins,
// shaders.cpp:1216-1230 and session.cpp:110-115).
__device__ int route_block(const int16_t* xn, const DMat& R, int D, int experts, Red& r) {
    const int k = scale_exponent(xn, D, r);
    const float sk = ldexpf(1.0f, k);
    int best = 0;
    float bestv = 0.0f;
    for (int e = 0; e < experts; ++e) {
        long long acc = 0;
        for (int c = threadIdx.x; c < D; c += kThreads) acc += (long long)R.w16[(size_t)e * D + c] * xscale(xn[c], k, sk);
        acc = block_sum_i64(acc, r);
        const int v = mv_epi(acc, R.rscale[e]);
        const float g = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), ldexpf(1.0f, -k));
        if (e == 0 || g > bestv) { best = e; bestv = g; }
    }
    return best;
}

// prep: one CTA per sequence (blockIdx.x = its batch position).
template <int WT>
__global__ void __launch_bounds__(kThreads) k_prep(DMat W, DMat E, const float* emb_scale, const float* rms_w,
                                                   DMat router, State s, Batch bt, Dims d, int layer, int op,
                                                   DownRec dr) {
    __shared__ Red red;
    extern __shared__ __align__(16) char smem[];
    if (!smem_ok(sizeof(int16_t) * (size_t)d.dim, s.err)) return;
    int16_t* x = reinterpret_cast<int16_t*>(smem);
    const int b = blockIdx.x;
    float nw[kPer];
    if (op != kOpWo) load_f32_regs(rms_w, d.dim, nw);
    pdl_launch_dependents();
    pdl_wait();
    if (op == kOpQkv && layer == 0) {
        // embedding (session.cpp:342-371) from the blocked q8 layout; also the residual x
        const int tok = bt.token[b];
        const float es = emb_scale[tok];
        const int8_t* eb = reinterpret_cast<const int8_t*>(E.body) + ((size_t)(tok / 32) * E.nchunks * 32 + (tok % 32)) * 16;
        for (int c = threadIdx.x; c < d.dim; c += kThreads) {
            const int16_t q = (int16_t)q16h(__fmul_rn((float)eb[(size_t)(c / 16) * 512 + (c % 16)], es));
            x[c] = q;
            s.x[(size_t)b * d.dim + c] = q;
        }
        if (threadIdx.x == 0) s.best[b] = 0ull;
    } else {
        const int16_t* src = op == kOpWo ? s.att : op == kOpGate ? s.x1 : s.x;
        load_vec(src + (size_t)b * d.dim, d.dim, x);
    }
    __syncthreads();
    if (op != kOpWo) rmsnorm_q16(x, nw, d.dim, d.eps, x, red);
    if (op == kOpGate && d.experts) {
        const int e = route_block(x, router, d.dim, d.experts, red);
        if (threadIdx.x == 0) s.route[(size_t)b * d.layers + layer] = e;
    }
    const int k = (op == kOpQkv || op == kOpWo) ? scale_exponent(x, d.dim, red) : 0;
    char* rec = s.xrec + (size_t)b * xrec_bytes(W);
    XStage xs;
    xs.stride = x_stride(W);
    xs.gstride = g_stride(W);
    xs.lo = reinterpret_cast<uint8_t*>(rec);
    xs.hi = reinterpret_cast<int8_t*>(rec + xs.stride);
    xs.gsum = reinterpret_cast<int*>(rec + 2 * (size_t)xs.stride);
    stage_one<WT>(xs, 0, x, d.dim, k, red);
    if (threadIdx.x == 0) xs.gsum[xs.gstride] = k;
    if (op == kOpGate && WT == W_T3 && threadIdx.x == 0) {
        // the gate matmat adds the hidden totals into the sequence's w2 record
        char* hr = s.hrec + (size_t)b * dr.bytes;
        *reinterpret_cast<int*>(hr + dr.g_a) = 0;
        if (d.chunk < d.ffn) *reinterpret_cast<int*>(hr + dr.g_b) = 0;
    }
}

// Sequences a matmat CTA serves: all of them, or (MoE) those routed to
// `expert`, in batch order; the route loads are issued by all threads at once
// and the list is compacted with warp ballots.
__device__ __forceinline__ int mm_members(const State& s, const Dims& d, int n, int layer, int expert, bool moe,
                                          int* members) {
    __shared__ int wc[32];
    __shared__ int base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (int)blockDim.x >> 5;   // any block size
    if (threadIdx.x == 0) base = 0;
    for (int r = 0; r < n; r += (int)blockDim.x) {
        const int b = r + threadIdx.x;
        const bool f = b < n && (!moe || __ldcg(s.route + (size_t)b * d.layers + layer) == expert);
        const unsigned m = __ballot_sync(0xffffffffu, f);
        if (lane == 0) wc[warp] = __popc(m);
        __syncthreads();
        int off = base;
        for (int w = 0; w < warp; ++w) off += wc[w];
        if (f) members[off + __popc(m & ((1u << lane) - 1u))] = b;
        __syncthreads();
        if (threadIdx.x == 0) for (int w = 0; w < nw; ++w) base += wc[w];
        __syncthreads();
    }
    return base;
}

// Dot products of `ni` staged inputs (records in shared memory) with the
// 32 rows of one weight block in shared memory; lane = row.
template <int WT>
__device__ __forceinline__ void mm_dots(const char* wsm, int nch, int stride, int gst, const char* const (&recs)[kMmNI],
                                        int ni, long long (&S)[kMmNI]) {
    constexpr int cpc = WT == W_Q8 ? 16 : WT == W_Q4 ? 32 : 64;
    const int lane = threadIdx.x & 31;
    const int4* wv = reinterpret_cast<const int4*>(wsm) + lane;
    const int* qp = reinterpret_cast<const int*>(wsm + (size_t)nch * 512) + lane;
#pragma unroll
    for (int i = 0; i < kMmNI; ++i) S[i] = 0;
#pragma unroll 2
    for (int j = 0; j < nch; ++j) {
        const int4 w = wv[(size_t)j * 32];
        const int sp = WT == W_Q4 ? qp[(size_t)j * 32] : 0;
#pragma unroll
        for (int i = 0; i < kMmNI; ++i) {
            if (i >= ni) break;
            const char* r = recs[i];
            S[i] += chunk_dot<WT>(w, sp, reinterpret_cast<const uint8_t*>(r) + j * cpc,
                                  reinterpret_cast<const int8_t*>(r + stride) + j * cpc,
                                  WT == W_Q4 ? reinterpret_cast<const int*>(r + 2 * (size_t)stride)[j] : 0);
        }
    }
    (void)gst;
}

__host__ __device__ inline size_t mm_smem(const DMat& W, int nmat, int group, int n) {
    return align128(nmat * mm_wbytes(W)) + (size_t)group * xrec_bytes(W) + align16(sizeof(int) * (size_t)n) + 64;
}

// matmat: one CTA per 32-row block (blockIdx.x) and expert (blockIdx.y).
template <int WT, int OP>
__global__ void __launch_bounds__(kThreads) k_mm(MatSet M, State s, Batch bt, Dims d, int layer, int group, int hs,
                                                 Finalize fz, DownRec dr) {
    constexpr int NM = OP == kOpGate ? 2 : 1;
    const int blk = blockIdx.x, expert = blockIdx.y;
    const DMat& W = M.a[expert];
    const DMat& W3 = M.b[expert];
    const int n = bt.n, nch = W.nchunks, stride = x_stride(W), gst = g_stride(W);
    const size_t wb = mm_wbytes(W), rb = xrec_bytes(W);
    if (!smem_ok(mm_smem(W, NM, group, n), s.err)) return;
    char* sm = SmemLayout::base();
    char* rsm = sm + align128(NM * wb);
    int* members = reinterpret_cast<int*>(rsm + (size_t)group * rb);
    unsigned long long* bar = reinterpret_cast<unsigned long long*>(
        sm + align128(NM * wb) + (size_t)group * rb + align16(sizeof(int) * (size_t)n));
    const unsigned wbody = (unsigned)nch * 512u, qbytes = WT == W_Q4 ? (unsigned)nch * 128u : 0u;
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
        mbar_expect_tx(&bar[0], NM * (wbody + qbytes + 128u));
        for (int m = 0; m < NM; ++m) {
            const DMat& X = m ? W3 : W;
            char* dst = sm + m * wb;
            bulk_g2s(dst, X.body + (size_t)blk * wbody, wbody, &bar[0]);
            if (WT == W_Q4) bulk_g2s(dst + wbody, X.q4p + (size_t)blk * nch * 32, qbytes, &bar[0]);
            bulk_g2s(dst + wbody + qbytes, X.rscale + (size_t)blk * 32, 128u, &bar[0]);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    // this CTA's share of the members (grid z splits them)
    const int nall = mm_members(s, d, n, layer, expert, OP == kOpGate && d.experts > 0, members);
    const int per = (nall + (int)gridDim.z - 1) / (int)gridDim.z;
    const int m0 = min(nall, (int)blockIdx.z * per), nm = min(nall, m0 + per) - m0;
    members += m0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blk * 32 + lane;
    const float* rs = reinterpret_cast<const float*>(sm + wbody + qbytes);
    const float* rs3 = reinterpret_cast<const float*>(sm + wb + wbody + qbytes);
    unsigned long long best[kMmNI];
    bool ok = !__syncthreads_or(!mbar_wait(&bar[0], 0));   // the same verdict in every thread
    for (int g0 = 0; g0 < nm && ok; g0 += group) {
        const int gn = min(group, nm - g0), gi = g0 / group;
        if (threadIdx.x == 0) {
            fence_proxy_async();
            mbar_expect_tx(&bar[1], (unsigned)(gn * rb));
            for (int i = 0; i < gn; ++i) bulk_g2s(rsm + i * rb, s.xrec + (size_t)members[g0 + i] * rb, (unsigned)rb, &bar[1]);
        }
        ok = mbar_wait(&bar[1], (unsigned)gi & 1u);
        if (__syncthreads_or(!ok)) { ok = false; break; }
        for (int i0 = warp * kMmNI; i0 < gn; i0 += kWarps * kMmNI) {
            const int ni = min(kMmNI, gn - i0);
            const char* recs[kMmNI];
#pragma unroll
            for (int i = 0; i < kMmNI; ++i) recs[i] = rsm + (size_t)(i0 + (i < ni ? i : 0)) * rb;
            long long S[kMmNI], S3[kMmNI];
            mm_dots<WT>(sm, nch, stride, gst, recs, ni, S);
            if (OP == kOpGate) mm_dots<WT>(sm + wb, nch, stride, gst, recs, ni, S3);
#pragma unroll
            for (int i = 0; i < kMmNI; ++i) {
                best[i] = 0ull;
                if (i >= ni) break;
                const int b = members[g0 + i0 + i];
                const int* gs = reinterpret_cast<const int*>(recs[i] + 2 * (size_t)stride);
                const int k = gs[gst];
                const long long corr = WT == W_T3 ? gs[0] : 0;
                const bool live = row < W.rows;
                const int v = live ? mv_epi(S[i] - corr, rs[lane]) : 0;
                if (OP == kOpQkv) {
                    if (live)
                        s.qkv[(size_t)b * (d.dim + 2 * d.kv_dim) + row] =
                            __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), ldexpf(1.0f, -k));
                } else if (OP == kOpWo) {
                    if (live) {
                        const float wo = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), ldexpf(1.0f, -k));
                        const float xr = __fmul_rn((float)__ldcg(s.x + (size_t)b * d.dim + row), 1.0f / 256.0f);
                        s.x1[(size_t)b * d.dim + row] = (int16_t)q16h(__fadd_rn(xr, wo));
                    }
                } else if (OP == kOpGate) {
                    int q = 0;
                    if (live) {
                        const int u = mv_epi(S3[i] - corr, rs3[lane]);
                        float y = swiglu1(__fmul_rn((float)v, 1.0f / 256.0f), __fmul_rn((float)u, 1.0f / 256.0f));
                        if (hs > 0) y = __fmul_rn(y, ldexpf(1.0f, -hs));     // metadata key 15 store scale
                        q = q16s(y);
                    }
                    // the w2 input record of sequence b: this block's 32 hidden rows are
                    // columns [c0, c0 + 32) of one w2 column half (the chunk is a multiple of 32)
                    const int half = (d.chunk < d.ffn && blk * 32 >= d.chunk) ? 1 : 0;
                    const int c0 = blk * 32 - (half ? d.chunk : 0);
                    char* hr = s.hrec + (size_t)b * dr.bytes;
                    const size_t lo = half ? dr.lo_b : dr.lo_a, hi = half ? dr.hi_b : dr.hi_a, g = half ? dr.g_b : dr.g_a;
                    if (live) {
                        hr[lo + c0 + lane] = (char)(q & 0xFF);
                        hr[hi + c0 + lane] = (char)(q >> 8);
                    }
                    const int sum = __reduce_add_sync(0xffffffffu, q);
                    if (lane == 0) {
                        if (WT == W_Q4) reinterpret_cast<int*>(hr + g)[c0 / 32] = sum;
                        if (WT == W_T3) atomicAdd(reinterpret_cast<int*>(hr + g), sum);
                    }
                } else if (live) {
                    s.logits[(size_t)b * d.vocab + row] = v;
                    best[i] = logit_key(v, row);
                }
            }
            if (OP == kOpLogits) {
#pragma unroll
                for (int i = 0; i < kMmNI; ++i) {
                    if (i >= ni) break;
                    unsigned long long kk = best[i];
                    for (int o = 16; o; o >>= 1) {
                        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, kk, o);
                        kk = k2 > kk ? k2 : kk;
                    }
                    if (lane == 0 && kk) atomicMax(&s.best[members[g0 + i0 + i]], kk);
                }
            }
        }
        __syncthreads();   // the group's records are consumed before the next group lands
    }
    if (!ok && threadIdx.x == 0) {
        // a copy did not land in time: report, and wait (bounded) for copies still in flight
        atomicExch(s.err, kErrCopyTimeout);
        mbar_wait(&bar[0], 0, 10000000ull);
        mbar_wait(&bar[1], 0, 10000000ull);
        mbar_wait(&bar[1], 1, 10000000ull);
    }
    if (OP == kOpLogits) logits_finish(s, 0, n, fz);
}

__host__ __device__ inline size_t mmdown_smem(const DMat& Wa, const DMat& Wb, bool two, int group, int n) {
    return align128(mm_wbytes(Wa) + (two ? mm_wbytes(Wb) : 0)) + (size_t)group * down_rec(Wa, Wb, two).bytes +
           align16(sizeof(int) * (size_t)n) + 64;
}

template <int WT>
__global__ void __launch_bounds__(kThreads) k_mmdown(MatSet M2, State s, Batch bt, Dims d, int layer, int group) {
    const int blk = blockIdx.x, expert = blockIdx.y;
    const bool two = d.chunk < d.ffn;
    const DMat& Wa = M2.a[expert];
    const DMat& Wb = M2.b[expert];
    const int n = bt.n;
    const size_t wba = mm_wbytes(Wa), wbb = two ? mm_wbytes(Wb) : 0;
    const DownRec R = down_rec(Wa, Wb, two);
    if (!smem_ok(mmdown_smem(Wa, Wb, two, group, n), s.err)) return;
    char* sm = SmemLayout::base();
    char* rsm = sm + align128(wba + wbb);
    int* members = reinterpret_cast<int*>(rsm + (size_t)group * R.bytes);
    unsigned long long* bar = reinterpret_cast<unsigned long long*>(
        sm + align128(wba + wbb) + (size_t)group * R.bytes + align16(sizeof(int) * (size_t)n));
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
        unsigned total = 0;
        for (int m = 0; m < (two ? 2 : 1); ++m) total += (unsigned)mm_wbytes(m ? Wb : Wa);
        mbar_expect_tx(&bar[0], total);
        for (int m = 0; m < (two ? 2 : 1); ++m) {
            const DMat& X = m ? Wb : Wa;
            char* dst = sm + (m ? wba : 0);
            const unsigned wbody = (unsigned)X.nchunks * 512u, qb = WT == W_Q4 ? (unsigned)X.nchunks * 128u : 0u;
            bulk_g2s(dst, X.body + (size_t)blk * wbody, wbody, &bar[0]);
            if (WT == W_Q4) bulk_g2s(dst + wbody, X.q4p + (size_t)blk * X.nchunks * 32, qb, &bar[0]);
            bulk_g2s(dst + wbody + qb, X.rscale + (size_t)blk * 32, 128u, &bar[0]);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    const int nall = mm_members(s, d, n, layer, expert, d.experts > 0, members);
    const int per = (nall + (int)gridDim.z - 1) / (int)gridDim.z;
    const int m0 = min(nall, (int)blockIdx.z * per), nm = min(nall, m0 + per) - m0;
    members += m0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blk * 32 + lane;
    const int sa = x_stride(Wa), sb = two ? x_stride(Wb) : 0;
    const float* rsa = reinterpret_cast<const float*>(sm + (size_t)Wa.nchunks * 512 + (WT == W_Q4 ? (size_t)Wa.nchunks * 128 : 0));
    const float* rsb = two ? reinterpret_cast<const float*>(sm + wba + (size_t)Wb.nchunks * 512 +
                                                           (WT == W_Q4 ? (size_t)Wb.nchunks * 128 : 0))
                           : rsa;
    bool ok = !__syncthreads_or(!mbar_wait(&bar[0], 0));   // the same verdict in every thread
    for (int g0 = 0; g0 < nm && ok; g0 += group) {
        const int gn = min(group, nm - g0), gi = g0 / group;
        if (threadIdx.x == 0) {
            fence_proxy_async();
            mbar_expect_tx(&bar[1], (unsigned)(gn * R.bytes));
            for (int i = 0; i < gn; ++i)
                bulk_g2s(rsm + i * R.bytes, s.hrec + (size_t)members[g0 + i] * R.bytes, (unsigned)R.bytes, &bar[1]);
        }
        ok = mbar_wait(&bar[1], (unsigned)gi & 1u);
        if (__syncthreads_or(!ok)) { ok = false; break; }
        for (int i0 = warp * kMmNI; i0 < gn; i0 += kWarps * kMmNI) {
            const int ni = min(kMmNI, gn - i0);
            const char* ra[kMmNI];
            const char* rb2[kMmNI];
#pragma unroll
            for (int i = 0; i < kMmNI; ++i) {
                ra[i] = rsm + (size_t)(i0 + (i < ni ? i : 0)) * R.bytes;
                rb2[i] = ra[i] + R.lo_b;
            }
            long long Sa[kMmNI], Sb[kMmNI];
            mm_dots<WT>(sm, Wa.nchunks, sa, g_stride(Wa), ra, ni, Sa);
            if (two) mm_dots<WT>(sm + wba, Wb.nchunks, sb, g_stride(Wb), rb2, ni, Sb);
#pragma unroll
            for (int i = 0; i < kMmNI; ++i) {
                if (i >= ni || row >= Wa.rows) continue;
                const int b = members[g0 + i0 + i];
                const long long ca = WT == W_T3 ? reinterpret_cast<const int*>(ra[i] + R.g_a)[0] : 0;
                float o2 = __fmul_rn((float)mv_epi(Sa[i] - ca, rsa[lane]), 1.0f / 256.0f);
                if (two) {
                    const long long cb = WT == W_T3 ? reinterpret_cast<const int*>(ra[i] + R.g_b)[0] : 0;
                    const int vb = mv_epi(Sb[i] - cb, rsb[lane]);
                    // add_q16 of the two chunk outputs (session.cpp:2052-2067)
                    o2 = __fmul_rn((float)q16h(__fadd_rn(o2, __fmul_rn((float)vb, 1.0f / 256.0f))), 1.0f / 256.0f);
                }
                const float x1 = __fmul_rn((float)__ldcg(s.x1 + (size_t)b * d.dim + row), 1.0f / 256.0f);
                s.x[(size_t)b * d.dim + row] = (int16_t)q16h(__fadd_rn(x1, o2));
            }
        }
        __syncthreads();
    }
    if (!ok && threadIdx.x == 0) {
        atomicExch(s.err, kErrCopyTimeout);
        mbar_wait(&bar[0], 0, 10000000ull);
        mbar_wait(&bar[1], 0, 10000000ull);
        mbar_wait(&bar[1], 1, 10000000ull);
    }
}

// ---------------------------------------------------------------------------
// Tensor-core matmat for q8 weights (tcgen05.mma kind::i8, TMEM accumulators).
//
// One CTA (one warpgroup) computes a 128-row tile of one matrix (or of two:
// w1 and w3 of the ffn, or the two column halves of a chunked w2) for a group
// of sequences.  The weights are 32-row blocks in HBM; 512-byte bulk copies
// place chunk j of row block q at shared offset j*2048 + q*512, which is the
// K-major core-matrix layout with the 8-row groups 128 bytes apart (SBO) and
// the 16-byte K chunks 2048 bytes apart (LBO).  The sequences' input bytes
// form the B operand [chunk][sequence][16 bytes] per plane: x' = lo + 256*hi
// with lo unsigned and hi signed, so every K step is two MMAs (s8 x u8 into
// one accumulator, s8 x s8 into another) and S = D_lo + 256*D_hi is the exact
// integer dot (|D| < 2^31 for every shape here).  tcgen05.ld brings row r of
// the accumulators to thread r of the warpgroup for the usual epilogues.
// ---------------------------------------------------------------------------

constexpr int kOpDown = 4;
constexpr int kTcThreads = 128;

__device__ __forceinline__ uint64_t umma_sdesc(unsigned addr, unsigned lbo, unsigned sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;   // descriptor version (sm_100); base offset 0, no swizzle
    return d;
}
__host__ __device__ constexpr uint32_t umma_idesc_i8(bool b_signed, int m, int n) {
    // D s32, A s8 (K-major), B u8 or s8 (K-major), shape m x n
    return (2u << 4) | (1u << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma_i8(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
                 ::"r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0) : "memory");
}
__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 16 consecutive 32-bit accumulator columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct TcPass {        // one matrix of a tensor-core matmat and where its B bytes live in a record
    DMat W;
    int lo_off, hi_off;
};
struct TcArgs {
    TcPass p[2];
    int npass;
    int rec_bytes;       // bytes per sequence record (State::xrec or State::hrec)
    int from_hrec;       // the records are w2 inputs (State::hrec)
    int group;           // sequences per MMA group (multiple of 16)
    int tmem_cols;       // power of two >= 2 * npass * group
    int hs;
    DownRec dr;
};

__host__ __device__ inline int tc_kchunks(const DMat& W) { return (W.nchunks + 1) & ~1; }   // even: K steps of 32
__host__ __device__ inline size_t tc_smem(const TcArgs& a, int n) {
    int kc = 0;
    for (int m = 0; m < a.npass; ++m) kc = kc > tc_kchunks(a.p[m].W) ? kc : tc_kchunks(a.p[m].W);
    return (size_t)kc * 2048 + (size_t)kc * a.group * 32 + align16(sizeof(int) * (size_t)n) + 64;
}

template <int OP>
__global__ void __launch_bounds__(kTcThreads) k_tmm(TcArgs a, State s, Batch bt, Dims d, int layer, Finalize fz) {
    const int tile = blockIdx.x, expert = blockIdx.y;
    const int n = bt.n, G = a.group;
    if (!smem_ok(tc_smem(a, n), s.err)) return;
    int kc = 0;
    for (int m = 0; m < a.npass; ++m) kc = max(kc, tc_kchunks(a.p[m].W));
    char* sm = SmemLayout::base();
    uint8_t* sa = reinterpret_cast<uint8_t*>(sm);                        // [kc][128 rows][16]
    uint8_t* sbl = sa + (size_t)kc * 2048;                              // [kc][G][16] lo plane
    uint8_t* sbh = sbl + (size_t)kc * G * 16;                            // [kc][G][16] hi plane
    int* members = reinterpret_cast<int*>(sbh + (size_t)kc * G * 16);
    unsigned long long* bar = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(members) +
                                                                   align16(sizeof(int) * (size_t)n));
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const TcPass P0 = a.p[0], P1 = a.p[a.npass > 1 ? 1 : 0];   // the passes have equal shapes
    auto issue_a = [&](const DMat& W) {   // warp 0: the tile's weights, one 512-byte copy per (chunk, row block)
        const int nch = W.nchunks;
        const int nq = min(4, W.rblocks - tile * 4);
        if (lane == 0) mbar_expect_tx(&bar[0], (unsigned)(nq * nch * 512));
        __syncwarp();
        for (int i = lane; i < nq * nch; i += 32) {
            const int q = i / nch, j = i % nch;
            bulk_g2s(sa + (size_t)j * 2048 + q * 512, W.body + ((size_t)(tile * 4 + q) * nch + j) * 512, 512u, &bar[0]);
        }
    };
    if (warp == 0) {
        if (lane == 0) {
            mbar_init(&bar[0], 1);
            mbar_init(&bar[1], 1);
            mbar_fence_init();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tslot)),
                     "r"(a.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        issue_a(P0.W);
    }
    // zero the padding the copies do not cover: row blocks past the matrix, the odd K chunk
    {
        const DMat& W = P0.W;
        const int nq = min(4, W.rblocks - tile * 4);
        for (int i = tid; i < kc * 128; i += kTcThreads) {
            const int j = i / 128, r = i % 128;
            if (j >= W.nchunks || r / 32 >= nq) *reinterpret_cast<uint4*>(sa + (size_t)j * 2048 + r * 16) = make_uint4(0, 0, 0, 0);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    const int nall = mm_members(s, d, n, layer, expert, false, members);
    const int per = (nall + (int)gridDim.z - 1) / (int)gridDim.z;
    const int m0 = min(nall, (int)blockIdx.z * per), nm = min(nall, m0 + per) - m0;
    members += m0;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const char* recs = a.from_hrec ? s.hrec : s.xrec;
    int a_issued = 1, a_waited = 0;   // weight-tile loads issued / waited for (phases of bar[0])
    unsigned mph = 0;                 // phase of bar[1] (MMA completion)
    bool ok = true;
    const int row = tile * 128 + tid;
    for (int g0 = 0; g0 < nm && ok; g0 += G) {
        const int gn = min(G, nm - g0);
        const int gp = (gn + 15) & ~15;                 // MMA N: a multiple of 16
        for (int m = 0; m < a.npass && ok; ++m) {
            const TcPass& P = m ? P1 : P0;
            const int nch = P.W.nchunks;
            if (a.npass > 1 && (m > 0 || g0 > 0)) {
                // reload the weight tile of this pass (the previous pass's MMAs are complete)
                if (warp == 0) { fence_proxy_async(); issue_a(P.W); }
                ++a_issued;
            }
            // B planes of this group: [chunk][sequence][16 bytes], each 16-byte
            // piece an independent cp.async (the transpose costs nothing)
            if (m == 0 || P.lo_off != P0.lo_off) {
                for (int i = tid; i < kc * gp; i += kTcThreads) {
                    const int j = i / gp, q = i % gp;
                    uint8_t* dl = sbl + ((size_t)j * gp + q) * 16;
                    uint8_t* dh = sbh + ((size_t)j * gp + q) * 16;
                    if (q < gn && j < nch) {
                        const char* r = recs + (size_t)members[g0 + q] * a.rec_bytes;
                        cp_async16(dl, r + P.lo_off + (size_t)j * 16);
                        cp_async16(dh, r + P.hi_off + (size_t)j * 16);
                    } else {
                        *reinterpret_cast<uint4*>(dl) = make_uint4(0, 0, 0, 0);
                        *reinterpret_cast<uint4*>(dh) = make_uint4(0, 0, 0, 0);
                    }
                }
                cp_async_wait_all();
            }
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                if (a_waited < a_issued) ok = mbar_wait(&bar[0], (unsigned)a_waited & 1u);
                if (ok) {
                    const uint32_t dlo = tmem + (uint32_t)(m * 2 * gp), dhi = dlo + (uint32_t)gp;
                    const uint32_t il = umma_idesc_i8(false, 128, gp), ih = umma_idesc_i8(true, 128, gp);
                    for (int k = 0; k < kc / 2; ++k) {
                        const uint64_t da = umma_sdesc(smem_addr(sa) + k * 4096, 2048, 128);
                        const uint64_t dbl = umma_sdesc(smem_addr(sbl) + k * 2 * gp * 16, gp * 16, 128);
                        const uint64_t dbh = umma_sdesc(smem_addr(sbh) + k * 2 * gp * 16, gp * 16, 128);
                        umma_i8(dlo, da, dbl, il, k > 0);
                        umma_i8(dhi, da, dbh, ih, k > 0);
                    }
                    umma_commit(&bar[1]);
                }
            }
            a_waited = a_issued;
            ok = !__syncthreads_or(!(tid != 0 || ok));
            if (!ok) break;
            ok = !__syncthreads_or(!mbar_wait(&bar[1], mph & 1u));
            ++mph;
            tc_fence_after();
        }
        if (!ok) break;
        // epilogue: row `row` (this thread's TMEM lane), sequences of the group in pieces of 16
        const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
        for (int c = 0; c < gp; c += 16) {
            uint32_t lo0[16], hi0[16], lo1[16], hi1[16];
            tmem_ld16(lane_base + c, lo0);
            tmem_ld16(lane_base + gp + c, hi0);
            if (a.npass > 1) {
                tmem_ld16(lane_base + 2 * gp + c, lo1);
                tmem_ld16(lane_base + 3 * gp + c, hi1);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int q = c + i;
                if (q >= gn) break;
                const int b = members[g0 + q];
                const long long S0 = (long long)(int)lo0[i] + 256LL * (long long)(int)hi0[i];
                const long long S1 = a.npass > 1 ? (long long)(int)lo1[i] + 256LL * (long long)(int)hi1[i] : 0;
                const bool live = row < P0.W.rows;
                const int* gs = reinterpret_cast<const int*>(recs + (size_t)b * a.rec_bytes + 2 * (size_t)x_stride(P0.W));
                if (OP == kOpQkv || OP == kOpWo) {
                    if (!live) continue;
                    const int k = gs[g_stride(P0.W)];
                    const float o = __fmul_rn(__fmul_rn((float)mv_epi(S0, __ldg(P0.W.rscale + row)), 1.0f / 256.0f),
                                              ldexpf(1.0f, -k));
                    if (OP == kOpQkv) {
                        s.qkv[(size_t)b * (d.dim + 2 * d.kv_dim) + row] = o;
                    } else {
                        const float xr = __fmul_rn((float)__ldcg(s.x + (size_t)b * d.dim + row), 1.0f / 256.0f);
                        s.x1[(size_t)b * d.dim + row] = (int16_t)q16h(__fadd_rn(xr, o));
                    }
                } else if (OP == kOpGate) {
                    if (!live) continue;
                    const int g = mv_epi(S0, __ldg(P0.W.rscale + row));
                    const int u = mv_epi(S1, __ldg(P1.W.rscale + row));
                    float y = swiglu1(__fmul_rn((float)g, 1.0f / 256.0f), __fmul_rn((float)u, 1.0f / 256.0f));
                    if (a.hs > 0) y = __fmul_rn(y, ldexpf(1.0f, -a.hs));   // metadata key 15 store scale
                    const int qv = q16s(y);
                    const int half = (d.chunk < d.ffn && row >= d.chunk) ? 1 : 0;
                    const int col = row - (half ? d.chunk : 0);
                    char* hr = s.hrec + (size_t)b * a.dr.bytes;
                    hr[(half ? a.dr.lo_b : a.dr.lo_a) + col] = (char)(qv & 0xFF);
                    hr[(half ? a.dr.hi_b : a.dr.hi_a) + col] = (char)(qv >> 8);
                } else if (OP == kOpDown) {
                    if (!live) continue;
                    float o2 = __fmul_rn((float)mv_epi(S0, __ldg(P0.W.rscale + row)), 1.0f / 256.0f);
                    if (a.npass > 1) {
                        const int vb = mv_epi(S1, __ldg(P1.W.rscale + row));
                        // add_q16 of the two chunk outputs (session.cpp:2052-2067)
                        o2 = __fmul_rn((float)q16h(__fadd_rn(o2, __fmul_rn((float)vb, 1.0f / 256.0f))), 1.0f / 256.0f);
                    }
                    const float x1 = __fmul_rn((float)__ldcg(s.x1 + (size_t)b * d.dim + row), 1.0f / 256.0f);
                    s.x[(size_t)b * d.dim + row] = (int16_t)q16h(__fadd_rn(x1, o2));
                } else {
                    unsigned long long key = 0ull;
                    if (live) {
                        const int v = mv_epi(S0, __ldg(P0.W.rscale + row));
                        s.logits[(size_t)b * d.vocab + row] = v;
                        key = logit_key(v, row);
                    }
                    for (int o = 16; o; o >>= 1) {
                        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                        key = k2 > key ? k2 : key;
                    }
                    if (lane == 0 && key) atomicMax(&s.best[b], key);
                }
            }
        }
        tc_fence_before();
        __syncthreads();   // accumulators and B planes are free for the next group
        tc_fence_after();
    }
    if (!ok && tid == 0) {
        // a copy or the MMAs did not complete in time: report, and wait (bounded) before freeing TMEM
        atomicExch(s.err, kErrCopyTimeout);
        mbar_wait(&bar[0], (unsigned)a_waited & 1u, 10000000ull);
        mbar_wait(&bar[1], mph & 1u, 10000000ull);
    }
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
    if (OP == kOpLogits) logits_finish(s, 0, n, fz);
}
