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
    __shared__ int wc[kWarps];
    __shared__ int base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) base = 0;
    for (int r = 0; r < n; r += kThreads) {
        const int b = r + threadIdx.x;
        const bool f = b < n && (!moe || __ldcg(s.route + (size_t)b * d.layers + layer) == expert);
        const unsigned m = __ballot_sync(0xffffffffu, f);
        if (lane == 0) wc[warp] = __popc(m);
        __syncthreads();
        int off = base;
        for (int w = 0; w < warp; ++w) off += wc[w];
        if (f) members[off + __popc(m & ((1u << lane) - 1u))] = b;
        __syncthreads();
        if (threadIdx.x == 0) for (int w = 0; w < kWarps; ++w) base += wc[w];
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
