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
        const float g = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), pow2f(-k));
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
    // matvec_s scales qkv, wo and, in the host FFN, the gate/up input
    const int k = (op == kOpQkv || op == kOpWo || (op == kOpGate && d.hostffn)) ? scale_exponent(x, d.dim, red) : 0;
    if (op == kOpGate && d.hostffn && threadIdx.x < 2) s.hmax[hmax_at(layer, b, threadIdx.x, s.slots)] = 0;
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
__device__ __forceinline__ void mm_dots(const char* wsm, int nch, int stride, int ja, int jb,
                                        const char* const (&recs)[kMmNI], int ni, long long (&S)[kMmNI]) {
    constexpr int cpc = WT == W_Q8 ? 16 : WT == W_Q4 ? 32 : 64;
    const int lane = threadIdx.x & 31;
    const int4* wv = reinterpret_cast<const int4*>(wsm) + lane;
    const int* qp = reinterpret_cast<const int*>(wsm + (size_t)nch * 512) + lane;
#pragma unroll
    for (int i = 0; i < kMmNI; ++i) S[i] = 0;
#pragma unroll 2
    for (int j = ja; j < jb; ++j) {
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
}

// partial dot products when the warps of a sequence pair split its chunks:
// reserved only for groups of at most two pairs, the ones that split
constexpr size_t kMmPartBytes = sizeof(long long) * kWarps * kMmNI * 32 * 2;
__host__ __device__ inline bool mm_splits_chunks(int group) { return group <= 2 * kMmNI; }
__host__ __device__ inline size_t mm_smem(const DMat& W, int nmat, int group, int n) {
    return align128(nmat * mm_wbytes(W)) + (size_t)group * xrec_bytes(W) + align16(sizeof(int) * (size_t)n) + 64 +
           (mm_splits_chunks(group) ? kMmPartBytes : 0);
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
    long long* part = reinterpret_cast<long long*>(reinterpret_cast<char*>(bar) + 64);
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
        // one copy per record, issued by lane 0 of every warp in turn: one
        // thread's bulk copies complete one after another
        if (lane == 0) {
            fence_proxy_async();
            if (warp == 0) mbar_expect_tx(&bar[1], (unsigned)(gn * rb));
            for (int i = warp; i < gn; i += kWarps)
                bulk_g2s(rsm + i * rb, s.xrec + (size_t)members[g0 + i] * rb, (unsigned)rb, &bar[1]);
        }
        ok = mbar_wait(&bar[1], (unsigned)gi & 1u);
        if (__syncthreads_or(!ok)) { ok = false; break; }
        // Groups of at most two sequence pairs (six of the eight warps would
        // idle): the warps of a pair split its chunks into nsl slices and add
        // their exact partial sums through shared memory.  Larger groups keep
        // one warp per pair and no partial-sum space (its 8 KB per CTA cost
        // c2, whose groups are larger, about 4%).
        // (not for q4: its gate form then needs 108 registers instead of 68, and
        // c2, the q4 many-sequence configuration, runs groups too large to split)
        const int npair = (gn + kMmNI - 1) / kMmNI;
        const int nsl = WT != W_Q4 && mm_splits_chunks(group) ? kWarps / npair : 1;
        if (nsl > 1) {
            const int p = warp % npair, sl = warp / npair;
            if (sl < nsl) {
                const int i0 = p * kMmNI, ni = min(kMmNI, gn - i0);
                const char* recs[kMmNI];
#pragma unroll
                for (int i = 0; i < kMmNI; ++i) recs[i] = rsm + (size_t)(i0 + (i < ni ? i : 0)) * rb;
                long long S[kMmNI], S3[kMmNI];
                const int ja = sl * nch / nsl, jb = (sl + 1) * nch / nsl;
                mm_dots<WT>(sm, nch, stride, ja, jb, recs, ni, S);
                if (OP == kOpGate) mm_dots<WT>(sm + wb, nch, stride, ja, jb, recs, ni, S3);
#pragma unroll
                for (int i = 0; i < kMmNI; ++i) {
                    part[((sl * npair + p) * kMmNI + i) * 32 + lane] = S[i];
                    if (OP == kOpGate) part[((kWarps + sl * npair + p) * kMmNI + i) * 32 + lane] = S3[i];
                }
            }
            __syncthreads();
        }
        for (int i0 = warp * kMmNI; i0 < gn; i0 += kWarps * kMmNI) {
            const int ni = min(kMmNI, gn - i0);
            const char* recs[kMmNI];
#pragma unroll
            for (int i = 0; i < kMmNI; ++i) recs[i] = rsm + (size_t)(i0 + (i < ni ? i : 0)) * rb;
            long long S[kMmNI], S3[kMmNI];
            if (nsl > 1) {   // this warp's pair is warp; its slices' sums
#pragma unroll
                for (int i = 0; i < kMmNI; ++i) {
                    S[i] = 0;
                    S3[i] = 0;
                    for (int sl = 0; sl < nsl; ++sl) {
                        S[i] += part[((sl * npair + warp) * kMmNI + i) * 32 + lane];
                        if (OP == kOpGate) S3[i] += part[((kWarps + sl * npair + warp) * kMmNI + i) * 32 + lane];
                    }
                }
            } else {
                mm_dots<WT>(sm, nch, stride, 0, nch, recs, ni, S);
                if (OP == kOpGate) mm_dots<WT>(sm + wb, nch, stride, 0, nch, recs, ni, S3);
            }
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
                            __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), pow2f(-k));
                } else if (OP == kOpWo) {
                    if (live) {
                        const float wo = __fmul_rn(__fmul_rn((float)v, 1.0f / 256.0f), pow2f(-k));
                        const float xr = __fmul_rn((float)__ldcg(s.x + (size_t)b * d.dim + row), 1.0f / 256.0f);
                        s.x1[(size_t)b * d.dim + row] = (int16_t)q16h(__fadd_rn(xr, wo));
                    }
                } else if (OP == kOpGate) {
                    int q = 0;
                    if (live) {
                        const int u = mv_epi(S3[i] - corr, rs3[lane]);
                        if (d.hostffn) {
                            q = host_hidden(v, u, k);
                        } else {
                            float y = swiglu1(__fmul_rn((float)v, 1.0f / 256.0f), __fmul_rn((float)u, 1.0f / 256.0f));
                            if (hs > 0) y = __fmul_rn(y, ldexpf(1.0f, -hs));     // metadata key 15 store scale
                            q = q16s(y);
                        }
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
                    if (d.hostffn) {
                        const int mq = __reduce_max_sync(0xffffffffu, abs(q));
                        if (lane == 0 && mq) atomicMax(s.hmax + hmax_at(layer, b, half, s.slots), mq);
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
__global__ void __launch_bounds__(kThreads) k_mmdown(MatSet M2, State s, Batch bt, Dims d, int layer, int group,
                                                     int hs) {
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
        if (lane == 0) {   // records issued by lane 0 of every warp in turn (as in k_mm)
            fence_proxy_async();
            if (warp == 0) mbar_expect_tx(&bar[1], (unsigned)(gn * R.bytes));
            for (int i = warp; i < gn; i += kWarps)
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
            mm_dots<WT>(sm, Wa.nchunks, sa, 0, Wa.nchunks, ra, ni, Sa);
            if (two) mm_dots<WT>(sm + wba, Wb.nchunks, sb, 0, Wb.nchunks, rb2, ni, Sb);
#pragma unroll
            for (int i = 0; i < kMmNI; ++i) {
                if (i >= ni || row >= Wa.rows) continue;
                const int b = members[g0 + i0 + i];
                const long long ca = WT == W_T3 ? reinterpret_cast<const int*>(ra[i] + R.g_a)[0] : 0;
                float o2;
                if (d.hostffn) {
                    const long long cb = WT == W_T3 ? reinterpret_cast<const int*>(ra[i] + R.g_b)[0] : 0;
                    const float oa = host_w2_out(Sa[i] - ca, rsa[lane], hidden_exp(s, layer, b, 0), hs, s.err);
                    const float ob = host_w2_out(Sb[i] - cb, rsb[lane], hidden_exp(s, layer, b, 1), hs, s.err);
                    o2 = __fmul_rn((float)q16h(__fadd_rn(oa, ob)), 1.0f / 256.0f);
                } else {
                    o2 = __fmul_rn((float)mv_epi(Sa[i] - ca, rsa[lane]), 1.0f / 256.0f);
                    if (two) {
                        const long long cb = WT == W_T3 ? reinterpret_cast<const int*>(ra[i] + R.g_b)[0] : 0;
                        const int vb = mv_epi(Sb[i] - cb, rsb[lane]);
                        // add_q16 of the two chunk outputs (session.cpp:2052-2067)
                        o2 = __fmul_rn((float)q16h(__fadd_rn(o2, __fmul_rn((float)vb, 1.0f / 256.0f))), 1.0f / 256.0f);
                    }
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
// Tensor-core matmat for q8 and t3 weights (tcgen05.mma kind::i8, TMEM accumulators).
//
// One CTA computes a 128-row tile of one matrix (or of two:
// w1 and w3 of the ffn, or the two column halves of a chunked w2) for a group
// of N consecutive sequences of the batch.  K streams through a ring of
// shared-memory stages of 128 bytes of every row, filled by 2-D TMA copies
// (cp.async.bulk.tensor, 128-byte swizzle) and completed on `full` mbarriers;
// one MMA thread consumes a stage as soon as it lands and hands it back
// through `empty` (tcgen05.commit), so copies and MMAs overlap and K has no
// shared-memory limit.
//  - A (weights): the matrix's row-major int8 copy (q8 levels, or t3's
//    -1/0/+1, so S is the plain integer dot); a stage holds 128 rows x 128
//    bytes, copied as two boxes of 64 rows.  Rows past the matrix and K past
//    its end read as zero (out-of-bounds fill).
//  - B (inputs): the sequences' staged records, n rows of rec_bytes; a stage
//    holds N rows x 128 bytes of the lo and of the hi plane, each copied as
//    two boxes of N/2 rows.  x' = lo + 256*hi with lo
//    unsigned and hi signed, so every K step is two MMAs (s8 x u8 into one
//    accumulator, s8 x s8 into another) and S = D_lo + 256*D_hi is the exact
//    integer dot (|D| < 2^31 for every shape here).
// Measured on B200: one thread's TMA copies complete one after another (about
// 0.2 us for a box with 16-byte rows, 0.55 us for a 16 KB box of 128-byte
// rows), while copies issued by different warps proceed side by side.  So
// every box is 128 bytes wide and each box of a stage has an issuing thread
// of its own (lane 0 of one warp each, up to 12).
// tcgen05.ld brings row r of the accumulators to lane r%32 of the warps of
// quarter r/32; sixteen warps share the epilogues (those of the CUDA-core
// kernels, so the results are theirs bit for bit), which are instruction-bound:
// with one warpgroup they took most of the kernel's time.
// ---------------------------------------------------------------------------

constexpr int kOpDown = 4;
// Epilogue variants for measurement builds (-D): the ffn matmats' piece width,
// and the double-precision rounding path instead of the integer form.
#ifndef VC4_TMM_PW_FFN
#define VC4_TMM_PW_FFN 2
#endif
#ifndef VC4_TMM_DBL
#define VC4_TMM_DBL 1
#endif
constexpr int kTcPwFfn = VC4_TMM_PW_FFN;
constexpr bool kTcDoubleEpi = VC4_TMM_DBL != 0;
constexpr int kTcThreads = 512;          // lane 0 of warp 1 issues the MMAs, of others the copies; all 16 run the epilogue
constexpr int kTcKs = 8;                  // 16-byte K chunks per ring stage: one 128-byte swizzle row
constexpr int kTcMaxStages = 8;
constexpr size_t kTcTileA = 128 * 128;    // bytes of one stage of a 128-row weight tile

// K-major operand in the 128-byte swizzle layout that a SWIZZLE_128B TMA box
// writes: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO); the leading
// offset is unused.  `addr` lies in a 1024-byte aligned atom, plus the K
// step's byte offset within the row.
__device__ __forceinline__ uint64_t umma_sdesc_sw128(unsigned addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                 // leading byte offset (unused): 16 bytes
    d |= (uint64_t)(1024u >> 4) << 32;      // stride byte offset
    d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                 // 128-byte swizzle
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
// 16 consecutive 32-bit accumulator columns of this thread's TMEM lane (the
// registers are valid after tmem_wait_ld)
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(addr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(addr));
}
__device__ __forceinline__ void tmem_ld4(uint32_t addr, uint32_t (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(addr));
}
__device__ __forceinline__ void tmem_ld2(uint32_t addr, uint32_t (&v)[2]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(v[0]), "=r"(v[1]) : "r"(addr));
}
template <int W>
__device__ __forceinline__ void tmem_ld(uint32_t addr, uint32_t (&v)[W]) {
    if constexpr (W == 16) tmem_ld16(addr, v);
    else if constexpr (W == 8) tmem_ld8(addr, v);
    else if constexpr (W == 4) tmem_ld4(addr, v);
    else tmem_ld2(addr, v);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Adds `bytes` to the transaction count of the barrier's current phase
// without arriving (the copies of a stage issued before its arrival).
__device__ __forceinline__ void mbar_add_tx(unsigned long long* bar, unsigned bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// 2-D tiled TMA load (no multicast) of box (x, y) of `map` into shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, unsigned long long* bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)) : "memory");
}

struct TcPass {        // one matrix of a tensor-core matmat and where its B bytes live in a record
    DMat W;
    int lo_off, hi_off;
};
struct TcMaps {        // TMA descriptors, passed by value (__grid_constant__)
    CUtensorMap a[2];  // weights of pass 0 / 1
    CUtensorMap b;     // the records
};
struct TcArgs {
    TcPass p[2];
    int npass;
    int nin;             // distinct B inputs: 2 when the passes read different record bytes
    int rec_bytes;       // bytes per sequence record (State::xrec or State::hrec)
    int from_hrec;       // the records are w2 inputs (State::hrec)
    int tiles;           // 128-row tiles of the matrix
    int groups;          // > 0: aligned split, CTA c = group c % groups of tile c / groups; 0: balanced ranges
    int group;           // N: sequences per round (multiple of 16, at most 256)
    int tmem_cols;       // power of two >= 2 * npass * group
    int stages;          // ring depth (at least 2)
    int kc;              // 16-byte K chunks of the longer pass (even)
    int t3;              // ternary weights: the gate also adds the hidden totals the CUDA-core w2 uses
    int hs;
    DownRec dr;
};

// 16-byte K chunks of a row-major row, even (K steps of 32)
__host__ __device__ inline int tc_kchunks(const DMat& W) { return (x_stride(W) / 16 + 1) & ~1; }
__host__ __device__ inline size_t tc_stage_bytes(const TcArgs& a) {
    return (size_t)a.npass * kTcTileA + (size_t)a.nin * 2 * a.group * 128;
}
// ring (1024-byte aligned) | full[stages] | empty[stages] | done | tfree |
// TMEM address (16 bytes) | two rounds' input exponents
__host__ __device__ inline size_t tc_smem(const TcArgs& a) {
    return 1024 + (size_t)a.stages * tc_stage_bytes(a) + 8 * (2 * (size_t)a.stages + 2) + 16 + 8 * (size_t)a.group;
}

// The work split.  The (tile, unit of 16 sequences) pairs, tile-major, are
// either cut into gridDim.x equal ranges (balanced) or grouped N/16 units at
// a time inside each tile (aligned, one CTA per group); a CTA takes its range
// in rounds, each inside one tile and at most N sequences.
struct TcRound {
    int tile, g0, gn;
};
__device__ __forceinline__ bool tc_round_at(int r, int u_begin, int u_end, int upt, int umax, int n, TcRound& o) {
    int u = u_begin;
    for (int i = 0;; ++i) {
        if (u >= u_end) return false;
        const int tile = u / upt, ut = u - tile * upt;
        const int nu = min(min(u_end - u, upt - ut), umax);
        if (i == r) {
            o.tile = tile;
            o.g0 = 16 * ut;
            o.gn = min(16 * nu, n - 16 * ut);
            return true;
        }
        u += nu;
    }
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Every instance keeps to 64 registers so that two CTAs share an SM: one's
// epilogue then overlaps the other's copies and MMAs, and each sub-partition
// has eight warps to hide the epilogue's latencies.
template <int OP>
__global__ void __launch_bounds__(kTcThreads, 2) k_tmm(const __grid_constant__ TcMaps maps, TcArgs a, State s, Batch bt,
                                                       Dims d, int layer, Finalize fz) {
    const int N = a.group, S = a.stages;
    const int n = bt.n, upt = (n + 15) / 16, umax = N / 16;
    const long long U = (long long)a.tiles * upt;
    int u_begin, u_end;
    if (a.groups) {   // aligned: CTA c is group c % groups of tile c / groups
        const int tile = (int)blockIdx.x / a.groups, grp = (int)blockIdx.x % a.groups;
        u_begin = tile * upt + grp * umax;
        u_end = min(u_begin + umax, (tile + 1) * upt);
    } else {          // balanced: equal ranges of the tile-major units
        u_begin = (int)(U * blockIdx.x / gridDim.x);
        u_end = (int)(U * (blockIdx.x + 1) / gridDim.x);
    }
    if (!smem_ok(tc_smem(a), s.err)) return;
    if (S < 2 || N % 16 || N < 16 || 2 * a.npass + 4 * a.nin > kTcThreads / 32 - 1) {   // see the issuers below
        if (threadIdx.x == 0) atomicExch(s.err, kErrRingShape);
        return;
    }
    int R = 0;
    for (TcRound t; tc_round_at(R, u_begin, u_end, upt, umax, n, t);) ++R;
    char* base = SmemLayout::base();
    char* ring = base + ((1024u - (smem_addr(base) & 1023u)) & 1023u);
    const size_t sb = tc_stage_bytes(a);
    unsigned long long* full = reinterpret_cast<unsigned long long*>(ring + (size_t)S * sb);
    unsigned long long* empty = full + S;
    unsigned long long* done = empty + S;
    unsigned long long* tfree = done + 1;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tfree + 1);
    int* kexp2 = reinterpret_cast<int*>(tslot + 4);        // [2][N]: the rounds' input exponents
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // qkv, wo and logits read one matrix: a constant, so the second
    // accumulator's code and registers compile away
    constexpr bool kOne = OP == kOpQkv || OP == kOpWo || OP == kOpLogits;
    const int npass = kOne ? 1 : a.npass, nin = kOne ? 1 : a.nin, kc = a.kc, nst = (kc + kTcKs - 1) / kTcKs;
    const int kcp[2] = {tc_kchunks(a.p[0].W), tc_kchunks(a.p[npass > 1 ? 1 : 0].W)};
    const size_t boff = (size_t)npass * kTcTileA;          // B planes inside a stage
    const unsigned bplane = (unsigned)N * 128u;            // bytes of one plane of one stage
    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < S; ++i) {
                mbar_init(&full[i], 1);
                mbar_init(&empty[i], 1);
            }
            mbar_init(done, 1);
            mbar_init(tfree, kTcThreads / 32);
            mbar_fence_init();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tslot)),
                     "r"(a.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // every CTA holds its TMEM before the dependent grid may start (a dependent
    // tensor-core grid allocates before its own wait)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_launch_dependents();

    // Global stage gi = r * nst + i covers K chunks 8i .. 8i+7 (128 bytes of
    // every row) of round r: one box per pass of the weights, one per plane
    // and input of the records.
    auto a_live = [&](int i, int p) { return i * kTcKs < kcp[p]; };
    auto b_live = [&](int i, int in) { return i * kTcKs < (nin > 1 ? kcp[in] : kc); };
    auto a_bytes = [&](int i) {
        unsigned b = 0;
        for (int p = 0; p < npass; ++p) b += a_live(i, p) ? (unsigned)kTcTileA : 0u;
        return b;
    };
    auto b_bytes = [&](int i) {
        unsigned b = 0;
        for (int in = 0; in < nin; ++in) b += b_live(i, in) ? 2u * bplane : 0u;
        return b;
    };
    // Box j of every stage has its own issuing thread (one thread's bulk
    // copies complete one after another, copies from different threads side
    // by side).  Each box is half of a tile: 64 weight rows, or N/2 records,
    // both whole 1024-byte swizzle atoms, so the halves land exactly where one
    // box of the whole tile would.  Boxes 0 .. 2*npass-1 are the weights
    // (pass j/2), then four per record input (plane, half).
    const int nbA = 2 * npass, nb = nbA + 4 * nin;
    const int my_box = warp == 0 ? 0 : warp - 1;        // warp 1 issues the MMAs
    const bool issuer = warp != 1 && lane == 0 && my_box < nb;
    auto box_live = [&](int i, int j) {
        return j < nbA ? a_live(i, j >> 1) : b_live(i, (j - nbA) >> 2);
    };
    auto issue_box = [&](int gi, int j, const TcRound& rd) {
        const int i = gi % nst;
        char* st = ring + (size_t)(gi % S) * sb;
        unsigned long long* bar = &full[gi % S];
        if (j < nbA) {
            const int p = j >> 1, h = j & 1;
            tma_load_2d(st + (size_t)p * kTcTileA + (size_t)h * (kTcTileA / 2), &maps.a[p], i * 128,
                        rd.tile * 128 + 64 * h, bar);
        } else {
            const int jb = j - nbA, in = jb >> 2, plane = (jb >> 1) & 1, h = jb & 1;
            const TcPass& Pi = a.p[in];
            tma_load_2d(st + boff + (size_t)(in * 2 + plane) * bplane + (size_t)h * (bplane / 2), &maps.b,
                        (plane ? Pi.hi_off : Pi.lo_off) + i * 128, rd.g0 + h * (N / 2), bar);
        }
    };

    // Every issuer takes every stage in order, so it refills a slot only after
    // the MMAs read the slot's previous contents, and the slot cannot be
    // consumed again before this issuer's own box of the next contents lands:
    // each wait on an `empty` barrier is for the phase right after the one the
    // issuer saw last (a parity wait cannot tell phases two apart).  Issuer 0
    // also arrives on the stage's `full` barrier with the stage's bytes.
    bool bad = false;        // one of this thread's bounded waits gave up
    int next = 0;            // the issuer's next global stage
    TcRound r0{0, 0, 0};
    if (R > 0) tc_round_at(0, u_begin, u_end, upt, umax, n, r0);
    const int pre = min(S, nst);
    if (issuer && R > 0) {
        if (my_box == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&maps.a[0]) : "memory");
            if (npass > 1) asm volatile("prefetch.tensormap [%0];" ::"l"(&maps.a[1]) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&maps.b) : "memory");
            for (int gi = 0; gi < pre; ++gi) mbar_expect_tx(&full[gi], a_bytes(gi) + b_bytes(gi));
        }
        // the first stages' weights before the grid-dependency wait
        if (my_box < nbA)
            for (int gi = 0; gi < pre; ++gi)
                if (box_live(gi, my_box)) issue_box(gi, my_box, r0);
    }
    pdl_wait();
    if (issuer && R > 0) {
        if (my_box >= nbA)
            for (int gi = 0; gi < pre; ++gi)
                if (box_live(gi, my_box)) issue_box(gi, my_box, r0);
        next = pre;
    }
    // Issues this thread's box of the stages below `limit`; a stage waits only
    // for the MMAs that read its slot before.
    auto produce_until = [&](int limit) {
        while (!bad && next < limit) {
            const int gi = next, i = gi % nst;
            TcRound rd;
            tc_round_at(gi / nst, u_begin, u_end, upt, umax, n, rd);
            if (gi >= S && !mbar_wait(&empty[gi % S], (unsigned)(gi / S - 1) & 1u)) {
                bad = true;
                break;
            }
            if (my_box == 0) mbar_expect_tx(&full[gi % S], a_bytes(i) + b_bytes(i));
            if (box_live(i, my_box)) issue_box(gi, my_box, rd);
            ++next;
        }
    };

    const TcPass P0 = a.p[0], P1 = a.p[npass > 1 ? 1 : 0];
    const int quarter = warp & 3, slice = warp >> 2, nslice = kTcThreads / 128;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
    bool failed = false;
    for (int r = 0; r < R; ++r) {
        TcRound rd;
        tc_round_at(r, u_begin, u_end, upt, umax, n, rd);
        const int g0 = rd.g0, gn = rd.gn, Nr = (gn + 15) & ~15;
        int* kexp = kexp2 + (r & 1) * N;
        // this round's remaining stages and the next round's first ones (their
        // slots are freed by this round's MMAs, never by its epilogue)
        if (issuer) produce_until(min(R * nst, (r + 1) * nst + (r + 1 < R ? pre : 0)));
        __syncwarp();
        if (warp == 1) {
            if (lane == 0) {
                // MMA issuer: four K steps of 32 bytes per stage, inside the
                // 128-byte swizzle row by advancing the descriptors' start
                // address; the accumulators are free once every warp has read
                // the previous round's
                if (r > 0 && !mbar_wait(tfree, (unsigned)(r - 1) & 1u)) bad = true;
                tc_fence_after();
                const uint32_t il = umma_idesc_i8(false, 128, Nr), ih = umma_idesc_i8(true, 128, Nr);
                for (int i = 0; i < nst && !bad; ++i) {
                    const int gi = r * nst + i;
                    if (!mbar_wait(&full[gi % S], (unsigned)(gi / S) & 1u)) {
                        bad = true;
                        break;
                    }
                    tc_fence_after();
                    const char* st = ring + (size_t)(gi % S) * sb;
                    for (int kk = 0; kk < kTcKs / 2; ++kk) {
                        const int j = i * kTcKs + 2 * kk;
                        for (int p = 0; p < npass; ++p) {
                            if (j >= kcp[p]) continue;
                            const int in = nin > 1 ? p : 0;
                            const uint64_t da = umma_sdesc_sw128(smem_addr(st + (size_t)p * kTcTileA) + 32u * kk);
                            const uint64_t dbl =
                                umma_sdesc_sw128(smem_addr(st + boff + (size_t)(in * 2 + 0) * bplane) + 32u * kk);
                            const uint64_t dbh =
                                umma_sdesc_sw128(smem_addr(st + boff + (size_t)(in * 2 + 1) * bplane) + 32u * kk);
                            const uint32_t dlo = tmem + (uint32_t)(p * 2 * N);
                            umma_i8(dlo, da, dbl, il, j > 0);
                            umma_i8(dlo + (uint32_t)N, da, dbh, ih, j > 0);
                        }
                    }
                    umma_commit(&empty[gi % S]);
                }
                umma_commit(done);   // every MMA issued above, also after a failure
            } else {
                // the other lanes fetch the round's input exponents for the epilogue
                if (OP == kOpQkv || OP == kOpWo || (OP == kOpGate && d.hostffn)) {
                    const char* recs = a.from_hrec ? s.hrec : s.xrec;
                    for (int q = lane - 1; q < gn; q += 31)
                        kexp[q] = reinterpret_cast<const int*>(recs + (size_t)(g0 + q) * a.rec_bytes +
                                                               2 * (size_t)x_stride(P0.W))[g_stride(P0.W)];
                }
                if (OP == kOpDown && d.hostffn)   // the w2 input exponents of both hidden halves
                    for (int q = lane - 1; q < gn; q += 31) {
                        const int ka = hidden_exp(s, layer, g0 + q, 0), kb = hidden_exp(s, layer, g0 + q, 1);
                        // a negative exponent (hidden value >= 64) is refused here, once per sequence
                        if (ka < 0 || kb < 0) atomicExch(s.err, kErrHiddenRange);
                        kexp[q] = (max(ka, 0) & 0xFFFF) | (max(kb, 0) << 16);
                    }
            }
            __syncwarp();
        }
        // epilogue of the round, by all sixteen warps once its accumulators are
        // complete: warp w reads TMEM lanes 32*(w%4) .. +31 (its rows) and
        // every fourth piece of sequences starting at piece w/4.  The
        // residuals it reads come from the previous grids.
        // One thread waits for the MMAs; the others wait at the block barrier
        // (in hardware, taking no issue slots from the copies and MMAs).
        if (tid == 0 && !mbar_wait(done, (unsigned)r & 1u)) bad = true;
        if (__syncthreads_or(bad)) {
            failed = true;
            break;
        }
        tc_fence_after();
        __syncwarp();   // tcgen05.ld below is warp-aligned
        // pieces of PW sequences: independent chains per warp within the 64
        // registers of two CTAs per SM (single-matrix ops 8; the ffn's two
        // accumulator pairs and SwiGLU or residual chains VC4_TMM_PW_FFN, 2)
        constexpr int PW = kOne ? 8 : kTcPwFfn;
        const int row = rd.tile * 128 + 32 * quarter + lane;
        const bool live = row < P0.W.rows;
        const float rs0 = live ? __ldg(P0.W.rscale + row) : 0.0f;
        const float rs1 = live && npass > 1 ? __ldg(P1.W.rscale + row) : 0.0f;
        const RowScale q0 = row_scale(rs0), q1 = row_scale(rs1);
        for (int c = PW * slice; c < gn; c += PW * nslice) {
            uint32_t lo0[PW], hi0[PW], lo1[PW], hi1[PW];
            tmem_ld<PW>(lane_base + c, lo0);
            tmem_ld<PW>(lane_base + N + c, hi0);
            if (npass > 1) {
                tmem_ld<PW>(lane_base + 2 * N + c, lo1);
                tmem_ld<PW>(lane_base + 3 * N + c, hi1);
            }
            int16_t res[PW];
            if (OP == kOpWo || OP == kOpDown) {
                const int16_t* src = OP == kOpWo ? s.x : s.x1;
#pragma unroll
                for (int i = 0; i < PW; ++i)
                    res[i] = live && c + i < gn ? __ldcg(src + (size_t)(g0 + c + i) * d.dim + row) : (int16_t)0;
            }
            tmem_wait_ld();
            // Every output of the piece is computed without branches (sequences
            // past the group's end compute on whatever their columns hold and are
            // not stored), so the piece's sequences' chains interleave; the stores
            // and the warp reductions follow in a loop of their own.  c and gn are
            // warp-uniform.
            auto S0 = [&](int i) { return (long long)(int)lo0[i] + 256LL * (long long)(int)hi0[i]; };
            auto S1 = [&](int i) { return npass > 1 ? (long long)(int)lo1[i] + 256LL * (long long)(int)hi1[i] : 0LL; };
            // w2 of the host FFN: each half's dot times its input scale 2^k
            auto sh0 = [&](int i) { return OP == kOpDown && d.hostffn ? (kexp[c + i] & 0xFFFF) : 0; };
            auto sh1 = [&](int i) { return OP == kOpDown && d.hostffn ? (kexp[c + i] >> 16) : 0; };
            // the exact rounding of every dot in the integer form, then (rarely,
            // |S| >= 2^28) the double path for the ones it cannot take
            int v0[PW], v1[PW];
            bool slow = false;
#pragma unroll
            for (int i = 0; i < PW; ++i) {
                if (kTcDoubleEpi) {
                    v0[i] = mv_epi(S0(i) * (1LL << sh0(i)), q0.sc);
                    v1[i] = npass > 1 ? mv_epi(S1(i) * (1LL << sh1(i)), q1.sc) : 0;
                    continue;
                }
                bool ok0, ok1 = true;
                v0[i] = mv_epi_int(S0(i) * (1LL << sh0(i)), q0, ok0);
                v1[i] = npass > 1 ? mv_epi_int(S1(i) * (1LL << sh1(i)), q1, ok1) : 0;
                slow |= !(ok0 && ok1);
            }
            if (__any_sync(0xffffffffu, slow)) {
                // the accumulators are read again (TMEM still holds them), so the
                // common path need not keep them live
                uint32_t l0[PW], h0[PW], l1[PW], h1[PW];
                tmem_ld<PW>(lane_base + c, l0);
                tmem_ld<PW>(lane_base + N + c, h0);
                if (npass > 1) {
                    tmem_ld<PW>(lane_base + 2 * N + c, l1);
                    tmem_ld<PW>(lane_base + 3 * N + c, h1);
                }
                tmem_wait_ld();
                for (int i = 0; i < PW; ++i) {
                    v0[i] = mv_epi(((long long)(int)l0[i] + 256LL * (long long)(int)h0[i]) * (1LL << sh0(i)), q0);
                    if (npass > 1)
                        v1[i] = mv_epi(((long long)(int)l1[i] + 256LL * (long long)(int)h1[i]) * (1LL << sh1(i)), q1);
                }
            }
            if (OP == kOpQkv || OP == kOpWo) {
                float o[PW];
#pragma unroll
                for (int i = 0; i < PW; ++i)
                    o[i] = __fmul_rn(__fmul_rn(i2f_small(v0[i]), 1.0f / 256.0f), pow2f(-kexp[c + i]));
                if (live) {
#pragma unroll
                    for (int i = 0; i < PW; ++i) {
                        if (c + i >= gn) continue;
                        const int b = g0 + c + i;
                        if (OP == kOpQkv) {
                            s.qkv[(size_t)b * (d.dim + 2 * d.kv_dim) + row] = o[i];
                        } else {
                            const float xr = __fmul_rn(i2f_small(res[i]), 1.0f / 256.0f);
                            s.x1[(size_t)b * d.dim + row] = (int16_t)q16h(__fadd_rn(xr, o[i]));
                        }
                    }
                }
            } else if (OP == kOpGate) {
                // dead rows have zero row scales, so g = u = 0 and their hidden value is 0
                int qv[PW];
                if (d.hostffn) {
#pragma unroll
                    for (int i = 0; i < PW; ++i) qv[i] = host_hidden(v0[i], v1[i], kexp[c + i]);
                } else {
                    const float hsc = pow2f(-a.hs);   // metadata key 15 store scale (exact)
#pragma unroll
                    for (int i = 0; i < PW; ++i) {
                        float y = swiglu1(__fmul_rn(i2f_small(v0[i]), 1.0f / 256.0f),
                                          __fmul_rn(i2f_small(v1[i]), 1.0f / 256.0f));
                        if (a.hs > 0) y = __fmul_rn(y, hsc);
                        qv[i] = q16s(y);
                    }
                }
                // a warp's 32 rows lie in one w2 column half (the chunk is a multiple of 32)
                const int half = (d.chunk < d.ffn && row >= d.chunk) ? 1 : 0;
                const int col = row - (half ? d.chunk : 0);
                const int off_lo = (half ? a.dr.lo_b : a.dr.lo_a) + col, off_hi = (half ? a.dr.hi_b : a.dr.hi_a) + col;
                const int off_g = half ? a.dr.g_b : a.dr.g_a;
#pragma unroll
                for (int i = 0; i < PW; ++i) {
                    if (c + i >= gn) continue;
                    char* hr = s.hrec + (size_t)(g0 + c + i) * a.dr.bytes;
                    if (live) {
                        hr[off_lo] = (char)(qv[i] & 0xFF);
                        hr[off_hi] = (char)(qv[i] >> 8);
                    }
                    if (a.t3) {   // the hidden total of the CUDA-core w2's offset codes
                        const int sum = __reduce_add_sync(0xffffffffu, qv[i]);
                        if (lane == 0) atomicAdd(reinterpret_cast<int*>(hr + off_g), sum);
                    }
                    if (d.hostffn) {
                        const int mq = __reduce_max_sync(0xffffffffu, abs(qv[i]));
                        if (lane == 0 && mq) atomicMax(s.hmax + hmax_at(layer, g0 + c + i, half, s.slots), mq);
                    }
                }
            } else if (OP == kOpDown) {
                float o2[PW];
                if (d.hostffn) {
                    // host_w2_out of each half, then add_q16 of the halves
#pragma unroll
                    for (int i = 0; i < PW; ++i) {
                        const float oa = __fmul_rn(__fmul_rn(i2f_small(v0[i]), 1.0f / 256.0f), pow2f(-(sh0(i) + a.hs)));
                        const float ob = __fmul_rn(__fmul_rn(i2f_small(v1[i]), 1.0f / 256.0f), pow2f(-(sh1(i) + a.hs)));
                        o2[i] = __fmul_rn(i2f_small(q16h(__fadd_rn(oa, ob))), 1.0f / 256.0f);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < PW; ++i) {
                        o2[i] = __fmul_rn(i2f_small(v0[i]), 1.0f / 256.0f);
                        if (npass > 1)   // add_q16 of the two chunk outputs (session.cpp:2052-2067)
                            o2[i] = __fmul_rn(i2f_small(q16h(__fadd_rn(o2[i], __fmul_rn(i2f_small(v1[i]), 1.0f / 256.0f)))),
                                              1.0f / 256.0f);
                    }
                }
                if (live) {
#pragma unroll
                    for (int i = 0; i < PW; ++i) {
                        if (c + i >= gn) continue;
                        const float x1 = __fmul_rn(i2f_small(res[i]), 1.0f / 256.0f);
                        s.x[(size_t)(g0 + c + i) * d.dim + row] = (int16_t)q16h(__fadd_rn(x1, o2[i]));
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < PW; ++i) {
                    const int q = c + i;
                    if (q >= gn) continue;
                    const int b = g0 + q;
                    unsigned long long key = 0ull;
                    if (live) {
                        s.logits[(size_t)b * d.vocab + row] = v0[i];
                        key = logit_key(v0[i], row);
                    }
                    for (int o = 16; o; o >>= 1) {
                        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                        key = k2 > key ? k2 : key;
                    }
                    if (lane == 0 && key) atomicMax(&s.best[b], key);
                }
            }
        }
        // the accumulators may be overwritten once every warp has read them
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tfree);
    }
    if (failed && tid == 0) {
        // a copy or the MMAs did not complete in time: report, and wait (bounded)
        // for the stages still in flight before the shared memory and TMEM go
        atomicExch(s.err, kErrCopyTimeout);
        for (int i = 0; i < S; ++i) mbar_wait(&full[i], 0u, 10000000ull), mbar_wait(&full[i], 1u, 10000000ull);
        mbar_wait(done, 0u, 10000000ull), mbar_wait(done, 1u, 10000000ull);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
    if (OP == kOpLogits) logits_finish(s, 0, n, fz);
}
