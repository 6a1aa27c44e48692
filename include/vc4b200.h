/*
 * vc4b200.h -- C ABI of the B200 quantized decode engine.
 *
 * The reference engine has no plugin or FFI layer: its decode path sits
 * behind the C++ class `GPU` (engine/src/gpu.h:41-633) as driven by
 * `Session` (engine/src/session.h:28-93).  These entry points are what that
 * class and the layer loop call, expressed as plain C: opaque handles,
 * pointers and sizes, int status codes (0 = OK) and a thread-local message.
 * Every entry point names the reference interface it replaces.
 *
 * Numerics: the reference CPU layer loop (session.cpp:373-556) with the
 * shader arithmetic of each matrix it draws and the packed KV codec; all
 * weight x activation products are exact integers.  Logits are on the q16
 * grid (1/256).
 */
#ifndef VC4B200_H
#define VC4B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VC4_API __attribute__((visibility("default")))
#else
#define VC4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define VC4_OK 0
#define VC4_EINVAL 1      /* bad argument (shape, slot, position, kv axis) */
#define VC4_EFORMAT 2     /* container refused (bad or unsupported file)    */
#define VC4_ECUDA 3       /* a CUDA call failed                             */
#define VC4_EIO 4         /* file I/O                                       */
#define VC4_ESTATE 5      /* wrong call order / mismatched cache            */
#define VC4_ERANGE 6      /* an activation left the range the kernels compute */

typedef struct vc4_gpu vc4_gpu;         /* device + stream (class GPU)            */
typedef struct vc4_model vc4_model;     /* uploaded weights (Model + GPU::upload) */
typedef struct vc4_session vc4_session; /* KV cache + activations, N slots        */

typedef struct {
    int dim, hidden, layers, heads, kv_heads, vocab, seq, head_dim, kv_dim;
    int experts, moe_hidden, ffn_width, ffn_chunked, ffn_chunk;
    int qk_norm, rope_half, head_dedup, wtype; /* wtype: 0 q8, 1 q4, 2 t3 */
    float rope_theta, rms_eps;
    uint64_t weight_bytes;                     /* device bytes of all matrices */
    uint64_t source_size, source_mtime;        /* container identity (MMKV1)   */
} vc4_model_info;

/* Message of the last failed call on this thread ("" when none). */
VC4_API const char* vc4_last_error(void);

/* GPU::GPU() / ~GPU (gpu.cpp:31-42): bind a CUDA device, create the stream. */
VC4_API int vc4_gpu_create(int device, vc4_gpu** out);
VC4_API void vc4_gpu_destroy(vc4_gpu* g);
/* GPU::sync (gpu.cpp:53): wait for all queued work. */
VC4_API int vc4_gpu_sync(vc4_gpu* g);

/* Model::load (model.cpp:23) + GPU::upload for every matrix
   (gpu_upload.cpp:20-192): parse the MMCF container, re-lay the quantised
   blocks into the device layout and copy them to HBM. */
VC4_API int vc4_model_load(vc4_gpu* g, const char* mmcf_path, vc4_model** out);
VC4_API int vc4_model_load_bytes(vc4_gpu* g, const void* data, size_t size, vc4_model** out);
VC4_API int vc4_model_info_get(const vc4_model* m, vc4_model_info* out);
/* Model::probe (model.h:209-216): parse and validate a container on the host
   without touching a GPU (this build validates every tensor record, not only
   the header and metadata); fills info, or returns VC4_EFORMAT / VC4_EIO with
   the reader's message. */
VC4_API int vc4_model_probe(const char* mmcf_path, vc4_model_info* out);
VC4_API void vc4_model_free(vc4_model* m);

/* Session::reset's device half: GPU::init_attention (gpu_attn.cpp:41-157)
   with the KV axis (kv_bits 16 = q16 grid 1/2048, 8 = q8 grid 1/16) and
   GPU::init_persistent (gpu_upload.cpp:196-220).  rope_cos / rope_sin are the
   caller's tables, seq x head_dim/2 floats (session.cpp:188-202; see
   vc4_rope_tables); NULL builds them from the container's theta.  A session
   holds `slots` independent sequences (the reference has one). */
VC4_API int vc4_session_create(vc4_model* m, int slots, int seq, int kv_bits,
                       const float* rope_cos, const float* rope_sin, vc4_session** out);
VC4_API void vc4_session_destroy(vc4_session* s);

/* The rope tables exactly as Session::reset builds them (session.cpp:188-202). */
VC4_API void vc4_rope_tables(float theta, int head_dim, int seq, const float* factors,
                     float* cos_out, float* sin_out);

/* Session::step (session.cpp:1797-1821) for one slot: run `token` at `pos`
   through every layer; when logits is not NULL copy the vocab q16 logits
   (as floats, value/256) to it.  Synchronous. */
VC4_API int vc4_step(vc4_session* s, int slot, int token, int pos, float* logits);
/* Session::step_greedy (session.cpp:1827-1842): same pass, returns the
   first-maximum token (sampling.cpp:160-162). */
VC4_API int vc4_step_greedy(vc4_session* s, int slot, int token, int pos, int* next_token);
/* Batched decode (new for this tier; the reference has no multi-sequence
   API): n sequences, each (slot, token, pos), host arrays.  next_tokens (n)
   and logits (n*vocab floats) may be NULL.  Synchronous. */
VC4_API int vc4_step_batch(vc4_session* s, int n, const int* slots, const int* tokens, const int* pos,
                   int* next_tokens, float* logits);
/* Device-resident form for benchmarking: the three int arrays live on the
   device; the pass is enqueued on the session stream (replayed from a CUDA
   graph) and returns without synchronising.  next_tokens (device, n) receives
   the greedy tokens; when `advance` is nonzero tokens[i] becomes the greedy
   token and pos[i] is incremented, so repeated calls decode autonomously. */
VC4_API int vc4_step_batch_device(vc4_session* s, int n, const int* d_slots, int* d_tokens, int* d_pos,
                          int* d_next_tokens, int advance);
/* The session's CUDA stream (cudaStream_t), for event timing. */
VC4_API void* vc4_session_stream(vc4_session* s);
/* The kernels' self-check word after device-resident passes (GPU::sync,
   gpu.cpp:53, plus the error the reference's shaders cannot report):
   synchronises the session stream; VC4_OK, or the status of the first
   failed check (VC4_ERANGE: an activation left the kernels' range; VC4_ECUDA:
   a launch or copy check).  vc4_step* calls check it themselves. */
VC4_API int vc4_session_check(vc4_session* s);

/* Prefill of a prompt on one slot: positions pos0 .. pos0+n-1 run in order
   (the serial prompt loop, chat.cpp:245-297); the logits of the last position
   are returned when logits is not NULL. */
VC4_API int vc4_prefill(vc4_session* s, int slot, const int* tokens, int n, int pos0, float* logits);
/* Batched prefill (the reference's step_pair / PREFILL_BATCH,
   session.cpp:1598-1795, which it accepts only byte-identical to the serial
   loop): the prompt's positions run as one batch of the many-sequence path,
   up to the session's slot count per pass (the activations are sized by it),
   with each layer's new K/V rows appended before any position attends.  The
   logits of the last position and every K/V row are those of vc4_prefill bit
   for bit.  Chunks below 16 positions, and models or sequence lengths the
   many-sequence kernels do not hold, run through the serial loop. */
VC4_API int vc4_prefill_batch(vc4_session* s, int slot, const int* tokens, int n, int pos0, float* logits);
/* vc4_prefill_batch that keeps every position's logits: logits_all receives
   n x vocab floats, row i the logits position pos0 + i produces (what
   Session::step returns for each scored token of the `--ppl` loop,
   ppl.cpp:50-75).  Positions of a serial tail are stepped one at a time. */
VC4_API int vc4_prefill_logits(vc4_session* s, int slot, const int* tokens, int n, int pos0, float* logits_all);

/* KV rows of one layer in the MMKV1 texel layout (the bytes
   prefix_cache.cpp:59-67 reads with glReadPixels and 176-189 writes with
   glTexSubImage2D): n rows of vc4_kv_row_bytes() each. */
VC4_API int vc4_kv_row_bytes(const vc4_session* s);
VC4_API int vc4_kv_read_rows(vc4_session* s, int slot, int layer, int n, void* host_out);
VC4_API int vc4_kv_write_rows(vc4_session* s, int slot, int layer, int n, const void* host_in);

/* Session::save_prefix_cache / load_prefix_cache (prefix_cache.cpp:25-207):
   the MMKV1 file (version 2) plus its .json sidecar.  load validates the
   header against the model and the KV axis and returns the token list. */
VC4_API int vc4_save_prefix_cache(vc4_session* s, int slot, const char* path, const int* toks, int n,
                          uint64_t system_fnv, uint64_t tools_fnv);
VC4_API int vc4_load_prefix_cache(vc4_session* s, int slot, const char* path, int* toks_out, int cap,
                          int* n_out);
/* load_prefix_cache restored into many slots at once, with the rows held
   once: the MMKV1 file (validated as vc4_load_prefix_cache does) is read into
   the session's shared-prefix rows, and each listed slot reads its positions
   below the prefix length from there instead of from a copy of its own.  A
   slot's own rows, and every result, are as after vc4_load_prefix_cache on
   that slot: vc4_kv_read_rows returns the prefix rows, and a write into the
   prefix (vc4_kv_write_rows, a prefill or a host-array step at such a
   position) first gives the slot its own copy.  A device-array step
   (vc4_step_batch_device) at a position inside a slot's shared prefix does
   not write the row and makes vc4_session_check report VC4_ESTATE.  One
   shared prefix per session: loading another one first gives the slots still
   reading the old one their own copies.  No counterpart in the reference,
   which restores a prefix into its one sequence (prefix_cache.cpp:135-207);
   this is the many-sequence form of that restore. */
VC4_API int vc4_load_prefix_cache_shared(vc4_session* s, const char* path, const int* slots, int count,
                                         int* toks_out, int cap, int* n_out);

/* build_prefix_cache (prefix_build.cpp:22-83, the `--build-prefix-cache
   PROMPTFILE OUT` mode) for a prompt the caller has already tokenised:
   refuses an empty prompt or one longer than the session's sequence length,
   prefills toks[0..n) on `slot` from position 0 with the serial prompt loop,
   then writes the MMKV1 file and its sidecar as vc4_save_prefix_cache does.
   system_fnv / tools_fnv are FNV-1a-64 hashes of the raw system prompt and
   tools text (common.cpp:63-67; 0 when the prompt came from a file). */
VC4_API int vc4_build_prefix_cache(vc4_session* s, int slot, const int* toks, int n, const char* path,
                                   uint64_t system_fnv, uint64_t tools_fnv);

/* GPU::matvec_s (gpu_conv.cpp:271-287), the CPU path's matvec: x (host
   floats, cols) is scaled by 2^k, quantised to q16, multiplied by one model
   matrix and read back as floats.  which: 0 qkv, 1 wo, 2 w1, 3 w3, 4 w2,
   5 router, 6 logits; expert selects an MoE expert. */
VC4_API int vc4_matvec_s(vc4_model* m, int which, int layer, int expert, const float* x, float* out);

/* Replay probe (the reference's MATVEC_DUP / ATTN_DUP, session.cpp:15-48 and
   gpu_attn.cpp:20-39): run one op of the decode pass `reps` times for the
   batch (slots, tokens, pos; host arrays) on the session stream, timing each
   launch with CUDA events.  op: 0 qkv, 1 attention, 2 wo, 3 ffn (gate/up,
   SwiGLU and the w2 partial sums), 5 logits; 4 is refused (w2 runs inside
   op 3).  With flush != 0 a 256 MiB buffer is written and read back between
   launches (outside the timed interval) so every launch starts from a cold
   L2 with no dirty line left to write back.  The KV
   cache and the sequences' state are unchanged afterwards (the FFN partial
   sums the replays accumulate are cleared before returning).  avg_ms receives
   the mean launch time. */
VC4_API int vc4_profile_op(vc4_session* s, int op, int layer, int n, const int* slots, const int* tokens,
                           const int* pos, int reps, int flush, double* avg_ms);
/* Algorithmic bytes one launch of `op` moves for n sequences at the given
   positions (sequence i in slot i): weights (with scale planes) + distinct KV
   rows read (a shared prefix once) and written + activations in and out. */
VC4_API int vc4_op_bytes(const vc4_session* s, int op, int layer, int n, const int* pos, double* bytes);

/* No counterpart in the reference (a measurement helper for the batch-1
   matvec roofline).  Times the matvec_s kernel, the one vc4_matvec_s
   launches, on a synthetic rows x cols matrix of weight type wtype (0 q8,
   1 q4, 2 t3) held in device memory: `reps` launches bracketed by CUDA
   events, each after a 256 MiB write and read that leave L2 cold and clean
   when flush != 0.  path
   selects the kernel: 0 as vc4_matvec_s picks it (by size), 1 one CTA per
   32-row block, 2 the streaming kernel.  ms_avg receives the mean launch
   time, bytes the algorithmic bytes of one launch (weights, q4 scale planes,
   row scales, input and output), digest an FNV-1a hash of the output (equal
   for equal results).  Allocates and frees its own device buffers. */
VC4_API int vc4_matvec_probe(int device, int wtype, int rows, int cols, int path, int reps, int flush,
                             double* ms_avg, double* bytes, unsigned long long* digest);

/* No counterpart in the reference (a test helper for the packed KV codec,
   shaders_attn.cpp:141-159).  Runs the attention kernels' own cache encoder
   on n arbitrary floats on `device` and writes each value's cache bytes to
   out: kv_bits 16 gives two bytes a value (q16 level on the 1/2048 grid,
   big-endian), 8 gives one (q8 level on the 1/16 grid).  Allocates and frees
   its own device buffers; synchronous. */
VC4_API int vc4_kv_codec_probe(int device, int kv_bits, const float* x, int n, void* out);

/* No counterpart in the reference.  vc4_matvec_s for callers that cannot
   allocate device memory: a host whose device memory belongs to its own pool,
   or a thread that must not risk the device synchronisation an allocation can
   cause.  d_x (cols floats) and d_out (rows floats) are the caller's device
   buffers; the scaled input and the integer results live in one static device
   array of at most 16384 columns and 81920 rows, resident on every GPU that
   uses the library until the process exits.  Larger matrices return
   VC4_EINVAL.  Nothing is allocated or freed.  The work is queued on `stream`
   (NULL: the model's stream) and the call returns without waiting.  The first
   call on a device looks up the array's device address (cudaGetSymbolAddress)
   and caches it, so make that first call before any stream capture.  Under
   CUDA's lazy module loading (the default since CUDA 12.2) that first call
   also loads the library's kernels onto the device, which the driver may pay
   for with an allocation and a synchronisation of its own: make it during
   set-up.  The cached address belongs to the device's primary context; after
   cudaDeviceReset it is stale, so do not call this entry point again in that
   process.  Every
   call shares the one array, so calls whose work can overlap on the GPU race:
   keep them on one stream. */
VC4_API int vc4_matvec_s_noalloc(vc4_model* m, int which, int layer, int expert, const float* d_x,
                                 float* d_out, void* stream);

/* ---- The per-op boundary ----------------------------------------------------
   The calls the reference's fused GPU layer loop makes on class GPU
   (Session::forward_gpu_hidden, session.cpp:1459-1584), one C function each.
   GL textures become per-slot device rows of q16 ints named by vc4_buf.  The
   reference's GPU path quantises at its own points; these calls compute what
   vc4_step computes (the CPU path's quantisation points, exact integer dots), so
   a layer loop written call for call against them gives vc4_step's token.  Work
   is queued on the session stream; calls that return host data synchronise. */
typedef enum {
    VC4_BUF_HIDDEN = 0,   /* the residual h (GPU::hidden_a_ / hidden_b_) */
    VC4_BUF_X1 = 1,       /* the residual after attention (hidden_b_ before the FFN) */
    VC4_BUF_XB = 2,       /* rmsnorm before attention (xb_) */
    VC4_BUF_XBF = 3,      /* rmsnorm before the FFN (xbf_) */
    VC4_BUF_XF = 4,       /* rmsnorm before the logits (xf_) */
    VC4_BUF_ATT = 5,      /* attention output (att_out_) */
    VC4_BUF_HA = 6,       /* FFN hidden: the whole row, or its first chunk (ffn_h_a_) */
    VC4_BUF_HB = 7,       /* FFN hidden: the second chunk (ffn_h_b_) */
    VC4_BUF_TMP = 8       /* the residual between the two w2 halves (hidden_a_) */
} vc4_buf;

/* Session::embedding (session.cpp:342-371) of `token` into buffer dst. */
VC4_API int vc4_embedding(vc4_session* s, int slot, int token, int dst);
/* GPU::upload_hidden (gpu.h:169): host floats (dim), quantised to q16 (lrintf). */
VC4_API int vc4_upload_hidden(vc4_session* s, int slot, const float* x, int dst);
/* GPU::rmsnorm (gpu.h:173): dst = rmsnorm(src) with the model's weights
   (weights 0: attention of `layer`, 1: FFN of `layer`, 2: final). */
VC4_API int vc4_rmsnorm(vc4_session* s, int slot, int src, int weights, int layer, int dst);
/* GPU::attention_block (gpu.h:142): qkv = matvec_s(qkv[layer], src), QK-norm,
   RoPE at `pos`, the packed KV row appended to the slot's cache, attention over
   positions 0..pos; the q16 attention output goes to dst. */
VC4_API int vc4_attention_block(vc4_session* s, int slot, int layer, int pos, int src, int dst);
/* GPU::matvec_add (gpu.h:175): dst = residual + the matrix times src.  which 1:
   wo (matvec_s, add_q16).  which 4 / 7: w2 / its second half.  For a chunked FFN
   the first half (4) goes to VC4_BUF_TMP and the second (7) takes VC4_BUF_TMP as
   its residual: dst = add_q16(x1, add_q16(w2a out, w2b out)), the CPU path's
   order (session.cpp:519-551).  The w2 input is read as matvec_s reads it in
   the host FFN of a two-chunk dense model, as is otherwise. */
VC4_API int vc4_matvec_add(vc4_session* s, int slot, int which, int layer, int expert, int src, int residual,
                           int dst);
/* GPU::matvec_from (gpu.h:84): the matrix times src read back as floats (rows).
   which 0 qkv, 1 wo, 5 router.  input_scale 1 reads src as matvec_s does
   (gpu_conv.cpp:271-287; the CPU path's router call, session.cpp:484), 0 as
   uploaded. */
VC4_API int vc4_matvec_from(vc4_session* s, int slot, int which, int layer, int expert, int src, int input_scale,
                            float* out);
/* GPU::ffn_split / ffn_split_chunked (gpu.h:89,107-108): the FFN hidden row of
   src for `layer` (and `expert`) into dst_a, and for a chunked FFN its second
   chunk into dst_b.  A two-chunk dense model uses the CPU path's host FFN
   (matvec_s gate/up, quantize_act); MoE and one-chunk FFNs the GPU FFN kernels'
   rounding. */
VC4_API int vc4_ffn_split(vc4_session* s, int slot, int layer, int expert, int src, int dst_a, int dst_b);
/* GPU::logits_from (gpu.h:256): the vocab logits (q16 grid, as floats) of src. */
VC4_API int vc4_logits_from(vc4_session* s, int slot, int src, float* logits);
/* GPU::logits_argmax_from (gpu.h:263-264): the first-maximum token of src. */
VC4_API int vc4_logits_argmax_from(vc4_session* s, int slot, int src, int* token);
/* GPU::read_bytes (gpu.h:270) of a buffer, as floats (n values, q16 / 256). */
VC4_API int vc4_read_buffer(vc4_session* s, int slot, int buf, int n, float* out);

/* draws()/syncs() (gpu.h:44-48): kernels launched and host syncs so far. */
VC4_API int vc4_counters(const vc4_session* s, long long* launches, long long* syncs);
/* Kernels one decode pass of n sequences launches. */
VC4_API int vc4_launches_per_step(const vc4_session* s, int n);

#ifdef __cplusplus
}
#endif
#endif
