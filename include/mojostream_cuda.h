/*
 * mojostream_cuda.h -- C-ABI of libmojostream_cuda.so, the B200 (sm_100a)
 * implementation of MojoStream's Gemma-4 token loop.
 *
 * A host written in Mojo binds these symbols with DLHandle / external_call,
 * the mechanism the reference already uses for libc (pread,
 * src/streaming/stream_runner.mojo:222-224).  Plain pointers and sizes only;
 * no CUDA, torch or C++ types cross the boundary.  Streams are passed as
 * `void*` (a cudaStream_t, or NULL for the context's own stream).
 *
 * Conventions
 *   - Every call returns ms_status (0 = MS_OK); ms_last_error() gives the
 *     message of the last failure on a context.  No exceptions cross the ABI.
 *   - Shapes, capacities and pointer alignment are validated on the host
 *     before anything is launched (the reference's kernels check nothing:
 *     a wrong packed_cols ran out of bounds, README.md:547-563).
 *   - A context owns all device memory it allocates.  Host buffers passed in
 *     are borrowed for the duration of the call only.
 *   - One context per host thread (thread-compatible, not thread-safe).
 *     Calls are asynchronous on the given stream unless stated otherwise;
 *     ms_sync() waits.  A context's split-K and attention partial sums are
 *     one buffer shared by all its calls and models: calls given different
 *     streams must not overlap in time (run them on one stream, or give each
 *     concurrent stream its own context).
 *   - Activations are fp32 row-major, Q4 weights are the reference's layout
 *     [K][N/2] (low nibble = even column, value (nibble - 8) * scale,
 *     src/linalg/kernels.mojo:64-70), fp32 lm_head is [D][V].
 */
#ifndef MOJOSTREAM_CUDA_H
#define MOJOSTREAM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MS_ABI_VERSION 1

#if defined(__GNUC__)
#define MS_API __attribute__((visibility("default")))
#else
#define MS_API
#endif

typedef enum {
  MS_OK = 0,
  MS_ERR_INVALID_ARG = 1,  /* null pointer, bad enum, bad layer index            */
  MS_ERR_SHAPE = 2,        /* unsupported or inconsistent dimensions             */
  MS_ERR_ALIGN = 3,        /* device pointer not aligned as required             */
  MS_ERR_CAPACITY = 4,     /* position beyond the KV cache, too many rows        */
  MS_ERR_CUDA = 5,         /* a CUDA runtime call failed                         */
  MS_ERR_NCCL = 6,         /* a collective failed                                */
  MS_ERR_OOM = 7,          /* device allocation failed                           */
  MS_ERR_STATE = 8,        /* objects from different contexts / wrong order      */
  MS_ERR_TIMEOUT = 9,      /* a bounded wait ran out                             */
  MS_ERR_UNSUPPORTED = 10  /* feature not built in this library                  */
} ms_status;

typedef struct ms_ctx ms_ctx;
typedef struct ms_model ms_model;
typedef struct ms_kv ms_kv;
typedef struct ms_q4_weight ms_q4_weight;

/* ---------------------------------------------------------------- context */

/* MS_ABI_VERSION of the built library: a binding compares it with the
 * header it was written against.  No counterpart in the reference. */
MS_API int ms_abi_version(void);
/* A short description of a status code ("capacity exceeded", ...); static
 * storage. */
MS_API const char *ms_status_string(ms_status s);

/* Bind to CUDA device `device` and create a context with its own stream. */
MS_API ms_status ms_init(int device, ms_ctx **out);
MS_API ms_status ms_destroy(ms_ctx *ctx);
/* The message of the context's last failed call; the text stays valid until
 * a later call on the context fails. */
MS_API const char *ms_last_error(const ms_ctx *ctx);
/* Wait for all work on `stream` (NULL = the context stream). */
MS_API ms_status ms_sync(ms_ctx *ctx, void *stream);

/* Device memory for hosts without CUDA headers.  kind: 0 host->device,
 * 1 device->host, 2 device->device.  ms_memcpy is stream-ordered. */
MS_API ms_status ms_malloc(ms_ctx *ctx, size_t bytes, void **dptr);
MS_API ms_status ms_free(ms_ctx *ctx, void *dptr);
MS_API ms_status ms_memcpy(ms_ctx *ctx, void *dst, const void *src, size_t bytes, int kind,
                    void *stream);

/* ------------------------------------------------- single Q4 projection */

/* Replaces matmul_q4_bpack_raw(C, A, bq_ptr, packed_cols, scale, workers)
 * (src/linalg/kernels.mojo:201-208).  The weight is repacked once into the
 * tensor-core tile layout; N is passed explicitly instead of packed_cols so a
 * wrong column count is rejected (MS_ERR_SHAPE) rather than read out of
 * bounds.  w_rx may be a host or a device pointer.  K % 64 == 0, N % 16 == 0. */
MS_API ms_status ms_q4_weight_create(ms_ctx *ctx, const uint8_t *w_rx, int K, int N, float scale,
                              ms_q4_weight **out);
MS_API ms_status ms_q4_weight_destroy(ms_ctx *ctx, ms_q4_weight *w);
/* C[M,N] = A[M,K] . deq(W)   (accumulate = 0)
 * C[M,N] += A[M,K] . deq(W)  (accumulate = 1, the reference's semantics,
 * matmul_q4_bpack_raw, src/linalg/kernels.mojo:201-267)
 * A, C: device pointers, row-major, A 16-byte and C 8-byte aligned.
 * MS_ERR_CAPACITY (before launch) when a decode call (M <= 8) would need a
 * k-split whose partial sums exceed the context's 32 MiB scratch: only for
 * very wide and long weights (N 262144 with K above 5120 at M 8, above
 * 20480 at M 4). */
MS_API ms_status ms_q4_gemm(ms_ctx *ctx, const ms_q4_weight *w, float *C, const float *A, int M,
                     int accumulate, void *stream);
/* No counterpart in the reference.  The same projection as ms_q4_gemm
 * (results within 2e-5 relative RMSE of it: rows above 8 run on the CUDA-core
 * tiled kernel, not the tensor-core GEMM) for callers that cannot have a call
 * allocate device memory or use the context's scratch (for example a host
 * that reserved all of HBM for its KV pages, or a path where an implicitly
 * synchronising allocation is not allowed).  It allocates nothing: its
 * scratch is one fixed device array of 1 MiB + 16 KiB inside the library
 * (split-K partial sums and arrival tickets).
 *   - Limit: the partial sums and tickets of the k-split must fit (262144
 *     floats, 4096 tickets); the call lowers the k-split until they do, down
 *     to the kernel's smallest split (unsplit for rows above 8), and returns
 *     MS_ERR_CAPACITY with both sizes in the message only if that does not
 *     fit.  Only decode rows (M 5..8) of wide or long projections reach the
 *     limit (e.g. M = 8, K = 13824, N = 5120); every projection of the E4B
 *     and 14B-class models fits at M <= 4.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, which may load the module): make that first
 *     call before any stream capture.  First calls from several host
 *     threads at once are safe.
 *   - The arrival tickets must be zero at launch; the call clears the ones
 *     it uses on `stream` before its kernel.
 *   - The scratch is shared by every call on the device: calls that overlap
 *     in time (other streams, other threads, other contexts) race; order
 *     them on one stream.
 *   - Kernel timeouts set the context's error word (reported by ms_sync). */
MS_API ms_status ms_q4_gemm_noalloc(ms_ctx *ctx, const ms_q4_weight *w, float *C, const float *A,
                             int M, int accumulate, void *stream);

/* ----------------------------------------------------------------- model */

/* One decoder layer (E4BLayerRef, src/inference/gemma4_e4b.mojo:125-174;
 * Gemma4LayerWeights, src/main.mojo:305-337).  window = 0 attends to every
 * cached position (the demo layers and E4B's full-attention layers); window > 0
 * is a sliding window over a circular cache.  RoPE rotates the leading
 * rotary_dims of each head, pairs (i, i + rotary_dims / 2), with base
 * rope_theta (src/linalg/kernels.mojo:553-595).  Matrices in the order
 * Q, K, V, O, Gate, Up, Down; host or device pointers, reference layout. */
typedef struct {
  int head_dim;
  int n_heads;
  int n_kv_heads;
  int window;
  int rotary_dims;
  int ffn_dim;
  float rope_theta;
  float ple;
  const uint8_t *w[7];
  float scale[7];
} ms_layer_desc;

typedef struct {
  int hidden;
  int n_layers;
  const ms_layer_desc *layers;
  int vocab;                /* 0 = no lm_head / embedding                    */
  const float *lm_head;     /* [hidden][vocab] fp32, host or device, or NULL */
  const float *final_gamma; /* [hidden] final RMSNorm gain, or NULL (= 1)    */
  int max_rows;             /* largest M of any forward call                 */
} ms_model_desc;

/* Copies and repacks all weights to the device (the caller's buffers may be
 * freed afterwards). */
MS_API ms_status ms_model_create(ms_ctx *ctx, const ms_model_desc *desc, ms_model **out);
MS_API ms_status ms_model_destroy(ms_ctx *ctx, ms_model *model);
/* Device bytes held for weights (Q4 tiles + lm_head). */
MS_API size_t ms_model_weight_bytes(const ms_model *model);

/* ------------------------------------------------------ .mojostream files */

/* Header of a .mojostream file (src/streaming/mojostream.mojo:95-160; written
 * by scripts/create_fake_model.py:194-281, format 1, and scripts/convert.py:
 * 359-414, format 2 with the Engram extension in header bytes 64-127). */
typedef struct {
  int format_tag;        /* 1: uniform demo stack, 2: layer-typed (sliding / full) */
  int n_layers, hidden, kv_dim, ffn_dim, n_heads, n_kv_heads;
  uint64_t n_tensors, data_start, data_end, file_size;
  /* format 2 (Engram extension; 0 when absent) */
  int kv_shared_layers, sliding_kv_dim, full_kv_dim, ple_dim, sliding_window;
} ms_file_info;

/* Open a .mojostream file, read its header and tensor directory and run the
 * reference's ShapeGuard and TensorGuard (src/streaming/stream_runner.mojo:
 * 288-400): head / KV-head divisibility, n_tensors = 8 n_layers, per entry the
 * (layer, type) sequence, its dims, scale > 0, 4096-aligned offset, inside the
 * file.  Format 2 accepts layer-typed dims (Q / K / V / O of a layer follow
 * its head_dim, one of sliding_kv_dim / n_kv and full_kv_dim / n_kv), which
 * the reference's StreamingRunner guard rejects for Gemma-4-E4B.  info may be
 * NULL.  On failure err (may be NULL) receives the message; MS_ERR_SHAPE for a
 * failed guard, MS_ERR_INVALID_ARG for an unreadable file.  No device use. */
MS_API ms_status ms_file_check(const char *path, ms_file_info *info, char *err, size_t err_bytes);

/* What the file does not say, per attention kind.  Zero fields take the
 * defaults in brackets. */
typedef struct {
  int full_every;         /* full attention iff (layer + 1) % full_every == 0
                             [format 1: every layer; format 2: 6, E4B's
                             rule, src/inference/gemma4_e4b.mojo:60-63]    */
  int window;             /* sliding window [the file's sliding_window]   */
  float slide_theta;      /* [1e4]                                          */
  float full_theta;       /* [1e6; format 1: slide_theta]                   */
  int full_rotary;        /* rotary dims of full layers [128, capped at
                             head_dim; format 1: head_dim]; sliding layers
                             rotate the whole head                          */
  int max_rows;           /* as ms_model_desc.max_rows [64]                 */
  size_t staging_bytes;   /* pinned host staging per reader thread [32 MiB] */
} ms_load_opts;

/* A model from a .mojostream file (and optionally an lm_head_proto.bin,
 * load_lm_head, src/inference/lm_head.mojo:61-116: v2 = fp32 weights, final
 * gamma and BOS embedding; v1 = Q4 weights, expanded to fp32 on the device,
 * gamma 1).  The file is checked as ms_file_check does, then its tensor data
 * streams to the device through pinned host buffers, one per reader thread
 * (up to 8 preads in parallel, each overlapping the others' cudaMemcpyAsync:
 * the reference's double buffer of sparse_pin.mojo:136-330, widened and aimed
 * at HBM) and is repacked as ms_model_create does.  With an lm_head file, token id 2 (BOS) embeds as the file's BOS
 * vector (apply_bos_embedding, lm_head.mojo:133-143).  Tensor parallel: each
 * rank loads the file and keeps its slices.  opts may be NULL. */
MS_API ms_status ms_model_load(ms_ctx *ctx, const char *path, const char *lm_head_path,
                               const ms_load_opts *opts, ms_model **out);
/* Seconds and bytes of the last ms_model_load on this context (file reads +
 * host-to-device copies, before the repack). */
MS_API ms_status ms_load_stats(const ms_ctx *ctx, double *seconds, uint64_t *bytes);

/* -------------------------------------------------------------- KV cache */

/* Paged KV cache for n_seq sequences (KVCache, src/main.mojo:257-301;
 * HybridKVCache, src/inference/gemma4_e4b.mojo:83-116).  Full-attention
 * layers hold max_pos positions; sliding layers hold slide_cap slots
 * (0 = the window, as in the reference; a prefill chunk of L tokens needs
 * slide_cap >= window + L - 1).  A cache refers to its model: destroy it
 * before the model (ms_kv_destroy alone may follow the model's destroy).
 * Calls that pair a cache with a model other than the one it was made for,
 * a later model at a freed one's address included, fail with MS_ERR_STATE. */
MS_API ms_status ms_kv_create(ms_ctx *ctx, const ms_model *model, int n_seq, int max_pos,
                       int slide_cap, ms_kv **out);
/* Element type of the cached K / V values. */
enum { MS_KV_F32 = 0, MS_KV_BF16 = 1, MS_KV_I8 = 2 };
/* ms_kv_create with an element type: MS_KV_F32 (the parity mode: the
 * reference's fp32 cache), MS_KV_BF16 (half the cache bytes; K / V rounded
 * to nearest bfloat16 when written, widened to fp32 when read; needs every
 * kv_dim % 8 == 0) or MS_KV_I8 (about a quarter of the bytes, the int8 KV
 * cache of the reference's roadmap, README.md:487-489: each K or V head row
 * of a position is stored as int8 q with one fp32 scale = max|v| / 127,
 * q = rint(v * 127 / max|v|); a value reads back as q * scale; a row whose
 * max|v| is below 2^-120 is stored as zeros; needs every head_dim % 16 ==
 * 0).  Attention, softmax and accumulation stay fp32. */
MS_API ms_status ms_kv_create_typed(ms_ctx *ctx, const ms_model *model, int n_seq, int max_pos,
                                    int slide_cap, int dtype, ms_kv **out);
/* A cache for serving requests that come and go (the reference's roadmap:
 * paged KV allocator / continuous batching, README.md:487-489).  The
 * full-attention layers draw 16-position pages from one pool of pool_pages
 * pages (a page id indexes every full layer's pool) instead of holding
 * max_pos positions for each of the n_seq sequence slots: a page is given to
 * a slot the first time a call writes (or a decode loop will reach) one of
 * its positions, together with every page below it, so short and long
 * sequences share the pool in proportion to their lengths.  Sliding layers
 * keep a ring of slide_cap slots per slot (they never grow past it).
 * MS_ERR_CAPACITY when the pool runs out, before any launch; the refused
 * call then holds no pages (every page it took is given back; ms_prefill:
 * its chunks of max_rows rows that ran keep theirs).  Every other call works
 * on it as on an ms_kv_create cache. */
MS_API ms_status ms_kv_create_pooled(ms_ctx *ctx, const ms_model *model, int n_seq, int max_pos,
                                     int slide_cap, int dtype, int pool_pages, ms_kv **out);
/* Slot `seq` is free for a new request: its pages go back to the pool (pages
 * it shares stay with the other holders) and its token history is cleared.
 * Any cache; stream-ordered on the context stream. */
MS_API ms_status ms_kv_release(ms_ctx *ctx, ms_kv *kv, int seq);
/* Slot dst starts as a copy of the first n_pos positions of slot src (a
 * prompt prefix computed once and reused): on a pooled cache dst's table
 * points at src's whole pages below n_pos (shared, reference-counted; a
 * later write into a shared page gets a private copy first) and the page the
 * prefix ends in is copied; the sliding rings and the token history are
 * copied.  dst must hold no pages (a new or released slot).  Continue dst at
 * position n_pos. */
MS_API ms_status ms_kv_share_prefix(ms_ctx *ctx, ms_kv *kv, int src_seq, int dst_seq, int n_pos);
/* Full-attention pages in use and in total (pooled: the pool; otherwise
 * n_seq x ceil(max_pos / 16), all of them in use). */
MS_API ms_status ms_kv_pages(const ms_kv *kv, int *used, int *total);
/* allow != 0: calls may hold rows of one sequence whose sliding-window slots
 * overlap slots that other rows of the same call still attend.  By default
 * such a call is rejected (MS_ERR_CAPACITY) before any kernel runs.  With it
 * allowed, the call behaves as the reference's E4B runner: every row's K / V
 * is written (slot p % slide_cap) before any row attends, so a row reads
 * whatever the call left in its window's slots.  That is the runner's
 * padding quirk: row 0 plus three zero rows at positions p+1..p+3
 * (src/inference/lm_head.mojo:133-143, gemma4_e4b_infer.mojo:45-54), whose
 * K / V overwrite slots 512 positions back once p >= 511
 * (write_kv_sliding, src/inference/gemma4_e4b.mojo:211-228).  Reproducing it
 * exactly needs slide_cap equal to the window (slide_cap 0 at ms_kv_create). */
MS_API ms_status ms_kv_allow_window_overwrite(ms_ctx *ctx, ms_kv *kv, int allow);
MS_API ms_status ms_kv_destroy(ms_ctx *ctx, ms_kv *kv);
/* K / V rows of positions pos0 .. pos0 + n - 1 of sequence seq in layer
 * `layer`, to or from dense fp32 device buffers k, v [n][kv_dim] (the
 * layer's n_kv_heads * head_dim).  write_kv_sliding / write_kv_full
 * (src/inference/gemma4_e4b.mojo:211-249) for n rows at once: full layers
 * hold position p at row p; sliding layers at slot p % slide_cap, so n <=
 * slide_cap, and a read of position p returns what the last write of a
 * position congruent to p mod slide_cap left there.  A bf16 cache rounds on
 * write as the forward pass does.  For importing or exporting a sequence's
 * cache (a shared prompt prefix copied into another slot, a sequence moved
 * between contexts); the token history is not touched.  Asynchronous on
 * `stream`; MS_ERR_CAPACITY for positions outside the cache. */
MS_API ms_status ms_kv_write(ms_ctx *ctx, ms_kv *kv, int layer, int seq, int pos0, int n,
                             const float *k, const float *v, void *stream);
MS_API ms_status ms_kv_read(ms_ctx *ctx, const ms_kv *kv, int layer, int seq, int pos0, int n,
                            float *k, float *v, void *stream);
/* Every slot empty again, as KVCache.reset (src/main.mojo:295-297) sets
 * cur_len to 0: K / V zeroed, token histories cleared, a pooled cache's
 * pages all free.  Stream-ordered on the context stream. */
MS_API ms_status ms_kv_reset(ms_ctx *ctx, ms_kv *kv);
/* Device bytes the cache holds (K / V pools of every layer). */
MS_API size_t ms_kv_bytes(const ms_kv *kv);

/* ---------------------------------------------------------------- forward */

/* Rows: row r of x belongs to sequence seq_ids[r] at absolute position pos[r]
 * (host arrays of M ints).  The reference's demo batch (B consecutive
 * positions of one sequence, src/main.mojo:584-592) is seq_ids = {0,0,0,0},
 * pos = {p, p+1, p+2, p+3}; independent sequences are seq_ids = {0,1,2,3}.
 * x is a device pointer [M][hidden], updated in place. */

/* gemma4_forward_layer (src/main.mojo:538-613) / e4b_forward_layer
 * (src/inference/gemma4_e4b.mojo:459-540) for one layer. */
MS_API ms_status ms_layer_forward(ms_ctx *ctx, const ms_model *model, int layer, float *x, ms_kv *kv,
                           const int *seq_ids, const int *pos, int M, void *stream);
/* All layers in order. */
MS_API ms_status ms_forward(ms_ctx *ctx, const ms_model *model, float *x, ms_kv *kv,
                     const int *seq_ids, const int *pos, int M, void *stream);
/* get_token_embedding (src/inference/lm_head.mojo:171-195): x[r] = column
 * ids[r] of the lm_head table.  ids: host array. */
MS_API ms_status ms_embed(ms_ctx *ctx, const ms_model *model, const int *ids, int M, float *x,
                   void *stream);
/* apply_final_norm + project_lm_head + greedy temperature_sampling
 * (src/inference/lm_head.mojo:119-168, 224-230).  x [M][hidden] device (not
 * modified); logits [M][vocab] device or NULL; argmax_out [M] device or NULL. */
MS_API ms_status ms_lm_head(ms_ctx *ctx, const ms_model *model, const float *x, int M, float *logits,
                     int *argmax_out, void *stream);

/* One greedy decode step with host buffers: embed ids, all layers, lm_head,
 * argmax -> next_ids (host).  Synchronous.  (The token loop of
 * gemma4_e4b_infer.mojo:163-186, one step.) */
MS_API ms_status ms_decode_step(ms_ctx *ctx, const ms_model *model, ms_kv *kv, const int *ids,
                         const int *seq_ids, const int *pos, int M, int *next_ids);

/* `steps` greedy decode steps entirely on the device, each a replay of the
 * captured decode-step graph followed by the on-device feedback (next ids
 * become inputs, positions advance): ids (host, M) are the first inputs, pos
 * (host, M) their positions; token t of step s is written to
 * out_ids[s * M + t] (host).  device_ms (nullable) receives the device time of
 * the replays (CUDA events on the context stream).  Synchronous. */
MS_API ms_status ms_generate(ms_ctx *ctx, const ms_model *model, ms_kv *kv, const int *ids,
                             const int *seq_ids, const int *pos, int M, int steps, int *out_ids,
                             float *device_ms);

/* The context's CUDA stream (a cudaStream_t), for callers that order their
 * own work or timing events with the library's. */
MS_API void *ms_ctx_stream(ms_ctx *ctx);

/* ---------------------------------------------------------------- sampling */

/* temperature_sampling (src/inference/lm_head.mojo:198-254) on M rows at once.
 * logits [M][V] fp32 device (read only: the reference rewrites its row in
 * place).  Row r's "generated" list is hist[hist_off[r] .. hist_off[r+1])
 * (device int arrays, hist_off with M + 1 entries; both NULL = empty).
 * penalty > 1: every occurrence of an id in the list divides its logit if
 * positive, multiplies it otherwise.  temperature <= 0.01: the first maximum.
 * Otherwise softmax(logits / temperature) and the first id whose running sum
 * reaches target = ((seed * 6364136223846793005 + 1442695040888963407) &
 * 0x7FFFFFFF) / 2^31 with seed = seeds[r] (device uint64 array; the reference
 * draws it from perf_counter_ns).  Where rounding leaves the running sum
 * short of the target, the last id with a nonzero weight (the reference
 * returns V - 1).  out_ids [M] device.  M <= 65535, V <= 8388608.
 * Asynchronous. */
MS_API ms_status ms_sample(ms_ctx *ctx, const float *logits, int M, int V, const int *hist,
                           const int *hist_off, float temperature, float penalty,
                           const uint64_t *seeds, int *out_ids, void *stream);

/* Sampling of the token loop (ms_decode_step, ms_generate and ms_prefill's
 * first ids; the reference's loop calls temperature_sampling with T = 0.7,
 * penalty 1.2, gemma4_e4b_infer.mojo:38-39, 139, 179).  Default: temperature
 * 0, penalty 1 (the plain greedy argmax).  A row's "generated" list is every
 * token the cache has been fed for its sequence up to and including the row's
 * position (prompt + generated ids; ms_kv_reset clears it), its seed
 * splitmix64(seed ^ (seq << 32 | pos)), so a generation repeats for a seed.
 * Under tensor parallelism every rank makes the same call. */
MS_API ms_status ms_set_sampling(ms_ctx *ctx, const ms_model *model, float temperature,
                                 float penalty, uint64_t seed);

/* ------------------------------------------------------ tensor parallelism */

/* No counterpart in the reference (which runs one CPU process): the larger
 * configurations split every layer's heads and FFN columns over W GPUs of one
 * node, one process (and one ms_ctx) per GPU.  Rank 0 creates an id
 * (ms_tp_unique_id, ms_tp_unique_id_bytes() bytes) and the host hands it to
 * every rank by its own means; each rank then calls ms_tp_init before
 * ms_model_create.  ms_model_create takes the FULL reference-layout weights
 * on every rank and keeps this rank's slices: Q/K/V and gate/up columns of
 * its heads / FFN columns, O and down rows, lm_head vocabulary columns
 * [rank V/W, (rank+1) V/W).  Per layer one all-reduce (NCCL) follows O and one
 * follows down; the embedding and the greedy argmax are combined over ranks,
 * so ms_embed / ms_decode_step / ms_generate / ms_prefill return the same
 * ids on every rank.  ms_lm_head's logits hold this rank's vocabulary slice
 * only.  Every rank must make the same calls in the same order.
 * Shapes: n_heads, n_kv_heads divisible by W, ffn_dim by 64 W, the local
 * q width by 64, vocab by 4 W (else MS_ERR_SHAPE).  W = 1: no-op. */
MS_API size_t ms_tp_unique_id_bytes(void);
MS_API ms_status ms_tp_unique_id(void *id_out, size_t bytes);
MS_API ms_status ms_tp_init(ms_ctx *ctx, int world, int rank, const void *unique_id);
/* Ranks of the context's tensor-parallel group (1 before / without ms_tp_init). */
MS_API int ms_tp_world(const ms_ctx *ctx);

/* Prefill (the TTFT pass): n_tokens rows (host arrays ids / seq_ids / pos,
 * any mix of sequences) run through all layers in chunks of at most max_rows
 * rows, writing the KV cache.  If first_ids is not NULL, the row with the
 * highest position of every sequence present goes through the lm_head and
 * its greedy token is written to first_ids[seq_id] (host, n_seq entries).
 * Synchronous. */
MS_API ms_status ms_prefill(ms_ctx *ctx, const ms_model *model, ms_kv *kv, const int *ids,
                     const int *seq_ids, const int *pos, int n_tokens, int *first_ids);

#ifdef __cplusplus
}
#endif
#endif /* MOJOSTREAM_CUDA_H */
