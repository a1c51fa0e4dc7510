// ms_kernels.h -- parameter blocks and launchers of the sm_100a kernels.
// Internal to libmojostream_cuda.so (the public C-ABI is include/mojostream_cuda.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ms {

// ------------------------------------------------------------------------
// Tiled Q4 weight layout ("fragment tiles").
//
// A matrix W[K][N] (reference layout: bytes [K][N/2], low nibble = even
// column) is cut into 16-column tiles, tiles into groups of 8, and stored as
//   [group][K/64 k-chunk][8 tiles of the group][32 lanes] x uint4,
// so one k-chunk of a whole group is 4 KB of contiguous memory (one bulk-copy
// piece that 8 warps consume together).  Tiles past N (group padding) hold
// nibble 8 (value 0).  Word s (0..3) of lane (g = lane/4, t = lane%4) in chunk
// c of tile j holds the eight nibbles that lane needs as the A operand
// (W^T, 16 x 16) of one mma.m16n8k16 for k-subtile 4c+s:
//   bits  0- 3 / 16-19 : rows g   , k 2t   / 2t+1
//   bits  4- 7 / 20-23 : rows g+8 , k 2t   / 2t+1
//   bits  8-11 / 24-27 : rows g   , k 2t+8 / 2t+9
//   bits 12-15 / 28-31 : rows g+8 , k 2t+8 / 2t+9
// Tile row r maps to a logical output column through a permutation chosen
// at repack time, so that the two rows a thread owns (g, g+8) are the pair an
// epilogue needs: RoPE partners (i, i + R/2), or gate/up of the same column.
// ------------------------------------------------------------------------
constexpr int kTileN = 16;
constexpr int kChunkK = 64;
constexpr int kGroupTiles = 8;
// uint4 offset of (tile, chunk) for lane 0
__host__ __device__ inline size_t tile_chunk_u4(int tile, int chunk, int nchunks) {
  return (((size_t)(tile / kGroupTiles) * nchunks + chunk) * kGroupTiles + tile % kGroupTiles) * 32;
}
__host__ __device__ inline int padded_tiles(int n_tiles) {
  return (n_tiles + kGroupTiles - 1) / kGroupTiles * kGroupTiles;
}

// Epilogues of the projection kernel.
enum Epilogue : int {
  kEpiStore = 0,   // out = s * acc
  kEpiAccum = 1,   // out += s * acc
  kEpiResid = 2,   // out = ple * resid * inv_rms(resid) + s * acc ; + row stats
  kEpiSwiGLU = 3,  // rows 0-7 gate, rows 8-15 up: h = up * g * sigmoid(g)
  kEpiQKV = 4,     // RoPE (rows g / g+8 partners) then Q store / K,V cache write
};

// Tile descriptor of a fused Q|K|V matrix: dst 0=Q 1=K 2=V, logical column of
// tile rows 0..7 (col_lo + g) and 8..15 (col_hi + g), RoPE frequency index of
// row 0 (or -1).
struct QkvTile {
  int dst, col_lo, col_hi, rope_i0;
};

struct KvView {
  float* k;                  // layer pool [n_pages][page][kv_dim]
  float* v;
  const int* block_table;    // [n_seq][bt_stride] physical page ids
  int bt_stride, page, cap, circular, kv_dim;
  int off32;                 // every row offset of the pool fits 32 bits
  int bf16;                  // K / V stored as bfloat16 (k, v then point at bf16 pools)
  // int8 cache: a position's row is kv_dim int8 values, then one fp32 scale
  // per KV head (hd values each), padded to row_bytes (a 16-byte multiple);
  // value = int8 * scale.  The projections write fp32 rows [M][kv_dim] to
  // stage_k / stage_v, and launch_kv_quant moves them into the cache.
  int i8, row_bytes, hd;
  float* stage_k;
  float* stage_v;
};

// Row index (page * page_size + slot within the page) of absolute position p
// of sequence seq in a layer's pool.
__device__ __forceinline__ size_t kv_row_index(const KvView& kv, int seq, int p) {
  const int slot = kv.circular ? (p % kv.cap) : p;
  const int phys = kv.block_table[seq * kv.bt_stride + slot / kv.page];
  return (size_t)phys * (size_t)kv.page + (size_t)(slot % kv.page);
}

// Where a projection writes the K (dst 1) or V (dst 2) values of its row m
// (sequence seq, position pos): element `off` of the returned fp32 / bf16
// pool, or for an int8 cache row m of the fp32 staging rows.
__device__ __forceinline__ float* kv_dst(const KvView& kv, int dst, int m, int seq, int pos,
                                         size_t& off, int& bf) {
  if (kv.i8) {
    off = (size_t)m * kv.kv_dim;
    bf = 0;
    return dst == 1 ? kv.stage_k : kv.stage_v;
  }
  off = kv_row_index(kv, seq, pos) * (size_t)kv.kv_dim;
  bf = kv.bf16;
  return dst == 1 ? kv.k : kv.v;
}

// int8 cache quantisation of one head row with absolute maximum amax:
// scale = amax / 127, q = rint(v * (127 / amax)) clamped to [-127, 127]
// (every step one IEEE-rounded operation, so a CPU restatement reproduces
// it bit for bit).  A row whose amax is below 2^-120 (zero rows included;
// 127 / amax would overflow below about 2^-121) is stored as scale 0, q 0.
constexpr float kI8MinAmax = 0x1p-120f;
__device__ __forceinline__ void i8_scale(float amax, float& scale, float& inv) {
  const bool live = amax >= kI8MinAmax;
  scale = live ? __fdiv_rn(amax, 127.0f) : 0.f;
  inv = live ? __fdiv_rn(127.0f, amax) : 0.f;
}
__device__ __forceinline__ int i8_quant(float v, float inv) {
  const float r = rintf(__fmul_rn(v, inv));
  return (int)fminf(fmaxf(r, -127.f), 127.f);
}

struct GemvParams {
  const uint4* w;    // fragment tiles
  int n_tiles, K, kseg, ksplit, M;  // kseg: k per CTA (multiple of 64), ksplit = ceil(K / kseg)
  // input rows x[M][K] (row stride ldx); optional RMSNorm in the prologue
  const float* x;
  int ldx;
  const float* in_stats;  // [in_nstat][M] partial sums of squares, or null
  int in_nstat;
  float in_ple;           // x is multiplied by ple before the norm
  int in_D;
  // epilogue
  int epi;
  float* out;
  int ldo;
  float scale, scale2;
  const float* resid;
  int ldr;
  const float* resid_stats;
  int resid_nstat;
  float resid_ple;
  float* out_stats;       // [n_tiles][M]
  // QKV epilogue
  const QkvTile* tiles;
  float sq, sk, sv;
  float* q_out;
  int ldq;
  const float* inv_freq;  // per RoPE frequency index
  const int* pos;
  const int* seq;
  KvView kv;
  // split-K scratch
  float* part;            // partial sums of k-segments
  int* counters;          // arrival tickets (reset by the last arrival)
  // decode kernel: the ksplit CTAs of a tile group run as one thread-block
  // cluster and sum their partials through distributed shared memory (part /
  // counters unused); set by the launcher
  int cluster;
  int* err;               // error bits for the host (bounded waits)
  // tensor-core path: activation limbs and per-row factors (quant_rows_kernel)
  uint8_t* lq;
  float2* rowf;
  // tensor parallel (tensor-core path): the finished output tile is summed
  // over the ranks inside the epilogue.  peer_tiles[r] / peer_flags[r]: rank
  // r's tile buffer ([tile][128 x 128] floats) and per-tile use counters, as
  // mapped in this process (CUDA IPC); null = no cross-rank sum.
  float* const* peer_tiles;
  int* const* peer_flags;
  int tp_world, tp_rank;
};

struct AttnParams {
  const float* q;
  int ldq;
  float* out;
  int ldo;
  KvView kv;
  const int* seq;
  const int* pos;
  int hd, n_heads, n_kv, window, chunk /* minimum positions per split */, n_splits, M;
  float scale;
  float* part;    // [M][n_kv][n_splits][G][hd + 4]
  int* counters;  // [M][n_kv]
  // decode kernel: the n_splits CTAs of (row, KV head) run as one cluster and
  // merge through distributed shared memory (part / counters unused);
  // n_splits <= attention_max_cluster()
  int cluster;
  int* err;       // error bits for the host (bounded waits)
  // prefill kernel: query blocks {row0, n_rows, seq, pos0} of consecutive
  // positions of one sequence (rows row0 .. row0 + n_rows - 1)
  const int4* blocks;
  int n_blocks;
};

struct LmHeadParams {
  const float* x;         // [M][D] raw residual rows
  const float* stats;     // [nstat][M]
  int nstat;
  const float* gamma;     // [D] or null
  const float* W;         // [D][V] fp32 (reference layout)
  int D, V, M;
  float* logits;          // [M][V] or null
  float* part_val;        // [M][n_ctas]
  int* part_idx;
  int* counter;
  int* argmax;            // [M] or null
  float* maxval;          // [M] the maximum itself (tensor-parallel combine), or null
  // tensor-core path (lm_tc_ok): scratch for the rows' bf16 hi / lo planes
  // and the error word of its bounded waits
  uint8_t* planes;
  size_t planes_bytes;
  int* err;
};


// Launchers (return cudaGetLastError of the launch).
cudaError_t launch_gemv(const GemvParams& p, int mg, int ch, cudaStream_t s, bool pdl);
cudaError_t launch_gemv_stream(const GemvParams& p, int mg, cudaStream_t s, bool pdl);
size_t gemv_stream_smem(int mg, int kseg);
// tcgen05 path (prefill / large batches): quantiser + GEMM, two launches
cudaError_t launch_gemm_tc(const GemvParams& p, cudaStream_t s, bool pdl);
int tc_rows_pad(int M);
// rows of limb planes + factors (quantiser only; the GEMMs launch it themselves)
cudaError_t launch_quant_rows(const GemvParams& p, int rows, cudaStream_t s, bool pdl);
// decode batches of 9..sk_rows_max() rows: weights on the MMA's 128-row side,
// k-slices (<= 8) merged inside a thread-block cluster; quantiser + GEMM
cudaError_t launch_gemm_sk(const GemvParams& p, cudaStream_t s, bool pdl);
cudaError_t prepare_gemm_sk();
int sk_rows_max();
size_t tc_limb_bytes(int M, int K);
cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl);
// tiled attention for prefill: one CTA per (query block, KV head)
cudaError_t launch_attention_prefill(const AttnParams& p, cudaStream_t s, bool pdl);
int attention_prefill_tokens(int head_dim, int group);  // tokens per query block
int attention_max_splits();
// Most splits that can run as one cluster (0: no cluster merge on this GPU).
int attention_max_cluster();
// one-time kernel attributes (dynamic shared memory above 48 KB)
cudaError_t prepare_gemv_stream();
cudaError_t prepare_attention();
cudaError_t prepare_gemm_tc();
cudaError_t prepare_attention_prefill();
cudaError_t launch_lm_head(const LmHeadParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_repack(uint4* out, const uint8_t* const* src, const int* src_n, int n_src,
                          const int* perm, int n_tiles, int K, cudaStream_t s);
// Per-sequence token table (the repetition-penalty history):
// tok[seq[m] * ld + pos[m]] = ids[m]; tok == null records nothing.
struct TokenLog {
  int* tok;
  int ld;
  const int* seq;
  const int* pos;
};
// x[m] = column ids[m] - v0 of the [D][V] table (zeros when that column is
// outside 0..V-1: another rank's vocabulary slice); stats per 16 columns;
// each id also goes to the token table.
// bos (may be null): token id bos_id embeds as bos[D] (rank 0's share under
// tensor parallelism) instead of its column.
cudaError_t launch_embed_stats(float* x, float* stats, const float* W,
                               const int* ids, int M, int D, int V, cudaStream_t s, bool pdl,
                               int v0 = 0, TokenLog log = TokenLog{nullptr, 0, nullptr, nullptr},
                               const float* bos = nullptr, int bos_id = -1);
// out[2 i + h] = ((q[i] >> 4 h) & 15) - 8) * scale: a Q4 [K][N/2] matrix as
// fp32 [K][N] (the reference's dequant, src/linalg/kernels.mojo:100-108).
cudaError_t launch_dequant_q4_f32(float* out, const uint8_t* q, size_t n_bytes, float scale,
                                  cudaStream_t s);
// Tensor-parallel epilogue of the row-parallel projections (O, down):
// out = resid * ple * inv_rms(resid * ple) + partial (already all-reduced),
// plus the per-16-column sums of squares of out.
cudaError_t launch_resid_add(float* out, float* out_stats, const float* partial,
                             const float* resid, const float* resid_stats, float resid_ple,
                             int M, int D, cudaStream_t s);
// Greedy argmax across vocabulary shards: pack (value, v0 + index) into keys
// whose unsigned maximum is the largest value, ties to the smallest index;
// then unpack the winning index.
cudaError_t launch_argmax_pack(unsigned long long* key, const float* val, const int* idx, int M,
                               int v0, cudaStream_t s);
cudaError_t launch_argmax_unpack(int* ids, const unsigned long long* key, int M, cudaStream_t s);
// K / V rows of positions pos0 .. pos0 + n - 1 of one sequence to (dir 0) or
// from (dir 1) dense fp32 device buffers [n][kv_dim].
cudaError_t launch_kv_copy(const KvView& kv, int seq, int pos0, int n, float* k, float* v,
                           int dir, cudaStream_t s);
// int8 cache: quantise the M staged fp32 K / V rows (kv.stage_k / stage_v)
// into the cache rows of (seq[m], pos[m]), one scale per KV head.
// lm_head on the tensor cores (ms_lm_tc.cu) for batches of 9+ rows:
// usable when lm_tc_ok(p) and a tensor map over W was made (lm_tc_make_map
// writes 128 bytes, 64-byte aligned, into map_out); at most `ctas`
// persistent CTAs.
bool lm_tc_ok(const LmHeadParams& p);
bool lm_tc_make_map(void* map_out, const float* W, int D, int V);
// Up to 8 rows on CUDA cores with the table streamed through a shared-memory
// ring of tensor copies (same tensor map); one persistent CTA per SM.
bool lm_ring_ok(const LmHeadParams& p);
cudaError_t launch_lm_ring(const LmHeadParams& p, const void* wmap, int ctas, cudaStream_t s,
                           bool pdl);
cudaError_t launch_lm_tc(const LmHeadParams& p, const void* wmap, int ctas, cudaStream_t s,
                         bool pdl);
cudaError_t prepare_lm_tc();
cudaError_t launch_kv_quant(const KvView& kv, const int* seq, const int* pos, int M,
                            cudaStream_t s, bool pdl);
cudaError_t launch_rowstats(float* stats, const float* x, int ldx, int M, int D,
                            cudaStream_t s, bool pdl);
cudaError_t launch_advance_step(int* ids, const int* next, int* pos, int* hist, int* step, int M,
                                cudaStream_t s, bool pdl);

// Repetition penalty + temperature sampling (temperature_sampling,
// src/inference/lm_head.mojo:198-254) over rows of fp32 logits.
constexpr int kSampChunk = 8192;   // logits columns per CTA
constexpr int kSampThreads = 256;
struct SampleParams {
  const float* logits;  // [M][ld]: this rank's V columns (global ids v0 ..)
  long long ld;
  int M, V, v0;
  int nchunk;           // ceil(V / kSampChunk)
  // history of row r ("generated"): CSR (hist + hist_off[r] .. hist_off[r+1])
  // when hist_off is set, else the token table tok[seq[r] * tok_ld + 0 .. pos[r]]
  const int* hist;
  const int* hist_off;
  const int* tok;
  const int* seq;
  const int* pos;
  int tok_ld;
  float temperature, penalty;
  const unsigned long long* seeds;  // per-row seeds (CSR mode) ...
  unsigned long long seed;          // ... else one seed mixed with (seq, pos)
  float2* part;        // [M][nchunk] chunk partials
  int* counter;        // [M] arrival tickets (zero between launches)
  float2* rowsum;      // tensor parallel: this rank's (max, sum) per row, or null
  const float2* rowsum_all;  // [W][M] all ranks' (max, sum), pick launch
  int tp_world, tp_rank;
  int* out;            // [M] global ids (greedy TP: this rank's local index)
  float* maxval;       // greedy TP: this rank's penalised maximum, or null
};
// Chunk pass (+ the pick for a single rank, by the last CTA of each row).
cudaError_t launch_sample(const SampleParams& p, cudaStream_t s);
// Tensor parallel, temperature mode: the pick after the all-gather of the
// ranks' (max, sum); the owning rank writes the id, the others -1.
cudaError_t launch_sample_pick(const SampleParams& p, cudaStream_t s);

}  // namespace ms
