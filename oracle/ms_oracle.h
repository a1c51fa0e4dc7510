/*
 * ms_oracle.h -- CPU restatement of MojoStream's Gemma-4 token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the parity checker for the CUDA library
 * (libmojostream_cuda.so) and the timed CPU baseline of bench.py.  Nothing in
 * the product path links, loads or calls it.
 *
 * Every function restates one routine of the reference (phunck/MojoStream,
 * Mojo 0.26.2); the routine is cited as path:line inside that project.
 * Pinned against the reference's own NumPy oracle (scripts/gen_reference.py)
 * through the golden fixtures in tests/golden/.
 */
#ifndef MS_ORACLE_H
#define MS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Matrix slots of one layer, in the order of the .mojostream directory
 * (src/streaming/mojostream.mojo:20-27: PLE=0, Q=1 ... Down=7; slot = tag-1). */
enum { ORC_Q = 0, ORC_K, ORC_V, ORC_O, ORC_GATE, ORC_UP, ORC_DOWN, ORC_NMAT };

typedef struct {
    int head_dim;      /* per-head width (demo: hidden/n_heads, main.mojo:551)       */
    int n_heads;       /* query heads                                                 */
    int n_kv_heads;    /* key/value heads (GQA)                                       */
    int window;        /* 0 = attend to all cached positions; >0 = sliding window     */
    int rotary_dims;   /* leading dims of each head that RoPE rotates                 */
    int ffn_dim;       /* SwiGLU intermediate width                                   */
    float rope_theta;  /* RoPE base                                                   */
    float ple;         /* per-layer scalar applied before the pre-norm                */
    const uint8_t *w[ORC_NMAT]; /* Q4 weights, reference layout [K][N/2]              */
    float scale[ORC_NMAT];      /* one fp32 scale per tensor                          */
} orc_layer_t;

/* KV cache of one layer: n_seq sequences x cap slots x kv_dim floats (K and V).
 * bf16 != 0 stores every K / V value rounded to bfloat16 (round to nearest,
 * ties to even): the reduced-precision cache of the GPU path, for its own
 * looser parity check. */
typedef struct {
    int n_seq;
    int cap;           /* slots per sequence (window>0: circular, slot = pos % cap)  */
    int kv_dim;
    float *k;
    float *v;
    int bf16;
    int frozen;        /* != 0: orc_layer_forward attends over the cache as it is and
                          writes no K / V row (a checker that has copied another
                          implementation's rows in compares only the arithmetic) */
    int i8;            /* != 0: every K / V head row is stored as the int8 cache
                          reads it back (orc_quant_i8, then q * scale) */
} orc_kv_layer_t;

/* int8 KV cache quantisation of one head row x[0..n): scale = amax / 127,
 * q[i] = rint(x[i] * (127 / amax)) clamped to [-127, 127] (amax = max |x|;
 * an all-zero row has scale 0).  Each step is one IEEE-rounded float
 * operation: the GPU cache computes the same bits. */
void orc_quant_i8(const float *x, int n, signed char *q, float *scale);
/* orc_quant_i8 over rows head rows of n values each (x, q: [rows][n]). */
void orc_quant_i8_rows(const float *x, int rows, int n, signed char *q, float *scale);

/* kernels.mojo:100-108 (dequant_vec): value of logical column n in row k. */
float orc_dequant(const uint8_t *w, int N, int k, int n, float scale);

/* kernels.mojo:201-267 (matmul_q4_bpack_raw): C[M,N] += A[M,K] . deq(W[K][N/2]).
 * workers: threads over 64-row M-blocks (the reference's parallelize). */
void orc_q4_matmul(float *C, const float *A, const uint8_t *W, int M, int K,
                   int N, float scale, int workers);

/* kernels.mojo:616-671 (matmul_fp32_raw): C[M,N] += A[M,K] . B[K,N]. */
void orc_fp32_matmul(float *C, const float *A, const float *B, int M, int K,
                     int N, int workers);

/* kernels.mojo:474-489 */
void orc_rmsnorm(float *x, int rows, int cols);
/* kernels.mojo:598-613 */
void orc_rmsnorm_weighted(float *x, const float *gamma, int rows, int cols);
/* kernels.mojo:506-516 */
void orc_ple_scale(float *x, int n, float s);
/* kernels.mojo:519-532: up <- up * gate * sigmoid(gate) */
void orc_swiglu(const float *gate, float *up, int n);
/* kernels.mojo:553-595: rotate pairs (i, i+hd/2) of n_heads heads of width hd
 * laid out back to back. */
void orc_rope(float *x, int n_heads, int hd, int pos, float theta);
/* The inverse-frequency table the rotation uses (kernels.mojo:573-575). */
void orc_rope_inv_freq(float *out, int hd, float theta);

/* main.mojo:445-519, gemma4_e4b.mojo:259-411: causal GQA attention of one row.
 * q: [n_heads*hd]; out: [n_heads*hd]; kc/vc: one sequence's cache
 * [cap][n_kv*hd]; the row attends positions lo..pos (inclusive). */
void orc_attention_row(float *out, const float *q, const float *kc,
                       const float *vc, int cap, int circular, int lo,
                       int pos, int n_heads, int n_kv, int hd);

/* main.mojo:538-613 / gemma4_e4b.mojo:459-540: one layer, in place on x[M,D].
 * Row r belongs to sequence seq[r] at position pos[r]. */
int orc_layer_forward(const orc_layer_t *L, int D, float *x, int M,
                      const int *seq, const int *pos, orc_kv_layer_t *kv,
                      int workers);

/* lm_head.mojo:119-130 + 146-168: final weighted norm then fp32 projection.
 * logits [M,V] are overwritten. x is normalised in place. */
void orc_lm_head(float *logits, float *x, const float *gamma, const float *W,
                 int M, int D, int V, int workers);

/* lm_head.mojo:224-230: greedy pick, strict '>' so the first maximum wins. */
int orc_argmax(const float *row, int n);

/* lm_head.mojo:198-254 (temperature_sampling), one logits row, modified in
 * place as there: repetition penalty once per entry of `generated` (divide
 * positive, multiply non-positive logits) when penalty > 1; temperature <=
 * 0.01 -> first maximum; else softmax(logits / T), normalised, and the first
 * id whose running sum reaches target = ((seed * 6364136223846793005 +
 * 1442695040888963407) & 0x7FFFFFFF) / 2^31 (the reference takes the seed
 * from perf_counter_ns), n - 1 if the sum never reaches it. */
int orc_temperature_sampling(float *row, int n, float temperature, const int *generated,
                             int n_generated, float penalty, uint64_t seed);
/* The target above, for a seed. */
float orc_sample_target(uint64_t seed);

/* lm_head.mojo:171-195: x = column `id` of the fp32 [D][V] table. */
void orc_embed(float *x, const float *W, int D, int V, int id);

#ifdef __cplusplus
}
#endif
#endif
