/*
 * ms_oracle.c -- CPU restatement of MojoStream's Gemma-4 token loop.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker of the CUDA library and the
 * timed CPU baseline (bench.py --impl reference).  Never part of the product.
 *
 * The reference is Mojo; it cannot be built here (no Mojo toolchain), so this
 * file restates its algorithm in C.  The blocking of the Q4 matmul follows the
 * reference (BK = 128 k-tiles, MR = 4 rows, NR = 2 * SIMD_W columns, a
 * dequantised B tile reused by all row blocks, C += acc after every k-tile,
 * threads over 64-row M blocks) so that the CPU baseline does the same work
 * in the same order.  SIMD_W = 16 (an AVX-512 host); reductions that the
 * reference does as SIMD lanes + reduce_add are done with the same 16 lanes.
 *
 * Parity is pinned by tests/golden (fixtures made by the reference's own
 * NumPy oracle, scripts/gen_reference.py).
 */
#include "ms_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define SIMD_W 16
#define MR 4
#define NR (2 * SIMD_W)
#define BM 64
#define BK 128

static int imin(int a, int b) { return a < b ? a : b; }

/* Nearest bfloat16 (ties to even) of a finite float, as a float: keep the top
 * 16 bits after adding half of the dropped range (IEEE 754 rounding). */
static float round_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) != 0x7f800000u) u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    memcpy(&f, &u, 4);
    return f;
}

void orc_quant_i8(const float *x, int n, signed char *q, float *scale)
{
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) {
        const float a = fabsf(x[i]);
        if (a > amax) amax = a;
    }
    /* rows below 2^-120 (127 / amax would overflow) are stored as zero rows;
     * the clamp is fminf(fmaxf()) as on the GPU, which also maps a NaN to -127 */
    const int live = amax >= 0x1p-120f;
    const float s = live ? amax / 127.0f : 0.0f;
    const float inv = live ? 127.0f / amax : 0.0f;
    for (int i = 0; i < n; ++i) {
        const float r = fminf(fmaxf(rintf(x[i] * inv), -127.0f), 127.0f);
        q[i] = (signed char)r;
    }
    *scale = s;
}

void orc_quant_i8_rows(const float *x, int rows, int n, signed char *q, float *scale)
{
    for (int r = 0; r < rows; ++r)
        orc_quant_i8(x + (size_t)r * n, n, q + (size_t)r * n, scale + r);
}

/* A head row as the int8 cache holds it: q * scale, in place. */
static void round_i8_row(float *x, int n)
{
    signed char q[1024];
    float s;
    orc_quant_i8(x, n, q, &s);
    for (int i = 0; i < n; ++i) x[i] = (float)q[i] * s;
}

/* kernels.mojo:100-108: low nibble -> even column, high nibble -> odd column,
 * value (nibble - 8) * scale. */
float orc_dequant(const uint8_t *w, int N, int k, int n, float scale)
{
    uint8_t b = w[(size_t)k * (size_t)(N / 2) + (size_t)(n / 2)];
    int nib = (n & 1) ? (b >> 4) : (b & 15);
    return (float)(nib - 8) * scale;
}

/* ---------------------------------------------------------------- threads */

typedef struct {
    void (*fn)(void *arg, int block);
    void *arg;
    int n_blocks;
    int next;
    pthread_mutex_t mu;
} pool_job_t;

static void *pool_worker(void *p)
{
    pool_job_t *job = (pool_job_t *)p;
    for (;;) {
        pthread_mutex_lock(&job->mu);
        int b = job->next++;
        pthread_mutex_unlock(&job->mu);
        if (b >= job->n_blocks) break;
        job->fn(job->arg, b);
    }
    return NULL;
}

/* The reference's parallelize[fn](n_blocks, workers) (kernels.mojo:266-267). */
static void parallel_blocks(void (*fn)(void *, int), void *arg, int n_blocks,
                            int workers)
{
    if (workers < 1) workers = 1;
    if (workers > n_blocks) workers = n_blocks;
    if (workers <= 1) {
        for (int b = 0; b < n_blocks; ++b) fn(arg, b);
        return;
    }
    pool_job_t job = {fn, arg, n_blocks, 0, PTHREAD_MUTEX_INITIALIZER};
    pthread_t th[64];
    if (workers > 64) workers = 64;
    for (int i = 0; i < workers; ++i) pthread_create(&th[i], NULL, pool_worker, &job);
    for (int i = 0; i < workers; ++i) pthread_join(th[i], NULL);
}

/* --------------------------------------------------------------- Q4 matmul */

typedef struct {
    float *C;
    const float *A;
    const uint8_t *W;
    int M, K, N;
    float scale;
} q4_args_t;

/* One 64-row M block of kernels.mojo:216-264. */
static void q4_mblock(void *p, int mb)
{
    const q4_args_t *a = (const q4_args_t *)p;
    const int m0 = mb * BM, m1 = imin(m0 + BM, a->M);
    const int K = a->K, N = a->N, pc = N / 2;
    float bbuf[BK * NR];
    for (int kt = 0; kt < K; kt += BK) {
        const int bk = imin(BK, K - kt);
        for (int nt = 0; nt < N; nt += NR) {
            const int nw = imin(NR, N - nt);
            /* pre-dequantise the (bk x NR) tile once for every row block */
            for (int kl = 0; kl < bk; ++kl) {
                const uint8_t *row = a->W + (size_t)(kt + kl) * pc + nt / 2;
                float *dst = bbuf + kl * NR;
                for (int j = 0; j < nw / 2; ++j) {
                    const uint8_t b = row[j];
                    dst[2 * j] = (float)((int)(b & 15) - 8) * a->scale;
                    dst[2 * j + 1] = (float)((int)(b >> 4) - 8) * a->scale;
                }
                for (int n = nw; n < NR; ++n) dst[n] = 0.f;
            }
            for (int m = m0; m < m1; m += MR) {
                const int mr = imin(MR, m1 - m);
                float acc[MR][NR];
                memset(acc, 0, sizeof acc);
                for (int kl = 0; kl < bk; ++kl) {
                    const float *brow = bbuf + kl * NR;
                    for (int r = 0; r < mr; ++r) {
                        const float av = a->A[(size_t)(m + r) * K + kt + kl];
                        for (int n = 0; n < NR; ++n) acc[r][n] = acc[r][n] + av * brow[n];
                    }
                }
                for (int r = 0; r < mr; ++r) {
                    float *crow = a->C + (size_t)(m + r) * N + nt;
                    for (int n = 0; n < nw; ++n) crow[n] = crow[n] + acc[r][n];
                }
            }
        }
    }
}

void orc_q4_matmul(float *C, const float *A, const uint8_t *W, int M, int K,
                   int N, float scale, int workers)
{
    q4_args_t a = {C, A, W, M, K, N, scale};
    parallel_blocks(q4_mblock, &a, (M + BM - 1) / BM, workers);
}

/* ------------------------------------------------------------- fp32 matmul */

typedef struct {
    float *C;
    const float *A;
    const float *B;
    int M, K, N;
} f32_args_t;

/* One M block of kernels.mojo:631-668 (tail columns beyond a multiple of NR
 * are skipped there; the same is done here). */
static void f32_mblock(void *p, int mb)
{
    const f32_args_t *a = (const f32_args_t *)p;
    const int m0 = mb * BM, m1 = imin(m0 + BM, a->M);
    const int K = a->K, N = a->N;
    for (int kt = 0; kt < K; kt += BK) {
        const int bk = imin(BK, K - kt);
        for (int nt = 0; nt + NR <= N; nt += NR) {
            for (int m = m0; m < m1; m += MR) {
                const int mr = imin(MR, m1 - m);
                float acc[MR][NR];
                memset(acc, 0, sizeof acc);
                for (int kl = 0; kl < bk; ++kl) {
                    const float *brow = a->B + (size_t)(kt + kl) * N + nt;
                    for (int r = 0; r < mr; ++r) {
                        const float av = a->A[(size_t)(m + r) * K + kt + kl];
                        for (int n = 0; n < NR; ++n) acc[r][n] = acc[r][n] + av * brow[n];
                    }
                }
                for (int r = 0; r < mr; ++r) {
                    float *crow = a->C + (size_t)(m + r) * N + nt;
                    for (int n = 0; n < NR; ++n) crow[n] = crow[n] + acc[r][n];
                }
            }
        }
    }
}

void orc_fp32_matmul(float *C, const float *A, const float *B, int M, int K,
                     int N, int workers)
{
    f32_args_t a = {C, A, B, M, K, N};
    parallel_blocks(f32_mblock, &a, (M + BM - 1) / BM, workers);
}

/* ------------------------------------------------------------ elementwise */

/* Sum of squares as SIMD_W lane partials followed by a lane reduction. */
static float sumsq_lanes(const float *x, int n)
{
    float lane[SIMD_W] = {0};
    int i = 0;
    for (; i + SIMD_W <= n; i += SIMD_W)
        for (int l = 0; l < SIMD_W; ++l) lane[l] = lane[l] + x[i + l] * x[i + l];
    for (int l = 0; i < n; ++i, ++l) lane[l] = lane[l] + x[i] * x[i];
    float s = 0.f;
    for (int l = 0; l < SIMD_W; ++l) s += lane[l];
    return s;
}

void orc_rmsnorm(float *x, int rows, int cols)
{
    for (int r = 0; r < rows; ++r) {
        float *rp = x + (size_t)r * cols;
        const float inv = 1.0f / sqrtf(sumsq_lanes(rp, cols) / (float)cols + 1e-6f);
        for (int i = 0; i < cols; ++i) rp[i] = rp[i] * inv;
    }
}

void orc_rmsnorm_weighted(float *x, const float *gamma, int rows, int cols)
{
    for (int r = 0; r < rows; ++r) {
        float *rp = x + (size_t)r * cols;
        const float inv = 1.0f / sqrtf(sumsq_lanes(rp, cols) / (float)cols + 1e-6f);
        for (int i = 0; i < cols; ++i) rp[i] = rp[i] * inv * gamma[i];
    }
}

void orc_ple_scale(float *x, int n, float s)
{
    for (int i = 0; i < n; ++i) x[i] = x[i] * s;
}

void orc_swiglu(const float *gate, float *up, int n)
{
    for (int i = 0; i < n; ++i) {
        const float g = gate[i];
        const float sig = 1.0f / (1.0f + expf(-g));
        up[i] = up[i] * g * sig;
    }
}

void orc_rope_inv_freq(float *out, int hd, float theta)
{
    const float ln_base = logf(theta);
    for (int i = 0; i < hd / 2; ++i)
        out[i] = expf(-(float)(2 * i) / (float)hd * ln_base);
}

void orc_rope(float *x, int n_heads, int hd, int pos, float theta)
{
    const int half = hd / 2;
    float inv[512], cs[512], sn[512];
    orc_rope_inv_freq(inv, hd, theta);
    const float pf = (float)pos;
    for (int i = 0; i < half; ++i) {
        const float th = pf * inv[i];
        cs[i] = cosf(th);
        sn[i] = sinf(th);
    }
    for (int h = 0; h < n_heads; ++h) {
        float *hp = x + (size_t)h * hd;
        for (int i = 0; i < half; ++i) {
            const float a = hp[i], b = hp[i + half];
            hp[i] = a * cs[i] - b * sn[i];
            hp[i + half] = a * sn[i] + b * cs[i];
        }
    }
}

/* -------------------------------------------------------------- attention */

static float dot_lanes(const float *a, const float *b, int n)
{
    float lane[SIMD_W] = {0};
    int i = 0;
    for (; i + SIMD_W <= n; i += SIMD_W)
        for (int l = 0; l < SIMD_W; ++l) lane[l] = lane[l] + a[i + l] * b[i + l];
    float s = 0.f;
    for (int l = 0; l < SIMD_W; ++l) s += lane[l];
    for (; i < n; ++i) s += a[i] * b[i];
    return s;
}

void orc_attention_row(float *out, const float *q, const float *kc,
                       const float *vc, int cap, int circular, int lo,
                       int pos, int n_heads, int n_kv, int hd)
{
    const int kv_dim = n_kv * hd;
    const int ratio = n_heads / n_kv;
    const float scale = 1.0f / sqrtf((float)hd);
    const int n = pos - lo + 1;
    float *sc = (float *)malloc(sizeof(float) * (size_t)n);
    for (int h = 0; h < n_heads; ++h) {
        const int hk = h / ratio;
        const float *qh = q + (size_t)h * hd;
        for (int i = 0; i < n; ++i) {
            const int t = lo + i;
            const int slot = circular ? t % cap : t;
            sc[i] = dot_lanes(qh, kc + (size_t)slot * kv_dim + (size_t)hk * hd, hd) * scale;
        }
        float mx = sc[0];
        for (int i = 1; i < n; ++i)
            if (sc[i] > mx) mx = sc[i];
        float sum = 0.f;
        for (int i = 0; i < n; ++i) {
            sc[i] = expf(sc[i] - mx);
            sum += sc[i];
        }
        const float inv = 1.0f / sum;
        for (int i = 0; i < n; ++i) sc[i] = sc[i] * inv;
        float *oh = out + (size_t)h * hd;
        for (int d = 0; d < hd; ++d) oh[d] = 0.f;
        for (int i = 0; i < n; ++i) {
            const int t = lo + i;
            const int slot = circular ? t % cap : t;
            const float *vh = vc + (size_t)slot * kv_dim + (size_t)hk * hd;
            const float p = sc[i];
            for (int d = 0; d < hd; ++d) oh[d] = oh[d] + p * vh[d];
        }
    }
    free(sc);
}

/* ------------------------------------------------------------------ layer */

int orc_layer_forward(const orc_layer_t *L, int D, float *x, int M,
                      const int *seq, const int *pos, orc_kv_layer_t *kv,
                      int workers)
{
    const int hd = L->head_dim, nh = L->n_heads, nkv = L->n_kv_heads;
    const int qd = nh * hd, kvd = nkv * hd, F = L->ffn_dim;
    if (kv->kv_dim != kvd) return -1;
    for (int r = 0; r < M; ++r) {
        if (seq[r] < 0 || seq[r] >= kv->n_seq || pos[r] < 0) return -2;
        if (L->window == 0 && pos[r] >= kv->cap) return -3;
    }
    float *q = (float *)calloc((size_t)M * qd, sizeof(float));
    float *k = (float *)calloc((size_t)M * kvd, sizeof(float));
    float *v = (float *)calloc((size_t)M * kvd, sizeof(float));
    float *att = (float *)calloc((size_t)M * qd, sizeof(float));
    float *prj = (float *)calloc((size_t)M * D, sizeof(float));
    float *g = (float *)calloc((size_t)M * F, sizeof(float));
    float *u = (float *)calloc((size_t)M * F, sizeof(float));

    /* 1. PLE + pre-norm (main.mojo:570-571; gemma4_e4b.mojo:474-475) */
    orc_ple_scale(x, M * D, L->ple);
    orc_rmsnorm(x, M, D);
    /* 2. Q/K/V into zeroed buffers (main.mojo:574-576) */
    orc_q4_matmul(q, x, L->w[ORC_Q], M, D, qd, L->scale[ORC_Q], workers);
    orc_q4_matmul(k, x, L->w[ORC_K], M, D, kvd, L->scale[ORC_K], workers);
    orc_q4_matmul(v, x, L->w[ORC_V], M, D, kvd, L->scale[ORC_V], workers);
    /* 3. RoPE: leading rotary_dims of every head (main.mojo:579-581;
     *    gemma4_e4b.mojo:489-505 for the partial-rotary full layers) */
    for (int r = 0; r < M; ++r) {
        float *qr = q + (size_t)r * qd, *kr = k + (size_t)r * kvd;
        if (L->rotary_dims == hd) {
            orc_rope(qr, nh, hd, pos[r], L->rope_theta);
            orc_rope(kr, nkv, hd, pos[r], L->rope_theta);
        } else {
            for (int h = 0; h < nh; ++h)
                orc_rope(qr + (size_t)h * hd, 1, L->rotary_dims, pos[r], L->rope_theta);
            for (int h = 0; h < nkv; ++h)
                orc_rope(kr + (size_t)h * hd, 1, L->rotary_dims, pos[r], L->rope_theta);
        }
    }
    /* 4. KV write (main.mojo:584-592; gemma4_e4b.mojo:211-249) */
    const int circular = L->window > 0;
    for (int r = 0; r < M && !kv->frozen; ++r) {
        const int slot = circular ? pos[r] % kv->cap : pos[r];
        const size_t off = ((size_t)seq[r] * kv->cap + slot) * kvd;
        memcpy(kv->k + off, k + (size_t)r * kvd, sizeof(float) * kvd);
        memcpy(kv->v + off, v + (size_t)r * kvd, sizeof(float) * kvd);
        if (kv->bf16)
            for (int j = 0; j < kvd; ++j) {
                kv->k[off + j] = round_bf16(kv->k[off + j]);
                kv->v[off + j] = round_bf16(kv->v[off + j]);
            }
        if (kv->i8)
            for (int h = 0; h < nkv; ++h) {
                round_i8_row(kv->k + off + (size_t)h * hd, hd);
                round_i8_row(kv->v + off + (size_t)h * hd, hd);
            }
    }
    /* 5. attention (main.mojo:445-519; gemma4_e4b.mojo:259-411) */
    for (int r = 0; r < M; ++r) {
        int lo = 0;
        if (circular) {
            lo = pos[r] + 1 - L->window;
            if (lo < 0) lo = 0;
        }
        const size_t base = (size_t)seq[r] * kv->cap * kvd;
        orc_attention_row(att + (size_t)r * qd, q + (size_t)r * qd, kv->k + base,
                          kv->v + base, kv->cap, circular, lo, pos[r], nh, nkv, hd);
    }
    /* 6. O projection + residual onto the normalised x (main.mojo:598-600) */
    orc_q4_matmul(prj, att, L->w[ORC_O], M, qd, D, L->scale[ORC_O], workers);
    for (int i = 0; i < M * D; ++i) x[i] = x[i] + prj[i];
    /* 7. post-attention norm (main.mojo:603) */
    orc_rmsnorm(x, M, D);
    /* 8. SwiGLU FFN + residual (main.mojo:606-613) */
    orc_q4_matmul(g, x, L->w[ORC_GATE], M, D, F, L->scale[ORC_GATE], workers);
    orc_q4_matmul(u, x, L->w[ORC_UP], M, D, F, L->scale[ORC_UP], workers);
    orc_swiglu(g, u, M * F);
    memset(prj, 0, sizeof(float) * (size_t)M * D);
    orc_q4_matmul(prj, u, L->w[ORC_DOWN], M, F, D, L->scale[ORC_DOWN], workers);
    for (int i = 0; i < M * D; ++i) x[i] = x[i] + prj[i];

    free(q); free(k); free(v); free(att); free(prj); free(g); free(u);
    return 0;
}

/* ---------------------------------------------------------------- lm head */

void orc_lm_head(float *logits, float *x, const float *gamma, const float *W,
                 int M, int D, int V, int workers)
{
    orc_rmsnorm_weighted(x, gamma, M, D);
    memset(logits, 0, sizeof(float) * (size_t)M * V);
    orc_fp32_matmul(logits, x, W, M, D, V, workers);
}

int orc_argmax(const float *row, int n)
{
    int best = 0;
    float bv = row[0];
    for (int j = 1; j < n; ++j)
        if (row[j] > bv) { bv = row[j]; best = j; }
    return best;
}

float orc_sample_target(uint64_t seed)
{
    /* lm_head.mojo:246-247: one LCG step, low 31 bits, divided by
     * Float32(0x7FFFFFFF), which rounds to 2^31. */
    uint64_t lcg = (seed * 6364136223846793005ull + 1442695040888963407ull) & 0x7FFFFFFFull;
    return (float)lcg / (float)0x7FFFFFFF;
}

int orc_temperature_sampling(float *row, int n, float temperature, const int *generated,
                             int n_generated, float penalty, uint64_t seed)
{
    /* lm_head.mojo:213-221 */
    if (penalty > 1.0f) {
        for (int i = 0; i < n_generated; ++i) {
            int tid = generated[i];
            if (tid >= 0 && tid < n) {
                float v = row[tid];
                row[tid] = v > 0.0f ? v / penalty : v * penalty;
            }
        }
    }
    /* :223-230 */
    if (temperature <= 0.01f) return orc_argmax(row, n);
    /* :232-243 */
    float inv_t = 1.0f / temperature;
    float max_v = row[0];
    for (int j = 1; j < n; ++j)
        if (row[j] > max_v) max_v = row[j];
    float sum_e = 0.0f;
    for (int j = 0; j < n; ++j) {
        float e = expf((row[j] - max_v) * inv_t);
        row[j] = e;
        sum_e += e;
    }
    float inv_s = 1.0f / sum_e;
    for (int j = 0; j < n; ++j) row[j] = row[j] * inv_s;
    /* :245-254 */
    float target = orc_sample_target(seed);
    float cdf = 0.0f;
    for (int j = 0; j < n; ++j) {
        cdf += row[j];
        if (cdf >= target) return j;
    }
    return n - 1;
}

void orc_embed(float *x, const float *W, int D, int V, int id)
{
    for (int r = 0; r < D; ++r) x[r] = W[(size_t)r * V + id];
}
