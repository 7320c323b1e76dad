/*
 * TEST INFRASTRUCTURE -- the CPU oracle.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg may load this library, and only as the
 * checker.  The product (freeml_b200/, include/) never links or calls it.
 *
 * A plain-C restatement of FreeML's reference CPU path for the NanoLLM token
 * loop (Model<float, MatrixCPU<float>>::Run + greedy argmax).  Every routine
 * keeps the reference's fp32 evaluation order (sequential-k accumulation,
 * sequential row sums), so that it can be pinned bit-for-bit against the
 * reference harness (oracle/ref_nanollm.cpp) on the committed golden vectors.
 * Each function cites the reference file:line it restates.
 *
 * Weight initialisation restates the reference's draw sequence: one global
 * std::mt19937 (ToolsLibrary/Tools.h:15-19) feeding a freshly constructed
 * std::normal_distribution<float> per value (Tools.h:22-27).  The libstdc++
 * algorithms behind those two names are restated here: MT19937 (Matsumoto &
 * Nishimura 1998, init_genrand seeding), generate_canonical<float,24> (one
 * 32-bit draw scaled by 2^-32) and Marsaglia's polar method, which returns the
 * second of the pair -- the first is cached in the distribution object and
 * lost, because the reference assigns a new distribution before every draw.
 *
 * FMA: the reference build (g++ -O3, x86-64-v3, GCC's default contraction)
 * fuses a multiply feeding an add into one fma -- except in loop-carried
 * accumulation chains such as `sum += a * b`, which GCC's generic tuning keeps
 * unfused.  This file is compiled with -ffp-contract=off and writes the
 * fused operations out with fmaf() exactly where the reference build has them
 * (pinned bit for bit by tests/test_oracle_golden.py):
 *   - every dot-product / row-sum accumulation: unfused (MAC below);
 *   - LayerNorm's `var * invCols + eps` and `xhat * gamma + beta`: fused;
 *   - ScaleAdd's `in * scale + add`: fused;
 *   - the normal draw's r2 = fma(y, y, x*x) and `v * stddev + mean`: fused.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifndef ORACLE_FUSED
#define ORACLE_FUSED 0
#endif
#if ORACLE_FUSED
#define MAC(acc, a, b) fmaf((a), (b), (acc))
#else
#define MAC(acc, a, b) ((acc) + (a) * (b))
#endif

/* ------------------------------------------------------------------ RNG -- */

typedef struct { uint32_t mt[624]; int idx; } mt19937_t;

static void mt_seed(mt19937_t* g, uint32_t s)
{
    g->mt[0] = s;
    for (int i = 1; i < 624; ++i)
        g->mt[i] = 1812433253u * (g->mt[i - 1] ^ (g->mt[i - 1] >> 30)) + (uint32_t)i;
    g->idx = 624;
}

static uint32_t mt_next(mt19937_t* g)
{
    if (g->idx >= 624)
    {
        for (int i = 0; i < 624; ++i)
        {
            uint32_t y = (g->mt[i] & 0x80000000u) | (g->mt[(i + 1) % 624] & 0x7fffffffu);
            uint32_t v = g->mt[(i + 397) % 624] ^ (y >> 1);
            if (y & 1u) v ^= 0x9908b0dfu;
            g->mt[i] = v;
        }
        g->idx = 0;
    }
    uint32_t y = g->mt[g->idx++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* generate_canonical<float, 24>: the 32-bit draw is converted to float (round
 * to nearest) and divided by 2^32; a result of 1.0 is pulled down to the
 * largest float below 1. */
static float canonical_f32(mt19937_t* g)
{
    float r = (float)mt_next(g) / 4294967296.0f;
    if (r >= 1.0f) r = nextafterf(1.0f, 0.0f);
    return r;
}

/* One draw of a fresh std::normal_distribution<float>(mean, stddev):
 * Marsaglia's polar method; the pair's second value is returned. */
static float normal_f32(mt19937_t* g, float mean, float stddev)
{
    float x, y, r2;
    do {
        x = 2.0f * canonical_f32(g) - 1.0f;
        y = 2.0f * canonical_f32(g) - 1.0f;
        r2 = fmaf(y, y, x * x);
    } while (r2 > 1.0f || r2 == 0.0f);
    const float mult = sqrtf(-2.0f * logf(r2) / r2);
    return fmaf(y * mult, stddev, mean);
}

/* Prompt recipe used by the harness, the tests and the bench: the first
 * (u32 & mask) <= V-1 per token, mask = 2^ceil(log2 V) - 1.  This is also what
 * numpy's legacy RandomState(seed).randint(0, V, n) draws. */
void oracle_prompt_tokens(uint32_t seed, uint32_t V, uint64_t n, uint32_t* out)
{
    mt19937_t g;
    mt_seed(&g, seed);
    uint32_t mask = 1;
    while (mask < V - 1u) mask = (mask << 1) | 1u;
    if (V == 1u) mask = 0u;
    for (uint64_t i = 0; i < n; ++i)
    {
        uint32_t v;
        do { v = mt_next(&g) & mask; } while (v > V - 1u);
        out[i] = v;
    }
}

/* ------------------------------------------------------------- config -- */

typedef struct
{
    uint32_t V, C, d, H, L;
} oracle_cfg;

/* Canonical parameter order (also the CUDA engine's):
 * tok_emb[V*d], pos_emb[C*d], per layer {ln0_g[d], w_qkv[d*3d], w_proj[d*d]
 * (out x in), ln1_g[d], w_fc[d*4d], w_mlp[4d*d]}, lnf_g[d]. */
uint64_t oracle_weight_count(const oracle_cfg* c)
{
    const uint64_t d = c->d;
    return (uint64_t)c->V * d + (uint64_t)c->C * d + (uint64_t)c->L * (2 * d + 12 * d * d) + d;
}

static void fill_normal(mt19937_t* g, float* p, uint64_t n)
{
    for (uint64_t i = 0; i < n; ++i) p[i] = normal_f32(g, 0.0f, 0.02f);
}

/* Draw order of BuildOrLoadModel + Model::Init:
 *   token table V*d   (InitEmbeddingBlob, LayerLibrary/Embedding.h:51-56)
 *   position table C*d
 *   lm_head V*d, discarded by weight tying (Examples/NanoLLM/NanoLLM.cpp:329-345)
 *   per block, in execution order (TransformerBlock.h:200-334):
 *     w_qkv [d x 3d], w_proj [d x d] then *= 1/sqrt(2L)  (CausalSelfAttentionLayer.h:45-50, TransformerBlock.h:247-256)
 *     w_fc [d x 4d], w_mlp [4d x d] then *= 1/sqrt(2L)   (TransformerBlock.h:279-325)
 * Dense weights are drawn in storage order (Dense.h:75-80, MapFunction_Zero).
 * LayerNorm gammas are 1 (LayerNorm.h:115). */
int oracle_init_weights(const oracle_cfg* c, uint32_t seed, float* w)
{
    mt19937_t* g = (mt19937_t*)malloc(sizeof(mt19937_t));
    if (!g) return -1;
    mt_seed(g, seed);
    const uint64_t d = c->d, V = c->V, C = c->C;
    float* p = w;
    fill_normal(g, p, V * d); p += V * d;
    fill_normal(g, p, C * d); p += C * d;
    for (uint64_t i = 0; i < V * d; ++i) (void)normal_f32(g, 0.0f, 0.02f);
    const float rscale = 1.0f / sqrtf(2.0f * (float)c->L);
    for (uint32_t l = 0; l < c->L; ++l)
    {
        for (uint64_t i = 0; i < d; ++i) p[i] = 1.0f;
        p += d;
        fill_normal(g, p, 3 * d * d); p += 3 * d * d;
        fill_normal(g, p, d * d);
        for (uint64_t i = 0; i < d * d; ++i) p[i] = p[i] * rscale;
        p += d * d;
        for (uint64_t i = 0; i < d; ++i) p[i] = 1.0f;
        p += d;
        fill_normal(g, p, 4 * d * d); p += 4 * d * d;
        fill_normal(g, p, 4 * d * d);
        for (uint64_t i = 0; i < 4 * d * d; ++i) p[i] = p[i] * rscale;
        p += 4 * d * d;
    }
    for (uint64_t i = 0; i < d; ++i) p[i] = 1.0f;
    free(g);
    return 0;
}

/* ------------------------------------------------------- thread helper -- */

typedef void (*range_fn)(void* ctx, uint32_t begin, uint32_t end);
typedef struct { range_fn fn; void* ctx; uint32_t b, e; } range_job;

static void* range_thunk(void* p)
{
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->b, j->e);
    return NULL;
}

static int g_threads = 1;
void oracle_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

static void parallel_rows(range_fn fn, void* ctx, uint32_t n)
{
    int nt = g_threads;
    if (nt <= 1 || n < 2) { fn(ctx, 0, n); return; }
    if ((uint32_t)nt > n) nt = (int)n;
    pthread_t th[256];
    range_job jobs[256];
    int started[256];
    const uint32_t per = (n + (uint32_t)nt - 1) / (uint32_t)nt;
    for (int t = 0; t < nt; ++t)
    {
        const uint32_t b = (uint32_t)t * per, e = b + per > n ? n : b + per;
        started[t] = 0;
        if (b >= e) continue;
        jobs[t] = (range_job){fn, ctx, b, e};
        if (pthread_create(&th[t], NULL, range_thunk, &jobs[t]) == 0) started[t] = 1;
        else fn(ctx, b, e);
    }
    for (int t = 0; t < nt; ++t)
        if (started[t]) pthread_join(th[t], NULL);
}

/* ---------------------------------------------------------------- ops -- */

/* GatherRows, MatrixLibrary/MatrixBase_Functions.h:203-242: out row r = src
 * row (uint32)idx[r]; ids are floats in the reference and are truncated. */
void oracle_gather_rows(float* out, const float* src, const float* idx, uint32_t rows, uint32_t width)
{
    for (uint32_t r = 0; r < rows; ++r)
        memcpy(out + (uint64_t)r * width, src + (uint64_t)((uint32_t)idx[r]) * width, sizeof(float) * width);
}

/* Add, MatrixBase_Functions.h:471-479. */
void oracle_add(float* out, const float* a, const float* b, uint64_t n)
{
    for (uint64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* LayerNormOp, MatrixBase_Functions.h:482-549: sequential mean, sequential
 * biased variance, invStd = 1/sqrt(var + eps), y = xhat*gamma + beta (beta 0
 * when absent). */
void oracle_layernorm(float* out, const float* in, const float* gamma, const float* beta,
                      uint32_t rows, uint32_t cols, float eps)
{
    const float invCols = 1.0f / (float)cols;
    for (uint32_t r = 0; r < rows; ++r)
    {
        const float* x = in + (uint64_t)r * cols;
        float* y = out + (uint64_t)r * cols;
        float mean = 0.0f;
        for (uint32_t c = 0; c < cols; ++c) mean += x[c];
        mean *= invCols;
        float var = 0.0f;
        for (uint32_t c = 0; c < cols; ++c) { const float df = x[c] - mean; var = MAC(var, df, df); }
        const float invStd = 1.0f / sqrtf(fmaf(var, invCols, eps));
        for (uint32_t c = 0; c < cols; ++c)
        {
            const float nrm = (x[c] - mean) * invStd;
            y[c] = fmaf(nrm, gamma[c], beta ? beta[c] : 0.0f);
        }
    }
}

/* GeluMat, MatrixBase_Functions.h:989-1000 (exact erf). */
void oracle_gelu(float* out, const float* in, uint64_t n)
{
    const float rs2 = sqrtf(2.0f);
    for (uint64_t i = 0; i < n; ++i)
    {
        const float x = in[i];
        out[i] = 0.5f * x * (1.0f + erff(x / rs2));
    }
}

/* Softmax, MatrixBase_Functions.h:50-80: row max, exp(x - max), sequential
 * sum, then division by the sum. */
void oracle_softmax(float* out, const float* in, uint32_t rows, uint32_t cols)
{
    for (uint32_t r = 0; r < rows; ++r)
    {
        const float* x = in + (uint64_t)r * cols;
        float* y = out + (uint64_t)r * cols;
        float mx = x[0];
        for (uint32_t c = 1; c < cols; ++c) mx = x[c] > mx ? x[c] : mx;
        float sum = 0.0f;
        for (uint32_t c = 0; c < cols; ++c) { const float v = expf(x[c] - mx); y[c] = v; sum += v; }
        for (uint32_t c = 0; c < cols; ++c) y[c] /= sum;
    }
}

/* ScaleAdd(out, in, Mat* scale, add), MatrixBase_Functions.h:1044-1060:
 * out = in*scale + add. */
void oracle_scale_add(float* out, const float* in, float scale, const float* add, uint64_t n)
{
    for (uint64_t i = 0; i < n; ++i) out[i] = fmaf(in[i], scale, add[i]);
}

/* Generic strided product with the reference's accumulation order:
 * C[i,j] = sum_k A(i,k) B(k,j), k ascending from 0, one fp32 accumulator
 * (MulBlock, MatrixBase_Mul.h:478-589; MulStridedBlock :244-381; MulStrided
 * :88-150; MulNoDynamicAlloc :37-86 -- all sum k in order).
 * transB: B(k,j) = B[j*ldb + k] (TransposeMode::Right), else B[k*ldb + j].
 * Rows of A/C are split across threads; the per-element order is unchanged. */
typedef struct
{
    const float* A; uint64_t lda;
    const float* B; uint64_t ldb;
    float* Cm; uint64_t ldc;
    uint32_t N, K;
    int transB;
} gemm_ctx;

static void gemm_rows(void* p, uint32_t i0, uint32_t i1)
{
    gemm_ctx* g = (gemm_ctx*)p;
    const uint32_t N = g->N, K = g->K;
    if (!g->transB)
    {
        for (uint32_t i = i0; i < i1; ++i)
        {
            float* c = g->Cm + (uint64_t)i * g->ldc;
            const float* a = g->A + (uint64_t)i * g->lda;
            for (uint32_t j = 0; j < N; ++j) c[j] = 0.0f;
            for (uint32_t k = 0; k < K; ++k)
            {
                const float av = a[k];
                const float* b = g->B + (uint64_t)k * g->ldb;
                for (uint32_t j = 0; j < N; ++j) c[j] = MAC(c[j], av, b[j]);
            }
        }
    }
    else
    {
        for (uint32_t i = i0; i < i1; ++i)
        {
            float* c = g->Cm + (uint64_t)i * g->ldc;
            const float* a = g->A + (uint64_t)i * g->lda;
            for (uint32_t j = 0; j < N; ++j)
            {
                const float* b = g->B + (uint64_t)j * g->ldb;
                float s = 0.0f;
                for (uint32_t k = 0; k < K; ++k) s = MAC(s, a[k], b[k]);
                c[j] = s;
            }
        }
    }
}

/* Mul<None|Right>(out[M x N], L[M x K], R), MatrixBase_Mul.h:591-615.
 * mode 0 = None (R is K x N), 1 = Right (R is N x K). */
void oracle_mul(float* out, const float* L, const float* R, uint32_t M, uint32_t N, uint32_t K, int mode)
{
    gemm_ctx g = {L, K, R, mode ? K : N, out, N, N, K, mode};
    parallel_rows(gemm_rows, &g, M);
}

/* MatMul_Strided<None|Right> for one z plane, MatrixBase_Mul.h:617-722,
 * with column strides 1 (the only form the attention layer uses):
 * out[i*ors + j] = sum_k L[i*lrs + k] * (Right ? R[j*rrs + k] : R[k*rrs + j]). */
void oracle_matmul_strided(float* out, const float* L, const float* R,
                           uint32_t M, uint32_t N, uint32_t K,
                           uint32_t lrs, uint32_t rrs, uint32_t ors, int mode)
{
    gemm_ctx g = {L, lrs, R, rrs, out, ors, N, K, mode};
    gemm_rows(&g, 0, M);
}

/* SplitQKV, MatrixBase_Functions.h:330-367. */
void oracle_split_qkv(float* q, float* k, float* v, const float* packed, uint32_t rows, uint32_t d)
{
    for (uint32_t r = 0; r < rows; ++r)
    {
        memcpy(q + (uint64_t)r * d, packed + (uint64_t)r * 3 * d, sizeof(float) * d);
        memcpy(k + (uint64_t)r * d, packed + (uint64_t)r * 3 * d + d, sizeof(float) * d);
        memcpy(v + (uint64_t)r * d, packed + (uint64_t)r * 3 * d + 2 * d, sizeof(float) * d);
    }
}

/* -------------------------------------------------------------- model -- */

typedef struct
{
    const float* qkv; /* T x 3d, q|k|v per row */
    float* y;         /* T x d */
    float* scratch;   /* per head T x T, H planes */
    uint32_t T, d, H, hd;
    float scale;
} attn_ctx;

/* One head of CausalSelfAttentionLayer::Forward (CausalSelfAttentionLayer.h:
 * 424-499): scores = Q_h K_h^T (MatMul_Strided<Right>), ScaleAdd with the
 * 0/-inf lower-triangular mask, Softmax, dropout p=0 (a copy), then
 * Y_h = P V_h (MatMul_Strided<None>) into column block h of Y. */
static void attn_heads(void* p, uint32_t h0, uint32_t h1)
{
    attn_ctx* a = (attn_ctx*)p;
    const uint32_t T = a->T, d = a->d, hd = a->hd;
    for (uint32_t h = h0; h < h1; ++h)
    {
        float* S = a->scratch + (uint64_t)h * T * T;
        const float* Q = a->qkv + (uint64_t)h * hd;
        const float* K = a->qkv + d + (uint64_t)h * hd;
        const float* Vv = a->qkv + 2 * (uint64_t)d + (uint64_t)h * hd;
        gemm_ctx g = {Q, 3 * (uint64_t)d, K, 3 * (uint64_t)d, S, T, T, hd, 1};
        gemm_rows(&g, 0, T);
        for (uint32_t i = 0; i < T; ++i)
            for (uint32_t j = 0; j < T; ++j)
            {
                const float m = j <= i ? 0.0f : -INFINITY;
                S[(uint64_t)i * T + j] = fmaf(S[(uint64_t)i * T + j], a->scale, m);
            }
        oracle_softmax(S, S, T, T);
        gemm_ctx g2 = {S, T, Vv, 3 * (uint64_t)d, a->y + (uint64_t)h * hd, d, hd, T, 0};
        gemm_rows(&g2, 0, T);
    }
}

/* Full NanoLLM forward over a T-token window (T <= C), following the layer
 * order of Model::Run (Model.h:780-788) for the graph of NanoLLM.cpp:268-358.
 * Row t of the output depends on tokens 0..t only, so a window shorter than
 * block_size gives the same rows as the reference's zero-padded C window.
 * Logits are produced for rows [row0, row0 + nrows) into out[nrows x V]. */
int oracle_forward(const oracle_cfg* c, const float* w, const uint32_t* tokens, uint32_t T,
                   uint32_t row0, uint32_t nrows, float* out)
{
    const uint32_t V = c->V, d = c->d, H = c->H, L = c->L;
    if (T == 0 || T > c->C || d % H || row0 + nrows > T) return -1;
    const uint32_t hd = d / H;
    const uint64_t Td = (uint64_t)T * d;
    float* x = (float*)malloc(sizeof(float) * Td);
    float* buf = (float*)malloc(sizeof(float) * Td);
    float* ln = (float*)malloc(sizeof(float) * Td);
    float* qkv = (float*)malloc(sizeof(float) * Td * 3);
    float* yat = (float*)malloc(sizeof(float) * Td);
    float* prj = (float*)malloc(sizeof(float) * Td);
    float* hid = (float*)malloc(sizeof(float) * Td * 4);
    float* sc = (float*)malloc(sizeof(float) * (uint64_t)H * T * T);
    float* tmp = (float*)malloc(sizeof(float) * Td);
    float* ids = (float*)malloc(sizeof(float) * T);
    if (!x || !buf || !ln || !qkv || !yat || !prj || !hid || !sc || !tmp || !ids) return -2;

    const float* tok = w;
    const float* pos = tok + (uint64_t)V * d;
    const float* p = pos + (uint64_t)c->C * d;

    /* embedding_token / embedding_pos GatherRows, token_pos_add Add,
     * embedding_dropout copy (Embedding.h:161-170, AddLayer.h:149,
     * DropoutLayer.h:125-150) */
    for (uint32_t t = 0; t < T; ++t) ids[t] = (float)tokens[t];
    oracle_gather_rows(tmp, tok, ids, T, d);
    for (uint32_t t = 0; t < T; ++t) ids[t] = (float)t;
    oracle_gather_rows(buf, pos, ids, T, d);
    oracle_add(x, tmp, buf, Td);

    const float scale = 1.0f / sqrtf((float)hd);
    for (uint32_t l = 0; l < L; ++l)
    {
        const float* g0 = p; p += d;
        const float* wqkv = p; p += 3 * (uint64_t)d * d;
        const float* wprj = p; p += (uint64_t)d * d;
        const float* g1 = p; p += d;
        const float* wfc = p; p += 4 * (uint64_t)d * d;
        const float* wmlp = p; p += 4 * (uint64_t)d * d;
        /* TransformerBlock.h:355-401 */
        oracle_layernorm(ln, x, g0, NULL, T, d, 1e-5f);
        oracle_mul(qkv, ln, wqkv, T, 3 * d, d, 0);
        attn_ctx a = {qkv, yat, sc, T, d, H, hd, scale};
        parallel_rows(attn_heads, &a, H);
        oracle_mul(prj, yat, wprj, T, d, d, 1);
        oracle_add(buf, x, prj, Td);
        oracle_layernorm(ln, buf, g1, NULL, T, d, 1e-5f);
        oracle_mul(hid, ln, wfc, T, 4 * d, d, 0);
        oracle_gelu(hid, hid, Td * 4);
        oracle_mul(prj, hid, wmlp, T, d, 4 * d, 0);
        oracle_add(x, buf, prj, Td);
    }
    /* ln_f, ln_f_flatten (a copy), lm_head Mul<Right> against the tied token
     * table (NanoLLM.cpp:315-348, Dense.h:203). */
    oracle_layernorm(ln, x, p, NULL, T, d, 1e-5f);
    oracle_mul(out, ln + (uint64_t)row0 * d, tok, nrows, V, d, 1);

    free(x); free(buf); free(ln); free(qkv); free(yat); free(prj); free(hid); free(sc); free(tmp); free(ids);
    return 0;
}

/* argmax with the reference's tie rule: strict '>' keeps the first maximum
 * (Examples/NanoLLM/NanoLLM.cpp:194-201). */
uint32_t oracle_argmax(const float* row, uint32_t n)
{
    uint32_t best = 0;
    float bv = row[0];
    for (uint32_t v = 1; v < n; ++v)
        if (row[v] > bv) { bv = row[v]; best = v; }
    return best;
}

/* The reference greedy loop (one full forward per generated token, argmax of
 * row plen+step-1).  tokens_out holds plen + nnew ids, logits_out nnew x V. */
int oracle_greedy(const oracle_cfg* c, const float* w, const uint32_t* prompt, uint32_t plen,
                  uint32_t nnew, uint32_t* tokens_out, float* logits_out)
{
    if (plen == 0 || plen + nnew > c->C) return -1;
    memcpy(tokens_out, prompt, sizeof(uint32_t) * plen);
    for (uint32_t s = 0; s < nnew; ++s)
    {
        const uint32_t T = plen + s;
        float* row = logits_out + (uint64_t)s * c->V;
        int rc = oracle_forward(c, w, tokens_out, T, T - 1, 1, row);
        if (rc) return rc;
        tokens_out[T] = oracle_argmax(row, c->V);
    }
    return 0;
}
