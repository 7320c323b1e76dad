// The decode engine: FreeML's NanoLLM token loop (Examples/NanoLLM/NanoLLM.cpp:
// 268-358 graph, Model::Run at ModelLibrary/Model.h:764-788, argmax at
// NanoLLM.cpp:189-204) rebuilt as a KV-cached, batched greedy loop on B200.
//
// Per generated token the reference recomputes the whole block_size window.
// Causality makes row t of that window depend on tokens 0..t only
// (CausalSelfAttentionLayer.h:66-67 mask; LayerNorm, Dense, Gelu and Add are
// row-wise), so the engine keeps each layer's K and V rows and computes only
// the new row: the logits are the reference's row t up to fp32 rounding.
//
// HBM layout (fp32):
//   weights, K-contiguous ("n-major": row n holds the n-th output's inputs)
//     tok     [V x d]      token table; also the tied lm_head rows
//     pos     [C x d]      position table
//     wqkv_t  [L][3d x d]  transpose of Dense_Weights [d x 3d]
//     wproj   [L][d x d]   Dense_Weights as stored (out x in)
//     wfc_t   [L][4d x d]  transpose of [d x 4d]
//     wmlp_t  [L][d x 4d]  transpose of [4d x d]
//     ln0, ln1 [L][d], lnf [d]
//   KV cache  kc, vc [L][B][H][C][hd]: one head's rows are contiguous, so a
//     split of the attention reads one dense block.
//   state     pending[B] (token to consume), pos[B] (rows held), keys[B]
//     (packed argmax), split partials + counters for attention.
//
// One decode step (B rows), every kernel reading positions and tokens from
// device memory so that one captured CUDA graph replays for every step:
//   embed -> L x { layernorm -> qkv gemv (q + K/V-cache scatter) ->
//   attention (split-KV, last CTA combines) -> proj gemv (+residual) ->
//   layernorm -> fc gemv (+gelu) -> mlp gemv (+residual) } -> layernorm ->
//   lm_head gemv (+argmax keys) -> finalize
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <utility>
#include <vector>

#include <cuda_bf16.h>
#include <nccl.h>

#include "attention.cuh"
#include "fml_common.cuh"

#ifdef FML_TIMELINE
// debug builds only: bind (buf, cap) as the kernels' timeline ring, this
// unit's kernels in the first half and the attention unit's in the second
extern "C" __attribute__((visibility("default"))) int fml_debug_timeline(void* buf, uint32_t cap)
{
    fml::TimelineRec* p = static_cast<fml::TimelineRec*>(buf);
    const uint32_t half = cap / 2;
    if (fml::timeline_bind_unit(p, half)) return 2;
    return fml::timeline_bind_attention(p ? p + half : nullptr, cap - half);
}
#endif

namespace fml {

int launch_layernorm(float* out, const float* in, const float* gamma, const float* beta, float* xhat, uint32_t rows,
                     uint32_t cols, uint64_t in_stride, uint64_t out_stride, float eps, cudaStream_t st);
int gemm_f32(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, bool trans_b,
             int batch, uint64_t pa, uint64_t pb, uint64_t pc, cudaStream_t st);
int gemm_tc(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, bool split3,
            int epi, const float* R, cudaStream_t st, const float* B_lo = nullptr);
int gemm_tc_qkv(float* q, int ldq, float* kc, float* vc, uint64_t seq_stride, int P, int hd, int ctx,
                const float* A, const float* B, int M, int dq, int K, bool split3, cudaStream_t st,
                const float* B_lo = nullptr);
int tf32_lo(float* lo, const float* x, uint64_t n, cudaStream_t st);
int gemm_tc_prepare(bool split3, int epi, bool blo = false);
int gemm_tc_splitk(float* part, const float* A, const float* B, int M, int N, int K, int lda, int ldb, bool split3,
                   int ksplit, cudaStream_t st, const float* B_lo = nullptr, bool pdl = false);
int gemv_nt(float* y, const float* x, const float* w, uint32_t M, uint32_t N, uint32_t K, cudaStream_t st);
int launch_prefill_attention(const float* q, uint32_t ldq, const float* kc, const float* vc, uint64_t seq_stride,
                             uint32_t C, float* out, uint32_t ldo, uint32_t B, uint32_t H, uint32_t P, uint32_t hd,
                             float scale, cudaStream_t st);
int launch_prefill_attention_tc(const float* q, uint32_t ldq, const float* kc, const float* vc, uint64_t seq_stride,
                                uint32_t C, float* out, uint32_t ldo, uint32_t B, uint32_t H, uint32_t P, uint32_t hd,
                                float scale, bool split3, cudaStream_t st);

// ---------------------------------------------------------------- kernels --

// Embedding GatherRows x2 + AddLayer (Embedding.h:161-170, AddLayer.h:149):
// x[r] = tok[id] + pos[t].  Decode: r = sequence b, id = pending[b],
// t = pos[b].  Prefill: r = b*P + t, id = prompt[r].
__global__ void embed_kernel(float* __restrict__ x, const float* __restrict__ tok, const float* __restrict__ posemb,
                             const uint32_t* __restrict__ ids, const uint32_t* __restrict__ pos, uint32_t rows,
                             uint32_t P, uint32_t d, uint32_t V, uint32_t C, uint32_t* zero, uint32_t nzero,
                             StepStamp stamp)
{
    FML_TIMELINE_SCOPE(1);
    const StampAtExit stamp_at_exit(stamp);
    griddep_launch_dependents();
    griddep_wait();
    FML_TIMELINE_MARK(1);
    // the step's first kernel clears the per-layer attention work counters
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0u;
    for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x)
    {
        const uint32_t t = pos ? pos[r] : r % P;
        uint32_t id = ids[r];
        const bool ok = id < V && t < C;
        if (!ok) id = 0;
        const float4* a = reinterpret_cast<const float4*>(tok + (uint64_t)id * d);
        const float4* b = reinterpret_cast<const float4*>(posemb + (uint64_t)(ok ? t : 0) * d);
        float4* o = reinterpret_cast<float4*>(x + (uint64_t)r * d);
        for (uint32_t c = threadIdx.x; c < d / 4; c += blockDim.x)
        {
            const float4 u = a[c], v = b[c];
            o[c] = ok ? make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w) : make_float4(0, 0, 0, 0);
        }
    }
}

enum GemvEpi { EPI_STORE = 0, EPI_GELU = 1, EPI_RESID = 2, EPI_QKV = 3, EPI_ARGMAX = 4 };

// One-shot all-reduce over NVLink peer memory (tensor parallel decode).
constexpr uint32_t AR_CTAS = 16;  // CTAs of the all-reduce kernel = flags per rank
constexpr uint64_t AR_WAIT_NS = 1000000000ull;
__device__ unsigned int g_tp_timeouts = 0;

// Flag tags of the one-shot all-reduce.  A step holds `nslot` all-reduces
// (2 per layer); use `slot` of step `epoch` raises every flag to
// epoch * nslot + slot + 1, so consecutive uses count up by one, modulo 2^32.
// A waiter passes once the flag has reached its tag, compared through the
// signed difference so the test holds across the 2^32 wrap (flags never lag
// a tag by 2^31 uses: every rank finishes use u before any starts u + 2).
__host__ __device__ __forceinline__ uint32_t ar_tag(uint32_t epoch, uint32_t slot, uint32_t nslot)
{
    return epoch * nslot + slot + 1u;
}
__host__ __device__ __forceinline__ bool ar_flag_reached(uint32_t flag, uint32_t tag)
{
    return (int32_t)(flag - tag) >= 0;
}

// Weight stream load: each weight is read once per step, so it bypasses L1
// and leaves L1 to the activation rows that every column group re-reads
// (measured: +4 % decode tokens/s on config 5, where the activation rows are
// 128 KB per CTA).
__device__ __forceinline__ float4 ldw(const float* p)
{
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// Eight bf16 weights packed in a 16-byte load (element i in bits
// [16 (i % 2), 16 (i % 2) + 16) of word i / 2), widened to fp32 exactly.
__device__ __forceinline__ void bf16x8_to_f32(const float4& w, float (&f)[8])
{
    const uint32_t u[4] = {__float_as_uint(w.x), __float_as_uint(w.y), __float_as_uint(w.z), __float_as_uint(w.w)};
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        f[2 * i] = __uint_as_float(u[i] << 16);
        f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
}

struct GemvArgs
{
    const float* x;  // [M x K], row stride ldx
    const float* w;  // [N x K]
    const uint16_t* wb;  // the same weights as bf16 (read instead of w by the WB kernels)
    uint32_t M, N, K, ldx;
    float* y;        // [M x N], row stride ldy
    uint32_t ldy;
    const float* r;  // residual [M x N], row stride ldr (EPI_RESID)
    uint32_t ldr;
    // EPI_QKV: columns [0,d) -> q[m*d + n], [d,2d) -> K cache, [2d,3d) -> V cache
    float* q;
    float* kc;
    float* vc;
    const uint32_t* pos;
    uint32_t d, H, hd, C;
    uint64_t seq_stride;  // H*C*hd: one sequence's block inside a layer
    // EPI_ARGMAX
    unsigned long long* keys;
    uint32_t n_off;  // global index of output column 0 (vocabulary-parallel lm_head)

    // LN prologue: gamma [K] (beta absent, NanoLLM's use_bias = false)
    const float* gamma;
    // split-K reduction with a LayerNorm of the finished rows: ln_out [M x N]
    // (row stride N) = LayerNormOp(y) with ln_gamma
    float* ln_out;
    const float* ln_gamma;
    StepStamp stamp;  // optional completion stamp
};

// y[m, n] = sum_k xn[m, k] W[n, k] for the small-M (decode) shapes, where
// xn = x, or LayerNormOp(x) with gamma (LN = true: LayerNorm.h:148-165 fused
// into the consumer -- every CTA recomputes the two-pass statistics of its
// rows, so no separate LayerNorm launch and no cross-CTA reduction).
//
// CTA = 4 warps, 4 output columns n, MT rows m.  The 128 threads partition K
// in float4 slices (thread t owns k = 4t + 512i), so each W element is read
// once per step and every load of an iteration is issued before any use.
// The CTA's first W slice is loaded before griddepcontrol.wait: with
// programmatic dependent launch it streams in while the previous kernel
// finishes.  Partial sums are combined by a warp transpose-reduce (each lane
// ends up owning distinct outputs) and a 4-way shared-memory sum; the
// epilogue runs on one thread per output.
template <int MT, int EPI, bool LN, bool WB>
__global__ void __launch_bounds__(128) gemv_kernel(GemvArgs a)
{
    FML_TIMELINE_SCOPE(10 + EPI);
    const StampAtExit stamp_at_exit(a.stamp);
    constexpr int NW = 4;
    constexpr uint32_t KV = WB ? 8u : 4u;  // k values per 16-byte W load
    constexpr uint32_t KSTEP = 128u * KV;  // k the CTA covers per iteration
    constexpr int CNT = MT * NW;
    constexpr int R = CNT >= 32 ? CNT / 32 : 1;
    constexpr int RM = MT >= 32 ? MT / 32 : 1;
    __shared__ float red[4][CNT];
    __shared__ float s_part[4][MT];
    __shared__ float s_mean[MT], s_rstd[MT];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t n0 = blockIdx.y * NW;
    const uint32_t m0 = blockIdx.x * MT;
    const uint32_t k_first = (uint32_t)tid * 4u;    // x rows (LayerNorm statistics; fp32 W slice)
    const uint32_t kw_first = (uint32_t)tid * KV;   // this thread's W slice
    // W rows: fp32 (a.w) or bf16 (a.wb) elements
    using WT = std::conditional_t<WB, uint16_t, float>;
    const WT* wbase = WB ? reinterpret_cast<const WT*>(a.wb) : reinterpret_cast<const WT*>(a.w);
    auto wptr = [](const WT* row, uint32_t k) { return reinterpret_cast<const float*>(row + k); };

    const WT* wrow[NW];
#pragma unroll
    for (int j = 0; j < NW; ++j) wrow[j] = wbase + (uint64_t)min(blockIdx.y * NW + j, a.N - 1) * a.K;
    // row pointers clamped into range: loads stay unconditional and in bounds
    const float* xrow[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) xrow[m] = a.x + (uint64_t)min(m0 + m, a.M - 1) * a.ldx;

    float4 wv[NW];
    const bool have_first = kw_first < a.K;
#pragma unroll
    for (int j = 0; j < NW; ++j)
        wv[j] = have_first ? ldw(wptr(wrow[j], kw_first)) : make_float4(0, 0, 0, 0);

    griddep_launch_dependents();
    griddep_wait();
    FML_TIMELINE_MARK(1);

    if constexpr (LN)
    {
        // two-pass mean / biased variance per row, like LayerNormOp
        float ps[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) ps[m] = 0.0f;
        for (uint32_t k = k_first; k < a.K; k += 512u)
        {
#pragma unroll
            for (int m = 0; m < MT; ++m)
            {
                const float4 xv = *reinterpret_cast<const float4*>(xrow[m] + k);
                ps[m] += (xv.x + xv.y) + (xv.z + xv.w);
            }
        }
        warp_transpose_reduce<MT>(ps, lane);
        if (reduce_owner<MT>(lane))
        {
            const int base = reduce_base<MT>(lane);
#pragma unroll
            for (int i = 0; i < RM; ++i) s_part[warp][base + i] = ps[i];
        }
        __syncthreads();
        const float invK = 1.0f / (float)a.K;
        if (tid < MT) s_mean[tid] = (s_part[0][tid] + s_part[1][tid] + s_part[2][tid] + s_part[3][tid]) * invK;
        __syncthreads();
        float mean[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) { mean[m] = s_mean[m]; ps[m] = 0.0f; }
        for (uint32_t k = k_first; k < a.K; k += 512u)
        {
#pragma unroll
            for (int m = 0; m < MT; ++m)
            {
                const float4 xv = *reinterpret_cast<const float4*>(xrow[m] + k);
                const float d0 = xv.x - mean[m], d1 = xv.y - mean[m], d2 = xv.z - mean[m], d3 = xv.w - mean[m];
                ps[m] = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, ps[m]))));
            }
        }
        warp_transpose_reduce<MT>(ps, lane);
        __syncthreads();  // s_part reuse
        if (reduce_owner<MT>(lane))
        {
            const int base = reduce_base<MT>(lane);
#pragma unroll
            for (int i = 0; i < RM; ++i) s_part[warp][base + i] = ps[i];
        }
        __syncthreads();
        if (tid < MT)
        {
            const float var = s_part[0][tid] + s_part[1][tid] + s_part[2][tid] + s_part[3][tid];
            s_rstd[tid] = 1.0f / sqrtf(fmaf(var, invK, 1e-5f));
        }
        __syncthreads();
    }

    FML_TIMELINE_MARK(2);
    // column groups of this CTA: n0 = 4 * (blockIdx.y + i * gridDim.y)
    const uint32_t ngroups = (a.N + NW - 1) / NW;
    for (uint32_t g = blockIdx.y; g < ngroups; g += gridDim.y)
    {
        const uint32_t n0 = g * NW;
        const uint32_t gnext = g + gridDim.y;
        float acc[CNT];
#pragma unroll
        for (int i = 0; i < CNT; ++i) acc[i] = 0.0f;

        // the W slice for the next k is requested as soon as this one is used
        if constexpr (WB)
        {
            for (uint32_t k = kw_first; k < a.K; k += KSTEP)
            {
                float4 xv[MT][2];  // x[m][k .. k + 7]
#pragma unroll
                for (int m = 0; m < MT; ++m)
#pragma unroll
                    for (int q = 0; q < 2; ++q) xv[m][q] = *reinterpret_cast<const float4*>(xrow[m] + k + 4 * q);
                if constexpr (LN)
                {
#pragma unroll
                    for (int q = 0; q < 2; ++q)
                    {
                        const float4 gm = *reinterpret_cast<const float4*>(a.gamma + k + 4 * q);
#pragma unroll
                        for (int m = 0; m < MT; ++m)
                        {
                            const float mu = s_mean[m], rs = s_rstd[m];
                            xv[m][q].x = (xv[m][q].x - mu) * rs * gm.x;
                            xv[m][q].y = (xv[m][q].y - mu) * rs * gm.y;
                            xv[m][q].z = (xv[m][q].z - mu) * rs * gm.z;
                            xv[m][q].w = (xv[m][q].w - mu) * rs * gm.w;
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < NW; ++j)
                {
                    float wf[8];
                    bf16x8_to_f32(wv[j], wf);
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                    {
                        float sacc = acc[m * NW + j];
#pragma unroll
                        for (int q = 0; q < 2; ++q)
                        {
                            sacc = fmaf(xv[m][q].x, wf[4 * q + 0], sacc);
                            sacc = fmaf(xv[m][q].y, wf[4 * q + 1], sacc);
                            sacc = fmaf(xv[m][q].z, wf[4 * q + 2], sacc);
                            sacc = fmaf(xv[m][q].w, wf[4 * q + 3], sacc);
                        }
                        acc[m * NW + j] = sacc;
                    }
                }
                if (k + KSTEP < a.K)
                {
#pragma unroll
                    for (int j = 0; j < NW; ++j) wv[j] = ldw(wptr(wrow[j], k + KSTEP));
                }
            }
        }
        else
        {
            for (uint32_t k = k_first; k < a.K; k += 512u)
            {
                float4 xv[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m) xv[m] = *reinterpret_cast<const float4*>(xrow[m] + k);
                if constexpr (LN)
                {
                    const float4 gm = *reinterpret_cast<const float4*>(a.gamma + k);
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                    {
                        const float mu = s_mean[m], rs = s_rstd[m];
                        xv[m].x = (xv[m].x - mu) * rs * gm.x;
                        xv[m].y = (xv[m].y - mu) * rs * gm.y;
                        xv[m].z = (xv[m].z - mu) * rs * gm.z;
                        xv[m].w = (xv[m].w - mu) * rs * gm.w;
                    }
                }
#pragma unroll
                for (int m = 0; m < MT; ++m)
                {
#pragma unroll
                    for (int j = 0; j < NW; ++j)
                    {
                        float sacc = acc[m * NW + j];
                        sacc = fmaf(xv[m].x, wv[j].x, sacc);
                        sacc = fmaf(xv[m].y, wv[j].y, sacc);
                        sacc = fmaf(xv[m].z, wv[j].z, sacc);
                        sacc = fmaf(xv[m].w, wv[j].w, sacc);
                        acc[m * NW + j] = sacc;
                    }
                }
                if (k + 512u < a.K)
                {
#pragma unroll
                    for (int j = 0; j < NW; ++j) wv[j] = ldw(wptr(wrow[j], k + 512u));
                }
            }
        }

        // prefetch the next group's first W slice while this one is reduced
        if (gnext < ngroups)
        {
#pragma unroll
            for (int j = 0; j < NW; ++j)
            {
                wrow[j] = wbase + (uint64_t)min(gnext * NW + j, a.N - 1) * a.K;
                wv[j] = have_first ? ldw(wptr(wrow[j], kw_first)) : make_float4(0, 0, 0, 0);
            }
        }

        warp_transpose_reduce<CNT>(acc, lane);
        __syncthreads();  // red[] of the previous group has been consumed
        if (reduce_owner<CNT>(lane))
        {
            const int base = reduce_base<CNT>(lane);
#pragma unroll
            for (int i = 0; i < R; ++i) red[warp][base + i] = acc[i];
        }
        __syncthreads();

        const int t = threadIdx.x;
        if (t < CNT || EPI == EPI_ARGMAX)
        {
            const int tt = t < CNT ? t : 0;
            const float v = red[0][tt] + red[1][tt] + red[2][tt] + red[3][tt];
            const uint32_t m = m0 + tt / NW, n = n0 + tt % NW;
            const bool valid = t < CNT && m < a.M && n < a.N;
            if constexpr (EPI == EPI_STORE)
            {
                if (valid) a.y[(uint64_t)m * a.ldy + n] = v;
            }
            else if constexpr (EPI == EPI_GELU)
            {
                if (valid) a.y[(uint64_t)m * a.ldy + n] = gelu_exact(v);
            }
            else if constexpr (EPI == EPI_RESID)
            {
                if (valid) a.y[(uint64_t)m * a.ldy + n] = a.r[(uint64_t)m * a.ldr + n] + v;
            }
            else if constexpr (EPI == EPI_QKV)
            {
                if (valid)
                {
                    if (n < a.d) a.q[(uint64_t)m * a.d + n] = v;
                    else
                    {
                        const uint32_t c = n % a.d, h = c / a.hd, e = c % a.hd;
                        float* cache = n < 2 * a.d ? a.kc : a.vc;
                        cache[(uint64_t)m * a.seq_stride + ((uint64_t)h * a.C + a.pos[m]) * a.hd + e] = v;
                    }
                }
            }
            else if constexpr (EPI == EPI_ARGMAX)
            {
                // logits (optional) and the per-row argmax over these 4
                // columns, folded into the row's global key with one atomicMax
                if (valid && a.y) a.y[(uint64_t)m * a.ldy + n] = v;
                if (t < 32 * ((CNT + 31) / 32))
                {
                    unsigned long long key = valid ? argmax_key(v, n + a.n_off) : 0ull;
                    unsigned long long o1 = __shfl_xor_sync(FULL_MASK, key, 1);
                    key = o1 > key ? o1 : key;
                    unsigned long long o2 = __shfl_xor_sync(FULL_MASK, key, 2);
                    key = o2 > key ? o2 : key;
                    if (valid && (t % NW) == 0) atomicMax(a.keys + m, key);
                }
            }
        }
    }

}

// Named barrier over `n` threads (a team of warps inside the CTA).
__device__ __forceinline__ void team_sync(uint32_t id, uint32_t n)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

#ifndef FML_GEMV_SB
#define FML_GEMV_SB 4
#endif
// packed fp32 FMA (fma.rn.f32x2, two products per instruction) with even / odd
// k partial sums: measured -1 % (32 sequences) and -4 % (8) us per decode
// step on config 3 against scalar fmaf, although the extra accumulators cost
// 3 instead of 4 resident CTAs per SM
#ifndef FML_GEMV_F2
#define FML_GEMV_F2 1
#endif

// Decode GEMV, team layout: y[m, n] = sum_k xn[m, k] W[n, k] for MT rows per
// CTA, xn = x or LayerNormOp(x) with gamma (LayerNorm.h:148-165, two-pass
// mean / biased variance).
//
// The CTA stages its MT rows of x once in shared memory, normalised in place
// when LN (warp w owns rows w, w + 4, ...), so the per-column-group work is
// only loads and fused multiply-adds.  Its 4 warps form 4 / KW teams; a team
// of KW warps owns one group of 4 output columns at a time and splits K
// between its 32 * KW lanes in float4 slices (lane k = 4 * (32 kw + lane) +
// 128 KW s), so each lane accumulates MT x 4 sums over S = K / (128 KW)
// slices before one warp transpose-reduce (and, for KW > 1, one sum of the
// team's warps through shared memory behind a named barrier).  W rows stream
// through SB register slots: a slot is refilled with the next slice of the
// group (or the next group's) as soon as it has been used, so SB slices per
// lane are always in flight; the first SB are requested before
// griddepcontrol.wait.  Measured against the one-group-per-CTA layout (every
// output a 128-thread reduction, the LayerNorm redone per column group):
// the per-group instruction count, not memory, bounded that kernel.
template <int MT, int KW, int EPI, bool LN, bool WB>
__global__ void __launch_bounds__(128) gemv_team_kernel(GemvArgs a)
{
    FML_TIMELINE_SCOPE(10 + EPI);
    const StampAtExit stamp_at_exit(a.stamp);
    constexpr int NW = 4;              // output columns per group
    constexpr int CNT = MT * NW;       // sums per lane (16 or 32)
    constexpr int TEAMS = 4 / KW;
    constexpr int SB = FML_GEMV_SB;    // W slices in flight per lane
    constexpr uint32_t KV = WB ? 8u : 4u;  // k values per 16-byte W slice (fp32 or bf16 weights)
    constexpr uint32_t KSTEP = 32u * KV * KW;  // K covered by one slice of the team
    static_assert(CNT == 16 || CNT == 32, "MT must be 4 or 8");
    extern __shared__ __align__(16) float xs[];  // [MT][K] x rows, then (LN) gamma [K]
    __shared__ float red[2][TEAMS][KW][CNT];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int team = warp / KW, kw = warp % KW;
    const uint32_t m0 = blockIdx.x * MT;
    const uint32_t K = a.K;
    const uint32_t k_lane = KV * (32u * kw + lane);
    const uint32_t S = (K + KSTEP - 1) / KSTEP;          // slices per lane
    const uint32_t nchunk = (S + SB - 1) / SB;
    const uint32_t ngroups = (a.N + NW - 1) / NW;
    const uint32_t gstride = gridDim.y * TEAMS;
    uint32_t g = blockIdx.y * TEAMS + team;

    // slice (group gg, slice s) of this lane: NW float4 of W, zero past K or
    // past the last group
    float4 wv[SB][NW];
    auto load_slot = [&](int b, uint32_t gg, uint32_t s) {
        const uint32_t k = k_lane + s * KSTEP;
        const bool ok = gg < ngroups && s < S && k < K;
#pragma unroll
        for (int j = 0; j < NW; ++j)
        {
            if constexpr (WB)
                wv[b][j] = ok ? ldw(reinterpret_cast<const float*>(a.wb + (uint64_t)min(gg * NW + j, a.N - 1) * K + k))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
            else
                wv[b][j] = ok ? ldw(a.w + (uint64_t)min(gg * NW + j, a.N - 1) * K + k)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
#pragma unroll
    for (int b = 0; b < SB; ++b) load_slot(b, g, b);

    // gamma is a weight: staged before the wait (after the x rows in shared
    // memory); every warp reads all of it, so a barrier follows
    const float4* gs4 = reinterpret_cast<const float4*>(xs + (uint64_t)MT * K);
    if constexpr (LN)
    {
        const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
        for (uint32_t c = tid; c < K / 4; c += 128) const_cast<float4*>(gs4)[c] = g4[c];
        __syncthreads();
    }

    griddep_launch_dependents();
    griddep_wait();
    FML_TIMELINE_MARK(1);

    // warp w stages rows w, w + 4, ... (zero past M) and, for LN, normalises
    // them in place; a lane only rereads the float4s it wrote itself
    const float invK = 1.0f / (float)K;
    for (int m = warp; m < MT; m += 4)
    {
        const bool in = m0 + m < a.M;
        const float4* src = reinterpret_cast<const float4*>(a.x + (uint64_t)(in ? m0 + m : 0) * a.ldx);
        float4* row = reinterpret_cast<float4*>(xs + (uint64_t)m * K);
        float sum = 0.f;
        // the row's loads are all requested before the first is used (at
        // most 16 float4 per lane, K <= 2048): one L2 round trip, not one per
        // iteration
        {
            float4 v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
            {
                const uint32_t c = lane + 32u * i;
                v[i] = in && c < K / 4 ? src[c] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i)
            {
                const uint32_t c = lane + 32u * i;
                if (c < K / 4)
                {
                    row[c] = v[i];
                    sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
                }
            }
        }
        if constexpr (LN)
        {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL_MASK, sum, o);
            const float mean = sum * invK;
            float q = 0.f;
            for (uint32_t c = lane; c < K / 4; c += 32)
            {
                const float4 v = row[c];
                const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
                q = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, q))));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(FULL_MASK, q, o);
            const float rstd = 1.0f / sqrtf(fmaf(q, invK, 1e-5f));
            for (uint32_t c = lane; c < K / 4; c += 32)
            {
                float4 v = row[c];
                const float4 gm = gs4[c];
                v.x = (v.x - mean) * rstd * gm.x;
                v.y = (v.y - mean) * rstd * gm.y;
                v.z = (v.z - mean) * rstd * gm.z;
                v.w = (v.w - mean) * rstd * gm.w;
                row[c] = v;
            }
        }
    }
    __syncthreads();
    FML_TIMELINE_MARK(2);

    const uint32_t hd_shift = EPI == EPI_QKV ? (uint32_t)(__ffs(a.hd) - 1) : 0u;
    uint32_t parity = 0;
    // the loop runs per team; its trip count is the same for the team's warps
    for (; g < ngroups; g += gstride, parity ^= 1u)
    {
        // the residual this lane's output adds (EPI_RESID), requested now so
        // that it arrives during the group's FMAs (the previous kernels that
        // wrote it finished before griddepcontrol.wait)
        [[maybe_unused]] float rres = 0.f;
        if constexpr (EPI == EPI_RESID)
        {
            const int ridx = reduce_base<CNT>(lane);
            const uint32_t rm = m0 + ridx / NW, rn = g * NW + ridx % NW;
            if (reduce_owner<CNT>(lane) && rm < a.M && rn < a.N) rres = __ldcg(a.r + (uint64_t)rm * a.ldr + rn);
        }
#if FML_GEMV_F2
        float2 acc2[CNT];  // even / odd k partial sums, packed fp32 FMA
#pragma unroll
        for (int i = 0; i < CNT; ++i) acc2[i] = make_float2(0.0f, 0.0f);
#else
        float acc[CNT];
#pragma unroll
        for (int i = 0; i < CNT; ++i) acc[i] = 0.0f;
#endif
        for (uint32_t c = 0; c < nchunk; ++c)
        {
#pragma unroll
            for (int b = 0; b < SB; ++b)
            {
                const uint32_t s = c * SB + b;
                const uint32_t k = k_lane + s * KSTEP;
                if constexpr (WB)
                {
                  if (s < S && k < K)
                  {
                    // eight bf16 weights per slot, widened to fp32 (exactly)
                    float wf[NW][8];
#pragma unroll
                    for (int j = 0; j < NW; ++j) bf16x8_to_f32(wv[b][j], wf[j]);
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                    {
#pragma unroll
                        for (int q = 0; q < 2; ++q)
                        {
                            const float4 xv = *reinterpret_cast<const float4*>(xs + (uint64_t)m * K + k + 4 * q);
#pragma unroll
                            for (int j = 0; j < NW; ++j)
                            {
#if FML_GEMV_F2
                                float2 t = acc2[m * NW + j];
                                t = __ffma2_rn(make_float2(xv.x, xv.y), make_float2(wf[j][4 * q], wf[j][4 * q + 1]), t);
                                t = __ffma2_rn(make_float2(xv.z, xv.w), make_float2(wf[j][4 * q + 2], wf[j][4 * q + 3]),
                                               t);
                                acc2[m * NW + j] = t;
#else
                                float t = acc[m * NW + j];
                                t = fmaf(xv.x, wf[j][4 * q], t);
                                t = fmaf(xv.y, wf[j][4 * q + 1], t);
                                t = fmaf(xv.z, wf[j][4 * q + 2], t);
                                t = fmaf(xv.w, wf[j][4 * q + 3], t);
                                acc[m * NW + j] = t;
#endif
                            }
                        }
                    }
                  }
                }
                else if (s < S && k < K)
                {
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                    {
                        const float4 xv = *reinterpret_cast<const float4*>(xs + (uint64_t)m * K + k);
#pragma unroll
                        for (int j = 0; j < NW; ++j)
                        {
#if FML_GEMV_F2
                            float2 t = acc2[m * NW + j];
                            t = __ffma2_rn(make_float2(xv.x, xv.y), make_float2(wv[b][j].x, wv[b][j].y), t);
                            t = __ffma2_rn(make_float2(xv.z, xv.w), make_float2(wv[b][j].z, wv[b][j].w), t);
                            acc2[m * NW + j] = t;
#else
                            float t = acc[m * NW + j];
                            t = fmaf(xv.x, wv[b][j].x, t);
                            t = fmaf(xv.y, wv[b][j].y, t);
                            t = fmaf(xv.z, wv[b][j].z, t);
                            t = fmaf(xv.w, wv[b][j].w, t);
                            acc[m * NW + j] = t;
#endif
                        }
                    }
                }
                // refill the slot: this group's slice s + SB, else the next
                // group's slice b
                if (c + 1 < nchunk) load_slot(b, g, s + SB);
                else load_slot(b, g + gstride, b);
            }
        }

#if FML_GEMV_F2
        float acc[CNT];
#pragma unroll
        for (int i = 0; i < CNT; ++i) acc[i] = acc2[i].x + acc2[i].y;
#endif
        warp_transpose_reduce<CNT>(acc, lane);
        const int idx = reduce_base<CNT>(lane);  // the sum this lane holds
        float v = acc[0];
        if constexpr (KW > 1)
        {
            if (reduce_owner<CNT>(lane)) red[parity][team][kw][idx] = v;
            team_sync(1 + team, 32 * KW);
            if (kw != 0) continue;
            v = red[parity][team][0][idx];
#pragma unroll
            for (int i = 1; i < KW; ++i) v += red[parity][team][i][idx];
        }

        const uint32_t m = m0 + idx / NW, n = g * NW + idx % NW;
        const bool valid = reduce_owner<CNT>(lane) && m < a.M && n < a.N;
        if constexpr (EPI == EPI_STORE)
        {
            if (valid) a.y[(uint64_t)m * a.ldy + n] = v;
        }
        else if constexpr (EPI == EPI_GELU)
        {
            if (valid) a.y[(uint64_t)m * a.ldy + n] = gelu_exact(v);
        }
        else if constexpr (EPI == EPI_RESID)
        {
            if (valid) a.y[(uint64_t)m * a.ldy + n] = rres + v;
        }
        else if constexpr (EPI == EPI_QKV)
        {
            if (valid)
            {
                if (n < a.d) a.q[(uint64_t)m * a.d + n] = v;
                else
                {
                    const uint32_t cc = n < 2 * a.d ? n - a.d : n - 2 * a.d;
                    float* cache = n < 2 * a.d ? a.kc : a.vc;
                    cache[(uint64_t)m * a.seq_stride + ((uint64_t)(cc >> hd_shift) * a.C + a.pos[m]) * a.hd +
                          (cc & (a.hd - 1))] = v;
                }
            }
        }
        else if constexpr (EPI == EPI_ARGMAX)
        {
            // logits (optional), then the max key over the group's 4 columns
            // of each row: the lanes holding row m's 4 sums differ in the
            // lane bits that carry idx % 4
            if (valid && a.y) a.y[(uint64_t)m * a.ldy + n] = v;
            unsigned long long key = valid ? argmax_key(v, n + a.n_off) : 0ull;
            constexpr int sh = CNT == 16 ? 1 : 0;
            unsigned long long o1 = __shfl_xor_sync(FULL_MASK, key, 1 << sh);
            key = o1 > key ? o1 : key;
            unsigned long long o2 = __shfl_xor_sync(FULL_MASK, key, 2 << sh);
            key = o2 > key ? o2 : key;
            if (valid && idx % NW == 0) atomicMax(a.keys + m, key);
        }
    }
}

// y = resid + sum over ranks (in rank order) of every rank's partial, for the
// row-parallel projections of a tensor-parallel decode step.  Each rank's
// projection GEMV wrote its partial into its own buffer `part` (mapped by
// every rank, double-buffered by use parity so that a rank one all-reduce
// ahead never overwrites a buffer a slower rank still reads).  CTA b raises
// flag b on every rank (release, system scope), waits until every rank has
// raised its flag b (acquire; bounded, expirations counted in
// g_tp_timeouts), then reads its 1/AR_CTAS slice of every rank's partial
// over NVLink and sums.  Every rank adds in the same order, so all ranks hold
// bit-identical activations.
__global__ void __launch_bounds__(256) ar_oneshot_kernel(float* __restrict__ y, const float* __restrict__ resid,
                                                         const float* const* parts, uint64_t part_off,
                                                         uint32_t* const* peer_flags, const uint32_t* flags,
                                                         const uint32_t* epoch, uint32_t slot, uint32_t nslot,
                                                         uint32_t world, uint32_t rank, uint64_t n, StepStamp stamp)
{
    const StampAtExit stamp_at_exit(stamp);
    griddep_wait();  // this rank's partial is complete
    griddep_launch_dependents();
    const uint32_t b = blockIdx.x;
    const uint32_t tag = ar_tag(__ldcg(epoch), slot, nslot);
    if (threadIdx.x < world)
    {
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peer_flags[threadIdx.x] + rank * AR_CTAS + b),
                     "r"(tag)
                     : "memory");
        const uint32_t* f = flags + threadIdx.x * AR_CTAS + b;
        uint64_t t0 = 0;
        for (uint32_t it = 0;; ++it)
        {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if (ar_flag_reached(v, tag)) break;
            uint64_t now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (it == 0) t0 = now;
            else if (now - t0 > AR_WAIT_NS)
            {
                atomicAdd(&g_tp_timeouts, 1u);  // the result is wrong; nothing waits forever
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();
    const uint64_t n4 = n / 4, per = (n4 + gridDim.x - 1) / gridDim.x;
    const uint64_t lo = b * per, hi = lo + per < n4 ? lo + per : n4;
    for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x)
    {
        float4 s = reinterpret_cast<const float4*>(resid)[i];
        for (uint32_t r = 0; r < world; ++r)
        {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(parts[r] + part_off) + i);
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        reinterpret_cast<float4*>(y)[i] = s;
    }
}

// Prefill: scatter the packed QKV rows of (b, t) into q and the cache.
__global__ void qkv_scatter_kernel(const float* __restrict__ qkv, float* __restrict__ q, float* __restrict__ kc,
                                   float* __restrict__ vc, uint32_t rows, uint32_t P, uint32_t d, uint32_t hd,
                                   uint32_t C, uint64_t seq_stride)
{
    const uint64_t n = (uint64_t)rows * 3u * d;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint64_t r = i / (3u * d);
        const uint32_t c3 = (uint32_t)(i - r * 3u * d);
        const float v = qkv[i];
        if (c3 < d) { q[r * d + c3] = v; continue; }
        const uint32_t b = (uint32_t)(r / P), t = (uint32_t)(r % P);
        const uint32_t c = c3 % d, h = c / hd, e = c % hd;
        float* cache = c3 < 2 * d ? kc : vc;
        cache[(uint64_t)b * seq_stride + ((uint64_t)h * C + t) * hd + e] = v;
    }
}

// Sum of the S partial planes at float4 offset i (plane stride `plane`
// floats), added in plane order; the loads of four planes are requested
// before any is added (one L2 round trip per four planes, not per plane).
__device__ __forceinline__ float4 sum_planes(const float* __restrict__ part, uint64_t plane, uint64_t i, uint32_t S)
{
    const float4* p4 = reinterpret_cast<const float4*>(part);
    const uint64_t pl4 = plane / 4;
    float4 v = p4[i];
    uint32_t s = 1;
    for (; s + 4 <= S; s += 4)
    {
        float4 w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) w[u] = p4[(s + u) * pl4 + i];
#pragma unroll
        for (int u = 0; u < 4; ++u)
        {
            v.x += w[u].x; v.y += w[u].y; v.z += w[u].z; v.w += w[u].w;
        }
    }
    for (; s < S; ++s)
    {
        const float4 w = p4[s * pl4 + i];
        v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
    }
    return v;
}

// The decode rows' split-K tensor-core contractions: v = sum of the S
// partial planes part[s] [M x N] in plane order (deterministic), then the
// GEMV's epilogue (a.y / a.r / a.q / K/V cache at a.pos, as in
// gemv_team_kernel), four consecutive columns per thread (N, the row
// strides and hd are multiples of 4, so the four share a head).
template <int EPI>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ part, uint32_t S, GemvArgs a)
{
    const StampAtExit stamp_at_exit(a.stamp);
    griddep_launch_dependents();
    griddep_wait();  // the partials come from the previous kernel
    const uint32_t N = a.N;
    const uint64_t plane = (uint64_t)a.M * N, n4 = plane / 4;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const float4 v = sum_planes(part, plane, i, S);
        const uint32_t m = (uint32_t)(4 * i / N), n = (uint32_t)(4 * i - (uint64_t)m * N);
        if constexpr (EPI == EPI_STORE)
            *reinterpret_cast<float4*>(a.y + (uint64_t)m * a.ldy + n) = v;
        else if constexpr (EPI == EPI_GELU)
            *reinterpret_cast<float4*>(a.y + (uint64_t)m * a.ldy + n) =
                make_float4(gelu_exact(v.x), gelu_exact(v.y), gelu_exact(v.z), gelu_exact(v.w));
        else if constexpr (EPI == EPI_RESID)
        {
            const float4 r = *reinterpret_cast<const float4*>(a.r + (uint64_t)m * a.ldr + n);
            *reinterpret_cast<float4*>(a.y + (uint64_t)m * a.ldy + n) =
                make_float4(r.x + v.x, r.y + v.y, r.z + v.z, r.w + v.w);
        }
        else if constexpr (EPI == EPI_QKV)
        {
            float* dst;
            if (n < a.d) dst = a.q + (uint64_t)m * a.d + n;
            else
            {
                const uint32_t cc = n < 2 * a.d ? n - a.d : n - 2 * a.d;
                dst = (n < 2 * a.d ? a.kc : a.vc) + (uint64_t)m * a.seq_stride +
                      ((uint64_t)(cc / a.hd) * a.C + a.pos[m]) * a.hd + cc % a.hd;
            }
            *reinterpret_cast<float4*>(dst) = v;
        }
    }
}

// The same reduction for a residual output, y = r + sum of the planes, one
// CTA per row, followed by the LayerNorm the next contraction needs
// (LayerNorm.h:148-165: two-pass mean and biased variance over the row held
// in registers): ln_out = LayerNormOp(y) with ln_gamma.  N = 1024 NV.
template <int NV>
__global__ void __launch_bounds__(256) splitk_reduce_ln_kernel(const float* __restrict__ part, uint32_t S, GemvArgs a)
{
    const StampAtExit stamp_at_exit(a.stamp);
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float red[8];
    const uint32_t m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t N = a.N;
    const uint64_t plane = (uint64_t)a.M * N;
    float4 v[NV];
    float s1 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
    {
        const uint32_t n = 4 * (tid + 256 * i);
        const uint64_t off = (uint64_t)m * N + n;
        float4 x = sum_planes(part, plane, off / 4, S);
        const float4 r = *reinterpret_cast<const float4*>(a.r + (uint64_t)m * a.ldr + n);
        x = make_float4(r.x + x.x, r.y + x.y, r.z + x.z, r.w + x.w);
        *reinterpret_cast<float4*>(a.y + (uint64_t)m * a.ldy + n) = x;
        v[i] = x;
        s1 += (x.x + x.y) + (x.z + x.w);
    }
    auto block_sum = [&](float t) {
        t = warp_sum(t);
        __syncthreads();  // red[] of a previous sum has been read
        if (lane == 0) red[warp] = t;
        __syncthreads();
        float u = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) u += red[w];
        return u;
    };
    const float invN = 1.0f / (float)N;
    const float mean = block_sum(s1) * invN;
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
    {
        const float d0 = v[i].x - mean, d1 = v[i].y - mean, d2 = v[i].z - mean, d3 = v[i].w - mean;
        s2 = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, s2))));
    }
    const float rstd = 1.0f / sqrtf(fmaf(block_sum(s2), invN, 1e-5f));
#pragma unroll
    for (int i = 0; i < NV; ++i)
    {
        const uint32_t n = 4 * (tid + 256 * i);
        const float4 g = *reinterpret_cast<const float4*>(a.ln_gamma + n);
        *reinterpret_cast<float4*>(a.ln_out + (uint64_t)m * N + n) =
            make_float4((v[i].x - mean) * rstd * g.x, (v[i].y - mean) * rstd * g.y, (v[i].z - mean) * rstd * g.z,
                        (v[i].w - mean) * rstd * g.w);
    }
}

// Argmax keys of logits rows (the tensor-core lm_head): keys[m] = max over
// this CTA's columns n of argmax_key(logits[m][n], n + n_off), folded into
// the row's key with one atomicMax per CTA (keys start at zero: finalize
// resets them).  grid = (column chunks, rows).
__global__ void __launch_bounds__(256) argmax_rows_kernel(const float* __restrict__ logits, uint32_t ld, uint32_t N,
                                                          uint32_t n_off, unsigned long long* keys, StepStamp stamp)
{
    const StampAtExit stamp_at_exit(stamp);
    __shared__ unsigned long long wbest[8];
    const uint32_t m = blockIdx.y;
    unsigned long long best = 0ull;
    for (uint32_t n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x)
    {
        const unsigned long long k = argmax_key(logits[(uint64_t)m * ld + n], n + n_off);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        const unsigned long long other = __shfl_xor_sync(FULL_MASK, best, o);
        best = other > best ? other : best;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) wbest[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0)
    {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = wbest[w] > best ? wbest[w] : best;
        atomicMax(keys + m, best);
    }
}

// After lm_head: pending token = argmax, advance the position, reset keys.
// With stamps on, thread 0 stamps the step's last slot and then advances the
// stamp step counter (every other kernel of the step has finished by then).
__global__ void finalize_kernel(unsigned long long* keys, uint32_t* pending, uint32_t* pos, uint32_t* next_out,
                                uint32_t B, uint32_t set_pos, uint32_t* epoch, StepStamp stamp, uint32_t* stamp_ctr)
{
    FML_TIMELINE_SCOPE(30);
    griddep_launch_dependents();
    griddep_wait();
    FML_TIMELINE_MARK(1);
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b == 0 && epoch) *epoch += 1u;
    if (b == 0 && stamp.buf)
    {
        stamp_write(stamp);
        *stamp_ctr += 1u;
    }
    if (b >= B) return;
    const uint32_t tok = argmax_key_index(keys[b]);
    pending[b] = tok;
    if (next_out) next_out[b] = tok;
    pos[b] = set_pos ? set_pos : pos[b] + 1u;
    keys[b] = 0ull;
}

// out[c * rows + r] = in[r * cols + c]: repack a [rows x cols] weight into
// [cols x rows] (K-contiguous) at bind time.
__global__ void transpose_kernel(float* __restrict__ out, const float* __restrict__ in, uint32_t rows, uint32_t cols)
{
    __shared__ float tile[32][33];
    const uint32_t c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y)
    {
        const uint32_t r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = in[(uint64_t)r * cols + c];
    }
    __syncthreads();
    for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y)
    {
        const uint32_t c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[(uint64_t)c * rows + r] = tile[threadIdx.x][i];
    }
}

// bf16 copy of fp32 weights, rounded to nearest even.
__global__ void to_bf16_kernel(uint16_t* __restrict__ out, const float* __restrict__ in, uint64_t n)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(in[i]));
}

__global__ void rewind_kernel(uint32_t* pos, uint32_t* pending, const uint32_t* src, uint32_t B, uint32_t p)
{
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    pos[b] = p;
    if (src) pending[b] = src[b];
}

__global__ void gelu_inplace_kernel(float* x, uint64_t n)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        x[i] = gelu_exact(x[i]);
}

__global__ void add_kernel(float* out, const float* a, const float* b, uint64_t n)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = a[i] + b[i];
}

}  // namespace fml

using namespace fml;

// ---------------------------------------------------------------- engine --

struct fml_lm
{
    fml_lm_config cfg{};
    int device = 0;
    uint32_t hd = 0;
    bool bound = false;

    // weights
    float* wbuf = nullptr;  // one allocation for every parameter
    // TF32x3 prefill: each layer weight's lo part (W - hi(W)) in W's layout,
    // so that the tensor-core kernel splits only the activations; made at
    // the first TF32x3 prefill after binding, when the memory is there
    float* wlo = nullptr;
    bool wlo_valid = false, wlo_failed = false;
    std::vector<float*> wqkv_lo, wproj_lo, wfc_lo, wmlp_lo;
    float *tok = nullptr, *pos_emb = nullptr, *lnf = nullptr;
    std::vector<float*> ln0, ln1, wqkv, wproj, wfc, wmlp;
    // FML_WEIGHTS_BF16: the decode step's GEMVs stream a bf16 copy of their
    // weights (layer matrices and the lm_head's vocabulary rows), made after
    // each bind before the next step; the prefill keeps the fp32 weights
    int weight_format = FML_WEIGHTS_FP32;
    uint16_t* wb16 = nullptr;
    bool wb16_valid = false;
    std::vector<const uint16_t*> wqkv_b, wproj_b, wfc_b, wmlp_b;
    const uint16_t* head_b = nullptr;

    // KV cache
    float *kc = nullptr, *vc = nullptr;
    uint64_t layer_stride = 0, seq_stride = 0;

    // activations (prefill rows = max_batch * context; decode uses the first rows)
    float *x = nullptr, *buf = nullptr, *ln = nullptr, *q = nullptr, *att = nullptr, *tmp = nullptr, *hid = nullptr;

    // state
    uint32_t* pending = nullptr;
    uint32_t* pos = nullptr;
    uint32_t* prompt_dev = nullptr;
    unsigned long long* keys = nullptr;
    float* part = nullptr;
    uint32_t* counters = nullptr;
    uint32_t* grab = nullptr;  // [L] attention work-unit counters
    uint32_t* host_io = nullptr;  // pinned [2 * max_batch]
    uint32_t* host_io_dev = nullptr;  // host_io as the device addresses it (null: not mapped)
    uint32_t S = 1, chunk = 0;

    uint32_t batch = 0;                // active sequences
    std::vector<uint32_t> hpos;        // host mirror of positions

    // graph / programmatic dependent launch
    bool use_graph = true;
    bool pdl = true;
    int prefill_math = FML_MATH_TF32X3;  // prefill contractions on the tensor cores

    // tensor parallelism: this rank's heads [h0, h0 + hl) (q/k/v width dl),
    // fc columns [j0, j0 + fl), vocabulary rows [v0, v0 + vl); proj and mlp
    // are row-parallel (partial sums all-reduced), the lm_head argmax keys
    // are max-reduced.  One rank: the whole model.
    int tp_rank = 0, tp_world = 1;
    ncclComm_t comm = nullptr;
    uint32_t hl = 0, dl = 0, fl = 0, h0 = 0, j0 = 0, v0 = 0, vl = 0;
    // fused all-reduce over peer memory (after fml_lm_tp_connect)
    bool ar_fused = false;
    float* ar_part = nullptr;        // [2][max_batch][d]: this rank's partial sums, read by every rank
    uint32_t* ar_flags = nullptr;    // [world][AR_CTAS]
    uint32_t* ar_epoch = nullptr;    // steps completed
    float** ar_peer_part = nullptr;  // device arrays of the world's pointers
    uint32_t** ar_peer_flags = nullptr;
    std::vector<void*> ar_opened;    // peer mappings to close

    // in-graph completion stamps (fml_lm_set_stamps): one slot per kernel of
    // a step, `stamp_stride` slots per step; the class of each slot
    unsigned long long* stamps = nullptr;
    uint32_t stamp_cap = 0, stamp_stride = 0, stamp_n = 0;
    uint32_t* stamp_step = nullptr;  // device step counter (advanced by finalize)
    std::vector<int> stamp_class;
    uint32_t step_kernels = 0;  // kernels one enqueued step launches
    cudaGraphExec_t graph_exec = nullptr;
    cudaStream_t graph_stream = nullptr;
    uint32_t* graph_next = nullptr;
    float* graph_logits = nullptr;
    uint32_t graph_batch = 0;
    // the host-buffer step (H2D of the tokens, the step, D2H of the next
    // tokens) as one graph: one launch per step instead of three calls
    cudaGraphExec_t host_graph_exec = nullptr;
    uint32_t host_graph_batch = 0;
    // several steps as one graph (fml_lm_steps): no launch gap between the
    // steps it holds, and each step's embed overlaps the previous finalize
    // (steps per graph, graph) for the current batch: the main size and the
    // remainder of a call
    std::vector<std::pair<uint32_t, cudaGraphExec_t>> multi_graphs;
    uint32_t multi_graph_batch = 0;

    // profiling
    bool profiling = false;
    double prof_ms[FML_LM_NCLASS] = {};
    uint64_t prof_n[FML_LM_NCLASS] = {};
    std::vector<cudaEvent_t> ev_pool;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> ev_pending;
    size_t ev_used = 0;
};

namespace {

uint64_t param_count(const fml_lm_config& c)
{
    const uint64_t d = c.d_model;
    return (uint64_t)c.vocab * d + (uint64_t)c.context * d + (uint64_t)c.n_layer * (2 * d + 12 * d * d) + d;
}

// Forget the recorded step graphs (their launch plan no longer holds).
void drop_graphs(fml_lm* lm)
{
    if (lm->graph_exec) cudaGraphExecDestroy(lm->graph_exec);
    lm->graph_exec = nullptr;
    if (lm->host_graph_exec) cudaGraphExecDestroy(lm->host_graph_exec);
    lm->host_graph_exec = nullptr;
    for (auto& g : lm->multi_graphs) cudaGraphExecDestroy(g.second);
    lm->multi_graphs.clear();
}

void free_all(fml_lm* lm)
{
    drop_graphs(lm);
    if (lm->comm) ncclCommDestroy(lm->comm);
    lm->comm = nullptr;
    for (void* p : lm->ar_opened) cudaIpcCloseMemHandle(p);
    lm->ar_opened.clear();
    void* arp[] = {lm->ar_part, lm->ar_flags, lm->ar_epoch, lm->ar_peer_part, lm->ar_peer_flags};
    for (void* p : arp)
        if (p) cudaFree(p);
    for (cudaEvent_t e : lm->ev_pool) cudaEventDestroy(e);
    if (lm->wlo) cudaFree(lm->wlo);
    lm->wlo = nullptr;
    if (lm->wb16) cudaFree(lm->wb16);
    lm->wb16 = nullptr;
    void* ptrs[] = {lm->wbuf, lm->kc,  lm->vc,      lm->x,          lm->buf,  lm->ln,   lm->q,
                    lm->att,  lm->tmp, lm->hid,     lm->pending,    lm->pos,  lm->keys, lm->part,
                    lm->counters, lm->prompt_dev, lm->grab, lm->stamp_step};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    if (lm->host_io) cudaFreeHost(lm->host_io);
}

// Event-pair timing of one kernel class (profiling mode only).
struct ProfScope
{
    fml_lm* lm;
    int cls;
    cudaStream_t st;
    cudaEvent_t b = nullptr, e = nullptr;
    ProfScope(fml_lm* l, int c, cudaStream_t s) : lm(l), cls(c), st(s)
    {
        if (!lm->profiling) return;
        while (lm->ev_pool.size() < lm->ev_used + 2)
        {
            cudaEvent_t ev;
            cudaEventCreate(&ev);
            lm->ev_pool.push_back(ev);
        }
        b = lm->ev_pool[lm->ev_used++];
        e = lm->ev_pool[lm->ev_used++];
        cudaEventRecord(b, st);
    }
    ~ProfScope()
    {
        if (!b) return;
        cudaEventRecord(e, st);
        lm->ev_pending.push_back({cls, {b, e}});
    }
};

int collect_profile(fml_lm* lm)
{
    if (lm->ev_pending.empty()) return FML_OK;
    FML_CUDA_TRY(cudaEventSynchronize(lm->ev_pending.back().second.second));
    for (auto& p : lm->ev_pending)
    {
        float ms = 0.0f;
        FML_CUDA_TRY(cudaEventElapsedTime(&ms, p.second.first, p.second.second));
        lm->prof_ms[p.first] += ms;
        lm->prof_n[p.first] += 1;
    }
    lm->ev_pending.clear();
    lm->ev_used = 0;
    return FML_OK;
}

// Launch with programmatic dependent launch when `pdl` is set: the kernel may
// start while the previous one in the stream finishes (it calls
// griddepcontrol.wait before reading that kernel's output).
template <typename... KArgs, typename... Args>
int launch_ks(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "cudaLaunchKernelEx: %s", cudaGetErrorString(e));
    FML_LAUNCH_CHECK();
    return FML_OK;
}

template <typename... KArgs, typename... Args>
int launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, bool pdl, Args... args)
{
    return launch_ks(kern, grid, block, 0, st, pdl, std::forward<Args>(args)...);
}

// Resident CTAs per SM of a gemv instantiation (cached per instantiation).
template <int MT, int EPI, bool LN, bool WB>
int gemv_blocks_per_sm()
{
    static int n = 0;
    if (!n)
    {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, gemv_kernel<MT, EPI, LN, WB>, 128, 0) != cudaSuccess ||
            b < 1)
            b = 1;
        n = b;
    }
    return n;
}

template <int MT, int EPI, bool LN, bool WB>
int launch_gemv_mt(const GemvArgs& a, cudaStream_t st, bool pdl, int sms)
{
    const unsigned gx = (a.M + MT - 1) / MT;
    const unsigned ngroups = (a.N + 3) / 4;
    // one wave: every CTA resident at once, each walking several column groups
    // (measured: capping the CTAs per SM to leave room for the next kernel's
    // early-launched CTAs only slows the step)
    const unsigned slots = (unsigned)(gemv_blocks_per_sm<MT, EPI, LN, WB>() * sms);
    unsigned gy = slots / gx;
    if (gy < 1) gy = 1;
    if (gy > ngroups) gy = ngroups;
    if (gy > 65535u) gy = 65535u;
    return launch_k(gemv_kernel<MT, EPI, LN, WB>, dim3(gx, gy), dim3(128), st, pdl, a);
}

constexpr size_t GEMV_TEAM_MAX_SMEM = 64 * 1024;  // staged x rows per CTA

template <int MT, int KW, int EPI, bool LN, bool WB>
int launch_gemv_team(const GemvArgs& a, cudaStream_t st, bool pdl, int sms)
{
    auto kern = gemv_team_kernel<MT, KW, EPI, LN, WB>;
    const size_t smem = (size_t)(MT + (LN ? 1 : 0)) * a.K * sizeof(float);
    static uint64_t attr_devices = 0;
    static size_t occ_smem = 0;
    static int occ = 0;
    FML_RC(smem_limit_once(reinterpret_cast<const void*>(kern), (int)GEMV_TEAM_MAX_SMEM, attr_devices));
    if (occ_smem != smem || occ == 0)
    {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, 128, smem) != cudaSuccess || b < 1) b = 1;
        occ = b;
        occ_smem = smem;
    }
    const int per_sm = occ;
    const unsigned gx = (a.M + MT - 1) / MT;
    const unsigned ngroups = (a.N + 3) / 4;
    const unsigned teams = 4 / KW;
    unsigned gy = (unsigned)(per_sm * sms) / gx;  // one wave
    gy = std::min(std::max(gy, 1u), (ngroups + teams - 1) / teams);
    gy = std::min(gy, 65535u);
    return launch_ks(kern, dim3(gx, gy), dim3(128), smem, st, pdl, a);
}

// K split: one warp per column group up to K = 1024 (8 float4 slices per
// lane), four above (FML_GEMV_KW1_MAX / FML_GEMV_KW2_MAX: the largest K for
// one and for two warps).  Measured on B200: one warp instead of two at
// K = 1024 (config 4) 2738 -> 2703 us per step; two instead of four at
// K = 2048 (config 3's mlp) 245 -> 251 us.
#ifndef FML_GEMV_KW1_MAX
#define FML_GEMV_KW1_MAX 1024
#endif
#ifndef FML_GEMV_KW2_MAX
#define FML_GEMV_KW2_MAX 1024
#endif
template <int MT, int EPI, bool LN, bool WB>
int launch_gemv_team_k(const GemvArgs& a, cudaStream_t st, bool pdl, int sms)
{
    uint32_t kw = a.K <= FML_GEMV_KW1_MAX ? 1u : (a.K <= FML_GEMV_KW2_MAX ? 2u : 4u);
    if (const char* e = getenv("FML_GEMV_KW"))  // tuning override: 1, 2 or 4
    {
        const long v = strtol(e, nullptr, 10);
        if (v == 1 || v == 2 || v == 4) kw = (uint32_t)v;
    }
    if (kw == 1) return launch_gemv_team<MT, 1, EPI, LN, WB>(a, st, pdl, sms);
    if (kw == 2) return launch_gemv_team<MT, 2, EPI, LN, WB>(a, st, pdl, sms);
    return launch_gemv_team<MT, 4, EPI, LN, WB>(a, st, pdl, sms);
}

template <int EPI, bool LN, bool WB>
int launch_gemv_w(const GemvArgs& a, cudaStream_t st, bool pdl)
{
    FML_REQUIRE(a.K % 4 == 0 && a.ldx % 4 == 0, "gemv: K and ldx must be multiples of 4");
    FML_REQUIRE(!WB || (a.K % 8 == 0 && a.wb), "gemv: bf16 weights need K a multiple of 8");
    FML_REQUIRE(!LN || a.gamma, "gemv: LayerNorm prologue without gamma");
    static int sms = 0;
    if (!sms)
    {
        int dev = 0;
        FML_CUDA_TRY(cudaGetDevice(&dev));
        FML_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    }
    // rows (tokens) per CTA: 4 up to 32 rows, 8 above.  Fewer rows per CTA
    // means more CTAs, fewer registers and more loads in flight, at the cost
    // of re-reading W from L2 once per row chunk; measured on B200 (decode
    // tokens/s against 16 rows per CTA): +13 % at 32 sequences (config 3),
    // +10 % at 8 (config 5); at 64 (config 4) 8 rows beat 4 and 16.
    // Tuning override: FML_GEMV_MT = 4, 8 or 16.
    const char* mt_env = getenv("FML_GEMV_MT");
    const long mt_v = mt_env ? strtol(mt_env, nullptr, 10) : (a.M > 32 ? 8 : 4);
    const uint32_t mt_cap = (uint32_t)(mt_v == 4 || mt_v == 8 ? mt_v : 16);
    // team layout for K <= 2048 when the CTA's x rows fit in shared memory;
    // measured on B200: config 3 decode 299 -> 265 us/step, config 4 +15 %
    // tokens/s, but config 5's K = 4096 projection 28 us slower per launch,
    // so larger K keeps the one-group layout (FML_GEMV_TEAM=0: always it)
    const char* team_env = getenv("FML_GEMV_TEAM");
    const bool team = !(team_env && strtol(team_env, nullptr, 10) == 0) && mt_cap <= 8 && a.K <= 2048;
    const uint32_t mt_team = a.M <= 4 || mt_cap == 4 ? 4u : 8u;
    if (team && (mt_team + (LN ? 1 : 0)) * a.K * sizeof(float) <= GEMV_TEAM_MAX_SMEM)
    {
        if (mt_team == 4) return launch_gemv_team_k<4, EPI, LN, WB>(a, st, pdl, sms);
        return launch_gemv_team_k<8, EPI, LN, WB>(a, st, pdl, sms);
    }
    if (a.M <= 4 || mt_cap == 4) return launch_gemv_mt<4, EPI, LN, WB>(a, st, pdl, sms);
    if (a.M <= 8 || mt_cap == 8) return launch_gemv_mt<8, EPI, LN, WB>(a, st, pdl, sms);
    return launch_gemv_mt<16, EPI, LN, WB>(a, st, pdl, sms);
}

// The decode GEMV: fp32 weights (a.w), or their bf16 copy when a.wb is set.
template <int EPI, bool LN>
int launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl)
{
    if (a.wb) return launch_gemv_w<EPI, LN, true>(a, st, pdl);
    return launch_gemv_w<EPI, LN, false>(a, st, pdl);
}

int launch_attention(fml_lm* lm, uint32_t layer, uint32_t row0, uint32_t rows, const uint32_t* pos, uint32_t P,
                     uint32_t S, uint32_t chunk, cudaStream_t st, bool pdl = false, StepStamp stamp = StepStamp{})
{
    AttnArgs a{};
    a.row0 = row0;
    a.q = lm->q;
    a.ldq = lm->dl;
    a.kc = lm->kc + (uint64_t)layer * lm->layer_stride;
    a.vc = lm->vc + (uint64_t)layer * lm->layer_stride;
    a.seq_stride = lm->seq_stride;
    a.H = lm->hl;
    a.C = lm->cfg.context;
    a.out = lm->att;
    a.ldo = lm->dl;
    a.pos = pos;
    a.P = P;
    a.S = S;
    a.chunk = chunk;
    a.scale = 1.0f / sqrtf((float)lm->hd);
    a.part = lm->part;
    a.counters = lm->counters;
    a.grab = lm->grab + layer;
    a.stamp = stamp;
    FML_REQUIRE(rows <= 65535u, "attention: too many rows in one launch (%u)", rows);
    FML_RC(launch_attention_kernel(a, lm->hd, dim3(lm->hl, rows, S), st, pdl));
    return FML_OK;
}

// Row-parallel partial sums: in-place NCCL all-reduce on the engine stream
// (captured into the step's graph like the kernels).
int all_reduce_sum(fml_lm* lm, float* buf, uint64_t n, cudaStream_t st)
{
    const ncclResult_t r = ncclAllReduce(buf, buf, n, ncclFloat32, ncclSum, lm->comm, st);
    if (r != ncclSuccess) return set_error(FML_ERR_CUDA, "ncclAllReduce: %s", ncclGetErrorString(r));
    return FML_OK;
}

// Vocabulary-parallel argmax: every rank's packed (value, ~index) keys hold
// its local best; the max over ranks is the global first-index argmax.
int all_reduce_max_keys(fml_lm* lm, uint32_t B, cudaStream_t st)
{
    const ncclResult_t r = ncclAllReduce(lm->keys, lm->keys, B, ncclUint64, ncclMax, lm->comm, st);
    if (r != ncclSuccess) return set_error(FML_ERR_CUDA, "ncclAllReduce: %s", ncclGetErrorString(r));
    return FML_OK;
}

// The stamp of the next kernel a step enqueues (class `cls`, FML_LM_* profile
// classes); a null stamp when stamps are off.
StepStamp next_stamp(fml_lm* lm, int cls)
{
    StepStamp s{};
    if (lm->stamps)
    {
        s.buf = lm->stamps;
        s.step = lm->stamp_step;
        s.stride = lm->stamp_stride;
        s.idx = lm->stamp_n;
        s.cap = lm->stamp_cap;
    }
    lm->stamp_class.push_back(cls);
    ++lm->stamp_n;
    return s;
}

// One decode contraction (the CUDA-core GEMV with its fused prologue and
// epilogue) with the step's next completion stamp.
template <int EPI, bool LN>
int decode_gemv(fml_lm* lm, GemvArgs a, int cls, cudaStream_t st, bool pdl)
{
    a.stamp = next_stamp(lm, cls);
    return launch_gemv<EPI, LN>(a, st, pdl);
}

// Row-parallel projection + all-reduce over peer memory: the GEMV writes this
// rank's partial into its shared buffer (parity `slot & 1`), the one-shot
// kernel sums the world's partials and the residual into y.
int gemv_allreduce(fml_lm* lm, GemvArgs a, float* y, const float* resid, uint32_t slot, int cls, cudaStream_t st,
                   bool pdl)
{
    const uint64_t n = (uint64_t)a.M * a.N, off = (uint64_t)(slot & 1u) * lm->cfg.max_batch * lm->cfg.d_model;
    a.y = lm->ar_part + off;
    a.ldy = a.N;
    FML_RC((decode_gemv<EPI_STORE, false>(lm, a, cls, st, pdl)));
    return launch_k(ar_oneshot_kernel, dim3(AR_CTAS), dim3(256), st, pdl, y, resid,
                    (const float* const*)lm->ar_peer_part, off, (uint32_t* const*)lm->ar_peer_flags,
                    (const uint32_t*)lm->ar_flags, (const uint32_t*)lm->ar_epoch, slot, 2u * lm->cfg.n_layer,
                    (uint32_t)lm->tp_world, (uint32_t)lm->tp_rank, n, next_stamp(lm, 9));
}

// The decode lm_head on the tcgen05 GEMM instead of the GEMV: TF32x3 math,
// fp32 weights, at least 32 rows and 148 column tiles of 128 (one per SM),
// and room for the logits in the engine's scratch rows.
bool lm_head_on_tensor_cores(const fml_lm* lm)
{
    const uint64_t d = lm->cfg.d_model;
    return lm->prefill_math == FML_MATH_TF32X3 && lm->weight_format == FML_WEIGHTS_FP32 && lm->batch >= 32 &&
           (lm->vl + 127) / 128 >= 148 && d % 4 == 0 &&
           (uint64_t)lm->batch * lm->vl <= (uint64_t)lm->cfg.max_batch * lm->cfg.context * 3 * lm->dl;
}

// The decode contractions on the tcgen05 GEMM (split K, then a reduction
// with the GEMV's epilogue): TF32x3 math, fp32 weights, one rank, at least
// 32 rows and d a multiple of 1024 -- there the CUDA-core GEMV's row chunks
// re-read each weight and walk many column-group rounds per warp.  Measured
// on config 4's shape (us per step, GEMV / tensor cores): 64 rows 2 620 /
// 2 170, 32 rows 1 469 / 1 387, 16 rows 838 / 989, 8 rows 584 / 828.
bool decode_on_tensor_cores(const fml_lm* lm)
{
    const bool able = lm->prefill_math == FML_MATH_TF32X3 && lm->weight_format == FML_WEIGHTS_FP32 &&
                      lm->tp_world == 1 && lm->cfg.d_model % 1024 == 0 && lm->cfg.d_model <= 4096;
    const char* e = getenv("FML_DECODE_TC");  // tuning override: 0 never, 1 at any batch
    if (e && e[0] == '0') return false;
    if (e && e[0] == '1') return able;
    return able && lm->batch >= 32;
}

// One decode contraction y = epilogue(A . W^T) on the tensor cores: the K
// split doubles (K / 32 divisible) while the tiles still fit one wave.
template <int EPI>
int decode_tc_gemm(fml_lm* lm, GemvArgs a, int cls, cudaStream_t st, bool pdl)
{
    const uint32_t tiles = (a.N + 127) / 128 * ((a.M + 127) / 128);
    uint32_t ks = 1;
    while (ks < 16 && tiles * ks * 2 <= 148 && (a.K / 32) % (ks * 2) == 0) ks *= 2;
    float* part = lm->tmp;
    FML_REQUIRE((uint64_t)ks * a.M * a.N <= (uint64_t)lm->cfg.max_batch * lm->cfg.context * 3 * lm->dl,
                "decode_tc_gemm: split-K partials exceed the scratch rows");
    // the weights' stored lo parts (the prefill's) would double the bytes a
    // decode step streams: the converter warps split the weight tiles
    // instead (measured on config 4: 2 192 -> 2 168 us per step)
    FML_RC(gemm_tc_splitk(part, a.x, a.w, (int)a.M, (int)a.N, (int)a.K, (int)a.ldx, (int)a.K, true, (int)ks, st,
                          nullptr, pdl));
    a.stamp = next_stamp(lm, cls);
    if (EPI == EPI_RESID && a.ln_out)
    {
        const uint32_t nv = a.N / 1024;
        auto k = nv == 1 ? splitk_reduce_ln_kernel<1> : (nv == 2 ? splitk_reduce_ln_kernel<2> : splitk_reduce_ln_kernel<4>);
        return launch_k(k, dim3(a.M), dim3(256), st, pdl, (const float*)part, ks, a);
    }
    const uint64_t n4 = (uint64_t)a.M * a.N / 4;
    return launch_k(splitk_reduce_kernel<EPI>, dim3((unsigned)std::min<uint64_t>((n4 + 255) / 256, 148u * 8u)),
                    dim3(256), st, pdl, (const float*)part, ks, a);
}

// The tcgen05 kernels a decode step may launch get their shared-memory
// limit before any capture records the step.
int prepare_tc_decode(const fml_lm* lm)
{
    if (lm_head_on_tensor_cores(lm) || decode_on_tensor_cores(lm))
    {
        FML_RC(gemm_tc_prepare(true, 0, false));
    }
    return FML_OK;
}

// Enqueue one decode step for the active batch: embed, per layer
// {qkv (LayerNorm fused) -> attention -> proj + residual -> fc (LayerNorm
// fused) + GELU -> mlp + residual}, lm_head (final LayerNorm fused) + argmax,
// finalize.  Every launch after the first uses programmatic dependent launch.
// ids: the tokens the step consumes (default: the pending tokens).
// chained: the previous kernel on `st` is this engine's finalize of the
// previous step (captured in the same graph), so the embed may launch under
// programmatic dependent launch too.
int enqueue_step(fml_lm* lm, uint32_t* next_out, float* logits, cudaStream_t st, const uint32_t* ids = nullptr,
                 bool chained = false)
{
    const fml_lm_config& c = lm->cfg;
    const uint32_t B = lm->batch, d = c.d_model;
    const bool pdl = lm->pdl && !lm->profiling;
    const uint64_t launched0 = launch_counter().load(std::memory_order_relaxed);
    lm->stamp_n = 0;
    lm->stamp_class.clear();
    {
        ProfScope ps(lm, 0, st);
        FML_RC(launch_k(embed_kernel, dim3(B), dim3(128), st, chained && pdl && lm->tp_world == 1, lm->x,
                        (const float*)lm->tok,
                        (const float*)lm->pos_emb, ids ? ids : (const uint32_t*)lm->pending, (const uint32_t*)lm->pos,
                        B, 1u, d, c.vocab, c.context, lm->grab, c.n_layer, next_stamp(lm, 0)));
    }
    const bool tp = lm->tp_world > 1;
    const bool resid_here = lm->tp_rank == 0;  // row-parallel sums take the residual once
    const bool wb = lm->weight_format == FML_WEIGHTS_BF16;
    FML_REQUIRE(!wb || lm->wb16_valid, "decode step: the bf16 weight copy is not ready");
    const bool dtc = decode_on_tensor_cores(lm);  // rows of LayerNorm, tcgen05 split-K, reduction
    for (uint32_t l = 0; l < c.n_layer; ++l)
    {
        {
            ProfScope ps(lm, 2, st);
            GemvArgs a{};
            a.x = lm->x; a.ldx = d; a.w = lm->wqkv[l]; a.M = B; a.N = 3 * lm->dl; a.K = d; a.gamma = lm->ln0[l];
            if (wb) a.wb = lm->wqkv_b[l];
            a.q = lm->q; a.kc = lm->kc + (uint64_t)l * lm->layer_stride; a.vc = lm->vc + (uint64_t)l * lm->layer_stride;
            a.pos = lm->pos; a.d = lm->dl; a.H = lm->hl; a.hd = lm->hd; a.C = c.context; a.seq_stride = lm->seq_stride;
            if (dtc)
            {
                // lm->ln holds LN0(x): the previous layer's mlp reduction (or,
                // for layer 0, the LayerNorm after the embedding) made it
                if (l == 0) FML_RC(launch_layernorm(lm->ln, lm->x, lm->ln0[0], nullptr, nullptr, B, d, d, d, 1e-5f, st));
                a.x = lm->ln;
                FML_RC(decode_tc_gemm<EPI_QKV>(lm, a, 2, st, pdl && l > 0));
            }
            else
                FML_RC((decode_gemv<EPI_QKV, true>(lm, a, 2, st, pdl)));
        }
        {
            ProfScope ps(lm, 3, st);
            FML_RC(launch_attention(lm, l, 0, B, lm->pos, 1, lm->S, 0, st, pdl, next_stamp(lm, 3)));
        }
        {
            ProfScope ps(lm, 4, st);
            GemvArgs a{};
            a.x = lm->att; a.ldx = lm->dl; a.w = lm->wproj[l]; a.M = B; a.N = d; a.K = lm->dl;
            if (wb) a.wb = lm->wproj_b[l];
            a.y = lm->buf; a.ldy = d; a.r = lm->x; a.ldr = d;
            if (dtc)
            {
                a.ln_out = lm->ln;  // LN1(buf) for fc
                a.ln_gamma = lm->ln1[l];
                FML_RC(decode_tc_gemm<EPI_RESID>(lm, a, 4, st, pdl));
            }
            else if (lm->ar_fused) FML_RC(gemv_allreduce(lm, a, lm->buf, lm->x, 2 * l, 4, st, pdl));
            else
            {
                if (resid_here) FML_RC((decode_gemv<EPI_RESID, false>(lm, a, 4, st, pdl)));
                else FML_RC((decode_gemv<EPI_STORE, false>(lm, a, 4, st, pdl)));
                if (tp) FML_RC(all_reduce_sum(lm, lm->buf, (uint64_t)B * d, st));
            }
        }
        {
            ProfScope ps(lm, 5, st);
            GemvArgs a{};
            a.x = lm->buf; a.ldx = d; a.w = lm->wfc[l]; a.M = B; a.N = lm->fl; a.K = d; a.gamma = lm->ln1[l];
            if (wb) a.wb = lm->wfc_b[l];
            a.y = lm->hid; a.ldy = lm->fl;
            if (dtc)
            {
                a.x = lm->ln;  // LN1(buf), made by the projection's reduction
                FML_RC(decode_tc_gemm<EPI_GELU>(lm, a, 5, st, pdl));
            }
            else
                FML_RC((decode_gemv<EPI_GELU, true>(lm, a, 5, st, pdl && (!tp || lm->ar_fused))));
        }
        {
            ProfScope ps(lm, 6, st);
            GemvArgs a{};
            a.x = lm->hid; a.ldx = lm->fl; a.w = lm->wmlp[l]; a.M = B; a.N = d; a.K = lm->fl;
            if (wb) a.wb = lm->wmlp_b[l];
            a.y = lm->x; a.ldy = d; a.r = lm->buf; a.ldr = d;
            if (dtc)
            {
                // LN0 of the next layer, or ln_f after the last, for the lm_head
                a.ln_out = lm->ln;
                a.ln_gamma = l + 1 < c.n_layer ? lm->ln0[l + 1] : lm->lnf;
                FML_RC(decode_tc_gemm<EPI_RESID>(lm, a, 6, st, pdl));
            }
            else if (lm->ar_fused) FML_RC(gemv_allreduce(lm, a, lm->x, lm->buf, 2 * l + 1, 6, st, pdl));
            else
            {
                if (resid_here) FML_RC((decode_gemv<EPI_RESID, false>(lm, a, 6, st, pdl)));
                else FML_RC((decode_gemv<EPI_STORE, false>(lm, a, 6, st, pdl)));
                if (tp) FML_RC(all_reduce_sum(lm, lm->x, (uint64_t)B * d, st));
            }
        }
    }
    {
        ProfScope ps(lm, 7, st);
        GemvArgs a{};
        a.x = lm->x; a.ldx = d; a.w = lm->tok + (uint64_t)lm->v0 * d; a.M = B; a.N = lm->vl; a.K = d;
        a.gamma = lm->lnf; a.y = logits; a.ldy = lm->vl; a.keys = lm->keys; a.n_off = lm->v0;
        if (wb) a.wb = lm->head_b;
        if (lm_head_on_tensor_cores(lm))
        {
            // at >= 32 rows and a vocabulary of >= 148 column tiles (config
            // 4: 64 rows x 32000) the GEMV's row chunks re-read the table
            // (131 MB, past L2): LayerNorm rows, then the tcgen05 GEMM (TF32x3)
            // streams the table once, then the argmax keys
            float* lg = logits ? logits : lm->tmp;
            // ln_f(x): made by the last mlp reduction on the tensor-core decode path
            if (!dtc) FML_RC(launch_layernorm(lm->ln, lm->x, lm->lnf, nullptr, nullptr, B, d, d, d, 1e-5f, st));
            FML_RC(gemm_tc(lg, lm->ln, lm->tok + (uint64_t)lm->v0 * d, (int)B, (int)lm->vl, (int)d, (int)d, (int)d,
                           (int)lm->vl, true, 0, nullptr, st));
            const uint32_t chunks = std::min<uint32_t>(64u, (lm->vl + 2047u) / 2048u);
            FML_RC(launch_k(argmax_rows_kernel, dim3(chunks, B), dim3(256), st, false, (const float*)lg, lm->vl,
                            lm->vl, lm->v0, lm->keys, next_stamp(lm, 7)));
        }
        else
            FML_RC((decode_gemv<EPI_ARGMAX, true>(lm, a, 7, st, pdl && !tp)));
        if (tp) FML_RC(all_reduce_max_keys(lm, B, st));
    }
    {
        ProfScope ps(lm, 8, st);
        FML_RC(launch_k(finalize_kernel, dim3((B + 127) / 128), dim3(128), st, pdl && !tp, lm->keys, lm->pending,
                        lm->pos, next_out, B, 0u, lm->ar_epoch, next_stamp(lm, 8), lm->stamp_step));
    }
    lm->step_kernels = (uint32_t)(launch_counter().load(std::memory_order_relaxed) - launched0);
    return FML_OK;
}

// The lo parts of the layer weights for TF32x3 prefill (see fml_lm::wlo):
// allocated once, recomputed after every bind; without the memory the
// kernel keeps splitting W itself.
int ensure_weight_lo(fml_lm* lm, cudaStream_t st)
{
    if (lm->wlo_valid || lm->wlo_failed || lm->prefill_math != FML_MATH_TF32X3) return FML_OK;
    const fml_lm_config& c = lm->cfg;
    const uint64_t d = c.d_model, dl = lm->dl, fl = lm->fl;
    const uint64_t per_layer = 3 * dl * d + d * dl + fl * d + d * fl;
    if (!lm->wlo)
    {
        size_t free_b = 0, total_b = 0;
        const uint64_t need = per_layer * c.n_layer * sizeof(float);
        if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess || free_b < need + (4ull << 30) ||
            cudaMalloc(&lm->wlo, need) != cudaSuccess)
        {
            cudaGetLastError();
            lm->wlo = nullptr;
            lm->wlo_failed = true;
            return FML_OK;
        }
        float* p = lm->wlo;
        for (uint32_t l = 0; l < c.n_layer; ++l)
        {
            lm->wqkv_lo.push_back(p); p += 3 * dl * d;
            lm->wproj_lo.push_back(p); p += d * dl;
            lm->wfc_lo.push_back(p); p += fl * d;
            lm->wmlp_lo.push_back(p); p += d * fl;
        }
    }
    for (uint32_t l = 0; l < c.n_layer; ++l)
    {
        FML_RC(tf32_lo(lm->wqkv_lo[l], lm->wqkv[l], 3 * dl * d, st));
        FML_RC(tf32_lo(lm->wproj_lo[l], lm->wproj[l], d * dl, st));
        FML_RC(tf32_lo(lm->wfc_lo[l], lm->wfc[l], fl * d, st));
        FML_RC(tf32_lo(lm->wmlp_lo[l], lm->wmlp[l], d * fl, st));
    }
    lm->wlo_valid = true;
    return FML_OK;
}

// The bf16 copy of the decode weights (FML_WEIGHTS_BF16): allocated once,
// refilled after every bind.  Called before a step is enqueued or recorded
// (never inside a stream capture).
int ensure_weight_bf16(fml_lm* lm, cudaStream_t st)
{
    if (lm->weight_format != FML_WEIGHTS_BF16 || lm->wb16_valid) return FML_OK;
    const fml_lm_config& c = lm->cfg;
    const uint64_t d = c.d_model, dl = lm->dl, fl = lm->fl;
    const uint64_t per_layer = 3 * dl * d + d * dl + fl * d + d * fl;
    const uint64_t head = (uint64_t)lm->vl * d;
    if (!lm->wb16)
    {
        if (cudaMalloc(&lm->wb16, (per_layer * c.n_layer + head) * sizeof(uint16_t)) != cudaSuccess)
        {
            cudaGetLastError();
            lm->wb16 = nullptr;
            return set_error(FML_ERR_NOMEM, "bf16 weight copy: cudaMalloc of %llu bytes failed",
                             (unsigned long long)((per_layer * c.n_layer + head) * sizeof(uint16_t)));
        }
        uint16_t* p = lm->wb16;
        lm->wqkv_b.clear(); lm->wproj_b.clear(); lm->wfc_b.clear(); lm->wmlp_b.clear();
        for (uint32_t l = 0; l < c.n_layer; ++l)
        {
            lm->wqkv_b.push_back(p); p += 3 * dl * d;
            lm->wproj_b.push_back(p); p += d * dl;
            lm->wfc_b.push_back(p); p += fl * d;
            lm->wmlp_b.push_back(p); p += d * fl;
        }
        lm->head_b = p;
    }
    auto conv = [&](const uint16_t* dst, const float* src, uint64_t n) -> int {
        to_bf16_kernel<<<grid_for(n, 256), 256, 0, st>>>(const_cast<uint16_t*>(dst), src, n);
        FML_LAUNCH_CHECK();
        return FML_OK;
    };
    for (uint32_t l = 0; l < c.n_layer; ++l)
    {
        FML_RC(conv(lm->wqkv_b[l], lm->wqkv[l], 3 * dl * d));
        FML_RC(conv(lm->wproj_b[l], lm->wproj[l], d * dl));
        FML_RC(conv(lm->wfc_b[l], lm->wfc[l], fl * d));
        FML_RC(conv(lm->wmlp_b[l], lm->wmlp[l], d * fl));
    }
    FML_RC(conv(lm->head_b, lm->tok + (uint64_t)lm->v0 * d, head));
    lm->wb16_valid = true;
    return FML_OK;
}

// Prefill contraction C = A . W^T (W [N x K] K-contiguous) with an epilogue:
// 0 store, 1 GELU, 2 C = R + A . W^T.  Tensor cores (tcgen05, TF32x3 or
// TF32) unless the engine is set to fp32 CUDA-core math or the rows are not
// 16-byte multiples (a TMA row stride must be).
int prefill_gemm(fml_lm* lm, float* C, const float* A, const float* W, int M, int N, int K, int epi, const float* R,
                 cudaStream_t st, const float* W_lo = nullptr)
{
    if (lm->prefill_math != FML_MATH_FP32 && K % 4 == 0)
        return gemm_tc(C, A, W, M, N, K, K, K, N, lm->prefill_math == FML_MATH_TF32X3, epi, R, st,
                       lm->wlo_valid ? W_lo : nullptr);
    FML_RC(gemm_f32(C, A, W, M, N, K, K, K, N, true, 1, 0, 0, 0, st));
    const uint64_t n = (uint64_t)M * N;
    if (epi == 1) gelu_inplace_kernel<<<grid_for(n, 256), 256, 0, st>>>(C, n);
    else if (epi == 2) add_kernel<<<grid_for(n, 256), 256, 0, st>>>(C, R, C, n);
    if (epi) FML_LAUNCH_CHECK();
    return FML_OK;
}

}  // namespace

// y[M x N] = x[M x K] . w[N x K]^T for M <= 64 rows (fml_matmul's small-batch
// Mul<Right>): the decode GEMV without epilogue or programmatic launch.
int fml::gemv_nt(float* y, const float* x, const float* w, uint32_t M, uint32_t N, uint32_t K, cudaStream_t st)
{
    GemvArgs a{};
    a.x = x;
    a.ldx = K;
    a.w = w;
    a.M = M;
    a.N = N;
    a.K = K;
    a.y = y;
    a.ldy = N;
    return launch_gemv<EPI_STORE, false>(a, st, false);
}

namespace {

// Kernels one recorded step launches (counted when it was enqueued).
uint32_t graph_nodes_per_step(fml_lm* lm) { return lm->step_kernels; }

}  // namespace

extern "C" {

uint64_t fml_lm_param_count(const fml_lm_config* cfg) { return cfg ? param_count(*cfg) : 0; }

int fml_lm_create(const fml_lm_config* cfg, int device, fml_lm** out)
{
    FML_REQUIRE(cfg && out, "fml_lm_create: null argument");
    const fml_lm_config c = *cfg;
    FML_REQUIRE(c.vocab && c.context && c.d_model && c.n_head && c.n_layer && c.max_batch,
                "fml_lm_create: zero-sized dimension");
    FML_REQUIRE(c.d_model % c.n_head == 0, "fml_lm_create: d_model %% n_head != 0");
    const uint32_t hd = c.d_model / c.n_head;
    if (hd != 32 && hd != 64 && hd != 128)
        return set_error(FML_ERR_UNSUPPORTED, "fml_lm_create: head dim %u (need 32, 64 or 128)", hd);
    FML_REQUIRE(c.d_model % 4 == 0, "fml_lm_create: d_model must be a multiple of 4");
    FML_CUDA_TRY(cudaSetDevice(device));
    fml_lm* lm = new fml_lm();
    lm->cfg = c;
    lm->device = device;
    lm->hd = hd;
    lm->hpos.assign(c.max_batch, 0);
    lm->hl = c.n_head;
    lm->dl = c.d_model;
    lm->fl = 4 * c.d_model;
    lm->vl = c.vocab;

    const uint64_t d = c.d_model, B = c.max_batch, Ctx = c.context, L = c.n_layer, H = c.n_head;
    lm->seq_stride = H * Ctx * hd;
    lm->layer_stride = B * lm->seq_stride;
    const uint64_t rows = B * Ctx;

    attention_splits(B * H, Ctx, &lm->S, &lm->chunk);
    if (const char* e = getenv("FML_ATTN_SPLITS"))  // tuning override (keys split over S CTAs)
    {
        const long v = strtol(e, nullptr, 10);
        if (v >= 1 && v <= 64) lm->S = (uint32_t)v;
    }

    auto alloc = [&](void** p, uint64_t bytes) -> int {
        cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
        if (e != cudaSuccess)
        {
            cudaGetLastError();
            return set_error(FML_ERR_NOMEM, "cudaMalloc(%llu bytes) failed: %s", (unsigned long long)bytes,
                             cudaGetErrorString(e));
        }
        return FML_OK;
    };
    int rc = FML_OK;
    const uint64_t f = sizeof(float);
    if (!rc) rc = alloc((void**)&lm->wbuf, param_count(c) * f);
    if (!rc) rc = alloc((void**)&lm->kc, L * lm->layer_stride * f);
    if (!rc) rc = alloc((void**)&lm->vc, L * lm->layer_stride * f);
    if (!rc) rc = alloc((void**)&lm->x, rows * d * f);
    if (!rc) rc = alloc((void**)&lm->buf, rows * d * f);
    if (!rc) rc = alloc((void**)&lm->ln, rows * d * f);
    if (!rc) rc = alloc((void**)&lm->q, rows * d * f);
    if (!rc) rc = alloc((void**)&lm->att, rows * d * f);
    if (!rc) rc = alloc((void**)&lm->tmp, rows * 3 * d * f);
    if (!rc) rc = alloc((void**)&lm->hid, rows * 4 * d * f);
    if (!rc) rc = alloc((void**)&lm->pending, B * 4);
    if (!rc) rc = alloc((void**)&lm->pos, B * 4);
    if (!rc) rc = alloc((void**)&lm->prompt_dev, rows * 4);
    if (!rc) rc = alloc((void**)&lm->keys, B * 8);
    if (!rc) rc = alloc((void**)&lm->part, B * H * lm->S * (hd + 2) * f);
    if (!rc) rc = alloc((void**)&lm->counters, B * H * 4);
    if (!rc) rc = alloc((void**)&lm->grab, L * 4);
    if (!rc) rc = alloc((void**)&lm->stamp_step, 4);
    if (!rc && cudaMallocHost((void**)&lm->host_io, 2 * B * 4) != cudaSuccess)
        rc = set_error(FML_ERR_NOMEM, "cudaMallocHost failed");
    if (!rc && cudaHostGetDevicePointer((void**)&lm->host_io_dev, lm->host_io, 0) != cudaSuccess)
    {
        cudaGetLastError();
        lm->host_io_dev = nullptr;  // the host-buffer step keeps its copies
    }
    if (rc)
    {
        free_all(lm);
        delete lm;
        return rc;
    }
    cudaMemset(lm->pending, 0, B * 4);
    cudaMemset(lm->pos, 0, B * 4);
    cudaMemset(lm->keys, 0, B * 8);
    cudaMemset(lm->counters, 0, B * H * 4);
    cudaMemset(lm->grab, 0, L * 4);
    cudaMemset(lm->stamp_step, 0, 4);

    // carve the weight buffer
    float* p = lm->wbuf;
    lm->tok = p; p += (uint64_t)c.vocab * d;
    lm->pos_emb = p; p += Ctx * d;
    for (uint32_t l = 0; l < L; ++l)
    {
        lm->ln0.push_back(p); p += d;
        lm->wqkv.push_back(p); p += 3 * d * d;
        lm->wproj.push_back(p); p += d * d;
        lm->ln1.push_back(p); p += d;
        lm->wfc.push_back(p); p += 4 * d * d;
        lm->wmlp.push_back(p); p += 4 * d * d;
    }
    lm->lnf = p;
    FML_CUDA_TRY(cudaDeviceSynchronize());
    *out = lm;
    return FML_OK;
}

int fml_lm_get_config(const fml_lm* lm, fml_lm_config* out)
{
    FML_REQUIRE(lm && out, "fml_lm_get_config: null argument");
    *out = lm->cfg;
    return FML_OK;
}

int fml_lm_destroy(fml_lm* lm)
{
    if (!lm) return FML_OK;
    cudaSetDevice(lm->device);
    cudaDeviceSynchronize();
    free_all(lm);
    delete lm;
    return FML_OK;
}

int fml_lm_bind_weights(fml_lm* lm, const fml_lm_weights* w, fml_stream_t stream)
{
    FML_REQUIRE(lm && w && w->tok_emb && w->pos_emb && w->lnf && w->ln0 && w->wqkv && w->wproj && w->ln1 && w->wfc &&
                    w->wmlp,
                "fml_lm_bind_weights: null pointer");
    cudaStream_t st = as_stream(stream);
    const fml_lm_config& c = lm->cfg;
    const uint64_t d = c.d_model, f = sizeof(float);
    lm->wlo_valid = false;  // the lo parts follow the new weights at the next prefill
    lm->wb16_valid = false;  // and the bf16 copy at the next step
    FML_CUDA_TRY(cudaMemcpyAsync(lm->tok, w->tok_emb, (uint64_t)c.vocab * d * f, cudaMemcpyDeviceToDevice, st));
    FML_CUDA_TRY(cudaMemcpyAsync(lm->pos_emb, w->pos_emb, (uint64_t)c.context * d * f, cudaMemcpyDeviceToDevice, st));
    FML_CUDA_TRY(cudaMemcpyAsync(lm->lnf, w->lnf, d * f, cudaMemcpyDeviceToDevice, st));
    const dim3 tb(32, 8);
    auto tr = [&](float* dst, const float* src, uint32_t rows, uint32_t cols) -> int {
        FML_REQUIRE(src, "fml_lm_bind_weights: null layer weight");
        transpose_kernel<<<dim3((cols + 31) / 32, (rows + 31) / 32), tb, 0, st>>>(dst, src, rows, cols);
        FML_LAUNCH_CHECK();
        return FML_OK;
    };
    // tensor parallel: full transposes go through a scratch matrix, then
    // this rank's rows (column-parallel QKV / fc) or input columns
    // (row-parallel proj / mlp) are packed K-contiguous
    const bool tp = lm->tp_world > 1;
    float* scratch = nullptr;
    if (tp) FML_CUDA_TRY(cudaMalloc(&scratch, 4 * d * d * f));
    const uint64_t dl = lm->dl, fl = lm->fl, hoff = (uint64_t)lm->h0 * lm->hd, j0 = lm->j0;
    int rc = FML_OK;
    for (uint32_t l = 0; l < c.n_layer && rc == FML_OK; ++l)
    {
        if (!(w->ln0[l] && w->ln1[l] && w->wproj[l]))
        {
            rc = set_error(FML_ERR_INVALID, "fml_lm_bind_weights: null layer weight");
            break;
        }
        auto cp = [&](void* dst, const void* src, uint64_t bytes) {
            if (rc == FML_OK && cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
                rc = set_error(FML_ERR_CUDA, "fml_lm_bind_weights: copy failed");
        };
        auto cp2d = [&](void* dst, uint64_t dpitch, const void* src, uint64_t spitch, uint64_t width, uint64_t h) {
            if (rc == FML_OK &&
                cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, h, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
                rc = set_error(FML_ERR_CUDA, "fml_lm_bind_weights: strided copy failed");
        };
        cp(lm->ln0[l], w->ln0[l], d * f);
        cp(lm->ln1[l], w->ln1[l], d * f);
        if (!tp)
        {
            cp(lm->wproj[l], w->wproj[l], d * d * f);
            if (rc == FML_OK) rc = tr(lm->wqkv[l], w->wqkv[l], (uint32_t)d, (uint32_t)(3 * d));
            if (rc == FML_OK) rc = tr(lm->wfc[l], w->wfc[l], (uint32_t)d, (uint32_t)(4 * d));
            if (rc == FML_OK) rc = tr(lm->wmlp[l], w->wmlp[l], (uint32_t)(4 * d), (uint32_t)d);
            continue;
        }
        // QKV [d x 3d] -> rows q|k|v of this rank's heads, each [dl x d]
        if (rc == FML_OK) rc = tr(scratch, w->wqkv[l], (uint32_t)d, (uint32_t)(3 * d));
        for (uint64_t part = 0; part < 3; ++part)
            cp(lm->wqkv[l] + part * dl * d, scratch + (part * d + hoff) * d, dl * d * f);
        // proj (out x in) -> its input columns of this rank's heads [d x dl]
        cp2d(lm->wproj[l], dl * f, w->wproj[l] + hoff, d * f, dl * f, d);
        // fc [d x 4d] -> this rank's fc rows [fl x d]
        if (rc == FML_OK) rc = tr(scratch, w->wfc[l], (uint32_t)d, (uint32_t)(4 * d));
        cp(lm->wfc[l], scratch + j0 * d, fl * d * f);
        // mlp [4d x d] -> [d x 4d] -> its input columns [d x fl]
        if (rc == FML_OK) rc = tr(scratch, w->wmlp[l], (uint32_t)(4 * d), (uint32_t)d);
        cp2d(lm->wmlp[l], fl * f, scratch + j0, 4 * d * f, fl * f, d);
    }
    const cudaError_t se = cudaStreamSynchronize(st);
    if (scratch) cudaFree(scratch);
    if (rc != FML_OK) return rc;
    if (se != cudaSuccess) return set_error(FML_ERR_CUDA, "fml_lm_bind_weights: %s", cudaGetErrorString(se));
    lm->bound = true;
    return FML_OK;
}

int fml_lm_bind_packed(fml_lm* lm, const float* params, int params_on_host, fml_stream_t stream)
{
    FML_REQUIRE(lm && params, "fml_lm_bind_packed: null argument");
    const fml_lm_config& c = lm->cfg;
    const uint64_t n = param_count(c), d = c.d_model;
    const float* src = params;
    float* staging = nullptr;
    if (params_on_host)
    {
        FML_CUDA_TRY(cudaMalloc(&staging, n * sizeof(float)));
        cudaError_t e = cudaMemcpy(staging, params, n * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess)
        {
            cudaFree(staging);
            return set_error(FML_ERR_CUDA, "cudaMemcpy params: %s", cudaGetErrorString(e));
        }
        src = staging;
    }
    std::vector<const float*> ln0, wqkv, wproj, ln1, wfc, wmlp;
    const float* p = src + (uint64_t)c.vocab * d + (uint64_t)c.context * d;
    for (uint32_t l = 0; l < c.n_layer; ++l)
    {
        ln0.push_back(p); p += d;
        wqkv.push_back(p); p += 3 * d * d;
        wproj.push_back(p); p += d * d;
        ln1.push_back(p); p += d;
        wfc.push_back(p); p += 4 * d * d;
        wmlp.push_back(p); p += 4 * d * d;
    }
    fml_lm_weights w{};
    w.tok_emb = src;
    w.pos_emb = src + (uint64_t)c.vocab * d;
    w.ln0 = ln0.data(); w.wqkv = wqkv.data(); w.wproj = wproj.data();
    w.ln1 = ln1.data(); w.wfc = wfc.data(); w.wmlp = wmlp.data();
    w.lnf = p;
    int rc = fml_lm_bind_weights(lm, &w, stream);
    if (staging) cudaFree(staging);
    return rc;
}

int fml_lm_prefill(fml_lm* lm, const uint32_t* prompts, uint32_t batch, uint32_t P, fml_stream_t stream)
{
    FML_REQUIRE(lm && prompts, "fml_lm_prefill: null argument");
    if (!lm->bound) return set_error(FML_ERR_STATE, "fml_lm_prefill: weights not bound");
    const fml_lm_config& c = lm->cfg;
    FML_REQUIRE(batch >= 1 && batch <= c.max_batch, "fml_lm_prefill: batch %u outside [1, %u]", batch, c.max_batch);
    FML_REQUIRE(P >= 1 && P < c.context, "fml_lm_prefill: prompt length %u outside [1, %u)", P, c.context);
    cudaStream_t st = as_stream(stream);
    const uint32_t d = c.d_model, R = batch * P;
    lm->batch = batch;
    FML_CUDA_TRY(cudaMemcpyAsync(lm->prompt_dev, prompts, (uint64_t)R * 4, cudaMemcpyDeviceToDevice, st));
    FML_CUDA_TRY(cudaMemsetAsync(lm->keys, 0, (uint64_t)c.max_batch * 8, st));
    embed_kernel<<<R < 65535u ? R : 65535u, 128, 0, st>>>(lm->x, lm->tok, lm->pos_emb, lm->prompt_dev, nullptr, R, P, d,
                                                          c.vocab, c.context, nullptr, 0u, StepStamp{});
    FML_LAUNCH_CHECK();
    const bool tp = lm->tp_world > 1;
    const int resid_epi = lm->tp_rank == 0 ? 2 : 0;  // row-parallel sums take the residual once
    FML_RC(ensure_weight_lo(lm, st));
    for (uint32_t l = 0; l < c.n_layer; ++l)
    {
        float* kc = lm->kc + (uint64_t)l * lm->layer_stride;
        float* vc = lm->vc + (uint64_t)l * lm->layer_stride;
        const uint32_t dl = lm->dl, fl = lm->fl;
        FML_RC(launch_layernorm(lm->ln, lm->x, lm->ln0[l], nullptr, nullptr, R, d, d, d, 1e-5f, st));
        // QKV: on the tensor cores the epilogue writes q and the cached K/V
        // rows directly (measured on config 3's prefill: the separate scatter
        // took 26.5 us of every layer's ~250); otherwise packed rows + scatter
        if (lm->prefill_math != FML_MATH_FP32 && d % 4 == 0 && dl % 32 == 0 && lm->hd % 32 == 0)
            FML_RC(gemm_tc_qkv(lm->q, (int)dl, kc, vc, lm->seq_stride, (int)P, (int)lm->hd, (int)c.context, lm->ln,
                               lm->wqkv[l], (int)R, (int)dl, (int)d, lm->prefill_math == FML_MATH_TF32X3, st,
                               lm->wlo_valid ? lm->wqkv_lo[l] : nullptr));
        else
        {
            FML_RC(prefill_gemm(lm, lm->tmp, lm->ln, lm->wqkv[l], (int)R, (int)(3 * dl), (int)d, 0, nullptr, st,
                                lm->wlo_valid ? lm->wqkv_lo[l] : nullptr));
            qkv_scatter_kernel<<<grid_for((uint64_t)R * 3 * dl, 256), 256, 0, st>>>(lm->tmp, lm->q, kc, vc, R, P, dl,
                                                                                   lm->hd, c.context, lm->seq_stride);
            FML_LAUNCH_CHECK();
        }
        // prefill attention: tensor cores in the TF32 modes (128-query tiles),
        // else (or for a layout that kernel does not take) the CUDA-core kernel
        {
            const float scale = 1.0f / sqrtf((float)lm->hd);
            int rc = FML_ERR_UNSUPPORTED;
            const char* pa_env = getenv("FML_PREFILL_ATTN_SIMT");  // tuning: 1 = the CUDA-core kernel
            if (lm->prefill_math != FML_MATH_FP32 && !(pa_env && pa_env[0] == '1'))
                rc = launch_prefill_attention_tc(lm->q, dl, kc, vc, lm->seq_stride, c.context, lm->att, dl, batch,
                                                 lm->hl, P, lm->hd, scale, lm->prefill_math == FML_MATH_TF32X3, st);
            if (rc == FML_ERR_UNSUPPORTED)
                rc = launch_prefill_attention(lm->q, dl, kc, vc, lm->seq_stride, c.context, lm->att, dl, batch, lm->hl,
                                              P, lm->hd, scale, st);
            FML_RC(rc);
        }
        // buf = x + att . Wproj^T ; hid = gelu(LN1(buf) . Wfc^T) ; x = buf + hid . Wmlp^T
        FML_RC(prefill_gemm(lm, lm->buf, lm->att, lm->wproj[l], (int)R, (int)d, (int)dl, resid_epi, lm->x, st,
                            lm->wlo_valid ? lm->wproj_lo[l] : nullptr));
        if (tp) FML_RC(all_reduce_sum(lm, lm->buf, (uint64_t)R * d, st));
        FML_RC(launch_layernorm(lm->ln, lm->buf, lm->ln1[l], nullptr, nullptr, R, d, d, d, 1e-5f, st));
        FML_RC(prefill_gemm(lm, lm->hid, lm->ln, lm->wfc[l], (int)R, (int)fl, (int)d, 1, nullptr, st,
                            lm->wlo_valid ? lm->wfc_lo[l] : nullptr));
        FML_RC(prefill_gemm(lm, lm->x, lm->hid, lm->wmlp[l], (int)R, (int)d, (int)fl, resid_epi, lm->buf, st,
                            lm->wlo_valid ? lm->wmlp_lo[l] : nullptr));
        if (tp) FML_RC(all_reduce_sum(lm, lm->x, (uint64_t)R * d, st));
    }
    // last prompt row of each sequence -> ln_f -> lm_head argmax
    FML_RC(launch_layernorm(lm->ln, lm->x + (uint64_t)(P - 1) * d, lm->lnf, nullptr, nullptr, batch, d,
                            (uint64_t)P * d, d, 1e-5f, st));
    GemvArgs a{};
    a.x = lm->ln; a.ldx = d; a.w = lm->tok + (uint64_t)lm->v0 * d; a.M = batch; a.N = lm->vl; a.K = d; a.y = nullptr;
    a.ldy = lm->vl; a.keys = lm->keys; a.n_off = lm->v0;
    FML_RC((launch_gemv<EPI_ARGMAX, false>(a, st, false)));
    if (tp) FML_RC(all_reduce_max_keys(lm, batch, st));
    finalize_kernel<<<(batch + 127) / 128, 128, 0, st>>>(lm->keys, lm->pending, lm->pos, nullptr, batch, P,
                                                         lm->ar_epoch, StepStamp{}, nullptr);
    FML_LAUNCH_CHECK();
    for (uint32_t b = 0; b < batch; ++b) lm->hpos[b] = P;
    return FML_OK;
}

int fml_lm_set_prefill_math(fml_lm* lm, int mode)
{
    FML_REQUIRE(lm, "fml_lm_set_prefill_math: null engine");
    FML_REQUIRE(mode == FML_MATH_FP32 || mode == FML_MATH_TF32X3 || mode == FML_MATH_TF32, "unknown math mode %d",
                mode);
    lm->prefill_math = mode;
    return FML_OK;
}

int fml_lm_set_weight_format(fml_lm* lm, int format)
{
    FML_REQUIRE(lm, "fml_lm_set_weight_format: null engine");
    FML_REQUIRE(format == FML_WEIGHTS_FP32 || format == FML_WEIGHTS_BF16, "unknown weight format %d", format);
    if (lm->weight_format == format) return FML_OK;
    lm->weight_format = format;
    lm->wb16_valid = false;
    drop_graphs(lm);  // the recorded steps read the other weights
    if (format == FML_WEIGHTS_FP32 && lm->wb16)
    {
        cudaFree(lm->wb16);
        lm->wb16 = nullptr;
    }
    return FML_OK;
}

int fml_nccl_unique_id(void* out)
{
    FML_REQUIRE(out, "fml_nccl_unique_id: null argument");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return set_error(FML_ERR_CUDA, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    std::memcpy(out, &id, sizeof(id));
    return FML_OK;
}

int fml_lm_set_tensor_parallel(fml_lm* lm, int rank, int world, const void* nccl_id)
{
    FML_REQUIRE(lm && world >= 1 && rank >= 0 && rank < world, "fml_lm_set_tensor_parallel: bad rank/world");
    FML_REQUIRE(!lm->bound, "fml_lm_set_tensor_parallel: call before binding weights");
    FML_REQUIRE(!lm->comm, "fml_lm_set_tensor_parallel: already set");
    const fml_lm_config& c = lm->cfg;
    FML_REQUIRE(c.n_head % (uint32_t)world == 0 && (4 * c.d_model) % (uint32_t)world == 0 &&
                    c.vocab >= (uint32_t)world,
                "fml_lm_set_tensor_parallel: %u heads / 4*%u fc columns / vocab %u do not split over %d ranks",
                c.n_head, c.d_model, c.vocab, world);
    if (world == 1) return FML_OK;
    FML_REQUIRE(nccl_id, "fml_lm_set_tensor_parallel: null NCCL id");
    FML_CUDA_TRY(cudaSetDevice(lm->device));
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t r = ncclCommInitRank(&lm->comm, world, id, rank);
    if (r != ncclSuccess)
    {
        lm->comm = nullptr;
        return set_error(FML_ERR_CUDA, "ncclCommInitRank: %s", ncclGetErrorString(r));
    }
    lm->tp_rank = rank;
    lm->tp_world = world;
    lm->hl = c.n_head / world;
    lm->h0 = rank * lm->hl;
    lm->dl = lm->hl * lm->hd;
    lm->fl = 4 * c.d_model / world;
    lm->j0 = rank * lm->fl;
    lm->vl = (c.vocab + world - 1) / world;
    lm->v0 = rank * lm->vl;
    if (lm->v0 + lm->vl > c.vocab) lm->vl = c.vocab - lm->v0;
    // this rank's heads only in the cache and in the attention splits
    lm->seq_stride = (uint64_t)lm->hl * c.context * lm->hd;
    lm->layer_stride = (uint64_t)c.max_batch * lm->seq_stride;
    attention_splits((uint64_t)c.max_batch * lm->hl, c.context, &lm->S, &lm->chunk);
    if (lm->part) cudaFree(lm->part);
    lm->part = nullptr;
    FML_CUDA_TRY(cudaMalloc(&lm->part, (uint64_t)c.max_batch * lm->hl * lm->S * (lm->hd + 2) * sizeof(float)));
    // buffers the fused all-reduce shares with the other ranks (fml_lm_tp_connect)
    FML_CUDA_TRY(cudaMalloc(&lm->ar_part, 2ull * c.max_batch * c.d_model * sizeof(float)));
    FML_CUDA_TRY(cudaMalloc(&lm->ar_flags, (uint64_t)world * AR_CTAS * sizeof(uint32_t)));
    FML_CUDA_TRY(cudaMalloc(&lm->ar_epoch, sizeof(uint32_t)));
    FML_CUDA_TRY(cudaMemset(lm->ar_flags, 0, (uint64_t)world * AR_CTAS * sizeof(uint32_t)));
    FML_CUDA_TRY(cudaMemset(lm->ar_epoch, 0, sizeof(uint32_t)));
    drop_graphs(lm);
    return FML_OK;
}

int fml_lm_tp_ipc_handles(fml_lm* lm, void* out)
{
    FML_REQUIRE(lm && out, "fml_lm_tp_ipc_handles: null argument");
    FML_REQUIRE(lm->tp_world > 1 && lm->ar_part, "fml_lm_tp_ipc_handles: call fml_lm_set_tensor_parallel first");
    cudaIpcMemHandle_t h[2];
    FML_CUDA_TRY(cudaIpcGetMemHandle(&h[0], lm->ar_part));
    FML_CUDA_TRY(cudaIpcGetMemHandle(&h[1], lm->ar_flags));
    std::memcpy(out, h, sizeof(h));
    return FML_OK;
}

int fml_lm_tp_connect(fml_lm* lm, const void* all)
{
    FML_REQUIRE(lm && all, "fml_lm_tp_connect: null argument");
    FML_REQUIRE(lm->tp_world > 1 && lm->ar_part, "fml_lm_tp_connect: call fml_lm_set_tensor_parallel first");
    FML_REQUIRE(!lm->ar_fused, "fml_lm_tp_connect: already connected");
    const int world = lm->tp_world;
    std::vector<float*> recv(world);
    std::vector<uint32_t*> flags(world);
    const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(all);
    for (int r = 0; r < world; ++r)
    {
        if (r == lm->tp_rank)
        {
            recv[r] = lm->ar_part;
            flags[r] = lm->ar_flags;
            continue;
        }
        void* p = nullptr;
        FML_CUDA_TRY(cudaIpcOpenMemHandle(&p, h[2 * r], cudaIpcMemLazyEnablePeerAccess));
        lm->ar_opened.push_back(p);
        recv[r] = static_cast<float*>(p);
        FML_CUDA_TRY(cudaIpcOpenMemHandle(&p, h[2 * r + 1], cudaIpcMemLazyEnablePeerAccess));
        lm->ar_opened.push_back(p);
        flags[r] = static_cast<uint32_t*>(p);
    }
    FML_CUDA_TRY(cudaMalloc(&lm->ar_peer_part, world * sizeof(float*)));
    FML_CUDA_TRY(cudaMalloc(&lm->ar_peer_flags, world * sizeof(uint32_t*)));
    FML_CUDA_TRY(cudaMemcpy(lm->ar_peer_part, recv.data(), world * sizeof(float*), cudaMemcpyHostToDevice));
    FML_CUDA_TRY(cudaMemcpy(lm->ar_peer_flags, flags.data(), world * sizeof(uint32_t*), cudaMemcpyHostToDevice));
    lm->ar_fused = true;
    drop_graphs(lm);
    return FML_OK;
}

int fml_tp_flag_check(uint32_t epoch, uint32_t slot, uint32_t nslot, uint32_t flag, int* reached)
{
    FML_REQUIRE(reached, "fml_tp_flag_check: null argument");
    FML_REQUIRE(slot < nslot, "fml_tp_flag_check: slot %u outside [0, %u)", slot, nslot);
    *reached = ar_flag_reached(flag, ar_tag(epoch, slot, nslot)) ? 1 : 0;
    return FML_OK;
}

int fml_lm_tp_error_count(uint64_t* out)
{
    FML_REQUIRE(out, "fml_lm_tp_error_count: null argument");
    unsigned int v = 0;
    FML_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tp_timeouts, sizeof(v)));
    *out = v;
    return FML_OK;
}

int fml_lm_set_stamps(fml_lm* lm, unsigned long long* stamps, uint32_t cap, uint32_t* stride)
{
    FML_REQUIRE(lm, "fml_lm_set_stamps: null engine");
    FML_REQUIRE(!stamps || aligned16(stamps), "fml_lm_set_stamps: the buffer must be 16-byte aligned");
    lm->stamps = cap ? stamps : nullptr;
    lm->stamp_cap = lm->stamps ? cap : 0u;
    // an upper bound of the kernels of one step: embed, per layer the QKV,
    // attention, proj and mlp GEMVs (with their all-reduce kernels under
    // tensor parallelism) and fc, lm_head, finalize
    lm->stamp_stride = 3u + 7u * lm->cfg.n_layer;
    if (stride) *stride = lm->stamp_stride;
    FML_CUDA_TRY(cudaMemset(lm->stamp_step, 0, 4));
    drop_graphs(lm);
    return FML_OK;
}

int fml_lm_stamp_classes(fml_lm* lm, int* classes, uint32_t n, uint32_t* kernels)
{
    FML_REQUIRE(lm && kernels, "fml_lm_stamp_classes: null argument");
    *kernels = (uint32_t)lm->stamp_class.size();
    for (uint32_t i = 0; i < n && i < lm->stamp_class.size(); ++i) classes[i] = lm->stamp_class[i];
    return FML_OK;
}

int fml_lm_set_graph(fml_lm* lm, int use_graph)
{
    FML_REQUIRE(lm, "fml_lm_set_graph: null engine");
    lm->use_graph = use_graph != 0;
    return FML_OK;
}

}  // extern "C"

namespace {

// A step may run only while every sequence has room for one more key.
int check_step_state(fml_lm* lm, const char* fn)
{
    if (!lm->bound || lm->batch == 0) return set_error(FML_ERR_STATE, "%s: call fml_lm_prefill first", fn);
    for (uint32_t b = 0; b < lm->batch; ++b)
        if (lm->hpos[b] >= lm->cfg.context)
            return set_error(FML_ERR_STATE, "%s: sequence %u is at the context limit (%u)", fn, b, lm->cfg.context);
    return FML_OK;
}

// Record one step into an executable graph.  With host_io the step takes
// its tokens from host_io[0, B) and leaves the next tokens in
// host_io[max_batch, max_batch + B) (pinned host memory): the step's first
// kernel reads them over the host link and its last kernel writes them back
// (mapped memory; otherwise copies bracket it).
int record_step(fml_lm* lm, uint32_t* next_tokens, float* logits, bool host_io, cudaGraphExec_t* out)
{
    *out = nullptr;
    const uint32_t B = lm->batch;
    const bool mapped = host_io && lm->host_io_dev;
    cudaStream_t cap;
    FML_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    FML_CUDA_TRY(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal));
    int rc = FML_OK;
    if (mapped) rc = enqueue_step(lm, lm->host_io_dev + lm->cfg.max_batch, logits, cap, lm->host_io_dev);
    else
    {
        if (host_io && cudaMemcpyAsync(lm->pending, lm->host_io, B * 4, cudaMemcpyHostToDevice, cap) != cudaSuccess)
            rc = set_error(FML_ERR_CUDA, "graph capture: token upload");
        if (!rc) rc = enqueue_step(lm, next_tokens, logits, cap);
        if (!rc && host_io &&
            cudaMemcpyAsync(lm->host_io + lm->cfg.max_batch, next_tokens, B * 4, cudaMemcpyDeviceToHost, cap) !=
                cudaSuccess)
            rc = set_error(FML_ERR_CUDA, "graph capture: token download");
    }
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(cap, &g);
    cudaStreamDestroy(cap);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    // capture counted the launches once; replays are counted at launch
    launch_counter().fetch_sub(graph_nodes_per_step(lm), std::memory_order_relaxed);
    return FML_OK;
}

// Record `n` consecutive steps (no outputs: each step leaves its tokens
// pending on the device) into one executable graph.
int record_steps(fml_lm* lm, uint32_t n, cudaGraphExec_t* out)
{
    *out = nullptr;
    cudaStream_t cap;
    FML_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    FML_CUDA_TRY(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal));
    int rc = FML_OK;
    for (uint32_t i = 0; i < n && rc == FML_OK; ++i) rc = enqueue_step(lm, nullptr, nullptr, cap, nullptr, i > 0);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(cap, &g);
    cudaStreamDestroy(cap);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    launch_counter().fetch_sub((uint64_t)n * graph_nodes_per_step(lm), std::memory_order_relaxed);
    return FML_OK;
}

// Enqueue one host-buffer step: tokens from host_io[0, B) in, the next
// tokens to host_io[max_batch, max_batch + B) out (read after a sync).
int enqueue_step_host(fml_lm* lm, cudaStream_t st)
{
    FML_RC(check_step_state(lm, "fml_lm_step_host"));
    FML_RC(ensure_weight_bf16(lm, st));
    FML_RC(prepare_tc_decode(lm));
    const uint32_t B = lm->batch;
    uint32_t* dev_next = lm->prompt_dev;  // scratch slot for the step's output tokens
    if (lm->use_graph && !lm->profiling)
    {
        if (!lm->host_graph_exec || lm->host_graph_batch != B)
        {
            if (lm->host_graph_exec) cudaGraphExecDestroy(lm->host_graph_exec);
            lm->host_graph_exec = nullptr;
            FML_RC(record_step(lm, dev_next, nullptr, true, &lm->host_graph_exec));
            lm->host_graph_batch = B;
        }
        FML_CUDA_TRY(cudaGraphLaunch(lm->host_graph_exec, st));
        launch_counter().fetch_add(graph_nodes_per_step(lm), std::memory_order_relaxed);
        for (uint32_t b = 0; b < B; ++b) lm->hpos[b] += 1;
        return FML_OK;
    }
    FML_CUDA_TRY(cudaMemcpyAsync(lm->pending, lm->host_io, B * 4, cudaMemcpyHostToDevice, st));
    FML_RC(fml_lm_step(lm, dev_next, nullptr, reinterpret_cast<fml_stream_t>(st)));
    FML_CUDA_TRY(cudaMemcpyAsync(lm->host_io + lm->cfg.max_batch, dev_next, B * 4, cudaMemcpyDeviceToHost, st));
    return FML_OK;
}

}  // namespace

extern "C" {

int fml_lm_step(fml_lm* lm, uint32_t* next_tokens, float* logits, fml_stream_t stream)
{
    FML_REQUIRE(lm, "fml_lm_step: null engine");
    FML_RC(check_step_state(lm, "fml_lm_step"));
    cudaStream_t st = as_stream(stream);
    FML_RC(ensure_weight_bf16(lm, st));
    FML_RC(prepare_tc_decode(lm));  // no attribute call inside a capture
    if (lm->use_graph && !lm->profiling)
    {
        if (!lm->graph_exec || lm->graph_next != next_tokens || lm->graph_logits != logits ||
            lm->graph_batch != lm->batch)
        {
            if (lm->graph_exec) cudaGraphExecDestroy(lm->graph_exec);
            lm->graph_exec = nullptr;
            FML_RC(record_step(lm, next_tokens, logits, false, &lm->graph_exec));
            lm->graph_next = next_tokens;
            lm->graph_logits = logits;
            lm->graph_batch = lm->batch;
        }
        FML_CUDA_TRY(cudaGraphLaunch(lm->graph_exec, st));
        launch_counter().fetch_add(graph_nodes_per_step(lm), std::memory_order_relaxed);
    }
    else
    {
        FML_RC(enqueue_step(lm, next_tokens, logits, st));
        if (lm->profiling) FML_RC(collect_profile(lm));
    }
    for (uint32_t b = 0; b < lm->batch; ++b) lm->hpos[b] += 1;
    return FML_OK;
}

int fml_lm_steps(fml_lm* lm, uint32_t n, fml_stream_t stream)
{
    FML_REQUIRE(lm, "fml_lm_steps: null engine");
    if (n == 0) return FML_OK;
    FML_RC(check_step_state(lm, "fml_lm_steps"));
    for (uint32_t b = 0; b < lm->batch; ++b)
        if ((uint64_t)lm->hpos[b] + n > lm->cfg.context)  // 64-bit: no wrap for any n
            return set_error(FML_ERR_STATE, "fml_lm_steps: %u steps take sequence %u past the context limit (%u)", n,
                             b, lm->cfg.context);
    cudaStream_t st = as_stream(stream);
    FML_RC(ensure_weight_bf16(lm, st));
    FML_RC(prepare_tc_decode(lm));
    if (!lm->use_graph || lm->profiling)
    {
        for (uint32_t i = 0; i < n; ++i) FML_RC(fml_lm_step(lm, nullptr, nullptr, stream));
        return FML_OK;
    }
    // graphs of G steps (FML_LM_GRAPH_STEPS, default 16), then one graph of
    // the remaining n mod G steps
    uint32_t G = 16;
    if (const char* e = getenv("FML_LM_GRAPH_STEPS"))
    {
        const long v = strtol(e, nullptr, 10);
        if (v >= 1 && v <= 256) G = (uint32_t)v;
    }
    if (lm->multi_graph_batch != lm->batch)
    {
        for (auto& g : lm->multi_graphs) cudaGraphExecDestroy(g.second);
        lm->multi_graphs.clear();
        lm->multi_graph_batch = lm->batch;
    }
    auto graph_of = [&](uint32_t k, cudaGraphExec_t* out) -> int {
        for (auto& g : lm->multi_graphs)
            if (g.first == k) { *out = g.second; return FML_OK; }
        if (lm->multi_graphs.size() >= 4)  // keep a few sizes only
        {
            cudaGraphExecDestroy(lm->multi_graphs.front().second);
            lm->multi_graphs.erase(lm->multi_graphs.begin());
        }
        FML_RC(record_steps(lm, k, out));
        lm->multi_graphs.emplace_back(k, *out);
        return FML_OK;
    };
    for (uint32_t done = 0; done < n;)
    {
        const uint32_t k = std::min(G, n - done);
        cudaGraphExec_t ge = nullptr;
        FML_RC(graph_of(k, &ge));
        FML_CUDA_TRY(cudaGraphLaunch(ge, st));
        launch_counter().fetch_add((uint64_t)k * graph_nodes_per_step(lm), std::memory_order_relaxed);
        for (uint32_t b = 0; b < lm->batch; ++b) lm->hpos[b] += k;
        done += k;
    }
    return FML_OK;
}

int fml_lm_step_host(fml_lm* lm, const uint32_t* tokens_in, uint32_t* tokens_out, fml_stream_t stream)
{
    FML_REQUIRE(lm && tokens_in && tokens_out, "fml_lm_step_host: null argument");
    if (lm->batch == 0) return set_error(FML_ERR_STATE, "fml_lm_step_host: call fml_lm_prefill first");
    cudaStream_t st = as_stream(stream);
    const uint32_t B = lm->batch;
    std::memcpy(lm->host_io, tokens_in, B * 4);
    FML_RC(enqueue_step_host(lm, st));
    FML_CUDA_TRY(cudaStreamSynchronize(st));
    std::memcpy(tokens_out, lm->host_io + lm->cfg.max_batch, B * 4);
    return FML_OK;
}

int fml_lm_generate_host(fml_lm* lm, uint32_t steps, const uint32_t* tokens_in, uint32_t* tokens_out,
                         fml_stream_t stream)
{
    FML_REQUIRE(lm && tokens_in && tokens_out, "fml_lm_generate_host: null argument");
    if (lm->batch == 0) return set_error(FML_ERR_STATE, "fml_lm_generate_host: call fml_lm_prefill first");
    cudaStream_t st = as_stream(stream);
    const uint32_t B = lm->batch;
    for (uint32_t t = 0; t < steps; ++t)
    {
        // every step's tokens go up from the host and come back before the next
        std::memcpy(lm->host_io, t == 0 ? tokens_in : tokens_out + (uint64_t)(t - 1) * B, B * 4);
        FML_RC(enqueue_step_host(lm, st));
        FML_CUDA_TRY(cudaStreamSynchronize(st));
        std::memcpy(tokens_out + (uint64_t)t * B, lm->host_io + lm->cfg.max_batch, B * 4);
    }
    return FML_OK;
}

int fml_lm_pending(fml_lm* lm, uint32_t* out, fml_stream_t stream)
{
    FML_REQUIRE(lm && out, "fml_lm_pending: null argument");
    if (lm->batch == 0) return set_error(FML_ERR_STATE, "fml_lm_pending: no active sequences");
    FML_CUDA_TRY(cudaMemcpyAsync(out, lm->pending, lm->batch * 4, cudaMemcpyDeviceToDevice, as_stream(stream)));
    return FML_OK;
}

int fml_lm_get_position(fml_lm* lm, uint32_t b, uint32_t* pos)
{
    FML_REQUIRE(lm && pos && b < lm->cfg.max_batch, "fml_lm_get_position: bad argument");
    *pos = lm->hpos[b];
    return FML_OK;
}

int fml_lm_rewind(fml_lm* lm, uint32_t pos, const uint32_t* pending, int pending_on_host, fml_stream_t stream)
{
    FML_REQUIRE(lm && pending, "fml_lm_rewind: null argument");
    FML_REQUIRE(lm->batch > 0 && pos >= 1 && pos < lm->cfg.context, "fml_lm_rewind: bad position %u", pos);
    cudaStream_t st = as_stream(stream);
    const uint32_t B = lm->batch;
    for (uint32_t b = 0; b < B; ++b)  // rows past a sequence's position were never written
        FML_REQUIRE(pos <= lm->hpos[b], "fml_lm_rewind: position %u is past sequence %u's %u cached rows", pos, b,
                    lm->hpos[b]);
    if (pending_on_host)
    {
        FML_CUDA_TRY(cudaStreamSynchronize(st));  // host_io may still feed an earlier copy
        std::memcpy(lm->host_io, pending, B * 4);
        FML_CUDA_TRY(cudaMemcpyAsync(lm->pending, lm->host_io, B * 4, cudaMemcpyHostToDevice, st));
        rewind_kernel<<<(B + 127) / 128, 128, 0, st>>>(lm->pos, lm->pending, nullptr, B, pos);
        FML_LAUNCH_CHECK();
        FML_CUDA_TRY(cudaStreamSynchronize(st));
    }
    else
    {
        rewind_kernel<<<(B + 127) / 128, 128, 0, st>>>(lm->pos, lm->pending, pending, B, pos);
        FML_LAUNCH_CHECK();
    }
    for (uint32_t b = 0; b < B; ++b) lm->hpos[b] = pos;
    return FML_OK;
}

uint64_t fml_lm_step_bytes(fml_lm* lm)
{
    if (!lm) return 0;
    const fml_lm_config& c = lm->cfg;
    const uint64_t d = c.d_model, L = c.n_layer, f = 4, dl = lm->dl, fl = lm->fl;
    // this rank's weights once (all of them on one rank)
    uint64_t bytes = f * (L * (4 * d * dl + 2 * d * fl) + (uint64_t)lm->vl * d + (2 * L + 1) * d);
    for (uint32_t b = 0; b < lm->batch; ++b)
    {
        const uint64_t len = lm->hpos[b] + 1;  // keys/values read this step, including the new row
        bytes += f * 2 * dl * L * len;         // K and V rows read (this rank's heads)
        bytes += f * 2 * dl * L;               // the new K and V rows written
        bytes += f * 2 * d;                    // token + position rows
    }
    return bytes;
}

uint64_t fml_lm_attention_bytes(fml_lm* lm)
{
    if (!lm) return 0;
    const fml_lm_config& c = lm->cfg;
    const uint64_t d = c.d_model, L = c.n_layer, f = 4;
    uint64_t bytes = 0;
    for (uint32_t b = 0; b < lm->batch; ++b)
        bytes += f * L * (2 * d * (uint64_t)(lm->hpos[b] + 1) + 2 * d);  // K,V rows + q in + out
    return bytes;
}

int fml_lm_set_profiling(fml_lm* lm, int on)
{
    FML_REQUIRE(lm, "fml_lm_set_profiling: null engine");
    lm->profiling = on != 0;
    for (int i = 0; i < FML_LM_NCLASS; ++i) { lm->prof_ms[i] = 0; lm->prof_n[i] = 0; }
    return FML_OK;
}

int fml_lm_get_profile(fml_lm* lm, double* ms, uint64_t* n, int ncls)
{
    FML_REQUIRE(lm && ms && n, "fml_lm_get_profile: null argument");
    for (int i = 0; i < ncls && i < FML_LM_NCLASS; ++i) { ms[i] = lm->prof_ms[i]; n[i] = lm->prof_n[i]; }
    return FML_OK;
}

}  // extern "C"
