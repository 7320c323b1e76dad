// Decode contractions on the tensor cores: y = LN(x) . W^T for the few rows
// of a decode step (the B sequences), with the step's epilogues fused -- the
// QKV projection with its K/V-cache scatter (CausalSelfAttentionLayer.h:
// 424-445 over Dense.h:179-223), fc + GELU (Dense<Gelu>, Gelu.h:32-38),
// projection / mlp + residual (AddLayer.h:131-165) and the tied lm_head with
// the greedy argmax keys (NanoLLM.cpp:189-204).  LN is LayerNormOp
// (MatrixBase_Functions.h:482-549) of every x row, fused as the prologue.
//
// Shape.  D[n, b] = sum_k W[n, k] xn[b, k]: the weight rows are the MMA's M
// side (128 per tile) and the B sequences its N side (NB = B rounded up to
// 16, zero rows past B), so one tcgen05.mma.kind::tf32 covers a 128 x NB x 8
// block.  A tile's K range is split over S CTAs (S = 1..16) that form one
// thread-block cluster: every weight byte is read from HBM by exactly one CTA,
// and every CTA needs only its K slice of x.
//
// Per CTA (4 warps):
//   1. one thread TMA-loads the CTA's W slice [128 x Kc] (128-byte swizzle),
//      then all threads write its TF32 lo part (W - hi(W)) -- before
//      griddepcontrol.wait: the weights do not depend on the previous
//      kernel, so with programmatic dependent launch this overlaps it;
//   2. after the wait, the x slice [NB x Kc] arrives by TMA (rows past B read
//      as zero);
//   3. LN: each CTA computes (mean, M2) of its slice of every row; one
//      cluster barrier; each CTA combines the S pairs in rank order (Chan's
//      parallel formula: mean = average of the slice means, M2 = sum of M2_i
//      + Kc sum (mean_i - mean)^2) -- the two-pass statistics of the whole
//      row without a second exchange -- and normalises its slice with gamma;
//   4. TF32x3: hi*hi + hi*lo + lo*hi per k step, fp32 accumulation in TMEM
//      (hi = the operand with its low 13 mantissa bits cleared, which is what
//      kind::tf32 reads from the fp32 tile itself);
//   5. tcgen05.ld of the 128 x NB partial into shared memory, one cluster
//      barrier, and CTA s sums rows [s 128/S, (s+1) 128/S) of all S partials
//      in rank order through distributed shared memory (deterministic: no
//      atomics on the data), applies the epilogue and stores; a last cluster
//      barrier keeps every CTA's shared memory alive until its peers have
//      read it.
// Every mbarrier wait is bounded (an expiry is counted in the device error
// count and the CTA winds down); the cluster barriers are reached by every
// thread of every CTA on every path.
#include <algorithm>
#include <cstdlib>

#include <cooperative_groups.h>

#include "gemv_tcgen05.cuh"
#include "tcgen05.cuh"

namespace fml {

__device__ int g_gemv_tc_timeouts;

namespace {

constexpr uint32_t WBLK = 128u * tc::BK * 4u;  // bytes of one 128 x 32 W block

template <int EPI>
__device__ __forceinline__ void epilogue4(const GemvTcArgs& a, uint32_t b, uint32_t n, float4 v,
                                          unsigned long long& key, uint32_t hd_shift)
{
    if constexpr (EPI == GTC_STORE)
    {
        *reinterpret_cast<float4*>(a.y + (uint64_t)b * a.ldy + n) = v;
    }
    else if constexpr (EPI == GTC_GELU)
    {
        v = make_float4(gelu_exact(v.x), gelu_exact(v.y), gelu_exact(v.z), gelu_exact(v.w));
        *reinterpret_cast<float4*>(a.y + (uint64_t)b * a.ldy + n) = v;
    }
    else if constexpr (EPI == GTC_RESID)
    {
        const float4 r = *reinterpret_cast<const float4*>(a.r + (uint64_t)b * a.ldr + n);
        *reinterpret_cast<float4*>(a.y + (uint64_t)b * a.ldy + n) =
            make_float4(r.x + v.x, r.y + v.y, r.z + v.z, r.w + v.w);
    }
    else if constexpr (EPI == GTC_QKV)
    {
        // columns [0, d) -> q, [d, 2d) -> K cache, [2d, 3d) -> V cache at the
        // sequence's position; four columns never straddle a head (hd % 4 == 0)
        if (n < a.d)
            *reinterpret_cast<float4*>(a.q + (uint64_t)b * a.d + n) = v;
        else
        {
            const uint32_t cc = n < 2 * a.d ? n - a.d : n - 2 * a.d;
            float* cache = n < 2 * a.d ? a.kc : a.vc;
            *reinterpret_cast<float4*>(cache + (uint64_t)b * a.seq_stride +
                                       ((uint64_t)(cc >> hd_shift) * a.C + a.pos[b]) * a.hd +
                                       (cc & (a.hd - 1))) = v;
        }
    }
    else if constexpr (EPI == GTC_ARGMAX)
    {
        if (a.y) *reinterpret_cast<float4*>(a.y + (uint64_t)b * a.ldy + n) = v;
        const uint32_t g = n + a.n_off;
        unsigned long long k = argmax_key(v.x, g);
        const unsigned long long k1 = argmax_key(v.y, g + 1), k2 = argmax_key(v.z, g + 2),
                                 k3 = argmax_key(v.w, g + 3);
        k = k1 > k ? k1 : k;
        k = k2 > k ? k2 : k;
        k = k3 > k ? k3 : k;
        key = k;
    }
}

}  // namespace

template <int NB, int EPI, bool LN>
__global__ void __launch_bounds__(128, 1) gemv_tc_kernel(const __grid_constant__ CUtensorMap map_w,
                                                         const __grid_constant__ CUtensorMap map_x, GemvTcArgs a)
{
    using namespace tc;
    namespace cg = cooperative_groups;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t XBLK = NB * 128u;                     // bytes of one NB x 32 x block
    constexpr uint32_t TCOLS = NB <= 32 ? 32u : (uint32_t)NB;  // TMEM columns (a power of 2 >= 32)
    constexpr uint32_t IDESC = idesc_tf32(128, NB);

    const uint32_t KB = a.kb;             // 32-wide K blocks of this CTA
    const uint32_t S = gridDim.x;         // K splits = CTAs of the cluster
    const uint32_t s = blockIdx.x;        // this CTA's split = its rank in the cluster
    const uint32_t n0 = blockIdx.y * 128u;
    const uint32_t k0 = s * KB * (uint32_t)BK;
    const uint32_t Kc = KB * (uint32_t)BK;

    unsigned char* w_s = smem;                  // KB x [128 x 32] W blocks
    unsigned char* wlo_s = w_s + KB * WBLK;     // their lo parts
    unsigned char* x_s = wlo_s + KB * WBLK;     // KB x [NB x 32] x blocks
    unsigned char* xlo_s = x_s + KB * XBLK;
    float* gam = reinterpret_cast<float*>(xlo_s + KB * XBLK);  // [Kc] gamma slice
    float* st_part = gam + Kc;                  // [NB][2] (mean, M2) of this CTA's slice
    float* st_row = st_part + 2 * NB;           // [NB][2] (mean, rstd) of the whole row
    uint64_t* bars = reinterpret_cast<uint64_t*>(st_row + 2 * NB);
    uint64_t* bar_w = bars;
    uint64_t* bar_x = bars + 1;
    uint64_t* bar_mma = bars + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
    float* red = reinterpret_cast<float*>(w_s);  // [NB][128] partial sums (W is dead by then)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    cg::cluster_group cluster = cg::this_cluster();

    if (tid == 0)
    {
        mbar_init(bar_w, 1);
        mbar_init(bar_x, 1);
        mbar_init(bar_mma, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    // 1. weights: TMA, gamma, lo parts -- none depends on the previous kernel
    if (tid == 0)
    {
        mbar_arrive_expect_tx(bar_w, KB * WBLK);
        for (uint32_t j = 0; j < KB; ++j) tma_load_2d(w_s + j * WBLK, &map_w, (int)(k0 + j * BK), (int)n0, bar_w);
    }
    if constexpr (LN)
        for (uint32_t i = tid; i < Kc; i += 128) gam[i] = a.gamma[k0 + i];
    bool ok = mbar_wait(bar_w, 0);
    if (ok)
    {
        const float4* w4 = reinterpret_cast<const float4*>(w_s);
        float4* wl4 = reinterpret_cast<float4*>(wlo_s);
        for (uint32_t i = tid; i < KB * (WBLK / 16); i += 128) wl4[i] = tf32_lo4(w4[i]);
    }

    griddep_launch_dependents();
    griddep_wait();

    // 2. this CTA's slice of the x rows
    if (tid == 0)
    {
        mbar_arrive_expect_tx(bar_x, KB * XBLK);
        for (uint32_t j = 0; j < KB; ++j) tma_load_2d(x_s + j * XBLK, &map_x, (int)(k0 + j * BK), 0, bar_x);
    }
    ok = mbar_wait(bar_x, 0) && ok;
    float4* x4 = reinterpret_cast<float4*>(x_s);
    float4* xl4 = reinterpret_cast<float4*>(xlo_s);

    // 3. LayerNorm of the x rows across the cluster
    if constexpr (LN)
    {
        const float invKc = 1.0f / (float)Kc;
        for (uint32_t m = warp; m < NB; m += 4)
        {
            // the 16-byte chunks of row m: KB blocks x 8 (their order does not
            // matter for a sum)
            float sum = 0.f;
            for (uint32_t c = lane; c < KB * 8; c += 32)
            {
                const float4 v = x4[((c >> 3) * NB + m) * 8 + (c & 7)];
                sum += (v.x + v.y) + (v.z + v.w);
            }
            sum = warp_sum(sum);
            const float mean = sum * invKc;
            float q = 0.f;
            for (uint32_t c = lane; c < KB * 8; c += 32)
            {
                const float4 v = x4[((c >> 3) * NB + m) * 8 + (c & 7)];
                const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
                q = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, q))));
            }
            q = warp_sum(q);
            if (lane == 0)
            {
                st_part[2 * m] = mean;
                st_part[2 * m + 1] = q;
            }
        }
        cluster.sync();  // every CTA's slice statistics are written
        if (tid < NB)
        {
            float mean = 0.f;
            for (uint32_t r = 0; r < S; ++r) mean += *cluster.map_shared_rank(st_part + 2 * tid, r);
            mean /= (float)S;
            float m2 = 0.f;
            for (uint32_t r = 0; r < S; ++r)
            {
                const float mi = *cluster.map_shared_rank(st_part + 2 * tid, r);
                const float di = mi - mean;
                m2 += *cluster.map_shared_rank(st_part + 2 * tid + 1, r) + (float)Kc * di * di;
            }
            const float var = m2 / (float)(Kc * S);
            st_row[2 * tid] = mean;
            st_row[2 * tid + 1] = 1.0f / sqrtf(var + 1e-5f);
        }
        __syncthreads();
        for (uint32_t i = tid; i < KB * NB * 8; i += 128)
        {
            const uint32_t j = i / (NB * 8), r = (i >> 3) % NB, p = i & 7;
            const uint32_t k = j * BK + 4u * (p ^ (r & 7u));  // 128-byte swizzle: chunk p holds k = 4 (p ^ r%8)
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < a.M)
            {
                const float4 u = x4[i];
                const float mean = st_row[2 * r], rstd = st_row[2 * r + 1];
                v.x = (u.x - mean) * rstd * gam[k];
                v.y = (u.y - mean) * rstd * gam[k + 1];
                v.z = (u.z - mean) * rstd * gam[k + 2];
                v.w = (u.w - mean) * rstd * gam[k + 3];
            }
            x4[i] = v;
            xl4[i] = tf32_lo4(v);
        }
    }
    else
    {
        for (uint32_t i = tid; i < KB * (XBLK / 16); i += 128) xl4[i] = tf32_lo4(x4[i]);
    }
    // generic-proxy writes of the operands -> visible to the tensor core
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    ok = __syncthreads_and(ok) != 0;

    // 4. TF32x3 MMAs, one thread
    if (tid == 0 && ok)
    {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (uint32_t j = 0; j < KB; ++j)
        {
#pragma unroll
            for (uint32_t kk = 0; kk < (uint32_t)BK / 8; ++kk)
            {
                const uint32_t off = kk * 32;
                const uint64_t da = smem_desc(w_s + j * WBLK, off);
                const uint64_t db = smem_desc(x_s + j * XBLK, off);
                mma_tf32(tmem, da, db, IDESC, j > 0 || kk > 0);
                mma_tf32(tmem, da, smem_desc(xlo_s + j * XBLK, off), IDESC, true);  // hi * lo
                mma_tf32(tmem, smem_desc(wlo_s + j * WBLK, off), db, IDESC, true);  // lo * hi
            }
        }
        mma_commit(bar_mma);
    }
    if (ok) ok = mbar_wait(bar_mma, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    ok = __syncthreads_and(ok) != 0;

    // 5. partial sums to shared memory: thread (warp w, lane l) holds row
    //    n0 + 32 w + l of D, all NB columns
    if (ok)
    {
        const uint32_t nl = 32u * warp + lane;
        const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16);
#pragma unroll
        for (int c0 = 0; c0 < NB; c0 += 16)
        {
            float v[16];
            tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) red[(c0 + i) * 128 + nl] = v[i];
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    cluster.sync();  // every CTA's partial is in its shared memory

    // CTA s owns rows [s R, s R + R) of the tile: sum the S partials in rank
    // order, four consecutive rows per thread
    if (ok)
    {
        const uint32_t R = 128u / S, QR = R / 4u;  // QR quads of rows per column b
        const uint32_t hd_shift = EPI == GTC_QKV ? (uint32_t)(__ffs(a.hd) - 1) : 0u;
        for (uint32_t t = tid; t < NB * QR; t += 128)
        {
            const uint32_t b = t / QR, nl = s * R + 4u * (t % QR), n = n0 + nl;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            for (uint32_t r = 0; r < S; ++r)
            {
                const float4 u = *reinterpret_cast<const float4*>(cluster.map_shared_rank(red + b * 128 + nl, r));
                v.x += u.x;
                v.y += u.y;
                v.z += u.z;
                v.w += u.w;
            }
            unsigned long long key = 0ull;
            const bool valid = b < a.M && n < a.N;
            if (valid) epilogue4<EPI>(a, b, n, v, key, hd_shift);
            if constexpr (EPI == GTC_ARGMAX)
            {
                // max over the QR threads of column b (consecutive, aligned
                // lanes: QR divides 32), one atomic per (CTA, column)
                for (uint32_t o = 1; o < QR && o < 32u; o <<= 1)
                {
                    const unsigned long long other = __shfl_xor_sync(FULL_MASK, key, o);
                    key = other > key ? other : key;
                }
                if (t % QR == 0 && b < a.M && key) atomicMax(a.keys + b, key);
            }
        }
    }
    cluster.sync();  // no CTA leaves while a peer may still read its partial

    if (!ok && tid == 0) atomicAdd(&g_gemv_tc_timeouts, 1);
    if (tid == 0 && a.stamp.buf) stamp_write(a.stamp);
    __syncthreads();
    if (warp == 0)
    {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
    }
}

// ---- host side ---------------------------------------------------------------

namespace {

size_t gemv_tc_smem(uint32_t NB, uint32_t KB)
{
    return 1024 + 2ull * KB * WBLK + 2ull * KB * NB * 128 + KB * tc::BK * 4 + 4ull * NB * 4 + 64;
}

// K blocks per CTA (Kc = 32 KB): the split count S = K / Kc must divide the
// 128 rows into quads (S <= 32, a power of two), stay a cluster (S <= 16) and
// the shared memory must fit; among those, the grid closest to one CTA per SM
// (FML_GEMV_TC_KB overrides).
uint32_t choose_kb(uint32_t K, uint32_t N, uint32_t NB, int sms)
{
    const uint32_t tiles = (N + 127) / 128;
    uint32_t best = 0, best_d = ~0u;
    for (uint32_t kb : {1u, 2u, 4u})
    {
        if (K % (kb * tc::BK)) continue;
        const uint32_t S = K / (kb * tc::BK);
        if (S < 1 || S > 16 || (S & (S - 1))) continue;
        if (gemv_tc_smem(NB, kb) > 227u * 1024u) continue;
        if (2ull * kb * tc::BK * 4 * 128 < (uint64_t)NB * 128 * 4) continue;  // the partials reuse W's space
        const uint32_t ctas = tiles * S;
        const uint32_t d = ctas > (uint32_t)sms ? ctas - (uint32_t)sms : (uint32_t)sms - ctas;
        if (d < best_d) { best_d = d; best = kb; }
    }
    if (const char* e = getenv("FML_GEMV_TC_KB"))
    {
        const long v = strtol(e, nullptr, 10);
        if ((v == 1 || v == 2 || v == 4) && K % (v * tc::BK) == 0)
        {
            const uint32_t S = K / ((uint32_t)v * tc::BK);
            if (S >= 1 && S <= 16 && !(S & (S - 1)) && gemv_tc_smem(NB, (uint32_t)v) <= 227u * 1024u &&
                (uint32_t)v * 2 * 32 >= NB)
                best = (uint32_t)v;
        }
    }
    return best;
}

template <int NB, int EPI, bool LN>
int launch_nb(const GemvTcArgs& args, uint32_t kb, cudaStream_t st, bool pdl)
{
    auto kern = gemv_tc_kernel<NB, EPI, LN>;
    static uint64_t attr_devices = 0;
    int dev = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
    if (!bit || !(attr_devices & bit))
    {
        FML_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        FML_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                          cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        attr_devices |= bit;
    }
    CUtensorMap mw, mx;
    FML_RC(tc::make_map(&mw, args.w, (int)args.N, (int)args.K, (int)args.K, 128));
    FML_RC(tc::make_map(&mx, args.x, (int)args.M, (int)args.K, (int)args.ldx, NB));
    GemvTcArgs a = args;
    a.kb = kb;
    const uint32_t S = args.K / (kb * tc::BK);
    const uint32_t tiles = (args.N + 127) / 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, tiles);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = gemv_tc_smem(NB, kb);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = S;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
    if (pdl)
    {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, mx, a);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "gemv_tc launch: %s", cudaGetErrorString(e));
    FML_LAUNCH_CHECK();
    return FML_OK;
}

template <int EPI, bool LN>
int launch_epi(const GemvTcArgs& a, uint32_t NB, uint32_t kb, cudaStream_t st, bool pdl)
{
    if (NB == 16) return launch_nb<16, EPI, LN>(a, kb, st, pdl);
    if (NB == 32) return launch_nb<32, EPI, LN>(a, kb, st, pdl);
    return launch_nb<64, EPI, LN>(a, kb, st, pdl);
}

uint32_t nb_for(uint32_t M) { return M <= 16 ? 16u : (M <= 32 ? 32u : 64u); }

int sm_count()
{
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace

bool gemv_tc_supported(const GemvTcArgs& a)
{
    if (const char* e = getenv("FML_GEMV_TC"))  // FML_GEMV_TC=0: CUDA-core GEMVs only
        if (strtol(e, nullptr, 10) == 0) return false;
    if (a.M < 1 || a.M > 64 || a.N < 4 || a.N % 4 || a.K % tc::BK || a.ldx % 4) return false;
    if (!aligned16(a.x) || !aligned16(a.w)) return false;
    if (a.epi == GTC_QKV && (a.hd % 4 || a.d % 4)) return false;
    // the instantiated prologues: LayerNorm before QKV, GELU and ARGMAX, none before RESID and STORE
    if (a.ln != (a.epi == GTC_QKV || a.epi == GTC_GELU || a.epi == GTC_ARGMAX) || (a.ln && !a.gamma)) return false;
    if ((a.epi == GTC_STORE || a.epi == GTC_GELU || a.epi == GTC_RESID) && (a.ldy % 4 || !aligned16(a.y))) return false;
    if (a.epi == GTC_RESID && (a.ldr % 4 || !aligned16(a.r))) return false;
    return choose_kb(a.K, a.N, nb_for(a.M), sm_count()) != 0;
}

int launch_gemv_tc(const GemvTcArgs& a, cudaStream_t st, bool pdl)
{
    FML_REQUIRE(gemv_tc_supported(a), "gemv_tc: unsupported shape M %u N %u K %u", a.M, a.N, a.K);
    FML_REQUIRE(!a.ln || a.gamma, "gemv_tc: LayerNorm prologue without gamma");
    const uint32_t NB = nb_for(a.M);
    const uint32_t kb = choose_kb(a.K, a.N, NB, sm_count());
    switch (a.epi)
    {
    case GTC_QKV: return launch_epi<GTC_QKV, true>(a, NB, kb, st, pdl);
    case GTC_GELU: return launch_epi<GTC_GELU, true>(a, NB, kb, st, pdl);
    case GTC_ARGMAX: return launch_epi<GTC_ARGMAX, true>(a, NB, kb, st, pdl);
    case GTC_RESID: return launch_epi<GTC_RESID, false>(a, NB, kb, st, pdl);
    case GTC_STORE: return launch_epi<GTC_STORE, false>(a, NB, kb, st, pdl);
    default: return set_error(FML_ERR_INVALID, "gemv_tc: unknown epilogue %d", a.epi);
    }
}

int gemv_tc_error_count(int* out)
{
    FML_CUDA_TRY(cudaMemcpyFromSymbol(out, g_gemv_tc_timeouts, sizeof(int)));
    return FML_OK;
}

}  // namespace fml
