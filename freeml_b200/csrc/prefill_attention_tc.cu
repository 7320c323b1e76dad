// Causal prefill attention on the tensor cores: CausalSelfAttentionLayer::
// Forward (CausalSelfAttentionLayer.h:424-499) over whole prompts -- per head
// S = Q K^T * 1/sqrt(hd) + causal mask, row softmax, Y = P V -- as a
// flash-attention loop on tcgen05 with fp32-level accuracy (TF32x3).
//
// CTA = 4 warps on (128 query rows, head, sequence); it walks the key tiles
// (KT keys) up to its last row.  Per tile:
//   1. K tile (TMA, 128-byte swizzle, K-major) -> its TF32 lo part; one
//      thread issues S = Q K^T (Q_hi K_hi + Q_hi K_lo + Q_lo K_hi) into TMEM;
//   2. thread r (= TMEM lane r) reads query row r's KT scores with
//      tcgen05.ld, scales and masks them (keys past the row and past the
//      prompt), and updates the row's online softmax (running max m and sum
//      l); it writes the row's probabilities P (and their lo part) into
//      shared memory as the K-major A operand of the next MMA;
//   3. V tile: TMA in the 128-byte swizzle of 32-byte atoms, the layout an
//      N-major tf32 operand needs (V is stored [keys x hd], hd contiguous);
//      rows past the last valid key are zeroed (the cache may hold anything
//      there); one thread issues O_tile = P V (TF32x3) into a second TMEM
//      accumulator;
//   4. thread r reads its O_tile row and accumulates O = O corr + O_tile in
//      registers (corr = exp(m_old - m_new)).
// At the end each valid row writes O / l.  The next tile's K and V copies
// start as soon as the MMAs that read the current ones have completed.
// Every mbarrier wait is bounded (expiries are counted in the device error
// count; the CTA then stops issuing work and still frees its TMEM).
#include <cmath>
#include <cstdlib>

#include "tcgen05.cuh"

namespace fml {

__device__ int g_prefill_tc_timeouts;

namespace {

constexpr int QB = 128;  // query rows per CTA (= TMEM lanes)

struct PfArgs
{
    float* out;       // [B*P x ldo], head h at column h * HD
    uint32_t ldo;
    uint32_t B, H, P, C;
    float scale;      // 1/sqrt(hd), CausalSelfAttentionLayer.h:73-77
};

template <int HD>
struct PfShape
{
    static constexpr int KT = HD <= 64 ? 64 : 32;           // keys per tile
    static constexpr uint32_t QBYTES = HD * QB * 4;          // Q tile: HD/32 blocks of [128 x 32]
    static constexpr uint32_t KBYTES = HD * KT * 4;          // K tile: HD/32 blocks of [KT x 32]
    static constexpr uint32_t VBYTES = HD * KT * 4;          // V tile: (KT/32) x (HD/32) boxes of [32 x 32]
    static constexpr uint32_t PBYTES = KT * QB * 4;          // P tile: KT/32 blocks of [128 x 32]
    static constexpr uint32_t SMEM = 2 * (QBYTES + KBYTES + VBYTES + PBYTES) + 1024 + 64;
    static constexpr uint32_t OCOL = KT < 32 ? 32 : KT;      // TMEM column of the O accumulator
    static constexpr uint32_t TCOLS = OCOL + HD <= 128 ? 128 : 256;
};

__device__ __forceinline__ void lo_inplace(float4* dst, const float4* src, uint32_t n4, int tid)
{
    for (uint32_t i = tid; i < n4; i += 128) dst[i] = tc::tf32_lo4(src[i]);
}

__device__ __forceinline__ uint64_t desc_mn(const void* tile)
{
    // MN-major, 128-byte swizzle with 32-byte atoms: the next 32 n one 4 KB
    // box on (LBO), the next 4 k one 512-byte atom on (SBO)
    const uint64_t start = (uint64_t)(tc::smem_u32(tile) >> 4) & 0x3FFFull;
    return start | ((uint64_t)(4096 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46) | (1ull << 61);
}

}  // namespace

template <int HD, bool SPLIT3>
__global__ void __launch_bounds__(128, 1) prefill_attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                                                                      const __grid_constant__ CUtensorMap map_k,
                                                                      const __grid_constant__ CUtensorMap map_v,
                                                                      PfArgs a)
{
    using namespace tc;
    using Sh = PfShape<HD>;
    constexpr int KT = Sh::KT;
    constexpr uint32_t IDESC_S = idesc_tf32(128, KT);
    constexpr uint32_t IDESC_O = idesc_tf32(128, HD) | (1u << 16);  // B (V) read MN-major
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* q_s = smem;
    unsigned char* qlo_s = q_s + Sh::QBYTES;
    unsigned char* k_s = qlo_s + Sh::QBYTES;
    unsigned char* klo_s = k_s + Sh::KBYTES;
    unsigned char* v_s = klo_s + Sh::KBYTES;
    unsigned char* vlo_s = v_s + Sh::VBYTES;
    unsigned char* p_s = vlo_s + Sh::VBYTES;
    unsigned char* plo_s = p_s + Sh::PBYTES;
    // barriers: Q, K, V copies; S, O products
    uint64_t* bars = reinterpret_cast<uint64_t*>(plo_s + Sh::PBYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
    enum { BQ = 0, BKEY = 1, BVAL = 2, BS = 3, BO = 4 };

    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t q0 = blockIdx.x * QB, h = blockIdx.y, b = blockIdx.z;
    const uint32_t P = a.P;
    const uint32_t nkeys = min(q0 + (uint32_t)QB, P);         // keys this CTA's rows can see
    const uint32_t ntiles = (nkeys + KT - 1) / KT;
    const int kv_row0 = (int)((b * a.H + h) * a.C);           // this (sequence, head)'s first cache row
    const uint32_t q = q0 + tid;                              // this thread's query row
    // thread 0's count of the phases it started / saw complete on each barrier
    // (the drain after an expired wait)
    uint32_t issued[5] = {0, 0, 0, 0, 0}, seen[5] = {0, 0, 0, 0, 0};

    if (tid == 0)
    {
        for (int i = 0; i < 5; ++i) mbar_init(&bars[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(Sh::TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_o = tmem + Sh::OCOL;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

    auto issue_k = [&](uint32_t t) {
        mbar_arrive_expect_tx(&bars[BKEY], Sh::KBYTES);
        for (int j = 0; j < HD / 32; ++j)
            tma_load_2d(k_s + j * (KT * 128), &map_k, 32 * j, kv_row0 + (int)(t * KT), &bars[BKEY]);
        ++issued[BKEY];
    };
    auto issue_v = [&](uint32_t t) {
        mbar_arrive_expect_tx(&bars[BVAL], Sh::VBYTES);
        for (int kb = 0; kb < KT / 32; ++kb)
            for (int j = 0; j < HD / 32; ++j)
                tma_load_2d(v_s + (kb * (HD / 32) + j) * 4096, &map_v, 32 * j, kv_row0 + (int)(t * KT) + 32 * kb,
                            &bars[BVAL]);
        ++issued[BVAL];
    };
    // bounded wait on phase `ph` of barrier i, the same answer in the whole warp
    auto wait = [&](int i, uint32_t ph) {
        const bool w = __all_sync(FULL_MASK, mbar_wait(&bars[i], ph & 1u));
        if (w) seen[i] = ph + 1;
        return w;
    };
    if (tid == 0)
    {
        mbar_arrive_expect_tx(&bars[BQ], Sh::QBYTES);
        for (int j = 0; j < HD / 32; ++j)
            tma_load_2d(q_s + j * (QB * 128), &map_q, (int)(h * HD) + 32 * j, (int)(b * P + q0), &bars[BQ]);
        issued[BQ] = 1;
        issue_k(0);
        issue_v(0);
    }

    bool ok = wait(BQ, 0);
    if constexpr (SPLIT3)
        if (ok)
            lo_inplace(reinterpret_cast<float4*>(qlo_s), reinterpret_cast<const float4*>(q_s), Sh::QBYTES / 16, tid);

    float o[HD];
#pragma unroll
    for (int e = 0; e < HD; ++e) o[e] = 0.f;
    float m = -INFINITY, l = 0.f;

    for (uint32_t t = 0; t < ntiles; ++t)
    {
        const uint32_t k0 = t * KT;
        // ---- S = Q K^T ----
        if (ok) ok = wait(BKEY, t);
        if constexpr (SPLIT3)
            if (ok)
                lo_inplace(reinterpret_cast<float4*>(klo_s), reinterpret_cast<const float4*>(k_s), Sh::KBYTES / 16,
                           tid);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        ok = __syncthreads_and(ok) != 0;
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (tid == 0)
        {
            for (int j = 0; j < HD / 32; ++j)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                {
                    const uint64_t da = smem_desc(q_s + j * (QB * 128), kk * 32);
                    const uint64_t db = smem_desc(k_s + j * (KT * 128), kk * 32);
                    mma_tf32(tmem, da, db, IDESC_S, j > 0 || kk > 0);
                    if constexpr (SPLIT3)
                    {
                        mma_tf32(tmem, da, smem_desc(klo_s + j * (KT * 128), kk * 32), IDESC_S, true);
                        mma_tf32(tmem, smem_desc(qlo_s + j * (QB * 128), kk * 32), db, IDESC_S, true);
                    }
                }
            mma_commit(&bars[BS]);
            ++issued[BS];
        }
        ok = wait(BS, t);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // the K tile is consumed: the next one's copy can start
        if (tid == 0 && ok && t + 1 < ntiles) issue_k(t + 1);

        // ---- row softmax (thread = query row) ----
        float sv[KT];
        if (ok)
        {
#pragma unroll
            for (int c = 0; c < KT; c += 32)
            {
                float v[32];
                tmem_ld32(tmem + lane_base + (uint32_t)c, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[c + i] = v[i];
            }
        }
        else
        {
#pragma unroll
            for (int i = 0; i < KT; ++i) sv[i] = 0.f;
        }
        float mx = m;
#pragma unroll
        for (int i = 0; i < KT; ++i)
        {
            const uint32_t key = k0 + i;
            const bool live = key <= q && key < P;
            sv[i] = live ? sv[i] * a.scale : -INFINITY;  // a select: masked slots may hold anything
            mx = fmaxf(mx, sv[i]);
        }
        const float corr = m == -INFINITY ? 0.f : expf(m - mx);
        float psum = 0.f;
#pragma unroll
        for (int i = 0; i < KT; ++i)
        {
            sv[i] = sv[i] == -INFINITY ? 0.f : expf(sv[i] - mx);
            psum += sv[i];
        }
        l = l * corr + psum;
        m = mx;
        // P row into the K-major 128-byte-swizzled A tile: keys kb*32 + 4c ..
        // + 3 of row tid sit in 16-byte chunk c ^ (tid % 8) of the row
#pragma unroll
        for (int kb = 0; kb < KT / 32; ++kb)
#pragma unroll
            for (int c = 0; c < 8; ++c)
            {
                const float4 pv = make_float4(sv[kb * 32 + 4 * c], sv[kb * 32 + 4 * c + 1], sv[kb * 32 + 4 * c + 2],
                                              sv[kb * 32 + 4 * c + 3]);
                const uint32_t off = kb * (QB * 128) + tid * 128 + ((c ^ (tid & 7)) * 16);
                *reinterpret_cast<float4*>(p_s + off) = pv;
                if constexpr (SPLIT3) *reinterpret_cast<float4*>(plo_s + off) = tf32_lo4(pv);
            }

        // ---- O_tile = P V ----
        if (ok) ok = wait(BVAL, t);
        if (ok)
        {
            // key rows past the last key any row of this CTA sees are zeroed
            // (the cache there may hold anything, and 0 * NaN is NaN); with
            // TF32x3 the same pass writes the lo part of the others.  Box
            // (kb, j) = keys kb*32.., head columns 32j.. is 4 KB of 32 rows.
            const uint32_t valid = nkeys - k0 < (uint32_t)KT ? nkeys - k0 : (uint32_t)KT;
            if (SPLIT3 || valid < (uint32_t)KT)
            {
                float4* v4 = reinterpret_cast<float4*>(v_s);
                float4* vlo4 = reinterpret_cast<float4*>(vlo_s);
                for (uint32_t i = tid; i < Sh::VBYTES / 16; i += 128)
                {
                    const uint32_t key = (i / 256) / (HD / 32) * 32 + (i % 256) / 8;
                    if (key >= valid)
                    {
                        v4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                        if constexpr (SPLIT3) vlo4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    else if constexpr (SPLIT3)
                        vlo4[i] = tf32_lo4(v4[i]);
                }
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        ok = __syncthreads_and(ok) != 0;
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (tid == 0)
        {
            for (int kb = 0; kb < KT / 32; ++kb)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                {
                    const uint64_t da = smem_desc(p_s + kb * (QB * 128), kk * 32);
                    const uint64_t db = desc_mn(v_s + kb * (HD / 32) * 4096 + kk * 1024);
                    mma_tf32(tmem_o, da, db, IDESC_O, kb > 0 || kk > 0);
                    if constexpr (SPLIT3)
                    {
                        mma_tf32(tmem_o, da, desc_mn(vlo_s + kb * (HD / 32) * 4096 + kk * 1024), IDESC_O, true);
                        mma_tf32(tmem_o, smem_desc(plo_s + kb * (QB * 128), kk * 32), db, IDESC_O, true);
                    }
                }
            mma_commit(&bars[BO]);
            ++issued[BO];
        }
        ok = wait(BO, t);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (tid == 0 && ok && t + 1 < ntiles) issue_v(t + 1);  // the V tile and P are consumed
        if (ok)
        {
#pragma unroll
            for (int c = 0; c < HD; c += 32)
            {
                float v[32];
                tmem_ld32(tmem_o + lane_base + (uint32_t)c, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) o[c + i] = fmaf(o[c + i], corr, v[i]);
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    ok = __syncthreads_and(ok) != 0;

    if (ok && q < P)
    {
        const float inv = 1.0f / l;  // l >= 1: the row's largest score contributes exp(0)
        float* dst = a.out + (uint64_t)(b * P + q) * a.ldo + h * HD;
#pragma unroll
        for (int e = 0; e < HD; e += 4)
            *reinterpret_cast<float4*>(dst + e) = make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
    }
    if (!ok && tid == 0)
    {
        atomicAdd(&g_prefill_tc_timeouts, 1);
        // copies and products still in flight must land before the CTA frees
        // its shared memory and TMEM (bounded waits)
        for (int i = 0; i < 5; ++i)
            for (uint32_t ph = seen[i]; ph < issued[i]; ++ph) mbar_wait(&bars[i], ph & 1u);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
    {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Sh::TCOLS) : "memory");
    }
}

// ---- head dim 64: two query tiles per CTA, warp-specialised ---------------
//
// CTA = 12 warps on (256 query rows as two 128-row tiles A and B, head,
// sequence); the two tiles share every K / V tile, and their softmax and
// MMA phases interleave so that the tensor pipe works on one tile while the
// CUDA cores work on the other:
//   warps 0-3   softmax of tile A (thread = TMEM lane = query row)
//   warps 4-7   softmax of tile B
//   warp 8      converter: the TF32 lo parts of K and V (TF32x3) and the
//               zeroing of V rows past the last key any row sees
//   warps 9-10  one thread each issues tile A's / tile B's tcgen05.mma
//   warp 11     one thread issues every TMA copy
// K and V operand tiles are double-buffered: the copy and the conversion of
// key tile t + 1 run while tile t's products do.
// TMEM per query tile (2 x 256 columns): S = Q K^T [64 keys | the hi.lo
// half], overwritten in place by P = exp(S - m) and P's lo part (the A
// operands of O += P V, read from TMEM); the O accumulator [64], which stays
// in TMEM over all key tiles; and Q's lo part [64] (the A operand of the
// lo.hi term of S).  A tf32 MMA of N = 64 costs 3/4 of one of N = 128 on
// this part (it runs the tensor pipe at 2/3 of its rate), so S's hi.hi and
// hi.lo terms are ONE MMA of N = 128 against [K hi | K lo] (the lo rows sit
// next to the hi rows of each K box); O's three terms stay 64 wide for the
// TMEM that Q lo needs.
// A row rescales O (tcgen05.ld / st) only when its running maximum rises by
// more than 2^8 over the one its P values were taken against, so P stays
// below 256 and fp32 keeps its precision; the result O / l does not depend
// on the reference maximum.
// The tensor pipe's instruction queue is short: while the thread that issues
// MMAs waits on an mbarrier (even one already complete, ~170 cycles), the
// pipe drains and idles.  So each query tile has its own issuing thread, in
// its own warp, and the pipe runs one tile's products while the other's
// thread waits (for its softmax, or for the completion of O_x(t-1): S_x(t)
// overwrites the columns P_x(t-1) is read from).
// Every wait is bounded and also returns early once any role has recorded an
// expiry in the CTA's abort flag; the MMA thread then waits for its MMAs and
// the copy thread for its copies (bounded) before TMEM is freed.
namespace {

constexpr int PP_HD = 64, PP_KT = 64;
constexpr uint32_t PP_QTILE = 128 * PP_HD * 4;  // one 128-row Q tile, 32 KB
constexpr uint32_t PP_KVT = PP_KT * PP_HD * 4;  // one K or V tile, 16 KB
constexpr int PP_THREADS = 12 * 32;
constexpr uint32_t PP_CONV = 32;  // converter threads
// operand tiles: K box j (head columns 32j..) = [64 hi rows | 64 lo rows] of
// 128 bytes (16 KB); V key block kb = four 4 KB boxes [hi columns 0-31, hi
// 32-63, lo 0-31, lo 32-63] of 32 keys (16 KB)
constexpr uint32_t PP_KBOX = 2 * PP_KT * 128, PP_VBLK = 4 * 4096, PP_KVOP = 2 * PP_KVT;
// Q hi tiles, then two K and two V operand tiles (hi and lo each)
constexpr uint32_t PP_SMEM = 2 * PP_QTILE + 4 * PP_KVOP + 1024 + 256;
// per operand buffer b: F copy landed, R converted, E[x] consumed by tile
// x's MMAs (index 2x + b); per query tile x: S, P, O and the final drain
enum PpBar { PB_QF, PB_QR, PB_KF, PB_KR = PB_KF + 2, PB_KE = PB_KR + 2, PB_VF = PB_KE + 4, PB_VR = PB_VF + 2,
             PB_VE = PB_VR + 2, PB_S0 = PB_VE + 4, PB_P0 = PB_S0 + 2, PB_O0 = PB_P0 + 2, PB_FIN = PB_O0 + 2,
             PB_N = PB_FIN + 2 };
// TMEM columns of tile x: S / P [0, 64), S's hi.lo half / P lo [64, 128), O
// [128, 192), Q lo [192, 256)
constexpr uint32_t PP_TX = 256, PP_PLO = 64, PP_O = 128, PP_QLO = 192;

__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for phase `ph` of `bar`; false when the limit ran out (the
// flag is then raised) or another role raised the flag.
__device__ __forceinline__ bool pp_wait(uint64_t* bar, uint32_t ph, volatile int* abort)
{
    const uint32_t addr = tc::smem_u32(bar);
    for (uint32_t it = 0; it < (1u << 24); ++it)
    {
        if (mbar_try(addr, ph & 1u)) return true;
        if ((it & 255u) == 255u && *abort) return false;
    }
    *abort = 1;
    return false;
}

// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32: relative error
// about 2^-22; 2^-inf = +0)
__device__ __forceinline__ float ex2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

}  // namespace

template <bool SPLIT3>
__global__ void __launch_bounds__(PP_THREADS, 1) prefill_attention_pp_kernel(const __grid_constant__ CUtensorMap map_q,
                                                                             const __grid_constant__ CUtensorMap map_k,
                                                                             const __grid_constant__ CUtensorMap map_v,
                                                                             PfArgs a)
{
    using namespace tc;
    constexpr uint32_t IDESC_S = idesc_tf32(128, PP_KT);
    constexpr uint32_t IDESC_S2 = idesc_tf32(128, 2 * PP_KT);          // [K hi | K lo]
    constexpr uint32_t IDESC_O = idesc_tf32(128, PP_HD) | (1u << 16);  // B (V) read MN-major
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* q_s = smem;                     // Q hi of tile x at x * QTILE
    unsigned char* k_op = smem + 2 * PP_QTILE;     // K operand buffer b at b * KVOP (PP_KBOX layout)
    unsigned char* v_op = k_op + 2 * PP_KVOP;      // V operand buffer b at b * KVOP (PP_VBLK layout)
    uint64_t* bars = reinterpret_cast<uint64_t*>(v_op + 2 * PP_KVOP);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + PB_N);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // heaviest query blocks (most key tiles) first
    const uint32_t qblk = gridDim.x - 1 - blockIdx.x;
    const uint32_t q0 = qblk * 256, h = blockIdx.y, b = blockIdx.z;
    const uint32_t P = a.P;
    const bool has_b = q0 + 128 < P;
    // key tiles of tile A / B and the keys any row of the CTA sees
    const uint32_t nt0 = (min(q0 + 128u, P) + PP_KT - 1) / PP_KT;
    const uint32_t nt1 = has_b ? (min(q0 + 256u, P) + PP_KT - 1) / PP_KT : 0u;
    const uint32_t ntiles = has_b ? nt1 : nt0;
    const uint32_t nkeys = min(q0 + 256u, P);
    const int kv_row0 = (int)((b * a.H + h) * a.C);

    if (tid == 0)
    {
        for (int i = 0; i < PB_N; ++i)
        {
            uint32_t count = 1;
            if (i == PB_QR) count = 256;  // every softmax thread writes its Q lo row
            if (i == PB_KR || i == PB_KR + 1 || i == PB_VR || i == PB_VR + 1) count = PP_CONV;
            if (i == PB_P0 || i == PB_P0 + 1) count = 128;
            mbar_init(&bars[i], count);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 8)
    {
        // ---------------- softmax of tile x ----------------
        const int x = warp >> 2;
        const uint32_t nt = x ? nt1 : nt0;
        const int r = 32 * (warp & 3) + lane;                 // row within the tile
        const uint32_t row = q0 + 128u * x + (uint32_t)r;     // this thread's query row
        const uint32_t tx = tmem + PP_TX * x + ((uint32_t)(32 * (warp & 3)) << 16);
        const float sl2 = a.scale * 1.4426950408889634f;  // scores in log2 units
        float m = -INFINITY, l = 0.f;
        bool ok = __all_sync(FULL_MASK, pp_wait(&bars[PB_QF], 0, abort));
        if (ok && SPLIT3)
        {
            // Q lo of this row into TMEM: row r of box j holds head columns
            // 32j + 4c.. in 16-byte chunk c ^ (r % 8)
            const unsigned char* qrow = q_s + x * PP_QTILE + r * 128;
#pragma unroll
            for (int j = 0; j < PP_HD / 32; ++j)
            {
                uint32_t u[32];
#pragma unroll
                for (int c = 0; c < 8; ++c)
                {
                    const float4 v = *reinterpret_cast<const float4*>(qrow + j * (128 * 128) + ((c ^ (r & 7)) * 16));
                    const float4 lo = tf32_lo4(v);
                    u[4 * c] = __float_as_uint(lo.x);
                    u[4 * c + 1] = __float_as_uint(lo.y);
                    u[4 * c + 2] = __float_as_uint(lo.z);
                    u[4 * c + 3] = __float_as_uint(lo.w);
                }
                tmem_st32(tx + PP_QLO + 32 * j, u);
            }
            tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(&bars[PB_QR]);
        for (uint32_t t = 0; ok && t < nt; ++t)
        {
            ok = __all_sync(FULL_MASK, pp_wait(&bars[PB_S0 + x], t, abort));
            if (!ok) break;
            tc_fence_after();
            float s[PP_KT];
#pragma unroll
            for (int c = 0; c < PP_KT; c += 32)
            {
                uint32_t u[32];
                tmem_ld32_async(tx + c, u);
                if constexpr (SPLIT3)
                {
                    uint32_t w[32];
                    tmem_ld32_async(tx + PP_PLO + c, w);
                    tmem_wait_ld(u);
                    tmem_wait_ld(w);
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(u[i]) + __uint_as_float(w[i]);
                }
                else
                {
                    tmem_wait_ld(u);
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(u[i]);
                }
            }
            const uint32_t k0 = t * PP_KT;
            // the mask only bites in tiles that reach past the warp's first
            // row or past the prompt (a warp-uniform test)
            const uint32_t row0 = row - lane;
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (k0 + PP_KT - 1 <= row0 && k0 + PP_KT <= P)
            {
#pragma unroll
                for (int i = 0; i < PP_KT; ++i)
                {
                    s[i] *= sl2;
                    mx4[i & 3] = fmaxf(mx4[i & 3], s[i]);
                }
            }
            else
            {
#pragma unroll
                for (int i = 0; i < PP_KT; ++i)
                {
                    const uint32_t key = k0 + i;
                    s[i] = (key <= row && key < P) ? s[i] * sl2 : -INFINITY;  // a select: masked slots may hold NaN
                    mx4[i & 3] = fmaxf(mx4[i & 3], s[i]);
                }
            }
            const float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            const bool need = mt > m + 8.0f;
            if (__any_sync(FULL_MASK, need))
            {
                const float mn = need ? mt : m;
                const float corr = ex2_approx(m - mn);  // 0 on the first tile (m = -inf)
                l *= corr;
                m = mn;
                if (t > 0)
                {
                    // O_x(t-1) has completed: S_x(t) was issued after it
#pragma unroll
                    for (int c = 0; c < PP_HD; c += 32)
                    {
                        float v[32];
                        uint32_t u[32];
                        tmem_ld32(tx + PP_O + c, v);
#pragma unroll
                        for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(v[i] * corr);
                        tmem_st32(tx + PP_O + c, u);
                    }
                }
            }
            float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < PP_KT; c += 32)
            {
                uint32_t u[32];
#pragma unroll
                for (int i = 0; i < 32; ++i)
                {
                    const float p = ex2_approx(s[c + i] - m);  // 0 for masked keys
                    ls[i & 3] += p;
                    s[c + i] = p;
                    u[i] = __float_as_uint(p);
                }
                tmem_st32(tx + c, u);  // P over S's columns (the MMA reads its TF32 part)
                if constexpr (SPLIT3)
                {
#pragma unroll
                    for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(s[c + i] - tf32_hi(s[c + i]));
                    tmem_st32(tx + PP_PLO + c, u);
                }
            }
            l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars[PB_P0 + x]);
        }
        if (ok && nt > 0)
        {
            ok = __all_sync(FULL_MASK, pp_wait(&bars[PB_O0 + x], nt - 1, abort));
            if (ok)
            {
                tc_fence_after();
                const float inv = 1.0f / l;
                float* dst = a.out + (uint64_t)(b * P + row) * a.ldo + h * PP_HD;
#pragma unroll
                for (int c = 0; c < PP_HD; c += 32)
                {
                    float v[32];
                    tmem_ld32(tx + PP_O + c, v);
                    if (row < P)
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4*>(dst + c + i) =
                                make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
                }
            }
        }
    }
    else if (warp == 8)
    {
        // ---------------- converter ----------------
        const int ct = tid - 256;
        for (uint32_t t = 0; t < ntiles; ++t)
        {
            const uint32_t bf = t & 1u, ph = t >> 1;
            // K(t): lo rows from the hi rows the copy wrote (box j = 512
            // float4 hi, then 512 lo)
            if (!pp_wait(&bars[PB_KF + bf], ph, abort)) break;
            if constexpr (SPLIT3)
            {
                // 16 loads in flight per thread before the stores
#pragma unroll
                for (int c = 0; c < PP_HD / 32; ++c)
                {
                    float4* box = reinterpret_cast<float4*>(k_op + bf * PP_KVOP + c * PP_KBOX);
                    float4 v[16];
#pragma unroll
                    for (int n = 0; n < 16; ++n) v[n] = box[ct + 32 * n];
#pragma unroll
                    for (int n = 0; n < 16; ++n) box[512 + ct + 32 * n] = tf32_lo4(v[n]);
                }
            }
            fence_async_smem();
            mbar_arrive(&bars[PB_KR + bf]);
            // V(t): key block kb = hi boxes (256 float4 each) then lo boxes;
            // rows at or past `nkeys` are zeroed (the cache there may hold
            // anything, and 0 * NaN is NaN)
            if (!pp_wait(&bars[PB_VF + bf], ph, abort)) break;
            {
                const uint32_t k0 = t * PP_KT;
                const uint32_t valid = nkeys - k0 < (uint32_t)PP_KT ? nkeys - k0 : (uint32_t)PP_KT;
#pragma unroll
                for (int c = 0; c < PP_KT / 32; ++c)
                {
                    float4* blk = reinterpret_cast<float4*>(v_op + bf * PP_KVOP + c * PP_VBLK);
                    if (valid == (uint32_t)PP_KT)
                    {
                        if constexpr (SPLIT3)
                        {
                            float4 v[16];
#pragma unroll
                            for (int n = 0; n < 16; ++n) v[n] = blk[ct + 32 * n];
#pragma unroll
                            for (int n = 0; n < 16; ++n) blk[512 + ct + 32 * n] = tf32_lo4(v[n]);
                        }
                    }
                    else
                    {
                        for (int n = 0; n < 16; ++n)
                        {
                            const uint32_t i = ct + 32 * n, key = c * 32 + (i % 256) / 8;
                            if (key >= valid)
                            {
                                blk[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                                if constexpr (SPLIT3) blk[512 + i] = make_float4(0.f, 0.f, 0.f, 0.f);
                            }
                            else if constexpr (SPLIT3)
                                blk[512 + i] = tf32_lo4(blk[i]);
                        }
                    }
                }
            }
            fence_async_smem();
            mbar_arrive(&bars[PB_VR + bf]);
        }
    }
    else if (warp < 11)
    {
        // ---------------- MMA issue for tile x ----------------
        const int x = warp - 9;
        const uint32_t nt = x ? nt1 : nt0;
        if (lane == 0 && nt > 0)
        {
            // descriptors: one base each, advanced by (byte offset >> 4) in
            // the start-address field (shared addresses stay below 2^18)
            const uint64_t dq = smem_desc(q_s + x * PP_QTILE, 0);
            const uint64_t dk = smem_desc(k_op, 0), dv = desc_mn(v_op);
            const uint32_t ts = tmem + PP_TX * x, to = ts + PP_O;
            bool ok = pp_wait(&bars[PB_QR], 0, abort);
            for (uint32_t t = 0; ok && t < nt; ++t)
            {
                const uint32_t bf = t & 1u, ph = t >> 1;
                // S_x(t) = Q_x K(t)^T, after O_x(t-1) has read P_x(t-1)
                if (!(ok = pp_wait(&bars[PB_KR + bf], ph, abort))) break;
                if (t > 0 && !(ok = pp_wait(&bars[PB_O0 + x], t - 1, abort))) break;
                tc_fence_after();
                const uint64_t kbase = dk + ((bf * PP_KVOP) >> 4);
#pragma unroll
                for (int j = 0; j < PP_HD / 32; ++j)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                    {
                        const uint64_t da = dq + ((j * (128 * 128) + kk * 32) >> 4);
                        const uint64_t db = kbase + ((j * PP_KBOX + kk * 32) >> 4);
                        if constexpr (SPLIT3)
                        {
                            // [hi.hi | hi.lo] in one MMA, then lo.hi (Q lo from TMEM) into the first half
                            mma_tf32(ts, da, db, IDESC_S2, j > 0 || kk > 0);
                            mma_tf32_tmem_a(ts, ts + PP_QLO + 32 * j + 8 * kk, db, IDESC_S, true);
                        }
                        else
                            mma_tf32(ts, da, db, IDESC_S, j > 0 || kk > 0);
                    }
                mma_commit(&bars[PB_S0 + x]);
                mma_commit(&bars[PB_KE + 2 * x + bf]);
                // O_x += P_x(t) V(t)
                if (!(ok = pp_wait(&bars[PB_VR + bf], ph, abort))) break;
                if (!(ok = pp_wait(&bars[PB_P0 + x], t, abort))) break;
                tc_fence_after();
                const uint64_t vbase = dv + ((bf * PP_KVOP) >> 4);
#pragma unroll
                for (int kb = 0; kb < PP_KT / 32; ++kb)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                    {
                        const uint64_t db = vbase + ((kb * PP_VBLK + kk * 1024) >> 4);
                        const uint32_t col = kb * 32 + kk * 8;
                        mma_tf32_tmem_a(to, ts + col, db, IDESC_O, t > 0 || kb > 0 || kk > 0);
                        if constexpr (SPLIT3)
                        {
                            mma_tf32_tmem_a(to, ts + col, db + (8192 >> 4), IDESC_O, true);  // P hi . V lo
                            mma_tf32_tmem_a(to, ts + PP_PLO + col, db, IDESC_O, true);      // P lo . V hi
                        }
                    }
                mma_commit(&bars[PB_O0 + x]);
                mma_commit(&bars[PB_VE + 2 * x + bf]);
            }
            // every MMA this thread issued completes before TMEM is freed
            mma_commit(&bars[PB_FIN + x]);
            mbar_wait(&bars[PB_FIN + x], 0);
        }
    }
    else
    {
        // ---------------- TMA copies ----------------
        if (lane == 0)
        {
            const int nq = has_b ? 2 : 1;
            mbar_arrive_expect_tx(&bars[PB_QF], nq * PP_QTILE);
            for (int x = 0; x < nq; ++x)
                for (int j = 0; j < PP_HD / 32; ++j)
                    tma_load_2d(q_s + x * PP_QTILE + j * (128 * 128), &map_q, (int)(h * PP_HD) + 32 * j,
                                (int)(b * P + q0 + 128 * x), &bars[PB_QF]);
            uint32_t issued = 0;
            for (uint32_t t = 0; t < ntiles; ++t)
            {
                const uint32_t bf = t & 1u;
                // K(t) into buffer t % 2 once S_A(t-2) and S_B(t-2) have read it
                if (t >= 2 && t - 2 < nt0 && !pp_wait(&bars[PB_KE + bf], (t >> 1) - 1, abort)) break;
                if (t >= 2 && t - 2 < nt1 && !pp_wait(&bars[PB_KE + 2 + bf], (t >> 1) - 1, abort)) break;
                mbar_arrive_expect_tx(&bars[PB_KF + bf], PP_KVT);
                for (int j = 0; j < PP_HD / 32; ++j)
                    tma_load_2d(k_op + bf * PP_KVOP + j * PP_KBOX, &map_k, 32 * j, kv_row0 + (int)(t * PP_KT),
                                &bars[PB_KF + bf]);
                // V(t) once O_A(t-2) and O_B(t-2) have
                if ((t >= 2 && t - 2 < nt0 && !pp_wait(&bars[PB_VE + bf], (t >> 1) - 1, abort)) ||
                    (t >= 2 && t - 2 < nt1 && !pp_wait(&bars[PB_VE + 2 + bf], (t >> 1) - 1, abort)))
                {
                    issued = 2 * t + 1;
                    break;
                }
                mbar_arrive_expect_tx(&bars[PB_VF + bf], PP_KVT);
                for (int kb = 0; kb < PP_KT / 32; ++kb)
                    for (int j = 0; j < PP_HD / 32; ++j)
                        tma_load_2d(v_op + bf * PP_KVOP + kb * PP_VBLK + j * 4096, &map_v, 32 * j,
                                    kv_row0 + (int)(t * PP_KT) + 32 * kb, &bars[PB_VF + bf]);
                issued = 2 * t + 2;
            }
            // the copies this thread started land before the CTA exits
            // (bounded; immediate on the normal path).  Copy n < issued is
            // K(n / 2) for even n, V(n / 2) for odd n.
            mbar_wait(&bars[PB_QF], 0);
            for (uint32_t n = issued >= 4 ? issued - 4 : 0; n < issued; ++n)
            {
                const uint32_t t = n >> 1;
                mbar_wait(&bars[(n & 1u ? PB_VF : PB_KF) + (t & 1u)], t >> 1);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort) atomicAdd(&g_prefill_tc_timeouts, 1);
    if (warp == 0)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

namespace {

template <int HD, bool SPLIT3>
int launch_tc_hd(const float* q, uint32_t ldq, const float* kc, const float* vc, uint32_t C, float* out, uint32_t ldo,
                 uint32_t B, uint32_t H, uint32_t P, float scale, cudaStream_t st)
{
    using Sh = PfShape<HD>;
    auto kern = prefill_attention_tc_kernel<HD, SPLIT3>;
    static uint64_t attr_devices = 0;
    FML_RC(smem_limit_once(reinterpret_cast<const void*>(kern), (int)Sh::SMEM, attr_devices));
    CUtensorMap mq, mk, mv;
    const uint64_t rows = (uint64_t)B * H * C;
    FML_REQUIRE(rows < (1ull << 31) && (uint64_t)B * P < (1ull << 31), "prefill attention: %llu cache rows",
                (unsigned long long)rows);
    FML_RC(tc::make_map(&mq, q, (int)(B * P), (int)(H * HD), (int)ldq, QB));
    FML_RC(tc::make_map(&mk, kc, (int)rows, HD, HD, Sh::KT));
    FML_RC(tc::make_map(&mv, vc, (int)rows, HD, HD, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
    PfArgs a{out, ldo, B, H, P, C, scale};
    dim3 grid((P + QB - 1) / QB, H, B);
    kern<<<grid, 128, Sh::SMEM, st>>>(mq, mk, mv, a);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

template <bool SPLIT3>
int launch_pp(const float* q, uint32_t ldq, const float* kc, const float* vc, uint32_t C, float* out, uint32_t ldo,
              uint32_t B, uint32_t H, uint32_t P, float scale, cudaStream_t st)
{
    auto kern = prefill_attention_pp_kernel<SPLIT3>;
    static uint64_t attr_devices = 0;
    FML_RC(smem_limit_once(reinterpret_cast<const void*>(kern), (int)PP_SMEM, attr_devices));
    CUtensorMap mq, mk, mv;
    const uint64_t rows = (uint64_t)B * H * C;
    FML_REQUIRE(rows < (1ull << 31) && (uint64_t)B * P < (1ull << 31), "prefill attention: %llu cache rows",
                (unsigned long long)rows);
    FML_RC(tc::make_map(&mq, q, (int)(B * P), (int)(H * PP_HD), (int)ldq, 128));
    FML_RC(tc::make_map(&mk, kc, (int)rows, PP_HD, PP_HD, PP_KT));
    FML_RC(tc::make_map(&mv, vc, (int)rows, PP_HD, PP_HD, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
    PfArgs a{out, ldo, B, H, P, C, scale};
    dim3 grid((P + 255) / 256, H, B);
    kern<<<grid, PP_THREADS, PP_SMEM, st>>>(mq, mk, mv, a);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

}  // namespace

// The tensor-core prefill attention.  q / out [B*P x ld] (head h at columns
// h*hd); keys and values of sequence b, head h at kc/vc + b*seq_stride +
// h*C*hd, rows 0..P-1 filled.  split3: TF32x3 (fp32-level), else one TF32
// product.  FML_ERR_UNSUPPORTED (no error recorded) for the layouts it does
// not take -- head dims other than 32 / 64 / 128, a cache whose sequences are
// not packed back to back, unaligned pointers or strides -- and the caller
// then uses the CUDA-core kernel.
int launch_prefill_attention_tc(const float* q, uint32_t ldq, const float* kc, const float* vc, uint64_t seq_stride,
                                uint32_t C, float* out, uint32_t ldo, uint32_t B, uint32_t H, uint32_t P, uint32_t hd,
                                float scale, bool split3, cudaStream_t st)
{
    if (!(hd == 32 || hd == 64 || hd == 128) || seq_stride != (uint64_t)H * C * hd || ldq % 4 || ldo % 4 ||
        !aligned16(q) || !aligned16(kc) || !aligned16(vc) || !aligned16(out) || B > 65535u || H > 65535u || P == 0)
        return FML_ERR_UNSUPPORTED;
    // FML_PREFILL_ATTN_SIMPLE=1: the one-tile kernel at head dim 64 as well
    // (tests run both)
    const char* simple = getenv("FML_PREFILL_ATTN_SIMPLE");
    if (hd == 64 && !(simple && simple[0] == '1'))
        return split3 ? launch_pp<true>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st)
                      : launch_pp<false>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st);
    if (split3)
    {
        if (hd == 32) return launch_tc_hd<32, true>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st);
        if (hd == 64) return launch_tc_hd<64, true>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st);
        return launch_tc_hd<128, true>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st);
    }
    if (hd == 32) return launch_tc_hd<32, false>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st);
    if (hd == 64) return launch_tc_hd<64, false>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st);
    return launch_tc_hd<128, false>(q, ldq, kc, vc, C, out, ldo, B, H, P, scale, st);
}

int launch_prefill_attention(const float* q, uint32_t ldq, const float* kc, const float* vc, uint64_t seq_stride,
                             uint32_t C, float* out, uint32_t ldo, uint32_t B, uint32_t H, uint32_t P, uint32_t hd,
                             float scale, cudaStream_t st);

int prefill_tc_error_count(int* out)
{
    FML_CUDA_TRY(cudaMemcpyFromSymbol(out, g_prefill_tc_timeouts, sizeof(int)));
    return FML_OK;
}

}  // namespace fml

using namespace fml;

extern "C" FML_API int fml_attention_prefill(float* out, const float* q, const float* kcache, const float* vcache,
                                             uint32_t batch, uint32_t heads, uint32_t head_dim, uint32_t context,
                                             uint32_t prompt_len, float scale, int mode, fml_stream_t stream)
{
    if (batch == 0 || prompt_len == 0) return FML_OK;
    FML_REQUIRE(out && q && kcache && vcache, "fml_attention_prefill: null pointer");
    FML_REQUIRE(heads >= 1 && prompt_len <= context, "fml_attention_prefill: %u heads, prompt %u, context %u", heads,
                prompt_len, context);
    FML_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128,
                "fml_attention_prefill: head_dim %u (need 32, 64 or 128)", head_dim);
    FML_REQUIRE(mode == FML_MATH_FP32 || mode == FML_MATH_TF32X3 || mode == FML_MATH_TF32,
                "fml_attention_prefill: unknown math mode %d", mode);
    const uint32_t ld = heads * head_dim;
    const uint64_t seq_stride = (uint64_t)heads * context * head_dim;
    cudaStream_t st = as_stream(stream);
    if (mode != FML_MATH_FP32)
    {
        const int rc = launch_prefill_attention_tc(q, ld, kcache, vcache, seq_stride, context, out, ld, batch, heads,
                                                   prompt_len, head_dim, scale, mode == FML_MATH_TF32X3, st);
        if (rc != FML_ERR_UNSUPPORTED) return rc;
    }
    return launch_prefill_attention(q, ld, kcache, vcache, seq_stride, context, out, ld, batch, heads, prompt_len,
                                    head_dim, scale, st);
}
