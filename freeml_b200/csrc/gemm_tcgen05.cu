// Tensor-core contractions on sm_100a (tcgen05 + TMEM + TMA): the batched /
// prefill Dense products Mul<None|Right> (MatrixBase_Mul.h:591-615) for the
// large-M shapes.
//
//   C[M x N] (+ epilogue) = A[M x K] . B[N x K]^T        (both K-contiguous)
//   C[M x N]                = A[M x K] . B[K x N]          (BMN: B row-major)
//
// 128 x 128 output tiles, K staged 32 fp32 (one 128-byte row) at a time
// through a 4-stage ring of TMA tensor loads (128-byte swizzle, each load into
// this CTA only); a persistent CTA per SM walks the tiles with the
// accumulator double-buffered in TMEM (2 x 128 lanes x 128 fp32 columns).
// Warp roles (10 warps):
//   warp 0      TMEM allocation; one thread issues the TMA loads
//   warp 1      one thread issues tcgen05.mma and tcgen05.commit
//   warps 2..5  TF32x3 split of each staged A tile into TMEM (and of the B
//               tile into shared memory, unless B's lo part is given)
//   warps 6..9  epilogue (tcgen05.ld of a finished accumulator, store to
//               global with the fused GELU or residual add)
//
// Precision: kind::tf32 reads only the top 19 bits of each fp32 operand.
// TF32x3 (default) splits x = hi + lo with hi = x with the low 13 bits
// cleared -- which is what the MMA reads from the staged tile itself, so hi
// is never written -- and lo = x - hi (exact in fp32), then sums
// hi*hi + hi*lo + lo*hi in the fp32 accumulator -- fp32-level results at
// three MMAs per k-step.  A's lo part goes to TMEM (the lo.hi MMA reads its
// A operand from there), which keeps a stage at three 16 KB tiles and the
// ring four stages deep.  TF32 (one MMA, hardware truncation) is the fast,
// looser mode.
//
// Every mbarrier wait is bounded; a wait that runs out sets the device error
// count (fml_device_error_count), waits (bounded) for the MMAs in flight and
// still frees the CTA's TMEM before returning.
#include <algorithm>

#include "tcgen05.cuh"

namespace fml {

__device__ int g_gemm_timeouts;

namespace tc {

constexpr int BM = 128, BN = 128;
constexpr int STAGES = 4;
constexpr uint32_t TILE_BYTES = BM * BK * 4;  // 16 KB (A or B tile)
constexpr uint32_t TMEM_COLS = 128;
// TMEM: two 128-column accumulators, then A's TF32 lo part of each stage (32
// columns: lane = A row, one column per k), the A operand of the lo.hi MMAs
constexpr uint32_t ALO_COL = 2 * TMEM_COLS, TMEM_ALLOC = 512;
constexpr uint32_t IDESC = idesc_tf32(BM, BN);
constexpr uint32_t IDESC_BMN = IDESC | (1u << 16);  // B read MN-major (bit 16: "transpose B")
constexpr uint32_t MN_BOX = 32;                      // n per 128-byte swizzle row of an MN-major B tile

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, bool accumulate)
{
    mma_tf32(tmem_d, da, db, IDESC, accumulate);
}

// MN-major B operand of one K = 8 step.  tf32 accepts only one MN-major
// shared-memory layout, the 128-byte swizzle with 32-byte atoms (descriptor
// layout type 1, "128B_BASE32B"): rows of 32 n (128 bytes) whose four 32-byte
// chunks are permuted by the row index mod 4, in 4-row / 512-byte atoms --
// what a 32 n x 32 k TMA box with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B lands.
// (The 16-byte-atom 128-byte swizzle of the K-major operands, with the
// transpose bit set, made every tf32 MMA produce zeros on B200.)  The tile
// holds BN / 32 such boxes of [32 k x 32 n] (4 KB each): the next 32 n one box
// on (LBO = 4 KB), the next 4 k one atom on (SBO = 512 B), so K step kk (8 k)
// starts 1 KB further.
__device__ __forceinline__ uint64_t smem_desc_mn(const void* tile, uint32_t kk)
{
    const uint64_t start = (uint64_t)((smem_u32(tile) + kk * 1024u) >> 4) & 0x3FFFull;
    const uint64_t lbo = (MN_BOX * BK * 4u) >> 4;  // next 32 n: the next box
    const uint64_t sbo = 512ull >> 4;              // next 4 k: the next atom
    return start | (lbo << 16) | (sbo << 32) | (1ull << 46) | (1ull << 61);
}

// One stage's MMAs (BK / 8 = 4 K steps) and the commit that frees the stage,
// in ONE asm block that first probes (mbarrier.test_wait, non-blocking) the
// barrier of the next stage and reads the probe's answer only after the MMAs
// are issued.  The tensor pipe's instruction queue is short, so a wait issued
// between two stages -- even on a barrier already complete, ~170 cycles --
// lets it drain; here the probe's latency overlaps the issue of the MMAs.
// Descriptors advance per K step by a_step / b_step (16-byte units: 32 bytes
// along a K-major row, 1 KB for the MN-major B).  Returns the probe's answer.
// The lo.hi term reads A's lo part from TMEM (talo: 8 columns per K step).
template <bool SPLIT3>
__device__ __forceinline__ bool issue_stage_probe(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t talo,
                                                  uint64_t dblo, uint32_t idesc, bool accumulate, uint64_t b_step,
                                                  uint64_t* empty_bar, uint64_t* next_bar, uint32_t next_parity)
{
    uint32_t ready;
    if constexpr (SPLIT3)
    {
        asm volatile(
            "{\n\t"
            ".reg .pred pr, pa, p1;\n\t"
            ".reg .b64 a, b, bl;\n\t"
            ".reg .b32 al;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 pr, [%1], %2;\n\t"
            "setp.ne.b32 pa, %8, 0;\n\t"
            "setp.eq.b32 p1, 0, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], %4, %5, %9, pa;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], %4, %7, %9, p1;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], [%6], %5, %9, p1;\n\t"
            "add.s64 a, %4, 2;\n\tadd.s64 b, %5, %10;\n\tadd.u32 al, %6, 8;\n\tadd.s64 bl, %7, %10;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, b, %9, p1;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, bl, %9, p1;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], [al], b, %9, p1;\n\t"
            "add.s64 a, a, 2;\n\tadd.s64 b, b, %10;\n\tadd.u32 al, al, 8;\n\tadd.s64 bl, bl, %10;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, b, %9, p1;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, bl, %9, p1;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], [al], b, %9, p1;\n\t"
            "add.s64 a, a, 2;\n\tadd.s64 b, b, %10;\n\tadd.u32 al, al, 8;\n\tadd.s64 bl, bl, %10;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, b, %9, p1;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, bl, %9, p1;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], [al], b, %9, p1;\n\t"
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%11];\n\t"
            "selp.u32 %0, 1, 0, pr;\n\t"
            "}"
            : "=r"(ready)
            : "r"(smem_u32(next_bar)), "r"(next_parity), "r"(tmem_d), "l"(da), "l"(db), "r"(talo), "l"(dblo),
              "r"((uint32_t)accumulate), "r"(idesc), "l"(b_step), "r"(smem_u32(empty_bar))
            : "memory");
    }
    else
    {
        asm volatile(
            "{\n\t"
            ".reg .pred pr, pa, p1;\n\t"
            ".reg .b64 a, b;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 pr, [%1], %2;\n\t"
            "setp.ne.b32 pa, %6, 0;\n\t"
            "setp.eq.b32 p1, 0, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], %4, %5, %7, pa;\n\t"
            "add.s64 a, %4, 2;\n\tadd.s64 b, %5, %8;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, b, %7, p1;\n\t"
            "add.s64 a, a, 2;\n\tadd.s64 b, b, %8;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, b, %7, p1;\n\t"
            "add.s64 a, a, 2;\n\tadd.s64 b, b, %8;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%3], a, b, %7, p1;\n\t"
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%9];\n\t"
            "selp.u32 %0, 1, 0, pr;\n\t"
            "}"
            : "=r"(ready)
            : "r"(smem_u32(next_bar)), "r"(next_parity), "r"(tmem_d), "l"(da), "l"(db), "r"((uint32_t)accumulate),
              "r"(idesc), "l"(b_step), "r"(smem_u32(empty_bar))
            : "memory");
    }
    return ready != 0;
}

}  // namespace tc

enum TcEpi { TC_STORE = 0, TC_GELU = 1, TC_RESID = 2, TC_QKV = 3 };

struct TcArgs
{
    int M, N, K;
    float* C;         // [M x N], row stride ldc
    int ldc;
    const float* R;   // TC_RESID: C = R + A.B^T (row stride ldc)
    bool vec4;        // C (and R) 16-byte aligned with ldc a multiple of 4
    // TC_QKV (the prefill's packed QKV rows, row = b * P + t): columns
    // [0, dq) go to C (row stride ldc), [dq, 2 dq) to the K cache and
    // [2 dq, 3 dq) to the V cache at cache + b * seq_stride +
    // (h * ctx + t) * hd + e for column h * hd + e of the part
    float* kc;
    float* vc;
    int P, hd, dq, ctx;
    uint64_t seq_stride;
    // split K (TC_STORE only): tile t covers k-blocks [ks kbs, (ks + 1) kbs)
    // of K with ks = t / (M and N tiles), and stores its partial product to
    // C + ks * M * ldc; 0 or 1 = no split
    int ksplit;
    bool pdl;  // launch under programmatic dependent launch
};

// One CTA per SM walks the output tiles t = blockIdx.x, blockIdx.x +
// gridDim.x, ... (n fastest, so that a wave shares its A rows).  The stage
// ring runs on across tile boundaries, and the accumulator is double-buffered
// in TMEM (2 x 128 columns) so that four epilogue warps drain tile j while
// the MMAs of tile j + 1 run (measured against one CTA per tile, whose
// tensor pipe idled while it filled its pipeline and drained its epilogue:
// config 4 prefill 339 -> 320 ms).
// Shared memory: STAGES x {A, B, B_lo} tiles (1024-byte aligned), then
// barriers and the TMEM base address.  TMEM: two accumulators and A_lo of
// each stage.  BLO (TF32x3 only): B's lo part is
// given in memory (map_blo, same geometry as map_b) and TMA-loaded into the
// B_lo tile; the converters split A only.
// Warp roles (10 warps):
//   warp 0      TMEM allocation; one thread issues the TMA loads
//   warp 1      one thread issues tcgen05.mma / tcgen05.commit
//   warps 2..5  TF32x3 split of each staged A tile into TMEM, and of B
//               without B_lo (relay only without split)
//   warps 6..9  epilogue: tcgen05.ld of a finished accumulator, store
// Barriers: full / conv / empty per stage (TMA landed / split done / MMAs have
// read it), acc_full / acc_empty per accumulator (MMAs done / drained).
// BMN: B is [K x N] row-major (Mul<None>, MatMul_Strided<None>): each stage
// loads it as BN / 32 boxes of 32 k x 32 n and the MMA reads it MN-major.
template <bool SPLIT3, int EPI, bool BLO = false, bool BMN = false>
__global__ void __launch_bounds__(320, 1) gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                         const __grid_constant__ CUtensorMap map_b,
                                                                         const __grid_constant__ CUtensorMap map_blo,
                                                                         TcArgs args)
{
    using namespace tc;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int NT = SPLIT3 ? 3 : 2;  // shared-memory tiles per stage: A, B (, B lo)
    unsigned char* tiles = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(tiles + STAGES * NT * TILE_BYTES);
    uint64_t* conv = full + STAGES;
    uint64_t* empty = conv + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* done = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ksplit = args.ksplit > 1 ? args.ksplit : 1;
    const int kblocks = (args.K + BK - 1) / BK / ksplit;  // k-blocks per tile (host: divisible)
    const int tiles_n = (args.N + BN - 1) / BN;
    const int tiles_mn = tiles_n * ((args.M + BM - 1) / BM);
    const int ntiles = tiles_mn * ksplit;

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < STAGES; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 4);  // one arrival per converter warp
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_ALLOC)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    bool ok = true;

    auto tile_ptr = [&](int stage, int which) { return tiles + (stage * NT + which) * TILE_BYTES; };

    // Programmatic dependent launch (the decode contractions): the weight
    // operand B does not depend on the previous kernel, so the first STAGES
    // stages' B tiles are requested before griddepcontrol.wait and their A
    // tiles after it; every role that touches global memory the previous
    // kernel writes (the A loads, the epilogue's residual reads and its
    // stores into buffers that kernel may still read) waits first.  Without
    // the launch attribute the wait returns at once.
    griddep_launch_dependents();
    if (warp == 0)
    {
        if (lane == 0)
        {
            // iteration it of this CTA: its (it / kblocks)-th tile, k-block it % kblocks
            auto coords = [&](uint32_t i, int& k, int& m0, int& n0) {
                const int t = (int)blockIdx.x + (int)(i / (uint32_t)kblocks) * (int)gridDim.x;
                const int tmn = t % tiles_mn;
                k = (t / tiles_mn) * kblocks * BK + (int)(i % (uint32_t)kblocks) * BK;
                m0 = (tmn / tiles_n) * BM;
                n0 = (tmn % tiles_n) * BN;
            };
            auto load_b = [&](int s, int k, int n0) {
                if constexpr (BMN)
                {
#pragma unroll
                    for (int j = 0; j < BN / (int)MN_BOX; ++j)
                        tma_load_2d(tile_ptr(s, 1) + j * (MN_BOX * BK * 4), &map_b, n0 + j * (int)MN_BOX, k, &full[s]);
                }
                else
                    tma_load_2d(tile_ptr(s, 1), &map_b, k, n0, &full[s]);
                if constexpr (BLO) tma_load_2d(tile_ptr(s, 2), &map_blo, k, n0, &full[s]);
            };
            const uint32_t mytiles = (uint32_t)((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x);
            const uint32_t total = (uint32_t)kblocks * (blockIdx.x < (unsigned)ntiles ? mytiles : 0u);
            const uint32_t pre = total < (uint32_t)STAGES ? total : (uint32_t)STAGES;
            for (uint32_t i = 0; i < pre; ++i)
            {
                int k, m0, n0;
                coords(i, k, m0, n0);
                mbar_arrive_expect_tx(&full[i], (BLO ? 3 : 2) * TILE_BYTES);
                load_b((int)i, k, n0);
            }
            griddep_wait();
            for (uint32_t i = 0; i < pre; ++i)
            {
                int k, m0, n0;
                coords(i, k, m0, n0);
                tma_load_2d(tile_ptr((int)i, 0), &map_a, k, m0, &full[i]);
            }
            uint32_t it = pre;  // k-blocks issued over all tiles
            for (; it < total && ok; ++it)
            {
                const int s = it % STAGES;
                if (!mbar_wait(&empty[s], ((it / STAGES) - 1) & 1)) { ok = false; break; }
                int k, m0, n0;
                coords(it, k, m0, n0);
                mbar_arrive_expect_tx(&full[s], (BLO ? 3 : 2) * TILE_BYTES);
                tma_load_2d(tile_ptr(s, 0), &map_a, k, m0, &full[s]);
                load_b(s, k, n0);
            }
            // the last STAGES loads issued (all earlier ones were consumed):
            // none may still be landing when the CTA exits
            for (uint32_t i = it > (uint32_t)STAGES ? it - STAGES : 0u; i < it; ++i)
                if (!mbar_wait(&full[i % STAGES], (i / STAGES) & 1)) ok = false;
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            static_assert(BK == 32, "issue_stage_probe issues 4 K steps of 8");
            uint32_t it = 0, j = 0;  // k-blocks consumed, tiles accumulated
            const uint32_t total = (uint32_t)kblocks * (uint32_t)((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) /
                                                                  (int)gridDim.x);
            bool ready = false;  // conv[it % STAGES] known complete (the previous stage's probe)
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++j)
            {
                const uint32_t buf = j & 1u, use = j >> 1;
                if (use >= 1 && !mbar_wait(&acc_empty[buf], (use - 1) & 1)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc_tmem = tmem_base + buf * TMEM_COLS;
                for (int kb = 0; kb < kblocks; ++kb, ++it)
                {
                    const int s = it % STAGES;
                    if (!ready && !mbar_wait(&conv[s], (it / STAGES) & 1)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // probe the next stage (the last one probes its own, already complete, barrier)
                    const uint32_t nx = it + 1 < total ? it + 1 : it;
                    const uint64_t da = smem_desc(tile_ptr(s, 0), 0);
                    const uint32_t talo = tmem_base + ALO_COL + 32u * (uint32_t)s;
                    uint64_t db, dblo;
                    if constexpr (BMN)
                    {
                        db = smem_desc_mn(tile_ptr(s, 1), 0);
                        dblo = smem_desc_mn(tile_ptr(s, 2), 0);
                    }
                    else
                    {
                        db = smem_desc(tile_ptr(s, 1), 0);
                        dblo = smem_desc(tile_ptr(s, 2), 0);
                    }
                    ready = issue_stage_probe<SPLIT3>(acc_tmem, da, db, talo, dblo, BMN ? IDESC_BMN : IDESC, kb > 0,
                                                      BMN ? 64u : 2u, &empty[s], &conv[nx % STAGES],
                                                      (nx / STAGES) & 1);
                    if (nx == it) ready = false;
                }
                if (!ok) break;
                mma_commit(&acc_full[buf]);  // the accumulator is complete
            }
            mma_commit(done);  // every MMA this thread issued
        }
    }
    else if (warp < 6)
    {
        // warps 2..5: A's lo part into TMEM (thread = TMEM lane = A row: warp
        // w may access lanes 32 (w % 4) ..), and B's into shared memory
        // unless B_lo is given
        const int ct = threadIdx.x - 64;  // 0..127
        const int r = 32 * (warp & 3) + lane;
        const uint32_t tlane = (uint32_t)(32 * (warp & 3)) << 16;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x)
        {
            for (int kb = 0; kb < kblocks; ++kb, ++it)
            {
                const int s = it % STAGES;
                if (!__all_sync(FULL_MASK, mbar_wait(&full[s], (it / STAGES) & 1))) { ok = false; break; }
                if constexpr (SPLIT3)
                {
                    // row r of the A tile: logical 16-byte chunk c (k = 4c..)
                    // at physical chunk c ^ (r % 8) (128-byte swizzle)
                    const unsigned char* arow = tile_ptr(s, 0) + r * 128;
                    uint32_t u[32];
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                    {
                        const float4 lo = tf32_lo4(*reinterpret_cast<const float4*>(arow + ((c ^ (r & 7)) * 16)));
                        u[4 * c] = __float_as_uint(lo.x);
                        u[4 * c + 1] = __float_as_uint(lo.y);
                        u[4 * c + 2] = __float_as_uint(lo.z);
                        u[4 * c + 3] = __float_as_uint(lo.w);
                    }
                    tmem_st32(tmem_base + tlane + ALO_COL + 32u * (uint32_t)s, u);
                    if constexpr (!BLO)
                    {
                        const float4* x4 = reinterpret_cast<const float4*>(tile_ptr(s, 1));
                        float4* lo = reinterpret_cast<float4*>(tile_ptr(s, 2));
#pragma unroll
                        for (int i = ct; i < (int)(TILE_BYTES / 16); i += 128) lo[i] = tf32_lo4(x4[i]);
                        // make these generic-proxy writes visible to the tensor core
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    }
                    tmem_wait_st();
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&conv[s]);
            }
        }
    }
    else
    {
        // warps 6..9: drain the accumulators; warp w reads TMEM lanes
        // 32 (w % 4) .. 32 (w % 4) + 31
        const int lg = warp & 3;
        griddep_wait();  // residual reads and output stores follow the previous kernel
        uint32_t j = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j)
        {
            const uint32_t buf = j & 1u, use = j >> 1;
            if (!__all_sync(FULL_MASK, mbar_wait(&acc_full[buf], use & 1))) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int tmn = t % tiles_mn;
            const int m0 = (tmn / tiles_n) * BM, n0 = (tmn % tiles_n) * BN;
            const int row = m0 + lg * 32 + lane;
            float* const cbase = args.C + (uint64_t)(t / tiles_mn) * args.M * args.ldc;  // split-K plane
            for (int c0 = 0; c0 < BN; c0 += 32)
            {
                float v[32];
                tc::tmem_ld32(tmem_base + ((uint32_t)(lg * 32) << 16) + buf * TMEM_COLS + (uint32_t)c0, v);
                if (row < args.M)
                {
                    float* crow = cbase + (uint64_t)row * args.ldc + n0 + c0;
                    if constexpr (EPI == TC_QKV)
                    {
                        // a 32-column slice lies inside one head of one part
                        // (dq and hd are multiples of 32): one base address
                        const int n = n0 + c0;
                        if (n >= args.dq)
                        {
                            const bool isk = n < 2 * args.dq;
                            const int c = isk ? n - args.dq : n - 2 * args.dq;
                            const int b = row / args.P, tq = row - b * args.P;
                            crow = (isk ? args.kc : args.vc) + (uint64_t)b * args.seq_stride +
                                   ((uint64_t)(c / args.hd) * args.ctx + tq) * args.hd + c % args.hd;
                        }
                        else
                            crow = args.C + (uint64_t)row * args.ldc + n;
                    }
                    const float* rrow = EPI == TC_RESID ? args.R + (uint64_t)row * args.ldc + n0 + c0 : nullptr;
                    if (args.vec4 && n0 + c0 + 32 <= args.N)
                    {
                        // whole 32-column slice, 16-byte aligned rows: float4
                        // stores (and residual loads), a quarter of the
                        // memory instructions of the scalar path
#pragma unroll
                        for (int jj = 0; jj < 32; jj += 4)
                        {
                            float4 x = make_float4(v[jj], v[jj + 1], v[jj + 2], v[jj + 3]);
                            if constexpr (EPI == TC_GELU)
                            {
                                x.x = gelu_exact(x.x); x.y = gelu_exact(x.y);
                                x.z = gelu_exact(x.z); x.w = gelu_exact(x.w);
                            }
                            if constexpr (EPI == TC_RESID)
                            {
                                const float4 r = *reinterpret_cast<const float4*>(rrow + jj);
                                x.x += r.x; x.y += r.y; x.z += r.z; x.w += r.w;
                            }
                            *reinterpret_cast<float4*>(crow + jj) = x;
                        }
                    }
                    else
                    {
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj)
                        {
                            if (n0 + c0 + jj < args.N)
                            {
                                float x = v[jj];
                                if constexpr (EPI == TC_GELU) x = gelu_exact(x);
                                if constexpr (EPI == TC_RESID) x += rrow[jj];
                                crow[jj] = x;
                            }
                        }
                    }
                }
            }
            // this warp's reads of the accumulator are complete
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }

    if (!ok && lane == 0) atomicAdd(&g_gemm_timeouts, 1);
    // the MMAs must have finished with TMEM before it is freed (bounded)
    if (warp == 1 && lane == 0) tc::mbar_wait(done, 0);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
    {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_ALLOC)
                     : "memory");
    }
}

// ---- host side ---------------------------------------------------------------

template <bool SPLIT3>
constexpr size_t tc_smem_bytes()
{
    return 1024 + (size_t)tc::STAGES * (SPLIT3 ? 3 : 2) * tc::TILE_BYTES + 32 * 8;
}

// The kernel's dynamic shared-memory limit, raised once per device.
template <bool SPLIT3, int EPI, bool BLO, bool BMN>
static int tc_smem_setup()
{
    static uint64_t attr_devices = 0;
    return smem_limit_once(reinterpret_cast<const void*>(gemm_tcgen05_kernel<SPLIT3, EPI, BLO, BMN>),
                           (int)tc_smem_bytes<SPLIT3>(), attr_devices);
}

template <bool SPLIT3, int EPI, bool BLO = false, bool BMN = false>
static int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mblo, const TcArgs& args,
                     cudaStream_t st)
{
    const size_t smem = tc_smem_bytes<SPLIT3>();
    FML_RC((tc_smem_setup<SPLIT3, EPI, BLO, BMN>()));
    int dev = 0, sms = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    FML_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int ntiles = ((args.N + tc::BN - 1) / tc::BN) * ((args.M + tc::BM - 1) / tc::BM) * std::max(1, args.ksplit);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min(ntiles, sms));
    cfg.blockDim = dim3(320);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = args.pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tcgen05_kernel<SPLIT3, EPI, BLO, BMN>, ma, mb, mblo, args);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "gemm_tcgen05 launch: %s", cudaGetErrorString(e));
    FML_LAUNCH_CHECK();
    return FML_OK;
}

// Raise the dynamic shared-memory limit of gemm_tc's kernel for (split3,
// epi, B_lo given) on the current device, so that a later launch inside a
// stream capture makes no attribute call.
int gemm_tc_prepare(bool split3, int epi, bool blo)
{
    if (split3 && blo)
    {
        if (epi == TC_GELU) return tc_smem_setup<true, TC_GELU, true, false>();
        if (epi == TC_RESID) return tc_smem_setup<true, TC_RESID, true, false>();
        return tc_smem_setup<true, TC_STORE, true, false>();
    }
    if (split3)
    {
        if (epi == TC_GELU) return tc_smem_setup<true, TC_GELU, false, false>();
        if (epi == TC_RESID) return tc_smem_setup<true, TC_RESID, false, false>();
        return tc_smem_setup<true, TC_STORE, false, false>();
    }
    if (epi == TC_GELU) return tc_smem_setup<false, TC_GELU, false, false>();
    if (epi == TC_RESID) return tc_smem_setup<false, TC_RESID, false, false>();
    return tc_smem_setup<false, TC_STORE, false, false>();
}

// C = A . B^T (+ epilogue) on the tensor cores.  A [M x K] (row stride lda),
// B [N x K] (row stride ldb), both 16-byte aligned with lda, ldb multiples of
// 4 (TMA's rules); split3 selects TF32x3.  B_lo (optional, TF32x3): B's lo
// part B - hi(B) in B's layout, so that only A is split in the kernel.
int gemm_tc(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, bool split3,
            int epi, const float* R, cudaStream_t st, const float* B_lo)
{
    if (M <= 0 || N <= 0) return FML_OK;
    FML_REQUIRE(K > 0, "gemm_tc: K must be positive");
    FML_REQUIRE(aligned16(A) && aligned16(B) && lda % 4 == 0 && ldb % 4 == 0 && (!B_lo || aligned16(B_lo)),
                "gemm_tc: operands must be 16-byte aligned with row strides that are multiples of 4");
    CUtensorMap ma, mb, mblo;
    FML_RC(tc::make_map(&ma, A, M, K, lda, tc::BM));
    FML_RC(tc::make_map(&mb, B, N, K, ldb, tc::BN));
    const bool blo = split3 && B_lo;
    if (blo) FML_RC(tc::make_map(&mblo, B_lo, N, K, ldb, tc::BN));
    else mblo = mb;
    TcArgs args{M, N, K, C, ldc, R, aligned16(C) && (!R || aligned16(R)) && ldc % 4 == 0};
    if (blo)
    {
        if (epi == TC_GELU) return launch_tc<true, TC_GELU, true>(ma, mb, mblo, args, st);
        if (epi == TC_RESID) return launch_tc<true, TC_RESID, true>(ma, mb, mblo, args, st);
        return launch_tc<true, TC_STORE, true>(ma, mb, mblo, args, st);
    }
    if (split3)
    {
        if (epi == TC_GELU) return launch_tc<true, TC_GELU>(ma, mb, mblo, args, st);
        if (epi == TC_RESID) return launch_tc<true, TC_RESID>(ma, mb, mblo, args, st);
        return launch_tc<true, TC_STORE>(ma, mb, mblo, args, st);
    }
    if (epi == TC_GELU) return launch_tc<false, TC_GELU>(ma, mb, mblo, args, st);
    if (epi == TC_RESID) return launch_tc<false, TC_RESID>(ma, mb, mblo, args, st);
    return launch_tc<false, TC_STORE>(ma, mb, mblo, args, st);
}

// The prefill's QKV contraction with its scatter fused into the epilogue:
// qkv = A . B^T (B [3 dq x K]) written as q [M x dq] (row stride ldq) and as
// the rows t of the K and V caches of sequence b = row / P (layout of
// TcArgs::kc).  dq and hd must be multiples of 32, q and the caches 16-byte
// aligned.
int gemm_tc_qkv(float* q, int ldq, float* kc, float* vc, uint64_t seq_stride, int P, int hd, int ctx,
                const float* A, const float* B, int M, int dq, int K, bool split3, cudaStream_t st, const float* B_lo)
{
    if (M <= 0 || dq <= 0) return FML_OK;
    FML_REQUIRE(K > 0 && P > 0, "gemm_tc_qkv: K and P must be positive");
    FML_REQUIRE(dq % 32 == 0 && hd % 32 == 0 && dq % hd == 0 && ldq % 4 == 0,
                "gemm_tc_qkv: dq and hd must be multiples of 32 (dq %d, hd %d)", dq, hd);
    FML_REQUIRE(aligned16(A) && aligned16(B) && aligned16(q) && aligned16(kc) && aligned16(vc) && K % 4 == 0 &&
                    (!B_lo || aligned16(B_lo)) && seq_stride % 4 == 0,
                "gemm_tc_qkv: operands must be 16-byte aligned with row strides that are multiples of 4");
    CUtensorMap ma, mb, mblo;
    FML_RC(tc::make_map(&ma, A, M, K, K, tc::BM));
    FML_RC(tc::make_map(&mb, B, 3 * dq, K, K, tc::BN));
    const bool blo = split3 && B_lo;
    if (blo) FML_RC(tc::make_map(&mblo, B_lo, 3 * dq, K, K, tc::BN));
    else mblo = mb;
    TcArgs args{M, 3 * dq, K, q, ldq, nullptr, true, kc, vc, P, hd, dq, ctx, seq_stride};
    if (blo) return launch_tc<true, TC_QKV, true>(ma, mb, mblo, args, st);
    if (split3) return launch_tc<true, TC_QKV>(ma, mb, mblo, args, st);
    return launch_tc<false, TC_QKV>(ma, mb, mblo, args, st);
}

// Split-K partial products for few rows (the decode contractions at 33-64
// rows): part[s] = A[:, s Ks:(s+1) Ks] . B[:, s Ks:(s+1) Ks]^T for s <
// ksplit (Ks = K / ksplit, a multiple of 32), each [M x N] (row stride N)
// at part + s M N.  The caller sums the planes in order.  pdl: launch under
// programmatic dependent launch (the B tiles of the first stages load
// while the previous kernel finishes).
int gemm_tc_splitk(float* part, const float* A, const float* B, int M, int N, int K, int lda, int ldb, bool split3,
                   int ksplit, cudaStream_t st, const float* B_lo, bool pdl)
{
    if (M <= 0 || N <= 0) return FML_OK;
    FML_REQUIRE(K > 0 && ksplit >= 1 && K % (32 * ksplit) == 0,
                "gemm_tc_splitk: K %d must be a multiple of 32 x ksplit (%d)", K, ksplit);
    FML_REQUIRE(aligned16(A) && aligned16(B) && aligned16(part) && lda % 4 == 0 && ldb % 4 == 0 && N % 4 == 0 &&
                    (!B_lo || aligned16(B_lo)),
                "gemm_tc_splitk: operands must be 16-byte aligned with row strides that are multiples of 4");
    CUtensorMap ma, mb, mblo;
    FML_RC(tc::make_map(&ma, A, M, K, lda, tc::BM));
    FML_RC(tc::make_map(&mb, B, N, K, ldb, tc::BN));
    const bool blo = split3 && B_lo;
    if (blo) FML_RC(tc::make_map(&mblo, B_lo, N, K, ldb, tc::BN));
    else mblo = mb;
    TcArgs args{M, N, K, part, N, nullptr, true};
    args.ksplit = ksplit;
    args.pdl = pdl;
    if (blo) return launch_tc<true, TC_STORE, true>(ma, mb, mblo, args, st);
    if (split3) return launch_tc<true, TC_STORE>(ma, mb, mblo, args, st);
    return launch_tc<false, TC_STORE>(ma, mb, mblo, args, st);
}

// C = A . B on the tensor cores with B [K x N] row-major (row stride ldb):
// Mul<None> and MatMul_Strided<None>.  B is staged MN-major (no transpose);
// the same alignment rules as gemm_tc (ldb a multiple of 4, B 16-byte
// aligned).
int gemm_tc_nn(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, bool split3,
               cudaStream_t st)
{
    if (M <= 0 || N <= 0) return FML_OK;
    FML_REQUIRE(K > 0, "gemm_tc_nn: K must be positive");
    FML_REQUIRE(aligned16(A) && aligned16(B) && lda % 4 == 0 && ldb % 4 == 0,
                "gemm_tc_nn: operands must be 16-byte aligned with row strides that are multiples of 4");
    CUtensorMap ma, mb;
    FML_RC(tc::make_map(&ma, A, M, K, lda, tc::BM));
    // B [K x N]: n is the contiguous (inner) dimension, 32 x 32 boxes in the
    // 32-byte-atom swizzle of an MN-major tf32 operand
    FML_RC(tc::make_map(&mb, B, K, N, ldb, (int)tc::MN_BOX, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
    TcArgs args{M, N, K, C, ldc, nullptr, aligned16(C) && ldc % 4 == 0};
    if (split3) return launch_tc<true, TC_STORE, false, true>(ma, mb, mb, args, st);
    return launch_tc<false, TC_STORE, false, true>(ma, mb, mb, args, st);
}

// lo = x - hi(x) (hi = x with the low 13 mantissa bits cleared), for B_lo.
__global__ void tf32_lo_kernel(float* __restrict__ lo, const float* __restrict__ x, uint64_t n)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        lo[i] = x[i] - __uint_as_float(__float_as_uint(x[i]) & 0xFFFFE000u);
}

int tf32_lo(float* lo, const float* x, uint64_t n, cudaStream_t st)
{
    if (n == 0) return FML_OK;
    tf32_lo_kernel<<<grid_for(n, 256), 256, 0, st>>>(lo, x, n);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int gemm_tc_error_count(int* out)
{
    FML_CUDA_TRY(cudaMemcpyFromSymbol(out, g_gemm_timeouts, sizeof(int)));
    return FML_OK;
}

}  // namespace fml
