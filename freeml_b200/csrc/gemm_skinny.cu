// Skinny contractions (M <= 64 rows): Mul<None> (MatrixBase_Mul.h:591-615)
// with B [K x N] row-major, the Dense forward of a batch of at most 64 rows
// (the drop-in's small-batch Dense and BASELINE config 2's Dense sweep).
//
// One launch, no scratch memory.  The 128-column blocks of the output are
// too few to fill the GPU at these shapes, so K is split over S CTAs (S = 1,
// 2, 4, 8 or 16) that form one thread-block cluster per column block:
//   * each CTA streams its K slice in chunks of KC rows through two
//     shared-memory buffers: the chunk's B rows (128 columns, 512 bytes each)
//     and A rows (KC floats each) arrive by bulk asynchronous copies
//     (cp.async.bulk, completing on an mbarrier), the next chunk's copies in
//     flight while the current chunk is multiplied;
//   * warp w accumulates rows m = w, w + 4, ... (at most 16) of the block in
//     fp32, lane l four consecutive columns (one float4 of each B row);
//   * the CTA's partial [M x 128] is split by columns over the cluster: CTA
//     o owns columns [o 128/S, (o+1) 128/S); every CTA stores its part of
//     each owner's columns into the owner's receive buffer (distributed
//     shared memory, slot = its rank), one cluster barrier, and each owner
//     sums the S partials in rank order from its own shared memory
//     (deterministic) and writes C.
// Every B element is read from DRAM once.  Every mbarrier wait is bounded
// (an expiry is counted in the device error count and the CTA winds down);
// the cluster barriers are reached by every thread on every path.
#include <algorithm>

#include <cooperative_groups.h>

#include "tcgen05.cuh"

namespace fml {

__device__ int g_skinny_timeouts;

namespace {

constexpr int SK_THREADS = 128, SK_COLS = 128, SK_KC = 64;

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

struct SkinnyArgs
{
    const float* A;  // [M x K], row stride lda
    const float* B;  // [K x N], row stride ldb
    float* C;        // [M x N], row stride ldc
    int M, N, K, lda, ldb, ldc;
    int kper;        // K rows per split (a multiple of 4)
};

// MT: rows per warp (M <= 4 MT)
template <int MT>
__global__ void __launch_bounds__(SK_THREADS, 1) skinny_nn_kernel(SkinnyArgs a)
{
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int M = a.M;
    const uint32_t S = gridDim.y;      // K splits = CTAs of the cluster
    const uint32_t s = blockIdx.y;     // this CTA's split = its cluster rank
    const int n0 = blockIdx.x * SK_COLS;
    const int ncols = min(SK_COLS, a.N - n0);  // a multiple of 4
    const int k0 = (int)s * a.kper;
    const int kend = min(a.K, k0 + a.kper);
    const int nchunks = kend > k0 ? (kend - k0 + SK_KC - 1) / SK_KC : 0;

    // shared memory: 2 x {B chunk [KC x 128], A chunk [M x KC]}, receive
    // buffer [S][M][128/S], two mbarriers
    float* bbuf = reinterpret_cast<float*>(smem_raw);                 // 2 x KC x 128
    float* abuf = bbuf + 2 * SK_KC * SK_COLS;                         // 2 x M x KC
    float* recv = abuf + 2 * M * SK_KC;                               // M x 128
    uint64_t* full = reinterpret_cast<uint64_t*>(recv + M * SK_COLS);  // [2]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    cg::cluster_group cluster = cg::this_cluster();
    cg::cluster_group::arrival_token started = cluster.barrier_arrive();
    if (tid == 0)
    {
        tc::mbar_init(&full[0], 1);
        tc::mbar_init(&full[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // warp 0 issues chunk c into buffer b: its B rows (ncols floats each) and
    // A rows (the chunk's kc floats of each of the M rows)
    auto issue = [&](int c, int b) {
        const int kb = k0 + c * SK_KC, kc = min(SK_KC, kend - kb);
        if (lane == 0)
            tc::mbar_arrive_expect_tx(&full[b], (uint32_t)(kc * ncols + M * kc) * 4u);
        __syncwarp();
        for (int r = lane; r < kc; r += 32)
            bulk_g2s(bbuf + (b * SK_KC + r) * SK_COLS, a.B + (uint64_t)(kb + r) * a.ldb + n0, ncols * 4u, &full[b]);
        for (int m = lane; m < M; m += 32)
            bulk_g2s(abuf + (b * M + m) * SK_KC, a.A + (uint64_t)m * a.lda + kb, kc * 4u, &full[b]);
    };
    if (warp == 0)
    {
        if (nchunks > 0) issue(0, 0);
        if (nchunks > 1) issue(1, 1);
    }

    float4 acc[MT];
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int c4 = 4 * lane;  // this lane's columns within the block
    bool ok = true;
    for (int c = 0; c < nchunks; ++c)
    {
        const int b = c & 1;
        ok = tc::mbar_wait(&full[b], (uint32_t)(c >> 1) & 1u) && ok;
        const int kc = min(SK_KC, kend - (k0 + c * SK_KC));
        if (ok && c4 < ncols)
        {
            const float* bb = bbuf + b * SK_KC * SK_COLS + c4;
            const float* ab = abuf + b * M * SK_KC;
            for (int k = 0; k < kc; ++k)
            {
                const float4 w = *reinterpret_cast<const float4*>(bb + k * SK_COLS);
#pragma unroll
                for (int i = 0; i < MT; ++i)
                {
                    const int m = warp + 4 * i;
                    if (m < M)
                    {
                        const float x = ab[m * SK_KC + k];
                        acc[i].x = fmaf(x, w.x, acc[i].x);
                        acc[i].y = fmaf(x, w.y, acc[i].y);
                        acc[i].z = fmaf(x, w.z, acc[i].z);
                        acc[i].w = fmaf(x, w.w, acc[i].w);
                    }
                }
            }
        }
        // every thread is done with buffer b; `ok` made uniform so that a
        // warp never splits around the issue's warp-synchronous steps
        ok = __syncthreads_and(ok) != 0;
        if (warp == 0 && c + 2 < nchunks && ok) issue(c + 2, b);
    }
    ok = __syncthreads_and(ok) != 0;

    // columns [o W, (o+1) W) of the block belong to CTA o
    const int W = SK_COLS / (int)S;
    cluster.barrier_wait(std::move(started));  // every CTA of the cluster is running
    if (ok)
    {
        const int o = c4 / W, j = c4 % W;
        float* dst = cluster.map_shared_rank(recv, o);
#pragma unroll
        for (int i = 0; i < MT; ++i)
        {
            const int m = warp + 4 * i;
            if (m < M) *reinterpret_cast<float4*>(dst + ((int)s * M + m) * W + j) = acc[i];
        }
    }
    cluster.sync();  // every partial is in its owner's receive buffer
    if (ok)
    {
        const int q = W / 4;  // float4 columns per row of this CTA's share
        for (int t = tid; t < M * q; t += SK_THREADS)
        {
            const int m = t / q, j = 4 * (t % q), n = n0 + (int)s * W + j;
            if (n >= a.N) continue;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            for (uint32_t r = 0; r < S; ++r)
            {
                const float4 u = *reinterpret_cast<const float4*>(recv + (r * M + m) * W + j);
                v.x += u.x;
                v.y += u.y;
                v.z += u.z;
                v.w += u.w;
            }
            *reinterpret_cast<float4*>(a.C + (uint64_t)m * a.ldc + n) = v;
        }
    }
    if (!ok && tid == 0) atomicAdd(&g_skinny_timeouts, 1);
}

size_t skinny_smem(int M) { return (size_t)(2 * SK_KC * SK_COLS + 2 * M * SK_KC + M * SK_COLS) * 4 + 64; }

template <int MT>
int launch_skinny(const SkinnyArgs& a, int S, cudaStream_t st)
{
    auto kern = skinny_nn_kernel<MT>;
    static uint64_t attr_devices = 0;
    int dev = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
    if (!bit || !(attr_devices & bit))
    {
        FML_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)skinny_smem(64)));
        FML_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                          cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        attr_devices |= bit;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.N + SK_COLS - 1) / SK_COLS, S);
    cfg.blockDim = dim3(SK_THREADS);
    cfg.dynamicSmemBytes = skinny_smem(a.M);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "skinny_nn launch: %s", cudaGetErrorString(e));
    FML_LAUNCH_CHECK();
    return FML_OK;
}

}  // namespace

bool skinny_nn_ok(const float* C, const float* A, const float* B, int M, int N, int K, int ldb, int ldc)
{
    // bulk copies need 16-byte aligned rows: A, B, C and their row strides
    return M > 0 && M <= 64 && N > 0 && K > 0 && N % 4 == 0 && K % 4 == 0 && ldb % 4 == 0 && ldc % 4 == 0 &&
           aligned16(A) && aligned16(B) && aligned16(C);
}

int skinny_nn(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc,
              cudaStream_t st)
{
    FML_REQUIRE(lda % 4 == 0, "skinny_nn: lda must be a multiple of 4");
    int dev = 0, sms = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    FML_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int blocks = (N + SK_COLS - 1) / SK_COLS;
    // splits: about two CTAs per SM, at least one 64-row chunk each, a power
    // of two up to 16 (the owners' column shares stay float4 multiples)
    int S = 1;
    while (S < 16 && blocks * S * 2 <= 2 * sms && (K + 2 * S - 1) / (2 * S) >= SK_KC) S *= 2;
    int kper = (K + S - 1) / S;
    kper = (kper + 3) & ~3;  // chunk starts stay 16-byte aligned
    SkinnyArgs a{A, B, C, M, N, K, lda, ldb, ldc, kper};
    if (M <= 4) return launch_skinny<1>(a, S, st);
    if (M <= 8) return launch_skinny<2>(a, S, st);
    if (M <= 16) return launch_skinny<4>(a, S, st);
    if (M <= 32) return launch_skinny<8>(a, S, st);
    return launch_skinny<16>(a, S, st);
}

int skinny_error_count(int* out)
{
    FML_CUDA_TRY(cudaMemcpyFromSymbol(out, g_skinny_timeouts, sizeof(int)));
    return FML_OK;
}

}  // namespace fml
