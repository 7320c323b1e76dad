// Skinny contractions (M <= 64 rows): Mul<None> (MatrixBase_Mul.h:591-615)
// with B [K x N] row-major, the Dense forward of a batch of at most 64 rows
// (the drop-in's decode-time Dense and BASELINE config 2's Dense sweep).
//
// The 128 x 128-tile GEMM leaves most of the GPU idle at such shapes (N/128
// CTAs), so this kernel splits K over grid.z instead: a CTA of 64 threads owns
// 256 consecutive columns (one float4 of B per thread per k: a warp reads
// 512 contiguous bytes of a B row, 8 rows in flight per thread) and MT rows,
// stages its rows of A in shared memory 128 k at a time (every lane reads the
// same A element: a broadcast), and accumulates in fp32 over its k range in
// ascending order.  With more than one split the partial results go to a
// stream-ordered scratch buffer and a second kernel sums them in split order,
// so the result is deterministic.  Every B element is read from DRAM once per
// row tile.  (A cluster-of-splits variant reducing through distributed shared
// memory was measured slower: at most 8-16 splits per column block leave too
// few bytes in flight for narrow outputs.)
#include <algorithm>

#include "fml_common.cuh"

namespace fml {

constexpr int SKN_THREADS = 64, SKN_COLS = SKN_THREADS * 4, SKN_K = 128;

template <int MT>
__global__ void __launch_bounds__(SKN_THREADS) skinny_nn_kernel(const float* __restrict__ A,
                                                                 const float* __restrict__ B, float* __restrict__ out,
                                                                 int M, int N, int K, int lda, int ldb, int ldo,
                                                                 int kper, uint64_t plane)
{
    __shared__ float xs[MT][SKN_K];
    const int tid = threadIdx.x;
    const int n = (blockIdx.x * SKN_THREADS + tid) * 4;
    const int m0 = blockIdx.y * MT;
    const int k0 = blockIdx.z * kper;
    const int k1 = min(K, k0 + kper);
    float4 acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int kc = k0; kc < k1; kc += SKN_K)
    {
        const int kn = min(SKN_K, k1 - kc);
        __syncthreads();
        for (int i = tid; i < MT * SKN_K; i += SKN_THREADS)
        {
            const int m = i / SKN_K, kk = i - m * SKN_K;
            xs[m][kk] = (m0 + m < M && kk < kn) ? A[(uint64_t)(m0 + m) * lda + kc + kk] : 0.f;
        }
        __syncthreads();
        if (n < N)
        {
            const float* bp = B + (uint64_t)kc * ldb + n;
#pragma unroll 8
            for (int kk = 0; kk < kn; ++kk)
            {
                const float4 w = __ldg(reinterpret_cast<const float4*>(bp + (uint64_t)kk * ldb));
#pragma unroll
                for (int m = 0; m < MT; ++m)
                {
                    const float x = xs[m][kk];
                    acc[m].x = fmaf(x, w.x, acc[m].x);
                    acc[m].y = fmaf(x, w.y, acc[m].y);
                    acc[m].z = fmaf(x, w.z, acc[m].z);
                    acc[m].w = fmaf(x, w.w, acc[m].w);
                }
            }
        }
    }
    if (n >= N) return;
    float* o = out + blockIdx.z * plane;
#pragma unroll
    for (int m = 0; m < MT; ++m)
        if (m0 + m < M) *reinterpret_cast<float4*>(o + (uint64_t)(m0 + m) * ldo + n) = acc[m];
}

// C[m, n] = sum over splits s (in order) of part[s][m][n]
__global__ void split_sum_kernel(float* __restrict__ C, const float* __restrict__ part, int M, int N, int ldc, int S)
{
    const uint64_t n4 = (uint64_t)N / 4, total = (uint64_t)M * n4;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint64_t m = i / n4, c = (i - m * n4) * 4;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int z = 0; z < S; ++z)
        {
            const float4 v = *reinterpret_cast<const float4*>(part + ((uint64_t)z * M + m) * N + c);
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        *reinterpret_cast<float4*>(C + m * ldc + c) = s;
    }
}

bool skinny_nn_ok(const float* C, const float* A, const float* B, int M, int N, int K, int ldb, int ldc)
{
    return M > 0 && M <= 64 && N > 0 && K > 0 && N % 4 == 0 && ldb % 4 == 0 && ldc % 4 == 0 &&
           (reinterpret_cast<uintptr_t>(B) & 15) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0;
}

template <int MT>
int launch_skinny(float* out, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldo,
                  int S, int kper, uint64_t plane, cudaStream_t st)
{
    dim3 grid((N + SKN_COLS - 1) / SKN_COLS, (M + MT - 1) / MT, S);
    skinny_nn_kernel<MT><<<grid, SKN_THREADS, 0, st>>>(A, B, out, M, N, K, lda, ldb, ldo, kper, plane);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int skinny_nn(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc,
              cudaStream_t st)
{
    static uint64_t pool_devices = 0;  // bit d: device d's pool is set up
    int dev = 0, sms = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    FML_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
    if (!(pool_devices & bit) || !bit)
    {
        // the split partials come from this device's stream-ordered pool;
        // keep freed blocks cached in this process (default threshold 0
        // would hand them back to the driver at every synchronisation)
        cudaMemPool_t pool;
        FML_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, dev));
        uint64_t keep = ~0ull;
        FML_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
        pool_devices |= bit;
    }
    const int MT = M <= 4 ? 4 : (M <= 8 ? 8 : 16);
    const int base = ((N + SKN_COLS - 1) / SKN_COLS) * ((M + MT - 1) / MT);
    // about eight CTAs per SM, at least 32 k per split, partials <= 64 MB
    int S = (8 * sms + base - 1) / base;
    S = std::min(S, (K + 31) / 32);
    S = std::min(S, std::max(1, (int)((64ull << 20) / (4ull * M * N))));
    S = std::max(S, 1);
    const int kper = (K + S - 1) / S;
    S = (K + kper - 1) / kper;
    float* part = nullptr;
    float* out = C;
    int ldo = ldc;
    if (S > 1)
    {
        FML_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&part), (size_t)S * M * N * sizeof(float), st));
        out = part;
        ldo = N;
    }
    const uint64_t plane = (uint64_t)M * N;
    int rc;
    if (MT == 4) rc = launch_skinny<4>(out, A, B, M, N, K, lda, ldb, ldo, S, kper, plane, st);
    else if (MT == 8) rc = launch_skinny<8>(out, A, B, M, N, K, lda, ldb, ldo, S, kper, plane, st);
    else rc = launch_skinny<16>(out, A, B, M, N, K, lda, ldb, ldo, S, kper, plane, st);
    if (rc == FML_OK && S > 1)
    {
        const uint64_t total = (uint64_t)M * N / 4;
        split_sum_kernel<<<(unsigned)std::min<uint64_t>((total + 255) / 256, 4096), 256, 0, st>>>(C, part, M, N, ldc,
                                                                                                  S);
        FML_LAUNCH_CHECK();
    }
    if (part) FML_CUDA_TRY(cudaFreeAsync(part, st));
    return rc;
}

}  // namespace fml
