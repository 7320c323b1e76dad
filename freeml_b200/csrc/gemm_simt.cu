// fp32 contractions on the CUDA cores: Mul<None|Right> (MatrixBase_Mul.h:
// 591-615) and MatMul_Strided<None|Right> (MatrixBase_Mul.h:617-722).
//
// C[M x N] = A[M x K] . op(B), op(B) = B[K x N] (trans_b = 0) or B[N x K]^T
// (trans_b = 1), arbitrary leading dimensions, batched over grid.z planes.
// Every output is one fp32 accumulator summed over k in ascending order,
// like the reference's MulBlock, so results differ from the CPU path only by
// the fused multiply-add rounding.
//
// Tiling: 128 x 128 output tile per 256-thread CTA, 8 x 8 outputs per
// thread, K staged through shared memory 16 at a time, double buffered.
// The tensor-core path (tcgen05, TF32x3 / TF32) lives in gemm_tcgen05.cu.
#include "fml_common.cuh"

namespace fml {

constexpr int GB_M = 128, GB_N = 128, GB_K = 16, GT_M = 8, GT_N = 8;

template <bool TRANS_B, bool TRANS_A = false>
__global__ void __launch_bounds__(256) gemm_f32_kernel(float* __restrict__ C, const float* __restrict__ A,
                                                       const float* __restrict__ B, int M, int N, int K, int lda,
                                                       int ldb, int ldc, uint64_t plane_a, uint64_t plane_b,
                                                       uint64_t plane_c)
{
    __shared__ __align__(16) float As[2][GB_K][GB_M + 4];
    __shared__ __align__(16) float Bs[2][GB_K][GB_N + 4];

    A += blockIdx.z * plane_a;
    B += blockIdx.z * plane_b;
    C += blockIdx.z * plane_c;

    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * GB_M, n0 = blockIdx.x * GB_N;
    const int tx = tid % 16, ty = tid / 16;  // 16 x 16 threads, 8x8 outputs each

    // Loader mapping: 256 threads load a 128 x 16 A tile (8 elements each) and
    // a 16 x 128 (or 128 x 16 for TRANS_B) B tile.
    float ra[8], rb[8];
    auto load_tiles = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const int e = tid + i * 256;           // 0..2047
            if (TRANS_A)
            {
                const int ak = e / GB_M, am = e % GB_M;  // A^T rows are k, contiguous in m
                const int gm = m0 + am, gk = k0 + ak;
                ra[i] = (gm < M && gk < K) ? A[(uint64_t)gk * lda + gm] : 0.0f;
            }
            else
            {
                const int am = e / GB_K, ak = e % GB_K;  // A tile row-major [128][16]
                const int gm = m0 + am, gk = k0 + ak;
                ra[i] = (gm < M && gk < K) ? A[(uint64_t)gm * lda + gk] : 0.0f;
            }
            if (TRANS_B)
            {
                const int bn = e / GB_K, bk = e % GB_K;  // B rows are n, contiguous in k
                const int gn = n0 + bn, gk2 = k0 + bk;
                rb[i] = (gn < N && gk2 < K) ? B[(uint64_t)gn * ldb + gk2] : 0.0f;
            }
            else
            {
                const int bk = e / GB_N, bn = e % GB_N;  // B rows are k, contiguous in n
                const int gn = n0 + bn, gk2 = k0 + bk;
                rb[i] = (gn < N && gk2 < K) ? B[(uint64_t)gk2 * ldb + gn] : 0.0f;
            }
        }
    };
    auto store_tiles = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const int e = tid + i * 256;
            if (TRANS_A) As[buf][e / GB_M][e % GB_M] = ra[i];
            else As[buf][e % GB_K][e / GB_K] = ra[i];
            if (TRANS_B) Bs[buf][e % GB_K][e / GB_K] = rb[i];
            else Bs[buf][e / GB_N][e % GB_N] = rb[i];
        }
    };

    float acc[GT_M][GT_N];
#pragma unroll
    for (int i = 0; i < GT_M; ++i)
#pragma unroll
        for (int j = 0; j < GT_N; ++j) acc[i][j] = 0.0f;

    const int ktiles = (K + GB_K - 1) / GB_K;
    load_tiles(0);
    store_tiles(0);
    __syncthreads();
    for (int kt = 0; kt < ktiles; ++kt)
    {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) load_tiles((kt + 1) * GB_K);
#pragma unroll
        for (int kk = 0; kk < GB_K; ++kk)
        {
            float a[GT_M], b[GT_N];
            // rows ty*4 + {0..3} and 64 + ty*4 + {0..3}: conflict-free float4 reads
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
            b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < GT_M; ++i)
#pragma unroll
                for (int j = 0; j < GT_N; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < ktiles) store_tiles(buf ^ 1);
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < GT_M; ++i)
    {
        const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < GT_N; ++j)
        {
            const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (gn < N) C[(uint64_t)gm * ldc + gn] = acc[i][j];
        }
    }
}

int gemm_f32(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, bool trans_b,
             int batch, uint64_t pa, uint64_t pb, uint64_t pc, cudaStream_t st)
{
    if (M <= 0 || N <= 0 || batch <= 0) return FML_OK;
    dim3 grid((N + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M, batch);
    FML_REQUIRE(grid.y <= 65535u && grid.z <= 65535u, "gemm: grid too large (M=%d batch=%d)", M, batch);
    if (K <= 0)
    {
        // empty contraction: zero output, like the reference's Clear + no terms
        for (int z = 0; z < batch; ++z)
            for (int m = 0; m < M; ++m)
                FML_CUDA_TRY(cudaMemsetAsync(C + z * pc + (uint64_t)m * ldc, 0, sizeof(float) * N, st));
        return FML_OK;
    }
    if (trans_b) gemm_f32_kernel<true><<<grid, 256, 0, st>>>(C, A, B, M, N, K, lda, ldb, ldc, pa, pb, pc);
    else gemm_f32_kernel<false><<<grid, 256, 0, st>>>(C, A, B, M, N, K, lda, ldb, ldc, pa, pb, pc);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

// C = A^T . B with A [K x M] (row stride lda), B [K x N] (row stride ldb):
// Mul<Left> / MatMul_Strided<Left> (MatrixBase_Mul.h:478-589, 617-722), one
// accumulator per output summed over k in ascending order.
int gemm_f32_ta(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, int batch,
                uint64_t pa, uint64_t pb, uint64_t pc, cudaStream_t st)
{
    if (M <= 0 || N <= 0 || batch <= 0) return FML_OK;
    dim3 grid((N + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M, batch);
    FML_REQUIRE(grid.y <= 65535u && grid.z <= 65535u, "gemm: grid too large (M=%d batch=%d)", M, batch);
    if (K <= 0)
    {
        for (int z = 0; z < batch; ++z)
            for (int m = 0; m < M; ++m)
                FML_CUDA_TRY(cudaMemsetAsync(C + z * pc + (uint64_t)m * ldc, 0, sizeof(float) * N, st));
        return FML_OK;
    }
    gemm_f32_kernel<false, true><<<grid, 256, 0, st>>>(C, A, B, M, N, K, lda, ldb, ldc, pa, pb, pc);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

// Batched / prefill contractions on the tensor cores by default: TF32x3 is
// fp32-level accuracy (fml_set_math_mode selects the fp32 CUDA-core kernels).
static int g_math_mode = FML_MATH_TF32X3;

int gemm_tc(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, bool split3,
            int epi, const float* R, cudaStream_t st, const float* B_lo = nullptr);
int gemm_tc_nn(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, bool split3,
               cudaStream_t st);
int gemv_nt(float* y, const float* x, const float* w, uint32_t M, uint32_t N, uint32_t K, cudaStream_t st);
bool skinny_nn_ok(const float* C, const float* A, const float* B, int M, int N, int K, int ldb, int ldc);
int skinny_nn(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc,
              cudaStream_t st);

int math_mode() { return g_math_mode; }

// Contraction with C = A . B^T: tensor cores (tcgen05) in the TF32 modes when
// the operands meet TMA's alignment rules, else the fp32 CUDA-core kernel.
int gemm_nt(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, int epi,
            const float* R, cudaStream_t st)
{
    const bool tc_ok = g_math_mode != FML_MATH_FP32 && K > 0 && aligned16(A) && aligned16(B) && lda % 4 == 0 &&
                       ldb % 4 == 0;
    if (tc_ok) return gemm_tc(C, A, B, M, N, K, lda, ldb, ldc, g_math_mode == FML_MATH_TF32X3, epi, R, st);
    FML_RC(gemm_f32(C, A, B, M, N, K, lda, ldb, ldc, true, 1, 0, 0, 0, st));
    if (epi == 0 || M <= 0 || N <= 0) return FML_OK;
    return set_error(FML_ERR_UNSUPPORTED, "gemm_nt: epilogue %d needs the tensor-core path", epi);
}

// C = A . B (B [K x N] row-major): tensor cores in the TF32 modes when the
// operands meet TMA's alignment rules, else the fp32 CUDA-core kernel.
int gemm_nn(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, cudaStream_t st)
{
    const bool tc_ok = g_math_mode != FML_MATH_FP32 && K > 0 && aligned16(A) && aligned16(B) && lda % 4 == 0 &&
                       ldb % 4 == 0;
    if (tc_ok) return gemm_tc_nn(C, A, B, M, N, K, lda, ldb, ldc, g_math_mode == FML_MATH_TF32X3, st);
    return gemm_f32(C, A, B, M, N, K, lda, ldb, ldc, false, 1, 0, 0, 0, st);
}

}  // namespace fml

using namespace fml;

extern "C" {

int fml_set_math_mode(int mode)
{
    FML_REQUIRE(mode == FML_MATH_FP32 || mode == FML_MATH_TF32X3 || mode == FML_MATH_TF32, "unknown math mode %d",
                mode);
    g_math_mode = mode;
    return FML_OK;
}

int fml_get_math_mode(void) { return g_math_mode; }

int fml_matmul(float* out, const float* a, const float* b, uint32_t M, uint32_t N, uint32_t K, int trans_b,
               fml_stream_t stream)
{
    FML_REQUIRE(M == 0 || N == 0 || (out && a && b), "fml_matmul: null pointer");
    FML_REQUIRE(M < (1u << 31) && N < (1u << 31) && K < (1u << 31), "fml_matmul: dimension too large");
    cudaStream_t st = as_stream(stream);
    // Few rows: the memory-bound fp32 CUDA-core kernels (every weight byte
    // read once, no tensor-core tile padding) -- up to 64 rows in the fp32
    // mode, up to 16 in the TF32 modes, where the tensor cores take over
    // (measured on B200, Mul<None> 4096 x 4096: 301 us on CUDA cores at 64
    // rows, CUDA-core FMA throughput bound)
    const uint32_t small = g_math_mode == FML_MATH_FP32 ? 64u : 16u;
    if (trans_b)
    {
        if (M >= 1 && M <= small && K > 0 && K % 4 == 0 && aligned16(a) && aligned16(b))
            return gemv_nt(out, a, b, M, N, K, st);
        return gemm_nt(out, a, b, (int)M, (int)N, (int)K, (int)K, (int)K, (int)N, 0, nullptr, st);
    }
    if (M <= small && skinny_nn_ok(out, a, b, (int)M, (int)N, (int)K, (int)N, (int)N))
        return skinny_nn(out, a, b, (int)M, (int)N, (int)K, (int)K, (int)N, (int)N, st);
    return gemm_nn(out, a, b, (int)M, (int)N, (int)K, (int)K, (int)N, (int)N, st);
}

int fml_matmul_strided(float* out, const float* a, const float* b, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                       uint32_t ldb, uint32_t ldc, int trans_b, uint32_t batch, uint64_t plane_a, uint64_t plane_b,
                       uint64_t plane_c, fml_stream_t stream)
{
    FML_REQUIRE(M == 0 || N == 0 || (out && a && b), "fml_matmul_strided: null pointer");
    FML_REQUIRE(batch >= 1, "fml_matmul_strided: batch must be >= 1");
    cudaStream_t st = as_stream(stream);
    // the per-head contractions of CausalSelfAttentionLayer.h:445-497 (scores
    // Q_h K_h^T and P V_h over row-strided head views): tensor cores in the
    // TF32 modes above 64 rows, one launch per plane
    if (g_math_mode != FML_MATH_FP32 && M > 64 && K > 0)
    {
        for (uint32_t z = 0; z < batch; ++z)
        {
            float* c = out + z * plane_c;
            const float* pa = a + z * plane_a;
            const float* pb = b + z * plane_b;
            if (trans_b) FML_RC(gemm_nt(c, pa, pb, (int)M, (int)N, (int)K, (int)lda, (int)ldb, (int)ldc, 0, nullptr, st));
            else FML_RC(gemm_nn(c, pa, pb, (int)M, (int)N, (int)K, (int)lda, (int)ldb, (int)ldc, st));
        }
        return FML_OK;
    }
    return gemm_f32(out, a, b, (int)M, (int)N, (int)K, (int)lda, (int)ldb, (int)ldc, trans_b != 0, (int)batch, plane_a,
                    plane_b, plane_c, st);
}

}  // extern "C"
