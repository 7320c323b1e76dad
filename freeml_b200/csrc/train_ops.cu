// Training-side operators of the NanoLLM graph (the backward pass, the loss
// and the optimiser step that Model::Run(input, target) performs,
// ModelLibrary/Model.h:785-840), on the device.  Each follows the reference
// function named in its comment; reductions keep the reference's order
// where it is a plain sequential loop over rows or columns (LayerNorm's
// dGamma, the per-row softmax sums), and the embedding gradient scatters
// with atomic adds (row order is not kept: results agree to rounding).
#include <cmath>

#include "fml_common.cuh"

namespace fml {
namespace {

// GeluDerivtiveMat (MatrixBase_Functions.h:1003-1018):
// 0.5 (1 + erf(x / sqrt 2)) + x exp(-x^2 / 2) / sqrt(2 pi)
__global__ void gelu_derivative_kernel(float* __restrict__ out, const float* __restrict__ in, uint64_t n)
{
    const float sqrt2 = 1.41421356237309515f;     // sqrt(2)
    const float sqrt2pi = 2.50662827463100024f;   // sqrt(2 pi)
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const float x = in[i];
        const float erf_term = erff(x / sqrt2);
        const float exp_term = expf(-0.5f * x * x);
        out[i] = 0.5f * (1.0f + erf_term) + (x * exp_term) / sqrt2pi;
    }
}

// SoftmaxBackwards (MatrixBase_Functions.h:82-111): per row
// out = y (g - sum(g y)).  One warp per row; the dot product is summed by
// lanes in column order, then across lanes.
__global__ void softmax_backward_kernel(float* __restrict__ out, const float* __restrict__ y,
                                        const float* __restrict__ g, uint32_t rows, uint32_t cols)
{
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* yr = y + (uint64_t)warp * cols;
    const float* gr = g + (uint64_t)warp * cols;
    float dot = 0.0f;
    for (uint32_t c = lane; c < cols; c += 32) dot = fmaf(gr[c], yr[c], dot);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(FULL_MASK, dot, o);
    float* orow = out + (uint64_t)warp * cols;
    for (uint32_t c = lane; c < cols; c += 32) orow[c] = yr[c] * (gr[c] - dot);
}

// ScatterAddRows (MatrixBase_Functions.h:285-320): out row idx[r] += src row
// r, per z plane (out plane 0 when out has one plane).
__global__ void scatter_add_rows_kernel(float* __restrict__ out, const float* __restrict__ src,
                                        const float* __restrict__ idx, uint32_t src_rows, uint32_t width,
                                        uint32_t out_rows, uint32_t out_planes)
{
    const uint32_t r = blockIdx.x, z = blockIdx.y;
    const uint32_t dst = (uint32_t)idx[(uint64_t)z * src_rows + r];
    if (dst >= out_rows) return;  // the reference asserts dst < out_rows
    const float* s = src + ((uint64_t)z * src_rows + r) * width;
    float* o = out + ((uint64_t)(out_planes == 1 ? 0 : z) * out_rows + dst) * width;
    for (uint32_t x = threadIdx.x; x < width; x += blockDim.x) atomicAdd(o + x, s[x]);
}

// LayerNormBackwardsOp (MatrixBase_Functions.h:552-705), part 1: dGamma (and
// dBeta) as column sums over rows in row order, with xHat given or
// recomputed per row as the reference does.  One thread per column.
__global__ void layernorm_backward_params_kernel(float* __restrict__ dgamma, float* __restrict__ dbeta,
                                                 const float* __restrict__ dy, const float* __restrict__ xhat,
                                                 const float* __restrict__ in, const float* __restrict__ stats,
                                                 uint32_t rows, uint32_t cols)
{
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    float g = 0.0f, b = 0.0f;
    for (uint32_t r = 0; r < rows; ++r)
    {
        const float d = dy[(uint64_t)r * cols + c];
        const float xh = xhat ? xhat[(uint64_t)r * cols + c]
                              : (in[(uint64_t)r * cols + c] - stats[2 * r]) * stats[2 * r + 1];
        b += d;
        g += d * xh;
    }
    dgamma[c] = g;
    if (dbeta) dbeta[c] = b;
}

// Part 2: dX per row (one warp per row): two-pass mean / variance, then
// dVar, dMean and dX exactly as the reference composes them; also leaves
// (mean, invStd) per row for part 1.
__global__ void layernorm_backward_dx_kernel(float* __restrict__ dx, float* __restrict__ stats,
                                             const float* __restrict__ dy, const float* __restrict__ in,
                                             const float* __restrict__ gamma, uint32_t rows, uint32_t cols, float eps)
{
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* x = in + (uint64_t)warp * cols;
    const float* d = dy + (uint64_t)warp * cols;
    const float invCols = 1.0f / (float)cols;
    float s = 0.0f;
    for (uint32_t c = lane; c < cols; c += 32) s += x[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL_MASK, s, o);
    const float mean = s * invCols;
    float v = 0.0f;
    for (uint32_t c = lane; c < cols; c += 32)
    {
        const float diff = x[c] - mean;
        v = fmaf(diff, diff, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
    const float invStd = 1.0f / sqrtf(v * invCols + eps);
    const float invStd3 = invStd * invStd * invStd;
    float dVar = 0.0f, dMean = 0.0f, sumDiff = 0.0f;
    for (uint32_t c = lane; c < cols; c += 32)
    {
        const float diff = x[c] - mean;
        const float dxh = d[c] * gamma[c];
        dVar += dxh * diff * -0.5f * invStd3;
        dMean += dxh * -invStd;
        sumDiff += diff;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        dVar += __shfl_xor_sync(FULL_MASK, dVar, o);
        dMean += __shfl_xor_sync(FULL_MASK, dMean, o);
        sumDiff += __shfl_xor_sync(FULL_MASK, sumDiff, o);
    }
    dMean += dVar * -2.0f * sumDiff * invCols;
    float* o = dx + (uint64_t)warp * cols;
    for (uint32_t c = lane; c < cols; c += 32)
    {
        const float diff = x[c] - mean;
        const float dxh = d[c] * gamma[c];
        o[c] = dxh * invStd + dVar * 2.0f * diff * invCols + dMean * invCols;
    }
    if (lane == 0 && stats)
    {
        stats[2 * warp] = mean;
        stats[2 * warp + 1] = invStd;
    }
}

// AdamWUpdate (MatrixBase_Functions.h:1498-1545), elementwise.
__global__ void adamw_kernel(float* __restrict__ param, const float* __restrict__ grad, float* __restrict__ mt,
                             float* __restrict__ vt, uint64_t n, float lr, float beta1, float beta2, float beta1_pow,
                             float beta2_pow, float eps, float wd)
{
    const float invB1 = 1.0f - beta1, invB2 = 1.0f - beta2;
    const float invB1Pow = 1.0f - beta1_pow, invB2Pow = 1.0f - beta2_pow;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const float g = grad[i];
        const float m = beta1 * mt[i] + invB1 * g;
        const float v = beta2 * vt[i] + invB2 * g * g;
        mt[i] = m;
        vt[i] = v;
        const float mh = m / invB1Pow, vh = v / invB2Pow;
        const float p = param[i];
        const float update = lr * mh / (sqrtf(vh) + eps);
        const float decay = lr * wd * p;
        param[i] = p + update - decay;
    }
}

// CategoricalCrossEntropyWithLogits (LossLibrary/
// CategoricalCrossEntropyWithLogits.h:29-217), one CTA per (step, batch)
// row.  ids = 1: the target holds one token id per row (-1 = ignored), the
// gradient is (onehot - softmax) / valid and the row loss logsumexp -
// logit[id]; ids = 0: the target is a dense [vocab] row per step, gradient
// (t - softmax), loss at the first t > 0.5.  `row_loss` gets each row's
// loss (0 for ignored rows), summed afterwards in row order.
__global__ void xent_kernel(float* __restrict__ grad, float* __restrict__ row_loss, const float* __restrict__ target,
                            const float* __restrict__ logits, uint32_t vocab, uint32_t steps, uint32_t target_planes,
                            int ids, uint32_t n_rows)
{
    __shared__ float red[32];
    __shared__ float s_bcast;
    const uint32_t row = blockIdx.x, t = row % steps, z = row / steps;
    const uint32_t tz = target_planes == 1 ? 0u : z;
    const float* lg = logits + (uint64_t)row * vocab;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    auto block_reduce = [&](float v, bool is_max) -> float {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
        {
            const float w = __shfl_xor_sync(FULL_MASK, v, o);
            v = is_max ? fmaxf(v, w) : v + w;
        }
        __syncthreads();
        if (lane == 0) red[warp] = v;
        __syncthreads();
        if (tid == 0)
        {
            float r = red[0];
            for (int i = 1; i < nw; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
            s_bcast = r;
        }
        __syncthreads();
        return s_bcast;
    };
    int idx = -1;
    float inv_valid = 1.0f;
    if (ids)
    {
        idx = (int)target[(uint64_t)tz * steps + t];
        // valid rows over the whole target (the reference counts them first)
        float cnt = 0.0f;
        for (uint32_t i = tid; i < n_rows; i += blockDim.x)
        {
            const uint32_t ti = i % steps, zi = i / steps;
            cnt += (int)target[(uint64_t)(target_planes == 1 ? 0u : zi) * steps + ti] != -1 ? 1.0f : 0.0f;
        }
        const float valid = block_reduce(cnt, false);
        inv_valid = valid > 0.0f ? 1.0f / valid : 0.0f;
        if (idx == -1)
        {
            for (uint32_t i = tid; i < vocab; i += blockDim.x) grad[(uint64_t)row * vocab + i] = 0.0f;
            if (tid == 0 && row_loss) row_loss[row] = 0.0f;
            return;
        }
    }
    float mx = -INFINITY;
    for (uint32_t i = tid; i < vocab; i += blockDim.x) mx = fmaxf(mx, lg[i]);
    mx = block_reduce(mx, true);
    float se = 0.0f;
    for (uint32_t i = tid; i < vocab; i += blockDim.x) se += expf(lg[i] - mx);
    se = block_reduce(se, false);
    const float* trow = ids ? nullptr : target + ((uint64_t)tz * steps + t) * vocab;
    for (uint32_t i = tid; i < vocab; i += blockDim.x)
    {
        const float p = expf(lg[i] - mx) / se;
        const float ti = ids ? ((uint32_t)idx == i ? 1.0f : 0.0f) : trow[i];
        grad[(uint64_t)row * vocab + i] = ids ? (ti - p) * inv_valid : (ti - p);
    }
    if (row_loss && tid == 0)
    {
        const float lse = mx + logf(se);
        if (ids) row_loss[row] = lse - lg[idx];
        else
        {
            float l = 0.0f;
            for (uint32_t i = 0; i < vocab; ++i)
                if (trow[i] > 0.5f) { l = lse - lg[i]; break; }
            row_loss[row] = l;
        }
    }
}

// Row losses summed in row order (one thread): the reference's sequential
// float total, divided by the valid count for the id form.
__global__ void xent_total_kernel(float* __restrict__ out, const float* __restrict__ row_loss,
                                  const float* __restrict__ target, uint32_t steps, uint32_t target_planes,
                                  uint32_t n_rows, int ids)
{
    float total = 0.0f;
    uint32_t valid = 0;
    for (uint32_t r = 0; r < n_rows; ++r)
    {
        if (ids)
        {
            const uint32_t t = r % steps, z = r / steps;
            if ((int)target[(uint64_t)(target_planes == 1 ? 0u : z) * steps + t] == -1) continue;
            ++valid;
        }
        total += row_loss[r];
    }
    *out = ids ? (valid ? total / (float)valid : 0.0f) : total;
}

// MergeQKV (MatrixBase_Functions.h:369-431): per-head gradients [heads][tokens]
// [head_dim] of q, k, v packed back into rows [tokens][3 * heads * head_dim].
__global__ void merge_qkv_kernel(float* __restrict__ packed, const float* __restrict__ q, const float* __restrict__ k,
                                 const float* __restrict__ v, uint32_t head_dim, uint32_t tokens, uint32_t heads)
{
    const uint32_t dC = head_dim * heads, cols = 3 * dC;
    const uint64_t n = (uint64_t)tokens * cols;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t row = (uint32_t)(i / cols), c = (uint32_t)(i % cols);
        const uint32_t part = c / dC, hc = c % dC, head = hc / head_dim, e = hc % head_dim;
        const float* src = part == 0 ? q : (part == 1 ? k : v);
        packed[i] = src[((uint64_t)head * tokens + row) * head_dim + e];
    }
}

}  // namespace

int gemm_f32_ta(float* C, const float* A, const float* B, int M, int N, int K, int lda, int ldb, int ldc, int batch,
                uint64_t pa, uint64_t pb, uint64_t pc, cudaStream_t st);

}  // namespace fml

using namespace fml;

extern "C" {

int fml_gelu_derivative(float* out, const float* in, uint64_t n, fml_stream_t stream)
{
    if (n == 0) return FML_OK;
    FML_REQUIRE(out && in, "fml_gelu_derivative: null pointer");
    gelu_derivative_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(out, in, n);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_softmax_backward(float* out, const float* y, const float* g, uint32_t rows, uint32_t cols,
                         fml_stream_t stream)
{
    if (rows == 0 || cols == 0) return FML_OK;
    FML_REQUIRE(out && y && g, "fml_softmax_backward: null pointer");
    const unsigned block = 256;
    softmax_backward_kernel<<<(unsigned)(((uint64_t)rows * 32 + block - 1) / block), block, 0, as_stream(stream)>>>(
        out, y, g, rows, cols);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_scatter_add_rows(float* out, const float* src, const float* indices, uint32_t src_rows, uint32_t width,
                         uint32_t out_rows, uint32_t planes, uint32_t out_planes, fml_stream_t stream)
{
    if (src_rows == 0 || width == 0 || planes == 0) return FML_OK;
    FML_REQUIRE(out && src && indices, "fml_scatter_add_rows: null pointer");
    FML_REQUIRE(out_planes == 1 || out_planes == planes, "fml_scatter_add_rows: %u output planes for %u", out_planes,
                planes);
    FML_REQUIRE(planes <= 65535u, "fml_scatter_add_rows: too many planes");
    scatter_add_rows_kernel<<<dim3(src_rows, planes), 128, 0, as_stream(stream)>>>(out, src, indices, src_rows, width,
                                                                                    out_rows, out_planes);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_layernorm_backward(float* dx, const float* dy, const float* in, const float* gamma, float* dgamma,
                           float* dbeta, const float* xhat, uint32_t rows, uint32_t cols, float eps, void* workspace,
                           fml_stream_t stream)
{
    if (rows == 0 || cols == 0) return FML_OK;
    FML_REQUIRE(dx && dy && in && gamma && dgamma, "fml_layernorm_backward: null pointer");
    FML_REQUIRE(xhat || workspace, "fml_layernorm_backward: workspace of 2 floats per row needed without xHat");
    cudaStream_t st = as_stream(stream);
    float* stats = static_cast<float*>(workspace);
    const unsigned block = 256;
    layernorm_backward_dx_kernel<<<(unsigned)(((uint64_t)rows * 32 + block - 1) / block), block, 0, st>>>(
        dx, stats, dy, in, gamma, rows, cols, eps);
    FML_LAUNCH_CHECK();
    layernorm_backward_params_kernel<<<(cols + 127) / 128, 128, 0, st>>>(dgamma, dbeta, dy, xhat, in, stats, rows,
                                                                         cols);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_adamw_update(float* param, const float* grad, float* mt, float* vt, uint64_t n, float lr, float beta1,
                     float beta2, float beta1_pow_t, float beta2_pow_t, float eps, float weight_decay,
                     fml_stream_t stream)
{
    if (n == 0) return FML_OK;
    FML_REQUIRE(param && grad && mt && vt, "fml_adamw_update: null pointer");
    adamw_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(param, grad, mt, vt, n, lr, beta1, beta2,
                                                                  beta1_pow_t, beta2_pow_t, eps, weight_decay);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_xent_with_logits(float* grad, float* loss_out, const float* target, const float* logits, uint32_t vocab,
                         uint32_t steps, uint32_t planes, uint32_t target_planes, int target_ids, void* workspace,
                         fml_stream_t stream)
{
    const uint64_t rows = (uint64_t)steps * planes;
    if (rows == 0 || vocab == 0) return FML_OK;
    FML_REQUIRE(grad && target && logits, "fml_xent_with_logits: null pointer");
    FML_REQUIRE(!loss_out || workspace, "fml_xent_with_logits: a loss needs a workspace of rows + 1 floats");
    FML_REQUIRE(rows <= 0x7fffffffu, "fml_xent_with_logits: too many rows");
    cudaStream_t st = as_stream(stream);
    float* row_loss = static_cast<float*>(workspace);
    xent_kernel<<<(unsigned)rows, 256, 0, st>>>(grad, loss_out ? row_loss : nullptr, target, logits, vocab, steps,
                                                target_planes, target_ids, (uint32_t)rows);
    FML_LAUNCH_CHECK();
    if (loss_out)
    {
        xent_total_kernel<<<1, 1, 0, st>>>(row_loss + rows, row_loss, target, steps, target_planes, (uint32_t)rows,
                                           target_ids);
        FML_LAUNCH_CHECK();
        FML_CUDA_TRY(cudaMemcpyAsync(loss_out, row_loss + rows, sizeof(float), cudaMemcpyDeviceToHost, st));
        FML_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return FML_OK;
}

int fml_merge_qkv(float* packed, const float* q, const float* k, const float* v, uint32_t head_dim, uint32_t tokens,
                  uint32_t heads, fml_stream_t stream)
{
    const uint64_t n = (uint64_t)tokens * 3 * head_dim * heads;
    if (n == 0) return FML_OK;
    FML_REQUIRE(packed && q && k && v, "fml_merge_qkv: null pointer");
    merge_qkv_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(packed, q, k, v, head_dim, tokens, heads);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_matmul_left(float* out, const float* a, const float* b, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                    uint32_t ldb, uint32_t ldc, uint32_t batch, uint64_t plane_a, uint64_t plane_b, uint64_t plane_c,
                    fml_stream_t stream)
{
    FML_REQUIRE(M == 0 || N == 0 || (out && a && b), "fml_matmul_left: null pointer");
    FML_REQUIRE(batch >= 1, "fml_matmul_left: batch must be >= 1");
    return gemm_f32_ta(out, a, b, (int)M, (int)N, (int)K, (int)lda, (int)ldb, (int)ldc, (int)batch, plane_a, plane_b,
                       plane_c, as_stream(stream));
}

}  // extern "C"
