// Operator entry points: the generic FreeML operators the NanoLLM forward
// reaches, as sm_100a kernels.  Each kernel cites the reference template it
// replaces; the MatrixCUDA<float> overloads call these through the C ABI.
#include <cmath>
#include <cstring>
#include <mutex>

#include "fml_common.cuh"

namespace fml {

static thread_local char g_err[512] = "";

int set_error(int status, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return status;
}

std::atomic<uint64_t>& launch_counter()
{
    static std::atomic<uint64_t> c{0};
    return c;
}

// ---- elementwise ------------------------------------------------------------

// Add / PerElementMul / BroadcastAdd (MatrixBase_Functions.h:471, :848, :717).
enum class EwOp { Add, Mul, BroadcastAdd };

template <EwOp OP>
__global__ void ew_binary_kernel(float* __restrict__ out, const float* a, const float* b, uint64_t n, uint32_t cols)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const float x = a[i];
        if constexpr (OP == EwOp::Add) out[i] = x + b[i];
        else if constexpr (OP == EwOp::Mul) out[i] = x * b[i];
        else out[i] = x + b[i % cols];
    }
}

// Vector form for 16-byte aligned, multiple-of-4 operands.
template <EwOp OP>
__global__ void ew_binary_kernel4(float4* __restrict__ out, const float4* a, const float4* b, uint64_t n4)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const float4 x = a[i], y = b[i];
        float4 r;
        if constexpr (OP == EwOp::Add) r = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
        else r = make_float4(x.x * y.x, x.y * y.y, x.z * y.z, x.w * y.w);
        out[i] = r;
    }
}

template <EwOp OP>
static int launch_binary(float* out, const float* a, const float* b, uint64_t n, uint32_t cols, cudaStream_t st)
{
    if (n == 0) return FML_OK;
    const unsigned block = 256;
    if (OP != EwOp::BroadcastAdd && (n % 4) == 0 && aligned16(out) && aligned16(a) && aligned16(b))
    {
        ew_binary_kernel4<OP><<<grid_for(n / 4, block), block, 0, st>>>((float4*)out, (const float4*)a,
                                                                        (const float4*)b, n / 4);
    }
    else
    {
        ew_binary_kernel<OP><<<grid_for(n, block), block, 0, st>>>(out, a, b, n, cols);
    }
    FML_LAUNCH_CHECK();
    return FML_OK;
}

// Scale (MatrixBase_Functions.h:1021-1039) and ScaleAdd (:1044-1070).  The
// reference build fuses `in * scale + add` into one fma.
__global__ void scale_kernel(float* out, const float* in, float s, const float* s_dev, uint64_t n)
{
    const float sc = s_dev ? s_dev[0] : s;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = in[i] * sc;
}

__global__ void scale_add_kernel(float* out, const float* in, const float* s_dev, const float* add, uint64_t n)
{
    const float sc = s_dev[0];
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = fmaf(in[i], sc, add[i]);
}

// Fill / Clear (MatrixBase_Functions.h:1073-1096).
__global__ void fill_kernel(float* out, float v, const float* v_dev, uint64_t n)
{
    const float val = v_dev ? v_dev[0] : v;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = val;
}

// GeluMat (MatrixBase_Functions.h:989-1000).
__global__ void gelu_kernel(float* out, const float* in, uint64_t n)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = gelu_exact(in[i]);
}

// GatherRows (MatrixBase_Functions.h:203-242): one CTA row-slab per output row.
__global__ void gather_rows_kernel(float* __restrict__ out, const float* __restrict__ src, const float* __restrict__ idx,
                                   uint32_t rows, uint32_t width, uint32_t src_rows)
{
    for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x)
    {
        const float fid = idx[r];
        const bool ok = fid >= 0.0f && fid < (float)src_rows;
        const uint32_t id = ok ? (uint32_t)fid : 0u;
        const float* s = src + (uint64_t)id * width;
        float* o = out + (uint64_t)r * width;
        for (uint32_t c = threadIdx.x; c < width; c += blockDim.x) o[c] = ok ? s[c] : 0.0f;
    }
}

// SplitQKV (MatrixBase_Functions.h:330-367).
__global__ void split_qkv_kernel(float* q, float* k, float* v, const float* packed, uint32_t rows, uint32_t d)
{
    const uint64_t n = (uint64_t)rows * 3u * d;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint64_t r = i / (3u * d);
        const uint32_t c = (uint32_t)(i - r * 3u * d);
        const float val = packed[i];
        if (c < d) q[r * d + c] = val;
        else if (c < 2 * d) k[r * d + c - d] = val;
        else v[r * d + c - 2 * d] = val;
    }
}

// LayerNormOp (MatrixBase_Functions.h:482-549): one warp per row.  Mean and
// biased variance are two separate passes like the reference (the variance
// is a sum of squared deviations from the finished mean, not E[x^2]-mean^2);
// invStd = 1/sqrt(var/cols + eps) with the same fused var*invCols+eps.
__global__ void layernorm_kernel(float* __restrict__ out, const float* __restrict__ in, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, float* __restrict__ xhat, uint32_t rows, uint32_t cols,
                                 uint64_t in_stride, uint64_t out_stride, float eps)
{
    const int lane = threadIdx.x & 31;
    const uint32_t warps = blockDim.x >> 5;
    const float invCols = 1.0f / (float)cols;
    for (uint32_t r = blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += gridDim.x * warps)
    {
        const float* x = in + r * in_stride;
        float s = 0.0f;
        for (uint32_t c = lane; c < cols; c += 32) s += x[c];
        const float mean = warp_sum(s) * invCols;
        float v = 0.0f;
        for (uint32_t c = lane; c < cols; c += 32)
        {
            const float df = x[c] - mean;
            v = fmaf(df, df, v);
        }
        v = warp_sum(v);
        const float invStd = 1.0f / sqrtf(fmaf(v, invCols, eps));
        float* y = out + r * out_stride;
        for (uint32_t c = lane; c < cols; c += 32)
        {
            const float nrm = (x[c] - mean) * invStd;
            if (xhat) xhat[r * (uint64_t)cols + c] = nrm;
            y[c] = fmaf(nrm, gamma[c], beta ? beta[c] : 0.0f);
        }
    }
}

// Softmax (MatrixBase_Functions.h:50-80): one warp per row, max, exp-sum,
// then division by the sum.
__global__ void softmax_kernel(float* __restrict__ out, const float* in, uint32_t rows, uint32_t cols)
{
    const int lane = threadIdx.x & 31;
    const uint32_t warps = blockDim.x >> 5;
    for (uint32_t r = blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += gridDim.x * warps)
    {
        const float* x = in + (uint64_t)r * cols;
        float* y = out + (uint64_t)r * cols;
        float m = -INFINITY;
        for (uint32_t c = lane; c < cols; c += 32) m = fmaxf(m, x[c]);
        m = warp_max(m);
        float s = 0.0f;
        for (uint32_t c = lane; c < cols; c += 32)
        {
            const float e = expf(x[c] - m);
            y[c] = e;
            s += e;
        }
        s = warp_sum(s);
        __syncwarp();
        for (uint32_t c = lane; c < cols; c += 32) y[c] = y[c] / s;
    }
}

// The same LayerNormOp for rows of up to 2048 columns in multiples of 128:
// one warp per row holds the row in registers (NV float4 per lane, requested
// together), so the row is read from memory once and the two statistics
// passes and the output pass run on registers.
template <int NV>
__global__ void layernorm_rows_kernel(float* __restrict__ out, const float* __restrict__ in,
                                      const float* __restrict__ gamma, const float* __restrict__ beta,
                                      float* __restrict__ xhat, uint32_t rows, uint32_t cols, uint64_t in_stride,
                                      uint64_t out_stride, float eps)
{
    const int lane = threadIdx.x & 31;
    const uint32_t warps = blockDim.x >> 5;
    const uint32_t c4 = cols / 4;  // float4 per row: 32 * nv, nv <= NV
    const float invCols = 1.0f / (float)cols;
    for (uint32_t r = blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += gridDim.x * warps)
    {
        const float4* x = reinterpret_cast<const float4*>(in + r * in_stride);
        float4 v[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if ((uint32_t)(lane + 32 * i) < c4) v[i] = x[lane + 32 * i];
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if ((uint32_t)(lane + 32 * i) < c4) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        const float mean = warp_sum(s) * invCols;
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if ((uint32_t)(lane + 32 * i) < c4)
            {
                const float d0 = v[i].x - mean, d1 = v[i].y - mean, d2 = v[i].z - mean, d3 = v[i].w - mean;
                q = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, q))));
            }
        const float invStd = 1.0f / sqrtf(fmaf(warp_sum(q), invCols, eps));
        float4* y = reinterpret_cast<float4*>(out + r * out_stride);
        const float4* g4 = reinterpret_cast<const float4*>(gamma);
        const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
        for (int i = 0; i < NV; ++i)
        {
            const uint32_t c = lane + 32 * i;
            if (c >= c4) continue;
            const float4 g = g4[c];
            const float4 b = beta ? b4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 n;
            n.x = (v[i].x - mean) * invStd; n.y = (v[i].y - mean) * invStd;
            n.z = (v[i].z - mean) * invStd; n.w = (v[i].w - mean) * invStd;
            if (xhat) reinterpret_cast<float4*>(xhat + r * (uint64_t)cols)[c] = n;
            y[c] = make_float4(fmaf(n.x, g.x, b.x), fmaf(n.y, g.y, b.y), fmaf(n.z, g.z, b.z), fmaf(n.w, g.w, b.w));
        }
    }
}

int launch_layernorm(float* out, const float* in, const float* gamma, const float* beta, float* xhat, uint32_t rows,
                     uint32_t cols, uint64_t in_stride, uint64_t out_stride, float eps, cudaStream_t st)
{
    if (rows == 0) return FML_OK;
    const unsigned block = 128;
    if (cols % 128 == 0 && cols <= 2048 && in_stride % 4 == 0 && out_stride % 4 == 0 && aligned16(in) &&
        aligned16(out) && aligned16(gamma) && (!beta || aligned16(beta)) && (!xhat || aligned16(xhat)))
    {
        const unsigned grid = (unsigned)((rows + 3) / 4);
        const unsigned g = grid < 65535u * 8 ? grid : 65535u * 8;
        if (cols <= 512)
            layernorm_rows_kernel<4><<<g, block, 0, st>>>(out, in, gamma, beta, xhat, rows, cols, in_stride, out_stride,
                                                           eps);
        else
            layernorm_rows_kernel<16><<<g, block, 0, st>>>(out, in, gamma, beta, xhat, rows, cols, in_stride,
                                                            out_stride, eps);
        FML_LAUNCH_CHECK();
        return FML_OK;
    }
    const unsigned grid = (unsigned)((rows + 3) / 4);
    layernorm_kernel<<<grid < 65535u * 8 ? grid : 65535u * 8, block, 0, st>>>(out, in, gamma, beta, xhat, rows, cols,
                                                                               in_stride, out_stride, eps);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

}  // namespace fml

using namespace fml;

extern "C" {

const char* fml_last_error(void) { return fml::g_err; }
const char* fml_version(void) { return "freeml_b200 0.1 (sm_100a)"; }
uint64_t fml_kernel_launch_count(void) { return launch_counter().load(); }

int fml_device_check(int* sm_count, int* cc_major, int* cc_minor)
{
    int dev = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    cudaDeviceProp p;
    FML_CUDA_TRY(cudaGetDeviceProperties(&p, dev));
    if (sm_count) *sm_count = p.multiProcessorCount;
    if (cc_major) *cc_major = p.major;
    if (cc_minor) *cc_minor = p.minor;
    if (p.major != 10) return set_error(FML_ERR_UNSUPPORTED, "built for sm_100a, device is sm_%d%d", p.major, p.minor);
    return FML_OK;
}

int fml_device_alloc(void** ptr, size_t bytes)
{
    FML_REQUIRE(ptr, "fml_device_alloc: null argument");
    *ptr = nullptr;
    const cudaError_t e = cudaMalloc(ptr, bytes ? bytes : 16);
    if (e != cudaSuccess)
    {
        cudaGetLastError();
        return set_error(FML_ERR_NOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    return FML_OK;
}

int fml_device_free(void* ptr)
{
    if (ptr) FML_CUDA_TRY(cudaFree(ptr));
    return FML_OK;
}

int fml_memcpy_to_device(void* dst, const void* src, size_t bytes)
{
    FML_REQUIRE(bytes == 0 || (dst && src), "fml_memcpy_to_device: null pointer");
    if (bytes) FML_CUDA_TRY(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return FML_OK;
}

int fml_memcpy_to_host(void* dst, const void* src, size_t bytes)
{
    FML_REQUIRE(bytes == 0 || (dst && src), "fml_memcpy_to_host: null pointer");
    FML_CUDA_TRY(cudaDeviceSynchronize());
    if (bytes) FML_CUDA_TRY(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return FML_OK;
}

int fml_synchronize(void)
{
    FML_CUDA_TRY(cudaDeviceSynchronize());
    return FML_OK;
}

int fml_gather_rows(float* out, const float* src, const float* idx, uint32_t rows, uint32_t width, uint32_t src_rows,
                    fml_stream_t stream)
{
    if (rows == 0 || width == 0) return FML_OK;
    FML_REQUIRE(out && src && idx, "fml_gather_rows: null pointer");
    gather_rows_kernel<<<rows < 65535u ? rows : 65535u, 128, 0, as_stream(stream)>>>(out, src, idx, rows, width, src_rows);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_add(float* out, const float* a, const float* b, uint64_t n, fml_stream_t stream)
{
    FML_REQUIRE(n == 0 || (out && a && b), "fml_add: null pointer");
    return launch_binary<EwOp::Add>(out, a, b, n, 1, as_stream(stream));
}

int fml_broadcast_add(float* out, const float* a, const float* row, uint64_t n, uint32_t cols, fml_stream_t stream)
{
    FML_REQUIRE(n == 0 || (out && a && row && cols), "fml_broadcast_add: bad arguments");
    return launch_binary<EwOp::BroadcastAdd>(out, a, row, n, cols, as_stream(stream));
}

int fml_mul_elementwise(float* out, const float* a, const float* b, uint64_t n, fml_stream_t stream)
{
    FML_REQUIRE(n == 0 || (out && a && b), "fml_mul_elementwise: null pointer");
    return launch_binary<EwOp::Mul>(out, a, b, n, 1, as_stream(stream));
}

int fml_scale(float* out, const float* in, float scale, const float* scale_dev, uint64_t n, fml_stream_t stream)
{
    if (n == 0) return FML_OK;
    FML_REQUIRE(out && in, "fml_scale: null pointer");
    scale_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(out, in, scale, scale_dev, n);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_scale_add(float* out, const float* in, const float* scale_dev, const float* add, uint64_t n, fml_stream_t stream)
{
    if (n == 0) return FML_OK;
    FML_REQUIRE(out && in && scale_dev && add, "fml_scale_add: null pointer");
    scale_add_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(out, in, scale_dev, add, n);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_fill(float* out, float value, const float* value_dev, uint64_t n, fml_stream_t stream)
{
    if (n == 0) return FML_OK;
    FML_REQUIRE(out, "fml_fill: null pointer");
    fill_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(out, value, value_dev, n);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_copy(float* out, const float* in, uint64_t n, fml_stream_t stream)
{
    if (n == 0 || out == in) return FML_OK;
    FML_REQUIRE(out && in, "fml_copy: null pointer");
    FML_CUDA_TRY(cudaMemcpyAsync(out, in, n * sizeof(float), cudaMemcpyDeviceToDevice, as_stream(stream)));
    return FML_OK;
}

int fml_layernorm(float* out, const float* in, const float* gamma, const float* beta, float* xhat, uint32_t rows,
                  uint32_t cols, float eps, fml_stream_t stream)
{
    FML_REQUIRE(rows == 0 || (out && in && gamma && cols), "fml_layernorm: bad arguments");
    return launch_layernorm(out, in, gamma, beta, xhat, rows, cols, cols, cols, eps, as_stream(stream));
}

int fml_gelu(float* out, const float* in, uint64_t n, fml_stream_t stream)
{
    if (n == 0) return FML_OK;
    FML_REQUIRE(out && in, "fml_gelu: null pointer");
    gelu_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(out, in, n);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_softmax(float* out, const float* in, uint32_t rows, uint32_t cols, fml_stream_t stream)
{
    if (rows == 0) return FML_OK;
    FML_REQUIRE(out && in && cols, "fml_softmax: bad arguments");
    const unsigned grid = (rows + 3) / 4;
    softmax_kernel<<<grid < 65535u * 8 ? grid : 65535u * 8, 128, 0, as_stream(stream)>>>(out, in, rows, cols);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int fml_split_qkv(float* q, float* k, float* v, const float* packed, uint32_t rows, uint32_t d, fml_stream_t stream)
{
    if (rows == 0 || d == 0) return FML_OK;
    FML_REQUIRE(q && k && v && packed, "fml_split_qkv: null pointer");
    split_qkv_kernel<<<grid_for((uint64_t)rows * 3 * d, 256), 256, 0, as_stream(stream)>>>(q, k, v, packed, rows, d);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

}  // extern "C"
