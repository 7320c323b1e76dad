// Causal decode attention over a KV cache: the attention core of
// CausalSelfAttentionLayer::Forward (CausalSelfAttentionLayer.h:424-499) for
// one query row at a time, used by the decode engine (decode and prefill
// rows) and exposed as the fml_attention_decode operator.
#include <cmath>
#include <mutex>

#include "attention.cuh"

namespace fml {

// Causal attention for one query row over the cached keys 0..t
// (CausalSelfAttentionLayer.h:424-499: Q_h K_h^T, * 1/sqrt(hd) + causal
// mask, Softmax, P V_h), as one pass with an online softmax.
// grid = (H, rows, S); 4 warps per CTA take 32-key tiles in turn.  Per tile a
// lane holds HD/32 dims of q; the 32 partial dot products are summed by a
// transpose-reduce, so lane j ends with key j's score; p_j is then
// broadcast for the P.V update.  With S > 1 each CTA writes (m, l, acc) and
// the last CTA of the (row, head) to finish merges the S partials.
template <int HD>
__global__ void __launch_bounds__(128) attention_kernel(AttnArgs a)
{
    constexpr int DPL = HD / 32;
    __shared__ float sm_m[4], sm_l[4];
    __shared__ float sm_acc[4][HD];
    __shared__ int sm_last;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t h = blockIdx.x, r = a.row0 + blockIdx.y, s = blockIdx.z;
    uint32_t b, len;
    if (a.lens) { b = r; len = a.lens[r]; }
    else if (a.pos) { b = r; len = a.pos[r] + 1; }
    else { b = r / a.P; len = r % a.P + 1; }
    const uint32_t begin = s * a.chunk;
    const uint32_t end = min(len, begin + a.chunk);

    const float* K = a.kc + (uint64_t)b * a.seq_stride + (uint64_t)h * a.C * HD;
    const float* Vv = a.vc + (uint64_t)b * a.seq_stride + (uint64_t)h * a.C * HD;

    float qv[DPL];
    const float* qp = a.q + (uint64_t)r * a.ldq + h * HD + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) qv[i] = qp[i];

    float m_run = -INFINITY, l_run = 0.0f;
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.0f;

    for (uint32_t j0 = begin + warp * 32u; j0 < end; j0 += 128u)
    {
        float part[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
        {
            float sdot = 0.0f;
            if (j0 + jj < end)
            {
                const float* kr = K + (uint64_t)(j0 + jj) * HD + lane * DPL;
                if constexpr (DPL == 4)
                {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr);
                    sdot = qv[0] * k4.x + qv[1] * k4.y + qv[2] * k4.z + qv[3] * k4.w;
                }
                else if constexpr (DPL == 2)
                {
                    const float2 k2 = *reinterpret_cast<const float2*>(kr);
                    sdot = qv[0] * k2.x + qv[1] * k2.y;
                }
                else
                {
                    sdot = qv[0] * kr[0];
                }
            }
            part[jj] = sdot;
        }
        warp_transpose_reduce<32>(part, lane);
        // lane now holds the full dot product of key j0 + lane
        const bool valid = j0 + lane < end;
        const float sc = valid ? part[0] * a.scale : -INFINITY;
        const float tile_max = warp_max(sc);
        const float m_new = fmaxf(m_run, tile_max);
        const float p = valid ? expf(sc - m_new) : 0.0f;
        const float corr = expf(m_run - m_new);
        l_run = l_run * corr + warp_sum(p);
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] *= corr;
        const uint32_t nvalid = min(32u, end - j0);
        for (uint32_t jj = 0; jj < nvalid; ++jj)
        {
            const float pj = __shfl_sync(FULL_MASK, p, jj);
            const float* vr = Vv + (uint64_t)(j0 + jj) * HD + lane * DPL;
            if constexpr (DPL == 4)
            {
                const float4 v4 = *reinterpret_cast<const float4*>(vr);
                acc[0] = fmaf(pj, v4.x, acc[0]);
                acc[1] = fmaf(pj, v4.y, acc[1]);
                acc[2] = fmaf(pj, v4.z, acc[2]);
                acc[3] = fmaf(pj, v4.w, acc[3]);
            }
            else if constexpr (DPL == 2)
            {
                const float2 v2 = *reinterpret_cast<const float2*>(vr);
                acc[0] = fmaf(pj, v2.x, acc[0]);
                acc[1] = fmaf(pj, v2.y, acc[1]);
            }
            else
            {
                acc[0] = fmaf(pj, vr[0], acc[0]);
            }
        }
        m_run = m_new;
    }

    if (lane == 0) { sm_m[warp] = m_run; sm_l[warp] = l_run; }
#pragma unroll
    for (int i = 0; i < DPL; ++i) sm_acc[warp][lane * DPL + i] = acc[i];
    __syncthreads();

    // merge the 4 warps
    const float M = fmaxf(fmaxf(sm_m[0], sm_m[1]), fmaxf(sm_m[2], sm_m[3]));
    float w4[4];
    float L = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        w4[i] = (M == -INFINITY) ? 0.0f : expf(sm_m[i] - M);
        L += sm_l[i] * w4[i];
    }
    const int e = threadIdx.x;
    if (a.S == 1)
    {
        if (e < HD)
        {
            const float A = sm_acc[0][e] * w4[0] + sm_acc[1][e] * w4[1] + sm_acc[2][e] * w4[2] + sm_acc[3][e] * w4[3];
            a.out[(uint64_t)r * a.ldo + h * HD + e] = L > 0.0f ? A / L : 0.0f;
        }
        return;
    }

    float* mypart = a.part + (((uint64_t)b * a.H + h) * a.S + s) * (HD + 2);
    if (e < HD)
        mypart[e] = sm_acc[0][e] * w4[0] + sm_acc[1][e] * w4[1] + sm_acc[2][e] * w4[2] + sm_acc[3][e] * w4[3];
    if (e == 0) { mypart[HD] = M; mypart[HD + 1] = L; }
    __threadfence();
    __syncthreads();
    if (e == 0)
    {
        const uint32_t prev = atomicAdd(a.counters + (uint64_t)b * a.H + h, 1u);
        sm_last = (prev == a.S - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!sm_last) return;
    __threadfence();
    const float* parts = a.part + ((uint64_t)b * a.H + h) * a.S * (HD + 2);
    float Mg = -INFINITY;
    for (uint32_t i = 0; i < a.S; ++i) Mg = fmaxf(Mg, __ldcg(parts + i * (HD + 2) + HD));
    float Lg = 0.0f, Ag = 0.0f;
    for (uint32_t i = 0; i < a.S; ++i)
    {
        const float mi = __ldcg(parts + i * (HD + 2) + HD);
        const float wi = (mi == -INFINITY) ? 0.0f : expf(mi - Mg);
        Lg += __ldcg(parts + i * (HD + 2) + HD + 1) * wi;
        if (e < HD) Ag += __ldcg(parts + i * (HD + 2) + e) * wi;
    }
    if (e < HD) a.out[(uint64_t)r * a.ldo + h * HD + e] = Lg > 0.0f ? Ag / Lg : 0.0f;
    if (e == 0) a.counters[(uint64_t)b * a.H + h] = 0u;
}


int launch_attention_kernel(const AttnArgs& a, uint32_t hd, dim3 grid, cudaStream_t st)
{
    switch (hd)
    {
    case 32: attention_kernel<32><<<grid, 128, 0, st>>>(a); break;
    case 64: attention_kernel<64><<<grid, 128, 0, st>>>(a); break;
    case 128: attention_kernel<128><<<grid, 128, 0, st>>>(a); break;
    default: return set_error(FML_ERR_UNSUPPORTED, "head dim %u not supported (32/64/128)", hd);
    }
    FML_LAUNCH_CHECK();
    return FML_OK;
}

// Split count for `pairs` (row, head) pairs over keys up to `ctx`: about two
// waves of 148 SMs, each split a multiple of 32 keys.
void attention_splits(uint64_t pairs, uint64_t ctx, uint32_t* S_out, uint32_t* chunk_out)
{
    uint64_t S = (2 * 148 + pairs - 1) / pairs;
    const uint64_t max_s = (ctx + 31) / 32;
    if (S > max_s) S = max_s;
    if (S < 1) S = 1;
    uint64_t chunk = (ctx + S - 1) / S;
    chunk = (chunk + 31) / 32 * 32;
    if (chunk < 32) chunk = 32;
    S = (ctx + chunk - 1) / chunk;
    *S_out = (uint32_t)S;
    *chunk_out = (uint32_t)chunk;
}

uint64_t attention_workspace_bytes(uint32_t B, uint32_t H, uint32_t hd, uint32_t S)
{
    // split partials (floats), then the per-(row, head) counters, 256-aligned
    const uint64_t part = (uint64_t)B * H * S * (hd + 2) * sizeof(float);
    return ((part + 255) / 256) * 256 + (uint64_t)B * H * sizeof(uint32_t);
}

}  // namespace fml

using namespace fml;

extern "C" {

size_t fml_attention_workspace_bytes(uint32_t batch, uint32_t heads, uint32_t head_dim, uint32_t context)
{
    if (!batch || !heads || !head_dim || !context) return 0;
    uint32_t S, chunk;
    attention_splits((uint64_t)batch * heads, context, &S, &chunk);
    return (size_t)attention_workspace_bytes(batch, heads, head_dim, S);
}

int fml_attention_decode(float* out, const float* q, const float* kcache, const float* vcache, const uint32_t* lens,
                         uint32_t batch, uint32_t heads, uint32_t head_dim, uint32_t context, float scale,
                         void* workspace, size_t workspace_bytes, fml_stream_t stream)
{
    if (batch == 0) return FML_OK;
    FML_REQUIRE(out && q && kcache && vcache && lens, "fml_attention_decode: null pointer");
    FML_REQUIRE(heads >= 1 && context >= 1, "fml_attention_decode: zero heads or context");
    FML_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128,
                "fml_attention_decode: head_dim %u (need 32, 64 or 128)", head_dim);
    FML_REQUIRE(batch <= 65535u, "fml_attention_decode: batch %u > 65535", batch);
    uint32_t S, chunk;
    attention_splits((uint64_t)batch * heads, context, &S, &chunk);
    const uint64_t need = attention_workspace_bytes(batch, heads, head_dim, S);
    FML_REQUIRE(workspace && workspace_bytes >= need,
                "fml_attention_decode: workspace of %llu bytes needed (fml_attention_workspace_bytes)",
                (unsigned long long)need);
    cudaStream_t st = as_stream(stream);
    const uint64_t part_bytes = need - (uint64_t)batch * heads * sizeof(uint32_t);
    uint32_t* counters = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + part_bytes);
    FML_CUDA_TRY(cudaMemsetAsync(counters, 0, (size_t)batch * heads * sizeof(uint32_t), st));
    AttnArgs a{};
    a.q = q; a.ldq = heads * head_dim; a.row0 = 0;
    a.kc = kcache; a.vc = vcache; a.seq_stride = (uint64_t)heads * context * head_dim;
    a.H = heads; a.C = context;
    a.out = out; a.ldo = heads * head_dim;
    a.pos = nullptr; a.lens = lens; a.P = 1;
    a.S = S; a.chunk = chunk; a.scale = scale;
    a.part = static_cast<float*>(workspace);
    a.counters = counters;
    return launch_attention_kernel(a, head_dim, dim3(heads, batch, S), st);
}

// ---------------------------------------------------------------------------
// Allocation-free attention (fml_attention_decode_noalloc).
//
// For callers that may not allocate device memory: a host runtime that hands
// every byte of the GPU to its own pool and forbids libraries from calling
// cudaMalloc, or code running inside such a pool's out-of-memory handling,
// where a new allocation could recurse or fail.  The split partials and the
// merge counters live in the fixed array below, part of this library's own
// device image: every GPU that loads the library holds these
// FML_NOALLOC_SCRATCH_BYTES until the process exits.
//
// Host code may not hand `g_attention_scratch` to a kernel: on the host that
// name is only a stand-in, not a device address.  The device address is
// fetched with cudaGetSymbolAddress once per device (with that device
// current) and cached; the first call on a device does this set-up, so make
// that first call outside any stream capture.
// ---------------------------------------------------------------------------

static __device__ __align__(256) unsigned char g_attention_scratch[FML_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

int noalloc_scratch(void** out)
{
    int dev = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(FML_ERR_UNSUPPORTED, "fml_attention_decode_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev])
    {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess || !p)
            return set_error(FML_ERR_CUDA, "fml_attention_decode_noalloc: cudaGetSymbolAddress failed: %s",
                             cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return FML_OK;
}
}  // namespace

int fml_attention_decode_noalloc(float* out, const float* q, const float* kcache, const float* vcache,
                                 const uint32_t* lens, uint32_t batch, uint32_t heads, uint32_t head_dim,
                                 uint32_t context, float scale, fml_stream_t stream)
{
    if (batch == 0) return FML_OK;
    FML_REQUIRE(out && q && kcache && vcache && lens, "fml_attention_decode_noalloc: null pointer");
    FML_REQUIRE(heads >= 1 && context >= 1, "fml_attention_decode_noalloc: zero heads or context");
    FML_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128,
                "fml_attention_decode_noalloc: head_dim %u (need 32, 64 or 128)", head_dim);
    FML_REQUIRE(batch <= 65535u, "fml_attention_decode_noalloc: batch %u > 65535", batch);
    uint32_t S, chunk;
    attention_splits((uint64_t)batch * heads, context, &S, &chunk);
    const uint64_t need = attention_workspace_bytes(batch, heads, head_dim, S);
    if (need > FML_NOALLOC_SCRATCH_BYTES)
        return set_error(FML_ERR_UNSUPPORTED,
                         "fml_attention_decode_noalloc: batch %u x heads %u x head_dim %u needs %llu bytes of "
                         "scratch, above the fixed %u-byte array; use fml_attention_decode with a workspace",
                         batch, heads, head_dim, (unsigned long long)need, (unsigned)FML_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    FML_RC(noalloc_scratch(&scratch));
    cudaStream_t st = as_stream(stream);
    // The array keeps whatever the previous call left; the merge counters must
    // start at zero, so clear them (a memset, not an allocation).
    const uint64_t part_bytes = need - (uint64_t)batch * heads * sizeof(uint32_t);
    uint32_t* counters = reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + part_bytes);
    FML_CUDA_TRY(cudaMemsetAsync(counters, 0, (size_t)batch * heads * sizeof(uint32_t), st));
    AttnArgs a{};
    a.q = q; a.ldq = heads * head_dim; a.row0 = 0;
    a.kc = kcache; a.vc = vcache; a.seq_stride = (uint64_t)heads * context * head_dim;
    a.H = heads; a.C = context;
    a.out = out; a.ldo = heads * head_dim;
    a.pos = nullptr; a.lens = lens; a.P = 1;
    a.S = S; a.chunk = chunk; a.scale = scale;
    a.part = static_cast<float*>(scratch);
    a.counters = counters;
    return launch_attention_kernel(a, head_dim, dim3(heads, batch, S), st);
}

}  // extern "C"
