// Causal decode attention over a KV cache: the attention core of
// CausalSelfAttentionLayer::Forward (CausalSelfAttentionLayer.h:424-499) for
// one query row at a time, used by the decode engine (decode and prefill
// rows) and exposed as the fml_attention_decode operator.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include <cooperative_groups.h>
#include <cuda.h>

#include "attention.cuh"

namespace fml {

#ifdef FML_TIMELINE
// debug builds: this unit's timeline ring (fml_debug_timeline binds it)
int timeline_bind_attention(TimelineRec* p, uint32_t cap) { return timeline_bind_unit(p, cap); }
#endif

// Causal attention for one query row over the cached keys 0..len-1
// (CausalSelfAttentionLayer.h:424-499: Q_h K_h^T, * 1/sqrt(hd) + causal
// mask, Softmax, P V_h) as one pass with an online softmax.
//
// CTA = NW warps (4 or 16) on one (row, head, key split); grid = (heads,
// rows, splits).
// Inside a warp, G = HD/4 lanes form a group that owns one key at a time,
// each lane holding 4 dims (one float4 of the K row and of the V row), so a
// score needs log2(G) shuffles and a warp covers 32/G keys per step.  Every
// group keeps its own running max / sum / accumulator (no per-key
// broadcast); U steps of K and V loads are issued before any is used, and a
// thread stays under 64 registers so that 32 warps (8 CTAs of 4, or 2 of 16)
// fit on an SM and the loads of many warps overlap.  Groups, warps and then
// splits are merged at the end; with S > 1 the splits of a (row, head) merge
// through a cluster's shared memory, or each CTA writes (m, l, acc) and the
// last CTA of the (row, head) to finish merges the partials.
struct AttnUnit
{
    uint32_t r, b, begin, end, nsplit;
    uint32_t newest;  // key written by the previous kernel (decode), else none
};

__device__ __forceinline__ AttnUnit attention_unit(const AttnArgs& a, uint32_t r, uint32_t s)
{
    AttnUnit t;
    t.r = r;
    uint32_t len;
    t.newest = 0xffffffffu;
    if (a.lens) { t.b = r; len = a.lens[r]; }
    else if (a.pos) { t.b = r; len = a.pos[r] + 1; t.newest = len - 1; }
    else { t.b = r / a.P; len = r % a.P + 1; }
    len = min(len, a.C);  // never past the (sequence, head) block
    // keys per split: fixed, or an even share of this row's keys
    const uint32_t chunk = a.chunk ? a.chunk : max(8u, ((len + a.S - 1) / a.S + 7u) & ~7u);
    t.begin = min(s * chunk, len);
    t.end = min(len, t.begin + chunk);
    t.nsplit = (len + chunk - 1) / chunk;  // non-empty splits of this row
    return t;
}

__device__ __forceinline__ float dot4(const float4& a, const float4& b)
{
    return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, a.w * b.w)));
}

// merge (m2, l2, acc2) into (m, l, acc)
__device__ __forceinline__ void softmax_merge(float& m, float& l, float4& acc, float m2, float l2, const float4& acc2)
{
    const float mn = fmaxf(m, m2);
    const float w1 = (m == -INFINITY) ? 0.0f : expf(m - mn);
    const float w2 = (m2 == -INFINITY) ? 0.0f : expf(m2 - mn);
    l = l * w1 + l2 * w2;
    acc.x = acc.x * w1 + acc2.x * w2;
    acc.y = acc.y * w1 + acc2.y * w2;
    acc.z = acc.z * w1 + acc2.z * w2;
    acc.w = acc.w * w1 + acc2.w * w2;
    m = mn;
}

// CL: the S splits of a (row, head) run as one thread-block cluster and are
// merged through distributed shared memory (cluster rank 0 reads every
// split's (m, l, acc) after a cluster barrier) instead of through global
// partials, a fence and a completion counter.
template <int HD, int NW, bool CL>
__global__ void __launch_bounds__(32 * NW, 32 / NW) attention_kernel(AttnArgs a)
{
    FML_TIMELINE_SCOPE(20);
    const StampAtExit stamp_at_exit(a.stamp);
    constexpr int G = HD / 4;       // lanes per key
    constexpr int KPW = 32 / G;     // keys per warp step
    constexpr int U = 4;            // steps whose loads are in flight together
    __shared__ float sm_m[NW], sm_l[NW];
    __shared__ __align__(16) float sm_acc[NW][HD];
    __shared__ int sm_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane / G, lig = lane % G;
    const uint32_t h = blockIdx.x, r = a.row0 + blockIdx.y, s = blockIdx.z;

    // CL: first arrival on the cluster barrier; its wait, before the first
    // write into another CTA's shared memory, guarantees every CTA of the
    // cluster is running by then
    [[maybe_unused]] cooperative_groups::cluster_group::arrival_token cl_started;
    if constexpr (CL) cl_started = cooperative_groups::this_cluster().barrier_arrive();

    griddep_launch_dependents();

    // Positions were set by the previous step's last kernel, which finished
    // before this step's first (non-overlapped) kernel began, and every cached
    // row below the newest was written by earlier steps: this CTA's first
    // batch of K/V rows is requested before waiting for the previous kernel.
    // Only the newest row (key len - 1) comes from that kernel; it is
    // re-read after the wait if the first batch holds it.
    const AttnUnit cu = attention_unit(a, r, s);
    const float* K = a.kc + (uint64_t)cu.b * a.seq_stride + (uint64_t)h * a.C * HD + lig * 4;
    const float* V = a.vc + (uint64_t)cu.b * a.seq_stride + (uint64_t)h * a.C * HD + lig * 4;
    constexpr uint32_t STEP = NW * KPW;  // keys per CTA step (NW warps)
    const uint32_t last = cu.end > 0 ? cu.end - 1 : 0;
    const uint32_t kw0 = cu.begin + warp * KPW;
    const uint32_t newest = cu.newest;
    // prefill rows (no positions, no lengths) read keys the previous kernel
    // wrote: no early loads there
    const bool early = a.pos != nullptr || a.lens != nullptr;
    if (!early) griddep_wait();
    float4 kk[U], vv[U];
    if (kw0 < cu.end)
    {
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const uint32_t j = min(kw0 + grp + u * STEP, last);
            kk[u] = *reinterpret_cast<const float4*>(K + (uint64_t)j * HD);
            vv[u] = *reinterpret_cast<const float4*>(V + (uint64_t)j * HD);
        }
    }
    if (early) griddep_wait();  // q and the newest K/V rows come from the previous kernel
    FML_TIMELINE_MARK(1);
    if (kw0 < cu.end)
    {
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const uint32_t j = min(kw0 + grp + u * STEP, last);
            if (j == newest)
            {
                kk[u] = __ldcg(reinterpret_cast<const float4*>(K + (uint64_t)j * HD));
                vv[u] = __ldcg(reinterpret_cast<const float4*>(V + (uint64_t)j * HD));
            }
        }
    }

    float4 q = *reinterpret_cast<const float4*>(a.q + (uint64_t)r * a.ldq + h * HD + lig * 4);
    q.x *= a.scale; q.y *= a.scale; q.z *= a.scale; q.w *= a.scale;

    float m = -INFINITY, l = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // the trip count depends on the warp only (never on the lane group): the
    // loop body has full-warp shuffles, so every lane must run every step
    for (uint32_t kw = kw0; kw < cu.end; kw += U * STEP)
    {
        const uint32_t kb = kw + grp;  // this group's first key of the step
        if (kw != kw0)
        {
#pragma unroll
            for (int u = 0; u < U; ++u)
            {
                const uint32_t j = min(kb + u * STEP, last);  // clamped in range, masked below
                kk[u] = *reinterpret_cast<const float4*>(K + (uint64_t)j * HD);
                vv[u] = *reinterpret_cast<const float4*>(V + (uint64_t)j * HD);
            }
        }
        float sc[U];
        float smax = -INFINITY;
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            float d = dot4(q, kk[u]);
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(FULL_MASK, d, o);
            sc[u] = (kb + u * STEP < cu.end) ? d : -INFINITY;
            smax = fmaxf(smax, sc[u]);
        }
        if (smax > m)  // rescale only when the running max grows
        {
            const float corr = (m == -INFINITY) ? 0.0f : expf(m - smax);
            l *= corr;
            acc.x *= corr; acc.y *= corr; acc.z *= corr; acc.w *= corr;
            m = smax;
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const float p = (sc[u] == -INFINITY) ? 0.0f : expf(sc[u] - m);
            l += p;
            acc.x = fmaf(p, vv[u].x, acc.x);
            acc.y = fmaf(p, vv[u].y, acc.y);
            acc.z = fmaf(p, vv[u].z, acc.z);
            acc.w = fmaf(p, vv[u].w, acc.w);
        }
    }

    FML_TIMELINE_MARK(2);
    // merge the KPW groups of the warp (xor across groups)
#pragma unroll
    for (int o = G; o < 32; o <<= 1)
    {
        const float m2 = __shfl_xor_sync(FULL_MASK, m, o);
        const float l2 = __shfl_xor_sync(FULL_MASK, l, o);
        float4 a2;
        a2.x = __shfl_xor_sync(FULL_MASK, acc.x, o);
        a2.y = __shfl_xor_sync(FULL_MASK, acc.y, o);
        a2.z = __shfl_xor_sync(FULL_MASK, acc.z, o);
        a2.w = __shfl_xor_sync(FULL_MASK, acc.w, o);
        softmax_merge(m, l, acc, m2, l2, a2);
    }
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
    if (grp == 0) *reinterpret_cast<float4*>(&sm_acc[warp][lig * 4]) = acc;
    __syncthreads();

    // merge the NW warps in warp order: thread e < HD owns output dim e
    const int e = tid;
    float M = sm_m[0];
#pragma unroll
    for (int i = 1; i < NW; ++i) M = fmaxf(M, sm_m[i]);
    float L = 0.0f, A = 0.0f;
#pragma unroll
    for (int i = 0; i < NW; ++i)
    {
        const float wi = (sm_m[i] == -INFINITY) ? 0.0f : expf(sm_m[i] - M);
        L += sm_l[i] * wi;
        if (e < HD) A += sm_acc[i][e] * wi;
    }
    if constexpr (CL)
    {
        // every split pushes (acc, m, l) into cluster rank 0's shared memory;
        // after the cluster barrier rank 0 merges them from its own shared
        // memory -- the same arithmetic as the global merge below, over every
        // split in order (an empty split has m = -inf and weight 0)
        __shared__ __align__(16) float cl_acc[8][HD];
        __shared__ float cl_ml[8][2];
        cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();
        cluster.barrier_wait(std::move(cl_started));
        if (e < HD) *cluster.map_shared_rank(&cl_acc[s][e], 0) = A;
        if (e == 0)
        {
            *cluster.map_shared_rank(&cl_ml[s][0], 0) = M;
            *cluster.map_shared_rank(&cl_ml[s][1], 0) = L;
        }
        cluster.sync();
        if (s == 0)
        {
            const uint32_t ns = gridDim.z;
            float Mg = -INFINITY;
            for (uint32_t i = 0; i < ns; ++i) Mg = fmaxf(Mg, cl_ml[i][0]);
            float Lg = 0.0f, Ag = 0.0f;
            for (uint32_t i = 0; i < ns; ++i)
            {
                const float mi = cl_ml[i][0];
                const float wi = mi == -INFINITY ? 0.0f : expf(mi - Mg);
                Lg += cl_ml[i][1] * wi;
                if (e < HD) Ag += cl_acc[i][e] * wi;
            }
            if (e < HD) a.out[(uint64_t)r * a.ldo + h * HD + e] = Lg > 0.0f ? Ag / Lg : 0.0f;
        }
        return;
    }
    if (cu.nsplit <= 1)
    {
        if (e < HD && s == 0) a.out[(uint64_t)r * a.ldo + h * HD + e] = L > 0.0f ? A / L : 0.0f;
        return;
    }
    if (cu.begin >= cu.end) return;  // an empty split beyond this row's keys
    float* mypart = a.part + (((uint64_t)cu.b * a.H + h) * a.S + s) * (HD + 2);
    if (e < HD) mypart[e] = A;
    if (e == 0) { mypart[HD] = M; mypart[HD + 1] = L; }
    __threadfence();
    __syncthreads();
    if (e == 0)
    {
        const uint32_t prev = atomicAdd(a.counters + (uint64_t)cu.b * a.H + h, 1u);
        sm_last = (prev == cu.nsplit - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!sm_last) return;
    __threadfence();
    const float* parts = a.part + ((uint64_t)cu.b * a.H + h) * a.S * (HD + 2);
    float Mg = -INFINITY;
    for (uint32_t i = 0; i < cu.nsplit; ++i) Mg = fmaxf(Mg, __ldcg(parts + i * (HD + 2) + HD));
    float Lg = 0.0f, Ag = 0.0f;
    for (uint32_t i = 0; i < cu.nsplit; ++i)
    {
        const float wi = expf(__ldcg(parts + i * (HD + 2) + HD) - Mg);
        Lg += __ldcg(parts + i * (HD + 2) + HD + 1) * wi;
        if (e < HD) Ag += __ldcg(parts + i * (HD + 2) + e) * wi;
    }
    if (e < HD) a.out[(uint64_t)r * a.ldo + h * HD + e] = Lg > 0.0f ? Ag / Lg : 0.0f;
    if (e == 0) a.counters[(uint64_t)cu.b * a.H + h] = 0u;
}

template <int HD>
static int launch_attention_hd(AttnArgs a, dim3 grid, cudaStream_t st, bool pdl)
{
    // warps per CTA: 16 in place of exactly 4 splits when the (row, head)
    // pairs alone give every SM a CTA (one CTA then merges four splits'
    // worth of warps in shared memory instead of four CTAs through a
    // cluster), else 4.  Measured on B200, config 3 decode, attention per
    // step (8 launches) at 4 / 8 / 16 warps: 32 sequences (256 pairs, 4
    // splits) 68.3 / 70.9 / 65.1 us; 16 sequences (8 splits) 56.9 / 56.6 /
    // 62.1; 8 sequences 39.3 / 41.8 / 47.3.  Tuning override:
    // FML_ATTN_WARPS = 4 | 8 | 16.
    int nw = (grid.z == 4 && (uint64_t)grid.x * grid.y >= 148) ? 16 : 4;
    if (const char* e = getenv("FML_ATTN_WARPS"))
    {
        const long v = strtol(e, nullptr, 10);
        if (v == 4 || (v == 8 && grid.z % 2 == 0) || (v == 16 && grid.z % 4 == 0)) nw = (int)v;
    }
    if (nw > 4)
    {
        grid.z /= (uint32_t)(nw / 4);
        a.S = grid.z;
    }
    // 2..8 splits: one cluster per (row, head), merged on chip
    // (FML_ATTN_CLUSTER=0: global partials and a completion counter)
    const char* cl_env = getenv("FML_ATTN_CLUSTER");
    const bool cl = !(cl_env && strtol(cl_env, nullptr, 10) == 0) && grid.z >= 2 && grid.z <= 8;
    a.rows = grid.y;
    if (grid.x == 0 || grid.y == 0 || grid.z == 0) return FML_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(32 * nw);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (pdl)
    {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cl)
    {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = 1;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = grid.z;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    cudaError_t e;
    if (nw == 16)
        e = cl ? cudaLaunchKernelEx(&cfg, attention_kernel<HD, 16, true>, a)
               : cudaLaunchKernelEx(&cfg, attention_kernel<HD, 16, false>, a);
    else if (nw == 8)
        e = cl ? cudaLaunchKernelEx(&cfg, attention_kernel<HD, 8, true>, a)
               : cudaLaunchKernelEx(&cfg, attention_kernel<HD, 8, false>, a);
    else
        e = cl ? cudaLaunchKernelEx(&cfg, attention_kernel<HD, 4, true>, a)
               : cudaLaunchKernelEx(&cfg, attention_kernel<HD, 4, false>, a);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int launch_attention_kernel(const AttnArgs& a, uint32_t hd, dim3 grid, cudaStream_t st, bool pdl)
{
    switch (hd)
    {
    case 32: return launch_attention_hd<32>(a, grid, st, pdl);
    case 64: return launch_attention_hd<64>(a, grid, st, pdl);
    case 128: return launch_attention_hd<128>(a, grid, st, pdl);
    default: return set_error(FML_ERR_UNSUPPORTED, "head dim %u not supported (32/64/128)", hd);
    }
}

// Split count for `pairs` (row, head) pairs over keys up to `ctx`: as many
// splits as still fit one wave of 4-warp CTAs (8 per SM on 148 SMs) -- a
// partial second wave would double the kernel's latency chain -- and at most
// 8, the largest portable cluster, so that the splits merge on chip
// (measured on config 3's shape: 8 clustered splits beat 16 merged through
// global memory by 8 % at 8 sequences and 11 % at one).
void attention_splits(uint64_t pairs, uint64_t ctx, uint32_t* S_out, uint32_t* chunk_out)
{
    uint64_t S = std::min<uint64_t>(8, (8 * 148) / pairs);
    if (const char* e = getenv("FML_ATTN_SPLITS"))  // tuning override
    {
        const long v = strtol(e, nullptr, 10);
        if (v >= 1 && v <= 256) S = (uint64_t)v;
    }
    const uint64_t max_s = (ctx + 31) / 32;
    if (S > max_s) S = max_s;
    if (S < 1) S = 1;
    *S_out = (uint32_t)S;
    *chunk_out = 0;  // keys per split follow each row's length
}

uint64_t attention_workspace_bytes(uint32_t B, uint32_t H, uint32_t hd, uint32_t S)
{
    // split partials (floats), then the per-(row, head) merge counters and
    // the work-unit counter, 256-aligned
    const uint64_t part = (uint64_t)B * H * S * (hd + 2) * sizeof(float);
    return ((part + 255) / 256) * 256 + ((uint64_t)B * H + 1) * sizeof(uint32_t);
}

}  // namespace fml

using namespace fml;

extern "C" {

int fml_device_error_count(uint64_t* count)
{
    FML_REQUIRE(count, "fml_device_error_count: null argument");
    int g = 0, k = 0, pf = 0;
    uint64_t tpw = 0;
    FML_CUDA_TRY(cudaDeviceSynchronize());
    FML_RC(gemm_tc_error_count(&g));
    FML_RC(skinny_error_count(&k));
    FML_RC(prefill_tc_error_count(&pf));
    FML_RC(fml_lm_tp_error_count(&tpw));
    *count = (uint64_t)g + (uint64_t)k + (uint64_t)pf + tpw;
    return FML_OK;
}

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
    FML_REQUIRE(aligned16(q) && aligned16(kcache) && aligned16(vcache),
                "fml_attention_decode: q and the K/V caches must be 16-byte aligned");
    uint32_t S, chunk;
    attention_splits((uint64_t)batch * heads, context, &S, &chunk);
    const uint64_t need = attention_workspace_bytes(batch, heads, head_dim, S);
    FML_REQUIRE(workspace && workspace_bytes >= need,
                "fml_attention_decode: workspace of %llu bytes needed (fml_attention_workspace_bytes)",
                (unsigned long long)need);
    cudaStream_t st = as_stream(stream);
    const uint64_t part_bytes = need - ((uint64_t)batch * heads + 1) * sizeof(uint32_t);
    uint32_t* counters = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + part_bytes);
    FML_CUDA_TRY(cudaMemsetAsync(counters, 0, ((size_t)batch * heads + 1) * sizeof(uint32_t), st));
    AttnArgs a{};
    a.q = q; a.ldq = heads * head_dim; a.row0 = 0;
    a.kc = kcache; a.vc = vcache; a.seq_stride = (uint64_t)heads * context * head_dim;
    a.H = heads; a.C = context;
    a.out = out; a.ldo = heads * head_dim;
    a.pos = nullptr; a.lens = lens; a.P = 1;
    a.S = S; a.chunk = chunk; a.scale = scale;
    a.part = static_cast<float*>(workspace);
    a.counters = counters;
    a.grab = counters + (uint64_t)batch * heads;
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
// current) and cached together with the CUDA context it belongs to; the first
// call on a device does this set-up, so make that first call outside any
// stream capture.  When the device's context changes (after a device reset the
// runtime loads this library's module into a new context) the address is
// fetched again.
// ---------------------------------------------------------------------------

static __device__ __align__(256) unsigned char g_attention_scratch[FML_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
struct ScratchAddr
{
    CUcontext ctx;
    void* addr;
};
ScratchAddr g_scratch_addr[kMaxDevices] = {};

// The calling thread's current context, through the driver entry point the
// runtime hands out (the library links no driver library directly); null
// when there is none or the entry point is unavailable.
CUcontext current_context()
{
    using GetCurrent = CUresult (*)(CUcontext*);
    static GetCurrent fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetCurrent>(p);
    });
    CUcontext ctx = nullptr;
    if (!fn || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

int noalloc_scratch(void** out)
{
    int dev = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(FML_ERR_UNSUPPORTED, "fml_attention_decode_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    CUcontext ctx = current_context();
    ScratchAddr& slot = g_scratch_addr[dev];
    if (!slot.addr || !ctx || ctx != slot.ctx)
    {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess || !p)
            return set_error(FML_ERR_CUDA, "fml_attention_decode_noalloc: cudaGetSymbolAddress failed: %s",
                             cudaGetErrorString(e));
        // the lookup made the device's context current if it was not yet
        ctx = current_context();
        slot.ctx = ctx;
        slot.addr = p;
    }
    *out = slot.addr;
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
    FML_REQUIRE(aligned16(q) && aligned16(kcache) && aligned16(vcache),
                "fml_attention_decode_noalloc: q and the K/V caches must be 16-byte aligned");
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
    const uint64_t part_bytes = need - ((uint64_t)batch * heads + 1) * sizeof(uint32_t);
    uint32_t* counters = reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + part_bytes);
    FML_CUDA_TRY(cudaMemsetAsync(counters, 0, ((size_t)batch * heads + 1) * sizeof(uint32_t), st));
    AttnArgs a{};
    a.q = q; a.ldq = heads * head_dim; a.row0 = 0;
    a.kc = kcache; a.vc = vcache; a.seq_stride = (uint64_t)heads * context * head_dim;
    a.H = heads; a.C = context;
    a.out = out; a.ldo = heads * head_dim;
    a.pos = nullptr; a.lens = lens; a.P = 1;
    a.S = S; a.chunk = chunk; a.scale = scale;
    a.part = static_cast<float*>(scratch);
    a.counters = counters;
    a.grab = counters + (uint64_t)batch * heads;
    return launch_attention_kernel(a, head_dim, dim3(heads, batch, S), st);
}

}  // extern "C"
