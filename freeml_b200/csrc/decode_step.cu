// The fused decode step: FreeML's per-token Model::Run (ModelLibrary/Model.h:
// 764-788 over the NanoLLM graph, Examples/NanoLLM/NanoLLM.cpp:268-358) for a
// batch of sequences as ONE persistent kernel launch per generated token.
//
// Why: a decode step is ~40 dependent phases (per layer: LayerNorm+QKV,
// attention, proj+residual, LayerNorm+fc+GELU, mlp+residual; then
// LayerNorm+lm_head+argmax), each only a few MB of weights or K/V rows.  As
// separate kernels every phase pays launch, ramp-up and tail, and DRAM idles
// between them.  Here the weights and the K/V rows written by earlier steps --
// all the bytes a step must stream -- do not depend on the step's own
// results, so each CTA's producer warp streams them into a shared-memory ring
// (cp.async.bulk + mbarrier) straight across phase boundaries, while the
// consumer warps wait only for the activations the previous phase wrote.
//
// Work decomposition.  The step is a fixed sequence of phases; phase p is
// split into work items and the items are numbered globally in phase order.
// CTA c takes items c, c + G, c + 2G, ... (G = grid size) and processes them
// in that order.  Item kinds:
//   * weight item: `rows` consecutive output rows of one Dense (or of the
//     tied lm_head), all K inputs, for one token group.  The rows' weights
//     (K-contiguous, one bulk copy) fill one ring entry.
//   * attention item: one (sequence, head).  Its K and V rows below the
//     sequence's position arrive through ceil(pos / kch) ring entries; the
//     new row (written by this step's QKV phase) is read from global memory.
// A consumer starts an item of phase p after phase p - ng (the previous
// phase of the same token group) has all its items done: one thread polls
// that phase's counter (ld.acquire.gpu), producers publish with
// __threadfence + atomicAdd.  Dependencies always point to earlier items, and
// every CTA is resident (cooperative launch), so the oldest unfinished item
// can always run: the schedule cannot deadlock.  Every wait is bounded
// (1 s); a wait that runs out sets the abort flag, which makes all other
// waits return at once, and counts itself in g_step_timeouts.
//
// Token groups.  With ng = 2 the batch is split in halves whose phases
// interleave (QKV g0, QKV g1, ATT g0, ATT g1, ...): one group's dependency
// wait overlaps the other group's work, and each group's staged activations
// are half the size.  The second group's weight reads hit L2.
//
// Completion signals leave the consumers' path: after an item's stores the
// consumers arrive on a CTA-local mbarrier queue, and a signal warp turns each
// arrival into __threadfence + atomicAdd on the phase counter (the
// barrier-then-release pattern), so no consumer thread waits on a fence.
//
// Consumer arithmetic (fp32, CUDA cores).  The phase input X (LayerNorm
// applied) is staged once per phase in shared memory, [tokens x d] with a
// padded row stride; all LayerNorm gammas stay resident in shared memory.
// Register blocking: lane = (token lane tb, k-group g), 8 x 4 per warp; a lane
// accumulates TB tokens x RM weight rows, so each weight float4 read from
// shared memory feeds 4 TB FMAs.  Warp w and k-group g own float4 columns
// c = 4w + g (mod 32).  Partial sums meet in a two-step transpose reduction
// over the k-groups and a fixed-order sum over warps: deterministic.
// The mlp input (4d per token) is staged whole when it fits beside the ring,
// else in four K segments accumulated in registers.
//
// Parity notes: LayerNorm two-pass mean / biased variance with
// 1/sqrt(var/d + 1e-5) (LayerNorm.h:148-165); exact erf GELU (Gelu.h);
// causal softmax over keys 0..pos (CausalSelfAttentionLayer.h:66-67) in the
// online (running max) form; argmax keeps the first maximal index
// (NanoLLM.cpp:189-204).
#include <cmath>
#include <cstdlib>

#include "decode_step.cuh"
#include "fml_common.cuh"

namespace fml {
namespace {

constexpr int NCW = 8;              // consumer warps
constexpr int NCT = NCW * 32;       // consumer threads
constexpr int NTHREADS = NCT + 64;  // + a producer warp and a signal warp
constexpr int NSIG = 4;             // completion queue depth (consumers -> signal warp)
constexpr int RMAX = 16;            // weight rows per item, at most
constexpr int MAX_SLOTS = 8;
constexpr int MAX_TOK = 32;
constexpr uint64_t WAIT_NS = 1000000000ull;

__device__ unsigned int g_step_timeouts = 0;

// Optional per-item timeline (debug builds with FML_STEP_TRACE): consumer
// thread 0 records globaltimer stamps of each item's stages.
#ifdef FML_STEP_TRACE
__device__ unsigned long long* g_step_trace = nullptr;
__device__ uint32_t g_step_trace_cap = 0;
struct Trace
{
    unsigned long long ts[12];
    __device__ void mark(int k, int tid)
    {
        if (tid == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ts[k]));
    }
    __device__ void flush(uint32_t j, uint32_t i, uint32_t p, int tid)
    {
        if (tid != 0 || !g_step_trace || j >= g_step_trace_cap) return;
        unsigned long long* r = g_step_trace + ((uint64_t)blockIdx.x * g_step_trace_cap + j) * 12;
        r[0] = ((unsigned long long)i << 32) | p;
        for (int k = 1; k < 12; ++k) r[k] = ts[k];
    }
};
#else
struct Trace
{
    __device__ void mark(int, int) {}
    __device__ void flush(uint32_t, uint32_t, uint32_t, int) {}
};
#endif

struct Misc
{
    uint64_t full[MAX_SLOTS];
    uint64_t empty[MAX_SLOTS];
    uint64_t sig_full[NSIG];
    uint64_t sig_empty[NSIG];
    uint32_t posv[MAX_TOK];
    uint32_t nch[MAX_TOK];
    float hv[RMAX][MAX_TOK];
    float mean[MAX_TOK], rstd[MAX_TOK];
    uint32_t flag;
};

// ---------------------------------------------------------- primitives --

__device__ __forceinline__ uint64_t gtimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Global -> shared bulk copy into this CTA only, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 16-byte global -> shared copy through L2 only (generic proxy; the source
// was written by other CTAs in this launch, so no L1 copy may be used).
__device__ __forceinline__ void cp_async16(void* dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Named barrier of the consumer warps (the producer warp never joins it).
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

__device__ __noinline__ void give_up(uint32_t* abortp)
{
    atomicAdd(&g_step_timeouts, 1u);
    atomicExch(abortp, 1u);
}

__device__ __forceinline__ bool aborted(const uint32_t* abortp) { return *(volatile const uint32_t*)abortp != 0u; }

__device__ bool wait_mbar(uint64_t* bar, uint32_t parity, uint32_t* abortp)
{
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t it = 1;; ++it)
    {
        if (mbar_try(bar, parity)) return true;
        if ((it & 15u) == 0u)
        {
            if (aborted(abortp)) return false;
            if (gtimer() - t0 > WAIT_NS)
            {
                give_up(abortp);
                return false;
            }
        }
    }
}

__device__ bool wait_count(const uint32_t* ctr, uint32_t target, uint32_t* abortp)
{
    if (ld_acquire(ctr) >= target) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t it = 1;; ++it)
    {
        __nanosleep(32);
        if (ld_acquire(ctr) >= target) return true;
        if ((it & 15u) == 0u)
        {
            if (aborted(abortp)) return false;
            if (gtimer() - t0 > WAIT_NS)
            {
                give_up(abortp);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------ geometry --

struct Phase
{
    uint32_t t, l, g;
};

__device__ __forceinline__ Phase phase_of(const StepArgs& a, uint32_t p)
{
    const uint32_t per = 5u * a.ng;
    if (p < a.L * per) return {(p % per) / a.ng, p / per, p % a.ng};
    return {SP_HEAD, a.L, p - a.L * per};
}

__device__ __forceinline__ uint32_t group_tokens(const StepArgs& a, uint32_t g)
{
    const uint32_t b0 = g * a.bg;
    return a.B - b0 < a.bg ? a.B - b0 : a.bg;
}

__device__ __forceinline__ uint32_t phase_items(const StepArgs& a, const Phase& ph)
{
    return ph.t == SP_ATT ? group_tokens(a, ph.g) * a.H : a.items[ph.t];
}

__device__ __forceinline__ uint32_t n_phases(const StepArgs& a) { return 5u * a.L * a.ng + a.ng; }

__device__ __forceinline__ const float* layer_base(const StepArgs& a, uint32_t l)
{
    const uint64_t d = a.d;
    return a.wbuf + (uint64_t)(a.V + a.C) * d + (uint64_t)l * (2 * d + 12 * d * d);
}

// weight rows of a phase type: base pointer, K (inputs) and N (outputs)
__device__ __forceinline__ const float* weight_base(const StepArgs& a, uint32_t t, uint32_t l, uint32_t& K,
                                                    uint32_t& N)
{
    const uint64_t d = a.d;
    const float* lb = layer_base(a, l);
    switch (t)
    {
    case SP_QKV: K = a.d; N = 3 * a.d; return lb + d;
    case SP_PROJ: K = a.d; N = a.d; return lb + d + 3 * d * d;
    case SP_FC: K = a.d; N = 4 * a.d; return lb + 2 * d + 4 * d * d;
    case SP_MLP: K = 4 * a.d; N = a.d; return lb + 2 * d + 8 * d * d;
    default: K = a.d; N = a.V; return a.wbuf;  // SP_HEAD: the token table
    }
}

__device__ __forceinline__ const float* ln_gamma(const StepArgs& a, uint32_t t, uint32_t l)
{
    const uint64_t d = a.d;
    if (t == SP_QKV) return layer_base(a, l);
    if (t == SP_FC) return layer_base(a, l) + d + 4 * d * d;
    return layer_base(a, a.L);  // lnf follows the last layer
}

// Row of the resident gamma table: ln0[l] -> 2l, ln1[l] -> 2l + 1, lnf -> 2L.
__device__ __forceinline__ uint32_t gamma_row(const StepArgs& a, uint32_t t, uint32_t l)
{
    return t == SP_QKV ? 2 * l : (t == SP_FC ? 2 * l + 1 : 2 * a.L);
}

struct Cursor
{
    uint32_t p = 0, base = 0, cnt = 0;
    Phase ph{};
    __device__ void start(const StepArgs& a)
    {
        p = 0;
        base = 0;
        ph = phase_of(a, 0);
        cnt = phase_items(a, ph);
    }
    __device__ void seek(const StepArgs& a, uint32_t i)
    {
        while (i >= base + cnt)
        {
            base += cnt;
            ++p;
            ph = phase_of(a, p);
            cnt = phase_items(a, ph);
        }
    }
};

// ------------------------------------------------------------- producer --

__device__ __forceinline__ void produce(const StepArgs& a, Misc& m, unsigned char* ring, uint32_t& e, const float* src,
                                        const float* src2, uint32_t bytes, uint32_t* abortp, int lane)
{
    const uint32_t s = e % a.nslot;
    if (e >= a.nslot) wait_mbar(&m.empty[s], ((e / a.nslot) - 1u) & 1u, abortp);
    if (lane == 0)
    {
        unsigned char* dst = ring + (uint64_t)s * a.slot;
        if (bytes == 0u) mbar_arrive(&m.full[s]);
        else
        {
            mbar_expect_tx(&m.full[s], src2 ? 2u * bytes : bytes);
            bulk_load(dst, src, bytes, &m.full[s]);
            if (src2) bulk_load(dst + a.slot / 2, src2, bytes, &m.full[s]);
        }
    }
    __syncwarp();
    ++e;
}

template <int HD>
__device__ void producer_loop(const StepArgs& a, Misc& m, unsigned char* ring, uint32_t T, uint32_t* abortp, int lane)
{
    Cursor cur;
    cur.start(a);
    uint32_t e = 0;
    for (uint32_t i = blockIdx.x; i < T; i += gridDim.x)
    {
        cur.seek(a, i);
        const uint32_t local = i - cur.base;
        const Phase ph = cur.ph;
        if (ph.t != SP_ATT)
        {
            uint32_t K, N;
            const float* w = weight_base(a, ph.t, ph.l, K, N);
            const uint32_t R = a.rows[ph.t], r0 = local * R;
            const uint32_t rows = N - r0 < R ? N - r0 : R;
            produce(a, m, ring, e, w + (uint64_t)r0 * K, nullptr, rows * K * 4u, abortp, lane);
        }
        else
        {
            const uint32_t bt = ph.g * a.bg + local / a.H, h = local % a.H;
            const uint32_t pb = m.posv[bt], nch = m.nch[bt];
            const uint64_t kvb = (uint64_t)ph.l * a.layer_stride + (uint64_t)bt * a.seq_stride + (uint64_t)h * a.C * HD;
            for (uint32_t c = 0; c < nch; ++c)
            {
                const uint32_t k0 = c * a.kch;
                const uint32_t nk = pb > k0 ? (pb - k0 < a.kch ? pb - k0 : a.kch) : 0u;
                produce(a, m, ring, e, a.kc + kvb + (uint64_t)k0 * HD, a.vc + kvb + (uint64_t)k0 * HD,
                        nk * HD * 4u, abortp, lane);
            }
        }
    }
}

// ------------------------------------------------------------ consumers --

// Stage a phase input for tokens [b0, b0 + nt) into xs, row stride
// (K4 + xpad4) float4: QKV / HEAD read the residual stream x, PROJ the
// attention output, FC buf, MLP one K segment of hid.  LayerNorm is applied
// in place for QKV / FC / HEAD.  Layer 0's QKV input is the embedding sum,
// computed here; the CTA that owns the phase's first item also writes it to x
// (the residual read by layer 0's proj).
__device__ void stage_x(const StepArgs& a, Misc& m, float* xs, float* gam, uint32_t t, uint32_t l, uint32_t seg,
                        uint32_t b0, uint32_t nt, bool owner0, int tid, Trace& tr)
{
    const bool ln = t == SP_QKV || t == SP_FC || t == SP_HEAD;
    const uint32_t d4 = a.d >> 2;
    const float* gs = gam;
    if (ln)
    {
        if (a.gam_all) gs = gam + (uint64_t)gamma_row(a, t, l) * a.d;
        else
        {
            const float4* g4 = reinterpret_cast<const float4*>(ln_gamma(a, t, l));
            for (uint32_t c = tid; c < d4; c += NCT) cp_async16(reinterpret_cast<float4*>(gam) + c, g4 + c);
        }
    }
    const uint32_t K4 = t == SP_MLP ? 4 * d4 / a.mlp_segs : d4;  // staged width
    const uint32_t xs4 = K4 + a.xpad4;
    float4* X = reinterpret_cast<float4*>(xs);
    const bool embed = t == SP_QKV && l == 0;
    // rows into X with 16-byte cp.async (L2 only: the rows were written by
    // other CTAs in this launch); layer 0 takes token-table rows and adds the
    // position rows below
    {
        const float* srcf = t == SP_PROJ ? a.att : (t == SP_FC ? a.buf : (t == SP_MLP ? a.hid : a.x));
        const uint32_t row4 = t == SP_MLP ? 4 * d4 : d4;
        for (uint32_t idx = tid; idx < nt * K4; idx += NCT)
        {
            const uint32_t b = idx / K4, c = idx - b * K4;
            const float4* src;
            if (embed)
            {
                const uint32_t id = a.pending[b0 + b];
                src = reinterpret_cast<const float4*>(a.wbuf) + (uint64_t)(id < a.V ? id : 0u) * d4 + c;
            }
            else src = reinterpret_cast<const float4*>(srcf) + (uint64_t)(b0 + b) * row4 + (uint64_t)seg * K4 + c;
            cp_async16(X + b * xs4 + c, src);
        }
    }
    if (embed)
    {
        const float4* pe = reinterpret_cast<const float4*>(a.wbuf + (uint64_t)a.V * a.d);
        float4* x4 = reinterpret_cast<float4*>(a.x);
        constexpr int BATCH = 8;
        for (uint32_t base = tid; base < nt * d4; base += NCT * BATCH)
        {
            float4 pv[BATCH];
#pragma unroll
            for (int k = 0; k < BATCH; ++k)
            {
                const uint32_t idx = base + (uint32_t)k * NCT;
                pv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (idx < nt * d4)
                {
                    const uint32_t b = idx / d4, c = idx - b * d4, ps = m.posv[b0 + b];
                    if (ps < a.C) pv[k] = __ldg(pe + (uint64_t)ps * d4 + c);
                }
            }
            cp_async_wait_all();  // this thread's own token-row copies
#pragma unroll
            for (int k = 0; k < BATCH; ++k)
            {
                const uint32_t idx = base + (uint32_t)k * NCT;
                if (idx >= nt * d4) break;
                const uint32_t b = idx / d4, c = idx - b * d4, bt = b0 + b;
                const bool ok = a.pending[bt] < a.V && m.posv[bt] < a.C;
                float4 v = X[b * xs4 + c];
                v = ok ? make_float4(v.x + pv[k].x, v.y + pv[k].y, v.z + pv[k].z, v.w + pv[k].w)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
                X[b * xs4 + c] = v;
                if (owner0) x4[(uint64_t)bt * d4 + c] = v;
            }
        }
    }
    cp_async_wait_all();
    tr.mark(8, tid);
    cbar();
    if (!ln) return;

    const int warp = tid >> 5, lane = tid & 31;
    const float invd = 1.0f / (float)a.d;
    for (uint32_t b = warp; b < nt; b += NCW)
    {
        float s = 0.f;
        for (uint32_t c = lane; c < d4; c += 32)
        {
            const float4 v = X[b * xs4 + c];
            s += (v.x + v.y) + (v.z + v.w);
        }
        const float mean = warp_sum(s) * invd;
        float q = 0.f;
        for (uint32_t c = lane; c < d4; c += 32)
        {
            const float4 v = X[b * xs4 + c];
            const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
            q = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, q))));
        }
        q = warp_sum(q);
        if (lane == 0)
        {
            m.mean[b] = mean;
            m.rstd[b] = 1.0f / sqrtf(fmaf(q, invd, 1e-5f));
        }
    }
    cbar();
    tr.mark(9, tid);
    const float4* g4 = reinterpret_cast<const float4*>(gs);
    for (uint32_t idx = tid; idx < nt * d4; idx += NCT)
    {
        const uint32_t b = idx / d4, c = idx - b * d4;
        float4 v = X[b * xs4 + c];
        const float4 g = g4[c];
        const float mu = m.mean[b], rs = m.rstd[b];
        v.x = (v.x - mu) * rs * g.x;
        v.y = (v.y - mu) * rs * g.y;
        v.z = (v.z - mu) * rs * g.z;
        v.w = (v.w - mu) * rs * g.w;
        X[b * xs4 + c] = v;
    }
    cbar();
}

// acc[r*TB + i] += sum_k X[tb*TB + i, k] W[r, col0 + k] over this lane's k
// columns of one staged segment (segK4 float4 columns; W rows have K4).  Rows
// past `rows` and tokens past `nt` re-read the last valid one (in bounds,
// never stored), so the loop has no branches and all of an iteration's loads
// issue before its FMAs.
template <int TB, int RM>
__device__ __forceinline__ void gemm_accumulate(float (&acc)[TB * RM], const float* __restrict__ wslot,
                                                const float* __restrict__ xs, uint32_t xs4, uint32_t K4,
                                                uint32_t col0, uint32_t segK4, uint32_t rows, uint32_t nt, int warp,
                                                int lane)
{
    const uint32_t tb = (uint32_t)lane >> 2, g = (uint32_t)lane & 3u;
    const uint32_t kp = (uint32_t)warp * 4u + g;
    constexpr uint32_t KP = NCW * 4;
    const float4* W4 = reinterpret_cast<const float4*>(wslot) + col0;
    const float4* X4[TB];
#pragma unroll
    for (int i = 0; i < TB; ++i)
    {
        const uint32_t b = tb * TB + i;
        X4[i] = reinterpret_cast<const float4*>(xs) + (uint64_t)(b < nt ? b : nt - 1u) * xs4;
    }
    uint32_t roff[RM];
#pragma unroll
    for (int r = 0; r < RM; ++r) roff[r] = ((uint32_t)r < rows ? (uint32_t)r : rows - 1u) * K4;
    for (uint32_t c = kp; c < segK4; c += KP)
    {
        float4 xv[TB], w[RM];
#pragma unroll
        for (int i = 0; i < TB; ++i) xv[i] = X4[i][c];
#pragma unroll
        for (int r = 0; r < RM; ++r) w[r] = W4[roff[r] + c];
#pragma unroll
        for (int r = 0; r < RM; ++r)
        {
#pragma unroll
            for (int i = 0; i < TB; ++i)
            {
                float s = acc[r * TB + i];
                s = fmaf(xv[i].x, w[r].x, s);
                s = fmaf(xv[i].y, w[r].y, s);
                s = fmaf(xv[i].z, w[r].z, s);
                s = fmaf(xv[i].w, w[r].w, s);
                acc[r * TB + i] = s;
            }
        }
    }
}

// Sum acc over the 4 k-groups of a token lane (two halving shuffle steps:
// lane keeps V/4 sums, those of indices base .. base + V/4) and publish them
// in red[warp][tb][*].
template <int V>
__device__ __forceinline__ void gemm_reduce(float (&acc)[V], float* red, int warp, int lane)
{
    const bool up1 = (lane & 1) != 0, up2 = (lane & 2) != 0;
#pragma unroll
    for (int i = 0; i < V / 2; ++i)
    {
        const float send = up1 ? acc[i] : acc[i + V / 2];
        const float keep = up1 ? acc[i + V / 2] : acc[i];
        acc[i] = keep + __shfl_xor_sync(FULL_MASK, send, 1);
    }
#pragma unroll
    for (int i = 0; i < V / 4; ++i)
    {
        const float send = up2 ? acc[i] : acc[i + V / 4];
        const float keep = up2 ? acc[i + V / 4] : acc[i];
        acc[i] = keep + __shfl_xor_sync(FULL_MASK, send, 2);
    }
    const int base = (up1 ? V / 2 : 0) + (up2 ? V / 4 : 0);
    float* dst = red + ((warp * 8 + (lane >> 2)) * V + base);
#pragma unroll
    for (int i = 0; i < V / 4; ++i) dst[i] = acc[i];
}

template <int TB, int RM>
__device__ __forceinline__ void gemm_rows(const StepArgs& a, Misc& m, float* xs, float* gam, float* red,
                                          const float* wslot, uint32_t& staged, const Cursor& cur,
                                          uint32_t t, uint32_t l, uint32_t b0, uint32_t nt, uint32_t K4,
                                          uint32_t rows, uint32_t s, uint32_t e, uint32_t* abortp, int tid,
                                          Trace& tr)
{
    const int warp = tid >> 5, lane = tid & 31;
    const uint32_t nseg = t == SP_MLP ? a.mlp_segs : 1u;
    const uint32_t segK4 = K4 / nseg;
    float acc[TB * RM];
#pragma unroll
    for (int i = 0; i < TB * RM; ++i) acc[i] = 0.f;
    for (uint32_t seg = 0; seg < nseg; ++seg)
    {
        const uint32_t key = cur.p * 8u + seg;
        if (staged != key)
        {
            if (seg > 0) cbar();  // the previous segment's readers are done
            stage_x(a, m, xs, gam, t, l, seg, b0, nt, (cur.base % gridDim.x) == blockIdx.x, tid, tr);
            staged = key;
        }
        if (seg == 0)
        {
            tr.mark(3, tid);
            wait_mbar(&m.full[s], (e / a.nslot) & 1u, abortp);
            tr.mark(4, tid);
        }
        gemm_accumulate<TB, RM>(acc, wslot, xs, segK4 + a.xpad4, K4, seg * segK4, segK4, rows, nt, warp, lane);
    }
    if (nseg > 1) staged = 0xffffffffu;  // xs holds a partial segment
    gemm_reduce<TB * RM>(acc, red, warp, lane);
}

__device__ __forceinline__ void signal_done(Misc& m, uint32_t j, uint32_t* abortp, int tid)
{
    if (tid == 0)
    {
        const uint32_t q = j % NSIG;
        if (j >= NSIG) wait_mbar(&m.sig_empty[q], ((j / NSIG) - 1u) & 1u, abortp);
        mbar_arrive(&m.sig_full[q]);
    }
}

template <int HD, int TB>
__device__ void gemm_item(const StepArgs& a, Misc& m, unsigned char* ring, float* red, float* xs, float* gam,
                          uint32_t& e, uint32_t& staged, const Cursor& cur, uint32_t local,
                          uint32_t j, uint32_t* abortp, int tid, Trace& tr)
{
    const Phase ph = cur.ph;
    const uint32_t t = ph.t, l = ph.l;
    const uint32_t b0 = ph.g * a.bg, nt = group_tokens(a, ph.g);
    const uint32_t d = a.d;
    uint32_t K, N;
    weight_base(a, t, l, K, N);
    const uint32_t K4 = K >> 2, R = a.rows[t], r0 = local * R;
    const uint32_t rows = N - r0 < R ? N - r0 : R;
    const uint32_t nout = rows * nt;

    // residual operands of this thread's outputs, fetched before the math
    float rv[2] = {0.f, 0.f};
    if (t == SP_PROJ || t == SP_MLP)
    {
        const float* rsrc = t == SP_PROJ ? a.x : a.buf;
#pragma unroll
        for (int k = 0; k < 2; ++k)
        {
            const uint32_t o = (uint32_t)tid + (uint32_t)k * NCT;
            if (o < nout)
            {
                const uint32_t b = o / rows, r = o - b * rows;
                rv[k] = __ldcg(rsrc + (uint64_t)(b0 + b) * d + r0 + r);
            }
        }
    }

    const uint32_t s = e % a.nslot;
    const float* wslot = reinterpret_cast<const float*>(ring + (uint64_t)s * a.slot);
    uint32_t RM;
    if (rows <= 4)
    {
        RM = 4;
        gemm_rows<TB, 4>(a, m, xs, gam, red, wslot, staged, cur, t, l, b0, nt, K4, rows, s, e, abortp, tid,
                               tr);
    }
    else if (rows <= 8)
    {
        RM = 8;
        gemm_rows<TB, 8>(a, m, xs, gam, red, wslot, staged, cur, t, l, b0, nt, K4, rows, s, e, abortp, tid,
                               tr);
    }
    else if (rows <= 12)
    {
        RM = 12;
        gemm_rows<TB, 12>(a, m, xs, gam, red, wslot, staged, cur, t, l, b0, nt, K4, rows, s, e, abortp, tid,
                               tr);
    }
    else
    {
        RM = 16;
        gemm_rows<TB, 16>(a, m, xs, gam, red, wslot, staged, cur, t, l, b0, nt, K4, rows, s, e, abortp, tid,
                               tr);
    }
    cbar();
    tr.mark(5, tid);
    if (tid == 0) mbar_arrive(&m.empty[s]);
    ++e;

    // outputs (r fastest: consecutive threads write consecutive columns)
    const uint32_t V = TB * RM;
#pragma unroll
    for (int k = 0; k < 2; ++k)
    {
        const uint32_t o = (uint32_t)tid + (uint32_t)k * NCT;
        if (o >= nout) break;
        const uint32_t b = o / rows, r = o - b * rows, bt = b0 + b, n = r0 + r;
        const uint32_t v = r * TB + (b % TB), tbb = b / TB;
        float val = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; ++w) val += red[((uint32_t)w * 8u + tbb) * V + v];
        switch (t)
        {
        case SP_QKV:
            if (n < d) a.q[(uint64_t)bt * d + n] = val;
            else
            {
                const uint32_t c = n < 2 * d ? n - d : n - 2 * d, h = c / HD, el = c % HD;
                float* cache = n < 2 * d ? a.kc : a.vc;
                cache[(uint64_t)l * a.layer_stride + (uint64_t)bt * a.seq_stride +
                      ((uint64_t)h * a.C + m.posv[bt]) * HD + el] = val;
            }
            break;
        case SP_PROJ: a.buf[(uint64_t)bt * d + n] = rv[k] + val; break;
        case SP_FC: a.hid[(uint64_t)bt * 4 * d + n] = gelu_exact(val); break;
        case SP_MLP: a.x[(uint64_t)bt * d + n] = rv[k] + val; break;
        default:
            if (a.logits) a.logits[(uint64_t)bt * a.V + n] = val;
            m.hv[r][b] = val;
            break;
        }
    }
    if (t == SP_HEAD)
    {
        cbar();
        if ((uint32_t)tid < nt)
        {
            unsigned long long best = 0ull;
            for (uint32_t r = 0; r < rows; ++r)
            {
                const unsigned long long key = argmax_key(m.hv[r][tid], r0 + r);
                best = key > best ? key : best;
            }
            atomicMax(a.keys + b0 + tid, best);
        }
    }
    tr.mark(6, tid);
    cbar();
    signal_done(m, j, abortp, tid);
    tr.mark(7, tid);
}

template <int HD>
__device__ void att_item(const StepArgs& a, Misc& m, unsigned char* ring, float* ws, uint32_t& e, const Cursor& cur,
                         uint32_t local, uint32_t j, uint32_t* abortp, int tid, Trace& tr)
{
    constexpr int EPL = HD / 32;
    const int lane = tid & 31, warp = tid >> 5;
    const Phase ph = cur.ph;
    const uint32_t bt = ph.g * a.bg + local / a.H, h = local % a.H;
    float* qs = ws;
    float* ored = ws + HD;
    float* mred = ored + NCW * HD;
    float* lred = mred + NCW;

    const uint32_t pb = m.posv[bt], nch = m.nch[bt];
    const uint64_t kvb = (uint64_t)ph.l * a.layer_stride + (uint64_t)bt * a.seq_stride + (uint64_t)h * a.C * HD;
    // the new row (key pos), written by this step's QKV phase: fetched now,
    // used after the cached rows
    float kn[EPL], vn[EPL];
    if (warp == NCW - 1)
    {
#pragma unroll
        for (int i = 0; i < EPL; ++i)
        {
            kn[i] = __ldcg(a.kc + kvb + (uint64_t)pb * HD + lane + 32 * i);
            vn[i] = __ldcg(a.vc + kvb + (uint64_t)pb * HD + lane + 32 * i);
        }
    }
    const float* qg = a.q + (uint64_t)bt * a.d + (uint64_t)h * HD;
    for (int i = tid; i < HD; i += NCT) qs[i] = __ldcg(qg + i) * a.scale;
    cbar();
    tr.mark(3, tid);
    float qr[EPL], o[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i)
    {
        qr[i] = qs[lane + 32 * i];
        o[i] = 0.f;
    }
    float mx = -INFINITY, ls = 0.f;
    for (uint32_t c = 0; c < nch; ++c)
    {
        const uint32_t s = e % a.nslot;
        wait_mbar(&m.full[s], (e / a.nslot) & 1u, abortp);
        if (c == 0) tr.mark(4, tid);
        const float* Ks = reinterpret_cast<const float*>(ring + (uint64_t)s * a.slot);
        const float* Vs = Ks + a.slot / 8;
        const uint32_t k0 = c * a.kch;
        const uint32_t nk = pb > k0 ? (pb - k0 < a.kch ? pb - k0 : a.kch) : 0u;
        // each warp takes blocks of 8 keys: 8 independent dot products, 8
        // interleaved butterfly sums, one running-max update per block
        for (uint32_t j0 = (uint32_t)warp * 8u; j0 < nk; j0 += NCW * 8u)
        {
            float sc[8];
            uint32_t jj[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
            {
                jj[u] = j0 + u < nk ? j0 + u : nk - 1u;
                float sd = 0.f;
#pragma unroll
                for (int i = 0; i < EPL; ++i) sd = fmaf(qr[i], Ks[jj[u] * HD + lane + 32 * i], sd);
                sc[u] = sd;
            }
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1)
            {
#pragma unroll
                for (int u = 0; u < 8; ++u) sc[u] += __shfl_xor_sync(FULL_MASK, sc[u], o2);
            }
            float bm = mx;
#pragma unroll
            for (int u = 0; u < 8; ++u)
            {
                if (j0 + u >= nk) sc[u] = -INFINITY;
                bm = fmaxf(bm, sc[u]);
            }
            const float corr = expf(mx - bm);
            float psum = 0.f, pj[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
            {
                pj[u] = expf(sc[u] - bm);
                psum += pj[u];
            }
            ls = fmaf(ls, corr, psum);
#pragma unroll
            for (int i = 0; i < EPL; ++i)
            {
                float acc = o[i] * corr;
#pragma unroll
                for (int u = 0; u < 8; ++u) acc = fmaf(pj[u], Vs[jj[u] * HD + lane + 32 * i], acc);
                o[i] = acc;
            }
            mx = bm;
        }
        cbar();
        if (tid == 0) mbar_arrive(&m.empty[s]);
        ++e;
    }
    if (warp == NCW - 1)
    {
        float sd = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) sd = fmaf(qr[i], kn[i], sd);
        sd = warp_sum(sd);
        const float mn = fmaxf(mx, sd);
        const float corr = expf(mx - mn), pj = expf(sd - mn);
        ls = fmaf(ls, corr, pj);
#pragma unroll
        for (int i = 0; i < EPL; ++i) o[i] = fmaf(pj, vn[i], o[i] * corr);
        mx = mn;
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) ored[warp * HD + lane + 32 * i] = o[i];
    if (lane == 0)
    {
        mred[warp] = mx;
        lred[warp] = ls;
    }
    cbar();
    if (tid < HD)
    {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NCW; ++w) M = fmaxf(M, mred[w]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; ++w)
        {
            const float f = expf(mred[w] - M);
            L = fmaf(lred[w], f, L);
            O = fmaf(ored[w * HD + tid], f, O);
        }
        a.att[(uint64_t)bt * a.d + (uint64_t)h * HD + tid] = O / L;
    }
    tr.mark(6, tid);
    cbar();
    signal_done(m, j, abortp, tid);
    tr.mark(7, tid);
}

template <int HD, int TB>
__global__ void __launch_bounds__(NTHREADS, 1) decode_step_kernel(const StepArgs a)
{
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* ring = smem;
    float* red = reinterpret_cast<float*>(smem + (uint64_t)a.nslot * a.slot);
    float* xs = red + a.red_floats;
    float* gam = xs + a.xs_floats;
    Misc& m = *reinterpret_cast<Misc*>(gam + a.gam_floats);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* abortp = a.sync + 1;

    if ((uint32_t)tid < a.B)
    {
        const uint32_t pb = a.pos[tid];
        m.posv[tid] = pb;
        m.nch[tid] = pb > 0u ? (pb + a.kch - 1u) / a.kch : 1u;
    }
    if (tid == 0)
    {
        for (uint32_t s = 0; s < a.nslot; ++s)
        {
            mbar_init(&m.full[s], 1);
            mbar_init(&m.empty[s], 1);
        }
        for (int q = 0; q < NSIG; ++q)
        {
            mbar_init(&m.sig_full[q], 1);
            mbar_init(&m.sig_empty[q], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    uint32_t T = 0;
    const uint32_t P = n_phases(a);
    for (uint32_t p = 0; p < P; ++p) T += phase_items(a, phase_of(a, p));

    if (warp == NCW)
        producer_loop<HD>(a, m, ring, T, abortp, lane);
    else if (warp == NCW + 1)
    {
        // signal warp: publish each finished item, in order
        Cursor cur;
        cur.start(a);
        uint32_t j = 0;
        for (uint32_t i = blockIdx.x; i < T; i += gridDim.x, ++j)
        {
            cur.seek(a, i);
            const uint32_t q = j % NSIG;
            wait_mbar(&m.sig_full[q], (j / NSIG) & 1u, abortp);
            if (lane == 0)
            {
                __threadfence();
                atomicAdd(a.sync + 2 + cur.p, 1u);
                mbar_arrive(&m.sig_empty[q]);
            }
            __syncwarp();
        }
    }
    else
    {
        if (a.gam_all)
        {
            // every LayerNorm gamma of the model, resident for the whole step
            const uint32_t d4 = a.d >> 2;
            for (uint32_t idx = tid; idx < (2 * a.L + 1) * d4; idx += NCT)
            {
                const uint32_t row = idx / d4, c = idx - row * d4;
                const uint32_t t = row == 2 * a.L ? (uint32_t)SP_HEAD : (row & 1u ? (uint32_t)SP_FC : (uint32_t)SP_QKV);
                cp_async16(reinterpret_cast<float4*>(gam) + idx,
                           reinterpret_cast<const float4*>(ln_gamma(a, t, row / 2)) + c);
            }
            cp_async_wait_all();
            cbar();
        }
        Cursor cur;
        cur.start(a);
        uint32_t e = 0, staged = 0xffffffffu, verified = 0, jt = 0;
        for (uint32_t i = blockIdx.x; i < T; i += gridDim.x, ++jt)
        {
            Trace tr;
            tr.mark(1, tid);
            cur.seek(a, i);
            const uint32_t local = i - cur.base;
            if (cur.p >= a.ng)
            {
                const uint32_t dp = cur.p - a.ng;
                if (dp + 1u > verified)
                {
                    if (tid == 0) wait_count(a.sync + 2 + dp, phase_items(a, phase_of(a, dp)), abortp);
                    cbar();
                    verified = dp + 1u;
                }
            }
            tr.mark(2, tid);
            if (cur.ph.t == SP_ATT) att_item<HD>(a, m, ring, red, e, cur, local, jt, abortp, tid, tr);
            else gemm_item<HD, TB>(a, m, ring, red, xs, gam, e, staged, cur, local, jt, abortp, tid, tr);
            tr.flush(jt, i, cur.p, tid);
        }
    }

    // the last CTA out finishes the step: next tokens, positions, and every
    // counter back to zero for the next launch
    __syncthreads();
    if (tid == 0)
    {
        __threadfence();
        m.flag = atomicAdd(a.sync, 1u) == gridDim.x - 1u;
    }
    __syncthreads();
    if (!m.flag) return;
    __threadfence();
    if ((uint32_t)tid < a.B)
    {
        const unsigned long long key = __ldcg(a.keys + tid);
        const uint32_t tok = argmax_key_index(key);
        a.pending[tid] = tok;
        if (a.next_out) a.next_out[tid] = tok;
        a.pos[tid] = m.posv[tid] + 1u;
        a.keys[tid] = 0ull;
    }
    for (uint32_t w = tid; w < P; w += NTHREADS) a.sync[2 + w] = 0u;
    if (tid == 0)
    {
        a.sync[1] = 0u;
        a.sync[0] = 0u;
    }
}

template <int HD>
void* kernel_tb(uint32_t tb)
{
    switch (tb)
    {
    case 1: return reinterpret_cast<void*>(&decode_step_kernel<HD, 1>);
    case 2: return reinterpret_cast<void*>(&decode_step_kernel<HD, 2>);
    case 4: return reinterpret_cast<void*>(&decode_step_kernel<HD, 4>);
    default: return nullptr;
    }
}

void* kernel_for(uint32_t hd, uint32_t tb)
{
    switch (hd)
    {
    case 32: return kernel_tb<32>(tb);
    case 64: return kernel_tb<64>(tb);
    case 128: return kernel_tb<128>(tb);
    default: return nullptr;
    }
}

uint32_t env_u32(const char* name, uint32_t dflt, uint32_t lo, uint32_t hi)
{
    if (const char* e = getenv(name))
    {
        const long v = strtol(e, nullptr, 10);
        if (v >= (long)lo && v <= (long)hi) return (uint32_t)v;
    }
    return dflt;
}

}  // namespace

uint32_t decode_step_sync_words(uint32_t L, uint32_t ng) { return 2u + 5u * L * ng + ng; }

int decode_step_plan(StepArgs& a, int device, int* grid, size_t* smem)
{
    if (a.B < 1 || a.B > (uint32_t)MAX_TOK)
        return set_error(FML_ERR_UNSUPPORTED, "fused step: batch %u outside [1, %d]", a.B, MAX_TOK);
    if (a.d % 32u) return set_error(FML_ERR_UNSUPPORTED, "fused step: d_model %u not a multiple of 32", a.d);
    if (a.hd != 32 && a.hd != 64 && a.hd != 128)
        return set_error(FML_ERR_UNSUPPORTED, "fused step: head dim %u", a.hd);

    // tuning knobs (defaults are the measured best)
    a.ng = env_u32("FML_STEP_GROUPS", 1u, 1u, 2u);
    if (a.ng > a.B) a.ng = 1;
    a.bg = (a.B + a.ng - 1) / a.ng;
    a.slot = 32768u;
    a.kch = a.slot / 2 / (a.hd * 4);
    if (4u * a.d * 4u > a.slot)
        return set_error(FML_ERR_UNSUPPORTED, "fused step: an mlp weight row (%u floats) exceeds a ring entry",
                         4u * a.d);
    // tokens per lane: 8 token lanes x 4 k-groups per warp
    a.tpw = a.bg <= 8 ? 1u : (a.bg <= 16 ? 2u : 4u);
    a.xpad4 = 4u / a.tpw;  // (TB * row stride) = 4 (mod 8) float4: conflict-free X reads
    void* kern = kernel_for(a.hd, a.tpw);
    const uint32_t att_ws = a.hd + NCW * a.hd + 2 * NCW;
    a.red_floats = NCW * 8u * a.tpw * RMAX;
    if (a.red_floats < att_ws) a.red_floats = att_ws;
    a.red_floats = (a.red_floats + 31u) & ~31u;
    a.scale = 1.0f / sqrtf((float)a.hd);

    int optin = 0, sms = 0;
    FML_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    FML_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    // shared memory: ring + reduction + staged activations + gammas.  Prefer
    // resident gammas, then a ring of >= 3 entries, then the whole mlp input
    // staged at once (else 4 K segments).
    const uint32_t want_slots = env_u32("FML_STEP_SLOTS", 0u, 2u, (uint32_t)MAX_SLOTS);
    size_t bytes = 0;
    bool ok = false;
    for (uint32_t min_slots = 3; min_slots >= 2 && !ok; --min_slots)
        for (uint32_t gall = 1; gall <= 1 && !ok; gall -= 1)
        {
            for (uint32_t segs = 1; segs <= 4 && !ok; segs *= 4)
            {
                a.gam_all = gall;
                a.gam_floats = gall ? (2 * a.L + 1) * a.d : a.d;
                a.mlp_segs = segs;
                const uint32_t w4 = a.d / segs > a.d / 4 ? a.d / segs : a.d / 4;  // staged float4 per row
                a.xs_floats = a.bg * (w4 + a.xpad4) * 4;
                const uint32_t hi = want_slots ? want_slots : 4u, lo = want_slots ? want_slots : min_slots;
                for (uint32_t ns = hi; ns >= lo && !ok; --ns)
                {
                    a.nslot = ns;
                    bytes = (size_t)a.nslot * a.slot + (size_t)(a.red_floats + a.xs_floats + a.gam_floats) * 4 +
                            sizeof(Misc);
                    ok = bytes <= (size_t)optin;
                }
            }
            if (gall == 0) break;
        }
    if (!ok)
    {
        // last resort: per-phase gammas
        for (uint32_t segs = 1; segs <= 4 && !ok; segs *= 4)
        {
            a.gam_all = 0;
            a.gam_floats = a.d;
            a.mlp_segs = segs;
            const uint32_t w4 = a.d / segs > a.d / 4 ? a.d / segs : a.d / 4;
            a.xs_floats = a.bg * (w4 + a.xpad4) * 4;
            a.nslot = 2;
            bytes = (size_t)a.nslot * a.slot + (size_t)(a.red_floats + a.xs_floats + a.gam_floats) * 4 + sizeof(Misc);
            ok = bytes <= (size_t)optin;
        }
    }
    if (!ok)
        return set_error(FML_ERR_UNSUPPORTED, "fused step: %zu bytes of shared memory (limit %d)", bytes, optin);
    FML_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    int occ = 0;
    FML_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NTHREADS, bytes));
    if (occ < 1) return set_error(FML_ERR_UNSUPPORTED, "fused step: kernel does not fit on an SM");
    const int G = sms;

    // weight items: about G / ng items per phase and group
    const uint32_t Ks[6] = {a.d, 0, a.d, a.d, 4 * a.d, a.d};
    const uint32_t Ns[6] = {3 * a.d, 0, a.d, 4 * a.d, a.d, a.V};
    for (int t = 0; t < 6; ++t)
    {
        if (t == SP_ATT)
        {
            a.rows[t] = 0;
            a.items[t] = 0;
            continue;
        }
        const uint32_t per = (uint32_t)G / a.ng;
        uint32_t R = (Ns[t] + per - 1) / per;
        const uint32_t cap = a.slot / (Ks[t] * 4);
        if (R > cap) R = cap;
        if (R > (uint32_t)RMAX) R = RMAX;
        if (R < 1) R = 1;
        a.rows[t] = R;
        a.items[t] = (Ns[t] + R - 1) / R;
    }
    *grid = G;
    *smem = bytes;
    return FML_OK;
}

int launch_decode_step(const StepArgs& a, int grid, size_t smem, cudaStream_t st)
{
    void* kern = kernel_for(a.hd, a.tpw);
    if (!kern) return set_error(FML_ERR_UNSUPPORTED, "fused step: head dim %u", a.hd);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<StepArgs*>(&a)};
    const cudaError_t e = cudaLaunchKernelExC(&cfg, kern, args);
    if (e != cudaSuccess) return set_error(FML_ERR_CUDA, "fused step launch: %s", cudaGetErrorString(e));
    FML_LAUNCH_CHECK();
    return FML_OK;
}

int decode_step_error_count(int* out)
{
    unsigned int v = 0;
    FML_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_step_timeouts, sizeof(v)));
    *out = (int)v;
    return FML_OK;
}

}  // namespace fml

#ifdef FML_STEP_TRACE
extern "C" __attribute__((visibility("default"))) int fml_debug_step_trace(void* buf, uint32_t cap)
{
    unsigned long long* p = static_cast<unsigned long long*>(buf);
    if (cudaMemcpyToSymbol(fml::g_step_trace, &p, sizeof(p)) != cudaSuccess) return 2;
    if (cudaMemcpyToSymbol(fml::g_step_trace_cap, &cap, sizeof(cap)) != cudaSuccess) return 2;
    return 0;
}
#endif
