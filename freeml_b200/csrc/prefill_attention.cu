// Causal attention over whole prompts (the engine's prefill):
// CausalSelfAttentionLayer::Forward (CausalSelfAttentionLayer.h:424-499) for
// all P rows of every sequence and head, Q K^T * 1/sqrt(hd) with the causal
// mask, softmax, times V, as tiles: one CTA per (64 query rows, head,
// sequence) walks the key tiles 0..(its last row) with an online softmax, so
// every K/V row of a (sequence, head) is read once per 64 queries instead of
// once per query.
//
// CTA = 256 threads, 16 x 16.  Thread (ty, tx) owns query rows
// ty + 16i and keys tx + 16j (i, j < 4) of the 64 x 64 score tile, and output
// columns tx + 16c of its rows.  Strided ownership keeps the float4 reads of
// the padded Q and K tiles bank-conflict free.  A row's 64 scores live in the
// 16 lanes of one half-warp: max and sum are 4-step shuffles.  P goes through
// shared memory for the P . V product.  The K / V tiles are double-buffered:
// tile k + 1 is copied (cp.async) while tile k is used.  fp32 throughout;
// expf.
#include <cmath>

#include "fml_common.cuh"

namespace fml {
namespace {

constexpr int PQ = 64, PK = 64;

__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy that bypasses registers (L2 only); with
// `fill` false it writes zeros and reads nothing
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool fill)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(fill ? 16 : 0)
                 : "memory");
}

template <int HD>
__global__ void __launch_bounds__(256) prefill_attention_kernel(const float* __restrict__ q, uint32_t ldq,
                                                                const float* __restrict__ kc,
                                                                const float* __restrict__ vc, uint64_t seq_stride,
                                                                uint32_t C, float* __restrict__ out, uint32_t ldo,
                                                                uint32_t P, float scale)
{
    constexpr int HP = HD + 4;  // padded row (floats)
    constexpr int OC = HD / 16; // output columns per thread
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;              // [PQ][HP]
    float* Kb = Qs + PQ * HP;    // 2 x [PK][HP]: K tiles, double-buffered
    float* Vb = Kb + 2 * PK * HP;  // 2 x [PK][HP]: V tiles
    float* Ps = Vb + 2 * PK * HP;  // [PQ][PK + 4]

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const uint32_t qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const uint32_t q0 = qt * PQ;
    const uint32_t nq = P - q0 < (uint32_t)PQ ? P - q0 : (uint32_t)PQ;
    const float* kbase = kc + (uint64_t)b * seq_stride + (uint64_t)h * C * HD;
    const float* vbase = vc + (uint64_t)b * seq_stride + (uint64_t)h * C * HD;

    // Q tile, pre-scaled
    for (int i = tid; i < PQ * (HD / 4); i += 256)
    {
        const int r = i / (HD / 4), c = i % (HD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if ((uint32_t)r < nq)
        {
            v = *reinterpret_cast<const float4*>(q + (uint64_t)(b * P + q0 + r) * ldq + h * HD + c * 4);
            v.x *= scale;
            v.y *= scale;
            v.z *= scale;
            v.w *= scale;
        }
        *reinterpret_cast<float4*>(Qs + r * HP + c * 4) = v;
    }

    float mrow[4], lrow[4], o[4][OC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        mrow[i] = -INFINITY;
        lrow[i] = 0.f;
#pragma unroll
        for (int c = 0; c < OC; ++c) o[i][c] = 0.f;
    }

    const uint32_t klast = q0 + nq - 1;  // last key any row of this tile sees
    // K / V tile kt into buffer kt & 1 (rows past klast zero-filled), issued
    // one tile ahead so that its copy overlaps the current tile's arithmetic
    auto issue_tile = [&](uint32_t kt) {
        const uint32_t k0 = kt * PK;
        float* Kd = Kb + (kt & 1u) * PK * HP;
        float* Vd = Vb + (kt & 1u) * PK * HP;
        for (int i = tid; i < PK * (HD / 4); i += 256)
        {
            const int r = i / (HD / 4), c = i % (HD / 4);
            const bool in = k0 + r <= klast;
            const uint64_t off = (uint64_t)(in ? k0 + r : 0u) * HD + c * 4;
            cp_async16_zfill(Kd + r * HP + c * 4, kbase + off, in);
            cp_async16_zfill(Vd + r * HP + c * 4, vbase + off, in);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const uint32_t ntiles = klast / PK + 1;
    issue_tile(0);
    for (uint32_t kt = 0; kt < ntiles; ++kt)
    {
        const uint32_t k0 = kt * PK;
        const float* Ks = Kb + (kt & 1u) * PK * HP;
        const float* Vs = Vb + (kt & 1u) * PK * HP;
        // the next tile's buffer was last read in iteration kt - 1, which
        // ended with a barrier
        if (kt + 1 < ntiles)
        {
            issue_tile(kt + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        }
        else
        {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // tile kt has landed for every thread

        // scores for rows ty + 16i, keys tx + 16j
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
        for (int e = 0; e < HD; e += 4)
        {
            float4 qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(Qs + (ty + 16 * i) * HP + e);
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * j) * HP + e);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                {
                    float a = s[i][j];
                    a = fmaf(qv[i].x, kv[j].x, a);
                    a = fmaf(qv[i].y, kv[j].y, a);
                    a = fmaf(qv[i].z, kv[j].z, a);
                    a = fmaf(qv[i].w, kv[j].w, a);
                    s[i][j] = a;
                }
        }
        // causal mask, online softmax per row (the row's 16 lanes)
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const uint32_t qi = q0 + ty + 16 * i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j)
            {
                const uint32_t kj = k0 + tx + 16 * j;
                if (kj > qi) s[i][j] = -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, off));
            const float mnew = fmaxf(mrow[i], mx);
            // every row sees key k0 of its last tile, so mnew is finite; the
            // guard only keeps the arithmetic finite if that ever changed
            const float base = mnew == -INFINITY ? 0.f : mnew;
            const float corr = expf(mrow[i] - base);
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j)
            {
                const float p = expf(s[i][j] - base);
                ps += p;
                Ps[(ty + 16 * i) * (PK + 4) + tx + 16 * j] = p;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ps += __shfl_xor_sync(FULL_MASK, ps, off);
            lrow[i] = fmaf(lrow[i], corr, ps);
#pragma unroll
            for (int c = 0; c < OC; ++c) o[i][c] *= corr;
            mrow[i] = mnew;
        }
        __syncthreads();
        // O[rows][cols] += P[rows][keys] . V[keys][cols]
        const uint32_t kn = klast - k0 + 1 < (uint32_t)PK ? klast - k0 + 1 : (uint32_t)PK;
        for (uint32_t k = 0; k < kn; ++k)
        {
            float pv[4], vv[OC];
#pragma unroll
            for (int i = 0; i < 4; ++i) pv[i] = Ps[(ty + 16 * i) * (PK + 4) + k];
#pragma unroll
            for (int c = 0; c < OC; ++c) vv[c] = Vs[k * HP + tx + 16 * c];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < OC; ++c) o[i][c] = fmaf(pv[i], vv[c], o[i][c]);
        }
        __syncthreads();  // this tile's K / V / P readers are done
    }

#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const uint32_t r = ty + 16 * i;
        if (r >= nq) continue;
        const float inv = 1.0f / lrow[i];
        float* dst = out + (uint64_t)(b * P + q0 + r) * ldo + h * HD;
#pragma unroll
        for (int c = 0; c < OC; ++c) dst[tx + 16 * c] = o[i][c] * inv;
    }
}

template <int HD>
int launch_hd(const float* q, uint32_t ldq, const float* kc, const float* vc, uint64_t seq_stride, uint32_t C,
              float* out, uint32_t ldo, uint32_t B, uint32_t H, uint32_t P, float scale, cudaStream_t st)
{
    const size_t smem = sizeof(float) * (5 * PQ * (HD + 4) + PQ * (PK + 4));
    static uint64_t attr_devices = 0;
    FML_RC(smem_limit_once(reinterpret_cast<const void*>(prefill_attention_kernel<HD>), (int)smem, attr_devices));
    const dim3 grid((P + PQ - 1) / PQ, H, B);
    prefill_attention_kernel<HD><<<grid, 256, smem, st>>>(q, ldq, kc, vc, seq_stride, C, out, ldo, P, scale);
    FML_LAUNCH_CHECK();
    return FML_OK;
}

}  // namespace

// Prefill attention for rows (b, t), t < P, of B sequences and H heads:
// q / out [B*P x ld] (head h at columns h*hd), keys and values of sequence b,
// head h at kc/vc + b*seq_stride + h*C*hd (rows 0..P-1 filled).
int launch_prefill_attention(const float* q, uint32_t ldq, const float* kc, const float* vc, uint64_t seq_stride,
                             uint32_t C, float* out, uint32_t ldo, uint32_t B, uint32_t H, uint32_t P, uint32_t hd,
                             float scale, cudaStream_t st)
{
    FML_REQUIRE(B <= 65535u && H <= 65535u, "prefill attention: %u sequences x %u heads", B, H);
    FML_REQUIRE(ldq % 4 == 0 && ldo % 4 == 0, "prefill attention: row strides must be multiples of 4");
    switch (hd)
    {
    case 32: return launch_hd<32>(q, ldq, kc, vc, seq_stride, C, out, ldo, B, H, P, scale, st);
    case 64: return launch_hd<64>(q, ldq, kc, vc, seq_stride, C, out, ldo, B, H, P, scale, st);
    case 128: return launch_hd<128>(q, ldq, kc, vc, seq_stride, C, out, ldo, B, H, P, scale, st);
    default: return set_error(FML_ERR_UNSUPPORTED, "prefill attention: head dim %u", hd);
    }
}

}  // namespace fml
