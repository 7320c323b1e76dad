// Shared helpers for the freeml_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "../../include/freeml_cuda.h"

namespace fml {

constexpr unsigned FULL_MASK = 0xffffffffu;

// ---- error reporting -------------------------------------------------------

int set_error(int status, const char* fmt, ...);
std::atomic<uint64_t>& launch_counter();
int gemm_tc_error_count(int* out);  // tensor-core GEMM wait limits hit
int skinny_error_count(int* out);   // skinny GEMM wait limits hit
int prefill_tc_error_count(int* out);  // tensor-core prefill attention wait limits hit

#define FML_CUDA_TRY(expr)                                                                     \
    do {                                                                                       \
        cudaError_t _e = (expr);                                                               \
        if (_e != cudaSuccess)                                                                 \
            return ::fml::set_error(FML_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,               \
                                    cudaGetErrorString(_e), __FILE__, __LINE__);               \
    } while (0)

// Checks the launch that was just issued and counts it.
#define FML_LAUNCH_CHECK()                                                                     \
    do {                                                                                       \
        cudaError_t _e = cudaGetLastError();                                                   \
        if (_e != cudaSuccess)                                                                 \
            return ::fml::set_error(FML_ERR_CUDA, "kernel launch failed: %s (%s:%d)",           \
                                    cudaGetErrorString(_e), __FILE__, __LINE__);               \
        ::fml::launch_counter().fetch_add(1, std::memory_order_relaxed);                       \
    } while (0)

#define FML_REQUIRE(cond, ...)                                                                 \
    do {                                                                                       \
        if (!(cond)) return ::fml::set_error(FML_ERR_INVALID, __VA_ARGS__);                    \
    } while (0)

#define FML_RC(expr)                   \
    do {                               \
        int _rc = (expr);              \
        if (_rc != FML_OK) return _rc; \
    } while (0)

inline cudaStream_t as_stream(fml_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline unsigned grid_for(uint64_t n, unsigned block, unsigned cap = 148u * 32u)
{
    uint64_t g = (n + block - 1) / block;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (unsigned)g;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A kernel's dynamic shared-memory limit (cudaFuncSetAttribute) holds for the
// device it was set on: raise it once per device a launcher runs on (bit
// `device` of `done`; devices past 63 set it on every call).
inline int smem_limit_once(const void* func, int bytes, uint64_t& done)
{
    int dev = 0;
    FML_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
    if (bit && (done & bit)) return FML_OK;
    FML_CUDA_TRY(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done |= bit;
    return FML_OK;
}

// ---- device helpers --------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, o));
    return v;
}

// Programmatic dependent launch (sm_90+): let the next kernel in the stream
// start its prologue now / wait until the previous kernel's writes are
// visible.  Both are no-ops when the launch did not opt in.
__device__ __forceinline__ void griddep_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- in-graph completion stamps of the decode step's kernels ------------
// When `buf` is set, thread 0 of every CTA of a step kernel raises
// buf[*step * stride + idx] to the global timer (ns) as the CTA exits, so the
// slot ends up holding the time the kernel's last CTA finished.  `step` is a
// device counter the step's last kernel advances; the host reads the slots of
// a replayed pass and takes differences of consecutive kernels' completions
// (the time each kernel adds to the step's dependent chain).  Off (null) in
// timed runs.
struct StepStamp
{
    unsigned long long* buf;
    const uint32_t* step;
    uint32_t stride, idx, cap;
};

__device__ __forceinline__ void stamp_write(const StepStamp& s)
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const uint32_t slot = *s.step * s.stride + s.idx;
    if (slot < s.cap) atomicMax(s.buf + slot, t);
}

// Writes the CTA's stamp when the kernel returns (any return path).
struct StampAtExit
{
    const StepStamp& s;
    __device__ explicit StampAtExit(const StepStamp& st) : s(st) {}
    __device__ ~StampAtExit()
    {
        if (s.buf && threadIdx.x == 0) stamp_write(s);
    }
};

// ---- optional per-CTA timeline (debug builds with -DFML_TIMELINE only) ----
// Thread 0 of every CTA appends (kernel id, start, end) global-timer stamps
// to a device ring that the host reads back; compiled out otherwise.
#ifdef FML_TIMELINE
struct TimelineRec
{
    unsigned long long start, mark1, mark2, end;  // marks: 0 when not set
    uint32_t kernel, cta;
};
// one ring per translation unit (device variables are not shared across
// units without relocatable device code); the host binds each to its own
// part of the caller's buffer
static __device__ TimelineRec* g_fml_timeline = nullptr;
static __device__ uint32_t g_fml_timeline_cap = 0;
static __device__ uint32_t g_fml_timeline_n = 0;
static inline int timeline_bind_unit(TimelineRec* p, uint32_t cap)
{
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(g_fml_timeline, &p, sizeof(p)) != cudaSuccess) return 2;
    if (cudaMemcpyToSymbol(g_fml_timeline_cap, &cap, sizeof(cap)) != cudaSuccess) return 2;
    if (cudaMemcpyToSymbol(g_fml_timeline_n, &zero, sizeof(zero)) != cudaSuccess) return 2;
    return 0;
}
int timeline_bind_attention(TimelineRec* p, uint32_t cap);
__device__ __forceinline__ unsigned long long fml_globaltimer()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
struct TimelineScope
{
    unsigned long long t0, t1 = 0, t2 = 0;
    uint32_t id;
    __device__ explicit TimelineScope(uint32_t k) : t0(fml_globaltimer()), id(k) {}
    __device__ void mark(int i) { (i == 1 ? t1 : t2) = fml_globaltimer(); }
    __device__ ~TimelineScope()
    {
        if (threadIdx.x == 0 && threadIdx.y == 0 && g_fml_timeline)
        {
            const uint32_t i = atomicAdd(&g_fml_timeline_n, 1u);
            if (i < g_fml_timeline_cap)
                g_fml_timeline[i] = {t0, t1, t2, fml_globaltimer(), id,
                                     blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)};
        }
    }
};
#define FML_TIMELINE_SCOPE(k) ::fml::TimelineScope _fml_tl_scope(k)
// stamp 1 (typically: past griddepcontrol.wait) or 2 (prologue done)
#define FML_TIMELINE_MARK(i) _fml_tl_scope.mark(i)
#else
#define FML_TIMELINE_SCOPE(k) \
    do {                      \
    } while (0)
#define FML_TIMELINE_MARK(i) \
    do {                     \
    } while (0)
#endif

// GeluMat's formula (MatrixBase_Functions.h:989-1000): 0.5 x (1 + erf(x / sqrt 2)).
__device__ __forceinline__ float gelu_exact(float x)
{
    return 0.5f * x * (1.0f + erff(x / 1.41421356237309515f));
}

// Orders floats as unsigned ints (larger float -> larger key).
__device__ __forceinline__ uint32_t float_order_key(float f)
{
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 64-bit argmax key: value in the high word, (~index) in the low word, so an
// unsigned max picks the largest value and, among equal values, the smallest
// index -- the reference's strict '>' scan (NanoLLM.cpp:194-201).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx)
{
    return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xffffffffu - idx);
}

__host__ __device__ __forceinline__ uint32_t argmax_key_index(unsigned long long key)
{
    return 0xffffffffu - (uint32_t)(key & 0xffffffffull);
}

// Sum-reduction of C values per lane across a warp without replicating the
// work: each step exchanges half of the lane's values with the partner lane,
// so after log2(min(C,32)) steps lane L holds C/32 complete sums (or one sum,
// replicated over the low lanes, when C < 32).  The value a[i] that lane L
// ends with is the sum of the original index i + reduce_base<C>(L).
template <int C>
__device__ __forceinline__ void warp_transpose_reduce(float (&a)[C], int lane)
{
    constexpr int HALV = C >= 32 ? 5 : (C >= 16 ? 4 : (C >= 8 ? 3 : (C >= 4 ? 2 : (C >= 2 ? 1 : 0))));
#pragma unroll
    for (int s = 0; s < HALV; ++s)
    {
        const int o = 16 >> s;
        const int n = C >> (s + 1);
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n; ++i)
        {
            const float send = up ? a[i] : a[i + n];
            const float keep = up ? a[i + n] : a[i];
            a[i] = keep + __shfl_xor_sync(FULL_MASK, send, o);
        }
    }
#pragma unroll
    for (int s = HALV; s < 5; ++s)
    {
        const int o = 16 >> s;
        a[0] += __shfl_xor_sync(FULL_MASK, a[0], o);
    }
}

template <int C>
__device__ __forceinline__ int reduce_base(int lane)
{
    constexpr int HALV = C >= 32 ? 5 : (C >= 16 ? 4 : (C >= 8 ? 3 : (C >= 4 ? 2 : (C >= 2 ? 1 : 0))));
    int base = 0;
#pragma unroll
    for (int s = 0; s < HALV; ++s)
        if (lane & (16 >> s)) base += C >> (s + 1);
    return base;
}

// True for the one lane of each replica group that should publish its sums.
template <int C>
__device__ __forceinline__ bool reduce_owner(int lane)
{
    constexpr int HALV = C >= 32 ? 5 : (C >= 16 ? 4 : (C >= 8 ? 3 : (C >= 4 ? 2 : (C >= 2 ? 1 : 0))));
    return (lane & ((1 << (5 - HALV)) - 1)) == 0;
}

}  // namespace fml
