// Decode contractions on the tensor cores (gemv_tcgen05.cu): the decode
// engine's y = LN(x) . W^T for B <= 64 rows with its fused epilogues.
#pragma once

#include "fml_common.cuh"

namespace fml {

enum GemvTcEpi { GTC_STORE = 0, GTC_GELU = 1, GTC_RESID = 2, GTC_QKV = 3, GTC_ARGMAX = 4 };

struct GemvTcArgs
{
    const float* x;  // [M x K] rows (the sequences), row stride ldx
    uint32_t ldx;
    const float* w;  // [N x K], K-contiguous
    uint32_t M, N, K;
    int epi;         // GemvTcEpi
    bool ln;         // LayerNormOp of every x row with gamma first (QKV, GELU, ARGMAX)
    const float* gamma;
    float* y;        // [M x N], row stride ldy (STORE, GELU, RESID; ARGMAX: optional logits)
    uint32_t ldy;
    const float* r;  // RESID: y = r + x.W^T, row stride ldr
    uint32_t ldr;
    // QKV: columns [0, d) -> q[m*d + n], [d, 2d) -> K cache, [2d, 3d) -> V cache
    float* q;
    float* kc;
    float* vc;
    const uint32_t* pos;
    uint32_t d, hd, C;
    uint64_t seq_stride;
    // ARGMAX: packed (value, ~index) keys, max-reduced per row
    unsigned long long* keys;
    uint32_t n_off;
    StepStamp stamp;  // optional completion stamp (fml_common.cuh)
    uint32_t kb;     // set by the launcher: 32-wide K blocks per CTA
};

// True when the tensor-core kernel takes this shape (M <= 64, K a multiple of
// 32 with at most 16 splits of <= 128, N a multiple of 4, aligned operands);
// FML_GEMV_TC=0 turns it off.
bool gemv_tc_supported(const GemvTcArgs& a);
int launch_gemv_tc(const GemvTcArgs& a, cudaStream_t st, bool pdl);
int gemv_tc_error_count(int* out);

}  // namespace fml
