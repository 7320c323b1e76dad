// Causal decode attention over a KV cache (shared by the decode engine and
// the fml_attention_decode operator entry point).
#pragma once

#include "fml_common.cuh"

namespace fml {

struct AttnArgs
{
    const float* q;  // row r, head h at q + r*ldq + h*HD
    uint32_t ldq;
    uint32_t row0;   // first row of this launch
    uint32_t rows;   // rows of this launch (set by the launcher)
    const float* kc;
    const float* vc;
    uint64_t seq_stride;  // H*C*HD
    uint32_t H, C;
    float* out;      // row r, head h at out + r*ldo + h*HD
    uint32_t ldo;
    const uint32_t* pos;  // decode: b = r, t = pos[r]; prefill (null): b = r / P, t = r % P
    const uint32_t* lens; // operator form: b = r, keys 0..lens[r]-1 (overrides pos / P)
    uint32_t P;
    uint32_t S, chunk;    // splits over the key range; keys per split (0: ceil(len / S) rounded up to 32)
    float scale;          // 1/sqrt(hd), CausalSelfAttentionLayer.h:73-77
    float* part;          // [B][H][S][HD + 2] split partials
    uint32_t* counters;   // [B][H] split-merge counters (zero between launches)
    uint32_t* grab;       // work-unit counter (zero before each launch)
    StepStamp stamp;      // optional completion stamp (decode engine)
};

void attention_splits(uint64_t pairs, uint64_t ctx, uint32_t* S_out, uint32_t* chunk_out);
uint64_t attention_workspace_bytes(uint32_t B, uint32_t H, uint32_t hd, uint32_t S);

// Launches attention_kernel<hd> on `grid` = (heads, rows, splits).
int launch_attention_kernel(const AttnArgs& a, uint32_t hd, dim3 grid, cudaStream_t st, bool pdl = false);

}  // namespace fml
