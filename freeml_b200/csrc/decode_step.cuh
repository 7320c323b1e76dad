// The fused decode step: one persistent kernel per generated token.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace fml {

// Phase types of one step, in layer order.  A step is
//   L x { QKV, ATT, PROJ, FC, MLP } then HEAD,
// each phase repeated once per token group.
enum StepPhase : uint32_t { SP_QKV = 0, SP_ATT = 1, SP_PROJ = 2, SP_FC = 3, SP_MLP = 4, SP_HEAD = 5 };

struct StepArgs
{
    // packed parameters, the engine's layout:
    //   tok [V x d], pos [C x d], L x {ln0 [d], wqkv [3d x d], wproj [d x d],
    //   ln1 [d], wfc [4d x d], wmlp [d x 4d]}, lnf [d]   (weights K-contiguous)
    const float* wbuf;
    float* kc;  // [L][B][H][C][hd]
    float* vc;
    uint64_t layer_stride, seq_stride;
    float *x, *buf, *q, *att, *hid;  // activations, [B x d] ([B x 4d] for hid)
    uint32_t* pending;               // token each sequence consumes this step
    uint32_t* pos;                   // rows held per sequence (the new row's index)
    uint32_t* next_out;              // optional copy of the step's tokens
    unsigned long long* keys;        // packed argmax per sequence (zero between steps)
    float* logits;                   // optional [B x V]
    uint32_t* sync;                  // [0] exit count, [1] abort flag, [2 + p] items done in phase p

    uint32_t B, V, C, d, H, hd, L;
    uint32_t ng, bg;      // token groups, tokens per group (the last group may hold fewer)
    uint32_t rows[6];     // weight rows per work item, per phase type (ATT: unused)
    uint32_t items[6];    // work items per phase and group (ATT: computed from the group's tokens)
    uint32_t kch;         // keys per attention ring entry
    uint32_t nslot, slot; // ring entries per CTA and bytes per entry
    uint32_t tpw;         // tokens per lane in the weight contractions (1, 2 or 4)
    uint32_t xpad4;       // staged-activation row padding, in float4
    uint32_t red_floats;  // reduction scratch
    uint32_t xs_floats;   // staged activations
    uint32_t gam_floats;  // LayerNorm gammas in shared memory
    uint32_t gam_all;     // 1: all (2L + 1) gammas resident; 0: one, staged per phase
    uint32_t mlp_segs;    // the mlp input (4d per token) is staged in this many K segments
    float scale;          // 1 / sqrt(hd)
};

// Number of sync words the step needs (zero them once; the kernel leaves
// them zero after every step).
uint32_t decode_step_sync_words(uint32_t L, uint32_t ng);

// Fills the geometry of `a` (its sizes and pointers already set) for this
// device; returns FML_ERR_UNSUPPORTED with a reason when the shape does not
// fit the fused kernel (the caller then runs the per-op kernels).
int decode_step_plan(StepArgs& a, int device, int* grid, size_t* smem);

int launch_decode_step(const StepArgs& a, int grid, size_t smem, cudaStream_t st);

// Waits in the fused step that ran out (each sets the abort flag).
int decode_step_error_count(int* out);

}  // namespace fml
