/*
 * freeml_cuda.h -- C ABI of the B200 (sm_100a) backend for FreeML's
 * language-model token loop.
 *
 * Two groups of entry points:
 *
 *  1. Operator entry points.  One per generic operator that the NanoLLM
 *     forward reaches (MatrixLibrary/MatrixBase_Functions.h,
 *     MatrixLibrary/MatrixBase_Mul.h).  The MatrixCUDA<float> overloads in
 *     include/freeml_b200/MatrixCUDA_Functions.h call these, the same way the
 *     DirectX11 backend's overloads (MatrixLibrary/GPU/DirectX11/
 *     MatrixDX11_Functions.h) dispatch shaders.  Each comment names the
 *     reference function it replaces.
 *
 *  2. The decode engine (fml_lm_*): a KV-cached, batched greedy token loop for
 *     the NanoLLM graph (Examples/NanoLLM/NanoLLM.cpp:268-358) -- prefill, then
 *     one fused step per generated token for B independent sequences.  The
 *     reference has no decode loop; the engine produces the logits that
 *     Model::Run (ModelLibrary/Model.h:764-788) would give for the same
 *     window, row by row, and the argmax of NanoLLM.cpp:189-204.
 *
 * Conventions (the reference has none -- it asserts or returns silently):
 *  - every function returns an int status, FML_OK (0) on success;
 *    fml_last_error() gives a message for the calling thread;
 *  - pointers are device pointers unless the name says host;
 *  - matrices are row-major fp32, FreeML's Dims3D{x = cols, y = rows};
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream);
 *  - allocation (fml_device_alloc aside, the allocator that MatrixCUDA
 *    uses): operator entry points allocate nothing (fml_attention_decode
 *    takes a caller workspace; fml_attention_decode_noalloc needs none);
 *    the engine
 *    allocates in fml_lm_create, fml_lm_bind_weights / fml_lm_bind_packed
 *    (a transient staging buffer), fml_lm_set_tensor_parallel /
 *    fml_lm_tp_connect, and at its first TF32x3 prefill after a bind (the
 *    weights' TF32 lo parts, left out when memory is short);
 *  - the engine's device must be current for every call on it
 *    (fml_lm_create leaves it current) and `stream` must belong to it;
 *  - callers are single-threaded per device, like MatrixManager
 *    (MatrixLibrary/MatrixManager.h:131-135).
 */
#ifndef FREEML_CUDA_H
#define FREEML_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FML_API __attribute__((visibility("default")))
#else
#define FML_API
#endif

typedef void* fml_stream_t; /* cudaStream_t */

enum fml_status
{
    FML_OK = 0,
    FML_ERR_INVALID = 1,     /* bad shape, null pointer, unsupported argument */
    FML_ERR_CUDA = 2,        /* a CUDA runtime call failed */
    FML_ERR_NOMEM = 3,       /* device allocation failed */
    FML_ERR_UNSUPPORTED = 4, /* shape outside what the kernels handle */
    FML_ERR_STATE = 5        /* engine used out of order */
};

/* Recorded launch plans: fml_capture_begin creates a stream and starts
 * capturing it (CUDA stream capture, relaxed mode); every entry point then
 * given that stream records its kernels instead of running them, in call
 * order.  fml_capture_end stops, instantiates the record as one CUDA graph
 * and releases the stream; fml_graph_launch replays it on `stream` (kernel
 * launch counts include the replayed kernels).  For host runtimes that issue
 * the same operator calls every step (FreeML's Model::Run over MatrixCUDA:
 * freeml_cuda::RunGraph in include/freeml_b200/MatrixCUDA_Functions.h). */
typedef struct fml_graph fml_graph;
FML_API int fml_capture_begin(fml_stream_t* stream_out);
FML_API int fml_capture_end(fml_stream_t stream, fml_graph** graph_out);
FML_API int fml_graph_launch(fml_graph* graph, fml_stream_t stream);
FML_API int fml_graph_destroy(fml_graph* graph);

/* Library / device information. */
FML_API const char* fml_last_error(void);
FML_API const char* fml_version(void);
FML_API int fml_device_check(int* sm_count, int* cc_major, int* cc_minor);
/* Device-side waits that hit their iteration limit since the library loaded
 * (every wait in these kernels is bounded; a non-zero count means a kernel
 * gave up and its output is invalid).  Synchronises the device. */
FML_API int fml_device_error_count(uint64_t* count);
/* Number of kernels this library has launched in this process (all entry
 * points, graph replays counted per kernel node). */
FML_API uint64_t fml_kernel_launch_count(void);

/* Device memory for host bindings (the MatrixCUDA<float> storage of
 * include/freeml_b200/MatrixCUDA.h): allocation, release, and synchronous
 * copies (the copy to the host waits for all prior work on the device). */
FML_API int fml_device_alloc(void** ptr, size_t bytes);
FML_API int fml_device_free(void* ptr);
FML_API int fml_memcpy_to_device(void* dst, const void* src, size_t bytes);
FML_API int fml_memcpy_to_host(void* dst, const void* src, size_t bytes);
FML_API int fml_synchronize(void);

/* ---------------------------------------------------------------------
 * 1. Operator entry points
 * ------------------------------------------------------------------- */

/* GatherRows(out, src, idx)  MatrixBase_Functions.h:203-242
 * out[r, :] = src[(uint32)idx[r], :]; idx holds float token ids (one per row).
 * The reference asserts ids < src_rows; here a row whose id is out of range
 * is written as zeros (the kernel never reads outside src). */
FML_API int fml_gather_rows(float* out, const float* src, const float* idx, uint32_t rows, uint32_t width,
                    uint32_t src_rows, fml_stream_t stream);

/* Add(out, L, R)  MatrixBase_Functions.h:471-479 (out may alias L or R). */
FML_API int fml_add(float* out, const float* a, const float* b, uint64_t n, fml_stream_t stream);

/* BroadcastAdd(out, L, R)  MatrixBase_Functions.h:717-731: out[i] = L[i] + R[i % cols]. */
FML_API int fml_broadcast_add(float* out, const float* a, const float* row, uint64_t n, uint32_t cols,
                      fml_stream_t stream);

/* PerElementMul(out, L, R)  MatrixBase_Functions.h:848-855. */
FML_API int fml_mul_elementwise(float* out, const float* a, const float* b, uint64_t n, fml_stream_t stream);

/* Scale(out, in, float)  MatrixBase_Functions.h:1032-1039 and
 * Scale(out, in, Mat*)  :1021-1030 (scale_dev != NULL: scale read on device). */
FML_API int fml_scale(float* out, const float* in, float scale, const float* scale_dev, uint64_t n,
              fml_stream_t stream);

/* ScaleAdd(out, in, Mat* scale, add)  MatrixBase_Functions.h:1056-1070:
 * out = in * scale[0] + add (fused multiply-add, as the reference build). */
FML_API int fml_scale_add(float* out, const float* in, const float* scale_dev, const float* add, uint64_t n,
                  fml_stream_t stream);

/* Fill(out, float) :1079-1086, Fill(out, Mat*) :1088-1096 (value_dev != NULL),
 * Clear(out) :1073-1077 (value 0). */
FML_API int fml_fill(float* out, float value, const float* value_dev, uint64_t n, fml_stream_t stream);

/* Copy(out, in) :157-162 and CopyRange(out, in, outOff, inOff, n) :164-181. */
FML_API int fml_copy(float* out, const float* in, uint64_t n, fml_stream_t stream);

/* LayerNormOp(out, in, gamma, beta, xHat, eps)  MatrixBase_Functions.h:482-549.
 * beta and xhat may be NULL. */
FML_API int fml_layernorm(float* out, const float* in, const float* gamma, const float* beta, float* xhat,
                  uint32_t rows, uint32_t cols, float eps, fml_stream_t stream);

/* GeluMat(out, in)  MatrixBase_Functions.h:989-1000 (exact erf). */
FML_API int fml_gelu(float* out, const float* in, uint64_t n, fml_stream_t stream);

/* Softmax(out, in)  MatrixBase_Functions.h:50-80 (row-wise). */
FML_API int fml_softmax(float* out, const float* in, uint32_t rows, uint32_t cols, fml_stream_t stream);

/* SplitQKV(q, k, v, packed)  MatrixBase_Functions.h:330-367. */
FML_API int fml_split_qkv(float* q, float* k, float* v, const float* packed, uint32_t rows, uint32_t d,
                  fml_stream_t stream);

/* Mul<Mode>(out, L, R)  MatrixBase_Mul.h:591-615 for Mode in {None, Right}:
 *   trans_b == 0: out[M x N] = L[M x K] . R[K x N]
 *   trans_b == 1: out[M x N] = L[M x K] . R[N x K]^T
 * Above 16 rows in the TF32 math modes: tcgen05 tensor cores (R read in its
 * stored layout, K-major for Right, N-major for None).  At most 16 rows (64
 * in FML_MATH_FP32): memory-bound fp32 CUDA-core kernels, the small-batch
 * Mul<None> one launch with no scratch memory.  Otherwise the fp32 CUDA-core
 * GEMM.  Precision follows fml_set_math_mode(). */
FML_API int fml_matmul(float* out, const float* a, const float* b, uint32_t M, uint32_t N, uint32_t K,
               int trans_b, fml_stream_t stream);

/* MatMul_Strided<Mode>(out, L, R, Lrs, 1, Rrs, 1, Ors, 1)  MatrixBase_Mul.h:617-722
 * (column strides of 1, the form CausalSelfAttentionLayer.h:445-497 uses),
 * for `batch` planes spaced by the plane strides (elements).  Above 64 rows
 * in the TF32 math modes: tcgen05 tensor cores, one launch per plane (the
 * row strides and plane offsets must keep every row 16-byte aligned, else
 * the CUDA-core kernel runs). */
FML_API int fml_matmul_strided(float* out, const float* a, const float* b, uint32_t M, uint32_t N, uint32_t K,
                       uint32_t lda, uint32_t ldb, uint32_t ldc, int trans_b, uint32_t batch,
                       uint64_t plane_a, uint64_t plane_b, uint64_t plane_c, fml_stream_t stream);

/* ---- Training (Model::Run(input, target), ModelLibrary/Model.h:785-840) ----
 * Mul<Left>(out, L, R) and MatMul_Strided<Left> with column strides of 1
 * (MatrixBase_Mul.h:478-589, 617-722): out[M x N] = L^T . R with L [K x M]
 * (row stride lda) and R [K x N] (row stride ldb), `batch` planes. */
FML_API int fml_matmul_left(float* out, const float* a, const float* b, uint32_t M, uint32_t N, uint32_t K,
                    uint32_t lda, uint32_t ldb, uint32_t ldc, uint32_t batch, uint64_t plane_a, uint64_t plane_b,
                    uint64_t plane_c, fml_stream_t stream);
/* MergeQKV(packed, qHeads, kHeads, vHeads)  MatrixBase_Functions.h:369-431:
 * per-head [heads][tokens][head_dim] back into [tokens][3 * heads * head_dim] */
FML_API int fml_merge_qkv(float* packed, const float* q, const float* k, const float* v, uint32_t head_dim,
                  uint32_t tokens, uint32_t heads, fml_stream_t stream);
/* GeluDerivtiveMat  MatrixBase_Functions.h:1003-1018 */
FML_API int fml_gelu_derivative(float* out, const float* in, uint64_t n, fml_stream_t stream);
/* SoftmaxBackwards(out, softmaxOut, gradIn)  MatrixBase_Functions.h:82-111 (row-wise) */
FML_API int fml_softmax_backward(float* out, const float* y, const float* g, uint32_t rows, uint32_t cols,
                         fml_stream_t stream);
/* ScatterAddRows(out, src, indices)  MatrixBase_Functions.h:285-320: out row
 * indices[r] += src row r for `planes` planes of src_rows rows; out has 1 or
 * `planes` planes of out_rows rows; indices are token ids stored as floats;
 * rows are added with atomics (the sum order is not the reference's). */
FML_API int fml_scatter_add_rows(float* out, const float* src, const float* indices, uint32_t src_rows,
                         uint32_t width, uint32_t out_rows, uint32_t planes, uint32_t out_planes,
                         fml_stream_t stream);
/* LayerNormBackwardsOp(dX, dY, in, gamma, dGamma, dBeta, xHat, eps)
 * MatrixBase_Functions.h:552-705 over rows x cols (dBeta, xHat optional);
 * without xHat, `workspace` holds 2 floats per row. */
FML_API int fml_layernorm_backward(float* dx, const float* dy, const float* in, const float* gamma, float* dgamma,
                           float* dbeta, const float* xhat, uint32_t rows, uint32_t cols, float eps,
                           void* workspace, fml_stream_t stream);
/* AdamWUpdate  MatrixBase_Functions.h:1498-1545 (param += update - decay) */
FML_API int fml_adamw_update(float* param, const float* grad, float* mt, float* vt, uint64_t n, float lr,
                     float beta1, float beta2, float beta1_pow_t, float beta2_pow_t, float eps,
                     float weight_decay, fml_stream_t stream);
/* CategoricalCrossEntropyWithLogits  LossLibrary/CategoricalCrossEntropyWithLogits.h:
 * 29-217 over `planes` x `steps` rows of `vocab` logits: the negative
 * gradient into `grad` and, when loss_out is not null, the loss into
 * *loss_out (host; synchronises the stream; `workspace` = rows + 1 floats).
 * target_ids = 1: target [target_planes][steps] token ids as floats (-1
 * ignored; gradient scaled by 1 / valid rows, loss = mean); 0: dense target
 * rows [target_planes][steps][vocab] (loss = sum). */
FML_API int fml_xent_with_logits(float* grad, float* loss_out, const float* target, const float* logits,
                         uint32_t vocab, uint32_t steps, uint32_t planes, uint32_t target_planes, int target_ids,
                         void* workspace, fml_stream_t stream);

/* Causal attention of one query row per sequence over a KV cache -- the
 * attention core of CausalSelfAttentionLayer::Forward
 * (LayerLibrary/CausalSelfAttentionLayer.h:424-499: MatMul_Strided<Right>
 * scores, ScaleAdd with the causal mask, Softmax, MatMul_Strided<None>) for
 * the newest row, where the mask leaves keys 0..len-1:
 *   q      [batch x heads*head_dim]
 *   kcache, vcache [batch][heads][context][head_dim]
 *   lens   [batch] (device): keys 0 .. lens[b]-1 attend (0 gives zeros)
 *   out    [batch x heads*head_dim]
 *   scale  1/sqrt(head_dim) in the reference ("ScalarScale", :73-77)
 * The key range is split across CTAs; `workspace` (device, at least
 * fml_attention_workspace_bytes(batch, heads, head_dim, context) bytes) holds
 * the per-split partial results. */
FML_API size_t fml_attention_workspace_bytes(uint32_t batch, uint32_t heads, uint32_t head_dim, uint32_t context);
FML_API int fml_attention_decode(float* out, const float* q, const float* kcache, const float* vcache,
                                 const uint32_t* lens, uint32_t batch, uint32_t heads, uint32_t head_dim,
                                 uint32_t context, float scale, void* workspace, size_t workspace_bytes,
                                 fml_stream_t stream);

/* fml_attention_decode without a workspace argument: it allocates nothing.
 * No counterpart in the reference (FreeML's CPU path never needs scratch
 * device memory).  It is for callers that may not allocate device memory --
 * a host runtime that owns the GPU's memory through its own pool and forbids
 * libraries to call cudaMalloc, or code running inside that pool's
 * out-of-memory handling.  The split partials live in a fixed
 * FML_NOALLOC_SCRATCH_BYTES array inside this library's device image, held by
 * every GPU that loads the library until the process exits.  Shapes whose
 * scratch would exceed it are rejected with FML_ERR_UNSUPPORTED (use
 * fml_attention_decode instead).  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress), so make that first call
 * outside any stream capture; after a device reset the next call looks it up
 * again (the address is cached per device and CUDA context).  Every call
 * shares the one array: calls that
 * overlap on the GPU (different streams, or different host threads on the same
 * device) race and must be serialised by the caller.  Same arguments and
 * results as fml_attention_decode otherwise. */
#define FML_NOALLOC_SCRATCH_BYTES (4u << 20)
FML_API int fml_attention_decode_noalloc(float* out, const float* q, const float* kcache, const float* vcache,
                                         const uint32_t* lens, uint32_t batch, uint32_t heads, uint32_t head_dim,
                                         uint32_t context, float scale, fml_stream_t stream);

/* Precision of fml_matmul / fml_matmul_strided (the drop-in's Mul and
 * MatMul_Strided) above 64 rows:
 *   FML_MATH_FP32  -- fp32 FFMA on the CUDA cores;
 *   FML_MATH_TF32X3 -- tcgen05 tensor cores, each fp32 operand split into a
 *                     TF32 pair and three products accumulated in fp32
 *                     (default: fp32-level accuracy, the logits bound of
 *                     1e-3 abs/rel against the reference holds);
 *   FML_MATH_TF32  -- tcgen05 tensor cores, one TF32 product (looser bound). */
enum fml_math_mode { FML_MATH_FP32 = 0, FML_MATH_TF32X3 = 1, FML_MATH_TF32 = 2 };
FML_API int fml_set_math_mode(int mode);
FML_API int fml_get_math_mode(void);

/* Causal attention over whole prompts -- the attention core of
 * CausalSelfAttentionLayer::Forward (LayerLibrary/CausalSelfAttentionLayer.h:
 * 424-499) for every row of a prompt, as the engine's prefill runs it:
 *   q, out [batch*prompt_len x heads*head_dim] (row b*prompt_len + t)
 *   kcache, vcache [batch][heads][context][head_dim], rows 0..prompt_len-1
 *          of each (sequence, head) filled; rows past them may hold anything
 *   row t attends keys 0..t; scale 1/sqrt(head_dim) in the reference
 * mode: FML_MATH_FP32 (CUDA cores), FML_MATH_TF32X3 (tcgen05 tensor cores,
 * fp32-level accuracy) or FML_MATH_TF32.  head_dim 32, 64 or 128;
 * prompt_len <= context.  Allocates nothing. */
FML_API int fml_attention_prefill(float* out, const float* q, const float* kcache, const float* vcache,
                                  uint32_t batch, uint32_t heads, uint32_t head_dim, uint32_t context,
                                  uint32_t prompt_len, float scale, int mode, fml_stream_t stream);

/* ---------------------------------------------------------------------
 * 2. Decode engine
 * ------------------------------------------------------------------- */

typedef struct fml_lm fml_lm;

typedef struct
{
    uint32_t vocab;      /* V: token table rows, lm_head columns */
    uint32_t context;    /* C: block_size, position table rows, max window */
    uint32_t d_model;    /* d */
    uint32_t n_head;     /* H (d % H == 0, head dim 32/64/128) */
    uint32_t n_layer;    /* L */
    uint32_t max_batch;  /* sequences held by this engine (KV-cache slots) */
} fml_lm_config;

/* Parameters in FreeML's storage layouts (device pointers, fp32):
 *   tok_emb   [V x d]   Embedding_Weights of embedding_token (also lm_head, tied)
 *   pos_emb   [C x d]   Embedding_Weights of embedding_pos
 *   per layer l (arrays of n_layer pointers):
 *     ln0[l]  [d]       GammaScale of LayerNorm0Data
 *     wqkv[l] [d x 3d]  Dense_Weights of CSA_AttentionLayer (y = x W)
 *     wproj[l][d x d]   Dense_Weights of CSA_ProjLayer (transposed: y = x W^T)
 *     ln1[l]  [d]       GammaScale of LayerNorm1Data
 *     wfc[l]  [d x 4d]  Dense_Weights of DenseFCData
 *     wmlp[l] [4d x d]  Dense_Weights of DenseProjData
 *   lnf       [d]       GammaScale of ln_f
 * The engine copies them into its own K-contiguous layout at bind time, so
 * the caller's buffers may be freed or changed afterwards. */
typedef struct
{
    const float* tok_emb;
    const float* pos_emb;
    const float* const* ln0;
    const float* const* wqkv;
    const float* const* wproj;
    const float* const* ln1;
    const float* const* wfc;
    const float* const* wmlp;
    const float* lnf;
} fml_lm_weights;

FML_API int fml_lm_create(const fml_lm_config* cfg, int device, fml_lm** out);
FML_API int fml_lm_destroy(fml_lm* lm);
FML_API int fml_lm_bind_weights(fml_lm* lm, const fml_lm_weights* w, fml_stream_t stream);
/* Convenience: all parameters in one host or device buffer, in the canonical
 * order tok_emb, pos_emb, per layer {ln0, wqkv, wproj, ln1, wfc, wmlp}, lnf. */
FML_API int fml_lm_bind_packed(fml_lm* lm, const float* params, int params_on_host, fml_stream_t stream);
FML_API uint64_t fml_lm_param_count(const fml_lm_config* cfg);
FML_API int fml_lm_get_config(const fml_lm* lm, fml_lm_config* out);

/* FreeML checkpoints: the directory Model::Save writes for a NanoLLM model
 * (ModelLibrary/Model.h:91-159; model.guide, *.blob_layer, *.blob_matrix,
 * *.blob_data, Loading/SaveLoader.h:499-577, 1523-1563), read without
 * building FreeML's layer graph.  fml_checkpoint_config gives V, C, d, H, L
 * (max_batch 0) from the stored shapes; fml_checkpoint_pack reads every
 * parameter into a host buffer of fml_lm_param_count floats in the packed
 * order of fml_lm_bind_packed; fml_lm_load_checkpoint does both and binds
 * the weights (the engine's shape must match).  A checkpoint with bias
 * terms, an untied lm_head or another layer naming than NanoLLM's
 * (Examples/NanoLLM/NanoLLM.cpp:268-348) is rejected (FML_ERR_UNSUPPORTED /
 * FML_ERR_INVALID).  Host-only except the final bind. */
FML_API int fml_checkpoint_config(const char* dir, fml_lm_config* cfg_out);
FML_API int fml_checkpoint_pack(const char* dir, float* params_out, uint64_t count);
FML_API int fml_lm_load_checkpoint(fml_lm* lm, const char* dir, fml_stream_t stream);

/* Start `batch` sequences (batch <= max_batch) from prompts of `prompt_len`
 * tokens each (device, sequence-major [batch x prompt_len]).  Runs the
 * prompt through batched contractions, fills the KV cache, and leaves the
 * argmax of each sequence's last prompt row as its next token. */
FML_API int fml_lm_prefill(fml_lm* lm, const uint32_t* prompts, uint32_t batch, uint32_t prompt_len,
                   fml_stream_t stream);

/* Tensor parallelism over `world` GPUs (one process and one engine each),
 * for models too slow or too large for one GPU.  Call
 * on every rank after fml_lm_create and before binding weights, with the
 * same 128-byte NCCL id on all ranks (from fml_nccl_unique_id on one rank,
 * shared by the caller).  Rank r then keeps heads [r*H/w, (r+1)*H/w) of
 * QKV and attention (column-parallel) and the matching input columns of
 * the attention projection (row-parallel), fc columns [r*4d/w, ...) and the
 * matching mlp inputs, and vocabulary rows [r*ceil(V/w), ...) of the tied
 * lm_head; the row-parallel partial sums are all-reduced (ncclSum, in
 * place) and the argmax keys max-reduced, so every rank ends each step with
 * the same tokens.  Logits returned by fml_lm_step are this rank's
 * vocabulary slice [B x ceil(V/w)].  Weights are given whole to
 * fml_lm_bind_weights / fml_lm_bind_packed; each rank packs its share. */
#define FML_NCCL_ID_BYTES 128
FML_API int fml_nccl_unique_id(void* id_out);
FML_API int fml_lm_set_tensor_parallel(fml_lm* lm, int rank, int world, const void* nccl_id);

/* All-reduce over NVLink peer memory for the decode step's row-parallel
 * projections: after fml_lm_set_tensor_parallel, each rank exports
 * FML_TP_IPC_BYTES of CUDA IPC handles (its partial-sum buffer and flags);
 * the caller gathers them from all ranks in rank order (world *
 * FML_TP_IPC_BYTES) and gives them to fml_lm_tp_connect on every rank.  From
 * then on each proj / mlp GEMV writes its partial sums locally and a
 * one-shot kernel of 16 CTAs signals every rank, waits for every rank, reads
 * all ranks' partials over NVLink and adds them in rank order plus the
 * residual (no NCCL call on the decode path; prefill keeps NCCL).  Waits are
 * bounded (1 s); fml_lm_tp_error_count reports expirations. */
#define FML_TP_IPC_BYTES 128
FML_API int fml_lm_tp_ipc_handles(fml_lm* lm, void* out);
FML_API int fml_lm_tp_connect(fml_lm* lm, const void* all_handles);
FML_API int fml_lm_tp_error_count(uint64_t* count);

/* The flag test of that all-reduce, on the host: *reached = 1 when a flag
 * holding `flag` satisfies a waiter of use `slot` (of `nslot` per step, 2 per
 * layer) in step `epoch`.  Tags count up by one per use modulo 2^32 and the
 * test is wrap-safe.  A test hook: no counterpart in the reference. */
FML_API int fml_tp_flag_check(uint32_t epoch, uint32_t slot, uint32_t nslot, uint32_t flag, int* reached);

/* Precision of the prefill contractions (FML_MATH_*; default
 * FML_MATH_TF32X3: tcgen05 tensor cores at fp32-level accuracy).  Under
 * FML_MATH_TF32X3 with fp32 weights on one rank, the decode step's
 * contractions also run on tcgen05 from 32 rows when d_model is a multiple
 * of 1024, and the logits head from 32 rows when the vocabulary spans at
 * least 148 column tiles of 128; fewer rows stay on the CUDA-core GEMVs.
 * FML_MATH_FP32 keeps every contraction on CUDA cores; FML_MATH_TF32 runs
 * the prefill as one tf32 pass and the decode step on CUDA cores. */
FML_API int fml_lm_set_prefill_math(fml_lm* lm, int mode);


/* Storage of the weights the decode step streams.  FML_WEIGHTS_FP32 (the
 * default): the fp32 weights, as the reference holds them.  FML_WEIGHTS_BF16:
 * the decode GEMVs (QKV, projection, fc, mlp and the tied lm_head) read a
 * bf16 copy, rounded to nearest even, and accumulate in fp32 -- half the
 * weight bytes per step.  The copy is made after each bind, before the next
 * step (2 bytes per weight of extra device memory); the prefill, the
 * embedding gathers, LayerNorm gammas and the K/V cache stay fp32.  Logits
 * then differ from the fp32 reference by more than the fp32 bound (tests
 * state the bf16 bound).  No counterpart in the reference, which holds fp32
 * (PRECISION=float) weights only. */
enum fml_weight_format { FML_WEIGHTS_FP32 = 0, FML_WEIGHTS_BF16 = 1 };
FML_API int fml_lm_set_weight_format(fml_lm* lm, int format);

/* One decode step for every active sequence: consume each sequence's pending
 * token, append its K/V, and produce the next token (greedy).  Optional
 * outputs (device): next tokens [batch] and logits [batch x V] of the row
 * just computed.  All work is enqueued on `stream`; nothing synchronises. */
FML_API int fml_lm_step(fml_lm* lm, uint32_t* next_tokens, float* logits, fml_stream_t stream);

/* `n` decode steps for every active sequence, each token left pending on the
 * device for the next (read them with fml_lm_pending).  With graphs on, the
 * steps replay as graphs of several steps each (FML_LM_GRAPH_STEPS, default
 * 16): no launch gap between the steps a graph holds, and each step's first
 * kernel starts under programmatic dependent launch while the previous
 * step's last one finishes.  The decode loop of NanoLLM.cpp:189-204 run n
 * times (one Model::Run and argmax per token there).  Fails before any work
 * if a sequence would pass the context. */
FML_API int fml_lm_steps(fml_lm* lm, uint32_t n, fml_stream_t stream);

/* The same step through host memory, the way a host caller drives the loop:
 * `tokens_in` (host, [batch]) go to the device, the step runs, the next
 * tokens come back into `tokens_out` (host) and the call waits for them.
 * With graphs on, the step's first kernel reads the tokens from the engine's
 * pinned host buffer and its last kernel writes the next tokens there. */
FML_API int fml_lm_step_host(fml_lm* lm, const uint32_t* tokens_in, uint32_t* tokens_out, fml_stream_t stream);

/* `steps` host-buffer steps in one call (the harness Generate() loop over
 * Model::Run, NanoLLM.cpp:189-204 for the token decode): step 0 reads
 * `tokens_in` (host, [batch]); step t > 0 reads the tokens step t - 1 wrote
 * back to the host; step t writes its next tokens to
 * tokens_out[t * batch, (t + 1) * batch) (host).  Every step copies its
 * tokens up and its result down and waits for it, like fml_lm_step_host. */
FML_API int fml_lm_generate_host(fml_lm* lm, uint32_t steps, const uint32_t* tokens_in, uint32_t* tokens_out,
                                 fml_stream_t stream);

/* Replay the step as one CUDA graph (captured on first use; the step reads
 * positions and tokens from device memory, so one graph serves every step).
 * use_graph = 0 launches the kernels one by one. */
FML_API int fml_lm_set_graph(fml_lm* lm, int use_graph);

/* Copy the pending token of each active sequence (the greedy token it will
 * consume next; after prefill, the argmax of its last prompt row) into
 * `out` (device, [batch]). */
FML_API int fml_lm_pending(fml_lm* lm, uint32_t* out, fml_stream_t stream);

/* Position (tokens held in the cache) of sequence b, and rewinding every
 * active sequence to `pos` (cache rows [0, pos) are kept; pos must not pass
 * any sequence's position) with the given pending tokens ([batch], host or
 * device memory).  The device form is stream-ordered and does not
 * synchronise. */
FML_API int fml_lm_get_position(fml_lm* lm, uint32_t b, uint32_t* pos);
FML_API int fml_lm_rewind(fml_lm* lm, uint32_t pos, const uint32_t* pending, int pending_on_host,
                          fml_stream_t stream);

/* Per-step algorithmic HBM bytes (weights once + K/V read + K/V written) for
 * the current positions, the quantity the bench divides by step time. */
FML_API uint64_t fml_lm_step_bytes(fml_lm* lm);

/* Kernel timing: with profiling on (and graphs off), every step records CUDA
 * events around each kernel class and accumulates milliseconds and launch
 * counts per class: 0 embed, 1 layernorm, 2 qkv, 3 attention, 4 proj,
 * 5 fc, 6 mlp, 7 lm_head, 8 argmax/finalize, 9 the tensor-parallel
 * all-reduce kernel.  Reset when turned on.  Eager launches without
 * programmatic dependent launch: not the timed execution (see stamps). */
enum { FML_LM_NCLASS = 10 };
FML_API int fml_lm_set_profiling(fml_lm* lm, int on);
FML_API int fml_lm_get_profile(fml_lm* lm, double* ms_by_class, uint64_t* launches_by_class, int n_classes);

/* In-graph kernel timing of the decode step as it is timed (CUDA graph,
 * programmatic dependent launch).  With `stamps` set (device memory,
 * `cap` zeroed uint64 slots), the step is recorded again with every kernel's
 * CTAs raising slot [s * stride + i] to the global timer (ns) as they
 * finish, where s counts the steps since this call and i is the kernel's
 * index within the step; *stride receives the slots per step.  The time a
 * kernel adds to the step is its slot minus the previous kernel's.
 * fml_lm_stamp_classes gives the profile class (above) of each index of the
 * last recorded step and *kernels their number.  Null turns stamps off
 * (re-records without them).  No counterpart in the reference. */
FML_API int fml_lm_set_stamps(fml_lm* lm, unsigned long long* stamps, uint32_t cap, uint32_t* stride);
FML_API int fml_lm_stamp_classes(fml_lm* lm, int* classes, uint32_t n, uint32_t* kernels);
/* Algorithmic bytes of the attention kernels of one step (K/V rows read,
 * queries read, outputs written), for the attention roofline. */
FML_API uint64_t fml_lm_attention_bytes(fml_lm* lm);

#ifdef __cplusplus
}
#endif
#endif /* FREEML_CUDA_H */
