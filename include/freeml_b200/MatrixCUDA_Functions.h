// FreeML operator overloads for MatrixCUDA<T>: the sm_100a kernels of
// libfreeml_cuda.so behind the names the layers call.  Include after the
// FreeML headers (and MatrixCUDA.h); argument-dependent lookup at template
// instantiation then picks these over the MatrixBase<T>* templates of
// MatrixLibrary/MatrixBase_Functions.h and MatrixBase_Mul.h -- the same
// mechanism as MatrixLibrary/GPU/DirectX11/MatrixDX11_Functions.h.
//
// Every operator the NanoLLM forward and training iteration (backward,
// CategoricalCrossEntropyWithLogits, AdamW) reach runs on the device.
// Other forms (Mul<Both>, MatMul_Strided with column strides other than 1)
// run FreeML's own host templates through the host mirror; MatrixCUDA counts
// those transfers so a test can assert that Model::Run performed none.
#pragma once

#include <algorithm>
#include <cmath>
#include <vector>

#include <MatrixLibrary/MatrixBase_Functions.h>
#include <MatrixLibrary/MatrixBase_Mul.h>
#include <LossLibrary/CategoricalCrossEntropyWithLogits.h>
#include <OptimiserLibrary/AdamWOptimiser.h>

#include "../freeml_cuda.h"
#include "MatrixCUDA.h"

namespace freeml_cuda {
// The stream the operators are issued on: the legacy default stream (ops run
// in call order), or the capture stream while a RunGraph records.
inline fml_stream_t& StreamSlot()
{
    static fml_stream_t s = nullptr;
    return s;
}
inline fml_stream_t Stream() { return StreamSlot(); }
}  // namespace freeml_cuda

#define FML_CALL(expr) ::freeml_cuda::Check((expr), #expr)

namespace freeml_cuda {

// A pre-resolved launch plan for a host runtime that repeats the same
// operator calls every step, such as Model::Run over a fixed window
// (ModelLibrary/Model.h:764-788: string-keyed blob lookups, view set-up and
// one C-ABI call per operator).  Record(f) calls f() once with every
// operator captured into a CUDA graph -- nothing executes then; Replay()
// uploads pending host writes of the buffers the recorded calls read (the
// token window written through DataWrite()), launches the graph in call
// order on the legacy default stream and marks the host mirrors of the
// buffers they wrote stale.  The recorded calls must not touch the host
// mirror (Model::Run does not once its inputs are flushed) and every buffer
// they use must stay allocated while the RunGraph lives.
class RunGraph
{
public:
    RunGraph() = default;
    RunGraph(const RunGraph&) = delete;
    RunGraph& operator=(const RunGraph&) = delete;
    ~RunGraph()
    {
        if (m_graph) fml_graph_destroy(m_graph);
    }

    template <class F>
    void Record(F&& f)
    {
        if (m_graph)
        {
            fml_graph_destroy(m_graph);
            m_graph = nullptr;
        }
        Recording rec;
        fml_stream_t s = nullptr;
        FML_CALL(fml_capture_begin(&s));
        StreamSlot() = s;
        ActiveRecording() = &rec;
        f();
        ActiveRecording() = nullptr;
        StreamSlot() = nullptr;
        FML_CALL(fml_capture_end(s, &m_graph));
        m_read = Unique(rec.read);
        m_written = Unique(rec.written);
    }

    void Replay()
    {
        for (Storage* s : m_read) s->Upload();
        FML_CALL(fml_graph_launch(m_graph, nullptr));
        for (Storage* s : m_written) s->host_valid = false;
    }

    bool Recorded() const { return m_graph != nullptr; }

private:
    static std::vector<Storage*> Unique(std::vector<Storage*> v)
    {
        std::sort(v.begin(), v.end());
        v.erase(std::unique(v.begin(), v.end()), v.end());
        return v;
    }

    fml_graph* m_graph = nullptr;
    std::vector<Storage*> m_read, m_written;
};

}  // namespace freeml_cuda

// GatherRows  MatrixBase_Functions.h:203-242 (token ids stored as floats)
template <class T>
void GatherRows(MatrixCUDA<T>* _out, MatrixCUDA<T>* _src, MatrixCUDA<T>* _indices)
{
    const uint32_t width = _src->GetDimsX();
    FML_CALL(fml_gather_rows(_out->DevOut(), _src->DevIn(), _indices->DevIn(), _indices->GetElementCount(), width,
                             _src->GetDimsY() * _src->GetDimsZ(), freeml_cuda::Stream()));
}

// Add  MatrixBase_Functions.h:471-479
template <class T>
void Add(MatrixCUDA<T>* _out, MatrixCUDA<T>* _L, MatrixCUDA<T>* _R)
{
    const float* l = _L->DevIn();
    const float* r = _R->DevIn();
    FML_CALL(fml_add(_out->DevOut(), l, r, _R->GetElementCount(), freeml_cuda::Stream()));
}

// BroadcastAdd  MatrixBase_Functions.h:717-731
template <class T>
void BroadcastAdd(MatrixCUDA<T>* _out, MatrixCUDA<T>* _L, MatrixCUDA<T>* _R)
{
    const float* l = _L->DevIn();
    const float* r = _R->DevIn();
    FML_CALL(fml_broadcast_add(_out->DevOut(), l, r, _L->GetElementCount(), _L->GetDimsX(), freeml_cuda::Stream()));
}

// PerElementMul  MatrixBase_Functions.h:848-855
template <class T>
void PerElementMul(MatrixCUDA<T>* _out, MatrixCUDA<T>* _L, MatrixCUDA<T>* _R)
{
    const float* l = _L->DevIn();
    const float* r = _R->DevIn();
    FML_CALL(fml_mul_elementwise(_out->DevOut(), l, r, _R->GetElementCount(), freeml_cuda::Stream()));
}

// Scale(out, in, Mat*)  MatrixBase_Functions.h:1021-1030 and Scale(out, in, float)  :1032-1039
template <class T>
void Scale(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in, MatrixCUDA<T>* _val)
{
    const float* in = _in->DevIn();
    const float* v = _val->DevIn();
    FML_CALL(fml_scale(_out->DevOut(), in, 0.0f, v, _in->GetElementCount(), freeml_cuda::Stream()));
}

template <class T>
void Scale(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in, float _val)
{
    const float* in = _in->DevIn();
    FML_CALL(fml_scale(_out->DevOut(), in, _val, nullptr, _in->GetElementCount(), freeml_cuda::Stream()));
}

// ScaleAdd(out, in, Mat* scale, add)  MatrixBase_Functions.h:1056-1070 and (out, in, float, add)  :1044-1054
template <class T>
void ScaleAdd(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in, MatrixCUDA<T>* _scale, MatrixCUDA<T>* _add)
{
    const float* in = _in->DevIn();
    const float* s = _scale->DevIn();
    const float* a = _add->DevIn();
    FML_CALL(fml_scale_add(_out->DevOut(), in, s, a, _out->GetElementCount(), freeml_cuda::Stream()));
}

// Fill(out, float)  :1079-1086, Fill(out, Mat*)  :1088-1096, Clear(out)  :1073-1077
template <class T>
void Fill(MatrixCUDA<T>* _out, float _val)
{
    FML_CALL(fml_fill(_out->DevOut(), _val, nullptr, _out->GetElementCount(), freeml_cuda::Stream()));
}

template <class T>
void Fill(MatrixCUDA<T>* _out, MatrixCUDA<T>* _val)
{
    const float* v = _val->DevIn();
    FML_CALL(fml_fill(_out->DevOut(), 0.0f, v, _out->GetElementCount(), freeml_cuda::Stream()));
}

template <class T>
void Clear(MatrixCUDA<T>* _out)
{
    FML_CALL(fml_fill(_out->DevOut(), 0.0f, nullptr, _out->GetElementCount(), freeml_cuda::Stream()));
}

// Copy  MatrixBase_Functions.h:157-162 and CopyRange  :164-181
template <class T>
void Copy(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in)
{
    const float* in = _in->DevIn();
    FML_CALL(fml_copy(_out->DevOut(), in, _in->GetElementCount(), freeml_cuda::Stream()));
}

template <class T>
void CopyRange(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in, uint32_t outOffset, uint32_t inOffset, uint32_t count)
{
    const float* in = _in->DevIn();
    FML_CALL(fml_copy(_out->DevOut() + outOffset, in + inOffset, count, freeml_cuda::Stream()));
}

// LayerNormOp  MatrixBase_Functions.h:482-549
template <class T>
void LayerNormOp(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in, MatrixCUDA<T>* _gamma, MatrixCUDA<T>* _beta = nullptr,
                 MatrixCUDA<T>* _xHat = nullptr, T _eps = static_cast<T>(1e-5))
{
    const float* in = _in->DevIn();
    const float* g = _gamma->DevIn();
    const float* b = _beta ? _beta->DevIn() : nullptr;
    float* xh = _xHat ? _xHat->DevOut() : nullptr;
    const uint32_t cols = _in->GetDimsX();
    FML_CALL(fml_layernorm(_out->DevOut(), in, g, b, xh, _in->GetDimsY() * _in->GetDimsZ(), cols, (float)_eps,
                           freeml_cuda::Stream()));
}

// GeluMat  MatrixBase_Functions.h:989-1000 (called by Gelu::activateMat, ActivationLibrary/Gelu.h:32-38)
template <class T>
void GeluMat(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in)
{
    const float* in = _in->DevIn();
    FML_CALL(fml_gelu(_out->DevOut(), in, _in->GetElementCount(), freeml_cuda::Stream()));
}

// Softmax  MatrixBase_Functions.h:50-80
template <class T>
void Softmax(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in)
{
    const float* in = _in->DevIn();
    FML_CALL(fml_softmax(_out->DevOut(), in, _in->GetDimsY() * _in->GetDimsZ(), _in->GetDimsX(),
                         freeml_cuda::Stream()));
}

// SplitQKV  MatrixBase_Functions.h:330-367
template <class T>
void SplitQKV(MatrixCUDA<T>* _q, MatrixCUDA<T>* _k, MatrixCUDA<T>* _v, MatrixCUDA<T>* _packed)
{
    const float* p = _packed->DevIn();
    FML_CALL(fml_split_qkv(_q->DevOut(), _k->DevOut(), _v->DevOut(), p, _q->GetDimsY() * _q->GetDimsZ(),
                           _q->GetDimsX(), freeml_cuda::Stream()));
}

// Mul<Mode>  MatrixBase_Mul.h:591-615.  None, Right and Left (the weight
// gradients, Dense.h:258-275) run on the device; Both uses FreeML's host
// template.
template <TransposeMode Mode = TransposeMode::None, class T>
void Mul(MatrixCUDA<T>* _out, MatrixCUDA<T>* _L, MatrixCUDA<T>* _R, uint32_t blockSize = 32, uint32_t numThreads = 12,
         ThreadPool* pool = nullptr)
{
    if constexpr (Mode == TransposeMode::None || Mode == TransposeMode::Right)
    {
        constexpr bool tb = Mode == TransposeMode::Right;
        const uint32_t M = _L->GetDimsY(), K = _L->GetDimsX();
        const uint32_t N = tb ? _R->GetDimsY() : _R->GetDimsX();
        const float* l = _L->DevIn();
        const float* r = _R->DevIn();
        FML_CALL(fml_matmul(_out->DevOut(), l, r, M, N, K, tb ? 1 : 0, freeml_cuda::Stream()));
    }
    else if constexpr (Mode == TransposeMode::Left)
    {
        const uint32_t M = _L->GetDimsX(), K = _L->GetDimsY(), N = _R->GetDimsX();
        const float* l = _L->DevIn();
        const float* r = _R->DevIn();
        FML_CALL(fml_matmul_left(_out->DevOut(), l, r, M, N, K, M, N, N, 1, 0, 0, 0, freeml_cuda::Stream()));
    }
    else
    {
        Mul<Mode, T>(static_cast<MatrixBase<T>*>(_out), static_cast<MatrixBase<T>*>(_L),
                     static_cast<MatrixBase<T>*>(_R), blockSize, numThreads, pool);
    }
}

// MatMul_Strided<Mode>  MatrixBase_Mul.h:617-722 for None / Right / Left with column
// strides of 1 (the form CausalSelfAttentionLayer.h:445-497 uses), one
// contraction per z plane with the reference's plane strides (row stride x
// rows).  Other forms use FreeML's host template.
template <TransposeMode Mode = TransposeMode::None, class T>
void MatMul_Strided(MatrixCUDA<T>* _out, MatrixCUDA<T>* _L, MatrixCUDA<T>* _R, uint32_t L_rowStride,
                    uint32_t L_colStride, uint32_t R_rowStride, uint32_t R_colStride, uint32_t outRowStride,
                    uint32_t outColStride, uint32_t blockSize = 32, uint32_t numThreads = 12,
                    ThreadPool* pool = nullptr)
{
    if constexpr (Mode == TransposeMode::Left)
    {
        if (L_colStride == 1 && R_colStride == 1 && outColStride == 1)
        {
            const uint32_t M = _L->GetDimsX(), K = _L->GetDimsY(), N = _R->GetDimsX();
            const uint32_t batch = _L->GetDimsZ() ? _L->GetDimsZ() : 1;
            const float* l = _L->DevIn();
            const float* r = _R->DevIn();
            FML_CALL(fml_matmul_left(_out->DevOut(), l, r, M, N, K, L_rowStride, R_rowStride, outRowStride, batch,
                                     (uint64_t)L_rowStride * _L->GetDimsY(), (uint64_t)R_rowStride * _R->GetDimsY(),
                                     (uint64_t)outRowStride * _out->GetDimsY(), freeml_cuda::Stream()));
            return;
        }
    }
    if constexpr (Mode == TransposeMode::None || Mode == TransposeMode::Right)
    {
        if (L_colStride == 1 && R_colStride == 1 && outColStride == 1)
        {
            constexpr bool tb = Mode == TransposeMode::Right;
            const uint32_t M = _L->GetDimsY(), K = _L->GetDimsX();
            const uint32_t N = tb ? _R->GetDimsY() : _R->GetDimsX();
            const uint32_t batch = _L->GetDimsZ() ? _L->GetDimsZ() : 1;
            const float* l = _L->DevIn();
            const float* r = _R->DevIn();
            FML_CALL(fml_matmul_strided(_out->DevOut(), l, r, M, N, K, L_rowStride, R_rowStride, outRowStride,
                                        tb ? 1 : 0, batch, (uint64_t)L_rowStride * _L->GetDimsY(),
                                        (uint64_t)R_rowStride * _R->GetDimsY(),
                                        (uint64_t)outRowStride * _out->GetDimsY(), freeml_cuda::Stream()));
            return;
        }
    }
    MatMul_Strided<Mode, T>(static_cast<MatrixBase<T>*>(_out), static_cast<MatrixBase<T>*>(_L),
                            static_cast<MatrixBase<T>*>(_R), L_rowStride, L_colStride, R_rowStride, R_colStride,
                            outRowStride, outColStride, blockSize, numThreads, pool);
}

// ---- training: backward operators, the loss and the optimiser step -------

namespace freeml_cuda {
// Grow-only device scratch for operators that need temporary space (slot:
// one per operator kind): the training entry points of the C ABI take their
// workspace from the caller.  One process-wide set, for the current device
// (the drop-in, like MatrixManager, drives one device per process).
inline float* Scratch(size_t floats, int slot)
{
    static float* ptr[4] = {};
    static size_t have[4] = {};
    if (have[slot] < floats)
    {
        if (ptr[slot]) fml_device_free(ptr[slot]);
        ptr[slot] = nullptr;
        Check(fml_device_alloc(reinterpret_cast<void**>(&ptr[slot]), floats * sizeof(float)), "fml_device_alloc");
        have[slot] = floats;
    }
    return ptr[slot];
}
}  // namespace freeml_cuda

// MergeQKV  MatrixBase_Functions.h:369-431 (CausalSelfAttentionLayer.h backward)
template <class T>
void MergeQKV(MatrixCUDA<T>* _packedQKV, MatrixCUDA<T>* _qHeads, MatrixCUDA<T>* _kHeads, MatrixCUDA<T>* _vHeads)
{
    const float* q = _qHeads->DevIn();
    const float* k = _kHeads->DevIn();
    const float* v = _vHeads->DevIn();
    FML_CALL(fml_merge_qkv(_packedQKV->DevOut(), q, k, v, _qHeads->GetDimsX(), _qHeads->GetDimsY(),
                           _qHeads->GetDimsZ() ? _qHeads->GetDimsZ() : 1, freeml_cuda::Stream()));
}

// GeluDerivtiveMat  MatrixBase_Functions.h:1003-1018 (Gelu.h:40-46)
template <class T>
void GeluDerivtiveMat(MatrixCUDA<T>* _out, MatrixCUDA<T>* _in)
{
    const float* in = _in->DevIn();
    FML_CALL(fml_gelu_derivative(_out->DevOut(), in, _in->GetElementCount(), freeml_cuda::Stream()));
}

// SoftmaxBackwards  MatrixBase_Functions.h:82-111 (rows = dims y, as there)
template <class T>
void SoftmaxBackwards(MatrixCUDA<T>* _out, MatrixCUDA<T>* _softmaxOut, MatrixCUDA<T>* _gradIn)
{
    const float* y = _softmaxOut->DevIn();
    const float* g = _gradIn->DevIn();
    FML_CALL(fml_softmax_backward(_out->DevOut(), y, g, _softmaxOut->GetDimsY(), _softmaxOut->GetDimsX(),
                                  freeml_cuda::Stream()));
}

// ScatterAddRows  MatrixBase_Functions.h:285-320 (Embedding.h backward)
template <class T>
void ScatterAddRows(MatrixCUDA<T>* _out, MatrixCUDA<T>* _src, MatrixCUDA<T>* _indices)
{
    const float* src = _src->DevIn();
    const float* idx = _indices->DevIn();
    // the output accumulates: read-modify-write on the device
    float* out = const_cast<float*>(_out->DevIn());
    _out->DevOut();
    FML_CALL(fml_scatter_add_rows(out, src, idx, _src->GetDimsY(), _src->GetDimsX(), _out->GetDimsY(),
                                  _src->GetDimsZ() ? _src->GetDimsZ() : 1, _out->GetDimsZ() ? _out->GetDimsZ() : 1,
                                  freeml_cuda::Stream()));
}

// LayerNormBackwardsOp  MatrixBase_Functions.h:552-705
template <class T>
void LayerNormBackwardsOp(MatrixCUDA<T>* _dX, MatrixCUDA<T>* _dY, MatrixCUDA<T>* _in, MatrixCUDA<T>* _gamma,
                          MatrixCUDA<T>* _dGamma, MatrixCUDA<T>* _dBeta = nullptr, MatrixCUDA<T>* _xHat = nullptr,
                          T _eps = static_cast<T>(1e-5))
{
    const uint32_t rows = _in->GetDimsY() * _in->GetDimsZ(), cols = _in->GetDimsX();
    const float* dy = _dY->DevIn();
    const float* in = _in->DevIn();
    const float* g = _gamma->DevIn();
    const float* xh = _xHat ? _xHat->DevIn() : nullptr;
    float* db = _dBeta ? _dBeta->DevOut() : nullptr;
    FML_CALL(fml_layernorm_backward(_dX->DevOut(), dy, in, g, _dGamma->DevOut(), db, xh, rows, cols, _eps,
                                    xh ? nullptr : freeml_cuda::Scratch(2 * (size_t)rows, 0), freeml_cuda::Stream()));
}

// AdamWUpdate  MatrixBase_Functions.h:1498-1545 (AdamWOptimiser::Step)
template <class T>
void AdamWUpdate(MatrixCUDA<T>* _param, MatrixCUDA<T>* _grad, MatrixCUDA<T>* _mt, MatrixCUDA<T>* _vt, T _lr,
                 T _beta1, T _beta2, T _beta1_pow_t, T _beta2_pow_t, T _eps, T _weightDecay)
{
    const float* g = _grad->DevIn();
    FML_CALL(fml_adamw_update(_param->DevOut(), g, _mt->DevOut(), _vt->DevOut(), _param->GetElementCount(), _lr,
                              _beta1, _beta2, _beta1_pow_t, _beta2_pow_t, _eps, _weightDecay, freeml_cuda::Stream()));
}

// CategoricalCrossEntropyWithLogits for MatrixCUDA: the loss and its
// (negative) gradient on the device -- the same class specialisation
// mechanism as the DirectX11 backend's
// (LossLibrary/CategoricalCrossEntropyWithLogits.h:219-222).
template <class T>
class CategoricalCrossEntropyWithLogits<T, MatrixCUDA<T>> : public LossBase<T, MatrixCUDA<T>>
{
public:
    const char* GetName() const override { return "CategoricalCrossEntropyWithLogits"; }

    T Loss(MatrixCUDA<T>* target, MatrixCUDA<T>* logits) override
    {
        float loss = 0.0f;
        Run(nullptr, target, logits, &loss);
        return loss;
    }

    void Gradient(MatrixCUDA<T>* out, MatrixCUDA<T>* target, MatrixCUDA<T>* logits) override
    {
        Run(out, target, logits, nullptr);
    }

private:
    static void Run(MatrixCUDA<T>* out, MatrixCUDA<T>* target, MatrixCUDA<T>* logits, float* loss)
    {
        const uint32_t vocab = logits->GetDimsX(), steps = logits->GetDimsY();
        const uint32_t planes = logits->GetDimsZ() ? logits->GetDimsZ() : 1;
        if (!vocab || !steps) return;
        const size_t rows = (size_t)steps * planes;
        const float* tg = target->DevIn();
        const float* lg = logits->DevIn();
        // the loss alone still computes the gradient rows: into scratch
        float* grad = out ? out->DevOut() : freeml_cuda::Scratch(rows * vocab, 1);
        FML_CALL(fml_xent_with_logits(grad, loss, tg, lg, vocab, steps, planes,
                                      target->GetDimsZ() ? target->GetDimsZ() : 1, target->GetDimsX() == 1u ? 1 : 0,
                                      loss ? freeml_cuda::Scratch(rows + 1, 2) : nullptr, freeml_cuda::Stream()));
    }
};

// AdamWOptimiser::Step (OptimiserLibrary/AdamWOptimiser.h:131-196) for
// MatrixCUDA: the reference's state handling (lazy moments cleared to zero,
// a step count per parameter, bias-correction powers) with the update on
// the device -- its generic branch casts to MatrixBase<T>*, which would
// select FreeML's host AdamWUpdate.
template <>
inline void AdamWOptimiser<float, MatrixCUDA<float>>::Step(MatrixCUDA<float>* param, MatrixCUDA<float>* grad)
{
    MatrixCUDA<float>* key = param;
    if (m_momentzero.find(key) == m_momentzero.end())
    {
        MatrixManager<float, MatrixCUDA<float>>& inst = MatrixManager<float, MatrixCUDA<float>>::Instance();
        m_momentzero[key] = inst.AllocateMatrix(param->GetDims(), "adamw_m");
        m_momentone[key] = inst.AllocateMatrix(param->GetDims(), "adamw_v");
        Clear(m_momentzero[key].get());
        Clear(m_momentone[key].get());
        m_timestep[key] = 0;
    }
    auto& mt = m_momentzero[key];
    auto& vt = m_momentone[key];
    uint64_t& t = m_timestep[key];
    ++t;
    const float beta1_pow_t = std::pow(m_beta1, t);
    const float beta2_pow_t = std::pow(m_beta2, t);
    AdamWUpdate(param, grad, mt.get(), vt.get(), m_learningRate, m_beta1, m_beta2, beta1_pow_t, beta2_pow_t, m_epsilon,
                m_weightDecay);
}

#undef FML_CALL
