// FreeML operator overloads for MatrixCUDA<T>: the sm_100a kernels of
// libfreeml_cuda.so behind the names the layers call.  Include after the
// FreeML headers (and MatrixCUDA.h); argument-dependent lookup at template
// instantiation then picks these over the MatrixBase<T>* templates of
// MatrixLibrary/MatrixBase_Functions.h and MatrixBase_Mul.h -- the same
// mechanism as MatrixLibrary/GPU/DirectX11/MatrixDX11_Functions.h.
//
// Every operator the NanoLLM inference forward reaches runs on the device.
// Training-only forms (Mul<Left|Both>, MatMul_Strided with column strides
// other than 1, the backward operators) are not overloaded and run FreeML's
// own host templates through the host mirror; MatrixCUDA counts those
// transfers so a test can assert that Model::Run performed none.
#pragma once

#include <algorithm>
#include <vector>

#include <MatrixLibrary/MatrixBase_Functions.h>
#include <MatrixLibrary/MatrixBase_Mul.h>

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

// Mul<Mode>  MatrixBase_Mul.h:591-615.  None and Right run on the device;
// Left / Both (gradient products) use FreeML's host template.
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
    else
    {
        Mul<Mode, T>(static_cast<MatrixBase<T>*>(_out), static_cast<MatrixBase<T>*>(_L),
                     static_cast<MatrixBase<T>*>(_R), blockSize, numThreads, pool);
    }
}

// MatMul_Strided<Mode>  MatrixBase_Mul.h:617-722 for None / Right with column
// strides of 1 (the form CausalSelfAttentionLayer.h:445-497 uses), one
// contraction per z plane with the reference's plane strides (row stride x
// rows).  Other forms use FreeML's host template.
template <TransposeMode Mode = TransposeMode::None, class T>
void MatMul_Strided(MatrixCUDA<T>* _out, MatrixCUDA<T>* _L, MatrixCUDA<T>* _R, uint32_t L_rowStride,
                    uint32_t L_colStride, uint32_t R_rowStride, uint32_t R_colStride, uint32_t outRowStride,
                    uint32_t outColStride, uint32_t blockSize = 32, uint32_t numThreads = 12,
                    ThreadPool* pool = nullptr)
{
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

#undef FML_CALL
