// MatrixCUDA<T> -- a FreeML matrix type whose storage lives in B200 device
// memory, so that Model<float, MatrixCUDA<float>> is a drop-in for
// Model<float, MatrixCPU<float>>.  Pair with MatrixCUDA_Functions.h, which
// overloads the generic operators for this type (the way
// MatrixLibrary/GPU/DirectX11/MatrixDX11_Functions.h does for MatrixDX11).
//
// Requires the FreeML root on the include path and libfreeml_cuda.so.
//
// Interface: MatrixLibrary/MatrixBase.h:34-160.  Storage semantics follow
// MatrixCPU (MatrixLibrary/CPU/MatrixCPU.h:9-143):
//   * AllocateMemory() owns a device buffer; FreeMemory() releases it and is
//     only called by MatrixManager::TryDeleteNow (MatrixManager.h:462-486);
//     the destructor frees nothing;
//   * GetData()/GetOffset()/SetData(ptr, offset) and GetSliceZ() make
//     non-owning views of the same buffer (CausalSelfAttentionLayer.h:
//     430-440, Model.h:773-777).  GetData() returns the buffer's storage
//     record (not a device address); only MatrixCUDA's own SetData reads it;
//   * DataWrite()/DataRead() give host-coherent access for FreeML's generic
//     host templates (weight init, masks, scalars): the whole buffer is
//     mirrored on the host, downloaded on first host access and uploaded
//     again before the next device use.  Every such transfer is counted
//     (HostTransfers()), so a caller can check that Model::Run did none.
#pragma once

#include <MatrixLibrary/MatrixBase.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include "../freeml_cuda.h"

namespace freeml_cuda {

// Aborts with the library's message when an entry point fails (the
// reference asserts on bad shapes; a failed device call cannot continue).
inline void Check(int status, const char* what)
{
    if (status != FML_OK)
    {
        std::fprintf(stderr, "freeml_b200: %s failed (%d): %s\n", what, status, fml_last_error());
        std::abort();
    }
}

struct Counters
{
    uint64_t downloads = 0, uploads = 0;
};

inline Counters& GlobalCounters()
{
    static Counters c;
    return c;
}

struct Storage;

// Buffers the operators read and write while a RunGraph records (see
// MatrixCUDA_Functions.h): a replay must upload pending host writes to the
// first and mark the host mirrors of the second stale, since the recorded
// calls -- and their DevIn() / DevOut() bookkeeping -- do not run again.
struct Recording
{
    std::vector<Storage*> read, written;
};

inline Recording*& ActiveRecording()
{
    static Recording* r = nullptr;
    return r;
}

// One device buffer and its host mirror, shared by the owner and all views.
struct Storage
{
    float* dev = nullptr;
    size_t count = 0;
    std::vector<float> host;
    bool host_valid = false;  // mirror holds the current contents
    bool host_dirty = false;  // mirror has writes not yet on the device

    void Download()
    {
        if (host_valid) return;
        host.resize(count);
        if (count) Check(fml_memcpy_to_host(host.data(), dev, count * sizeof(float)), "fml_memcpy_to_host");
        host_valid = true;
        ++GlobalCounters().downloads;
    }

    void Upload()
    {
        if (!host_dirty) return;
        if (count) Check(fml_memcpy_to_device(dev, host.data(), count * sizeof(float)), "fml_memcpy_to_device");
        host_dirty = false;
        ++GlobalCounters().uploads;
    }
};

}  // namespace freeml_cuda

template <class T>
class MatrixCUDA : public MatrixBase<T>
{
    static_assert(sizeof(T) == sizeof(float), "MatrixCUDA stores fp32");

public:
    MatrixCUDA(void* _data = nullptr)
    {
        MatrixBase<T>::m_hardwareName = "CUDA";
        SetData(_data);
    }

    MatrixCUDA(T* _data, Dims3D _dims, std::string _name = "NoName") : MatrixCUDA(static_cast<void*>(_data))
    {
        MatrixBase<T>::m_name = _name;
        MatrixBase<T>::m_dims = _dims;
    }

    ~MatrixCUDA() {}

    bool AllocateMemory(uint32_t _elementCount) override
    {
        auto* s = new freeml_cuda::Storage();
        s->count = _elementCount;
        if (_elementCount && fml_device_alloc(reinterpret_cast<void**>(&s->dev), _elementCount * sizeof(float)) != FML_OK)
        {
            delete s;
            return false;
        }
        m_storage = s;
        m_offset = 0;
        m_owner = true;
        return true;
    }

    void FreeMemory() override
    {
        if (!m_owner || !m_storage) return;
        if (m_storage->dev) fml_device_free(m_storage->dev);
        delete m_storage;
        m_storage = nullptr;
        m_owner = false;
    }

    // ---- views ----------------------------------------------------------
    void GetSliceZ(MatrixBase<T>* _matrixOut, uint32_t _zIndex) override
    {
        auto* out = static_cast<MatrixCUDA<T>*>(_matrixOut);
        out->SetData(m_storage, m_offset + this->GetDimsX() * this->GetDimsY() * _zIndex);
        out->SetDims({this->GetDimsX(), this->GetDimsY(), 1});
    }

    void SetData(void* _ptr, uint32_t _offset = 0u) override
    {
        m_storage = static_cast<freeml_cuda::Storage*>(_ptr);
        m_offset = _offset;
        m_owner = false;
    }

    void* GetData() override { return m_storage; }
    uint32_t GetOffset() override { return m_offset; }

    // ---- device access (used by MatrixCUDA_Functions.h) -----------------
    // Device address of element 0 for reading; pending host writes go first.
    const float* DevIn()
    {
        if (!m_storage) return nullptr;
        m_storage->Upload();
        if (auto* r = freeml_cuda::ActiveRecording()) r->read.push_back(m_storage);
        return m_storage->dev + m_offset;
    }

    // Device address for a kernel that writes this matrix: pending host
    // writes are flushed first (a kernel may write only part of the buffer)
    // and the host mirror becomes stale.
    float* DevOut()
    {
        if (!m_storage) return nullptr;
        m_storage->Upload();
        m_storage->host_valid = false;
        if (auto* r = freeml_cuda::ActiveRecording()) r->written.push_back(m_storage);
        return m_storage->dev + m_offset;
    }

    // Uploads pending host writes now (e.g. a token window written through
    // DataWrite() before Model::Run), so that the transfer happens here.
    void Flush()
    {
        if (m_storage) m_storage->Upload();
    }

    static freeml_cuda::Counters HostTransfers() { return freeml_cuda::GlobalCounters(); }

    // ---- host access ----------------------------------------------------
    // FML_TRACE_HOST=1: name every matrix whose host access moves data
    // (debugging aid for finding operators that run on the host mirror)
    void TraceHost(const char* what) const
    {
        static const bool on = std::getenv("FML_TRACE_HOST") != nullptr;
        if (on && m_storage && !m_storage->host_valid)
            std::fprintf(stderr, "freeml_b200 host %s: %s [%u x %u x %u]\n", what, this->m_name.c_str(),
                         this->GetDimsX(), this->GetDimsY(), this->GetDimsZ());
    }

    T* DataWrite() override
    {
        if (!m_storage) return nullptr;
        TraceHost("write");
        m_storage->Download();
        m_storage->host_dirty = true;
        return reinterpret_cast<T*>(m_storage->host.data()) + m_offset;
    }

    const T* DataRead() override
    {
        if (!m_storage) return nullptr;
        TraceHost("read");
        m_storage->Download();
        return reinterpret_cast<const T*>(m_storage->host.data()) + m_offset;
    }

    T GetValue(uint32_t _x, uint32_t _y) override { return DataRead()[_y * this->GetDimsX() + _x]; }
    T GetValue(uint32_t _x, uint32_t _y, uint32_t _z) override
    {
        return DataRead()[this->GetDimsX() * this->GetDimsY() * _z + _y * this->GetDimsX() + _x];
    }
    void SetValue(uint32_t _x, uint32_t _y, T _val) override { DataWrite()[_y * this->GetDimsX() + _x] = _val; }
    void SetValue(uint32_t _x, uint32_t _y, uint32_t _z, T _val) override
    {
        DataWrite()[this->GetDimsX() * this->GetDimsY() * _z + _y * this->GetDimsX() + _x] = _val;
    }

    std::vector<T> GetRow(uint32_t _r) override
    {
        const T* start = DataRead() + _r * this->GetDimsX();
        return std::vector<T>(start, start + this->GetDimsX());
    }

    std::vector<T> GetColumn(uint32_t _c) override
    {
        std::vector<T> col;
        const T* d = DataRead();
        for (uint32_t y = 0; y < this->GetDimsY(); ++y) col.push_back(d[y * this->GetDimsX() + _c]);
        return col;
    }

    uint32_t GetElementCount() const override
    {
        return this->GetDimsX() * this->GetDimsY() * this->GetDimsZ();
    }

    void GetRawData(std::vector<char>& _out) override
    {
        const uint32_t count = GetElementCount();
        if (!count || !m_storage)
        {
            _out.clear();
            return;
        }
        const T* d = DataRead();
        _out.resize(count * sizeof(T));
        std::memcpy(_out.data(), d, count * sizeof(T));
    }

private:
    freeml_cuda::Storage* m_storage = nullptr;
    uint32_t m_offset = 0;
    bool m_owner = false;
};
