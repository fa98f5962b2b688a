// om_tensor_storage.hpp — the engine's TensorStorage on the B200 backend: a drop-in for the
// reference's om::TensorStorage (src/engine/om.engine.tensor_storage.ixx:41-192).
//
// The engine's Tensor, tensor_ops and autograd code use exactly the reference's surface: the two
// constructors (bytes, device, device id) and (source, bytes, device, device id), data(),
// mutableData(), bytes(), deviceType(), deviceId() and copyTo(). Those keep the reference's
// meaning: an untyped byte buffer holding fp32 NCHW-contiguous data, on the host (64-byte
// aligned) or on a device through omCudaMalloc/omCudaFree, with synchronous copies.
//
// Differences from the reference:
//   * device memory is allocated, freed and copied with ITS device current (the reference uses
//     whatever device the process last selected; it only ever drives device 0), and a device a
//     thread has not initialised yet is initialised on first use;
//   * every failing call throws std::runtime_error with the backend status (the reference
//     ignores the status of omCudaFree);
//   * new, for the 16-bit fused path: a storage knows its element type (fp32, bf16, fp16) and
//     its layout (Flat = the engine's NCHW-contiguous fp32, or NHWC with the channel count
//     padded to omCudaStoredChannels), the logical NCHW shape of an NHWC storage, and the
//     device's compute stream that orders every operation on it;
//   * copyTo(CPU) always yields flat NCHW fp32, converting an NHWC / 16-bit device storage on the
//     device first, so code that reads tensors back (ModelSerializer::save, Tensor::cpu) keeps
//     working unchanged;
//   * contiguousCopy() makes a strided fp32 view contiguous on the device (omCudaStridedCopy),
//     in place of the reference's device -> host -> device round trip (om.engine.tensor.ixx:
//     390-391).
//
// DeviceType comes from the engine's om_types.h when it is on the include path; on its own this
// header declares the same enum (same enumerators and values).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#if __has_include("om_types.h")
#include "om_types.h"
#else
namespace om {
enum class DeviceType { CPU = 0, CUDA, OpenCL };
}  // namespace om
#endif

#include "om_cuda.h"

namespace om {

// Element type of a storage (values are the C ABI's OM_DTYPE_* codes).
enum class StorageDtype : int { Float32 = OM_DTYPE_F32, BFloat16 = OM_DTYPE_BF16, Float16 = OM_DTYPE_F16 };
// Flat: the engine's NCHW-contiguous buffer (the Tensor's shape and strides describe it).
// NHWC: [N, H, W, Cs] with Cs = omCudaStoredChannels(C), channels C..Cs-1 zero.
enum class StorageLayout : int { Flat = 0, NHWC = 1 };

inline size_t storageElemSize(StorageDtype d) { return d == StorageDtype::Float32 ? 4 : 2; }

namespace storage_detail {

inline void check(int st, const char* what) {
    if (st != OM_OK)
        throw std::runtime_error(std::string("TensorStorage: ") + what + " failed (status " +
                                 std::to_string(st) + ")");
}

// Makes `dev` the calling thread's device for the scope's lifetime (initialising it the first
// time this thread uses it) and restores the previous device afterwards.
class DeviceScope {
public:
    explicit DeviceScope(int dev) : m_prev(omCudaGetCurrentDevice()) {
        if (m_prev == dev) return;
        int st = omCudaSetDevice(dev);
        if (st == OM_ERR_NOT_INIT) st = omCudaInit(dev);
        check(st, "selecting the storage's device");
        m_switched = true;
    }
    ~DeviceScope() {
        if (m_switched && m_prev >= 0) omCudaSetDevice(m_prev);
    }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;

private:
    int m_prev;
    bool m_switched = false;
};

}  // namespace storage_detail

class TensorStorage {
public:
    // Same as the reference: nBytes of 64-byte-aligned host memory, or device memory on
    // device nDeviceId. A flat fp32 storage.
    explicit TensorStorage(size_t nBytes, DeviceType eDevice = DeviceType::CPU, int nDeviceId = 0)
        : m_pData(nullptr), m_nBytes(nBytes), m_deviceType(eDevice), m_nDeviceId(nDeviceId) {
        allocate();
    }

    // Same as the reference: a copy of nBytes host bytes at pSrcData on the given device.
    TensorStorage(const void* pSrcData, size_t nBytes, DeviceType eDevice = DeviceType::CPU,
                  int nDeviceId = 0)
        : TensorStorage(nBytes, eDevice, nDeviceId) {
        if (!pSrcData || nBytes == 0) return;
        if (eDevice == DeviceType::CUDA) {
            storage_detail::DeviceScope g(m_nDeviceId);
            storage_detail::check(omCudaCopyH2D(m_pData, pSrcData, nBytes), "omCudaCopyH2D");
        } else {
            std::memcpy(m_pData, pSrcData, nBytes);
        }
    }

    // New: an uninitialised NHWC device storage for the logical NCHW shape [N, C, H, W] with
    // element type dt (bf16 or fp16), channels padded to omCudaStoredChannels(C).
    static std::shared_ptr<TensorStorage> makeNhwc(int N, int C, int H, int W, StorageDtype dt,
                                                   int nDeviceId) {
        if (dt == StorageDtype::Float32)
            throw std::invalid_argument("TensorStorage: NHWC storage is bf16 or fp16");
        if (N <= 0 || C <= 0 || H <= 0 || W <= 0)
            throw std::invalid_argument("TensorStorage: NHWC shape must be positive");
        const int cs = omCudaStoredChannels(C);
        const size_t bytes = (size_t)N * H * W * cs * storageElemSize(dt);
        auto s = std::make_shared<TensorStorage>(bytes, DeviceType::CUDA, nDeviceId);
        s->m_dtype = dt;
        s->m_layout = StorageLayout::NHWC;
        s->m_shape = {N, C, H, W};
        s->m_storedChannels = cs;
        return s;
    }

    TensorStorage(const TensorStorage&) = delete;
    TensorStorage& operator=(const TensorStorage&) = delete;

    ~TensorStorage() { release(); }

    // ---- the reference's accessors
    const void* data() const { return m_pData; }
    void* mutableData() { return m_pData; }
    size_t bytes() const { return m_nBytes; }
    DeviceType deviceType() const { return m_deviceType; }
    int deviceId() const { return m_nDeviceId; }

    // ---- new accessors
    StorageDtype dtype() const { return m_dtype; }
    StorageLayout layout() const { return m_layout; }
    // logical [N, C, H, W] of an NHWC storage (zeros for a flat one)
    const std::array<int, 4>& nchwShape() const { return m_shape; }
    int storedChannels() const { return m_storedChannels; }
    // The compute stream (a cudaStream_t) of the storage's device; nullptr for host storage.
    // Every backend call on this storage's data is ordered on it.
    void* stream() const {
        if (m_deviceType != DeviceType::CUDA) return nullptr;
        storage_detail::DeviceScope g(m_nDeviceId);
        return omCudaGetStream();
    }

    // The reference's copyTo, in all four directions. A CPU target always receives flat NCHW
    // fp32: an NHWC or 16-bit device storage is first converted on its device.
    std::shared_ptr<TensorStorage> copyTo(DeviceType eTargetDevice, int nTargetDeviceId = 0) const {
        using storage_detail::check;
        using storage_detail::DeviceScope;
        if (m_deviceType == DeviceType::CUDA && m_layout == StorageLayout::NHWC) {
            auto flat = toNchwFloat();
            return eTargetDevice == DeviceType::CUDA && nTargetDeviceId == m_nDeviceId
                       ? flat
                       : flat->copyTo(eTargetDevice, nTargetDeviceId);
        }
        auto pNew = std::make_shared<TensorStorage>(m_nBytes, eTargetDevice, nTargetDeviceId);
        if (m_nBytes == 0) return pNew;
        const bool srcDev = m_deviceType == DeviceType::CUDA;
        const bool dstDev = eTargetDevice == DeviceType::CUDA;
        if (!srcDev && !dstDev) {
            std::memcpy(pNew->m_pData, m_pData, m_nBytes);
        } else if (!srcDev && dstDev) {
            DeviceScope g(nTargetDeviceId);
            check(omCudaCopyH2D(pNew->m_pData, m_pData, m_nBytes), "omCudaCopyH2D");
        } else if (srcDev && !dstDev) {
            DeviceScope g(m_nDeviceId);
            check(omCudaCopyD2H(pNew->m_pData, m_pData, m_nBytes), "omCudaCopyD2H");
        } else if (nTargetDeviceId == m_nDeviceId) {
            DeviceScope g(m_nDeviceId);
            check(omCudaCopyD2D(pNew->m_pData, m_pData, m_nBytes), "omCudaCopyD2D");
        } else {
            // across devices: the source's pending work first, then a peer copy issued on the
            // target device, complete on return like the reference's synchronous copies
            {
                DeviceScope g(m_nDeviceId);
                check(omCudaSynchronize(), "omCudaSynchronize");
            }
            DeviceScope g(nTargetDeviceId);
            check(omCudaCopyD2D(pNew->m_pData, m_pData, m_nBytes), "omCudaCopyD2D");
            check(omCudaSynchronize(), "omCudaSynchronize");
        }
        return pNew;
    }

    // New: an NHWC copy (dt = bf16 or fp16) on the same device of this flat fp32 device storage,
    // read as the NCHW tensor [N, C, H, W].
    std::shared_ptr<TensorStorage> toNhwc(int N, int C, int H, int W, StorageDtype dt) const {
        if (m_deviceType != DeviceType::CUDA || m_layout != StorageLayout::Flat)
            throw std::invalid_argument("TensorStorage::toNhwc: needs a flat device storage");
        if ((size_t)N * C * H * W * 4 > m_nBytes)
            throw std::invalid_argument("TensorStorage::toNhwc: shape exceeds the storage");
        auto out = makeNhwc(N, C, H, W, dt, m_nDeviceId);
        storage_detail::DeviceScope g(m_nDeviceId);
        storage_detail::check(omCudaNchwToNhwc(static_cast<const float*>(m_pData), out->m_pData, N,
                                               C, H, W, out->m_storedChannels, (int)dt),
                              "omCudaNchwToNhwc");
        return out;
    }

    // New: the flat NCHW fp32 copy, on the same device, of this NHWC storage.
    std::shared_ptr<TensorStorage> toNchwFloat() const {
        if (m_layout != StorageLayout::NHWC)
            throw std::invalid_argument("TensorStorage::toNchwFloat: needs an NHWC storage");
        const auto& s = m_shape;
        auto out = std::make_shared<TensorStorage>((size_t)s[0] * s[1] * s[2] * s[3] * 4,
                                                   DeviceType::CUDA, m_nDeviceId);
        storage_detail::DeviceScope g(m_nDeviceId);
        storage_detail::check(omCudaNhwcToNchw(m_pData, static_cast<float*>(out->m_pData), s[0],
                                               s[1], s[2], s[3], m_storedChannels, (int)m_dtype),
                              "omCudaNhwcToNchw");
        return out;
    }

    // New: a contiguous flat fp32 copy of the strided view (shape, strides and offset in
    // elements, as om::Tensor keeps them) of this storage, made on the storage's own device
    // (on the host for host storage, with the same element order).
    std::shared_ptr<TensorStorage> contiguousCopy(const std::vector<int>& shape,
                                                  const std::vector<int>& strides,
                                                  int offset) const {
        if (shape.size() != strides.size() || shape.size() > 8)
            throw std::invalid_argument("TensorStorage::contiguousCopy: bad view");
        size_t n = 1;
        for (int d : shape) n *= (size_t)(d < 0 ? 0 : d);
        auto out = std::make_shared<TensorStorage>(n * 4, m_deviceType, m_nDeviceId);
        if (n == 0) return out;
        if (m_deviceType == DeviceType::CUDA) {
            storage_detail::DeviceScope g(m_nDeviceId);
            storage_detail::check(
                omCudaStridedCopy(static_cast<const float*>(m_pData),
                                  static_cast<float*>(out->m_pData), shape.data(), strides.data(),
                                  (int)shape.size(), offset),
                "omCudaStridedCopy");
        } else {
            const float* src = static_cast<const float*>(m_pData);
            float* dst = static_cast<float*>(out->m_pData);
            for (size_t i = 0; i < n; ++i) {
                size_t rem = i, off = (size_t)offset;
                for (int d = (int)shape.size() - 1; d >= 0; --d) {
                    off += (rem % (size_t)shape[d]) * (size_t)strides[d];
                    rem /= (size_t)shape[d];
                }
                dst[i] = src[off];
            }
        }
        return out;
    }

private:
    void allocate() {
        if (m_nBytes == 0) return;
        if (m_deviceType == DeviceType::CUDA) {
            storage_detail::DeviceScope g(m_nDeviceId);
            int st = omCudaMalloc(&m_pData, m_nBytes);
            if (st != OM_OK || !m_pData)
                throw std::runtime_error("TensorStorage: omCudaMalloc failed, bytes=" +
                                         std::to_string(m_nBytes) + " status " +
                                         std::to_string(st));
        } else if (m_deviceType == DeviceType::CPU) {
            m_pData = std::aligned_alloc(64, (m_nBytes + 63) & ~size_t(63));
            if (!m_pData) throw std::bad_alloc();
        } else {
            throw std::runtime_error("TensorStorage: unsupported device type");
        }
    }

    void release() noexcept {
        if (!m_pData) return;
        if (m_deviceType == DeviceType::CUDA) {
            try {
                storage_detail::DeviceScope g(m_nDeviceId);
                omCudaFree(m_pData);
            } catch (...) {
                // the device is gone (process teardown): nothing left to return the block to
            }
        } else {
            std::free(m_pData);
        }
        m_pData = nullptr;
    }

    void* m_pData;
    size_t m_nBytes;
    DeviceType m_deviceType;
    int m_nDeviceId;
    StorageDtype m_dtype = StorageDtype::Float32;
    StorageLayout m_layout = StorageLayout::Flat;
    std::array<int, 4> m_shape{{0, 0, 0, 0}};
    int m_storedChannels = 0;
};

}  // namespace om
