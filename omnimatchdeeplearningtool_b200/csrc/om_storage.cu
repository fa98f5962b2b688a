// Device-side helpers of the engine's tensor storage (include/om_tensor_storage.hpp).
//
// omCudaStridedCopy gathers a strided fp32 view into a contiguous buffer on the device. The
// reference makes a non-contiguous GPU tensor contiguous by copying it to the host, running
// CPUBackend::stridedCopy there and copying the result back (om.engine.tensor.ixx:385-408,
// cpu_backend stridedCopy); this keeps the data on the device, with the same element order:
// dst[i] = src[offset + sum_d coord_d(i) * stride_d], coords of i in row-major order of shape.
#include "om_common.cuh"

namespace omb {
namespace storage {

constexpr int kMaxDims = 8;

struct StridedView {
    int ndim;
    long long shape[kMaxDims];
    long long stride[kMaxDims];
    long long offset;
    long long total;
};

__global__ void strided_copy_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                    StridedView v) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < v.total;
         i += (long long)gridDim.x * blockDim.x) {
        long long rem = i, off = v.offset;
        for (int d = v.ndim - 1; d >= 0; --d) {
            const long long q = rem / v.shape[d];
            off += (rem - q * v.shape[d]) * v.stride[d];
            rem = q;
        }
        dst[i] = src[off];
    }
}

}  // namespace storage
}  // namespace omb

extern "C" int omCudaStridedCopy(const float* pSrc, float* pDst, const int* pShape,
                                 const int* pStrides, int nDims, long long nOffset) {
    OMB_CTX_OR_FAIL(c);
    using omb::storage::StridedView;
    if (!pSrc || !pDst || nDims < 0 || nDims > omb::storage::kMaxDims || nOffset < 0 ||
        (nDims > 0 && (!pShape || !pStrides)))
        return OM_ERR_INVALID;
    StridedView v;
    v.ndim = nDims;
    v.offset = nOffset;
    v.total = 1;
    for (int d = 0; d < nDims; ++d) {
        if (pShape[d] < 0 || pStrides[d] < 0) return OM_ERR_INVALID;
        v.shape[d] = pShape[d];
        v.stride[d] = pStrides[d];
        v.total *= pShape[d];
    }
    if (v.total == 0) return OM_OK;
    omb::storage::strided_copy_kernel<<<omb::ew_grid(c, v.total, 256), 256, 0, c->compute>>>(
        pSrc, pDst, v);
    return omb::after_launch(c);
}
