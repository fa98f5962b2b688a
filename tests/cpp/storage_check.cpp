// GPU check of om::TensorStorage (include/om_tensor_storage.hpp), run by
// tests/test_gpu_storage.py: compiled with g++ against the header and libomcuda.so, it prints
// "storage ok" when every check passes and exits non-zero at the first failure.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "om_tensor_storage.hpp"

using om::DeviceType;
using om::StorageDtype;
using om::StorageLayout;
using om::TensorStorage;

#define CHECK(cond)                                                       \
    do {                                                                  \
        if (!(cond)) {                                                    \
            std::printf("FAILED line %d: %s\n", __LINE__, #cond);         \
            return 1;                                                     \
        }                                                                 \
    } while (0)

static std::vector<float> host_floats(const TensorStorage& s) {
    std::vector<float> v(s.bytes() / 4);
    std::memcpy(v.data(), s.data(), s.bytes());
    return v;
}

int main() {
    const int N = 2, C = 3, H = 5, W = 7;
    const size_t n = (size_t)N * C * H * W;
    // values exactly representable in bf16 and fp16: k/8 for |k| < 256
    std::vector<float> x(n);
    for (size_t i = 0; i < n; ++i) x[i] = (float)((int)(i * 37 % 401) - 200) / 8.0f;

    // host storage: 64-byte aligned copy, as the reference
    TensorStorage hs(x.data(), n * 4);
    CHECK(((uintptr_t)hs.data() & 63) == 0);
    CHECK(hs.deviceType() == DeviceType::CPU && hs.stream() == nullptr);
    CHECK(std::memcmp(hs.data(), x.data(), n * 4) == 0);

    // host -> device -> host, byte for byte
    auto ds = hs.copyTo(DeviceType::CUDA, 0);
    CHECK(ds->deviceType() == DeviceType::CUDA && ds->deviceId() == 0);
    CHECK(ds->dtype() == StorageDtype::Float32 && ds->layout() == StorageLayout::Flat);
    CHECK(ds->stream() != nullptr);
    auto back = ds->copyTo(DeviceType::CPU);
    CHECK(back->bytes() == n * 4 && std::memcmp(back->data(), x.data(), n * 4) == 0);
    auto dd = ds->copyTo(DeviceType::CUDA, 0);  // device -> device
    CHECK(std::memcmp(dd->copyTo(DeviceType::CPU)->data(), x.data(), n * 4) == 0);

    // NCHW fp32 -> NHWC 16-bit -> copyTo(CPU) gives NCHW fp32 again, bit-exact here
    for (StorageDtype dt : {StorageDtype::BFloat16, StorageDtype::Float16}) {
        auto nh = ds->toNhwc(N, C, H, W, dt);
        CHECK(nh->layout() == StorageLayout::NHWC && nh->dtype() == dt);
        CHECK(nh->nchwShape()[0] == N && nh->nchwShape()[1] == C && nh->nchwShape()[2] == H &&
              nh->nchwShape()[3] == W);
        CHECK(nh->storedChannels() == omCudaStoredChannels(C));
        CHECK(nh->bytes() == (size_t)N * H * W * nh->storedChannels() * 2);
        auto flat = nh->copyTo(DeviceType::CPU);
        CHECK(flat->deviceType() == DeviceType::CPU && flat->bytes() == n * 4);
        CHECK(std::memcmp(flat->data(), x.data(), n * 4) == 0);
        auto dflat = nh->toNchwFloat();
        CHECK(dflat->deviceType() == DeviceType::CUDA && dflat->layout() == StorageLayout::Flat);
        CHECK(std::memcmp(dflat->copyTo(DeviceType::CPU)->data(), x.data(), n * 4) == 0);
    }

    // contiguous copy of strided views on the device equals the host walk of the same view
    struct View {
        std::vector<int> shape, strides;
        int offset;
    };
    const View views[] = {
        {{N, W, H, C}, {C * H * W, 1, W, H * W}, 0},  // NCHW read as N, W, H, C (a permute)
        {{N, 2, H, 3}, {C * H * W, H * W, W, 2}, 1},  // a strided slice with an offset
        {{(int)n}, {1}, 0},                          // already contiguous
    };
    for (const View& v : views) {
        auto dv = ds->contiguousCopy(v.shape, v.strides, v.offset);
        auto hv = hs.contiguousCopy(v.shape, v.strides, v.offset);
        CHECK(dv->deviceType() == DeviceType::CUDA && hv->deviceType() == DeviceType::CPU);
        CHECK(dv->bytes() == hv->bytes());
        auto got = host_floats(*dv->copyTo(DeviceType::CPU));
        auto want = host_floats(*hv);
        CHECK(got == want);
    }
    // spot-check the permute against the definition
    {
        auto hv = host_floats(*hs.contiguousCopy(views[0].shape, views[0].strides, 0));
        const int nn = 1, ww = 4, hh = 2, cc = 2;
        CHECK(hv[((nn * W + ww) * H + hh) * C + cc] == x[((nn * C + cc) * H + hh) * W + ww]);
    }

    // misuse is reported, not run
    bool threw = false;
    try {
        hs.toNhwc(N, C, H, W, StorageDtype::BFloat16);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    CHECK(threw);
    threw = false;
    try {
        TensorStorage bad(64, DeviceType::CUDA, omCudaGetDeviceCount());  // no such device
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw);
    CHECK(omCudaGetCurrentDevice() == 0);  // the thread stays on its device
    std::printf("storage ok\n");
    return 0;
}
