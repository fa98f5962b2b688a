// Compiles the C++ CUDABackend mirror the way the reference's tensor_ops would use it and
// checks, without a GPU, that a failing call throws instead of being silently ignored.
#include <cstdio>

#include "om_cuda_backend.hpp"

int main() {
    float* p = nullptr;
    try {
        // no omCudaInit on this thread: the backend must report OM_ERR_NOT_INIT
        om::CUDABackend::relu(p, p, 16);
        std::puts("no-throw");
        return 1;
    } catch (const om::CudaBackendError& e) {
        std::printf("threw %d\n", e.status());
        return e.status() == OM_ERR_NOT_INIT ? 0 : 2;
    }
}
