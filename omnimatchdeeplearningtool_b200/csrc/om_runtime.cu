// Device lifecycle, memory and stream entry points (replaces the reference's
// cuda_kernels.cu:63-445 and :4887-4954).
//
// Differences by design from the reference:
//  - a context per device, selected per host thread (the reference keeps one global device,
//    cuda_kernels.cu:63-64), so one process can drive all GPUs of a node;
//  - allocation uses the device's stream-ordered memory pool with an unlimited release
//    threshold, which caches freed blocks like the reference's size-bucketed pool
//    (cuda_kernels.cu:187-285) without a global mutex; on OOM the pool is trimmed and the
//    allocation retried once, as the reference does (:208-240);
//  - every call returns a status; nothing is silently ignored.
#include <mutex>
#include <string.h>

#include "om_common.cuh"

namespace omb {

static DeviceCtx g_ctx[64];
static std::mutex g_ctx_mu;
static thread_local int t_device = -1;

DeviceCtx* ctx() {
    if (t_device < 0) return nullptr;
    DeviceCtx* c = &g_ctx[t_device];
    return c->inited ? c : nullptr;
}

static int init_device(int dev) {
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    DeviceCtx* c = &g_ctx[dev];
    OMB_CHECK(cudaSetDevice(dev));
    if (!c->inited) {
        OMB_CHECK(cudaStreamCreateWithFlags(&c->compute, cudaStreamNonBlocking));
        OMB_CHECK(cudaStreamCreateWithFlags(&c->transfer, cudaStreamNonBlocking));
        OMB_CHECK(cudaEventCreateWithFlags(&c->transfer_done, cudaEventDisableTiming));
        OMB_CHECK(cudaEventCreateWithFlags(&c->compute_done, cudaEventDisableTiming));
        OMB_CHECK(cudaMalloc(&c->err_word, sizeof(unsigned int)));
        OMB_CHECK(cudaMemset(c->err_word, 0, sizeof(unsigned int)));
        OMB_CHECK(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, dev));
        cudaMemPool_t pool;
        OMB_CHECK(cudaDeviceGetDefaultMemPool(&pool, dev));
        unsigned long long thr = ~0ull;
        OMB_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
        OMB_CHECK(cudaDeviceSynchronize());
        c->device = dev;
        c->inited = true;
    }
    t_device = dev;
    return OM_OK;
}

}  // namespace omb

using omb::DeviceCtx;

extern "C" {

int omCudaInit(int nDeviceId) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return OM_ERR_CUDA;
    if (nDeviceId < 0 || nDeviceId >= n || nDeviceId >= 64) return OM_ERR_INVALID;
    return omb::init_device(nDeviceId);
}

int omCudaSetDevice(int nDeviceId) {
    if (nDeviceId < 0 || nDeviceId >= 64 || !omb::g_ctx[nDeviceId].inited) return OM_ERR_NOT_INIT;
    OMB_CHECK(cudaSetDevice(nDeviceId));
    omb::t_device = nDeviceId;
    return OM_OK;
}

int omCudaGetCurrentDevice(void) {
    DeviceCtx* c = omb::ctx();
    return c ? c->device : -1;
}

void* omCudaGetStream(void) {
    DeviceCtx* c = omb::ctx();
    return c ? (void*)c->compute : nullptr;
}

int omCudaGetDeviceCount(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int omCudaGetDeviceName(int nDeviceId, char* pNameBuf, int nBufSize) {
    if (!pNameBuf || nBufSize <= 0) return OM_ERR_INVALID;
    cudaDeviceProp p;
    OMB_CHECK(cudaGetDeviceProperties(&p, nDeviceId));
    strncpy(pNameBuf, p.name, nBufSize - 1);
    pNameBuf[nBufSize - 1] = 0;
    return OM_OK;
}

int omCudaGetMemInfo(int nDeviceId, size_t* pFreeMem, size_t* pTotalMem) {
    int prev = 0;
    OMB_CHECK(cudaGetDevice(&prev));
    OMB_CHECK(cudaSetDevice(nDeviceId));
    cudaError_t e = cudaMemGetInfo(pFreeMem, pTotalMem);
    cudaSetDevice(prev);
    return omb::status_of(e);
}

int omCudaGetComputeCapability(int nDeviceId, int* pMajor, int* pMinor) {
    OMB_CHECK(cudaDeviceGetAttribute(pMajor, cudaDevAttrComputeCapabilityMajor, nDeviceId));
    OMB_CHECK(cudaDeviceGetAttribute(pMinor, cudaDevAttrComputeCapabilityMinor, nDeviceId));
    return OM_OK;
}

int omCudaMalloc(void** ppDevPtr, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    if (!ppDevPtr) return OM_ERR_INVALID;
    if (nBytes == 0) nBytes = 256;
    cudaError_t e = cudaMallocAsync(ppDevPtr, nBytes, c->compute);
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        cudaMemPool_t pool;
        OMB_CHECK(cudaDeviceGetDefaultMemPool(&pool, c->device));
        OMB_CHECK(cudaStreamSynchronize(c->compute));
        OMB_CHECK(cudaMemPoolTrimTo(pool, 0));
        e = cudaMallocAsync(ppDevPtr, nBytes, c->compute);
        if (e == cudaErrorMemoryAllocation) {
            cudaGetLastError();
            return OM_ERR_OOM;
        }
    }
    if (e != cudaSuccess) return OM_ERR_CUDA;
    // The reference's allocation is immediately usable by any stream; keep that contract.
    return omb::status_of(cudaStreamSynchronize(c->compute));
}

int omCudaFree(void* pDevPtr) {
    OMB_CTX_OR_FAIL(c);
    if (!pDevPtr) return OM_OK;
    return omb::status_of(cudaFreeAsync(pDevPtr, c->compute));
}

int omCudaCopyH2D(void* pDst, const void* pSrc, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    OMB_CHECK(cudaMemcpyAsync(pDst, pSrc, nBytes, cudaMemcpyHostToDevice, c->compute));
    return omb::status_of(cudaStreamSynchronize(c->compute));
}

int omCudaCopyD2H(void* pDst, const void* pSrc, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    OMB_CHECK(cudaMemcpyAsync(pDst, pSrc, nBytes, cudaMemcpyDeviceToHost, c->compute));
    return omb::status_of(cudaStreamSynchronize(c->compute));
}

int omCudaCopyD2D(void* pDst, const void* pSrc, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaMemcpyAsync(pDst, pSrc, nBytes, cudaMemcpyDeviceToDevice, c->compute));
}

int omCudaMemset(void* pDev, int nValue, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaMemsetAsync(pDev, nValue, nBytes, c->compute));
}

int omCudaSynchronize(void) {
    OMB_CTX_OR_FAIL(c);
    OMB_CHECK(cudaStreamSynchronize(c->transfer));
    return omb::status_of(cudaStreamSynchronize(c->compute));
}

// Async copies are issued on the compute stream so that they stay ordered with the kernels
// that produce or consume them (the reference uses a second stream plus explicit syncs).
int omCudaAsyncCopyH2D(void* pDst, const void* pSrc, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaMemcpyAsync(pDst, pSrc, nBytes, cudaMemcpyHostToDevice, c->compute));
}

int omCudaAsyncCopyD2H(void* pDst, const void* pSrc, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaMemcpyAsync(pDst, pSrc, nBytes, cudaMemcpyDeviceToHost, c->compute));
}

int omCudaTransferH2D(void* pDst, const void* pSrcHost, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaMemcpyAsync(pDst, pSrcHost, nBytes, cudaMemcpyHostToDevice, c->transfer));
}

int omCudaTransferD2H(void* pDstHost, const void* pSrc, size_t nBytes) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaMemcpyAsync(pDstHost, pSrc, nBytes, cudaMemcpyDeviceToHost, c->transfer));
}

// One reusable event per direction and device: a stream wait binds to the event's most recent
// record at the time the wait is enqueued, so re-recording it afterwards is safe.
static int stream_wait(cudaStream_t waiter, cudaStream_t producer, cudaEvent_t e) {
    OMB_CHECK(cudaEventRecord(e, producer));
    return omb::status_of(cudaStreamWaitEvent(waiter, e, 0));
}

int omCudaComputeWaitTransfer(void) {
    OMB_CTX_OR_FAIL(c);
    return stream_wait(c->compute, c->transfer, c->transfer_done);
}

int omCudaTransferWaitCompute(void) {
    OMB_CTX_OR_FAIL(c);
    return stream_wait(c->transfer, c->compute, c->compute_done);
}

int omCudaSyncTransferStream(void) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaStreamSynchronize(c->transfer));
}

int omCudaSyncComputeStream(void) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaStreamSynchronize(c->compute));
}

int omCudaCleanup(void) {
    OMB_CTX_OR_FAIL(c);
    OMB_CHECK(cudaStreamSynchronize(c->compute));
    cudaMemPool_t pool;
    OMB_CHECK(cudaDeviceGetDefaultMemPool(&pool, c->device));
    return omb::status_of(cudaMemPoolTrimTo(pool, 0));
}

// Recovery after an engine-level failure (the reference's cuda_kernels.cu:429-437, called by
// EngineBridge.cpp:4047): wait for all work on the device, clear a sticky-free last error and
// release the cached pool blocks. Like the reference it does not call cudaDeviceReset, so device
// pointers that tensors still hold stay valid. The context's streams are kept (the reference
// destroys and lazily re-creates its global streams; here every entry point uses them).
int omCudaForceReset(void) {
    OMB_CTX_OR_FAIL(c);
    cudaError_t e = cudaDeviceSynchronize();
    cudaGetLastError();
    if (e != cudaSuccess) return OM_ERR_CUDA;
    cudaMemPool_t pool;
    OMB_CHECK(cudaDeviceGetDefaultMemPool(&pool, c->device));
    return omb::status_of(cudaMemPoolTrimTo(pool, 0));
}

int omCudaMallocHost(void** ppPtr, size_t nBytes) {
    return omb::status_of(cudaMallocHost(ppPtr, nBytes));
}

int omCudaFreeHost(void* pPtr) { return omb::status_of(cudaFreeHost(pPtr)); }

int omCudaGraphBeginCapture(void) {
    OMB_CTX_OR_FAIL(c);
    return omb::status_of(cudaStreamBeginCapture(c->compute, cudaStreamCaptureModeThreadLocal));
}

int omCudaGraphEndCapture(void** pGraphExec) {
    OMB_CTX_OR_FAIL(c);
    if (!pGraphExec) return OM_ERR_INVALID;
    cudaGraph_t g = nullptr;
    OMB_CHECK(cudaStreamEndCapture(c->compute, &g));
    cudaGraphExec_t ge = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return OM_ERR_CUDA;
    *pGraphExec = (void*)ge;
    return OM_OK;
}

int omCudaGraphLaunch(void* pGraphExec) {
    OMB_CTX_OR_FAIL(c);
    if (!pGraphExec) return OM_ERR_INVALID;
    return omb::status_of(cudaGraphLaunch((cudaGraphExec_t)pGraphExec, c->compute));
}

int omCudaGraphDestroy(void* pGraphExec) {
    if (!pGraphExec) return OM_OK;
    return omb::status_of(cudaGraphExecDestroy((cudaGraphExec_t)pGraphExec));
}

int omCudaGetKernelError(unsigned int* pCode) {
    OMB_CTX_OR_FAIL(c);
    if (!pCode) return OM_ERR_INVALID;
    OMB_CHECK(cudaStreamSynchronize(c->compute));
    OMB_CHECK(cudaMemcpy(pCode, c->err_word, sizeof(unsigned int), cudaMemcpyDeviceToHost));
    OMB_CHECK(cudaMemset(c->err_word, 0, sizeof(unsigned int)));
    return OM_OK;
}

int omCudaSynchronizeChecked(void) {
    unsigned int code = 0;
    int st = omCudaGetKernelError(&code);
    if (st != OM_OK) return st;
    return code ? OM_ERR_KERNEL_TIMEOUT : OM_OK;
}

int omCudaGetLaunchCount(unsigned long long* pCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pCount) return OM_ERR_INVALID;
    *pCount = c->launches;
    return OM_OK;
}

}  // extern "C"
