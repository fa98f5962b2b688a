// Data-parallel gradient exchange over NCCL: the working version of the reference's
// DataParallel::synchronizeGradients (om.engine.distributed.ixx:132-161), which is a stub that
// only names ncclAllReduce in a comment.
//
// One process (or host thread) per GPU. Each device joins one communicator (omNcclInit) whose
// collectives run on a communication stream of their own:
//   omCudaAllreduceAsync  enqueues an in-place all-reduce that starts once the compute work
//                         issued so far has finished, and runs while later compute work (the
//                         rest of the backward pass) proceeds;
//   omCudaAllreduceJoin   makes later compute work (the optimiser step) wait for every
//                         all-reduce issued so far;
//   omNcclPoll            watches the communicator from the host with a time limit.
//
// Failure handling. The communicator is created non-blocking and its initialisation is polled
// with a time limit; an NCCL call that reports an error, or a poll that runs out of time (a peer
// that died or never joined), aborts the communicator (ncclCommAbort) and every later call on
// it returns OM_ERR_COMM, so a rank never waits for good on a peer. Only host threads wait here;
// no kernel of this file spins.
//
// NCCL is loaded when a communicator is first needed, not linked: the process may already hold
// another NCCL build under the same soname (PyTorch's), and a library linked here would claim
// the soname first and break that one. The copy already loaded in the process is used when
// there is one, else $OM_NCCL_LIBRARY, else libnccl.so.2 from the loader's search path. The
// header is used for types only.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

#include "om_common.cuh"

namespace omb {
namespace dist {

struct NcclApi {
    ncclResult_t (*getUniqueId)(ncclUniqueId*);
    ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*commAbort)(ncclComm_t);
    ncclResult_t (*commFinalize)(ncclComm_t);
    ncclResult_t (*commDestroy)(ncclComm_t);
    ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t);
};
static NcclApi g_nccl;
static bool g_nccl_ok = false;

static bool load_nccl() {
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        const char* path = std::getenv("OM_NCCL_LIBRARY");
        if (!h && path && *path) h = dlopen(path, RTLD_NOW);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
        if (!h) return;
        bool ok = true;
        auto sym = [&](const char* name) {
            void* f = dlsym(h, name);
            ok = ok && f != nullptr;
            return f;
        };
        g_nccl.getUniqueId = reinterpret_cast<decltype(g_nccl.getUniqueId)>(sym("ncclGetUniqueId"));
        g_nccl.commInitRankConfig =
            reinterpret_cast<decltype(g_nccl.commInitRankConfig)>(sym("ncclCommInitRankConfig"));
        g_nccl.commGetAsyncError =
            reinterpret_cast<decltype(g_nccl.commGetAsyncError)>(sym("ncclCommGetAsyncError"));
        g_nccl.commAbort = reinterpret_cast<decltype(g_nccl.commAbort)>(sym("ncclCommAbort"));
        g_nccl.commFinalize = reinterpret_cast<decltype(g_nccl.commFinalize)>(sym("ncclCommFinalize"));
        g_nccl.commDestroy = reinterpret_cast<decltype(g_nccl.commDestroy)>(sym("ncclCommDestroy"));
        g_nccl.allReduce = reinterpret_cast<decltype(g_nccl.allReduce)>(sym("ncclAllReduce"));
        g_nccl_ok = ok;
    });
    return g_nccl_ok;
}

struct CommCtx {
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ready = nullptr;  // recorded on the compute stream, waited on by `stream`
    cudaEvent_t done = nullptr;   // recorded on `stream` after each collective
    int rank = -1;
    int world = 0;
    bool aborted = false;
};

static CommCtx g_comm[64];
// limit for an NCCL call that answers "in progress" (non-blocking communicators)
constexpr long long kCallLimitMs = 60000;

static long long now_ms() {
    using namespace std::chrono;
    return duration_cast<milliseconds>(steady_clock::now().time_since_epoch()).count();
}

static void release(CommCtx* cc) {
    if (cc->stream) cudaStreamDestroy(cc->stream);
    if (cc->ready) cudaEventDestroy(cc->ready);
    if (cc->done) cudaEventDestroy(cc->done);
    *cc = CommCtx();
}

static void abort_comm(CommCtx* cc) {
    if (cc->comm && !cc->aborted) g_nccl.commAbort(cc->comm);
    cc->comm = nullptr;
    cc->aborted = true;
}

// Polls the communicator until its pending host-side work (initialisation, or a collective
// that answered ncclInProgress) is complete, an error is reported, or limit_ms passes.
static int settle(CommCtx* cc, long long limit_ms) {
    const long long t0 = now_ms();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        if (g_nccl.commGetAsyncError(cc->comm, &st) != ncclSuccess) return OM_ERR_COMM;
        if (st == ncclSuccess) return OM_OK;
        if (st != ncclInProgress) return OM_ERR_COMM;
        if (now_ms() - t0 > limit_ms) return OM_ERR_COMM;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

static CommCtx* comm_of(DeviceCtx* c) {
    CommCtx* cc = &g_comm[c->device];
    return cc->comm && !cc->aborted ? cc : nullptr;
}

}  // namespace dist
}  // namespace omb

using omb::dist::CommCtx;

extern "C" {

int omNcclGetUniqueId(void* pId) {
    if (!pId) return OM_ERR_INVALID;
    static_assert(sizeof(ncclUniqueId) == OM_NCCL_ID_BYTES, "NCCL unique id size");
    if (!omb::dist::load_nccl()) return OM_ERR_UNSUPPORTED;
    ncclUniqueId id;
    if (omb::dist::g_nccl.getUniqueId(&id) != ncclSuccess) return OM_ERR_COMM;
    std::memcpy(pId, &id, sizeof(id));
    return OM_OK;
}

int omNcclInit(int nRank, int nWorld, const void* pId, int nTimeoutMs) {
    OMB_CTX_OR_FAIL(c);
    if (!pId || nWorld < 1 || nRank < 0 || nRank >= nWorld || nTimeoutMs <= 0)
        return OM_ERR_INVALID;
    if (!omb::dist::load_nccl()) return OM_ERR_UNSUPPORTED;
    CommCtx* cc = &omb::dist::g_comm[c->device];
    if (cc->comm) return OM_ERR_INVALID;  // one communicator per device
    omb::dist::release(cc);
    OMB_CHECK(cudaStreamCreateWithFlags(&cc->stream, cudaStreamNonBlocking));
    OMB_CHECK(cudaEventCreateWithFlags(&cc->ready, cudaEventDisableTiming));
    OMB_CHECK(cudaEventCreateWithFlags(&cc->done, cudaEventDisableTiming));
    ncclUniqueId id;
    std::memcpy(&id, pId, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = omb::dist::g_nccl.commInitRankConfig(&cc->comm, nWorld, id, nRank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (cc->comm) omb::dist::g_nccl.commAbort(cc->comm);
        omb::dist::release(cc);
        return OM_ERR_COMM;
    }
    if (omb::dist::settle(cc, nTimeoutMs) != OM_OK) {
        omb::dist::abort_comm(cc);
        omb::dist::release(cc);
        return OM_ERR_COMM;
    }
    cc->rank = nRank;
    cc->world = nWorld;
    return OM_OK;
}

int omCudaAllreduceAsync(float* pData, long long nCount, int nOp) {
    OMB_CTX_OR_FAIL(c);
    CommCtx* cc = omb::dist::comm_of(c);
    if (!cc) return OM_ERR_COMM;
    if (!pData || nCount < 0 || (nOp != OM_REDUCE_SUM && nOp != OM_REDUCE_MAX))
        return OM_ERR_INVALID;
    if (nCount == 0) return OM_OK;
    OMB_CHECK(cudaEventRecord(cc->ready, c->compute));
    OMB_CHECK(cudaStreamWaitEvent(cc->stream, cc->ready, 0));
    ncclResult_t r = omb::dist::g_nccl.allReduce(pData, pData, (size_t)nCount, ncclFloat32,
                                   nOp == OM_REDUCE_MAX ? ncclMax : ncclSum, cc->comm, cc->stream);
    if (r == ncclInProgress) r = omb::dist::settle(cc, omb::dist::kCallLimitMs) == OM_OK
                                     ? ncclSuccess : ncclInternalError;
    if (r != ncclSuccess) {
        omb::dist::abort_comm(cc);
        return OM_ERR_COMM;
    }
    return omb::status_of(cudaEventRecord(cc->done, cc->stream));
}

int omCudaAllreduceJoin(void) {
    OMB_CTX_OR_FAIL(c);
    CommCtx* cc = omb::dist::comm_of(c);
    if (!cc) return OM_ERR_COMM;
    // `done` was recorded after the last collective; the stream runs them in order
    return omb::status_of(cudaStreamWaitEvent(c->compute, cc->done, 0));
}

int omCudaAllreduce(float* pData, long long nCount, int nOp) {
    int st = omCudaAllreduceAsync(pData, nCount, nOp);
    return st != OM_OK ? st : omCudaAllreduceJoin();
}

int omNcclPoll(int nTimeoutMs) {
    OMB_CTX_OR_FAIL(c);
    CommCtx* cc = omb::dist::comm_of(c);
    if (!cc) return OM_ERR_COMM;
    const long long t0 = omb::dist::now_ms();
    for (;;) {
        cudaError_t q = cudaEventQuery(cc->done);
        ncclResult_t st = ncclSuccess;
        if (omb::dist::g_nccl.commGetAsyncError(cc->comm, &st) != ncclSuccess ||
            (st != ncclSuccess && st != ncclInProgress)) {
            omb::dist::abort_comm(cc);
            return OM_ERR_COMM;
        }
        if (q == cudaSuccess) return OM_OK;
        if (q != cudaErrorNotReady) return OM_ERR_CUDA;
        if (omb::dist::now_ms() - t0 > nTimeoutMs) {
            omb::dist::abort_comm(cc);
            return OM_ERR_COMM;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

int omNcclRankInfo(int* pRank, int* pWorld) {
    OMB_CTX_OR_FAIL(c);
    CommCtx* cc = omb::dist::comm_of(c);
    if (!cc) return OM_ERR_COMM;
    if (pRank) *pRank = cc->rank;
    if (pWorld) *pWorld = cc->world;
    return OM_OK;
}

int omNcclAbort(void) {
    OMB_CTX_OR_FAIL(c);
    CommCtx* cc = &omb::dist::g_comm[c->device];
    omb::dist::abort_comm(cc);
    omb::dist::release(cc);
    return OM_OK;
}

int omNcclDestroy(void) {
    OMB_CTX_OR_FAIL(c);
    CommCtx* cc = &omb::dist::g_comm[c->device];
    if (!cc->comm) {
        omb::dist::release(cc);
        return OM_OK;
    }
    int st = omb::status_of(cudaStreamSynchronize(cc->stream));
    // a non-blocking communicator finalises asynchronously: flush it, then free it
    ncclResult_t r = omb::dist::g_nccl.commFinalize(cc->comm);
    if (r == ncclInProgress) r = omb::dist::settle(cc, omb::dist::kCallLimitMs) == OM_OK
                                     ? ncclSuccess : ncclInternalError;
    if (r != ncclSuccess) {
        omb::dist::abort_comm(cc);
        omb::dist::release(cc);
        return OM_ERR_COMM;
    }
    if (omb::dist::g_nccl.commDestroy(cc->comm) != ncclSuccess) st = OM_ERR_COMM;
    cc->comm = nullptr;
    omb::dist::release(cc);
    return st;
}

}  // extern "C"
