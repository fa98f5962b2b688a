/*
 * om_cuda.h — C ABI of the B200 (sm_100a) compute backend for the OmniMatch engine.
 *
 * Drop-in for all 97 entry points of the reference's src/cuda/cuda_kernels.cuh: every
 * function below that carries a "replaces" line has the same name, argument order and
 * argument meaning as the reference entry point it names (cuda_kernels.cu:<line>), so the
 * reference's CUDABackend (src/hal/om.hal.cuda_backend.ixx) links against this library
 * unchanged. Functions marked "new" extend the ABI for NHWC / bf16 / fp16 fused execution.
 *
 * Conventions (same as the reference unless stated):
 *   - return 0 on success, a negative OM_* status on failure (the reference returns -1 for
 *     every failure; all our codes are negative, so `!= 0` checks keep working);
 *   - all pointers are device pointers unless the name says Host;
 *   - calls are asynchronous on the calling thread's current device's compute stream and
 *     stream-ordered with each other; omCudaSynchronize waits for them;
 *   - layouts of the reference ops are NCHW fp32; weights [Cout, Cin/groups, KH, KW];
 *   - one host thread may drive one device at a time (omCudaInit/omCudaSetDevice select it
 *     for the calling thread), so one process can drive all 8 GPUs from 8 threads.
 */
#ifndef OM_CUDA_H
#define OM_CUDA_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes (all failures are negative) */
#define OM_OK 0
#define OM_ERR_CUDA (-1)          /* a CUDA runtime call failed */
#define OM_ERR_INVALID (-2)       /* bad argument: size, alignment, null pointer */
#define OM_ERR_UNSUPPORTED (-3)   /* shape/dtype combination this kernel does not cover */
#define OM_ERR_NOT_INIT (-4)      /* omCudaInit was not called on this thread */
#define OM_ERR_OOM (-5)           /* device allocation failed after releasing the cache */
#define OM_ERR_KERNEL_TIMEOUT (-6)/* a bounded in-kernel wait gave up (see omCudaGetKernelError) */
#define OM_ERR_DRIVER (-7)        /* a driver entry point (tensor-map encode) was unavailable */
#define OM_ERR_TOO_LARGE (-8)     /* request exceeds the fixed capacity of an allocation-free entry point */
#define OM_ERR_COMM (-9)          /* a collective failed or timed out; the communicator was aborted */

/* element types for the NHWC entry points */
#define OM_DTYPE_F32 0
#define OM_DTYPE_BF16 1
#define OM_DTYPE_F16 2
/* 8-bit image samples (value = sample / 255): only as the image input of the stem entry points */
#define OM_DTYPE_U8 3

/* fused epilogue activations */
#define OM_ACT_NONE 0
#define OM_ACT_RELU 1
#define OM_ACT_RELU6 2

/* ---------------- device, memory, streams ---------------- */
int omCudaInit(int nDeviceId);                                         /* replaces :287 */
int omCudaGetDeviceCount(void);                                        /* replaces :299 */
int omCudaGetDeviceName(int nDeviceId, char* pNameBuf, int nBufSize);  /* replaces :306 */
int omCudaGetMemInfo(int nDeviceId, size_t* pFreeMem, size_t* pTotalMem); /* replaces :314 */
int omCudaGetComputeCapability(int nDeviceId, int* pMajor, int* pMinor);  /* replaces :324 */
int omCudaMalloc(void** ppDevPtr, size_t nBytes);                      /* replaces :336 */
int omCudaFree(void* pDevPtr);                                         /* replaces :345 */
int omCudaCopyH2D(void* pDst, const void* pSrc, size_t nBytes);        /* replaces :353 */
int omCudaCopyD2H(void* pDst, const void* pSrc, size_t nBytes);        /* replaces :365 */
int omCudaCopyD2D(void* pDst, const void* pSrc, size_t nBytes);        /* replaces :371 */
int omCudaMemset(void* pDev, int nValue, size_t nBytes);               /* replaces :377 */
int omCudaSynchronize(void);                                           /* replaces :383 */
int omCudaAsyncCopyH2D(void* pDst, const void* pSrc, size_t nBytes);   /* replaces :390 */
int omCudaAsyncCopyD2H(void* pDst, const void* pSrc, size_t nBytes);   /* replaces :397 */
int omCudaSyncTransferStream(void);                                    /* replaces :404 */
int omCudaSyncComputeStream(void);                                     /* replaces :412 */
int omCudaCleanup(void);                                               /* replaces :420 */
/* replaces :429 (declared by the engine at EngineBridge.cpp:143, called at :4047): wait for the
 * device, clear the last error, release cached pool blocks; no cudaDeviceReset */
int omCudaForceReset(void);
int omCudaMallocHost(void** ppPtr, size_t nBytes);                     /* replaces :4887 */
int omCudaFreeHost(void* pPtr);                                        /* replaces :4895 */
int omCudaGraphBeginCapture(void);                                     /* replaces :4909 */
int omCudaGraphEndCapture(void** pGraphExec);                          /* replaces :4919 */
int omCudaGraphLaunch(void* pGraphExec);                               /* replaces :4941 */
int omCudaGraphDestroy(void* pGraphExec);                              /* replaces :4949 */
/* new: copies on the device's transfer stream, and ordering between the transfer and compute
 * streams, so a serving loop can upload step i+1's input while step i computes:
 * omCudaTransferH2D/D2H enqueue on the transfer stream; omCudaComputeWaitTransfer makes later
 * compute work wait for the transfer work issued so far, omCudaTransferWaitCompute the
 * opposite (e.g. before overwriting an input buffer the previous step still reads). */
int omCudaTransferH2D(void* pDst, const void* pSrcHost, size_t nBytes);
int omCudaTransferD2H(void* pDstHost, const void* pSrc, size_t nBytes);
int omCudaComputeWaitTransfer(void);
int omCudaTransferWaitCompute(void);
/* new: select the calling thread's device (must have been omCudaInit'ed once per thread) */
int omCudaSetDevice(int nDeviceId);
/* new: the compute stream of the calling thread's device, as a cudaStream_t */
void* omCudaGetStream(void);
/* new: the calling thread's current device (set by omCudaInit / omCudaSetDevice), -1 if none */
int omCudaGetCurrentDevice(void);
/* new: device-side gather of a strided fp32 view into a contiguous buffer (Tensor::contiguous
 * without the host round trip of om.engine.tensor.ixx:390-391):
 * dst[i] = src[nOffset + sum_d coord_d(i) * pStrides[d]], with coord(i) the row-major coordinates
 * of i in pShape. pShape / pStrides are host arrays of nDims <= 8 entries (elements, >= 0). */
int omCudaStridedCopy(const float* pSrc, float* pDst, const int* pShape, const int* pStrides,
                      int nDims, long long nOffset);
/* new: read and clear the device error word that bounded in-kernel waits set; *pCode is 0
 * when no kernel gave up since the last call. Synchronises the compute stream. */
int omCudaGetKernelError(unsigned int* pCode);
/* new: wait for the compute stream, then OM_ERR_KERNEL_TIMEOUT if a bounded in-kernel wait gave
 * up since the last check (the error word is read and cleared), else OM_OK */
int omCudaSynchronizeChecked(void);
/* new, for tests of the bounded waits: the next tensor-core conv launch on the calling thread's
 * device gets role waits limited to nWaitNs (1 ms .. 2 s) and a producer that stops issuing
 * loads after nLoadsBeforeStall of them, so the MMA issuer waits for a load that never comes
 * and gives up; every load issued has landed before the kernel exits. One launch only. */
int omCudaTestStallNextConv(long long nLoadsBeforeStall, unsigned long long nWaitNs);
/* new: number of kernels this library has launched on the calling thread's device */
int omCudaGetLaunchCount(unsigned long long* pCount);

/* ---------------- elementwise / fills (fp32) ---------------- */
int omCudaAdd(const float* pA, const float* pB, float* pC, int nCount);          /* replaces :467 */
int omCudaMulScalar(const float* pA, float fScalar, float* pC, int nCount);      /* replaces :542 */
int omCudaReLU(const float* pIn, float* pOut, int nCount);                       /* replaces :585 */
int omCudaReLUBackward(const float* pIn, const float* pGradOut, float* pGradIn, int nCount); /* :600 */
int omCudaClip(const float* pIn, float* pOut, int nCount, float fMin, float fMax); /* replaces :3763 */
int omCudaFillZeros(float* pData, int nCount);                                   /* replaces :2346 */
int omCudaFillOnes(float* pData, int nCount);                                    /* replaces :2363 */
int omCudaFillValue(float* pData, int nCount, float fValue);                     /* replaces :2380 */
int omCudaCopy(const float* pSrc, float* pDst, int nCount);                      /* replaces :2388 */
int omCudaSum(const float* pData, float* pResult, int nCount);                   /* replaces :1473 */
int omCudaArgmax(const float* pData, int* pOut, int nBatch, int nClasses);       /* replaces :2415 */
int omCudaTranspose(const float* pIn, float* pOut, int nRows, int nCols);        /* replaces :707 */
int omCudaSub(const float* pA, const float* pB, float* pC, int nCount);          /* replaces :493 */
int omCudaMul(const float* pA, const float* pB, float* pC, int nCount);          /* replaces :518 */
int omCudaDiv(const float* pA, const float* pB, float* pC, int nCount);          /* replaces :3743 */
int omCudaAddScalar(const float* pA, float fScalar, float* pC, int nCount);      /* replaces :566 */
/* *pResult (device) = sum / nCount */
int omCudaMean(const float* pData, float* pResult, int nCount);                  /* replaces :1506 */
/* activations and their backwards; the Sigmoid / Tanh backwards take the forward output,
 * the GELU (tanh form) / SiLU / LeakyReLU backwards the forward input */
int omCudaSigmoid(const float* pIn, float* pOut, int nCount);                    /* replaces :615 */
int omCudaSigmoidBackward(const float* pGrad, const float* pOutput, float* pOut, int nCount); /* :1978 */
int omCudaTanh(const float* pIn, float* pOut, int nCount);                       /* replaces :1889 */
int omCudaTanhBackward(const float* pGrad, const float* pOutput, float* pOut, int nCount); /* :1910 */
int omCudaGELU(const float* pIn, float* pOut, int nCount);                       /* replaces :635 */
int omCudaGeluBackward(const float* pGrad, const float* pInput, float* pOut, int nCount); /* :1936 */
int omCudaSiLU(const float* pIn, float* pOut, int nCount);                       /* replaces :653 */
int omCudaSiluBackward(const float* pGrad, const float* pInput, float* pOut, int nCount); /* :1957 */
int omCudaLeakyRelu(const float* pIn, float* pOut, int nCount, float fSlope);    /* replaces :1871 */
int omCudaLeakyReluBackward(const float* pGrad, const float* pInput, float* pOut, int nCount,
                            float fSlope);                                       /* replaces :1997 */

/* ---------------- dense contractions (fp32, reference layouts) ---------------- */
/* C[M,N] = A[M,K] . B[K,N], row-major */
int omCudaMatmul(const float* pA, const float* pB, float* pC, int nM, int nK, int nN); /* :768 */
/* out = conv(in, w) + b, NCHW; pBias may be NULL */
int omCudaConv2d(const float* pInput, const float* pWeight, const float* pBias, float* pOutput,
                 int nBatch, int nCin, int nH, int nW, int nCout, int nKH, int nKW,
                 int nStride, int nPad);                                         /* replaces :1076 */
/* grouped / dilated direct conv (groups == Cin == Cout is depthwise) */
int omCudaDilatedConv2d(const float* pInput, const float* pWeight, const float* pBias,
                        float* pOutput, int nBatch, int nCin, int nH, int nW, int nCout,
                        int nKH, int nKW, int nStride, int nPad, int nDilation,
                        int nGroups);                                            /* replaces :1201 */
/* dX = conv^T(dY, W); overwrites pGradInput */
int omCudaConv2dBackwardInput(const float* pGradOutput, const float* pWeight, float* pGradInput,
                              int nBatch, int nCin, int nH, int nW, int nCout, int nKH, int nKW,
                              int nStride, int nPad);                            /* replaces :2600 */
/* dW = sum_n dY (x) im2col(X), dB = sum dY; overwrites both (pGradBias may be NULL) */
int omCudaConv2dBackwardWeight(const float* pInput, const float* pGradOutput, float* pGradWeight,
                               float* pGradBias, int nBatch, int nCin, int nH, int nW,
                               int nCout, int nKH, int nKW, int nStride, int nPad); /* :2739 */

/* ---------------- normalisation, pooling, losses, optimiser (fp32 NCHW) ---------------- */
int omCudaBatchNorm2d(const float* pInput, float* pOutput, const float* pGamma,
                      const float* pBeta, float* pRunMean, float* pRunVar, float* pSavedMean,
                      float* pSavedInvStd, int nBatch, int nChannels, int nH, int nW,
                      float fEps, float fMomentum, int bTraining);              /* replaces :1648 */
/* No counterpart in the reference. Same arguments and results as omCudaBatchNorm2d, for
 * callers that must not allocate device memory once they are running (for example an
 * inspection loop that reserved its whole VRAM budget at start-up, or an engine embedded in a
 * host whose allocator owns the device): it never calls cudaMalloc/cudaFree or an allocating
 * routine. Training-mode statistics use a fixed 2 MiB per-device array inside this library
 * (up to 4096 channels; more returns OM_ERR_TOO_LARGE without launching). The first call on a
 * device looks that array up; make that first call before any stream capture. All calls on a
 * device share the array, so calls whose kernels overlap on the GPU race with each other. */
int omCudaBatchNorm2dNoAlloc(const float* pInput, float* pOutput, const float* pGamma,
                             const float* pBeta, float* pRunMean, float* pRunVar,
                             float* pSavedMean, float* pSavedInvStd, int nBatch, int nChannels,
                             int nH, int nW, float fEps, float fMomentum, int bTraining);
int omCudaBatchNorm2dBackward(const float* pGradOutput, const float* pInput, const float* pMean,
                              const float* pInvStd, const float* pGamma, float* pGradInput,
                              float* pGradGamma, float* pGradBeta, int nBatch, int nChannels,
                              int nH, int nW, float fEps);                       /* replaces :3130 */
/* new: BatchNorm with the activation that follows it (nAct: OM_ACT_NONE or OM_ACT_RELU)
 * applied in the same pass, for conv -> BN -> ReLU chains (the reference calls :1648 and then
 * its ReLU kernel). Same arguments as omCudaBatchNorm2d plus nAct; pOutput receives the
 * activated result, bit-identical to omCudaBatchNorm2d followed by omCudaReLU. */
int omCudaBatchNorm2dAct(const float* pInput, float* pOutput, const float* pGamma,
                         const float* pBeta, float* pRunMean, float* pRunVar, float* pSavedMean,
                         float* pSavedInvStd, int nBatch, int nChannels, int nH, int nW,
                         float fEps, float fMomentum, int bTraining, int nAct);
/* new: train-mode conv -> BatchNorm (-> ReLU) with the BatchNorm statistics taken in the
 * convolution's epilogue (the reference calls :1076, then :1648 and its ReLU kernel). The conv
 * (arguments as omCudaConv2d, square stride and padding) writes pConvOut [N, Cout, P, Q]; the
 * BatchNorm (arguments as omCudaBatchNorm2d, always training: batch statistics with the biased
 * variance, running statistics updated with fMomentum) writes pOutput with nAct (OM_ACT_NONE or
 * OM_ACT_RELU) applied, and the saved mean and 1/sqrt(var + eps) its backward needs. The
 * statistics are combined in a fixed order, so the result is deterministic; they agree with
 * omCudaBatchNorm2d's two-pass statistics to fp32 rounding. pConvOut is written once and read
 * once. pInputSplit (may be NULL): a device buffer of omCudaConvInputSplitBytes(nBatch, nCin,
 * nH, nW, nStride) bytes (when that is not 0) that receives the convolution's tensor-core copy
 * of pInput and keeps it for omCudaConv2dBackwardWeightSplit, which then does not make it
 * again. */
int omCudaConv2dBatchNorm2dAct(const float* pInput, const float* pWeight, const float* pBias,
                               float* pConvOut, float* pOutput, const float* pGamma,
                               const float* pBeta, float* pRunMean, float* pRunVar,
                               float* pSavedMean, float* pSavedInvStd, int nBatch, int nCin,
                               int nH, int nW, int nCout, int nKH, int nKW, int nStride, int nPad,
                               float fEps, float fMomentum, int nAct, void* pInputSplit);
/* new: omCudaConv2dBatchNorm2dAct with a residual branch pResidual [N, Cout, P, Q] added to the
 * normalised output before nAct (a ResNet block's last conv, its shortcut add and the block's
 * ReLU): pOutput = act(BN(conv) + pResidual). Bit-identical to omCudaConv2dBatchNorm2dAct with
 * OM_ACT_NONE, omCudaAdd and omCudaReLU; pOutput > 0 is the block ReLU's backward mask. */
int omCudaConv2dBatchNorm2dAddAct(const float* pInput, const float* pWeight, const float* pBias,
                                  float* pConvOut, float* pOutput, const float* pGamma,
                                  const float* pBeta, float* pRunMean, float* pRunVar,
                                  float* pSavedMean, float* pSavedInvStd, int nBatch, int nCin,
                                  int nH, int nW, int nCout, int nKH, int nKW, int nStride,
                                  int nPad, float fEps, float fMomentum, int nAct,
                                  void* pInputSplit, const float* pResidual);
/* new: bytes of the kept input copy that omCudaConv2dBatchNorm2dAct writes and
 * omCudaConv2dBackwardWeightSplit reads (the hi and lo fp32 parts of the NHWC input with the
 * channels padded to 32); 0 when the weight gradient of this shape makes its own copy (stride-2
 * convs of at most 8 input channels) or the arguments are invalid */
long long omCudaConvInputSplitBytes(int nBatch, int nCin, int nH, int nW, int nStride);
/* new: omCudaConv2dBatchNorm2dAct for the image stem (stride 2, at most 8 input channels) with
 * the convolution in its space-to-depth form: a stride-1 ceil(KH/2) x ceil(KW/2) convolution
 * over a 32-channel copy of the image holding each 2x2 block's pixels as channels (16 taps of 32
 * channels for the 7x7/2 ImageNet stem instead of 49 taps of 3). Same arguments and outputs;
 * the sums run in another order, so results agree with omCudaConv2dBatchNorm2dAct to fp32
 * rounding, not bit for bit. pInputSplit (may be NULL): a device buffer of
 * omCudaStemInputSplitBytes(...) bytes that keeps that copy for
 * omCudaConv2dBackwardWeightSplit. OM_ERR_UNSUPPORTED for any other shape. */
int omCudaStemConv2dBatchNorm2dAct(const float* pInput, const float* pWeight, const float* pBias,
                                   float* pConvOut, float* pOutput, const float* pGamma,
                                   const float* pBeta, float* pRunMean, float* pRunVar,
                                   float* pSavedMean, float* pSavedInvStd, int nBatch, int nCin,
                                   int nH, int nW, int nCout, int nKH, int nKW, int nStride,
                                   int nPad, float fEps, float fMomentum, int nAct,
                                   void* pInputSplit);
/* new: bytes of the space-to-depth copy omCudaStemConv2dBatchNorm2dAct keeps (hi and lo fp32
 * parts of [N, P + ceil(KH/2) - 1, Q + ceil(KW/2) - 1, 32]); 0 for shapes it does not take */
long long omCudaStemInputSplitBytes(int nBatch, int nCin, int nH, int nW, int nKH, int nKW,
                                    int nStride, int nPad);
/* new: omCudaConv2dBackwardWeight reading the input's kept copy (pInputSplit, written by the
 * forward omCudaConv2dBatchNorm2dAct of the same pInput and shape, or for the stem shapes by
 * omCudaStemConv2dBatchNorm2dAct, unchanged since) instead of copying pInput again; pInput is
 * still read where the tensor path does not take the shape. Bit-identical to
 * omCudaConv2dBackwardWeight. */
int omCudaConv2dBackwardWeightSplit(const float* pInput, const void* pInputSplit,
                                    const float* pGradOutput, float* pGradWeight,
                                    float* pGradBias, int nBatch, int nCin, int nH, int nW,
                                    int nCout, int nKH, int nKW, int nStride, int nPad);
/* new: a conv's whole backward, omCudaConv2dBackwardInput (skipped when pGradInput is NULL)
 * then omCudaConv2dBackwardWeightSplit (pInputSplit may be NULL: omCudaConv2dBackwardWeight),
 * with one tensor-core copy of pGradOutput read by both passes instead of one copy each.
 * Bit-identical to the two calls. */
int omCudaConv2dBackwardSplit(const float* pGradOutput, const float* pInput,
                              const void* pInputSplit, const float* pWeight, float* pGradInput,
                              float* pGradWeight, float* pGradBias, int nBatch, int nCin, int nH,
                              int nW, int nCout, int nKH, int nKW, int nStride, int nPad);
/* new: the backward of omCudaBatchNorm2dAct (the reference calls its ReLU backward, then :3130). pOutput is the
 * forward's activated output: the incoming gradient is zeroed where pOutput <= 0 inside the BN
 * backward passes. Bit-identical to omCudaReLUBackward followed by omCudaBatchNorm2dBackward. */
int omCudaBatchNorm2dBackwardAct(const float* pGradOutput, const float* pInput,
                                 const float* pMean, const float* pInvStd, const float* pGamma,
                                 const float* pOutput, float* pGradInput, float* pGradGamma,
                                 float* pGradBeta, int nBatch, int nChannels, int nH, int nW,
                                 float fEps, int nAct);
int omCudaMaxPool2d(const float* pIn, float* pOut, int* pIndices, int nN, int nC, int nH, int nW,
                    int nKH, int nKW, int nSH, int nSW, int nPH, int nPW);       /* replaces :2052 */
/* accumulates into pGradIn (callers zero it first, as CUDABackend::maxPool2dBackward does) */
int omCudaMaxPool2dBackward(const float* pGradOut, const int* pIndices, float* pGradIn, int nN,
                            int nC, int nH, int nW, int nHout, int nWout);       /* replaces :2083 */
/* new: the max-pool backward with the window geometry (as omCudaMaxPool2d), as a gather: each
 * element of pGradIn is written (not accumulated; no zeroing needed) with the sum of the output
 * gradients whose argmax picked it, added in increasing output order. That is the reference CPU
 * backend's loop (cpu_backend.ixx:937-953) sum for sum: deterministic, unlike the scatter with
 * atomics of omCudaMaxPool2dBackward where windows overlap. */
int omCudaMaxPool2dBackwardGather(const float* pGradOut, const int* pIndices, float* pGradIn,
                                  int nN, int nC, int nH, int nW, int nKH, int nKW, int nSH,
                                  int nSW, int nPH, int nPW);
int omCudaAvgPool2d(const float* pIn, float* pOut, int nN, int nC, int nH, int nW, int nKH,
                    int nKW, int nSH, int nSW, int nPH, int nPW);                /* replaces :2127 */
/* accumulates into pGradIn (callers zero it first) */
int omCudaAvgPool2dBackward(const float* pGradOut, float* pGradIn, int nN, int nC, int nH,
                            int nW, int nKH, int nKW, int nSH, int nSW, int nPH, int nPW); /* :2175 */
int omCudaAdaptiveAvgPool2d(const float* pIn, float* pOut, int nN, int nC, int nH, int nW,
                            int nOutH, int nOutW);                               /* replaces :2225 */
int omCudaAdaptiveAvgPool2dBackward(const float* pGradOut, float* pGradIn, int nBatch,
                                    int nChannels, int nH, int nW, int nOutH, int nOutW); /* :3532 */
/* out[n,c,hw] = in[n,c,hw] + bias[c] */
int omCudaAddBias(const float* pData, const float* pBias, float* pOut, int nN, int nC, int nHW); /* :2253 */
/* gradBias[c] = sum_{n,hw} gradOut[n,c,hw] (overwrites) */
int omCudaAddBiasBackward(const float* pGradOut, float* pGradBias, int nN, int nC, int nHW); /* :3569 */
/* row softmax; divides by the plain sum as the CPU backend does (cpu_backend.ixx:352-370) */
int omCudaSoftmax(const float* pIn, float* pOut, int nBatch, int nClasses);      /* replaces :1456 */
/* *pResult (device) = -sum_{target>0.5} log(max(p,1e-7)) / nBatch (cpu_backend.ixx:375-388) */
int omCudaCrossEntropy(const float* pSoftmax, const float* pTarget, float* pResult, int nBatch,
                       int nClasses);                                            /* replaces :3973 */
int omCudaSoftmaxCrossEntropyBackward(const float* pSoftmax, const float* pTarget,
                                      float* pGradLogits, int nBatch, int nClasses); /* :2539 */
/* new: softmax (:1387), cross-entropy (:3934) and its gradient (:2539) in one pass over the
 * logits, with the CPU backend's semantics: pSoftmax (may be NULL) = softmax(logits), *pLoss
 * (device) = -sum over targets > 0.5 of log(max(p, 1e-7)) / nBatch, pGradLogits = (p - t) /
 * nBatch. The loss is summed in a fixed order (deterministic) through a per-device array that
 * every call shares: two calls on one device must not overlap. nBatch <= 65536. */
int omCudaSoftmaxCrossEntropyFused(const float* pLogits, const float* pTarget, float* pSoftmax,
                                   float* pGradLogits, float* pLoss, int nBatch, int nClasses);
/* v = m*v + g; p -= lr*v (m == 0 or pVelocity == NULL: p -= lr*g) */
int omCudaSgdStep(float* pParam, const float* pGrad, float* pVelocity, int nCount, float fLr,
                  float fMomentum);                                              /* replaces :2511 */
/* new: omCudaSgdStep on fGradScale * grad (1/world after a summing all-reduce), one pass */
int omCudaSgdStepScaled(float* pParam, const float* pGrad, float* pVelocity, int nCount,
                        float fLr, float fMomentum, float fGradScale);
/* new: the training loop's gradient guard (EngineBridge.cpp:1885-1925) on the device, in place of
 * its per-step host copy of every gradient. pStatus (device, 3 floats) receives the L2 norm (NaN
 * when an element is not finite), the verdict (1 = step, 0 = skip: a NaN/Inf element) and the
 * clip coefficient. When the step goes ahead, pGrad is multiplied by fMaxNorm / norm if the norm
 * exceeds fMaxNorm (fMaxNorm <= 0: no clipping), then by fAccumScale (1 = none); when it is
 * skipped, pGrad is left unchanged. The reduction order is fixed (deterministic). Its partial
 * sums and last-block ticket live in a per-device array that every call shares: two calls on
 * one device must not overlap (for example from graphs replayed on different streams). */
int omCudaGradNormClip(float* pGrad, int nCount, float fMaxNorm, float fAccumScale, float* pStatus);
/* new: omCudaSgdStep that does nothing when the guard's verdict pStatus[1] is 0, so a skipped
 * step needs no host round trip */
int omCudaSgdStepGuarded(float* pParam, const float* pGrad, float* pVelocity, int nCount,
                         float fLr, float fMomentum, const float* pStatus);
/* Adam with bias correction (beta^step from nStep >= 1) */
int omCudaAdamStep(float* pParam, const float* pGrad, float* pM, float* pV, int nCount,
                   float fLr, float fBeta1, float fBeta2, float fEps, int nStep); /* :2468 */

/* ---------------- off the hot path: the reference's remaining entry points ----------------
 * Plain SIMT kernels with the reference's arithmetic, for the engine's segmentation and
 * transformer models. Reductions run in a fixed order (deterministic); the reference's
 * host round trips for loss values are replaced by device-side finishing. */
/* C[b] = A[b][M,K] . B[b][K,N], batches contiguous */
int omCudaBatchedMatmul(const float* pA, const float* pB, float* pC, int nBatch, int nM, int nK,
                        int nN);                                                 /* replaces :843 */
/* same as omCudaConv2d */
int omCudaConv2dIm2col(const float* pInput, const float* pWeight, const float* pBias,
                       float* pOutput, int nBatch, int nCin, int nH, int nW, int nCout, int nKH,
                       int nKW, int nStride, int nPad);                          /* replaces :991 */
/* weight [Cin, Cout, KH, KW]; output side (in-1)*stride - 2*pad + K; pBias may be NULL */
int omCudaConvTranspose2d(const float* pInput, const float* pWeight, const float* pBias,
                          float* pOutput, int nBatch, int nCin, int nHin, int nWin, int nCout,
                          int nKH, int nKW, int nStride, int nPad);              /* replaces :4187 */
/* dW and dB (pGradBias may be NULL) of a dilated convolution, overwritten */
int omCudaDilatedConv2dBackwardWeight(const float* pInput, const float* pGradOutput,
                                      float* pGradWeight, float* pGradBias, int nBatch,
                                      int nCin, int nH, int nW, int nCout, int nKH, int nKW,
                                      int nStride, int nPad, int nDilation);     /* :2911 */
/* LayerNorm over the last nDim of nBatch rows, saving mean and 1/sqrt(var + eps) per row */
int omCudaLayerNorm(const float* pInput, float* pOutput, const float* pGamma, const float* pBeta,
                    float* pSavedMean, float* pSavedInvStd, int nBatch, int nDim,
                    float fEps);                                                 /* replaces :1829 */
int omCudaLayerNormBackward(const float* pGradOut, const float* pInput, const float* pMean,
                            const float* pInvStd, const float* pGamma, float* pGradInput,
                            float* pGradGamma, float* pGradBeta, int nBatch, int nDim); /* :4096 */
/* GroupNorm of NCHW with nGroups channel groups; saves per (n, group) mean and invstd */
int omCudaGroupNorm2d(const float* pInput, float* pOutput, const float* pGamma, const float* pBeta,
                      float* pSavedMean, float* pSavedInvStd, int nBatch, int nChannels, int nH,
                      int nW, int nGroups, float fEps);                          /* replaces :3299 */
int omCudaGroupNorm2dBackward(const float* pGradOutput, const float* pInput, const float* pMean,
                              const float* pInvStd, const float* pGamma, float* pGradInput,
                              float* pGradGamma, float* pGradBeta, int nBatch, int nChannels,
                              int nH, int nW, int nGroups, float fEps);          /* :3458 */
/* dx = s * (dy - sum(dy * s)) per row */
int omCudaSoftmaxLastDimBackward(const float* pGradOut, const float* pSoftmax, float* pGradIn,
                                 int nOuter, int nLastDim);                      /* :4409 */
/* bilinear resize (half-pixel centres, clamped edges); the backward zeroes pGradIn first */
int omCudaUpsampleBilinear(const float* pIn, float* pOut, int nBatch, int nChannels, int nH,
                           int nW, int nOutH, int nOutW);                        /* replaces :3825 */
int omCudaUpsampleBilinearBackward(const float* pGradOut, float* pGradIn, int nBatch,
                                   int nChannels, int nInH, int nInW, int nOutH, int nOutW); /* :3639 */
int omCudaConcatChannels(const float* pA, const float* pB, float* pOut, int nBatch, int nC1,
                         int nC2, int nHW);                                      /* replaces :3866 */
int omCudaConcatChannelsBackward(const float* pGradOut, float* pGradA, float* pGradB, int nBatch,
                                 int nCA, int nCB, int nHW);                     /* :3686 */
int omCudaConcatLastDim(const float* pA, const float* pB, float* pOut, int nOuter, int nDimA,
                        int nDimB);                                              /* replaces :4244 */
int omCudaConcatLastDimBackward(const float* pGradOut, float* pGradA, float* pGradB, int nOuter,
                                int nDimA, int nDimB);                           /* :4281 */
/* columns [nStart, nStart + nLen) of each row; the backward writes only those columns */
int omCudaSliceLastDim(const float* pIn, float* pOut, int nOuter, int nFullDim, int nStart,
                       int nLen);                                                /* replaces :4315 */
int omCudaSliceLastDimBackward(const float* pGradOut, float* pGradIn, int nOuter, int nFullDim,
                               int nStart, int nLen);                            /* :4345 */
/* [N, S, 3, H, Dh] -> Q (times fScale), K, V as [N, H, S, Dh]; and [N, H, S, Dh] -> [N, S, H*Dh] */
int omCudaQkvSplitHeads(const float* pQkv, float* pQ, float* pK, float* pV, int nBatch,
                        int nSeqLen, int nHeads, int nHeadDim, float fScale);    /* :4854 */
int omCudaMergeHeads(const float* pIn, float* pOut, int nBatch, int nSeqLen, int nHeads,
                     int nHeadDim);                                              /* replaces :4866 */
/* *pResult (device) = sum of max(x,0) - x*y + log(1 + exp(-|x|)); grad (sigmoid(x) - y) * fInvN */
int omCudaBCEWithLogits(const float* pLogits, const float* pTargets, float* pResult,
                        int nCount);                                             /* replaces :3921 */
int omCudaBCEWithLogitsBackward(const float* pLogits, const float* pTargets, float* pGradLogits,
                                int nCount, float fInvN);                        /* :3717 */
/* soft Dice on sigmoid(logits): pStats = (sum s*t, sum s, sum t), *pLoss = 1 - 2 I/(P+T+1e-6) */
int omCudaDiceLossForward(const float* pLogits, const float* pTarget, float* pLoss,
                          float* pSigmoidOut, float* pStats, int nCount);        /* :4541 */
int omCudaDiceLossBackward(const float* pSigmoidOut, const float* pTarget, const float* pStats,
                           const float* pGradOutput, float* pGradLogits, int nCount); /* :4575 */
/* class-weighted focal (gamma 2) cross-entropy per pixel of [B, K, S] logits against class-id
 * targets; pStats = (weighted loss sum, weight sum), *pLoss = their ratio */
int omCudaWeightedPixelCEForward(const float* pLogits, const float* pTarget,
                                 const float* pClassWeights, float* pSoftmax, float* pLoss,
                                 float* pStats, int nPixels, int nClasses, int nSpatial); /* :4747 */
int omCudaWeightedPixelCEBackward(const float* pSoftmax, const float* pTarget,
                                  const float* pClassWeights, const float* pGradOutput,
                                  const float* pStats, float* pGradLogits, int nPixels,
                                  int nClasses, int nSpatial);                   /* :4778 */
/* out = in * mask / (1 - p) when training with p > 0, else a copy */
int omCudaDropout(const float* pIn, float* pOut, const float* pMask, int nCount, float fProb,
                  int bTraining);                                                /* replaces :2279 */
/* mask from the reference's per-index hash of nSeed: 1/keep with probability keep, else 0 */
int omCudaDropoutForward(const float* pIn, float* pOut, float* pMask, int nCount,
                         float fKeepProb, unsigned long long nSeed);             /* :2324 */

/* ---------------- new: data-parallel gradient exchange over NCCL ----------------
 * Replaces the stub DataParallel::synchronizeGradients (om.engine.distributed.ixx:132-161),
 * which names ncclAllReduce but does nothing. One communicator per device, joined by the
 * thread that drives the device; its collectives run on a communication stream of their own.
 * Every failure (an NCCL error, a time limit passed) aborts the communicator: later calls on it
 * return OM_ERR_COMM instead of waiting for a peer that is gone. */
#define OM_NCCL_ID_BYTES 128
#define OM_REDUCE_SUM 0
#define OM_REDUCE_MAX 1
/* rank 0 creates the communicator's id (OM_NCCL_ID_BYTES opaque bytes) and hands it to all ranks */
int omNcclGetUniqueId(void* pId);
/* the calling thread's device joins as nRank of nWorld; initialisation is non-blocking and
 * polled for at most nTimeoutMs (a rank that never joins makes every rank return OM_ERR_COMM) */
int omNcclInit(int nRank, int nWorld, const void* pId, int nTimeoutMs);
/* in-place all-reduce (sum or max) of nCount floats that starts once the compute work issued
 * so far has finished and overlaps the compute work issued after it */
int omCudaAllreduceAsync(float* pData, long long nCount, int nOp);
/* later compute work waits for every all-reduce issued so far (stream-ordered, no host wait) */
int omCudaAllreduceJoin(void);
/* omCudaAllreduceAsync + omCudaAllreduceJoin */
int omCudaAllreduce(float* pData, long long nCount, int nOp);
/* host: wait up to nTimeoutMs for the issued all-reduces, polling the communicator's error
 * state; an error or the time limit aborts the communicator and returns OM_ERR_COMM */
int omNcclPoll(int nTimeoutMs);
/* rank and world size of the device's communicator */
int omNcclRankInfo(int* pRank, int* pWorld);
/* abort the communicator (pending collectives are cancelled) and release it */
int omNcclAbort(void);
/* finalise and release the communicator after its work has finished */
int omNcclDestroy(void);

/* ---------------- new: NHWC bf16/fp16 fused inference path ---------------- */
/* Elements of the packed K-major weight [Cout, Kpad] that omCudaPackConvWeight writes, where
 * Kpad = round_up(KH*KW*Cs, 64) and Cs = stored input channels (omCudaStoredChannels). */
long long omCudaPackedConvWeightElems(int nCout, int nKH, int nKW, int nCs);
/* stored channel count for an NHWC activation with nC logical channels: nC when it is a
 * multiple of 64, else nC rounded up to a multiple of 8 */
int omCudaStoredChannels(int nC);
/* Fold eval-mode BatchNorm (gamma,beta,mean,var,eps; any may be NULL for "no BN") and an
 * optional conv bias into a packed K-major weight (dtype) and an fp32 bias[Cout]:
 * w' = w*gamma/sqrt(var+eps), b' = beta + (b - mean)*gamma/sqrt(var+eps). */
int omCudaPackConvWeight(const float* pWeight, const float* pConvBias, const float* pGamma,
                         const float* pBeta, const float* pMean, const float* pVar, float fEps,
                         void* pPacked, float* pBiasOut, int nCout, int nCin, int nKH, int nKW,
                         int nCs, int nDtype);
/* Implicit-GEMM conv on tcgen05 tensor cores, NHWC, no im2col buffer:
 *   out[n,p,q,k] = act( sum_{r,s,c} in[n, p*st-pad+r, q*st-pad+s, c] * W'[k,(r,s,c)]
 *                       + bias[k] + residual[n,p,q,k] )
 * in: [N,H,W,Cs] (nDtype), out/residual: [N,P,Q,Cout] (nOutDtype; residual may be NULL),
 * bias fp32 [Cout] (may be NULL), W' from omCudaPackConvWeight. Cs % 8 == 0, Cout % 8 == 0. */
int omCudaConv2dBnAct(const void* pInput, const void* pPacked, const float* pBias,
                      const void* pResidual, void* pOutput, int nBatch, int nH, int nW, int nCs,
                      int nCout, int nKH, int nKW, int nStride, int nPad, int nAct, int nDtype,
                      int nOutDtype);
/* new: the tile plan omCudaConv2dBnAct picks on the current device for these arguments (no
 * launch): pPlan[0] = tile width BN (32/64/128/256 output channels), [1] = CTAs per SM,
 * [2] = 128-row sub-tiles per tile, [3] = epilogue warps. For tests that must cover a variant. */
int omCudaConvTilePlan(int nBatch, int nH, int nW, int nCs, int nCout, int nKH, int nKW,
                       int nStride, int nPad, int bResidual, int* pPlan);
/* new: launch-duration stamps for measurement. With pStamps (device, 2 * nCapacity u64) set,
 * every tcgen05 conv launch on the calling thread's device (omCudaConv2dBnAct, the stem, the
 * fp32 3xTF32 convs) takes one pair per CTA, in launch order: %globaltimer (ns) at the CTA's
 * start and at its end; a launch that no longer fits records nothing. NULL switches it off.
 * Each call resets the launch list. A launch captured into a CUDA graph keeps its slots. */
int omCudaConvStamps(unsigned long long* pStamps, int nCapacity);
/* the launches recorded since omCudaConvStamps: first pair index and CTA count of each (up to
 * nMax of them); *pCount = number recorded */
int omCudaConvStampLaunches(int* pFirst, int* pCtas, int nMax, int* pCount);
/* new: a conv and the 1x1 conv after it in one kernel (a bottleneck's 3x3 and its expansion):
 *   mid = act1(conv(in, W1') + bias1)             [N, P, Q, nMid], kept on chip in nDtype
 *   out = act2(mid . W2' + bias2 + residual)      [N, P, Q, nCout] (residual may be NULL)
 * in: NHWC [N, H, W, nCs]; W1' from omCudaPackConvWeight (nCs inputs, nKH x nKW), W2' from it as
 * a 1x1 conv with nMid inputs. The intermediate map never reaches device memory; the results
 * are those of omCudaConv2dBnAct twice (the same roundings and summation order). nCs % 64 == 0,
 * nMid 64 or 128, nCout a multiple of 128 up to 512 (omCudaConvPairSupported). */
int omCudaConvPairBnAct(const void* pInput, const void* pPacked1, const float* pBias1,
                        const void* pPacked2, const float* pBias2, const void* pResidual,
                        void* pOutput, int nBatch, int nH, int nW, int nCs, int nMid, int nCout,
                        int nKH, int nKW, int nStride, int nPad, int nAct1, int nAct2,
                        int nDtype);
/* 1 when omCudaConvPairBnAct takes these channel counts and dtype, else 0 */
int omCudaConvPairSupported(int nCs, int nMid, int nCout, int nDtype);
/* new: the image stem (stride 1 or 2, Cin * stride^2 <= 16, Cout % 8 == 0) from the NCHW fp32
 * image: out[n,p,q,k] = act(sum_{c,r,s} x[n,c,p*st-pad+r,q*st-pad+s] * W[k,c,r,s] * scale[k]
 * + bias[k]), NHWC 16-bit output, BN folded as in omCudaPackConvWeight. A first launch writes a
 * space-to-depth 16-bit copy of the image into pWorkspace (omCudaStemWorkspaceBytes bytes,
 * 16-byte aligned): 16 channels (c, py, px) per pixel, padding included, so the stem runs as a
 * stride-1 ceil(KH/st) x ceil(KW/st) convolution through the same tcgen05 kernel as
 * omCudaConv2dBnAct; omCudaPackStemWeight packs the filter for it. */
long long omCudaPackedStemWeightElems(int nCout, int nCin, int nKH, int nKW, int nStride);
long long omCudaStemWorkspaceBytes(int nBatch, int nCin, int nH, int nW, int nKH, int nKW,
                                   int nStride, int nPad);
int omCudaPackStemWeight(const float* pWeight, const float* pConvBias, const float* pGamma,
                         const float* pBeta, const float* pMean, const float* pVar, float fEps,
                         void* pPacked, float* pBiasOut, int nCout, int nCin, int nKH, int nKW,
                         int nStride, int nDtype);
int omCudaStemConvBnAct(const float* pInput, void* pWorkspace, const void* pPacked,
                        const float* pBias, void* pOutput, int nBatch, int nCin, int nH, int nW,
                        int nCout, int nKH, int nKW, int nStride, int nPad, int nAct, int nDtype);
/* new: omCudaStemConvBnAct from an NCHW image in nInDtype: OM_DTYPE_F32, the conv's own
 * 16-bit nDtype (half the bytes to move to the device; a 16-bit image gives the same output as
 * its fp32 form, since the stem rounds its input to nDtype anyway), or OM_DTYPE_U8, 8-bit
 * samples read as sample / 255 in fp32 (a quarter of the bytes; the same output as the fp32
 * image sample / 255.0f). The same input dtypes apply to omCudaStemConvBnActPoolIn and
 * omCudaStemConvBnActNormIn. */
int omCudaStemConvBnActIn(const void* pInput, int nInDtype, void* pWorkspace, const void* pPacked,
                          const float* pBias, void* pOutput, int nBatch, int nCin, int nH, int nW,
                          int nCout, int nKH, int nKW, int nStride, int nPad, int nAct,
                          int nDtype);
/* new: the stem followed by its 3x3 / stride 2 / pad 1 max pool in one kernel (the stem output
 * never reaches device memory). pPooled: NHWC [nBatch, P2, Q2, nCout] with P2 = (P - 1) / 2 + 1,
 * Q2 likewise, P x Q the stem's output. Bit-identical to omCudaStemConvBnActIn followed by
 * omCudaMaxPool2dNhwc(..., 3, 2, 1, ...). Shapes omCudaStemPoolSupported rejects return
 * OM_ERR_UNSUPPORTED (nothing launched). Fuses the reference ResNet's stem sequence
 * conv1 -> bn1 -> relu -> maxpool(3, 2, 1) (om.engine.resnet.ixx:236-241). */
int omCudaStemConvBnActPoolIn(const void* pInput, int nInDtype, void* pWorkspace,
                              const void* pPacked, const float* pBias, void* pPooled, int nBatch,
                              int nCin, int nH, int nW, int nCout, int nKH, int nKW, int nStride,
                              int nPad, int nAct, int nDtype);
/* 1 when omCudaStemConvBnActPoolIn takes these shapes: nCout 64, a filter whose space-to-depth
 * form has 4 tap columns and at most 4 tap rows (the 7x7 / stride 2 ImageNet stem), output
 * width <= 128, a 16-bit dtype; else 0 */
int omCudaStemPoolSupported(int nBatch, int nCin, int nH, int nW, int nCout, int nKH, int nKW,
                            int nStride, int nPad, int nDtype);
/* new: the stem (bPool = 0: omCudaStemConvBnActIn; 1: omCudaStemConvBnActPoolIn) on an image
 * that is not normalised yet: channel c of the image becomes (x - pNormMean[c]) * pNormInvStd[c]
 * in fp32, subtract then multiply, before the rounding to 16 bits; padding stays 0. That is the
 * reference's ImageNet normalisation of inferBatch (EngineBridge.cpp:3580-3594, normalizeImage
 * om.engine.data_pipeline.ixx:744-803, invstd = 1.0f / std), done inside the stem's pre-pass
 * instead of on the host: with an fp32 image the result is bit-identical to normalising on the
 * host and calling the plain entry point. pNormMean and pNormInvStd are HOST arrays of nCin
 * floats (nCin <= 16). */
int omCudaStemConvBnActNormIn(const void* pInput, int nInDtype, const float* pNormMean,
                              const float* pNormInvStd, void* pWorkspace, const void* pPacked,
                              const float* pBias, void* pOutput, int nBatch, int nCin, int nH,
                              int nW, int nCout, int nKH, int nKW, int nStride, int nPad,
                              int nAct, int nDtype, int bPool);
/* NCHW fp32 -> NHWC (nDtype) with channels zero-padded to nCs */
int omCudaNchwToNhwc(const float* pIn, void* pOut, int nN, int nC, int nH, int nW, int nCs,
                     int nDtype);
/* NHWC (nDtype, nCs stored channels) -> NCHW fp32 with nC channels */
int omCudaNhwcToNchw(const void* pIn, float* pOut, int nN, int nC, int nH, int nW, int nCs,
                     int nDtype);
/* NHWC max pool (nDtype), same window semantics as omCudaMaxPool2d, no indices */
int omCudaMaxPool2dNhwc(const void* pIn, void* pOut, int nN, int nH, int nW, int nCs, int nK,
                        int nStride, int nPad, int nDtype);
/* NHWC global average pool: out[n,c] = mean_{h,w} in[n,h,w,c] (out in nOutDtype) */
int omCudaGlobalAvgPoolNhwc(const void* pIn, void* pOut, int nN, int nHW, int nCs, int nDtype,
                            int nOutDtype);
/* Fold BN into a depthwise weight [C,1,KH,KW] -> fp32 [KH*KW, Cs] plus bias [Cs] */
int omCudaPackDepthwiseWeight(const float* pWeight, const float* pGamma, const float* pBeta,
                              const float* pMean, const float* pVar, float fEps, float* pPacked,
                              float* pBiasOut, int nC, int nKH, int nKW, int nCs);
/* NHWC depthwise conv with fused bias + activation (bandwidth-bound, CUDA cores) */
int omCudaDepthwiseConv2dNhwc(const void* pIn, const float* pPacked, const float* pBias,
                              void* pOut, int nN, int nH, int nW, int nCs, int nKH, int nKW,
                              int nStride, int nPad, int nAct, int nDtype);
/* elementwise NHWC residual add + activation: out = act(a + b) (nDtype) */
int omCudaAddActNhwc(const void* pA, const void* pB, void* pOut, long long nCount, int nAct,
                     int nDtype);

#ifdef __cplusplus
}
#endif
#endif /* OM_CUDA_H */
