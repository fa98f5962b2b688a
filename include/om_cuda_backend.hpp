// om_cuda_backend.hpp — C++ host side of the B200 backend: a drop-in for the reference's
// om::CUDABackend (src/hal/om.hal.cuda_backend.ixx:283-984).
//
// Same class name, static method names and argument orders as the reference wrapper, so
// tensor_ops / autograd / optimizer code that calls `CUDABackend::conv2d(...)` compiles
// unchanged against this header. Two deliberate differences:
//   * every call checks the C-ABI status and throws om::CudaBackendError on failure (the
//     reference discards it, e.g. cuda_backend.ixx:325-329, :438-452);
//   * conv2d/conv2dBackward* reject asymmetric kernel/pad/stride instead of silently using
//     the H values for both dimensions as the reference does (cuda_backend.ixx:446-449).
#pragma once

#include <cstddef>
#include <stdexcept>
#include <string>

#include "om_cuda.h"

namespace om {

class CudaBackendError : public std::runtime_error {
public:
    CudaBackendError(const char* fn, int status)
        : std::runtime_error(std::string(fn) + " failed with status " + std::to_string(status)),
          m_status(status) {}
    int status() const { return m_status; }

private:
    int m_status;
};

namespace detail {
inline void omCheck(int status, const char* fn) {
    if (status != OM_OK) throw CudaBackendError(fn, status);
}
}  // namespace detail

#define OM_CALL(expr) ::om::detail::omCheck((expr), #expr)

class CUDABackend {
public:
    static void add(const float* pA, const float* pB, float* pOut, size_t nCount) {
        OM_CALL(omCudaAdd(pA, pB, pOut, static_cast<int>(nCount)));
    }
    static void mulScalar(const float* pA, float fScalar, float* pOut, size_t nCount) {
        OM_CALL(omCudaMulScalar(pA, fScalar, pOut, static_cast<int>(nCount)));
    }
    static void matmul(const float* pA, const float* pB, float* pC, int nM, int nK, int nN) {
        OM_CALL(omCudaMatmul(pA, pB, pC, nM, nK, nN));
    }
    static void transpose(const float* pIn, float* pOut, int nRows, int nCols) {
        OM_CALL(omCudaTranspose(pIn, pOut, nRows, nCols));
    }
    static void relu(const float* pIn, float* pOut, size_t nCount) {
        OM_CALL(omCudaReLU(pIn, pOut, static_cast<int>(nCount)));
    }
    static void reluBackward(const float* pInput, const float* pGradOut, float* pGradIn,
                             size_t nCount) {
        OM_CALL(omCudaReLUBackward(pInput, pGradOut, pGradIn, static_cast<int>(nCount)));
    }
    static void conv2d(const float* pInput, const float* pWeight, const float* pBias,
                       float* pOutput, int nBatch, int nCin, int nH, int nW, int nCout, int nKH,
                       int nKW, int nPadH, int nPadW, int nStrH, int nStrW) {
        symmetric(nKH, nKW, nPadH, nPadW, nStrH, nStrW, "conv2d");
        OM_CALL(omCudaConv2d(pInput, pWeight, pBias, pOutput, nBatch, nCin, nH, nW, nCout, nKH,
                             nKW, nStrH, nPadH));
    }
    static void dilatedConv2d(const float* pInput, const float* pWeight, const float* pBias,
                              float* pOutput, int nBatch, int nCin, int nH, int nW, int nCout,
                              int nKH, int nKW, int nStride, int nPad, int nDilation,
                              int nGroups) {
        OM_CALL(omCudaDilatedConv2d(pInput, pWeight, pBias, pOutput, nBatch, nCin, nH, nW, nCout,
                                    nKH, nKW, nStride, nPad, nDilation, nGroups));
    }
    static void conv2dBackwardInput(const float* pGradOutput, const float* pWeight,
                                    float* pGradInput, int nBatch, int nCin, int nH, int nW,
                                    int nCout, int nKH, int nKW, int nPadH, int nPadW, int nStrH,
                                    int nStrW) {
        symmetric(nKH, nKW, nPadH, nPadW, nStrH, nStrW, "conv2dBackwardInput");
        OM_CALL(omCudaConv2dBackwardInput(pGradOutput, pWeight, pGradInput, nBatch, nCin, nH, nW,
                                          nCout, nKH, nKW, nStrH, nPadH));
    }
    static void conv2dBackwardWeight(const float* pInput, const float* pGradOutput,
                                     float* pGradWeight, float* pGradBias, int nBatch, int nCin,
                                     int nH, int nW, int nCout, int nKH, int nKW, int nPadH,
                                     int nPadW, int nStrH, int nStrW) {
        symmetric(nKH, nKW, nPadH, nPadW, nStrH, nStrW, "conv2dBackwardWeight");
        OM_CALL(omCudaConv2dBackwardWeight(pInput, pGradOutput, pGradWeight, pGradBias, nBatch,
                                           nCin, nH, nW, nCout, nKH, nKW, nStrH, nPadH));
    }
    static void maxPool2d(const float* pIn, float* pOut, int* pIndices, int nBatch, int nChannels,
                          int nH, int nW, int nKH, int nKW, int nStride, int nPad) {
        OM_CALL(omCudaMaxPool2d(pIn, pOut, pIndices, nBatch, nChannels, nH, nW, nKH, nKW,
                                nStride, nStride, nPad, nPad));
    }
    static void maxPool2dBackward(const float* pGradOut, const int* pIndices, float* pGradIn,
                                  int nBatch, int nChannels, int nH, int nW, int nHout,
                                  int nWout) {
        size_t n = static_cast<size_t>(nBatch) * nChannels * nH * nW;
        OM_CALL(omCudaMemset(pGradIn, 0, n * sizeof(float)));
        OM_CALL(omCudaMaxPool2dBackward(pGradOut, pIndices, pGradIn, nBatch, nChannels, nH, nW,
                                        nHout, nWout));
    }
    static void avgPool2d(const float* pIn, float* pOut, int nBatch, int nChannels, int nH,
                          int nW, int nKH, int nKW, int nStride, int nPad) {
        OM_CALL(omCudaAvgPool2d(pIn, pOut, nBatch, nChannels, nH, nW, nKH, nKW, nStride, nStride,
                                nPad, nPad));
    }
    static void avgPool2dBackward(const float* pGradOut, float* pGradIn, int nBatch,
                                  int nChannels, int nH, int nW, int nKH, int nKW, int nStride,
                                  int nPad) {
        size_t n = static_cast<size_t>(nBatch) * nChannels * nH * nW;
        OM_CALL(omCudaMemset(pGradIn, 0, n * sizeof(float)));
        OM_CALL(omCudaAvgPool2dBackward(pGradOut, pGradIn, nBatch, nChannels, nH, nW, nKH, nKW,
                                        nStride, nStride, nPad, nPad));
    }
    static void adaptiveAvgPool2d(const float* pIn, float* pOut, int nBatch, int nChannels,
                                  int nH, int nW, int nOutH, int nOutW) {
        OM_CALL(omCudaAdaptiveAvgPool2d(pIn, pOut, nBatch, nChannels, nH, nW, nOutH, nOutW));
    }
    static void adaptiveAvgPool2dBackward(const float* pGradOut, float* pGradIn, int nBatch,
                                          int nChannels, int nH, int nW, int nOutH, int nOutW) {
        OM_CALL(omCudaAdaptiveAvgPool2dBackward(pGradOut, pGradIn, nBatch, nChannels, nH, nW,
                                                nOutH, nOutW));
    }
    // note the reference order: gamma/beta before the output (cuda_backend.ixx:571)
    static void batchNorm2d(const float* pInput, const float* pGamma, const float* pBeta,
                            float* pOutput, float* pRunMean, float* pRunVar, float* pSavedMean,
                            float* pSavedInvStd, int nBatch, int nChannels, int nHW, float fEps,
                            float fMomentum, bool bTraining) {
        OM_CALL(omCudaBatchNorm2d(pInput, pOutput, pGamma, pBeta, pRunMean, pRunVar, pSavedMean,
                                  pSavedInvStd, nBatch, nChannels, 1, nHW, fEps, fMomentum,
                                  bTraining ? 1 : 0));
    }
    static void batchNorm2dBackward(const float* pGradOutput, const float* pInput,
                                    const float* pMean, const float* pInvStd, const float* pGamma,
                                    float* pGradInput, float* pGradGamma, float* pGradBeta,
                                    int nBatch, int nChannels, int nH, int nW,
                                    float fEps = 1e-5f) {
        OM_CALL(omCudaBatchNorm2dBackward(pGradOutput, pInput, pMean, pInvStd, pGamma, pGradInput,
                                          pGradGamma, pGradBeta, nBatch, nChannels, nH, nW, fEps));
    }
    static void softmax(const float* pIn, float* pOut, int nBatch, int nClasses) {
        OM_CALL(omCudaSoftmax(pIn, pOut, nBatch, nClasses));
    }
    static void crossEntropySoftmaxBackward(const float* pSoftmax, const float* pTarget,
                                            float* pGradLogits, int nBatch, int nClasses) {
        OM_CALL(omCudaSoftmaxCrossEntropyBackward(pSoftmax, pTarget, pGradLogits, nBatch,
                                                  nClasses));
    }
    static void crossEntropyForward(const float* pSoftmax, const float* pTarget, float* pResult,
                                    int nBatch, int nClasses) {
        OM_CALL(omCudaCrossEntropy(pSoftmax, pTarget, pResult, nBatch, nClasses));
    }
    static void sgdStep(float* pParam, const float* pGrad, float* pVelocity, int nCount,
                        float fLr, float fMomentum) {
        OM_CALL(omCudaSgdStep(pParam, pGrad, pVelocity, nCount, fLr, fMomentum));
    }
    static void fillZeros(float* pData, size_t nCount) {
        OM_CALL(omCudaFillZeros(pData, static_cast<int>(nCount)));
    }
    static void fillOnes(float* pData, size_t nCount) {
        OM_CALL(omCudaFillOnes(pData, static_cast<int>(nCount)));
    }
    static void fillValue(float* pData, size_t nCount, float fValue) {
        OM_CALL(omCudaFillValue(pData, static_cast<int>(nCount), fValue));
    }
    static void copy(const float* pSrc, float* pDst, size_t nCount) {
        OM_CALL(omCudaCopy(pSrc, pDst, static_cast<int>(nCount)));
    }
    static void addBias(const float* pData, const float* pBias, float* pOut, int nBatch,
                        int nChannels, int nHW) {
        OM_CALL(omCudaAddBias(pData, pBias, pOut, nBatch, nChannels, nHW));
    }
    static void addBiasBackward(const float* pGradOut, float* pGradBias, int nBatch,
                                int nChannels, int nHW) {
        OM_CALL(omCudaAddBiasBackward(pGradOut, pGradBias, nBatch, nChannels, nHW));
    }
    static void clip(const float* pIn, float* pOut, size_t nCount, float fMin, float fMax) {
        OM_CALL(omCudaClip(pIn, pOut, static_cast<int>(nCount), fMin, fMax));
    }
    static void argmax(const float* pData, int* pOut, int nBatch, int nClasses) {
        OM_CALL(omCudaArgmax(pData, pOut, nBatch, nClasses));
    }
    static void sum(const float* pData, float* pResult, int nCount) {
        OM_CALL(omCudaSum(pData, pResult, nCount));
    }

private:
    static void symmetric(int kh, int kw, int ph, int pw, int sh, int sw, const char* fn) {
        if (kh != kw || ph != pw || sh != sw) throw CudaBackendError(fn, OM_ERR_UNSUPPORTED);
    }
};

#undef OM_CALL

}  // namespace om
