// om_cuda_backend.hpp — C++ host side of the B200 backend: a drop-in for the reference's
// om::CUDABackend (src/hal/om.hal.cuda_backend.ixx:283-984).
//
// Same class name, static method names and argument orders as the reference wrapper, so
// tensor_ops / autograd / optimizer code that calls `CUDABackend::conv2d(...)` compiles
// unchanged against this header. Two deliberate differences:
//   * every call checks the C-ABI status and throws om::CudaBackendError on failure (the
//     reference discards it, e.g. cuda_backend.ixx:325-329, :438-452);
//   * conv2d/conv2dBackward* reject asymmetric pad or stride instead of silently using the H
//     values for both dimensions as the reference does (cuda_backend.ixx:446-449); rectangular
//     filters (KH != KW) pass through, as the C ABI takes both.
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
        symmetric(nPadH, nPadW, nStrH, nStrW, "conv2d");
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
        symmetric(nPadH, nPadW, nStrH, nStrW, "conv2dBackwardInput");
        OM_CALL(omCudaConv2dBackwardInput(pGradOutput, pWeight, pGradInput, nBatch, nCin, nH, nW,
                                          nCout, nKH, nKW, nStrH, nPadH));
    }
    static void conv2dBackwardWeight(const float* pInput, const float* pGradOutput,
                                     float* pGradWeight, float* pGradBias, int nBatch, int nCin,
                                     int nH, int nW, int nCout, int nKH, int nKW, int nPadH,
                                     int nPadW, int nStrH, int nStrW) {
        symmetric(nPadH, nPadW, nStrH, nStrW, "conv2dBackwardWeight");
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

    // ---- the wrapper's remaining methods (cuda_backend.ixx:295-984), each forwarding its
    // arguments unchanged to the C-ABI entry point of the same name
    static void sub(const float* pA, const float* pB, float* pOut, size_t nCount) {
        OM_CALL(omCudaSub(pA, pB, pOut, static_cast<int>(nCount)));
    }
    static void mul(const float* pA, const float* pB, float* pOut, size_t nCount) {
        OM_CALL(omCudaMul(pA, pB, pOut, static_cast<int>(nCount)));
    }
    static void div(const float* pA, const float* pB, float* pOut, size_t nCount) {
        OM_CALL(omCudaDiv(pA, pB, pOut, static_cast<int>(nCount)));
    }
    static void addScalar(const float* pA, float fScalar, float* pOut, size_t nCount) {
        OM_CALL(omCudaAddScalar(pA, fScalar, pOut, static_cast<int>(nCount)));
    }
    static void batchedMatmul(const float* pA, const float* pB, float* pC, int nBatch, int nM,
                              int nK, int nN) {
        OM_CALL(omCudaBatchedMatmul(pA, pB, pC, nBatch, nM, nK, nN));
    }
    static void sigmoid(const float* pIn, float* pOut, size_t nCount) {
        OM_CALL(omCudaSigmoid(pIn, pOut, static_cast<int>(nCount)));
    }
    static void sigmoidBackward(const float* pGrad, const float* pOutput, float* pOut,
                                size_t nCount) {
        OM_CALL(omCudaSigmoidBackward(pGrad, pOutput, pOut, static_cast<int>(nCount)));
    }
    static void gelu(const float* pIn, float* pOut, size_t nCount) {
        OM_CALL(omCudaGELU(pIn, pOut, static_cast<int>(nCount)));
    }
    static void geluBackward(const float* pGrad, const float* pInput, float* pOut, size_t nCount) {
        OM_CALL(omCudaGeluBackward(pGrad, pInput, pOut, static_cast<int>(nCount)));
    }
    static void silu(const float* pIn, float* pOut, size_t nCount) {
        OM_CALL(omCudaSiLU(pIn, pOut, static_cast<int>(nCount)));
    }
    static void siluBackward(const float* pGrad, const float* pInput, float* pOut, size_t nCount) {
        OM_CALL(omCudaSiluBackward(pGrad, pInput, pOut, static_cast<int>(nCount)));
    }
    static void leakyRelu(const float* pIn, float* pOut, size_t nCount, float fSlope = 0.01f) {
        OM_CALL(omCudaLeakyRelu(pIn, pOut, static_cast<int>(nCount), fSlope));
    }
    static void leakyReluBackward(const float* pGrad, const float* pInput, float* pOut,
                                  size_t nCount, float fSlope = 0.01f) {
        OM_CALL(omCudaLeakyReluBackward(pGrad, pInput, pOut, static_cast<int>(nCount), fSlope));
    }
    static void tanhForward(const float* pIn, float* pOut, size_t nCount) {
        OM_CALL(omCudaTanh(pIn, pOut, static_cast<int>(nCount)));
    }
    static void tanhBackward(const float* pGrad, const float* pOutput, float* pOut, size_t nCount) {
        OM_CALL(omCudaTanhBackward(pGrad, pOutput, pOut, static_cast<int>(nCount)));
    }
    static void dilatedConv2dBackwardWeight(const float* pInput, const float* pGradOutput,
                                            float* pGradWeight, float* pGradBias, int nBatch,
                                            int nCin, int nH, int nW, int nCout, int nKH, int nKW,
                                            int nStride, int nPad, int nDilation) {
        OM_CALL(omCudaDilatedConv2dBackwardWeight(pInput, pGradOutput, pGradWeight, pGradBias,
                                                  nBatch, nCin, nH, nW, nCout, nKH, nKW, nStride,
                                                  nPad, nDilation));
    }
    static void groupNorm2d(const float* pInput, float* pOutput, const float* pGamma,
                            const float* pBeta, float* pSavedMean, float* pSavedInvStd, int nBatch,
                            int nChannels, int nH, int nW, int nGroups, float fEps) {
        OM_CALL(omCudaGroupNorm2d(pInput, pOutput, pGamma, pBeta, pSavedMean, pSavedInvStd,
                                  nBatch, nChannels, nH, nW, nGroups, fEps));
    }
    static void groupNorm2dBackward(const float* pGradOutput, const float* pInput,
                                    const float* pMean, const float* pInvStd, const float* pGamma,
                                    float* pGradInput, float* pGradGamma, float* pGradBeta,
                                    int nBatch, int nChannels, int nH, int nW, int nGroups,
                                    float fEps) {
        OM_CALL(omCudaGroupNorm2dBackward(pGradOutput, pInput, pMean, pInvStd, pGamma, pGradInput,
                                          pGradGamma, pGradBeta, nBatch, nChannels, nH, nW,
                                          nGroups, fEps));
    }
    static void layerNorm(const float* pInput, float* pOutput, const float* pGamma,
                          const float* pBeta, float* pSavedMean, float* pSavedInvStd, int nBatch,
                          int nDim, float fEps) {
        OM_CALL(omCudaLayerNorm(pInput, pOutput, pGamma, pBeta, pSavedMean, pSavedInvStd, nBatch,
                                nDim, fEps));
    }
    static void layerNormBackward(const float* pGradOut, const float* pInput, const float* pMean,
                                  const float* pInvStd, const float* pGamma, float* pGradInput,
                                  float* pGradGamma, float* pGradBeta, int nBatch, int nDim) {
        OM_CALL(omCudaLayerNormBackward(pGradOut, pInput, pMean, pInvStd, pGamma, pGradInput,
                                        pGradGamma, pGradBeta, nBatch, nDim));
    }
    static void adamStep(float* pParam, const float* pGrad, float* pM, float* pV, int nCount,
                         float fLr, float fBeta1, float fBeta2, float fEps, int nStep) {
        OM_CALL(omCudaAdamStep(pParam, pGrad, pM, pV, nCount, fLr, fBeta1, fBeta2, fEps, nStep));
    }
    static void upsampleBilinear(const float* pIn, float* pOut, int nBatch, int nChannels, int nH,
                                 int nW, int nOutH, int nOutW) {
        OM_CALL(omCudaUpsampleBilinear(pIn, pOut, nBatch, nChannels, nH, nW, nOutH, nOutW));
    }
    static void upsampleBilinearBackward(const float* pGradOut, float* pGradIn, int nBatch,
                                         int nChannels, int nInH, int nInW, int nOutH,
                                         int nOutW) {
        OM_CALL(omCudaUpsampleBilinearBackward(pGradOut, pGradIn, nBatch, nChannels, nInH, nInW,
                                               nOutH, nOutW));
    }
    static void concatChannels(const float* pA, const float* pB, float* pOut, int nBatch, int nC1,
                               int nC2, int nHW) {
        OM_CALL(omCudaConcatChannels(pA, pB, pOut, nBatch, nC1, nC2, nHW));
    }
    static void concatChannelsBackward(const float* pGradOut, float* pGradA, float* pGradB,
                                       int nBatch, int nCA, int nCB, int nHW) {
        OM_CALL(omCudaConcatChannelsBackward(pGradOut, pGradA, pGradB, nBatch, nCA, nCB, nHW));
    }
    static void bceWithLogitsForward(const float* pLogits, const float* pTargets, float* pResult,
                                     int nCount) {
        OM_CALL(omCudaBCEWithLogits(pLogits, pTargets, pResult, nCount));
    }
    static void bceWithLogitsBackward(const float* pLogits, const float* pTargets,
                                      float* pGradLogits, int nCount, float fInvN) {
        OM_CALL(omCudaBCEWithLogitsBackward(pLogits, pTargets, pGradLogits, nCount, fInvN));
    }
    static void convTranspose2d(const float* pInput, const float* pWeight, const float* pBias,
                                float* pOutput, int nBatch, int nCin, int nHin, int nWin,
                                int nCout, int nKH, int nKW, int nStride, int nPad) {
        OM_CALL(omCudaConvTranspose2d(pInput, pWeight, pBias, pOutput, nBatch, nCin, nHin, nWin,
                                      nCout, nKH, nKW, nStride, nPad));
    }
    static void concatLastDim(const float* pA, const float* pB, float* pOut, int nOuter,
                              int nDimA, int nDimB) {
        OM_CALL(omCudaConcatLastDim(pA, pB, pOut, nOuter, nDimA, nDimB));
    }
    static void concatLastDimBackward(const float* pGradOut, float* pGradA, float* pGradB,
                                      int nOuter, int nDimA, int nDimB) {
        OM_CALL(omCudaConcatLastDimBackward(pGradOut, pGradA, pGradB, nOuter, nDimA, nDimB));
    }
    static void sliceLastDim(const float* pIn, float* pOut, int nOuter, int nFullDim, int nStart,
                             int nLen) {
        OM_CALL(omCudaSliceLastDim(pIn, pOut, nOuter, nFullDim, nStart, nLen));
    }
    static void sliceLastDimBackward(const float* pGradOut, float* pGradIn, int nOuter,
                                     int nFullDim, int nStart, int nLen) {
        OM_CALL(omCudaSliceLastDimBackward(pGradOut, pGradIn, nOuter, nFullDim, nStart, nLen));
    }
    static void softmaxLastDimBackward(const float* pGradOut, const float* pSoftmax,
                                       float* pGradIn, int nOuter, int nLastDim) {
        OM_CALL(omCudaSoftmaxLastDimBackward(pGradOut, pSoftmax, pGradIn, nOuter, nLastDim));
    }
    static void dropoutForward(const float* pIn, float* pOut, float* pMask, int nCount,
                               float fKeepProb, unsigned long long nSeed) {
        OM_CALL(omCudaDropoutForward(pIn, pOut, pMask, nCount, fKeepProb, nSeed));
    }
    static void diceLossForward(const float* pLogits, const float* pTarget, float* pLoss,
                                float* pSigmoidOut, float* pStats, int nCount) {
        OM_CALL(omCudaDiceLossForward(pLogits, pTarget, pLoss, pSigmoidOut, pStats, nCount));
    }
    static void diceLossBackward(const float* pSigmoidOut, const float* pTarget,
                                 const float* pStats, const float* pGradOutput,
                                 float* pGradLogits, int nCount) {
        OM_CALL(omCudaDiceLossBackward(pSigmoidOut, pTarget, pStats, pGradOutput, pGradLogits,
                                       nCount));
    }
    static void weightedPixelCEForward(const float* pLogits, const float* pTarget,
                                       const float* pClassWeights, float* pSoftmax, float* pLoss,
                                       float* pStats, int nPixels, int nClasses, int nSpatial) {
        OM_CALL(omCudaWeightedPixelCEForward(pLogits, pTarget, pClassWeights, pSoftmax, pLoss,
                                             pStats, nPixels, nClasses, nSpatial));
    }
    static void weightedPixelCEBackward(const float* pSoftmax, const float* pTarget,
                                        const float* pClassWeights, const float* pGradOutput,
                                        const float* pStats, float* pGradLogits, int nPixels,
                                        int nClasses, int nSpatial) {
        OM_CALL(omCudaWeightedPixelCEBackward(pSoftmax, pTarget, pClassWeights, pGradOutput,
                                              pStats, pGradLogits, nPixels, nClasses, nSpatial));
    }
    static void qkvSplitHeads(const float* pQkv, float* pQ, float* pK, float* pV, int nBatch,
                              int nSeqLen, int nHeads, int nHeadDim, float fScale) {
        OM_CALL(omCudaQkvSplitHeads(pQkv, pQ, pK, pV, nBatch, nSeqLen, nHeads, nHeadDim, fScale));
    }
    static void mergeHeads(const float* pIn, float* pOut, int nBatch, int nSeqLen, int nHeads,
                           int nHeadDim) {
        OM_CALL(omCudaMergeHeads(pIn, pOut, nBatch, nSeqLen, nHeads, nHeadDim));
    }

private:
    // The C ABI takes one padding and one stride for both dimensions (the reference wrapper
    // passes the H values, cuda_backend.ixx:447-448); a rectangular filter is fine.
    static void symmetric(int ph, int pw, int sh, int sw, const char* fn) {
        if (ph != pw || sh != sw) throw CudaBackendError(fn, OM_ERR_UNSUPPORTED);
    }
};

#undef OM_CALL

}  // namespace om
