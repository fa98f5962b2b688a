// Compiles the C++ CUDABackend mirror the way the reference's tensor_ops would use it and
// checks, without a GPU, that a failing call throws instead of being silently ignored.
#include <cstdio>

#include "om_cuda_backend.hpp"

// every static method of the reference's om::CUDABackend (cuda_backend.ixx:283-984): the
// program does not compile if the mirror lacks one
#define OMB_HAS(name) (void)&om::CUDABackend::name;
static void reference_methods_exist() {
    OMB_HAS(add) OMB_HAS(sub) OMB_HAS(mul) OMB_HAS(addScalar)
    OMB_HAS(mulScalar) OMB_HAS(matmul) OMB_HAS(batchedMatmul) OMB_HAS(transpose)
    OMB_HAS(relu) OMB_HAS(reluBackward) OMB_HAS(sigmoid) OMB_HAS(sigmoidBackward)
    OMB_HAS(gelu) OMB_HAS(geluBackward) OMB_HAS(silu) OMB_HAS(siluBackward)
    OMB_HAS(leakyRelu) OMB_HAS(leakyReluBackward) OMB_HAS(tanhForward) OMB_HAS(tanhBackward)
    OMB_HAS(conv2d) OMB_HAS(dilatedConv2d) OMB_HAS(dilatedConv2dBackwardWeight) OMB_HAS(conv2dBackwardInput)
    OMB_HAS(conv2dBackwardWeight) OMB_HAS(maxPool2d) OMB_HAS(maxPool2dBackward) OMB_HAS(avgPool2d)
    OMB_HAS(avgPool2dBackward) OMB_HAS(adaptiveAvgPool2d) OMB_HAS(batchNorm2d) OMB_HAS(batchNorm2dBackward)
    OMB_HAS(groupNorm2d) OMB_HAS(groupNorm2dBackward) OMB_HAS(layerNorm) OMB_HAS(softmax)
    OMB_HAS(crossEntropySoftmaxBackward) OMB_HAS(adamStep) OMB_HAS(sgdStep) OMB_HAS(fillZeros)
    OMB_HAS(fillOnes) OMB_HAS(fillValue) OMB_HAS(copy) OMB_HAS(addBias)
    OMB_HAS(argmax) OMB_HAS(sum) OMB_HAS(adaptiveAvgPool2dBackward) OMB_HAS(addBiasBackward)
    OMB_HAS(upsampleBilinearBackward) OMB_HAS(concatChannelsBackward) OMB_HAS(bceWithLogitsBackward) OMB_HAS(div)
    OMB_HAS(clip) OMB_HAS(upsampleBilinear) OMB_HAS(concatChannels) OMB_HAS(bceWithLogitsForward)
    OMB_HAS(crossEntropyForward) OMB_HAS(layerNormBackward) OMB_HAS(convTranspose2d) OMB_HAS(concatLastDim)
    OMB_HAS(concatLastDimBackward) OMB_HAS(sliceLastDim) OMB_HAS(sliceLastDimBackward) OMB_HAS(softmaxLastDimBackward)
    OMB_HAS(dropoutForward) OMB_HAS(diceLossForward) OMB_HAS(diceLossBackward) OMB_HAS(weightedPixelCEForward)
    OMB_HAS(weightedPixelCEBackward) OMB_HAS(qkvSplitHeads) OMB_HAS(mergeHeads)
}
#undef OMB_HAS

int main() {
    reference_methods_exist();
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
