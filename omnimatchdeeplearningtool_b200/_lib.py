"""ctypes binding of libomcuda.so, the sm_100a backend declared in include/om_cuda.h.

The library is built in-tree (``make -C omnimatchdeeplearningtool_b200``). There is no CPU
fallback: importing this module on a machine without the built library raises immediately,
and every entry point's status is checked by :func:`check`.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_longlong, c_size_t, c_uint, c_ulonglong, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libomcuda.so")

OM_OK = 0
STATUS_NAMES = {
    -1: "OM_ERR_CUDA",
    -2: "OM_ERR_INVALID",
    -3: "OM_ERR_UNSUPPORTED",
    -4: "OM_ERR_NOT_INIT",
    -5: "OM_ERR_OOM",
    -6: "OM_ERR_KERNEL_TIMEOUT",
    -7: "OM_ERR_DRIVER",
    -8: "OM_ERR_TOO_LARGE",
    -9: "OM_ERR_COMM",
}
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
DTYPE_U8 = 3   # 8-bit image samples (value / 255), an input dtype of the stem entry points
ACT_NONE, ACT_RELU, ACT_RELU6 = 0, 1, 2


class OmCudaError(RuntimeError):
    """Raised for every non-zero status returned by the backend."""

    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: {STATUS_NAMES.get(status, status)}")
        self.status = status


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C {_HERE}` "
            "(the backend has no CPU fallback)")
    return ctypes.CDLL(LIB_PATH)


lib = _load()

P = c_void_p
F = c_float
I = c_int
_SIGS = {
    # runtime
    "omCudaInit": [I], "omCudaSetDevice": [I], "omCudaGetDeviceCount": [],
    "omCudaGetDeviceName": [I, ctypes.c_char_p, I],
    "omCudaGetMemInfo": [I, POINTER(c_size_t), POINTER(c_size_t)],
    "omCudaGetComputeCapability": [I, POINTER(c_int), POINTER(c_int)],
    "omCudaMalloc": [POINTER(c_void_p), c_size_t], "omCudaFree": [P],
    "omCudaCopyH2D": [P, P, c_size_t], "omCudaCopyD2H": [P, P, c_size_t],
    "omCudaCopyD2D": [P, P, c_size_t], "omCudaMemset": [P, I, c_size_t],
    "omCudaSynchronize": [], "omCudaAsyncCopyH2D": [P, P, c_size_t],
    "omCudaAsyncCopyD2H": [P, P, c_size_t], "omCudaSyncTransferStream": [],
    "omCudaSyncComputeStream": [], "omCudaCleanup": [], "omCudaForceReset": [],
    "omCudaTransferH2D": [P, P, c_size_t], "omCudaTransferD2H": [P, P, c_size_t],
    "omCudaComputeWaitTransfer": [], "omCudaTransferWaitCompute": [],
    "omCudaMallocHost": [POINTER(c_void_p), c_size_t], "omCudaFreeHost": [P],
    "omCudaGraphBeginCapture": [], "omCudaGraphEndCapture": [POINTER(c_void_p)],
    "omCudaGraphLaunch": [P], "omCudaGraphDestroy": [P],
    "omCudaGetKernelError": [POINTER(c_uint)], "omCudaGetLaunchCount": [POINTER(c_ulonglong)],
    "omCudaGetCurrentDevice": [],
    "omCudaSynchronizeChecked": [], "omCudaTestStallNextConv": [c_longlong, c_ulonglong],
    # data-parallel gradient exchange
    "omNcclGetUniqueId": [P], "omNcclInit": [I, I, P, I],
    "omCudaAllreduceAsync": [P, c_longlong, I], "omCudaAllreduceJoin": [],
    "omCudaAllreduce": [P, c_longlong, I], "omNcclPoll": [I],
    "omNcclRankInfo": [POINTER(c_int), POINTER(c_int)], "omNcclAbort": [], "omNcclDestroy": [],
    "omCudaStridedCopy": [P, P, POINTER(c_int), POINTER(c_int), I, c_longlong],
    # elementwise
    "omCudaAdd": [P, P, P, I], "omCudaMulScalar": [P, F, P, I], "omCudaReLU": [P, P, I],
    "omCudaReLUBackward": [P, P, P, I], "omCudaClip": [P, P, I, F, F],
    "omCudaFillZeros": [P, I], "omCudaFillOnes": [P, I], "omCudaFillValue": [P, I, F],
    "omCudaCopy": [P, P, I], "omCudaSum": [P, P, I], "omCudaArgmax": [P, P, I, I],
    "omCudaTranspose": [P, P, I, I],
    # contractions
    "omCudaMatmul": [P, P, P, I, I, I],
    "omCudaConv2d": [P, P, P, P, I, I, I, I, I, I, I, I, I],
    "omCudaDilatedConv2d": [P, P, P, P, I, I, I, I, I, I, I, I, I, I, I],
    "omCudaConv2dBackwardInput": [P, P, P, I, I, I, I, I, I, I, I, I],
    "omCudaConv2dBackwardWeight": [P, P, P, P, I, I, I, I, I, I, I, I, I],
    # norm / pool / loss / optimiser
    "omCudaBatchNorm2d": [P, P, P, P, P, P, P, P, I, I, I, I, F, F, I],
    "omCudaBatchNorm2dBackward": [P, P, P, P, P, P, P, P, I, I, I, I, F],
    "omCudaBatchNorm2dAct": [P, P, P, P, P, P, P, P, I, I, I, I, F, F, I, I],
    "omCudaConv2dBatchNorm2dAct": [P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, I,
                                   F, F, I, P],
    "omCudaConv2dBatchNorm2dAddAct": [P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I,
                                      I, F, F, I, P, P],
    "omCudaStemConv2dBatchNorm2dAct": [P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I,
                                       I, F, F, I, P],
    "omCudaConv2dBackwardWeightSplit": [P, P, P, P, P, I, I, I, I, I, I, I, I, I],
    "omCudaConv2dBackwardSplit": [P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, I],
    "omCudaMaxPool2dBackwardGather": [P, P, P, I, I, I, I, I, I, I, I, I, I],
    "omCudaBatchNorm2dBackwardAct": [P, P, P, P, P, P, P, P, P, I, I, I, I, F, I],
    "omCudaBatchNorm2dNoAlloc": [P, P, P, P, P, P, P, P, I, I, I, I, F, F, I],
    "omCudaMaxPool2d": [P, P, P, I, I, I, I, I, I, I, I, I, I],
    "omCudaMaxPool2dBackward": [P, P, P, I, I, I, I, I, I],
    "omCudaAvgPool2d": [P, P, I, I, I, I, I, I, I, I, I, I],
    "omCudaAvgPool2dBackward": [P, P, I, I, I, I, I, I, I, I, I, I],
    "omCudaAdaptiveAvgPool2d": [P, P, I, I, I, I, I, I],
    "omCudaAdaptiveAvgPool2dBackward": [P, P, I, I, I, I, I, I],
    "omCudaAddBias": [P, P, P, I, I, I], "omCudaAddBiasBackward": [P, P, I, I, I],
    "omCudaSoftmax": [P, P, I, I], "omCudaCrossEntropy": [P, P, P, I, I],
    "omCudaSoftmaxCrossEntropyBackward": [P, P, P, I, I],
    "omCudaSgdStepScaled": [P, P, P, I, F, F, F],
    "omCudaSoftmaxCrossEntropyFused": [P, P, P, P, P, I, I], "omCudaSgdStep": [P, P, P, I, F, F],
    "omCudaAdamStep": [P, P, P, P, I, F, F, F, F, I],
    "omCudaGradNormClip": [P, I, F, F, P], "omCudaSgdStepGuarded": [P, P, P, I, F, F, P],
    # further elementwise ops and activations
    "omCudaSub": [P, P, P, I], "omCudaMul": [P, P, P, I], "omCudaDiv": [P, P, P, I],
    "omCudaAddScalar": [P, F, P, I], "omCudaMean": [P, P, I],
    "omCudaSigmoid": [P, P, I], "omCudaSigmoidBackward": [P, P, P, I],
    "omCudaTanh": [P, P, I], "omCudaTanhBackward": [P, P, P, I],
    "omCudaGELU": [P, P, I], "omCudaGeluBackward": [P, P, P, I],
    "omCudaSiLU": [P, P, I], "omCudaSiluBackward": [P, P, P, I],
    "omCudaLeakyRelu": [P, P, I, F], "omCudaLeakyReluBackward": [P, P, P, I, F],
    # off the hot path: the remaining reference entry points
    "omCudaBatchedMatmul": [P, P, P, I, I, I, I],
    "omCudaConv2dIm2col": [P, P, P, P, I, I, I, I, I, I, I, I, I],
    "omCudaConvTranspose2d": [P, P, P, P, I, I, I, I, I, I, I, I, I],
    "omCudaDilatedConv2dBackwardWeight": [P, P, P, P, I, I, I, I, I, I, I, I, I, I],
    "omCudaLayerNorm": [P, P, P, P, P, P, I, I, F],
    "omCudaLayerNormBackward": [P, P, P, P, P, P, P, P, I, I],
    "omCudaGroupNorm2d": [P, P, P, P, P, P, I, I, I, I, I, F],
    "omCudaGroupNorm2dBackward": [P, P, P, P, P, P, P, P, I, I, I, I, I, F],
    "omCudaSoftmaxLastDimBackward": [P, P, P, I, I],
    "omCudaUpsampleBilinear": [P, P, I, I, I, I, I, I],
    "omCudaUpsampleBilinearBackward": [P, P, I, I, I, I, I, I],
    "omCudaConcatChannels": [P, P, P, I, I, I, I],
    "omCudaConcatChannelsBackward": [P, P, P, I, I, I, I],
    "omCudaConcatLastDim": [P, P, P, I, I, I], "omCudaConcatLastDimBackward": [P, P, P, I, I, I],
    "omCudaSliceLastDim": [P, P, I, I, I, I], "omCudaSliceLastDimBackward": [P, P, I, I, I, I],
    "omCudaQkvSplitHeads": [P, P, P, P, I, I, I, I, F],
    "omCudaMergeHeads": [P, P, I, I, I, I],
    "omCudaBCEWithLogits": [P, P, P, I], "omCudaBCEWithLogitsBackward": [P, P, P, I, F],
    "omCudaDiceLossForward": [P, P, P, P, P, I], "omCudaDiceLossBackward": [P, P, P, P, P, I],
    "omCudaWeightedPixelCEForward": [P, P, P, P, P, P, I, I, I],
    "omCudaWeightedPixelCEBackward": [P, P, P, P, P, P, I, I, I],
    "omCudaDropout": [P, P, P, I, F, I],
    "omCudaDropoutForward": [P, P, P, I, F, c_ulonglong],
    # NHWC fused path
    "omCudaPackConvWeight": [P, P, P, P, P, P, F, P, P, I, I, I, I, I, I],
    "omCudaConv2dBnAct": [P, P, P, P, P, I, I, I, I, I, I, I, I, I, I, I, I],
    "omCudaConvTilePlan": [I, I, I, I, I, I, I, I, I, I, POINTER(c_int)],
    "omCudaConvPairBnAct": [P, P, P, P, P, P, P] + [I] * 13,
    "omCudaConvPairSupported": [I, I, I, I],
    "omCudaConvStamps": [P, I],
    "omCudaConvStampLaunches": [POINTER(c_int), POINTER(c_int), I, POINTER(c_int)],
    "omCudaPackStemWeight": [P, P, P, P, P, P, F, P, P, I, I, I, I, I, I],
    "omCudaStemConvBnAct": [P, P, P, P, P, I, I, I, I, I, I, I, I, I, I, I],
    "omCudaStemConvBnActIn": [P, I, P, P, P, P, I, I, I, I, I, I, I, I, I, I, I],
    "omCudaStemConvBnActPoolIn": [P, I, P, P, P, P, I, I, I, I, I, I, I, I, I, I, I],
    "omCudaStemConvBnActNormIn": [P, I, P, P, P, P, P, P, I, I, I, I, I, I, I, I, I, I, I, I],
    "omCudaStemPoolSupported": [I, I, I, I, I, I, I, I, I, I],
    "omCudaNchwToNhwc": [P, P, I, I, I, I, I, I], "omCudaNhwcToNchw": [P, P, I, I, I, I, I, I],
    "omCudaMaxPool2dNhwc": [P, P, I, I, I, I, I, I, I, I],
    "omCudaGlobalAvgPoolNhwc": [P, P, I, I, I, I, I],
    "omCudaPackDepthwiseWeight": [P, P, P, P, P, F, P, P, I, I, I, I],
    "omCudaDepthwiseConv2dNhwc": [P, P, P, P, I, I, I, I, I, I, I, I, I, I],
    "omCudaAddActNhwc": [P, P, P, c_longlong, I, I],
}
for _name, _args in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = c_int
lib.omCudaGetStream.argtypes = []
lib.omCudaGetStream.restype = c_void_p
lib.omCudaPackedConvWeightElems.argtypes = [I, I, I, I]
lib.omCudaPackedConvWeightElems.restype = c_longlong
lib.omCudaPackedStemWeightElems.argtypes = [I, I, I, I, I]
lib.omCudaPackedStemWeightElems.restype = c_longlong
lib.omCudaStemWorkspaceBytes.argtypes = [I, I, I, I, I, I, I, I]
lib.omCudaStemWorkspaceBytes.restype = c_longlong
lib.omCudaStoredChannels.argtypes = [I]
lib.omCudaStoredChannels.restype = c_int
lib.omCudaConvInputSplitBytes.argtypes = [I, I, I, I, I]
lib.omCudaConvInputSplitBytes.restype = c_longlong
lib.omCudaStemInputSplitBytes.argtypes = [I, I, I, I, I, I, I, I]
lib.omCudaStemInputSplitBytes.restype = c_longlong

EXPORTED = sorted(list(_SIGS) + ["omCudaGetStream", "omCudaPackedConvWeightElems",
                                 "omCudaPackedStemWeightElems", "omCudaStemWorkspaceBytes",
                                 "omCudaStoredChannels", "omCudaConvInputSplitBytes",
                                 "omCudaStemInputSplitBytes"])


def check(status: int, fn: str = "omCuda") -> None:
    if status != OM_OK:
        raise OmCudaError(fn, status)


def call(name: str, *args) -> None:
    """Call an entry point by name and raise OmCudaError on a non-zero status."""
    check(getattr(lib, name)(*args), name)
