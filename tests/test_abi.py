"""CPU-only checks of the drop-in boundary: the library loads and exports every entry point
that include/om_cuda.h declares, and entry points report errors instead of faulting when no
device has been initialised on the calling thread."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "om_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(om(?:Cuda|Nccl)\w+)\s*\(", src)))


def test_header_declares_reference_hot_path():
    names = _declared()
    for ref_name in ("omCudaConv2d", "omCudaConv2dBackwardInput", "omCudaConv2dBackwardWeight",
                     "omCudaBatchNorm2d", "omCudaBatchNorm2dBackward", "omCudaMaxPool2d",
                     "omCudaMaxPool2dBackward", "omCudaAdaptiveAvgPool2d", "omCudaReLU",
                     "omCudaSoftmax", "omCudaCrossEntropy", "omCudaSoftmaxCrossEntropyBackward",
                     "omCudaSgdStep", "omCudaMatmul", "omCudaAddBias", "omCudaMalloc",
                     "omCudaGraphLaunch"):
        assert ref_name in names


def test_library_exports_every_declared_symbol():
    from omnimatchdeeplearningtool_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding covers the header exactly
    assert sorted(_lib.EXPORTED) == _declared()


def test_calls_without_init_report_not_init():
    # a fresh thread has no current device: every entry point must return OM_ERR_NOT_INIT
    import threading
    from omnimatchdeeplearningtool_b200._lib import lib
    res = {}

    def probe():
        res["relu"] = lib.omCudaReLU(None, None, 0)
        res["conv"] = lib.omCudaConv2dBnAct(None, None, None, None, None, 1, 1, 1, 8, 8, 1, 1, 1,
                                            0, 0, 1, 1)
        res["sync"] = lib.omCudaSynchronize()

    t = threading.Thread(target=probe)
    t.start()
    t.join()
    assert res == {"relu": -4, "conv": -4, "sync": -4}


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    import importlib
    import omnimatchdeeplearningtool_b200._lib as L
    monkeypatch.setattr(L, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(ImportError):
        L._load()


# every extern "C" entry point of the reference's src/cuda/cuda_kernels.cuh (97 functions)
REFERENCE_ENTRY_POINTS = [
    "omCudaAdamStep", "omCudaAdaptiveAvgPool2d", "omCudaAdaptiveAvgPool2dBackward", "omCudaAdd",
    "omCudaAddBias", "omCudaAddBiasBackward", "omCudaAddScalar", "omCudaArgmax",
    "omCudaAsyncCopyD2H", "omCudaAsyncCopyH2D", "omCudaAvgPool2d", "omCudaAvgPool2dBackward",
    "omCudaBCEWithLogits", "omCudaBCEWithLogitsBackward", "omCudaBatchNorm2d",
    "omCudaBatchNorm2dBackward", "omCudaBatchedMatmul", "omCudaCleanup", "omCudaClip",
    "omCudaConcatChannels", "omCudaConcatChannelsBackward", "omCudaConcatLastDim",
    "omCudaConcatLastDimBackward", "omCudaConv2d", "omCudaConv2dBackwardInput",
    "omCudaConv2dBackwardWeight", "omCudaConv2dIm2col", "omCudaConvTranspose2d", "omCudaCopy",
    "omCudaCopyD2D", "omCudaCopyD2H", "omCudaCopyH2D", "omCudaCrossEntropy",
    "omCudaDiceLossBackward", "omCudaDiceLossForward", "omCudaDilatedConv2d",
    "omCudaDilatedConv2dBackwardWeight", "omCudaDiv", "omCudaDropout", "omCudaDropoutForward",
    "omCudaFillOnes", "omCudaFillValue", "omCudaFillZeros", "omCudaFree", "omCudaFreeHost",
    "omCudaGELU", "omCudaGeluBackward", "omCudaGetComputeCapability", "omCudaGetDeviceCount",
    "omCudaGetDeviceName", "omCudaGetMemInfo", "omCudaGraphBeginCapture", "omCudaGraphDestroy",
    "omCudaGraphEndCapture", "omCudaGraphLaunch", "omCudaGroupNorm2d",
    "omCudaGroupNorm2dBackward", "omCudaInit", "omCudaLayerNorm", "omCudaLayerNormBackward",
    "omCudaLeakyRelu", "omCudaLeakyReluBackward", "omCudaMalloc", "omCudaMallocHost",
    "omCudaMatmul", "omCudaMaxPool2d", "omCudaMaxPool2dBackward", "omCudaMean", "omCudaMemset",
    "omCudaMergeHeads", "omCudaMul", "omCudaMulScalar", "omCudaQkvSplitHeads", "omCudaReLU",
    "omCudaReLUBackward", "omCudaSgdStep", "omCudaSiLU", "omCudaSigmoid",
    "omCudaSigmoidBackward", "omCudaSiluBackward", "omCudaSliceLastDim",
    "omCudaSliceLastDimBackward", "omCudaSoftmax", "omCudaSoftmaxCrossEntropyBackward",
    "omCudaSoftmaxLastDimBackward", "omCudaSub", "omCudaSum", "omCudaSyncComputeStream",
    "omCudaSyncTransferStream", "omCudaSynchronize", "omCudaTanh", "omCudaTanhBackward",
    "omCudaTranspose", "omCudaUpsampleBilinear", "omCudaUpsampleBilinearBackward",
    "omCudaWeightedPixelCEBackward", "omCudaWeightedPixelCEForward",
]


def test_header_and_library_cover_every_reference_entry_point():
    from omnimatchdeeplearningtool_b200 import _lib
    assert len(REFERENCE_ENTRY_POINTS) == 97
    declared = set(_declared())
    assert not [n for n in REFERENCE_ENTRY_POINTS if n not in declared]
    lib = ctypes.CDLL(_lib.LIB_PATH)
    assert not [n for n in REFERENCE_ENTRY_POINTS if not hasattr(lib, n)]
