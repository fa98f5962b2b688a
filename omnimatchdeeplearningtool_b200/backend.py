"""Host-side mirror of the reference's ``om::CUDABackend`` (src/hal/om.hal.cuda_backend.ixx).

Each static method keeps the reference method's name and argument order (including the
argument orders that differ from the C ABI, e.g. ``conv2d``'s pad-before-stride and
``batchNorm2d``'s gamma/beta-before-output) and forwards to one C-ABI entry point of
libomcuda.so. Unlike the reference wrapper, which discards every return code
(cuda_backend.ixx:325-329, :438-452), a non-zero status raises :class:`OmCudaError`.

Pointers are plain device addresses (``int``) such as :attr:`DeviceBuffer.ptr`.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import OmCudaError, call, lib  # noqa: F401  (re-exported)

_NP_FROM_DT = {0: np.float32}


def init(device: int = 0) -> None:
    """omCudaInit for the calling thread (cuda_kernels.cu:287)."""
    call("omCudaInit", device)


def synchronize() -> None:
    call("omCudaSynchronize")


def stream_handle() -> int:
    """The library's compute stream on the calling thread's device (cudaStream_t)."""
    return int(lib.omCudaGetStream() or 0)


def kernel_error() -> int:
    code = ctypes.c_uint(0)
    call("omCudaGetKernelError", ctypes.byref(code))
    return int(code.value)


def launch_count() -> int:
    n = ctypes.c_ulonglong(0)
    call("omCudaGetLaunchCount", ctypes.byref(n))
    return int(n.value)


class DeviceBuffer:
    """A device allocation from omCudaMalloc, freed with omCudaFree."""

    def __init__(self, nbytes: int):
        self.nbytes = int(max(nbytes, 1))
        p = ctypes.c_void_p()
        call("omCudaMalloc", ctypes.byref(p), self.nbytes)
        self.ptr = int(p.value)

    @classmethod
    def from_numpy(cls, arr: np.ndarray) -> "DeviceBuffer":
        arr = np.ascontiguousarray(arr)
        buf = cls(arr.nbytes)
        call("omCudaCopyH2D", buf.ptr, arr.ctypes.data, arr.nbytes)
        return buf

    @classmethod
    def zeros(cls, nbytes: int) -> "DeviceBuffer":
        buf = cls(nbytes)
        call("omCudaMemset", buf.ptr, 0, buf.nbytes)
        return buf

    def upload(self, arr: np.ndarray) -> None:
        arr = np.ascontiguousarray(arr)
        assert arr.nbytes <= self.nbytes
        call("omCudaCopyH2D", self.ptr, arr.ctypes.data, arr.nbytes)

    def to_numpy(self, shape, dtype=np.float32) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        assert out.nbytes <= self.nbytes
        call("omCudaCopyD2H", out.ctypes.data, self.ptr, out.nbytes)
        return out

    def free(self) -> None:
        if getattr(self, "ptr", 0):
            try:
                lib.omCudaFree(self.ptr)
            finally:
                self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class CUDABackend:
    """Static methods named and ordered as om::CUDABackend (om.hal.cuda_backend.ixx:283-984)."""

    @staticmethod
    def add(a, b, out, n):  # :288
        call("omCudaAdd", a, b, out, n)

    @staticmethod
    def mulScalar(a, s, out, n):
        call("omCudaMulScalar", a, s, out, n)

    @staticmethod
    def matmul(a, b, c, m, k, n):  # :325
        call("omCudaMatmul", a, b, c, m, k, n)

    @staticmethod
    def transpose(inp, out, rows, cols):
        call("omCudaTranspose", inp, out, rows, cols)

    @staticmethod
    def relu(inp, out, n):  # :349
        call("omCudaReLU", inp, out, n)

    @staticmethod
    def reluBackward(inp, grad_out, grad_in, n):
        call("omCudaReLUBackward", inp, grad_out, grad_in, n)

    @staticmethod
    def conv2d(inp, w, b, out, N, Cin, H, W, Cout, KH, KW, padH, padW, strH, strW):  # :438
        if padH != padW or strH != strW:
            raise OmCudaError("conv2d (asymmetric pad/stride)", -3)
        call("omCudaConv2d", inp, w, b, out, N, Cin, H, W, Cout, KH, KW, strH, padH)

    @staticmethod
    def dilatedConv2d(inp, w, b, out, N, Cin, H, W, Cout, KH, KW, stride, pad, dil, groups):
        call("omCudaDilatedConv2d", inp, w, b, out, N, Cin, H, W, Cout, KH, KW, stride, pad,
             dil, groups)

    @staticmethod
    def conv2dBackwardInput(dy, w, dx, N, Cin, H, W, Cout, KH, KW, padH, padW, strH, strW):  # :480
        call("omCudaConv2dBackwardInput", dy, w, dx, N, Cin, H, W, Cout, KH, KW, strH, padH)

    @staticmethod
    def conv2dBackwardWeight(x, dy, dw, db, N, Cin, H, W, Cout, KH, KW, padH, padW, strH, strW):  # :492
        call("omCudaConv2dBackwardWeight", x, dy, dw, db, N, Cin, H, W, Cout, KH, KW, strH, padH)

    @staticmethod
    def maxPool2d(inp, out, idx, N, C, H, W, KH, KW, stride, pad):  # :506
        call("omCudaMaxPool2d", inp, out, idx, N, C, H, W, KH, KW, stride, stride, pad, pad)

    @staticmethod
    def maxPool2dBackward(dy, idx, dx, N, C, H, W, Hout, Wout):  # :519
        call("omCudaMemset", dx, 0, N * C * H * W * 4)
        call("omCudaMaxPool2dBackward", dy, idx, dx, N, C, H, W, Hout, Wout)

    @staticmethod
    def avgPool2d(inp, out, N, C, H, W, KH, KW, stride, pad):
        call("omCudaAvgPool2d", inp, out, N, C, H, W, KH, KW, stride, stride, pad, pad)

    @staticmethod
    def avgPool2dBackward(dy, dx, N, C, H, W, KH, KW, stride, pad):
        call("omCudaMemset", dx, 0, N * C * H * W * 4)
        call("omCudaAvgPool2dBackward", dy, dx, N, C, H, W, KH, KW, stride, stride, pad, pad)

    @staticmethod
    def adaptiveAvgPool2d(inp, out, N, C, H, W, OH, OW):  # :560
        call("omCudaAdaptiveAvgPool2d", inp, out, N, C, H, W, OH, OW)

    @staticmethod
    def adaptiveAvgPool2dBackward(dy, dx, N, C, H, W, OH, OW):
        call("omCudaAdaptiveAvgPool2dBackward", dy, dx, N, C, H, W, OH, OW)

    @staticmethod
    def batchNorm2d(inp, gamma, beta, out, run_mean, run_var, saved_mean, saved_invstd, N, C,
                    HW, eps, momentum, training):  # :571 (note: gamma/beta before out)
        call("omCudaBatchNorm2d", inp, out, gamma, beta, run_mean, run_var, saved_mean,
             saved_invstd, N, C, 1, HW, eps, momentum, 1 if training else 0)

    @staticmethod
    def batchNorm2dBackward(dy, x, mean, invstd, gamma, dx, dgamma, dbeta, N, C, H, W,
                            eps=1e-5):  # :590
        call("omCudaBatchNorm2dBackward", dy, x, mean, invstd, gamma, dx, dgamma, dbeta, N, C,
             H, W, eps)

    @staticmethod
    def softmax(inp, out, N, C):  # :652
        call("omCudaSoftmax", inp, out, N, C)

    @staticmethod
    def crossEntropySoftmaxBackward(p, target, grad, N, C):  # :659
        call("omCudaSoftmaxCrossEntropyBackward", p, target, grad, N, C)

    @staticmethod
    def crossEntropyForward(p, target, result, N, C):  # :823
        call("omCudaCrossEntropy", p, target, result, N, C)

    @staticmethod
    def sgdStep(param, grad, vel, n, lr, momentum):  # :679
        call("omCudaSgdStep", param, grad, vel, n, lr, momentum)

    @staticmethod
    def fillZeros(data, n):  # :689
        call("omCudaFillZeros", data, n)

    @staticmethod
    def fillOnes(data, n):
        call("omCudaFillOnes", data, n)

    @staticmethod
    def fillValue(data, n, v):
        call("omCudaFillValue", data, n, v)

    @staticmethod
    def copy(src, dst, n):  # :710
        call("omCudaCopy", src, dst, n)

    @staticmethod
    def addBias(data, bias, out, N, C, HW):  # :717
        call("omCudaAddBias", data, bias, out, N, C, HW)

    @staticmethod
    def addBiasBackward(dy, db, N, C, HW):
        call("omCudaAddBiasBackward", dy, db, N, C, HW)

    @staticmethod
    def clip(inp, out, n, lo, hi):  # :789
        call("omCudaClip", inp, out, n, lo, hi)

    @staticmethod
    def argmax(data, out, N, C):
        call("omCudaArgmax", data, out, N, C)

    @staticmethod
    def sum(data, result, n):
        call("omCudaSum", data, result, n)

    # ---- the reference wrapper's remaining methods (same names and argument orders; all
    # forward their arguments unchanged to the C-ABI entry point of the same name)
    @staticmethod
    def sub(a, b, out, n):  # :295
        call("omCudaSub", a, b, out, n)

    @staticmethod
    def mul(a, b, out, n):  # :302
        call("omCudaMul", a, b, out, n)

    @staticmethod
    def addScalar(a, s, out, n):  # :309
        call("omCudaAddScalar", a, s, out, n)

    @staticmethod
    def div(a, b, out, n):  # :782
        call("omCudaDiv", a, b, out, n)

    @staticmethod
    def batchedMatmul(a, b, c, batch, m, k, n):  # :332
        call("omCudaBatchedMatmul", a, b, c, batch, m, k, n)

    @staticmethod
    def sigmoid(inp, out, n):  # :363
        call("omCudaSigmoid", inp, out, n)

    @staticmethod
    def sigmoidBackward(grad, output, out, n):  # :370
        call("omCudaSigmoidBackward", grad, output, out, n)

    @staticmethod
    def gelu(inp, out, n):  # :377
        call("omCudaGELU", inp, out, n)

    @staticmethod
    def geluBackward(grad, inp, out, n):  # :384
        call("omCudaGeluBackward", grad, inp, out, n)

    @staticmethod
    def silu(inp, out, n):  # :391
        call("omCudaSiLU", inp, out, n)

    @staticmethod
    def siluBackward(grad, inp, out, n):  # :398
        call("omCudaSiluBackward", grad, inp, out, n)

    @staticmethod
    def leakyRelu(inp, out, n, slope=0.01):  # :405
        call("omCudaLeakyRelu", inp, out, n, slope)

    @staticmethod
    def leakyReluBackward(grad, inp, out, n, slope=0.01):  # :412
        call("omCudaLeakyReluBackward", grad, inp, out, n, slope)

    @staticmethod
    def tanhForward(inp, out, n):  # :420
        call("omCudaTanh", inp, out, n)

    @staticmethod
    def tanhBackward(grad, output, out, n):  # :427
        call("omCudaTanhBackward", grad, output, out, n)

    @staticmethod
    def dilatedConv2dBackwardWeight(x, dy, dw, db, N, Cin, H, W, Cout, KH, KW, stride, pad,
                                    dil):  # :467
        call("omCudaDilatedConv2dBackwardWeight", x, dy, dw, db, N, Cin, H, W, Cout, KH, KW,
             stride, pad, dil)

    @staticmethod
    def groupNorm2d(inp, out, gamma, beta, mean, invstd, N, C, H, W, groups, eps):  # :607
        call("omCudaGroupNorm2d", inp, out, gamma, beta, mean, invstd, N, C, H, W, groups, eps)

    @staticmethod
    def groupNorm2dBackward(dy, x, mean, invstd, gamma, dx, dgamma, dbeta, N, C, H, W, groups,
                            eps):  # :624
        call("omCudaGroupNorm2dBackward", dy, x, mean, invstd, gamma, dx, dgamma, dbeta, N, C, H,
             W, groups, eps)

    @staticmethod
    def layerNorm(inp, out, gamma, beta, mean, invstd, batch, dim, eps):  # :639
        call("omCudaLayerNorm", inp, out, gamma, beta, mean, invstd, batch, dim, eps)

    @staticmethod
    def layerNormBackward(dy, x, mean, invstd, gamma, dx, dgamma, dbeta, batch, dim):  # :833
        call("omCudaLayerNormBackward", dy, x, mean, invstd, gamma, dx, dgamma, dbeta, batch, dim)

    @staticmethod
    def adamStep(param, grad, m, v, n, lr, b1, b2, eps, step):  # :670
        call("omCudaAdamStep", param, grad, m, v, n, lr, b1, b2, eps, step)

    @staticmethod
    def upsampleBilinear(inp, out, N, C, H, W, OH, OW):  # :796
        call("omCudaUpsampleBilinear", inp, out, N, C, H, W, OH, OW)

    @staticmethod
    def upsampleBilinearBackward(dy, dx, N, C, IH, IW, OH, OW):  # :755
        call("omCudaUpsampleBilinearBackward", dy, dx, N, C, IH, IW, OH, OW)

    @staticmethod
    def concatChannels(a, b, out, N, C1, C2, HW):  # :804
        call("omCudaConcatChannels", a, b, out, N, C1, C2, HW)

    @staticmethod
    def concatChannelsBackward(dy, da, db, N, CA, CB, HW):  # :763
        call("omCudaConcatChannelsBackward", dy, da, db, N, CA, CB, HW)

    @staticmethod
    def bceWithLogitsForward(logits, targets, result, n):  # :813
        call("omCudaBCEWithLogits", logits, targets, result, n)

    @staticmethod
    def bceWithLogitsBackward(logits, targets, grad, n, inv_n):  # :772
        call("omCudaBCEWithLogitsBackward", logits, targets, grad, n, inv_n)

    @staticmethod
    def convTranspose2d(inp, w, b, out, N, Cin, H, W, Cout, KH, KW, stride, pad):  # :846
        call("omCudaConvTranspose2d", inp, w, b, out, N, Cin, H, W, Cout, KH, KW, stride, pad)

    @staticmethod
    def concatLastDim(a, b, out, outer, da, db):  # :857
        call("omCudaConcatLastDim", a, b, out, outer, da, db)

    @staticmethod
    def concatLastDimBackward(dy, ga, gb, outer, da, db):  # :865
        call("omCudaConcatLastDimBackward", dy, ga, gb, outer, da, db)

    @staticmethod
    def sliceLastDim(inp, out, outer, full, start, length):  # :874
        call("omCudaSliceLastDim", inp, out, outer, full, start, length)

    @staticmethod
    def sliceLastDimBackward(dy, dx, outer, full, start, length):  # :882
        call("omCudaSliceLastDimBackward", dy, dx, outer, full, start, length)

    @staticmethod
    def softmaxLastDimBackward(dy, s, dx, outer, last):  # :894
        call("omCudaSoftmaxLastDimBackward", dy, s, dx, outer, last)

    @staticmethod
    def dropoutForward(inp, out, mask, n, keep, seed):  # :905
        call("omCudaDropoutForward", inp, out, mask, n, keep, seed)

    @staticmethod
    def diceLossForward(logits, target, loss, sig, stats, n):  # :916
        call("omCudaDiceLossForward", logits, target, loss, sig, stats, n)

    @staticmethod
    def diceLossBackward(sig, target, stats, gout, grad, n):  # :927
        call("omCudaDiceLossBackward", sig, target, stats, gout, grad, n)

    @staticmethod
    def weightedPixelCEForward(logits, target, cw, soft, loss, stats, P, K, S):  # :938
        call("omCudaWeightedPixelCEForward", logits, target, cw, soft, loss, stats, P, K, S)

    @staticmethod
    def weightedPixelCEBackward(soft, target, cw, gout, stats, grad, P, K, S):  # :951
        call("omCudaWeightedPixelCEBackward", soft, target, cw, gout, stats, grad, P, K, S)

    @staticmethod
    def qkvSplitHeads(qkv, q, k, v, N, S, H, D, scale):  # :967
        call("omCudaQkvSplitHeads", qkv, q, k, v, N, S, H, D, scale)

    @staticmethod
    def mergeHeads(inp, out, N, S, H, D):  # :977
        call("omCudaMergeHeads", inp, out, N, S, H, D)
