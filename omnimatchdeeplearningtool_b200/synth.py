"""Architectures and seeded synthetic data for the benchmark configurations.

Architectures are described layer by layer with the parameter names, shapes and order that
the reference's modules report through ``Module::namedParameters()`` / ``namedBuffers()``
(om.engine.module.ixx:71-166):

* ImageNet ResNet-18/50: Conv2d(3,64,7,2,3) + BatchNorm2d + ReLU + MaxPool2d(3,2,1), then
  BasicBlock (om.engine.resnet.ixx:31-177) or Bottleneck (om.engine.resnet50.ixx:28-191)
  stages, AdaptiveAvgPool2d(1,1), Flatten, Linear(in, classes) with weight ``[in, out]`` and
  bias ``[1, out]`` (om.engine.linear.ixx:27-45). Stride sits on the 3x3 conv of a
  Bottleneck and on conv1 of a BasicBlock; the downsample is a strided 1x1 conv + BN.
* MobileNet-style stack: ConvBnReLU6(3,32,3,s2,p1) stem, 12 InvertedResidual(expand 4)
  blocks (om.engine.mobilenet.ixx:177-240), 3 per stage at widths 32/64/128/256, stride 2 on
  the first block of stages 2-4, global pool, Linear(256, classes).

Synthetic data (the reference ships no weights or dataset; BASELINE fixes the recipe):
inputs U[0,1) from seed 0, normalised per channel with the ImageNet mean/std (config 1) or
N(0,1) (configs 3-5); He-normal conv and FC weights N(0, 2/fan_in) drawn in parameter order
from seed 1; BN gamma=1, beta=0, running_mean ~ N(0, 0.1^2), running_var ~ U(0.5, 1.5) drawn
in buffer order from seed 2. All draws use numpy's PCG64 so both sides of every comparison
see identical bits.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Tuple

import numpy as np

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


@dataclass
class ConvSpec:
    name: str            # e.g. "layer1.0.conv1"
    cin: int
    cout: int
    k: int
    stride: int
    pad: int
    groups: int = 1
    bn: str = ""         # BatchNorm2d name that follows, e.g. "layer1.0.bn1"


@dataclass
class BlockSpec:
    kind: str                      # "basic" | "bottleneck" | "inverted"
    convs: List[ConvSpec]          # main path in execution order
    downsample: ConvSpec = None    # 1x1 strided conv + BN on the shortcut, or None
    residual: bool = True          # inverted blocks add the input only when shapes match


@dataclass
class NetSpec:
    name: str
    stem: List[ConvSpec]
    stem_act: str                  # "relu" | "relu6"
    maxpool: bool
    blocks: List[BlockSpec]
    fc_in: int
    classes: int
    params: List[Tuple[str, Tuple[int, ...]]] = field(default_factory=list)
    buffers: List[Tuple[str, Tuple[int, ...]]] = field(default_factory=list)


def _bn_entries(bn: str, c: int):
    return [(bn + ".gamma", (c,)), (bn + ".beta", (c,))], \
           [(bn + ".running_mean", (c,)), (bn + ".running_var", (c,))]


def _add_conv(net: NetSpec, cv: ConvSpec):
    net.params.append((cv.name + ".weight", (cv.cout, cv.cin // cv.groups, cv.k, cv.k)))
    p, b = _bn_entries(cv.bn, cv.cout)
    net.params.extend(p)
    return b


def resnet_spec(depth: int, classes: int = 1000) -> NetSpec:
    """ImageNet-stem ResNet-18 (depth 18) or ResNet-50 (depth 50)."""
    assert depth in (18, 50)
    stem = [ConvSpec("conv1", 3, 64, 7, 2, 3, bn="bn1")]
    blocks: List[BlockSpec] = []
    counts = (2, 2, 2, 2) if depth == 18 else (3, 4, 6, 3)
    cin = 64
    for s, n in enumerate(counts):
        planes = 64 << s
        for b in range(n):
            stride = 2 if (s > 0 and b == 0) else 1
            pre = f"layer{s + 1}.{b}"
            if depth == 18:
                convs = [ConvSpec(pre + ".conv1", cin, planes, 3, stride, 1, bn=pre + ".bn1"),
                         ConvSpec(pre + ".conv2", planes, planes, 3, 1, 1, bn=pre + ".bn2")]
                cout = planes
                kind = "basic"
            else:
                convs = [ConvSpec(pre + ".conv1", cin, planes, 1, 1, 0, bn=pre + ".bn1"),
                         ConvSpec(pre + ".conv2", planes, planes, 3, stride, 1, bn=pre + ".bn2"),
                         ConvSpec(pre + ".conv3", planes, planes * 4, 1, 1, 0, bn=pre + ".bn3")]
                cout = planes * 4
                kind = "bottleneck"
            ds = None
            if stride != 1 or cin != cout:
                ds = ConvSpec(pre + ".downsample_conv", cin, cout, 1, stride, 0,
                              bn=pre + ".downsample_bn")
            blocks.append(BlockSpec(kind, convs, ds))
            cin = cout
    net = NetSpec(f"resnet{depth}", stem, "relu", True, blocks, cin, classes)
    bufs = _add_conv(net, stem[0])
    net.buffers.extend(bufs)
    for blk in blocks:
        # parameters: convs with their BNs in order, then downsample; buffers: the BNs in the
        # same order (resnet.ixx:109-152, resnet50.ixx:304-366)
        for cv in blk.convs:
            net.buffers.extend(_add_conv(net, cv))
        if blk.downsample is not None:
            net.buffers.extend(_add_conv(net, blk.downsample))
    net.params.append(("fc.weight", (cin, classes)))
    net.params.append(("fc.bias", (1, classes)))
    return net


def mobilenet_spec(classes: int = 1000) -> NetSpec:
    """MobileNet-style depthwise-separable stack (config 5)."""
    stem = [ConvSpec("stem.conv", 3, 32, 3, 2, 1, bn="stem.bn")]
    blocks: List[BlockSpec] = []
    widths = (32, 64, 128, 256)
    cin = 32
    for s in range(4):
        for b in range(3):
            stride = 2 if (s > 0 and b == 0) else 1
            pre = f"blocks.{s * 3 + b}"
            hid = cin * 4
            cout = widths[s]
            convs = [ConvSpec(pre + ".expand.conv", cin, hid, 1, 1, 0, bn=pre + ".expand.bn"),
                     ConvSpec(pre + ".depthwise.conv", hid, hid, 3, stride, 1, groups=hid,
                              bn=pre + ".depthwise.bn"),
                     ConvSpec(pre + ".project.conv", hid, cout, 1, 1, 0, bn=pre + ".project.bn")]
            blocks.append(BlockSpec("inverted", convs, None,
                                    residual=(stride == 1 and cin == cout)))
            cin = cout
    net = NetSpec("mobilenet", stem, "relu6", False, blocks, cin, classes)
    net.buffers.extend(_add_conv(net, stem[0]))
    for blk in blocks:
        for cv in blk.convs:
            net.buffers.extend(_add_conv(net, cv))
    net.params.append(("fc.weight", (cin, classes)))
    net.params.append(("fc.bias", (1, classes)))
    return net


def make_weights(net: NetSpec, weight_seed: int = 1, buffer_seed: int = 2) -> Dict[str, np.ndarray]:
    """He-normal conv/FC weights, BN gamma=1/beta=0, FC bias 0; BN running stats seeded."""
    rng = np.random.Generator(np.random.PCG64(weight_seed))
    out: Dict[str, np.ndarray] = {}
    for name, shape in net.params:
        if name.endswith(".gamma"):
            out[name] = np.ones(shape, np.float32)
        elif name.endswith(".beta") or name == "fc.bias":
            out[name] = np.zeros(shape, np.float32)
        elif name == "fc.weight":
            fan_in = shape[0]
            out[name] = (rng.standard_normal(shape) * np.sqrt(2.0 / fan_in)).astype(np.float32)
        else:
            fan_in = int(np.prod(shape[1:]))
            out[name] = (rng.standard_normal(shape) * np.sqrt(2.0 / fan_in)).astype(np.float32)
    rng = np.random.Generator(np.random.PCG64(buffer_seed))
    for name, shape in net.buffers:
        if name.endswith("running_mean"):
            out[name] = (rng.standard_normal(shape) * 0.1).astype(np.float32)
        else:
            out[name] = rng.uniform(0.5, 1.5, shape).astype(np.float32)
    return out


def imagenet_input(n: int, h: int = 224, w: int = 224, seed: int = 0) -> np.ndarray:
    """Config 1 input: U[0,1) from seed 0, then per-channel (x - mean) / std."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.random((n, 3, h, w), dtype=np.float32)
    mean = np.array(IMAGENET_MEAN, np.float32).reshape(1, 3, 1, 1)
    std = np.array(IMAGENET_STD, np.float32).reshape(1, 3, 1, 1)
    return ((x - mean) / std).astype(np.float32)


def normal_input(n: int, c: int = 3, h: int = 224, w: int = 224, seed: int = 0) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((n, c, h, w), dtype=np.float32)


def onehot_labels(n: int, classes: int = 1000, seed: int = 3) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    y = rng.integers(0, classes, n)
    oh = np.zeros((n, classes), np.float32)
    oh[np.arange(n), y] = 1.0
    return oh


def conv_flops(net: NetSpec, h: int = 224, w: int = 224) -> int:
    """Algorithmic FLOPs per image: 2*K*(C/g)*R*S*P*Q per conv plus 2*F*classes for the FC."""
    total = 0

    def conv(cv: ConvSpec, hh, ww):
        nonlocal total
        p = (hh + 2 * cv.pad - cv.k) // cv.stride + 1
        q = (ww + 2 * cv.pad - cv.k) // cv.stride + 1
        total += 2 * cv.cout * (cv.cin // cv.groups) * cv.k * cv.k * p * q
        return p, q

    hh, ww = h, w
    for cv in net.stem:
        hh, ww = conv(cv, hh, ww)
    if net.maxpool:
        hh, ww = (hh + 2 - 3) // 2 + 1, (ww + 2 - 3) // 2 + 1
    for blk in net.blocks:
        h0, w0 = hh, ww
        for cv in blk.convs:
            hh, ww = conv(cv, hh, ww)
        if blk.downsample is not None:
            conv(blk.downsample, h0, w0)
    total += 2 * net.fc_in * net.classes
    return total


def conv_layer_data(c: int, h: int, ks: int, n: int, seed: int):
    """Config 2's single conv2d + BatchNorm2d + ReLU layer with C = K = c on an h x h input:
    N(0,1) input, He-normal weights, BN gamma U(0.5,1.5), beta N(0,0.1), running mean N(0,0.1),
    running var U(0.5,1.5), all from one seed. Returns (x, w, gamma, beta, mean, var)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((c, c, ks, ks)) * np.sqrt(2.0 / (c * ks * ks))).astype(np.float32)
    g = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = (rng.standard_normal(c) * 0.1).astype(np.float32)
    mu = (rng.standard_normal(c) * 0.1).astype(np.float32)
    var = rng.uniform(0.5, 1.5, c).astype(np.float32)
    return x, w, g, b, mu, var
