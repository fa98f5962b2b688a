"""Multi-device batch classification (omnimatchdeeplearningtool_b200/serving.py), the form of the
reference's EngineBridge::inferBatch that uses every GPU.

CPU tests replace the per-device plan with a fake that records what it was given, to check the
dealing of chunks, the zero padding of the ragged end, the order of the results and error
reporting. classify_logits is checked against a restatement of the reference's per-image loop
(EngineBridge.cpp:3691-3717). The GPU test compares the classifier's logits with one plan's on
the same images, on every visible device."""
import math
import threading

import numpy as np
import pytest

from omnimatchdeeplearningtool_b200 import serving


class _FakePlan:
    """Logit row = [device, first pixel of the image, count of calls so far on this plan]."""

    def __init__(self, device, log):
        self.device, self.log, self.calls = device, log, 0

    def run(self, x):
        self.log.append((self.device, threading.current_thread().name, x.shape[0],
                         float(x[-1].sum())))
        self.calls += 1
        return np.stack([np.array([self.device, img.flat[0], self.calls], np.float32)
                         for img in x])

    def close(self):
        self.log.append((self.device, "closed"))


def _classifier(devices, batch, log, init_log=None):
    def init(d):
        if init_log is not None:
            init_log.append((d, threading.current_thread().name))
    return serving.MultiDeviceClassifier(None, {}, devices, batch, h=2, w=2,
                                         make_plan=lambda d: _FakePlan(d, log), init_device=init)


def test_chunks_are_dealt_round_robin_padded_and_reassembled():
    log, inits = [], []
    clf = _classifier([3, 5, 7], 4, log, inits)
    n = 4 * 7 + 2  # seven full chunks and a ragged one of 2
    x = np.zeros((n, 3, 2, 2), np.float32)
    x[:, 0, 0, 0] = np.arange(n) + 1
    out = clf.infer_logits(x)
    assert out.shape == (n, 3)
    assert np.array_equal(out[:, 1], np.arange(n) + 1)  # input order kept
    chunk_dev = [out[i * 4, 0] for i in range(math.ceil(n / 4))]
    assert chunk_dev == [3, 5, 7, 3, 5, 7, 3, 5]  # chunk i on device i mod 3
    runs = [e for e in log if len(e) == 4]
    assert all(e[2] == 4 for e in runs)  # every call sees a full batch
    assert any(e[3] == 0.0 for e in runs)  # the padded rows of the last chunk are zeros
    # each device is initialised and driven by its own thread
    names = {d: t for d, t in inits}
    assert sorted(names) == [3, 5, 7] and len(set(names.values())) == 3
    assert all(names[e[0]] == e[1] for e in runs)
    clf.close()
    assert sorted(e[0] for e in log if e[1] == "closed") == [3, 5, 7]


def test_single_image_infer():
    """infer(image): one [C, H, W] image through the first device, the reference's single-image
    result; a wrongly shaped image is refused."""
    log = []
    clf = _classifier([2, 4], 1, log)
    x = np.zeros((3, 2, 2), np.float32)
    x[0, 0, 0] = 9.0
    r = clf.infer(x)
    assert isinstance(r, serving.InferResult)
    assert r.probs.shape == (3,)
    runs = [e for e in log if len(e) == 4]
    assert [e[0] for e in runs] == [2]
    with pytest.raises(ValueError):
        clf.infer(np.zeros((1, 3, 2, 2), np.float32))
    clf.close()


def test_arguments_and_failures_are_reported():
    log = []
    with pytest.raises(ValueError):
        _classifier([0, 0], 2, log)
    with pytest.raises(ValueError):
        _classifier([], 2, log)
    clf = _classifier([0], 2, log)
    with pytest.raises(ValueError):
        clf.infer_logits(np.zeros((2, 3, 4, 4), np.float32))  # wrong image size
    clf.close()

    def bad_init(d):
        raise RuntimeError("no such device")
    with pytest.raises(RuntimeError, match="setup failed"):
        serving.MultiDeviceClassifier(None, {}, [0, 1], 2, h=2, w=2,
                                      make_plan=lambda d: _FakePlan(d, log), init_device=bad_init)

    class Failing(_FakePlan):
        def run(self, x):
            raise RuntimeError("kernel failed")
    clf = serving.MultiDeviceClassifier(None, {}, [0], 2, h=2, w=2,
                                        make_plan=lambda d: Failing(d, log),
                                        init_device=lambda d: None)
    with pytest.raises(RuntimeError, match="chunk 0 failed"):
        clf.infer_logits(np.zeros((2, 3, 2, 2), np.float32))
    clf.close()


def _reference_result(row, threshold):
    """The reference's per-image loop, element by element in float32."""
    m = max(row)
    probs = [np.float32(math.exp(np.float32(v) - m)) for v in row]
    s = np.float32(0)
    for p in probs:
        s = np.float32(s + p)
    best, best_p = 0, 0.0
    out = []
    for c, p in enumerate(probs):
        q = np.float32(p / max(s, np.float32(1e-8)))
        out.append(q)
        if q > best_p:
            best, best_p = c, q
    return (best if best_p >= threshold else -1), best_p, np.array(out, np.float32)


def test_classify_logits_follows_the_reference():
    rng = np.random.Generator(np.random.PCG64(3))
    z = (rng.standard_normal((50, 7)) * 3).astype(np.float32)
    z[0] = 0.0  # uniform: confidence 1/7, below the threshold -> class -1
    res = serving.classify_logits(z, 0.5)
    for row, r in zip(z, res):
        cls, conf, probs = _reference_result(row.tolist(), 0.5)
        assert r.predicted_class == cls
        assert abs(r.confidence - conf) <= 1e-6
        assert np.allclose(r.probs, probs, rtol=1e-6, atol=1e-7)
    assert res[0].predicted_class == -1


@pytest.mark.gpu
def test_multi_device_logits_match_one_plan(gpu):
    """Every visible device (one thread each) against a single plan on device 0: identical
    logits for the same images, including a ragged last chunk; and the images each device
    processed against the fp32 oracle (<= 2e-2, identical top-1)."""
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    ndev = _lib.lib.omCudaGetDeviceCount()
    devices = list(range(min(ndev, 8)))
    net = synth.resnet_spec(18)
    w = synth.make_weights(net)
    b = 8
    n = b * len(devices) + 3
    x = synth.imagenet_input(n)
    clf = serving.MultiDeviceClassifier(net, w, devices, b)
    try:
        got = clf.infer_logits(x)
        results = clf.infer_batch(x)
    finally:
        clf.close()
    plan = InferencePlan(net, w, batch=b)
    want = []
    for s in range(0, n, b):
        part = x[s:s + b]
        pad = np.zeros((b - part.shape[0],) + part.shape[1:], np.float32)
        want.append(plan.run(np.concatenate([part, pad]))[:part.shape[0]])
    plan.close()
    want = np.concatenate(want)
    assert np.array_equal(got, want)
    ref = serving.classify_logits(want)
    assert [r.predicted_class for r in results] == [r.predicted_class for r in ref]
    assert gpu.kernel_error() == 0
    # and against the fp32 oracle: the first image of every device's chunks and the ragged tail
    import oracle as orc
    from conftest import rel_err
    idx = sorted({i * b for i in range(len(devices))} | {n - 1})
    want_o = orc.forward(net, w, np.ascontiguousarray(x[idx]))
    assert rel_err(got[idx], want_o) <= 2e-2
    assert np.array_equal(got[idx].argmax(1), want_o.argmax(1))


def _host_normalise(raw, mean, std):
    """The reference's normalizeImage on the host: (x - mean) * (1 / std) in fp32."""
    m = np.asarray(mean, np.float32).reshape(1, -1, 1, 1)
    inv = (np.float32(1.0) / np.asarray(std, np.float32)).reshape(1, -1, 1, 1)
    return ((raw - m) * inv).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("arch", ["resnet18", "mobilenet"])
def test_normalisation_on_the_device_matches_the_host(gpu, arch):
    """Images in [0, 1] normalised inside the stem's pre-pass (InferencePlan input_norm,
    omCudaStemConvBnActNormIn; ResNet: the stem fused with its max pool, MobileNet: the plain
    stem) give the logits of host-normalised images, bit for bit; so does the multi-device
    classifier with normalize=IMAGENET_NORM on every visible device."""
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import IMAGENET_NORM, InferencePlan
    net = synth.resnet_spec(18) if arch == "resnet18" else synth.mobilenet_spec()
    w = synth.make_weights(net)
    b = 4
    rng = np.random.Generator(np.random.PCG64(77))
    raw = rng.random((b, 3, 224, 224), dtype=np.float32)
    dt = _lib.DTYPE_BF16 if arch == "resnet18" else _lib.DTYPE_F16
    plain = InferencePlan(net, w, batch=b, dtype=dt)
    want = plain.run(_host_normalise(raw, *IMAGENET_NORM))
    plain.close()
    normed = InferencePlan(net, w, batch=b, dtype=dt, input_norm=IMAGENET_NORM)
    got = normed.run(raw)
    normed.close()
    assert np.array_equal(got, want)
    assert gpu.kernel_error() == 0
    if arch == "resnet18":
        devices = list(range(min(_lib.lib.omCudaGetDeviceCount(), 8)))
        clf = serving.MultiDeviceClassifier(net, w, devices, b, dtype=dt,
                                            normalize=IMAGENET_NORM)
        try:
            got2 = clf.infer_logits(np.concatenate([raw] * len(devices)))
        finally:
            clf.close()
        assert np.array_equal(got2, np.concatenate([want] * len(devices)))


@pytest.mark.gpu
@pytest.mark.parametrize("pool", [True, False])
def test_u8_images_match_their_float_form(gpu, pool):
    """8-bit images (input_dtype DTYPE_U8, sample / 255 on the device) normalised on the device
    give the logits of the fp32 images sample / 255.0f normalised on the host, bit for bit;
    with the stem fused with its max pool and without (omCudaStemConvBnActNormIn bPool 1 / 0);
    and through the multi-device classifier."""
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import IMAGENET_NORM, InferencePlan
    net = synth.resnet_spec(18)
    w = synth.make_weights(net)
    b = 4
    rng = np.random.Generator(np.random.PCG64(78))
    u8 = rng.integers(0, 256, (b, 3, 224, 224), dtype=np.uint8)
    as_float = (u8.astype(np.float32) / np.float32(255.0)).astype(np.float32)
    plain = InferencePlan(net, w, batch=b, fuse_stem_pool=pool)
    want = plain.run(_host_normalise(as_float, *IMAGENET_NORM))
    plain.close()
    p8 = InferencePlan(net, w, batch=b, fuse_stem_pool=pool, input_dtype=_lib.DTYPE_U8,
                       input_norm=IMAGENET_NORM)
    assert p8.in_bytes == b * 3 * 224 * 224
    got = p8.run(u8)
    p8.close()
    assert np.array_equal(got, want)
    assert gpu.kernel_error() == 0
    if pool:
        clf = serving.MultiDeviceClassifier(net, w, [0], b, normalize=IMAGENET_NORM,
                                            input_dtype=_lib.DTYPE_U8)
        try:
            got2 = clf.infer_logits(u8[:3])
        finally:
            clf.close()
        assert np.array_equal(got2, want[:3])
