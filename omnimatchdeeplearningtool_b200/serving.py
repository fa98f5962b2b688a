"""Batch classification over several GPUs from one process: the multi-device form of the
reference's ``EngineBridge::inferBatch`` (src/engine/bridge/EngineBridge.cpp:3525-3720), which
runs every batch on device 0.

Each device gets one worker thread. The thread selects its device (``omCudaInit``), builds its own
:class:`~omnimatchdeeplearningtool_b200.plan.InferencePlan` (weights resident on that GPU,
CUDA-graph replay) and runs the chunks of images it is given. The ctypes calls release the GIL,
so the devices work at the same time. Images are cut into chunks of ``batch_per_device`` in
order, and chunk i goes to device i mod D; a short last chunk is zero-padded (eval-mode
BatchNorm keeps the images independent) and its padding rows are dropped.

:func:`classify_logits` turns logits into the reference's per-image result
(EngineBridge.cpp:3691-3717): softmax with the maximum subtracted and the sum floored at 1e-8,
the most probable class and its probability, and class -1 when that probability is below the
confidence threshold (``BridgeInferParams::fConfThreshold``, default 0.5).

The reference normalises each image on the host before its forward (EngineBridge.cpp:3580-3594:
the ImageNet preset for ResNet/MobileNet models). With ``normalize=IMAGENET_NORM`` (or any
(mean, std) pair) the classifier takes the images as the reference's inferBatch does, in [0, 1],
and each plan normalises them inside its stem's pre-pass on the GPU, with the reference's
arithmetic; with ``normalize=None`` the images come normalised.
"""
from __future__ import annotations

import queue
import threading
from typing import Callable, Dict, List, NamedTuple, Optional, Sequence

import numpy as np

from ._lib import DTYPE_BF16, DTYPE_F32, DTYPE_U8


class InferResult(NamedTuple):
    """One image's result, as the reference's ``BridgeInferResult`` for a classifier."""
    predicted_class: int
    confidence: float
    probs: np.ndarray


def classify_logits(logits: np.ndarray, conf_threshold: float = 0.5) -> List[InferResult]:
    """Per-row softmax, best class and confidence, in float32 as the reference computes them."""
    z = np.asarray(logits, np.float32)
    e = np.exp(z - z.max(axis=1, keepdims=True))
    p = e / np.maximum(e.sum(axis=1, keepdims=True, dtype=np.float32), np.float32(1e-8))
    best = p.argmax(axis=1)
    out = []
    for i in range(p.shape[0]):
        conf = float(p[i, best[i]])
        out.append(InferResult(int(best[i]) if conf >= conf_threshold else -1, conf, p[i]))
    return out


class _Worker:
    """A thread that owns one device and one plan, and runs the chunks put on its queue."""

    def __init__(self, device: int, make_plan: Callable[[], object],
                 init_device: Callable[[int], None]):
        self.device = device
        self.jobs: "queue.Queue" = queue.Queue()
        self.error: Optional[BaseException] = None
        self._ready = threading.Event()
        self._thread = threading.Thread(target=self._main, args=(make_plan, init_device),
                                        name=f"omb-device-{device}", daemon=True)
        self._thread.start()

    def _main(self, make_plan, init_device) -> None:
        plan = None
        try:
            init_device(self.device)
            plan = make_plan()
        except BaseException as e:  # reported to the caller by wait_ready
            self.error = e
        self._ready.set()
        while True:
            job = self.jobs.get()
            if job is None:
                break
            x, results, key, done = job
            try:
                if plan is None:
                    raise RuntimeError(f"device {self.device} has no plan: {self.error!r}")
                results[key] = plan.run(x)
            except BaseException as e:
                results[key] = e
            done.release()
        if plan is not None:
            plan.close()

    def wait_ready(self) -> None:
        self._ready.wait()
        if self.error is not None:
            raise RuntimeError(f"device {self.device}: setup failed") from self.error

    def stop(self) -> None:
        self.jobs.put(None)
        self._thread.join()


class MultiDeviceClassifier:
    """``inferBatch`` over ``devices``: one resident plan per GPU, chunks dealt round-robin.

    ``make_plan(device)`` and ``init_device(device)`` default to an ``InferencePlan`` of ``net``
    and ``weights`` (``batch_per_device`` images, ``dtype``) and ``omCudaInit``; tests replace
    them to check the dealing without a GPU."""

    def __init__(self, net, weights: Dict[str, np.ndarray], devices: Sequence[int],
                 batch_per_device: int, dtype: int = DTYPE_BF16, h: int = 224, w: int = 224,
                 make_plan: Optional[Callable[[int], object]] = None,
                 init_device: Optional[Callable[[int], None]] = None,
                 normalize=None, input_dtype: int = DTYPE_F32):
        if not devices:
            raise ValueError("MultiDeviceClassifier needs at least one device")
        if len(set(devices)) != len(devices):
            raise ValueError("each device may appear once (one driving thread per device)")
        if batch_per_device <= 0:
            raise ValueError("batch_per_device must be positive")
        if make_plan is None:
            from .plan import InferencePlan

            def make_plan(_device):
                return InferencePlan(net, weights, batch=batch_per_device, dtype=dtype, h=h, w=w,
                                     input_norm=normalize, input_dtype=input_dtype)
        if init_device is None:
            from . import backend
            init_device = backend.init
        self.batch = batch_per_device
        # DTYPE_U8: the images are uint8 samples (value / 255), a quarter of the bytes to copy
        self.u8 = input_dtype == DTYPE_U8
        self.shape = (3, h, w) if net is None else (net.stem[0].cin, h, w)
        self.workers = [_Worker(d, (lambda d=d: make_plan(d)), init_device) for d in devices]
        try:
            for wk in self.workers:
                wk.wait_ready()
        except BaseException:
            self.close()
            raise

    def infer_logits(self, images: np.ndarray) -> np.ndarray:
        """[n, C, H, W] fp32 host images (uint8 with input_dtype=DTYPE_U8) -> [n, classes] fp32
        logits, in input order."""
        if self.u8 and np.asarray(images).dtype != np.uint8:
            raise TypeError("an 8-bit classifier takes uint8 images")
        x = np.ascontiguousarray(images, np.uint8 if self.u8 else np.float32)
        if x.ndim != 4 or x.shape[1:] != self.shape:
            raise ValueError(f"images must be [n, {self.shape[0]}, {self.shape[1]}, "
                             f"{self.shape[2]}], got {x.shape}")
        n = x.shape[0]
        if n == 0:
            raise ValueError("no images")
        chunks = [(s, min(s + self.batch, n)) for s in range(0, n, self.batch)]
        results: Dict[int, object] = {}
        done = threading.Semaphore(0)
        for i, (s, e) in enumerate(chunks):
            part = x[s:e]
            if e - s < self.batch:  # the ragged end: zero rows, dropped again below
                part = np.concatenate([part, np.zeros((self.batch - (e - s),) + self.shape,
                                                      x.dtype)])
            self.workers[i % len(self.workers)].jobs.put((part, results, i, done))
        for _ in chunks:
            done.acquire()
        outs = []
        for i, (s, e) in enumerate(chunks):
            r = results[i]
            if isinstance(r, BaseException):
                raise RuntimeError(f"chunk {i} failed") from r
            outs.append(np.asarray(r)[:e - s])
        return np.concatenate(outs)

    def infer_batch(self, images: np.ndarray, conf_threshold: float = 0.5) -> List[InferResult]:
        """The reference's ``inferBatch`` result for each image."""
        return classify_logits(self.infer_logits(images), conf_threshold)

    def infer(self, image: np.ndarray, conf_threshold: float = 0.5) -> InferResult:
        """The reference's single-image ``infer`` (EngineBridge.cpp:3100-3200) for a
        classifier: one [C, H, W] image, on the first device's plan (build the classifier with
        ``batch_per_device=1`` for the lowest latency; a larger plan pads the image)."""
        x = np.asarray(image)
        if x.shape != self.shape:
            raise ValueError(f"image must be {list(self.shape)}, got {list(x.shape)}")
        return self.infer_batch(x[None], conf_threshold)[0]

    def close(self) -> None:
        for wk in self.workers:
            wk.stop()
        self.workers = []
