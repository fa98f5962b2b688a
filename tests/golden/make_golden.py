"""Writes tests/golden/golden.npz: fixtures produced by the reference engine itself.

Runs the reference's own CPU code (oracle/_ref/libomref.so, built from the reference sources by
`make -C oracle ref`) on small seeded inputs: single ops of the conv/BN/pool/softmax hot path,
eval-mode network forwards (ResNet-18, ResNet-50, the MobileNet stack; 10 classes, 64x64) and a
ResNet-18 training step. The CPU tests check the C restatement (oracle/om_oracle.c) against these
numbers, so the oracle is pinned to the reference even where the reference is not built.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as orc  # noqa: E402
from omnimatchdeeplearningtool_b200 import synth  # noqa: E402


def main():
    L = orc.ref()
    if L is None:
        raise SystemExit("oracle/_ref/libomref.so is not built (make -C oracle ref)")
    rng = np.random.Generator(np.random.PCG64(2024))
    g = {}
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    P = lambda a: a.ctypes.data

    # conv forward / backward, two geometries
    for tag, (n, c, h, k, r, st, pad) in {"a": (2, 3, 9, 4, 3, 1, 1), "b": (2, 4, 11, 6, 3, 2, 1)}.items():
        x, w, b = f(n, c, h, h), f(k, c, r, r), f(k)
        p = (h + 2 * pad - r) // st + 1
        y = np.empty((n, k, p, p), np.float32)
        L.omref_conv2d(P(x), P(w), P(b), P(y), n, c, h, h, k, r, st, pad)
        dy = f(n, k, p, p)
        dx = np.empty_like(x)
        L.omref_conv2d_backward_input(P(dy), P(w), P(dx), n, c, h, h, k, r, st, pad)
        dw, db = np.empty_like(w), np.empty(k, np.float32)
        L.omref_conv2d_backward_weight(P(x), P(dy), P(dw), P(db), n, c, h, h, k, r, st, pad)
        g.update({f"conv_{tag}_x": x, f"conv_{tag}_w": w, f"conv_{tag}_b": b, f"conv_{tag}_y": y,
                  f"conv_{tag}_dy": dy, f"conv_{tag}_dx": dx, f"conv_{tag}_dw": dw,
                  f"conv_{tag}_db": db,
                  f"conv_{tag}_geom": np.array([n, c, h, k, r, st, pad], np.int32)})
    # depthwise (grouped) conv
    x, w = f(2, 6, 8, 8), f(6, 1, 3, 3)
    y = np.empty((2, 6, 4, 4), np.float32)
    L.omref_dilated_conv2d(P(x), P(w), None, P(y), 2, 6, 8, 8, 6, 3, 2, 1, 1, 6)
    g.update({"dw_x": x, "dw_w": w, "dw_y": y})
    # batch norm, training and eval, and backward
    x = (f(3, 5, 4, 6) * 2 + 0.5).astype(np.float32)
    gm, bt = rng.uniform(0.5, 1.5, 5).astype(np.float32), f(5)
    for mode in (0, 1):
        rm, rv = (f(5) * 0.1).astype(np.float32), rng.uniform(0.5, 1.5, 5).astype(np.float32)
        g[f"bn{mode}_rm_in"], g[f"bn{mode}_rv_in"] = rm.copy(), rv.copy()
        y, sm, si = np.empty_like(x), np.empty(5, np.float32), np.empty(5, np.float32)
        L.omref_batchnorm2d(P(x), P(y), P(gm), P(bt), P(rm), P(rv), P(sm), P(si), 3, 5, 4, 6,
                            1e-5, 0.1, mode)
        g.update({f"bn{mode}_y": y, f"bn{mode}_rm": rm, f"bn{mode}_rv": rv, f"bn{mode}_sm": sm,
                  f"bn{mode}_si": si})
    dy = f(3, 5, 4, 6)
    dx, dg, db = np.empty_like(x), np.empty(5, np.float32), np.empty(5, np.float32)
    L.omref_batchnorm2d_backward(P(dy), P(x), P(g["bn1_sm"]), P(g["bn1_si"]), P(gm), P(dx), P(dg),
                                 P(db), 3, 5, 4, 6)
    g.update({"bn_x": x, "bn_gamma": gm, "bn_beta": bt, "bn_dy": dy, "bn_dx": dx, "bn_dg": dg,
              "bn_db": db})
    # pooling
    x = f(2, 3, 9, 9)
    y, idx = np.empty((2, 3, 5, 5), np.float32), np.empty((2, 3, 5, 5), np.int32)
    L.omref_maxpool2d(P(x), P(y), P(idx), 2, 3, 9, 9, 3, 2, 1)
    dy = f(2, 3, 5, 5)
    dx = np.empty_like(x)
    L.omref_maxpool2d_backward(P(dy), P(idx), P(dx), 2, 3, 5, 5, 9, 9)
    ya = np.empty((2, 3, 5, 5), np.float32)
    L.omref_avgpool2d(P(x), P(ya), 2, 3, 9, 9, 3, 2, 1)
    yg = np.empty((2, 3, 2, 3), np.float32)
    L.omref_adaptive_avgpool2d(P(x), P(yg), 2, 3, 9, 9, 2, 3)
    dg_ = f(2, 3, 2, 3)
    dxg = np.empty_like(x)
    L.omref_adaptive_avgpool2d_backward(P(dg_), P(dxg), 2, 3, 9, 9, 2, 3)
    g.update({"pool_x": x, "maxpool_y": y, "maxpool_idx": idx, "maxpool_dy": dy,
              "maxpool_dx": dx, "avgpool_y": ya, "adapool_y": yg, "adapool_dy": dg_,
              "adapool_dx": dxg})
    # elementwise, matmul, bias
    a, b = f(257), f(257)
    out = np.empty_like(a)
    L.omref_relu(P(a), P(out), 257)
    g["relu_y"] = out.copy()
    L.omref_relu_backward(P(a), P(b), P(out), 257)
    g["relu_dx"] = out.copy()
    L.omref_clip(P(a), P(out), 257, 0.0, 0.75)
    g["clip_y"] = out.copy()
    L.omref_add(P(a), P(b), P(out), 257)
    g["add_y"] = out.copy()
    g.update({"ew_a": a, "ew_b": b})
    A, B = f(7, 13), f(13, 9)
    C = np.empty((7, 9), np.float32)
    L.omref_matmul(P(A), P(B), P(C), 7, 13, 9)
    bias = f(9)
    Cb = np.empty_like(C)
    L.omref_add_bias(P(C), P(bias), P(Cb), 7, 9)
    g.update({"mm_a": A, "mm_b": B, "mm_c": C, "mm_bias": bias, "mm_cb": Cb})
    # softmax / cross-entropy
    z = (f(4, 11) * 3).astype(np.float32)
    oh = np.zeros((4, 11), np.float32)
    oh[np.arange(4), [3, 0, 10, 7]] = 1
    sp = np.empty_like(z)
    L.omref_softmax(P(z), P(sp), 4, 11)
    ce = np.array([L.omref_cross_entropy(P(sp), P(oh), 4, 11)], np.float32)
    dz = np.empty_like(z)
    L.omref_ce_softmax_backward(P(sp), P(oh), P(dz), 4, 11)
    g.update({"sm_z": z, "sm_onehot": oh, "sm_p": sp, "ce_loss": ce, "ce_dz": dz})

    # networks: eval forward logits (batch 2, 64x64, 10 classes) from the reference modules
    for kind, net in ((0, synth.resnet_spec(18, 10)), (1, synth.resnet_spec(50, 10)),
                      (2, synth.mobilenet_spec(10))):
        w = synth.make_weights(net)
        h = orc.ref_model(kind, 10, w, net)
        x = synth.normal_input(2, 3, 64, 64, seed=5)
        out = np.empty((2, 10), np.float32)
        L.omref_model_forward(h, P(x), 2, 64, 64, P(out))
        g[f"net_{net.name}_logits"] = out
        L.omref_model_destroy(h)
    # ResNet-18 training step (batch 4, 64x64, 10 classes): loss and per-parameter gradient
    # summaries [sum, L2 norm, first four values]
    net = synth.resnet_spec(18, 10)
    w = synth.make_weights(net)
    h = orc.ref_model(0, 10, w, net)
    x = synth.normal_input(4, 3, 64, 64, seed=6)
    y = synth.onehot_labels(4, 10, seed=7)
    tot = sum(int(np.prod(s)) for _, s in net.params)
    grads = np.empty(tot, np.float32)
    loss = L.omref_model_train_step(h, P(x), P(y), 4, 64, 64, 10, 0.01, 0.9, 0, P(grads))
    summ = []
    off = 0
    for _, shape in net.params:
        m = int(np.prod(shape))
        v = grads[off:off + m].astype(np.float64)
        off += m
        summ.append([v.sum(), np.sqrt((v * v).sum()), *v[:4]])
    g["train_r18_loss"] = np.array([loss], np.float32)
    g["train_r18_grad_summary"] = np.array(summ, np.float64)
    L.omref_model_destroy(h)

    # Config 3 at its parity size (ResNet-18, 1000 classes, batch 8 at 224x224): how far the
    # reference's own fp32 gradients sit from the oracle's double-precision ones, per parameter
    # as max|ref - oracle| / max|oracle|. The GPU training step is held to this spread.
    net = synth.resnet_spec(18, 1000)
    w = synth.make_weights(net)
    h = orc.ref_model(0, 1000, w, net)
    x = synth.normal_input(8, 3, 224, 224, seed=11)
    y = synth.onehot_labels(8, 1000, seed=12)
    tot = sum(int(np.prod(s)) for _, s in net.params)
    gref = np.empty(tot, np.float32)
    loss = L.omref_model_train_step(h, P(x), P(y), 8, 224, 224, 1000, 0.01, 0.9, 0, P(gref))
    _, gor = orc.train_step(net, {k: v.copy() for k, v in w.items()}, x, y)
    errs = []
    off = 0
    for name, shape in net.params:
        m = int(np.prod(shape))
        o = gor[name].reshape(-1)
        errs.append(float(np.abs(gref[off:off + m] - o).max() / np.abs(o).max()))
        off += m
    g["train_r18_224_ref_loss"] = np.array([loss], np.float32)
    g["train_r18_224_ref_grad_err"] = np.array(errs, np.float64)
    L.omref_model_destroy(h)

    out = os.path.join(HERE, "golden.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out} ({os.path.getsize(out)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
