"""Parity of the off-hot-path C-ABI entry points (the reference's remaining omCuda* functions,
src/cuda/cuda_kernels.cu) with numpy restatements of the reference kernels' arithmetic.

Tolerances: data movement, + - * /, LeakyReLU and dropout must match exactly; elementwise ops
built on expf / tanhf within 1e-5 relative (CUDA's functions are within a few ulp); reductions
and contractions within the fp32 path's 1e-4 (max |a-b| / max |b| per output; numpy sums in
double).
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4
TOL_EW = 1e-5

_KEEP = []


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    _KEEP.clear()


def _dev(a):
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    b = DeviceBuffer.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    _KEEP.append(b)
    return b


def _out(shape):
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    b = DeviceBuffer.zeros(max(int(np.prod(shape)), 1) * 4)
    _KEEP.append(b)
    return b


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def _sig(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def test_binary_and_scalar_ops_exact(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(1)
    n = 1029
    a = rng.standard_normal(n).astype(np.float32)
    b = (rng.standard_normal(n) + 3.0).astype(np.float32)
    da, db, o = _dev(a), _dev(b), _out((n,))
    for fn, want in ((B.sub, a - b), (B.mul, a * b), (B.div, a / b)):
        fn(da.ptr, db.ptr, o.ptr, n)
        assert np.array_equal(o.to_numpy((n,)), want)
    B.addScalar(da.ptr, np.float32(0.375), o.ptr, n)
    assert np.array_equal(o.to_numpy((n,)), a + np.float32(0.375))
    B.leakyRelu(da.ptr, o.ptr, n, 0.1)
    assert np.array_equal(o.to_numpy((n,)), np.where(a > 0, a, np.float32(0.1) * a))
    B.leakyReluBackward(db.ptr, da.ptr, o.ptr, n, 0.2)
    assert np.array_equal(o.to_numpy((n,)), np.where(a > 0, b, np.float32(0.2) * b))
    # misaligned start (scalar path) and an empty call
    B.sub(da.ptr + 4, db.ptr + 4, o.ptr + 4, n - 1)
    assert np.array_equal(o.to_numpy((n,))[1:], (a - b)[1:])
    B.sub(da.ptr, db.ptr, o.ptr, 0)


def test_activations(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(2)
    n = 4099
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    dx, dg, o = _dev(x), _dev(g), _out((n,))
    x64, g64 = x.astype(np.float64), g.astype(np.float64)
    s = _sig(x64)
    c = 0.7978845608
    t = np.tanh(c * (x64 + 0.044715 * x64 ** 3))
    cases = [
        (lambda: B.sigmoid(dx.ptr, o.ptr, n), s),
        (lambda: B.tanhForward(dx.ptr, o.ptr, n), np.tanh(x64)),
        (lambda: B.gelu(dx.ptr, o.ptr, n), 0.5 * x64 * (1 + t)),
        (lambda: B.silu(dx.ptr, o.ptr, n), x64 * s),
        (lambda: B.geluBackward(dg.ptr, dx.ptr, o.ptr, n),
         g64 * (0.5 * (1 + t) + 0.5 * x64 * (1 - t * t) * c * (1 + 3 * 0.044715 * x64 ** 2))),
        (lambda: B.siluBackward(dg.ptr, dx.ptr, o.ptr, n), g64 * s * (1 + x64 * (1 - s))),
    ]
    for run, want in cases:
        run()
        assert rel_err(o.to_numpy((n,)), want) < TOL_EW
    # the Sigmoid / Tanh backwards take the forward output
    y = np.float32(_sig(x64))
    dy = _dev(y)
    B.sigmoidBackward(dg.ptr, dy.ptr, o.ptr, n)
    assert rel_err(o.to_numpy((n,)), g64 * y * (1.0 - y.astype(np.float64))) < TOL_EW
    B.tanhBackward(dg.ptr, dy.ptr, o.ptr, n)
    assert rel_err(o.to_numpy((n,)), g64 * (1.0 - y.astype(np.float64) ** 2)) < TOL_EW


def test_mean_and_batched_matmul(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    from omnimatchdeeplearningtool_b200._lib import call
    rng = _rng(3)
    x = rng.standard_normal(100003).astype(np.float32) + 0.25
    r = _out((1,))
    call("omCudaMean", _dev(x).ptr, r.ptr, x.size)
    assert abs(r.to_numpy((1,))[0] - x.astype(np.float64).mean()) < 1e-5
    bt, m, k, n = 3, 17, 33, 20
    a = rng.standard_normal((bt, m, k)).astype(np.float32)
    b = rng.standard_normal((bt, k, n)).astype(np.float32)
    c = _out((bt, m, n))
    B.batchedMatmul(_dev(a).ptr, _dev(b).ptr, c.ptr, bt, m, k, n)
    want = np.einsum("bmk,bkn->bmn", a.astype(np.float64), b.astype(np.float64))
    assert rel_err(c.to_numpy((bt, m, n)), want) < TOL


def test_concat_slice_and_heads_exact(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(4)
    n, c1, c2, hw = 3, 5, 7, 11
    a = rng.standard_normal((n, c1, hw)).astype(np.float32)
    b = rng.standard_normal((n, c2, hw)).astype(np.float32)
    o = _out((n, c1 + c2, hw))
    B.concatChannels(_dev(a).ptr, _dev(b).ptr, o.ptr, n, c1, c2, hw)
    cat = np.concatenate([a, b], axis=1)
    assert np.array_equal(o.to_numpy(cat.shape), cat)
    ga, gb = _out(a.shape), _out(b.shape)
    B.concatChannelsBackward(_dev(cat).ptr, ga.ptr, gb.ptr, n, c1, c2, hw)
    assert np.array_equal(ga.to_numpy(a.shape), a) and np.array_equal(gb.to_numpy(b.shape), b)

    outer, da, db = 13, 6, 9
    a = rng.standard_normal((outer, da)).astype(np.float32)
    b = rng.standard_normal((outer, db)).astype(np.float32)
    o = _out((outer, da + db))
    B.concatLastDim(_dev(a).ptr, _dev(b).ptr, o.ptr, outer, da, db)
    cat = np.concatenate([a, b], axis=1)
    assert np.array_equal(o.to_numpy(cat.shape), cat)
    ga, gb = _out(a.shape), _out(b.shape)
    B.concatLastDimBackward(_dev(cat).ptr, ga.ptr, gb.ptr, outer, da, db)
    assert np.array_equal(ga.to_numpy(a.shape), a) and np.array_equal(gb.to_numpy(b.shape), b)

    full, start, ln = 15, 4, 7
    x = rng.standard_normal((outer, full)).astype(np.float32)
    s = _out((outer, ln))
    B.sliceLastDim(_dev(x).ptr, s.ptr, outer, full, start, ln)
    assert np.array_equal(s.to_numpy((outer, ln)), x[:, start:start + ln])
    # the backward writes the slice columns only; the rest keeps what the buffer held
    pre = np.full((outer, full), 7.0, np.float32)
    gi = _dev(pre)
    B.sliceLastDimBackward(_dev(x[:, :ln]).ptr, gi.ptr, outer, full, start, ln)
    want = pre.copy()
    want[:, start:start + ln] = x[:, :ln]
    assert np.array_equal(gi.to_numpy((outer, full)), want)

    N, S, H, D = 2, 5, 3, 4
    qkv = rng.standard_normal((N, S, 3, H, D)).astype(np.float32)
    q, k, v = _out((N, H, S, D)), _out((N, H, S, D)), _out((N, H, S, D))
    B.qkvSplitHeads(_dev(qkv).ptr, q.ptr, k.ptr, v.ptr, N, S, H, D, 0.5)
    sh = (N, H, S, D)
    assert np.array_equal(q.to_numpy(sh), qkv[:, :, 0].transpose(0, 2, 1, 3) * np.float32(0.5))
    assert np.array_equal(k.to_numpy(sh), qkv[:, :, 1].transpose(0, 2, 1, 3))
    assert np.array_equal(v.to_numpy(sh), qkv[:, :, 2].transpose(0, 2, 1, 3))
    m = _out((N, S, H * D))
    B.mergeHeads(k.ptr, m.ptr, N, S, H, D)
    assert np.array_equal(m.to_numpy((N, S, H * D)), qkv[:, :, 1].reshape(N, S, H * D))


def test_invalid_arguments_raise(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B, OmCudaError
    x, o = _out((16,)), _out((16,))
    with pytest.raises(OmCudaError):
        B.sliceLastDim(x.ptr, o.ptr, 2, 8, 5, 4)  # slice runs past the row
    with pytest.raises(OmCudaError):
        B.groupNorm2d(x.ptr, o.ptr, x.ptr, x.ptr, x.ptr, x.ptr, 1, 6, 2, 1, 4, 1e-5)  # 6 % 4
    with pytest.raises(OmCudaError):
        B.adamStep(x.ptr, x.ptr, x.ptr, x.ptr, 16, 1e-3, 0.9, 0.999, 1e-8, 0)  # step 0


def test_softmax_last_dim_backward(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(5)
    outer, d = 37, 300
    z = rng.standard_normal((outer, d))
    s = np.exp(z - z.max(1, keepdims=True))
    s = (s / s.sum(1, keepdims=True)).astype(np.float32)
    g = rng.standard_normal((outer, d)).astype(np.float32)
    o = _out((outer, d))
    B.softmaxLastDimBackward(_dev(g).ptr, _dev(s).ptr, o.ptr, outer, d)
    s64, g64 = s.astype(np.float64), g.astype(np.float64)
    want = s64 * (g64 - (g64 * s64).sum(1, keepdims=True))
    assert rel_err(o.to_numpy((outer, d)), want) < TOL


@pytest.mark.parametrize("rows,dim", [(7, 64), (33, 257), (2, 1024)])
def test_layer_norm_fwd_bwd(gpu, rows, dim):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(6 + dim)
    x = (rng.standard_normal((rows, dim)) * 2 + 0.5).astype(np.float32)
    gam = rng.standard_normal(dim).astype(np.float32)
    bet = rng.standard_normal(dim).astype(np.float32)
    dy = rng.standard_normal((rows, dim)).astype(np.float32)
    eps = 1e-5
    dX, dG = _dev(x), _dev(gam)
    y, mu, iv = _out(x.shape), _out((rows,)), _out((rows,))
    B.layerNorm(dX.ptr, y.ptr, dG.ptr, _dev(bet).ptr, mu.ptr, iv.ptr, rows, dim, eps)
    x64 = x.astype(np.float64)
    m = x64.mean(1, keepdims=True)
    inv = 1.0 / np.sqrt(x64.var(1, keepdims=True) + eps)
    xh = (x64 - m) * inv
    assert rel_err(y.to_numpy(x.shape), gam * xh + bet) < TOL
    assert rel_err(mu.to_numpy((rows,)), m[:, 0]) < TOL
    assert rel_err(iv.to_numpy((rows,)), inv[:, 0]) < TOL
    gx, gg, gb = _out(x.shape), _out((dim,)), _out((dim,))
    B.layerNormBackward(_dev(dy).ptr, dX.ptr, mu.ptr, iv.ptr, dG.ptr, gx.ptr, gg.ptr, gb.ptr, rows,
                        dim)
    d64 = dy.astype(np.float64)
    gdy = gam * d64
    want = inv * (gdy - gdy.mean(1, keepdims=True) - xh * (gdy * xh).mean(1, keepdims=True))
    assert rel_err(gx.to_numpy(x.shape), want) < TOL
    assert rel_err(gg.to_numpy((dim,)), (d64 * xh).sum(0)) < TOL
    assert rel_err(gb.to_numpy((dim,)), d64.sum(0)) < TOL


@pytest.mark.parametrize("n,c,h,w,groups", [(2, 8, 5, 7, 4), (3, 32, 8, 8, 8), (1, 6, 3, 3, 1)])
def test_group_norm_fwd_bwd(gpu, n, c, h, w, groups):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(7 + c)
    x = (rng.standard_normal((n, c, h, w)) + 0.3).astype(np.float32)
    gam = rng.standard_normal(c).astype(np.float32)
    bet = rng.standard_normal(c).astype(np.float32)
    dy = rng.standard_normal(x.shape).astype(np.float32)
    eps = 1e-5
    dX, dG = _dev(x), _dev(gam)
    y, mu, iv = _out(x.shape), _out((n * groups,)), _out((n * groups,))
    B.groupNorm2d(dX.ptr, y.ptr, dG.ptr, _dev(bet).ptr, mu.ptr, iv.ptr, n, c, h, w, groups, eps)
    xg = x.astype(np.float64).reshape(n, groups, -1)
    m = xg.mean(2, keepdims=True)
    inv = 1.0 / np.sqrt(xg.var(2, keepdims=True) + eps)
    xh = ((xg - m) * inv).reshape(x.shape)
    assert rel_err(y.to_numpy(x.shape), gam[None, :, None, None] * xh +
                   bet[None, :, None, None]) < TOL
    gx, gg, gb = _out(x.shape), _out((c,)), _out((c,))
    B.groupNorm2dBackward(_dev(dy).ptr, dX.ptr, mu.ptr, iv.ptr, dG.ptr, gx.ptr, gg.ptr, gb.ptr,
                          n, c, h, w, groups, eps)
    d64 = dy.astype(np.float64)
    dgam = (d64 * xh).sum((0, 2, 3))
    dbet = d64.sum((0, 2, 3))
    assert rel_err(gg.to_numpy((c,)), dgam) < TOL
    assert rel_err(gb.to_numpy((c,)), dbet) < TOL
    # the reference's dx: batch-total parameter gradients summed over each group's channels
    cpg, M = c // groups, (c // groups) * h * w
    GG = np.repeat(dgam.reshape(groups, cpg).sum(1), cpg)[None, :, None, None]
    GB = np.repeat(dbet.reshape(groups, cpg).sum(1), cpg)[None, :, None, None]
    invc = np.repeat(inv.reshape(n, groups), cpg, axis=1)[:, :, None, None]
    want = gam[None, :, None, None] * invc * (d64 - GB / M - xh * GG / M)
    assert rel_err(gx.to_numpy(x.shape), want) < TOL


def _bilinear_taps(out_size, in_size):
    sc = in_size / out_size
    src = (np.arange(out_size) + 0.5) * np.float32(sc) - 0.5
    i0 = np.floor(src).astype(np.int64)
    lam = src - i0
    return np.clip(i0, 0, in_size - 1), np.clip(i0 + 1, 0, in_size - 1), lam


@pytest.mark.parametrize("h,w,oh,ow", [(5, 7, 10, 14), (8, 8, 3, 5), (4, 6, 4, 6)])
def test_upsample_bilinear(gpu, h, w, oh, ow):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(8 + h)
    n, c = 2, 3
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    o = _out((n, c, oh, ow))
    B.upsampleBilinear(_dev(x).ptr, o.ptr, n, c, h, w, oh, ow)
    h0, h1, lh = _bilinear_taps(oh, h)
    w0, w1, lw = _bilinear_taps(ow, w)
    x64 = x.astype(np.float64)
    lh, lw = lh[:, None], lw[None, :]

    def at(hi, wi):
        return x64[:, :, hi][:, :, :, wi]
    want = (1 - lh) * ((1 - lw) * at(h0, w0) + lw * at(h0, w1)) + \
        lh * ((1 - lw) * at(h1, w0) + lw * at(h1, w1))
    assert rel_err(o.to_numpy(want.shape), want) < TOL_EW
    g = rng.standard_normal((n, c, oh, ow)).astype(np.float32)
    gi = _dev(np.full(x.shape, 5.0, np.float32))  # the backward zeroes it first
    B.upsampleBilinearBackward(_dev(g).ptr, gi.ptr, n, c, h, w, oh, ow)
    ref = np.zeros(x.shape)
    g64 = g.astype(np.float64)
    for i in range(oh):
        for j in range(ow):
            for hi, wh in ((h0[i], 1 - lh[i, 0]), (h1[i], lh[i, 0])):
                for wi, ww in ((w0[j], 1 - lw[0, j]), (w1[j], lw[0, j])):
                    ref[:, :, hi, wi] += g64[:, :, i, j] * wh * ww
    assert rel_err(gi.to_numpy(x.shape), ref) < TOL


@pytest.mark.parametrize("cin,h,cout,k,stride,pad,bias",
                         [(3, 5, 4, 4, 2, 1, True), (8, 7, 6, 3, 1, 1, False),
                          (4, 6, 5, 2, 2, 0, True),
                          (64, 14, 32, 2, 2, 0, True),    # UNet-style 2x upsampling
                          (48, 9, 40, 4, 2, 1, False),    # 4x4 / 2 with padding
                          (6, 5, 7, 3, 2, 3, True)])      # pad > K-1: the direct kernel
def test_conv_transpose2d(gpu, cin, h, cout, k, stride, pad, bias):
    """omCudaConvTranspose2d (cuda_kernels.cu:4187) against a float64 scatter; pad <= K-1 runs
    on the 3xTF32 tensor-core conv (the input gradient of the matching convolution)."""
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(9 + cin)
    n, w_ = 2, h + 1
    x = rng.standard_normal((n, cin, h, w_)).astype(np.float32)
    wt = rng.standard_normal((cin, cout, k, k)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    ho, wo = (h - 1) * stride - 2 * pad + k, (w_ - 1) * stride - 2 * pad + k
    o = _out((n, cout, ho, wo))
    B.convTranspose2d(_dev(x).ptr, _dev(wt).ptr, _dev(b).ptr if bias else 0, o.ptr, n, cin, h,
                      w_, cout, k, k, stride, pad)
    ref = np.zeros((n, cout, ho, wo))
    x64, w64 = x.astype(np.float64), wt.astype(np.float64)
    for ih in range(h):
        for iw in range(w_):
            for kh in range(k):
                for kw in range(k):
                    oh, ow = ih * stride - pad + kh, iw * stride - pad + kw
                    if 0 <= oh < ho and 0 <= ow < wo:
                        ref[:, :, oh, ow] += x64[:, :, ih, iw] @ w64[:, :, kh, kw]
    if bias:
        ref += b[None, :, None, None]
    assert rel_err(o.to_numpy(ref.shape), ref) < TOL


@pytest.mark.parametrize("stride,pad,dil", [(1, 2, 2), (2, 1, 1), (1, 3, 3)])
def test_dilated_conv_backward_weight(gpu, stride, pad, dil):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(10 + dil)
    n, cin, h, w_, cout, k = 2, 3, 11, 9, 4, 3
    ek = k + (k - 1) * (dil - 1)
    p, q = (h + 2 * pad - ek) // stride + 1, (w_ + 2 * pad - ek) // stride + 1
    x = rng.standard_normal((n, cin, h, w_)).astype(np.float32)
    dy = rng.standard_normal((n, cout, p, q)).astype(np.float32)
    dw, db = _out((cout, cin, k, k)), _out((cout,))
    B.dilatedConv2dBackwardWeight(_dev(x).ptr, _dev(dy).ptr, dw.ptr, db.ptr, n, cin, h, w_, cout,
                                  k, k, stride, pad, dil)
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    ref = np.zeros((cout, cin, k, k))
    for kh in range(k):
        for kw in range(k):
            patch = xp[:, :, kh * dil:kh * dil + stride * (p - 1) + 1:stride,
                       kw * dil:kw * dil + stride * (q - 1) + 1:stride]
            ref[:, :, kh, kw] = np.einsum("nopq,nipq->oi", dy.astype(np.float64), patch)
    assert rel_err(dw.to_numpy(ref.shape), ref) < TOL
    assert rel_err(db.to_numpy((cout,)), dy.astype(np.float64).sum((0, 2, 3))) < TOL


def test_conv2d_im2col_is_conv2d(gpu):
    from omnimatchdeeplearningtool_b200._lib import call
    rng = _rng(11)
    n, cin, h, cout, k = 2, 16, 12, 24, 3
    x = rng.standard_normal((n, cin, h, h)).astype(np.float32)
    wt = rng.standard_normal((cout, cin, k, k)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    args = (_dev(x).ptr, _dev(wt).ptr, _dev(b).ptr)
    o1, o2 = _out((n, cout, h, h)), _out((n, cout, h, h))
    call("omCudaConv2d", *args, o1.ptr, n, cin, h, h, cout, k, k, 1, 1)
    call("omCudaConv2dIm2col", *args, o2.ptr, n, cin, h, h, cout, k, k, 1, 1)
    assert np.array_equal(o1.to_numpy((n, cout, h, h)), o2.to_numpy((n, cout, h, h)))


def test_bce_with_logits(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(12)
    n = 50001
    x = (rng.standard_normal(n) * 4).astype(np.float32)
    t = (rng.random(n) < 0.3).astype(np.float32)
    dx, dt, r = _dev(x), _dev(t), _out((1,))
    B.bceWithLogitsForward(dx.ptr, dt.ptr, r.ptr, n)
    x64 = x.astype(np.float64)
    want = (np.maximum(x64, 0) - x64 * t + np.log1p(np.exp(-np.abs(x64)))).sum()
    assert abs(r.to_numpy((1,))[0] - want) / want < TOL
    g = _out((n,))
    B.bceWithLogitsBackward(dx.ptr, dt.ptr, g.ptr, n, 1.0 / n)
    assert rel_err(g.to_numpy((n,)), (_sig(x64) - t) / n) < TOL_EW


def test_dice_loss(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(13)
    n = 2 * 64 * 64
    x = (rng.standard_normal(n) * 2).astype(np.float32)
    t = (rng.random(n) < 0.4).astype(np.float32)
    dT = _dev(t)
    loss, sig, st = _out((1,)), _out((n,)), _out((3,))
    B.diceLossForward(_dev(x).ptr, dT.ptr, loss.ptr, sig.ptr, st.ptr, n)
    s = _sig(x)
    I, P, T = (s * t).sum(), s.sum(), t.sum()
    assert rel_err(st.to_numpy((3,)), [I, P, T]) < TOL
    assert abs(loss.to_numpy((1,))[0] - (1 - 2 * I / (P + T + 1e-6))) < 1e-5
    assert rel_err(sig.to_numpy((n,)), s) < TOL_EW
    g = _out((n,))
    B.diceLossBackward(sig.ptr, dT.ptr, st.ptr, _dev(np.array([0.5], np.float32)).ptr, g.ptr, n)
    D = P + T + 1e-6
    want = -0.5 * 2 * (t * D - I) / D ** 2 * s * (1 - s)
    assert rel_err(g.to_numpy((n,)), want) < TOL


def test_weighted_pixel_ce(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(14)
    b, k, hw = 2, 5, 300
    logits = (rng.standard_normal((b, k, hw)) * 2).astype(np.float32)
    tgt = rng.integers(0, k, (b, hw)).astype(np.float32)
    tgt[0, :17] = 255.0  # ignored pixels (out of the class range)
    tgt[1, :5] = -1.0
    cw = (rng.random(k) + 0.5).astype(np.float32)
    dT, dW = _dev(tgt), _dev(cw)
    soft, loss, st = _out(logits.shape), _out((1,)), _out((2,))
    B.weightedPixelCEForward(_dev(logits).ptr, dT.ptr, dW.ptr, soft.ptr, loss.ptr, st.ptr, b * hw,
                             k, hw)
    z = logits.astype(np.float64)
    sm = np.exp(z - z.max(1, keepdims=True))
    sm /= sm.sum(1, keepdims=True)
    ti = np.rint(tgt).astype(np.int64)
    valid = (ti >= 0) & (ti < k)
    tc = np.where(valid, ti, 0)
    pt = np.take_along_axis(sm, tc[:, None, :], 1)[:, 0]
    w = np.where(valid, cw[tc], 0.0)
    L = (-w * (1 - pt) ** 2 * np.log(pt + 1e-7)).sum()
    W = w.sum()
    assert rel_err(soft.to_numpy(logits.shape), sm) < TOL_EW
    assert rel_err(st.to_numpy((2,)), [L, W]) < TOL
    assert abs(loss.to_numpy((1,))[0] - L / W) / (L / W) < TOL
    g = _out(logits.shape)
    B.weightedPixelCEBackward(soft.ptr, dT.ptr, dW.ptr, _dev(np.array([2.0], np.float32)).ptr,
                              st.ptr, g.ptr, b * hw, k, hw)
    pt_v = np.where(valid, pt, 1.0)
    onehot = (np.arange(k)[None, :, None] == ti[:, None, :]).astype(np.float64)
    scale = (w * 2.0 / W)[:, None, :]
    want = scale * ((1 - pt_v)[:, None] ** 2 * (sm - onehot) +
                    onehot * (-2 * (1 - pt_v) * np.log(pt_v + 1e-7))[:, None] * sm)
    assert rel_err(g.to_numpy(logits.shape), want) < TOL


def _dropout_uniform(seed, n):
    """The reference's per-index hash (cuda_kernels.cu:2300-2320) in numpy uint64."""
    with np.errstate(over="ignore"):
        i = np.arange(n, dtype=np.uint64)
        s = np.uint64(seed) + i * np.uint64(6364136223846793005) + np.uint64(1442695040888963407)
        s ^= s >> np.uint64(33)
        s *= np.uint64(0xFF51AFD7ED558CCD)
        s ^= s >> np.uint64(33)
    return (s & np.uint64(0xFFFFFF)).astype(np.float32) / np.float32(16777216.0)


def test_dropout_exact(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    from omnimatchdeeplearningtool_b200._lib import call
    rng = _rng(15)
    n = 10007
    x = rng.standard_normal(n).astype(np.float32)
    dx, o, m = _dev(x), _out((n,)), _out((n,))
    keep, seed = 0.7, 0x1234ABCD5678
    B.dropoutForward(dx.ptr, o.ptr, m.ptr, n, keep, seed)
    want_m = np.where(_dropout_uniform(seed, n) < np.float32(keep),
                      np.float32(1) / np.float32(keep), np.float32(0))
    assert np.array_equal(m.to_numpy((n,)), want_m)
    assert np.array_equal(o.to_numpy((n,)), x * want_m)
    assert abs((want_m > 0).mean() - keep) < 0.02
    # omCudaDropout: mask times 1/(1-p) in training, a plain copy otherwise
    mask = (rng.random(n) < 0.5).astype(np.float32)
    call("omCudaDropout", dx.ptr, o.ptr, _dev(mask).ptr, n, 0.5, 1)
    assert np.array_equal(o.to_numpy((n,)), x * mask * (np.float32(1) / np.float32(0.5)))
    call("omCudaDropout", dx.ptr, o.ptr, 0, n, 0.5, 0)
    assert np.array_equal(o.to_numpy((n,)), x)


def test_adam_step(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(16)
    n = 3001
    p = rng.standard_normal(n).astype(np.float32)
    m = (rng.standard_normal(n) * 0.1).astype(np.float32)
    v = (rng.random(n) * 0.01).astype(np.float32)
    dp, dm, dv = _dev(p), _dev(m), _dev(v)
    lr, b1, b2, eps = 1e-3, 0.9, 0.999, 1e-8
    p64, m64, v64 = p.astype(np.float64), m.astype(np.float64), v.astype(np.float64)
    for step in (1, 2, 3):
        g = rng.standard_normal(n).astype(np.float32)
        B.adamStep(dp.ptr, _dev(g).ptr, dm.ptr, dv.ptr, n, lr, b1, b2, eps, step)
        m64 = b1 * m64 + (1 - b1) * g
        v64 = b2 * v64 + (1 - b2) * g.astype(np.float64) ** 2
        p64 = p64 - lr * (m64 / (1 - b1 ** step)) / (np.sqrt(v64 / (1 - b2 ** step)) + eps)
    assert rel_err(dm.to_numpy((n,)), m64) < TOL_EW
    assert rel_err(dv.to_numpy((n,)), v64) < TOL
    assert rel_err(dp.to_numpy((n,)) - p, p64 - p) < 1e-3  # the update itself, within 0.1%
    assert gpu.kernel_error() == 0


@pytest.mark.parametrize("n", [5, 100003, 3 * 2 ** 20 + 7])
def test_gradient_guard_clip_and_skip(gpu, n):
    """omCudaGradNormClip + omCudaSgdStepGuarded: the training loop's NaN/Inf skip, norm clip
    to max_norm and accumulation scale (EngineBridge.cpp:1885-1925), on the device."""
    from omnimatchdeeplearningtool_b200._lib import call
    rng = _rng(17)
    g = rng.standard_normal(n).astype(np.float32)
    g64 = g.astype(np.float64)
    norm = float(np.sqrt((g64 ** 2).sum()))
    st = _out((4,))
    # below the limit: the gradient is untouched, the step goes ahead
    dg = _dev(g)
    call("omCudaGradNormClip", dg.ptr, n, norm * 2, 1.0, st.ptr)
    s = st.to_numpy((4,))
    assert abs(s[0] - norm) / norm < 1e-5 and s[1] == 1.0 and s[2] == 1.0
    assert np.array_equal(dg.to_numpy((n,)), g)
    # above the limit, then the accumulation scale, as two multiplies in that order
    for _ in range(3):  # repeated calls: the cross-block ticket resets itself
        dg = _dev(g)
        call("omCudaGradNormClip", dg.ptr, n, norm / 4, 0.5, st.ptr)
        s = st.to_numpy((4,))
        assert s[1] == 1.0 and abs(s[2] - 0.25) < 1e-5
        want = (g * np.float32(s[2])) * np.float32(0.5)
        assert np.array_equal(dg.to_numpy((n,)), want)
    first = s.copy()
    call("omCudaGradNormClip", _dev(g).ptr, n, norm / 4, 0.5, st.ptr)
    assert np.array_equal(st.to_numpy((4,)), first)  # deterministic
    # guarded SGD after a passing guard equals the plain step
    p = rng.standard_normal(n).astype(np.float32)
    v = rng.standard_normal(n).astype(np.float32)
    dp, dv = _dev(p), _dev(v)
    call("omCudaSgdStepGuarded", dp.ptr, dg.ptr, dv.ptr, n, 0.01, 0.9, st.ptr)
    dp2, dv2 = _dev(p), _dev(v)
    call("omCudaSgdStep", dp2.ptr, dg.ptr, dv2.ptr, n, 0.01, 0.9)
    assert np.array_equal(dp.to_numpy((n,)), dp2.to_numpy((n,)))
    assert np.array_equal(dv.to_numpy((n,)), dv2.to_numpy((n,)))
    # a non-finite element: verdict 0, gradient, parameters and velocity all unchanged
    bad = g.copy()
    bad[n // 2] = np.nan if n % 2 else np.inf
    dg = _dev(bad)
    call("omCudaGradNormClip", dg.ptr, n, 1.0, 0.5, st.ptr)
    s = st.to_numpy((4,))
    assert np.isnan(s[0]) and s[1] == 0.0
    assert np.array_equal(dg.to_numpy((n,)), bad, equal_nan=True)
    call("omCudaSgdStepGuarded", dp.ptr, dg.ptr, dv.ptr, n, 0.01, 0.9, st.ptr)
    assert np.array_equal(dp.to_numpy((n,)), dp2.to_numpy((n,)))
    assert np.array_equal(dv.to_numpy((n,)), dv2.to_numpy((n,)))
    assert gpu.kernel_error() == 0
