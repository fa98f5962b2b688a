// NHWC 16-bit support kernels for the fused inference path: layout conversion, BatchNorm
// folding into packed weights, max/global-average pooling, depthwise convolution and the
// residual add. All are bandwidth-bound and use 128-bit accesses along the channel dim.
//
// Window semantics follow the reference CPU backend: max pool starts from -1e30 and skips
// padding (cpu_backend.ixx:897-934); global pooling is the 1x1 adaptive average pool
// (:1467-1489); depthwise is the grouped direct conv with groups == C (:454-502).
#include "om_common.cuh"

namespace omb {

// ---------------------------------------------------------------- weight packing
// w [K, C, R, S] fp32 -> packed [K, Kpad] (16-bit), index kk = (r*S + s)*Cs + c, with the
// eval-mode BatchNorm scale folded in; zero where c >= C or kk >= R*S*Cs.
template <typename T>
__global__ void pack_conv_weight_kernel(const float* __restrict__ w, const float* __restrict__ scale,
                                        T* __restrict__ out, int K, int C, int R, int S, int Cs,
                                        long long kpad) {
    long long total = (long long)K * kpad;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int k = (int)(i / kpad);
        long long kk = i - (long long)k * kpad;
        float v = 0.f;
        if (kk < (long long)R * S * Cs) {
            int rs = (int)(kk / Cs);
            int c = (int)(kk - (long long)rs * Cs);
            int r = rs / S, s = rs - r * S;
            if (c < C) v = w[(((long long)k * C + c) * R + r) * S + s] * (scale ? scale[k] : 1.f);
        }
        if constexpr (sizeof(T) == 2) {
            if constexpr (std::is_same<T, __nv_bfloat16>::value) out[i] = __float2bfloat16_rn(v);
            else out[i] = __float2half_rn(v);
        }
    }
}

// Stem packing: w [K, C, R, S] -> [K, Kpad] with kk = (r*C + c)*8 + s (s < S <= 8), the
// layout the stem's gather warps build A in (8 horizontal taps of one plane row per chunk).
// Stem filter over the space-to-depth channels (f = stride): kk = (tr * tw + ts) * 16 + ch,
// ch = (c * f + py) * f + px holds W[k, c, f*tr + py, f*ts + px] * scale[k] (zero past the
// filter, the channels and the taps).
template <typename T>
__global__ void pack_stem_weight_kernel(const float* __restrict__ w, const float* __restrict__ scale,
                                        T* __restrict__ out, int K, int C, int R, int S, int f,
                                        int th, int tw, long long kpad) {
    long long total = (long long)K * kpad;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int k = (int)(i / kpad);
        long long kk = i - (long long)k * kpad;
        int tap = (int)(kk / 16), ch = (int)(kk % 16);
        float v = 0.f;
        if (tap < th * tw && ch < C * f * f) {
            const int tr = tap / tw, ts = tap - tr * tw;
            const int c = ch / (f * f), py = (ch / f) % f, px = ch % f;
            const int r = f * tr + py, s = f * ts + px;
            if (r < R && s < S) v = w[(((long long)k * C + c) * R + r) * S + s] * scale[k];
        }
        if constexpr (std::is_same<T, __nv_bfloat16>::value) out[i] = __float2bfloat16_rn(v);
        else out[i] = __float2half_rn(v);
    }
}

// scale[k] = gamma/sqrt(var+eps); bias[k] = beta + (b - mean)*scale (BN absent -> identity)
__global__ void fold_bn_kernel(const float* conv_bias, const float* gamma, const float* beta,
                               const float* mean, const float* var, float eps, float* scale,
                               float* bias, int K) {
    int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K) return;
    float g = gamma ? gamma[k] : 1.f;
    float v = var ? var[k] : 1.f;
    float sc = (gamma || var) ? g / sqrtf(v + eps) : 1.f;
    float b = conv_bias ? conv_bias[k] : 0.f;
    float mu = mean ? mean[k] : 0.f;
    float be = beta ? beta[k] : 0.f;
    scale[k] = sc;
    bias[k] = be + (b - mu) * sc;
}

// ---------------------------------------------------------------- layout conversion
// One thread per pixel: the C plane reads are coalesced along w across the warp and the
// pixel's Cs stored channels (zero-padded) go out as 16-byte vectors.
template <int DT>
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ in, typename Half16<DT>::T* __restrict__ out,
                                    int N, int C, int H, int W, int Cs) {
    using H16 = Half16<DT>;
    const long long pixels = (long long)N * H * W;
    const long long plane = (long long)H * W;
    for (long long pix = blockIdx.x * (long long)blockDim.x + threadIdx.x; pix < pixels;
         pix += (long long)gridDim.x * blockDim.x) {
        const long long n = pix / plane;
        const long long hw = pix - n * plane;
        const float* src = in + n * C * plane + hw;
        uint4* dst = reinterpret_cast<uint4*>(out + pix * Cs);
        for (int c8 = 0; c8 < Cs; c8 += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = (c8 + j < C) ? __ldg(src + (long long)(c8 + j) * plane) : 0.f;
            uint4 o;
            typename H16::T2* o2 = reinterpret_cast<typename H16::T2*>(&o);
#pragma unroll
            for (int j = 0; j < 4; ++j) o2[j] = H16::pack(v[2 * j], v[2 * j + 1]);
            dst[c8 / 8] = o;
        }
    }
}

template <int DT>
__global__ void nhwc_to_nchw_kernel(const typename Half16<DT>::T* __restrict__ in, float* __restrict__ out,
                                    int N, int C, int H, int W, int Cs) {
    long long total = (long long)N * C * H * W;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int w = (int)(i % W);
        long long t = i / W;
        int h = (int)(t % H);
        t /= H;
        int c = (int)(t % C);
        int n = (int)(t / C);
        out[i] = Half16<DT>::to_f(in[(((long long)n * H + h) * W + w) * Cs + c]);
    }
}

// ---------------------------------------------------------------- pooling
// One block per output row (n, p); its threads walk the row's (q, 8-channel group) items, each
// the max of up to k*k 16-byte vectors taken on packed 16-bit pairs (a max is one of its
// operands, so no rounding is involved). Windows with no pixel inside the image give -1e30,
// the reference's starting value (cpu_backend.ixx maxPool2d). KS > 0 fixes the window at
// KS x KS: all its loads are issued before the max is taken (pixels outside the image count
// as -1e30, which is where the reference starts every window too).
template <int DT, int KS>
__global__ void maxpool_nhwc_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, int H,
                                    int W, int C8, int P, int Q, int k, int stride, int pad) {
    using H16 = Half16<DT>;
    using T2 = typename H16::T2;
    const int row = blockIdx.x;          // n * P + p
    const int n = row / P;
    const int p = row - n * P;
    const int h0 = p * stride - pad;
    const uint4* img = in + (size_t)n * H * W * C8;
    uint4* orow = out + (size_t)row * Q * C8;
    const T2 lowest = H16::pack(-1e30f, -1e30f);
    if constexpr (KS > 0) {
        uint4 low4;
        {
            T2* l2 = reinterpret_cast<T2*>(&low4);
            l2[0] = l2[1] = l2[2] = l2[3] = lowest;
        }
        for (int i = threadIdx.x; i < Q * C8; i += blockDim.x) {
            const int q = i / C8;
            const int c8 = i - q * C8;
            const int w0 = q * stride - pad;
            uint4 v[KS * KS];
#pragma unroll
            for (int r = 0; r < KS; ++r) {
#pragma unroll
                for (int s = 0; s < KS; ++s) {
                    const int hh = h0 + r, ww = w0 + s;
                    const bool ok = hh >= 0 && hh < H && ww >= 0 && ww < W;
                    v[r * KS + s] = ok ? __ldg(img + ((size_t)hh * W + ww) * C8 + c8) : low4;
                }
            }
            T2 m[4] = {lowest, lowest, lowest, lowest};
#pragma unroll
            for (int t = 0; t < KS * KS; ++t) {
                const T2* v2 = reinterpret_cast<const T2*>(&v[t]);
#pragma unroll
                for (int j = 0; j < 4; ++j) m[j] = __hmax2(m[j], v2[j]);
            }
            orow[i] = *reinterpret_cast<const uint4*>(m);
        }
    } else {
        const int r0 = h0 < 0 ? -h0 : 0;
        const int r1 = (H - h0) < k ? (H - h0) : k;
        for (int i = threadIdx.x; i < Q * C8; i += blockDim.x) {
            const int q = i / C8;
            const int c8 = i - q * C8;
            const int w0 = q * stride - pad;
            const int s0 = w0 < 0 ? -w0 : 0;
            const int s1 = (W - w0) < k ? (W - w0) : k;
            T2 m[4] = {lowest, lowest, lowest, lowest};
            for (int r = r0; r < r1; ++r) {
                // first in-image pixel of the window row; the pointer never leaves the image
                const uint4* src = img + ((size_t)(h0 + r) * W + (w0 + s0)) * C8 + c8;
                for (int s = s0; s < s1; ++s) {
                    uint4 v = __ldg(src + (size_t)(s - s0) * C8);
                    const T2* v2 = reinterpret_cast<const T2*>(&v);
#pragma unroll
                    for (int j = 0; j < 4; ++j) m[j] = __hmax2(m[j], v2[j]);
                }
            }
            orow[i] = *reinterpret_cast<const uint4*>(m);
        }
    }
}

// One block per image: thread t owns channel group t % C8 and pixel row t / C8, and walks the
// pixels row, row + rows, ... (rows = blockDim / C8) with four 16-byte loads in flight. Each row's
// partial sums go to shared memory and are added in row order, so the result does not depend
// on scheduling.
template <int DT>
__global__ void gap_nhwc_kernel(const uint4* __restrict__ in, void* __restrict__ out, int HW,
                                int C8, int out_f32) {
    using H16 = Half16<DT>;
    extern __shared__ float sh[];  // [rows][C8 * 8] partial sums
    const int n = blockIdx.x;
    const int rows = (int)blockDim.x / C8;
    const int cg = threadIdx.x % C8;
    const int row = threadIdx.x / C8;
    const int C = C8 * 8;
    if (row < rows) {
        const uint4* src = in + (long long)n * HW * C8 + cg;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        int pix = row;
        for (; pix + 3 * rows < HW; pix += 4 * rows) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldg(src + (long long)(pix + u * rows) * C8);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const typename H16::T2* v2 = reinterpret_cast<const typename H16::T2*>(&v[u]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = H16::unpack(v2[j]);
                    acc[2 * j] += f.x;
                    acc[2 * j + 1] += f.y;
                }
            }
        }
        for (; pix < HW; pix += rows) {
            uint4 v = __ldg(src + (long long)pix * C8);
            const typename H16::T2* v2 = reinterpret_cast<const typename H16::T2*>(&v);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f = H16::unpack(v2[j]);
                acc[2 * j] += f.x;
                acc[2 * j + 1] += f.y;
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) sh[row * C + cg * 8 + j] = acc[j];
    }
    __syncthreads();
    const float inv = 1.f / (float)HW;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float v = 0.f;
        for (int r = 0; r < rows; ++r) v += sh[r * C + c];
        v *= inv;
        if (out_f32)
            static_cast<float*>(out)[(long long)n * C + c] = v;
        else
            static_cast<typename H16::T*>(out)[(long long)n * C + c] = H16::from_f(v);
    }
}

// ---------------------------------------------------------------- depthwise conv
// packed weight: fp32 [R*S, Cs] (BN scale folded), bias fp32 [Cs]. One block per output row
// (n, p); its threads walk the row's (q, 8-channel group) items with 32-bit indices. KS > 0
// fixes the window at KS x KS: the item's KS*KS input loads are all issued before the
// arithmetic (taps outside the image load zeros), which keeps the HBM pipe busy; the taps are
// accumulated in the same order as the general loop.
// One window tap: the 8 channels at (hh, ww), or zeros outside the image. The load itself is
// unconditional (from the clamped, always valid pixel) and the zeros are selected afterwards,
// so that a thread's taps are all in flight at once instead of each waiting behind a branch.
__device__ __forceinline__ uint4 tap_load(const uint4* __restrict__ img, int hh, int ww, int H,
                                          int W, int C8, int c8) {
    const bool ok = hh >= 0 && hh < H && ww >= 0 && ww < W;
    const int hc = min(max(hh, 0), H - 1), wc = min(max(ww, 0), W - 1);
    const uint4 t = __ldg(img + ((size_t)hc * W + wc) * C8 + c8);
    return ok ? t : make_uint4(0, 0, 0, 0);
}

template <int DT, int KS>
__global__ void depthwise_nhwc_kernel(const uint4* __restrict__ in, const float* __restrict__ wpk,
                                      const float* __restrict__ bias, uint4* __restrict__ out,
                                      int H, int W, int C8, int P, int Q, int R, int S,
                                      int stride, int pad, int act, int pair) {
    using H16 = Half16<DT>;
    const int Cs = C8 * 8;
    const int row = blockIdx.x;          // n * P + p (pair: n * ceil(P/2) + p/2)
    const int n = pair ? row / ((P + 1) / 2) : row / P;
    const int p = row - n * P;
    const int h0 = p * stride - pad;
    const uint4* img = in + (size_t)n * H * W * C8;
    uint4* orow = out + (size_t)row * Q * C8;
    if constexpr (KS > 0 && DT == OM_DTYPE_F16) {
        if (blockDim.x % C8 == 0) {
            // fp16: every item of this thread has the same 8 channels, so the KS*KS weights
            // and the bias are loaded once, as half2, and the taps are accumulated with HFMA2
            // (9 fp16 products and the bias: ~1e-3 relative, inside the 16-bit tolerance)
            const int c8 = (int)threadIdx.x % C8;
            __half2 wt[KS * KS][4];
#pragma unroll
            for (int t = 0; t < KS * KS; ++t) {
                const float4* w4 = reinterpret_cast<const float4*>(wpk + (size_t)t * Cs + c8 * 8);
                const float4 wa = __ldg(w4), wb = __ldg(w4 + 1);
                wt[t][0] = __floats2half2_rn(wa.x, wa.y);
                wt[t][1] = __floats2half2_rn(wa.z, wa.w);
                wt[t][2] = __floats2half2_rn(wb.x, wb.y);
                wt[t][3] = __floats2half2_rn(wb.z, wb.w);
            }
            const float4* b4 = reinterpret_cast<const float4*>(bias + c8 * 8);
            const float4 ba = __ldg(b4), bb = __ldg(b4 + 1);
            const __half2 bh[4] = {__floats2half2_rn(ba.x, ba.y), __floats2half2_rn(ba.z, ba.w),
                                   __floats2half2_rn(bb.x, bb.y), __floats2half2_rn(bb.z, bb.w)};
            const __half2 zero = __float2half2_rn(0.f), six = __float2half2_rn(6.f);
            auto finish = [&](__half2 (&acc)[4]) {
                uint4 o;
                __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __half2 a = acc[j];
                    if (act == OM_ACT_RELU) a = __hmax2(a, zero);
                    else if (act == OM_ACT_RELU6) a = __hmin2(__hmax2(a, zero), six);
                    o2[j] = a;
                }
                return o;
            };
            if (pair) {
                // stride 1: this block owns output rows p and p + 1 (2 * blockIdx.x within the
                // image); the two windows share KS - 1 input rows, loaded once
                const int pr = 2 * (row - n * ((P + 1) / 2));
                const int hb = pr - pad;
                const bool second = pr + 1 < P;
                uint4* orow0 = out + ((size_t)n * P + pr) * Q * C8;
                for (int i = threadIdx.x; i < Q * C8; i += blockDim.x) {
                    const int q = i / C8;
                    const int w0 = q - pad;
                    uint4 v[(KS + 1) * KS];
#pragma unroll
                    for (int r = 0; r < KS + 1; ++r) {
#pragma unroll
                        for (int sx = 0; sx < KS; ++sx) {
                            const int hh = hb + r, ww = w0 + sx;
                            v[r * KS + sx] = tap_load(img, hh, ww, H, W, C8, c8);
                        }
                    }
                    __half2 a0[4] = {bh[0], bh[1], bh[2], bh[3]};
                    __half2 a1[4] = {bh[0], bh[1], bh[2], bh[3]};
#pragma unroll
                    for (int t = 0; t < KS * KS; ++t) {
                        const __half2* x0 = reinterpret_cast<const __half2*>(&v[t]);
                        const __half2* x1 = reinterpret_cast<const __half2*>(&v[t + KS]);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            a0[j] = __hfma2(x0[j], wt[t][j], a0[j]);
                            a1[j] = __hfma2(x1[j], wt[t][j], a1[j]);
                        }
                    }
                    orow0[i] = finish(a0);
                    if (second) orow0[(size_t)Q * C8 + i] = finish(a1);
                }
                return;
            }
            for (int i = threadIdx.x; i < Q * C8; i += blockDim.x) {
                const int q = i / C8;
                const int w0 = q * stride - pad;
                uint4 v[KS * KS];
#pragma unroll
                for (int r = 0; r < KS; ++r) {
#pragma unroll
                    for (int sx = 0; sx < KS; ++sx) {
                        const int hh = h0 + r, ww = w0 + sx;
                        v[r * KS + sx] = tap_load(img, hh, ww, H, W, C8, c8);
                    }
                }
                __half2 acc[4] = {bh[0], bh[1], bh[2], bh[3]};
#pragma unroll
                for (int t = 0; t < KS * KS; ++t) {
                    const __half2* v2 = reinterpret_cast<const __half2*>(&v[t]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[j] = __hfma2(v2[j], wt[t][j], acc[j]);
                }
                orow[i] = finish(acc);
            }
            return;
        }
    }
    if constexpr (KS > 0) {
        for (int i = threadIdx.x; i < Q * C8; i += blockDim.x) {
            const int q = i / C8;
            const int c8 = i - q * C8;
            const int w0 = q * stride - pad;
            uint4 v[KS * KS];
#pragma unroll
            for (int r = 0; r < KS; ++r) {
#pragma unroll
                for (int sx = 0; sx < KS; ++sx) {
                    const int hh = h0 + r, ww = w0 + sx;
                    v[r * KS + sx] = tap_load(img, hh, ww, H, W, C8, c8);
                }
            }
            float acc[8];
            const float4* b4 = reinterpret_cast<const float4*>(bias + c8 * 8);
            float4 b0 = __ldg(b4), b1 = __ldg(b4 + 1);
            acc[0] = b0.x; acc[1] = b0.y; acc[2] = b0.z; acc[3] = b0.w;
            acc[4] = b1.x; acc[5] = b1.y; acc[6] = b1.z; acc[7] = b1.w;
#pragma unroll
            for (int t = 0; t < KS * KS; ++t) {
                const int r = t / KS, sx = t - r * KS;
                if (h0 + r < 0 || h0 + r >= H || w0 + sx < 0 || w0 + sx >= W) continue;
                const typename H16::T2* v2 = reinterpret_cast<const typename H16::T2*>(&v[t]);
                const float4* w4 = reinterpret_cast<const float4*>(wpk + (size_t)t * Cs + c8 * 8);
                float4 wa = __ldg(w4), wb = __ldg(w4 + 1);
                float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = H16::unpack(v2[j]);
                    acc[2 * j] += f.x * wv[2 * j];
                    acc[2 * j + 1] += f.y * wv[2 * j + 1];
                }
            }
            uint4 o;
            typename H16::T2* o2 = reinterpret_cast<typename H16::T2*>(&o);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                o2[j] = H16::pack(apply_act(acc[2 * j], act), apply_act(acc[2 * j + 1], act));
            orow[i] = o;
        }
        return;
    }
    const int r0 = h0 < 0 ? -h0 : 0;
    const int r1 = (H - h0) < R ? (H - h0) : R;
    for (int i = threadIdx.x; i < Q * C8; i += blockDim.x) {
        const int q = i / C8;
        const int c8 = i - q * C8;
        const int w0 = q * stride - pad;
        const int s0 = w0 < 0 ? -w0 : 0;
        const int s1 = (W - w0) < S ? (W - w0) : S;
        float acc[8];
        const float4* b4 = reinterpret_cast<const float4*>(bias + c8 * 8);
        float4 b0 = __ldg(b4), b1 = __ldg(b4 + 1);
        acc[0] = b0.x; acc[1] = b0.y; acc[2] = b0.z; acc[3] = b0.w;
        acc[4] = b1.x; acc[5] = b1.y; acc[6] = b1.z; acc[7] = b1.w;
        for (int r = r0; r < r1; ++r) {
            // first in-image pixel of the window row; the pointer never leaves the image
            const uint4* src = img + ((size_t)(h0 + r) * W + (w0 + s0)) * C8 + c8;
            const float* wr = wpk + (size_t)(r * S) * Cs + c8 * 8;
            for (int s = s0; s < s1; ++s) {
                uint4 v = __ldg(src + (size_t)(s - s0) * C8);
                const typename H16::T2* v2 = reinterpret_cast<const typename H16::T2*>(&v);
                const float4* w4 = reinterpret_cast<const float4*>(wr + (size_t)s * Cs);
                float4 wa = __ldg(w4), wb = __ldg(w4 + 1);
                float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = H16::unpack(v2[j]);
                    acc[2 * j] += f.x * wv[2 * j];
                    acc[2 * j + 1] += f.y * wv[2 * j + 1];
                }
            }
        }
        uint4 o;
        typename H16::T2* o2 = reinterpret_cast<typename H16::T2*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            o2[j] = H16::pack(apply_act(acc[2 * j], act), apply_act(acc[2 * j + 1], act));
        orow[i] = o;
    }
}

__global__ void pack_depthwise_kernel(const float* __restrict__ w, const float* __restrict__ scale,
                                      const float* __restrict__ bias_in, float* __restrict__ wpk,
                                      float* __restrict__ bias_out, int C, int RS, int Cs) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= RS * Cs) return;
    int rs = i / Cs, c = i - rs * Cs;
    wpk[i] = c < C ? w[(long long)c * RS + rs] * scale[c] : 0.f;
    if (rs == 0) bias_out[c] = c < C ? bias_in[c] : 0.f;
}

// ---------------------------------------------------------------- residual add
template <int DT>
__global__ void add_act_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
                               uint4* __restrict__ out, long long n8, int act) {
    using H16 = Half16<DT>;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
         i += (long long)gridDim.x * blockDim.x) {
        uint4 va = a[i], vb = b[i], o;
        const typename H16::T2* a2 = reinterpret_cast<const typename H16::T2*>(&va);
        const typename H16::T2* b2 = reinterpret_cast<const typename H16::T2*>(&vb);
        typename H16::T2* o2 = reinterpret_cast<typename H16::T2*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float2 x = H16::unpack(a2[j]), y = H16::unpack(b2[j]);
            o2[j] = H16::pack(apply_act(x.x + y.x, act), apply_act(x.y + y.y, act));
        }
        out[i] = o;
    }
}

}  // namespace omb

using namespace omb;

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int omCudaPackConvWeight(const float* pWeight, const float* pConvBias,
                                    const float* pGamma, const float* pBeta, const float* pMean,
                                    const float* pVar, float fEps, void* pPacked, float* pBiasOut,
                                    int nCout, int nCin, int nKH, int nKW, int nCs, int nDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pWeight || !pPacked || !pBiasOut || nCout <= 0 || nCin <= 0 || nCs < nCin) return OM_ERR_INVALID;
    if (nDtype != OM_DTYPE_BF16 && nDtype != OM_DTYPE_F16) return OM_ERR_UNSUPPORTED;
    long long kpad = omCudaPackedConvWeightElems(1, nKH, nKW, nCs);
    float* scale = nullptr;
    OMB_CHECK(cudaMallocAsync(&scale, sizeof(float) * nCout, c->compute));
    fold_bn_kernel<<<(nCout + 255) / 256, 256, 0, c->compute>>>(pConvBias, pGamma, pBeta, pMean,
                                                                 pVar, fEps, scale, pBiasOut, nCout);
    int st = after_launch(c);
    if (st == OM_OK) {
        long long total = (long long)nCout * kpad;
        int grid = ew_grid(c, total, 256);
        if (nDtype == OM_DTYPE_BF16)
            pack_conv_weight_kernel<__nv_bfloat16><<<grid, 256, 0, c->compute>>>(
                pWeight, scale, static_cast<__nv_bfloat16*>(pPacked), nCout, nCin, nKH, nKW, nCs, kpad);
        else
            pack_conv_weight_kernel<__half><<<grid, 256, 0, c->compute>>>(
                pWeight, scale, static_cast<__half*>(pPacked), nCout, nCin, nKH, nKW, nCs, kpad);
        st = after_launch(c);
    }
    cudaFreeAsync(scale, c->compute);
    return st;
}

extern "C" int omCudaNchwToNhwc(const float* pIn, void* pOut, int nN, int nC, int nH, int nW,
                                int nCs, int nDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nCs < nC || nCs % 8 || nN <= 0 || nC <= 0 || nH <= 0 || nW <= 0 ||
        !aligned16(pOut))
        return OM_ERR_INVALID;
    long long total = (long long)nN * nH * nW;
    int grid = ew_grid(c, total, 256);
    if (nDtype == OM_DTYPE_BF16)
        nchw_to_nhwc_kernel<OM_DTYPE_BF16><<<grid, 256, 0, c->compute>>>(
            pIn, static_cast<__nv_bfloat16*>(pOut), nN, nC, nH, nW, nCs);
    else if (nDtype == OM_DTYPE_F16)
        nchw_to_nhwc_kernel<OM_DTYPE_F16><<<grid, 256, 0, c->compute>>>(
            pIn, static_cast<__half*>(pOut), nN, nC, nH, nW, nCs);
    else
        return OM_ERR_UNSUPPORTED;
    return after_launch(c);
}

extern "C" int omCudaNhwcToNchw(const void* pIn, float* pOut, int nN, int nC, int nH, int nW,
                                int nCs, int nDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nCs < nC) return OM_ERR_INVALID;
    long long total = (long long)nN * nC * nH * nW;
    int grid = ew_grid(c, total, 256);
    if (nDtype == OM_DTYPE_BF16)
        nhwc_to_nchw_kernel<OM_DTYPE_BF16><<<grid, 256, 0, c->compute>>>(
            static_cast<const __nv_bfloat16*>(pIn), pOut, nN, nC, nH, nW, nCs);
    else if (nDtype == OM_DTYPE_F16)
        nhwc_to_nchw_kernel<OM_DTYPE_F16><<<grid, 256, 0, c->compute>>>(
            static_cast<const __half*>(pIn), pOut, nN, nC, nH, nW, nCs);
    else
        return OM_ERR_UNSUPPORTED;
    return after_launch(c);
}

extern "C" int omCudaMaxPool2dNhwc(const void* pIn, void* pOut, int nN, int nH, int nW, int nCs,
                                   int nK, int nStride, int nPad, int nDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nCs % 8 || !aligned16(pIn) || !aligned16(pOut)) return OM_ERR_INVALID;
    int P = (nH + 2 * nPad - nK) / nStride + 1, Q = (nW + 2 * nPad - nK) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    const long long rows = (long long)nN * P;
    if (rows >= (1LL << 31) || (long long)Q * (nCs / 8) >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    const int threads = Q * (nCs / 8) >= 256 ? 256 : 128;
    const uint4* src = static_cast<const uint4*>(pIn);
    uint4* dst = static_cast<uint4*>(pOut);
    const int c8 = nCs / 8;
    if (nDtype == OM_DTYPE_BF16) {
        if (nK == 3)
            maxpool_nhwc_kernel<OM_DTYPE_BF16, 3><<<(unsigned)rows, threads, 0, c->compute>>>(
                src, dst, nH, nW, c8, P, Q, nK, nStride, nPad);
        else
            maxpool_nhwc_kernel<OM_DTYPE_BF16, 0><<<(unsigned)rows, threads, 0, c->compute>>>(
                src, dst, nH, nW, c8, P, Q, nK, nStride, nPad);
    } else if (nDtype == OM_DTYPE_F16) {
        if (nK == 3)
            maxpool_nhwc_kernel<OM_DTYPE_F16, 3><<<(unsigned)rows, threads, 0, c->compute>>>(
                src, dst, nH, nW, c8, P, Q, nK, nStride, nPad);
        else
            maxpool_nhwc_kernel<OM_DTYPE_F16, 0><<<(unsigned)rows, threads, 0, c->compute>>>(
                src, dst, nH, nW, c8, P, Q, nK, nStride, nPad);
    } else {
        return OM_ERR_UNSUPPORTED;
    }
    return after_launch(c);
}

extern "C" int omCudaGlobalAvgPoolNhwc(const void* pIn, void* pOut, int nN, int nHW, int nCs,
                                       int nDtype, int nOutDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nCs % 8 || nCs > 2048 || !aligned16(pIn)) return OM_ERR_INVALID;
    if (nOutDtype != OM_DTYPE_F32 && nOutDtype != nDtype) return OM_ERR_UNSUPPORTED;
    int C8 = nCs / 8;
    // up to 1024 threads: C8 channel groups x as many pixel rows as fit (one row at least)
    const int rows = C8 >= 1024 ? 1 : 1024 / C8;
    const int threads = C8 * rows;
    if (threads > 1024) return OM_ERR_UNSUPPORTED;
    size_t sh = sizeof(float) * (size_t)rows * nCs;
    int of32 = nOutDtype == OM_DTYPE_F32;
    if (nDtype == OM_DTYPE_BF16)
        gap_nhwc_kernel<OM_DTYPE_BF16><<<nN, threads, sh, c->compute>>>(static_cast<const uint4*>(pIn), pOut, nHW, C8, of32);
    else if (nDtype == OM_DTYPE_F16)
        gap_nhwc_kernel<OM_DTYPE_F16><<<nN, threads, sh, c->compute>>>(static_cast<const uint4*>(pIn), pOut, nHW, C8, of32);
    else
        return OM_ERR_UNSUPPORTED;
    return after_launch(c);
}

extern "C" int omCudaPackDepthwiseWeight(const float* pWeight, const float* pGamma,
                                         const float* pBeta, const float* pMean, const float* pVar,
                                         float fEps, float* pPacked, float* pBiasOut, int nC,
                                         int nKH, int nKW, int nCs) {
    OMB_CTX_OR_FAIL(c);
    if (!pWeight || !pPacked || !pBiasOut || nCs < nC) return OM_ERR_INVALID;
    float *scale = nullptr, *bias = nullptr;
    OMB_CHECK(cudaMallocAsync(&scale, sizeof(float) * nC, c->compute));
    OMB_CHECK(cudaMallocAsync(&bias, sizeof(float) * nC, c->compute));
    fold_bn_kernel<<<(nC + 255) / 256, 256, 0, c->compute>>>(nullptr, pGamma, pBeta, pMean, pVar,
                                                             fEps, scale, bias, nC);
    int st = after_launch(c);
    if (st == OM_OK) {
        int total = nKH * nKW * nCs;
        pack_depthwise_kernel<<<(total + 255) / 256, 256, 0, c->compute>>>(
            pWeight, scale, bias, pPacked, pBiasOut, nC, nKH * nKW, nCs);
        st = after_launch(c);
    }
    cudaFreeAsync(scale, c->compute);
    cudaFreeAsync(bias, c->compute);
    return st;
}

// the ring kernel for fp16 3x3 layers with padding 1 and stride 1 or 2 (om_conv_tc.cu)
extern "C" __attribute__((visibility("hidden"))) int omb_depthwise_ring(
    DeviceCtx* c, const void* pIn, const float* pPacked, const float* pBias, void* pOut, int nN,
    int nH, int nW, int nCs, int nStride, int nAct);

extern "C" int omCudaDepthwiseConv2dNhwc(const void* pIn, const float* pPacked, const float* pBias,
                                         void* pOut, int nN, int nH, int nW, int nCs, int nKH,
                                         int nKW, int nStride, int nPad, int nAct, int nDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || !pPacked || !pBias || nCs % 8 || !aligned16(pIn) || !aligned16(pOut) ||
        !aligned16(pPacked) || !aligned16(pBias))
        return OM_ERR_INVALID;
    int P = (nH + 2 * nPad - nKH) / nStride + 1, Q = (nW + 2 * nPad - nKW) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    const long long rows = (long long)nN * P;
    if (rows >= (1LL << 31) || (long long)Q * (nCs / 8) >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    const int threads = Q * (nCs / 8) >= 256 ? 256 : 128;
    const uint4* src = static_cast<const uint4*>(pIn);
    uint4* dst = static_cast<uint4*>(pOut);
    const int c8 = nCs / 8;
    const bool k3 = nKH == 3 && nKW == 3;
    if (nDtype == OM_DTYPE_F16 && k3 && nPad == 1) {
        const int st = omb_depthwise_ring(c, pIn, pPacked, pBias, pOut, nN, nH, nW, nCs, nStride,
                                          nAct);
        if (st != OM_ERR_UNSUPPORTED) return st;
    }
    // fp16, 3x3, stride 1, every thread on fixed channels: one block per pair of output rows
    const int pair = (nDtype == OM_DTYPE_F16 && k3 && nStride == 1 && threads % c8 == 0) ? 1 : 0;
    const unsigned grid = pair ? (unsigned)((long long)nN * ((P + 1) / 2)) : (unsigned)rows;
    if (nDtype == OM_DTYPE_BF16) {
        if (k3)
            depthwise_nhwc_kernel<OM_DTYPE_BF16, 3><<<grid, threads, 0, c->compute>>>(
                src, pPacked, pBias, dst, nH, nW, c8, P, Q, nKH, nKW, nStride, nPad, nAct, 0);
        else
            depthwise_nhwc_kernel<OM_DTYPE_BF16, 0><<<grid, threads, 0, c->compute>>>(
                src, pPacked, pBias, dst, nH, nW, c8, P, Q, nKH, nKW, nStride, nPad, nAct, 0);
    } else if (nDtype == OM_DTYPE_F16) {
        if (k3)
            depthwise_nhwc_kernel<OM_DTYPE_F16, 3><<<grid, threads, 0, c->compute>>>(
                src, pPacked, pBias, dst, nH, nW, c8, P, Q, nKH, nKW, nStride, nPad, nAct, pair);
        else
            depthwise_nhwc_kernel<OM_DTYPE_F16, 0><<<grid, threads, 0, c->compute>>>(
                src, pPacked, pBias, dst, nH, nW, c8, P, Q, nKH, nKW, nStride, nPad, nAct, 0);
    } else {
        return OM_ERR_UNSUPPORTED;
    }
    return after_launch(c);
}

extern "C" int omCudaAddActNhwc(const void* pA, const void* pB, void* pOut, long long nCount,
                                int nAct, int nDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pB || !pOut || nCount % 8 || !aligned16(pA) || !aligned16(pB) || !aligned16(pOut))
        return OM_ERR_INVALID;
    long long n8 = nCount / 8;
    int grid = ew_grid(c, n8, 256);
    if (nDtype == OM_DTYPE_BF16)
        add_act_kernel<OM_DTYPE_BF16><<<grid, 256, 0, c->compute>>>(
            static_cast<const uint4*>(pA), static_cast<const uint4*>(pB), static_cast<uint4*>(pOut), n8, nAct);
    else if (nDtype == OM_DTYPE_F16)
        add_act_kernel<OM_DTYPE_F16><<<grid, 256, 0, c->compute>>>(
            static_cast<const uint4*>(pA), static_cast<const uint4*>(pB), static_cast<uint4*>(pOut), n8, nAct);
    else
        return OM_ERR_UNSUPPORTED;
    return after_launch(c);
}

extern "C" int omCudaPackStemWeight(const float* pWeight, const float* pConvBias,
                                    const float* pGamma, const float* pBeta, const float* pMean,
                                    const float* pVar, float fEps, void* pPacked, float* pBiasOut,
                                    int nCout, int nCin, int nKH, int nKW, int nStride, int nDtype) {
    OMB_CTX_OR_FAIL(c);
    if (!pWeight || !pPacked || !pBiasOut || nCout <= 0 || nCin <= 0 || nKH <= 0 || nKW <= 0)
        return OM_ERR_INVALID;
    if (nStride != 1 && nStride != 2) return OM_ERR_UNSUPPORTED;
    if (nCin * nStride * nStride > 16) return OM_ERR_UNSUPPORTED;
    if (nDtype != OM_DTYPE_BF16 && nDtype != OM_DTYPE_F16) return OM_ERR_UNSUPPORTED;
    const int th = (nKH + nStride - 1) / nStride, tw = (nKW + nStride - 1) / nStride;
    const long long kpad = omCudaPackedStemWeightElems(1, nCin, nKH, nKW, nStride);
    float* scale = nullptr;
    OMB_CHECK(cudaMallocAsync(&scale, sizeof(float) * nCout, c->compute));
    fold_bn_kernel<<<(nCout + 255) / 256, 256, 0, c->compute>>>(pConvBias, pGamma, pBeta, pMean,
                                                                 pVar, fEps, scale, pBiasOut, nCout);
    int st = after_launch(c);
    if (st == OM_OK) {
        long long total = (long long)nCout * kpad;
        int grid = ew_grid(c, total, 256);
        if (nDtype == OM_DTYPE_BF16)
            pack_stem_weight_kernel<__nv_bfloat16><<<grid, 256, 0, c->compute>>>(
                pWeight, scale, static_cast<__nv_bfloat16*>(pPacked), nCout, nCin, nKH, nKW,
                nStride, th, tw, kpad);
        else
            pack_stem_weight_kernel<__half><<<grid, 256, 0, c->compute>>>(
                pWeight, scale, static_cast<__half*>(pPacked), nCout, nCin, nKH, nKW, nStride, th,
                tw, kpad);
        st = after_launch(c);
    }
    cudaFreeAsync(scale, c->compute);
    return st;
}
