// fp32 NCHW bandwidth-bound ops behind the reference C ABI: BatchNorm forward/backward,
// pooling, softmax / cross-entropy, SGD, bias add and elementwise kernels.
//
// Numerics follow the reference CPU backend (the parity target), not the reference GPU
// kernels where the two disagree:
//   - softmax divides by the plain sum (cpu_backend.ixx:352-370; the reference GPU kernel
//     adds 1e-7, cuda_kernels.cu:1450);
//   - cross-entropy clamps p at 1e-7 and counts targets > 0.5 (cpu_backend.ixx:375-388; the
//     GPU kernel uses log(p + 1e-10), cuda_kernels.cu:3934);
//   - BatchNorm updates the running variance with the biased batch variance, as the CPU
//     backend does (cpu_backend.ixx:781-842).
// BatchNorm statistics are reduced per channel over N*H*W by a (channel x split) grid whose
// per-split partial sums go to a small scratch buffer, then combined in a fixed order, so
// the result is deterministic and large feature maps still fill all SMs.
#include <mutex>

#include <algorithm>

#include "om_common.cuh"

namespace omb {
namespace ops {

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}
// block-wide sum, result valid in thread 0
__device__ __forceinline__ float block_sum(float v) {
    __shared__ float sh[32];
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < ((blockDim.x + 31) >> 5) ? sh[threadIdx.x] : 0.f;
        v = warp_sum(v);
    }
    return v;
}

// ---------------------------------------------------------------- BatchNorm
// Channel c's reduction domain is the N*HW elements j = n*HW + hw (n-major), element j at
// (n*C + c)*HW + hw. A reduction block covers [z*chunk, (z+1)*chunk); thread t sums j = beg+t,
// beg+t+256, ... in that order, so the result depends only on (C, HW, N, splits), never on
// timing. n = j / HW comes from a 32-bit multiply-shift division by the invariant HW (the
// round-up method of Granlund and Montgomery), valid for j < 2^31; the loop is unrolled so that
// loads overlap while the additions keep their order.
struct FastDiv {
    uint32_t d, mul, shift;
};
static FastDiv make_fastdiv(uint32_t d) {
    uint32_t shift = 0;
    while (shift < 32 && (1ull << shift) < d) ++shift;
    const uint64_t one = 1;
    const uint64_t magic = ((one << 32) * ((one << shift) - d)) / d + 1;
    return FastDiv{d, (uint32_t)magic, shift};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
    return (__umulhi(n, f.mul) + n) >> f.shift;
}
__device__ __forceinline__ size_t bn_index(uint32_t j, int c, int C, const FastDiv& hw) {
    const uint32_t n = fdiv(j, hw);
    return ((size_t)n * C + c) * hw.d + (j - n * hw.d);
}

__global__ void bn_partial_sum_kernel(const float* __restrict__ x, float* __restrict__ part, int C,
                                      FastDiv hw, long long cnt, long long chunk) {
    const int c = blockIdx.x, z = blockIdx.y;
    const long long beg = z * chunk, end = min(cnt, beg + chunk);
    float s = 0.f;
#pragma unroll 8
    for (long long j = beg + threadIdx.x; j < end; j += blockDim.x)
        s += __ldg(x + bn_index((uint32_t)j, c, C, hw));
    s = block_sum(s);
    if (threadIdx.x == 0) part[(long long)c * gridDim.y + z] = s;
}

__global__ void bn_partial_m2_kernel(const float* __restrict__ x, const float* __restrict__ psum,
                                     float* __restrict__ part, int C, FastDiv hw, long long cnt,
                                     long long chunk) {
    const int c = blockIdx.x, z = blockIdx.y, S = gridDim.y;
    float tot = 0.f;
    for (int i = 0; i < S; ++i) tot += psum[(long long)c * S + i];
    const float mean = tot / (float)cnt;
    const long long beg = z * chunk, end = min(cnt, beg + chunk);
    float s = 0.f;
#pragma unroll 8
    for (long long j = beg + threadIdx.x; j < end; j += blockDim.x) {
        const float d = __ldg(x + bn_index((uint32_t)j, c, C, hw)) - mean;
        s += d * d;
    }
    s = block_sum(s);
    if (threadIdx.x == 0) part[(long long)c * S + z] = s;
}

// mean/invstd per channel into saved buffers; running statistics updated in training mode
__global__ void bn_finalize_kernel(const float* __restrict__ psum, const float* __restrict__ pm2,
                                   int S, long long cnt, float* run_mean, float* run_var,
                                   float* saved_mean, float* saved_invstd, float eps,
                                   float momentum, int training, int C) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float mean, var;
    if (training) {
        float s = 0.f, m2 = 0.f;
        for (int i = 0; i < S; ++i) {
            s += psum[(long long)c * S + i];
            m2 += pm2[(long long)c * S + i];
        }
        mean = s / (float)cnt;
        var = m2 / (float)cnt;
        run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mean;
        run_var[c] = (1.f - momentum) * run_var[c] + momentum * var;
    } else {
        mean = run_mean[c];
        var = run_var[c];
    }
    saved_mean[c] = mean;
    saved_invstd[c] = 1.f / sqrtf(var + eps);
}

// Elementwise BN kernels over the NCHW tensor. V = 4: vectors of 4 floats that share a channel
// (HW % 4 == 0), one 32-bit division per vector (total < 2^32); V = 1: any shape.
// relu = 1: the ReLU of the result, written with the reference's expression (v > 0 ? v : 0).
__device__ __forceinline__ float bn_act(float v, int relu) { return relu ? (v > 0.f ? v : 0.f) : v; }
// y = act(gamma * (x - mean) * invstd + beta [+ res]): with res (a residual branch, same shape)
// the sum is taken before the activation, as an add and then a ReLU would. V = 4: float4
// vectors; PE: a vector may span channels (HW % 4 != 0), each element looks up its own channel.
// Every element gets the same expression as with V = 1.
template <int V, bool PE = false>
__global__ void bn_apply_kernel(const float* __restrict__ x, float* __restrict__ y,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                const float* __restrict__ mean, const float* __restrict__ invstd,
                                long long total, int C, int HW, int relu,
                                const float* __restrict__ res) {
    const long long nv = total / V;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv;
         i += (long long)gridDim.x * blockDim.x) {
        int c;
        if constexpr (V == 4) c = (int)(((unsigned)i * 4u / (unsigned)HW) % (unsigned)C);
        else c = (int)((i / HW) % C);
        if constexpr (V == 4) {
            int c1 = c, c2 = c, c3 = c;
            if constexpr (PE) {
                const unsigned e = (unsigned)i * 4u;
                c = (int)((e / (unsigned)HW) % (unsigned)C);
                c1 = (int)(((e + 1u) / (unsigned)HW) % (unsigned)C);
                c2 = (int)(((e + 2u) / (unsigned)HW) % (unsigned)C);
                c3 = (int)(((e + 3u) / (unsigned)HW) % (unsigned)C);
            }
            const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
            float4 o = make_float4(gamma[c] * (v.x - mean[c]) * invstd[c] + beta[c],
                                   gamma[c1] * (v.y - mean[c1]) * invstd[c1] + beta[c1],
                                   gamma[c2] * (v.z - mean[c2]) * invstd[c2] + beta[c2],
                                   gamma[c3] * (v.w - mean[c3]) * invstd[c3] + beta[c3]);
            if (res) {
                const float4 r = __ldg(reinterpret_cast<const float4*>(res) + i);
                o.x += r.x; o.y += r.y; o.z += r.z; o.w += r.w;
            }
            reinterpret_cast<float4*>(y)[i] = make_float4(bn_act(o.x, relu), bn_act(o.y, relu),
                                                          bn_act(o.z, relu), bn_act(o.w, relu));
        } else {
            float o = gamma[c] * (x[i] - mean[c]) * invstd[c] + beta[c];
            if (res) o += res[i];
            y[i] = bn_act(o, relu);
        }
    }
}

__global__ void bn_bwd_partial_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                      const float* __restrict__ mean, const float* __restrict__ invstd,
                                      const float* __restrict__ mask, float* __restrict__ pg,
                                      float* __restrict__ pb, int C, FastDiv hw, long long cnt,
                                      long long chunk) {
    const int c = blockIdx.x, z = blockIdx.y;
    const float mu = mean[c], is = invstd[c];
    const long long beg = z * chunk, end = min(cnt, beg + chunk);
    float sg = 0.f, sb = 0.f;
#pragma unroll 8
    for (long long j = beg + threadIdx.x; j < end; j += blockDim.x) {
        const size_t idx = bn_index((uint32_t)j, c, C, hw);
        float g = __ldg(dy + idx);
        if (mask) g = __ldg(mask + idx) > 0.f ? g : 0.f;   // the ReLU backward, fused
        sg += g * (__ldg(x + idx) - mu) * is;
        sb += g;
    }
    sg = block_sum(sg);
    if (threadIdx.x == 0) pg[(long long)c * gridDim.y + z] = sg;
    sb = block_sum(sb);
    if (threadIdx.x == 0) pb[(long long)c * gridDim.y + z] = sb;
}

// The same partial sums four pixels at a time (HW % 4 == 0, chunk % 4 == 0, 16-byte aligned
// tensors): the four share an image and a channel plane, so one index computation and one
// 16-byte load per tensor cover them. The pass is bound by instruction issue, not bandwidth.
__global__ void bn_bwd_partial4_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                       const float* __restrict__ mean,
                                       const float* __restrict__ invstd,
                                       const float* __restrict__ mask, float* __restrict__ pg,
                                       float* __restrict__ pb, int C, FastDiv hw, long long cnt,
                                       long long chunk) {
    const int c = blockIdx.x, z = blockIdx.y;
    const float mu = mean[c], is = invstd[c];
    const long long beg = z * chunk, end = min(cnt, beg + chunk);
    float sg = 0.f, sb = 0.f;
#pragma unroll 4
    for (long long j = beg + 4 * threadIdx.x; j < end; j += 4 * blockDim.x) {
        const size_t idx = bn_index((uint32_t)j, c, C, hw);
        float4 g = __ldg(reinterpret_cast<const float4*>(dy + idx));
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + idx));
        if (mask) {   // the ReLU backward, fused
            const float4 m = __ldg(reinterpret_cast<const float4*>(mask + idx));
            g.x = m.x > 0.f ? g.x : 0.f; g.y = m.y > 0.f ? g.y : 0.f;
            g.z = m.z > 0.f ? g.z : 0.f; g.w = m.w > 0.f ? g.w : 0.f;
        }
        sg += g.x * (v.x - mu) * is;
        sg += g.y * (v.y - mu) * is;
        sg += g.z * (v.z - mu) * is;
        sg += g.w * (v.w - mu) * is;
        sb += g.x;
        sb += g.y;
        sb += g.z;
        sb += g.w;
    }
    sg = block_sum(sg);
    if (threadIdx.x == 0) pg[(long long)c * gridDim.y + z] = sg;
    sb = block_sum(sb);
    if (threadIdx.x == 0) pb[(long long)c * gridDim.y + z] = sb;
}

__global__ void bn_bwd_finalize_kernel(const float* __restrict__ pg, const float* __restrict__ pb,
                                       int S, float* dgamma, float* dbeta, int C) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float g = 0.f, b = 0.f;
    for (int i = 0; i < S; ++i) {
        g += pg[(long long)c * S + i];
        b += pb[(long long)c * S + i];
    }
    dgamma[c] = g;
    dbeta[c] = b;
}

// dx = gamma*invstd/M * (M*dy - dbeta - xhat*dgamma)   (cpu_backend.ixx:847-892)
template <int V, bool PE = false>   // V and PE as in bn_apply_kernel
__global__ void bn_bwd_apply_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                    const float* __restrict__ mean, const float* __restrict__ invstd,
                                    const float* __restrict__ gamma, const float* __restrict__ dgamma,
                                    const float* __restrict__ dbeta, float* __restrict__ dx,
                                    long long total, int C, int HW, float M,
                                    const float* __restrict__ mask) {
    const long long nv = total / V;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv;
         i += (long long)gridDim.x * blockDim.x) {
        int c;
        if constexpr (V == 4) c = (int)(((unsigned)i * 4u / (unsigned)HW) % (unsigned)C);
        else c = (int)((i / HW) % C);
        const float is = invstd[c], mu = mean[c], k = gamma[c] * is / M, db = dbeta[c],
                    dg = dgamma[c];
        if constexpr (V == 4) {
            float4 g = __ldg(reinterpret_cast<const float4*>(dy) + i);
            if (mask) {
                const float4 m = __ldg(reinterpret_cast<const float4*>(mask) + i);
                g.x = m.x > 0.f ? g.x : 0.f; g.y = m.y > 0.f ? g.y : 0.f;
                g.z = m.z > 0.f ? g.z : 0.f; g.w = m.w > 0.f ? g.w : 0.f;
            }
            const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
            if constexpr (PE) {
                float o[4];
                const float gv[4] = {g.x, g.y, g.z, g.w}, xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int ce = (int)((((unsigned)i * 4u + e) / (unsigned)HW) % (unsigned)C);
                    const float ise = invstd[ce], mue = mean[ce], ke = gamma[ce] * ise / M;
                    o[e] = ke * (M * gv[e] - dbeta[ce] - (xv[e] - mue) * ise * dgamma[ce]);
                }
                reinterpret_cast<float4*>(dx)[i] = make_float4(o[0], o[1], o[2], o[3]);
            } else {
                reinterpret_cast<float4*>(dx)[i] =
                    make_float4(k * (M * g.x - db - (v.x - mu) * is * dg),
                                k * (M * g.y - db - (v.y - mu) * is * dg),
                                k * (M * g.z - db - (v.z - mu) * is * dg),
                                k * (M * g.w - db - (v.w - mu) * is * dg));
            }
        } else {
            const float xh = (x[i] - mu) * is;
            const float g = mask ? (mask[i] > 0.f ? dy[i] : 0.f) : dy[i];
            dx[i] = k * (M * g - db - xh * dg);
        }
    }
}

// ---------------------------------------------------------------- pooling (NCHW)
__global__ void maxpool_kernel(const float* __restrict__ in, float* __restrict__ out,
                               int* __restrict__ idx, int N, int C, int H, int W, int kh, int kw,
                               int sh, int sw, int ph, int pw, int P, int Q) {
    long long total = (long long)N * C * P * Q;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int q = (int)(i % Q);
        long long t = i / Q;
        int p = (int)(t % P);
        long long nc = t / P;
        float m = -1e30f;
        int mi = -1;
        for (int r = 0; r < kh; ++r) {
            int ih = p * sh - ph + r;
            if (ih < 0 || ih >= H) continue;
            for (int s = 0; s < kw; ++s) {
                int iw = q * sw - pw + s;
                if (iw < 0 || iw >= W) continue;
                long long ii = (nc * H + ih) * W + iw;
                float v = in[ii];
                if (v > m) {
                    m = v;
                    mi = (int)ii;
                }
            }
        }
        out[i] = m;
        if (idx) idx[i] = mi;
    }
}

// The 3x3 / stride 2 / padding 1 pool with 32-bit indices (input < 2^31 elements): the nine
// taps are loaded together (clamped addresses, out-of-image taps never win) and scanned in
// the generic kernel's order with its strict '>', so values and argmax indices are the same.
__global__ void maxpool_3s2_kernel(const float* __restrict__ in, float* __restrict__ out,
                                   int* __restrict__ idx, int total, FastDiv fpq, FastDiv fq,
                                   int H, int W, int P, int Q) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int nc = (int)fdiv((uint32_t)i, fpq);
        const int pq = i - nc * (int)fpq.d;
        const int p = (int)fdiv((uint32_t)pq, fq);
        const int q = pq - p * (int)fq.d;
        const int base = nc * H * W;
        float v[9];
        int ii[9];
        bool ok[9];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int s = 0; s < 3; ++s) {
                const int ih = 2 * p - 1 + r, iw = 2 * q - 1 + s;
                const bool in_img = ih >= 0 && ih < H && iw >= 0 && iw < W;
                const int a = base + min(max(ih, 0), H - 1) * W + min(max(iw, 0), W - 1);
                v[r * 3 + s] = __ldg(in + a);
                ii[r * 3 + s] = a;
                ok[r * 3 + s] = in_img;
            }
        float m = -1e30f;
        int mi = -1;
#pragma unroll
        for (int t = 0; t < 9; ++t)
            if (ok[t] && v[t] > m) {
                m = v[t];
                mi = ii[t];
            }
        out[i] = m;
        if (idx) idx[i] = mi;
    }
}

__global__ void maxpool_bwd_kernel(const float* __restrict__ dy, const int* __restrict__ idx,
                                   float* __restrict__ dx, long long nout) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nout;
         i += (long long)gridDim.x * blockDim.x) {
        int s = idx[i];
        if (s >= 0) atomicAdd(&dx[s], dy[i]);
    }
}

// Max-pool backward as a gather: each input element adds the gradients of the output windows
// that picked it (argmax index == its flat index), in increasing output order, from 0. These
// are the sums of the reference CPU backend's sequential scatter loop (cpu_backend.ixx:937-953)
// in its order, so the result is deterministic and the same bits; no atomics, no zeroing.
__global__ void maxpool_bwd_gather_kernel(const float* __restrict__ dy, const int* __restrict__ idx,
                                          float* __restrict__ dx, int total, FastDiv fhw,
                                          FastDiv fw, int kh, int kw, int sh, int sw, int ph,
                                          int pw, int P, int Q) {
    // 32-bit indices (the caller checks N*C*H*W < 2^31): consecutive threads take consecutive
    // w of a row, so their candidate windows' index and gradient reads are close together
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int nc = (int)fdiv((uint32_t)i, fhw);
        const int hw = i - nc * (int)fhw.d;
        const int h = (int)fdiv((uint32_t)hw, fw);
        const int w = hw - h * (int)fw.d;
        // windows p with p*sh - ph <= h <= p*sh - ph + kh - 1, likewise q
        const int a = h + ph - kh + 1, b = w + pw - kw + 1;
        const int p0 = a <= 0 ? 0 : (a + sh - 1) / sh, p1 = min(P - 1, (h + ph) / sh);
        const int q0 = b <= 0 ? 0 : (b + sw - 1) / sw, q1 = min(Q - 1, (w + pw) / sw);
        const int* ip = idx + nc * P * Q;
        const float* gp = dy + nc * P * Q;
        float acc = 0.f;
        for (int p = p0; p <= p1; ++p)
            for (int q = q0; q <= q1; ++q) {
                const int o = p * Q + q;
                if (__ldg(ip + o) == i) acc += __ldg(gp + o);
            }
        dx[i] = acc;
    }
}

// The 3x3 / stride 2 / padding 1 pool (the ResNet stem's): a thread takes the 2x2 input block
// (2r.., 2s..). Every pixel of it lies in window (r, s); the odd row also in (r + 1, s), the
// odd column also in (r, s + 1), the odd corner in all four. The four windows' argmax indices
// and gradients are read once, and each pixel adds its matches in output order (r, s),
// (r, s + 1), (r + 1, s), (r + 1, s + 1), as the generic kernel and the CPU loop do.
__global__ void maxpool_bwd_gather_3s2_kernel(const float* __restrict__ dy,
                                              const int* __restrict__ idx, float* __restrict__ dx,
                                              int blocks, FastDiv frs, FastDiv fs2, int H, int W,
                                              int P, int Q) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < blocks; t += gridDim.x * blockDim.x) {
        const int nc = (int)fdiv((uint32_t)t, frs);
        const int rem = t - nc * (int)frs.d;
        const int r = (int)fdiv((uint32_t)rem, fs2);
        const int s = rem - r * (int)fs2.d;
        const int base_o = nc * P * Q;
        int iv[4] = {-1, -1, -1, -1};
        float gv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int p = r + (k >> 1), q = s + (k & 1);
            if (p < P && q < Q) {
                iv[k] = __ldg(idx + base_o + p * Q + q);
                gv[k] = __ldg(dy + base_o + p * Q + q);
            }
        }
        const int base_i = nc * H * W;
#pragma unroll
        for (int dh = 0; dh < 2; ++dh) {
            const int h = 2 * r + dh;
            if (h >= H) continue;
#pragma unroll
            for (int dw = 0; dw < 2; ++dw) {
                const int w = 2 * s + dw;
                if (w >= W) continue;
                const int pix = base_i + h * W + w;
                float acc = 0.f;
                if (iv[0] == pix) acc += gv[0];
                if (dw && iv[1] == pix) acc += gv[1];
                if (dh && iv[2] == pix) acc += gv[2];
                if (dh && dw && iv[3] == pix) acc += gv[3];
                dx[pix] = acc;
            }
        }
    }
}

__global__ void avgpool_kernel(const float* __restrict__ in, float* __restrict__ out, int N, int C,
                               int H, int W, int kh, int kw, int sh, int sw, int ph, int pw, int P,
                               int Q) {
    long long total = (long long)N * C * P * Q;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int q = (int)(i % Q);
        long long t = i / Q;
        int p = (int)(t % P);
        long long nc = t / P;
        float s = 0.f;
        for (int r = 0; r < kh; ++r) {
            int ih = p * sh - ph + r;
            if (ih < 0 || ih >= H) continue;
            for (int u = 0; u < kw; ++u) {
                int iw = q * sw - pw + u;
                if (iw >= 0 && iw < W) s += in[(nc * H + ih) * W + iw];
            }
        }
        out[i] = s / (float)(kh * kw);
    }
}

__global__ void avgpool_bwd_kernel(const float* __restrict__ dy, float* __restrict__ dx, int N,
                                   int C, int H, int W, int kh, int kw, int sh, int sw, int ph,
                                   int pw, int P, int Q) {
    long long total = (long long)N * C * P * Q;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int q = (int)(i % Q);
        long long t = i / Q;
        int p = (int)(t % P);
        long long nc = t / P;
        float g = dy[i] / (float)(kh * kw);
        for (int r = 0; r < kh; ++r) {
            int ih = p * sh - ph + r;
            if (ih < 0 || ih >= H) continue;
            for (int u = 0; u < kw; ++u) {
                int iw = q * sw - pw + u;
                if (iw >= 0 && iw < W) atomicAdd(&dx[(nc * H + ih) * W + iw], g);
            }
        }
    }
}

__global__ void adaptive_avgpool_kernel(const float* __restrict__ in, float* __restrict__ out,
                                        int N, int C, int H, int W, int OH, int OW) {
    // one warp per output element: the window can be the whole plane (global pooling)
    long long total = (long long)N * C * OH * OW;
    long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    int lane = threadIdx.x & 31;
    for (long long i = warp; i < total; i += nwarps) {
        int ow = (int)(i % OW);
        long long t = i / OW;
        int oh = (int)(t % OH);
        long long nc = t / OH;
        int h0 = oh * H / OH, h1 = (oh + 1) * H / OH, w0 = ow * W / OW, w1 = (ow + 1) * W / OW;
        int wn = w1 - w0, cnt = (h1 - h0) * wn;
        float s = 0.f;
        for (int j = lane; j < cnt; j += 32) {
            int ih = h0 + j / wn, iw = w0 + j % wn;
            s += in[(nc * H + ih) * W + iw];
        }
        s = warp_sum(s);
        if (lane == 0) out[i] = s / (float)cnt;
    }
}

__global__ void adaptive_avgpool_bwd_kernel(const float* __restrict__ dy, float* __restrict__ dx,
                                            int N, int C, int H, int W, int OH, int OW) {
    long long total = (long long)N * C * H * W;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int w = (int)(i % W);
        long long t = i / W;
        int h = (int)(t % H);
        long long nc = t / H;
        float g = 0.f;
        for (int oh = 0; oh < OH; ++oh) {
            int h0 = oh * H / OH, h1 = (oh + 1) * H / OH;
            if (h < h0 || h >= h1) continue;
            for (int ow = 0; ow < OW; ++ow) {
                int w0 = ow * W / OW, w1 = (ow + 1) * W / OW;
                if (w < w0 || w >= w1) continue;
                g += dy[(nc * OH + oh) * OW + ow] / (float)((h1 - h0) * (w1 - w0));
            }
        }
        dx[i] = g;
    }
}

// ---------------------------------------------------------------- softmax / CE
__global__ void softmax_kernel(const float* __restrict__ in, float* __restrict__ out, int N, int C) {
    long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= N) return;
    const float* x = in + warp * C;
    float* y = out + warp * C;
    float m = -INFINITY;
    for (int j = lane; j < C; j += 32) m = fmaxf(m, x[j]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int j = lane; j < C; j += 32) s += expf(x[j] - m);
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.f / s;
    for (int j = lane; j < C; j += 32) y[j] = expf(x[j] - m) * inv;
}

__global__ void cross_entropy_kernel(const float* __restrict__ p, const float* __restrict__ t,
                                     float* __restrict__ result, long long n, int N) {
    float s = 0.f;
    for (long long i = threadIdx.x; i < n; i += blockDim.x)
        if (t[i] > 0.5f) s -= logf(fmaxf(p[i], 1e-7f));
    s = block_sum(s);
    if (threadIdx.x == 0) *result = s / (float)N;
}

__global__ void ce_softmax_bwd_kernel(const float* __restrict__ p, const float* __restrict__ t,
                                      float* __restrict__ g, long long n, float scale) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        g[i] = (p[i] - t[i]) * scale;
}

// Softmax, cross-entropy and its gradient in one pass over the logits (the three reference
// kernels cuda_kernels.cu:1387, :3934 and :2539 with the CPU backend's semantics: divide by the
// sum, loss = -sum over targets > 0.5 of log(max(p, 1e-7)) / N, grad = (p - t) / N). One warp
// per row, 8 rows per block; each block adds its rows' losses in row order into a per-block
// partial, and the last block to finish adds the partials in block order (deterministic).
namespace sce {
constexpr int kRows = 8;
constexpr int kMaxBlocks = 8192;   // 65536 rows
__device__ float g_part[kMaxBlocks];
__device__ unsigned int g_ticket;  // zero between calls: the last block resets it
}  // namespace sce

__global__ void __launch_bounds__(256) softmax_ce_fused_kernel(
    const float* __restrict__ x, const float* __restrict__ t, float* __restrict__ prob,
    float* __restrict__ grad, float* __restrict__ loss, int N, int C, float invN) {
    __shared__ float rowloss[sce::kRows];
    __shared__ int is_last;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * sce::kRows + w;
    float rl = 0.f;
    if (row < N) {
        const float* xr = x + row * C;
        const float* tr = t + row * C;
        float m = -INFINITY;
        for (int j = lane; j < C; j += 32) m = fmaxf(m, xr[j]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float s = 0.f;
        for (int j = lane; j < C; j += 32) s += expf(xr[j] - m);
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float inv = 1.f / s;
        for (int j = lane; j < C; j += 32) {
            const float p = expf(xr[j] - m) * inv;
            const float tj = tr[j];
            if (prob) prob[row * C + j] = p;
            grad[row * C + j] = (p - tj) * invN;
            if (tj > 0.5f) rl -= logf(fmaxf(p, 1e-7f));
        }
        for (int o = 16; o; o >>= 1) rl += __shfl_xor_sync(0xffffffffu, rl, o);
    }
    if (lane == 0) rowloss[w] = rl;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = 0.f;
        for (int i = 0; i < sce::kRows; ++i) b += rowloss[i];
        sce::g_part[blockIdx.x] = b;
        __threadfence();
        is_last = atomicAdd(&sce::g_ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last && w == 0) {
        __threadfence();
        float v = 0.f;
        for (int b = lane; b < (int)gridDim.x; b += 32) v += __ldcg(&sce::g_part[b]);
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) {
            *loss = v * invN;
            sce::g_ticket = 0;
        }
    }
}

// ---------------------------------------------------------------- optimiser, elementwise
// status (nullable): the gradient guard's verdict; status[1] == 0 skips the step
// gs scales the gradient first (1/world after a summing all-reduce; exactly 1 otherwise)
__global__ void sgd_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ v,
                           long long n, float lr, float mom, const float* __restrict__ status,
                           float gs = 1.f) {
    if (status && status[1] == 0.f) return;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float gi = gs == 1.f ? g[i] : gs * g[i];
        if (v) {
            float nv = mom * v[i] + gi;
            v[i] = nv;
            p[i] -= lr * nv;
        } else {
            p[i] -= lr * gi;
        }
    }
}

template <class F>
__global__ void map_kernel(long long n, F f) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        f(i);
}

// y[i] = f(a[i], b[i]) (b absent: f(a[i], a[i])) in vectors of 4 floats, then the n % 4 tail.
// The pointers are 16-byte aligned; y may be a or b (in place), so no restrict or
// read-only-cache loads.
template <class F>
__global__ void zip_kernel(const float* a, const float* b, float* y, long long n, F f) {
    const long long n4 = n >> 2;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    float4* y4 = reinterpret_cast<float4*>(y);
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    for (long long i = t; i < n4; i += stride) {
        const float4 u = a4[i];
        const float4 v = b ? b4[i] : u;
        y4[i] = make_float4(f(u.x, v.x), f(u.y, v.y), f(u.z, v.z), f(u.w, v.w));
    }
    for (long long i = (n4 << 2) + t; i < n; i += stride) y[i] = f(a[i], b ? b[i] : a[i]);
}

__global__ void sum_kernel(const float* __restrict__ x, float* __restrict__ out, long long n) {
    float s = 0.f;
    for (long long i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
    s = block_sum(s);
    if (threadIdx.x == 0) *out = s;
}

__global__ void argmax_kernel(const float* __restrict__ x, int* __restrict__ out, int N, int C) {
    long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= N) return;
    const float* r = x + warp * C;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = lane; j < C; j += 32)
        if (r[j] > best) { best = r[j]; bi = j; }
    for (int o = 16; o; o >>= 1) {
        float ob = __shfl_xor_sync(0xffffffffu, best, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) out[warp] = bi == 0x7fffffff ? 0 : bi;
}

__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out, int R, int C) {
    __shared__ float tile[32][33];
    int x = blockIdx.x * 32 + threadIdx.x, y = blockIdx.y * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (x < C && y + j < R) tile[threadIdx.y + j][threadIdx.x] = in[(long long)(y + j) * C + x];
    __syncthreads();
    x = blockIdx.y * 32 + threadIdx.x;
    y = blockIdx.x * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (x < R && y + j < C) out[(long long)(y + j) * R + x] = tile[threadIdx.x][threadIdx.y + j];
}

__global__ void bias_grad_kernel(const float* __restrict__ dy, float* __restrict__ db, int N, int C,
                                 FastDiv hw) {
    const int c = blockIdx.x;
    const long long cnt = (long long)N * hw.d;
    float s = 0.f;
#pragma unroll 8
    for (long long j = threadIdx.x; j < cnt; j += blockDim.x) s += __ldg(dy + bn_index((uint32_t)j, c, C, hw));
    s = block_sum(s);
    if (threadIdx.x == 0) db[c] = s;
}

// Reduction blocks per channel for the BN statistics: >= 4 blocks per SM overall, each split
// covering at least 4096 elements, at most 64.
static int bn_splits(DeviceCtx* c, int C, long long cnt) {
    long long want = (4LL * c->num_sms + C - 1) / C;
    long long maxs = cnt / 4096 > 0 ? cnt / 4096 : 1;
    long long s = want < maxs ? want : maxs;
    if (s > 64) s = 64;
    return s < 1 ? 1 : (int)s;
}
static bool aligned16f(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
// 4-float vectors for the elementwise BN kernels: whole vectors share a channel, every pointer is
// 16-byte aligned and the 32-bit vector index math holds
// 4-float vectors that may span channels (the kernels' PE form): whole vectors, aligned pointers
static bool bn_vec_any(long long total, const void* a, const void* b, const void* d = nullptr) {
    return total % 4 == 0 && aligned16f(a) && aligned16f(b) && (!d || aligned16f(d)) &&
           total < (1LL << 32);
}
static bool bn_vec_flat(int HW, long long total, const void* a, const void* b,
                        const void* d = nullptr) {
    return HW % 4 == 0 && aligned16f(a) && aligned16f(b) && (!d || aligned16f(d)) &&
           total < (1LL << 32);
}

// The BN training statistics of x into part (sums) and part + C*S (centred squares).
static int bn_stats(DeviceCtx* c, const float* x, float* part, int N, int C, int HW, int S) {
    const long long cnt = (long long)N * HW;
    const long long chunk = (cnt + S - 1) / S;
    const FastDiv hw = make_fastdiv((uint32_t)HW);
    const dim3 grid(C, S);
    bn_partial_sum_kernel<<<grid, 256, 0, c->compute>>>(x, part, C, hw, cnt, chunk);
    int st = after_launch(c);
    if (st != OM_OK) return st;
    bn_partial_m2_kernel<<<grid, 256, 0, c->compute>>>(x, part, part + (long long)C * S, C, hw, cnt,
                                                       chunk);
    return after_launch(c);
}
static int bn_apply(DeviceCtx* c, const float* x, float* y, const float* gamma, const float* beta,
                    const float* mean, const float* invstd, long long total, int C, int HW,
                    int relu = 0, const float* res = nullptr) {
    if (bn_vec_flat(HW, total, x, y, res))
        bn_apply_kernel<4><<<ew_grid(c, total / 4, 256), 256, 0, c->compute>>>(
            x, y, gamma, beta, mean, invstd, total, C, HW, relu, res);
    else if (bn_vec_any(total, x, y, res))
        bn_apply_kernel<4, true><<<ew_grid(c, total / 4, 256), 256, 0, c->compute>>>(
            x, y, gamma, beta, mean, invstd, total, C, HW, relu, res);
    else
        bn_apply_kernel<1><<<ew_grid(c, total, 256), 256, 0, c->compute>>>(
            x, y, gamma, beta, mean, invstd, total, C, HW, relu, res);
    return after_launch(c);
}

// BatchNorm statistics from a convolution's per-group partials (the 3xTF32 conv epilogue with
// bn_part): for channel c, G groups of 32 output pixels (the last one holds cnt - 32 (G - 1)),
// each with its mean m_g and sum of squared deviations q_g. The channel's mean is
// sum n_g m_g / cnt and its sum of squared deviations sum (q_g + n_g (m_g - mean)^2) (the
// parallel form of the two-pass variance, exact in real arithmetic), each summed in a fixed
// order: thread t takes groups t, t + 256, ..., then the 256 partial sums are added pairwise
// down a tree. Then, as bn_finalize_kernel: biased variance, running statistics with momentum,
// saved mean and 1/sqrt(var + eps). One block per channel.
__device__ __forceinline__ float bn_tree_sum(float v, float* sh) {
    sh[threadIdx.x] = v;
    __syncthreads();
    for (int h = 128; h >= 1; h >>= 1) {
        if ((int)threadIdx.x < h) sh[threadIdx.x] += sh[threadIdx.x + h];
        __syncthreads();
    }
    const float r = sh[0];
    __syncthreads();
    return r;
}
__global__ void __launch_bounds__(256) bn_chan_finalize_kernel(
    const float* __restrict__ part, int G, long long cnt, int C, float* run_mean, float* run_var,
    float* saved_mean, float* saved_invstd, float eps, float momentum) {
    const int c = blockIdx.x;
    const float* pm = part + (size_t)c * G;
    const float* pq = part + ((size_t)C + c) * G;
    __shared__ float sh[256];
    // every group holds 32 pixels except possibly the last
    const float n_last = (float)(cnt - 32LL * (G - 1));
    float s = 0.f;
    for (int g = threadIdx.x; g < G; g += 256) s += (g == G - 1 ? n_last : 32.f) * pm[g];
    const float mean = bn_tree_sum(s, sh) / (float)cnt;
    float q = 0.f;
    for (int g = threadIdx.x; g < G; g += 256) {
        const float d = pm[g] - mean;
        q += pq[g] + (g == G - 1 ? n_last : 32.f) * d * d;
    }
    const float m2 = bn_tree_sum(q, sh);
    if (threadIdx.x == 0) {
        const float var = m2 / (float)cnt;
        run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mean;
        run_var[c] = (1.f - momentum) * run_var[c] + momentum * var;
        saved_mean[c] = mean;
        saved_invstd[c] = 1.f / sqrtf(var + eps);
    }
}

}  // namespace ops
}  // namespace omb

using namespace omb;
using namespace omb::ops;

#define OMB_EW(n) ew_grid(c, (n), 256), 256, 0, c->compute

// Elementwise y = f(a, b) over n floats: float4 vectors when every pointer is 16-byte aligned,
// else one float per thread.
template <class F>
static int zip(DeviceCtx* c, const float* a, const float* b, float* y, long long n, F f) {
    const bool vec = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                       reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    if (vec)
        zip_kernel<<<ew_grid(c, (n + 3) / 4, 256), 256, 0, c->compute>>>(a, b, y, n, f);
    else
        map_kernel<<<OMB_EW(n)>>>(n, [=] __device__(long long i) { y[i] = f(a[i], b ? b[i] : a[i]); });
    return after_launch(c);
}

// BatchNorm forward, with the ReLU of the result applied in the same pass when relu = 1.
static int bn_forward(const float* pInput, float* pOutput, const float* pGamma, const float* pBeta,
                      float* pRunMean, float* pRunVar, float* pSavedMean, float* pSavedInvStd,
                      int nBatch, int nChannels, int nH, int nW, float fEps, float fMomentum,
                      int bTraining, int relu) {
    OMB_CTX_OR_FAIL(c);
    if (!pInput || !pOutput || !pGamma || !pBeta || !pRunMean || !pRunVar || !pSavedMean ||
        !pSavedInvStd || nBatch <= 0 || nChannels <= 0 || nH <= 0 || nW <= 0)
        return OM_ERR_INVALID;
    const int HW = nH * nW;
    const long long cnt = (long long)nBatch * HW;
    if (cnt >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    int S = 1;
    float* scratch = nullptr;
    if (bTraining) {
        S = bn_splits(c, nChannels, cnt);
        OMB_CHECK(cudaMallocAsync(&scratch, sizeof(float) * 2 * nChannels * S, c->compute));
        const int st = bn_stats(c, pInput, scratch, nBatch, nChannels, HW, S);
        if (st != OM_OK) {
            cudaFreeAsync(scratch, c->compute);
            return st;
        }
    }
    bn_finalize_kernel<<<(nChannels + 127) / 128, 128, 0, c->compute>>>(
        scratch, scratch ? scratch + (long long)nChannels * S : nullptr, S, cnt, pRunMean, pRunVar,
        pSavedMean, pSavedInvStd, fEps, fMomentum, bTraining, nChannels);
    int st = after_launch(c);
    if (scratch) cudaFreeAsync(scratch, c->compute);
    if (st != OM_OK) return st;
    return bn_apply(c, pInput, pOutput, pGamma, pBeta, pSavedMean, pSavedInvStd,
                    cnt * nChannels, nChannels, HW, relu);
}

// BatchNorm backward; with pMask (the ReLU output of a fused forward), the incoming gradient
// first goes through the ReLU backward (zero where pMask <= 0), in the same passes.
static int bn_backward(const float* pGradOutput, const float* pInput, const float* pMean,
                       const float* pInvStd, const float* pGamma, const float* pMask,
                       float* pGradInput, float* pGradGamma, float* pGradBeta, int nBatch,
                       int nChannels, int nH, int nW) {
    OMB_CTX_OR_FAIL(c);
    if (!pGradOutput || !pInput || !pMean || !pInvStd || !pGamma || !pGradInput || !pGradGamma ||
        !pGradBeta || nBatch <= 0 || nChannels <= 0 || nH <= 0 || nW <= 0)
        return OM_ERR_INVALID;
    const int HW = nH * nW;
    const long long cnt = (long long)nBatch * HW;
    if (cnt >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    const int S = bn_splits(c, nChannels, cnt);
    float* scratch = nullptr;
    OMB_CHECK(cudaMallocAsync(&scratch, sizeof(float) * 2 * nChannels * S, c->compute));
    const long long chunk = (cnt + S - 1) / S;
    if (HW % 4 == 0 && aligned16f(pGradOutput) && aligned16f(pInput) &&
        (!pMask || aligned16f(pMask)))
        bn_bwd_partial4_kernel<<<dim3(nChannels, S), 256, 0, c->compute>>>(
            pGradOutput, pInput, pMean, pInvStd, pMask, scratch,
            scratch + (long long)nChannels * S, nChannels, make_fastdiv((uint32_t)HW), cnt,
            (chunk + 3) / 4 * 4);
    else
        bn_bwd_partial_kernel<<<dim3(nChannels, S), 256, 0, c->compute>>>(
            pGradOutput, pInput, pMean, pInvStd, pMask, scratch,
            scratch + (long long)nChannels * S, nChannels, make_fastdiv((uint32_t)HW), cnt, chunk);
    int st = after_launch(c);
    if (st == OM_OK) {
        bn_bwd_finalize_kernel<<<(nChannels + 127) / 128, 128, 0, c->compute>>>(
            scratch, scratch + (long long)nChannels * S, S, pGradGamma, pGradBeta, nChannels);
        st = after_launch(c);
    }
    cudaFreeAsync(scratch, c->compute);
    if (st != OM_OK) return st;
    const long long total = cnt * nChannels;
    if (bn_vec_flat(HW, total, pGradOutput, pInput, pGradInput) && (!pMask || aligned16f(pMask)))
        bn_bwd_apply_kernel<4><<<ew_grid(c, total / 4, 256), 256, 0, c->compute>>>(
            pGradOutput, pInput, pMean, pInvStd, pGamma, pGradGamma, pGradBeta, pGradInput, total,
            nChannels, HW, (float)cnt, pMask);
    else if (bn_vec_any(total, pGradOutput, pInput, pGradInput) && (!pMask || aligned16f(pMask)))
        bn_bwd_apply_kernel<4, true><<<ew_grid(c, total / 4, 256), 256, 0, c->compute>>>(
            pGradOutput, pInput, pMean, pInvStd, pGamma, pGradGamma, pGradBeta, pGradInput, total,
            nChannels, HW, (float)cnt, pMask);
    else
        bn_bwd_apply_kernel<1><<<OMB_EW(total)>>>(pGradOutput, pInput, pMean, pInvStd, pGamma,
                                                  pGradGamma, pGradBeta, pGradInput, total,
                                                  nChannels, HW, (float)cnt, pMask);
    return after_launch(c);
}

extern "C" int omCudaBatchNorm2d(const float* pInput, float* pOutput, const float* pGamma,
                                 const float* pBeta, float* pRunMean, float* pRunVar,
                                 float* pSavedMean, float* pSavedInvStd, int nBatch, int nChannels,
                                 int nH, int nW, float fEps, float fMomentum, int bTraining) {
    return bn_forward(pInput, pOutput, pGamma, pBeta, pRunMean, pRunVar, pSavedMean, pSavedInvStd,
                      nBatch, nChannels, nH, nW, fEps, fMomentum, bTraining, 0);
}

extern "C" int omCudaBatchNorm2dBackward(const float* pGradOutput, const float* pInput,
                                         const float* pMean, const float* pInvStd,
                                         const float* pGamma, float* pGradInput, float* pGradGamma,
                                         float* pGradBeta, int nBatch, int nChannels, int nH,
                                         int nW, float fEps) {
    (void)fEps;
    return bn_backward(pGradOutput, pInput, pMean, pInvStd, pGamma, nullptr, pGradInput,
                       pGradGamma, pGradBeta, nBatch, nChannels, nH, nW);
}

extern "C" int omCudaBatchNorm2dAct(const float* pInput, float* pOutput, const float* pGamma,
                                    const float* pBeta, float* pRunMean, float* pRunVar,
                                    float* pSavedMean, float* pSavedInvStd, int nBatch,
                                    int nChannels, int nH, int nW, float fEps, float fMomentum,
                                    int bTraining, int nAct) {
    if (nAct != OM_ACT_NONE && nAct != OM_ACT_RELU) return OM_ERR_UNSUPPORTED;
    return bn_forward(pInput, pOutput, pGamma, pBeta, pRunMean, pRunVar, pSavedMean, pSavedInvStd,
                      nBatch, nChannels, nH, nW, fEps, fMomentum, bTraining,
                      nAct == OM_ACT_RELU ? 1 : 0);
}

// Train-mode conv -> BatchNorm (-> ReLU) with the statistics taken in the conv's epilogue: the
// conv output is written once and read once (by the normalisation), instead of three times
// (two statistics passes and the normalisation).
// s2d: the convolution in its space-to-depth form (tf32_conv_s2d; stride-2 shapes of at most 8
// input channels only), pInputSplit then receiving that form's copy. pResidual (optional): added
// to the normalised output before the activation.
static int conv_bn_act(const float* pInput, const float* pWeight, const float* pBias,
                       float* pConvOut, float* pOutput, const float* pGamma, const float* pBeta,
                       float* pRunMean, float* pRunVar, float* pSavedMean, float* pSavedInvStd,
                       int nBatch, int nCin, int nH, int nW, int nCout, int nKH, int nKW,
                       int nStride, int nPad, float fEps, float fMomentum, int nAct,
                       void* pInputSplit, bool s2d, const float* pResidual = nullptr) {
    OMB_CTX_OR_FAIL(c);
    if (!pInput || !pWeight || !pConvOut || !pOutput || !pGamma || !pBeta || !pRunMean ||
        !pRunVar || !pSavedMean || !pSavedInvStd || nBatch <= 0 || nCin <= 0 || nCout <= 0 ||
        nStride <= 0 || nPad < 0)
        return OM_ERR_INVALID;
    if (nAct != OM_ACT_NONE && nAct != OM_ACT_RELU) return OM_ERR_UNSUPPORTED;
    const int P = (nH + 2 * nPad - nKH) / nStride + 1, Q = (nW + 2 * nPad - nKW) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    const long long cnt = (long long)nBatch * P * Q;
    if (cnt >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    if (s2d && omb::tc::s2d_split_half_bytes(nBatch, nCin, nH, nW, nKH, nKW, nStride, nPad) == 0)
        return OM_ERR_UNSUPPORTED;
    const long long G = (cnt + 31) / 32;
    float* part = nullptr;
    OMB_CHECK(cudaMallocAsync(&part, sizeof(float) * 2 * (size_t)nCout * G, c->compute));
    // the input's tensor-core copy is kept in pInputSplit for the weight gradient when the
    // caller gave one (omCudaConvInputSplitBytes / omCudaStemInputSplitBytes say whether the
    // weight gradient reads it)
    float* keep = static_cast<float*>(pInputSplit);
    if (keep && !s2d && !omb::tc::wgrad_reads_kept_split(nCin, nStride)) keep = nullptr;
    int st = s2d ? omb::tc::tf32_conv_s2d(c, pInput, nBatch, nCin, nH, nW, pWeight, nCout, nKH,
                                          nKW, nStride, nPad, pBias, pConvOut, part, keep)
                 : omb::tc::tf32_conv(c, pInput, nBatch, nCin, nH, nW, nH, nW, 0, 0, 1, pWeight,
                                      nCout, nKH, nKW, false, nCin, pBias, pConvOut, nStride,
                                      nPad, 1, 0, 0, part, keep);
    if (st == OM_OK) {
        bn_chan_finalize_kernel<<<nCout, 256, 0, c->compute>>>(part, (int)G, cnt, nCout,
                                                               pRunMean, pRunVar, pSavedMean,
                                                               pSavedInvStd, fEps, fMomentum);
        st = after_launch(c);
    }
    cudaFreeAsync(part, c->compute);
    if (st == OM_ERR_UNSUPPORTED || st == OM_ERR_OOM) {
        // the tensor path did not take the shape: the conv and the BatchNorm separately, and the
        // kept copy written on its own
        st = omCudaConv2d(pInput, pWeight, pBias, pConvOut, nBatch, nCin, nH, nW, nCout, nKH, nKW,
                          nStride, nPad);
        if (st != OM_OK) return st;
        if (keep) {
            st = s2d ? omb::tc::tf32_s2d_split_input(c, pInput, nBatch, nCin, nH, nW, nKH, nKW,
                                                     nStride, nPad, keep)
                     : omb::tc::tf32_split_input(c, pInput, nBatch, nCin, nH, nW, keep);
            if (st != OM_OK) return st;
        }
        if (!pResidual)
            return omCudaBatchNorm2dAct(pConvOut, pOutput, pGamma, pBeta, pRunMean, pRunVar,
                                        pSavedMean, pSavedInvStd, nBatch, nCout, P, Q, fEps,
                                        fMomentum, 1, nAct);
        st = omCudaBatchNorm2dAct(pConvOut, pOutput, pGamma, pBeta, pRunMean, pRunVar, pSavedMean,
                                  pSavedInvStd, nBatch, nCout, P, Q, fEps, fMomentum, 1,
                                  OM_ACT_NONE);
        if (st == OM_OK) st = omCudaAdd(pOutput, pResidual, pOutput, (int)(cnt * nCout));
        if (st == OM_OK && nAct == OM_ACT_RELU)
            st = omCudaReLU(pOutput, pOutput, (int)(cnt * nCout));
        return st;
    }
    if (st != OM_OK) return st;
    return bn_apply(c, pConvOut, pOutput, pGamma, pBeta, pSavedMean, pSavedInvStd,
                    cnt * nCout, nCout, P * Q, nAct == OM_ACT_RELU ? 1 : 0, pResidual);
}

extern "C" int omCudaConv2dBatchNorm2dAct(const float* pInput, const float* pWeight,
                                          const float* pBias, float* pConvOut, float* pOutput,
                                          const float* pGamma, const float* pBeta,
                                          float* pRunMean, float* pRunVar, float* pSavedMean,
                                          float* pSavedInvStd, int nBatch, int nCin, int nH,
                                          int nW, int nCout, int nKH, int nKW, int nStride,
                                          int nPad, float fEps, float fMomentum, int nAct,
                                          void* pInputSplit) {
    return conv_bn_act(pInput, pWeight, pBias, pConvOut, pOutput, pGamma, pBeta, pRunMean,
                       pRunVar, pSavedMean, pSavedInvStd, nBatch, nCin, nH, nW, nCout, nKH, nKW,
                       nStride, nPad, fEps, fMomentum, nAct, pInputSplit, false);
}

extern "C" int omCudaConv2dBatchNorm2dAddAct(const float* pInput, const float* pWeight,
                                             const float* pBias, float* pConvOut, float* pOutput,
                                             const float* pGamma, const float* pBeta,
                                             float* pRunMean, float* pRunVar, float* pSavedMean,
                                             float* pSavedInvStd, int nBatch, int nCin, int nH,
                                             int nW, int nCout, int nKH, int nKW, int nStride,
                                             int nPad, float fEps, float fMomentum, int nAct,
                                             void* pInputSplit, const float* pResidual) {
    if (!pResidual || nStride <= 0) return OM_ERR_INVALID;
    if ((long long)nBatch * nCout * ((nH + 2 * nPad - nKH) / nStride + 1) *
            ((nW + 2 * nPad - nKW) / nStride + 1) >= (1LL << 31))
        return OM_ERR_UNSUPPORTED;   // the fallback's elementwise ops take int counts
    return conv_bn_act(pInput, pWeight, pBias, pConvOut, pOutput, pGamma, pBeta, pRunMean,
                       pRunVar, pSavedMean, pSavedInvStd, nBatch, nCin, nH, nW, nCout, nKH, nKW,
                       nStride, nPad, fEps, fMomentum, nAct, pInputSplit, false, pResidual);
}

extern "C" int omCudaStemConv2dBatchNorm2dAct(const float* pInput, const float* pWeight,
                                              const float* pBias, float* pConvOut,
                                              float* pOutput, const float* pGamma,
                                              const float* pBeta, float* pRunMean,
                                              float* pRunVar, float* pSavedMean,
                                              float* pSavedInvStd, int nBatch, int nCin, int nH,
                                              int nW, int nCout, int nKH, int nKW, int nStride,
                                              int nPad, float fEps, float fMomentum, int nAct,
                                              void* pInputSplit) {
    return conv_bn_act(pInput, pWeight, pBias, pConvOut, pOutput, pGamma, pBeta, pRunMean,
                       pRunVar, pSavedMean, pSavedInvStd, nBatch, nCin, nH, nW, nCout, nKH, nKW,
                       nStride, nPad, fEps, fMomentum, nAct, pInputSplit, true);
}

extern "C" int omCudaBatchNorm2dBackwardAct(const float* pGradOutput, const float* pInput,
                                            const float* pMean, const float* pInvStd,
                                            const float* pGamma, const float* pOutput,
                                            float* pGradInput, float* pGradGamma,
                                            float* pGradBeta, int nBatch, int nChannels, int nH,
                                            int nW, float fEps, int nAct) {
    (void)fEps;
    if (nAct != OM_ACT_NONE && nAct != OM_ACT_RELU) return OM_ERR_UNSUPPORTED;
    if (nAct == OM_ACT_RELU && !pOutput) return OM_ERR_INVALID;
    return bn_backward(pGradOutput, pInput, pMean, pInvStd, pGamma,
                       nAct == OM_ACT_RELU ? pOutput : nullptr, pGradInput, pGradGamma, pGradBeta,
                       nBatch, nChannels, nH, nW);
}

extern "C" int omCudaMaxPool2d(const float* pIn, float* pOut, int* pIndices, int nN, int nC,
                               int nH, int nW, int nKH, int nKW, int nSH, int nSW, int nPH,
                               int nPW) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nSH <= 0 || nSW <= 0) return OM_ERR_INVALID;
    int P = (nH + 2 * nPH - nKH) / nSH + 1, Q = (nW + 2 * nPW - nKW) / nSW + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    if ((long long)nN * nC * nH * nW >= (1LL << 31)) return OM_ERR_UNSUPPORTED;  // int32 indices
    long long total = (long long)nN * nC * P * Q;
    if (nKH == 3 && nKW == 3 && nSH == 2 && nSW == 2 && nPH == 1 && nPW == 1)
        maxpool_3s2_kernel<<<OMB_EW(total)>>>(pIn, pOut, pIndices, (int)total,
                                              make_fastdiv((uint32_t)(P * Q)),
                                              make_fastdiv((uint32_t)Q), nH, nW, P, Q);
    else
        maxpool_kernel<<<OMB_EW(total)>>>(pIn, pOut, pIndices, nN, nC, nH, nW, nKH, nKW, nSH, nSW,
                                          nPH, nPW, P, Q);
    return after_launch(c);
}

extern "C" int omCudaMaxPool2dBackward(const float* pGradOut, const int* pIndices, float* pGradIn,
                                       int nN, int nC, int nH, int nW, int nHout, int nWout) {
    (void)nH; (void)nW;
    OMB_CTX_OR_FAIL(c);
    if (!pGradOut || !pIndices || !pGradIn) return OM_ERR_INVALID;
    long long n = (long long)nN * nC * nHout * nWout;
    maxpool_bwd_kernel<<<OMB_EW(n)>>>(pGradOut, pIndices, pGradIn, n);
    return after_launch(c);
}

extern "C" int omCudaMaxPool2dBackwardGather(const float* pGradOut, const int* pIndices,
                                             float* pGradIn, int nN, int nC, int nH, int nW,
                                             int nKH, int nKW, int nSH, int nSW, int nPH,
                                             int nPW) {
    OMB_CTX_OR_FAIL(c);
    if (!pGradOut || !pIndices || !pGradIn || nSH <= 0 || nSW <= 0 || nKH <= 0 || nKW <= 0)
        return OM_ERR_INVALID;
    const int P = (nH + 2 * nPH - nKH) / nSH + 1, Q = (nW + 2 * nPW - nKW) / nSW + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    const long long total = (long long)nN * nC * nH * nW;
    if (total >= (1LL << 31)) return OM_ERR_UNSUPPORTED;   // int32 indices
    const FastDiv fhw = make_fastdiv((uint32_t)(nH * nW)), fw = make_fastdiv((uint32_t)nW);
    if (nKH == 3 && nKW == 3 && nSH == 2 && nSW == 2 && nPH == 1 && nPW == 1) {
        const int R2 = (nH + 1) / 2, S2 = (nW + 1) / 2;
        const long long blocks = (long long)nN * nC * R2 * S2;
        maxpool_bwd_gather_3s2_kernel<<<OMB_EW(blocks)>>>(
            pGradOut, pIndices, pGradIn, (int)blocks, make_fastdiv((uint32_t)(R2 * S2)),
            make_fastdiv((uint32_t)S2), nH, nW, P, Q);
    } else
        maxpool_bwd_gather_kernel<<<OMB_EW(total)>>>(
            pGradOut, pIndices, pGradIn, (int)total, fhw, fw, nKH, nKW, nSH, nSW, nPH, nPW, P, Q);
    return after_launch(c);
}

extern "C" int omCudaAvgPool2d(const float* pIn, float* pOut, int nN, int nC, int nH, int nW,
                               int nKH, int nKW, int nSH, int nSW, int nPH, int nPW) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nSH <= 0 || nSW <= 0) return OM_ERR_INVALID;
    int P = (nH + 2 * nPH - nKH) / nSH + 1, Q = (nW + 2 * nPW - nKW) / nSW + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    long long total = (long long)nN * nC * P * Q;
    avgpool_kernel<<<OMB_EW(total)>>>(pIn, pOut, nN, nC, nH, nW, nKH, nKW, nSH, nSW, nPH, nPW, P, Q);
    return after_launch(c);
}

extern "C" int omCudaAvgPool2dBackward(const float* pGradOut, float* pGradIn, int nN, int nC,
                                       int nH, int nW, int nKH, int nKW, int nSH, int nSW, int nPH,
                                       int nPW) {
    OMB_CTX_OR_FAIL(c);
    if (!pGradOut || !pGradIn || nSH <= 0 || nSW <= 0) return OM_ERR_INVALID;
    int P = (nH + 2 * nPH - nKH) / nSH + 1, Q = (nW + 2 * nPW - nKW) / nSW + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    long long total = (long long)nN * nC * P * Q;
    avgpool_bwd_kernel<<<OMB_EW(total)>>>(pGradOut, pGradIn, nN, nC, nH, nW, nKH, nKW, nSH, nSW, nPH, nPW, P, Q);
    return after_launch(c);
}

extern "C" int omCudaAdaptiveAvgPool2d(const float* pIn, float* pOut, int nN, int nC, int nH,
                                       int nW, int nOutH, int nOutW) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nOutH <= 0 || nOutW <= 0 || nOutH > nH || nOutW > nW) return OM_ERR_INVALID;
    long long total = (long long)nN * nC * nOutH * nOutW;
    adaptive_avgpool_kernel<<<OMB_EW(total * 32)>>>(pIn, pOut, nN, nC, nH, nW, nOutH, nOutW);
    return after_launch(c);
}

extern "C" int omCudaAdaptiveAvgPool2dBackward(const float* pGradOut, float* pGradIn, int nBatch,
                                               int nChannels, int nH, int nW, int nOutH,
                                               int nOutW) {
    OMB_CTX_OR_FAIL(c);
    if (!pGradOut || !pGradIn || nOutH <= 0 || nOutW <= 0) return OM_ERR_INVALID;
    long long total = (long long)nBatch * nChannels * nH * nW;
    adaptive_avgpool_bwd_kernel<<<OMB_EW(total)>>>(pGradOut, pGradIn, nBatch, nChannels, nH, nW, nOutH, nOutW);
    return after_launch(c);
}

extern "C" int omCudaAddBias(const float* pData, const float* pBias, float* pOut, int nN, int nC,
                             int nHW) {
    OMB_CTX_OR_FAIL(c);
    if (!pData || !pBias || !pOut) return OM_ERR_INVALID;
    long long total = (long long)nN * nC * nHW;
    map_kernel<<<OMB_EW(total)>>>(total, [=] __device__(long long i) {
        pOut[i] = pData[i] + pBias[(i / nHW) % nC];
    });
    return after_launch(c);
}

extern "C" int omCudaAddBiasBackward(const float* pGradOut, float* pGradBias, int nN, int nC,
                                     int nHW) {
    OMB_CTX_OR_FAIL(c);
    if (!pGradOut || !pGradBias) return OM_ERR_INVALID;
    if ((long long)nN * nHW >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    bias_grad_kernel<<<nC, 256, 0, c->compute>>>(pGradOut, pGradBias, nN, nC,
                                                 make_fastdiv((uint32_t)nHW));
    return after_launch(c);
}

extern "C" int omCudaSoftmax(const float* pIn, float* pOut, int nBatch, int nClasses) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nBatch <= 0 || nClasses <= 0) return OM_ERR_INVALID;
    long long threads = (long long)nBatch * 32;
    softmax_kernel<<<(int)((threads + 255) / 256), 256, 0, c->compute>>>(pIn, pOut, nBatch, nClasses);
    return after_launch(c);
}

extern "C" int omCudaCrossEntropy(const float* pSoftmax, const float* pTarget, float* pResult,
                                  int nBatch, int nClasses) {
    OMB_CTX_OR_FAIL(c);
    if (!pSoftmax || !pTarget || !pResult || nBatch <= 0) return OM_ERR_INVALID;
    cross_entropy_kernel<<<1, 1024, 0, c->compute>>>(pSoftmax, pTarget, pResult,
                                                     (long long)nBatch * nClasses, nBatch);
    return after_launch(c);
}

extern "C" int omCudaSoftmaxCrossEntropyFused(const float* pLogits, const float* pTarget,
                                              float* pSoftmax, float* pGradLogits, float* pLoss,
                                              int nBatch, int nClasses) {
    OMB_CTX_OR_FAIL(c);
    if (!pLogits || !pTarget || !pGradLogits || !pLoss || nBatch <= 0 || nClasses <= 0)
        return OM_ERR_INVALID;
    const long long blocks = ((long long)nBatch + sce::kRows - 1) / sce::kRows;
    if (blocks > sce::kMaxBlocks) return OM_ERR_UNSUPPORTED;
    softmax_ce_fused_kernel<<<(int)blocks, 32 * sce::kRows, 0, c->compute>>>(
        pLogits, pTarget, pSoftmax, pGradLogits, pLoss, nBatch, nClasses, 1.f / (float)nBatch);
    return after_launch(c);
}

extern "C" int omCudaSoftmaxCrossEntropyBackward(const float* pSoftmax, const float* pTarget,
                                                 float* pGradLogits, int nBatch, int nClasses) {
    OMB_CTX_OR_FAIL(c);
    if (!pSoftmax || !pTarget || !pGradLogits || nBatch <= 0) return OM_ERR_INVALID;
    long long n = (long long)nBatch * nClasses;
    ce_softmax_bwd_kernel<<<OMB_EW(n)>>>(pSoftmax, pTarget, pGradLogits, n, 1.f / (float)nBatch);
    return after_launch(c);
}

extern "C" int omCudaSgdStep(float* pParam, const float* pGrad, float* pVelocity, int nCount,
                             float fLr, float fMomentum) {
    OMB_CTX_OR_FAIL(c);
    if (!pParam || !pGrad || nCount < 0) return OM_ERR_INVALID;
    float* v = fMomentum > 0.f ? pVelocity : nullptr;
    if (fMomentum > 0.f && !pVelocity) return OM_ERR_INVALID;
    sgd_kernel<<<OMB_EW(nCount)>>>(pParam, pGrad, v, nCount, fLr, fMomentum, nullptr);
    return after_launch(c);
}

// Data-parallel SGD: the summed gradient of `world` ranks scaled by fGradScale (1/world) inside
// the update, so the scale costs no extra pass over the gradient.
extern "C" int omCudaSgdStepScaled(float* pParam, const float* pGrad, float* pVelocity,
                                   int nCount, float fLr, float fMomentum, float fGradScale) {
    OMB_CTX_OR_FAIL(c);
    if (!pParam || !pGrad || nCount < 0) return OM_ERR_INVALID;
    float* v = fMomentum > 0.f ? pVelocity : nullptr;
    if (fMomentum > 0.f && !pVelocity) return OM_ERR_INVALID;
    sgd_kernel<<<OMB_EW(nCount)>>>(pParam, pGrad, v, nCount, fLr, fMomentum, nullptr, fGradScale);
    return after_launch(c);
}

// ---------------------------------------------------------------- gradient guard
// The training loop's check before each optimiser step (EngineBridge.cpp:1885-1925), on the
// device instead of through a host copy of every gradient: a non-finite gradient skips the
// step; otherwise the gradient is scaled by maxNorm / ||g|| when its L2 norm exceeds maxNorm,
// then by the accumulation scale. One pass reduces (each block's partial, then the last block
// to finish sums the partials in block order, so the result is deterministic) and one scales.
namespace gradguard {
constexpr int kMaxBlocks = 1024;
__device__ float g_partial[kMaxBlocks];
__device__ int g_bad[kMaxBlocks];
__device__ unsigned int g_ticket;  // zero between calls: the last block resets it

__global__ void reduce_kernel(const float* __restrict__ g, long long n, float max_norm,
                              float* __restrict__ status) {
    __shared__ float sh[32];
    __shared__ bool last;
    float s = 0.f;
    int bad = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float x = g[i];
        bad |= !isfinite(x);
        s += x * x;
    }
    bad = __syncthreads_or(bad);
    for (int o = 16; o; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sh[w];
        g_partial[blockIdx.x] = t;
        g_bad[blockIdx.x] = bad;
        __threadfence();
        last = atomicAdd(&g_ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        float t = 0.f;
        int any_bad = 0;
        for (int b = 0; b < (int)gridDim.x; ++b) {
            t += __ldcg(&g_partial[b]);
            any_bad |= __ldcg(&g_bad[b]);
        }
        const float norm = sqrtf(t);
        status[0] = any_bad ? __int_as_float(0x7fc00000) : norm;
        status[1] = any_bad ? 0.f : 1.f;
        status[2] = (!any_bad && max_norm > 0.f && norm > max_norm) ? max_norm / norm : 1.f;
        g_ticket = 0;
    }
}

__global__ void scale_kernel(float* __restrict__ g, long long n, float accum_scale,
                             const float* __restrict__ status) {
    if (status[1] == 0.f) return;  // the step is skipped; the gradient stays as it was
    const float clip = status[2];
    if (clip == 1.f && accum_scale == 1.f) return;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float x = g[i];
        if (clip != 1.f) x *= clip;
        if (accum_scale != 1.f) x *= accum_scale;
        g[i] = x;
    }
}
}  // namespace gradguard

extern "C" int omCudaGradNormClip(float* pGrad, int nCount, float fMaxNorm, float fAccumScale,
                                  float* pStatus) {
    OMB_CTX_OR_FAIL(c);
    if (!pGrad || !pStatus || nCount <= 0) return OM_ERR_INVALID;
    const int blocks = (int)std::min<long long>(2LL * c->num_sms, gradguard::kMaxBlocks);
    gradguard::reduce_kernel<<<blocks, 512, 0, c->compute>>>(pGrad, nCount, fMaxNorm, pStatus);
    int st = after_launch(c);
    if (st != OM_OK) return st;
    gradguard::scale_kernel<<<OMB_EW(nCount)>>>(pGrad, nCount, fAccumScale, pStatus);
    return after_launch(c);
}

extern "C" int omCudaSgdStepGuarded(float* pParam, const float* pGrad, float* pVelocity,
                                    int nCount, float fLr, float fMomentum,
                                    const float* pStatus) {
    OMB_CTX_OR_FAIL(c);
    if (!pParam || !pGrad || !pStatus || nCount < 0) return OM_ERR_INVALID;
    float* v = fMomentum > 0.f ? pVelocity : nullptr;
    if (fMomentum > 0.f && !pVelocity) return OM_ERR_INVALID;
    sgd_kernel<<<OMB_EW(nCount)>>>(pParam, pGrad, v, nCount, fLr, fMomentum, pStatus);
    return after_launch(c);
}

extern "C" int omCudaAdd(const float* pA, const float* pB, float* pC, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pB || !pC || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pA, pB, pC, nCount, [] __device__(float a, float b) { return a + b; });
}

extern "C" int omCudaMulScalar(const float* pA, float fScalar, float* pC, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pC || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pA, nullptr, pC, nCount,
               [=] __device__(float a, float) { return a * fScalar; });
}

extern "C" int omCudaReLU(const float* pIn, float* pOut, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pIn, nullptr, pOut, nCount,
               [] __device__(float v, float) { return v > 0.f ? v : 0.f; });
}

extern "C" int omCudaReLUBackward(const float* pIn, const float* pGradOut, float* pGradIn,
                                  int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pGradOut || !pGradIn || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pIn, pGradOut, pGradIn, nCount,
               [] __device__(float x, float g) { return x > 0.f ? g : 0.f; });
}

extern "C" int omCudaClip(const float* pIn, float* pOut, int nCount, float fMin, float fMax) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pIn, nullptr, pOut, nCount, [=] __device__(float v, float) {
        v = v < fMin ? fMin : v;
        return v > fMax ? fMax : v;
    });
}

// ---------------------------------------------------------------- more elementwise ops
// The reference's remaining elementwise entry points (cuda_kernels.cu:477-660, 1871-2005,
// 3735), with its formulas; the math functions are CUDA's own expf / tanhf.
#define OMB_ZIP_ENTRY(NAME, A, B, FN)                                              \
    extern "C" int NAME {                                                          \
        OMB_CTX_OR_FAIL(c);                                                        \
        if (!(A) || !pOut || nCount < 0) return OM_ERR_INVALID;                    \
        return zip(c, A, B, pOut, nCount, FN);                                     \
    }
extern "C" int omCudaSub(const float* pA, const float* pB, float* pC, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pB || !pC || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pA, pB, pC, nCount, [] __device__(float a, float b) { return a - b; });
}
extern "C" int omCudaMul(const float* pA, const float* pB, float* pC, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pB || !pC || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pA, pB, pC, nCount, [] __device__(float a, float b) { return a * b; });
}
extern "C" int omCudaDiv(const float* pA, const float* pB, float* pC, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pB || !pC || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pA, pB, pC, nCount, [] __device__(float a, float b) { return a / b; });
}
extern "C" int omCudaAddScalar(const float* pA, float fScalar, float* pC, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pC || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pA, nullptr, pC, nCount, [=] __device__(float a, float) { return a + fScalar; });
}
// sigmoid(x) = 1 / (1 + exp(-x)); its backward from the output o: g * o * (1 - o)
OMB_ZIP_ENTRY(omCudaSigmoid(const float* pIn, float* pOut, int nCount), pIn, nullptr,
              [] __device__(float x, float) { return 1.0f / (1.0f + expf(-x)); })
OMB_ZIP_ENTRY(omCudaSigmoidBackward(const float* pGrad, const float* pOutput, float* pOut,
                                    int nCount), pGrad, pOutput,
              [] __device__(float g, float o) { return g * o * (1.0f - o); })
OMB_ZIP_ENTRY(omCudaTanh(const float* pIn, float* pOut, int nCount), pIn, nullptr,
              [] __device__(float x, float) { return tanhf(x); })
OMB_ZIP_ENTRY(omCudaTanhBackward(const float* pGrad, const float* pOutput, float* pOut,
                                 int nCount), pGrad, pOutput,
              [] __device__(float g, float o) { return g * (1.0f - o * o); })
// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
OMB_ZIP_ENTRY(omCudaGELU(const float* pIn, float* pOut, int nCount), pIn, nullptr,
              [] __device__(float x, float) {
                  const float u = 0.7978845608f * (x + 0.044715f * x * x * x);
                  return 0.5f * x * (1.0f + tanhf(u));
              })
OMB_ZIP_ENTRY(omCudaGeluBackward(const float* pGrad, const float* pInput, float* pOut,
                                 int nCount), pGrad, pInput,
              [] __device__(float g, float x) {
                  const float t = tanhf(0.7978845608f * (x + 0.044715f * x * x * x));
                  const float du = 0.7978845608f * (1.0f + 3.0f * 0.044715f * x * x);
                  return g * (0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * du);
              })
OMB_ZIP_ENTRY(omCudaSiLU(const float* pIn, float* pOut, int nCount), pIn, nullptr,
              [] __device__(float x, float) { return x * (1.0f / (1.0f + expf(-x))); })
OMB_ZIP_ENTRY(omCudaSiluBackward(const float* pGrad, const float* pInput, float* pOut,
                                 int nCount), pGrad, pInput,
              [] __device__(float g, float x) {
                  const float s = 1.0f / (1.0f + expf(-x));
                  return g * s * (1.0f + x * (1.0f - s));
              })
extern "C" int omCudaLeakyRelu(const float* pIn, float* pOut, int nCount, float fSlope) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pIn, nullptr, pOut, nCount,
               [=] __device__(float x, float) { return x > 0.0f ? x : fSlope * x; });
}
extern "C" int omCudaLeakyReluBackward(const float* pGrad, const float* pInput, float* pOut,
                                       int nCount, float fSlope) {
    OMB_CTX_OR_FAIL(c);
    if (!pGrad || !pInput || !pOut || nCount < 0) return OM_ERR_INVALID;
    return zip(c, pGrad, pInput, pOut, nCount,
               [=] __device__(float g, float x) { return x > 0.0f ? g : fSlope * g; });
}
#undef OMB_ZIP_ENTRY

extern "C" int omCudaFillValue(float* pData, int nCount, float fValue) {
    OMB_CTX_OR_FAIL(c);
    if (!pData || nCount < 0) return OM_ERR_INVALID;
    map_kernel<<<OMB_EW(nCount)>>>((long long)nCount, [=] __device__(long long i) { pData[i] = fValue; });
    return after_launch(c);
}

extern "C" int omCudaFillZeros(float* pData, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pData || nCount < 0) return OM_ERR_INVALID;
    return omb::status_of(cudaMemsetAsync(pData, 0, sizeof(float) * (size_t)nCount, c->compute));
}

extern "C" int omCudaFillOnes(float* pData, int nCount) { return omCudaFillValue(pData, nCount, 1.f); }

extern "C" int omCudaCopy(const float* pSrc, float* pDst, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pSrc || !pDst || nCount < 0) return OM_ERR_INVALID;
    return omb::status_of(cudaMemcpyAsync(pDst, pSrc, sizeof(float) * (size_t)nCount,
                                          cudaMemcpyDeviceToDevice, c->compute));
}

extern "C" int omCudaSum(const float* pData, float* pResult, int nCount) {
    OMB_CTX_OR_FAIL(c);
    if (!pData || !pResult || nCount < 0) return OM_ERR_INVALID;
    sum_kernel<<<1, 1024, 0, c->compute>>>(pData, pResult, nCount);
    return after_launch(c);
}

extern "C" int omCudaArgmax(const float* pData, int* pOut, int nBatch, int nClasses) {
    OMB_CTX_OR_FAIL(c);
    if (!pData || !pOut || nBatch <= 0 || nClasses <= 0) return OM_ERR_INVALID;
    long long threads = (long long)nBatch * 32;
    argmax_kernel<<<(int)((threads + 255) / 256), 256, 0, c->compute>>>(pData, pOut, nBatch, nClasses);
    return after_launch(c);
}

extern "C" int omCudaTranspose(const float* pIn, float* pOut, int nRows, int nCols) {
    OMB_CTX_OR_FAIL(c);
    if (!pIn || !pOut || nRows <= 0 || nCols <= 0) return OM_ERR_INVALID;
    dim3 grid((nCols + 31) / 32, (nRows + 31) / 32);
    transpose_kernel<<<grid, dim3(32, 8), 0, c->compute>>>(pIn, pOut, nRows, nCols);
    return after_launch(c);
}

// ---------------------------------------------------------------- allocation-free BatchNorm
// For callers that cannot allocate device memory while they run (a fixed VRAM budget reserved
// up front, or a host process that owns the device allocator): the training-mode partial sums
// live in a file-scope device array instead of pool memory. The array costs 2 MiB on every
// device that loads this library, for as long as the process lives.
namespace omb {
namespace ops {
constexpr int kNoAllocMaxChannels = 4096;
constexpr int kNoAllocMaxSplits = 64;  // bn_splits never returns more
static __device__ __align__(256) float g_bnNoAllocScratch[2 * kNoAllocMaxChannels * kNoAllocMaxSplits];
// Device address of the array per device. In host code the array's name is only a host-side
// stand-in, so the real address is looked up once per device with that device current.
static float* g_bnNoAllocAddr[64] = {nullptr};
static std::mutex g_bnNoAllocMu;
}  // namespace ops
}  // namespace omb

extern "C" int omCudaBatchNorm2dNoAlloc(const float* pInput, float* pOutput, const float* pGamma,
                                        const float* pBeta, float* pRunMean, float* pRunVar,
                                        float* pSavedMean, float* pSavedInvStd, int nBatch,
                                        int nChannels, int nH, int nW, float fEps,
                                        float fMomentum, int bTraining) {
    OMB_CTX_OR_FAIL(c);
    if (!pInput || !pOutput || !pGamma || !pBeta || !pRunMean || !pRunVar || !pSavedMean ||
        !pSavedInvStd || nBatch <= 0 || nChannels <= 0 || nH <= 0 || nW <= 0)
        return OM_ERR_INVALID;
    if (nChannels > kNoAllocMaxChannels) return OM_ERR_TOO_LARGE;
    const int HW = nH * nW;
    const long long cnt = (long long)nBatch * HW;
    if (cnt >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    int S = 1;
    float* scratch = nullptr;
    if (bTraining) {
        {
            std::lock_guard<std::mutex> lock(g_bnNoAllocMu);
            if (!g_bnNoAllocAddr[c->device]) {
                void* addr = nullptr;
                OMB_CHECK(cudaGetSymbolAddress(&addr, g_bnNoAllocScratch));
                g_bnNoAllocAddr[c->device] = static_cast<float*>(addr);
            }
            scratch = g_bnNoAllocAddr[c->device];
        }
        S = bn_splits(c, nChannels, cnt);
        if (S > kNoAllocMaxSplits) S = kNoAllocMaxSplits;
        // Nothing needs clearing: each call writes every partial-sum slot it later reads.
        const int st = bn_stats(c, pInput, scratch, nBatch, nChannels, HW, S);
        if (st != OM_OK) return st;
    }
    bn_finalize_kernel<<<(nChannels + 127) / 128, 128, 0, c->compute>>>(
        scratch, scratch ? scratch + (long long)nChannels * S : nullptr, S, cnt, pRunMean, pRunVar,
        pSavedMean, pSavedInvStd, fEps, fMomentum, bTraining, nChannels);
    int st = after_launch(c);
    if (st != OM_OK) return st;
    return bn_apply(c, pInput, pOutput, pGamma, pBeta, pSavedMean, pSavedInvStd,
                    cnt * nChannels, nChannels, HW);
}
