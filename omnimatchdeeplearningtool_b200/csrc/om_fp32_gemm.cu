// fp32 dense contractions in the reference's NCHW layout: conv forward, conv backward-input,
// conv backward-weight, grouped/depthwise conv and matmul. These back the ≤1e-4 fp32 path
// (ResNet-18 inference and training configs) and keep the reference's C ABI signatures.
//
// One SIMT implicit-GEMM template (64x64 tile, K-step 16, 256 threads, 4x4 FFMA micro-tile)
// serves all contractions; the operand "views" gather A and B on the fly, so no im2col or
// col2im buffer is ever materialised (the reference materialises one per sample,
// cuda_kernels.cu:991-1037, :2600-2690, :2739-2910).
//
// Backward-weight splits the long N*P*Q reduction over blocks; the partial tiles go to a
// scratch buffer and a second kernel sums them in a fixed order, so results are
// deterministic run to run.
#include "om_common.cuh"

namespace omb {
namespace simt {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

template <class Op>
__global__ void __launch_bounds__(NT) gemm_kernel(Op op, int M, int N, int Kd, int k_per_split) {
    __shared__ __align__(16) float As[BK][BM];
    __shared__ __align__(16) float Bs[BK][BN];
    const int t = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int kbeg = blockIdx.z * k_per_split;
    const int kend = min(Kd, kbeg + k_per_split);
    const int tx = t & 15, ty = t >> 4;
    float acc[4][4] = {};
    for (int kt = kbeg; kt < kend; kt += BK) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int row = (t >> 4) + 16 * i, col = t & 15;
            int m = m0 + row, kk = kt + col;
            As[col][row] = (m < M && kk < kend) ? op.a(m, kk) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int row = (t >> 6) + 4 * i, col = t & 63;
            int kk = kt + row, n = n0 + col;
            Bs[row][col] = (n < N && kk < kend) ? op.b(kk, n) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
            float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int n = n0 + tx * 4 + j;
            if (n < N) op.store(m, n, acc[i][j], blockIdx.z);
        }
    }
}

// C[M,N] = A[M,K] . B[K,N]
struct MatmulOp {
    const float *A, *B;
    float* C;
    int K, N;
    __device__ float a(int m, int k) const { return A[(long long)m * K + k]; }
    __device__ float b(int k, int n) const { return B[(long long)k * N + n]; }
    __device__ void store(int m, int n, float v, int) const { C[(long long)m * N + n] = v; }
};

// forward: rows = output channel k, cols = output pixel (img, p, q), reduction = (c, r, s)
struct ConvFwdOp {
    const float *X, *Wt, *bias;
    float* Y;
    int C, H, W, R, S, stride, pad, P, Q, CRS;
    __device__ float a(int k, int kk) const { return Wt[(long long)k * CRS + kk]; }
    __device__ float b(int kk, int pix) const {
        int c = kk / (R * S), rs = kk - c * (R * S), r = rs / S, s = rs - r * S;
        int img = pix / (P * Q), pq = pix - img * (P * Q), p = pq / Q, q = pq - p * Q;
        int ih = p * stride - pad + r, iw = q * stride - pad + s;
        if (ih < 0 || ih >= H || iw < 0 || iw >= W) return 0.f;
        return X[(((long long)img * C + c) * H + ih) * W + iw];
    }
    int Kout;
    __device__ void store(int k, int pix, float v, int) const {
        int img = pix / (P * Q), pq = pix - img * (P * Q);
        Y[((long long)img * Kout + k) * (P * Q) + pq] = v + (bias ? bias[k] : 0.f);
    }
};

// backward-input: rows = input channel c, cols = input pixel (img, h, w), reduction = (k, r, s)
struct ConvDgradOp {
    const float *dY, *Wt;
    float* dX;
    int C, H, W, K, R, S, stride, pad, P, Q;
    __device__ float a(int c, int kk) const {
        int k = kk / (R * S), rs = kk - k * (R * S);
        return Wt[((long long)k * C + c) * (R * S) + rs];
    }
    __device__ float b(int kk, int pix) const {
        int k = kk / (R * S), rs = kk - k * (R * S), r = rs / S, s = rs - r * S;
        int img = pix / (H * W), hw = pix - img * (H * W), h = hw / W, w = hw - h * W;
        int ph = h + pad - r, pw = w + pad - s;
        if (ph < 0 || pw < 0) return 0.f;
        if (ph % stride || pw % stride) return 0.f;
        int p = ph / stride, q = pw / stride;
        if (p >= P || q >= Q) return 0.f;
        return dY[(((long long)img * K + k) * P + p) * Q + q];
    }
    __device__ void store(int c, int pix, float v, int) const {
        int img = pix / (H * W), hw = pix - img * (H * W);
        dX[((long long)img * C + c) * (H * W) + hw] = v;
    }
};

// backward-weight: rows = k, cols = (c, r, s), reduction = (img, p, q), split over blockIdx.z
struct ConvWgradOp {
    const float *X, *dY;
    float* part;  // [splits][K][CRS]
    int C, H, W, K, R, S, stride, pad, P, Q, CRS;
    __device__ float a(int k, int kk) const {
        int img = kk / (P * Q), pq = kk - img * (P * Q);
        return dY[((long long)img * K + k) * (P * Q) + pq];
    }
    __device__ float b(int kk, int crs) const {
        int c = crs / (R * S), rs = crs - c * (R * S), r = rs / S, s = rs - r * S;
        int img = kk / (P * Q), pq = kk - img * (P * Q), p = pq / Q, q = pq - p * Q;
        int ih = p * stride - pad + r, iw = q * stride - pad + s;
        if (ih < 0 || ih >= H || iw < 0 || iw >= W) return 0.f;
        return X[(((long long)img * C + c) * H + ih) * W + iw];
    }
    __device__ void store(int k, int crs, float v, int split) const {
        part[((long long)split * K + k) * CRS + crs] = v;
    }
};

__global__ void sum_splits_kernel(const float* __restrict__ part, float* __restrict__ out,
                                  long long n, int splits) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int z = 0; z < splits; ++z) s += part[(long long)z * n + i];
        out[i] = s;
    }
}

// db[k] = sum over (img, pq) of dY[img, k, pq]; one block per channel, fixed order
__global__ void bias_grad_nchw_kernel(const float* __restrict__ dY, float* __restrict__ db, int N,
                                      int K, int PQ) {
    int k = blockIdx.x;
    float s = 0.f;
    for (long long i = threadIdx.x; i < (long long)N * PQ; i += blockDim.x) {
        int img = (int)(i / PQ), pq = (int)(i - (long long)img * PQ);
        s += dY[((long long)img * K + k) * PQ + pq];
    }
    __shared__ float sh[32];
    for (int o = 16; o; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) db[k] = s;
    }
}

// grouped / dilated direct conv (depthwise when groups == C): one thread per output element
__global__ void grouped_conv_kernel(const float* __restrict__ X, const float* __restrict__ Wt,
                                    const float* __restrict__ bias, float* __restrict__ Y, int N,
                                    int C, int H, int W, int K, int R, int S, int stride, int pad,
                                    int dil, int groups, int P, int Q) {
    long long total = (long long)N * K * P * Q;
    int cg = C / groups, kg = K / groups;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int q = (int)(i % Q);
        long long t = i / Q;
        int p = (int)(t % P);
        t /= P;
        int k = (int)(t % K);
        int img = (int)(t / K);
        int g = k / kg;
        float acc = 0.f;
        for (int ci = 0; ci < cg; ++ci)
            for (int r = 0; r < R; ++r) {
                int ih = p * stride - pad + r * dil;
                if (ih < 0 || ih >= H) continue;
                for (int s = 0; s < S; ++s) {
                    int iw = q * stride - pad + s * dil;
                    if (iw < 0 || iw >= W) continue;
                    acc = fmaf(X[(((long long)img * C + g * cg + ci) * H + ih) * W + iw],
                               Wt[(((long long)k * cg + ci) * R + r) * S + s], acc);
                }
            }
        Y[i] = acc + (bias ? bias[k] : 0.f);
    }
}

template <class Op>
static int run_gemm(DeviceCtx* c, const Op& op, int M, int N, int Kd, int splits) {
    if (M <= 0 || N <= 0) return OM_OK;
    int kps = Kd;
    if (splits > 1) {
        kps = (Kd + splits - 1) / splits;
        kps = (kps + BK - 1) / BK * BK;
        splits = (Kd + kps - 1) / kps;
    } else {
        splits = 1;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, splits);
    if (grid.y > 65535) return OM_ERR_UNSUPPORTED;
    gemm_kernel<Op><<<grid, NT, 0, c->compute>>>(op, M, N, Kd, kps);
    return after_launch(c);
}

}  // namespace simt
}  // namespace omb

using namespace omb;
using namespace omb::simt;

extern "C" int omCudaMatmul(const float* pA, const float* pB, float* pC, int nM, int nK, int nN) {
    OMB_CTX_OR_FAIL(c);
    if (!pA || !pB || !pC || nM < 0 || nK < 0 || nN < 0) return OM_ERR_INVALID;
    if (nK == 0) return omb::status_of(cudaMemsetAsync(pC, 0, sizeof(float) * (size_t)nM * nN, c->compute));
    // Tensor cores (3xTF32) first: C = A . B is the 1x1 convolution of the NCHW "image" A
    // [M, K, 1, 1] with the filter B^T, which the pack step takes transposed from B [K, N] (its
    // flip mode, a 180-degree turn of a 1x1 filter being the identity); the result is NCHW
    // [M, N, 1, 1] = C. The SIMT kernel covers what that path does not take.
    if (nM > 0 && nN > 0) {
        int st = omb::tc::tf32_conv(c, pA, nM, nK, 1, 1, 1, 1, 0, 0, 1, pB, nN, 1, 1, true, nN,
                                    nullptr, pC, 1, 0);
        if (st != OM_ERR_UNSUPPORTED && st != OM_ERR_OOM) return st;
    }
    MatmulOp op{pA, pB, pC, nK, nN};
    return run_gemm(c, op, nM, nN, nK, 1);
}

extern "C" int omCudaConv2d(const float* pInput, const float* pWeight, const float* pBias,
                            float* pOutput, int nBatch, int nCin, int nH, int nW, int nCout,
                            int nKH, int nKW, int nStride, int nPad) {
    OMB_CTX_OR_FAIL(c);
    if (!pInput || !pWeight || !pOutput || nStride <= 0) return OM_ERR_INVALID;
    int P = (nH + 2 * nPad - nKH) / nStride + 1, Q = (nW + 2 * nPad - nKW) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    // tensor cores (3xTF32) first; the SIMT kernel, which needs no scratch, covers the shapes
    // they do not take and the case where their operand copies do not fit in device memory
    int st = omb::tc::tf32_conv(c, pInput, nBatch, nCin, nH, nW, nH, nW, 0, 0, 1, pWeight, nCout,
                                nKH, nKW, false, nCin, pBias, pOutput, nStride, nPad);
    if (st != OM_ERR_UNSUPPORTED && st != OM_ERR_OOM) return st;
    ConvFwdOp op{pInput, pWeight, pBias, pOutput, nCin, nH, nW, nKH, nKW, nStride, nPad, P, Q,
                 nCin * nKH * nKW, nCout};
    return run_gemm(c, op, nCout, nBatch * P * Q, nCin * nKH * nKW, 1);
}

extern "C" int omCudaDilatedConv2d(const float* pInput, const float* pWeight, const float* pBias,
                                   float* pOutput, int nBatch, int nCin, int nH, int nW, int nCout,
                                   int nKH, int nKW, int nStride, int nPad, int nDilation,
                                   int nGroups) {
    OMB_CTX_OR_FAIL(c);
    if (!pInput || !pWeight || !pOutput || nGroups <= 0 || nCin % nGroups || nCout % nGroups ||
        nStride <= 0 || nDilation <= 0)
        return OM_ERR_INVALID;
    int eR = nKH + (nKH - 1) * (nDilation - 1), eS = nKW + (nKW - 1) * (nDilation - 1);
    int P = (nH + 2 * nPad - eR) / nStride + 1, Q = (nW + 2 * nPad - eS) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    if (nGroups == 1) {
        // dense: the 3xTF32 tensor-core conv walks the dilated taps directly (tap (r, s) reads
        // input offset (r*d, s*d)), so no zero-inserted filter and no extra arithmetic. Shapes
        // that path does not take, or whose operand copies do not fit in device memory, run on
        // the direct kernel below, which needs no scratch.
        int st = omb::tc::tf32_conv(c, pInput, nBatch, nCin, nH, nW, nH, nW, 0, 0, 1, pWeight,
                                    nCout, nKH, nKW, false, nCin, pBias, pOutput, nStride, nPad,
                                    nDilation);
        if (st != OM_ERR_UNSUPPORTED && st != OM_ERR_OOM) return st;
    } else if (nCin / nGroups >= 16 && nCout / nGroups >= 16 && nGroups <= 64) {
        // grouped, with enough channels per group for a GEMM: one 3xTF32 tensor-core conv per
        // group, reading its Cin/g channels of every input image and writing its Cout/g
        // channels of every output image in place (weights [Cout, Cin/g, R, S] are grouped by
        // output channel already). Depthwise and other thin groups stay on the direct kernel.
        const int cg = nCin / nGroups, kg = nCout / nGroups;
        int st = OM_OK;
        for (int g = 0; g < nGroups && st == OM_OK; ++g)
            st = omb::tc::tf32_conv(c, pInput + (size_t)g * cg * nH * nW, nBatch, cg, nH, nW, nH,
                                    nW, 0, 0, 1, pWeight + (size_t)g * kg * cg * nKH * nKW, kg,
                                    nKH, nKW, false, cg, pBias ? pBias + (size_t)g * kg : nullptr,
                                    pOutput + (size_t)g * kg * P * Q, nStride, nPad, nDilation,
                                    nCin, nCout);
        // a refusal comes at the first group (every group has the same shape); the direct
        // kernel then writes the whole output
        if (st != OM_ERR_UNSUPPORTED && st != OM_ERR_OOM) return st;
    }
    long long total = (long long)nBatch * nCout * P * Q;
    grouped_conv_kernel<<<ew_grid(c, total, 256), 256, 0, c->compute>>>(
        pInput, pWeight, pBias, pOutput, nBatch, nCin, nH, nW, nCout, nKH, nKW, nStride, nPad,
        nDilation, nGroups, P, Q);
    return after_launch(c);
}

extern "C" int omCudaConv2dBackwardInput(const float* pGradOutput, const float* pWeight,
                                         float* pGradInput, int nBatch, int nCin, int nH, int nW,
                                         int nCout, int nKH, int nKW, int nStride, int nPad) {
    OMB_CTX_OR_FAIL(c);
    if (!pGradOutput || !pWeight || !pGradInput || nStride <= 0) return OM_ERR_INVALID;
    int P = (nH + 2 * nPad - nKH) / nStride + 1, Q = (nW + 2 * nPad - nKW) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    // stride 2: one stride-1 convolution per output phase, no inserted zeros
    if (nStride == 2) {
        int st = omb::tc::tf32_dgrad_s2(c, pGradOutput, pWeight, pGradInput, nBatch, nCin, nH, nW,
                                        nCout, nKH, nKW, nPad);
        if (st != OM_ERR_UNSUPPORTED && st != OM_ERR_OOM) return st;
    }
    // dX = (zero-inserted, padded dY) convolved with the rotated, transposed filter, stride 1:
    // dY[n,k,p,q] lands at (R-1-pad + p*stride, S-1-pad + q*stride) of an (H+R-1) x (W+S-1) grid
    if (nPad <= nKH - 1 && nPad <= nKW - 1) {
        int st = omb::tc::tf32_conv(c, pGradOutput, nBatch, nCout, P, Q, nH + nKH - 1, nW + nKW - 1,
                                    nKH - 1 - nPad, nKW - 1 - nPad, nStride, pWeight, nCin, nKH,
                                    nKW, true, nCin, nullptr, pGradInput, 1, 0);
        if (st != OM_ERR_UNSUPPORTED && st != OM_ERR_OOM) return st;
    }
    ConvDgradOp op{pGradOutput, pWeight, pGradInput, nCin, nH, nW, nCout, nKH, nKW, nStride, nPad, P, Q};
    return run_gemm(c, op, nCin, nBatch * nH * nW, nCout * nKH * nKW, 1);
}

// The weight gradient; pInputSplit (optional): the forward's kept tensor-core copy of pInput
// (omCudaConv2dBatchNorm2dAct), which the tensor path then reads instead of splitting pInput.
// given_dy (optional): an NHWC hi/lo copy of pGradOutput the tensor path reads in place.
static int conv_wgrad(const float* pInput, const void* pInputSplit, const float* pGradOutput,
                      float* pGradWeight, float* pGradBias, int nBatch, int nCin, int nH, int nW,
                      int nCout, int nKH, int nKW, int nStride, int nPad,
                      const float* given_dy = nullptr) {
    OMB_CTX_OR_FAIL(c);
    if (!pInput || !pGradOutput || !pGradWeight || nStride <= 0) return OM_ERR_INVALID;
    int P = (nH + 2 * nPad - nKH) / nStride + 1, Q = (nW + 2 * nPad - nKW) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    const int CRS = nCin * nKH * nKW;
    const long long red = (long long)nBatch * P * Q;
    if (red >= (1LL << 31)) return OM_ERR_UNSUPPORTED;
    // tensor cores (3xTF32) first; the SIMT kernel covers what they do not
    int tst = omb::tc::tf32_wgrad(c, pInput, pGradOutput, pGradWeight, nBatch, nCin, nH, nW, nCout,
                                  nKH, nKW, nStride, nPad,
                                  static_cast<const float*>(pInputSplit), given_dy);
    if (tst != OM_ERR_UNSUPPORTED) {
        if (tst != OM_OK || !pGradBias) return tst;
        bias_grad_nchw_kernel<<<nCout, 256, 0, c->compute>>>(pGradOutput, pGradBias, nBatch, nCout, P * Q);
        return after_launch(c);
    }
    // enough splits to give every SM a few blocks, each split at least 256 long
    long long tiles = (long long)((CRS + BN - 1) / BN) * ((nCout + BM - 1) / BM);
    long long want = (4LL * c->num_sms + tiles - 1) / tiles;
    long long maxs = red / 256 > 0 ? red / 256 : 1;
    int splits = (int)(want < maxs ? want : maxs);
    if (splits < 1) splits = 1;
    if (splits > 256) splits = 256;
    int kps = (int)((red + splits - 1) / splits);
    kps = (kps + BK - 1) / BK * BK;
    splits = (int)((red + kps - 1) / kps);
    const long long n = (long long)nCout * CRS;
    float* part = nullptr;
    int st = OM_OK;
    if (splits > 1) {
        OMB_CHECK(cudaMallocAsync(&part, sizeof(float) * n * splits, c->compute));
        ConvWgradOp op{pInput, pGradOutput, part, nCin, nH, nW, nCout, nKH, nKW, nStride, nPad, P, Q, CRS};
        st = run_gemm(c, op, nCout, CRS, (int)red, splits);
        if (st == OM_OK) {
            sum_splits_kernel<<<ew_grid(c, n, 256), 256, 0, c->compute>>>(part, pGradWeight, n, splits);
            st = after_launch(c);
        }
        cudaFreeAsync(part, c->compute);
    } else {
        ConvWgradOp op{pInput, pGradOutput, pGradWeight, nCin, nH, nW, nCout, nKH, nKW, nStride, nPad, P, Q, CRS};
        st = run_gemm(c, op, nCout, CRS, (int)red, 1);
    }
    if (st == OM_OK && pGradBias) {
        bias_grad_nchw_kernel<<<nCout, 256, 0, c->compute>>>(pGradOutput, pGradBias, nBatch, nCout, P * Q);
        st = after_launch(c);
    }
    return st;
}

extern "C" int omCudaConv2dBackwardWeight(const float* pInput, const float* pGradOutput,
                                          float* pGradWeight, float* pGradBias, int nBatch,
                                          int nCin, int nH, int nW, int nCout, int nKH, int nKW,
                                          int nStride, int nPad) {
    return conv_wgrad(pInput, nullptr, pGradOutput, pGradWeight, pGradBias, nBatch, nCin, nH, nW,
                      nCout, nKH, nKW, nStride, nPad);
}

extern "C" int omCudaConv2dBackwardWeightSplit(const float* pInput, const void* pInputSplit,
                                               const float* pGradOutput, float* pGradWeight,
                                               float* pGradBias, int nBatch, int nCin, int nH,
                                               int nW, int nCout, int nKH, int nKW, int nStride,
                                               int nPad) {
    if (!pInputSplit) return OM_ERR_INVALID;
    return conv_wgrad(pInput, pInputSplit, pGradOutput, pGradWeight, pGradBias, nBatch, nCin, nH,
                      nW, nCout, nKH, nKW, nStride, nPad);
}

extern "C" int omCudaConv2dBackwardSplit(const float* pGradOutput, const float* pInput,
                                         const void* pInputSplit, const float* pWeight,
                                         float* pGradInput, float* pGradWeight, float* pGradBias,
                                         int nBatch, int nCin, int nH, int nW, int nCout,
                                         int nKH, int nKW, int nStride, int nPad) {
    OMB_CTX_OR_FAIL(c);
    if (!pGradOutput || !pInput || !pWeight || !pGradWeight || nStride <= 0 || nPad < 0)
        return OM_ERR_INVALID;
    const int P = (nH + 2 * nPad - nKH) / nStride + 1, Q = (nW + 2 * nPad - nKW) / nStride + 1;
    if (P <= 0 || Q <= 0) return OM_ERR_INVALID;
    // one NHWC hi/lo copy of dY for both passes (each makes its own where this is not possible)
    const size_t yb = omb::tc::dy_split_half_bytes(nBatch, P, Q, nCout);
    float* ys = nullptr;
    if ((long long)nBatch * P * Q + 128 < (1LL << 31) &&
        cudaMallocAsync(reinterpret_cast<void**>(&ys), 2 * yb, c->compute) != cudaSuccess) {
        cudaGetLastError();
        ys = nullptr;
    }
    const float* yhi = ys;
    const float* ylo = ys ? ys + yb / 4 : nullptr;
    int st = OM_OK;
    if (ys) {
        omb::tc::split_nhwc(c, pGradOutput, ys, ys + yb / 4, nBatch, nCout, P, Q);
        st = after_launch(c);
    }
    if (st == OM_OK && pGradInput) {
        st = ys ? omb::tc::tf32_dgrad_split(c, yhi, ylo, pWeight, pGradInput, nBatch, nCin, nH,
                                            nW, nCout, nKH, nKW, nStride, nPad)
                : OM_ERR_UNSUPPORTED;
        if (st == OM_ERR_UNSUPPORTED || st == OM_ERR_OOM)
            st = omCudaConv2dBackwardInput(pGradOutput, pWeight, pGradInput, nBatch, nCin, nH, nW,
                                           nCout, nKH, nKW, nStride, nPad);
    }
    if (st == OM_OK)
        st = conv_wgrad(pInput, pInputSplit, pGradOutput, pGradWeight, pGradBias, nBatch, nCin,
                        nH, nW, nCout, nKH, nKW, nStride, nPad, yhi);
    if (ys) cudaFreeAsync(ys, c->compute);
    return st;
}

extern "C" long long omCudaConvInputSplitBytes(int nBatch, int nCin, int nH, int nW,
                                               int nStride) {
    if (nBatch <= 0 || nCin <= 0 || nH <= 0 || nW <= 0 || nStride <= 0) return 0;
    if (!omb::tc::wgrad_reads_kept_split(nCin, nStride)) return 0;
    return 2LL * (long long)omb::tc::conv_split_half_bytes(nBatch, nH, nW, nCin);
}

extern "C" long long omCudaStemInputSplitBytes(int nBatch, int nCin, int nH, int nW, int nKH,
                                               int nKW, int nStride, int nPad) {
    if (nBatch <= 0 || nCin <= 0 || nH <= 0 || nW <= 0 || nKH <= 0 || nKW <= 0) return 0;
    return 2LL * (long long)omb::tc::s2d_split_half_bytes(nBatch, nCin, nH, nW, nKH, nKW, nStride,
                                                         nPad);
}
