// Internal helpers shared by the backend's translation units: per-device context,
// status handling, launch accounting and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "om_cuda.h"

namespace omb {

// One context per device: the compute stream every entry point launches on, a transfer
// stream, the device error word that bounded waits write, and the SM count.
struct DeviceCtx {
    int device = -1;
    cudaStream_t compute = nullptr;
    cudaStream_t transfer = nullptr;
    cudaEvent_t transfer_done = nullptr;  // recorded on `transfer`, waited on by `compute`
    cudaEvent_t compute_done = nullptr;   // recorded on `compute`, waited on by `transfer`
    unsigned int* err_word = nullptr;   // device memory, 0 = no error
    int num_sms = 0;
    unsigned long long launches = 0;    // kernels launched through this library
    bool inited = false;
};

// Context of the calling thread's current device, or nullptr before omCudaInit.
DeviceCtx* ctx();

namespace tc {
// 3xTF32 tensor-core convolution of an NCHW fp32 source (om_conv_tc.cu): the source is copied
// to NHWC [N, Hp, Wp, ceil32(Cin)] with out[n,hp,wp,c] = src[n,c,(hp-offh)/up,(wp-offw)/up]
// (exact divisions inside the source, else 0), convolved (stride, pad) with W [Kw, Cw, R, S]
// (flip = false: Kout = Kw output channels; flip = true: Kout = Cw, the filter transposed and
// rotated by 180 degrees, for the backward-input pass) and written NCHW [N, Kout, P, Q] (+bias).
// With dil > 1 the filter is dilated: tap (r, s) reads input offset (r*dil, s*dil), so P and Q
// follow the dilated extent (R-1)*dil+1. One group of a grouped convolution reads Cin of the
// source's src_ctot channels per image (src points at its first) and writes Kout of the
// output's out_ktot channels per image (0: Cin and Kout, the whole tensors). With bn_part the
// epilogue also writes BatchNorm statistics of the output per 32-pixel group g = m / 32 of the
// N*P*Q output pixels m (G = ceil(N*P*Q / 32) groups) and channel k: the group's mean at
// bn_part[k*G + g], its sum of squared deviations from that mean at bn_part[(Kout + k)*G + g].
// With keep_split the NHWC hi/lo copy of the source is written to that caller buffer (hi at
// byte 0, lo at byte conv_split_half_bytes(N, Hp, Wp, Cin)) instead of scratch, and stays
// there for the weight gradient. Returns OM_ERR_UNSUPPORTED for shapes the tensor path does
// not take and OM_ERR_OOM when its operand copies do not fit; nothing is launched then.
int tf32_conv(DeviceCtx* c, const float* src, int N, int Cin, int Hin, int Win, int Hp, int Wp,
              int offh, int offw, int up, const float* w, int Kout, int R, int S, bool flip,
              int Cw, const float* bias, float* out, int stride, int pad, int dil = 1,
              int src_ctot = 0, int out_ktot = 0, float* bn_part = nullptr,
              float* keep_split = nullptr);
// The backward input of a stride-2 convolution (dY [N, Kout, P, Q] and W [Kout, Cin, R, S] to
// dX [N, Cin, H, W], NCHW fp32) as one stride-1 3xTF32 convolution per output phase over the
// plain copy of dY. OM_ERR_UNSUPPORTED for shapes it does not take (nothing launched then).
int tf32_dgrad_s2(DeviceCtx* c, const float* dy, const float* w, float* dx, int N, int Cin,
                  int H, int W, int Kout, int R, int S, int pad, const float* yhi_in = nullptr,
                  const float* ylo_in = nullptr);
// Bytes of one half (hi or lo) of a kept input copy: N*H*W*ceil32(C) floats, rounded up to 256.
inline size_t conv_split_half_bytes(long long N, long long H, long long W, long long C) {
    return ((size_t)(N * H * W * ((C + 31) / 32 * 32)) * 4 + 255) / 256 * 256;
}
// The kept input copy of tf32_conv's keep_split written on its own (for a forward that did not
// take the tensor path).
int tf32_split_input(DeviceCtx* c, const float* x, int N, int C, int H, int W, float* keep_split);
// Whether tf32_wgrad reads a kept input copy in tf32_conv's layout for this shape: stride-2
// convs of at most 8 input channels take the space-to-depth form, whose copy only
// tf32_conv_s2d keeps.
inline bool wgrad_reads_kept_split(int Cin, int stride) { return !(stride == 2 && Cin * 4 <= 32); }
// Space-to-depth form of a stride-2 convolution of at most 8 input channels (the image stem):
// bytes of one half (hi or lo) of its 32-channel input copy [N, Hs, Ws, 32], rounded up to 256
// (0 for any other shape); the copy written on its own into keep_split; and the forward
// convolution in that form (arguments as tf32_conv's; OM_ERR_UNSUPPORTED for other shapes),
// keeping the copy for tf32_wgrad when keep_split is given.
size_t s2d_split_half_bytes(int N, int Cin, int H, int W, int R, int S, int stride, int pad);
int tf32_s2d_split_input(DeviceCtx* c, const float* x, int N, int Cin, int H, int W, int R, int S,
                         int stride, int pad, float* keep_split);
int tf32_conv_s2d(DeviceCtx* c, const float* x, int N, int Cin, int H, int W, const float* w,
                  int Kout, int R, int S, int stride, int pad, const float* bias, float* out,
                  float* bn_part, float* keep_split);
// 3xTF32 tensor-core weight gradient of a (stride, pad) convolution: dW [K, Cin, R, S] from
// X [N, Cin, H, W] and dY [N, K, P, Q], all NCHW fp32 (om_conv_tc.cu). given_split: the kept
// input copy (tf32_conv's layout, or tf32_conv_s2d's for the space-to-depth shapes). given_dy:
// an NHWC hi/lo copy of dY [N, P, Q, ceil32(K)] (hi at byte 0, lo at dy_split_half_bytes),
// read in place of a copy of its own.
int tf32_wgrad(DeviceCtx* c, const float* x, const float* dy, float* dw, int N, int Cin, int H,
               int W, int K, int R, int S, int stride, int pad, const float* given_split = nullptr,
               const float* given_dy = nullptr);
inline size_t dy_split_half_bytes(long long N, long long P, long long Q, long long K) {
    return ((size_t)(N * P * Q * ((K + 31) / 32 * 32)) * 4 + 255) / 256 * 256;
}
// The backward input from an NHWC hi/lo copy of dY (as tf32_wgrad's given_dy): stride 1 (square
// filter, pad <= R-1) as one convolution with the rotated filter, stride 2 by output phase.
// OM_ERR_UNSUPPORTED for other shapes (nothing launched then).
int tf32_dgrad_split(DeviceCtx* c, const float* yhi, const float* ylo, const float* w, float* dx,
                     int N, int Cin, int H, int W, int Kout, int R, int S, int stride, int pad);
// NHWC hi/lo copy of an NCHW tensor [N, C, P, Q] into hi, lo (channels padded to 32).
void split_nhwc(DeviceCtx* c, const float* x, float* hi, float* lo, int N, int C, int P, int Q);
}  // namespace tc

inline int status_of(cudaError_t e) { return e == cudaSuccess ? OM_OK : OM_ERR_CUDA; }

// Called after every launch: records the launch and turns a launch error into a status.
inline int after_launch(DeviceCtx* c) {
    c->launches++;
    return status_of(cudaGetLastError());
}

#define OMB_CTX_OR_FAIL(c)                       \
    omb::DeviceCtx* c = omb::ctx();              \
    if (!c) return OM_ERR_NOT_INIT;

#define OMB_CHECK(call)                          \
    do {                                         \
        cudaError_t e_ = (call);                 \
        if (e_ != cudaSuccess) return OM_ERR_CUDA; \
    } while (0)

// Grid size for grid-stride elementwise kernels: a multiple of the SM count.
inline int ew_grid(DeviceCtx* c, long long n, int block) {
    long long want = (n + block - 1) / block;
    long long cap = (long long)c->num_sms * 8;
    if (want > cap) want = cap;
    return want < 1 ? 1 : (int)want;
}

// device error codes written into DeviceCtx::err_word by bounded waits
enum : unsigned int {
    ERRBIT_TC_PRODUCER = 1u << 0,
    ERRBIT_TC_MMA = 1u << 1,
    ERRBIT_TC_EPILOGUE = 1u << 2,
    ERRBIT_TC_DRAIN = 1u << 3,
};

// 16-bit storage type helpers for the NHWC path
template <int DT> struct Half16;
template <> struct Half16<OM_DTYPE_BF16> {
    using T = __nv_bfloat16;
    using T2 = __nv_bfloat162;
    static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
    static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ T2 pack(float a, float b) { return __floats2bfloat162_rn(a, b); }
    static __device__ __forceinline__ float2 unpack(T2 v) { return __bfloat1622float2(v); }
};
template <> struct Half16<OM_DTYPE_F16> {
    using T = __half;
    using T2 = __half2;
    static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
    static __device__ __forceinline__ T from_f(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ T2 pack(float a, float b) { return __floats2half2_rn(a, b); }
    static __device__ __forceinline__ float2 unpack(T2 v) { return __half22float2(v); }
};

__device__ __forceinline__ float apply_act(float v, int act) {
    if (act == OM_ACT_RELU) return v > 0.f ? v : 0.f;
    if (act == OM_ACT_RELU6) return v < 0.f ? 0.f : (v > 6.f ? 6.f : v);
    return v;
}

}  // namespace omb
