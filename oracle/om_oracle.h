/* TEST INFRASTRUCTURE ONLY — declarations of the CPU oracle (om_oracle.c). The product never
 * includes this header; see om_oracle.c for what each function restates. */
#ifndef OM_ORACLE_H
#define OM_ORACLE_H
#include <stddef.h>
#ifdef __cplusplus
extern "C" {
#endif
void oracle_conv2d(const float* in, const float* w, const float* b, float* out, int N, int C,
                   int H, int W, int K, int R, int S, int stride, int pad);
void oracle_grouped_conv2d(const float* in, const float* w, const float* b, float* out, int N,
                           int C, int H, int W, int K, int R, int S, int stride, int pad,
                           int dil, int groups);
void oracle_conv2d_backward_input(const float* dy, const float* w, float* dx, int N, int C,
                                  int H, int W, int K, int R, int S, int stride, int pad);
void oracle_conv2d_backward_weight(const float* x, const float* dy, float* dw, float* db, int N,
                                   int C, int H, int W, int K, int R, int S, int stride, int pad);
void oracle_batchnorm2d(const float* in, float* out, const float* gamma, const float* beta,
                        float* run_mean, float* run_var, float* saved_mean, float* saved_invstd,
                        int N, int C, int H, int W, float eps, float momentum, int training);
void oracle_batchnorm2d_backward(const float* dy, const float* x, const float* mean,
                                 const float* invstd, const float* gamma, float* dx,
                                 float* dgamma, float* dbeta, int N, int C, int H, int W);
void oracle_maxpool2d(const float* in, float* out, int* idx, int N, int C, int H, int W, int k,
                      int stride, int pad);
void oracle_maxpool2d_backward(const float* dy, const int* idx, float* dx, int N, int C, int P,
                               int Q, int H, int W);
void oracle_avgpool2d(const float* in, float* out, int N, int C, int H, int W, int k, int stride,
                      int pad);
void oracle_avgpool2d_backward(const float* dy, float* dx, int N, int C, int H, int W, int k,
                               int stride, int pad);
void oracle_adaptive_avgpool2d(const float* in, float* out, int N, int C, int H, int W, int OH,
                               int OW);
void oracle_adaptive_avgpool2d_backward(const float* dy, float* dx, int N, int C, int H, int W,
                                        int OH, int OW);
void oracle_relu(const float* in, float* out, size_t n);
void oracle_relu_backward(const float* x, const float* dy, float* dx, size_t n);
void oracle_add(const float* a, const float* b, float* out, size_t n);
void oracle_clip(const float* in, float* out, size_t n, float lo, float hi);
void oracle_matmul(const float* a, const float* b, float* c, int M, int K, int N);
void oracle_add_bias(const float* a, const float* bias, float* out, int rows, int cols);
void oracle_add_bias_backward(const float* dy, float* dbias, int rows, int cols);
void oracle_softmax(const float* in, float* out, int N, int C);
float oracle_cross_entropy(const float* p, const float* onehot, int N, int C);
void oracle_ce_softmax_backward(const float* p, const float* onehot, float* grad, int N, int C);
void oracle_sgd_step(float* param, const float* grad, float* vel, size_t n, float lr,
                     float momentum);
void oracle_set_num_threads(int n);
#ifdef __cplusplus
}
#endif
#endif
