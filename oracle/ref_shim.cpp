// Test infrastructure only: a C-ABI shim over the reference engine's own CPU code.
//
// This file is compiled against headers produced by gen_ref_headers.sh from the read-only
// reference checkout (src/hal/*.ixx, src/engine/*.ixx), with OM_HAS_CUDA undefined so every
// op takes the reference CPUBackend path. The resulting library (oracle/_ref/libomref.so)
// is the *reference itself*, used (a) to pin the C restatement in om_oracle.c, (b) to write
// the golden fixtures under tests/golden/, and (c) as the timed CPU baseline. Nothing in the
// product links it.
//
// Models are composed from the reference's exported building blocks exactly as the
// BASELINE configs describe (ImageNet 7x7/2 stem + 3x3/2 maxpool), because the reference's
// own ResNet18/ResNet50 classes use a CIFAR stem (om.engine.resnet.ixx:195-197,
// om.engine.resnet50.ixx:205).
#include <cmath>
#include <omp.h>
namespace std { using ::sqrtf; }  // om.engine.tensor_ops.ixx:901 names std::sqrtf

#include "om.hal.cpu_backend.hpp"
#include "om.engine.tensor.hpp"
#include "om.engine.tensor_ops.hpp"
#include "om.engine.module.hpp"
#include "om.engine.conv.hpp"
#include "om.engine.linear.hpp"
#include "om.engine.activations.hpp"
#include "om.engine.resnet.hpp"
#include "om.engine.resnet50.hpp"
#include "om.engine.mobilenet.hpp"
#include "om.engine.optimizer.hpp"
#include "om.engine.loss.hpp"
#include "om.engine.serializer.hpp"
#include "ref_models.hpp"

#include <cstring>
#include <memory>
#include <string>
#include <vector>

using om::CPUBackend;
using om::Tensor;

extern "C" {

// ---- single ops: straight calls into om::CPUBackend (om.hal.cpu_backend.ixx) ----------

void omref_conv2d(const float* in, const float* w, const float* b, float* out, int N, int C,
                  int H, int W, int K, int R, int stride, int pad) {
    CPUBackend::conv2d(in, w, b, out, N, C, H, W, K, R, R, stride, pad);  // :619
}
void omref_conv2d_backward_input(const float* dy, const float* w, float* dx, int N, int C, int H,
                                 int W, int K, int R, int stride, int pad) {
    CPUBackend::conv2dBackwardInput(dy, w, dx, N, C, H, W, K, R, R, stride, pad);  // :666
}
void omref_conv2d_backward_weight(const float* x, const float* dy, float* dw, float* db, int N,
                                  int C, int H, int W, int K, int R, int stride, int pad) {
    CPUBackend::conv2dBackwardWeight(x, dy, dw, db, N, C, H, W, K, R, R, stride, pad);  // :710
}
void omref_dilated_conv2d(const float* in, const float* w, const float* b, float* out, int N,
                          int C, int H, int W, int K, int R, int stride, int pad, int dil,
                          int groups) {
    CPUBackend::dilatedConv2d(in, w, b, out, N, C, H, W, K, R, R, stride, pad, dil, groups);
}
void omref_batchnorm2d(const float* in, float* out, const float* gamma, const float* beta,
                       float* run_mean, float* run_var, float* saved_mean, float* saved_invstd,
                       int N, int C, int H, int W, float eps, float momentum, int training) {
    CPUBackend::batchNorm2d(in, out, gamma, beta, run_mean, run_var, saved_mean, saved_invstd,
                            N, C, H, W, eps, momentum, training != 0);  // :781
}
void omref_batchnorm2d_backward(const float* dy, const float* x, const float* mean,
                                const float* invstd, const float* gamma, float* dx,
                                float* dgamma, float* dbeta, int N, int C, int H, int W) {
    CPUBackend::batchNorm2dBackward(dy, x, mean, invstd, gamma, dx, dgamma, dbeta, N, C, H, W);
}
void omref_maxpool2d(const float* in, float* out, int* idx, int N, int C, int H, int W, int k,
                     int stride, int pad) {
    CPUBackend::maxPool2d(in, out, idx, N, C, H, W, k, k, stride, pad);  // :897
}
void omref_maxpool2d_backward(const float* dy, const int* idx, float* dx, int N, int C, int P,
                              int Q, int H, int W) {
    CPUBackend::maxPool2dBackward(dy, idx, dx, N, C, P, Q, H, W);  // :937
}
void omref_avgpool2d(const float* in, float* out, int N, int C, int H, int W, int k, int stride,
                     int pad) {
    CPUBackend::avgPool2d(in, out, N, C, H, W, k, k, stride, pad);
}
void omref_adaptive_avgpool2d(const float* in, float* out, int N, int C, int H, int W, int OH,
                              int OW) {
    CPUBackend::adaptiveAvgPool2d(in, out, N, C, H, W, OH, OW);  // :1467
}
void omref_adaptive_avgpool2d_backward(const float* dy, float* dx, int N, int C, int H, int W,
                                       int OH, int OW) {
    CPUBackend::adaptiveAvgPool2dBackward(dy, dx, N, C, H, W, OH, OW);
}
void omref_relu(const float* in, float* out, long n) { CPUBackend::relu(in, out, (size_t)n); }
void omref_relu_backward(const float* x, const float* dy, float* dx, long n) {
    CPUBackend::reluBackward(x, dy, dx, (size_t)n);
}
void omref_add(const float* a, const float* b, float* out, long n) {
    CPUBackend::add(a, b, out, (size_t)n);
}
void omref_clip(const float* in, float* out, long n, float lo, float hi) {
    CPUBackend::clipForward(in, out, (size_t)n, lo, hi);
}
void omref_matmul(const float* a, const float* b, float* c, int M, int K, int N) {
    CPUBackend::matmul(a, b, c, M, K, N);  // :239
}
void omref_add_bias(const float* a, const float* bias, float* out, int rows, int cols) {
    CPUBackend::addBias(a, bias, out, rows, cols);
}
void omref_softmax(const float* in, float* out, int N, int C) {
    CPUBackend::softmax(in, out, N, C);
}
float omref_cross_entropy(const float* p, const float* onehot, int N, int C) {
    return CPUBackend::crossEntropy(p, onehot, N, C);
}
void omref_ce_softmax_backward(const float* p, const float* onehot, float* grad, int N, int C) {
    CPUBackend::crossEntropySoftmaxBackward(p, onehot, grad, N, C);
}

// ---- models composed from the reference's modules (ref_models.hpp) --------------------

namespace {

using omref_models::ImageNetResNet;
using omref_models::MobileStack;
using omref_models::TinyNet;

struct RefModel {
    std::unique_ptr<om::Module> mod;
    std::vector<std::pair<std::string, Tensor*>> params, bufs;
    std::unique_ptr<om::SGD> sgd;
};

}  // namespace

void* omref_model_create(int kind, int classes) {
    auto* m = new RefModel();
    if (kind == 3)
        m->mod = std::make_unique<TinyNet>(classes);
    else if (kind == 2)
        m->mod = std::make_unique<MobileStack>(classes);
    else
        m->mod = std::make_unique<ImageNetResNet>(kind, classes);
    m->params = m->mod->namedParameters();
    m->bufs = m->mod->namedBuffers();
    return m;
}
void omref_model_destroy(void* h) { delete static_cast<RefModel*>(h); }
// The model's parameters and buffers written by the reference's own ModelSerializer::save
// (format v5, om.engine.serializer.ixx:174), XOR-encrypted with `password` when it is not
// empty. Returns 0, or -1 when save threw.
int omref_model_save(void* h, const char* path, const char* password) {
    try {
        om::ModelEncryptConfig enc;
        if (password && password[0]) {
            enc.bEncrypt = true;
            enc.strPassword = password;
        }
        om::ModelMeta meta;
        meta.strModelType = "TinyNet";
        meta.nModelTypeHash = om::ModelMeta::hashString(meta.strModelType);
        meta.nNumClasses = 3;
        om::ModelSerializer::save(*static_cast<RefModel*>(h)->mod, path, meta, enc);
        return 0;
    } catch (...) {
        return -1;
    }
}
int omref_model_num_params(void* h) { return (int)static_cast<RefModel*>(h)->params.size(); }
int omref_model_num_buffers(void* h) { return (int)static_cast<RefModel*>(h)->bufs.size(); }

// Writes the tensor's name into buf and its shape into shape[0..3]; returns its rank.
static int describe(const std::pair<std::string, Tensor*>& e, char* buf, int buflen, int* shape) {
    std::snprintf(buf, buflen, "%s", e.first.c_str());
    const auto& s = e.second->shapeVec();
    for (size_t i = 0; i < s.size() && i < 4; ++i) shape[i] = s[i];
    return (int)s.size();
}
int omref_model_param_info(void* h, int i, char* name, int len, int* shape) {
    return describe(static_cast<RefModel*>(h)->params[i], name, len, shape);
}
int omref_model_buffer_info(void* h, int i, char* name, int len, int* shape) {
    return describe(static_cast<RefModel*>(h)->bufs[i], name, len, shape);
}
void omref_model_set_param(void* h, int i, const float* data) {
    Tensor* t = static_cast<RefModel*>(h)->params[i].second;
    std::memcpy(t->mutableFloatDataPtr(), data, sizeof(float) * t->numel());
}
void omref_model_get_param(void* h, int i, float* data) {
    Tensor* t = static_cast<RefModel*>(h)->params[i].second;
    std::memcpy(data, t->floatDataPtr(), sizeof(float) * t->numel());
}
void omref_model_set_buffer(void* h, int i, const float* data) {
    Tensor* t = static_cast<RefModel*>(h)->bufs[i].second;
    std::memcpy(t->mutableFloatDataPtr(), data, sizeof(float) * t->numel());
}
void omref_model_get_buffer(void* h, int i, float* data) {
    Tensor* t = static_cast<RefModel*>(h)->bufs[i].second;
    std::memcpy(data, t->floatDataPtr(), sizeof(float) * t->numel());
}

// Eval-mode forward: x is [N,3,H,W] NCHW fp32, logits [N,classes].
void omref_model_forward(void* h, const float* x, int N, int H, int W, float* logits) {
    auto* m = static_cast<RefModel*>(h);
    m->mod->eval();
    Tensor in = Tensor::fromData(x, {N, 3, H, W});
    Tensor out = m->mod->forward(in);
    Tensor c = out.contiguous();
    std::memcpy(logits, c.floatDataPtr(), sizeof(float) * c.numel());
}

// One training step in the reference's own order (train_main.cpp:226-277): train-mode forward,
// CrossEntropyLoss on one-hot targets, zeroGrad, tensorBackward, then (if apply_sgd) SGD with
// momentum. grads (optional) receives every parameter gradient in namedParameters order,
// concatenated, taken after backward and before the update.
float omref_model_train_step(void* h, const float* x, const float* onehot, int N, int H, int W,
                             int classes, float lr, float momentum, int apply_sgd, float* grads) {
    auto* m = static_cast<RefModel*>(h);
    m->mod->train(true);
    if (!m->sgd) {
        std::vector<Tensor*> ps;
        for (auto& p : m->params) ps.push_back(p.second);
        m->sgd = std::make_unique<om::SGD>(ps, lr, momentum);
    }
    Tensor in = Tensor::fromData(x, {N, 3, H, W});
    Tensor tgt = Tensor::fromData(onehot, {N, classes});
    m->mod->zeroGrad();
    Tensor logits = m->mod->forward(in);
    om::CrossEntropyLoss ce;
    Tensor loss = ce.forward(logits, tgt);
    float lv = loss.item();
    om::tensorBackward(loss);
    if (grads) {
        size_t off = 0;
        for (auto& p : m->params) {
            Tensor g = om::tensorGetGrad(*p.second);
            size_t n = (size_t)p.second->numel();
            if (g.numel() == 0) {
                std::memset(grads + off, 0, n * sizeof(float));
            } else {
                Tensor cg = g.contiguous();
                std::memcpy(grads + off, cg.floatDataPtr(), n * sizeof(float));
            }
            off += n;
        }
    }
    if (apply_sgd) m->sgd->step();
    return lv;
}

// OpenMP threads for the reference engine's parallel loops (a launcher may have set 1).
void omref_set_num_threads(int n) { omp_set_num_threads(n); }
int omref_get_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
