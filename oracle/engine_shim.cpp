// Test infrastructure only: the reference engine, unchanged, running on this repository's
// backend.
//
// The reference's own Tensor, tensor_ops, autograd, Module/Conv2d/BatchNorm2d/Linear, SGD and
// CrossEntropyLoss code (headers generated from the read-only checkout by gen_ref_headers.sh)
// is compiled with OM_HAS_CUDA defined, so every op on a CUDA tensor dispatches through
// om::CUDABackend into the C ABI. The three subsystems the backend replaces come from this
// repository instead of the reference: om::TensorStorage (include/om_tensor_storage.hpp, in
// place of om.engine.tensor_storage.ixx), om::CUDABackend (include/om_cuda_backend.hpp, in
// place of om.hal.cuda_backend.ixx) and the kernels (libomcuda.so, in place of
// src/cuda/cuda_kernels.cu). Models are composed exactly as in ref_shim.cpp (ref_models.hpp),
// moved to the GPU the way EngineBridge.cpp:915-931 moves a model (every parameter and buffer
// replaced by its .cuda() copy), and trained in train_main.cpp's order.
//
// tests/test_gpu_engine.py compares this library with the same engine code on the CPU
// (oracle/_ref/libomref.so) and with the oracle's double-precision training step.
#include <cmath>
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
#include "ref_models.hpp"

#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

using om::Tensor;

namespace {

struct EngineModel {
    std::unique_ptr<om::Module> mod;
    std::unique_ptr<om::SGD> sgd;
    bool on_cuda = false;
};

std::string g_last_error;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_last_error = e.what();
    } catch (...) {
        g_last_error = "unknown exception";
    }
    return -1;
}

std::vector<std::pair<std::string, Tensor*>> params_of(EngineModel* m) {
    return m->mod->namedParameters();
}
std::vector<std::pair<std::string, Tensor*>> buffers_of(EngineModel* m) {
    return m->mod->namedBuffers();
}

// host copy of any tensor (device tensors come back through TensorStorage::copyTo(CPU))
void read_back(const Tensor& t, float* dst) {
    Tensor c = (t.isCuda() ? t.cpu() : t).contiguous();
    std::memcpy(dst, c.floatDataPtr(), sizeof(float) * (size_t)c.numel());
}

// name of a parameter / buffer into buf; returns its rank, shape into shape[0..3]
int describe(const std::pair<std::string, Tensor*>& e, char* buf, int buflen, int* shape) {
    std::snprintf(buf, buflen, "%s", e.first.c_str());
    const auto& s = e.second->shapeVec();
    for (size_t i = 0; i < s.size() && i < 4; ++i) shape[i] = s[i];
    return (int)s.size();
}

}  // namespace

extern "C" {

const char* omeng_last_error(void) { return g_last_error.c_str(); }

int omeng_init(int device) { return omCudaInit(device); }

void* omeng_model_create(int kind, int classes) {
    auto* m = new EngineModel();
    if (kind == 2)
        m->mod = std::make_unique<omref_models::MobileStack>(classes);
    else
        m->mod = std::make_unique<omref_models::ImageNetResNet>(kind, classes);
    return m;
}
void omeng_model_destroy(void* h) { delete static_cast<EngineModel*>(h); }
int omeng_model_num_params(void* h) { return (int)params_of(static_cast<EngineModel*>(h)).size(); }
int omeng_model_num_buffers(void* h) { return (int)buffers_of(static_cast<EngineModel*>(h)).size(); }
int omeng_model_param_info(void* h, int i, char* name, int len, int* shape) {
    return describe(params_of(static_cast<EngineModel*>(h))[i], name, len, shape);
}
int omeng_model_buffer_info(void* h, int i, char* name, int len, int* shape) {
    return describe(buffers_of(static_cast<EngineModel*>(h))[i], name, len, shape);
}

// Values are set while the model is still on the host (before omeng_model_to_cuda).
void omeng_model_set_param(void* h, int i, const float* data) {
    Tensor* t = params_of(static_cast<EngineModel*>(h))[i].second;
    std::memcpy(t->mutableFloatDataPtr(), data, sizeof(float) * t->numel());
}
void omeng_model_set_buffer(void* h, int i, const float* data) {
    Tensor* t = buffers_of(static_cast<EngineModel*>(h))[i].second;
    std::memcpy(t->mutableFloatDataPtr(), data, sizeof(float) * t->numel());
}
int omeng_model_get_param(void* h, int i, float* data) {
    return guarded([&] { read_back(*params_of(static_cast<EngineModel*>(h))[i].second, data); });
}
int omeng_model_get_buffer(void* h, int i, float* data) {
    return guarded([&] { read_back(*buffers_of(static_cast<EngineModel*>(h))[i].second, data); });
}
// 1 when the parameter's data lives on a device
int omeng_model_param_is_cuda(void* h, int i) {
    return params_of(static_cast<EngineModel*>(h))[i].second->isCuda() ? 1 : 0;
}

// Every parameter and buffer replaced by its device copy (EngineBridge.cpp:915-931). The
// reference's Tensor::to() does not carry the leaf's GradAccumulator over (om.engine.tensor.ixx:
// 264), and every op takes its tensors by value, so a parameter moved exactly as EngineBridge
// moves it would record no gradient: backward would accumulate into an accumulator created on a
// temporary copy (tensor_ops.ixx:81-98). The shim re-arms each moved parameter the way
// Module::registerParameter arms it at construction (module.ixx:39, tensorSetRequiresGrad).
int omeng_model_to_cuda(void* h) {
    auto* m = static_cast<EngineModel*>(h);
    return guarded([&] {
        for (auto& p : params_of(m)) {
            *p.second = p.second->cuda();
            om::tensorSetRequiresGrad(*p.second, true);
        }
        for (auto& b : buffers_of(m)) *b.second = b.second->cuda();
        m->on_cuda = true;
    });
}

// Eval-mode forward of x [N,3,H,W] (host, NCHW fp32) on the model's device; logits to host.
int omeng_model_forward(void* h, const float* x, int N, int H, int W, float* logits) {
    auto* m = static_cast<EngineModel*>(h);
    return guarded([&] {
        m->mod->eval();
        Tensor in = Tensor::fromData(x, {N, 3, H, W});
        if (m->on_cuda) in = in.cuda();
        Tensor out = m->mod->forward(in);
        read_back(out, logits);
    });
}

// One training step in the reference's own order (train_main.cpp:226-277): train-mode forward,
// CrossEntropyLoss on one-hot targets, zeroGrad, tensorBackward, then (if apply_sgd) SGD with
// momentum. grads (optional) receives every parameter gradient in namedParameters order,
// concatenated, after backward and before the update. *loss receives the loss.
int omeng_model_train_step(void* h, const float* x, const float* onehot, int N, int H, int W,
                           int classes, float lr, float momentum, int apply_sgd, float* grads,
                           float* loss) {
    auto* m = static_cast<EngineModel*>(h);
    return guarded([&] {
        m->mod->train(true);
        auto ps = params_of(m);
        if (!m->sgd) {
            std::vector<Tensor*> v;
            for (auto& p : ps) v.push_back(p.second);
            m->sgd = std::make_unique<om::SGD>(v, lr, momentum);
        }
        Tensor in = Tensor::fromData(x, {N, 3, H, W});
        Tensor tgt = Tensor::fromData(onehot, {N, classes});
        if (m->on_cuda) {
            in = in.cuda();
            tgt = tgt.cuda();
        }
        m->mod->zeroGrad();
        Tensor logits = m->mod->forward(in);
        om::CrossEntropyLoss ce;
        Tensor l = ce.forward(logits, tgt);
        *loss = l.item();
        om::tensorBackward(l);
        if (grads) {
            size_t off = 0;
            for (auto& p : ps) {
                Tensor g = om::tensorGetGrad(*p.second);
                const size_t n = (size_t)p.second->numel();
                if (g.numel() == 0)
                    std::memset(grads + off, 0, n * sizeof(float));
                else
                    read_back(g, grads + off);
                off += n;
            }
        }
        if (apply_sgd) m->sgd->step();
    });
}

}  // extern "C"
