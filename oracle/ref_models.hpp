// Test infrastructure only: models composed from the reference engine's own modules, shared by
// the CPU shim (ref_shim.cpp, the parity reference) and the engine-on-backend shim
// (engine_shim.cpp). Include after the generated reference headers.
//
// The BASELINE configs' ImageNet 7x7/2 stem + 3x3/2 maxpool variants are composed from the
// reference's exported building blocks, because the reference's own ResNet18/ResNet50 classes
// use a CIFAR stem (om.engine.resnet.ixx:195-197, om.engine.resnet50.ixx:205).
#pragma once

#include <memory>
#include <string>
#include <vector>

namespace omref_models {

using om::Tensor;

// ImageNet-stem ResNet built from the reference's BasicBlock/Bottleneck (resnet.ixx:31,
// resnet50.ixx:28). kind 0 = ResNet-18 (BasicBlock x [2,2,2,2]), 1 = ResNet-50
// (Bottleneck x [3,4,6,3]).
class ImageNetResNet : public om::Module {
public:
    ImageNetResNet(int kind, int classes) {
        conv1 = std::make_shared<om::Conv2d>(3, 64, 7, 2, 3, false);
        bn1 = std::make_shared<om::BatchNorm2d>(64);
        registerModule("conv1", conv1);
        registerModule("bn1", bn1);
        static const int r18[4] = {2, 2, 2, 2}, r50[4] = {3, 4, 6, 3};
        const int* depth = kind == 0 ? r18 : r50;
        int inC = 64;
        for (int s = 0; s < 4; ++s) {
            int planes = 64 << s;
            for (int b = 0; b < depth[s]; ++b) {
                int stride = (s > 0 && b == 0) ? 2 : 1;
                std::shared_ptr<om::Module> blk;
                if (kind == 0) {
                    blk = std::make_shared<om::BasicBlock>(inC, planes, stride);
                    inC = planes;
                } else {
                    blk = std::make_shared<om::Bottleneck>(inC, planes, stride);
                    inC = planes * 4;
                }
                registerModule("layer" + std::to_string(s + 1) + "." + std::to_string(b), blk);
                blocks.push_back(blk);
            }
        }
        fc = std::make_shared<om::Linear>(inC, classes, true);
        registerModule("fc", fc);
    }
    Tensor forward(const Tensor& x) override {
        auto out = conv1->forward(x);
        out = bn1->forward(out);
        out = relu.forward(out);
        out = pool.forward(out);
        for (auto& b : blocks) out = b->forward(out);
        out = gap.forward(out);
        out = flat.forward(out);
        return fc->forward(out);
    }
    std::shared_ptr<om::Conv2d> conv1;
    std::shared_ptr<om::BatchNorm2d> bn1;
    om::ReLU relu;
    om::MaxPool2d pool{3, 2, 1};
    std::vector<std::shared_ptr<om::Module>> blocks;
    om::AdaptiveAvgPool2d gap{1, 1};
    om::Flatten flat{1};
    std::shared_ptr<om::Linear> fc;
};

// MobileNet-style stack: ConvBnReLU6(3,32,3,s2,p1) stem, then 12 InvertedResidual(expand 4)
// blocks, 3 per stage at widths 32/64/128/256 with stride 2 on the first block of stages
// 2-4 (mobilenet.ixx:44, :177), global pool, Linear(256, classes).
class MobileStack : public om::Module {
public:
    explicit MobileStack(int classes) {
        stem = std::make_shared<om::ConvBnReLU6>(3, 32, 3, 2, 1);
        registerModule("stem", stem);
        static const int widths[4] = {32, 64, 128, 256};
        int inC = 32;
        for (int s = 0; s < 4; ++s) {
            for (int b = 0; b < 3; ++b) {
                int stride = (s > 0 && b == 0) ? 2 : 1;
                auto blk = std::make_shared<om::InvertedResidual>(inC, widths[s], stride, 4);
                registerModule("blocks." + std::to_string(s * 3 + b), blk);
                blocks.push_back(blk);
                inC = widths[s];
            }
        }
        fc = std::make_shared<om::Linear>(inC, classes, true);
        registerModule("fc", fc);
    }
    Tensor forward(const Tensor& x) override {
        auto out = stem->forward(x);
        for (auto& b : blocks) out = b->forward(out);
        out = gap.forward(out);
        out = flat.forward(out);
        return fc->forward(out);
    }
    std::shared_ptr<om::ConvBnReLU6> stem;
    std::vector<std::shared_ptr<om::Module>> blocks;
    om::AdaptiveAvgPool2d gap{1, 1};
    om::Flatten flat{1};
    std::shared_ptr<om::Linear> fc;
};

// A few-hundred-parameter model (conv with bias, BN, FC) whose .omm files the golden fixtures
// keep: small enough to commit, with every entry kind (4-D, 1-D and 2-D parameters, BN buffers).
class TinyNet : public om::Module {
public:
    explicit TinyNet(int classes) {
        conv = std::make_shared<om::Conv2d>(3, 4, 3, 1, 1, true);
        bn = std::make_shared<om::BatchNorm2d>(4);
        fc = std::make_shared<om::Linear>(4, classes, true);
        registerModule("conv", conv);
        registerModule("bn", bn);
        registerModule("fc", fc);
    }
    Tensor forward(const Tensor& x) override { return x; }
    std::shared_ptr<om::Conv2d> conv;
    std::shared_ptr<om::BatchNorm2d> bn;
    std::shared_ptr<om::Linear> fc;
};

}  // namespace omref_models
