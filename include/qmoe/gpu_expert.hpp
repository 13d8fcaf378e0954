// qmoe/gpu_expert.hpp -- the reference's GpuExpert host API
// (src/gpu_expert.hpp:6-21, behaviour src/hip/expert.hip:183-241) for C++20
// callers, over the C ABI of libqwen_moe_b200.so (moe_expert_*): one resident
// expert on a B200, its own stream, borrowed host spans in and out.
//
// Contract kept from the reference:
//  * the constructor checks shapes and types (gate/up Q4_0 [I][H/32], down Q4_0
//    or Q4_1 [H][I/32], H and I multiples of 32 up to 16384, 1..1024 columns)
//    and exact byte sizes, throwing std::invalid_argument, then uploads;
//  * check_quantization() requires the GPU Q8_1 bytes of `input` to equal
//    `expected` byte for byte: std::invalid_argument for bad spans or a block
//    that is not representable, std::runtime_error on a byte mismatch;
//  * linear() runs one projection (down, else up, else gate) of Q8_1 input;
//  * run() times `repeats` resident float -> Q8_1 -> gate/up -> SiLU*up ->
//    Q8_1 -> down passes after one untimed warm-up;
//  * CUDA failures throw std::runtime_error.
// The weights are always held in this library's planar layout, so `planar`
// is accepted for source compatibility and has no effect.
#pragma once

#include <memory>
#include <span>
#include <stdexcept>
#include <string>

#include "../qwen_moe_b200.h"
#include "quant.hpp"

namespace qmoe {

struct ExpertTiming {
    double upload_ms, resident_ms, completed_wall_ms;
};

class GpuExpert {
public:
    GpuExpert(QMatrix gate, QMatrix up, QMatrix down, int device, int max_columns, bool planar)
        : hidden_(gate.input), inter_(gate.output), max_columns_(max_columns) {
        (void)planar;
        if (max_columns <= 0 || max_columns > 1024 || gate.input <= 0 || gate.input > 16384 || gate.input % 32 ||
            gate.output <= 0 || gate.output > 16384 || gate.output % 32 || up.input != gate.input ||
            up.output != gate.output || down.input != gate.output || down.output != gate.input ||
            gate.type != TensorType::Q4_0 || up.type != TensorType::Q4_0 ||
            (down.type != TensorType::Q4_0 && down.type != TensorType::Q4_1))
            throw std::invalid_argument("GPU expert shape/type");
        for (const QMatrix &m : {gate, up, down})
            if (m.weights.size() != static_cast<std::size_t>(m.input / 32) * m.output * block_bytes(m.type))
                throw std::invalid_argument("GPU expert byte size");
        moe_expert_t h = nullptr;
        check(moe_expert_create_typed(gate.weights.data(), up.weights.data(), down.weights.data(),
                                      static_cast<int>(down.type), hidden_, inter_, device, max_columns, &h));
        handle_.reset(h);
    }

    GpuExpert(const GpuExpert &) = delete;
    GpuExpert &operator=(const GpuExpert &) = delete;

    void check_quantization(std::span<const float> input, std::span<const Q8_1> expected) {
        if (input.empty() || input.size() > static_cast<std::size_t>(hidden_) * max_columns_ || input.size() % 32 ||
            expected.size() != input.size() / 32)
            throw std::invalid_argument("GPU quantization span");
        const int st = moe_expert_check_quantization(handle_.get(), input.data(), input.size(), expected.data());
        if (st == MOE_NUMERIC_ERROR) throw std::runtime_error("CPU/GPU Q8_1 ABI mismatch");
        if (st == MOE_INVALID_ARGUMENT) throw std::invalid_argument("GPU activation not representable in Q8_1");
        check(st);
    }

    void linear(bool down, bool up, std::span<const Q8_1> input, int columns, std::span<float> output) {
        const int in = down ? inter_ : hidden_, out = down ? hidden_ : inter_;
        if (columns <= 0 || columns > max_columns_ || input.size() != static_cast<std::size_t>(in / 32) * columns ||
            output.size() != static_cast<std::size_t>(out) * columns)
            throw std::invalid_argument("GPU linear span");
        check(moe_expert_linear(handle_.get(), down ? 1 : 0, up ? 1 : 0, input.data(), columns, output.data()));
    }

    ExpertTiming run(std::span<const float> input, int columns, std::span<float> output, int repeats) {
        if (columns <= 0 || columns > max_columns_ || repeats <= 0 || repeats > 10000 ||
            input.size() != static_cast<std::size_t>(hidden_) * columns || output.size() != input.size())
            throw std::invalid_argument("GPU expert input/output");
        ExpertTiming t{};
        const int st = moe_expert_run(handle_.get(), input.data(), columns, output.data(), repeats, &t.upload_ms,
                                      &t.resident_ms, &t.completed_wall_ms);
        if (st == MOE_NUMERIC_ERROR) throw std::invalid_argument("GPU activation not representable in Q8_1");
        check(st);
        return t;
    }

private:
    struct Destroy {
        void operator()(moe_expert_t h) const noexcept { moe_expert_destroy(h); }
    };
    static void check(int st) {
        if (st == MOE_OK) return;
        const char *msg = moe_last_error_message();
        std::string what = std::string(moe_status_string(st)) + ": " + (msg ? msg : "");
        if (st == MOE_INVALID_ARGUMENT || st == MOE_NOT_SUPPORTED) throw std::invalid_argument(what);
        throw std::runtime_error(what);
    }
    int hidden_, inter_, max_columns_;
    std::unique_ptr<moe_expert_s, Destroy> handle_;
};

}  // namespace qmoe
