// qwen/gpu_expert.hpp -- drop-in for the reference's src/gpu_expert.hpp:5-21:
// qwen::GpuExpert and qwen::ExpertTiming with the reference's constructor,
// check_quantization, linear and run, implemented by qmoe::GpuExpert over the
// C ABI of libqwen_moe_b200.so (sm_100a kernels instead of the HIP ones).
#pragma once

#include "../qmoe/gpu_expert.hpp"
#include "quant.hpp"

namespace qwen {
using qmoe::ExpertTiming;
using qmoe::GpuExpert;
}  // namespace qwen
