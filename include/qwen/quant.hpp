// qwen/quant.hpp -- drop-in for the block formats and the borrowed-matrix view
// of the reference's src/quant.hpp:6-33 (TensorType from src/model.hpp:17-20):
// the same byte layouts and names in namespace qwen.  The reference's CPU
// matmul/quantize functions stay the reference's own code (this library has
// no CPU path); this header covers what the GPU expert API takes.
#pragma once

#include "../qmoe/quant.hpp"

namespace qwen {
using qmoe::block_bytes;
using qmoe::Q4_0;
using qmoe::Q4_1;
using qmoe::Q8_1;
using qmoe::QMatrix;
using qmoe::TensorType;
}  // namespace qwen
