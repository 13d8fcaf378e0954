// qmoe/quant.hpp -- the block formats and the borrowed-matrix view of the
// reference's quantisation ABI (src/quant.hpp:8-33, src/model.hpp:17-20),
// restated for C++20 callers of libqwen_moe_b200.so.  The byte layouts are
// the reference's (canonical GGML Q4_0 / Q4_1 and its 36-byte Q8_1) so
// buffers pass between the two without conversion; the tensor type numbers
// are the GGUF type ids the reference uses.
#pragma once

#include <cstddef>
#include <cstdint>
#include <span>

namespace qmoe {

enum class TensorType : std::uint32_t { F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3 };

// Q4_0: half scale d, 16 code bytes; element j = d * ((byte j & 15) - 8),
// element j + 16 = d * ((byte j >> 4) - 8).
struct Q4_0 {
    std::uint16_t d;
    std::uint8_t qs[16];
};
// Q4_1: half scale d and minimum m; element = d * code + m.
struct Q4_1 {
    std::uint16_t d, m;
    std::uint8_t qs[16];
};
// Q8_1 activations: half(amax / 127), half(raw float sum), 32 int8 codes.
struct Q8_1 {
    std::uint16_t d, s;
    std::int8_t qs[32];
};
static_assert(sizeof(Q4_0) == 18 && sizeof(Q4_1) == 20 && sizeof(Q8_1) == 36);

[[nodiscard]] constexpr std::size_t block_bytes(TensorType t) noexcept {
    return t == TensorType::Q4_0 ? sizeof(Q4_0) : t == TensorType::Q4_1 ? sizeof(Q4_1) : 0;
}

// Borrowed canonical weights of one matrix: `output` rows of `input / 32`
// blocks, row-major (the reference's QMatrix).
struct QMatrix {
    TensorType type;
    int input, output;
    std::span<const std::byte> weights;
};

}  // namespace qmoe
