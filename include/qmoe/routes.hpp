// qmoe/routes.hpp -- host route grouping with the reference's RouteGroups
// contract (src/routes.hpp:11-65), implemented in libqwen_moe_b200.so.
//
// Fixed 512-expert / top-10 routing map.  All storage is allocated once in the
// constructor; prepare() and the accessors allocate nothing.  prepare()
// validates the whole input (ids 0..511 and unique within each token, weights
// finite and nonnegative, exact tokens*10 extents, no byte overlap with this
// object's storage) before mutating anything, throwing std::invalid_argument
// otherwise, and keeps every raw weight bit.  Groups ascend by expert; inside
// a group the order is token, then original rank.  Not copyable or movable.
//
// The forward path on the GPU (moe_forward) builds the same grouping on the
// device; this class keeps the reference's host API for callers that group on
// the host (e.g. the reference Session's hybrid CPU/GPU path).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <span>
#include <vector>

namespace qmoe {

struct RouteAssignment {
    int token;
    int rank;
    int expert;
    float weight;
};
static_assert(sizeof(RouteAssignment) == 16);

// Exported from libqwen_moe_b200.so (built with hidden default visibility).
class __attribute__((visibility("default"))) RouteGroups {
public:
    enum class Bound { chunk1024, layerwise16384 };
    explicit RouteGroups(int token_capacity, Bound bound = Bound::chunk1024);
    RouteGroups(const RouteGroups&) = delete;
    RouteGroups& operator=(const RouteGroups&) = delete;
    RouteGroups(RouteGroups&&) = delete;
    RouteGroups& operator=(RouteGroups&&) = delete;

    void prepare(std::span<const std::int32_t> ids, std::span<const float> weights, int tokens);
    std::span<const RouteAssignment> assignments() const noexcept;
    std::span<const RouteAssignment> group(int expert) const;
    std::span<const int> counts() const noexcept;

private:
    static constexpr int expert_count = 512;
    static constexpr int top_k = 10;
    static constexpr int max_tokens = 16384;
    bool owns(const void* data, std::size_t bytes) const noexcept;

    int capacity_;
    std::vector<RouteAssignment> storage_;
    std::array<int, expert_count> counts_{};
    std::array<int, expert_count + 1> offsets_{};
    std::array<int, expert_count> cursor_{};
    std::size_t size_ = 0;
};

}  // namespace qmoe
