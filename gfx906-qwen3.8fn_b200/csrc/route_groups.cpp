// route_groups.cpp -- host RouteGroups (contract of src/routes.hpp:28-65,
// behaviour of src/routes.cpp:59-130) and its C entry points.
#include "../../include/qmoe/routes.hpp"

#include <cmath>
#include <cstring>
#include <limits>
#include <stdexcept>

#include "../../include/qwen_moe_b200.h"

namespace qmoe {
namespace {

[[noreturn]] void reject(const char* why) { throw std::invalid_argument(why); }

// Byte-range overlap on a flat address space, without forming out-of-range pointers.
bool ranges_overlap(std::uintptr_t a, std::size_t an, std::uintptr_t b, std::size_t bn) noexcept {
    return a < b ? b - a < an : a - b < bn;
}

}  // namespace

RouteGroups::RouteGroups(int token_capacity, Bound bound) : capacity_(token_capacity) {
    int limit;
    switch (bound) {
    case Bound::chunk1024: limit = 1024; break;
    case Bound::layerwise16384: limit = max_tokens; break;
    default: reject("routes: unknown constructor bound");
    }
    if (token_capacity < 1 || token_capacity > limit)
        reject("routes: token capacity outside explicit constructor bound");
    storage_.resize(static_cast<std::size_t>(token_capacity) * top_k);
}

bool RouteGroups::owns(const void* data, std::size_t bytes) const noexcept {
    const auto p = reinterpret_cast<std::uintptr_t>(data);
    return ranges_overlap(p, bytes, reinterpret_cast<std::uintptr_t>(this), sizeof(*this)) ||
           ranges_overlap(p, bytes, reinterpret_cast<std::uintptr_t>(storage_.data()),
                          storage_.capacity() * sizeof(RouteAssignment));
}

void RouteGroups::prepare(std::span<const std::int32_t> ids, std::span<const float> weights, int tokens) {
    if (tokens < 1 || tokens > capacity_) reject("routes: tokens outside constructor capacity");
    const std::size_t n = static_cast<std::size_t>(tokens) * top_k;
    if (ids.size() != n || weights.size() != n) reject("routes: expected exactly tokens*10 IDs and weights");
    const auto ip = reinterpret_cast<std::uintptr_t>(ids.data());
    const auto wp = reinterpret_cast<std::uintptr_t>(weights.data());
    const auto max = std::numeric_limits<std::uintptr_t>::max();
    if (!ids.data() || !weights.data() || n * 4 > max - ip || n * 4 > max - wp)
        reject("routes: null or wrapping input range");
    if (owns(ids.data(), n * 4) || owns(weights.data(), n * 4)) reject("routes: input overlaps owned storage");
    // Validate everything before touching any member.
    for (int t = 0; t < tokens; ++t) {
        const std::int32_t* row = ids.data() + static_cast<std::size_t>(t) * top_k;
        const float* wrow = weights.data() + static_cast<std::size_t>(t) * top_k;
        for (int r = 0; r < top_k; ++r) {
            if (row[r] < 0 || row[r] >= expert_count) reject("routes: expert ID must be 0..511");
            if (!std::isfinite(wrow[r]) || wrow[r] < 0.0f) reject("routes: weight must be finite and nonnegative");
            for (int q = 0; q < r; ++q)
                if (row[q] == row[r]) reject("routes: duplicate expert ID within token");
        }
    }
    // Stable counting sort by expert; ties keep (token, rank) order.
    counts_.fill(0);
    for (std::size_t i = 0; i < n; ++i) ++counts_[static_cast<std::size_t>(ids[i])];
    int run = 0;
    for (int e = 0; e < expert_count; ++e) {
        offsets_[static_cast<std::size_t>(e)] = run;
        cursor_[static_cast<std::size_t>(e)] = run;
        run += counts_[static_cast<std::size_t>(e)];
    }
    offsets_[expert_count] = run;
    for (std::size_t i = 0; i < n; ++i) {
        const auto e = static_cast<std::size_t>(ids[i]);
        RouteAssignment& a = storage_[static_cast<std::size_t>(cursor_[e]++)];
        a.token = static_cast<int>(i / top_k);
        a.rank = static_cast<int>(i % top_k);
        a.expert = static_cast<int>(e);
        std::memcpy(&a.weight, &weights[i], sizeof(float));  // raw bits, including -0
    }
    size_ = n;
}

std::span<const RouteAssignment> RouteGroups::assignments() const noexcept { return {storage_.data(), size_}; }

std::span<const RouteAssignment> RouteGroups::group(int expert) const {
    if (expert < 0 || expert >= expert_count) reject("routes: group expert must be 0..511");
    const auto e = static_cast<std::size_t>(expert);
    return {storage_.data() + offsets_[e], static_cast<std::size_t>(counts_[e])};
}

std::span<const int> RouteGroups::counts() const noexcept { return counts_; }

}  // namespace qmoe

// ------------------------------------------------------------ C entry points
struct moe_route_groups_s {
    qmoe::RouteGroups groups;
    explicit moe_route_groups_s(int capacity, qmoe::RouteGroups::Bound b) : groups(capacity, b) {}
};

namespace {
thread_local char route_message[256];
}

extern "C" {

int moe_route_groups_create(int token_capacity, int bound, moe_route_groups_t* out) {
    if (!out) return MOE_INVALID_ARGUMENT;
    *out = nullptr;
    try {
        *out = new moe_route_groups_s(token_capacity, bound ? qmoe::RouteGroups::Bound::layerwise16384
                                                            : qmoe::RouteGroups::Bound::chunk1024);
        return MOE_OK;
    } catch (const std::invalid_argument& e) {
        std::snprintf(route_message, sizeof(route_message), "%s", e.what());
        return MOE_INVALID_ARGUMENT;
    } catch (...) {
        return MOE_OUT_OF_MEMORY;
    }
}

int moe_route_groups_destroy(moe_route_groups_t g) {
    delete g;
    return MOE_OK;
}

int moe_route_groups_prepare(moe_route_groups_t g, const int32_t* ids, const float* weights, size_t n, int tokens) {
    if (!g) return MOE_INVALID_ARGUMENT;
    try {
        g->groups.prepare({ids, n}, {weights, n}, tokens);
        return MOE_OK;
    } catch (const std::invalid_argument& e) {
        std::snprintf(route_message, sizeof(route_message), "%s", e.what());
        return MOE_INVALID_ARGUMENT;
    } catch (...) {
        return MOE_INVALID_ARGUMENT;
    }
}

size_t moe_route_groups_assignments(moe_route_groups_t g, void* out, size_t capacity) {
    if (!g) return 0;
    const auto a = g->groups.assignments();
    if (out) std::memcpy(out, a.data(), (a.size() < capacity ? a.size() : capacity) * sizeof(qmoe::RouteAssignment));
    return a.size();
}

int moe_route_groups_counts(moe_route_groups_t g, int32_t* out512) {
    if (!g || !out512) return MOE_INVALID_ARGUMENT;
    const auto c = g->groups.counts();
    std::memcpy(out512, c.data(), c.size() * sizeof(int));
    return MOE_OK;
}

const char* moe_route_groups_message(void) { return route_message; }

}  // extern "C"
