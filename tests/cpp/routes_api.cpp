// C++20 exercise of qwen::RouteGroups through include/qwen/routes.hpp (the
// reference's header name and namespace) with the reference's contract
// (src/routes.hpp:18-65): grouping order, raw weight bits, validation before
// mutation, and the Bound capacities.  Runs on the host only; prints "ok".
#include <cstdint>
#include <cstring>
#include <iostream>
#include <stdexcept>
#include <vector>

#include "routes.hpp"   // include/qwen/

namespace {
int fails = 0;
void expect(bool ok, const char *what) {
    if (!ok) {
        std::cout << "FAIL " << what << "\n";
        ++fails;
    }
}
template <class F> bool throws_invalid(F f) {
    try {
        f();
    } catch (const std::invalid_argument &) {
        return true;
    }
    return false;
}
}  // namespace

int main() {
    constexpr int T = 6, K = 10;
    std::vector<std::int32_t> ids(T * K);
    std::vector<float> w(T * K);
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < K; ++k) {
            ids[t * K + k] = (t * 7 + k * 53) % 512;   // unique within a token, reused across tokens
            w[t * K + k] = 0.01f * static_cast<float>(k + 1) + 0.001f * static_cast<float>(t);
        }
    w[3] = -0.0f;   // a signed zero is a valid weight and keeps its bits
    qwen::RouteGroups rg(T);
    rg.prepare(ids, w, T);
    const auto a = rg.assignments();
    expect(a.size() == static_cast<std::size_t>(T * K), "every contribution kept");
    for (std::size_t i = 1; i < a.size(); ++i) {
        const auto &p = a[i - 1], &q = a[i];
        expect(p.expert < q.expert ||
                   (p.expert == q.expert && (p.token < q.token || (p.token == q.token && p.rank < q.rank))),
               "groups ascend by expert, then token, then rank");
    }
    for (const auto &x : a) {
        expect(ids[x.token * K + x.rank] == x.expert, "assignment names its source id");
        expect(std::memcmp(&w[x.token * K + x.rank], &x.weight, 4) == 0, "raw weight bits kept");
    }
    int total = 0;
    for (int c : rg.counts()) total += c;
    expect(total == T * K, "counts sum to tokens*10");
    const auto g = rg.group(ids[0]);
    expect(!g.empty() && g[0].expert == ids[0], "group view");
    expect(throws_invalid([&] { (void)rg.group(512); }), "group expert range");

    // rejected calls leave the published views unchanged
    const std::vector<qwen::RouteAssignment> before(a.begin(), a.end());
    std::vector<std::int32_t> dup = ids;
    dup[1] = dup[0];
    expect(throws_invalid([&] { rg.prepare(dup, w, T); }), "duplicate id within a token");
    std::vector<float> bad = w;
    bad[5] = -1.0f;
    expect(throws_invalid([&] { rg.prepare(ids, bad, T); }), "negative weight");
    expect(throws_invalid([&] { rg.prepare(std::span(ids).first(T * K - 1), std::span(w).first(T * K - 1), T); }),
           "extent must be tokens*10");
    expect(throws_invalid([&] { rg.prepare(ids, w, T + 1); }), "tokens above capacity");
    const auto after = rg.assignments();
    expect(after.size() == before.size() &&
               std::memcmp(after.data(), before.data(), before.size() * sizeof(qwen::RouteAssignment)) == 0,
           "views unchanged after a rejected prepare");

    expect(throws_invalid([] { qwen::RouteGroups too_big(1025); }), "chunk bound 1024");
    qwen::RouteGroups layerwise(16384, qwen::RouteGroups::Bound::layerwise16384);
    expect(throws_invalid([] { qwen::RouteGroups too_big(16385, qwen::RouteGroups::Bound::layerwise16384); }),
           "layerwise bound 16384");
    if (fails) return 1;
    std::cout << "ok\n";
    return 0;
}
