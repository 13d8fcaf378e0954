// ref_shim.cpp -- C entry points over the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/build_ref.py together with the
// reference's src/routes.cpp, src/quant.cpp, src/model.cpp and src/cpu_expert.cpp
// (the last one shape-patched for the 2048/512 build) into oracle/_ref/*.so.
// Used by tests/ to pin the oracle restatement, and by bench.py as the timed
// CPU baseline (the reference's CpuExpertPool on the host cores).  No product
// code loads it.
#include "cpu_expert.hpp"
#include "quant.hpp"
#include "routes.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <new>
#include <span>
#include <stdexcept>

using namespace qwen;

namespace {
thread_local char last_message[256];
void remember(const std::exception& e) {
    std::strncpy(last_message, e.what(), sizeof(last_message) - 1);
    last_message[sizeof(last_message) - 1] = 0;
}
QMatrix view(int type, int input, int output, const void* w, std::size_t bytes) {
    return {static_cast<TensorType>(type), input, output,
            std::span<const std::byte>(static_cast<const std::byte*>(w), bytes)};
}
}  // namespace

extern "C" {

const char* ref_last_message() { return last_message; }

int ref_shape_hidden() {
    // The patched build validates [hidden, inter] gate/up views; report what it accepts.
    return sizeof(CpuExpertScratch::down) / sizeof(float) / 3;
}
int ref_shape_inter() { return sizeof(CpuExpertScratch::gate) / sizeof(float) / 3; }

float ref_half_to_float(std::uint16_t h) { return half_to_float(h); }
std::uint16_t ref_float_to_half(float f) { return float_to_half(f); }

// 0 ok, 1 invalid_argument (reference throws), 2 other
int ref_quantize_q8(const float* input, std::size_t n, void* output) {
    try {
        quantize_q8({input, n}, {static_cast<Q8_1*>(output), n / 32});
        return 0;
    } catch (const std::invalid_argument& e) { remember(e); return 1; }
    catch (const std::exception& e) { remember(e); return 2; }
}

int ref_matmul(int avx2, int type, int input, int output, const void* w, std::size_t wbytes,
               const void* x, std::size_t nx, int columns, float* out, std::size_t nout) {
    try {
        const auto m = view(type, input, output, w, wbytes);
        std::span<const Q8_1> xs(static_cast<const Q8_1*>(x), nx);
        std::span<float> os(out, nout);
        if (avx2) matmul_avx2(m, xs, columns, os);
        else matmul_scalar(m, xs, columns, os);
        return 0;
    } catch (const std::invalid_argument& e) { remember(e); return 1; }
    catch (const std::exception& e) { remember(e); return 2; }
}

float ref_dot(int avx2, int type, const void* block, const void* activation) {
    const auto& a = *static_cast<const Q8_1*>(activation);
    return avx2 ? dot_q4_avx2(block, static_cast<TensorType>(type), a)
                : dot_q4_scalar(block, static_cast<TensorType>(type), a);
}

void* ref_routes_new(int capacity, int layerwise) {
    try {
        return new RouteGroups(capacity, layerwise ? RouteGroups::Bound::layerwise16384
                                                   : RouteGroups::Bound::chunk1024);
    } catch (const std::exception& e) { remember(e); return nullptr; }
}
void ref_routes_free(void* h) { delete static_cast<RouteGroups*>(h); }
int ref_routes_prepare(void* h, const std::int32_t* ids, const float* weights, std::size_t n,
                       int tokens) {
    try {
        static_cast<RouteGroups*>(h)->prepare({ids, n}, {weights, n}, tokens);
        return 0;
    } catch (const std::invalid_argument& e) { remember(e); return 1; }
    catch (const std::exception& e) { remember(e); return 2; }
}
// 16-byte RouteAssignment records {token, rank, expert, weight}.
std::size_t ref_routes_assignments(void* h, void* out, std::size_t capacity) {
    const auto a = static_cast<RouteGroups*>(h)->assignments();
    const auto n = a.size() < capacity ? a.size() : capacity;
    std::memcpy(out, a.data(), n * sizeof(RouteAssignment));
    return a.size();
}
void ref_routes_counts(void* h, int* out) {
    const auto c = static_cast<RouteGroups*>(h)->counts();
    std::memcpy(out, c.data(), c.size() * sizeof(int));
}

void* ref_expert_new(const void* gate, const void* up, const void* down, std::size_t gate_bytes,
                     std::size_t down_bytes, int hidden, int inter) {
    try {
        return new CpuExpert(view(2, hidden, inter, gate, gate_bytes),
                             view(2, hidden, inter, up, gate_bytes),
                             view(2, inter, hidden, down, down_bytes));
    } catch (const std::exception& e) { remember(e); return nullptr; }
}
// down_type: the reference's TensorType value of the down matrix (2 Q4_0, 3 Q4_1).
void* ref_expert_new_typed(const void* gate, const void* up, const void* down, int down_type,
                           std::size_t gate_bytes, std::size_t down_bytes, int hidden, int inter) {
    try {
        return new CpuExpert(view(2, hidden, inter, gate, gate_bytes),
                             view(2, hidden, inter, up, gate_bytes),
                             view(down_type, inter, hidden, down, down_bytes));
    } catch (const std::exception& e) { remember(e); return nullptr; }
}
void ref_expert_free(void* h) { delete static_cast<CpuExpert*>(h); }

// CpuExpertStatus as int. inputs: `columns` pointers to Q8_1 spans of
// blocks_per_column blocks.  stage 0 whole, 1 gate_up, 2 down.
int ref_run_cpu_expert(void* expert, int columns, const void* const* inputs,
                       std::size_t blocks_per_column, int stage, float* out, std::size_t nout) {
    CpuExpertJob job;
    job.expert = static_cast<const CpuExpert*>(expert);
    job.columns = columns;
    for (int c = 0; c < columns && c < 3; ++c)
        job.input[c] = {static_cast<const Q8_1*>(inputs[c]), blocks_per_column};
    job.output = {out, nout};
    job.stage = static_cast<CpuExpertStage>(stage);
    auto* scratch = new (std::align_val_t(64)) CpuExpertScratch;
    const auto status = run_cpu_expert(job, *scratch);
    ::operator delete(scratch, std::align_val_t(64));
    return static_cast<int>(status);
}

int ref_allowed_physical_cpus(int* dest, std::size_t capacity, std::size_t* count) {
    return static_cast<int>(cpu_expert_allowed_physical_cpus({dest, capacity}, *count));
}

void* ref_pool_new(std::size_t workers, int pin, const int* cpus, std::size_t ncpus) {
    try {
        CpuExpertPoolConfig config;
        config.workers = workers;
        config.pin_workers = pin != 0;
        if (pin) config.cpus = {cpus, ncpus};
        return new CpuExpertPool(config);
    } catch (const std::exception& e) { remember(e); return nullptr; }
}
void ref_pool_free(void* p) { delete static_cast<CpuExpertPool*>(p); }

// Job descriptors must stay alive until drain: the pool copies the descriptor,
// but inputs/outputs are borrowed.  Returns CpuExpertStatus as int.
int ref_pool_submit(void* pool, void* expert, int columns, const void* const* inputs,
                    std::size_t blocks_per_column, int stage, float* out, std::size_t nout,
                    std::size_t* ticket) {
    CpuExpertJob job;
    job.expert = static_cast<const CpuExpert*>(expert);
    job.columns = columns;
    for (int c = 0; c < columns && c < 3; ++c)
        job.input[c] = {static_cast<const Q8_1*>(inputs[c]), blocks_per_column};
    job.output = {out, nout};
    job.stage = static_cast<CpuExpertStage>(stage);
    return static_cast<int>(static_cast<CpuExpertPool*>(pool)->submit(job, *ticket));
}
int ref_pool_drain(void* pool) { return static_cast<int>(static_cast<CpuExpertPool*>(pool)->drain()); }
int ref_pool_reset(void* pool) { return static_cast<int>(static_cast<CpuExpertPool*>(pool)->reset()); }

}  // extern "C"
