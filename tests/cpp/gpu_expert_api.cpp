// C++20 exercise of qwen::GpuExpert (include/qwen/gpu_expert.hpp, a drop-in for the
// reference's src/gpu_expert.hpp implemented by include/qmoe/gpu_expert.hpp) with the
// reference GpuExpert's calls and error behaviour (src/gpu_expert.hpp,
// src/hip/expert.hip:183-241).  Reads fixtures written by
// tests/test_cpp_api.py into <dir>, writes the GPU results back there.
//
//   gpu_expert_api <dir>
//     meta.txt   hidden inter columns down_type
//     gate.bin up.bin down.bin   canonical weight bytes
//     x.bin      float [columns][hidden]
//     xq.bin     Q8_1 [columns][hidden/32] (expected quantisation)
//     mid.bin    Q8_1 [columns][inter/32]  (input of the down projection)
//   writes gate_out.bin (float [columns][inter]), down_out.bin (float
//   [columns][hidden]), run_out.bin (float [columns][hidden]); prints "ok".
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

#include "gpu_expert.hpp"   // include/qwen/: the reference's header name and namespace

namespace {
std::vector<std::byte> read_file(const std::string &path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot read " + path);
    std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<std::byte> out(raw.size());
    std::memcpy(out.data(), raw.data(), raw.size());
    return out;
}
template <class T> std::vector<T> read_as(const std::string &path) {
    const auto b = read_file(path);
    std::vector<T> out(b.size() / sizeof(T));
    std::memcpy(out.data(), b.data(), out.size() * sizeof(T));
    return out;
}
template <class T> void write_file(const std::string &path, const std::vector<T> &v) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char *>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
}
template <class E, class F> bool throws(F &&f) {
    try {
        f();
    } catch (const E &) {
        return true;
    } catch (...) {
        return false;
    }
    return false;
}
int fail(const char *what) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    return 1;
}
}  // namespace

int main(int argc, char **argv) {
    if (argc != 2) return fail("usage: gpu_expert_api <dir>");
    const std::string dir = argv[1];
    int H = 0, I = 0, cols = 0, down_type = 2;
    std::ifstream(dir + "/meta.txt") >> H >> I >> cols >> down_type;
    const auto gate = read_file(dir + "/gate.bin"), up = read_file(dir + "/up.bin"), down = read_file(dir + "/down.bin");
    const auto x = read_as<float>(dir + "/x.bin");
    const auto xq = read_as<qwen::Q8_1>(dir + "/xq.bin");
    const auto mid = read_as<qwen::Q8_1>(dir + "/mid.bin");
    const auto dt = static_cast<qwen::TensorType>(down_type);
    const qwen::QMatrix g{qwen::TensorType::Q4_0, H, I, gate}, u{qwen::TensorType::Q4_0, H, I, up}, d{dt, I, H, down};

    // constructor checks: shape/type and byte size, before any device work
    if (!throws<std::invalid_argument>([&] { qwen::GpuExpert(g, u, g, 0, cols, true); }))
        return fail("mismatched down shape accepted");
    if (!throws<std::invalid_argument>([&] { qwen::GpuExpert(g, u, d, 0, 0, true); }))
        return fail("zero max_columns accepted");
    const qwen::QMatrix short_gate{qwen::TensorType::Q4_0, H, I, std::span(gate).first(gate.size() - 1)};
    if (!throws<std::invalid_argument>([&] { qwen::GpuExpert(short_gate, u, d, 0, cols, true); }))
        return fail("short weight span accepted");

    qwen::GpuExpert expert(g, u, d, 0, cols, true);
    expert.check_quantization(x, xq);
    auto bad = xq;
    bad[0].qs[0] ^= 1;
    if (!throws<std::runtime_error>([&] { expert.check_quantization(x, bad); })) return fail("Q8_1 mismatch not reported");
    if (!throws<std::invalid_argument>([&] { expert.check_quantization(std::span(x).first(31), xq); }))
        return fail("ragged quantization span accepted");

    std::vector<float> gate_out(static_cast<std::size_t>(cols) * I), down_out(static_cast<std::size_t>(cols) * H),
        run_out(static_cast<std::size_t>(cols) * H);
    expert.linear(false, false, xq, cols, gate_out);
    expert.linear(true, false, mid, cols, down_out);
    if (!throws<std::invalid_argument>([&] { expert.linear(true, false, xq, cols, down_out); }))
        return fail("wrong linear input extent accepted");
    const auto timing = expert.run(x, cols, run_out, 3);
    if (!(timing.resident_ms > 0.0)) return fail("no resident time");
    write_file(dir + "/gate_out.bin", gate_out);
    write_file(dir + "/down_out.bin", down_out);
    write_file(dir + "/run_out.bin", run_out);
    std::printf("ok upload_ms=%.3f resident_ms=%.4f\n", timing.upload_ms, timing.resident_ms);
    return 0;
}
