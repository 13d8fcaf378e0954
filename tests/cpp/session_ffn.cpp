// C++20 replay of the FFN section of the reference's Layer::ffn
// (src/session.hip:1412-1556) for a stack of MoE layers, through the C ABI
// of libqwen_moe_b200.so: one layer workspace shared by every layer (the
// reference's Session device buffers), one weights object per layer, the
// residual stream on the device.  Layer::ffn reads the normalised hidden
// state and its output is added into the residual; the normalisation belongs
// to the attention side of the session, so here the host applies an
// unweighted RMS norm (per token: h / sqrt(mean(h^2) + 1e-6)) to the
// residual to form each layer's input.  Per layer
//   * the router taps the reference records under a probe (router logits,
//     src/session.hip:1420-1428) -- here moe_router_logits, whose output the
//     test routes with;
//   * the trace capture of ffn_expert_down_unweighted_rank_N
//     (src/session.hip:1544-1553: rank N's unweighted down rows, stride
//     10*H over tokens) -- here moe_forward_contributions, which stores the
//     reference's [T][10][H] contribution layout and folds it in the
//     reference's rank order;
//   * the fast path: residual += ffn(input) with moe_forward_hidden
//     (router GEMM, routing, experts and the scatter-add on the device, no
//     host round trip), MOE_OUT_ACCUMULATE into the next residual buffer;
//   * the per-layer flag check (the reference's d.check after each layer's
//     router, src/session.hip:1425): moe_layer_read_flags, which fails the
//     run on any sticky flag.
//
//   session_ffn <dir>
//     meta.txt          hidden inter tokens layers seed
//     x0.bin            float [tokens][hidden], the first layer's input
//     router_<l>.bin    float [512][hidden], layer l's ffn_gate_inp
//     gate_<l>.bin      float [hidden], layer l's shared-expert gate vector
//   Expert weights of layer l are the library's seeded synthetic Q4_0
//   experts (moe_weights_synthesize(seed, l)).  Writes, per layer l,
//   res_<l>.bin (the residual before it), x_<l>.bin (its input),
//   logits_<l>.bin, det_<l>.bin (the trace-mode output, overwrite),
//   ffn_expert_down_unweighted_rank_<N>_<l>.bin (float [tokens][hidden]) and
//   res_<layers>.bin (the final residual); prints "ok".
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

#include "qwen_moe_b200.h"

namespace {
template <class T> std::vector<T> read_as(const std::string &path, size_t count) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot read " + path);
    std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (raw.size() != count * sizeof(T)) throw std::runtime_error("wrong size: " + path);
    std::vector<T> out(count);
    std::memcpy(out.data(), raw.data(), raw.size());
    return out;
}
void write_floats(const std::string &path, const float *p, size_t n) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char *>(p), static_cast<std::streamsize>(n * sizeof(float)));
    if (!f) throw std::runtime_error("cannot write " + path);
}
void moe(int status, const char *what) {
    if (status != MOE_OK) throw std::runtime_error(std::string(what) + ": " + moe_status_string(status));
}
void cuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Device buffer owned for the program's lifetime.
struct DeviceFloats {
    float *p = nullptr;
    explicit DeviceFloats(size_t n) { cuda(cudaMalloc(&p, n * sizeof(float)), "cudaMalloc"); }
    ~DeviceFloats() { cudaFree(p); }
    DeviceFloats(const DeviceFloats &) = delete;
    DeviceFloats &operator=(const DeviceFloats &) = delete;
};

std::vector<float> to_host(const float *dev, size_t n, cudaStream_t s) {
    std::vector<float> h(n);
    cuda(cudaMemcpyAsync(h.data(), dev, n * sizeof(float), cudaMemcpyDeviceToHost, s), "D2H");
    cuda(cudaStreamSynchronize(s), "sync");
    return h;
}

int run(const std::string &dir) {
    int H = 0, I = 0, T = 0, L = 0;
    unsigned long long seed = 0;
    {
        std::ifstream m(dir + "/meta.txt");
        if (!(m >> H >> I >> T >> L >> seed)) throw std::runtime_error("bad meta.txt");
    }
    const moe_layer_desc desc{H, I, 512, 10, 1, 0, T};
    cuda(cudaSetDevice(0), "cudaSetDevice");
    cudaStream_t stream;
    cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");

    std::vector<moe_weights_t> weights(L, nullptr);
    for (int l = 0; l < L; ++l) {
        moe(moe_weights_create(&desc, &weights[l]), "moe_weights_create");
        moe(moe_weights_synthesize(weights[l], seed, static_cast<uint32_t>(l), stream), "synthesize");
        const auto router = read_as<float>(dir + "/router_" + std::to_string(l) + ".bin", size_t(512) * H);
        const auto gate = read_as<float>(dir + "/gate_" + std::to_string(l) + ".bin", size_t(H));
        moe(moe_weights_upload_router(weights[l], router.data(), stream), "upload_router");
        moe(moe_weights_upload_shared_gate(weights[l], gate.data(), stream), "upload_shared_gate");
    }
    moe_layer_t layer = nullptr;
    moe(moe_layer_create(&desc, &layer), "moe_layer_create");

    const size_t n = size_t(T) * H;
    DeviceFloats res(n), xin(n), logits(size_t(T) * 512), contrib(size_t(T) * 10 * H), shared(n), det(n);
    {
        const auto x0 = read_as<float>(dir + "/x0.bin", n);
        cuda(cudaMemcpyAsync(res.p, x0.data(), n * sizeof(float), cudaMemcpyHostToDevice, stream), "H2D");
    }
    float *a = xin.p;
    for (int l = 0; l < L; ++l) {
        const std::string tag = "_" + std::to_string(l) + ".bin";
        // the layer's input: the RMS-normalised residual
        std::vector<float> h = to_host(res.p, n, stream);
        write_floats(dir + "/res" + tag, h.data(), n);
        for (int t = 0; t < T; ++t) {
            double ss = 0.0;
            for (int i = 0; i < H; ++i) ss += double(h[size_t(t) * H + i]) * h[size_t(t) * H + i];
            const float inv = static_cast<float>(1.0 / std::sqrt(ss / H + 1e-6));
            for (int i = 0; i < H; ++i) h[size_t(t) * H + i] *= inv;
        }
        cuda(cudaMemcpyAsync(a, h.data(), n * sizeof(float), cudaMemcpyHostToDevice, stream), "H2D");
        write_floats(dir + "/x" + tag, h.data(), n);
        // probe taps: router logits, then the deterministic trace pass
        moe(moe_router_logits(weights[l], a, T, logits.p, stream), "moe_router_logits");
        write_floats(dir + "/logits" + tag, to_host(logits.p, size_t(T) * 512, stream).data(), size_t(T) * 512);
        moe(moe_forward_contributions(layer, weights[l], a, logits.p, T, contrib.p, shared.p, det.p,
                                      MOE_OUT_OVERWRITE, stream),
            "moe_forward_contributions");
        const auto c = to_host(contrib.p, size_t(T) * 10 * H, stream);
        for (int rank = 0; rank < 10; ++rank) {
            std::vector<float> rows(n);   // rank's row of every token: offset rank*H, stride 10*H
            for (int t = 0; t < T; ++t)
                std::memcpy(rows.data() + size_t(t) * H, c.data() + (size_t(t) * 10 + rank) * H, H * sizeof(float));
            write_floats(dir + "/ffn_expert_down_unweighted_rank_" + std::to_string(rank) + tag, rows.data(), n);
        }
        write_floats(dir + "/det" + tag, to_host(det.p, n, stream).data(), n);
        // the fast path: residual += ffn(input), all on the device
        moe(moe_forward_hidden(layer, weights[l], a, T, res.p, MOE_OUT_ACCUMULATE, stream), "moe_forward_hidden");
        int flags = 0;
        moe(moe_layer_read_flags(layer, &flags, 1, stream), "moe_layer_read_flags");
        if (flags != 0) throw std::runtime_error("layer " + std::to_string(l) + " raised flags " + std::to_string(flags));
    }
    write_floats(dir + "/res_" + std::to_string(L) + ".bin", to_host(res.p, n, stream).data(), n);

    moe(moe_layer_destroy(layer), "moe_layer_destroy");
    for (auto w : weights) moe(moe_weights_destroy(w), "moe_weights_destroy");
    cuda(cudaStreamDestroy(stream), "stream destroy");
    return 0;
}
}  // namespace

int main(int argc, char **argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
        return 2;
    }
    try {
        if (run(argv[1]) != 0) return 1;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "FAILED: %s\n", e.what());
        return 1;
    }
    std::printf("ok\n");
    return 0;
}
