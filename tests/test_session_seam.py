"""The Session integration seam: the FFN section of the reference's Layer::ffn
(src/session.hip:1412-1556) replayed by a C++20 host program
(tests/cpp/session_ffn.cpp) over a stack of layers through the C ABI, with
the residual stream on the device, the router-logit and
ffn_expert_down_unweighted_rank_N trace taps (src/session.hip:1420-1428,
1544-1553) and the per-layer flag check.

CPU: the program compiles as C++20 against include/qwen_moe_b200.h and the
CUDA runtime and links against libqwen_moe_b200.so.
The program forms each layer's input as the unweighted RMS norm of the
residual (the session's pre-FFN norm, which is not on this path) and adds the
FFN output into the residual.
GPU: every layer is checked against the oracle on that layer's own input (the
normalised residual the program fed it) and router logits:
* the logits against fp64 within an fp32 accumulation bound (the reference's
  router is a BLAS GEMM of unspecified order);
* the fast path's residual update res[l+1] - res[l] and the trace pass's
  output against the oracle layer within 1e-3 * RMS;
* each rank's unweighted down rows against the oracle's CPU expert for that
  token's expert of that rank (1e-3 * RMS), the trace layout of the reference.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

from cases import assert_close

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gfx906-qwen3.8fn_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "session_ffn.cpp")
H, I, E = 2048, 512, 512
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build_program(out_dir):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    inc, lib = os.path.join(CUDA_HOME, "include"), os.path.join(CUDA_HOME, "lib64")
    if not os.path.exists(os.path.join(inc, "cuda_runtime.h")):
        pytest.skip("no CUDA runtime headers")
    exe = os.path.join(out_dir, "session_ffn")
    cmd = [cxx, "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), "-I", inc,
           SRC, "-L", PKG, "-lqwen_moe_b200", f"-Wl,-rpath,{PKG}", "-L", lib, "-lcudart", f"-Wl,-rpath,{lib}",
           "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_session_program_compiles_and_links(pkg, tmp_path):
    assert os.path.exists(build_program(str(tmp_path)))


@pytest.mark.gpu
@pytest.mark.parametrize("T", [8, 64])
def test_session_layer_stack(pkg, O, tmp_path, T):
    L, seed = 4, 4100 + T
    exe = build_program(str(tmp_path))
    rng = np.random.default_rng(seed)
    x0 = rng.standard_normal((T, H)).astype(np.float32)
    routers = [(rng.standard_normal((E, H)) * 0.02).astype(np.float32) for _ in range(L)]
    gates = [(rng.standard_normal(H) * 0.02).astype(np.float32) for _ in range(L)]
    x0.tofile(os.path.join(tmp_path, "x0.bin"))
    for l in range(L):
        routers[l].tofile(os.path.join(tmp_path, f"router_{l}.bin"))
        gates[l].tofile(os.path.join(tmp_path, f"gate_{l}.bin"))
    with open(os.path.join(tmp_path, "meta.txt"), "w") as f:
        f.write(f"{H} {I} {T} {L} {seed}\n")
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr

    def load(name, shape):
        return np.fromfile(os.path.join(tmp_path, name), np.float32).reshape(shape)

    res = [load(f"res_{l}.bin", (T, H)) for l in range(L + 1)]
    assert np.array_equal(res[0], x0)
    for l in range(L):
        x, lg = load(f"x_{l}.bin", (T, H)), load(f"logits_{l}.bin", (T, E))
        r64 = res[l].astype(np.float64)
        want_x = r64 / np.sqrt(np.mean(r64 ** 2, axis=1, keepdims=True) + 1e-6)
        assert np.max(np.abs(x - want_x)) <= 1e-5 * np.max(np.abs(want_x)), f"layer {l} input norm"
        ref64 = x.astype(np.float64) @ routers[l].astype(np.float64).T
        bound = 2e-5 * (np.abs(x).astype(np.float64) @ np.abs(routers[l]).astype(np.float64).T)
        assert np.all(np.abs(lg - ref64) <= bound), f"layer {l} router logits"
        want, ids, _, flags = O.moe_layer(x, lg, lambda e: O.synth_expert(seed, l, e), O.synth_expert(seed, l, 512),
                                          gates[l], threads=8)
        assert flags == 0
        ffn = (res[l + 1].astype(np.float64) - res[l]).astype(np.float32)
        assert_close(ffn, want)
        assert_close(load(f"det_{l}.bin", (T, H)), want)
        xq, _ = O.quantize(x)
        for rank in range(10):
            rows = load(f"ffn_expert_down_unweighted_rank_{rank}_{l}.bin", (T, H))
            for t in range(2):
                y, _ = O.expert_whole(*O.synth_expert(seed, l, int(ids[t, rank])), xq[t:t + 1])
                assert_close(rows[t][None], y)
