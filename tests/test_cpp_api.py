"""The C++20 host API headers at the reference's names (include/qwen/*.hpp, namespace
qwen, over include/qmoe/*.hpp and the C ABI): qwen::GpuExpert exercised by
tests/cpp/gpu_expert_api.cpp the way the reference's own GpuExpert is used
(src/gpu_expert.hpp, src/hip/expert.hip:183-241), and qwen::RouteGroups by
tests/cpp/routes_api.cpp (src/routes.hpp:18-65).

CPU: the program compiles as C++20 and links against libqwen_moe_b200.so.
GPU: it runs on oracle fixtures (Q4_0 and Q4_1 down) and its outputs match
the oracle (projection gate 2e-4 + 2e-5*|ref|, expert output 1e-3 * RMS)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gfx906-qwen3.8fn_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "gpu_expert_api.cpp")


def build_program(out_dir, src=SRC, name="gpu_expert_api"):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    exe = os.path.join(out_dir, name)
    # include/qwen/ first, as a caller of the reference's headers would put it
    cmd = [cxx, "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include", "qwen"), src,
           "-L", PKG, "-lqwen_moe_b200", f"-Wl,-rpath,{PKG}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_gpu_expert_header_compiles_and_links(pkg, tmp_path):
    assert os.path.exists(build_program(str(tmp_path)))


def test_route_groups_drop_in_header(pkg, tmp_path):
    """qwen::RouteGroups through include/qwen/routes.hpp: grouping order, raw
    weight bits, validation before mutation (host code, no GPU needed)."""
    exe = build_program(str(tmp_path), os.path.join(ROOT, "tests", "cpp", "routes_api.cpp"), "routes_api")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("down_type", [2, 3])
def test_gpu_expert_cpp_api(pkg, O, tmp_path, down_type):
    exe = build_program(str(tmp_path))
    H, I, cols = 2048, 512, 3
    g, u, d = O.synth_expert(6, 1, 2, down_type=down_type)
    rng = np.random.default_rng(down_type)
    x = rng.standard_normal((cols, H)).astype(np.float32)
    xq, _ = O.quantize(x)
    mid, _ = O.quantize(rng.standard_normal((cols, I)).astype(np.float32))
    files = dict(gate=g, up=u, down=d, x=x, xq=xq, mid=mid)
    for name, a in files.items():
        np.ascontiguousarray(a).tofile(os.path.join(tmp_path, name + ".bin"))
    with open(os.path.join(tmp_path, "meta.txt"), "w") as f:
        f.write(f"{H} {I} {cols} {down_type}\n")
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr
    got_gate = np.fromfile(os.path.join(tmp_path, "gate_out.bin"), np.float32).reshape(cols, I)
    ref = O.matrix_serial(g, xq, I, H // 32)
    assert np.all(np.abs(got_gate - ref) <= 2e-4 + 2e-5 * np.abs(ref))
    got_down = np.fromfile(os.path.join(tmp_path, "down_out.bin"), np.float32).reshape(cols, H)
    ref = (O.matrix_serial_q4_1 if down_type == 3 else O.matrix_serial)(d, mid, H, I // 32)
    assert np.all(np.abs(got_down - ref) <= 2e-4 + 2e-5 * np.abs(ref))
    y = np.fromfile(os.path.join(tmp_path, "run_out.bin"), np.float32).reshape(cols, H)
    want, _ = O.expert_whole(g, u, d, xq, down_type=down_type)
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    assert float(np.max(np.abs(y - want))) <= 1e-3 * rms
