#!/usr/bin/env python3
"""Generate tests/golden/*.npz from the reference's own CPU code.

Run here, where the reference tree is mounted and oracle/build_ref.py has
built oracle/_ref/libqwen_ref{,_native}.so.  The fixtures travel with the
repository; nothing at test time needs the reference tree.

Fixtures:
* quant_cases.npz   -- float blocks from the reference's quantize tests
  (tests/quant_test.cpp:200-330: ties, raw-sum, original-scale, cancellation,
  tiny-scale cases) and random blocks, with the reference quantize_q8 bytes;
* expert_native.npz -- the reference cpu_expert test fixture
  (tests/cpu_expert_test.cpp:219-261: xorshift Q4_0 weights, sin/cos input)
  at the reference's 2560/640 shape: input Q8_1 bytes and run_cpu_expert
  'whole' outputs for 3 columns;
* expert_2048.npz   -- seeded synthetic weights (the repository generator) at
  2048/512 with run_cpu_expert outputs of the shape-patched reference build;
* routes.npz        -- RouteGroups::prepare on the reference test's fixture
  patterns (tests/routes_test.cpp:89-112) for several token counts;
* expert_q4_1.npz   -- Q4_1 down matrices: the reference cpu_expert test's
  Fixture(TensorType::Q4_1) at 2560/640 (tests/cpu_expert_test.cpp:219-261)
  and the repository's seeded Q4_1 generator at 2048/512, each with the
  reference run_cpu_expert 'whole' outputs, plus matmul_scalar outputs of a
  generated Q4_1 matrix.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402


def quant_cases():
    blocks = []
    z = np.array([-0.0 if i % 2 == 0 else 0.0 for i in range(32)], np.float32)
    blocks.append(z)
    v = np.zeros(32, np.float32)
    v[0] = 127.0
    v[1:9] = [0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 126.5, -126.5]
    blocks.append(v.copy())
    v[1] = np.nextafter(np.float32(0.5), np.float32(0.0))
    v[2] = -v[1]
    v[3] = np.nextafter(np.float32(0.5), np.float32(1.0))
    v[4] = -v[3]
    blocks.append(v.copy())
    v = np.full(32, 0.4, np.float32)
    v[0] = 127.0
    blocks.append(v)
    v = np.zeros(32, np.float32)
    v[0] = 1.0
    v[1] = np.nextafter(np.float32(1.0 / 127.0) * np.float32(0.5), np.float32(0.0))
    blocks.append(v)
    v = np.zeros(32, np.float32)
    v[0], v[1], v[2], v[3] = 1048576.0, 0.03125, -1048576.0, 0.03125
    blocks.append(v)
    v = np.zeros(32, np.float32)
    v[0] = np.float32(127.0) * np.nextafter(np.float32(2.0 ** -25), np.float32(1.0))
    v[1] = -v[0]
    blocks.append(v)
    for sign in (1.0, -1.0):
        blocks.append(np.full(32, sign * 3.4e-6, np.float32))
        v = np.zeros(32, np.float32)
        v[0], v[1], v[2], v[3] = sign * 3.4e-6, -sign * 3.4e-6, sign * 3.4e-6 * 0.4, -sign * 3.4e-6 * 0.1
        blocks.append(v)
    rng = np.random.default_rng(20240601)
    for _ in range(256):
        blocks.append((rng.integers(-100000, 100001, 32) / 4096.0).astype(np.float32))
    for _ in range(64):
        blocks.append((rng.standard_normal(32) * 10.0 ** rng.uniform(-6, 3)).astype(np.float32))
    x = np.stack(blocks).astype(np.float32)
    R = O.ref()
    out = np.zeros(len(blocks), O.Q8_DTYPE)
    for i in range(len(blocks)):
        st = R.ref_quantize_q8(O.ptr(x[i]), 32, O.ptr(out[i:i + 1]))
        assert st == 0, R.ref_last_message()
    return dict(x=x, q8=out.view(np.uint8).reshape(len(blocks), 36))


def expert_native():
    RN = O.ref_native()
    H, I = 2560, 640
    gate = O.fixture_xorshift_q4_0(0x70af451, I, H // 32)
    up = O.fixture_xorshift_q4_0(0xa5f726e, I, H // 32)
    down = O.fixture_xorshift_q4_0(0x525a31, H, I // 32)
    floats = (np.float32(0.7) * np.sin(np.arange(10240, dtype=np.float32) * np.float32(0.137)).astype(np.float32)
              + np.float32(0.2) * np.cos(np.arange(10240, dtype=np.float32) * np.float32(0.071)).astype(np.float32))
    floats = floats.astype(np.float32)
    q = np.zeros(320, O.Q8_DTYPE)
    assert RN.ref_quantize_q8(O.ptr(floats), floats.size, O.ptr(q)) == 0
    starts = [0, 160, 80]
    h = RN.ref_expert_new(O.ptr(gate), O.ptr(up), O.ptr(down), gate.size, down.size, H, I)
    assert h, RN.ref_last_message()
    cols = np.ascontiguousarray(np.stack([q[s:s + 80] for s in starts]))
    ptrs = (ctypes.c_void_p * 3)(*[cols[c].ctypes.data for c in range(3)])
    out = np.zeros(3 * H, np.float32)
    assert RN.ref_run_cpu_expert(h, 3, ptrs, 80, 0, O.ptr(out), out.size) == 0
    RN.ref_expert_free(h)
    return dict(xq=cols.view(np.uint8).reshape(3, 80 * 36), out=out.reshape(3, H))


def expert_2048():
    R = O.ref()
    H, I, seed = 2048, 512, 77
    g, u, d = O.synth_expert(seed, 3, 17)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, H)).astype(np.float32)
    q = np.zeros((3, H // 32), O.Q8_DTYPE)
    for c in range(3):
        assert R.ref_quantize_q8(O.ptr(x[c]), H, O.ptr(q[c])) == 0
    h = R.ref_expert_new(O.ptr(g), O.ptr(u), O.ptr(d), g.size, d.size, H, I)
    assert h, R.ref_last_message()
    ptrs = (ctypes.c_void_p * 3)(*[q[c].ctypes.data for c in range(3)])
    out = np.zeros(3 * H, np.float32)
    assert R.ref_run_cpu_expert(h, 3, ptrs, H // 32, 0, O.ptr(out), out.size) == 0
    R.ref_expert_free(h)
    return dict(seed=np.array([seed, 3, 17]), x=x, xq=q.view(np.uint8).reshape(3, H // 32 * 36),
                out=out.reshape(3, H))


def _run_expert(R, g, u, d, down_type, H, I, cols):
    h = R.ref_expert_new_typed(O.ptr(g), O.ptr(u), O.ptr(d), down_type, g.size, d.size, H, I)
    assert h, R.ref_last_message()
    ptrs = (ctypes.c_void_p * 3)(*[cols[c].ctypes.data for c in range(3)])
    out = np.zeros(3 * H, np.float32)
    assert R.ref_run_cpu_expert(h, 3, ptrs, H // 32, 0, O.ptr(out), out.size) == 0, R.ref_last_message()
    R.ref_expert_free(h)
    return out.reshape(3, H)


def expert_q4_1():
    out = {}
    # reference fixture, native shape
    RN = O.ref_native()
    H, I = 2560, 640
    gate = O.fixture_xorshift_q4_0(0x70af451, I, H // 32)
    up = O.fixture_xorshift_q4_0(0xa5f726e, I, H // 32)
    down = O.fixture_xorshift_q4_1(0x525a31, H, I // 32)
    floats = (np.float32(0.7) * np.sin(np.arange(10240, dtype=np.float32) * np.float32(0.137)).astype(np.float32)
              + np.float32(0.2) * np.cos(np.arange(10240, dtype=np.float32) * np.float32(0.071)).astype(np.float32))
    floats = np.ascontiguousarray(floats, dtype=np.float32)
    q = np.zeros(320, O.Q8_DTYPE)
    assert RN.ref_quantize_q8(O.ptr(floats), floats.size, O.ptr(q)) == 0
    cols = np.ascontiguousarray(np.stack([q[s:s + 80] for s in (0, 160, 80)]))
    out["native_xq"] = cols.view(np.uint8).reshape(3, 80 * 36)
    out["native_out"] = _run_expert(RN, gate, up, down, 3, H, I, cols)
    # repository generator, 2048/512
    R = O.ref()
    H, I, seed = 2048, 512, 41
    g, u, d = O.synth_expert(seed, 2, 33, down_type=O.Q4_1)
    x = np.random.default_rng(9).standard_normal((3, H)).astype(np.float32)
    q = np.zeros((3, H // 32), O.Q8_DTYPE)
    for c in range(3):
        assert R.ref_quantize_q8(O.ptr(x[c]), H, O.ptr(q[c])) == 0
    out["seed"] = np.array([seed, 2, 33])
    out["x"] = x
    out["out"] = _run_expert(R, g, u, d, 3, H, I, q)
    # matmul_scalar of one generated Q4_1 matrix (rows 2048, K 512)
    w = O.synth_q4_1(5, 1, 2, 2, 2048, 16)
    xm = np.random.default_rng(10).standard_normal((3, 512)).astype(np.float32)
    qm = np.zeros((3, 16), O.Q8_DTYPE)
    for c in range(3):
        assert R.ref_quantize_q8(O.ptr(xm[c]), 512, O.ptr(qm[c])) == 0
    mo = np.zeros(3 * 2048, np.float32)
    assert R.ref_matmul(0, 3, 512, 2048, O.ptr(w), w.size, O.ptr(qm), qm.size, 3, O.ptr(mo), mo.size) == 0
    out["matmul_x"] = xm
    out["matmul_out"] = mo.reshape(3, 2048)
    return out


def route_fixture(tokens, pattern):
    # tests/routes_test.cpp:89-112
    repeated = [511, 0, 510, 1, 127, 255, 256, 257, 400, 41]
    bits = [0, 0x80000000, 1, 0x007fffff, 0x00800000, 0x3dcccccd, 0x3f800000, 0x7f7fffff, 0x3f000001, 0x4f123456]
    ids = np.empty(tokens * 10, np.int32)
    raw = np.empty(tokens * 10, np.uint32)
    for t in range(tokens):
        for r in range(10):
            i = t * 10 + r
            ids[i] = (511 + 37 * t + 73 * r) % 512 if pattern == 0 else repeated[(r + 3 * t) % 10]
            raw[i] = ((0 if (t + r) % 2 == 0 else 0x80000000) if pattern == 2 else bits[(11 * t + 3 * r) % 10])
    return ids, raw.view(np.float32)


def routes():
    R = O.ref()
    result = {}
    for tokens in (1, 2, 3, 37, 128):
        for pattern in (0, 1, 2):
            ids, w = route_fixture(tokens, pattern)
            h = R.ref_routes_new(128, 0)
            assert R.ref_routes_prepare(h, O.ptr(ids), O.ptr(w), ids.size, tokens) == 0, R.ref_last_message()
            a = np.zeros(ids.size, O.ASSIGN_DTYPE)
            n = R.ref_routes_assignments(h, O.ptr(a), a.size)
            c = np.zeros(512, np.int32)
            R.ref_routes_counts(h, O.ptr(c))
            R.ref_routes_free(h)
            assert n == ids.size
            key = f"t{tokens}_p{pattern}"
            result[key + "_ids"] = ids
            result[key + "_weights"] = w
            result[key + "_assign"] = a.view(np.int32).reshape(-1, 4)
            result[key + "_counts"] = c
    return result


def main():
    if O.ref() is None or O.ref_native() is None:
        raise SystemExit("oracle/_ref is not built: run python oracle/build_ref.py first")
    np.savez_compressed(os.path.join(HERE, "quant_cases.npz"), **quant_cases())
    np.savez_compressed(os.path.join(HERE, "expert_native.npz"), **expert_native())
    np.savez_compressed(os.path.join(HERE, "expert_2048.npz"), **expert_2048())
    np.savez_compressed(os.path.join(HERE, "routes.npz"), **routes())
    np.savez_compressed(os.path.join(HERE, "expert_q4_1.npz"), **expert_q4_1())
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
