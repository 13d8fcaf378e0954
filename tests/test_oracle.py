"""CPU tests: the oracle restatement pinned against the reference's own code
(oracle/_ref, when built) and against the committed golden vectors."""
import math

import numpy as np
import pytest

from conftest import golden


def _ref_or_skip(O, native=False):
    r = O.ref_native() if native else O.ref()
    if r is None:
        pytest.skip("reference CPU build (oracle/_ref) not present")
    return r


def test_half_conversion_exhaustive(O):
    L = O.lib()
    # decode: every half against the mathematical definition
    for h in range(0, 65536, 1):
        e, m = (h >> 10) & 31, h & 1023
        v = L.o_half_to_float(h)
        if e == 31:
            assert (math.isinf(v) if m == 0 else math.isnan(v))
            continue
        want = math.ldexp(m, -24) if e == 0 else math.ldexp(1024 + m, e - 25)
        assert v == (-want if h & 0x8000 else want) and math.copysign(1, v) == (-1 if h & 0x8000 else 1)
    # encode: round trip of every finite half and RNE at every midpoint
    vals = np.array([L.o_half_to_float(h) for h in range(0x7c00)], np.float64)
    for h in range(0, 0x7bff, 7):
        assert L.o_float_to_half(float(vals[h])) == h
        mid = np.float32((vals[h] + vals[h + 1]) / 2)
        even = h + (h & 1)
        assert L.o_float_to_half(float(mid)) == even
        assert L.o_float_to_half(float(np.nextafter(mid, np.float32(0)))) == h
        assert L.o_float_to_half(float(np.nextafter(mid, np.float32(np.inf)))) == h + 1
    assert L.o_float_to_half(65519.0) == 0x7bff and L.o_float_to_half(65520.0) == 0x7c00


def test_half_conversion_matches_reference(O):
    R = _ref_or_skip(O)
    L = O.lib()
    rng = np.random.default_rng(3)
    for f in rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32):
        assert L.o_float_to_half(float(f)) == R.ref_float_to_half(float(f))


def test_quantize_golden_cases(O):
    g = golden("quant_cases.npz")
    q, flags = O.quantize(g["x"])
    assert flags == 0
    assert np.array_equal(q.view(np.uint8).reshape(-1, 36), g["q8"])


def test_quantize_reference_tie_and_raw_sum_rules(O):
    # tests/quant_test.cpp:206-240: ties away from zero, raw float sum kept
    v = np.zeros(32, np.float32)
    v[0] = 127.0
    v[1:9] = [0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 126.5, -126.5]
    q, _ = O.quantize(v)
    assert list(q[0]["qs"][1:9]) == [1, -1, 2, -2, 3, -3, 127, -127]
    v = np.full(32, 0.4, np.float32)
    v[0] = 127.0
    q, _ = O.quantize(v)
    assert q[0]["s"] == O.lib().o_float_to_half(139.4)
    # tiny scale: stored half d == 0 keeps codes and raw sum (quant_test.cpp:336-356)
    q, f = O.quantize(np.full(32, 3.4e-6, np.float32))
    assert f == 0 and q[0]["d"] == 0 and all(c == 127 for c in q[0]["qs"]) and q[0]["s"] != 0


def test_quantize_invalid_blocks_flag_and_zero(O):
    for bad in (np.inf, -np.inf, np.nan):
        v = np.ones(32, np.float32)
        v[5] = bad
        q, f = O.quantize(v)
        assert f & 1 and not q.view(np.uint8).any()
    v = np.zeros(32, np.float32)
    v[0] = np.float32(1e-45)  # original FP32 scale underflows to zero
    q, f = O.quantize(v)
    assert f & 2 and not q.view(np.uint8).any()
    q, f = O.quantize(np.full(32, 3000.0, np.float32))  # raw sum overflows half
    assert f & 2 and not q.view(np.uint8).any()


def test_literal_matrix_known_answer(O):
    # tests/quant_test.cpp:572-603: Q4_0 expected {-96, -224, -6120, -24552}
    x = np.zeros(2, O.Q8_DTYPE)
    x["d"] = 0x3c00
    x[0]["s"], x[1]["s"] = 0x4000, 0xc200
    x[0]["qs"] = [3] * 16 + [-4] * 16
    x[1]["qs"] = [-128] * 32
    w = np.zeros((2, 18), np.uint8)
    for row, code in ((0, 0x21), (1, 0x75)):
        w[row, 0:2] = [0x00, 0x3c]
        w[row, 2:] = code
    out = O.matrix_serial(w.ravel(), x, 2, 1)
    assert out.ravel().tolist() == [-96.0, -224.0, -6120.0, -24552.0]
    assert O.matrix_mmvq(w.ravel(), x, 2, 1).ravel().tolist() == [-96.0, -224.0, -6120.0, -24552.0]


def test_block_dot_full_range(O):
    # tests/quant_test.cpp:404-418: every nibble against every int8 code
    L = O.lib()
    for code in range(16):
        w = np.full(16, code * 17, np.uint8)
        for val in range(-128, 128, 5):
            qs = np.full(32, val, np.int8)
            assert L.o_block_dot(O.ptr(w), O.ptr(qs)) == 32 * code * val


def test_matrix_serial_matches_reference(O):
    R = _ref_or_skip(O)
    rng = np.random.default_rng(11)
    for rows, blocks in ((512, 64), (2048, 16), (7, 3)):
        w = O.synth_q4_0(9, 0, 1, 2, rows, blocks)
        xq, _ = O.quantize(rng.standard_normal((3, blocks * 32)).astype(np.float32))
        a = O.matrix_serial(w, xq, rows, blocks)
        out = np.zeros(3 * rows, np.float32)
        assert R.ref_matmul(0, 2, blocks * 32, rows, O.ptr(w), w.size, O.ptr(xq), xq.size, 3, O.ptr(out), out.size) == 0
        assert np.array_equal(a.ravel().view(np.uint32), out.view(np.uint32))


def test_expert_whole_matches_reference_native_fixture(O):
    g = golden("expert_native.npz")
    H, I = 2560, 640
    gate = O.fixture_xorshift_q4_0(0x70af451, I, H // 32)
    up = O.fixture_xorshift_q4_0(0xa5f726e, I, H // 32)
    down = O.fixture_xorshift_q4_0(0x525a31, H, I // 32)
    xq = np.ascontiguousarray(g["xq"]).view(O.Q8_DTYPE).reshape(3, 80)
    out, flags = O.expert_whole(gate, up, down, xq, H, I)
    assert flags == 0
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))


def test_expert_whole_matches_patched_reference_2048(O):
    g = golden("expert_2048.npz")
    seed, layer, expert = (int(v) for v in g["seed"])
    gate, up, down = O.synth_expert(seed, layer, expert)
    xq, _ = O.quantize(g["x"])
    assert np.array_equal(xq.view(np.uint8).reshape(3, -1), g["xq"])
    out, flags = O.expert_whole(gate, up, down, xq)
    assert flags == 0
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))


def test_route_groups_golden(O):
    g = golden("routes.npz")
    for key in [k[:-4] for k in g.files if k.endswith("_ids")]:
        ids, w = g[key + "_ids"], g[key + "_weights"]
        tokens = ids.size // 10
        r = O.route_groups(ids.reshape(tokens, 10), w.reshape(tokens, 10))
        a = g[key + "_assign"]
        assert np.array_equal(r["token"], a[:, 0]) and np.array_equal(r["rank"], a[:, 1])
        assert np.array_equal(r["expert"], a[:, 2])
        assert np.array_equal(r["weight"].view(np.int32), a[:, 3])
        assert np.array_equal(r["counts"], g[key + "_counts"])


def _select_python(row):
    order = sorted(range(512), key=lambda i: (-row[i], i))[:10]
    buckets = [np.float32(0)] * 32
    for i in order:
        buckets[i % 32] = np.float32(buckets[i % 32] + row[i])
    d = 1
    while d < 32:
        prev = list(buckets)
        buckets = [np.float32(prev[l] + prev[l ^ d]) for l in range(32)]
        d *= 2
    den = max(buckets[0], np.float32(1.0 / 16384.0))
    inv = np.float32(np.float32(1.0) / den)
    return order, [np.float32(row[i] * inv) for i in order]


def test_select_routes_matches_independent_restatement(O):
    rng = np.random.default_rng(8)
    logits = rng.standard_normal((64, 512)).astype(np.float32)
    logits[3, 100] = logits[3, 200] = 9.0  # exact tie -> lower id first
    logits[5] = 0.0                         # all equal -> ids 0..9
    probs, flags = O.router_softmax(logits)
    assert flags == 0
    ids, w = O.select_routes(probs)
    for t in range(64):
        order, weights = _select_python(probs[t])
        assert ids[t].tolist() == order
        assert np.array_equal(np.array(weights, np.float32).view(np.uint32), w[t].view(np.uint32))
    assert ids[3, 0] == 100 and ids[3, 1] == 200
    assert ids[5].tolist() == list(range(10))


def test_router_softmax_properties(O):
    rng = np.random.default_rng(9)
    logits = (rng.standard_normal((16, 512)) * 4).astype(np.float32)
    p, flags = O.router_softmax(logits)
    assert flags == 0
    ref = np.exp(logits.astype(np.float64) - logits.max(1, keepdims=True))
    ref /= ref.sum(1, keepdims=True)
    assert np.max(np.abs(p - ref)) < 1e-6
    bad = logits.copy()
    bad[2, 7] = np.nan
    p, flags = O.router_softmax(bad)
    assert flags & 1 and not p[2].any() and p[3].any()


def test_route_exp_accuracy(O):
    L = O.lib()
    xs = np.concatenate([np.linspace(-103.9, 0, 20001), -np.logspace(-8, 2, 2000)]).astype(np.float32)
    worst = 0
    for x in xs:
        a = np.float32(L.o_route_exp(float(x)))
        b = np.float32(math.exp(float(x)))
        if b == 0:
            continue
        ulp = np.spacing(b)
        worst = max(worst, abs(float(a) - float(b)) / float(ulp))
    assert worst <= 2.0
    assert L.o_route_exp(0.0) == 1.0 and L.o_route_exp(-200.0) == 0.0


def test_synth_generator_statistics(O):
    w = O.synth_q4_0(1, 0, 0, 0, 512, 64).reshape(-1, 18)
    d = w[:, :2].copy().view(np.uint16).ravel()
    vals = np.array([O.lib().o_half_to_float(int(h)) for h in d[:4096]])
    assert 0.003 < np.median(vals) < 0.009
    codes = w[:, 2:].ravel()
    lo, hi = codes & 15, codes >> 4
    assert abs(lo.mean() - 7.5) < 0.05 and abs(hi.mean() - 7.5) < 0.05
    # different streams differ, same stream repeats
    assert not np.array_equal(O.synth_q4_0(1, 0, 0, 0, 4, 4), O.synth_q4_0(1, 0, 1, 0, 4, 4))
    assert np.array_equal(O.synth_q4_0(1, 2, 3, 1, 4, 4), O.synth_q4_0(1, 2, 3, 1, 4, 4))


def test_layer_oracle_composition(O):
    """Whole-layer composition on a tiny synthetic case, compared with an
    independent numpy composition of the same restated pieces."""
    rng = np.random.default_rng(21)
    T, seed = 2, 5
    x = rng.standard_normal((T, 2048)).astype(np.float32)
    logits = rng.standard_normal((T, 512)).astype(np.float32)
    gv = (rng.standard_normal(2048) * 0.02).astype(np.float32)
    out, ids, w, flags = O.moe_layer(x, logits, lambda e: O.synth_expert(seed, 0, e), O.synth_expert(seed, 0, 512), gv)
    assert flags == 0
    xq, _ = O.quantize(x)
    acc = np.zeros((T, 2048), np.float64)
    for t in range(T):
        for r in range(10):
            y, _ = O.expert_whole(*O.synth_expert(seed, 0, int(ids[t, r])), xq[t:t + 1])
            acc[t] += float(w[t, r]) * y[0]
        ys, _ = O.expert_whole(*O.synth_expert(seed, 0, 512), xq[t:t + 1])
        raw = float(np.dot(x[t].astype(np.float64), gv))
        acc[t] += ys[0] / (1 + math.exp(-raw))
    rms = np.sqrt(np.mean(acc ** 2))
    assert np.max(np.abs(out - acc)) <= 1e-5 * rms


# ------------------------------------------------------------------- Q4_1 --
def _q4_1_rows(d, m, codes):
    w = np.zeros((len(codes), 20), np.uint8)
    for r, c in enumerate(codes):
        w[r, 0:2] = np.array([d], np.uint16).view(np.uint8)
        w[r, 2:4] = np.array([m], np.uint16).view(np.uint8)
        w[r, 4:] = c
    return w.ravel()


def test_q4_1_literal_matrix_known_answer(O):
    # tests/quant_test.cpp:575-603: Q4_1 (d 1, m 0.5) expected {-79, -207, -6145.5, -24577.5}
    x = np.zeros(2, O.Q8_DTYPE)
    x["d"] = 0x3c00
    x[0]["s"], x[1]["s"] = 0x4000, 0xc200
    x[0]["qs"] = [3] * 16 + [-4] * 16
    x[1]["qs"] = [-128] * 32
    w = _q4_1_rows(0x3c00, 0x3800, (0x21, 0x75))
    want = [-79.0, -207.0, -6145.5, -24577.5]
    assert O.matrix_serial_q4_1(w, x, 2, 1).ravel().tolist() == want
    assert O.matrix_mmvq_q4_1(w, x, 2, 1).ravel().tolist() == want


def test_q4_1_half_rounded_products(O):
    # tests/quant_test.cpp:480-500: the products d4*d8 and m4*s8 are rounded to half
    x = np.zeros(1, O.Q8_DTYPE)
    x["d"], x["s"] = 0x3c01, 0x3c01
    x[0]["qs"] = [127] * 32
    w = _q4_1_rows(0x3c01, 0xbc01, (0xff,))
    got = O.matrix_serial_q4_1(w, x, 1, 1).item()
    h = O.lib().o_half_to_float
    dd = np.float32(h(O.lib().o_float_to_half(np.float32(h(0x3c01)) * np.float32(h(0x3c01)))))
    ms = np.float32(h(O.lib().o_float_to_half(np.float32(h(0xbc01)) * np.float32(h(0x3c01)))))
    assert got == np.float32(np.float32(32 * 15 * 127) * dd) + ms
    unrounded = float(32 * 15 * 127) * h(0x3c01) * h(0x3c01) + h(0xbc01) * h(0x3c01)
    assert abs(unrounded - got) > 0.01
    # 2^-14 * 2^-14 rounds to half zero; the offset m*s = 0.5 * 3 remains
    x["d"], x["s"] = 0x0400, 0x4200
    w = _q4_1_rows(0x0400, 0x3800, (0xff,))
    assert O.matrix_serial_q4_1(w, x, 1, 1).item() == 1.5


def test_q4_1_block_dots_and_serial_match_golden(O):
    g = golden("expert_q4_1.npz")
    w = O.synth_q4_1(5, 1, 2, 2, 2048, 16)
    xq, _ = O.quantize(g["matmul_x"])
    out = O.matrix_serial_q4_1(w, xq, 2048, 16)
    assert np.array_equal(out.view(np.uint32), g["matmul_out"].view(np.uint32))
    # uncentred block dots: the Q4_0 dot routine over the same code bytes
    dots = O.block_dots_q4_1(w, xq, 2048, 16)
    w0 = np.concatenate([np.zeros((2048 * 16, 2), np.uint8), w.reshape(-1, 20)[:, 4:]], axis=1).ravel()
    assert np.array_equal(dots, O.block_dots(w0, xq, 2048, 16))


def test_q4_1_serial_matches_reference(O):
    R = _ref_or_skip(O)
    rng = np.random.default_rng(12)
    for rows, blocks in ((512, 64), (2048, 16), (7, 3)):
        w = O.synth_q4_1(9, 0, 1, 2, rows, blocks)
        xq, _ = O.quantize(rng.standard_normal((3, blocks * 32)).astype(np.float32))
        a = O.matrix_serial_q4_1(w, xq, rows, blocks)
        for avx2 in (0, 1):
            out = np.zeros(3 * rows, np.float32)
            assert R.ref_matmul(avx2, 3, blocks * 32, rows, O.ptr(w), w.size, O.ptr(xq), xq.size, 3, O.ptr(out),
                                out.size) == 0
            assert np.array_equal(a.ravel().view(np.uint32), out.view(np.uint32))


def test_q4_1_expert_whole_matches_reference_fixtures(O):
    g = golden("expert_q4_1.npz")
    # the reference cpu_expert test's Fixture(TensorType::Q4_1) at 2560/640
    H, I = 2560, 640
    gate = O.fixture_xorshift_q4_0(0x70af451, I, H // 32)
    up = O.fixture_xorshift_q4_0(0xa5f726e, I, H // 32)
    down = O.fixture_xorshift_q4_1(0x525a31, H, I // 32)
    xq = np.ascontiguousarray(g["native_xq"]).view(O.Q8_DTYPE).reshape(3, 80)
    out, flags = O.expert_whole(gate, up, down, xq, H, I, down_type=O.Q4_1)
    assert flags == 0
    assert np.array_equal(out.view(np.uint32), g["native_out"].view(np.uint32))
    # the repository's Q4_1 generator at 2048/512
    seed, layer, expert = (int(v) for v in g["seed"])
    gate, up, down = O.synth_expert(seed, layer, expert, down_type=O.Q4_1)
    xq, _ = O.quantize(g["x"])
    out, flags = O.expert_whole(gate, up, down, xq, down_type=O.Q4_1)
    assert flags == 0
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))


def test_q4_1_generator(O):
    """Q4_1 down matrices share the Q4_0 generator's codes and scales; the
    minimum lies in [-12 d, -4 d]."""
    w1 = O.synth_q4_1(3, 4, 5, 2, 64, 16).reshape(-1, 20)
    w0 = O.synth_q4_0(3, 4, 5, 2, 64, 16).reshape(-1, 18)
    assert np.array_equal(w1[:, :2], w0[:, :2]) and np.array_equal(w1[:, 4:], w0[:, 2:])
    h = O.lib().o_half_to_float
    d = np.array([h(int(v)) for v in w1[:, :2].copy().view(np.uint16).ravel()])
    m = np.array([h(int(v)) for v in w1[:, 2:4].copy().view(np.uint16).ravel()])
    assert np.all(m <= -4 * d * (1 - 1e-3)) and np.all(m >= -12 * d * (1 + 1e-3))
