"""GPU parity tests: the sm_100a kernels through the C ABI against the CPU
oracle (itself pinned to the reference's own code).

Bars (from the build's contract):
* Q8_1 bytes, per-block int32 dots, routing ids/weights/probabilities and the
  grouped (expert, token, rank) order: bit-exact;
* layer outputs: max|err| <= 1e-3 * RMS(output) in fp32 (TOL_RMS below);
* single linear projections: the reference's own common-Q8 gate
  2e-4 + 2e-5*|ref| (tests/cpu_expert_test.cpp:296-324).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from cases import H, I, E, LayerCase, assert_close, f32bits, zipf_logits  # noqa: E402


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


# ------------------------------------------------------------------ kernels --
def test_quantize_bytes_match_oracle(pkg, O, torch):
    from conftest import golden
    g = golden("quant_cases.npz")
    rng = np.random.default_rng(1)
    x = np.concatenate([g["x"].reshape(-1, 32),
                        (rng.standard_normal((4096, 32)) * 10.0 ** rng.uniform(-5, 3, (4096, 1))).astype(np.float32)])
    x = np.ascontiguousarray(x)  # one 32-wide column per block
    q, err = pkg.quantize_q8_1(torch.from_numpy(x).cuda())
    want, flags = O.quantize(x)
    assert int(err.item()) == flags == 0
    assert np.array_equal(q.cpu().numpy().ravel(), want.view(np.uint8).ravel())


def test_quantize_invalid_blocks(pkg, O, torch):
    x = np.ones((2, 64), np.float32)
    x[0, 3] = np.nan
    x[1, 32:] = 0.0
    x[1, 40] = 1e-45   # whole block's original FP32 scale underflows to zero
    q, err = pkg.quantize_q8_1(torch.from_numpy(x).cuda())
    want, flags = O.quantize(x)
    assert int(err.item()) == flags == 3
    assert np.array_equal(q.cpu().numpy().ravel(), want.view(np.uint8).ravel())


@pytest.mark.parametrize("rows,k,cols", [(512, 2048, 3), (2048, 512, 5), (96, 64, 1)])
def test_block_dots_bit_exact(pkg, O, torch, rows, k, cols):
    rng = np.random.default_rng(rows + cols)
    w = O.synth_q4_0(3, 0, rows % 7, 0, rows, k // 32)
    x = rng.standard_normal((cols, k)).astype(np.float32)
    xq, _ = O.quantize(x)
    out, dots = pkg.q4_linear(torch.from_numpy(w).cuda(), rows, k,
                              torch.from_numpy(xq.view(np.uint8).reshape(cols, -1).copy()).cuda(), cols,
                              with_dots=True)
    assert np.array_equal(dots.cpu().numpy(), O.block_dots(w, xq, rows, k // 32))
    ref = O.matrix_serial(w, xq, rows, k // 32)
    got = out.cpu().numpy()
    assert np.all(np.abs(got - ref) <= 2e-4 + 2e-5 * np.abs(ref))


def test_synthesized_weights_match_oracle_generator(pkg, O, torch):
    desc = pkg.make_desc(max_tokens=1)
    w = pkg.MoeWeights(desc)
    w.synthesize(99, 7)
    torch.cuda.synchronize()
    for e in (0, 255, 511, 512):
        got = w.download_expert(e)
        want = O.synth_expert(99, 7, e)
        for a, b in zip(got, want):
            assert np.array_equal(a, b), e


def test_upload_download_roundtrip(pkg, O, torch):
    desc = pkg.make_desc(max_tokens=1)
    w = pkg.MoeWeights(desc)
    g, u, d = O.synth_expert(1, 1, 1)
    w.upload_expert(3, g, u, d)
    for a, b in zip(w.download_expert(3), (g, u, d)):
        assert np.array_equal(a, b)


# ------------------------------------------------------------------ routing --
@pytest.mark.parametrize("T,kind", [(1, "normal"), (8, "normal"), (37, "ties"), (300, "normal"),
                                    (4096, "zipf"), (2500, "nonfinite")])
def test_route_bit_exact(pkg, O, torch, T, kind):
    rng = np.random.default_rng(T)
    if kind == "zipf":
        logits = zipf_logits(rng, T)
    else:
        logits = rng.standard_normal((T, E)).astype(np.float32)
    if kind == "ties":
        logits[0, :] = 0.0
        logits[1, 10] = logits[1, 20] = 7.0
        logits[2] = np.round(logits[2])
    if kind == "nonfinite":
        logits[5, 9] = np.inf
        logits[77, 0] = np.nan
    layer = pkg.MoeLayer(pkg.make_desc(max_tokens=T))
    r = layer.route(torch.from_numpy(logits).cuda())
    torch.cuda.synchronize()
    probs, flags = O.router_softmax(logits)
    ids, w = O.select_routes(probs)
    grp = O.route_groups(ids, w)
    assert np.array_equal(f32bits(r["probs"].cpu().numpy()), f32bits(probs))
    assert np.array_equal(r["ids"].cpu().numpy(), ids)
    assert np.array_equal(f32bits(r["weights"].cpu().numpy()), f32bits(w))
    assert np.array_equal(r["offsets"].cpu().numpy(), grp["offsets"])
    assert np.array_equal(r["token"].cpu().numpy(), grp["token"])
    assert np.array_equal(r["rank"].cpu().numpy(), grp["rank"])
    assert layer.read_flags() == flags


# -------------------------------------------------------------------- layer --
@pytest.mark.parametrize("T", [1, 8, 3, 33])
def test_forward_matches_oracle(pkg, O, torch, T):
    c = LayerCase(pkg, O, torch, T, seed=100 + T)
    out = torch.zeros(T, H, device="cuda")
    c.layer.forward(c.weights, c.xd, c.ld, out, accumulate=False)
    torch.cuda.synchronize()
    assert c.layer.read_flags() == 0
    assert_close(out.cpu().numpy(), c.oracle())


def test_forward_accumulates_into_residual_in_place(pkg, O, torch):
    T = 8
    c = LayerCase(pkg, O, torch, T, seed=7)
    h = c.xd.clone()
    c.layer.forward(c.weights, h, c.ld, h, accumulate=True)  # residual += FFN(residual)
    torch.cuda.synchronize()
    assert_close(h.cpu().numpy() - c.x, c.oracle())


def test_forward_flags_nonfinite_input(pkg, O, torch):
    T = 4
    c = LayerCase(pkg, O, torch, T, seed=11)
    x = c.xd.clone()
    x[2, 100] = float("nan")
    out = torch.zeros(T, H, device="cuda")
    c.layer.forward(c.weights, x, c.ld, out, accumulate=False)
    assert c.layer.read_flags() & 1


def test_forward_rejects_bad_arguments(pkg, O, torch):
    c = LayerCase(pkg, O, torch, 2, seed=12)
    out = torch.zeros(2, H, device="cuda")
    with pytest.raises(ValueError):
        c.layer.forward(c.weights, c.xd, c.ld, c.xd, accumulate=False)  # overwrite aliasing x
    big = torch.zeros(3, H, device="cuda")
    with pytest.raises(ValueError):
        c.layer.forward(c.weights, big, torch.zeros(3, E, device="cuda"), big.clone(), accumulate=False)


def test_forward_in_cuda_graph(pkg, O, torch):
    T = 8
    c = LayerCase(pkg, O, torch, T, seed=13)
    out = torch.zeros(T, H, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        c.layer.forward(c.weights, c.xd, c.ld, out, accumulate=False, stream=s)  # warm-up
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        c.layer.forward(c.weights, c.xd, c.ld, out, accumulate=False, stream=s)
    out.fill_(123.0)
    g.replay()
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), c.oracle())


# -------------------------------------------------- single-expert fixture --
def test_gpu_expert_api(pkg, O, torch):
    g, u, d = O.synth_expert(4, 0, 9)
    ex = pkg.GpuExpert(g, u, d, max_columns=5)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((5, H)).astype(np.float32)
    xq, _ = O.quantize(x)
    ex.check_quantization(x, xq)
    bad = xq.copy()
    bad[0, 0]["qs"][0] ^= 1
    with pytest.raises(RuntimeError):
        ex.check_quantization(x, bad)
    for which, (w, rows, blocks) in {"gate": (g, I, H // 32), "up": (u, I, H // 32)}.items():
        got = ex.linear(False, which == "up", xq, 5)
        ref = O.matrix_serial(w, xq, rows, blocks)
        assert np.all(np.abs(got - ref) <= 2e-4 + 2e-5 * np.abs(ref))
    y, timing = ex.run(x, 5, repeats=3)
    want, _ = O.expert_whole(g, u, d, xq)
    assert_close(y, want)
    assert timing["resident_ms"] > 0


# ------------------------------------------------------------------- Q4_1 --
# Q4_1 down matrices (the reference's layers 0-5): block term
# acc + fma(dot, half(d4*d8), half(m4*s8)).
@pytest.mark.parametrize("rows,k,cols", [(2048, 512, 5), (96, 64, 1)])
def test_q4_1_linear_dots_bit_exact(pkg, O, torch, rows, k, cols):
    rng = np.random.default_rng(rows + 3 * cols)
    w = O.synth_q4_1(8, 1, rows % 5, 2, rows, k // 32)
    xq, _ = O.quantize(rng.standard_normal((cols, k)).astype(np.float32))
    out, dots = pkg.q4_1_linear(torch.from_numpy(w).cuda(), rows, k,
                                torch.from_numpy(xq.view(np.uint8).reshape(cols, -1).copy()).cuda(), cols,
                                with_dots=True)
    assert np.array_equal(dots.cpu().numpy(), O.block_dots_q4_1(w, xq, rows, k // 32))
    ref = O.matrix_serial_q4_1(w, xq, rows, k // 32)
    assert np.all(np.abs(out.cpu().numpy() - ref) <= 2e-4 + 2e-5 * np.abs(ref))


def test_q4_1_weights_generator_and_roundtrip(pkg, O, torch):
    desc = pkg.make_desc(max_tokens=1)
    w = pkg.MoeWeights(desc, pkg.MOE_Q4_1)
    w.synthesize(99, 7)
    torch.cuda.synchronize()
    for e in (0, 300, 512):
        for a, b in zip(w.download_expert(e), O.synth_expert(99, 7, e, down_type=O.Q4_1)):
            assert np.array_equal(a, b), e
    g, u, d = O.synth_expert(1, 1, 1, down_type=O.Q4_1)
    w.upload_expert(3, g, u, d)
    for a, b in zip(w.download_expert(3), (g, u, d)):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("T,kind", [(1, "normal"), (8, "normal"), (33, "normal"), (300, "zipf"), (1024, "normal")])
def test_q4_1_forward_matches_oracle(pkg, O, torch, T, kind):
    """Decode sizes on the streaming kernels, prefill sizes on the tensor-core
    kernels (the down kernel with the Q4_1 block term)."""
    c = LayerCase(pkg, O, torch, T, seed=500 + T, logits_kind=kind, down_type=pkg.MOE_Q4_1)
    out = torch.zeros(T, H, device="cuda")
    c.layer.forward(c.weights, c.xd, c.ld, out, accumulate=False)
    torch.cuda.synchronize()
    assert c.layer.read_flags() == 0
    sample = None if T <= 33 else np.random.default_rng(1).choice(T, 12, replace=False)
    got = out.cpu().numpy() if sample is None else out.cpu().numpy()[sample]
    assert_close(got, c.oracle(sample))


def test_q4_1_gpu_expert_api(pkg, O, torch):
    """GpuExpert with the reference's native type mix (Q4_0 gate/up, Q4_1 down)."""
    g, u, d = O.synth_expert(4, 0, 9, down_type=O.Q4_1)
    ex = pkg.GpuExpert(g, u, d, max_columns=5, down_type=pkg.MOE_Q4_1)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, H)).astype(np.float32)
    xq, _ = O.quantize(x)
    mid, _ = O.quantize(rng.standard_normal((5, I)).astype(np.float32))
    got = ex.linear(True, False, mid, 5)
    ref = O.matrix_serial_q4_1(d, mid, H, I // 32)
    assert np.all(np.abs(got - ref) <= 2e-4 + 2e-5 * np.abs(ref))
    y, _ = ex.run(x, 5, repeats=2)
    want, _ = O.expert_whole(g, u, d, xq, down_type=O.Q4_1)
    assert_close(y, want)


# -------------------------------------------------------------- trace mode --
@pytest.mark.parametrize("T,kind,shared", [(8, "normal", True), (8, "normal", False), (100, "zipf", True)])
def test_forward_contributions_trace_mode(pkg, O, torch, T, kind, shared):
    """moe_forward_contributions: deterministic [T][10][H] contributions and the
    reference's rank-order fold over them (src/hip/session_ops.hip:305-391)."""
    seed = 900 + T
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H)).astype(np.float32)
    logits = zipf_logits(rng, T) if kind == "zipf" else rng.standard_normal((T, E)).astype(np.float32)
    gate_vec = (rng.standard_normal(H) * 0.02).astype(np.float32)
    desc = pkg.make_desc(max_tokens=T, has_shared=int(shared))
    weights = pkg.MoeWeights(desc)
    weights.synthesize(seed, 0)
    if shared:
        weights.upload_shared_gate(gate_vec)
    layer = pkg.MoeLayer(desc)
    xd, ld = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
    runs = []
    for _ in range(2):
        out = torch.zeros(T, H, device="cuda")
        contrib, sh = layer.forward_contributions(weights, xd, ld, out, accumulate=False)
        torch.cuda.synchronize()
        runs.append((out.cpu().numpy(), contrib.cpu().numpy(), None if sh is None else sh.cpu().numpy()))
    assert layer.read_flags() == 0
    (out, contrib, sh), (out2, contrib2, sh2) = runs
    assert np.array_equal(f32bits(out), f32bits(out2)) and np.array_equal(f32bits(contrib), f32bits(contrib2))
    probs, _ = O.router_softmax(logits)
    ids, w = O.select_routes(probs)
    fold = np.empty((T, H), np.float32)
    O.lib().o_routed_fold(O.ptr(np.ascontiguousarray(contrib)), O.ptr(w), T, H, O.ptr(fold))
    if not shared:
        assert np.array_equal(f32bits(out), f32bits(fold))   # the fold itself is the reference's, bit for bit
    # each stored contribution is its expert's unweighted output for that token
    xq, _ = O.quantize(x)
    for t in range(min(T, 4)):
        for r in range(10):
            want, _ = O.expert_whole(*O.synth_expert(seed, 0, int(ids[t, r])), xq[t:t + 1])
            assert_close(contrib[t, r][None], want)
    if shared:
        want, _ = O.expert_whole(*O.synth_expert(seed, 0, 512), xq[:min(T, 4)])
        assert_close(sh[:min(T, 4)], want)
        ref, _, _, _ = O.moe_layer(x, logits, lambda e: O.synth_expert(seed, 0, e), O.synth_expert(seed, 0, 512),
                                   gate_vec, np.arange(min(T, 8)))
        assert_close(out[:min(T, 8)], ref)


# ------------------------------------------------------------- router GEMM --
@pytest.mark.parametrize("T", [1, 8, 33, 300])
def test_router_logits_fp32(pkg, O, torch, T):
    """x * W_router^T on the device: fp32 sums of 2048 products, checked against
    fp64 with an fp32 accumulation bound (the reference's BLAS order is unspecified)."""
    rng = np.random.default_rng(40 + T)
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    desc = pkg.make_desc(max_tokens=T)
    w = pkg.MoeWeights(desc)
    w.upload_router(W)
    got = w.router_logits(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = x.astype(np.float64) @ W.astype(np.float64).T
    bound = 2e-5 * (np.abs(x).astype(np.float64) @ np.abs(W).astype(np.float64).T)
    assert np.all(np.abs(got - ref) <= bound)


@pytest.mark.parametrize("T", [8, 100])
def test_forward_hidden_routes_device_logits(pkg, O, torch, T):
    """moe_forward_hidden == moe_forward over the device logits, and those
    logits route exactly as the oracle routes them."""
    seed = 70 + T
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    gate_vec = (rng.standard_normal(H) * 0.02).astype(np.float32)
    desc = pkg.make_desc(max_tokens=T)
    w = pkg.MoeWeights(desc)
    w.synthesize(seed, 0)
    w.upload_shared_gate(gate_vec)
    w.upload_router(W)
    layer = pkg.MoeLayer(desc)
    xd = torch.from_numpy(x).cuda()
    out_h = torch.zeros(T, H, device="cuda")
    layer.forward_hidden(w, xd, out_h, accumulate=False)
    logits = w.router_logits(xd)
    out_l = torch.zeros(T, H, device="cuda")
    layer.forward(w, xd, logits, out_l, accumulate=False)
    torch.cuda.synchronize()
    assert layer.read_flags() == 0
    lg = logits.cpu().numpy()
    assert_close(out_h.cpu().numpy(), out_l.cpu().numpy())
    r = layer.route(logits)
    probs, _ = O.router_softmax(lg)
    ids, wts = O.select_routes(probs)
    assert np.array_equal(r["ids"].cpu().numpy(), ids)
    assert np.array_equal(f32bits(r["weights"].cpu().numpy()), f32bits(wts))
    sample = np.arange(min(T, 6))
    ref, _, _, _ = O.moe_layer(x, lg, lambda e: O.synth_expert(seed, 0, e), O.synth_expert(seed, 0, 512), gate_vec,
                               sample)
    assert_close(out_h.cpu().numpy()[sample], ref)
