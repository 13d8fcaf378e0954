"""Expert parallelism over peer memory (moe_ep_*).

CPU: argument checks before any device call and the host-side handle
exchange over a 2-rank gloo group.  GPU: the world-1 path (self-dispatch)
against moe_forward on one B200, and 2 ranks on 2 B200s (skipped with fewer
GPUs) against the single-GPU forward of the same tokens.  Bar: max|err| <=
1e-3 * RMS(output), the layer bar; in practice only fp32 summation order
differs."""
import ctypes
import multiprocessing as mp
import socket

import numpy as np
import pytest

TOL_RMS = 1e-3


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(target, world, *args, timeout=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=timeout))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return sorted(results, key=lambda r: r[0])


def test_ep_arguments_rejected_before_device_calls(pkg):
    L = pkg.library()
    h = ctypes.c_void_p()
    d = pkg.make_desc(max_tokens=8)
    for rank, world in ((0, 3), (2, 2), (-1, 2), (0, 16)):
        assert L.moe_ep_create(ctypes.byref(d), rank, world, ctypes.byref(h)) == pkg.MOE_INVALID_ARGUMENT
        assert L.moe_ep_weights_create(ctypes.byref(d), rank, world, ctypes.byref(h)) == pkg.MOE_INVALID_ARGUMENT
        assert not h.value
    big = pkg.make_desc(max_tokens=40000)
    assert L.moe_ep_create(ctypes.byref(big), 0, 2, ctypes.byref(h)) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_ep_forward(None, None, None, None, 1, None, 0, None) == pkg.MOE_INVALID_ARGUMENT


def test_handle_exchange_two_ranks_gloo():
    import ep_worker
    res = run_ranks(ep_worker.exchange_worker, 2, timeout=120)
    for rank, got, n in res:
        assert got == [1, 2], (rank, got, n)
        assert n == 64


@pytest.mark.gpu
@pytest.mark.parametrize("tokens,routing,down_type", [(8, "normal", 2), (100, "normal", 2), (300, "zipf", 2),
                                                      (8, "normal", 3), (300, "zipf", 3)])
def test_ep_world1_matches_forward(pkg, tokens, routing, down_type):
    import torch
    desc = pkg.make_desc(max_tokens=tokens)
    rng = np.random.default_rng(tokens)
    x = torch.from_numpy(rng.standard_normal((tokens, 2048)).astype(np.float32)).cuda()
    if routing == "zipf":
        perm = rng.permutation(512)
        g = -np.log(-np.log(rng.random((tokens, 512))))
        lg = (-1.1 * np.log1p(perm.astype(np.float64))[None, :] + g).astype(np.float32)
    else:
        lg = rng.standard_normal((tokens, 512)).astype(np.float32)
    logits = torch.from_numpy(lg).cuda()
    gate = (rng.standard_normal(2048) * 0.05).astype(np.float32)
    full = pkg.MoeWeights(desc, down_type)
    full.synthesize(3, 1)
    full.upload_shared_gate(gate)
    ref = torch.zeros(tokens, 2048, device="cuda")
    pkg.MoeLayer(desc).forward(full, x, logits, ref)
    shard = pkg.EpWeights(desc, 0, 1, down_type)
    shard.synthesize(3, 1)
    shard.upload_shared_gate(gate)
    ep = pkg.EpLayer(desc, 0, 1)
    for _ in range(3):
        out = x.clone()
        ep.forward(shard, x, logits, out)          # accumulate into a residual copy
        torch.cuda.synchronize()
        r = ref.cpu().numpy()
        err = np.abs((out - x).cpu().numpy() - r).max()
        rms = np.sqrt(np.mean(r.astype(np.float64) ** 2))
        assert err <= TOL_RMS * rms, (err, rms)
    assert ep.read_flags() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("tokens,routing", [(8, "normal"), (256, "zipf")])
def test_ep_two_ranks_match_single_gpu(tokens, routing):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import ep_worker
    res = run_ranks(ep_worker.forward_worker, 2, tokens, routing, timeout=600)
    for rank, flags, errs, rms in res:
        assert flags != "error", (rank, errs)
        assert flags == 0, (rank, flags)
        for e in errs:
            assert e <= TOL_RMS * rms, (rank, e, rms)


@pytest.mark.gpu
def test_ep_silent_peer_times_out_with_flag(pkg):
    """A peer that never publishes: the bounded device waits give up after ~1 s
    each and report MOE_FLAG_TIMEOUT; nothing hangs and the context stays
    usable.  Two processes on one GPU; only one of them launches kernels."""
    import ep_worker
    res = run_ranks(ep_worker.silent_peer_worker, 2, timeout=240)
    rank0 = res[0]
    assert rank0[1] != "error", rank0
    _, flags, waited, after = rank0
    assert flags & 4, flags          # MOE_FLAG_TIMEOUT
    assert 0.5 < waited < 30.0, waited
    assert after == 0
    assert res[1][1] != "error", res[1]


@pytest.mark.gpu
def test_ep_world1_forward_hidden(pkg):
    """moe_ep_forward_hidden (router logits on the device from the shard's router
    matrix) equals the single-GPU moe_forward_hidden."""
    import torch
    T = 8
    desc = pkg.make_desc(max_tokens=T)
    rng = np.random.default_rng(77)
    x = torch.from_numpy(rng.standard_normal((T, 2048)).astype(np.float32)).cuda()
    router = (rng.standard_normal((512, 2048)) * 0.02).astype(np.float32)
    gate = (rng.standard_normal(2048) * 0.05).astype(np.float32)
    full = pkg.MoeWeights(desc)
    full.synthesize(9, 2)
    full.upload_shared_gate(gate)
    full.upload_router(router)
    ref = torch.zeros(T, 2048, device="cuda")
    pkg.MoeLayer(desc).forward_hidden(full, x, ref, accumulate=False)
    shard = pkg.EpWeights(desc, 0, 1)
    shard.synthesize(9, 2)
    shard.upload_shared_gate(gate)
    shard.upload_router(router)
    ep = pkg.EpLayer(desc, 0, 1)
    ep.connect(lambda h: [h])
    out = torch.zeros(T, 2048, device="cuda")
    ep.forward_hidden(shard, x, out, accumulate=False)
    torch.cuda.synchronize()
    r = ref.cpu().numpy()
    rms = np.sqrt(np.mean(r.astype(np.float64) ** 2))
    assert np.abs(out.cpu().numpy() - r).max() <= TOL_RMS * rms
    assert ep.read_flags() == 0
