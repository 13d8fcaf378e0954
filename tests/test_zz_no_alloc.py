"""GPU test of moe_route_noalloc, the routing entry point that allocates no
device memory.

Some callers cannot allocate: work enqueued while a CUDA graph is being
captured (an allocation is not part of a capture and would have to outlive
the graph), and hosts whose device memory is owned by another allocator or a
fixed arena.  For them moe_route_noalloc keeps its scratch in one static
device array (at most 1024 tokens) and writes only into the caller's buffers.

The test calls it through the C ABI twice in a row per case -- up to the
array's 1024-token limit, and a skewed routing whose tile list nears the
array's tile capacity -- checks that the device's free memory does not change
across a call, and compares every output with the allocating entry point
(moe_route through a layer workspace).  It also captures the call in a CUDA
graph (after one eager call, as the header requires) and replays the graph
on new logits written into the captured input.  Routing results are compared exactly
-- the tolerance the other routing tests use.  This file is collected last on
purpose.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def _bits(t):
    return t.cpu().numpy().view(np.uint32)


def _logits(torch, T, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "skewed":
        # a third of the experts unused, many with one or two pairs, a few
        # with ~900: 1-pair tiles beside long groups
        base = -3.0 * np.log1p(rng.permutation(512).astype(np.float64))
        lg = base[None, :] + 4.0 * rng.standard_normal((T, 512))
    else:
        lg = rng.standard_normal((T, 512))
    return torch.from_numpy(lg.astype(np.float32)).cuda()


def _raw_call(pkg, torch, logits, outs):
    L = pkg.library()
    st = L.moe_route_noalloc(ctypes.c_void_p(logits.data_ptr()), logits.shape[0],
                             *[ctypes.c_void_p(outs[k].data_ptr()) for k in ("ids", "weights", "offsets", "token",
                                                                             "rank", "error")],
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == pkg.MOE_OK, L.moe_last_error_message()


@pytest.mark.parametrize("T,kind", [(8, "normal"), (300, "normal"), (1024, "normal"), (1024, "skewed")])
def test_noalloc_route_matches_allocating_route_twice(pkg, torch, T, kind):
    layer = pkg.MoeLayer(pkg.make_desc(max_tokens=T))
    outs = _outputs(torch, T)
    # the first call on a device resolves the static array's address; after it,
    # calls allocate nothing: the device's free memory is unchanged around them
    _raw_call(pkg, torch, _logits(torch, T, kind, 1), outs)
    torch.cuda.synchronize()
    for call in range(2):
        logits = _logits(torch, T, kind, 1000 * T + call)
        want = layer.route(logits)
        torch.cuda.synchronize()
        outs["error"].zero_()
        free_before = torch.cuda.mem_get_info()[0]
        _raw_call(pkg, torch, logits, outs)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before, "moe_route_noalloc allocated device memory"
        assert int(outs["error"].item()) == 0
        assert np.array_equal(outs["ids"].cpu().numpy(), want["ids"].cpu().numpy())
        assert np.array_equal(_bits(outs["weights"]), _bits(want["weights"]))
        assert np.array_equal(outs["offsets"].cpu().numpy(), want["offsets"].cpu().numpy())
        assert np.array_equal(outs["token"].cpu().numpy(), want["token"].cpu().numpy())
        assert np.array_equal(outs["rank"].cpu().numpy(), want["rank"].cpu().numpy())
        if T == 1024:   # the tile list (<= 4 pairs per tile) nears the array's 3072-tile capacity
            counts = np.diff(want["offsets"].cpu().numpy())
            assert int(np.sum((counts + 3) // 4)) > 2600


def _outputs(torch, T):
    return dict(ids=torch.empty(T, 10, dtype=torch.int32, device="cuda"),
                weights=torch.empty(T, 10, device="cuda"),
                offsets=torch.empty(513, dtype=torch.int32, device="cuda"),
                token=torch.empty(T * 10, dtype=torch.int32, device="cuda"),
                rank=torch.empty(T * 10, dtype=torch.int32, device="cuda"),
                error=torch.zeros(1, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("T", [8, 300])
def test_noalloc_route_captured_in_cuda_graph(pkg, torch, T):
    layer = pkg.MoeLayer(pkg.make_desc(max_tokens=T))
    outs = _outputs(torch, T)
    logits = torch.empty(T, 512, device="cuda")
    logits.copy_(_logits(torch, T, "normal", 5))
    _raw_call(pkg, torch, logits, outs)          # the eager first call resolves the array's address
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):   # the call is enqueued on the capturing stream
        _raw_call(pkg, torch, logits, outs)
    for replay in range(2):
        logits.copy_(_logits(torch, T, "normal", 77 + replay))
        outs["error"].zero_()
        graph.replay()
        torch.cuda.synchronize()
        want = layer.route(logits)
        torch.cuda.synchronize()
        assert int(outs["error"].item()) == 0
        assert np.array_equal(outs["ids"].cpu().numpy(), want["ids"].cpu().numpy())
        assert np.array_equal(_bits(outs["weights"]), _bits(want["weights"]))
        assert np.array_equal(outs["offsets"].cpu().numpy(), want["offsets"].cpu().numpy())
        assert np.array_equal(outs["token"].cpu().numpy(), want["token"].cpu().numpy())
        assert np.array_equal(outs["rank"].cpu().numpy(), want["rank"].cpu().numpy())
    del graph


def test_noalloc_python_wrapper_checks_arguments(pkg, torch):
    with pytest.raises(ValueError):
        pkg.route_noalloc(torch.zeros(4, 256, device="cuda"))             # not 512 experts wide
    with pytest.raises(ValueError):
        pkg.route_noalloc(torch.zeros(4, 512, device="cuda", dtype=torch.float64))
    with pytest.raises(ValueError):
        pkg.route_noalloc(torch.zeros(512, 4, device="cuda").t())         # not contiguous


def test_noalloc_route_rejects_more_tokens_than_its_scratch(pkg, torch):
    L = pkg.library()
    T = 1025
    logits = torch.zeros(T, 512, device="cuda")
    bufs = [torch.empty(T * 10 + 1024, dtype=torch.int32, device="cuda") for _ in range(6)]
    st = L.moe_route_noalloc(ctypes.c_void_p(logits.data_ptr()), T,
                             *[ctypes.c_void_p(b.data_ptr()) for b in bufs],
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == pkg.MOE_INVALID_ARGUMENT
    assert b"1..1024" in L.moe_last_error_message()
