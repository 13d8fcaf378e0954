"""GPU test of moe_route_noalloc, the routing entry point that allocates no
device memory.

Some callers cannot allocate: work enqueued while a CUDA graph is being
captured (an allocation is not part of a capture and would have to outlive
the graph), and hosts whose device memory is owned by another allocator or a
fixed arena.  For them moe_route_noalloc keeps its scratch in one static
device array (at most 1024 tokens) and writes only into the caller's buffers.

The test calls it through the C ABI twice in a row per size and compares
every output with the allocating entry point (moe_route through a layer
workspace).  Routing results are compared exactly -- the tolerance the other
routing tests use.  This file is collected last on purpose.
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


@pytest.mark.parametrize("T", [8, 300])
def test_noalloc_route_matches_allocating_route_twice(pkg, torch, T):
    layer = pkg.MoeLayer(pkg.make_desc(max_tokens=T))
    for call in range(2):
        rng = np.random.default_rng(1000 * T + call)
        logits = torch.from_numpy(rng.standard_normal((T, 512)).astype(np.float32)).cuda()
        want = layer.route(logits)
        got, err = pkg.route_noalloc(logits)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert np.array_equal(got["ids"].cpu().numpy(), want["ids"].cpu().numpy())
        assert np.array_equal(_bits(got["weights"]), _bits(want["weights"]))
        assert np.array_equal(got["offsets"].cpu().numpy(), want["offsets"].cpu().numpy())
        assert np.array_equal(got["token"].cpu().numpy(), want["token"].cpu().numpy())
        assert np.array_equal(got["rank"].cpu().numpy(), want["rank"].cpu().numpy())


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
