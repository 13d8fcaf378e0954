"""Bit-exact per-block dot parity of the kernels the forward actually runs.

moe_debug_block_dots runs an ordinary forward through the same kernels a
batch of that size uses -- the streaming dp4a kernels at decode sizes (two
items in flight per CTA at T=1, one at T=8), the tcgen05 tensor-core kernels
above -- and records, for one expert's pairs, every
per-block int32 dot those kernels formed plus the middle Q8_1 the gate/up
kernel produced.  The checks mirror the reference's own producer-kernel
comparison against its CPU expert (src/cpu_expert_shadow.hip:333-341) and its
"down on common middle Q8" case (tests/cpu_expert_test.cpp:323-326):

* gate and up dots == the oracle's uncentred block dots of that expert's
  weights against the quantised x rows of its pairs (bit-exact);
* down dots == the oracle's block dots of the down matrix (Q4_0, or Q4_1 as
  in the reference's layers 0-5) against the middle Q8_1 the GPU itself
  produced (bit-exact);
* that middle Q8_1 is byte-identical to the oracle's CPU-expert middle: the
  gate/up kernels sum in the reference's MMVQ order and the SiLU's exp is
  correctly rounded, so the fp32 gate and up values are the reference's.
"""
import numpy as np
import pytest

from cases import H, I, LayerCase

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def tap_and_check(O, torch, c, expert, max_pairs=None):
    xq, _ = O.quantize(c.x)
    probs, _ = O.router_softmax(c.logits)
    ids, w = O.select_routes(probs)
    if expert == 512:
        tokens = np.arange(c.T)
    else:
        grp = O.route_groups(ids, w)
        tokens = grp["token"][grp["offsets"][expert]:grp["offsets"][expert + 1]]
    n = len(tokens) if max_pairs is None else min(max_pairs, len(tokens))
    assert n > 0
    tokens = tokens[:n]
    r = c.layer.block_dots(c.weights, c.xd, c.ld, expert, n)
    torch.cuda.synchronize()
    assert c.layer.read_flags() == 0
    g, u, d = c.expert(expert)
    xs = np.ascontiguousarray(xq[tokens])
    assert np.array_equal(r["gate"].cpu().numpy(), O.block_dots(g, xs, I, H // 32)), "gate dots"
    assert np.array_equal(r["up"].cpu().numpy(), O.block_dots(u, xs, I, H // 32)), "up dots"
    mid = np.zeros((n, I // 32), O.Q8_DTYPE)
    ds = r["mid_ds"].cpu().numpy().view(np.uint32)
    mid["d"] = ds & 0xffff
    mid["s"] = ds >> 16
    mid["qs"] = r["mid_codes"].cpu().numpy().reshape(n, I // 32, 32)
    down_dots = O.block_dots_q4_1 if c.down_type == O.Q4_1 else O.block_dots
    assert np.array_equal(r["down"].cpu().numpy(), down_dots(d, mid, H, I // 32)), "down dots on the GPU's middle"
    # the GPU's middle against the CPU expert's own middle Q8_1
    mq = np.zeros(n * I // 32, O.Q8_DTYPE)
    scratch = np.empty(n * I * 3, np.float32)
    out = np.empty(n * H, np.float32)
    O.lib().o_expert_whole_typed(O.ptr(g), O.ptr(u), O.ptr(d), c.down_type, H, I, O.ptr(xs), n, O.ptr(out),
                                 O.ptr(scratch), O.ptr(mq))
    mq = mq.reshape(n, I // 32)
    flips = int(np.sum(mid["qs"] != mq["qs"]))
    assert flips == 0, f"{flips} middle codes differ from the CPU expert's"
    assert np.array_equal(mid["d"], mq["d"]) and np.array_equal(mid["s"], mq["s"]), "middle scales"
    return n


@pytest.mark.parametrize("T,kind,pick", [(1, "normal", "first"), (1, "normal", "shared"),
                                         (8, "normal", "first"), (8, "normal", "shared"),
                                         (1024, "normal", "largest"), (1024, "normal", "smallest"),
                                         (1024, "normal", "shared"), (4096, "zipf", "largest"),
                                         (4096, "zipf", "median")])
def test_block_dots_of_forward_kernels(pkg, O, torch, T, kind, pick):
    c = LayerCase(pkg, O, torch, T, seed=600 + T, logits_kind=kind)
    probs, _ = O.router_softmax(c.logits)
    ids, _ = O.select_routes(probs)
    counts = np.bincount(ids.ravel(), minlength=512)
    if pick == "shared":
        expert = 512
    elif pick == "first":
        expert = int(ids[0, 0])
    elif pick == "largest":
        expert = int(np.argmax(counts))
    elif pick == "smallest":
        expert = int(np.argmin(np.where(counts > 0, counts, 1 << 30)))
    else:
        live = np.nonzero(counts)[0]
        expert = int(live[np.argsort(counts[live])[len(live) // 2]])
    # the shared expert of a large batch: its first 160 pairs (three tiles)
    assert tap_and_check(O, torch, c, expert, max_pairs=160 if expert == 512 else None) >= 1


@pytest.mark.parametrize("T,kind,pick", [(300, "zipf", "largest"), (1024, "normal", "largest"),
                                         (1024, "normal", "shared")])
def test_block_dots_q4_1_down(pkg, O, torch, T, kind, pick):
    """Q4_1 down matrices on the tensor-core down kernel: its dots on the
    GPU's own middle, bit-exact."""
    c = LayerCase(pkg, O, torch, T, seed=650 + T, logits_kind=kind, down_type=pkg.MOE_Q4_1)
    probs, _ = O.router_softmax(c.logits)
    ids, _ = O.select_routes(probs)
    expert = 512 if pick == "shared" else int(np.argmax(np.bincount(ids.ravel(), minlength=512)))
    assert tap_and_check(O, torch, c, expert, max_pairs=160 if expert == 512 else None) >= 1
