"""Layer parity at the BASELINE configurations' own shapes.

Each case runs the whole routed-MoE layer on the GPU through the C ABI and
checks it against the CPU oracle (the reference's restated Layer::ffn:
quantise, softmax, select_routes, grouping, CpuExpert 'whole' per pair,
rank-order fold, sigmoid-gated shared expert) within
max|err| <= 1e-3 * RMS(output).  A token's output depends only on its own
routing, so checking a sample of the tokens of a large batch is exact for
those tokens.

* config 4's micro-batch: T=1024, uniform routing, ~20 pairs per expert
  (the mid-size tensor-core regime), every token checked;
* T=2048 uniform (~40 pairs per expert), every 4th token;
* config 3: T=4096 with Zipf(1.1) routing, 256 sampled tokens;
* config 5: T=32,768 continuous-batching pack, 256 tokens: all 56 decode
  tokens, both ends of every prefill chunk, the rest random.
"""
import numpy as np
import pytest

from cases import LayerCase, assert_close, mixed_sample

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def run(c, torch):
    out = torch.zeros(c.T, 2048, device="cuda")
    c.layer.forward(c.weights, c.xd, c.ld, out, accumulate=False)
    torch.cuda.synchronize()
    assert c.layer.read_flags() == 0
    return out


def test_config4_ubatch_T1024_uniform_all_tokens(pkg, O, torch):
    c = LayerCase(pkg, O, torch, 1024, seed=4)
    out = run(c, torch)
    assert_close(out.cpu().numpy(), c.oracle())


def test_uniform_T2048_every_fourth_token(pkg, O, torch):
    c = LayerCase(pkg, O, torch, 2048, seed=41)
    out = run(c, torch)
    sample = np.arange(0, 2048, 4)
    assert_close(out.cpu().numpy()[sample], c.oracle(sample))


def test_config3_prefill_T4096_zipf_256_tokens(pkg, O, torch):
    c = LayerCase(pkg, O, torch, 4096, seed=3, logits_kind="zipf")
    out = run(c, torch)
    sample = np.sort(np.random.default_rng(0).choice(4096, 256, replace=False))
    assert_close(out.cpu().numpy()[sample], c.oracle(sample))


def test_config5_mixed_T32768_256_tokens(pkg, O, torch):
    c = LayerCase(pkg, O, torch, 32768, seed=5)
    out = run(c, torch)
    sample = mixed_sample(5)
    assert len(sample) == 256
    assert_close(out.cpu().numpy()[sample], c.oracle(sample))


def test_config4_ubatch_accumulates_twice(pkg, O, torch):
    """Two consecutive micro-batch forwards into one residual (the bench's
    layer loop): out = FFN(x) + FFN(x)."""
    c = LayerCase(pkg, O, torch, 1024, seed=44)
    out = torch.zeros(1024, 2048, device="cuda")
    for _ in range(2):
        c.layer.forward(c.weights, c.xd, c.ld, out, accumulate=True)
    torch.cuda.synchronize()
    assert c.layer.read_flags() == 0
    sample = np.arange(0, 1024, 8)
    want = c.oracle(sample)
    assert_close(out.cpu().numpy()[sample], (want.astype(np.float64) * 2).astype(np.float32))
