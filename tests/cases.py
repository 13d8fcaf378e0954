"""Shared inputs and checks of the GPU parity tests.

* `zipf_logits` -- config 3's Zipf(1.1) route skew as router logits;
* `mixed_layout` / `mixed_sample` -- config 5's continuous-batching pack
  (56 decode tokens and 8 prefill chunks, 32,768 tokens) and the tokens of it
  that are checked;
* `LayerCase` -- one seeded layer (synthetic Q4_0 weights, x, logits, shared
  gate) on the GPU plus its CPU oracle;
* `assert_close` -- the layer-output bar max|err| <= 1e-3 * RMS(output).
"""
import os

import numpy as np

TOL_RMS = 1e-3
H, I, E = 2048, 512, 512
ORACLE_THREADS = max(1, min(32, os.cpu_count() or 1))


def f32bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def zipf_logits(rng, T, s=1.1):
    """Zipf(s) route skew: -s*ln(1+pi(e)) + Gumbel noise (top-10 of Gumbel-perturbed
    log-weights samples experts without replacement in proportion to the weights)."""
    perm = rng.permutation(E)
    base = -s * np.log1p(perm.astype(np.float64))
    g = -np.log(-np.log(rng.random((T, E))))
    return (base[None, :] + g).astype(np.float32)


def mixed_layout(seed, total=32768, decode=56, chunks=8, lo=256, hi=4096):
    """Config 5's ragged pack: `decode` single-token sequences first, then
    `chunks` prefill chunks.  Chunk lengths are drawn uniformly from [lo, hi]
    and scaled to fill the rest of `total` (the draws alone cannot reach it).
    Returns (chunk start offsets, chunk lengths)."""
    rng = np.random.default_rng(seed)
    draw = rng.integers(lo, hi + 1, chunks).astype(np.float64)
    rest = total - decode
    lens = np.floor(draw / draw.sum() * rest).astype(np.int64)
    lens[-1] += rest - lens.sum()
    starts = decode + np.concatenate([[0], np.cumsum(lens)[:-1]])
    return starts, lens


def mixed_sample(seed, n=256, decode=56):
    """Tokens of the config 5 pack to check: every decode token, the first and
    last 8 tokens of each prefill chunk, and random tokens to make up `n`."""
    starts, lens = mixed_layout(seed, decode=decode)
    pick = set(range(decode))
    for s, l in zip(starts, lens):
        pick.update(range(int(s), int(s) + 8))
        pick.update(range(int(s + l) - 8, int(s + l)))
    rng = np.random.default_rng(seed + 1)
    total = int(starts[-1] + lens[-1])
    while len(pick) < n:
        pick.add(int(rng.integers(0, total)))
    return np.array(sorted(pick))


class LayerCase:
    """One seeded layer on the GPU plus its oracle (synthetic weights are
    generated bit-identically on both sides)."""

    def __init__(self, pkg, O, torch, T, seed, logits_kind="normal", max_tokens=None, down_type=2):
        self.pkg, self.O, self.T, self.seed, self.down_type = pkg, O, T, seed, down_type
        rng = np.random.default_rng(seed)
        self.x = rng.standard_normal((T, H)).astype(np.float32)
        self.logits = zipf_logits(rng, T) if logits_kind == "zipf" else rng.standard_normal((T, E)).astype(np.float32)
        self.gate_vec = (rng.standard_normal(H) * 0.02).astype(np.float32)
        self.desc = pkg.make_desc(max_tokens=max_tokens or T)
        self.weights = pkg.MoeWeights(self.desc, down_type)
        self.weights.synthesize(seed, 0)
        self.weights.upload_shared_gate(self.gate_vec)
        self.layer = pkg.MoeLayer(self.desc)
        self.xd = torch.from_numpy(self.x).cuda()
        self.ld = torch.from_numpy(self.logits).cuda()

    def expert(self, e):
        return self.O.synth_expert(self.seed, 0, e, down_type=self.down_type)

    def oracle(self, tokens=None):
        out, _, _, _ = self.O.moe_layer(self.x, self.logits, self.expert, self.expert(512), self.gate_vec, tokens,
                                        down_type=self.down_type, threads=ORACLE_THREADS)
        return out


def assert_close(got, want):
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    err = float(np.max(np.abs(got.astype(np.float64) - want)))
    assert err <= TOL_RMS * rms, f"max|err|={err:.3e} rms={rms:.3e}"
    return err / rms
