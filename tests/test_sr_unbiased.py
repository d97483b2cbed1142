"""Stochastic rounding of the 1Q re-quantisation is unbiased over 10^4 draws.

One 128-element block state is tiled over 10^4 blocks with identical inputs;
the Philox counter includes the block index, so every block draws fresh
uniforms and each element position gets 10^4 independent roundings of the
same continuous index c = (ln v - min) / span * 2^bits. The mean stored
index must equal E[r] = floor(c) + frac(c) (or the clamp value 2^bits - 1)
within 5 standard errors, per element and pooled (reference semantics:
quantize.py:276-294, round up iff u < frac).
"""
import numpy as np
import pytest
import torch

DRAWS = 10_000


def _case(oracle, nbits, seed=3):
    rng = np.random.default_rng(seed)
    idx, hdr = oracle.v_init(128)
    for _ in range(3):  # evolve to a spread-out block state
        g = (rng.standard_normal(128) * 10.0 ** rng.uniform(-5, -1, 128)).astype(np.float32)
        idx, hdr, _ = oracle.v_update(idx, hdr, g, nbits, 0.999, rng.random(128, np.float32))
    g = (rng.standard_normal(128) * 10.0 ** rng.uniform(-4, -2, 128)).astype(np.float32)
    return (np.tile(idx, DRAWS), np.tile(hdr, DRAWS), np.tile(g, DRAWS))


def _expected(oracle, v_block, nbits):
    """E[stored index] per element from the fp32 steps of the re-quantisation."""
    f32 = np.float32
    L = oracle.logf(np.maximum(v_block, f32(1e-38)))
    vmin, vmax = L.min(), L.max()
    nspan = np.maximum(f32(vmax - vmin), f32(1e-10))
    c = ((L - vmin) / nspan) * f32(1 << nbits)
    fl = np.floor(c)
    fr = (c - fl).astype(np.float64)
    top = (1 << nbits) - 1
    mean = np.where(fl >= top, float(top), fl + fr)
    var = np.where(fl >= top, 0.0, fr * (1.0 - fr))
    return mean, var


def _check(r, mean, var):
    r = r.reshape(DRAWS, 128).astype(np.float64)
    got = r.mean(axis=0)
    se = np.sqrt(var / DRAWS)
    assert np.all(np.abs(got - mean) <= 5.0 * se + 1e-9), np.max(np.abs(got - mean) - 5 * se)
    pooled = (r - mean).mean()
    assert abs(pooled) <= 5.0 * np.sqrt(var.sum() / DRAWS) / 128 + 1e-12
    assert (var > 0.01).sum() >= 32  # the case really exercises fractional roundings


@pytest.mark.parametrize("nbits", [2, 4, 8])
def test_sr_unbiased_checker(oracle, nbits):
    idx, hdr, g = _case(oracle, nbits)
    n = g.size
    u = oracle.sr_uniforms(n, 5, 9, 0x1234)
    oi, _, v = oracle.v_update(idx, hdr, g, nbits, 0.999, u)
    mean, var = _expected(oracle, v[:128], nbits)
    _check(oi, mean, var)


@pytest.mark.gpu
@pytest.mark.parametrize("nbits", [2, 4, 8])
def test_sr_unbiased_cuda(oracle, nbits):
    from turboadam_b200.oneq import fused_v_update

    idx, hdr, g = _case(oracle, nbits)
    n = g.size
    ni, _, v = fused_v_update(torch.from_numpy(idx).cuda(),
                              torch.from_numpy(hdr.view(np.float16)).cuda(),
                              torch.from_numpy(g).cuda(), 0.999, nbits, 128, n,
                              seed=0xABCDEF, tensor_id=3, step=11)
    v = v.cpu().numpy()
    assert np.array_equal(v.reshape(DRAWS, 128), np.tile(v[:128], (DRAWS, 1)))
    mean, var = _expected(oracle, v[:128], nbits)
    _check(ni.cpu().numpy(), mean, var)
