"""The sampler's float functions and virtual logits (CPU oracle).

The kernel's softmax sampler computes its noise with its own ln / cos(2 pi u)
/ exp, written as fixed sequences of IEEE operations so that the oracle
reproduces them bit for bit (the GPU parity tests check that the choices and
log-probs are identical).  Here: the functions' error bounds against float64
references, and the moments of the virtual N(0,1) logits and Gumbel noise.
"""

from __future__ import annotations

import math

import numpy as np

import oracle


def _ulps(got: float, ref: float) -> float:
    return abs(got - ref) / float(np.spacing(np.float32(abs(ref))))


def test_ln_within_three_ulp():
    rng = np.random.default_rng(1)
    xs = np.exp(rng.uniform(math.log(2.0 ** -25), math.log(40.0), 20000)).astype(np.float32)
    grid = (np.arange(1, 2 ** 24, 65537) * 2.0 ** -24).astype(np.float32)  # the sampler's uniforms
    for x in np.concatenate([xs, grid, np.float32([0.5, 2.0, 1 - 2 ** -24, 2 ** -24])]):
        assert _ulps(oracle.noise_fn("ln", float(x)), math.log(float(x))) <= 3.0, x
    assert oracle.noise_fn("ln", 1.0) == 0.0


def test_cos2pi_within_1e7():
    rng = np.random.default_rng(2)
    us = (rng.integers(1, 2 ** 24, 20000) * 2.0 ** -24).astype(np.float32)
    for u in np.concatenate([us, np.float32([0.25, 0.5, 0.75, 0.125, 2 ** -24, 1 - 2 ** -24])]):
        assert abs(oracle.noise_fn("cos2pi", float(u)) - math.cos(2 * math.pi * float(u))) <= 1.2e-7, u


def test_exp_within_one_ulp():
    rng = np.random.default_rng(3)
    for z in np.concatenate([rng.uniform(-80, 12, 20000).astype(np.float32), np.float32([0.0, -1.0, 1.0])]):
        assert _ulps(oracle.noise_fn("exp", float(z)), math.exp(float(z))) <= 1.0, z
    assert oracle.noise_fn("exp", -81.0) == 0.0


def test_virtual_logits_and_gumbel_moments():
    z, g = np.array([oracle.logit_noise(7, e, 3, a) for e in range(40) for a in range(0, 10000, 7)]).T
    n = z.size
    assert abs(z.mean()) < 4 / math.sqrt(n) and abs(z.std() - 1) < 0.01
    assert abs(np.mean(np.abs(z) > 1.959964) - 0.05) < 0.005
    assert abs(g.mean() - 0.5772157) < 4 * 1.28 / math.sqrt(n)  # Gumbel(0,1): mean Euler's gamma, sd pi/sqrt 6
