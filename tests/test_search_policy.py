"""The batched search's policy arithmetic against the reference's formulas (CPU).

``compute_search_policy`` must give, row by row, what the reference's
``compute_search_policy`` (stratego/search/mirror_descent.py:32-76) gives on
the legal moves of that row, and ``magnet_policy`` what
``SearchEngine._compute_magnet_probs`` (:156-177) gives.  Both reference
functions are restated here in numpy, line for line.
"""

from __future__ import annotations

import numpy as np
import torch

from ataraxos_b200.search import compute_search_policy, magnet_policy


def _ref_search_policy(q, net, mag, alpha, beta):
    eps = 1e-8
    log_unnorm = (q + alpha * np.log(mag + eps) + beta * np.log(net + eps)) / (alpha + beta)
    log_unnorm -= np.max(log_unnorm)
    pi = np.exp(log_unnorm)
    pi /= np.sum(pi)
    return pi


def _ref_magnet(legal):
    piece_moves = {}
    for i, a in enumerate(legal):
        piece_moves.setdefault(a // 100, []).append(i)
    probs = np.zeros(len(legal))
    for idx in piece_moves.values():
        for i in idx:
            probs[i] = 1.0 / len(piece_moves) / len(idx)
    return probs


def test_search_policy_matches_reference_rows():
    rng = np.random.default_rng(0)
    R = 7
    legal = np.zeros((R, 10000), dtype=bool)
    for r in range(R):
        legal[r, rng.choice(10000, size=int(rng.integers(1, 60)), replace=False)] = True
    q = rng.uniform(-1, 1, size=(R, 10000))
    net = rng.dirichlet(np.ones(10000), size=R)
    mag = rng.dirichlet(np.ones(10000), size=R)
    for alpha, beta in ((0.002, 0.02), (0.1, 0.5)):
        pi = compute_search_policy(torch.from_numpy(q), torch.from_numpy(net), torch.from_numpy(mag), alpha, beta,
                                   legal=torch.from_numpy(legal)).numpy()
        for r in range(R):
            idx = np.nonzero(legal[r])[0]
            ref = _ref_search_policy(q[r, idx], net[r, idx], mag[r, idx], alpha, beta)
            np.testing.assert_allclose(pi[r, idx], ref, rtol=1e-12, atol=1e-15)
            assert (pi[r, ~legal[r]] == 0).all()


def test_magnet_policy_matches_reference():
    rng = np.random.default_rng(1)
    R = 5
    mask = np.zeros((R, 100, 100), dtype=bool)
    for r in range(R):
        for src in rng.choice(100, size=int(rng.integers(1, 20)), replace=False):
            mask[r, src, rng.choice(100, size=int(rng.integers(1, 8)), replace=False)] = True
    rho = magnet_policy(torch.from_numpy(mask)).numpy()
    for r in range(R):
        legal = np.nonzero(mask[r].reshape(-1))[0]
        np.testing.assert_allclose(rho[r, legal], _ref_magnet(legal), rtol=1e-15)
        assert abs(rho[r].sum() - 1.0) < 1e-12
