"""The rank-128 LoRA slot fold restated in oracle.packs.fold_slots (moss/mossrun/lorafold.cpp:200-284
`fold`), checked on the CPU against its definition: B'^T A' is the best rank-128 approximation of
BT^T AM (Eckart-Young, numpy SVD of the full product), exact when the stacked rank is at most 128,
with the singular values carried by B' (the rows of A' orthonormal)."""
import numpy as np
import pytest

from oracle import packs as op


def _factors(seed, eff, ur, N=300, I=256):
    rng = np.random.default_rng(seed)
    BT, AM = np.zeros((128 + ur, N)), np.zeros((128 + ur, I))
    BT[:eff], AM[:eff] = rng.standard_normal((eff, N)), rng.standard_normal((eff, I))
    BT[128:], AM[128:] = rng.standard_normal((ur, N)), rng.standard_normal((ur, I))
    return BT, AM


def _rel(a, b):
    return np.linalg.norm(a - b) / np.linalg.norm(b)


@pytest.mark.parametrize("eff,ur", [(40, 64), (0, 128), (127, 1)])
def test_fold_is_exact_up_to_rank_128(eff, ur):
    BT, AM = _factors(1, eff, ur)
    Bo, Ao = op.fold_slots(BT, AM)
    assert _rel(Bo.astype(np.float64).T @ Ao, BT.T @ AM) < 1e-6


@pytest.mark.parametrize("ur", [1, 64, 128])
def test_fold_is_the_best_rank_128_approximation(ur):
    BT, AM = _factors(2, 128, ur)
    P = BT.T @ AM
    U, S, Vt = np.linalg.svd(P)
    T = (U[:, :128] * S[:128]) @ Vt[:128]
    Bo, Ao = op.fold_slots(BT, AM)
    Q = Bo.astype(np.float64).T @ Ao
    assert _rel(Q, T) < 1e-6
    # the residual is what the truncation leaves: the tail singular values
    assert abs(np.linalg.norm(P - Q) - np.sqrt((S[128:] ** 2).sum())) < 1e-4 * np.linalg.norm(P)
    # A' rows orthonormal, B' carries the singular values
    G = Ao.astype(np.float64) @ Ao.T
    assert np.allclose(G, np.eye(128), atol=1e-5)
    assert np.allclose(np.linalg.norm(Bo.astype(np.float64), axis=1), S[:128], rtol=1e-5)
