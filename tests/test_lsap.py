"""Host LSAP solver vs scipy (the reference's solver is a port of scipy's
rectangular LSAP, `src/rfdetr/utils/scipy_rectangular_lsap.cpp`)."""
import numpy as np
import pytest
import torch
from scipy.optimize import linear_sum_assignment

from mmltk_b200.ops import native


@pytest.mark.parametrize("shape", [(1, 1), (3, 3), (7, 4), (4, 7), (30, 10), (10, 30), (300, 9), (50, 50)])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_lsap_matches_scipy(shape, seed):
    rng = np.random.default_rng(seed)
    c = rng.normal(size=shape)
    r, k = native().lsap(torch.from_numpy(c), False)
    sr, sk = linear_sum_assignment(c)
    assert np.array_equal(r.numpy(), sr)
    assert np.array_equal(k.numpy(), sk)


def test_lsap_maximize_and_integer_ties():
    rng = np.random.default_rng(5)
    c = rng.integers(0, 4, size=(12, 20)).astype(np.float64)
    r, k = native().lsap(torch.from_numpy(c), False)
    sr, sk = linear_sum_assignment(c)
    assert c[r.numpy(), k.numpy()].sum() == c[sr, sk].sum()
    r, k = native().lsap(torch.from_numpy(c), True)
    sr, sk = linear_sum_assignment(c, maximize=True)
    assert c[r.numpy(), k.numpy()].sum() == c[sr, sk].sum()


def test_lsap_rejects_nan():
    c = torch.tensor([[1.0, float("nan")], [0.0, 1.0]], dtype=torch.float64)
    with pytest.raises(RuntimeError):
        native().lsap(c, False)


def test_match_batched_groups_and_sanitize():
    torch.manual_seed(0)
    NL, B, G, Qg, T = 2, 3, 4, 25, 6
    cost = torch.randn(NL, B, G * Qg, T)
    cost[0, 0, 3, 0] = float("inf")
    counts = torch.tensor([6, 0, 3])
    m = native().match_batched(cost, counts, G)
    assert m.shape == (NL, B, G, T)
    for l in range(NL):
        for b in range(B):
            n = int(counts[b])
            for g in range(G):
                sub = cost[l, b, g * Qg:(g + 1) * Qg, :n].double().numpy()
                if n == 0:
                    assert (m[l, b, g] == -1).all()
                    continue
                finite = np.isfinite(sub)
                fmax, amax = sub[finite].max(), np.abs(sub[finite]).max()
                sub = np.where(finite, sub, fmax + amax + 1.0)
                rows, cols = linear_sum_assignment(sub)
                exp = np.full(T, -1)
                exp[cols] = rows + g * Qg
                assert np.array_equal(m[l, b, g].numpy(), exp)
