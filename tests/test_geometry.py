"""Rotated-surface tables: counts, the reference's table/inverse conventions, the code's algebra, the XOR map."""
import numpy as np
import pytest

from codecoder_b200.geometry import CHECK_X, CHECK_Z, CORNERS, RotatedSurface, pad_fraction, place_type
from codecoder_b200.sampler import sample


@pytest.mark.parametrize("d,R", [(3, 3), (5, 5), (9, 9), (13, 13), (17, 3)])
def test_counts(d, R):
    g = RotatedSurface(d, R)
    assert g.n_check_round == d * d - 1 and g.n_data_round == d * d
    assert g.N_c == R * (d * d - 1) and g.N_d == R * d * d
    assert g.c2d[0].shape == (g.N_d, 8) and g.d2c_all.shape == (g.N_c, 8)
    assert len(g.d2c) == 2 and g.d2c[0].shape == (R * g.nh, 8)


def test_config_sizes():
    # the workload sizes the path is specified on: checks / data qubits per round
    assert RotatedSurface(5, 5).n_check_round == 24
    assert RotatedSurface(9, 9).n_check_round == 80 and RotatedSurface(9, 9).n_data_round == 81
    g = RotatedSurface(13, 13)
    assert (g.n_check_round, g.n_data_round, g.N_c, g.N_d) == (168, 169, 2184, 2197)
    g = RotatedSurface(17, 3)
    assert (g.n_check_round, g.N_c, g.N_d) == (288, 864, 867)


@pytest.mark.parametrize("d", [3, 5, 7, 13])
def test_stabilizers_commute_and_are_independent(d):
    g = RotatedSurface(d, 1)
    assert not ((g.hx.astype(int) @ g.hz.T.astype(int)) % 2).any()
    # weights 2 or 4, each data qubit in 1..2 checks of each type
    for h in (g.hx, g.hz):
        w = h.sum(1)
        assert set(w.tolist()) <= {2, 4}
        col = h.sum(0)
        assert col.min() >= 1 and col.max() <= 2
    # GF(2) rank of each type = (d^2 - 1) / 2 (independent generators)
    for h in (g.hx, g.hz):
        m = h.copy() % 2
        rank = 0
        for c in range(m.shape[1]):
            piv = np.nonzero(m[rank:, c])[0]
            if len(piv) == 0:
                continue
            p = rank + piv[0]
            m[[rank, p]] = m[[p, rank]]
            for r in range(m.shape[0]):
                if r != rank and m[r, c]:
                    m[r] ^= m[rank]
            rank += 1
        assert rank == g.nh


def test_checkerboard_and_boundaries():
    d = 5
    assert place_type(d, 0, 0) == -1 and place_type(d, 0, d) == -1
    for j in range(1, d):
        assert place_type(d, 0, j) in (CHECK_X, -1)
        assert place_type(d, j, 0) in (CHECK_Z, -1)
    for i in range(1, d):
        for j in range(1, d):
            assert place_type(d, i, j) == (i + j) % 2


@pytest.mark.parametrize("d,R", [(3, 3), (5, 4), (9, 9)])
def test_tables_follow_reference_conventions(d, R):
    g = RotatedSurface(d, R)
    # pad = number of sources, every relation reads a source at most once (cascade_net.py:119-127)
    for idx, ns, inv in ((g.c2d[0], g.N_c, g.inv_c2d[0]), (g.d2c[0], g.N_d, g.inv_d2c[0]),
                         (g.d2c[1], g.N_d, g.inv_d2c[1])):
        assert idx.min() >= 0 and idx.max() <= ns
        nt, K = idx.shape
        assert inv.shape == (ns, K)
        n, r = np.nonzero(idx < ns)
        assert (inv[idx[n, r], r] == n * K + r).all()
        assert ((inv == nt * K) | (inv < nt * K)).all()
        assert (inv < nt * K).sum() == len(n)
    # check -> data and data -> check are the same adjacency (corner j of a data qubit <-> corner 3 - j of a check)
    for n in range(g.N_d):
        t, q = divmod(n, g.n_data_round)
        for jc in range(4):
            c = g.c2d[0][n, 2 * jc]             # dt = 0
            if c == g.N_c:
                continue
            assert g.d2c_all[c, 2 * (3 - jc) + 1] == n   # the check reads this data qubit at dt = 0
    # time offsets: c2d dt = (0, +1), d2c dt = (-1, 0)
    T = g.T
    for n in range(g.N_d):
        t = n // g.n_data_round
        for jc in range(4):
            a, b = g.c2d[0][n, 2 * jc], g.c2d[0][n, 2 * jc + 1]
            if t == T - 1:
                assert b == g.N_c
            if a < g.N_c and b < g.N_c:
                assert g.check_t[b] == g.check_t[a] + 1


def test_pad_fraction_d13():
    g = RotatedSurface(13, 13)
    f_c2d = pad_fraction(g.c2d[0], g.N_c)
    f_d2c = pad_fraction(g.d2c_all, g.N_d)
    assert 0.05 < f_c2d < 0.25 and 0.05 < f_d2c < 0.25


@pytest.mark.parametrize("d,R", [(3, 4), (5, 5), (7, 3)])
def test_perfect_prediction_cancels_every_detector(d, R):
    """With no measurement flips, XOR-ing the true data flips into the detectors leaves a zero residual: the
    xor_nbr map is exactly the detector model of the sampler."""
    import sys, os
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle.predecoder_oracle import cancel
    g = RotatedSurface(d, R)
    det, err = sample(g, 0.05, 200, seed=3, q=0.0)
    assert det.any()
    res = cancel(det, err, g)
    assert not res.any()
    # with measurement flips the residual is exactly the measurement-flip pattern m[t] ^ m[t-1]
    det2, err2 = sample(g, 0.05, 200, seed=4, q=0.05)
    res2 = cancel(det2, err2, g)
    assert res2.any()
