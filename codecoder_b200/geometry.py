"""Rotated-surface-code Tanner graph in the reference's gather-table format.

The reference keeps one `Geometry` per code: for every target type a `(NT, K)` table of source node indices (the value
N_sources is the zero pad row) and an inverse `(N_sources, K)` table giving, for every source and relation, the flat
position `n K + r` of the target that reads it (`NT K` = none); every relation reads each source at most once
(training/bb/ising_compare/bb/cascade_net.py:84-127).  This module builds the same tables for the rotated surface code
of distance d over R rounds of phenomenological noise.

Plaquette grid.  Data qubit (r, c), 0 <= r, c < d, sits in the cell whose corners are the plaquette places
(r + di, c + dj), di, dj in {0, 1}, of the (d + 1) x (d + 1) place grid (cascade/d13/surface/surface_net.py:20-26 and
surface_layout.py "data qubit (r, c) is the one cell (r, c) .. (r + 1, c + 1)").  Interior places (1 <= i, j <= d - 1)
all hold a stabilizer, X where i + j is even and Z where it is odd (a checkerboard, as surface_layout.Layout checks);
on the top and bottom rows only the X places hold one (weight-2 X checks), on the left and right columns only the Z
places.  That gives d^2 - 1 checks per round, (d^2 - 1) / 2 of each type.

Nodes.  Check node (c, t, s) has index (c T + t) nh + s with c = 0 X / 1 Z, t = 0 .. T - 1 (T = R: one detector layer
per round), nh = (d^2 - 1) / 2 and s the place's rank among the places of type c in row-major order: the reference's
type-major order (cascade_net.py:5-8).  Data node (t, q) has index t d^2 + q, q = r d + c.

Relations.  K = 8 = 4 corners x 2 time offsets, relation r = 2 j + k (corner j, offset k) as in cascade_net.py:86-87.
check -> data: data (t, r, c) reads the plaquette at corner j = (di, dj) in NW, NE, SW, SE order at time t + dt,
dt in DT_C2D = (0, +1); data -> check: check (t, i, j) reads the data qubit (i - 1 + a, j - 1 + b) at its corner
(a, b) in NW, NE, SW, SE order at time t + dt, dt in DT_D2C = (-1, 0) (cascade_net.py:42-43).  Missing corners and
times outside 0 .. T - 1 read the pad row.
"""
from __future__ import annotations

import numpy as np

DT_C2D = (0, 1)          # data (t) <- checks (t + dt)            (cascade_net.py:42)
DT_D2C = (-1, 0)         # check (t) <- data (t + dt)             (cascade_net.py:43)
CORNERS = ((0, 0), (0, 1), (1, 0), (1, 1))   # NW, NE, SW, SE
CHECK_X, CHECK_Z = 0, 1
ERR_X, ERR_Z = 0, 1      # logit channels: predicted X flip, predicted Z flip of a data qubit


def place_type(d: int, i: int, j: int) -> int:
    """Stabilizer type at place (i, j) of the (d + 1) x (d + 1) grid: 0 X, 1 Z, -1 no stabilizer."""
    if not (0 <= i <= d and 0 <= j <= d):
        return -1
    t = (i + j) & 1                       # X on even, Z on odd
    if 1 <= i <= d - 1 and 1 <= j <= d - 1:
        return t
    if (i == 0 or i == d) and 1 <= j <= d - 1:
        return CHECK_X if t == CHECK_X else -1
    if (j == 0 or j == d) and 1 <= i <= d - 1:
        return CHECK_Z if t == CHECK_Z else -1
    return -1                             # the four corners of the grid


class RotatedSurface:
    """Node layout and gather tables of the rotated surface code (module docstring).

    Attributes in the reference's Geometry format (cascade_net.py:84-127):
      c2d[0]      (N_d, K) int64   source check per data node and relation, pad = N_c
      d2c[c]      (T nh, K) int64  source data node per check of type c and relation, pad = N_d
      inv_c2d[0]  (N_c, K) int64   flat target position n K + r reading check u through r, none = N_d K
      inv_d2c[c]  (N_d, K) int64   likewise for the checks of type c, none = T nh K
    Extra tables for the pre-decoder:
      d2c_all     (N_c, K)         d2c[0] and d2c[1] stacked in node order
      xor_nbr     (N_d, 2, 2)      for a predicted X (Z) flip of data node n, the Z (X) checks at the same round
                                   whose detector it flips; -1 = none
      check_type  (N_c,)           0 X / 1 Z
    """

    def __init__(self, d: int, rounds: int | None = None):
        if d < 3 or d % 2 == 0:
            raise ValueError("the rotated surface code needs an odd distance d >= 3")
        self.d = d
        self.R = self.T = T = d if rounds is None else int(rounds)
        if T < 1:
            raise ValueError("rounds must be >= 1")
        self.K = K = len(CORNERS) * 2
        self.n_data_round = nq = d * d
        self.nh = nh = (d * d - 1) // 2
        self.n_check_round = 2 * nh
        self.N_d = N_d = T * nq
        self.N_c = N_c = T * 2 * nh
        # places of each type, row-major
        places = [[], []]
        for i in range(d + 1):
            for j in range(d + 1):
                ty = place_type(d, i, j)
                if ty >= 0:
                    places[ty].append((i, j))
        if len(places[0]) != nh or len(places[1]) != nh:
            raise ValueError("unexpected stabilizer count")
        self.places = places
        rank = {}
        for ty in range(2):
            for s, ij in enumerate(places[ty]):
                rank[ij] = (ty, s)
        self._rank = rank

        def check_node(ty, t, s):
            return (ty * T + t) * nh + s

        # check -> data: data (t, r, c) <- plaquette (r + di, c + dj) at t + dt
        c2d = np.full((T, nq, K), N_c, np.int64)
        for r in range(d):
            for c in range(d):
                q = r * d + c
                for jc, (di, dj) in enumerate(CORNERS):
                    ij = (r + di, c + dj)
                    if ij not in rank:
                        continue
                    ty, s = rank[ij]
                    for k, dt in enumerate(DT_C2D):
                        for t in range(T):
                            ts = t + dt
                            if 0 <= ts < T:
                                c2d[t, q, 2 * jc + k] = check_node(ty, ts, s)
        self.c2d = [c2d.reshape(N_d, K)]

        # data -> check: check (t, i, j) <- data (i - 1 + a, j - 1 + b) at t + dt
        d2c = []
        for ty in range(2):
            tab = np.full((T, nh, K), N_d, np.int64)
            for s, (i, j) in enumerate(places[ty]):
                for jc, (a, b) in enumerate(CORNERS):
                    r, c = i - 1 + a, j - 1 + b
                    if not (0 <= r < d and 0 <= c < d):
                        continue
                    for k, dt in enumerate(DT_D2C):
                        for t in range(T):
                            ts = t + dt
                            if 0 <= ts < T:
                                tab[t, s, 2 * jc + k] = ts * nq + r * d + c
            d2c.append(tab.reshape(T * nh, K))
        self.d2c = d2c
        self.d2c_all = np.concatenate(d2c, 0)
        self.inv_c2d = [self.inverse(self.c2d[0], N_c)]
        self.inv_d2c = [self.inverse(x, N_d) for x in self.d2c]

        # node attributes
        self.check_type = np.repeat(np.arange(2), T * nh).astype(np.int64)
        self.check_t = np.tile(np.repeat(np.arange(T), nh), 2).astype(np.int64)
        # the checks round by round, X then Z within a round: the order a data -> check step visits them so the data
        # nodes of a round are swept once for both check types (node order keeps the types apart)
        self.check_round_order = np.lexsort((np.arange(N_c), self.check_type, self.check_t)).astype(np.int64)
        self.check_place = np.array([places[ty][s] for ty in range(2) for _ in range(T) for s in range(nh)], np.int64)

        # syndrome cancellation: a predicted X flip of data (t, q) flips the Z checks around q at round t,
        # a predicted Z flip the X checks (phenomenological detectors, sampler below)
        xor_nbr = np.full((T, nq, 2, 2), -1, np.int64)
        for r in range(d):
            for c in range(d):
                q = r * d + c
                fill = [0, 0]
                for di, dj in CORNERS:
                    ij = (r + di, c + dj)
                    if ij not in rank:
                        continue
                    ty, s = rank[ij]
                    e = ERR_X if ty == CHECK_Z else ERR_Z
                    for t in range(T):
                        xor_nbr[t, q, e, fill[e]] = check_node(ty, t, s)
                    fill[e] += 1
        self.xor_nbr = xor_nbr.reshape(N_d, 2, 2)

        # parity-check matrices per round (checks of one type x data qubits)
        hx = np.zeros((nh, nq), np.uint8)
        hz = np.zeros((nh, nq), np.uint8)
        for ty, h in ((CHECK_X, hx), (CHECK_Z, hz)):
            for s, (i, j) in enumerate(places[ty]):
                for a, b in CORNERS:
                    r, c = i - 1 + a, j - 1 + b
                    if 0 <= r < d and 0 <= c < d:
                        h[s, r * d + c] = 1
        self.hx, self.hz = hx, hz

    def inverse(self, idx: np.ndarray, n_src: int) -> np.ndarray:
        """Inverse gather table (cascade_net.py:119-127): inv[u, r] = n K + r for the target n reading source u
        through relation r, n_targets K where none; raises if a relation reads one source twice."""
        nt, K = idx.shape
        inv = np.full((n_src, K), nt * K, np.int64)
        n, r = np.nonzero(idx < n_src)
        u = idx[n, r]
        if len(np.unique(u * K + r)) != len(u):
            raise ValueError("a relation reads one source twice")
        inv[u, r] = n * K + r
        return inv

    def check_node(self, ty: int, t: int, s: int) -> int:
        return (ty * self.T + t) * self.nh + s

    def describe(self) -> dict:
        return {"d": self.d, "rounds": self.R, "K": self.K, "checks_per_round": self.n_check_round,
                "data_per_round": self.n_data_round, "N_c": self.N_c, "N_d": self.N_d}


def pad_fraction(idx: np.ndarray, pad: int) -> float:
    """Fraction of (target, relation) slots that read the pad row."""
    return float((idx == pad).mean())
