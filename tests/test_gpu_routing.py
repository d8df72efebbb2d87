"""Routing of pre-decoded shots to a fallback decoder (C ABI bpc_route) against the oracle's restatement of the
reference's rule (evaluation/convlines/decoder.py:116-142): the routed mask, the ordered indices, the hand-off rows,
the per-shot confidence and residual weight, bit for bit; and decode() with a matcher."""
import numpy as np
import pytest
import torch

from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.modules import PreDecoder
from codecoder_b200.params import CONFIGS, init_params
from codecoder_b200.routing import decode, route
from codecoder_b200.sampler import sample
from oracle import predecoder_oracle as orc

pytestmark = pytest.mark.gpu


def check(lg, rs, tau, route_residual):
    r = route(torch.as_tensor(lg).cuda(), torch.as_tensor(rs).cuda(), tau, route_residual)
    routed, index, handoff, conf, weight = orc.route(lg, rs, tau, route_residual)
    assert np.array_equal(r.routed.cpu().numpy(), routed)
    assert np.array_equal(r.index.cpu().numpy(), index)
    assert np.array_equal(r.handoff.cpu().numpy(), handoff)
    assert np.array_equal(r.conf.cpu().numpy(), conf)
    assert np.array_equal(r.weight.cpu().numpy(), weight)
    return r


@pytest.mark.parametrize("B", [0, 1, 1023, 1024, 5000])
@pytest.mark.parametrize("tau,route_residual", [(0.05, True), (0.05, False), (0.0, True), (10.0, False)])
def test_route_matches_oracle(B, tau, route_residual):
    rng = np.random.default_rng(B + int(tau * 100))
    N_d, N_c = 169, 168
    lg = rng.standard_normal((B, N_d, 2)).astype(np.float32)
    rs = (rng.random((B, N_c)) < 0.002).astype(np.uint8)
    r = check(lg, rs, tau, route_residual)
    if tau == 10.0:
        assert r.index.numel() == B                    # every shot routed
    if tau == 0.0 and not route_residual:
        assert r.index.numel() == 0


def test_route_on_the_predecoder_and_decode_with_a_matcher():
    cfg = CONFIGS["d9_bf16"]
    g = RotatedSurface(cfg.d, cfg.rounds)
    pd = PreDecoder(g, cfg, init_params(cfg, 31), device="cuda")
    det, _ = sample(g, cfg.p, 700, 32)
    d = torch.as_tensor(det).cuda()
    lg, rs = pd(d)
    check(lg.cpu().numpy(), rs.cpu().numpy(), 0.02, True)
    # a matcher that flips data qubit 0's X component for every residual it sees: the routed shots' corrections
    # are the network's flips with that bit toggled, the other shots' the network's flips
    seen = []

    def matcher(h):
        seen.append(h.copy())
        f = np.zeros((len(h), g.N_d, 2), np.uint8)
        f[:, 0, 0] = 1
        return f

    lg2, rs2, r, corr = decode(pd, d, 0.02, matcher)
    assert torch.equal(lg2, lg) and torch.equal(rs2, rs)
    base = (lg > 0).to(torch.uint8)
    expect = base.clone()
    expect[r.index, 0, 0] ^= 1
    assert torch.equal(corr, expect)
    assert len(seen) == (1 if r.index.numel() else 0)
    if seen:
        assert np.array_equal(seen[0], rs.cpu().numpy()[r.index.cpu().numpy()])
