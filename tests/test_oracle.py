"""The CPU oracle against the golden fixtures written by the reference's own gather_mm / BipartiteConv."""
import os

import numpy as np
import pytest
import torch

from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.params import PreDecoderConfig, init_params, storage_params
from oracle import predecoder_oracle as orc


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32)


@pytest.fixture(scope="module")
def bb72(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "bb72_c14_conv.npz")))


def test_oracle_gather_mm_matches_reference_bb72_c14(bb72):
    x = torch.as_tensor(bf16_to_f32(bb72["x_bf16"]))
    w = torch.as_tensor(bf16_to_f32(bb72["w_c2d_0_bf16"]))
    y = orc.gather_mm(x, w, bb72["c2d0"])
    np.testing.assert_allclose(y.numpy(), bb72["y_c2d0"], rtol=1e-5, atol=1e-5)
    y64 = orc.gather_mm_loop(x.numpy(), w.numpy(), bb72["c2d0"].astype(np.int64))
    np.testing.assert_allclose(y64, bb72["y_c2d0"], rtol=1e-4, atol=1e-4)


def test_oracle_bipartite_conv_matches_reference_module(bb72):
    x = torch.as_tensor(bf16_to_f32(bb72["x_bf16"]))
    w = {k: torch.as_tensor(bf16_to_f32(bb72[k + "_bf16"])) for k in ("w_c2d_0", "w_c2d_1", "w_d2c_0", "w_d2c_1")}
    y = orc.bipartite_conv(x, [w["w_c2d_0"], w["w_c2d_1"]], [w["w_d2c_0"], w["w_d2c_1"]],
                           [bb72["c2d0"], bb72["c2d1"]], [bb72["d2c0"], bb72["d2c1"]])
    np.testing.assert_allclose(y.numpy(), bb72["y_module"], rtol=1e-4, atol=1e-4)


def test_oracle_gather_mm_matches_reference_surface(golden_dir):
    z = np.load(os.path.join(golden_dir, "surface_gmm.npz"))
    keys = sorted({k.rsplit("_", 1)[0] for k in z.files})
    assert len(keys) == 10
    for key in keys:
        x = torch.as_tensor(bf16_to_f32(z[key + "_x"]))
        w = torch.as_tensor(bf16_to_f32(z[key + "_w"]))
        idx = z[key + "_idx"]
        d, R, ci, co, B, ns = z[key + "_meta"]
        g = RotatedSurface(int(d), int(R))
        table = g.c2d[0] if key.endswith("c2d") else g.d2c_all
        assert np.array_equal(table, idx), "fixture tables = this geometry's tables"
        np.testing.assert_allclose(orc.gather_mm(x, w, idx).numpy(), z[key + "_y"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["d3_fp32", "d5_fp32", "d5_bf16_c64"])
def test_oracle_predecoder_matches_reference_composition(golden_dir, name):
    z = np.load(os.path.join(golden_dir, f"predecoder_{name}.npz"))
    cfg = PreDecoderConfig(d=int(z["d"]), rounds=int(z["rounds"]), layers=int(z["layers"]),
                           channels=int(z["channels"]), dtype=str(z["dtype"]))
    g = RotatedSurface(cfg.d, cfg.rounds)
    params = init_params(cfg, int(z["seed"]))
    import hashlib
    h = hashlib.sha256()
    for k in sorted(params):
        h.update(k.encode())
        h.update(np.ascontiguousarray(params[k], np.float32).tobytes())
    assert h.hexdigest() == str(z["params_sha256"]), "seeded weights changed"
    p = storage_params(cfg, params)
    logits, res = orc.predecoder(g, cfg, p, z["det"])
    tol = 1e-4 if cfg.dtype == "f32" else 2e-2
    assert orc.logit_error(logits, z["logits"]) < (1e-5 if cfg.dtype == "f32" else 1e-2)
    assert orc.residual_mismatch_outside_band(res, z["residual"], z["logits"], g, tol) == 0
    # the fixture's residual is exactly det ^ cancel(its own logits)
    e = (z["logits"] > 0).astype(np.uint8)
    assert np.array_equal(orc.cancel(z["det"], e, g), z["residual"])


def test_band_helpers():
    ref = np.array([[[1.0, -2.0], [1e-6, 0.5]]])
    assert orc.band_mask(ref, 1e-3).sum() == 1
    assert orc.logit_error(ref, ref) == 0.0


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.fixture(scope="module")
def bwd(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "gather_mm_bwd.npz")))


def test_oracle_backward_matches_reference_op(bwd):
    names = sorted({k.rsplit("_", 1)[0] for k in bwd if not k.startswith("bb72")})
    assert len(names) == 4
    for nm in names:
        x = bf16_to_f32(bwd[nm + "_x"])
        w = bf16_to_f32(bwd[nm + "_w"])
        gy = bf16_to_f32(bwd[nm + "_gy"])
        idx = bwd[nm + "_idx"].astype(np.int64)
        NT, K = idx.shape
        Ci = x.shape[2]
        tgt = orc.target_table(bwd[nm + "_inv"], NT, K)
        assert _rel(orc.gather_mm_dgrad(gy, w, tgt, Ci), bwd[nm + "_gx"]) < 1e-5, nm
        assert _rel(orc.gather_mm_wgrad(x, gy, idx), bwd[nm + "_gw"]) < 1e-5, nm


def test_oracle_backward_matches_reference_module(bb72, bwd):
    w = [torch.as_tensor(bf16_to_f32(bb72[k + "_bf16"]), dtype=torch.float64).requires_grad_()
         for k in ("w_c2d_0", "w_c2d_1", "w_d2c_0", "w_d2c_1")]
    x = torch.as_tensor(bf16_to_f32(bwd["bb72_x"]), dtype=torch.float64).requires_grad_()
    y = orc.bipartite_conv(x, w[:2], w[2:], [bb72["c2d0"], bb72["c2d1"]], [bb72["d2c0"], bb72["d2c1"]])
    y.backward(torch.as_tensor(bf16_to_f32(bwd["bb72_gy"]), dtype=torch.float64))
    assert _rel(x.grad.numpy(), bwd["bb72_gx"]) < 1e-5
    assert _rel(w[0].grad.numpy(), bwd["bb72_gw_c2d0"]) < 1e-5
    assert _rel(w[3].grad.numpy(), bwd["bb72_gw_d2c1"]) < 1e-5


def test_oracle_cascade_block_matches_reference_c14(bb72, golden_dir):
    z = dict(np.load(os.path.join(golden_dir, "cascade_block_c14.npz")))
    p = {k: z[k] for k in z if k.startswith("bn")}
    p["down"] = bf16_to_f32(z["down_bf16"])
    p["up"] = bf16_to_f32(z["up_bf16"])
    p["w_c2d"] = [bf16_to_f32(bb72["w_c2d_0_bf16"]), bf16_to_f32(bb72["w_c2d_1_bf16"])]
    p["w_d2c"] = [bf16_to_f32(bb72["w_d2c_0_bf16"]), bf16_to_f32(bb72["w_d2c_1_bf16"])]
    out = orc.cascade_block(bf16_to_f32(z["h_bf16"]), p, [bb72["c2d0"], bb72["c2d1"]], [bb72["d2c0"], bb72["d2c1"]],
                            int(z["L"]), str(z["res"]), float(z["eps"]))
    assert _rel(out.numpy(), z["out"]) < 1e-5


def test_deep_parity_bar_accepts_a_correct_restatement_and_catches_planted_mistakes():
    """The full-depth bf16 bar: the oracle's own float32 restatement passes against the float64 one; a residual bit
    flipped outside the band, a residual that is not the XOR of its own logits, and logits off by a few percent
    everywhere all fail.  The mistakes are planted in copies of the oracle's outputs, on the CPU."""
    from codecoder_b200.sampler import sample
    cfg = PreDecoderConfig(d=5, rounds=5, layers=6, channels=32, dtype="bf16", p=0.02)
    g = RotatedSurface(cfg.d, cfg.rounds)
    sp = storage_params(cfg, init_params(cfg, 41))
    det, _ = sample(g, cfg.p, 96, 42)
    ref64, res64 = orc.predecoder_batched(g, cfg, sp, det, dtype=torch.float64, batch=32)
    ref32, res32 = orc.predecoder_batched(g, cfg, sp, det, dtype=torch.float32, batch=32)
    ok = orc.deep_parity(g, det, ref32, res32, ref64, res64, ref32)
    assert ok["pass"], ok
    # a residual bit flipped at a check far from every band logit
    rep = orc.deep_parity(g, det, ref32, res32, ref64, res64, ref32)
    band = orc.band_mask(ref64, max(2e-2, rep["logit_max_rel_err"]))
    touched = np.zeros(res64.shape, bool)
    for j in range(2):
        for k in range(2):
            c = g.xor_nbr[:, j, k]
            okc = c >= 0
            bi, ni = np.nonzero(band[:, okc, j])
            touched[bi, c[okc][ni]] = True
    b, c = np.argwhere(~touched)[0]
    bad = res32.copy()
    bad[b, c] ^= 1
    r = orc.deep_parity(g, det, ref32, bad, ref64, res64, ref32)
    assert not r["pass"] and r["residual_mismatch_outside_band"] == 1 and not r["residual_is_own_xor"]
    # logits 5 % off everywhere
    r = orc.deep_parity(g, det, ref32 * 1.05, res32, ref64, res64, ref32)
    assert not r["pass"]


def test_route_rule_on_a_hand_made_batch():
    """The routing rule: a shot goes to the fallback decoder when its least confident logit is inside tau or its
    residual is not empty; the hand-off keeps ascending shot order and the shots' residual rows."""
    lg = np.ones((4, 3, 2), np.float32)
    lg[1, 2, 1] = -0.01                     # shot 1: one unsure logit
    rs = np.zeros((4, 5), np.uint8)
    rs[3, 4] = 1                            # shot 3: a detector left over
    routed, index, handoff, conf, weight = orc.route(lg, rs, 0.05, True)
    assert routed.tolist() == [False, True, False, True] and index.tolist() == [1, 3]
    assert np.array_equal(handoff, rs[[1, 3]]) and weight.tolist() == [0, 0, 0, 1]
    assert np.isclose(conf[1], 0.01) and conf[0] == 1.0
    assert orc.route(lg, rs, 0.05, False)[1].tolist() == [1]
    assert orc.route(lg, rs, 0.0, False)[1].tolist() == []
