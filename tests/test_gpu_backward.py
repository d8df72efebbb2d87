"""Backward of the gather_mm op on the GPU (input gradient through the target table, weight gradient) against the
reference's own backward (golden fixtures) and the CPU oracle.

Tolerances: relative to max |ref|, 1e-5 for fp32 inputs on the CUDA cores, 2e-2 for bf16 outputs (input gradient)
and 2e-3 for the fp32 weight gradient of bf16 inputs (fp32 accumulation of exact bf16 products)."""
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from codecoder_b200 import ops
from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.modules import BipartiteConv
from oracle import predecoder_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32)


def rel(a, b):
    a = a.detach().float().cpu().numpy() if torch.is_tensor(a) else a
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.fixture(scope="module")
def bwd(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "gather_mm_bwd.npz")))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_backward_ops_golden(bwd, dtype):
    names = sorted({k.rsplit("_", 1)[0] for k in bwd if not k.startswith("bb72")})
    for nm in names:
        x = torch.as_tensor(bf16_to_f32(bwd[nm + "_x"])).to(DEV, dtype)
        w = torch.as_tensor(bf16_to_f32(bwd[nm + "_w"])).to(DEV, dtype)
        gy = torch.as_tensor(bf16_to_f32(bwd[nm + "_gy"])).to(DEV, dtype)
        idx = torch.as_tensor(bwd[nm + "_idx"]).to(DEV)
        inv = torch.as_tensor(bwd[nm + "_inv"]).to(DEV)
        NT, K = idx.shape
        gx = ops.gmm(gy, ops.target_table(inv, NT, K), w, True)
        gw = ops.gmm_wgrad(x, gy, idx)
        tx, tw = (2e-2, 2e-3) if dtype == torch.bfloat16 else (1e-5, 1e-5)
        assert gx.dtype == dtype and gw.dtype == torch.float32
        assert rel(gx, bwd[nm + "_gx"]) < tx, (nm, rel(gx, bwd[nm + "_gx"]))
        assert rel(gw, bwd[nm + "_gw"]) < tw, (nm, rel(gw, bwd[nm + "_gw"]))
    assert ops.op_status() == 0


def _bb72_geo(z):
    return SimpleNamespace(c2d=[z["c2d0"], z["c2d1"]], d2c=[z["d2c0"], z["d2c1"]],
                           inv_c2d=[z["inv_c2d0"].astype(np.int64), z["inv_c2d1"].astype(np.int64)],
                           inv_d2c=[z["inv_d2c0"].astype(np.int64), z["inv_d2c1"].astype(np.int64)])


@pytest.mark.parametrize("autocast", [True, False])
def test_bipartite_conv_backward_bb72_c14(golden_dir, bwd, autocast):
    z = dict(np.load(os.path.join(golden_dir, "bb72_c14_conv.npz")))
    conv = BipartiteConv(int(z["C"]), _bb72_geo(z)).to(DEV)
    with torch.no_grad():
        for k in range(2):
            conv.w_c2d[k].copy_(torch.as_tensor(bf16_to_f32(z[f"w_c2d_{k}_bf16"])))
            conv.w_d2c[k].copy_(torch.as_tensor(bf16_to_f32(z[f"w_d2c_{k}_bf16"])))
    x = torch.as_tensor(bf16_to_f32(bwd["bb72_x"])).to(DEV).requires_grad_()
    gy = torch.as_tensor(bf16_to_f32(bwd["bb72_gy"])).to(DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        y = conv(x)
    y.backward(gy.to(y.dtype))
    # bf16: the intermediate data features are stored in bf16, so the gradients carry two bf16 roundings
    tol = 3e-2 if autocast else 1e-4
    assert rel(x.grad, bwd["bb72_gx"]) < tol
    assert rel(conv.w_c2d[0].grad, bwd["bb72_gw_c2d0"]) < tol
    assert rel(conv.w_d2c[1].grad, bwd["bb72_gw_d2c1"]) < tol


@pytest.mark.parametrize("d,C,B,step", [(13, 128, 300, "c2d"), (11, 96, 200, "d2c"), (9, 64, 129, "c2d"),
                                        (13, 128, 1, "d2c")])
def test_backward_vs_oracle_surface(d, C, B, step):
    g = RotatedSurface(d, d)
    idx, ns = (g.c2d[0], g.N_c) if step == "c2d" else (g.d2c_all, g.N_d)
    inv = g.inverse(idx, ns)
    rng = np.random.default_rng(d * 1000 + C + B)
    x = torch.as_tensor(rng.standard_normal((B, ns, C)), dtype=torch.float32).to(torch.bfloat16)
    w = torch.as_tensor(rng.standard_normal((C, g.K * C)) / np.sqrt(g.K * C), dtype=torch.float32).to(torch.bfloat16)
    gy = torch.as_tensor(rng.standard_normal((B, idx.shape[0], C)), dtype=torch.float32).to(torch.bfloat16)
    NT, K = idx.shape
    gx = ops.gmm(gy.to(DEV), ops.target_table(torch.as_tensor(inv).to(DEV), NT, K), w.to(DEV), True)
    gw = ops.gmm_wgrad(x.to(DEV), gy.to(DEV), torch.as_tensor(idx).to(DEV))
    tgt = orc.target_table(inv, NT, K)
    ref_gx = orc.gather_mm_dgrad(gy.float().numpy(), w.float().numpy(), tgt, C)
    ref_gw = orc.gather_mm_wgrad(x.float().numpy(), gy.float().numpy(), idx)
    assert rel(gx, ref_gx) < 2e-2
    assert rel(gw, ref_gw) < 2e-3
    assert ops.op_status() == 0


def test_wgrad_deterministic_and_pads():
    g = RotatedSurface(11, 11)
    idx = torch.as_tensor(g.d2c_all).to(DEV)
    B, C = 777, 96
    torch.manual_seed(5)
    x = torch.randn(B, g.N_d, C, device=DEV).to(torch.bfloat16)
    gy = torch.randn(B, g.N_c, C, device=DEV).to(torch.bfloat16)
    a = ops.gmm_wgrad(x, gy, idx)
    b = ops.gmm_wgrad(x, gy, idx)
    assert torch.equal(a, b)
    # a relation that is a pad for every target has a zero gradient
    idx2 = idx.clone()
    idx2[:, 3] = g.N_d
    c = ops.gmm_wgrad(x, gy, idx2).view(C, g.K, C)
    assert torch.count_nonzero(c[:, 3]) == 0
    assert torch.equal(c[:, :3], a.view(C, g.K, C)[:, :3])


def test_autograd_matches_oracle_autograd():
    g = RotatedSurface(5, 5)
    C, B = 64, 33
    idx = torch.as_tensor(g.c2d[0])
    inv = torch.as_tensor(g.inverse(g.c2d[0], g.N_c))
    torch.manual_seed(3)
    x0 = torch.randn(B, g.N_c, C).to(torch.bfloat16).float()
    w0 = (torch.randn(C, g.K * C) / 16).to(torch.bfloat16).float()
    gy = torch.randn(B, g.N_d, C).to(torch.bfloat16).float()
    x = x0.to(DEV).requires_grad_()
    w = w0.to(DEV).requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = ops.gather_mm(x, w, idx.to(DEV), inv.to(DEV))
    y.backward(gy.to(DEV, y.dtype))
    xr = x0.double().requires_grad_()
    wr = w0.double().requires_grad_()
    orc.gather_mm(xr, wr, g.c2d[0]).backward(gy.double())
    assert x.grad.dtype == torch.float32 and w.grad.dtype == torch.float32
    assert rel(x.grad, xr.grad.numpy()) < 2e-2
    # the Function returns the weight gradient in the weight's autocast dtype, bf16, as the reference's does
    # (cascade_triton.py:185): one bf16 rounding
    assert rel(w.grad, wr.grad.numpy()) < 1e-2
