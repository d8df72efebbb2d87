"""gather_mm on the GPU through the C ABI against the reference's outputs (golden fixtures) and the CPU oracle.

Tolerances: bf16 outputs within 1e-2 of the fp32 reference (relative to max(|ref|, rms(ref))): the output rounding
to bf16 is 2^-9 relative and the accumulation is fp32; fp32 within 1e-4."""
import os

import numpy as np
import pytest
import torch

from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.modules import BipartiteConv
from codecoder_b200.ops import gather_mm, gmm
from oracle import predecoder_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return orc.logit_error(a, b)


@pytest.fixture(scope="module")
def bb72(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "bb72_c14_conv.npz")))


def test_gmm_bb72_c14_trained_weights(bb72):
    x = torch.as_tensor(bf16_to_f32(bb72["x_bf16"])).to(DEV, torch.bfloat16)
    w = torch.as_tensor(bf16_to_f32(bb72["w_c2d_0_bf16"])).to(DEV, torch.bfloat16)
    idx = torch.as_tensor(bb72["c2d0"]).to(DEV)
    y = gmm(x, idx, w)
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu().numpy(), bb72["y_c2d0"]) < 1e-2


def test_bipartite_conv_module_bb72_c14(bb72):
    class Geo:
        pass
    g = Geo()
    g.c2d = [bb72["c2d0"].astype(np.int64), bb72["c2d1"].astype(np.int64)]
    g.d2c = [bb72["d2c0"].astype(np.int64), bb72["d2c1"].astype(np.int64)]
    g.inv_c2d = [bb72["inv_c2d0"].astype(np.int64), bb72["inv_c2d1"].astype(np.int64)]
    g.inv_d2c = [bb72["inv_d2c0"].astype(np.int64), bb72["inv_d2c1"].astype(np.int64)]
    conv = BipartiteConv(int(bb72["C"]), g).to(DEV)
    with torch.no_grad():
        for name, plist in (("w_c2d", conv.w_c2d), ("w_d2c", conv.w_d2c)):
            for k in range(2):
                plist[k].copy_(torch.as_tensor(bf16_to_f32(bb72[f"{name}_{k}_bf16"])))
        x = torch.as_tensor(bf16_to_f32(bb72["x_bf16"])).to(DEV)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = conv(x)
    assert y.dtype == torch.bfloat16
    assert rel_err(y.float().cpu().numpy(), bb72["y_module"]) < 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gmm_surface_fixtures(golden_dir, dtype):
    z = np.load(os.path.join(golden_dir, "surface_gmm.npz"))
    keys = sorted({k.rsplit("_", 1)[0] for k in z.files})
    for key in keys:
        x = torch.as_tensor(bf16_to_f32(z[key + "_x"])).to(DEV, dtype)
        w = torch.as_tensor(bf16_to_f32(z[key + "_w"])).to(DEV, dtype)
        idx = torch.as_tensor(z[key + "_idx"]).to(DEV)
        y = gmm(x, idx, w).float().cpu().numpy()
        tol = 1e-2 if dtype == torch.bfloat16 else 1e-4
        assert rel_err(y, z[key + "_y"]) < tol, key


@pytest.mark.parametrize("B", [1, 127, 128, 129, 300])
@pytest.mark.parametrize("C", [64, 128])
def test_gmm_ragged_batches(B, C):
    g = RotatedSurface(5, 5)
    rng = np.random.default_rng(B * 1000 + C)
    x = torch.as_tensor(rng.standard_normal((B, g.N_c, C)).astype(np.float32)).to(torch.bfloat16)
    w = torch.as_tensor((rng.standard_normal((C, 8 * C)) / np.sqrt(8 * C)).astype(np.float32)).to(torch.bfloat16)
    ref = orc.gather_mm(x.float(), w.float(), g.c2d[0]).numpy()
    y = gmm(x.to(DEV), torch.as_tensor(g.c2d[0]).to(DEV), w.to(DEV)).float().cpu().numpy()
    assert rel_err(y, ref) < 1e-2


@pytest.mark.parametrize("Ci,Co", [(64, 96), (96, 64), (96, 96), (128, 96), (96, 128), (64, 128)])
def test_gmm_rectangular_channels(Ci, Co):
    """C_in and C_out in {64, 96, 128} in any pair (the wide-tile kernel: M = 128 output channels, rows past C_out
    unused; a 96-channel input is one full and one half 64-channel block), over two 256-shot tiles, the second
    partial."""
    g = RotatedSurface(5, 5)
    B = 300
    rng = np.random.default_rng(Ci * 1000 + Co)
    x = torch.as_tensor(rng.standard_normal((B, g.N_d, Ci)).astype(np.float32)).to(torch.bfloat16)
    w = torch.as_tensor((rng.standard_normal((Co, 8 * Ci)) / np.sqrt(8 * Ci)).astype(np.float32)).to(torch.bfloat16)
    idx = g.d2c[0]
    ref = orc.gather_mm(x.float(), w.float(), idx).numpy()
    y = gmm(x.to(DEV), torch.as_tensor(idx).to(DEV), w.to(DEV)).float().cpu().numpy()
    assert y.shape == (B, idx.shape[0], Co)
    assert rel_err(y, ref) < 1e-2


def test_dgrad_accumulate_adds_the_second_type():
    """bpc_gather_mm_dgrad_ex with accumulate: the input gradient of a source read by X- and Z-check targets is the
    first type's gradient plus the second's, the second added in the kernel's epilogue."""
    from codecoder_b200.ops import _dgrad_into, target_table
    g = RotatedSurface(5, 5)
    B, C, K = 200, 96, 8
    rng = np.random.default_rng(7)
    gx = torch.empty(B, g.N_d, C, dtype=torch.bfloat16, device=DEV)
    ref = np.zeros((B, g.N_d, C))
    for t in range(2):
        NT = g.d2c[t].shape[0]
        gy = torch.as_tensor(rng.standard_normal((B, NT, C)).astype(np.float32)).to(torch.bfloat16)
        w = torch.as_tensor((rng.standard_normal((C, K * C)) / np.sqrt(K * C)).astype(np.float32)).to(torch.bfloat16)
        tgt = target_table(torch.as_tensor(g.inverse(g.d2c[t], g.N_d)), NT, K)
        _dgrad_into(gy.to(DEV), tgt.to(DEV), w.to(DEV), gx, accumulate=t > 0)
        ref += orc.gather_mm_dgrad(gy.float().numpy(), w.float().numpy(), tgt.numpy(), C)
    assert rel_err(gx.float().cpu().numpy(), ref) < 2e-2


def test_gmm_pad_rows_and_negative_indices_read_zeros():
    NS, NT, K, C, B = 50, 40, 8, 128, 130
    rng = np.random.default_rng(5)
    idx = rng.integers(0, NS, (NT, K)).astype(np.int32)
    idx[3, :] = NS                      # a target whose every relation is a pad
    idx[7, 2] = -1                      # out-of-range reads zeros too
    idx[9, :4] = NS
    x = torch.as_tensor(rng.standard_normal((B, NS, C)).astype(np.float32)).to(torch.bfloat16)
    w = torch.as_tensor((rng.standard_normal((C, K * C)) / 30).astype(np.float32)).to(torch.bfloat16)
    safe = np.where((idx < 0) | (idx >= NS), NS, idx)
    ref = orc.gather_mm(x.float(), w.float(), safe).numpy()
    y = gmm(x.to(DEV), torch.as_tensor(idx).to(DEV), w.to(DEV)).float().cpu().numpy()
    assert np.all(y[:, 3] == 0)
    assert rel_err(y, ref) < 1e-2


def test_gmm_deterministic():
    g = RotatedSurface(9, 9)
    rng = np.random.default_rng(9)
    x = torch.as_tensor(rng.standard_normal((256, g.N_c, 128)).astype(np.float32)).to(DEV, torch.bfloat16)
    w = torch.as_tensor((rng.standard_normal((128, 1024)) / 32).astype(np.float32)).to(DEV, torch.bfloat16)
    idx = torch.as_tensor(g.c2d[0]).to(DEV)
    a = gmm(x, idx, w)
    b = gmm(x, idx, w)
    assert torch.equal(a, b)


def test_gather_mm_dropin_signature():
    g = RotatedSurface(3, 3)
    rng = np.random.default_rng(11)
    x = torch.as_tensor(rng.standard_normal((4, g.N_c, 64)).astype(np.float32)).to(DEV)
    w = torch.as_tensor((rng.standard_normal((64, 512)) / 20).astype(np.float32)).to(DEV)
    idx = torch.as_tensor(g.c2d[0]).to(DEV)
    inv = torch.as_tensor(g.inv_c2d[0]).to(DEV)
    y32 = gather_mm(x, w, idx, inv)                      # fp32, CUDA cores
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y16 = gather_mm(x, w, idx, inv)                  # cast to bf16, tensor cores
    ref = orc.gather_mm(x.cpu(), w.cpu(), g.c2d[0]).numpy()
    assert y32.dtype == torch.float32 and rel_err(y32.cpu().numpy(), ref) < 1e-4
    assert y16.dtype == torch.bfloat16 and rel_err(y16.float().cpu().numpy(), ref) < 2e-2
    assert torch.ops.cascade.gmm(x, idx.to(torch.int32), w, False).shape == (4, g.N_d, 64)


@pytest.mark.parametrize("B", [0, 1])
def test_gather_mm_empty_and_single_shot_batches(B):
    """gather_mm forward and backward on the tensor-core path (bf16 autocast, C = 64) for an empty batch and a single
    shot: an empty batch gives empty outputs and input gradient and a zero weight gradient; one shot matches the
    oracle's forward and its autograd gradients (bf16 tolerances as the other op tests)."""
    g = RotatedSurface(5, 5)
    rng = np.random.default_rng(12 + B)
    x0 = rng.standard_normal((B, g.N_c, 64)).astype(np.float32)
    w0 = (rng.standard_normal((64, 8 * 64)) / 20).astype(np.float32)
    idx = torch.as_tensor(g.c2d[0]).to(DEV)
    inv = torch.as_tensor(g.inv_c2d[0]).to(DEV)
    x = torch.as_tensor(x0).to(DEV).requires_grad_()
    w = torch.as_tensor(w0).to(DEV).requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = gather_mm(x, w, idx, inv)
    gy = torch.as_tensor(rng.standard_normal((B, g.N_d, 64)).astype(np.float32)).to(DEV)
    (y.float() * gy).sum().backward()
    torch.cuda.synchronize()
    assert y.shape == (B, g.N_d, 64) and x.grad.shape == x.shape and w.grad.shape == w.shape
    if B == 0:
        assert torch.count_nonzero(w.grad) == 0
        return
    xr = torch.as_tensor(x0).requires_grad_()
    wr = torch.as_tensor(w0).requires_grad_()
    yr = orc.gather_mm(xr, wr, g.c2d[0])
    (yr * gy.cpu()).sum().backward()
    assert rel_err(y.detach().float().cpu().numpy(), yr.detach().numpy()) < 2e-2
    assert rel_err(x.grad.cpu().numpy(), xr.grad.numpy()) < 5e-2
    assert rel_err(w.grad.cpu().numpy(), wr.grad.numpy()) < 5e-2


@pytest.mark.parametrize("C,B", [(128, 300), (64, 257), (96, 130)])
def test_affine_silu_epilogue_two_weight_sets(C, B):
    """The op with two weight sets and the affine + SiLU epilogue (the Cascade block's data -> check convolution with
    its BN3 + SiLU, bpc_gather_mm_fwd_ex): y = SiLU(scale * op(x) + shift), checked against an fp32 restatement on
    the rotated-surface d = 9 graph; ragged batches (partial shot tiles).  Tolerance 2e-2 of max |ref|:
    the bf16 output rounding plus the hardware-tanh SiLU."""
    from codecoder_b200.ops import gmm_ex
    g = RotatedSurface(9, 9)
    gen = torch.Generator(device=DEV).manual_seed(C + B)
    x = torch.randn(B, g.N_d, C, device=DEV, generator=gen).bfloat16()
    w = (torch.randn(2, C, g.K * C, device=DEV, generator=gen) / (g.K * C) ** 0.5).bfloat16()
    scale = 0.5 + torch.rand(C, device=DEV, generator=gen)
    shift = 0.2 * torch.randn(C, device=DEV, generator=gen)
    idx = torch.as_tensor(g.d2c_all, dtype=torch.int32, device=DEV)
    split = g.T * g.nh
    y = gmm_ex(x, idx, w, type_split=split, scale=scale, shift=shift)
    torch.cuda.synchronize()
    xp = torch.cat([x.float(), torch.zeros(B, 1, C, device=DEV)], 1)
    gat = xp[:, idx.long()].reshape(B, idx.shape[0], g.K * C)
    ref = torch.cat([gat[:, :split] @ w[0].float().t(), gat[:, split:] @ w[1].float().t()], 1)
    ref = torch.nn.functional.silu(ref * scale + shift)
    assert rel_err(y.float().cpu().numpy(), ref.cpu().numpy()) < 2e-2
