"""The reference's bottleneck Block (cascade_net.py:236-259) on the B200 op: the fused inference path against the
reference's own Block with the trained C14 block-0 weights (golden fixture), training mode (batch statistics,
backward through the op) against an fp64 composition, and the time of a 14-block C14 stack.  The whole network
(CascadeBB, cascade_net.py:262-343, as CascadeNet): eval logits against the reference's on seeded shots, and a
training-mode step under bf16 autocast.

Tolerances: relative to max |ref|; 2e-2 for the bf16 inference path (four bf16 roundings of bottleneck activations
around an fp32 residual), 1e-4 for training mode in fp32.  The whole network's logits: 2e-2 of max |ref|, and 5e-2
of the largest shot-to-shot deviation for the logits less their mean over shots (the bf16 read-out GEMMs add their
roundings to the blocks'), and neither above the same statistic of the reference's own bf16 autocast run against
its fp32 run."""
import os
import time
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.modules import CascadeBlock, CascadeNet, CascadeStack
from oracle import predecoder_oracle as orc

pytestmark = pytest.mark.gpu


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32)


def rel(a, b):
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else a
    b = b.detach().double().cpu().numpy() if torch.is_tensor(b) else b
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def bb72_geo(z):
    return SimpleNamespace(c2d=[z["c2d0"], z["c2d1"]], d2c=[z["d2c0"], z["d2c1"]],
                           inv_c2d=[z["inv_c2d0"].astype(np.int64), z["inv_c2d1"].astype(np.int64)],
                           inv_d2c=[z["inv_d2c0"].astype(np.int64), z["inv_d2c1"].astype(np.int64)])


@pytest.fixture(scope="module")
def c14(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "bb72_c14_conv.npz"))), \
        dict(np.load(os.path.join(golden_dir, "cascade_block_c14.npz")))


def load_block(blk, conv_z, z):
    with torch.no_grad():
        for i in (1, 2, 3):
            bn = getattr(blk, f"bn{i}")
            bn.weight.copy_(torch.as_tensor(z[f"bn{i}_weight"]))
            bn.bias.copy_(torch.as_tensor(z[f"bn{i}_bias"]))
            bn.running_mean.copy_(torch.as_tensor(z[f"bn{i}_mean"]))
            bn.running_var.copy_(torch.as_tensor(z[f"bn{i}_var"]))
        blk.down.weight.copy_(torch.as_tensor(bf16_to_f32(z["down_bf16"])))
        blk.up.weight.copy_(torch.as_tensor(bf16_to_f32(z["up_bf16"])))
        for k in range(2):
            blk.conv.w_c2d[k].copy_(torch.as_tensor(bf16_to_f32(conv_z[f"w_c2d_{k}_bf16"])))
            blk.conv.w_d2c[k].copy_(torch.as_tensor(bf16_to_f32(conv_z[f"w_d2c_{k}_bf16"])))


def test_cascade_block_inference_matches_reference_c14(c14):
    conv_z, z = c14
    blk = CascadeBlock(int(z["H"]), bb72_geo(conv_z), int(z["L"]), res=str(z["res"]))
    load_block(blk, conv_z, z)
    blk = blk.cuda().eval()
    h = torch.as_tensor(bf16_to_f32(z["h_bf16"])).cuda()
    with torch.no_grad():
        out = blk(h)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == h.shape
    err = rel(out, z["out"])
    print("C14 block-0 inference vs the reference Block: rel err %.2e" % err)
    assert err < 2e-2


def test_cascade_block_training_mode_matches_fp64():
    g = RotatedSurface(5, 5)
    torch.manual_seed(7)
    blk = CascadeBlock(256, g, 4, res="branch").cuda().train()
    h = torch.randn(3, g.N_c, 256, device="cuda", requires_grad=True)
    out = blk(h)
    gy = torch.randn_like(out)
    out.backward(gy)
    # fp64 restatement with batch statistics over every node of every shot
    p = {n: t.detach().double().cpu().requires_grad_() for n, t in blk.named_parameters()}
    hr = h.detach().double().cpu().requires_grad_()

    def bn(x, i):
        C = x.shape[-1]
        m = getattr(blk, f"bn{i}")
        return F.batch_norm(x.reshape(-1, C), None, None, p[f"bn{i}.weight"], p[f"bn{i}.bias"], True, 0.0,
                            m.eps).view(x.shape)

    u = F.silu(bn(hr, 1)) @ p["down.weight"].t()
    u = orc.bipartite_conv(F.silu(bn(u, 2)), [p["conv.w_c2d.0"]], [p["conv.w_d2c.0"], p["conv.w_d2c.1"]], g.c2d, g.d2c)
    ref = hr + blk.scale * (F.silu(bn(u, 3)) @ p["up.weight"].t())
    ref.backward(gy.double().cpu())
    assert rel(out, ref) < 1e-4
    assert rel(h.grad, hr.grad) < 1e-4
    for n, t in blk.named_parameters():
        assert rel(t.grad, p[n].grad) < 1e-4, n


def test_cascade_c14_stack_time(c14):
    """14 C14-shaped blocks (H = 512, bb72) in eval mode: device time per shot at a batch of 512 shots."""
    conv_z, z = c14
    geo = bb72_geo(conv_z)
    torch.manual_seed(3)
    blocks = CascadeStack([CascadeBlock(512, geo, 14, res="skip") for _ in range(14)]).cuda().eval()
    for b in blocks.blocks:
        for i in (1, 2, 3):
            getattr(b, f"bn{i}").running_var.uniform_(0.5, 2.0)
    h = torch.randn(512, int(conv_z["N"]), 512, device="cuda")
    with torch.no_grad():
        for _ in range(3):
            blocks(h)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for _ in range(5):
            out = blocks(h)
        e.record()
        e.synchronize()
    us = s.elapsed_time(e) * 1000 / 5 / h.shape[0]
    assert torch.isfinite(out).all()
    # the stack's fused hand-over gives what the blocks give one by one
    with torch.no_grad():
        one = h[:4]
        for b in blocks.blocks:
            one = b(one)
        assert rel(blocks(h[:4]), one) < 1e-5
    print("C14 block stack (14 blocks, bb72, H=512): %.2f us/shot at 512 shots" % us)


@pytest.fixture(scope="module")
def cascade_net_z(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "cascade_net_bb72.npz")))


def make_cascade_net(z, conv_z):
    geo = bb72_geo(conv_z)
    geo.T, geo.n2, geo.N = int(z["T"]), int(z["n2"]), int(z["N"])
    net = CascadeNet(geo, int(z["H"]), int(z["L"]), z["det_t"], z["det_typ"], z["det_site"], z["logicals"],
                     res=str(z["res"]))
    net.load_state_dict({k[3:]: torch.as_tensor(v) for k, v in z.items() if k.startswith("sd.")})
    return net.cuda()


def test_cascade_net_inference_matches_reference_bb72(c14, cascade_net_z):
    conv_z, _ = c14
    z = cascade_net_z
    net = make_cascade_net(z, conv_z).eval()
    with torch.no_grad():
        out = net(torch.as_tensor(z["det"]).cuda())
    torch.cuda.synchronize()
    ref = z["logits"]
    assert out.shape == ref.shape and out.dtype == torch.float32
    err = rel(out, ref)
    dev = rel(out - out.mean(0), ref - ref.mean(0))
    # the reference's own bf16 autocast run, against its fp32 run: the same two statistics
    ra = z["logits_autocast"]
    err_ref, dev_ref = rel(ra, ref), rel(ra - ra.mean(0), ref - ref.mean(0))
    print("CascadeNet (H=128, L=2, bb72) vs the reference: rel err %.2e, of the shot deviations %.2e "
          "(the reference's own bf16 run: %.2e, %.2e)" % (err, dev, err_ref, dev_ref))
    assert err < 2e-2 and dev < 5e-2
    assert err <= err_ref and dev <= dev_ref


def test_cascade_net_training_step_under_autocast(c14, cascade_net_z):
    conv_z, _ = c14
    z = cascade_net_z
    net = make_cascade_net(z, conv_z).train()
    det = torch.as_tensor(z["det"]).cuda()
    target = torch.randint(0, 2, (det.shape[0], int(net.k)), device="cuda").float()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = net(det)
        loss = F.binary_cross_entropy_with_logits(logits.float(), target)
    loss.backward()
    assert torch.isfinite(loss)
    for n, p in net.named_parameters():
        assert p.grad is not None and bool(torch.isfinite(p.grad).all()), n
    assert float(net.scatter.grad.abs().max()) > 0 and float(net.blocks[0].conv.w_c2d[0].grad.abs().max()) > 0
