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
import math
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


def boundary_case(rows, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    x3 = r(rows, 128).bfloat16()
    w_up = (r(512, 128) / 11.3).bfloat16()
    w_down = (r(128, 512) / 22.6).bfloat16()
    h = r(rows, 512)
    a1, b1 = 0.5 + r(512).abs(), 0.1 * r(512)
    a2, b2 = 0.5 + r(128).abs(), 0.1 * r(128)
    return x3, w_up, w_down, h, a1, b1, a2, b2


@pytest.mark.parametrize("rows", [1512, 4096 * 3 + 77])
def test_cascade_boundary_matches_the_unfused_launches(rows):
    """bpc_cascade_boundary against the launches it replaces: the bf16 up GEMM (cuBLAS), the residual + BN1 + SiLU
    pass and the op's down projection with the BN2 + SiLU epilogue.  The same operations in the same order: h' and x2
    equal bit for bit wherever the two up GEMMs round u alike (all elements in practice; the bar allows one bf16 step
    of u in h' and the resulting step in x2).  Ragged row counts (partial last tile), in-place h, and the last-block
    mode that writes x1 instead of running the down projection."""
    from codecoder_b200.ops import cascade_boundary, gmm_ex, residual_affine_silu
    x3, w_up, w_down, h, a1, b1, a2, b2 = boundary_case(rows, rows)
    sh, su = 1 / math.sqrt(28), 1.0
    u = torch.matmul(x3, w_up.t())
    h_ref, x1_ref = residual_affine_silu(h, u, sh, su, a1, b1)
    ident = torch.zeros(1, 1, dtype=torch.int32, device="cuda")
    x2_ref = gmm_ex(x1_ref.view(rows, 1, 512), ident, w_down, scale=a2, shift=b2).view(rows, 128)
    h_new, x2 = cascade_boundary(x3, w_up, h, sh, su, a1, b1, w_down, a2, b2)
    torch.cuda.synchronize()
    dh = (h_new - h_ref).abs()
    assert bool((dh <= su * u.float().abs() * 2 ** -7 + 1e-6).all())
    exact_h = float((dh == 0).float().mean())
    dx = (x2.float() - x2_ref.float()).abs()
    exact_x = float((dx == 0).float().mean())
    print("boundary rows=%d: h' exact %.6f, x2 exact %.6f" % (rows, exact_h, exact_x))
    assert exact_h > 0.999 and exact_x > 0.99
    assert rel(x2, x2_ref) < 2e-2
    # in place, and the last-block mode (x1 out, no down projection)
    h2 = h.clone()
    out, x1 = cascade_boundary(x3, w_up, h2, sh, su, a1, b1, h_out=h2)
    torch.cuda.synchronize()
    assert out.data_ptr() == h2.data_ptr()
    assert torch.equal(h2, h_new)
    assert x1.shape == (rows, 512) and float(((x1.float() - x1_ref.float()).abs() > 0).float().mean()) < 1e-3
    # h' only
    out, none = cascade_boundary(x3, w_up, h, sh, su, want_y=False)
    torch.cuda.synchronize()
    assert none is None and torch.equal(out, h_new)


def test_cascade_stack_of_one_block_matches_reference_c14(c14):
    """The stack path (one launch per block boundary) on the reference Block's C14 block-0 fixture: the same bar as
    the block-by-block path."""
    conv_z, z = c14
    blk = CascadeBlock(int(z["H"]), bb72_geo(conv_z), int(z["L"]), res=str(z["res"]))
    load_block(blk, conv_z, z)
    stack = CascadeStack([blk]).cuda().eval()
    h = torch.as_tensor(bf16_to_f32(z["h_bf16"])).cuda()
    h_in = h.clone()
    with torch.no_grad():
        out = stack(h)
    torch.cuda.synchronize()
    assert torch.equal(h, h_in)                     # the caller's stream is not written
    err = rel(out, z["out"])
    print("C14 block-0 through the boundary kernel vs the reference Block: rel err %.2e" % err)
    assert err < 2e-2
    with torch.no_grad():
        assert rel(out, blk(h)) < 1e-5


def test_cascade_net_c14_width_matches_reference(golden_dir, c14):
    """The whole network at C14's width (H = 512, 128-channel bottleneck, 2 blocks) through the block-boundary
    kernel and the wide-tile convolutions, against the reference's own CascadeBB (fp32 CPU) with the same seeded
    weights (tests/cascade_weights.py rebuilds them).  Bars: 2e-2 of max |ref| and 5e-2 of the largest shot-to-shot
    deviation, and each at most twice the same statistic of the reference's own bf16 autocast run."""
    from cascade_weights import cascade_state
    conv_z, _ = c14
    z = dict(np.load(os.path.join(golden_dir, "cascade_net_bb72_h512.npz")))
    geo = bb72_geo(conv_z)
    geo.T, geo.n2, geo.N = int(z["T"]), int(z["n2"]), int(z["N"])
    net = CascadeNet(geo, int(z["H"]), int(z["L"]), z["det_t"], z["det_typ"], z["det_site"], z["logicals"],
                     res=str(z["res"]))
    state = cascade_state({k: tuple(v.shape) for k, v in net.state_dict().items()}, int(z["seed"]))
    net.load_state_dict({k: torch.as_tensor(v) for k, v in state.items()})
    net = net.cuda().eval()
    with torch.no_grad():
        out = net(torch.as_tensor(z["det"]).cuda())
    torch.cuda.synchronize()
    ref, ra = z["logits"], z["logits_autocast"]
    err, dev = rel(out, ref), rel(out - out.mean(0), ref - ref.mean(0))
    err_ref, dev_ref = rel(ra, ref), rel(ra - ra.mean(0), ref - ref.mean(0))
    print("CascadeNet (H=512, L=2, bb72) vs the reference: rel err %.2e, of the shot deviations %.2e "
          "(the reference's own bf16 run: %.2e, %.2e)" % (err, dev, err_ref, dev_ref))
    assert err < 2e-2 and dev < 5e-2
    assert err <= 2 * err_ref and dev <= 2 * dev_ref


def test_token_stem_and_boundary_match_the_embedded_stream():
    """bpc_cascade_stem and bpc_cascade_boundary_tokens read the embedding table by detector token instead of an
    embedded stream: both give the same bits as the residual pass and the boundary kernel on the materialised
    stream h0 = E[token] (tokens as CascadeBB.tokens: 2 type + bit at a detector's node, 4 elsewhere)."""
    from codecoder_b200.ops import cascade_boundary, cascade_boundary_tokens, cascade_stem, residual_affine_silu
    B, D, N = 5, 360, 504
    cpu = torch.Generator().manual_seed(77)
    nodes = torch.randperm(N, generator=cpu)[:D]
    gidx = torch.full((N,), D, dtype=torch.int32)
    gidx[nodes] = torch.arange(D, dtype=torch.int32)
    tbase = torch.full((N,), 4, dtype=torch.int32)
    tbase[nodes] = 2 * torch.randint(0, 2, (D,), generator=cpu, dtype=torch.int32)
    det = (torch.rand(B, D, generator=cpu) < 0.3).to(torch.uint8)
    E = torch.randn(5, 512, generator=cpu)
    det, gidx, tbase, E = det.cuda(), gidx.cuda(), tbase.cuda(), E.cuda()
    tok = tbase.long() + F.pad(det, (0, 1))[:, gidx.long()].long()
    h0 = E[tok].contiguous()
    x3, w_up, w_down, _, a1, b1, a2, b2 = boundary_case(B * N, 9)
    x3 = x3.view(B, N, 128)
    sh, su = 1 / math.sqrt(28), 1.0
    x1 = cascade_stem(det, gidx, tbase, E, a1, b1)
    _, x1_ref = residual_affine_silu(h0, None, 1.0, 0.0, a1, b1, want_out=False)
    h_t, x2_t = cascade_boundary_tokens(x3, w_up, det, gidx, tbase, E, sh, su, a1, b1, w_down, a2, b2)
    h_r, x2_r = cascade_boundary(x3, w_up, h0, sh, su, a1, b1, w_down, a2, b2)
    _, xl_t = cascade_boundary_tokens(x3, w_up, det, gidx, tbase, E, sh, su, a1, b1, want_h=False)
    _, xl_r = cascade_boundary(x3, w_up, h0, sh, su, a1, b1, h_out=None)
    torch.cuda.synchronize()
    assert torch.equal(x1, x1_ref)
    assert torch.equal(h_t, h_r) and torch.equal(x2_t, x2_r)
    assert torch.equal(xl_t, xl_r)


def test_cascade_net_single_shot_and_empty_batch(golden_dir, c14):
    """The C14-width network on one shot (504 node rows: a partial last tile in every kernel) gives that shot's logits
    of a larger batch, and an empty batch gives an empty result."""
    from cascade_weights import cascade_state
    conv_z, _ = c14
    z = dict(np.load(os.path.join(golden_dir, "cascade_net_bb72_h512.npz")))
    geo = bb72_geo(conv_z)
    geo.T, geo.n2, geo.N = int(z["T"]), int(z["n2"]), int(z["N"])
    net = CascadeNet(geo, int(z["H"]), int(z["L"]), z["det_t"], z["det_typ"], z["det_site"], z["logicals"],
                     res=str(z["res"]))
    state = cascade_state({k: tuple(v.shape) for k, v in net.state_dict().items()}, int(z["seed"]))
    net.load_state_dict({k: torch.as_tensor(v) for k, v in state.items()})
    net = net.cuda().eval()
    det = torch.as_tensor(z["det"]).cuda()
    with torch.no_grad():
        many = net(det)
        one = net(det[5:6])
        none = net(det[:0])
    torch.cuda.synchronize()
    assert one.shape == (1, many.shape[1]) and none.shape == (0, many.shape[1])
    assert rel(one[0], many[5]) < 1e-5
