"""The training step on the GPU: PreDecoderNet on the B200 op against the same network on the CPU oracle's
gather_mm (float64 autograd), and a short training run that lowers the loss.

Tolerances: fp32 network (CUDA-core kernels) 1e-4 relative to max |ref|; bf16 autocast (tensor cores) 5e-2 on the
gradients (every stored activation and gradient is rounded to bf16 along the way)."""
from dataclasses import replace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.params import CONFIGS, init_params
from codecoder_b200.sampler import sample, sample_torch
from codecoder_b200.train import PreDecoderNet, Trainer
from oracle import predecoder_oracle as orc

pytestmark = pytest.mark.gpu


def oracle_gmm(x, w, idx, inv):
    return orc.gather_mm(x, w, idx.cpu())


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def grads(cfg, seed, B, autocast):
    g = RotatedSurface(cfg.d, cfg.rounds)
    params = init_params(cfg, seed)
    det, err = sample(g, 0.03, B, seed + 1)
    dev_net = PreDecoderNet(g, cfg, params).cuda()
    ref_net = PreDecoderNet(g, cfg, params, gmm=oracle_gmm).double()
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        z = dev_net(torch.as_tensor(det).cuda())
    F.binary_cross_entropy_with_logits(z.float(), torch.as_tensor(err).cuda().float()).backward()
    zr = ref_net(torch.as_tensor(det))
    F.binary_cross_entropy_with_logits(zr, torch.as_tensor(err).double()).backward()
    return z, zr, dict(dev_net.named_parameters()), dict(ref_net.named_parameters())


def test_train_gradients_fp32_match_oracle():
    cfg = replace(CONFIGS["d5_fp32"], d=3, rounds=3, layers=2)
    z, zr, pd, pr = grads(cfg, 31, 24, autocast=False)
    assert rel(z, zr) < 1e-4
    for k in pr:
        if pr[k].requires_grad:
            assert rel(pd[k].grad, pr[k].grad) < 1e-4, k


def test_train_gradients_bf16_match_oracle():
    cfg = replace(CONFIGS["d11_train"], d=5, rounds=5, layers=2)          # C = 96: tensor-core kernels
    z, zr, pd, pr = grads(cfg, 32, 40, autocast=True)
    assert rel(z, zr) < 3e-2
    for k in pr:
        if pr[k].requires_grad:
            assert rel(pd[k].grad, pr[k].grad) < 5e-2, (k, rel(pd[k].grad, pr[k].grad))


def test_training_lowers_the_loss():
    cfg = replace(CONFIGS["d11_train"], d=5, rounds=5, layers=3, channels=64)
    g = RotatedSurface(cfg.d, cfg.rounds)
    torch.manual_seed(0)
    tr = Trainer(PreDecoderNet(g, cfg, init_params(cfg, 41)).cuda(), lr=1e-3)
    losses = []
    for step in range(60):
        det, err = sample_torch(g, 0.01, 1024, 1000 + step, device="cuda")
        losses.append(float(tr.step(det, err)))
    assert np.isfinite(losses).all()
    assert np.mean(losses[-10:]) < 0.7 * np.mean(losses[:5]), losses


def test_graphed_training_steps_match_eager_steps():
    """Trainer(graph=True).step_graphed replays forward, backward, clipping and the Adam step from one CUDA graph:
    from the same weights and the same batches it gives the eager steps' losses and weights bit for bit (its first
    call runs two eager warm-up steps on its batch before the captured one, so the eager run does the same)."""
    cfg = replace(CONFIGS["d11_train"], d=5, rounds=5, layers=3)            # C = 96: tensor-core kernels
    g = RotatedSurface(cfg.d, cfg.rounds)
    batches = [sample_torch(g, 0.03, 384, 60 + i, device="cuda") for i in range(3)]
    eager = Trainer(PreDecoderNet(g, cfg, init_params(cfg, 59)).cuda(), lr=1e-3, graph=True)
    graphed = Trainer(PreDecoderNet(g, cfg, init_params(cfg, 59)).cuda(), lr=1e-3, graph=True)
    order = [0, 1, 2, 1, 0]
    le = [eager.step(*batches[0]) for _ in range(2)]
    le += [eager.step(*batches[i]) for i in order]
    lg = [graphed.step_graphed(*batches[i]) for i in order]
    torch.cuda.synchronize()
    assert torch.equal(torch.stack(le[2:]), torch.stack(lg))
    for pe, pg in zip(eager.model.parameters(), graphed.model.parameters()):
        assert torch.equal(pe, pg)


def test_fused_gelu_launch_matches_the_two_launch_form(monkeypatch):
    """The training network's residual steps run the op and their GELU / residual pass in one launch
    (bpc_gather_mm_fwd_gelu: the step kernel's epilogue writes the kept pre-activation and the residual stream).  It
    gives the bits of the op followed by bpc_gelu_residual_fwd in every mode (the first check -> data step without a
    residual, the bf16 data stream, the fp32 check stream with two target types), over a partial tile: the same
    loss and gradients."""
    from codecoder_b200 import ops
    cfg = replace(CONFIGS["d11_train"], d=5, rounds=5, layers=3)            # C = 96: the wide-tile kernel
    g = RotatedSurface(cfg.d, cfg.rounds)
    det, err = sample_torch(g, 0.03, 384, 71, device="cuda")
    out = []
    for fused in (True, False):
        monkeypatch.setattr(ops, "_FUSED_GELU", fused)
        net = PreDecoderNet(g, cfg, init_params(cfg, 70)).cuda()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = net(det, err)
        loss.backward()
        out.append((loss.detach(), [p.grad.clone() for p in net.parameters() if p.grad is not None]))
    torch.cuda.synchronize()
    (lf, gf), (lu, gu) = out
    assert torch.equal(lf, lu)
    assert len(gf) == len(gu) and all(torch.equal(a, b) for a, b in zip(gf, gu))


def test_fused_steps_match_the_unfused_network():
    """Under bf16 autocast PreDecoderNet runs each residual step as ops.bipartite_step (op kernels + one GELU /
    residual pass each way, both check types in one pre-activation block); the unfused torch composition of the same
    network gives the same logits and gradients up to bf16 rounding (GELU on tanh.approx vs tanhf, one rounding of
    the summed input gradient instead of two)."""
    cfg = replace(CONFIGS["d11_train"], d=5, rounds=5, layers=3)
    g = RotatedSurface(cfg.d, cfg.rounds)
    params = init_params(cfg, 51)
    det, err = sample(g, 0.03, 300, 52)
    out = []
    for fused in (True, False):
        net = PreDecoderNet(g, cfg, params, fused=fused).cuda()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            z = net(torch.as_tensor(det).cuda())
        F.binary_cross_entropy_with_logits(z.float(), torch.as_tensor(err).cuda().float()).backward()
        out.append((z, dict(net.named_parameters())))
    (zf, pf), (zu, pu) = out
    assert rel(zf, zu) < 1e-2
    for k in pu:
        if pu[k].requires_grad:
            assert rel(pf[k].grad, pu[k].grad) < 2e-2, (k, rel(pf[k].grad, pu[k].grad))


@pytest.mark.parametrize("f32", [True, False])
def test_gelu_residual_passes_match_torch(f32):
    """bpc_gelu_residual_fwd / _bwd through the C ABI against torch's composition of the same step (bf16 GELU in the
    tanh form, residual add, cast; and back): the residual gradient exactly, GELU and its gradient to bf16 rounding
    (the kernels use the hardware tanh.approx)."""
    from codecoder_b200 import _lib
    torch.manual_seed(3)
    T, B, NTt, C = 2, 40, 37, 96
    NT = T * NTt
    dev = "cuda"
    a = torch.randn(T, B, NTt, C, device=dev).to(torch.bfloat16)
    a_rows = a.permute(1, 0, 2, 3).reshape(B, NT, C)          # type-major block -> (B, NT, C)
    h = torch.randn(B, NT, C, device=dev, dtype=torch.float32 if f32 else torch.bfloat16)
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    dt = _lib.BPC_DTYPE_F32 if f32 else _lib.BPC_DTYPE_BF16
    y = torch.empty_like(h)
    y16 = torch.empty(B, NT, C, device=dev, dtype=torch.bfloat16) if f32 else None
    _lib.check(L.bpc_gelu_residual_fwd(a.data_ptr(), h.data_ptr(), y.data_ptr(), y16.data_ptr() if f32 else None,
                                       B, NT, C, T, dt, st), "fwd")
    u = F.gelu(a_rows.float(), approximate="tanh").to(torch.bfloat16)
    y_ref = h + u.float() if f32 else (h.float() + u.float()).to(torch.bfloat16)
    assert rel(y, y_ref) < 1e-2
    if f32:
        assert torch.equal(y16, y.to(torch.bfloat16))
    gy = torch.randn(B, NT, C, device=dev, dtype=torch.float32 if f32 else torch.bfloat16)
    gy16 = torch.randn(B, NT, C, device=dev).to(torch.bfloat16) if f32 else None
    gh = torch.empty(B, NT, C, device=dev, dtype=torch.float32) if f32 else None
    ga = torch.empty_like(a)
    _lib.check(L.bpc_gelu_residual_bwd(gy.data_ptr(), gy16.data_ptr() if f32 else None, a.data_ptr(),
                                       gh.data_ptr() if f32 else None, ga.data_ptr(), B, NT, C, T, dt, st), "bwd")
    g = gy + gy16.float() if f32 else gy.float()
    if f32:
        assert torch.equal(gh, g)
    x = a_rows.float().requires_grad_(True)
    F.gelu(x, approximate="tanh").backward(g.to(torch.bfloat16).float())
    ga_ref = x.grad.to(torch.bfloat16).reshape(B, T, NTt, C).permute(1, 0, 2, 3)
    assert rel(ga, ga_ref) < 2e-2


def test_embed_tokens_match_torch():
    """bpc_embed_tokens_fwd / _bwd through ops.embed_tokens against F.embedding and its autograd gradient: the
    features exactly, the weight gradient to fp32 summation order."""
    from codecoder_b200.ops import embed_tokens
    g = RotatedSurface(5, 5)
    det, _ = sample(g, 0.05, 300, 61)
    det = torch.as_tensor(det).cuda()
    ctype = torch.as_tensor(g.check_type.astype(np.uint8)).cuda()
    E = torch.randn(4, 64, device="cuda", requires_grad=True)
    h, h16 = embed_tokens(det, ctype, E)
    E_ref = E.detach().clone().requires_grad_(True)
    h_ref = F.embedding(2 * ctype.long() + det.long(), E_ref)
    assert torch.equal(h, h_ref) and torch.equal(h16, h_ref.to(torch.bfloat16))
    gh = torch.randn_like(h)
    gh16 = torch.randn_like(h).to(torch.bfloat16)
    (h * gh).sum().backward(retain_graph=True)
    (h16.float() * gh16.float()).sum().backward()
    (h_ref * (gh + gh16.float())).sum().backward()
    assert rel(E.grad, E_ref.grad) < 1e-5


def test_head_loss_matches_the_torch_composition():
    """ops.head_bce (the training network's head and loss in one pass each way) against F.linear under bf16 autocast
    followed by binary_cross_entropy_with_logits on the logits in fp32: the loss within 1e-3 relative (bf16 logits
    whose fp32 sums run in another order may round one step apart), the input, weight and bias gradients within
    2e-2 of max |ref| (bf16 outputs); an upstream gradient of 2 doubles them."""
    from codecoder_b200.ops import head_bce
    gen = torch.Generator(device="cuda").manual_seed(5)
    rows, C = 5000, 96
    hd = torch.randn(rows, C, device="cuda", generator=gen).bfloat16()
    W0 = torch.randn(2, C, device="cuda", generator=gen) / C ** 0.5
    b0 = 0.1 * torch.randn(2, device="cuda", generator=gen)
    y = (torch.rand(rows, 2, device="cuda", generator=gen) < 0.1).to(torch.uint8)
    out = []
    for fused in (True, False):
        h = hd.clone().requires_grad_()
        W = W0.clone().requires_grad_()
        b = b0.clone().requires_grad_()
        if fused:
            loss = head_bce(h, W, b, y)
        else:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                z = F.linear(h, W, b)
            loss = F.binary_cross_entropy_with_logits(z.float(), y.float())
        (2.0 * loss).backward()
        out.append((loss.detach(), h.grad, W.grad, b.grad))
    (lf, hf, Wf, bf), (lu, hu, Wu, bu) = out
    assert abs(float(lf) - float(lu)) <= 1e-3 * abs(float(lu))
    assert rel(hf, hu) < 2e-2 and rel(Wf, Wu) < 2e-2 and rel(bf, bu) < 2e-2, (rel(hf, hu), rel(Wf, Wu), rel(bf, bu))
