"""Generate the golden fixtures of tests/golden from the reference's own code.

Run where the reference tree is checked out, naming its root in REFERENCE_ROOT:
    REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py
It imports the reference's bb.cascade_net (training/bb/ising_compare/bb/cascade_net.py) unchanged and records:
  bb72_c14_conv.npz      the reference's Geometry('bb72') tables, the trained relation matrices of the released C14
                         network's first block (weights/cascade_bb72/C14.pt, key 'ema', rounded to bf16), a seeded
                         input, and the outputs of the reference's gather_mm, gather_mm_ref and BipartiteConv.forward
                         (fp32, CPU)
  surface_gmm.npz        the rotated-surface tables of codecoder_b200.geometry run through the reference's gather_mm
                         (several channel widths, including C_in != C_out)
  predecoder_<cfg>.npz   the pre-decoder composed from the reference's gather_mm on seeded shots: det, logits,
                         residual (weights regenerate from the stored seed with codecoder_b200.params.init_params)
  cascade_block_c14.npz  the reference's Block(512, Geometry('bb72'), L=14, res='skip') in eval mode with the C14
                         network's block-0 weights (relation, down and up matrices rounded to bf16; BatchNorm in
                         fp32) on a seeded bf16-valued input, and its output (fp32, CPU)
  cascade_net_bb72.npz   the reference's whole CascadeBB (H = 128, L = 2) on the BB72 graph with a seeded synthetic
                         detector layout (the Stim layout is absent): its state_dict, the layout, seeded shots and
                         the fp32 CPU forward's logits
  gather_mm_bwd.npz      input and weight gradients from the reference's _GatherMM.backward (autograd through
                         cn.gather_mm, fp32, CPU) for seeded upstream gradients: rotated-surface steps at several
                         widths and BipartiteConv(128, Geometry('bb72')) with the C14 relation matrices (its
                         input gradient and two of its four weight gradients)
The fixtures are small; the device never reads the reference tree.
"""
import hashlib
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("REFERENCE_ROOT")
if not REF or not os.path.isdir(REF):
    sys.exit("make_golden.py: set REFERENCE_ROOT to the root of the reference checkout")
sys.path[:0] = [REPO, os.path.join(REF, "training/bb/ising_compare"), os.path.join(REF, "training/bb/qldpc_neural")]

from bb import cascade_net as cn  # noqa: E402  (the reference, unchanged)

from codecoder_b200.geometry import RotatedSurface  # noqa: E402
from codecoder_b200.params import CONFIGS, init_params, round_bf16, storage_params  # noqa: E402
from codecoder_b200.sampler import sample  # noqa: E402


def bf16_bits(a):
    return (np.ascontiguousarray(round_bf16(a)).view(np.uint32) >> 16).astype(np.uint16)


def params_sha(params):
    h = hashlib.sha256()
    for k in sorted(params):
        h.update(k.encode())
        h.update(np.ascontiguousarray(params[k], np.float32).tobytes())
    return h.hexdigest()


def make_bb72():
    geo = cn.Geometry("bb72")
    ck = torch.load(os.path.join(REF, "weights/cascade_bb72/C14.pt"), map_location="cpu", weights_only=False)
    ema = ck["ema"]
    C = ck["cfg"]["H"] // 4
    conv = cn.BipartiteConv(C, geo, impl="torch")
    names = ["w_c2d.0", "w_c2d.1", "w_d2c.0", "w_d2c.1"]
    ws = {n: torch.as_tensor(round_bf16(ema["blocks.0.conv." + n].float().numpy())) for n in names}
    with torch.no_grad():
        conv.w_c2d[0].copy_(ws["w_c2d.0"])
        conv.w_c2d[1].copy_(ws["w_c2d.1"])
        conv.w_d2c[0].copy_(ws["w_d2c.0"])
        conv.w_d2c[1].copy_(ws["w_d2c.1"])
    rng = np.random.default_rng(1401)
    B = 2
    x = torch.as_tensor(round_bf16(rng.standard_normal((B, geo.N, C)).astype(np.float32)))
    with torch.no_grad():
        y_mod = conv(x)
        y0 = cn.gather_mm(x, conv.w_c2d[0], torch.as_tensor(geo.c2d[0]), torch.as_tensor(geo.inv_c2d[0]))
        y0_ref = cn.gather_mm_ref(x, conv.w_c2d[0], torch.as_tensor(geo.c2d[0]))
    assert torch.allclose(y0, y0_ref, atol=1e-4), "reference gather_mm != gather_mm_ref"
    out = {"x_bf16": bf16_bits(x.numpy()), "y_module": y_mod.numpy(), "y_c2d0": y0.numpy(), "C": C, "B": B,
           "N": geo.N, "T": geo.T, "n2": geo.n2}
    for n in names:
        out[n.replace(".", "_") + "_bf16"] = bf16_bits(ws[n].numpy())
    for k in range(2):
        out[f"c2d{k}"] = geo.c2d[k].astype(np.int32)
        out[f"d2c{k}"] = geo.d2c[k].astype(np.int32)
        out[f"inv_c2d{k}"] = geo.inv_c2d[k].astype(np.int32)
        out[f"inv_d2c{k}"] = geo.inv_d2c[k].astype(np.int32)
    np.savez_compressed(os.path.join(HERE, "bb72_c14_conv.npz"), **out)
    print("bb72_c14_conv", {k: getattr(v, "shape", v) for k, v in out.items()})


def make_surface_gmm():
    out = {}
    rng = np.random.default_rng(1402)
    cases = [("d5_c64", 5, 5, 64, 64, 3), ("d5_c128", 5, 5, 128, 128, 2), ("d3_ci64_co128", 3, 3, 64, 128, 5),
             ("d3_c96", 3, 3, 96, 96, 4), ("d5_c32", 5, 5, 32, 32, 4)]
    for name, d, R, ci, co, B in cases:
        geo = RotatedSurface(d, R)
        for step, idx, ns in (("c2d", geo.c2d[0], geo.N_c), ("d2c", geo.d2c_all, geo.N_d)):
            x = round_bf16(rng.standard_normal((B, ns, ci)).astype(np.float32))
            w = round_bf16((rng.standard_normal((co, geo.K * ci)) / np.sqrt(geo.K * ci)).astype(np.float32))
            inv = geo.inverse(idx, ns)
            with torch.no_grad():
                y = cn.gather_mm(torch.as_tensor(x), torch.as_tensor(w), torch.as_tensor(idx), torch.as_tensor(inv))
            key = f"{name}_{step}"
            out[key + "_x"] = bf16_bits(x)
            out[key + "_w"] = bf16_bits(w)
            out[key + "_idx"] = idx.astype(np.int32)
            out[key + "_y"] = y.numpy()
            out[key + "_meta"] = np.array([d, R, ci, co, B, ns], np.int64)
    np.savez_compressed(os.path.join(HERE, "surface_gmm.npz"), **out)
    print("surface_gmm", len(out) // 5, "cases")


def reference_predecoder(geo, cfg, params, det):
    """The pre-decoder composed from the reference's gather_mm (fp32, CPU), bf16 storage rounding for a bf16
    network applied where the device stores bf16."""
    bf = cfg.dtype == "bf16"

    def st(a):
        return a.to(torch.bfloat16).float() if bf else a

    p = storage_params(cfg, params)
    det_t = torch.as_tensor(det).long()
    tok = 2 * torch.as_tensor(geo.check_type) + det_t
    hc = st(torch.as_tensor(p["embed"])[tok])
    hd = None
    for layer in range(cfg.layers):
        acc = torch.cat([cn.gather_mm(hc, torch.as_tensor(w), torch.as_tensor(t), torch.as_tensor(geo.inverse(t, geo.N_c)))
                         for w, t in zip(p["w_c2d"][layer], geo.c2d)], 1)
        g_ = F.gelu(acc, approximate="tanh")
        hd = st(g_ if hd is None else hd + g_)
        acc = torch.cat([cn.gather_mm(hd, torch.as_tensor(w), torch.as_tensor(t), torch.as_tensor(geo.inverse(t, geo.N_d)))
                         for w, t in zip(p["w_d2c"][layer], geo.d2c)], 1)
        hc = st(hc + F.gelu(acc, approximate="tanh"))
    logits = hd @ torch.as_tensor(p["head_w"]).t() + torch.as_tensor(p["head_b"])
    e = (logits > 0).numpy().astype(np.uint8)
    res = det.astype(np.uint8).copy()
    for n in range(geo.N_d):                      # literal per-node XOR loop (small cases)
        for j in range(2):
            for c in geo.xor_nbr[n, j]:
                if c >= 0:
                    res[:, c] ^= e[:, n, j]
    return logits.numpy(), res, hc.numpy()


def make_predecoder():
    from dataclasses import replace
    cases = [("d3_fp32", replace(CONFIGS["d5_fp32"], d=3, rounds=3, layers=2, channels=32), 64),
             ("d5_fp32", CONFIGS["d5_fp32"], 64),
             ("d5_bf16_c64", replace(CONFIGS["d9_bf16"], d=5, rounds=5, layers=3, channels=64), 32)]
    for name, cfg, B in cases:
        geo = RotatedSurface(cfg.d, cfg.rounds)
        seed = 7000 + cfg.d
        params = init_params(cfg, seed)
        det, err = sample(geo, cfg.p * 10, B, seed + 1)       # denser than the workload so the fixture has events
        with torch.no_grad():
            logits, res, hc = reference_predecoder(geo, cfg, params, det)
        np.savez_compressed(os.path.join(HERE, f"predecoder_{name}.npz"), det=det, logits=logits, residual=res,
                            seed=seed, d=cfg.d, rounds=cfg.rounds, layers=cfg.layers,
                            channels=cfg.channels, dtype=cfg.dtype, params_sha256=params_sha(params))
        print("predecoder", name, det.shape, logits.shape, float(np.abs(logits).mean()))


def make_backward():
    out = {}
    rng = np.random.default_rng(1403)
    cases = [("d5_c64_c2d", 5, 64, 64, 3, "c2d"), ("d3_c96_d2c", 3, 96, 96, 4, "d2c"),
             ("d3_ci64_co128_c2d", 3, 64, 128, 3, "c2d"), ("d5_c32_c2d", 5, 32, 32, 4, "c2d")]
    for name, d, ci, co, B, step in cases:
        geo = RotatedSurface(d, d)
        idx, ns = (geo.c2d[0], geo.N_c) if step == "c2d" else (geo.d2c_all, geo.N_d)
        inv = geo.inverse(idx, ns)
        x = torch.as_tensor(round_bf16(rng.standard_normal((B, ns, ci)).astype(np.float32))).requires_grad_()
        w = torch.as_tensor(round_bf16((rng.standard_normal((co, geo.K * ci)) / np.sqrt(geo.K * ci))
                                       .astype(np.float32))).requires_grad_()
        gy = round_bf16(rng.standard_normal((B, idx.shape[0], co)).astype(np.float32))
        y = cn.gather_mm(x, w, torch.as_tensor(idx), torch.as_tensor(inv))
        y.backward(torch.as_tensor(gy))
        out[name + "_x"] = bf16_bits(x.detach().numpy())
        out[name + "_w"] = bf16_bits(w.detach().numpy())
        out[name + "_gy"] = bf16_bits(gy)
        out[name + "_idx"] = idx.astype(np.int32)
        out[name + "_inv"] = inv.astype(np.int64)
        out[name + "_gx"] = x.grad.numpy()
        out[name + "_gw"] = w.grad.numpy()
    # the reference module with the C14 relation matrices on Geometry('bb72'), one shot
    geo = cn.Geometry("bb72")
    z = np.load(os.path.join(HERE, "bb72_c14_conv.npz"))
    C = int(z["C"])
    conv = cn.BipartiteConv(C, geo, impl="torch")
    with torch.no_grad():
        for k in range(2):
            conv.w_c2d[k].copy_(torch.as_tensor((z[f"w_c2d_{k}_bf16"].astype(np.uint32) << 16).view(np.float32)))
            conv.w_d2c[k].copy_(torch.as_tensor((z[f"w_d2c_{k}_bf16"].astype(np.uint32) << 16).view(np.float32)))
    x = torch.as_tensor(round_bf16(rng.standard_normal((1, geo.N, C)).astype(np.float32))).requires_grad_()
    gy = round_bf16(rng.standard_normal((1, geo.N, C)).astype(np.float32))
    conv(x).backward(torch.as_tensor(gy))
    out["bb72_x"] = bf16_bits(x.detach().numpy())
    out["bb72_gy"] = bf16_bits(gy)
    out["bb72_gx"] = x.grad.numpy()
    out["bb72_gw_c2d0"] = conv.w_c2d[0].grad.numpy()     # two of the four weight gradients keep the file small
    out["bb72_gw_d2c1"] = conv.w_d2c[1].grad.numpy()
    np.savez_compressed(os.path.join(HERE, "gather_mm_bwd.npz"), **out)
    print("gather_mm_bwd", len(cases), "op cases + bb72 module")


def make_cascade_block():
    geo = cn.Geometry("bb72")
    ck = torch.load(os.path.join(REF, "weights/cascade_bb72/C14.pt"), map_location="cpu", weights_only=False)
    ema, cfg = ck["ema"], ck["cfg"]
    blk = cn.Block(cfg["H"], geo, cfg["L"], res=cfg["res"], impl="torch")
    sd = {k[len("blocks.0."):]: v for k, v in ema.items() if k.startswith("blocks.0.")}
    for k in list(sd):
        if k.startswith(("conv.", "down.", "up.")):
            sd[k] = torch.as_tensor(round_bf16(sd[k].float().numpy()))
    blk.load_state_dict(sd)
    blk.eval()
    rng = np.random.default_rng(1404)
    h = torch.as_tensor(round_bf16(rng.standard_normal((1, geo.N, cfg["H"])).astype(np.float32)))
    with torch.no_grad():
        out = blk(h)
    o = {"h_bf16": bf16_bits(h.numpy()), "out": out.numpy(), "H": cfg["H"], "L": cfg["L"], "res": cfg["res"],
         "eps": blk.bn1.eps, "down_bf16": bf16_bits(sd["down.weight"].numpy()), "up_bf16": bf16_bits(sd["up.weight"].numpy())}
    for i in (1, 2, 3):
        for a, b in (("weight", "weight"), ("bias", "bias"), ("mean", "running_mean"), ("var", "running_var")):
            o[f"bn{i}_{a}"] = sd[f"bn{i}.{b}"].float().numpy()
    np.savez_compressed(os.path.join(HERE, "cascade_block_c14.npz"), **o)
    print("cascade_block_c14", h.shape, float(out.abs().mean()))


def synthetic_bb72_layout(geo, rng, D=360, k=12):
    """A seeded stand-in for the Relay-BP circuit layout (bb.code.Layout needs Stim, which is absent): D detectors on
    distinct nodes of the (type, round, site) grid and k observables with supports on the 2 n2 data qubits."""
    T, n2 = geo.T, geo.n2
    node = np.sort(rng.choice(2 * T * n2, size=D, replace=False))
    det_typ, rem = np.divmod(node, T * n2)
    det_t, det_site = np.divmod(rem, n2)
    logicals = np.zeros((k, 2 * n2), np.int64)
    for o in range(k):
        logicals[o, rng.choice(2 * n2, size=12, replace=False)] = 1
    return det_t.astype(np.int64), det_typ.astype(np.int64), det_site.astype(np.int64), logicals


def make_cascade_net():
    """The reference's whole CascadeBB (stem, blocks, bn_out, pooled scatter read-out, MLP) at H = 128, L = 2 on the
    BB72 graph with a seeded synthetic layout; BatchNorm statistics and the (zero-initialised) last MLP layer drawn at
    random and the scatter projection scaled by 4, with a detector density of 0.25, so that the logits vary from shot
    to shot by ~15 % of their size (at initialisation they hardly depend on the detectors); matrices of the blocks
    rounded to bf16; fp32 CPU forward on 16 seeded shots, and the same forward under CPU bf16 autocast (the
    reference's own bf16 rounding error, the scale of the parity bar)."""
    geo = cn.Geometry("bb72")
    rng = np.random.default_rng(1405)
    det_t, det_typ, det_site, logicals = synthetic_bb72_layout(geo, rng)
    torch.manual_seed(1405)
    m = cn.CascadeBB("bb72", 128, 2, det_t, det_typ, det_site, logicals, res="skip", conv_impl="torch")
    with torch.no_grad():
        for name, mod in m.named_modules():
            if isinstance(mod, torch.nn.BatchNorm1d):
                mod.running_mean.copy_(torch.as_tensor(rng.standard_normal(mod.num_features) * 0.1, dtype=torch.float32))
                mod.running_var.copy_(torch.as_tensor(rng.uniform(0.5, 2.0, mod.num_features), dtype=torch.float32))
                mod.weight.copy_(torch.as_tensor(rng.uniform(0.5, 1.5, mod.num_features), dtype=torch.float32))
                mod.bias.copy_(torch.as_tensor(rng.standard_normal(mod.num_features) * 0.1, dtype=torch.float32))
        m.mlp2.weight.copy_(torch.as_tensor(rng.standard_normal(m.mlp2.weight.shape), dtype=torch.float32))
        m.mlp2.bias.copy_(torch.as_tensor(rng.standard_normal(1) * 0.1, dtype=torch.float32))
        m.scatter.mul_(4.0)
        for name, p in m.named_parameters():
            if name.startswith("blocks.") and p.ndim == 2:
                p.copy_(torch.as_tensor(round_bf16(p.numpy())))
    m.eval()
    det = (rng.random((16, len(det_t))) < 0.25).astype(np.uint8)
    with torch.no_grad():
        logits = m(torch.as_tensor(det))
    o = {"det": det, "logits": logits.numpy(), "det_t": det_t, "det_typ": det_typ, "det_site": det_site,
         "logicals": logicals, "H": 128, "L": 2, "res": "skip", "T": geo.T, "n2": geo.n2, "N": geo.N}
    for k in range(2):
        o[f"c2d{k}"] = np.asarray(geo.c2d[k], np.int32)
        o[f"d2c{k}"] = np.asarray(geo.d2c[k], np.int32)
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        o["logits_autocast"] = m(torch.as_tensor(det)).float().numpy()     # the reference's own bf16 run
    o["tokens"] = m.tokens(torch.as_tensor(det)).numpy().astype(np.uint8)
    o["pool"] = m.pool.numpy()
    for name, v in m.state_dict().items():
        o["sd." + name] = v.numpy()
    np.savez_compressed(os.path.join(HERE, "cascade_net_bb72.npz"), **o)
    print("cascade_net_bb72", det.shape, logits.shape, float(logits.abs().mean()), float(logits.std(0).mean()))


def make_cascade_net_h512():
    """The reference's CascadeBB at C14's width (H = 512, the 128-channel bottleneck; L = 2 blocks, res = 'skip') on
    the BB72 graph with the synthetic layout, every weight drawn by tests/cascade_weights.cascade_state (seed 512, so
    the test rebuilds them instead of the fixture storing ~9 M parameters); fp32 and CPU bf16 autocast logits of 16
    seeded shots at detector density 0.25."""
    sys.path.insert(0, os.path.dirname(HERE))
    from cascade_weights import cascade_state
    geo = cn.Geometry("bb72")
    rng = np.random.default_rng(512)
    det_t, det_typ, det_site, logicals = synthetic_bb72_layout(geo, rng)
    m = cn.CascadeBB("bb72", 512, 2, det_t, det_typ, det_site, logicals, res="skip", conv_impl="torch")
    state = cascade_state({k: tuple(v.shape) for k, v in m.state_dict().items()}, 512)
    m.load_state_dict({k: torch.as_tensor(v) for k, v in state.items()})
    m.eval()
    det = (rng.random((16, len(det_t))) < 0.25).astype(np.uint8)
    with torch.no_grad():
        logits = m(torch.as_tensor(det))
        with torch.autocast("cpu", dtype=torch.bfloat16):
            logits_ac = m(torch.as_tensor(det)).float()
    np.savez_compressed(os.path.join(HERE, "cascade_net_bb72_h512.npz"), det=det, logits=logits.numpy(),
                        logits_autocast=logits_ac.numpy(), det_t=det_t, det_typ=det_typ, det_site=det_site,
                        logicals=logicals, H=512, L=2, res="skip", seed=512, T=geo.T, n2=geo.n2, N=geo.N)
    print("cascade_net_bb72_h512", det.shape, logits.shape, float(logits.abs().mean()), float(logits.std(0).mean()),
          float((logits_ac - logits).abs().max() / logits.abs().max()))


if __name__ == "__main__":
    torch.manual_seed(0)
    if len(sys.argv) > 1:
        for name in sys.argv[1:]:
            globals()[name]()
        sys.exit(0)
    make_bb72()
    make_surface_gmm()
    make_predecoder()
    make_backward()
    make_cascade_block()
    make_cascade_net()
    make_cascade_net_h512()
