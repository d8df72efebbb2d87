#!/usr/bin/env python
"""Throughput benchmark of the rotated-surface bipartite-conv pre-decoder (d = 13, 13 rounds, 8 layers, C = 128, bf16).

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]
    (N > 1: torchrun --nproc-per-node N bench.py --gpus N ..., one rank per GPU)

A step is one forward pass of the pre-decoder over this rank's shard of a 262,144-shot batch (shards of
262144 / N shots, no collective on the data path): detectors -> 16 bipartite steps -> X/Z logits -> residual
syndrome.  Inputs are seeded phenomenological shots (p = 0.005) drawn on the device; weights are seeded.
`value` times K steps on device-resident inputs with CUDA events (max over ranks); `e2e` times the same steps through
the public PreDecoder API from pinned host memory, copies in and out included; `roofline` is the bipartite-step
kernel's algorithmic tensor FLOP rate (CUDA events around every step launch of the last timed step) against the
measured sustained bf16 peak; `cpu_baseline` times the CPU oracle (the reference's fp32 index_select + matmul path,
restated) on this host's cores for a bounded sample.  --impl reference times only that CPU path.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from dataclasses import replace

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "syndromes/sec/GPU at d=13 (1/2/4/8 B200, % roofline); p99 per-round latency d=17"
UNIT = "syndromes/s (aggregate over all GPUs)"
TOTAL_SHOTS = 262144
SEED = 1234
# DRAM bytes per (target node x shot) of one d = 13 bipartite step of gmm_wide_kernel, from one ncu capture of a
# 4,096-shot check -> data launch: (dram__bytes_read.sum + dram__bytes_write.sum) / (2,197 nodes x 4,096 shots).
# Traffic grows in proportion to the shots, so it is scaled to the shots of a launch.
WIDE_D13_DRAM_BYTES_PER_NODE_SHOT = 766.4
PARITY_SHOTS = 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="d13_bf16")
    ap.add_argument("--shots", type=int, default=TOTAL_SHOTS, help="total shots per step over all GPUs")
    ap.add_argument("--chunk", type=int, default=16384, help="shots per pass through the network")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-stream", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the d=5 fp32, d=9 bf16 and Cascade workloads")
    ap.add_argument("--cascade-only", action="store_true",
                    help="time only the C14-size Cascade network (one JSON object; for launch lists and profiles)")
    ap.add_argument("--cascade-shots", type=int, default=4096, help="shots of the Cascade network's batch")
    ap.add_argument("--stream-rounds", type=int, default=20000)
    ap.add_argument("--no-train", action="store_true")
    ap.add_argument("--train-steps", type=int, default=6)
    ap.add_argument("--train-batch", type=int, default=8192, help="shots per GPU per training step")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"bf16_tflops": p["bf16_tflops"], "bf16_tflops_sustained": p["bf16_tflops_sustained"],
                "hbm_gbs": p["hbm_gbs"], "source": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def workload(cfg, g, shots_per_gpu, n):
    return {"workload": f"rotated surface d={cfg.d}, {cfg.rounds} rounds, phenomenological p={cfg.p}; "
                        f"{cfg.layers} layers x [check->data, data->check], C={cfg.channels}, K={cfg.K}, "
                        f"{cfg.dtype}; X/Z head + residual syndrome",
            "d": cfg.d, "rounds": cfg.rounds, "layers": cfg.layers, "channels": cfg.channels, "K": cfg.K,
            "checks": g.N_c, "data_nodes": g.N_d, "global_batch": shots_per_gpu * n, "shots_per_gpu": shots_per_gpu,
            "parallelism": f"shots sharded over {n} GPU(s), no collective",
            "l2": "inputs larger than L2 (detectors 573 MB per 262144 shots; 18 GB activations per 16384-shot pass)"}


class ClockSampler:
    """nvidia-smi samples of this GPU's clocks and throttle reasons while the timed region runs."""
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, device_index):
        import torch
        self.sel = []
        try:
            u = str(torch.cuda.get_device_properties(device_index).uuid)
            if u:
                self.sel = ["-i", u if u.startswith("GPU-") else "GPU-" + u]
        except Exception:
            self.sel = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", *self.sel, "--query-gpu=" + ",".join(self.FIELDS),
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=10)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != len(self.FIELDS):
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        busy = [r for r in rows if r[2] > 0.5 * max(x[2] for x in rows)] or rows
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in busy:
            for nm, v in zip(names, r[3][1:]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r[0] for r in busy), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(busy), "power_w_max": max(r[2] for r in rows)}


CPU_BATCHES = (1, 2, 4, 8, 16, 64)


def best_cpu_batch(g, cfg32, params, det):
    """The reference's CPU path (restated by the oracle: fp32 torch index_select + matmul on every host thread) is
    fastest at a small batch, where the materialised (B, NT, K C) gather stays in cache.  One warm-up and one timed
    call per candidate batch -> (batch, shots/s at that batch)."""
    import torch
    from oracle import predecoder_oracle as orc
    best = (1, 0.0)
    with torch.no_grad():
        for b in CPU_BATCHES:
            if b > len(det):
                break
            orc.predecoder(g, cfg32, params, det[:b], dtype=torch.float32)
            t = time.perf_counter()
            orc.predecoder(g, cfg32, params, det[:b], dtype=torch.float32)
            rate = b / (time.perf_counter() - t)
            if rate > best[1]:
                best = (b, rate)
    return best


def cpu_rate(g, cfg, params, det, seconds):
    """The CPU oracle (fp32 torch on every host thread) at its best batch on a bounded sample
    -> (shots/s, shots, threads, batch)."""
    import torch
    from oracle import predecoder_oracle as orc
    torch.set_num_threads(os.cpu_count() or 1)
    cfg32 = replace(cfg, dtype="f32")
    batch, _ = best_cpu_batch(g, cfg32, params, det)
    done = 0
    with torch.no_grad():
        t0 = time.perf_counter()
        while True:
            b0 = (done // batch * batch) % (len(det) - batch + 1)
            orc.predecoder(g, cfg32, params, det[b0:b0 + batch], dtype=torch.float32)
            done += batch
            if time.perf_counter() - t0 >= seconds:
                break
    dt = time.perf_counter() - t0
    return done / dt, done, torch.get_num_threads(), batch


FP32_FMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12   # nominal: 148 SMs x 128 FP32 FMA/clk x 2 x max SM clock


def measure_config(name, shots, steps, warmup, dev, pk, cpu_seconds):
    """One of the other workloads on one GPU: device-resident throughput, the step kernel's rate against its
    roofline, a parity sample against the oracle and the CPU oracle at its best batch."""
    import numpy as np
    import torch
    from codecoder_b200.geometry import RotatedSurface
    from codecoder_b200.modules import PreDecoder
    from codecoder_b200.params import CONFIGS, flops_per_shot, init_params, storage_params
    from codecoder_b200.sampler import sample_torch
    from oracle import predecoder_oracle as orc
    cfg = CONFIGS[name]
    g = RotatedSurface(cfg.d, cfg.rounds)
    params = init_params(cfg, SEED)
    det, _ = sample_torch(g, cfg.p, shots, SEED + 31, device=dev)
    pd = PreDecoder(g, cfg, params, device=dev, chunk_shots=16384)
    logits = torch.empty(shots, g.N_d, 2, dtype=torch.float32, device=dev)
    resid = torch.empty(shots, g.N_c, dtype=torch.uint8, device=dev)
    S = ((min(16384, shots) + 255) // 256) * 256
    chunks = [min(S, shots - b) for b in range(0, shots, S)]
    step_flops = [2.0 * cfg.K * cfg.channels ** 2 * (g.N_d if i % 2 == 0 else g.N_c) * sb
                  for sb in chunks for i in range(2 * cfg.layers)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in step_flops]
    for _ in range(warmup):
        pd.forward_into(det, logits, resid)
    torch.cuda.synchronize()
    pd.record_step_events(ev)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(steps):
        pd.forward_into(det, logits, resid)
    s1.record()
    s1.synchronize()
    pd.record_step_events([])
    if pd.status() != 0:
        raise RuntimeError(f"device watchdog fired in the {name} measurement")
    ms = s0.elapsed_time(s1)
    tc_ms = sum(a.elapsed_time(b) for a, b in ev)
    achieved = sum(step_flops) / (tc_ms / 1000.0) / 1e12
    f32 = cfg.dtype == "f32"
    if f32:
        narrow = cfg.channels in (8, 16, 32)        # equal widths <= 32: the resident-weight CUDA-core kernel
        peak, peak_kind, kernel, bound = FP32_FMA_PEAK_TFLOPS, "nominal FP32 FMA (148 SMs x 128 FMA/clk x 2 x 1965 MHz)", \
            (f"gmm_fma_narrow_kernel<float, {cfg.channels}>" if narrow else "gmm_fma_kernel<float>"), "fma"
    else:
        peak, peak_kind, kernel, bound = pk["bf16_tflops_sustained"], f"{pk['source']} sustained bf16 (cuBLAS)", \
            "gmm_wide_kernel", "tensor"
    pick = np.unique(np.linspace(0, shots - 1, min(16, shots)).astype(np.int64))
    sel = torch.as_tensor(pick, device=dev)
    det_s = det.index_select(0, sel).cpu().numpy()
    lg_s = logits.index_select(0, sel).cpu().numpy()
    rs_s = resid.index_select(0, sel).cpu().numpy()
    sp = storage_params(cfg, params)
    torch.set_num_threads(os.cpu_count() or 1)
    ref64, res64 = orc.predecoder_batched(g, cfg, sp, det_s, dtype=torch.float64, batch=16)
    if f32:
        parity = orc.parity_report(g, det_s, lg_s, rs_s, ref64, res64, 1e-4)
        parity["pass"] = bool(parity["logit_max_rel_err"] < 1e-4 and parity["residual_mismatch_outside_band"] == 0
                              and parity["residual_is_own_xor"])
    else:
        ref32, _ = orc.predecoder_batched(g, cfg, sp, det_s, dtype=torch.float32, batch=16)
        parity = orc.deep_parity(g, det_s, lg_s, rs_s, ref64, res64, ref32, 2e-2)
    rate, n_shots, threads, cb = cpu_rate(g, cfg, params, det[:64].cpu().numpy(), cpu_seconds)
    return {"workload": f"rotated surface d={cfg.d}, {cfg.rounds} rounds, p={cfg.p}; {cfg.layers} layers, "
                        f"C={cfg.channels}, K={cfg.K}, {cfg.dtype}; {shots} shots on one GPU",
            "value": steps * shots / (ms / 1000.0), "unit": "syndromes/s", "ms_per_step": ms / steps,
            "steps": steps, "warmup": warmup, "flop_per_shot": flops_per_shot(cfg, g.N_c, g.N_d),
            "roofline": {"bound": bound, "kernel": kernel, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "avg_launch_ms": tc_ms / len(ev),
                         "launches": len(ev)},
            "parity": parity,
            "cpu_baseline": {"value": rate, "unit": "syndromes/s", "cores": threads, "kind": "port", "batch": cb,
                             "sample": f"{n_shots} shots through the CPU oracle (fp32) at batch {cb}"}}


def synthetic_bb_layout(T, n2, n_det, k, seed):
    """A seeded stand-in for a BB code memory's circuit layout (the reference reads it from its Stim circuit):
    n_det detectors on distinct nodes of the (type, round, site) grid and k observables of 12 data qubits each."""
    import numpy as np
    rng = np.random.default_rng(seed)
    node = np.sort(rng.choice(2 * T * n2, size=n_det, replace=False))
    det_typ, rem = np.divmod(node, T * n2)
    det_t, det_site = np.divmod(rem, n2)
    logicals = np.zeros((k, 2 * n2), np.int64)
    for o in range(k):
        logicals[o, rng.choice(2 * n2, size=12, replace=False)] = 1
    return det_t, det_typ, det_site, logicals


def measure_cascade_net(tables_npz, dev, pk, shots=4096, steps=5, warmup=3):
    """The reference's Cascade BB72 network at C14's size (CascadeBB, cascade_net.py:262-343: H = 512, 14 bottleneck
    blocks with the bipartite convolution at 128 channels, pooled scatter read-out, 12 observables) in eval mode,
    seeded weights and BatchNorm statistics, on a seeded synthetic detector layout: device time per shot at `shots`
    shots with the detector bits resident on the GPU (the reference quotes C14 at batch 4,096, input on GPU), and
    the backbone (the 14 blocks alone) beside it.  The graph's tables are the reference's Geometry('bb72') tables as
    recorded in the test fixture."""
    import numpy as np
    import torch
    from types import SimpleNamespace
    from codecoder_b200.modules import CascadeNet, CascadeStack
    z = np.load(tables_npz)
    T, n2, N = int(z["T"]), int(z["n2"]), int(z["N"])
    geo = SimpleNamespace(T=T, n2=n2, N=N, c2d=[z["c2d0"], z["c2d1"]], d2c=[z["d2c0"], z["d2c1"]],
                          inv_c2d=[z["inv_c2d0"].astype(np.int64), z["inv_c2d1"].astype(np.int64)],
                          inv_d2c=[z["inv_d2c0"].astype(np.int64), z["inv_d2c1"].astype(np.int64)])
    H, L, n_det, k = 512, 14, 360, 12
    torch.manual_seed(SEED)
    net = CascadeNet(geo, H, L, *synthetic_bb_layout(T, n2, n_det, k, SEED), res="skip").to(dev).eval()
    with torch.no_grad():
        for m in net.modules():
            if isinstance(m, torch.nn.BatchNorm1d):
                m.running_var.uniform_(0.5, 2.0)
        net.mlp2.weight.normal_()
    rng = np.random.default_rng(SEED)
    det = torch.as_tensor((rng.random((shots, n_det)) < 0.05).astype(np.uint8), device=dev)
    h0 = torch.randn(shots, N, H, device=dev)

    def timed(fn):
        with torch.no_grad():
            for _ in range(warmup):
                out = fn()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(steps):
                out = fn()
            e.record()
            e.synchronize()
        if not bool(torch.isfinite(out).all()):
            raise RuntimeError("C14-sized Cascade network produced non-finite values")
        return s.elapsed_time(e) / steps

    ms = timed(lambda: net(det))
    ms_blocks = timed(lambda: CascadeStack.forward_blocks(net.blocks, h0)[0])
    Hb, K = H // 4, int(z["c2d0"].shape[1])
    flop = L * (2 * 2 * N * K * Hb * Hb + 2 * 2 * N * H * Hb) + 2 * k * 2 * K * N * H + 2 * k * 2 * K * H * H \
        + 2 * k * (H * 2 * H + 2 * H)
    return {"workload": f"Cascade network at C14 size: H=512, 14 bottleneck blocks (conv at 128 channels), BB72 graph "
                        f"({N} nodes), {n_det} detectors (seeded synthetic layout), {k} observables, eval, bf16 "
                        f"bottleneck and read-out GEMMs + fp32 residual stream, {shots} shots, input on the GPU",
            "shots": shots, "ms_per_batch": ms, "us_per_shot": ms * 1000.0 / shots,
            "backbone_us_per_shot": ms_blocks * 1000.0 / shots, "flop_per_shot": flop,
            "tflops": flop * shots / (ms * 1e-3) / 1e12, "tensor_frac_of_sustained": flop * shots / (ms * 1e-3) / 1e12
            / pk["bf16_tflops_sustained"],
            "kernels": "cascade_stem_kernel (tokens -> the first block's BN1 + SiLU, the embedded stream not written) "
                       "and gmm_tc_kernel (down + BN2 + SiLU); per block: the two-type conv (gmm_wide_kernel check -> "
                       "data, gmm_wide_kernel data -> check + BN3 + SiLU) and cascade_boundary_kernel (up, residual, "
                       "the next block's BN1 + SiLU + down + BN2 + SiLU, or bn_out + SiLU after the last; the first "
                       "reads the embedding by token); read-out: cuBLAS GEMMs (bf16 pooling and scatter, fp32 MLP); "
                       "backbone_us_per_shot: the 14 blocks from a materialised stream"}


def run_reference(args, cfg, g, params, rank, world):
    """--impl reference: the CPU path of the reference (restated by the oracle) at its best batch, rank 0 only."""
    if rank != 0:
        return
    import torch
    from codecoder_b200.sampler import sample
    from oracle import predecoder_oracle as orc
    torch.set_num_threads(os.cpu_count() or 1)
    det, _ = sample(g, cfg.p, 64, SEED)
    cfg32 = replace(cfg, dtype="f32")
    batch, probe_rate = best_cpu_batch(g, cfg32, params, det)
    # a step is n_batch calls at the best batch, about 2 s of CPU work
    n_batch = int(max(1, min(64, round(2.0 * probe_rate / batch))))
    times = []
    with torch.no_grad():
        for k in range(args.warmup + args.steps):
            t = time.perf_counter()
            for i in range(n_batch):
                b0 = (i * batch) % (len(det) - batch + 1)
                orc.predecoder(g, cfg32, params, det[b0:b0 + batch], dtype=torch.float32)
            if k >= args.warmup:
                times.append(time.perf_counter() - t)
    total = sum(times)
    shots = n_batch * batch
    rate = shots * len(times) / total
    sample_desc = (f"{shots} shots per step of the d={cfg.d} workload ({n_batch} calls at batch {batch}, the fastest of "
                   f"{list(CPU_BATCHES)}), fp32 CPU oracle of the reference's gather_mm path")
    line = {"metric": METRIC, "value": rate, "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload(cfg, g, args.shots // world, world),
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample_desc, "batch": batch},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    from codecoder_b200.geometry import RotatedSurface
    from codecoder_b200.params import CONFIGS, flops_per_shot, init_params
    cfg = CONFIGS[args.config]
    g = RotatedSurface(cfg.d, cfg.rounds)
    params = init_params(cfg, SEED)
    if args.impl == "reference":
        run_reference(args, cfg, g, params, rank, world)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    from codecoder_b200.build import build
    from codecoder_b200.modules import PreDecoder
    from codecoder_b200.sampler import sample_torch

    if rank == 0:
        build()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.cascade_only:
        if rank == 0:
            print(json.dumps(measure_cascade_net(os.path.join(REPO, "tests", "golden", "bb72_c14_conv.npz"), dev,
                                                 peaks(), shots=args.cascade_shots, steps=args.steps,
                                                 warmup=args.warmup)))
        return
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
        dist.barrier()
        build()                                         # no-op once rank 0 built it

    from codecoder_b200.shard import shard
    _, shots = shard(args.shots, world, rank)
    det, _ = sample_torch(g, cfg.p, shots, SEED + 7919 * rank, device=dev)
    pd = PreDecoder(g, cfg, params, device=dev, chunk_shots=args.chunk)
    logits = torch.empty(shots, g.N_d, 2, dtype=torch.float32, device=dev)
    resid = torch.empty(shots, g.N_c, dtype=torch.uint8, device=dev)

    S = ((min(args.chunk, shots) + 127) // 128) * 128
    chunks = [min(S, shots - b) for b in range(0, shots, S)]
    launches_per_fwd = len(chunks) * (2 * cfg.layers + 2)
    step_flops = []                                     # algorithmic FLOPs of each bipartite-step launch in order
    exec_flops = []                                     # the MMA work actually done (pad relations are skipped)
    live_c2d = float((g.c2d[0] < g.N_c).sum()) / g.K
    live_d2c = float((g.d2c_all < g.N_d).sum()) / g.K
    for sb in chunks:
        for _ in range(cfg.layers):
            step_flops.append(2.0 * cfg.K * cfg.channels ** 2 * g.N_d * sb)
            step_flops.append(2.0 * cfg.K * cfg.channels ** 2 * g.N_c * sb)
            exec_flops.append(2.0 * cfg.K * cfg.channels ** 2 * live_c2d * sb)
            exec_flops.append(2.0 * cfg.K * cfg.channels ** 2 * live_d2c * sb)
    ev_pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in step_flops]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        pd.forward_into(det, logits, resid)
    torch.cuda.synchronize()
    if pd.status() != 0:
        raise RuntimeError("device watchdog fired during warm-up")

    pd.record_step_events(ev_pairs)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record()
        for _ in range(args.steps):
            pd.forward_into(det, logits, resid)
        end.record()
        end.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    pd.record_step_events([])
    step_ms = [a.elapsed_time(b) for a, b in ev_pairs]
    tc_ms = sum(step_ms)
    tc_flops = sum(step_flops)
    if pd.status() != 0:
        raise RuntimeError("device watchdog fired in the timed region")

    value = args.steps * args.shots / (ms / 1000.0)
    pk = peaks()
    achieved = tc_flops / (tc_ms / 1000.0) / 1e12
    fps = flops_per_shot(cfg, g.N_c, g.N_d)
    step_kernel = "gmm_pair_kernel" if (cfg.channels == 128 and os.environ.get("BPC_STEP_KERNEL") in
                                        ("pair", "pair_stream")) else "gmm_wide_kernel"
    roof = {"bound": "tensor", "kernel": f"{step_kernel} (bipartite step)", "achieved": achieved,
            "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops_sustained"],
            "peak_kind": f"{pk['source']} sustained bf16 (cuBLAS)", "traffic": None,
            "avg_launch_ms": tc_ms / len(step_ms), "launches": len(step_ms),
            "flop_per_unit": 2 * cfg.K * cfg.channels ** 2, "unit_desc": "target node x shot",
            "executed_tflops": sum(exec_flops) / (tc_ms / 1000.0) / 1e12,
            "whole_step_frac": value / world * fps / 1e12 / pk["bf16_tflops_sustained"]}
    if args.config == "d13_bf16":
        units_per_launch = (sum(step_flops) / len(step_flops)) / (2 * cfg.K * cfg.channels ** 2)
        roof["traffic"] = WIDE_D13_DRAM_BYTES_PER_NODE_SHOT * units_per_launch
        roof["traffic_unit"] = "DRAM bytes per launch"
        roof["traffic_source"] = ("ncu capture of one gmm_wide_kernel launch, d=13 check->data step, 4,096 shots "
                                  "(dram__bytes_read.sum + dram__bytes_write.sum / (2,197 nodes x 4,096 shots)), "
                                  "scaled by the shots of a launch")
        # sources read once + residual read + write, each 2C bytes per node and shot, averaged over the launches
        roof["algorithmic_bytes_per_launch"] = sum(
            (g.N_c + 2 * g.N_d if i % 2 == 0 else g.N_d + 2 * g.N_c) * sb * 2 * cfg.channels
            for i, sb in enumerate(sb for sb in chunks for _ in range(2 * cfg.layers))) / len(step_flops)

    parity = None
    if rank == 0 and not args.no_parity:
        # the timed run's own outputs for a fixed sample of its shots (spread over every pass) against the CPU
        # oracle, outside the timed region: the logit error, the band count and the residual bits
        import torch as _t
        from oracle import predecoder_oracle as orc
        from codecoder_b200.params import storage_params
        _t.set_num_threads(os.cpu_count() or 1)
        pick = np.unique(np.linspace(0, shots - 1, min(PARITY_SHOTS, shots)).astype(np.int64))
        sel = _t.as_tensor(pick, device=dev)
        det_s = det.index_select(0, sel).cpu().numpy()
        lg_s = logits.index_select(0, sel).cpu().numpy()
        rs_s = resid.index_select(0, sel).cpu().numpy()
        sp = storage_params(cfg, params)
        ref64, res64 = orc.predecoder_batched(g, cfg, sp, det_s, dtype=_t.float64, batch=16)
        if cfg.dtype == "f32":
            parity = orc.parity_report(g, det_s, lg_s, rs_s, ref64, res64, 1e-4)
            parity["pass"] = bool(parity["logit_max_rel_err"] < 1e-4 and parity["residual_mismatch_outside_band"] == 0
                                  and parity["residual_is_own_xor"])
        else:
            ref32, _ = orc.predecoder_batched(g, cfg, sp, det_s, dtype=_t.float32, batch=16)
            parity = orc.deep_parity(g, det_s, lg_s, rs_s, ref64, res64, ref32, 2e-2)
        parity["sample"] = (f"{len(pick)} shots spread over the timed batch (the last timed step's outputs) against "
                            f"the CPU oracle (float64 accumulation, bf16 storage rounding emulated; float32 "
                            f"accumulation for the oracle's own spread)")

    e2e = None
    if not args.no_e2e:
        # the public API from pinned host memory: PreDecoder.forward_host copies slices in and out on a copy stream
        # while the previous slice runs (C ABI bpc_predecoder_forward per slice)
        det_h = det.cpu().pin_memory()
        lg_h = torch.empty(logits.shape, dtype=logits.dtype, pin_memory=True)
        rs_h = torch.empty(resid.shape, dtype=resid.dtype, pin_memory=True)
        pd.forward_host(det_h, lg_h, rs_h)
        barrier()
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            pd.forward_host(det_h, lg_h, rs_h)
        e2.record()
        e2.synchronize()
        barrier()
        ms2 = max_over_ranks(s2.elapsed_time(e2))
        e2e = {"value": args.steps * args.shots / (ms2 / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": args.shots * g.N_c,
               "d2h_bytes_per_step": args.shots * (g.N_d * 2 * 4 + g.N_c),
               "api": "codecoder_b200.modules.PreDecoder.forward_host (C ABI bpc_predecoder_forward per slice)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        det_np = det[:64].cpu().numpy()
        rate, n_shots, threads, cb = cpu_rate(g, cfg, params, det_np, args.cpu_seconds)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port", "batch": cb,
               "sample": f"{n_shots} shots of the d={cfg.d} workload through the CPU oracle (fp32 torch "
                         f"index_select + matmul, the reference's gather_mm path) at batch {cb}, the fastest of "
                         f"{list(CPU_BATCHES)}, {threads} threads"}

    stream = None
    if rank == 0 and world == 1 and not args.no_stream:
        # d = 17 streaming: sliding window of 3 rounds, batch 1, one new round per step, one graph replay per round
        from codecoder_b200.sampler import sample_stream
        from codecoder_b200.streaming import PersistentStreamingDecoder, StreamingDecoder
        scfg = CONFIGS["d17_stream"]
        sparams = init_params(scfg, SEED)
        rounds = sample_stream(RotatedSurface(scfg.d, 1), scfg.p, args.stream_rounds + 200, SEED + 17)
        sd = StreamingDecoder(scfg.d, scfg.rounds, scfg, sparams, device=dev)
        lat_g = sd.latency(rounds[:min(len(rounds), 5200)], warmup=200)
        del sd
        # the resident kernel in both layouts; the headline is the one the default (auto) layout runs: the 8 clusters
        lats, used = {}, {}
        for layout in ("clusters", "one_cluster"):
            ps = PersistentStreamingDecoder(scfg.d, scfg.rounds, scfg, sparams, device=dev, layout=layout)
            try:
                ps.start()
                used[layout] = ps.layout()
                lats[layout] = ps.latency(rounds if layout == "clusters" else rounds[:5200], warmup=200)
                ps.stop()
            except RuntimeError as e:
                used[layout] = f"unavailable: {e}"
            finally:
                ps.close()
        # the kernels' own phase stamps of one round (tracing on, a short run of each layout)
        phases = {}
        for layout in lats:
            ps = PersistentStreamingDecoder(scfg.d, scfg.rounds, scfg, sparams, device=dev, layout=layout, trace=True)
            try:
                ps.latency(rounds[:600], warmup=100)
                ps.stop()
                tab = ps.phase_table()
                keys = list(PersistentStreamingDecoder.PHASES) + ["total"]
                phases[layout] = {"median_ns_per_step": {k: float(np.median([st[k] for st in tab["steps"]]))
                                                         for k in keys},
                                  "round_ns": tab["round"], "steps": len(tab["steps"])}
            finally:
                ps.close()
        head = "clusters" if "clusters" in lats else "one_cluster"
        lat = lats[head]
        sg = ps.geo
        sflop = flops_per_shot(scfg, sg.N_c, sg.N_d)
        sms = {"one_cluster": f"one cluster of {2 * max((sg.N_d + 127) // 128, 2 * ((sg.nh * scfg.rounds + 127) // 128))}"
                              f" CTAs", "clusters": "8 clusters x 8 CTAs"}
        stream = {"config": f"d={scfg.d}, window {scfg.rounds} rounds, batch 1, {scfg.layers} layers, C={scfg.channels},"
                            f" {scfg.dtype}, p={scfg.p}; one resident kernel ({sms[head]}) served through a request "
                            f"line in mapped host memory (C ABI bpc_stream_run)",
                  "layout": head,
                  "rounds": int(len(lat)), "p50_us": float(np.percentile(lat, 50)),
                  "p99_us": float(np.percentile(lat, 99)), "mean_us": float(lat.mean()),
                  "clock": "host wall clock in the library's loop, from writing a round's request to reading its "
                           "response (residual + newest logits) in host memory",
                  "graph_replay": {"p50_us": float(np.percentile(lat_g, 50)), "p99_us": float(np.percentile(lat_g, 99)),
                                   "rounds": int(len(lat_g)),
                                   "how": "StreamingDecoder: one CUDA-graph replay per round (node-tiled kernels)"},
                  "phases": phases,
                  "layouts": {k: ({"p50_us": float(np.percentile(v, 50)), "p99_us": float(np.percentile(v, 99)),
                                   "rounds": int(len(v)), "kernel": sms[k]} if k in lats else used[k])
                              for k, v in list(lats.items()) + [(k, None) for k in used if k not in lats]},
                  "flop_per_round": sflop, "roofline_us_all_sms": sflop / (pk["bf16_tflops"] * 1e12) * 1e6}

    cascade = None
    golden_bb72 = os.path.join(REPO, "tests", "golden", "bb72_c14_conv.npz")
    if rank == 0 and world == 1 and not args.no_configs and os.path.exists(golden_bb72):
        cascade = measure_cascade_net(golden_bb72, dev, pk)

    configs = None
    if rank == 0 and world == 1 and not args.no_configs:
        # the d = 5 fp32 (CUDA-core) and d = 9 bf16 workloads at their stated batches
        # the d = 5 step is ~1.5 ms: time 20 of them so that clock ramps and launch jitter average out
        configs = {"d5_fp32": measure_config("d5_fp32", 1024, max(args.steps, 20), max(args.warmup, 3), dev, pk, 4.0),
                   "d9_bf16": measure_config("d9_bf16", 65536, max(args.steps, 5), max(args.warmup, 3), dev, pk, 6.0)}

    train = None
    if not args.no_train:
        # d = 11 training step (bf16 autocast, BCE, Adam 1e-3) with DDP over NCCL at world > 1: fixed shots per GPU
        del det, logits, resid, pd
        if not args.no_e2e:
            del det_h, lg_h, rs_h
        torch.cuda.empty_cache()
        from codecoder_b200.train import PreDecoderNet, Trainer, train_flops_per_shot
        tcfg = CONFIGS["d11_train"]
        tg = RotatedSurface(tcfg.d, tcfg.rounds)
        torch.manual_seed(SEED)
        # one GPU: each step replays one CUDA graph (forward, backward, clipping, Adam); DDP steps run eagerly
        graphed = world == 1
        trn = Trainer(PreDecoderNet(tg, tcfg, init_params(tcfg, SEED)).to(dev), lr=1e-3, graph=graphed)
        tstep = trn.step_graphed if graphed else trn.step
        batches = [sample_torch(tg, tcfg.p, args.train_batch, SEED + 1000 * rank + i, device=dev) for i in range(4)]
        losses = []
        for i in range(args.warmup):
            losses.append(tstep(*batches[i % 4]))
        torch.cuda.synchronize()
        barrier()
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s3.record()
        for i in range(args.train_steps):
            losses.append(tstep(*batches[(args.warmup + i) % 4]))
        e3.record()
        e3.synchronize()
        barrier()
        ms3 = max_over_ranks(s3.elapsed_time(e3))
        losses = [float(l) for l in losses]
        tfps = train_flops_per_shot(tg, tcfg)
        train = {"config": f"d={tcfg.d}, {tcfg.rounds} rounds, p={tcfg.p}, {tcfg.layers} layers, C={tcfg.channels}, "
                           f"bf16 autocast, BCE vs sampled data-qubit errors, Adam lr 1e-3, grad-norm clip 1, "
                           f"{'DDP over NCCL, eager steps' if world > 1 else 'one GPU, each step one CUDA graph replay'}",
                 "shots_per_gpu": args.train_batch, "steps": args.train_steps, "warmup": args.warmup,
                 "ms_per_step": ms3 / args.train_steps,
                 "shots_per_s": args.train_steps * args.train_batch * world / (ms3 / 1000.0),
                 "flop_per_shot": tfps,
                 "tflops_per_gpu": args.train_steps * args.train_batch * tfps / (ms3 / 1000.0) / 1e12,
                 "loss_first": losses[0], "loss_last": losses[-1], "scaling": "weak",
                 "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9}

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": cfg.dtype, "data": "synthetic",
                "config": workload(cfg, g, shots, world), "per_gpu": value / world, "roofline": roof,
                "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
                "gpu_launches": launches_per_fwd * args.steps, "flop_per_shot": fps, "parity": parity,
                "streaming": stream, "configs": configs, "cascade_c14": cascade, "train": train}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
