"""The multi-GPU path's host logic on CPU: two gloo ranks shard a batch of shots, each computes its shard alone
(no collective on the data path), and the gathered results equal the single-process result; the timing reduction
takes the max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from codecoder_b200.shard import shard


def test_shard_partitions_exactly():
    for total in (0, 1, 7, 262144, 262145):
        for world in (1, 2, 3, 4, 8):
            spans = [shard(total, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == total
            pos = 0
            for s, c in spans:
                assert s == pos
                pos += c
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from codecoder_b200.geometry import RotatedSurface
    from codecoder_b200.params import CONFIGS, init_params, storage_params
    from codecoder_b200.sampler import sample
    from dataclasses import replace
    from oracle import predecoder_oracle as orc
    cfg = replace(CONFIGS["d5_fp32"], d=3, rounds=3, layers=2)
    g = RotatedSurface(cfg.d, cfg.rounds)
    det, _ = sample(g, 0.05, 37, 11)                         # the job's batch
    start, count = shard(len(det), world, rank)
    lg, res = orc.predecoder(g, cfg, storage_params(cfg, init_params(cfg, 5)), det[start:start + count])
    t = torch.tensor([float(rank + 1)])                      # per-rank "elapsed time"
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    parts = [None] * world
    dist.all_gather_object(parts, (start, res, lg))
    if rank == 0:
        out.put((float(t.item()), parts))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharding_matches_single_process():
    from dataclasses import replace
    from codecoder_b200.geometry import RotatedSurface
    from codecoder_b200.params import CONFIGS, init_params, storage_params
    from codecoder_b200.sampler import sample
    from oracle import predecoder_oracle as orc
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    tmax, parts = q.get(timeout=240)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert tmax == 2.0
    cfg = replace(CONFIGS["d5_fp32"], d=3, rounds=3, layers=2)
    g = RotatedSurface(cfg.d, cfg.rounds)
    det, _ = sample(g, 0.05, 37, 11)
    lg, res = orc.predecoder(g, cfg, storage_params(cfg, init_params(cfg, 5)), det)
    parts.sort(key=lambda p: p[0])
    assert np.array_equal(np.concatenate([p[1] for p in parts]), res)
    np.testing.assert_allclose(np.concatenate([p[2] for p in parts]), lg, rtol=1e-12, atol=1e-12)


def _train_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from dataclasses import replace
    from codecoder_b200.geometry import RotatedSurface
    from codecoder_b200.params import CONFIGS, init_params
    from codecoder_b200.sampler import sample
    from codecoder_b200.train import PreDecoderNet, Trainer
    from oracle import predecoder_oracle as orc
    cfg = replace(CONFIGS["d5_fp32"], d=3, rounds=3, layers=2, channels=16)
    g = RotatedSurface(cfg.d, cfg.rounds)
    det, err = sample(g, 0.05, 16, 21)                       # the global batch; each rank takes its half
    start, count = shard(len(det), world, rank)
    net = PreDecoderNet(g, cfg, init_params(cfg, 9), gmm=lambda x, w, i, v: orc.gather_mm(x, w, i))
    tr = Trainer(net, lr=1e-2)
    for _ in range(2):
        tr.step(torch.as_tensor(det[start:start + count]), torch.as_tensor(err[start:start + count]))
    stop, bad = tr.agree(stop=rank == 1, bad=False)
    state = {k: v.detach().numpy().copy() for k, v in net.state_dict().items()}   # numpy: picklable by value
    parts = [None] * world
    dist.all_gather_object(parts, state)
    if rank == 0:
        out.put((stop, bad, parts))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_ddp_training_step_matches_single_process():
    """DDP over gloo: two ranks on halves of a batch end with identical weights, equal to one process on the whole
    batch (the all-reduce averages the gradients; the loss is a mean), and the flag reduction is a MAX."""
    from dataclasses import replace
    from codecoder_b200.geometry import RotatedSurface
    from codecoder_b200.params import CONFIGS, init_params
    from codecoder_b200.sampler import sample
    from codecoder_b200.train import PreDecoderNet, Trainer
    from oracle import predecoder_oracle as orc
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_train_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    stop, bad, parts = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert stop is True and bad is False
    for k in parts[0]:
        assert np.array_equal(parts[0][k], parts[1][k]), k
    cfg = replace(CONFIGS["d5_fp32"], d=3, rounds=3, layers=2, channels=16)
    g = RotatedSurface(cfg.d, cfg.rounds)
    det, err = sample(g, 0.05, 16, 21)
    net = PreDecoderNet(g, cfg, init_params(cfg, 9), gmm=lambda x, w, i, v: orc.gather_mm(x, w, i))
    tr = Trainer(net, lr=1e-2)
    for _ in range(2):
        tr.step(torch.as_tensor(det), torch.as_tensor(err))
    for k, v in net.state_dict().items():
        np.testing.assert_allclose(parts[0][k], v.numpy(), rtol=1e-5, atol=1e-6)
