"""Streaming (sliding window, batch 1, CUDA-graph replay) against the batch forward on the same windows."""
import numpy as np
import pytest
import torch
from dataclasses import replace

from codecoder_b200.geometry import RotatedSurface
from codecoder_b200.modules import PreDecoder
from codecoder_b200.params import CONFIGS, init_params
from codecoder_b200.sampler import sample_stream
from codecoder_b200.streaming import StreamingDecoder

pytestmark = pytest.mark.gpu


def test_streaming_matches_batch_windows():
    cfg = replace(CONFIGS["d17_stream"], d=9, layers=3)
    W = cfg.rounds
    params = init_params(cfg, 31)
    sd = StreamingDecoder(cfg.d, W, cfg, params, device="cuda")
    g = RotatedSurface(cfg.d, W)
    stream = sample_stream(g, 0.05, 8, 32)
    batch = PreDecoder(g, cfg, params, device="cuda")
    nh = g.nh
    win = np.zeros((2, W, nh), np.uint8)
    for t in range(len(stream)):
        res, lg_new = sd.step(stream[t])
        win[:, :-1] = win[:, 1:].copy()
        win[0, -1], win[1, -1] = stream[t][:nh], stream[t][nh:]
        ref_lg, ref_rs = batch(torch.as_tensor(win.reshape(1, -1)).cuda())
        assert torch.equal(res.clone(), ref_rs[0].cpu())
        assert torch.equal(lg_new.clone(), ref_lg[0, (W - 1) * g.n_data_round:].cpu())


def test_streaming_latency_is_measured():
    cfg = CONFIGS["d17_stream"]
    sd = StreamingDecoder(cfg.d, cfg.rounds, cfg, init_params(cfg, 33), device="cuda")
    lat = sd.latency(sample_stream(RotatedSurface(cfg.d, 1), cfg.p, 300, 34), warmup=50)
    assert len(lat) == 250 and np.all(lat > 0)
    print("d17 window-3 per-round latency us p50 %.1f p99 %.1f" % (np.percentile(lat, 50), np.percentile(lat, 99)))


@pytest.mark.parametrize("layout", ["clusters", "one_cluster"])
@pytest.mark.parametrize("d", [9, 13, 17])
def test_persistent_stream_matches_graph_stream(d, layout):
    """The resident kernel (mapped request line) gives the graph-replay decoder's bits round after round, in both
    layouts (the one-cluster layout adds relations 0-3 in one CTA and 4-7 in its partner, in the same order)."""
    from codecoder_b200.streaming import PersistentStreamingDecoder
    cfg = replace(CONFIGS["d17_stream"], d=d)
    params = init_params(cfg, 41)
    stream = sample_stream(RotatedSurface(d, 1), 0.02, 12, 42)
    ref = StreamingDecoder(d, cfg.rounds, cfg, params, device="cuda")
    ref.capture()                          # before the resident kernel starts: capture synchronises
    ps = PersistentStreamingDecoder(d, cfg.rounds, cfg, params, device="cuda", layout=layout)
    try:
        ps.start()
        assert ps.layout() == layout
        for t in range(len(stream)):
            r_res, r_lg = ref.step(stream[t])
            p_res, p_lg = ps.step(stream[t])
            assert np.array_equal(p_res, r_res.numpy()), t
            assert np.array_equal(p_lg, r_lg.numpy()), t
        lat = ps.latency(sample_stream(RotatedSurface(d, 1), cfg.p, 400, 43), warmup=100)
        print("persistent %s d%d window-3 per-round latency us p50 %.1f p99 %.1f" %
              (layout, d, np.percentile(lat, 50), np.percentile(lat, 99)))
        ps.stop()
        assert ps.status() == 2
    finally:
        ps.close()


@pytest.mark.parametrize("layout", ["clusters", "one_cluster"])
def test_persistent_stream_idle_watchdog_leaves_a_usable_context(layout):
    """No request within the idle limit: the kernel leaves by itself with status 4; a round afterwards is an error,
    not a hang, and the device keeps working."""
    import time
    from codecoder_b200.sampler import sample
    from codecoder_b200.streaming import PersistentStreamingDecoder
    cfg = replace(CONFIGS["d17_stream"], d=9)
    params = init_params(cfg, 5)
    ps = PersistentStreamingDecoder(9, cfg.rounds, cfg, params, device="cuda", idle_timeout_ms=200, layout=layout)
    try:
        ps.start()
        time.sleep(1.0)
        assert ps.status() == 4
        with pytest.raises(RuntimeError):
            ps.step(np.zeros(2 * ps.nh, np.uint8), timeout_us=200_000)
    finally:
        ps.close()
    g = RotatedSurface(9, cfg.rounds)
    det, _ = sample(g, 0.02, 8, 6)
    lg, rs = PreDecoder(g, cfg, params, device="cuda")(torch.as_tensor(det).cuda())
    torch.cuda.synchronize()
    assert torch.isfinite(lg).all()


@pytest.mark.parametrize("layout", ["clusters", "one_cluster"])
def test_persistent_stream_round_timeout_refuses_rounds_until_restart(layout):
    """A round the host gives up on (its timeout ends before the response) leaves the kernel still working on it:
    a later request would overwrite the line it may be reading, so every later round is refused until the stream is
    stopped and started again; after the restart rounds are answered again."""
    from codecoder_b200.streaming import PersistentStreamingDecoder
    cfg = replace(CONFIGS["d17_stream"], d=9)
    params = init_params(cfg, 7)
    rounds = sample_stream(RotatedSurface(9, 1), 0.02, 4, 8)
    ps = PersistentStreamingDecoder(9, cfg.rounds, cfg, params, device="cuda", idle_timeout_ms=2000, layout=layout)
    try:
        ps.start()
        ps.step(rounds[0])
        with pytest.raises(RuntimeError, match="within the timeout"):
            ps.step(rounds[1], timeout_us=1)             # no round is answered within a microsecond
        with pytest.raises(RuntimeError, match="stop and start"):
            ps.step(rounds[2])
        ps.stop()
        ps.start()
        res, lg = ps.step(rounds[3])
        assert np.isfinite(lg).all() and res.shape == (ps.geo.N_c,)
        ps.stop()
        assert ps.status() == 2
    finally:
        ps.close()


@pytest.mark.parametrize("layout", ["clusters", "one_cluster"])
def test_persistent_stream_trace_gives_a_phase_table(layout):
    """With tracing on, the kernel's global-timer stamps of the last round served come back after stop: every step
    has its phases in order, and the round's embedding and publication are stamped."""
    from codecoder_b200.streaming import PersistentStreamingDecoder
    cfg = replace(CONFIGS["d17_stream"], d=9)
    params = init_params(cfg, 9)
    rounds = sample_stream(RotatedSurface(9, 1), 0.02, 40, 10)
    ps = PersistentStreamingDecoder(9, cfg.rounds, cfg, params, device="cuda", layout=layout, trace=True)
    try:
        ps.latency(rounds, warmup=10)
        ps.stop()
        tab = ps.phase_table()
        assert [s["step"] for s in tab["steps"]] == list(range(2 * cfg.layers - 1))
        for s in tab["steps"]:
            assert all(s[p] >= 0 for p in ps.PHASES) and 0 < s["total"] < 1e6
        assert tab["round"]["embed"] >= 0 and tab["round"]["publish"] > 0
        tr = ps.trace()
        assert np.all(np.diff(tr[0, 0, :7]) >= 0)
    finally:
        ps.close()
