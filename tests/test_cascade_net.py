"""CascadeNet (the reference's CascadeBB, cascade_net.py:262-343) on the host: its stem tokens and pooling matrix
against the reference's own buffers (recorded in the golden fixture by tests/golden/make_golden.py), its state_dict
keys against the reference's, and the pooled read-out against the read-out as the paper writes it (scatter the
relations to the data nodes, then average over each observable's support, cascade_net.py:331-340), restated here in
numpy.  Tolerance of the read-out: 1e-5 relative to max |ref| (fp32 against fp64)."""
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from codecoder_b200.modules import CascadeNet


@pytest.fixture(scope="module")
def fixtures(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "cascade_net_bb72.npz"))), \
        dict(np.load(os.path.join(golden_dir, "bb72_c14_conv.npz")))


def net_geo(z, conv_z):
    for k in range(2):
        assert np.array_equal(z[f"c2d{k}"], conv_z[f"c2d{k}"]) and np.array_equal(z[f"d2c{k}"], conv_z[f"d2c{k}"])
    return SimpleNamespace(T=int(z["T"]), n2=int(z["n2"]), N=int(z["N"]),
                           c2d=[z["c2d0"], z["c2d1"]], d2c=[z["d2c0"], z["d2c1"]],
                           inv_c2d=[conv_z["inv_c2d0"].astype(np.int64), conv_z["inv_c2d1"].astype(np.int64)],
                           inv_d2c=[conv_z["inv_d2c0"].astype(np.int64), conv_z["inv_d2c1"].astype(np.int64)])


def make_net(z, conv_z, H=None, L=None):
    return CascadeNet(net_geo(z, conv_z), H or int(z["H"]), L or int(z["L"]), z["det_t"], z["det_typ"], z["det_site"],
                      z["logicals"], res=str(z["res"]))


def test_cascade_net_tokens_pool_and_keys_match_the_reference(fixtures):
    z, conv_z = fixtures
    net = make_net(z, conv_z)
    assert np.array_equal(net.tokens(torch.as_tensor(z["det"])).numpy(), z["tokens"].astype(np.int64))
    assert np.array_equal(net.pool.numpy(), z["pool"])
    sd = {k[3:]: torch.as_tensor(v) for k, v in z.items() if k.startswith("sd.")}
    net.load_state_dict(sd, strict=True)
    assert sorted(net.state_dict()) == sorted(sd)


def test_cascade_net_rejects_colliding_detectors(fixtures):
    z, conv_z = fixtures
    place = [z[n].copy() for n in ("det_t", "det_typ", "det_site")]
    for a in place:
        a[1] = a[0]                                   # detectors 0 and 1 on one node
    with pytest.raises(ValueError):
        CascadeNet(net_geo(z, conv_z), 128, 2, *place, z["logicals"])


def readout_paper(net, h, c2d, T, n2):
    """The read-out as a scatter to every data node and an average over each support (fp64 numpy)."""
    B, N, H = h.shape
    W = net.scatter.detach().double().numpy().reshape(H, 2, c2d[0].shape[1], H)     # (out, d, r, in)
    hp = np.concatenate([h, np.zeros((B, 1, H))], 1)                                  # pad source N -> zero row
    data = np.stack([np.einsum("bnri,ori->bno", hp[:, c2d[d]], W[:, d]) for d in range(2)], 1)   # (B, 2, T n2, H)
    data = data.reshape(B, 2, T, n2, H).transpose(0, 1, 3, 2, 4).reshape(B, 2 * n2, T, H)
    z = np.stack([data[:, sup].mean((1, 2)) for sup in net.support], 1)   # (B, k, H)
    w1, b1 = net.mlp1.weight.detach().double().numpy(), net.mlp1.bias.detach().double().numpy()
    w2, b2 = net.mlp2.weight.detach().double().numpy(), net.mlp2.bias.detach().double().numpy()
    a = z @ w1.T + b1
    a = a / (1 + np.exp(-a))
    return (a @ w2.T + b2)[..., 0]


def test_cascade_net_pooled_readout_matches_the_paper_form(fixtures):
    z, conv_z = fixtures
    net = make_net(z, conv_z)
    net.load_state_dict({k[3:]: torch.as_tensor(v) for k, v in z.items() if k.startswith("sd.")})
    rng = np.random.default_rng(11)
    h = rng.standard_normal((3, int(z["N"]), int(z["H"])))
    with torch.no_grad():
        got = net.readout(torch.as_tensor(h, dtype=torch.float32)).double().numpy()
    ref = readout_paper(net, h, [z["c2d0"], z["c2d1"]], int(z["T"]), int(z["n2"]))
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) < 1e-5


def test_seeded_weights_fit_cascade_net_at_c14_width(golden_dir, fixtures):
    """The H = 512 fixture's network is rebuilt from seeded weights (tests/cascade_weights.py): they load strictly
    into CascadeNet and are the same on every call."""
    from cascade_weights import cascade_state
    _, conv_z = fixtures
    z = dict(np.load(os.path.join(golden_dir, "cascade_net_bb72_h512.npz")))
    net = CascadeNet(net_geo_h512(z, conv_z), int(z["H"]), int(z["L"]), z["det_t"], z["det_typ"], z["det_site"],
                     z["logicals"], res=str(z["res"]))
    shapes = {k: tuple(v.shape) for k, v in net.state_dict().items()}
    a, b = cascade_state(shapes, int(z["seed"])), cascade_state(shapes, int(z["seed"]))
    net.load_state_dict({k: torch.as_tensor(v) for k, v in a.items()}, strict=True)
    assert all(np.array_equal(a[k], b[k]) for k in a)


def net_geo_h512(z, conv_z):
    return SimpleNamespace(T=int(z["T"]), n2=int(z["n2"]), N=int(z["N"]), c2d=[conv_z["c2d0"], conv_z["c2d1"]],
                           d2c=[conv_z["d2c0"], conv_z["d2c1"]],
                           inv_c2d=[conv_z["inv_c2d0"].astype(np.int64), conv_z["inv_c2d1"].astype(np.int64)],
                           inv_d2c=[conv_z["inv_d2c0"].astype(np.int64), conv_z["inv_d2c1"].astype(np.int64)])
