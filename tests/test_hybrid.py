"""The hybrid FNN-transformer mirror against the reference module's own
seeded weights and outputs (tests/golden/hybrid_reference_seed0.npz)."""
import hashlib
import os

import numpy as np
import pytest
import torch

from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridGNNConfig, HybridPieceTensorBatch

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "hybrid_reference_seed0.npz")


@pytest.fixture(scope="module")
def g():
    return dict(np.load(GOLD))


def _pb(g, d):
    return HybridPieceTensorBatch(
        token_features=torch.from_numpy(g["token_features"][..., :d]), token_q=torch.from_numpy(g["token_q"]).long(),
        token_r=torch.from_numpy(g["token_r"]).long(), token_z=torch.from_numpy(g["token_z"]).long(),
        token_mask=torch.from_numpy(g["token_mask"]).bool(), global_features=torch.from_numpy(g["global_features"]),
        num_tokens=torch.from_numpy(g["num_tokens"]))


@pytest.mark.parametrize("name,cfg", [("default", HybridGNNConfig), ("small", HybridGNNConfig.small)])
def test_hybrid_mirror_matches_reference(g, name, cfg):
    torch.manual_seed(0)
    net = HiveHybridGNN(cfg()).eval()
    h = hashlib.sha256()
    for n, p in net.named_parameters():
        h.update(n.encode())
        h.update(p.detach().float().contiguous().numpy().tobytes())
    assert h.hexdigest() == str(g[f"{name}/params_sha256"]), "parameter names, order or seeded init differ"
    assert net.count_parameters() == int(g[f"{name}/param_count"])
    n = g["num_legal"]
    valid = np.arange(256)[None, :] < n[:, None]
    pb = _pb(g, net.config.node_feat_dim)
    with torch.no_grad():
        logits, values = net(torch.from_numpy(g["root_features"]), torch.from_numpy(g["succ_features"]),
                             torch.from_numpy(g["succ_roots"]), torch.from_numpy(n.astype(np.int64)), pb,
                             torch.from_numpy(g["move_features"][valid]))
        gs = net.graph_trunk(pb)
    np.testing.assert_allclose(gs.numpy(), g[f"{name}/graph_summary"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(logits.numpy(), g[f"{name}/logits"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(values.numpy(), g[f"{name}/values"], rtol=1e-5, atol=1e-5)
