"""CPU tests: the HiveFNN mirror against the reference module's golden outputs."""
import os

import numpy as np
import pytest
import torch

from hive_neuralnet_b200 import _lib
from hive_neuralnet_b200.fnn import FNNConfig, HiveFNN, pack_weights

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fnn_reference_seed0.npz")


@pytest.mark.parametrize("preset,params", [("small", 1226), ("medium", 7202), ("large", 20546)])
def test_seeded_init_and_forward_match_reference(preset, params):
    g = np.load(GOLD)
    torch.manual_seed(0)
    net = HiveFNN(getattr(FNNConfig, preset)())
    assert net.count_parameters() == params == int(g[f"{preset}/params"])
    for k, v in net.state_dict().items():
        assert np.array_equal(v.numpy(), g[f"{preset}/{k}"]), k
    with torch.no_grad():
        logits, values = net(torch.from_numpy(g["in/root"]), torch.from_numpy(g["in/succ"]),
                             torch.from_numpy(g["in/action_to_root"]), None)
    assert np.array_equal(logits.numpy(), g[f"{preset}/out_logits"])
    assert np.array_equal(values.numpy(), g[f"{preset}/out_values"])


@pytest.mark.parametrize("preset", ["small", "medium", "large"])
def test_packed_size_matches_kernel(preset):
    if not os.path.exists(_lib.LIB_PATH):
        _lib.build()
    lib = _lib.load()
    net = HiveFNN(getattr(FNNConfig, preset)())
    w = pack_weights(net, "cpu")
    c = net.config
    assert w.numel() == lib.hv_fnn_weights_size(c.hidden_dim, c.embed_dim, c.action_hidden)
    assert w.numel() == net.count_parameters()
