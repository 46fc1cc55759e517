"""Arena host logic on the CPU: the score tally (arena.py:1101-1151) and
loading checkpoints written by the reference (pickled config classes of
the reference's modules; fc1 padding, fnn_network.py:74-94; hybrid resize,
fnn_transformer_net.py:244-286)."""
import dataclasses
import sys
import types

import numpy as np
import torch

from hive_neuralnet_b200.arena import load_checkpoint, parse_wave_schedule, read_checkpoint, tally
from hive_neuralnet_b200.fnn import HiveFNN
from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridGNNConfig


def test_tally():
    res = np.array([1, 2, 3, 0, 1, 2])
    a_white = np.array([True, True, False, False, False, True])
    t = tally(res, a_white)
    # game 0: A white, white wins -> A; 1: A white, black wins -> B; 2: draw; 3: capped;
    # 4: A black, white wins -> B; 5: A white, black wins -> B
    assert t["white_wins"] == 1 and t["black_wins"] == 3 and t["draws"] == 2 and t["capped"] == 1
    assert t["model_a_score"] == 2.0 and t["white_score"] == 2.0
    assert t["model_a_white_games"] == 3 and t["model_a_white_score"] == 1.0
    assert t["model_a_black_games"] == 3 and t["model_a_black_score"] == 1.0


def test_wave_schedule():
    assert parse_wave_schedule("1, 2,4,,0") == [1, 2, 4, 1]
    assert parse_wave_schedule("") is None and parse_wave_schedule(None) is None


def _fake_reference_module(name, cls_name, fields):
    mod = types.ModuleType(name)
    cls = dataclasses.make_dataclass(cls_name, fields)
    cls.__module__ = name
    setattr(mod, cls_name, cls)
    return mod, cls


def _save_with_reference_class(tmp_path, module, cls_name, fields, values, state):
    parts = module.split(".")
    saved = {k: sys.modules.get(k) for k in (parts[0], module)}
    mod, cls = _fake_reference_module(module, cls_name, fields)
    sys.modules[parts[0]] = types.ModuleType(parts[0])
    sys.modules[module] = mod
    try:
        path = tmp_path / "ckpt.pt"
        torch.save({"net_config": cls(**values), "model_state_dict": state, "iteration": 7}, path)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return str(path)


def test_fnn_checkpoint_from_reference_pickle(tmp_path):
    torch.manual_seed(0)
    src = HiveFNN()
    state = src.state_dict()
    state["fc1.weight"] = state["fc1.weight"][:, :100].clone()  # an older, narrower feature width
    fields = [("feat_dim", int), ("hidden_dim", int), ("embed_dim", int), ("action_hidden", int)]
    path = _save_with_reference_class(tmp_path, "hive_fnn.fnn_network", "FNNConfig", fields,
                                      dict(feat_dim=100, hidden_dim=64, embed_dim=64, action_hidden=64), state)
    assert "hive_fnn.fnn_network" not in sys.modules
    ck = read_checkpoint(path)
    assert type(ck["net_config"]).__module__ == "hive_neuralnet_b200.fnn" and ck["iteration"] == 7
    net = load_checkpoint("fnn", path, device="cpu")
    w = net.fc1.weight.detach()
    assert w.shape == (64, 122)
    assert torch.equal(w[:, :100], state["fc1.weight"])
    assert float(w[:, 100:].abs().max()) < 0.01  # N(0, 1e-3) padding
    assert torch.equal(net.action_fc1.weight, src.action_fc1.weight)


def test_hybrid_checkpoint_resize(tmp_path):
    torch.manual_seed(1)
    small = HiveHybridGNN(HybridGNNConfig.small())
    state = small.state_dict()
    state["legacy.unused"] = torch.zeros(3)
    torch.manual_seed(2)
    big = HiveHybridGNN()
    before = {k: v.clone() for k, v in big.state_dict().items()}
    big.load_state_dict(state)
    after = big.state_dict()
    for key, t in after.items():
        if key not in state:
            assert torch.equal(t, before[key])
        elif state[key].shape == t.shape:
            assert torch.equal(t, state[key])
        else:
            ov = tuple(slice(0, min(a, b)) for a, b in zip(state[key].shape, t.shape))
            assert torch.equal(t[ov], state[key][ov].to(t.dtype))
