"""GPU parity of the Gumbel root driver against the reference's OWN driver
code (tests/golden/make_gumbel_golden.py ran the reference's
FNNMCTSOrchestrator.self_play_batch on the CPU over the reference's
compiled game logic and tree kernels and recorded its decisions).

The B200 orchestrator replays the same searches: same start positions and
config, the same leaf evaluator (tests/hash_eval.py, exact on any device)
and the reference run's recorded torch.rand draws.  Compared, per searched
move: the candidate slots of every sequential-halving round and of the final
choice (_root_candidate_slots, fnn_mcts_orchestrator.py:384-444, and the
halving loop, :670-731), the root children's visit counts, the improved-policy
target (_build_policy_target, :144-191, :733-748); and the training examples
of every game (state bytes = the chosen moves, policy and value targets,
flags).  Counts and slots bit-exact; policy targets within 1e-6 (softmax and
log on two devices)."""
import ast
import os

import numpy as np
import pytest
import torch

from tests.hash_eval import hash_eval

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(os.path.join(GOLD, "golden_gumbel.npz")))


@pytest.mark.parametrize("name", ["full_schedule", "multi_move", "gumbel_topk"])
def test_gumbel_driver_matches_reference_driver(gold, name):
    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.orchestrator import FNNMCTSConfig, FNNMCTSOrchestrator
    cfg = FNNMCTSConfig(**ast.literal_eval(str(gold[f"{name}/cfg"])))
    orch = FNNMCTSOrchestrator(HiveFNN(), cfg)
    dev = orch.device
    draws = [gold[f"{name}/draw{i}"] for i in range(int(gold[f"{name}/n_draws"]))]
    used = []

    def uniform(*shape):
        d = draws[len(used)]
        assert tuple(d.shape) == tuple(shape), (d.shape, shape)
        used.append(d)
        return torch.from_numpy(d).to(dev)

    cands, visits, probs = [], [], []
    root_stats, build_target = orch._root_stats, orch._build_policy_target

    def stats(tree, B, slots, min_visits):
        v, q = root_stats(tree, B, slots, min_visits)
        if slots.shape[1] == 256:
            visits.append(v.cpu().numpy())
        else:
            cands.append(slots.to(torch.int32).cpu().numpy())
        return v, q

    def target(logits, valid):
        p, t = build_target(logits, valid)
        probs.append(p.cpu().numpy())
        return p, t

    orch._uniform = uniform
    orch._eval_states = hash_eval
    orch._root_stats = stats
    orch._build_policy_target = target
    examples = orch.self_play_batch(torch.from_numpy(gold[f"{name}/start"]).to(dev))

    assert len(used) == len(draws)
    n_cand = int(gold[f"{name}/n_cand"])
    assert len(cands) == n_cand
    for i in range(n_cand):
        assert np.array_equal(cands[i], gold[f"{name}/cand{i}"]), f"candidate set {i} differs"
    assert np.array_equal(np.array(visits), gold[f"{name}/visits"])
    np.testing.assert_allclose(np.array(probs), gold[f"{name}/probs"], rtol=0, atol=1e-6)

    flat = [(g, e) for g, games in enumerate(examples) for e in games]
    assert len(flat) == len(gold[f"{name}/ex_game"])
    for k, (g, e) in enumerate(flat):
        assert g == gold[f"{name}/ex_game"][k]
        assert np.array_equal(e.state_bytes, gold[f"{name}/ex_state"][k]), f"example {k}: position differs"
        n = int(gold[f"{name}/ex_len"][k])
        assert len(e.policy_target) == n
        np.testing.assert_allclose(e.policy_target, gold[f"{name}/ex_policy"][k, :n], rtol=0, atol=1e-6)
        assert [e.value_target, e.value_weight] == gold[f"{name}/ex_value"][k].tolist()
        assert [int(e.use_for_policy), int(e.use_for_value)] == gold[f"{name}/ex_flags"][k].tolist()
