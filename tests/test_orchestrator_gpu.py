"""GPU tests of the self-play orchestrators.

The key check replays a recorded B200 search on the CPU oracle: the same
root expansion, the same candidate slots / alive masks and wave widths, and
the B200 evaluator's priors, values and child Q fed into the oracle's
sequential tree operations.  The resulting trees must be bit-identical, i.e.
visit counts are reproduced exactly given the evaluator outputs and the
Gumbel noise (drawn from a seeded Philox generator)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _start(B, seed, mask=7, max_ply=40):
    """In-progress positions past the opening with no immediately winning
    move (the reference PUCT driver skips the whole batch's search when any
    game has one, fnn_puct_orchestrator.py:203-208)."""
    orc = O.oracle()
    st = orc.generate_positions(seed, 0, 8 * B, max_ply, mask)
    mv, nl, _ = orc.legal_moves_features(st)
    keep = []
    for i in np.where((st[:, 3415] == 0) & (nl > 3) & (st[:, 3412] >= 8))[0]:
        kids = orc.apply_moves(np.repeat(st[i:i + 1], nl[i], 0), mv[i, :nl[i]])
        if (kids[:, 3415] == 0).all():
            keep.append(i)
        if len(keep) == B:
            break
    assert len(keep) == B
    return st[keep]


def _tree_np(tree_t, B, M):
    t = O.TreeArrays(B, M)
    names = ["visit_count", "total_value", "prior", "parent_idx", "virtual_q_penalty", "move_bytes", "action_idx",
             "first_child", "num_children", "is_terminal", "terminal_value", "node_count"]
    for a, n in zip(t.arrays(), names):
        a[...] = tree_t[n].cpu().numpy()
    t.child_init_q[...] = tree_t["child_init_q"].cpu().numpy()
    return t


def _replay(trace, B, M, mode, c_puct):
    orc = O.oracle()
    root = next(x for x in trace if x["kind"] == "root")
    st = root["states"].cpu().numpy()
    tree = O.TreeArrays(B, M)
    ga = root["game_active"].cpu().numpy()
    leaf0 = np.where(ga != 0, 0, -1).astype(np.int32)
    O.mcts_expand_dense("orc", tree, root["child_q"].cpu().numpy(), leaf0, st, root["legal"].cpu().numpy(),
                        root["nl"].cpu().numpy(), root["priors"].cpu().numpy(), st[:, 3415].astype(np.int32),
                        with_backprop=False)
    valid = (np.arange(256)[None, :] < root["nl"].cpu().numpy()[:, None]).astype(np.int8)
    for w in (x for x in trace if x["kind"] == "wave"):
        if mode == 2:
            slots = w["root_slots"].cpu().numpy()
            sel = O.mcts_select("orc", tree, mode=2, game_active=ga, root_nodes=np.zeros(B, np.int32),
                                root_slots=slots, num_candidates=slots.shape[1], W=w["W"], c_puct=c_puct)
        else:
            sel = O.mcts_select("orc", tree, mode=1, game_active=ga, root_nodes=np.zeros(B, np.int32),
                                alive_mask=valid, W=w["W"], c_puct=c_puct)
        leaf, paths, plen, vlp, vll = sel
        assert np.array_equal(leaf, w["leaf"].cpu().numpy())
        ls = O.mcts_replay("orc", st, paths, plen, leaf, B)
        lmv, lnl, _ = orc.legal_moves_features(ls)
        O.mcts_expand_dense("orc", tree, w["child_q"].cpu().numpy(), leaf, ls, lmv, lnl, w["priors"].cpu().numpy(),
                            ls[:, 3415].astype(np.int32), w["values"].cpu().numpy(), vlp, vll)
    return tree


@pytest.mark.parametrize("sims,reserve", [(64, 6), (96, 0)])
def test_gumbel_search_replays_bit_exact_on_oracle(sims, reserve):
    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.orchestrator import FNNMCTSConfig, FNNMCTSOrchestrator
    B, M = 12, 8192
    torch.manual_seed(0)
    cfg = FNNMCTSConfig(num_simulations=sims, batch_size=B, max_game_length=1, dirichlet_epsilon=0.0, seed=5,
                        max_tree_nodes=M, queen_surround_reserve_slots=reserve)
    orch = FNNMCTSOrchestrator(HiveFNN(), cfg)
    orch.trace = []
    ex = orch.self_play_batch(torch.from_numpy(_start(B, 3)).cuda())
    searched = next(x for x in orch.trace if x["kind"] == "searched")
    got = _tree_np(searched["tree"], B, M)
    want = _replay(orch.trace, B, M, 2, cfg.c_puct)
    assert got.equal(want) == []
    assert sum(len(e) for e in ex) == B
    for games in ex:
        for e in games:
            assert e.policy_target.shape == (len(e.policy_target),)
            assert abs(float(e.policy_target.sum()) - 1.0) < 1e-5


def test_puct_search_replays_bit_exact_on_oracle():
    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.orchestrator import FNNPUCTConfig, FNNPUCTOrchestrator
    B, M = 10, 8192
    torch.manual_seed(1)
    cfg = FNNPUCTConfig(num_simulations=48, batch_size=B, max_game_length=1, dirichlet_epsilon=0.0, seed=2,
                        max_tree_nodes=M, wave_size=16)
    orch = FNNPUCTOrchestrator(HiveFNN(), cfg)
    orch.trace = []
    orch.self_play_batch(torch.from_numpy(_start(B, 9)).cuda())
    searched = next(x for x in orch.trace if x["kind"] == "searched")
    assert _tree_np(searched["tree"], B, M).equal(_replay(orch.trace, B, M, 1, cfg.c_puct)) == []


def test_self_play_games_deterministic_with_seed():
    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.orchestrator import FNNMCTSConfig, FNNMCTSOrchestrator
    torch.manual_seed(0)
    net = HiveFNN()
    runs = []
    for _ in range(2):
        cfg = FNNMCTSConfig(num_simulations=32, batch_size=6, max_game_length=8, seed=11, max_tree_nodes=4096,
                            expansion_mask=7)
        runs.append(FNNMCTSOrchestrator(net, cfg).self_play_batch())
    for a, b in zip(*runs):
        assert len(a) == len(b) > 0
        for x, y in zip(a, b):
            assert np.array_equal(x.state_bytes, y.state_bytes)
            assert np.array_equal(x.policy_target, y.policy_target)
            assert x.value_target == y.value_target


def test_gumbel_with_short_forced_win_probe():
    """short_forced_win_probe=True (the trainer's default): rows the root
    tactical probe decides are not searched, a found win is played with a
    one-hot policy target, and the searched rows still replay bit-exact."""
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_tactical_golden as T
    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.orchestrator import FNNMCTSConfig, FNNMCTSOrchestrator
    import json
    orc = O.oracle()
    st, sel = T.tactical_inputs(orc)
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_tactical.json")) as f:
        case = json.load(f)["cases"]["111"]
    w_all, f_all = np.array(case["winning"]), np.array(case["forced"])
    rows = np.concatenate([np.where(w_all >= 0)[0][:6], np.where(f_all == 1)[0][:2],
                           np.where((w_all < 0) & (f_all == 0))[0][:8]])
    B, M = len(rows), 8192
    start = st[sel[rows]]
    torch.manual_seed(0)
    cfg = FNNMCTSConfig(num_simulations=64, batch_size=B, max_game_length=1, dirichlet_epsilon=0.0, seed=7,
                        max_tree_nodes=M, short_forced_win_probe=True, expansion_mask=7)
    orch = FNNMCTSOrchestrator(HiveFNN(), cfg)
    orch.trace = []
    ex = orch.self_play_batch(torch.from_numpy(start).cuda())
    root = next(x for x in orch.trace if x["kind"] == "root")
    mv, nl, _ = orc.legal_moves_features(start)
    win, _, forced = orc.tactical_probe(start, mv, nl, root["priors"].cpu().numpy())
    ga = root["game_active"].cpu().numpy()
    assert ((win >= 0) | (forced == 1)).any(), "fixture rows should include decided roots"
    assert np.array_equal(ga != 0, (win < 0) & (forced == 0) & (nl > 0))
    for b in range(B):
        if win[b] >= 0:
            (e,) = ex[b]
            assert e.policy_target[win[b]] == 1.0 and e.policy_target.sum() == 1.0
    if ga.any():
        searched = next(x for x in orch.trace if x["kind"] == "searched")
        assert _tree_np(searched["tree"], B, M).equal(_replay(orch.trace, B, M, 2, cfg.c_puct)) == []
