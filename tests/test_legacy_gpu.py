"""Legacy action-space PUCT driver (hive_gpu/gpu_native_mcts.py) on the
kernels: its first search replays bit-exact on the oracle's sequential
action-space tree operations given the evaluator outputs and the Dirichlet
noise, and self-play produces legal moves with visit-share policy targets."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
A = 85834


def _evaluate(states, total):
    """A fixed, seeded stand-in for the archived action-space networks."""
    s = states[:total].float().sum(dim=1, keepdim=True) % 97.0
    a = torch.arange(A, device=states.device, dtype=torch.float32).unsqueeze(0)
    return torch.sin(0.0007 * a * (1.0 + s)) * 3.0, torch.tanh(s.squeeze(1) / 50.0 - 1.0)


def _run(seed, B=6, sims=40, W=8, games=2):
    from hive_neuralnet_b200.legacy import GPUMCTSConfig, GPUNativeMCTSOrchestrator
    cfg = GPUMCTSConfig(num_simulations=sims, batch_size=B, wave_size=W, max_game_length=games, seed=seed,
                        playout_cap_randomize=False, max_tree_nodes=8192, expansion_mask=7)
    orch = GPUNativeMCTSOrchestrator(_evaluate, cfg)
    orch.trace = []
    orc = O.oracle()
    st = orc.generate_positions(seed, 0, 4 * B, 30, 7)
    st = st[st[:, 3415] == 0][:B]
    return orch, st, orch.self_play_batch(torch.from_numpy(st).cuda())


def test_first_search_replays_bit_exact_on_oracle():
    orch, st, _ = _run(5)
    B, M = len(st), orch._max_nodes
    orc = O.oracle()
    root = next(x for x in orch.trace if x["kind"] == "root")
    noise = next(x for x in orch.trace if x["kind"] == "noise")["noise"].cpu().numpy()
    tree = O.TreeArrays(B, M)
    mv, nl, _ = orc.legal_moves_features(st)
    O.mcts_expand_action("orc", tree, 0, np.zeros(B, np.int32), st, mv, nl, root["probs"].cpu().numpy(),
                         root["results"].cpu().numpy())
    O.mcts_root_noise("orc", tree, noise, np.zeros(B, np.int32), orch.config.dirichlet_epsilon,
                      orch.config.root_policy_temp)
    for w in orch.trace:
        if w["kind"] == "searched":
            break  # the waves of the first move only
        if w["kind"] != "wave":
            continue
        leaf, paths, plen, vlp, vll = O.mcts_select("orc", tree, mode=0, game_active=np.ones(B, np.int8),
                                                    root_nodes=np.zeros(B, np.int32), W=w["W"],
                                                    c_puct=orch.config.c_puct)
        assert np.array_equal(leaf, w["leaf"].cpu().numpy())
        ls = O.mcts_replay("orc", st, paths, plen, leaf, B)
        lmv, lnl, _ = orc.legal_moves_features(ls)
        O.mcts_expand_action("orc", tree, 1, leaf, ls, lmv, lnl, w["probs"].cpu().numpy(),
                             ls[:, 3415].astype(np.int32), w["values"].cpu().numpy(), vlp, vll)
    searched = next(x for x in orch.trace if x["kind"] == "searched")["tree"]
    names = ["visit_count", "total_value", "prior", "parent_idx", "virtual_q_penalty", "move_bytes",
             "action_idx", "first_child", "num_children", "is_terminal", "terminal_value", "node_count"]
    got = O.TreeArrays(B, M)
    for a, n in zip(got.arrays(), names):
        a[...] = searched[n].cpu().numpy()
    # root priors pass through powf(p, 1 / root_policy_temp), whose last ulp
    # differs between CUDA and libm: compared at 1e-6, everything else bit-exact
    assert [d for d in got.equal(tree) if d != "prior"] == []
    np.testing.assert_allclose(got.prior, tree.prior, rtol=1e-6, atol=1e-9)


def test_self_play_moves_are_legal_and_targets_are_visit_shares():
    orch, st, ex = _run(9, games=3)
    orc = O.oracle()
    for games in ex:
        for e in games:
            mv, nl, _ = orc.legal_moves_features(e.state_bytes[None])
            acts, _ = orc.actions(e.state_bytes[None], mv, nl)
            legal_actions = set(int(a) for a in acts[0, :nl[0]] if a >= 0)
            support = set(np.nonzero(e.policy_target)[0].tolist())
            assert support and support <= legal_actions
            # mcts_extract_policy_kernel (mcts_tree.cuh:643-680) normalises by the sum
            # over all root children but writes by action index: children that share
            # an action (duplicate moves with expansions on) leave the sum below 1
            assert (e.policy_target >= 0).all() and 0.0 < float(e.policy_target.sum()) <= 1.0 + 1e-4
            assert e.value_target in (-1.0, 0.0, 1.0)
    assert sum(len(g) for g in ex) > len(st)
