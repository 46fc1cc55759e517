"""Arena / match evaluation (reference arena.py) on the kernels.

The Gumbel-root chooser's search replays bit-exact on the oracle's
sequential tree operations (root expansion, root-mask waves per halving
round, the recorded evaluator outputs); each halving keeps the best-scored
live slots; the chosen move is the most visited root child.  Whole matches
finish with a consistent tally and are deterministic given the seeds."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_orchestrator_gpu import _start, _tree_np

pytestmark = pytest.mark.gpu


def _root_scores(tree, B, legal_logits, c_visit, c_scale):
    fc, nc = tree.first_child[:, 0], tree.num_children[:, 0]
    visits = np.zeros((B, 256), np.int64)
    q = np.zeros((B, 256), np.float32)
    for i in range(B):
        if fc[i] < 0:
            continue
        n = int(nc[i])
        v = tree.visit_count[i, fc[i]:fc[i] + n]
        w = tree.total_value[i, fc[i]:fc[i] + n]
        visits[i, :n] = v
        q[i, :n] = np.where(v > 0, -w / np.maximum(v, 1).astype(np.float32), 0.0)
    sigma = np.float32((c_visit + visits.max()) * c_scale)
    return legal_logits + sigma * q, visits


@pytest.mark.parametrize("k,sims,wave", [(8, 48, 4), (16, 64, 8)])
def test_gumbel_chooser_replays_bit_exact_on_oracle(k, sims, wave):
    from hive_neuralnet_b200.arena import build_orchestrator, choose_fnn_moves
    from hive_neuralnet_b200.fnn import HiveFNN
    B, M = 8, 8192
    torch.manual_seed(0)
    orch, cfg = build_orchestrator("fnn", HiveFNN().cuda(), B, sims, k, True, wave, 7, 300, 1.0, 20, seed=3)
    cfg.max_tree_nodes = M
    orch._max_nodes = M
    orch.trace = []
    st = _start(B, 21)
    res = choose_fnn_moves(orch, torch.from_numpy(st).cuda(), np.ones(B, bool))
    tr = orch.trace
    root = next(x for x in tr if x["kind"] == "root")
    assert not root["any_win"]
    orc = O.oracle()
    tree = O.TreeArrays(B, M)
    nl = root["nl"].cpu().numpy()
    pri = root["priors"].cpu().numpy()
    ga = root["game_active"].cpu().numpy()
    O.mcts_expand_dense("orc", tree, root["child_q"].cpu().numpy(), np.where(ga != 0, 0, -1).astype(np.int32), st,
                        root["legal"].cpu().numpy(), nl, pri, st[:, 3415].astype(np.int32), with_backprop=False)
    valid = np.arange(256)[None, :] < nl[:, None]
    legal_logits = np.where(valid, np.log(np.maximum(pri, np.float32(1e-20))), np.float32(-1e30)).astype(np.float32)
    alive, rounds = None, 0
    for x in tr:
        if x["kind"] == "round":
            new = x["alive"].cpu().numpy().astype(bool)
            if alive is None:
                # the first top-k (no noise) spans the batch-wide k: every row's
                # min(nl, k) best priors, padded with slots past its legal moves
                max_k = min(k, int(nl.max()))
                assert (new.sum(1) == max_k).all() and ((new & valid).sum(1) == np.minimum(nl, max_k)).all()
                for i in range(B):
                    p = pri[i, :nl[i]]
                    if (new[i] & valid[i]).any() and not (new[i, :nl[i]]).all():
                        assert p[new[i, :nl[i]]].min() >= p[~new[i, :nl[i]]].max()
            else:
                assert not (new & ~valid).any()
                score, _ = _root_scores(tree, B, legal_logits, cfg.c_visit, cfg.c_scale)
                keep = max(1, int(alive.sum(1).max()) // 2)
                for i in range(B):
                    live = alive[i] & valid[i]
                    dropped, kept = live & ~new[i], live & new[i]
                    if dropped.any() and kept.any():
                        assert score[i, dropped].max() <= score[i, kept].min() + 1e-5 * abs(score[i, kept].min())
                    if live.sum() >= keep:
                        assert new[i].sum() == keep and not (new[i] & ~live).any()
            alive = new
            rounds += 1
        elif x["kind"] == "wave":
            leaf, paths, plen, vlp, vll = O.mcts_select("orc", tree, mode=1, game_active=ga,
                                                        root_nodes=np.zeros(B, np.int32),
                                                        alive_mask=alive.astype(np.int8), W=x["W"],
                                                        c_puct=cfg.c_puct)
            assert np.array_equal(leaf, x["leaf"].cpu().numpy())
            ls = O.mcts_replay("orc", st, paths, plen, leaf, B)
            lmv, lnl, _ = orc.legal_moves_features(ls)
            O.mcts_expand_dense("orc", tree, x["child_q"].cpu().numpy(), leaf, ls, lmv, lnl,
                                x["priors"].cpu().numpy(), ls[:, 3415].astype(np.int32), x["values"].cpu().numpy(),
                                vlp, vll)
    assert rounds == max(1, int(np.ceil(np.log2(max(min(k, int(nl.max())), 2)))))
    searched = next(x for x in tr if x["kind"] == "searched")
    assert _tree_np(searched["tree"], B, M).equal(tree) == []
    _, visits = _root_scores(tree, B, legal_logits, cfg.c_visit, cfg.c_scale)
    assert np.array_equal(res.chosen_slots, visits.argmax(axis=1))
    mv, _, _ = orc.legal_moves_features(st)
    assert np.array_equal(res.move_bytes, mv[np.arange(B), res.chosen_slots])


def _match(seed, stochastic):
    from hive_neuralnet_b200.arena import build_orchestrator, play_arena
    from hive_neuralnet_b200.fnn import FNNConfig, HiveFNN
    G = 6
    torch.manual_seed(seed)
    a = HiveFNN().cuda()
    b = HiveFNN(FNNConfig.medium()).cuda()
    wo, _ = build_orchestrator("fnn", a, G, 32, 8, True, 4, 7, 10, 1.0, 20, eval_mode=not stochastic, seed=seed)
    bo, _ = build_orchestrator("fnn", b, G, 32, 8, True, 8, 7, 10, 1.0, 20, use_puct=True,
                               eval_mode=not stochastic, seed=seed + 1)
    for o in (wo, bo):
        o._max_nodes = 4096
    st = torch.from_numpy(_start(G, 40 + seed)).cuda()
    return play_arena("fnn", wo, "fnn", bo, G, max_game_length=10, alternate_colors=True, stochastic=stochastic,
                      gumbel_noise_scale=0.1, start_states=st), st


@pytest.mark.parametrize("stochastic", [False, True])
def test_match_tally_and_determinism(stochastic):
    r1, st = _match(4, stochastic)
    r2, _ = _match(4, stochastic)
    assert np.array_equal(r1.final_results, r2.final_results)
    assert np.array_equal(r1.move_numbers, r2.move_numbers)
    assert set(np.unique(r1.final_results).tolist()) <= {0, 1, 2, 3}
    assert (r1.move_numbers <= 10).all() and (r1.move_numbers >= 1).all()
    assert (r1.final_results[r1.move_numbers < 10] != 0).all()
    assert r1.white_wins + r1.black_wins + r1.draws == 6
    assert r1.model_a_white_games + r1.model_a_black_games == 6
    assert abs(r1.model_a_score - (r1.model_a_white_score + r1.model_a_black_score)) < 1e-9
    assert r1.white_is_model_a.tolist() == [True, False] * 3


def test_policy_only_side_plays_the_prior_argmax():
    from hive_neuralnet_b200.arena import build_orchestrator, choose_fnn_policy_moves
    from hive_neuralnet_b200.fnn import HiveFNN
    B = 16
    torch.manual_seed(2)
    orch, _ = build_orchestrator("fnn", HiveFNN().cuda(), B, 8, 4, True, 4, 7, 300, 1.0, 20, seed=1)
    st = torch.from_numpy(_start(B, 8)).cuda()
    res = choose_fnn_policy_moves(orch, st, np.ones(B, bool))
    legal, nl, feats = orch.ext.generate_legal_moves_and_fnn_features_batch(st, B)
    pri, _, _ = orch._eval_states(st, legal, nl, B, feats)
    pri = pri.cpu().numpy()
    for i in range(B):
        assert res.chosen_slots[i] == int(np.argmax(pri[i, :int(nl[i])]))
