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


# ---------------------------------------------------------------------------
# one-ply Gumbel driver (hive_gpu/gumbel_mcts.py)
# ---------------------------------------------------------------------------
def _np_softmax(x):
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp((x - m).astype(np.float64))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def _gumbel_replay(orch, st, k, sims):
    """The search restated in numpy over oracle move generation, action
    lookup and move application, fed with the driver's recorded network
    outputs (looked up by state bytes) and Gumbel draws."""
    cfg, orc, B = orch.config, O.oracle(), len(st)
    evals = {}
    for x in orch.trace:
        if x["kind"] == "eval":
            s, lg, v = x["states"].cpu().numpy(), x["logits"].cpu().numpy(), x["values"].cpu().numpy()
            for j in range(len(s)):
                evals[s[j].tobytes()] = (lg[j], v[j])

    def nn(state):
        return evals[state.tobytes()]  # KeyError: the driver never evaluated this state

    def legal_info(states):
        mv, nl, _ = orc.legal_moves_features(states)
        acts, _ = orc.actions(states, mv, nl)
        acts = np.where(np.arange(256)[None, :] < nl[:, None], acts, -1)
        mask = np.zeros((len(states), A), bool)
        for i in range(len(states)):
            a = acts[i, :nl[i]]
            mask[i, a[a >= 0]] = True
        return mv, nl, acts, mask

    mv, nl, acts, mask = legal_info(st)
    g = next(x for x in orch.trace if x["kind"] == "gumbel")["gumbel"].cpu().numpy()
    logits = np.stack([np.where(mask[i], nn(st[i])[0], -np.inf).astype(np.float32) for i in range(B)])
    root_v = np.array([nn(st[i])[1] for i in range(B)], np.float32)
    perturbed = (g + logits).astype(np.float32)
    n_legal = mask.sum(1)
    max_k = min(k, int(n_legal.max()))
    eff = np.minimum(n_legal, k)
    gpu = next(x for x in orch.trace if x["kind"] == "searched")
    topk = gpu["topk"].cpu().numpy()
    for i in range(B):
        want = np.argsort(-perturbed[i], kind="stable")[:eff[i]]
        assert np.array_equal(topk[i, :eff[i]], want)
    cand = np.arange(max_k)[None, :] < eff[:, None]
    q_sums = np.zeros((B, max_k), np.float32)
    visits_n = np.zeros((B, max_k), np.int32)
    remaining = np.full(B, sims, np.int32)
    rounds = max(1, int(np.ceil(np.log2(int(cand.sum(1).max())))))
    for r in range(rounds):
        n_rem = cand.sum(1).astype(np.int32)
        if n_rem.max() == 0:
            break
        vis = np.where(n_rem > 0, np.maximum(remaining // np.maximum(n_rem, 1), 1), 0).astype(np.int32)
        cv = np.zeros((B, max_k), np.float32)
        for i, j in zip(*np.nonzero(cand)):
            hit = np.nonzero(acts[i, :nl[i]] == topk[i, j])[0]
            if hit.size == 0:
                continue
            child = orc.apply_moves(st[i:i + 1], mv[i, hit[0]:hit[0] + 1])
            res = int(child[0, 3415])
            clog, cval = nn(child[0])
            if res != 0:
                root_white = int(st[i, 3412]) % 2 == 0
                won = (res == 1 and root_white) or (res == 2 and not root_white)
                cval = np.float32(0.0 if res == 3 else (-1.0 if won else 1.0))
            val = -np.float32(cval)
            if vis.max() > 1 and res == 0 and vis[i] - 1 > 0:
                cmv, cnl, cacts, cmask = legal_info(child)
                if cnl[0] > 0:
                    ml = np.where(cmask[0], clog, -np.inf).astype(np.float32)
                    sc = np.where(cacts[0] >= 0, ml[np.maximum(cacts[0], 0)], -np.inf)
                    best = int(np.argmax(sc))
                    if np.isfinite(sc[best]):
                        gc = orc.apply_moves(child, cmv[0, best:best + 1])
                        gres = int(gc[0, 3415])
                        gval = np.float32(nn(gc[0])[1])
                        if gres != 0:
                            rw = int(child[0, 3412]) % 2 == 1
                            won = (gres == 1 and rw) or (gres == 2 and not rw)
                            gval = np.float32(0.0 if gres == 3 else (1.0 if won else -1.0))
                        val = gval
            cv[i, j] = val
        q_sums += (cv * vis[:, None].astype(np.float32)) * cand.astype(np.float32)
        visits_n += vis[:, None] * cand.astype(np.int32)
        remaining = np.maximum(remaining - vis * n_rem, 0)
        if r < rounds - 1:
            max_n = np.maximum(visits_n.max(1, keepdims=True).astype(np.float32), 1)
            q_mean = np.where(visits_n > 0, q_sums / np.maximum(visits_n, 1).astype(np.float32), 0).astype(np.float32)
            qt = (np.float32(cfg.c_visit) + max_n) * np.float32(cfg.c_scale) * q_mean
            tk = topk[:, :max_k]
            sigma = (np.take_along_axis(g, tk, 1) + np.take_along_axis(logits, tk, 1) + qt).astype(np.float32)
            sigma = np.where(cand, sigma, -np.inf)
            keep = np.maximum(np.ceil(n_rem / 2).astype(np.int32), 1)
            new = np.zeros_like(cand)
            for i in range(B):
                order = np.argsort(-sigma[i], kind="stable")
                new[i, order[:keep[i]]] = True
            cand = new & cand
    return topk, q_sums, visits_n, cand, logits, root_v


def test_gumbel_one_ply_search_replays_on_oracle():
    from hive_neuralnet_b200.legacy import GumbelAlphaZeroOrchestrator, GumbelConfig
    B, k, sims = 5, 8, 16
    cfg = GumbelConfig(num_simulations=sims, max_num_considered_actions=k, batch_size=B, max_game_length=1,
                       seed=11, expansion_mask=7)
    orch = GumbelAlphaZeroOrchestrator(_evaluate, cfg)
    orch.trace = []
    orc = O.oracle()
    st = orc.generate_positions(12, 0, 4 * B, 30, 7)
    st = st[st[:, 3415] == 0][:B]
    ex = orch.self_play_batch(torch.from_numpy(st).cuda())
    topk, q_sums, visits, cand, logits, root_v = _gumbel_replay(orch, st, k, sims)
    gpu = next(x for x in orch.trace if x["kind"] == "searched")
    assert np.array_equal(gpu["visits"].cpu().numpy(), visits)
    assert np.array_equal(gpu["candidates"].cpu().numpy(), cand)
    np.testing.assert_allclose(gpu["q_sums"].cpu().numpy(), q_sums, rtol=1e-6, atol=1e-6)
    # improved policy: softmax over the candidates of logit + sigma(completed Q)
    max_n = np.maximum(visits.max(1, keepdims=True).astype(np.float32), 1)
    q = np.where(visits > 0, q_sums / np.maximum(visits, 1), -root_v[:, None]).astype(np.float32)
    want = _np_softmax(np.take_along_axis(logits, topk, 1) + (50.0 + max_n) * q)
    for i, (acts, probs) in enumerate(gpu["policies"]):
        np.testing.assert_allclose(probs, np.nan_to_num(want[i]), rtol=1e-5, atol=1e-7)
    for i, games in enumerate(ex):
        (e,) = games
        assert np.array_equal(e.state_bytes, st[i])
        mv, nl, _ = orc.legal_moves_features(st[i:i + 1])
        a, _ = orc.actions(st[i:i + 1], mv, nl)
        legal = set(int(x) for x in a[0, :nl[0]] if x >= 0)
        support = set(np.nonzero(e.policy_target)[0].tolist())
        assert legal <= support  # every legal action carries at least the 1e-4 floor
        assert e.value_target in (-1.0, 0.0, 1.0)


def test_gumbel_match_plays_to_the_end():
    from hive_neuralnet_b200.legacy import gumbel_match

    def other(states, total):
        lg, v = _evaluate(states, total)
        return -lg, -v

    orc = O.oracle()
    st = orc.generate_positions(3, 0, 40, 30, 7)
    st = torch.from_numpy(st[st[:, 3415] == 0][:6]).cuda()
    r1 = gumbel_match(_evaluate, other, 6, 8, 4, max_moves=6, expansion_mask=7, seed=1, start_states=st)
    r2 = gumbel_match(_evaluate, other, 6, 8, 4, max_moves=6, expansion_mask=7, seed=1, start_states=st)
    assert np.array_equal(r1["results"], r2["results"]) and np.array_equal(r1["move_numbers"], r2["move_numbers"])
    assert (r1["move_numbers"] <= 6).all() and ((r1["move_numbers"] == 6) | (r1["results"] != 0)).all()
    assert 0.0 <= r1["a_score"] <= 6.0 and r1["a_is_white"].tolist() == [True] * 3 + [False] * 3
