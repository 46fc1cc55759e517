"""Pin the Gumbel root driver to the REFERENCE's own code (run where the
reference tree exists; see oracle.reference_dir()).

Runs the reference's ``FNNMCTSOrchestrator.self_play_batch``
(hive_fnn/fnn_mcts_orchestrator.py:561-875) unmodified, on the CPU: the
orchestrator is built with ``__new__`` (as the reference's own
tests/test_gpu_training_logic.py builds its orchestrators) and given

* an extension object with the reference's binding names whose functions
  call the reference's own hive_gpu/csrc code compiled on the host
  (oracle/_ref/libhive_ref.so): move generation, features, apply / results,
  queen-escape flags, the root tactical probe, and the MCTS tree kernels run
  one simulation at a time in simulation-index order (the order the B200
  kernels define, since the reference's wave-parallel order is a race);
* the leaf evaluator of tests/hash_eval.py in place of ``_eval_states``
  (exact on any device, so the network cannot blur a decision);
* ``torch`` factory calls and ``.cuda()`` mapped to the CPU while it runs.

Each case uses the first seed whose search meets no immediate win: a win
anywhere in the batch zeroes every game's priors (:621-625), after which the
candidate top-k breaks ties, in an order that differs between CPU and CUDA.

Every ``torch.rand`` draw of the search (Gumbel uniforms, forced-random
moves) is recorded, so the B200 run can replay the same noise.  Recorded per
searched move: the candidate slots of every halving round and of the final
choice, the root children's visit counts, the improved-policy target; per
game the training examples (state bytes, policy target, value target,
flags).  Cases:

* ``full_schedule`` -- BASELINE config 4 at 64 games: 4,096 simulations,
  16 considered actions, the (2, 4, 8, 16) wave schedule, queen-surround
  reserve 6, 65,536-node trees (which fill: expansions past the pool revert,
  mcts_tree.cuh:1014-1020), one move;
* ``multi_move`` -- 16 games, 64 simulations, all expansions, the short
  forced-win probe on (wins, forced random moves, allowed-slot masks), up to
  8 moves per game with tree rebasing;
* ``gumbel_topk`` -- the reserve off (candidates by Gumbel top-k,
  :402-408), 16 games, 256 simulations, 3 moves, fixed policy-target
  temperature.

    python tests/golden/make_gumbel_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from tests.hash_eval import hash_eval  # noqa: E402
from tests.reference_cpu import reference_module, torch_on_cpu  # noqa: E402

R = reference_module("hive_fnn.fnn_mcts_orchestrator")  # the reference module

TREE_NAMES = [n for n, _, _ in O.TREE_FIELDS]

CASES = {
    "full_schedule": dict(games=64, seed=11, max_ply=30, mask=0,
                          cfg=dict(num_simulations=4096, batch_size=64, max_game_length=1, expansion_mask=0,
                                   dirichlet_epsilon=0.0, max_tree_nodes=65536)),
    "multi_move": dict(games=16, seed=12, max_ply=40, mask=7,
                       cfg=dict(num_simulations=64, batch_size=16, max_game_length=8, expansion_mask=7,
                                dirichlet_epsilon=0.0, max_tree_nodes=8192, short_forced_win_probe=True)),
    "gumbel_topk": dict(games=16, seed=13, max_ply=30, mask=7,
                        cfg=dict(num_simulations=256, batch_size=16, max_game_length=3, expansion_mask=7,
                                 dirichlet_epsilon=0.0, max_tree_nodes=16384, queen_surround_reserve_slots=0,
                                 adaptive_policy_target_temperature=False, policy_target_temperature=1.5)),
}


def start_states(lib, games, seed, max_ply, mask):
    """Seeded in-progress positions with at least one legal move."""
    st = lib.generate_positions(seed, 0, games * 4, max_ply, mask)
    _, nl, _ = lib.legal_moves_features(st)
    keep = np.where((st[:, 3415] == 0) & (nl > 0))[0][:games]
    assert len(keep) == games
    return st[keep]


def _tree(args, child_init_q):
    """The 12 tree tensors (binding order) as the oracle's TreeArrays, sharing memory."""
    t = O.TreeArrays.__new__(O.TreeArrays)
    t.B, t.max_nodes = args[0].shape
    for name, a in zip(TREE_NAMES, args):
        assert a.is_contiguous()
        setattr(t, name, a.numpy())
    t.child_init_q = child_init_q.numpy()
    return t


def _np(x):
    return x.contiguous().numpy()


class RefHostExt:
    """The reference extension's functions over CPU tensors, computed by the
    reference's own headers compiled on the host."""

    def __init__(self):
        self.lib = O.ref()

    def generate_legal_moves_and_fnn_features_batch(self, states, n):
        return tuple(torch.from_numpy(a) for a in self.lib.legal_moves_features(_np(states[:n])))

    def generate_legal_moves_batch(self, states, n):
        mv, nl, _ = self.lib.legal_moves_features(_np(states[:n]))
        return torch.from_numpy(mv), torch.from_numpy(nl)

    def apply_moves_batch(self, states, moves, n):
        states[:n].copy_(torch.from_numpy(self.lib.apply_moves(_np(states[:n]), _np(moves[:n]))))

    def check_results_batch(self, states, n):
        return states[:n, 3415].to(torch.int32).contiguous()

    def queen_escape_flags_batch(self, states, n):
        return torch.from_numpy(self.lib.queen_escape(_np(states[:n])))

    def root_tactical_probe_batch(self, states, legal, nl, priors, n, w1, chk, w2):
        win, allowed, forced = self.lib.tactical_probe(_np(states[:n]), _np(legal[:n]), _np(nl[:n]),
                                                       _np(priors[:n].float()), w1, chk, w2)
        return torch.from_numpy(win), torch.from_numpy(allowed), torch.from_numpy(forced)

    def mcts_expand_dense_priors_batch(self, *a):
        tree = _tree(a[:12], a[12])
        child_q, leaf, states, legal, nl, priors, results, B, total = a[13:22]
        O.mcts_expand_dense("ref", tree, _np(child_q), _np(leaf.to(torch.int32)), _np(states[:total]),
                            _np(legal), _np(nl), _np(priors), _np(results), with_backprop=False)

    def mcts_select_replay_legal_fnn_root_slots_batch(self, *a):
        tree = _tree(a[:12], a[12])
        root_states, game_active, root_nodes, root_slots, C, max_legal, c_puct, B, W = a[13:22]
        det = bool(a[23]) if len(a) > 23 else False
        sigma = float(a[24]) if len(a) > 24 else 4.0
        qpen = float(a[25]) if len(a) > 25 else 0.0
        leaf, paths, plen, vlp, vll = O.mcts_select(
            "ref", tree, mode=2, game_active=_np(game_active), root_nodes=_np(root_nodes),
            root_slots=_np(root_slots.to(torch.int32)), num_candidates=C, max_root_children=max_legal,
            c_puct=c_puct, W=W, det=det, sigma=sigma, q_penalty=qpen)
        ls = O.mcts_replay("ref", _np(root_states), paths, plen, leaf, B)
        mv, nl, ft = self.lib.legal_moves_features(ls)
        res = ls[:, 3415].astype(np.int32)
        return tuple(torch.from_numpy(x) for x in (leaf, ls, mv, nl, ft, res, vlp, vll))

    def mcts_expand_and_backprop_dense_priors_batch(self, *a):
        tree = _tree(a[:12], a[12])
        cq, leaf, leaf_states, legal, nl, pri, results, vals, vlp, vll, B, total, max_nodes, qpen = a[13:27]
        O.mcts_expand_dense("ref", tree, _np(cq), _np(leaf), _np(leaf_states), _np(legal), _np(nl), _np(pri),
                            _np(results), _np(vals), _np(vlp), _np(vll), q_penalty=float(qpen), with_backprop=True)

    def mcts_apply_root_noise(self, *a):
        tree = _tree(a[:12], torch.zeros(tuple(a[0].shape), dtype=torch.float32))
        noise, root_nodes, pad, eps, temp = a[12:17]
        O.mcts_root_noise("ref", tree, _np(noise), _np(root_nodes), float(eps), float(temp))


def run_reference(case: dict, start: np.ndarray, seed: int):
    cfg = R.FNNMCTSConfig(**case["cfg"])
    orch = R.FNNMCTSOrchestrator.__new__(R.FNNMCTSOrchestrator)
    orch.ext = RefHostExt()
    orch.config = cfg
    orch.net = None
    orch._move_size = 6
    orch._max_nodes = int(cfg.max_tree_nodes)
    orch._max_legal = 256
    orch._row_idx_cache = {}
    orch._keep_rank_cache = {}
    orch.last_policy_temperature_stats = {}
    draws, cands, visits, probs = [], [], [], []
    with torch_on_cpu([]):
        orch._slot_idx = torch.arange(256, dtype=torch.int64).unsqueeze(0)
        orch._neighbor_cells = orch._build_neighbor_cells()
    orch._eval_states = hash_eval
    cand_fn, child_fn, target_fn = (orch._gather_root_candidate_stats, orch._gather_root_child_stats,
                                    orch._build_policy_target)

    def cand_stats(tree, B, slots):
        cands.append(slots.numpy().astype(np.int32).copy())
        return cand_fn(tree, B, slots)

    def child_stats(tree, B):
        v, q = child_fn(tree, B)
        visits.append(v.numpy().copy())
        return v, q

    def target(logits, valid):
        p, t = target_fn(logits, valid)
        probs.append(p.numpy().copy())
        return p, t

    orch._gather_root_candidate_stats = cand_stats
    orch._gather_root_child_stats = child_stats
    orch._build_policy_target = target
    # an immediate win anywhere in the batch zeroes every game's priors
    # (fnn_mcts_orchestrator.py:621-625): the candidate top-k then breaks ties
    # among equal priors, and CPU and CUDA top-k break ties differently, so a
    # case is kept only if its search never meets one
    wins_seen = []
    imm_fn, tac_fn = orch._find_immediate_wins, orch._analyze_short_tactics

    def find_wins(*a, **k):
        w = imm_fn(*a, **k)
        wins_seen.append(bool((w >= 0).any()))
        return w

    def tactics(*a, **k):
        t = tac_fn(*a, **k)
        wins_seen.append(bool((t.winning_moves >= 0).any()))
        return t

    orch._find_immediate_wins = find_wins
    orch._analyze_short_tactics = tactics
    torch.manual_seed(seed)
    with torch_on_cpu(draws):
        examples = orch.self_play_batch(torch.from_numpy(start.copy()))
    ex_game, ex_state, ex_pi, ex_n, ex_val, ex_flags = [], [], [], [], [], []
    for g, games in enumerate(examples):
        for e in games:
            ex_game.append(g)
            ex_state.append(e.state_bytes)
            pi = np.zeros(256, np.float32)
            pi[:len(e.policy_target)] = e.policy_target
            ex_pi.append(pi)
            ex_n.append(len(e.policy_target))
            ex_val.append([e.value_target, e.value_weight])
            ex_flags.append([int(e.use_for_policy), int(e.use_for_value)])
    return dict(any_win=any(wins_seen), draws=draws, candidates=cands, visits=np.array(visits), probs=np.array(probs),
                ex_game=np.array(ex_game, np.int32), ex_state=np.array(ex_state, np.uint8),
                ex_policy=np.array(ex_pi, np.float32), ex_len=np.array(ex_n, np.int32),
                ex_value=np.array(ex_val, np.float32), ex_flags=np.array(ex_flags, np.int8))


def main() -> None:
    O.build(ref=True)
    if O.ref() is None:
        raise SystemExit("reference build unavailable: the reference tree is needed to make goldens")
    out = {}
    for name, case in CASES.items():
        for attempt in range(60):
            seed = case["seed"] + 1000 * attempt
            start = start_states(O.ref(), case["games"], seed, case["max_ply"], case["mask"])
            rec = run_reference(case, start, 1000 + seed)
            if not rec["any_win"]:
                break
        else:
            raise SystemExit(f"{name}: every seed met an immediate win")
        out[f"{name}/start"] = start
        out[f"{name}/cfg"] = np.array(repr(case["cfg"]))
        out[f"{name}/n_draws"] = np.array(len(rec["draws"]), np.int32)
        for i, d in enumerate(rec["draws"]):
            out[f"{name}/draw{i}"] = d
        out[f"{name}/n_cand"] = np.array(len(rec["candidates"]), np.int32)
        for i, c in enumerate(rec["candidates"]):
            out[f"{name}/cand{i}"] = c
        for k in ("visits", "probs", "ex_game", "ex_state", "ex_policy", "ex_len", "ex_value", "ex_flags"):
            out[f"{name}/{k}"] = rec[k]
        print(name, "moves searched", len(rec["visits"]), "examples", len(rec["ex_game"]),
              "draws", len(rec["draws"]), "candidate sets", len(rec["candidates"]),
              "max root visits", int(rec["visits"].max()) if len(rec["visits"]) else 0, flush=True)
    np.savez_compressed(os.path.join(HERE, "golden_gumbel.npz"), **out)


if __name__ == "__main__":
    main()
