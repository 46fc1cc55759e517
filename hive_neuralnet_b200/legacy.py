"""Legacy action-space search driver (hive_gpu/gpu_native_mcts.py).

``GPUNativeMCTSOrchestrator`` keeps the reference driver's search: PUCT
waves over the 85,834-wide action space (select with virtual loss, replay,
dense legal mask, masked softmax of the network's action logits, fused
expand + backup), tree reuse across moves (the chosen child becomes the
root), shaped Dirichlet noise with a root policy temperature, visit-count
policy targets with pruning, the immediate-win override and playout-cap
randomisation -- all on this build's kernels.

The reference driver feeds its network through the archived GNN /
transformer encoders (``encode_states_batch`` / ``hybrid_gnn_*``) and
records mobility and queen-surround targets (``compute_mobility_batch``);
those encoders and targets are outside the self-play hot path.  Here the
network is a callable ``evaluate(states, total) -> (policy_logits [T, 85834],
values [T])`` on device tensors, and an example is (state bytes, policy
target over the action space, value target, network prior of the root).
The reference passes 11 tree tensors to the 12-tensor bindings
(gpu_native_mcts.py:103-110 vs bindings.cpp:130-135); this driver passes
the 12 in binding order.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass
from typing import Callable, NamedTuple

import numpy as np
import torch

from .hive_gpu import ACTION_SPACE_SIZE, SIZEOF_GPU_MOVE, load_extension


@dataclass
class GPUMCTSConfig:
    """The fields of the reference's GPUMCTSConfig that the search uses
    (archive/modules/hive_gpu_hybrid/gpu_mcts.py:38-73), plus ``seed`` and
    ``max_tree_nodes``."""

    num_simulations: int = 100
    c_puct: float = 1.5
    dirichlet_alpha: float = 0.3
    dirichlet_epsilon: float = 0.25
    temperature: float = 1.0
    temperature_drop_move: int = 20
    batch_size: int = 64
    max_game_length: int = 300
    expansion_mask: int = 0
    wave_size: int = 8
    playout_cap_randomize: bool = True
    playout_cap_randomize_prob: float = 0.25
    playout_cap_fast_sims: int = 0
    policy_target_pruning: float = 0.02
    root_policy_temp: float = 1.1
    shaped_dirichlet: bool = True
    max_tree_nodes: int = 65536
    seed: int | None = None


class ActionSpaceExample(NamedTuple):
    state_bytes: np.ndarray      # [3424] u8, the searched root
    policy_target: np.ndarray    # [85834] f32, visit distribution (pruned)
    value_target: float          # +1 / -1 / 0 from the root player's view
    nn_prior: np.ndarray | None  # [85834] f32, the network's root prior before noise


Evaluator = Callable[[torch.Tensor, int], "tuple[torch.Tensor, torch.Tensor]"]


class GPUNativeMCTSOrchestrator:
    """Action-space PUCT self-play with tree reuse (gpu_native_mcts.py:35-886)."""

    def __init__(self, evaluate: Evaluator, config: GPUMCTSConfig | None = None, device: str = "cuda") -> None:
        self.ext = load_extension()
        self.evaluate = evaluate
        self.config = config or GPUMCTSConfig()
        self.device = torch.device(device)
        self.rng = np.random.default_rng(self.config.seed)
        self._max_nodes = int(self.config.max_tree_nodes)
        self.trace: list | None = None  # set to a list to record the first move's search

    # -- tree -----------------------------------------------------------------
    def _alloc_tree(self, B: int) -> dict[str, torch.Tensor]:
        M, dev = self._max_nodes, self.device
        return {
            "visit_count": torch.zeros(B, M, dtype=torch.int32, device=dev),
            "total_value": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "prior": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "parent_idx": torch.full((B, M), -1, dtype=torch.int32, device=dev),
            "virtual_q_penalty": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "move_bytes": torch.zeros(B, M, SIZEOF_GPU_MOVE, dtype=torch.uint8, device=dev),
            "action_idx": torch.full((B, M), -1, dtype=torch.int32, device=dev),
            "first_child": torch.full((B, M), -1, dtype=torch.int32, device=dev),
            "num_children": torch.zeros(B, M, dtype=torch.int32, device=dev),
            "is_terminal": torch.zeros(B, M, dtype=torch.int8, device=dev),
            "terminal_value": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "node_count": torch.ones(B, dtype=torch.int32, device=dev),
            "root_node": torch.zeros(B, dtype=torch.int32, device=dev),
        }

    @staticmethod
    def _tree_args(tree):
        return [tree[k] for k in ("visit_count", "total_value", "prior", "parent_idx", "virtual_q_penalty",
                                  "move_bytes", "action_idx", "first_child", "num_children", "is_terminal",
                                  "terminal_value", "node_count")]

    def _probs(self, states: torch.Tensor, total: int, masks: torch.Tensor):
        logits, values = self.evaluate(states, total)
        logits = logits.float().masked_fill(masks == 0, float("-inf"))
        return torch.softmax(logits, dim=-1), values.float().reshape(-1)

    # -- per move ---------------------------------------------------------------
    def _root_children(self, tree, B):
        row = torch.arange(B, device=self.device)
        rn = tree["root_node"].long()
        return tree["first_child"][row, rn].cpu().numpy(), tree["num_children"][row, rn].cpu().numpy()

    def _expand_roots(self, states, B, tree, active):
        """gpu_native_mcts.py:374-448: network on the roots, expand, record priors."""
        results = self.ext.check_results_batch(states, B)
        legal, nl, masks = self.ext.generate_legal_moves_and_mask_batch(states, B)
        probs, _ = self._probs(states, B, masks)
        if self.trace is not None:
            self.trace.append(dict(kind="root", states=states.clone(), probs=probs.clone(), results=results.clone()))
        self.ext.mcts_expand_batch(*self._tree_args(tree), torch.zeros(B, dtype=torch.int32, device=self.device),
                                   states, legal, nl, probs, results, B, B, self._max_nodes)
        return self._priors_from_tree(tree, B, active)

    def _priors_from_tree(self, tree, B, active):
        """gpu_native_mcts.py:507-538: the stored (noise-free) priors of the root's children."""
        fc, nc = self._root_children(tree, B)
        ai, pr = tree["action_idx"].cpu().numpy(), tree["prior"].cpu().numpy()
        out = [None] * B
        for i in range(B):
            if not active[i] or fc[i] < 0 or nc[i] == 0:
                continue
            p = np.zeros(ACTION_SPACE_SIZE, np.float32)
            a = ai[i, fc[i]:fc[i] + nc[i]]
            ok = (a >= 0) & (a < ACTION_SPACE_SIZE)
            p[a[ok]] = pr[i, fc[i]:fc[i] + nc[i]][ok]
            out[i] = p
        return out

    def _root_noise(self, tree, B, active):
        """gpu_native_mcts.py:450-484: shaped Dirichlet noise and root policy temperature."""
        cfg = self.config
        _, nc = self._root_children(tree, B)
        pad = max(int(nc.max()), 1)
        noise = np.zeros((B, pad), np.float32)
        for i in range(B):
            n = int(nc[i])
            if n == 0 or not active[i]:
                continue
            alpha = max(0.03, 10.0 / n) if cfg.shaped_dirichlet else cfg.dirichlet_alpha
            noise[i, :n] = self.rng.dirichlet([alpha] * n)
        noise_t = torch.from_numpy(noise).to(self.device)
        self.ext.mcts_apply_root_noise(*self._tree_args(tree), noise_t, tree["root_node"], pad,
                                       cfg.dirichlet_epsilon, cfg.root_policy_temp, B, self._max_nodes)
        return noise_t

    def _search(self, states, B, active, move_numbers, tree, num_sims):
        """gpu_native_mcts.py:259-371: waves of select / replay / evaluate / expand + backup."""
        cfg = self.config
        game_active = torch.tensor([1 if a else 0 for a in active], dtype=torch.int8, device=self.device)
        W = cfg.wave_size
        leaf_states = torch.zeros(W * B, states.shape[1], dtype=torch.uint8, device=self.device)
        for wave in range(math.ceil(num_sims / W)):
            w = min(W, num_sims - wave * W)
            total = w * B
            leaf, paths, plen, vlp, vll = self.ext.mcts_select_batch(*self._tree_args(tree), game_active,
                                                                     tree["root_node"], cfg.c_puct, B, w,
                                                                     self._max_nodes)
            ls = leaf_states[:total]
            self.ext.mcts_replay_batch(states, ls, paths, plen, leaf, B, total)
            results = self.ext.check_results_batch(ls, total)
            legal, nl, masks = self.ext.generate_legal_moves_and_mask_batch(ls, total)
            probs, values = self._probs(ls, total, masks)
            if self.trace is not None:
                self.trace.append(dict(kind="wave", W=w, leaf=leaf.clone(), probs=probs.clone(),
                                       values=values.clone()))
            self.ext.mcts_expand_and_backprop_batch(*self._tree_args(tree), leaf, ls, legal, nl, probs, results,
                                                    values, vlp, vll, B, total, self._max_nodes)
        mn = torch.tensor(move_numbers, dtype=torch.int32, device=self.device)
        return self.ext.mcts_extract_policy_batch(*self._tree_args(tree), mn, tree["root_node"], cfg.temperature,
                                                  cfg.temperature_drop_move, cfg.policy_target_pruning, B,
                                                  self._max_nodes).cpu().numpy()

    def _immediate_wins(self, states, B, active, turns, tree, policies):
        """gpu_native_mcts.py:569-653: a root child whose move wins at once takes the whole policy."""
        fc, nc = self._root_children(tree, B)
        games, kids = [], []
        for i in range(B):
            if active[i] and fc[i] >= 0 and nc[i] > 0:
                games += [i] * int(nc[i])
                kids += list(range(int(fc[i]), int(fc[i] + nc[i])))
        if not games:
            return
        g = torch.tensor(games, dtype=torch.int64, device=self.device)
        k = torch.tensor(kids, dtype=torch.int64, device=self.device)
        test = states[g].clone()
        self.ext.apply_moves_batch(test, tree["move_bytes"][g, k].contiguous(), len(games))
        res = self.ext.check_results_batch(test, len(games)).cpu().numpy()
        acts = tree["action_idx"][g, k].cpu().numpy()
        done = set()
        for j, i in enumerate(games):
            if i in done or res[j] == 0:
                continue
            if res[j] == (1 if turns[i] % 2 == 0 else 2) and 0 <= acts[j] < ACTION_SPACE_SIZE:
                policies[i][:] = 0.0
                policies[i][acts[j]] = 1.0
                done.add(i)

    def _move_for_action(self, tree, states, i, action):
        """gpu_native_mcts.py:655-702: the root child with this action (or a legal fallback)."""
        rn = int(tree["root_node"][i])
        fc, nc = int(tree["first_child"][i, rn]), int(tree["num_children"][i, rn])
        if fc >= 0 and nc > 0:
            ai = tree["action_idx"][i, fc:fc + nc].cpu().numpy()
            hit = np.nonzero(ai == action)[0]
            if hit.size:
                return tree["move_bytes"][i, fc + hit[0]].cpu().numpy(), fc + int(hit[0])
        legal, nl = self.ext.generate_legal_moves_batch(states[i:i + 1].contiguous(), 1)
        n = int(nl[0])
        if n == 0:
            return None, -1
        acts = self.ext.legal_moves_to_actions_batch(states[i:i + 1].contiguous(), legal, nl, 1)[0, :n].cpu().numpy()
        hit = np.nonzero(acts == action)[0]
        return legal[0, int(hit[0]) if hit.size else 0].cpu().numpy(), -1

    def self_play_batch(self, start_states: torch.Tensor | None = None) -> list[list[ActionSpaceExample]]:
        """gpu_native_mcts.py:114-257."""
        cfg = self.config
        B = cfg.batch_size
        states = (start_states.to(self.device).contiguous().clone() if start_states is not None
                  else self.ext.create_initial_states(B, cfg.expansion_mask))
        tree = self._alloc_tree(B)
        active = [True] * B
        move_numbers = [0] * B
        histories: list[list[tuple]] = [[] for _ in range(B)]
        first = True
        while any(active):
            sh = states.cpu().numpy()
            turns = [int(sh[i, 3412]) | (int(sh[i, 3413]) << 8) for i in range(B)]
            if cfg.playout_cap_randomize:
                use_full = self.rng.random() < cfg.playout_cap_randomize_prob
                sims = cfg.num_simulations if use_full else (cfg.playout_cap_fast_sims or
                                                             max(1, cfg.num_simulations // 8))
            else:
                use_full, sims = True, cfg.num_simulations
            if first:
                nn_priors = self._expand_roots(states, B, tree, active)
            else:
                nn_priors = self._priors_from_tree(tree, B, active)
            noise = self._root_noise(tree, B, active)
            if self.trace is not None and first:
                self.trace.append(dict(kind="noise", noise=noise.clone()))
            first = False
            policies = self._search(states, B, active, move_numbers, tree, sims)
            if self.trace is not None and len([x for x in self.trace if x["kind"] == "searched"]) == 0:
                self.trace.append(dict(kind="searched", tree={k: v.clone() for k, v in tree.items()},
                                       policies=policies.copy()))
            self._immediate_wins(states, B, active, turns, tree, policies)
            moves = np.zeros((B, SIZEOF_GPU_MOVE), np.uint8)
            chosen = [-1] * B
            for i in range(B):
                if not active[i]:
                    continue
                pol = policies[i]
                if use_full:
                    histories[i].append((sh[i].copy(), pol.copy(), turns[i], nn_priors[i]))
                if move_numbers[i] >= cfg.temperature_drop_move:
                    action = int(np.argmax(pol))
                else:
                    s = pol.sum()
                    p = pol / s if (s > 0 and np.isfinite(s)) else np.full(pol.shape, 1.0 / pol.size)
                    action = int(self.rng.choice(pol.size, p=p))
                mb, child = self._move_for_action(tree, states, i, action)
                chosen[i] = child
                if mb is not None:
                    moves[i] = mb
            # re-root at the chosen children (gpu_native_mcts.py:540-567)
            new_roots = tree["root_node"].clone()
            for i in range(B):
                if active[i] and chosen[i] >= 0:
                    new_roots[i] = chosen[i]
            tree["root_node"].copy_(new_roots)
            tree["parent_idx"].scatter_(1, new_roots.long().unsqueeze(1),
                                        torch.full((B, 1), -1, dtype=torch.int32, device=self.device))
            self.ext.apply_moves_batch(states, torch.from_numpy(moves).to(self.device), B)
            res = self.ext.check_results_batch(states, B).cpu().numpy()
            for i in range(B):
                if active[i]:
                    move_numbers[i] += 1
                    if res[i] != 0 or move_numbers[i] >= cfg.max_game_length:
                        active[i] = False
        final = self.ext.check_results_batch(states, B).cpu().numpy()
        out = []
        for i, hist in enumerate(histories):
            r = int(final[i])
            ex = []
            for sb, pol, turn, prior in hist:
                white = turn % 2 == 0
                v = 0.0 if r in (0, 3) else (1.0 if (r == 1) == white else -1.0)
                ex.append(ActionSpaceExample(sb, pol, v, prior))
            out.append(ex)
        return out


# ---------------------------------------------------------------------------
# one-ply Gumbel AlphaZero (hive_gpu/gumbel_mcts.py) and its match driver
# (gumbel_match.py)
# ---------------------------------------------------------------------------
@dataclass
class GumbelConfig:
    """hive_gpu/gumbel_mcts.py:45-68, plus ``seed``.  ``encoder_type`` is kept
    for signature compatibility; the network is the ``evaluate`` callable."""

    num_simulations: int = 128
    max_num_considered_actions: int = 32
    c_visit: float = 50.0
    c_scale: float = 1.0
    temperature: float = 1.0
    temperature_drop_move: int = 20
    batch_size: int = 256
    max_game_length: int = 300
    encoder_type: str = "transformer"
    expansion_mask: int = 0
    nn_max_batch: int = 0
    seed: int | None = None


class GumbelAlphaZeroOrchestrator:
    """Tree-free Gumbel search with sequential halving over the action space
    (gumbel_mcts.py:72-1020): the root's top-k Gumbel-perturbed actions are
    evaluated one ply deep (a candidate with more than one simulation of
    budget also probes the opponent's most likely reply), halved by
    g + logit + sigma(Q) per round, and the policy target is the softmax of
    logit + sigma(completed Q) over the candidates.

    Differences: the Gumbel uniforms come from a seeded CUDA generator and
    the move draws from a seeded numpy generator (``config.seed``); the
    immediate-win scan is one child-probe launch instead of a host loop over
    every legal move; the halving sort is stable; with no legal action in
    the whole batch the reference returns a 4-tuple its caller cannot unpack
    (gumbel_mcts.py:294-298), here the search returns empty candidate lists.
    An example is (state bytes, dense policy target with the 1e-4 floor on
    legal actions, value target, dense network prior at the candidates)."""

    _OFF_TURN = 3412

    def __init__(self, evaluate: Evaluator, config: GumbelConfig | None = None, device: str = "cuda") -> None:
        self.ext = load_extension()
        self.evaluate = evaluate
        self.config = config or GumbelConfig()
        self.device = torch.device(device)
        self.gen = torch.Generator(device=self.device)
        if self.config.seed is not None:
            self.gen.manual_seed(int(self.config.seed))
        else:
            self.gen.seed()
        self.rng = np.random.default_rng(self.config.seed)
        self._action_space_size = ACTION_SPACE_SIZE
        self._move_size = SIZEOF_GPU_MOVE
        self.trace: list | None = None  # set to a list to record the first search's evaluations

    def _recording(self) -> bool:
        return self.trace is not None and not any(x["kind"] == "searched" for x in self.trace)

    def _nn(self, states: torch.Tensor, total: int):
        """(logits [T, 85834] f32, values [T] f32), in chunks of ``nn_max_batch``
        (gumbel_mcts.py:854-866)."""
        mb = int(self.config.nn_max_batch)
        if mb > 0 and total > mb:
            parts = [self.evaluate(states[s:min(s + mb, total)], min(s + mb, total) - s) for s in range(0, total, mb)]
            logits = torch.cat([p[0].float() for p in parts])
            values = torch.cat([p[1].float().reshape(-1) for p in parts])
        else:
            logits, values = self.evaluate(states, total)
            logits, values = logits.float(), values.float().reshape(-1)
        if self._recording():
            self.trace.append(dict(kind="eval", states=states[:total].clone(), logits=logits.clone(),
                                   values=values.clone()))
        return logits, values

    def _get_turns(self, states: torch.Tensor, B: int) -> list[int]:
        off = self._OFF_TURN
        return (states[:B, off].to(torch.int32) | (states[:B, off + 1].to(torch.int32) << 8)).cpu().tolist()

    @staticmethod
    def _match_actions_to_legal_moves(actions, legal_action_indices, num_legal):
        """gumbel_mcts.py:641-662: first legal slot holding each action, or -1."""
        matches = legal_action_indices.unsqueeze(1).eq(actions.unsqueeze(-1))
        slots = torch.arange(legal_action_indices.shape[1], device=legal_action_indices.device).unsqueeze(0)
        matches &= (slots < num_legal.unsqueeze(1)).unsqueeze(1)
        first = matches.to(torch.int8).argmax(dim=-1).to(torch.int64)
        return torch.where(matches.any(dim=-1), first, torch.full_like(first, -1))

    @staticmethod
    def _gather_legal_action_scores(action_scores, legal_action_indices):
        """gumbel_mcts.py:664-673"""
        g = action_scores.gather(1, legal_action_indices.clamp(min=0).long())
        return g.masked_fill(legal_action_indices < 0, float("-inf"))

    # -- search -------------------------------------------------------------------
    def _gumbel_search(self, root_states: torch.Tensor, B: int, active: list[bool], move_numbers: list[int]):
        """gumbel_mcts.py:238-411 -> (policies, graphs, seqs, nn_priors,
        legal_moves, legal_action_indices, num_legal_moves); graphs and seqs
        (archived encoders) are ``None`` per game."""
        cfg, A, dev = self.config, self._action_space_size, self.device
        legal_moves, num_legal_moves, mask = self.ext.generate_legal_moves_and_mask_batch(root_states, B)
        legal_action_indices = self.ext.legal_moves_to_actions_batch(root_states, legal_moves, num_legal_moves, B)
        legal_mask = mask != 0
        policy_logits, root_values = self._nn(root_states, B)
        policy_logits = policy_logits.masked_fill(~legal_mask, float("-inf"))
        nn_prior_probs = torch.softmax(policy_logits, dim=-1)
        u = torch.rand(B, A, device=dev, generator=self.gen).clamp(1e-10, 1.0 - 1e-7)
        gumbel = (-torch.log(-torch.log(u))).masked_fill(~legal_mask, float("-inf"))
        if self._recording():
            self.trace.append(dict(kind="gumbel", gumbel=gumbel.clone()))
        perturbed = gumbel + policy_logits
        num_legal = legal_mask.sum(dim=1)
        k = int(cfg.max_num_considered_actions)
        max_k = min(k, int(num_legal.max().item()))
        none = [None] * B
        if max_k == 0:
            empty = (np.zeros(0, np.int64), np.zeros(0, np.float32))
            return [empty] * B, none, none, [None] * B, legal_moves, legal_action_indices, num_legal_moves
        topk_actions = torch.topk(perturbed, max_k, dim=1).indices
        q_sums = torch.zeros(B, max_k, device=dev)
        visit_counts = torch.zeros(B, max_k, dtype=torch.int32, device=dev)
        candidate_mask = (torch.arange(max_k, device=dev).unsqueeze(0)
                          < torch.clamp(num_legal, max=k).unsqueeze(1))
        num_rounds = max(1, math.ceil(math.log2(int(candidate_mask.sum(dim=1).max().item()))))
        remaining = torch.full((B,), int(cfg.num_simulations), dtype=torch.int32, device=dev)
        for round_idx in range(num_rounds):
            n_remaining = candidate_mask.sum(dim=1).float()
            if int(n_remaining.max().item()) == 0:
                break
            n_rem_i = candidate_mask.sum(dim=1).int()
            visits = torch.where(n_rem_i > 0, torch.clamp(remaining // n_rem_i.clamp(min=1), min=1),
                                 torch.zeros_like(remaining))
            if int(visits.max().item()) == 0:
                break
            child_values = self._evaluate_candidates(root_states, B, topk_actions, candidate_mask, visits,
                                                     legal_moves, num_legal_moves, legal_action_indices)
            q_sums += child_values * visits.unsqueeze(1).float() * candidate_mask.float()
            visit_counts += visits.unsqueeze(1) * candidate_mask.int()
            remaining = torch.clamp(remaining - visits * n_rem_i, min=0)
            if round_idx < num_rounds - 1:
                max_n = visit_counts.max(dim=1, keepdim=True).values.float().clamp(min=1)
                q_mean = torch.where(visit_counts > 0, q_sums / visit_counts.float(), torch.zeros_like(q_sums))
                qtransform = (cfg.c_visit + max_n) * cfg.c_scale * q_mean
                sigma = gumbel.gather(1, topk_actions) + policy_logits.gather(1, topk_actions) + qtransform
                sigma = sigma.masked_fill(~candidate_mask, float("-inf"))
                n_keep = (n_remaining / 2).ceil().int().clamp(min=1)
                order = sigma.argsort(dim=1, descending=True, stable=True)
                rank = torch.empty_like(order)
                rank.scatter_(1, order, torch.arange(max_k, device=dev).unsqueeze(0).expand(B, -1).contiguous())
                candidate_mask = (rank < n_keep.unsqueeze(1)) & candidate_mask
        policies, nn_priors = self._compute_improved_policy(policy_logits, topk_actions, q_sums, visit_counts,
                                                            root_values, nn_prior_probs, B, active)
        if self._recording():
            self.trace.append(dict(kind="searched", topk=topk_actions.clone(), q_sums=q_sums.clone(),
                                   visits=visit_counts.clone(), candidates=candidate_mask.clone(),
                                   policies=policies))
        return policies, none, none, nn_priors, legal_moves, legal_action_indices, num_legal_moves

    def _evaluate_candidates(self, root_states, B, topk_actions, candidate_mask, visits_per_action, legal_moves,
                             num_legal_moves, legal_action_indices):
        """gumbel_mcts.py:416-514: one-ply values of the live candidates, from
        the root player's view, [B, max_k]."""
        max_k = topk_actions.shape[1]
        matched = self._match_actions_to_legal_moves(topk_actions, legal_action_indices, num_legal_moves)
        pairs = torch.nonzero(candidate_mask & (matched >= 0), as_tuple=False)
        out = torch.zeros(B, max_k, device=self.device)
        if pairs.numel() == 0:
            return out
        gi, cj = pairs[:, 0], pairs[:, 1]
        total = int(pairs.shape[0])
        child_states = root_states[gi].clone()
        self.ext.apply_moves_batch(child_states, legal_moves[gi, matched[gi, cj]].contiguous(), total)
        results = self.ext.check_results_batch(child_states, total)
        child_logits, child_values = self._nn(child_states, total)
        root_white = root_states[gi, self._OFF_TURN] % 2 == 0
        root_won = ((results == 1) & root_white) | ((results == 2) & ~root_white)
        terminal = torch.where(results == 3, torch.zeros_like(child_values),
                               torch.where(root_won, torch.full_like(child_values, -1.0),
                                           torch.full_like(child_values, 1.0)))
        neg = -torch.where(results != 0, terminal, child_values)
        if int(visits_per_action.max().item()) > 1:
            c_legal, c_nl, c_mask = self.ext.generate_legal_moves_and_mask_batch(child_states, total)
            c_lai = self.ext.legal_moves_to_actions_batch(child_states, c_legal, c_nl, total)
            masked = child_logits.masked_fill(c_mask == 0, float("-inf"))
            neg = self._probe_child_replies(child_states, neg, results, gi, visits_per_action, c_legal, c_nl,
                                            c_lai, masked)
        out[gi, cj] = neg
        return out

    def _probe_child_replies(self, child_states, default_root_values, child_results, root_game_indices,
                             visits_per_action, child_legal_moves, child_num_legal, child_legal_action_indices,
                             child_policy_logits):
        """gumbel_mcts.py:516-639: a child with reply budget takes the value of
        the grandchild after the opponent's most likely reply."""
        root_values = default_root_values.clone()
        scores = self._gather_legal_action_scores(torch.softmax(child_policy_logits, dim=-1),
                                                  child_legal_action_indices)
        best = scores.argmax(dim=1)
        best_score = scores.gather(1, best.unsqueeze(1)).squeeze(1)
        budget = (visits_per_action[root_game_indices] - 1).clamp(min=0)
        eligible = (child_results == 0) & (budget > 0) & (child_num_legal > 0) & best_score.isfinite()
        parent = torch.nonzero(eligible, as_tuple=True)[0]
        n = int(parent.numel())
        if n == 0:
            return root_values
        gc = child_states[parent].clone()
        self.ext.apply_moves_batch(gc, child_legal_moves[parent, best[parent]].contiguous(), n)
        gc_res = self.ext.check_results_batch(gc, n)
        _, gc_vals = self._nn(gc, n)
        root_white = child_states[parent, self._OFF_TURN] % 2 == 1
        root_won = ((gc_res == 1) & root_white) | ((gc_res == 2) & ~root_white)
        terminal = torch.where(gc_res == 3, torch.zeros_like(gc_vals),
                               torch.where(root_won, torch.full_like(gc_vals, 1.0), torch.full_like(gc_vals, -1.0)))
        root_values[parent] = torch.where(gc_res != 0, terminal, gc_vals)
        return root_values

    def _compute_improved_policy(self, logits, topk_actions, q_sums, visit_counts, root_values, nn_prior_probs, B,
                                 active):
        """gumbel_mcts.py:677-769: softmax over the candidates of logit +
        sigma(completed Q); unvisited candidates take -V(root)."""
        cfg = self.config
        q_mean = torch.where(visit_counts > 0, q_sums / visit_counts.float(), torch.zeros_like(q_sums))
        max_n = visit_counts.max(dim=1, keepdim=True).values.float().clamp(min=1)
        q = torch.where(visit_counts > 0, q_mean, (-root_values).unsqueeze(1).expand_as(q_mean))
        improved = logits.gather(1, topk_actions) + (cfg.c_visit + max_n) * cfg.c_scale * q
        probs = torch.nan_to_num(torch.softmax(improved, dim=-1), nan=0.0)
        prior = nn_prior_probs.gather(1, topk_actions)
        acts, pr, nnp = topk_actions.cpu().numpy(), probs.cpu().numpy(), prior.cpu().numpy()
        policies = [(acts[i], pr[i]) for i in range(B)]
        nn_priors = [(acts[i], nnp[i]) if active[i] else None for i in range(B)]
        return policies, nn_priors

    def _check_immediate_wins(self, root_states, B, active, current_turns) -> dict[int, int]:
        """gumbel_mcts.py:773-832: {game: action of its first winning legal move}."""
        legal, nl = self.ext.generate_legal_moves_batch(root_states, B)
        lai = self.ext.legal_moves_to_actions_batch(root_states, legal, nl, B)
        res, _, _ = self.ext.child_probe_batch(root_states, legal, nl, B, False)
        act = torch.tensor(active, dtype=torch.bool, device=self.device)
        white = torch.tensor([t % 2 == 0 for t in current_turns], dtype=torch.bool, device=self.device)
        slots = torch.arange(legal.shape[1], device=self.device).unsqueeze(0)
        target = torch.where(white, 1, 2).unsqueeze(1)
        win = (slots < nl.unsqueeze(1)) & act.unsqueeze(1) & (res == target)
        first = win.to(torch.int8).argmax(dim=1)
        has = win.any(dim=1)
        action = lai.gather(1, first.unsqueeze(1)).squeeze(1)
        rows = torch.nonzero(has).squeeze(1).cpu().tolist()
        vals = action[has].cpu().tolist()
        return dict(zip(rows, vals))

    def _select_and_apply(self, states, B, policies, active, move_numbers, legal_moves, legal_action_indices,
                          num_legal, win_overrides=None, greedy=False):
        """Action choice (greedy after the temperature drop, else a draw from
        the candidate distribution) and the batched move application
        (gumbel_mcts.py:176-219)."""
        cfg = self.config
        selected = np.full(B, -1, dtype=np.int64)
        for i in range(B):
            if not active[i]:
                continue
            acts, probs = policies[i]
            if win_overrides and i in win_overrides:
                selected[i] = win_overrides[i]
            elif greedy:
                selected[i] = int(acts[int(np.argmax(probs))]) if len(acts) else -1
            elif move_numbers[i] >= cfg.temperature_drop_move:
                selected[i] = int(acts[int(np.argmax(probs))])
            else:
                p = probs.astype(np.float64)
                s = p.sum()
                p = p / s if (s > 0 and np.isfinite(s)) else np.full(len(p), 1.0 / len(p))
                selected[i] = int(acts[int(self.rng.choice(len(p), p=p))])
        a = torch.from_numpy(selected).to(self.device).unsqueeze(1)
        matched = self._match_actions_to_legal_moves(a, legal_action_indices, num_legal).squeeze(1)
        mb = legal_moves[torch.arange(B, device=self.device), matched.clamp(min=0)]
        mb = torch.where((matched >= 0).unsqueeze(1), mb, torch.zeros_like(mb)).contiguous()
        self.ext.apply_moves_batch(states, mb, B)
        return selected

    def self_play_batch(self, start_states: torch.Tensor | None = None) -> list[list[ActionSpaceExample]]:
        """gumbel_mcts.py:101-234"""
        cfg = self.config
        B = cfg.batch_size
        states = (start_states.to(self.device).contiguous().clone() if start_states is not None
                  else self.ext.create_initial_states(B, cfg.expansion_mask))
        active = [True] * B
        move_numbers = [0] * B
        histories: list[list[tuple]] = [[] for _ in range(B)]
        while any(active):
            turns = self._get_turns(states, B)
            policies, _, _, nn_priors, legal, lai, nl = self._gumbel_search(states, B, active, move_numbers)
            lai_np, nl_np = lai.cpu().numpy(), nl.cpu().numpy()
            wins = self._check_immediate_wins(states, B, active, turns)
            sh = states.cpu().numpy()
            for i in range(B):
                if not active[i]:
                    continue
                acts, probs = policies[i]
                legal_acts = lai_np[i, :int(nl_np[i])].copy()
                if i in wins:
                    acts, probs = np.array([wins[i]], dtype=acts.dtype), np.array([1.0], dtype=probs.dtype)
                histories[i].append((sh[i].copy(), (acts, probs), turns[i], nn_priors[i], legal_acts))
            self._select_and_apply(states, B, policies, active, move_numbers, legal, lai, nl, wins)
            for i in range(B):
                if active[i]:
                    move_numbers[i] += 1
            results = self.ext.check_results_batch(states, B).cpu().numpy()
            for i in range(B):
                if active[i] and (results[i] != 0 or move_numbers[i] >= cfg.max_game_length):
                    active[i] = False
        return self._build_examples(histories, self.ext.check_results_batch(states, B).cpu().numpy())

    def _build_examples(self, histories, final_results) -> list[list[ActionSpaceExample]]:
        """gumbel_mcts.py:936-1020 without the archived encoders' mobility and
        queen-surround targets."""
        A = self._action_space_size
        out = []
        for i, hist in enumerate(histories):
            r = int(final_results[i])
            ex = []
            for sb, (acts, probs), turn, prior, legal_acts in hist:
                white = turn % 2 == 0
                v = 0.0 if r in (0, 3) else (1.0 if (r == 1) == white else -1.0)
                policy = np.zeros(A, np.float32)
                policy[acts] = probs
                ok = legal_acts[legal_acts >= 0]
                if ok.size:
                    policy[ok] = np.maximum(policy[ok], 1e-4)
                nn_prior = None
                if prior is not None:
                    nn_prior = np.zeros(A, np.float32)
                    nn_prior[prior[0]] = prior[1]
                ex.append(ActionSpaceExample(sb, policy, v, nn_prior))
            out.append(ex)
        return out


def gumbel_match(evaluate_a: Evaluator, evaluate_b: Evaluator, num_games: int, num_sims: int, gumbel_k: int,
                 max_moves: int = 300, expansion_mask: int = 0, seed: int | None = None,
                 start_states: torch.Tensor | None = None) -> dict:
    """gumbel_match.py:79-197: two evaluators play ``num_games`` greedy games
    (A is white in the first half); each step the games are split by the side
    to move and searched in two sub-batches.  Returns the per-game results,
    move counts and A's score."""
    cfg = GumbelConfig(num_simulations=num_sims, max_num_considered_actions=gumbel_k, temperature=0.0,
                       temperature_drop_move=0, batch_size=num_games, expansion_mask=expansion_mask, seed=seed)
    orch_a = GumbelAlphaZeroOrchestrator(evaluate_a, cfg)
    orch_b = GumbelAlphaZeroOrchestrator(evaluate_b, dataclasses.replace(cfg, seed=None if seed is None else seed + 1))
    ext = orch_a.ext
    dev = orch_a.device
    a_is_white = np.arange(num_games) < num_games // 2
    states = (start_states.to(dev).contiguous().clone() if start_states is not None
              else ext.create_initial_states(num_games, expansion_mask))
    active = np.ones(num_games, dtype=bool)
    move_numbers = np.zeros(num_games, dtype=np.int64)
    while active.any():
        turns = np.array(orch_a._get_turns(states, num_games))
        a_turn = active & (a_is_white == (turns % 2 == 0))
        b_turn = active & ~a_turn
        for orch, idx in ((orch_a, np.flatnonzero(a_turn)), (orch_b, np.flatnonzero(b_turn))):
            n = int(idx.size)
            if n == 0:
                continue
            it = torch.from_numpy(idx.astype(np.int64)).to(dev)
            sub = states[it].contiguous()
            pol, _, _, _, legal, lai, nl = orch._gumbel_search(sub, n, [True] * n, list(move_numbers[idx]))
            orch._select_and_apply(sub, n, pol, [True] * n, list(move_numbers[idx]), legal, lai, nl, greedy=True)
            states[it] = sub
        move_numbers[active] += 1
        res = ext.check_results_batch(states, num_games).cpu().numpy()
        active &= ~((res != 0) | (move_numbers >= max_moves))
    final = ext.check_results_batch(states, num_games).cpu().numpy()
    score = np.where(final == 1, a_is_white.astype(float), np.where(final == 2, (~a_is_white).astype(float), 0.5))
    return dict(results=final, move_numbers=move_numbers, a_is_white=a_is_white, a_score=float(score.sum()))
