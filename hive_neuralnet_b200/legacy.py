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
