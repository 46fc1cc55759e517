"""Self-play orchestrators: drop-ins for the reference's FNN search drivers.

* :class:`FNNMCTSOrchestrator` -- Gumbel-root MCTS with sequential halving
  (reference hive_fnn/fnn_mcts_orchestrator.py:91-1161);
* :class:`FNNPUCTOrchestrator` -- plain PUCT with wave virtual loss
  (reference hive_fnn/fnn_puct_orchestrator.py:46-451).

Same constructors, configs and ``self_play_batch(start_states=None) ->
list[list[FNNTrainingExample]]``.  What changes is where the work runs:

* leaf evaluation is one fused kernel (successors + FNN + softmax,
  :class:`hive_neuralnet_b200.fnn.FusedFNNEvaluator`);
* every per-game Python loop of the reference (immediate wins, root stats,
  re-rooting, Dirichlet noise) is a batched device operation, and a search
  wave has no host synchronisation;
* tree kernels process each game's simulations in simulation order, so the
  search is deterministic given the noise (Gumbel and Dirichlet draws come
  from a seeded CUDA generator when ``config.seed`` is set);
* ``FNNPUCTOrchestrator`` passes the tree tensors in the binding order.  The
  reference's ``_tree_args`` (fnn_puct_orchestrator.py:110-117) swaps
  ``virtual_q_penalty`` and ``parent_idx``; here that swap would be rejected
  by dtype checks, so the intended order of FNNMCTSOrchestrator._tree_args
  (fnn_mcts_orchestrator.py:232-239) is used.

Reference behaviours kept on purpose (parity): when any game of the batch has
an immediate win, all games' priors and child Q are reset
(fnn_mcts_orchestrator.py:621-625); the halving score's sigma uses the
batch-wide maximum visit count (:692-697); re-rooting does not reset
virtual_q_penalty (:1126-1141).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np
import torch

from .fnn import FusedFNNEvaluator, HiveFNN
from .hive_gpu import load_extension

_OFF_TURN = 3412
_OFF_HEIGHT = 2645
_OFF_QUEEN_CELL = 3392
_NUM_CELLS = 529
_BOARD_SIZE = 23
_GUMBEL_ROUNDS = 4
_GUMBEL_WAVE_SCHEDULE = (2, 4, 8, 16)


class FNNTrainingExample(NamedTuple):
    """Same fields as hive_fnn/fnn_replay_buffer.py:21-31."""

    state_bytes: np.ndarray
    policy_target: np.ndarray
    value_target: float
    use_for_policy: bool = True
    use_for_value: bool = True
    value_weight: float = 1.0
    surprise_weight: float = 1.0


@dataclass
class FNNMCTSConfig:
    """Fields and defaults of hive_fnn/fnn_mcts_orchestrator.py:45-82, plus ``seed``."""

    num_simulations: int = 128
    max_num_considered_actions: int = 16
    c_puct: float = 1.25
    c_visit: float = 50.0
    c_scale: float = 1.0
    temperature: float = 1.0
    temperature_drop_move: int = 20
    batch_size: int = 128
    max_game_length: int = 300
    expansion_mask: int = 0
    wave_parallel: bool = True
    wave_size: int = 4
    deterministic_non_root: bool = False
    virtual_q_penalty: float = 0.25
    non_root_sigma: float = 4.0
    dirichlet_alpha: float = 0.3
    dirichlet_epsilon: float = 0.25
    max_tree_nodes: int = 65536
    queen_surround_reserve_slots: int = 6
    queen_surround_reserve_immobile_only: bool = True
    root_q_min_visits: int = 0
    short_forced_win_probe: bool = False
    probe_win_in_one: bool = True
    probe_check_opponent_wins: bool = True
    probe_win_in_two: bool = True
    policy_target_temperature: float = 1.0
    adaptive_policy_target_temperature: bool = True
    policy_target_top1_cap: float = 0.7
    policy_target_min_temperature: float = 1.0
    policy_target_max_temperature: float = 7.0
    final_value_ply_count: int = 3
    final_value_weight: float = 2.0
    rebase_tree_each_move: bool = True
    seed: int | None = None


@dataclass
class FNNPUCTConfig:
    """Fields and defaults of hive_fnn/fnn_puct_orchestrator.py:24-42, plus ``seed``."""

    num_simulations: int = 128
    c_puct: float = 1.25
    temperature: float = 1.0
    temperature_drop_move: int = 20
    batch_size: int = 128
    max_game_length: int = 300
    expansion_mask: int = 0
    wave_size: int = 16
    dirichlet_alpha: float = 0.3
    dirichlet_epsilon: float = 0.25
    max_tree_nodes: int = 65536
    final_value_ply_count: int = 3
    final_value_weight: float = 2.0
    rebase_tree_each_move: bool = True
    seed: int | None = None


def _result_to_value(result: int, turn: int) -> float:
    """fnn_mcts_orchestrator.py:1155-1161"""
    if result == 0 or result == 3:
        return 0.0
    is_white = turn % 2 == 0
    return 1.0 if (result == 1 and is_white) or (result == 2 and not is_white) else -1.0


def _neighbor_cells(device) -> torch.Tensor:
    neigh = torch.full((_NUM_CELLS, 6), -1, dtype=torch.int64)
    dirs = ((1, 0), (1, -1), (0, -1), (-1, 0), (-1, 1), (0, 1))
    for cell in range(_NUM_CELLS):
        row, col = divmod(cell, _BOARD_SIZE)
        for i, (dq, dr) in enumerate(dirs):
            nr, nc = row + dr, col + dq
            if 0 <= nr < _BOARD_SIZE and 0 <= nc < _BOARD_SIZE:
                neigh[cell, i] = nr * _BOARD_SIZE + nc
    return neigh.to(device)


class _SearchBase:
    """Tree storage, evaluation and the root helpers shared by both drivers."""

    def _setup(self, net: HiveFNN, cfg, device) -> None:
        self.ext = load_extension()
        self.net = net
        self.config = cfg
        self.device = torch.device(device)
        self.evaluator = FusedFNNEvaluator(net, self.device)
        self._move_size = self.ext.SIZEOF_GPU_MOVE
        self._max_nodes = int(cfg.max_tree_nodes)
        self._max_legal = int(self.ext.MAX_LEGAL_MOVES)
        self._slot_idx = torch.arange(self._max_legal, device=self.device, dtype=torch.int64).unsqueeze(0)
        self._neighbor = _neighbor_cells(self.device)
        self.gen = torch.Generator(device=self.device)
        if cfg.seed is not None:
            self.gen.manual_seed(int(cfg.seed))
        else:
            self.gen.seed()
        self.trace: list | None = None  # set to a list to record per-wave evaluator outputs
        # simulations executed (leaves with a node), accumulated on the device
        self.sims_done = torch.zeros((), dtype=torch.int64, device=self.device)
        # positions and successor rows the evaluator ran (the work behind the
        # FLOP count of a step): a host count and a device count, no sync
        self.leaves_evaluated = 0
        self.rows_evaluated = torch.zeros((), dtype=torch.int64, device=self.device)

    def _uniform(self, *shape: int) -> torch.Tensor:
        """U[0, 1) float32 draws of the search (the reference's torch.rand
        calls), from the driver's seeded generator; the single place a test
        substitutes recorded draws."""
        return torch.rand(shape, device=self.device, generator=self.gen)

    # -- tree ---------------------------------------------------------------
    def _alloc_tree(self, B: int) -> dict[str, torch.Tensor]:
        M, dev = self._max_nodes, self.device
        return {
            "visit_count": torch.zeros(B, M, dtype=torch.int32, device=dev),
            "total_value": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "prior": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "virtual_q_penalty": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "parent_idx": torch.full((B, M), -1, dtype=torch.int32, device=dev),
            "move_bytes": torch.zeros(B, M, self._move_size, dtype=torch.uint8, device=dev),
            "action_idx": torch.full((B, M), -1, dtype=torch.int32, device=dev),
            "first_child": torch.full((B, M), -1, dtype=torch.int32, device=dev),
            "num_children": torch.zeros(B, M, dtype=torch.int32, device=dev),
            "is_terminal": torch.zeros(B, M, dtype=torch.int8, device=dev),
            "terminal_value": torch.zeros(B, M, dtype=torch.float32, device=dev),
            "node_count": torch.ones(B, dtype=torch.int32, device=dev),
            "root_node": torch.zeros(B, dtype=torch.int32, device=dev),
            "child_init_q": torch.zeros(B, M, dtype=torch.float32, device=dev),
        }

    def _reset_tree(self, tree: dict[str, torch.Tensor]) -> None:
        """fnn_mcts_orchestrator.py:216-230"""
        for key, fill in (("visit_count", 0), ("total_value", 0.0), ("prior", 0.0), ("virtual_q_penalty", 0.0),
                          ("parent_idx", -1), ("move_bytes", 0), ("action_idx", -1), ("first_child", -1),
                          ("num_children", 0), ("is_terminal", 0), ("terminal_value", 0.0), ("node_count", 1),
                          ("root_node", 0), ("child_init_q", 0.0)):
            tree[key].fill_(fill)

    @staticmethod
    def _tree_args(tree: dict[str, torch.Tensor]) -> list[torch.Tensor]:
        return [tree["visit_count"], tree["total_value"], tree["prior"], tree["parent_idx"],
                tree["virtual_q_penalty"], tree["move_bytes"], tree["action_idx"], tree["first_child"],
                tree["num_children"], tree["is_terminal"], tree["terminal_value"], tree["node_count"]]

    def _reroot_tree(self, tree, moved: torch.Tensor, chosen_child: torch.Tensor) -> None:
        """Batched form of fnn_mcts_orchestrator.py:1122-1153 (moved: [B] bool)."""
        if self.config.rebase_tree_each_move:
            m = moved.unsqueeze(1)
            for key, fill in (("visit_count", 0), ("total_value", 0.0), ("prior", 0.0), ("parent_idx", -1),
                              ("action_idx", -1), ("first_child", -1), ("num_children", 0), ("is_terminal", 0),
                              ("terminal_value", 0.0), ("child_init_q", 0.0)):
                tree[key].masked_fill_(m, fill)
            tree["move_bytes"].masked_fill_(m.unsqueeze(2), 0)
            tree["node_count"].masked_fill_(moved, 1)
            tree["root_node"].masked_fill_(moved, 0)
            return
        new_roots = torch.where(moved, chosen_child.to(torch.int32), tree["root_node"])
        tree["root_node"].copy_(new_roots)
        tree["parent_idx"].scatter_(1, new_roots.long().unsqueeze(1),
                                    torch.full_like(new_roots.unsqueeze(1), -1))

    def _expand_root_if_needed(self, tree, states, legal_moves, num_legal, priors, child_q, game_active, B):
        row = torch.arange(B, device=self.device)
        root = tree["root_node"]
        needs = (tree["first_child"][row, root.long()] < 0) & game_active.to(torch.bool)
        leaf = torch.where(needs, root, torch.full_like(root, -1)).to(torch.int32).contiguous()
        results = self.ext.check_results_batch(states, B)
        self.ext.mcts_expand_dense_priors_batch(*self._tree_args(tree), tree["child_init_q"], child_q, leaf, states,
                                                legal_moves, num_legal, priors, results, B, B, self._max_nodes)

    def _apply_root_dirichlet(self, tree, B: int, active: torch.Tensor) -> None:
        """fnn_mcts_orchestrator.py:904-925 with the per-game numpy draws
        replaced by batched Gamma draws on the device (Dirichlet = normalised
        Gamma(alpha, 1))."""
        cfg = self.config
        if cfg.dirichlet_epsilon <= 0.0:
            return
        row = torch.arange(B, device=self.device)
        nc = tree["num_children"][row, tree["root_node"].long()]
        pad = self._max_legal
        alpha = torch.clamp(10.0 / nc.clamp(min=1).float(), max=cfg.dirichlet_alpha).clamp(min=0.03)
        valid = (self._slot_idx < nc.unsqueeze(1)) & active.unsqueeze(1)
        conc = alpha.unsqueeze(1).expand(B, pad).contiguous()
        g = torch._standard_gamma(conc, generator=self.gen)
        g = torch.where(valid, g, torch.zeros_like(g))
        noise = (g / g.sum(dim=1, keepdim=True).clamp(min=1e-30)).float().contiguous()
        self.ext.mcts_apply_root_noise(*self._tree_args(tree), noise, tree["root_node"], pad, cfg.dirichlet_epsilon,
                                       1.0, B, self._max_nodes)

    def _root_stats(self, tree, B: int, slots: torch.Tensor, min_visits: int):
        """Visits and Q of root children at `slots` ([B, k] slot indices,
        negative = none): fnn_mcts_orchestrator.py:1072-1120."""
        row = torch.arange(B, device=self.device, dtype=torch.long)
        root = tree["root_node"].long()
        fc = tree["first_child"][row, root].long()
        nc = tree["num_children"][row, root].long()
        sl = slots.long()
        valid = (sl >= 0) & (fc.unsqueeze(1) >= 0) & (sl < nc.unsqueeze(1))
        child = (fc.unsqueeze(1) + sl.clamp(min=0)).clamp(min=0, max=self._max_nodes - 1)
        row2 = row.unsqueeze(1).expand_as(child)
        v_raw = tree["visit_count"][row2, child]
        t_raw = tree["total_value"][row2, child]
        visits = torch.where(valid, v_raw, torch.zeros_like(v_raw))
        q = torch.where(valid & (v_raw > min_visits), -t_raw / v_raw.clamp(min=1).float(), torch.zeros_like(t_raw))
        return visits, q

    def _gather_root_child_stats(self, tree, B: int):
        """Visits and Q of every root child slot (fnn_mcts_orchestrator.py:1098-1120,
        fnn_puct_orchestrator.py:388-410)."""
        return self._root_stats(tree, B, self._slot_idx.expand(B, -1), int(getattr(self.config, "root_q_min_visits", 0)))

    def _run_simulations(self, tree, root_states, game_active, alive_mask, B, num_sims, wave_size=None):
        """Waves of root-mask select / replay / evaluate / expand + backup
        (fnn_mcts_orchestrator.py:927-980, fnn_puct_orchestrator.py:341-386)."""
        cfg = self.config
        W = max(1, int(cfg.wave_size if wave_size is None else wave_size))
        q_pen = float(cfg.virtual_q_penalty) if getattr(cfg, "deterministic_non_root", False) and W > 1 else 0.0
        leaf_states = torch.zeros(W * B, root_states.shape[1], dtype=torch.uint8, device=self.device)
        for wave in range((num_sims + W - 1) // W):
            aw = min(W, num_sims - wave * W)
            total = aw * B
            leaf, paths, plen, vlp, vll = self.ext.mcts_select_with_root_mask_batch(
                *self._tree_args(tree), tree["child_init_q"], game_active, tree["root_node"], alive_mask,
                self._max_legal, cfg.c_puct, B, aw, self._max_nodes, False, 4.0, 0.0)
            ls = leaf_states[:total]
            self.ext.mcts_replay_batch(root_states, ls, paths, plen, leaf, B, total)
            results = self.ext.check_results_batch(ls, total)
            legal, nl, feats = self.ext.generate_legal_moves_and_fnn_features_batch(ls, total)
            pri, vals, cq = self._eval_states(ls, legal, nl, total, feats)
            self.sims_done += (leaf >= 0).sum()
            if self.trace is not None:
                self.trace.append(dict(kind="wave", W=aw, leaf=leaf.clone(), priors=pri.clone(),
                                       values=vals.clone(), child_q=cq.clone()))
            self.ext.mcts_expand_and_backprop_dense_priors_slots_batch(
                *self._tree_args(tree), tree["child_init_q"], cq, leaf, ls, legal, nl, pri, results, vals, vlp, vll,
                tree["root_node"], None, 1, B, total, self._max_nodes, q_pen)

    def _find_immediate_wins(self, states, legal_moves, num_legal, total, *, row_mask=None, slot_mask=None):
        """First winning legal slot per game or -1 (fnn_mcts_orchestrator.py:446-493)."""
        winners = torch.full((total,), -1, dtype=torch.int64, device=self.device)
        if total == 0:
            return winners
        valid = self._slot_idx < num_legal.to(torch.int64).unsqueeze(1)
        if row_mask is not None:
            valid &= row_mask.unsqueeze(1)
        if slot_mask is not None:
            valid &= slot_mask
        res, _, _ = self.ext.child_probe_batch(states, legal_moves, num_legal, total, False)
        white = (states[:, _OFF_TURN].to(torch.int32) % 2 == 0).unsqueeze(1)
        win = valid & (((res == 1) & white) | ((res == 2) & ~white))
        first = torch.argmax(win.to(torch.int8), dim=1)
        return torch.where(win.any(dim=1), first, winners)

    def _queen_surround_count(self, states, queen_color):
        """fnn_mcts_orchestrator.py:318-337"""
        rows = torch.arange(states.shape[0], device=self.device, dtype=torch.int64)
        qbase = (_OFF_QUEEN_CELL + 2 * queen_color).to(torch.int64)
        qcell = states[rows, qbase].to(torch.int32) | (states[rows, qbase + 1].to(torch.int32) << 8)
        valid_queen = qcell != 0xFFFF
        neigh = self._neighbor[qcell.clamp(min=0, max=_NUM_CELLS - 1).to(torch.int64)]
        heights = states[:, _OFF_HEIGHT:_OFF_HEIGHT + _NUM_CELLS].to(torch.int16)
        nh = heights.gather(1, neigh.clamp(min=0))
        surround = ((neigh >= 0) & (nh > 0)).sum(dim=1).to(torch.int32)
        return torch.where(valid_queen, surround, torch.zeros_like(surround)), qcell

    def _eval_states(self, states, legal_moves, num_legal, total, root_features=None):
        self.leaves_evaluated += int(total)
        if total:
            self.rows_evaluated += num_legal[:total].to(torch.int64).clamp(0, self._max_legal).sum()
        return self.evaluator.eval_states(states, legal_moves, num_legal, total, root_features)


class FNNMCTSOrchestrator(_SearchBase):
    """Gumbel AlphaZero with MCTS below the root (FNN leaf evaluation)."""

    def __init__(self, net: HiveFNN, config: FNNMCTSConfig | None = None, device: str = "cuda") -> None:
        self._setup(net, config or FNNMCTSConfig(), device)
        self.last_policy_temperature_stats: dict[str, float] = {}

    # fnn_mcts_orchestrator.py:144-191
    def _build_policy_target(self, sampled_logits, valid_slot):
        cfg = self.config

        def soft(temp):
            p = torch.softmax(sampled_logits / temp, dim=1)
            p = torch.where(valid_slot, p, torch.zeros_like(p))
            return p / p.sum(dim=1, keepdim=True).clamp_min(1e-12)

        if not cfg.adaptive_policy_target_temperature:
            t = torch.full((sampled_logits.shape[0], 1), max(float(cfg.policy_target_temperature), 1e-6),
                           dtype=sampled_logits.dtype, device=sampled_logits.device)
            return soft(t), t.squeeze(1)
        min_t = max(float(cfg.policy_target_min_temperature), 1.0)
        max_t = max(float(cfg.policy_target_max_temperature), min_t)
        cap = min(max(float(cfg.policy_target_top1_cap), 0.0), 1.0)
        base = torch.full((sampled_logits.shape[0], 1), min_t, dtype=sampled_logits.dtype,
                          device=sampled_logits.device)
        probs = soft(base)
        need = probs.max(dim=1, keepdim=True).values > cap
        if max_t <= min_t:
            return probs, base.squeeze(1)
        low, high = base.clone(), torch.full_like(base, max_t)
        for _ in range(12):
            mid = (low + high) * 0.5
            sharp = soft(mid).max(dim=1, keepdim=True).values > cap
            low = torch.where(need & sharp, mid, low)
            high = torch.where(need & ~sharp, mid, high)
        final = torch.where(need, high, base)
        return soft(final), final.squeeze(1)

    # fnn_mcts_orchestrator.py:339-382
    def _queen_surround_qualifying_mask(self, states, legal_moves, num_legal, total):
        valid = self._slot_idx < num_legal.to(torch.int64).unsqueeze(1)
        _, after, esc = self.ext.child_probe_batch(states, legal_moves, num_legal, total,
                                                   bool(self.config.queen_surround_reserve_immobile_only))
        turn = states[:, _OFF_TURN].to(torch.int32) | (states[:, _OFF_TURN + 1].to(torch.int32) << 8)
        before, _ = self._queen_surround_count(states, ((turn + 1) & 1).to(torch.int64))
        qual = valid & (after > before.unsqueeze(1))
        if esc is not None:
            qual &= esc == 0
        return qual

    # fnn_mcts_orchestrator.py:384-444
    def _root_candidate_slots(self, states, legal_moves, num_legal, priors, legal_logits, total,
                              allowed_slot_mask=None):
        cfg = self.config
        k = min(int(cfg.max_num_considered_actions), self._max_legal)
        valid = self._slot_idx < num_legal.to(torch.int64).unsqueeze(1)
        if allowed_slot_mask is not None:
            valid = valid & allowed_slot_mask
        reserve = min(int(cfg.queen_surround_reserve_slots), k)
        if reserve <= 0:
            u = self._uniform(total, self._max_legal).clamp(1e-4, 1 - 1e-4)
            g = torch.where(valid, -torch.log(-torch.log(u)), torch.full_like(u, -1e30))
            return torch.topk(g + legal_logits, k, dim=1).indices.to(torch.int32)
        qual = self._queen_surround_qualifying_mask(states, legal_moves, num_legal, total)
        rs = torch.where(qual, priors, torch.full_like(priors, -1e30))
        per_game = qual.sum(dim=1).clamp(max=reserve)
        r_order = torch.topk(rs, reserve, dim=1).indices
        r_valid = torch.arange(reserve, device=self.device).unsqueeze(0) < per_game.unsqueeze(1)
        r_cand = torch.where(r_valid, r_order.to(torch.int32), torch.full_like(r_order, -1, dtype=torch.int32))
        # reserved slots marked in an extra column's worth of room: entries past
        # a game's reserve count land in the spare column, never on a real slot
        chosen = torch.zeros((total, self._max_legal + 1), dtype=torch.bool, device=valid.device)
        chosen.scatter_(1, torch.where(r_valid, r_order, torch.full_like(r_order, self._max_legal)),
                        torch.ones_like(r_valid))
        chosen = chosen[:, :self._max_legal]
        fs = torch.where(valid & ~chosen, priors, torch.full_like(priors, -1e30))
        f_order = torch.topk(fs, k, dim=1).indices
        f_keep = (k - per_game).clamp(min=0)
        f_valid = torch.arange(k, device=self.device).unsqueeze(0) < f_keep.unsqueeze(1)
        f_cand = torch.where(f_valid, f_order.to(torch.int32), torch.full_like(f_order, -1, dtype=torch.int32))
        return torch.cat([r_cand, f_cand], dim=1)[:, :k].contiguous()

    # fnn_mcts_orchestrator.py:982-1055
    def _run_simulations_for_root_slots(self, tree, root_states, game_active, root_slots, B, sims_per_slot,
                                        wave_size=None):
        cfg = self.config
        C = int(root_slots.shape[1])
        W = max(1, int(cfg.wave_size if wave_size is None else wave_size))
        q_pen = float(cfg.virtual_q_penalty) if cfg.deterministic_non_root and W > 1 else 0.0
        for wave in range(math.ceil(sims_per_slot / W)):
            aw = min(W, sims_per_slot - wave * W)
            total = aw * C * B
            leaf, leaf_states, legal, nl, feats, results, vlp, vll = \
                self.ext.mcts_select_replay_legal_fnn_root_slots_batch(
                    *self._tree_args(tree), tree["child_init_q"], root_states, game_active, tree["root_node"],
                    root_slots, C, self._max_legal, cfg.c_puct, B, aw, self._max_nodes, cfg.deterministic_non_root,
                    cfg.non_root_sigma, cfg.virtual_q_penalty)
            pri, vals, cq = self._eval_states(leaf_states, legal, nl, total, feats)
            self.sims_done += (leaf >= 0).sum()
            if self.trace is not None:
                self.trace.append(dict(kind="wave", root_slots=root_slots.clone(), W=aw, leaf=leaf.clone(),
                                       priors=pri.clone(),
                                       values=vals.clone(), child_q=cq.clone()))
            self.ext.mcts_expand_and_backprop_dense_priors_slots_batch(
                *self._tree_args(tree), tree["child_init_q"], cq, leaf, leaf_states, legal, nl, pri, results, vals,
                vlp, vll, tree["root_node"], root_slots, C, B, total, self._max_nodes, q_pen)

    def self_play_batch(self, start_states: torch.Tensor | None = None) -> list[list[FNNTrainingExample]]:
        """fnn_mcts_orchestrator.py:561-875"""
        cfg, dev = self.config, self.device
        B = cfg.batch_size
        states = (start_states.to(dev).contiguous().clone() if start_states is not None
                  else self.ext.create_initial_states(B, cfg.expansion_mask))
        tree = self._alloc_tree(B)
        active = torch.ones((B,), dtype=torch.bool, device=dev)
        move_numbers = torch.zeros((B,), dtype=torch.int64, device=dev)
        records = []  # per move: (states, probs, nl, has_actions, forced) on the host
        temps = []
        L = self._max_legal
        while bool(active.any().item()):
            legal, nl, root_feats = self.ext.generate_legal_moves_and_fnn_features_batch(states, B)
            n64 = nl.to(torch.int64)
            has_actions = active & (n64 > 0)
            active = active & ~(active & (n64 == 0))
            if int(n64.max().item()) == 0:
                break
            priors, _, child_q = self._eval_states(states, legal, nl, B, root_feats)
            valid_slot = self._slot_idx < n64.unsqueeze(1)
            forced = torch.zeros((B,), dtype=torch.bool, device=dev)
            allowed = valid_slot
            if cfg.short_forced_win_probe:
                win, allowed_t, forced_t = self.ext.root_tactical_probe_batch(
                    states, legal, nl, priors, B, cfg.probe_win_in_one, cfg.probe_check_opponent_wins,
                    cfg.probe_win_in_two)
                wins = win.to(torch.int64)
                allowed = allowed_t.to(torch.bool) & valid_slot
                forced = forced_t.to(torch.bool) & has_actions
            else:
                wins = self._find_immediate_wins(states, legal, nl, B)
            has_win = wins >= 0
            any_win = bool(has_win.any().item())
            if any_win:
                rows_w = torch.nonzero(has_win).squeeze(1)
                priors.zero_()
                priors[rows_w, wins[rows_w]] = 1.0
                child_q.zero_()
            search_rows = has_actions & ~has_win & ~forced
            legal_logits = torch.where(allowed, priors.clamp(min=1e-20).log(), torch.full_like(priors, -1e30))
            u = self._uniform(B, L).clamp(1e-4, 1 - 1e-4)
            gumbel = torch.where(allowed, -torch.log(-torch.log(u)), torch.full_like(u, -1e30))
            topk_slots = self._root_candidate_slots(states, legal, nl, priors, legal_logits, B, allowed)
            game_active = search_rows.to(torch.int8)
            if self.trace is not None:
                self.trace.append(dict(kind="root", states=states.clone(), legal=legal.clone(), nl=nl.clone(),
                                       priors=priors.clone(), child_q=child_q.clone(),
                                       game_active=game_active.clone()))
            self._expand_root_if_needed(tree, states, legal, nl, priors, child_q, game_active, B)
            self._apply_root_dirichlet(tree, B, search_rows)

            slot_visits = torch.zeros(B, L, dtype=torch.int32, device=dev)
            probs = torch.zeros(B, L, dtype=torch.float32, device=dev)
            chosen = torch.zeros((B,), dtype=torch.long, device=dev)
            if bool(search_rows.any().item()):
                cand = topk_slots.to(torch.int32)
                cidx = cand.long().clamp(min=0)
                cvalid = torch.gather(valid_slot, 1, cidx) & (cand >= 0)
                cand = torch.where(cvalid, cand, torch.full_like(cand, -1))
                per_round = max(1, cfg.num_simulations // _GUMBEL_ROUNDS)
                score_base = gumbel + legal_logits
                for r in range(_GUMBEL_ROUNDS):
                    slots = cand.contiguous()
                    cvalid = slots >= 0
                    C = int(slots.shape[1])
                    spc = max(1, per_round // C)
                    W = _GUMBEL_WAVE_SCHEDULE[min(r, len(_GUMBEL_WAVE_SCHEDULE) - 1)] if cfg.wave_parallel else 1
                    self._run_simulations_for_root_slots(tree, states, game_active, slots, B, spc, wave_size=W)
                    if C <= 1:
                        continue
                    per_keep = (cvalid.sum(dim=1) // 2).clamp(min=1)
                    max_keep = C // 2
                    cv, cq = self._root_stats(tree, B, slots, int(cfg.root_q_min_visits))
                    sigma = (cfg.c_visit + cv.max()) * cfg.c_scale
                    score = (torch.gather(score_base, 1, slots.long().clamp(min=0)) + sigma * cq).float()
                    score = torch.where(cvalid, score, torch.full_like(score, -1e30))
                    keep_pos = torch.topk(score, max_keep, dim=1).indices
                    kvalid = torch.arange(max_keep, device=dev).unsqueeze(0) < per_keep.unsqueeze(1)
                    ns = torch.gather(slots, 1, keep_pos)
                    cand = torch.where(kvalid, ns, torch.full_like(ns, -1))
                cvalid = cand >= 0
                cv, cq = self._root_stats(tree, B, cand, int(cfg.root_q_min_visits))
                sigma = (cfg.c_visit + cv.max()) * cfg.c_scale
                final = (torch.gather(score_base, 1, cand.long().clamp(min=0)) + sigma * cq).float()
                final = torch.where(cvalid, final, torch.full_like(final, -1e30))
                pos = torch.argmax(final, dim=1)
                chosen = torch.gather(cand, 1, pos.unsqueeze(1)).squeeze(1).clamp(min=0).to(torch.long)
                slot_visits, slot_q = self._root_stats(tree, B, self._slot_idx.expand(B, -1),
                                                       int(cfg.root_q_min_visits))
                visited = (slot_visits > 0) & valid_slot
                max_n = slot_visits.float().max(dim=1, keepdim=True).values
                sig = (cfg.c_visit + max_n) * cfg.c_scale
                sampled = torch.where(visited, legal_logits + sig * slot_q, torch.full_like(legal_logits, -1e30))
                probs, used = self._build_policy_target(sampled, valid_slot)
                tmask = search_rows & visited.any(dim=1)
                temps.append(used[tmask])
            if self.trace is not None:
                self.trace.append(dict(kind="searched", tree={k: v.clone() for k, v in tree.items()},
                                       chosen=chosen.clone(), probs=probs.clone()))
            if any_win:
                rows_w = torch.nonzero(has_win).squeeze(1)
                slot_visits[rows_w] = 0
                slot_visits[rows_w, wins[rows_w]] = cfg.num_simulations
                probs[rows_w] = 0.0
                probs[rows_w, wins[rows_w]] = 1.0
                chosen = torch.where(has_win, wins, chosen)
            if bool(forced.any().item()):
                rnd = (self._uniform(B) * n64.clamp(min=1).float()).to(torch.int64)
                chosen = torch.where(forced, rnd, chosen)
                probs = torch.where(forced.unsqueeze(1), torch.zeros_like(probs), probs)
            records.append((states.cpu().numpy(), probs.cpu().numpy(), nl.cpu().numpy(),
                            has_actions.cpu().numpy(), forced.cpu().numpy()))
            row = torch.arange(B, device=dev)
            move_bytes = torch.where(has_actions.unsqueeze(1), legal[row, chosen.clamp(max=L - 1)],
                                     torch.zeros((B, self._move_size), dtype=torch.uint8, device=dev)).contiguous()
            self.ext.apply_moves_batch(states, move_bytes, B)
            fc = tree["first_child"][row, tree["root_node"].long()]
            moved = has_actions & (fc >= 0)
            self._reroot_tree(tree, moved, fc + chosen.to(torch.int32))
            move_numbers = move_numbers + has_actions.to(torch.int64)
            results = self.ext.check_results_batch(states, B)
            active = active & (results == 0) & (move_numbers < cfg.max_game_length)
        final_results = self.ext.check_results_batch(states, B).cpu().numpy()
        if temps:
            t = torch.cat(temps).float().cpu().numpy()
            if t.size:
                self.last_policy_temperature_stats = {"mean": float(t.mean()), "min": float(t.min()),
                                                      "max": float(t.max()), "count": float(t.size)}
        return self._examples(records, final_results, B)

    def _examples(self, records, final_results, B):
        cfg = self.config
        histories = [[] for _ in range(B)]
        for st, pr, nl, has, forced in records:
            for i in range(B):
                if not has[i]:
                    continue
                n = int(nl[i])
                if forced[i]:
                    histories[i].append((st[i].copy(), np.zeros((n,), np.float32), False))
                else:
                    histories[i].append((st[i].copy(), pr[i, :n].astype(np.float32, copy=True), True))
        out = [[] for _ in range(B)]
        for i in range(B):
            winner = int(final_results[i])
            use_v = winner != 0
            w_from = len(histories[i]) - max(0, int(cfg.final_value_ply_count))
            for k, (sb, pi, use_p) in enumerate(histories[i]):
                turn = int(sb[_OFF_TURN]) | (int(sb[_OFF_TURN + 1]) << 8)
                vw = float(cfg.final_value_weight) if (use_v and k >= w_from and
                                                       float(cfg.final_value_weight) != 1.0) else 1.0
                out[i].append(FNNTrainingExample(sb, pi.astype(np.float32), float(_result_to_value(winner, turn)),
                                                 bool(use_p), use_v, vw))
        return out


class FNNPUCTOrchestrator(_SearchBase):
    """Plain PUCT MCTS with wave virtual loss (FNN leaf evaluation)."""

    def __init__(self, net: HiveFNN, config: FNNPUCTConfig | None = None, device: str = "cuda") -> None:
        self._setup(net, config or FNNPUCTConfig(), device)

    def self_play_batch(self, start_states: torch.Tensor | None = None) -> list[list[FNNTrainingExample]]:
        """fnn_puct_orchestrator.py:140-298"""
        cfg, dev = self.config, self.device
        B, L = cfg.batch_size, self._max_legal
        states = (start_states.to(dev).contiguous().clone() if start_states is not None
                  else self.ext.create_initial_states(B, cfg.expansion_mask))
        tree = self._alloc_tree(B)
        active = torch.ones((B,), dtype=torch.bool, device=dev)
        move_numbers = torch.zeros((B,), dtype=torch.int64, device=dev)
        records = []
        while bool(active.any().item()):
            legal, nl, root_feats = self.ext.generate_legal_moves_and_fnn_features_batch(states, B)
            n64 = nl.to(torch.int64)
            has_actions = active & (n64 > 0)
            active = active & ~(active & (n64 == 0))
            wins = self._find_immediate_wins(states, legal, nl, B)
            has_win = wins >= 0
            if int(n64.max().item()) == 0:
                break
            priors, _, child_q = self._eval_states(states, legal, nl, B, root_feats)
            any_win = bool(has_win.any().item())
            if any_win:
                rows_w = torch.nonzero(has_win).squeeze(1)
                priors.zero_()
                priors[rows_w, wins[rows_w]] = 1.0
                child_q.zero_()
            game_active = has_actions.to(torch.int8)
            if self.trace is not None:
                self.trace.append(dict(kind="root", states=states.clone(), legal=legal.clone(), nl=nl.clone(),
                                       priors=priors.clone(), child_q=child_q.clone(),
                                       game_active=game_active.clone()))
            self._expand_root_if_needed(tree, states, legal, nl, priors, child_q, game_active, B)
            self._apply_root_dirichlet(tree, B, has_actions)
            valid_slot = self._slot_idx < n64.unsqueeze(1)
            if any_win:
                probs = torch.zeros(B, L, dtype=torch.float32, device=dev)
                probs[rows_w, wins[rows_w]] = 1.0
            else:
                self._run_simulations(tree, states, game_active, valid_slot.to(torch.int8).contiguous(), B,
                                      cfg.num_simulations)
                if self.trace is not None:
                    self.trace.append(dict(kind="searched", tree={k: v.clone() for k, v in tree.items()}))
                visits, _ = self._root_stats(tree, B, self._slot_idx.expand(B, -1), 0)
                vf = visits.float()
                vsum = vf.sum(dim=1, keepdim=True)
                probs = torch.where(vsum > 0, vf / vsum.clamp(min=1.0), torch.zeros_like(vf))
                uni = valid_slot.float()
                uni = uni / uni.sum(dim=1, keepdim=True).clamp(min=1.0)
                probs = torch.where(vsum > 0, probs, uni)
            records.append((states.cpu().numpy(), probs.cpu().numpy(), nl.cpu().numpy(), has_actions.cpu().numpy()))
            chosen = torch.zeros((B,), dtype=torch.int64, device=dev)
            if any_win:
                chosen = torch.where(has_win, wins, chosen)
            else:
                greedy = move_numbers >= cfg.temperature_drop_move
                arg = probs.argmax(dim=1)
                sp = probs / probs.sum(dim=1, keepdim=True).clamp_min(1e-8)
                sp = torch.where(has_actions.unsqueeze(1), sp, torch.full_like(sp, 1.0 / L))
                samp = torch.multinomial(sp, 1, generator=self.gen).squeeze(1)
                chosen = torch.where(has_actions, torch.where(greedy, arg, samp), chosen)
            row = torch.arange(B, device=dev)
            move_bytes = torch.where(has_actions.unsqueeze(1), legal[row, chosen.clamp(max=L - 1)],
                                     torch.zeros((B, self._move_size), dtype=torch.uint8, device=dev)).contiguous()
            self.ext.apply_moves_batch(states, move_bytes, B)
            fc = tree["first_child"][row, tree["root_node"].long()]
            self._reroot_tree(tree, has_actions & (fc >= 0), fc + chosen.to(torch.int32))
            move_numbers = move_numbers + has_actions.to(torch.int64)
            results = self.ext.check_results_batch(states, B)
            active = active & (results == 0) & (move_numbers < cfg.max_game_length)
        final_results = self.ext.check_results_batch(states, B).cpu().numpy()
        hist = [[] for _ in range(B)]
        for st, pr, nl, has in records:
            for i in range(B):
                if has[i]:
                    hist[i].append((st[i].copy(), pr[i, :int(nl[i])].astype(np.float32, copy=True)))
        out = [[] for _ in range(B)]
        for i in range(B):
            winner = int(final_results[i])
            use_v = winner != 0
            w_from = len(hist[i]) - max(0, int(cfg.final_value_ply_count))
            for k, (sb, pi) in enumerate(hist[i]):
                turn = int(sb[_OFF_TURN]) | (int(sb[_OFF_TURN + 1]) << 8)
                vw = float(cfg.final_value_weight) if (use_v and k >= w_from and
                                                       float(cfg.final_value_weight) != 1.0) else 1.0
                out[i].append(FNNTrainingExample(sb, pi, float(_result_to_value(winner, turn)), True, use_v, vw))
        return out


# ---------------------------------------------------------------------------
# hybrid FNN-transformer drivers
# ---------------------------------------------------------------------------
@dataclass
class HybridMCTSConfig(FNNMCTSConfig):
    """hive_fnn_transformer/fnn_transformer_mcts_orchestrator.py:20-22."""


@dataclass
class HybridPUCTConfig(FNNPUCTConfig):
    """PUCT waves with the hybrid evaluator (the FNNPUCTConfig fields)."""


class HybridMCTSOrchestrator(FNNMCTSOrchestrator):
    """Gumbel-root MCTS with relative-transformer policy / value evaluation
    (fnn_transformer_mcts_orchestrator.py:25-169): child initial Q is zero."""

    def __init__(self, net, config: HybridMCTSConfig | None = None, device: str = "cuda") -> None:
        from .hybrid import HybridEvaluator
        super().__init__(net.fnn, config or HybridMCTSConfig(), device)
        self.net = net
        self.evaluator = HybridEvaluator(net, self.device)


class HybridPUCTOrchestrator(FNNPUCTOrchestrator):
    """PUCT MCTS (fnn_puct_orchestrator.py:140-386) with the hybrid evaluator."""

    def __init__(self, net, config: HybridPUCTConfig | None = None, device: str = "cuda") -> None:
        from .hybrid import HybridEvaluator
        super().__init__(net.fnn, config or HybridPUCTConfig(), device)
        self.net = net
        self.evaluator = HybridEvaluator(net, self.device)
