"""CPU restatement of the reference's FNN CPU player (TEST INFRASTRUCTURE ONLY).

The reference's CPU path for the Gumbel search, ``FNNNativeCPUPlayer``
(hive_fnn/fnn_native_cpu_player.py:72-281), is a Python tree search over the
reference's native state backend (hive_gpu/csrc/cpu_native.cpp, bound as
``hive_cpu_native_ext``) with a torch CPU FNN.  This module restates that
search step for step and runs it over the same native backend, compiled from
the reference's own source into oracle/_ref by ``make -C oracle ref-player``:

* ``evaluate`` -- cpu_native's legal moves + root features, successor
  features / states / results of every legal move (the full move list,
  cpu_native.cpp:130-174), FNN encode, root value, action scores, softmax
  over the legal moves (fnn_native_cpu_player.py:126-157);
* ``expand`` / ``select`` / ``backup`` -- one node per legal move, PUCT with
  sqrt(max(1, N)), the first maximum kept, values alternating in sign up the
  path (:159-209);
* ``gumbel_search`` -- top-k of log prior + scaled Gumbel noise, ceil(log2 k)
  rounds of sequential halving with sims_per_round // k' simulations under
  each candidate, score log prior + noise + (c_visit + max N) * c_scale * Q,
  final argmax (:211-266).

tests/test_cpu_player.py pins it to the reference player itself (same chosen
moves and root visit counts) where the reference tree exists.  Only the
tests and bench.py's cpu_baseline leg use it; the product path never does.
"""
from __future__ import annotations

import glob
import importlib.util
import math
import os
import sys
import time
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def backend_path() -> str | None:
    hits = glob.glob(os.path.join(HERE, "_ref", "hive_cpu_native_ext*.so"))
    return hits[0] if hits else None


def load_backend():
    """The reference's cpu_native extension built into oracle/_ref (None if absent)."""
    path = backend_path()
    if path is None:
        return None
    if "hive_cpu_native_ext" in sys.modules:
        return sys.modules["hive_cpu_native_ext"]
    import torch  # noqa: F401  (the extension links libtorch)
    spec = importlib.util.spec_from_file_location("hive_cpu_native_ext", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules["hive_cpu_native_ext"] = mod
    return mod


@dataclass
class PlayerConfig:
    """Fields and defaults of FNNNativeCPUConfig (fnn_native_cpu_player.py:16-24)."""

    num_simulations: int = 512
    c_puct: float = 1.25
    c_visit: float = 50.0
    c_scale: float = 1.0
    use_gumbel_root: bool = True
    gumbel_considered: int = 16
    gumbel_noise_scale: float = 0.0


class _Stop(Exception):
    pass


class Node:
    __slots__ = ("state", "parent", "move", "prior", "n", "w", "kids", "moves", "expanded", "result")

    def __init__(self, state: bytes, parent=None, move=None, prior=0.0, result=0):
        self.state = state
        self.parent = parent
        self.move = move
        self.prior = float(prior)
        self.n = 0
        self.w = 0.0
        self.kids: list[Node] = []
        self.moves = None
        self.expanded = False
        self.result = int(result)

    def q(self) -> float:
        return self.w / self.n if self.n else 0.0


def _value_of_result(result: int, state: bytes) -> float:
    if result in (0, 3):
        return 0.0
    white = ((state[3412] | (state[3413] << 8)) % 2) == 0
    return 1.0 if (result == 1 and white) or (result == 2 and not white) else -1.0


class CPUPlayer:
    """One game's search; ``sims`` counts simulations run (leaf visits)."""

    def __init__(self, net, config: PlayerConfig, backend=None, deadline: float | None = None):
        import torch
        self.torch = torch
        self.net = net.eval()
        self.cfg = config
        self.ext = backend or load_backend()
        if self.ext is None:
            raise RuntimeError("reference cpu_native backend not built (make -C oracle ref-player)")
        self.deadline = deadline
        self.sims = 0

    def evaluate(self, node: Node):
        mv, n, rf = self.ext.legal_moves_and_fnn_features(node.state)
        n = int(n)
        moves = np.asarray(mv, np.uint8)[:n].copy()
        if n <= 0:
            return moves, np.zeros(0, np.float32), 0.0, [], np.zeros(0, np.int32)
        sf, kid_states, kid_res = self.ext.successor_features(node.state, moves, n)
        torch = self.torch
        with torch.inference_mode():
            re = self.net.encode(torch.from_numpy(np.asarray(rf, np.float32).copy()).unsqueeze(0))
            se = self.net.encode(torch.from_numpy(np.asarray(sf, np.float32)))
            value = float(self.net.value_head(re).squeeze().item())
            logits = self.net.score_actions(re.expand(se.shape[0], -1), se).float()
            priors = torch.softmax(logits, dim=0).numpy().astype(np.float32)
        return moves, priors, value, list(kid_states), np.asarray(kid_res, np.int32)

    def _make_children(self, node: Node, moves, priors, kid_states, kid_res) -> None:
        node.moves = moves
        node.kids = [Node(kid_states[i], node, moves[i].copy(), priors[i], kid_res[i]) for i in range(len(moves))]
        node.expanded = True

    def expand(self, node: Node) -> float:
        if node.result != 0:
            return _value_of_result(node.result, node.state)
        moves, priors, value, kid_states, kid_res = self.evaluate(node)
        self._make_children(node, moves, priors, kid_states, kid_res)
        return value

    def select(self, node: Node) -> Node:
        sq = math.sqrt(max(1, node.n))
        best, best_s = node.kids[0], -1e30
        for k in node.kids:
            s = (-k.q() if k.n > 0 else 0.0) + self.cfg.c_puct * k.prior * sq / (1 + k.n)
            if s > best_s:
                best, best_s = k, s
        return best

    @staticmethod
    def backup(node: Node, value: float) -> None:
        while node is not None:
            node.n += 1
            node.w += value
            value = -value
            node = node.parent

    def search_under(self, root: Node, sims: int) -> None:
        for _ in range(max(0, int(sims))):
            if self.deadline is not None and time.perf_counter() > self.deadline:
                raise _Stop
            node = root
            while node.expanded and node.kids:
                node = self.select(node)
            value = node.q() if node.expanded else self.expand(node)
            self.backup(node, value)
            self.sims += 1

    def gumbel_search(self, root: Node) -> int:
        cfg = self.cfg
        moves, priors, _, kid_states, kid_res = self.evaluate(root)
        if len(moves) == 0:
            root.moves = moves
            return -1
        self._make_children(root, moves, priors, kid_states, kid_res)
        k = min(int(cfg.gumbel_considered), len(moves))
        rounds = max(1, math.ceil(math.log2(max(k, 1))))
        per_round = max(1, int(cfg.num_simulations) // rounds)
        logp = np.log(np.clip(priors, 1e-30, None))
        u = np.clip(np.random.random(len(moves)), 1e-12, 1.0 - 1e-12)
        base = logp + (-np.log(-np.log(u)) * float(cfg.gumbel_noise_scale)).astype(np.float32)
        cand = np.argsort(base)[-k:][::-1].tolist()

        def scores(ids):
            n = np.array([root.kids[i].n for i in ids], np.float32)
            q = np.array([-root.kids[i].q() for i in ids], np.float32)
            sigma = (float(cfg.c_visit) + float(n.max())) * float(cfg.c_scale)
            return np.array([base[i] for i in ids], np.float32) + sigma * q

        for _ in range(rounds):
            if len(cand) <= 1:
                break
            spc = max(1, per_round // len(cand))
            for i in cand:
                self.search_under(root.kids[i], spc)
            keep = max(1, len(cand) // 2)
            order = np.argsort(scores(cand))[-keep:][::-1]
            cand = [cand[i] for i in order]
        if len(cand) == 1:
            return int(cand[0])
        return int(cand[int(np.argmax(scores(cand)))])

    def choose_move(self, state: bytes) -> np.ndarray:
        root = Node(state, result=int(self.ext.check_result(state)))
        if self.cfg.use_gumbel_root:
            i = self.gumbel_search(root)
            return np.zeros(6, np.uint8) if i < 0 or root.moves is None else root.moves[i].copy()
        self.search_under(root, self.cfg.num_simulations)
        if not root.kids:
            return np.zeros(6, np.uint8)
        return root.moves[int(np.argmax([k.n for k in root.kids]))].copy()


def _worker(args):
    """One process, one game at a time, torch on one thread: simulations run
    before the deadline."""
    import torch
    states, sims, seed, seconds = args
    torch.set_num_threads(1)
    sys.path.insert(0, os.path.dirname(HERE))
    from hive_neuralnet_b200.fnn import HiveFNN
    torch.manual_seed(0)
    net = HiveFNN()
    np.random.seed(seed)
    t0 = time.perf_counter()
    player = CPUPlayer(net, PlayerConfig(num_simulations=sims), deadline=t0 + seconds)
    moves = 0
    try:
        while True:
            for st in states:
                player.choose_move(bytes(st))
                moves += 1
    except _Stop:
        pass
    return player.sims, time.perf_counter() - t0, moves


def timed_rate(states: np.ndarray, sims: int, processes: int, seconds: float):
    """Simulations per second of the reference CPU player, one game per
    process over `processes` spawned processes for about `seconds`."""
    import multiprocessing as mp
    chunks = [states[i::processes] for i in range(processes)]
    ctx = mp.get_context("spawn")
    with ctx.Pool(processes) as pool:
        out = pool.map(_worker, [(c, sims, 1000 + i, seconds) for i, c in enumerate(chunks) if len(c)])
    done = sum(o[0] for o in out)
    wall = max(o[1] for o in out)
    return done / wall, done, wall, sum(o[2] for o in out)
