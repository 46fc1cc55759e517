"""Test helper: drive several MCTS waves through a tree backend.

A backend provides select / replay / expand_dense with the numpy-level
signatures of oracle/oracle.py (the sequential C restatement "orc", the
reference kernels run sequentially "ref", or the B200 kernels "gpu" in
tests/test_mcts_gpu.py).  Leaf priors, child Q and values are seeded random
numbers (the tree kernels do not care where they come from), legal moves and
results come from the oracle, so the final trees of two backends must be
bit-identical.
"""
from __future__ import annotations

import numpy as np

from oracle import oracle as O


class OracleBackend:
    def __init__(self, name: str):
        self.name = name

    def select(self, tree, **kw):
        return O.mcts_select(self.name, tree, **kw)

    def replay(self, root_states, paths, plen, leaf, B):
        return O.mcts_replay(self.name, root_states, paths, plen, leaf, B)

    def expand_dense(self, tree, *args, slots=None, **kw):
        # (the oracle's sequential expansion serves the root-slot waves too)
        return O.mcts_expand_dense(self.name, tree, *args, **kw)


def _priors(rng, nl):
    logits = rng.normal(size=(len(nl), 256)).astype(np.float32)
    valid = np.arange(256)[None, :] < nl[:, None]
    logits = np.where(valid, logits, -1e30).astype(np.float32)
    e = np.where(valid, np.exp(logits - logits.max(1, keepdims=True)), 0).astype(np.float32)
    s = e.sum(1, keepdims=True)
    return np.where(valid, e / np.maximum(s, 1e-30), 0).astype(np.float32)


def run_waves(backend, states: np.ndarray, waves: int, W: int, mode: int, seed: int, C: int = 4,
              max_nodes: int = 4096, det: bool = False, q_penalty: float = 0.0, c_puct: float = 1.25,
              repeat_slots: bool = False, grouped: bool = True):
    orc = O.oracle()
    B = states.shape[0]
    rng = np.random.default_rng(seed)
    tree = O.TreeArrays(B, max_nodes)
    mv, nl, _ = orc.legal_moves_features(states)
    results = states[:, 3415].astype(np.int32)
    valid = np.arange(256)[None, :] < nl[:, None]
    child_q = np.where(valid, rng.uniform(-1, 1, (B, 256)), 0).astype(np.float32)
    backend.expand_dense(tree, child_q, np.zeros(B, np.int32), states, mv, nl, _priors(rng, nl), results,
                         with_backprop=False)
    active = ((results == 0) & (nl > 0)).astype(np.int8)
    roots = np.zeros(B, np.int32)
    log = []
    for w in range(waves):
        kw = dict(mode=mode, game_active=active, root_nodes=roots, W=W, det=det, q_penalty=q_penalty,
                  c_puct=c_puct)
        if mode == 1:
            kw["alive_mask"] = (rng.uniform(size=(B, 256)) < 0.6).astype(np.int8)
            kw["max_root_children"] = 256
        if mode == 2:
            slots = np.stack([rng.permutation(256)[:C] for _ in range(B)]).astype(np.int32)
            slots = np.where(slots < nl[:, None], slots, -1).astype(np.int32)
            slots[:, 0] = np.where(nl > 0, rng.integers(0, np.maximum(nl, 1)), -1)
            if repeat_slots:  # every other game lists its first candidate twice
                slots[::2, 1] = slots[::2, 0]
            kw.update(root_slots=slots, num_candidates=C, max_root_children=256)
        leaf, paths, plen, vlp, vll = backend.select(tree, **kw)
        ls = backend.replay(states, paths, plen, leaf, B)
        lmv, lnl, _ = orc.legal_moves_features(ls)
        lres = ls[:, 3415].astype(np.int32)
        lvalid = np.arange(256)[None, :] < lnl[:, None]
        cq = np.where(lvalid, rng.uniform(-1, 1, (len(leaf), 256)), 0).astype(np.float32)
        vals = rng.uniform(-1, 1, len(leaf)).astype(np.float32)
        backend.expand_dense(tree, cq, leaf, ls, lmv, lnl, _priors(rng, lnl), lres, vals, vlp, vll,
                             q_penalty=q_penalty if det and W > 1 else 0.0, with_backprop=True,
                             slots=(roots, kw["root_slots"] if mode == 2 else None, C) if grouped else None)
        log.append((leaf.copy(), plen.copy(), vll.copy()))
    return tree, log
