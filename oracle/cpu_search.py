"""CPU restatement of the self-play search, timed as the host-CPU baseline.

TEST INFRASTRUCTURE ONLY: bench.py's cpu_baseline legs (configs 3-5) time
it on a bounded sample, tests use its evaluators as fp32 checkers.  Nothing
in hive_neuralnet_b200 imports it.

One search = PUCT waves over the sequential C restatement of the
reference's tree kernels (oracle/hive_oracle_mcts.c: select with the root
alive mask, replay, dense-prior expand + backup), the C oracle's move
generation, features and successor features (OpenMP over all host threads)
and an fp32 torch CPU leaf evaluator:

* FNN (hive_fnn/fnn_mcts_orchestrator.py:243-316) -- fnn_reference.py;
* hybrid FNN-transformer (hive_fnn_transformer/
  fnn_transformer_mcts_orchestrator.py:42-169) -- :func:`hybrid_eval`.

Per simulation this is the same work the B200 path does (select, replay,
leaf move generation + root features, one successor-feature row per legal
move, network, expand, backup); the Gumbel root's sequential halving adds
only per-move root work, so the same loop stands in for configs 4 and 5.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import oracle as O
from .fnn_reference import eval_states_reference


def _successors(orc, states, moves, nl):
    roots = np.repeat(np.arange(len(states), dtype=np.int64), nl)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in nl]) if len(nl) else np.zeros(0, np.int64)
    return orc.successor_features(states, moves, roots, idx), roots


def fnn_eval(net, orc, states, moves, nl, feats):
    """(priors, values, child_q) of the FNN evaluator in fp32 on the CPU."""
    sf, _ = _successors(orc, states, moves, nl)
    pri, val, cq, _ = eval_states_reference(net, feats, sf, nl)
    return pri, val, cq


def hybrid_eval(net, orc, states, moves, nl, feats):
    """(priors, values, child_q = 0) of the hybrid evaluator in fp32 on the CPU."""
    from hive_neuralnet_b200.hybrid import HybridPieceTensorBatch
    sf, roots = _successors(orc, states, moves, nl)
    tf, tq, tr, tz, tm, gf, nt, mf = orc.hybrid_encode(states, moves, nl)
    d = net.config.node_feat_dim
    pb = HybridPieceTensorBatch(torch.from_numpy(tf[..., :d]), torch.from_numpy(tq).long(),
                                torch.from_numpy(tr).long(), torch.from_numpy(tz).long(),
                                torch.from_numpy(tm).bool(), torch.from_numpy(gf), torch.from_numpy(nt))
    valid = np.arange(256)[None, :] < nl[:, None]
    with torch.no_grad():
        lg, vals = net(torch.from_numpy(feats), torch.from_numpy(sf), torch.from_numpy(roots),
                       torch.from_numpy(nl.astype(np.int64)), pb, torch.from_numpy(mf[valid]))
    logits = torch.full((len(states), 256), -1e30)
    logits[torch.from_numpy(valid)] = lg
    pri = torch.softmax(logits, dim=1).numpy() * valid
    return pri.astype(np.float32), vals.numpy().reshape(-1), np.zeros((len(states), 256), np.float32)


def puct_search(evaluate, root_states: np.ndarray, sims: int, wave: int, c_puct: float,
                max_nodes: int = 16384) -> int:
    """Run ``sims`` simulations per root in waves of ``wave``; returns the
    number of simulations that reached a leaf."""
    orc = O.oracle()
    B = len(root_states)
    tree = O.TreeArrays(B, max_nodes)
    mv, nl, feats = orc.legal_moves_features(root_states)
    pri, _, cq = evaluate(root_states, mv, nl, feats)
    res = root_states[:, 3415].astype(np.int32)
    O.mcts_expand_dense("orc", tree, cq, np.zeros(B, np.int32), root_states, mv, nl, pri, res,
                        with_backprop=False)
    active = ((res == 0) & (nl > 0)).astype(np.int8)
    alive = (np.arange(256)[None, :] < nl[:, None]).astype(np.int8)
    roots = np.zeros(B, np.int32)
    done = 0
    for w0 in range(0, sims, wave):
        W = min(wave, sims - w0)
        leaf, paths, plen, vlp, vll = O.mcts_select("orc", tree, mode=1, game_active=active, root_nodes=roots,
                                                    alive_mask=alive, W=W, c_puct=c_puct)
        ls = O.mcts_replay("orc", root_states, paths, plen, leaf, B)
        lmv, lnl, lf = orc.legal_moves_features(ls)
        lpri, lval, lcq = evaluate(ls, lmv, lnl, lf)
        O.mcts_expand_dense("orc", tree, lcq, leaf, ls, lmv, lnl, lpri, ls[:, 3415].astype(np.int32), lval, vlp,
                            vll)
        done += int((leaf >= 0).sum())
    return done


def timed_search(evaluate, root_states, sims, wave, c_puct, min_seconds=10.0):
    """Repeat the search on the sample until ``min_seconds`` of work; (sims/s, sims, seconds)."""
    total, t0 = 0, time.perf_counter()
    while True:
        total += puct_search(evaluate, root_states, sims, wave, c_puct)
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            return total / dt, total, dt
