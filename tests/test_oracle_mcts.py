"""CPU tests: the MCTS oracle restatement against the reference's tree kernels
(hive_gpu/csrc/mcts_tree.cuh) executed sequentially in simulation order."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.mcts_sim import OracleBackend, run_waves

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference host build not present")


def _states(seed, n=24):
    orc = O.oracle()
    return np.concatenate([orc.generate_positions(seed, 0, n // 2, 40, 0),
                           orc.generate_positions(seed + 1, 0, n - n // 2, 90, 7)])


@needs_ref
@pytest.mark.parametrize("mode,W,det", [(0, 1, False), (0, 4, False), (1, 3, False), (2, 2, False),
                                        (2, 4, False), (1, 4, True), (2, 3, True)])
def test_oracle_tree_matches_reference(mode, W, det):
    st = _states(100 + mode * 10 + W)
    a, la = run_waves(OracleBackend("orc"), st, waves=6, W=W, mode=mode, seed=7, det=det,
                      q_penalty=0.25 if det else 0.0)
    b, lb = run_waves(OracleBackend("ref"), st, waves=6, W=W, mode=mode, seed=7, det=det,
                      q_penalty=0.25 if det else 0.0)
    assert a.equal(b) == []
    for (x1, y1, z1), (x2, y2, z2) in zip(la, lb):
        assert np.array_equal(x1, x2) and np.array_equal(y1, y2) and np.array_equal(z1, z2)
    assert a.visit_count[:, 0].max() > 0


@needs_ref
def test_oracle_action_space_path_matches_reference():
    orc = O.oracle()
    st = _states(5, 16)
    B = len(st)
    rng = np.random.default_rng(3)
    trees = {n: O.TreeArrays(B, 2048) for n in ("orc", "ref")}
    mv, nl, _ = orc.legal_moves_features(st)
    res = st[:, 3415].astype(np.int32)
    probs = rng.uniform(size=(B, 85834)).astype(np.float32)
    for n, t in trees.items():
        was = O.mcts_expand_action(n, t, 0, np.zeros(B, np.int32), st, mv, nl, probs, res)
        O.mcts_expand_action(n, t, 2, np.zeros(B, np.int32), st, mv, nl, probs, res,
                             values=np.full(B, 0.5, np.float32), was_expanded=was)
    for wave in range(4):
        out = {}
        for n, t in trees.items():
            leaf, paths, plen, vlp, vll = O.mcts_select(n, t, mode=0, game_active=np.ones(B, np.int8),
                                                        root_nodes=np.zeros(B, np.int32), W=2)
            ls = O.mcts_replay(n, st, paths, plen, leaf, B)
            lmv, lnl, _ = orc.legal_moves_features(ls)
            vals = np.linspace(-0.9, 0.9, len(leaf)).astype(np.float32)
            lp = np.random.default_rng(wave).uniform(size=(len(leaf), 85834)).astype(np.float32)
            O.mcts_expand_action(n, t, 1, leaf, ls, lmv, lnl, lp, ls[:, 3415].astype(np.int32), vals, vlp, vll)
            out[n] = leaf
        assert np.array_equal(out["orc"], out["ref"])
    assert trees["orc"].equal(trees["ref"]) == []
    for temp, drop, prune in [(1.0, 30, 0.0), (0.5, 30, 0.1), (1.0, 0, 0.0)]:
        pa = O.mcts_extract_policy("orc", trees["orc"], np.zeros(B), np.zeros(B), temp, drop, prune)
        pb = O.mcts_extract_policy("ref", trees["ref"], np.zeros(B), np.zeros(B), temp, drop, prune)
        assert np.array_equal(pa.view(np.uint32), pb.view(np.uint32))
    noise = np.random.default_rng(9).dirichlet(np.full(256, 0.3), size=B).astype(np.float32)
    for temp in (1.0, 1.5):
        O.mcts_root_noise("orc", trees["orc"], noise, np.zeros(B), 0.25, temp)
        O.mcts_root_noise("ref", trees["ref"], noise, np.zeros(B), 0.25, temp)
        assert trees["orc"].equal(trees["ref"]) == []
