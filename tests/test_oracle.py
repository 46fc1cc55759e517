"""CPU tests: the oracle against the reference's golden vectors.

The oracle (oracle/hive_oracle.c) is pinned three ways:
1. bit-exact against tests/golden/golden_small.npz, produced by the
   reference's own headers compiled on the host (tests/golden/make_golden.py);
2. SHA-256 digests of the reference's outputs on the full config-1 set
   (4,096 base-game positions) and an 8,192-position all-expansion set;
3. live against oracle/_ref/libhive_ref.so on fresh seeds, where built;
plus the reference test-suite's known answers
(tests/test_gpu_move_gen.py:137-154: grid constants, 4 opening moves).
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def orc():
    return O.oracle()


@pytest.fixture(scope="module")
def small():
    return dict(np.load(os.path.join(GOLD, "golden_small.npz")))


def _digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _outputs(lib, states):
    moves, nl, feats = lib.legal_moves_features(states)
    cm, cn = lib.compact_moves(states)
    act, cen = lib.actions(states, moves, nl)
    roots = np.repeat(np.arange(states.shape[0], dtype=np.int64), nl)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in nl])
    succ = lib.successor_features(states, moves, roots, idx)
    return dict(moves=moves, num_legal=nl, features=feats, compact_moves=cm, compact_num=cn,
                articulation=lib.articulation(states), actions=act, centroids=cen,
                queen_escape=lib.queen_escape(states), succ_roots=roots, succ_moves=idx,
                succ_features=succ)


def test_known_answers_opening(orc):
    # reference tests/test_gpu_move_gen.py:148-154: turn 0 base game = 4 placements
    st = orc.generate_positions(1, 0, 1, 0, 0)  # stop ply 0 -> initial state
    moves, nl, feats = orc.legal_moves_features(st)
    assert nl[0] == 4
    assert [tuple(m) for m in moves[0, :4, :2]] == [(0, 2), (0, 3), (0, 4), (0, 5)]
    cells = {int(m[4]) | (int(m[5]) << 8) for m in moves[0, :4]}
    assert cells == {11 * 23 + 11}
    # with all expansions: 7 types (no queen on the first turn)
    st7 = orc.generate_positions(1, 0, 1, 0, 7)
    assert orc.legal_moves_features(st7)[1][0] == 7
    # turn 0 features: hands full, moves_to_draw 1, move_number 0
    assert feats[0, 102] == 1.0 and feats[0, 103] == 0.0
    assert np.all(feats[0, 16:26] == 1.0)


def test_oracle_matches_golden_small(orc, small):
    got = _outputs(orc, small["states"])
    for k, v in got.items():
        ref = small[k]
        if v.dtype == np.float32:
            assert np.array_equal(v.view(np.uint32), ref.view(np.uint32)), k
        else:
            assert np.array_equal(v, ref), k


@pytest.mark.parametrize("name", ["config1_base_4096", "expansions_8192"])
def test_oracle_matches_reference_digests(orc, name):
    with open(os.path.join(GOLD, "golden_digests.json")) as f:
        d = json.load(f)[name]
    p = d["params"]
    st = orc.generate_positions(p["seed"], p["first_game"], p["count"], p["max_ply"], p["expansion_mask"])
    assert _digest(st) == d["states"]
    o = _outputs(orc, st)
    assert _digest(o["moves"], o["num_legal"]) == d["moves"]
    assert _digest(o["features"]) == d["features"]
    assert _digest(o["compact_moves"], o["compact_num"]) == d["compact"]
    assert _digest(o["articulation"]) == d["articulation"]
    assert _digest(o["actions"], o["centroids"]) == d["actions"]
    assert _digest(o["queen_escape"]) == d["queen_escape"]
    assert _digest(o["succ_features"]) == d["successor_features"]
    hyb = orc.hybrid_encode(st, o["moves"], o["num_legal"])
    assert _digest(*hyb[:7]) == d["hybrid_tokens"]
    assert _digest(hyb[7]) == d["hybrid_move_features"]


@pytest.mark.skipif(not O.ref_available(), reason="reference host build not present")
@pytest.mark.parametrize("mask,max_ply", [(0, 60), (7, 120), (7, 200)])
def test_oracle_matches_reference_live(orc, mask, max_ply):
    ref = O.ref()
    st = ref.generate_positions(777 + mask + max_ply, 1000, 2048, max_ply, mask)
    assert np.array_equal(st, orc.generate_positions(777 + mask + max_ply, 1000, 2048, max_ply, mask))
    a, b = _outputs(orc, st), _outputs(ref, st)
    for k in a:
        if a[k].dtype == np.float32:
            assert np.array_equal(a[k].view(np.uint32), b[k].view(np.uint32)), k
        else:
            assert np.array_equal(a[k], b[k]), k


def test_oracle_apply_matches_golden_transitions(orc, small):
    # every legal move of every golden position, applied by the oracle, has
    # successor features equal to the reference's (checked above); here the
    # successor states themselves are checked to stay internally consistent
    st = small["states"]
    nl = small["num_legal"]
    moves = small["moves"]
    picks = np.array([moves[i, (7 * i) % max(1, nl[i])] for i in range(len(st))], np.uint8)
    after = orc.apply_moves(st, picks)
    occ = after[:, 3176:3176 + 72].copy().view(np.uint64)
    heights = after[:, 2645:2645 + 529]
    for i in range(len(st)):
        bits = np.unpackbits(occ[i].view(np.uint8), bitorder="little")[:529]
        assert np.array_equal(bits.astype(bool), heights[i] > 0)


@pytest.mark.skipif(not O.ref_available(), reason="reference host build not present")
def test_action_indices_give_the_reference_legal_mask(orc):
    """The dense mask built from the oracle's action indices equals the reference's
    legal_mask_kernel output (the GPU mask test builds its expectation the same way)."""
    st = np.concatenate([orc.generate_positions(515, 0, 256, 60, 0), orc.generate_positions(516, 0, 256, 150, 7)])
    mo, no, _ = orc.legal_moves_features(st)
    act, _ = orc.actions(st, mo, no)
    want = np.zeros((len(st), 85834), np.float32)
    for i in range(len(st)):
        a = act[i, :no[i]]
        want[i, a[a >= 0]] = 1.0
    assert np.array_equal(O.ref().legal_mask(st, mo, no), want)


def test_oracle_matches_reference_edge_fixtures(orc):
    """The C oracle on the reference's edge-case fixtures (move lists cut at
    256, 5-high stacks, grid edge, pillbug / mosquito rule scenarios;
    tests/golden/make_edge_golden.py), every output bit-exact."""
    g = dict(np.load(os.path.join(GOLD, "golden_edge.npz")))
    with open(os.path.join(GOLD, "golden_edge.json")) as f:
        d = json.load(f)
    st = g["states"]
    o = _outputs(orc, st)
    for k in ("moves", "num_legal", "compact_moves", "compact_num", "articulation", "actions", "centroids"):
        assert np.array_equal(o[k], g[k]), k
    assert np.array_equal(o["features"].view(np.uint32), g["features"].view(np.uint32))
    offs = np.concatenate([[0], np.cumsum(o["num_legal"])])
    hyb = orc.hybrid_encode(st, o["moves"], o["num_legal"])
    for i in range(len(st)):
        n = int(o["num_legal"][i])
        assert _digest(o["succ_features"][offs[i]:offs[i + 1]]) == d["successor_features"][i], g["case"][i]
        kids = orc.apply_moves(np.repeat(st[i:i + 1], n, 0), o["moves"][i, :n])
        assert _digest(kids) == d["successor_states"][i], g["case"][i]
        assert _digest(*(a[i:i + 1] for a in hyb[:7])) == d["hybrid_tokens"][i], g["case"][i]
        assert _digest(hyb[7][i, :n]) == d["hybrid_move_features"][i], g["case"][i]


@pytest.mark.skipif(not O.ref_available(), reason="reference build not present")
def test_oracle_tactical_probe_matches_reference_on_edge_fixtures(orc):
    g = dict(np.load(os.path.join(GOLD, "golden_edge.npz")))
    st, mv, nl = g["states"], g["moves"], g["num_legal"]
    rng = np.random.default_rng(17)
    pri = rng.uniform(0.01, 1, (len(st), 256)).astype(np.float32)
    pri = np.where(np.arange(256)[None, :] < nl[:, None], pri, 0).astype(np.float32)
    for a, b in zip(orc.tactical_probe(st, mv, nl, pri), O.ref().tactical_probe(st, mv, nl, pri)):
        assert np.array_equal(a, b)
