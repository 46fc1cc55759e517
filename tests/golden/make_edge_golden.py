"""Edge-case fixtures from the REFERENCE itself (run where the reference tree
exists; see oracle.reference_dir()).

Random playouts almost never reach the limits of the reference's move
generator, so this script searches for positions that do, by seeded beam
searches over legal play and by filtering seeded playouts, and records the
reference build's outputs (oracle/_ref: the reference's hive_gpu/csrc headers
compiled on the host) for each of them:

* ``cap256``   -- the side to move has 256 legal moves: the list is cut at
  MAX_LEGAL_MOVES (hive_gpu/csrc/move_gen.cuh:351, :1188-1357);
* ``stack5``   -- a 5-high stack (MAX_STACK, hive_state.cuh:75) with a
  beetle or mosquito of the side to move beside it, so a climb onto it is
  generated and applying it meets the refusal of a 6th piece (:331, :400);
* ``stack4``   -- 4-high stacks (one below the cap);
* ``edge``     -- pieces on the outermost rows or columns of the 23x23 grid,
  where destinations off the grid are dropped (hex_grid.cuh:57-161);
* ``pill_stunned``  -- the side to move's pillbug sits on the stunned cell
  with a throwable neighbour (the reference lets it throw: the throw pass,
  move_gen.cuh:1308-1345, does not test the thrower against the stunned cell);
* ``pill_pinned``   -- the side to move's pillbug is an articulation point
  (it cannot move, it can still throw);
* ``pill_covered``  -- a pillbug under a beetle (not the top piece: no throws);
* ``mosq_pill``     -- a ground mosquito of the side to move beside a
  pillbug (it copies the pillbug's throw, move_gen.cuh:907-1008);
* ``stunned_next_pill`` -- the piece on the stunned cell is beside the side
  to move's pillbug (a piece that just moved cannot be thrown).

The MAX_ANT_DESTS cap (128, move_gen.cuh:29, :271) has no case: an ant's
destinations are empty cells adjacent to the other pieces, and a connected
group of n hex cells has at most 2n + 4 such cells, so with at most 27 other
pieces an ant reaches at most 58 cells (and a mosquito's union at most 64).

Recorded per position: state bytes, the full move list, num_legal, the 122
features, the compact successor list, articulation points, action indices
and centroids; per position SHA-256 digests of the successor features of
every legal move, of the successor states (apply_move of every legal move)
and of their game results, and of the hybrid transformer inputs.

    python tests/golden/make_edge_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

SEED = 20261202
OFF_HEIGHT, OFF_TURN, OFF_RESULT, OFF_STUN = 2645, 3412, 3415, 3416
T_BEETLE, T_MOSQ, T_PILL = 5, 6, 8
DIRS = ((1, 0), (1, -1), (0, -1), (-1, 0), (-1, 1), (0, 1))  # (dq, dr) = (dcol, drow)

# neighbour table of the 23x23 grid, -1 off the grid
NEIGH = np.full((529, 6), -1, np.int64)
for _c in range(529):
    _r, _q = divmod(_c, 23)
    for _d, (_dq, _dr) in enumerate(DIRS):
        if 0 <= _r + _dr < 23 and 0 <= _q + _dq < 23:
            NEIGH[_c, _d] = (_r + _dr) * 23 + _q + _dq


def heights(st):
    return st[:, OFF_HEIGHT:OFF_HEIGHT + 529].astype(np.int64)


def tops(st):
    """Top piece byte of every cell (0 where empty)."""
    h = heights(st)
    lv = st[:, :5 * 529].reshape(-1, 5, 529)
    idx = np.clip(h - 1, 0, 4)
    t = np.take_along_axis(lv, idx[:, None, :], 1)[:, 0, :]
    return np.where(h > 0, t, 0)


def side(st):
    return (st[:, OFF_TURN].astype(np.int64) | (st[:, OFF_TURN + 1].astype(np.int64) << 8)) & 1


def stunned(st):
    return st[:, OFF_STUN].astype(np.int64) | (st[:, OFF_STUN + 1].astype(np.int64) << 8)


def nbr_vals(arr, cells):
    """arr [n, 529] gathered at the 6 neighbours of cells [n] -> [n, 6] (-1 off the grid)."""
    nb = NEIGH[cells]
    v = np.take_along_axis(arr, np.clip(nb, 0, 528), 1)
    return np.where(nb >= 0, v, -1)


def climber_beside(st, cell_mask):
    """Rows where a top beetle / mosquito of the side to move stands next to a cell of cell_mask."""
    t = tops(st)
    own = ((t >> 4) & 1) == side(st)[:, None]
    climb = own & (((t & 15) == T_BEETLE) | ((t & 15) == T_MOSQ)) & (heights(st) > 0)
    ok = np.zeros(len(st), bool)
    for d in range(6):
        nb = NEIGH[:, d]
        shifted = np.where(nb[None, :] >= 0, np.take(cell_mask, np.clip(nb, 0, 528), axis=1), False)
        ok |= (climb & shifted).any(1)
    return ok


def children(lib, frontier, rng=None, sample=None):
    """Every (or, with `sample`, up to `sample` seeded random) legal successor
    of each state whose game is not over."""
    mv, nl, _ = lib.legal_moves_features(frontier)
    roots = np.repeat(np.arange(len(frontier)), nl)
    idx = np.concatenate([np.arange(n) for n in nl]) if len(nl) else np.zeros(0, np.int64)
    if sample is not None:
        sel, start = [], 0
        for n in nl:
            sel.extend(start + rng.choice(n, min(n, sample), replace=False))
            start += n
        sel = np.asarray(sel, np.int64)
        roots, idx = roots[sel], idx[sel]
    kids = lib.apply_moves(frontier[roots], mv[roots, idx])
    return kids[kids[:, OFF_RESULT] == 0]


def beam(lib, starts, score, width, depth, rng, reply_sample=None):
    """Beam search over legal play: keep the `width` states with the highest
    score (seeded jitter breaks ties); returns every state scored.  With
    `reply_sample`, one step is a move of the side to move followed by up to
    `reply_sample` random replies, so the score always rates the same side."""
    frontier, seen, out = starts, set(), []
    for _ in range(depth):
        kids = children(lib, frontier)
        if reply_sample is not None and len(kids):
            kids = children(lib, kids, rng, reply_sample)
        keep = []
        for i, k in enumerate(kids):
            h = hashlib.sha1(k.tobytes()).digest()
            if h not in seen:
                seen.add(h)
                keep.append(i)
        kids = kids[keep]
        if len(kids) == 0:
            break
        out.append(kids)
        s = score(lib, kids) + rng.uniform(0, 0.5, len(kids))
        frontier = kids[np.argsort(-s, kind="stable")[:width]]
    return np.concatenate(out) if out else np.zeros((0, 3424), np.uint8)


def score_moves(lib, st):
    _, nl, _ = lib.legal_moves_features(st)
    return nl.astype(np.float64)


def score_stack(lib, st):
    """Tallest stack first, then a beetle / mosquito of the side to move beside
    it, then climbers of either side beside it, then the number of stacks."""
    h = heights(st)
    mx = h.max(1)
    top = h == mx[:, None]
    t = tops(st)
    climb = (((t & 15) == T_BEETLE) | ((t & 15) == T_MOSQ)) & (h > 0)
    near = np.zeros(len(st), np.int64)
    for d in range(6):
        nb = NEIGH[:, d]
        shifted = np.where(nb[None, :] >= 0, np.take(top, np.clip(nb, 0, 528), axis=1), False)
        near += (climb & shifted & ~top).sum(1)
    return mx * 10.0 + climber_beside(st, top) * 4 + np.minimum(near, 3) + (h >= 2).sum(1) * 0.5


def score_edge(lib, st):
    occ = heights(st) > 0
    r = np.arange(529) // 23
    q = np.arange(529) % 23
    d = np.maximum(np.abs(r - 11), np.abs(q - 11))
    return np.where(occ, d[None, :], 0).max(1) * 10.0 + occ.sum(1) * 0.1


def pick(rng, rows, k):
    rows = np.asarray(rows)
    if len(rows) <= k:
        return rows
    return np.sort(rng.choice(rows, k, replace=False))


def find_cases(lib):
    rng = np.random.default_rng(SEED)
    cases = {}
    # -- searches over legal play -------------------------------------------
    starts = lib.generate_positions(SEED, 0, 256, 16, 7)
    starts = starts[(starts[:, OFF_RESULT] == 0) & (side(starts) == 0)][:16]
    many = beam(lib, starts, score_moves, 16, 12, rng, reply_sample=6)
    _, nl, _ = lib.legal_moves_features(many)
    cases["cap256"] = many[pick(rng, np.where(nl >= 256)[0], 12)]
    cases["near_cap"] = many[pick(rng, np.where((nl >= 240) & (nl < 256))[0], 4)]

    starts = lib.generate_positions(SEED + 1, 0, 256, 24, 7)
    starts = starts[starts[:, OFF_RESULT] == 0][:48]
    tall = beam(lib, starts, score_stack, 48, 60, rng)
    h = heights(tall)
    five = h.max(1) >= 5
    # a legal climb onto a 5-high stack (applying it meets the refusal of a 6th piece)
    cand = np.where(five & climber_beside(tall, h >= 5))[0][:4000]
    mv, nl, _ = lib.legal_moves_features(tall[cand])
    to = mv[:, :, 4].astype(np.int64) | (mv[:, :, 5].astype(np.int64) << 8)
    valid = np.arange(256)[None, :] < nl[:, None]
    onto5 = valid & (mv[:, :, 0] == 1) & (np.take_along_axis(h[cand], np.clip(to, 0, 528), 1) >= 5)
    cases["stack5"] = tall[cand[pick(rng, np.where(onto5.any(1))[0], 10)]]
    cases["stack5_any"] = tall[pick(rng, np.where(five)[0], 4)]
    cases["stack4"] = tall[pick(rng, np.where(h.max(1) == 4)[0], 6)]

    starts = lib.generate_positions(SEED + 2, 0, 256, 20, 7)
    starts = starts[starts[:, OFF_RESULT] == 0][:32]
    far = beam(lib, starts, score_edge, 32, 60, rng)
    occ = heights(far) > 0
    r = np.arange(529) // 23
    q = np.arange(529) % 23
    border = (r == 0) | (r == 22) | (q == 0) | (q == 22)
    near = (r == 1) | (r == 21) | (q == 1) | (q == 21)
    cases["edge"] = far[pick(rng, np.where((occ & border[None, :]).any(1))[0], 12)]
    cases["near_edge"] = far[pick(rng, np.where((occ & near[None, :]).any(1) & ~(occ & border[None, :]).any(1))[0],
                                  4)]

    # -- pillbug situations from seeded playouts (all expansions) ------------
    pool = lib.generate_positions(SEED + 3, 0, 200000, 160, 7)
    pool = pool[pool[:, OFF_RESULT] == 0]
    t, h, me = tops(pool), heights(pool), side(pool)
    ttype, tcol = t & 15, (t >> 4) & 1
    ap = lib.articulation(pool)
    apbits = np.unpackbits(ap.view(np.uint8), axis=1, bitorder="little")[:, :529].astype(bool)
    stun = stunned(pool)
    has_stun = stun < 529
    sc = np.clip(stun, 0, 528)
    rows = np.arange(len(pool))
    own_pill = (ttype == T_PILL) & (tcol == me[:, None]) & (h > 0)
    ground1 = (h == 1)
    # a pillbug of the side to move on the stunned cell with a ground neighbour and an empty neighbour
    pill_on_stun = has_stun & own_pill[rows, sc]
    nb_h = nbr_vals(h, sc)
    stun_ok = pill_on_stun & (nb_h == 1).any(1) & (nb_h == 0).any(1)
    cases["pill_stunned"] = pool[pick(rng, np.where(stun_ok)[0], 10)]
    # a pinned pillbug of the side to move (articulation point, height 1) with throwable neighbours
    pinned = own_pill & ground1 & apbits
    cells = np.argmax(pinned, 1)
    nb_h = nbr_vals(h, cells)
    cases["pill_pinned"] = pool[pick(rng, np.where(pinned.any(1) & (nb_h == 1).any(1) & (nb_h == 0).any(1))[0], 10)]
    # a pillbug covered by a beetle (level 0 is a pillbug, height >= 2)
    lv0 = pool[:, :529] & 15
    covered = (lv0 == T_PILL) & (h >= 2)
    cases["pill_covered"] = pool[pick(rng, np.where(covered.any(1))[0], 8)]
    # a ground mosquito of the side to move beside any pillbug (top), with a ground neighbour
    mosq = (ttype == T_MOSQ) & (tcol == me[:, None]) & ground1
    pill_any = (ttype == T_PILL) & (h > 0)
    beside = np.zeros_like(mosq)
    for d in range(6):
        nb = NEIGH[:, d]
        beside |= mosq & np.where(nb[None, :] >= 0, np.take(pill_any, np.clip(nb, 0, 528), axis=1), False)
    cases["mosq_pill"] = pool[pick(rng, np.where(beside.any(1))[0], 10)]
    # the stunned piece is beside a pillbug of the side to move
    nb_pill = nbr_vals(own_pill.astype(np.int64), sc)
    cases["stunned_next_pill"] = pool[pick(rng, np.where(has_stun & ~pill_on_stun & (nb_pill == 1).any(1))[0], 8)]
    return cases


# -- hand-built rule scenarios -------------------------------------------------
# Small boards written piece by piece (the kind of setup a rules test uses):
# each piece is (type, colour, q, r) in axial coordinates around the grid's
# centre cell, listed bottom to top where pieces share a cell.
TYPES = "QAGSBMLP"


def build_state(pieces, turn, stunned=None, mask=7):
    """HiveState bytes (hive_state.cuh:239-269 layout) for the given pieces:
    hands reduced by the pieces on the board, queen cells and flags set,
    result in progress, no stunned cell unless given ((q, r))."""
    st = np.zeros(3424, np.uint8)
    height = np.zeros(529, np.int64)
    hands = np.array([[1, 3, 3, 2, 2, mask & 1, (mask >> 1) & 1, (mask >> 2) & 1]] * 2, np.int64)
    qcell = [0xFFFF, 0xFFFF]
    qplaced = 0
    top = {}
    for t, colour, q, r in pieces:
        pt = TYPES.index(t) + 1
        c = (r + 11) * 23 + (q + 11)
        h = height[c]
        st[h * 529 + c] = pt | (colour << 4)
        height[c] = h + 1
        top[c] = colour
        hands[colour, pt - 1] -= 1
        assert hands[colour, pt - 1] >= 0, (t, colour)
        if pt == 1:
            qcell[colour] = c
            qplaced |= 1 << colour
    st[OFF_HEIGHT:OFF_HEIGHT + 529] = height
    occ = np.zeros(9, np.uint64)
    wt = np.zeros(9, np.uint64)
    bt = np.zeros(9, np.uint64)
    for c, colour in top.items():
        bit = np.uint64(1) << np.uint64(c % 64)
        occ[c // 64] |= bit
        (bt if colour else wt)[c // 64] |= bit
    st[3176:3248] = occ.view(np.uint8)
    st[3248:3320] = wt.view(np.uint8)
    st[3320:3392] = bt.view(np.uint8)
    st[3392:3396] = np.array(qcell, np.uint16).view(np.uint8)
    st[3396:3412] = hands.astype(np.uint8).reshape(-1)
    st[3412:3414] = np.array([turn], np.uint16).view(np.uint8)
    st[3414] = qplaced
    st[3415] = 0
    sc = 0xFFFF if stunned is None else (stunned[1] + 11) * 23 + (stunned[0] + 11)
    st[3416:3418] = np.array([sc], np.uint16).view(np.uint8)
    st[3418] = 0
    st[3419] = 0
    return st


W, B = 0, 1
SCENARIOS = {
    # pillbug throws a friendly / an enemy neighbour onto an empty neighbour of its own
    "throw_friend": ([("Q", W, 0, 0), ("P", W, 1, 0), ("A", W, 1, -1), ("Q", B, -1, 0)], 8),
    "throw_enemy": ([("Q", W, 0, 0), ("P", W, 1, 0), ("Q", B, 2, 0), ("A", B, 3, 0)], 8),
    # the queen between the chain and the pillbug holds the hive together: it is not thrown
    "throw_pinned_neighbour": ([("A", W, -2, 0), ("B", W, -1, 0), ("Q", W, 0, 0), ("P", W, 1, 0),
                                ("Q", B, -3, 0)], 8),
    # the pillbug itself holds the hive together: it cannot move, it still throws
    "pillbug_articulation": ([("A", W, -1, 0), ("P", W, 0, 0), ("Q", W, 1, 0), ("Q", B, -2, 0)], 8),
    # a beetle on the pillbug: the pillbug is not a top piece and throws nothing
    "pillbug_covered": ([("Q", W, 0, 0), ("P", W, 1, 0), ("B", W, 1, 0), ("A", W, 2, 0), ("Q", B, -1, 0)], 8),
    "pillbug_covered_by_enemy": ([("Q", W, 0, 0), ("P", W, 1, 0), ("B", B, 1, 0), ("A", W, 2, 0),
                                  ("Q", B, -1, 0)], 8),
    # a stacked neighbour cannot be thrown, nor a piece that just moved (stunned)
    "throw_stacked_neighbour": ([("Q", W, 0, 0), ("P", W, 1, 0), ("G", W, 1, -1), ("B", B, 1, -1),
                                 ("Q", B, 2, -1)], 8),
    "throw_stunned_neighbour": ([("Q", W, 0, 0), ("P", W, 1, 0), ("A", B, 2, 0), ("Q", B, 3, 0)], 8, (2, 0)),
    "stunned_pillbug_throws": ([("Q", W, 0, 0), ("P", W, 1, 0), ("A", W, 1, -1), ("Q", B, -1, 0)], 8, (1, 0)),
    # a throw over a gate: both cells beside the path are stacked higher
    "throw_through_gate": ([("Q", W, 0, 0), ("P", W, 1, 0), ("A", W, 2, 0), ("G", B, 1, -1), ("B", B, 1, -1),
                            ("S", B, 2, -1), ("B", W, 2, -1), ("Q", B, 0, -1)], 8),
    # ground mosquito beside a pillbug throws its own neighbours; beside a mosquito only: nothing
    "mosquito_throws": ([("Q", W, 0, 0), ("P", W, 1, 0), ("M", W, 0, 1), ("A", W, -1, 1), ("Q", B, -1, 0)], 8),
    "mosquito_beside_enemy_pillbug": ([("Q", W, 0, 0), ("M", W, 0, 1), ("P", B, 1, 1), ("A", B, 2, 1),
                                       ("Q", B, -1, 0)], 8),
    "mosquito_beside_mosquito": ([("Q", W, 0, 0), ("M", W, 1, 0), ("M", B, 2, 0), ("Q", B, 3, 0)], 8),
    # a mosquito copies ant, grasshopper, spider, beetle, ladybug, queen moves of its neighbours
    "mosquito_copies_all": ([("Q", W, 0, 0), ("A", W, 1, 0), ("M", W, 1, 1), ("G", W, 2, 1), ("S", W, 0, 2),
                             ("B", B, 1, 2), ("L", B, 2, 2), ("Q", B, 2, 3)], 8),
    # a mosquito on top of the hive moves as a beetle only
    "mosquito_on_top": ([("Q", W, 0, 0), ("A", W, 1, 0), ("M", W, 1, 0), ("G", W, 2, 0), ("Q", B, -1, 0)], 8),
    # ladybug: two steps on top of the hive, one down
    "ladybug": ([("Q", W, 0, 0), ("L", W, 1, 0), ("A", B, 2, 0), ("S", B, 2, 1), ("Q", B, 1, 2)], 8),
    # beetle on a stack between two higher stacks (gate on top of the hive)
    "beetle_gate_on_top": ([("Q", W, 0, 0), ("B", W, 0, 0), ("A", B, 1, 0), ("B", B, 1, 0), ("G", W, 1, -1),
                            ("B", W, 1, -1), ("G", B, 0, -1), ("B", B, 0, -1), ("Q", B, -1, 1)], 8),
    # grasshopper jumps that would land off the grid, an ant on the outer column
    "edge_grasshopper": ([("Q", W, 8, 0), ("G", W, 9, 0), ("A", B, 10, 0), ("S", B, 11, 0), ("Q", B, 11, -1)], 8),
    "edge_ant": ([("Q", W, 0, 0), ("A", W, 1, -11), ("G", W, 1, -10), ("S", W, 1, -9), ("G", W, 1, -8),
                  ("S", W, 1, -7), ("G", W, 1, -6), ("A", W, 1, -5), ("B", W, 1, -4), ("B", W, 1, -3),
                  ("A", W, 1, -2), ("L", W, 1, -1), ("Q", B, -1, 0)], 8),
    # black to move versions of two of the above
    "throw_friend_black": ([("Q", B, 0, 0), ("P", B, 1, 0), ("A", B, 1, -1), ("Q", W, -1, 0)], 9),
    "mosquito_throws_black": ([("Q", B, 0, 0), ("P", B, 1, 0), ("M", B, 0, 1), ("A", B, -1, 1),
                               ("Q", W, -1, 0)], 9),
    # queen not yet placed at the side's fourth turn: placements only, queen forced
    "queen_forced": ([("A", W, 0, 0), ("G", W, 1, 0), ("S", W, 2, 0), ("Q", B, -1, 0), ("A", B, -2, 0),
                      ("G", B, -3, 0)], 6),
}


def scenario_states():
    names, states = [], []
    for name, spec in SCENARIOS.items():
        pieces, turn = spec[0], spec[1]
        stunned = spec[2] if len(spec) > 2 else None
        names.append(name)
        states.append(build_state(pieces, turn, stunned))
    return names, np.stack(states)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def record(lib, states):
    moves, nl, feats = lib.legal_moves_features(states)
    cm, cn = lib.compact_moves(states)
    ap = lib.articulation(states)
    act, cen = lib.actions(states, moves, nl)
    succ_dig, kid_dig, res_dig = [], [], []
    for i in range(len(states)):
        n = int(nl[i])
        roots = np.full(n, i, np.int64)
        idx = np.arange(n, dtype=np.int64)
        sf = lib.successor_features(states, moves, roots, idx)
        kids = lib.apply_moves(np.repeat(states[i:i + 1], n, 0), moves[i, :n])
        succ_dig.append(digest(sf))
        kid_dig.append(digest(kids))
        res_dig.append(digest(kids[:, OFF_RESULT]))
    hyb = lib.hybrid_encode(states, moves, nl)
    hyb_dig = [digest(*(a[i:i + 1] for a in hyb[:7])) for i in range(len(states))]
    mf_dig = [digest(hyb[7][i, :int(nl[i])]) for i in range(len(states))]
    return dict(moves=moves, num_legal=nl, features=feats, compact_moves=cm, compact_num=cn, articulation=ap,
                actions=act, centroids=cen), dict(successor_features=succ_dig, successor_states=kid_dig,
                                                  successor_results=res_dig, hybrid_tokens=hyb_dig,
                                                  hybrid_move_features=mf_dig)


def main() -> None:
    O.build(ref=True)
    ref = O.ref()
    if ref is None:
        raise SystemExit("reference build unavailable: the reference tree is needed to make goldens")
    cases = find_cases(ref)
    names, states = [], []
    for k, v in cases.items():
        names += [k] * len(v)
        states.append(v)
    snames, sstates = scenario_states()
    names += ["scenario:" + n for n in snames]
    states.append(sstates)
    cases["scenarios"] = sstates
    states = np.concatenate(states)
    arrays, digests = record(ref, states)
    np.savez_compressed(os.path.join(HERE, "golden_edge.npz"), states=states, case=np.array(names), **arrays)
    with open(os.path.join(HERE, "golden_edge.json"), "w") as f:
        json.dump({"seed": SEED, "cases": {k: int(len(v)) for k, v in cases.items()}, **digests}, f, indent=0)
    print(json.dumps({k: int(len(v)) for k, v in cases.items()}),
          "max legal", int(arrays["num_legal"].max()), "max height", int(heights(states).max()))


if __name__ == "__main__":
    main()
