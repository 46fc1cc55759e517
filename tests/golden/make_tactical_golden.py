"""Generate tests/golden/golden_tactical.json from the REFERENCE itself.

Positions: the seeded playout generator (all expansions, stop ply
U[0, 160]); the fixture keeps those where the root tactical probe has work
(game in progress and the opponent queen has 4 or 5 occupied neighbours, or
the own queen 5).  Priors are seeded uniforms.  The reference outputs come
from oracle/_ref/libhive_ref.so: root_tactical_probe_kernel's steps
(hive_gpu/csrc/game_logic.cu:290-397) over the reference's own move_gen.cuh
helpers, compiled on the host.

    python tests/golden/make_tactical_golden.py
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

PARAMS = {"seed": 777, "first_game": 0, "count": 20000, "max_ply": 160, "expansion_mask": 7, "prior_seed": 5}
_DIRS = ((0, 1), (-1, 1), (-1, 0), (0, -1), (1, -1), (1, 0))


def surround_counts(states: np.ndarray) -> np.ndarray:
    """[B, 2] occupied on-grid neighbours of each colour's queen (0 if not placed)."""
    occ = states[:, 3176:3176 + 72].copy().view(np.uint64)
    qc = states[:, 3392:3396].copy().view(np.uint16).astype(np.int64)
    qp = states[:, 3414].astype(np.int64)
    out = np.zeros((len(states), 2), np.int64)
    for c in range(2):
        placed = ((qp >> c) & 1).astype(bool) & (qc[:, c] < 529)
        q = np.where(placed, qc[:, c], 0)
        r, col = q // 23, q % 23
        for dr, dc in _DIRS:
            rr, cc = r + dr, col + dc
            on = (rr >= 0) & (rr < 23) & (cc >= 0) & (cc < 23) & placed
            cell = np.where(on, rr * 23 + cc, 0)
            bit = (occ[np.arange(len(states)), cell >> 6] >> (cell & 63).astype(np.uint64)) & np.uint64(1)
            out[:, c] += (on & (bit == 1)).astype(np.int64)
    return out


def tactical_inputs(lib):
    p = PARAMS
    st = lib.generate_positions(p["seed"], p["first_game"], p["count"], p["max_ply"], p["expansion_mask"])
    s = surround_counts(st)
    me = (st[:, 3412] & 1).astype(np.int64)
    rows = np.arange(len(st))
    opp_s, own_s = s[rows, 1 - me], s[rows, me]
    sel = np.where((st[:, 3415] == 0) & ((opp_s >= 4) & (opp_s <= 5) | (own_s == 5)))[0]
    return st, sel


def priors_for(n: int) -> np.ndarray:
    return np.random.default_rng(PARAMS["prior_seed"]).random((n, 256)).astype(np.float32)


def main() -> None:
    O.build(ref=True)
    ref = O.ref()
    if ref is None:
        raise SystemExit("reference build unavailable: the reference tree is needed to make goldens")
    st, sel = tactical_inputs(ref)
    sub = st[sel]
    mo, no, _ = ref.legal_moves_features(sub)
    pri = priors_for(len(sel))
    out = {"params": PARAMS, "indices": sel.tolist(), "cases": {}}
    for flags in ((1, 1, 1), (1, 0, 0), (0, 1, 0), (0, 0, 1)):
        win, allowed, forced = ref.tactical_probe(sub, mo, no, pri, *flags)
        out["cases"]["%d%d%d" % flags] = {
            "winning": win.tolist(), "forced": forced.tolist(),
            "allowed_sha256": hashlib.sha256(allowed.tobytes()).hexdigest(),
            "wins": int((win >= 0).sum()), "forced_count": int(forced.sum()),
        }
        print(flags, "wins", int((win >= 0).sum()), "forced", int(forced.sum()))
    with open(os.path.join(HERE, "golden_tactical.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("positions", len(sel))


if __name__ == "__main__":
    main()
