"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Run in a container that has the reference tree: it builds
oracle/_ref/libhive_ref.so (the reference's own hive_gpu/csrc headers compiled
on the host by oracle/ref_driver.cpp) and records its outputs:

* ``golden_small.npz`` -- explicit arrays for 96 positions (48 base game,
  ply U[0,60]; 48 all expansions, ply U[0,120]): state bytes, full move lists,
  num_legal, features, compact lists, articulation points, centroids, action
  indices, queen-escape flags, and successor features of every legal move;
* ``golden_digests.json`` -- SHA-256 digests of the same outputs (plus the
  hybrid transformer's piece tokens and move features) for the
  BASELINE config-1 set (4,096 base positions) and an 8,192-position
  all-expansion set, so the larger parity sets are pinned without storing them.

The position generator is the seeded counter-based playout recipe shared by
oracle/hive_oracle.c (orc_playout) and the CUDA kernel k_playouts.

    python tests/golden/make_golden.py
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

SEED = 20251201
SETS = {
    # name: (seed, first_game, count, max_ply, expansion_mask)
    "config1_base_4096": (SEED, 0, 4096, 60, 0),
    "expansions_8192": (SEED + 1, 0, 8192, 120, 7),
}


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def outputs(lib, states: np.ndarray) -> dict:
    moves, nl, feats = lib.legal_moves_features(states)
    cm, cn = lib.compact_moves(states)
    ap = lib.articulation(states)
    act, cen = lib.actions(states, moves, nl)
    qe = lib.queen_escape(states)
    roots = np.repeat(np.arange(states.shape[0], dtype=np.int64), nl)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in nl]) if len(nl) else np.zeros(0, np.int64)
    succ = lib.successor_features(states, moves, roots, idx)
    return dict(moves=moves, num_legal=nl, features=feats, compact_moves=cm, compact_num=cn,
                articulation=ap, actions=act, centroids=cen, queen_escape=qe,
                succ_roots=roots, succ_moves=idx, succ_features=succ)


def hybrid(lib, states: np.ndarray, o: dict):
    """Hybrid transformer inputs (state_encoder.cuh:372-550): tokens, q, r, z, mask, global,
    num_tokens, move features."""
    return lib.hybrid_encode(states, o["moves"], o["num_legal"])


def main() -> None:
    O.build(ref=True)
    ref = O.ref()
    if ref is None:
        raise SystemExit("reference build unavailable: the reference tree is needed to make goldens")
    small_b = ref.generate_positions(SEED + 7, 0, 48, 60, 0)
    small_x = ref.generate_positions(SEED + 8, 0, 48, 120, 7)
    states = np.concatenate([small_b, small_x])
    out = outputs(ref, states)
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"), states=states, **out)
    dig = {}
    for name, (seed, first, count, max_ply, mask) in SETS.items():
        st = ref.generate_positions(seed, first, count, max_ply, mask)
        o = outputs(ref, st)
        dig[name] = {
            "params": {"seed": seed, "first_game": first, "count": count, "max_ply": max_ply,
                       "expansion_mask": mask},
            "states": digest(st),
            "moves": digest(o["moves"], o["num_legal"]),
            "features": digest(o["features"]),
            "compact": digest(o["compact_moves"], o["compact_num"]),
            "articulation": digest(o["articulation"]),
            "actions": digest(o["actions"], o["centroids"]),
            "queen_escape": digest(o["queen_escape"]),
            "successor_features": digest(o["succ_features"]),
            "hybrid_tokens": digest(*hybrid(ref, st, o)[:7]),
            "hybrid_move_features": digest(hybrid(ref, st, o)[7]),
            "num_successors": int(len(o["succ_roots"])),
            "mean_legal": float(o["num_legal"].mean()),
        }
    with open(os.path.join(HERE, "golden_digests.json"), "w") as f:
        json.dump(dig, f, indent=1, sort_keys=True)
    print(json.dumps({k: (v["num_successors"], v["mean_legal"]) for k, v in dig.items()}))


if __name__ == "__main__":
    main()
