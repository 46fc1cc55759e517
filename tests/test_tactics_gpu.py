"""GPU parity of root_tactical_probe_batch against the reference's outputs
(golden_tactical.json) and the C oracle, bit-exact."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLD)
import make_tactical_golden as T  # noqa: E402


@pytest.fixture(scope="module")
def setup():
    from hive_neuralnet_b200.hive_gpu import load_extension
    ext = load_extension()
    with open(os.path.join(GOLD, "golden_tactical.json")) as f:
        fx = json.load(f)
    p = T.PARAMS
    st = ext.generate_positions(p["seed"], p["first_game"], p["count"], p["max_ply"], p["expansion_mask"])
    idx = torch.tensor(fx["indices"], dtype=torch.int64, device="cuda")
    sub = st[idx].contiguous()
    mo, no = ext.generate_legal_moves_batch(sub, len(idx))
    pri = torch.from_numpy(T.priors_for(len(idx))).cuda()
    return ext, fx, sub, mo, no, pri


@pytest.mark.parametrize("flags", ["111", "100", "010", "001"])
def test_tactical_probe_matches_reference(setup, flags):
    ext, fx, sub, mo, no, pri = setup
    want = fx["cases"][flags]
    win, allowed, forced = ext.root_tactical_probe_batch(sub, mo, no, pri, len(sub), *(c == "1" for c in flags))
    assert win.dtype == torch.int64 and allowed.dtype == torch.uint8 and forced.dtype == torch.uint8
    w = win.cpu().numpy()
    bad = np.where(w != np.array(want["winning"]))[0]
    assert len(bad) == 0, f"winning differs at {bad[:10]}"
    assert forced.cpu().numpy().tolist() == want["forced"]
    assert hashlib.sha256(allowed.cpu().numpy().tobytes()).hexdigest() == want["allowed_sha256"]
    assert ext.device_error_word(clear=True) == 0


def test_tactical_probe_all_off_and_random_positions(setup):
    ext, fx, sub, mo, no, pri = setup
    win, allowed, forced = ext.root_tactical_probe_batch(sub, mo, no, pri, len(sub), False, False, False)
    n = no.cpu().numpy()
    assert (win.cpu().numpy() == -1).all() and (forced.cpu().numpy() == 0).all()
    assert np.array_equal(allowed.cpu().numpy(), (np.arange(256)[None] < n[:, None]).astype(np.uint8))
    # ordinary positions (mostly no tactics) against the oracle
    orc = O.oracle()
    st = orc.generate_positions(4242, 0, 2048, 120, 7)
    m, nl, _ = orc.legal_moves_features(st)
    pr = np.random.default_rng(1).random((2048, 256)).astype(np.float32)
    want = orc.tactical_probe(st, m, nl, pr)
    got = ext.root_tactical_probe_batch(*(torch.from_numpy(a).cuda() for a in (st, m, nl, pr)), 2048)
    for g, o in zip(got, want):
        assert np.array_equal(g.cpu().numpy(), o)
