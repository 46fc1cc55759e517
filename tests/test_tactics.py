"""Root tactical probe: the C oracle against the reference's own outputs.

golden_tactical.json holds the reference's results (root_tactical_probe_kernel,
hive_gpu/csrc/game_logic.cu:290-397, run on the host over the reference
headers) for 4,376 seeded positions where the probe has work, under four
combinations of the enable flags.
"""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLD)
import make_tactical_golden as T  # noqa: E402


@pytest.fixture(scope="module")
def fixture():
    with open(os.path.join(GOLD, "golden_tactical.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def inputs(fixture):
    orc = O.oracle()
    st, sel = T.tactical_inputs(orc)
    assert sel.tolist() == fixture["indices"], "position generator or selection drifted from the fixture"
    sub = st[sel]
    mo, no, _ = orc.legal_moves_features(sub)
    return orc, sub, mo, no, T.priors_for(len(sel))


@pytest.mark.parametrize("flags", ["111", "100", "010", "001"])
def test_oracle_tactical_probe_matches_reference(fixture, inputs, flags):
    orc, sub, mo, no, pri = inputs
    want = fixture["cases"][flags]
    win, allowed, forced = orc.tactical_probe(sub, mo, no, pri, *(int(c) for c in flags))
    assert win.tolist() == want["winning"]
    assert forced.tolist() == want["forced"]
    assert hashlib.sha256(allowed.tobytes()).hexdigest() == want["allowed_sha256"]


def test_tactical_fixture_exercises_every_branch(fixture):
    c = fixture["cases"]
    assert c["100"]["wins"] > 0 and c["010"]["forced_count"] > 0
    # win-in-two wins that are not wins in one
    w1 = np.array(c["100"]["winning"])
    w2 = np.array(c["001"]["winning"])
    assert ((w2 >= 0) & (w1 < 0)).sum() > 0
