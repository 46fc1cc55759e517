"""GPU parity: the fused successor + FNN leaf evaluator against the fp32
PyTorch restatement of the reference's _eval_states (oracle/fnn_reference.py)
fed with the oracle's bit-exact successor features.

Tolerance (fp32, different summation order and transcendental
implementations): |gpu - ref| <= 1e-5 * |ref| + 1e-6 for values, logits,
child Q and priors."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle.fnn_reference import eval_states_reference

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-5, 1e-6


def _close(a, b):
    return np.abs(a - b) <= RTOL * np.abs(b) + ATOL


@pytest.mark.parametrize("preset", ["large", "medium", "small"])
@pytest.mark.parametrize("with_root_features", [True, False])
@pytest.mark.parametrize("path", ["rows", "fused"])
def test_fused_eval_matches_reference(preset, with_root_features, path):
    from hive_neuralnet_b200.fnn import FNNConfig, FusedFNNEvaluator, HiveFNN
    orc = O.oracle()
    torch.manual_seed(0)
    net = HiveFNN(getattr(FNNConfig, preset)()).eval()
    st = np.concatenate([orc.generate_positions(71, 0, 384, 60, 0), orc.generate_positions(72, 0, 640, 150, 7)])
    mo, no, fo = orc.legal_moves_features(st)
    roots = np.repeat(np.arange(len(st), dtype=np.int64), no)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in no])
    sf = orc.successor_features(st, mo, roots, idx)
    pr, vr, cr, lr = eval_states_reference(net, fo, sf, no)
    ev = FusedFNNEvaluator(net)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    fn = ev.eval_states if path == "rows" else ev.eval_states_fused
    out = fn(t(st), t(mo), t(no), len(st), t(fo) if with_root_features else None, return_logits=True)
    pg, vg, cg, lg = (x.cpu().numpy() for x in out)
    assert _close(vg, vr).all(), np.abs(vg - vr).max()
    valid = np.arange(256)[None, :] < no[:, None]
    assert _close(lg[valid], lr[valid]).all(), np.abs(lg - lr)[valid].max()
    assert _close(cg, cr).all(), np.abs(cg - cr).max()
    assert _close(pg, pr).all(), np.abs(pg - pr).max()
    assert (pg[~valid] == 0).all() and (cg[~valid] == 0).all()
    np.testing.assert_allclose(pg.sum(1)[no > 0], 1.0, rtol=1e-5)


def test_terminal_and_empty_rows():
    from hive_neuralnet_b200.fnn import FusedFNNEvaluator, HiveFNN
    torch.manual_seed(1)
    net = HiveFNN()
    ev = FusedFNNEvaluator(net)
    st = torch.zeros((3, 3424), dtype=torch.uint8, device="cuda")
    mv = torch.zeros((3, 256, 6), dtype=torch.uint8, device="cuda")
    nl = torch.zeros((3,), dtype=torch.int32, device="cuda")
    for fn in (ev.eval_states, ev.eval_states_fused):
        p, v, c = fn(st, mv, nl, 3)
        assert (p == 0).all() and (c == 0).all() and torch.isfinite(v).all()
    p0, v0, c0 = ev.eval_states(st[:0], mv[:0], nl[:0], 0)
    assert p0.shape == (0, 256) and v0.shape == (0,)


@pytest.mark.parametrize("count", [1, 2, 5, 17])
def test_rows_small_batches(count):
    """Ragged row counts: one partial 64-row tile (a CTA whose second group
    has no tile), two tiles in one CTA, and a partial last tile."""
    from hive_neuralnet_b200.fnn import FusedFNNEvaluator, HiveFNN
    orc = O.oracle()
    torch.manual_seed(2)
    net = HiveFNN().eval()
    st = orc.generate_positions(900 + count, 0, count, 90, 7)
    mo, no, fo = orc.legal_moves_features(st)
    roots = np.repeat(np.arange(len(st), dtype=np.int64), no)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in no])
    sf = orc.successor_features(st, mo, roots, idx)
    pr, vr, cr, lr = eval_states_reference(net, fo, sf, no)
    ev = FusedFNNEvaluator(net)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    pg, vg, cg, lg = (x.cpu().numpy() for x in ev.eval_states(t(st), t(mo), t(no), count, t(fo), return_logits=True))
    valid = np.arange(256)[None, :] < no[:, None]
    assert _close(vg, vr).all() and _close(cg, cr).all() and _close(pg, pr).all()
    assert _close(lg[valid], lr[valid]).all()
