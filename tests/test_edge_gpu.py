"""GPU parity on the reference's edge cases, bit-exact against fixtures the
reference build itself produced (tests/golden/make_edge_golden.py):
positions whose move list is cut at 256, 5-high stacks with a climb onto
them (the refused 6th piece), pieces on the grid's outer rows and columns,
and pillbug / mosquito rule situations, found by search and written by hand.

Every output of the path is compared: move lists (order, duplicates,
truncation), num_legal, the 122 features as float bits, the successor
features of every legal move, the successor states and their results, the
action indices and centroids, the hybrid transformer inputs, the FNN leaf
evaluation (1e-5 against the fp32 statement) and the tactical probe."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def ext():
    from hive_neuralnet_b200.hive_gpu import load_extension
    return load_extension()


@pytest.fixture(scope="module")
def gold():
    g = dict(np.load(os.path.join(GOLD, "golden_edge.npz")))
    with open(os.path.join(GOLD, "golden_edge.json")) as f:
        g.update(json.load(f))
    return g


def _where(gold, rows):
    return sorted({str(gold["case"][i]) for i in rows})


def test_fixture_reaches_the_limits(gold):
    nl, st = gold["num_legal"], gold["states"]
    assert (nl[gold["case"] == "cap256"] == 256).all()
    assert st[:, 2645:2645 + 529].max() == 5
    assert int(gold["cases"]["scenarios"]) >= 20


def test_moves_and_features(ext, gold):
    st = _cuda(gold["states"])
    n = len(gold["states"])
    mg, ng, fg = (x.cpu().numpy() for x in ext.generate_legal_moves_and_fnn_features_batch(st, n))
    bad = np.where(ng != gold["num_legal"])[0]
    assert len(bad) == 0, f"num_legal differs: {_where(gold, bad)}"
    bad = np.where((mg != gold["moves"]).reshape(n, -1).any(1))[0]
    assert len(bad) == 0, f"move lists differ: {_where(gold, bad)}"
    bad = np.where((_bits(fg) != _bits(gold["features"])).any(1))[0]
    assert len(bad) == 0, f"features differ: {_where(gold, bad)}"
    # the standalone generator and the features of a supplied list
    m2, n2 = ext.generate_legal_moves_batch(st, n)
    assert np.array_equal(m2.cpu().numpy(), gold["moves"]) and np.array_equal(n2.cpu().numpy(), gold["num_legal"])
    f2 = ext.extract_fnn_features_batch(st, _cuda(gold["moves"]), _cuda(gold["num_legal"]), n).cpu().numpy()
    assert np.array_equal(_bits(f2), _bits(gold["features"]))
    # the compact list's features (the successor path's list)
    fc = ext.extract_fnn_features_batch(st, _cuda(gold["compact_moves"]), _cuda(gold["compact_num"]), n)
    orc = O.oracle()
    want = orc.features(gold["states"], gold["compact_moves"], gold["compact_num"])
    assert np.array_equal(_bits(fc.cpu().numpy()), _bits(want))


def test_successors(ext, gold):
    st, mv, nl = gold["states"], gold["moves"], gold["num_legal"]
    roots = np.repeat(np.arange(len(st), dtype=np.int64), nl)
    idx = np.concatenate([np.arange(k, dtype=np.int64) for k in nl])
    sf = ext.fnn_successor_features_batch(_cuda(st), _cuda(mv), _cuda(roots), _cuda(idx), len(roots))
    sf = sf.cpu().numpy()
    kids = _cuda(st[roots])
    ext.apply_moves_batch(kids, _cuda(mv[roots, idx]), len(roots))
    res = ext.check_results_batch(kids, len(roots)).cpu().numpy()
    kids = kids.cpu().numpy()
    assert np.array_equal(res, kids[:, 3415].astype(np.int32))
    bad_f, bad_s, bad_r = [], [], []
    start = 0
    for i, k in enumerate(nl):
        sl = slice(start, start + k)
        start += k
        if _digest(sf[sl]) != gold["successor_features"][i]:
            bad_f.append(i)
        if _digest(kids[sl]) != gold["successor_states"][i]:
            bad_s.append(i)
        if _digest(kids[sl, 3415]) != gold["successor_results"][i]:
            bad_r.append(i)
    assert not bad_f, f"successor features differ: {_where(gold, bad_f)}"
    assert not bad_s, f"successor states differ: {_where(gold, bad_s)}"
    assert not bad_r, f"successor results differ: {_where(gold, bad_r)}"
    # a climb onto a 5-high stack is generated and its application leaves the stack at 5
    h = st[:, 2645:2645 + 529]
    to = mv[..., 4].astype(np.int64) | (mv[..., 5].astype(np.int64) << 8)
    onto5 = [(i, j) for i in range(len(st)) for j in range(nl[i])
             if mv[i, j, 0] == 1 and h[i, to[i, j]] >= 5]
    assert onto5, "the fixture should hold a climb onto a 5-high stack"
    offs = np.concatenate([[0], np.cumsum(nl)])
    for i, j in onto5:
        assert kids[offs[i] + j, 2645 + to[i, j]] == 5


def test_actions_and_centroids(ext, gold):
    st, mv, nl = _cuda(gold["states"]), _cuda(gold["moves"]), _cuda(gold["num_legal"])
    n = len(gold["states"])
    act = ext.legal_moves_to_actions_batch(st, mv, nl, n).cpu().numpy()
    cen = ext.compute_centroids_batch(st, n).cpu().numpy()
    assert np.array_equal(act, gold["actions"])
    assert np.array_equal(cen, gold["centroids"])


def test_hybrid_inputs(ext, gold):
    st, mv, nl = _cuda(gold["states"]), _cuda(gold["moves"]), _cuda(gold["num_legal"])
    n = len(gold["states"])
    tok = [t.cpu().numpy() for t in ext.hybrid_transformer_encode_with_moves_batch(st, mv, nl, n)]
    tok[4] = tok[4].astype(np.uint8)
    mf = ext.hybrid_transformer_move_features_batch(st, mv, nl, n).cpu().numpy()
    bad_t = [i for i in range(n) if _digest(*(a[i:i + 1] for a in tok[:7])) != gold["hybrid_tokens"][i]]
    bad_m = [i for i in range(n)
             if _digest(mf[i, :int(gold["num_legal"][i])]) != gold["hybrid_move_features"][i]]
    assert not bad_t, f"hybrid tokens differ: {_where(gold, bad_t)}"
    assert not bad_m, f"hybrid move features differ: {_where(gold, bad_m)}"


def test_fnn_leaf_evaluation(gold):
    """Leaves with 256 successors and stacked / edge / throw positions through
    the row pipeline, against the fp32 statement on the fixture's own
    successor features (1e-5)."""
    from hive_neuralnet_b200.fnn import FusedFNNEvaluator, HiveFNN
    from oracle.fnn_reference import eval_states_reference
    st, mv, nl, ft = gold["states"], gold["moves"], gold["num_legal"], gold["features"]
    orc = O.oracle()
    roots = np.repeat(np.arange(len(st), dtype=np.int64), nl)
    idx = np.concatenate([np.arange(k, dtype=np.int64) for k in nl])
    sf = orc.successor_features(st, mv, roots, idx)
    torch.manual_seed(3)
    net = HiveFNN().eval()
    pr, vr, cr, lr = eval_states_reference(net, ft, sf, nl)
    ev = FusedFNNEvaluator(net)
    pg, vg, cg, lg = (x.cpu().numpy() for x in ev.eval_states(_cuda(st), _cuda(mv), _cuda(nl), len(st), _cuda(ft),
                                                              return_logits=True))
    close = lambda a, b: np.abs(a - b) <= 1e-5 * np.abs(b) + 1e-6
    valid = np.arange(256)[None, :] < nl[:, None]
    assert close(vg, vr).all() and close(cg, cr).all() and close(pg, pr).all()
    assert close(lg[valid], lr[valid]).all()


def test_tactical_probe(ext, gold):
    st, mv, nl = gold["states"], gold["moves"], gold["num_legal"]
    rng = np.random.default_rng(17)
    pri = rng.uniform(0.01, 1, (len(st), 256)).astype(np.float32)
    pri = np.where(np.arange(256)[None, :] < nl[:, None], pri, 0).astype(np.float32)
    win, allowed, forced = ext.root_tactical_probe_batch(_cuda(st), _cuda(mv), _cuda(nl), _cuda(pri), len(st),
                                                         True, True, True)
    w, a, f = O.oracle().tactical_probe(st, mv, nl, pri)
    assert np.array_equal(win.cpu().numpy(), w)
    assert np.array_equal(allowed.cpu().numpy().astype(np.uint8), a)
    assert np.array_equal(forced.cpu().numpy().astype(np.uint8), f)
