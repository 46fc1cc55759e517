"""Parity at BASELINE.json's full sizes.

Config 2: all 262,144 positions of the bench workload (seed 20260101, all
expansions, ply U[0,120]) -- move lists, counts and features bit-exact
against the oracle.  Config 3: every successor of the 65,536 roots
(~4.7 M rows) bit-exact, and the row-pipeline evaluator on all roots checked
against the fp32 reference on a seeded sample of 512 leaves (1e-5 rel)."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle.fnn_reference import eval_states_reference

pytestmark = pytest.mark.gpu


def _digest(*a):
    h = hashlib.sha256()
    for x in a:
        h.update(np.ascontiguousarray(x).tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def ext():
    from hive_neuralnet_b200.hive_gpu import load_extension
    return load_extension()


def test_config2_full_size_bit_exact(ext):
    P = 262144
    st = ext.generate_positions(20260101, 0, P, 120, 7)
    mg, ng, fg = ext.generate_legal_moves_and_fnn_features_batch(st, P)
    sth = st.cpu().numpy()
    mo, no, fo = O.oracle().legal_moves_features(sth)
    assert _digest(mg.cpu().numpy(), ng.cpu().numpy()) == _digest(mo, no)
    assert _digest(fg.cpu().numpy()) == _digest(fo)


def test_config3_full_size_successors_and_evaluator(ext):
    from hive_neuralnet_b200.fnn import FusedFNNEvaluator, HiveFNN
    P = 65536
    st = ext.generate_positions(20260101 + 3, 0, P, 120, 7)
    mv, nl, feats = ext.generate_legal_moves_and_fnn_features_batch(st, P)
    n = nl.cpu().numpy()
    roots = np.repeat(np.arange(P, dtype=np.int64), n)
    idx = np.concatenate([np.arange(k, dtype=np.int64) for k in n])
    sf_g = ext.fnn_successor_features_batch(st, mv, torch.from_numpy(roots).cuda(), torch.from_numpy(idx).cuda(),
                                            len(roots)).cpu().numpy()
    orc = O.oracle()
    sth, mvh = st.cpu().numpy(), mv.cpu().numpy()
    sf_o = orc.successor_features(sth, mvh, roots, idx)
    assert len(roots) > 4_000_000
    assert _digest(sf_g) == _digest(sf_o)
    torch.manual_seed(0)
    net = HiveFNN().eval()
    pr, va, cq = (x.cpu().numpy() for x in FusedFNNEvaluator(net).eval_states(st, mv, nl, P, feats))
    pick = np.sort(np.random.default_rng(3).choice(P, 512, replace=False))
    sub_rows = np.concatenate([np.arange(k) + s for k, s in zip(n[pick], np.concatenate([[0], np.cumsum(n)])[pick])])
    rp, rv, rc, _ = eval_states_reference(net, feats.cpu().numpy()[pick], sf_o[sub_rows], n[pick])
    tol = lambda a, b: np.abs(a - b) <= 1e-5 * np.abs(b) + 1e-6
    assert tol(va[pick], rv).all() and tol(pr[pick], rp).all() and tol(cq[pick], rc).all()


def test_config4_full_size_tree_invariants():
    """One searched move of BASELINE config 4 (512 games x 4,096 simulations):
    every root child's visits sum to the simulations its game ran (counted
    on the device), parent links are consistent, |W| <= N, the pool is not
    exceeded."""
    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.hive_gpu import load_extension
    from hive_neuralnet_b200.orchestrator import FNNMCTSConfig, FNNMCTSOrchestrator
    ext = load_extension()
    B, M = 512, 65536
    st = ext.generate_positions(99, 0, 4 * B, 30, 0)
    st = st[torch.nonzero(ext.check_results_batch(st, 4 * B) == 0).squeeze(1)[:B]].contiguous()
    torch.manual_seed(0)
    cfg = FNNMCTSConfig(num_simulations=4096, batch_size=B, max_game_length=1, dirichlet_epsilon=0.0, seed=3,
                        max_tree_nodes=M, short_forced_win_probe=True)
    orch = FNNMCTSOrchestrator(HiveFNN(), cfg)
    orch.trace = []
    orch.sims_done.zero_()
    ex = orch.self_play_batch(st.cpu())
    tree = next(x for x in orch.trace if x["kind"] == "searched")["tree"]
    root = next(x for x in orch.trace if x["kind"] == "root")
    vc, tv, pa, fc, nc, cnt = (tree[k] for k in ("visit_count", "total_value", "parent_idx", "first_child",
                                                  "num_children", "node_count"))
    assert (cnt <= M).all() and (cnt >= 1).all()
    rows = torch.arange(B, device=vc.device)
    active = root["game_active"] != 0
    f0, n0 = fc[rows, 0].long(), nc[rows, 0].long()
    slot = torch.arange(256, device=vc.device)
    kid = (f0.unsqueeze(1) + slot).clamp(0, M - 1)
    kid_vis = torch.where(slot < n0.unsqueeze(1), torch.gather(vc, 1, kid), torch.zeros_like(kid, dtype=vc.dtype))
    per_game = kid_vis.sum(1)
    assert int(per_game[active].min()) > 0 and int(per_game.sum()) == int(orch.sims_done.item())
    used = torch.arange(M, device=vc.device).unsqueeze(0) < cnt.unsqueeze(1).long()
    assert (tv.abs() <= vc.float() + 1e-3)[used].all()
    # each child's parent is the node whose child range holds it
    has = used & (fc >= 0) & (nc > 0)
    g, node = torch.nonzero(has, as_tuple=True)
    for j in range(0, 3):
        c = (fc[g, node] + j).long()
        ok = j < nc[g, node]
        assert (pa[g[ok], c[ok]] == node[ok].int()).all()
    assert sum(len(e) for e in ex) == B
