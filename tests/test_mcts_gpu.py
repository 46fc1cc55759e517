"""GPU parity of the MCTS tree kernels (hive_gpu mirror -> C ABI -> sm_100a)
against the sequential oracle: after several select / replay / expand+backup
waves the whole tree (visit counts, value sums as raw float bits, priors,
parents, moves, actions, children, terminal flags, node counts, child Q)
must be bit-identical, for every select mode and wave width.  The waves run
the parallel select and expansion forms (one warp per root candidate in
root-slot waves, the root steps first and then the root children's
subtrees in parallel in plain and root-mask waves); root-slot tables that
repeat a slot take the per-game order, so both forms are compared with the
oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.mcts_sim import OracleBackend, run_waves

pytestmark = pytest.mark.gpu


class GpuBackend:
    """Runs each tree operation on the GPU through the reference-named API."""

    def __init__(self):
        from hive_neuralnet_b200.hive_gpu import load_extension
        self.ext = load_extension()

    @staticmethod
    def _up(tree):
        ts = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in tree.arrays()]
        return ts, torch.from_numpy(tree.child_init_q).cuda()

    @staticmethod
    def _down(tree, ts, ciq):
        for a, t in zip(tree.arrays(), ts):
            a[...] = t.cpu().numpy()
        tree.child_init_q[...] = ciq.cpu().numpy()

    @staticmethod
    def _t(a, dt=None):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        return t if dt is None else t.to(dt)

    def select(self, tree, mode, game_active, root_nodes, alive_mask=None, root_slots=None, num_candidates=1,
               max_root_children=256, c_puct=1.25, W=1, det=False, sigma=4.0, q_penalty=0.0):
        ts, ciq = self._up(tree)
        B, M = tree.B, tree.max_nodes
        ga, rn = self._t(game_active), self._t(root_nodes)
        if mode == 0:
            out = self.ext.mcts_select_batch(*ts, ga, rn, c_puct, B, W, M)
        elif mode == 1:
            out = self.ext.mcts_select_with_root_mask_batch(*ts, ciq, ga, rn, self._t(alive_mask),
                                                            max_root_children, c_puct, B, W, M, det, sigma, q_penalty)
        else:
            out = self.ext.mcts_select_with_root_slots_batch(*ts, ciq, ga, rn, self._t(root_slots), num_candidates,
                                                             max_root_children, c_puct, B, W, M, det, sigma,
                                                             q_penalty)
        torch.cuda.synchronize()
        self._down(tree, ts, ciq)
        return tuple(x.cpu().numpy() for x in out)

    def replay(self, root_states, paths, plen, leaf, B):
        out = torch.zeros((len(leaf), 3424), dtype=torch.uint8, device="cuda")
        self.ext.mcts_replay_batch(self._t(root_states), out, self._t(paths), self._t(plen), self._t(leaf), B,
                                   len(leaf))
        return out.cpu().numpy()

    def expand_dense(self, tree, child_q, leaf, leaf_states, legal, num_legal, priors, results, values=None,
                     vl_paths=None, vl_len=None, q_penalty=0.0, with_backprop=True, slots=None):
        ts, ciq = self._up(tree)
        B, M, total = tree.B, tree.max_nodes, len(leaf)
        args = (self._t(child_q), self._t(leaf), self._t(leaf_states), self._t(legal), self._t(num_legal),
                self._t(priors), self._t(results))
        was = None
        if with_backprop and slots is not None:
            # the grouped expansion (hv_mcts_expand_slots): by candidate, or by root child
            roots, root_slots, C = slots
            self.ext.mcts_expand_and_backprop_dense_priors_slots_batch(
                *ts, ciq, *args, self._t(values), self._t(vl_paths), self._t(vl_len), self._t(roots),
                None if root_slots is None else self._t(root_slots), C, B, total, M, q_penalty)
        elif with_backprop:
            self.ext.mcts_expand_and_backprop_dense_priors_batch(*ts, ciq, *args, self._t(values), self._t(vl_paths),
                                                                 self._t(vl_len), B, total, M, q_penalty)
        else:
            was = self.ext.mcts_expand_dense_priors_batch(*ts, ciq, *args, B, total, M).cpu().numpy()
        torch.cuda.synchronize()
        self._down(tree, ts, ciq)
        return was


def _states(seed, n=32):
    orc = O.oracle()
    return np.concatenate([orc.generate_positions(seed, 0, n // 2, 40, 0),
                           orc.generate_positions(seed + 1, 0, n - n // 2, 90, 7)])


@pytest.mark.parametrize("grouped", [True, False])
@pytest.mark.parametrize("mode,W", [(0, 1), (0, 4), (1, 1), (1, 4), (2, 1), (2, 4), (2, 16)])
def test_tree_waves_bit_exact(mode, W, grouped):
    # grouped: the waves' expansion + backup through hv_mcts_expand_slots,
    # else through the per-game hv_mcts_expand
    st = _states(300 + 7 * mode + W)
    a, la = run_waves(OracleBackend("orc"), st, waves=8, W=W, mode=mode, seed=11)
    b, lb = run_waves(GpuBackend(), st, waves=8, W=W, mode=mode, seed=11, grouped=grouped)
    for (x1, y1, z1), (x2, y2, z2) in zip(la, lb):
        assert np.array_equal(x1, x2) and np.array_equal(y1, y2) and np.array_equal(z1, z2)
    assert a.equal(b) == []
    assert a.visit_count[:, 0].sum() > 0


@pytest.mark.parametrize("W", [1, 4])
def test_root_slot_waves_with_repeated_slots_bit_exact(W):
    # games whose candidate table lists a slot twice share a subtree between
    # two candidates: select and expansion keep the per-game order there
    st = _states(900 + W)
    a, la = run_waves(OracleBackend("orc"), st, waves=8, W=W, mode=2, seed=13, repeat_slots=True)
    b, lb = run_waves(GpuBackend(), st, waves=8, W=W, mode=2, seed=13, repeat_slots=True)
    for (x1, y1, z1), (x2, y2, z2) in zip(la, lb):
        assert np.array_equal(x1, x2) and np.array_equal(y1, y2) and np.array_equal(z1, z2)
    assert a.equal(b) == []
    assert a.visit_count[:, 0].sum() > 0


def test_deterministic_completed_q_runs():
    # logf/expf differ in the last ulp between libm and CUDA, so this mode is
    # checked for tree invariants rather than bit equality
    st = _states(900, 16)
    b, _ = run_waves(GpuBackend(), st, waves=5, W=4, mode=2, seed=5, det=True, q_penalty=0.25)
    assert np.abs(b.virtual_q_penalty).max() < 1e-6
    assert (b.visit_count >= 0).all()


def test_action_space_policy_and_noise():
    from hive_neuralnet_b200.hive_gpu import load_extension
    ext = load_extension()
    orc = O.oracle()
    st = _states(77, 16)
    B, M = len(st), 2048
    tree_o = O.TreeArrays(B, M)
    mv, nl, _ = orc.legal_moves_features(st)
    res = st[:, 3415].astype(np.int32)
    probs = np.random.default_rng(3).uniform(size=(B, 85834)).astype(np.float32)
    was_o = O.mcts_expand_action("orc", tree_o, 0, np.zeros(B, np.int32), st, mv, nl, probs, res)
    ts = [torch.from_numpy(x.copy()).cuda() for x in O.TreeArrays(B, M).arrays()]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    was_g = ext.mcts_expand_batch(*ts, t(np.zeros(B, np.int32)), t(st), t(mv), t(nl), t(probs), t(res), B, B, M)
    assert np.array_equal(was_g.cpu().numpy(), was_o)
    vals = np.full(B, 0.25, np.float32)
    O.mcts_expand_action("orc", tree_o, 2, np.zeros(B, np.int32), st, mv, nl, probs, res, values=vals,
                         was_expanded=was_o)
    ext.mcts_backprop_batch(*ts, t(np.zeros(B, np.int32)), t(vals), t(np.zeros((B, 128), np.int32)),
                            t(np.zeros(B, np.int32)), was_g, B, B, M)
    for wave in range(3):
        lo = O.mcts_select("orc", tree_o, mode=0, game_active=np.ones(B, np.int8), root_nodes=np.zeros(B, np.int32), W=2)
        lg = ext.mcts_select_batch(*ts, t(np.ones(B, np.int8)), t(np.zeros(B, np.int32)), 1.25, B, 2, M)
        assert np.array_equal(lo[0], lg[0].cpu().numpy())
        ls = O.mcts_replay("orc", st, lo[1], lo[2], lo[0], B)
        lmv, lnl, _ = orc.legal_moves_features(ls)
        lp = np.random.default_rng(wave).uniform(size=(len(lo[0]), 85834)).astype(np.float32)
        v = np.linspace(-0.9, 0.9, len(lo[0])).astype(np.float32)
        lres = ls[:, 3415].astype(np.int32)
        O.mcts_expand_action("orc", tree_o, 1, lo[0], ls, lmv, lnl, lp, lres, v, lo[3], lo[4])
        ext.mcts_expand_and_backprop_batch(*ts, lg[0], t(ls), t(lmv), t(lnl), t(lp), t(lres), t(v), lg[3], lg[4],
                                           B, len(lo[0]), M)
    tree_g = O.TreeArrays(B, M)
    for a, x in zip(tree_g.arrays(), ts):
        a[...] = x.cpu().numpy()
    assert tree_o.equal(tree_g) == []
    for temp, drop, prune in [(1.0, 30, 0.0), (1.0, 30, 0.2), (1.0, 0, 0.0)]:
        po = O.mcts_extract_policy("orc", tree_o, np.zeros(B), np.zeros(B), temp, drop, prune)
        pg = ext.mcts_extract_policy_batch(*ts, t(np.zeros(B, np.int32)), t(np.zeros(B, np.int32)), temp, drop,
                                           prune, B, M).cpu().numpy()
        assert np.array_equal(po.view(np.uint32), pg.view(np.uint32))
    noise = np.random.default_rng(9).dirichlet(np.full(256, 0.3), size=B).astype(np.float32)
    O.mcts_root_noise("orc", tree_o, noise, np.zeros(B), 0.25, 1.0)
    ext.mcts_apply_root_noise(*ts, t(noise), t(np.zeros(B, np.int32)), 256, 0.25, 1.0, B, M)
    tree_g = O.TreeArrays(B, M)
    for a, x in zip(tree_g.arrays(), ts):
        a[...] = x.cpu().numpy()
    assert tree_o.equal(tree_g) == []


def test_fused_wave_prefix_matches_components():
    from hive_neuralnet_b200.hive_gpu import load_extension
    ext = load_extension()
    orc = O.oracle()
    st = _states(55, 16)
    B, M, C, W = len(st), 2048, 4, 2
    tree = O.TreeArrays(B, M)
    mv, nl, _ = orc.legal_moves_features(st)
    valid = np.arange(256)[None, :] < nl[:, None]
    pri = np.where(valid, 1.0 / np.maximum(nl, 1)[:, None], 0).astype(np.float32)
    O.mcts_expand_dense("orc", tree, np.zeros((B, 256), np.float32), np.zeros(B, np.int32), st, mv, nl, pri,
                        st[:, 3415].astype(np.int32), with_backprop=False)
    slots = np.tile(np.arange(C, dtype=np.int32), (B, 1))
    slots = np.where(slots < nl[:, None], slots, -1).astype(np.int32)
    ts = [torch.from_numpy(x.copy()).cuda() for x in tree.arrays()]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = ext.mcts_select_replay_legal_fnn_root_slots_batch(
        *ts, t(tree.child_init_q), t(st), t(((st[:, 3415] == 0) & (nl > 0)).astype(np.int8)), t(np.zeros(B, np.int32)),
        t(slots), C, 256, 1.25, B, W, M)
    leaf, ls, lm, ln, lf, lr, vlp, vll = (x.cpu().numpy() for x in out)
    lo = O.mcts_select("orc", tree, mode=2, game_active=((st[:, 3415] == 0) & (nl > 0)).astype(np.int8),
                       root_nodes=np.zeros(B, np.int32), root_slots=slots, num_candidates=C, W=W)
    assert np.array_equal(leaf, lo[0]) and np.array_equal(vll, lo[4])
    ls_o = O.mcts_replay("orc", st, lo[1], lo[2], lo[0], B)
    assert np.array_equal(ls, ls_o)
    m_o, n_o, f_o = orc.legal_moves_features(ls_o)
    assert np.array_equal(lm, m_o) and np.array_equal(ln, n_o)
    assert np.array_equal(lf.view(np.uint32), f_o.view(np.uint32))
    assert np.array_equal(lr, ls_o[:, 3415].astype(np.int32))
