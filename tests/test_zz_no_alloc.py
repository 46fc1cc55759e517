"""hv_hybrid_evaluate_noalloc (fixed file-scope device scratch) against the
workspace entry point hv_hybrid_evaluate (eval_states_fused), on two calls in a row; and the
oversize rejection.  Collected last; needs nothing from other test files."""

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _inputs(n):
    orc = O.oracle()
    st = np.concatenate([orc.generate_positions(901, 0, n // 2, 60, 0), orc.generate_positions(902, 0, n - n // 2,
                                                                                                 140, 7)])
    mo, no, fo = orc.legal_moves_features(st)
    return [torch.from_numpy(a).cuda() for a in (st, mo, no, fo)]


def test_noalloc_matches_workspace_entry_point_twice():
    from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridEvaluator
    torch.manual_seed(21)
    ev = HybridEvaluator(HiveHybridGNN().eval())
    st, mo, no, fo = _inputs(700)
    want = ev.eval_states_fused(st, mo, no, len(st), fo)
    for _ in range(2):
        got = ev.eval_states_noalloc(st, mo, no, len(st), fo)
        for g, w in zip(got, want):
            assert torch.equal(g, w)
    # root features computed in the kernel, then a smaller call reusing the scratch
    want2 = ev.eval_states_fused(st[:123], mo[:123], no[:123], 123)
    got2 = ev.eval_states_noalloc(st[:123], mo[:123], no[:123], 123)
    for g, w in zip(got2, want2):
        assert torch.equal(g, w)


def test_noalloc_rejects_oversize_request():
    from hive_neuralnet_b200 import _lib
    lib = _lib.load()
    n = 9138  # one more than the fixed scratch holds
    buf = torch.zeros((n, 3424), dtype=torch.uint8, device="cuda")
    mv = torch.zeros((n, 256, 6), dtype=torch.uint8, device="cuda")
    nl = torch.zeros((n,), dtype=torch.int32, device="cuda")
    out = torch.zeros((n, 256), dtype=torch.float32, device="cuda")
    rc = lib.hv_hybrid_evaluate_noalloc(buf.data_ptr(), mv.data_ptr(), nl.data_ptr(), None, n, 26, buf.data_ptr(),
                                        out.data_ptr(), out.data_ptr(), 64, 64, 64, out.data_ptr(), 128,
                                        out.data_ptr(), out.data_ptr(), out.data_ptr(), None,
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 6
    assert b"9137" in lib.hv_status_string(rc)
