"""GPU test of the tensor-core kernels' give-up path.

Every mbarrier wait of the bulk-copy / tcgen05 kernels (the hybrid trunk,
the hybrid row and leaf networks, the FP32 row network) is bounded.  With the
test-only limit hv_set_wait_limit_ns(0) each such wait gives up at once while
the copy or MMA it waits for is still in flight: the kernel records its error
bit, waits (up to 1 s, the fixed drain limit) for the work it started, frees
its tensor memory and returns.  Checked: the call returns, the error bits
are set, and with the limit restored the next call on the same context is
clean and gives the same bytes as before.  No wait here is left without an
end: the copies and MMAs complete on their own, only the waiting stops."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEFAULT_LIMIT_NS = 1_000_000_000


def _inputs(count, seed):
    orc = O.oracle()
    st = orc.generate_positions(seed, 0, count, 60, 7)
    mv, nl, ft = orc.legal_moves_features(st)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t(st), t(mv), t(nl), t(ft)


def _give_up_once(ext, run):
    lib = ext._lib
    assert ext.device_error_word(clear=True) == 0
    want = [x.clone() for x in run()]
    torch.cuda.synchronize()
    assert ext.device_error_word(clear=True) == 0
    assert lib.hv_set_wait_limit_ns(0) == 0
    try:
        run()
        torch.cuda.synchronize()
        err = ext.device_error_word(clear=True)
    finally:
        assert lib.hv_set_wait_limit_ns(DEFAULT_LIMIT_NS) == 0
    again = run()
    torch.cuda.synchronize()
    assert ext.device_error_word(clear=True) == 0
    for a, b in zip(again, want):
        assert torch.equal(a, b)
    return err


def test_hybrid_kernels_give_up_and_recover():
    from hive_neuralnet_b200.hive_gpu import load_extension
    from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridEvaluator
    ext = load_extension()
    torch.manual_seed(0)
    ev = HybridEvaluator(HiveHybridGNN().eval())
    st, mv, nl, ft = _inputs(300, 61)
    err = _give_up_once(ext, lambda: ev.eval_states(st, mv, nl, len(st), ft))
    assert err & 4, f"trunk give-up bit missing: {err:#x}"
    assert err & 8, f"row / leaf network give-up bit missing: {err:#x}"


def test_fnn_row_network_gives_up_and_recovers():
    from hive_neuralnet_b200.fnn import FusedFNNEvaluator, HiveFNN
    from hive_neuralnet_b200.hive_gpu import load_extension
    ext = load_extension()
    torch.manual_seed(0)
    ev = FusedFNNEvaluator(HiveFNN().eval())
    st, mv, nl, ft = _inputs(300, 62)
    err = _give_up_once(ext, lambda: ev.eval_states(st, mv, nl, len(st), ft))
    assert err & 8, f"row network give-up bit missing: {err:#x}"
