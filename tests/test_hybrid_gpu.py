"""Hybrid FNN-transformer leaf evaluation on the B200 against the fp32 torch
statement of the network on the same seeded positions (tolerance 1e-2: the
trunk's GEMM operands are fp16), and the hybrid PUCT driver replaying
bit-exact on the oracle's tree operations given the evaluator's outputs."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _reference_eval(net, orc, st):
    """priors / values / logits of HybridMCTSOrchestrator._eval_states in fp32 (CPU)."""
    from hive_neuralnet_b200.hybrid import HybridPieceTensorBatch
    mo, no, fo = orc.legal_moves_features(st)
    tf, tq, tr, tz, tm, gf, nt, mf = orc.hybrid_encode(st, mo, no)
    roots = np.repeat(np.arange(len(st), dtype=np.int64), no)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in no])
    sf = orc.successor_features(st, mo, roots, idx)
    pb = HybridPieceTensorBatch(torch.from_numpy(tf[..., :net.config.node_feat_dim]), torch.from_numpy(tq).long(),
                                torch.from_numpy(tr).long(), torch.from_numpy(tz).long(),
                                torch.from_numpy(tm).bool(), torch.from_numpy(gf), torch.from_numpy(nt))
    valid = np.arange(256)[None, :] < no[:, None]
    with torch.no_grad():
        lg, vals = net(torch.from_numpy(fo), torch.from_numpy(sf), torch.from_numpy(roots),
                       torch.from_numpy(no.astype(np.int64)), pb, torch.from_numpy(mf[valid]))
    logits = np.full((len(st), 256), -1e30, np.float32)
    logits[valid] = lg.numpy()
    pri = torch.softmax(torch.from_numpy(logits), dim=1).numpy() * valid
    return mo, no, fo, logits, pri, vals.numpy().reshape(-1), valid


@pytest.mark.parametrize("preset", ["default", "small"])
@pytest.mark.parametrize("with_root_features", [True, False])
@pytest.mark.parametrize("path", ["rows", "fused"])
def test_hybrid_eval_matches_fp32_statement(preset, with_root_features, path):
    from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridEvaluator, HybridGNNConfig
    torch.manual_seed(11)
    net = HiveHybridGNN(HybridGNNConfig() if preset == "default" else HybridGNNConfig.small()).eval()
    orc = O.oracle()
    st = np.concatenate([orc.generate_positions(81, 0, 200, 60, 0), orc.generate_positions(82, 0, 200, 150, 7)])
    mo, no, fo, logits, pri, vals, valid = _reference_eval(net, orc, st)
    ev = HybridEvaluator(net)
    d = lambda a: torch.from_numpy(a).cuda()
    fn = ev.eval_states if path == "rows" else ev.eval_states_fused
    p, v, cq, lg = fn(d(st), d(mo), d(no), len(st), d(fo) if with_root_features else None, return_logits=True)
    p, v, cq, lg = (t.cpu().numpy() for t in (p, v, cq, lg))
    assert np.abs(lg - np.where(valid, logits, 0))[valid].max() < TOL
    assert np.abs(p - pri).max() < TOL
    assert np.abs(v - vals).max() < TOL
    assert (cq == 0).all() and (p[~valid] == 0).all()


def test_hybrid_puct_replays_bit_exact_on_oracle():
    from tests.test_orchestrator_gpu import _replay, _start, _tree_np
    from hive_neuralnet_b200.hybrid import HiveHybridGNN
    from hive_neuralnet_b200.orchestrator import HybridPUCTConfig, HybridPUCTOrchestrator
    B, M = 10, 8192
    torch.manual_seed(2)
    cfg = HybridPUCTConfig(num_simulations=64, batch_size=B, max_game_length=1, dirichlet_epsilon=0.0, seed=4,
                           max_tree_nodes=M, wave_size=32, c_puct=1.5)
    orch = HybridPUCTOrchestrator(HiveHybridGNN(), cfg)
    orch.trace = []
    ex = orch.self_play_batch(torch.from_numpy(_start(B, 19)).cuda())
    searched = next(x for x in orch.trace if x["kind"] == "searched")
    assert _tree_np(searched["tree"], B, M).equal(_replay(orch.trace, B, M, 1, cfg.c_puct)) == []
    assert sum(len(e) for e in ex) == B
