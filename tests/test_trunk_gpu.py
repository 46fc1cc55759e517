"""The hybrid evaluator's transformer trunk on the tensor cores (fp16 tcgen05
GEMMs, fp32 attention) against the fp32 torch statement of the network and
the reference module's own outputs; tolerance 1e-2 (16-bit operands, the bound the
reference's autocast network is held to)."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "hybrid_reference_seed0.npz")
TOL = 1e-2


def _batch(ext, st):
    from hive_neuralnet_b200.hybrid import HybridPieceTensorBatch
    d = torch.from_numpy(st).cuda()
    mo, no = ext.generate_legal_moves_batch(d, len(st))
    tf, tq, tr, tz, tm, gf, nt = ext.hybrid_transformer_encode_with_moves_batch(d, mo, no, len(st))
    return HybridPieceTensorBatch(tf, tq, tr, tz, tm, gf, nt)


def _cpu(pb, nfeat):
    from hive_neuralnet_b200.hybrid import HybridPieceTensorBatch
    return HybridPieceTensorBatch(pb.token_features[..., :nfeat].cpu(), pb.token_q.cpu().long(),
                                  pb.token_r.cpu().long(), pb.token_z.cpu().long(), pb.token_mask.cpu(),
                                  pb.global_features.cpu(), pb.num_tokens.cpu())


@pytest.mark.parametrize("preset", ["default", "small"])
def test_trunk_matches_fp32_statement(preset):
    from hive_neuralnet_b200.hive_gpu import load_extension
    from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridGNNConfig, HybridTrunk
    ext = load_extension()
    torch.manual_seed(3)
    net = HiveHybridGNN(HybridGNNConfig() if preset == "default" else HybridGNNConfig.small()).eval()
    # exercise the learned parts that are zero at init
    with torch.no_grad():
        net.graph_trunk.cls_token.normal_(0, 0.5)
    orc = O.oracle()
    st = np.concatenate([orc.generate_positions(71, 0, 300, 60, 0), orc.generate_positions(72, 0, 301, 150, 7)])
    pb = _batch(ext, st)
    got = HybridTrunk(net)(pb).cpu()
    with torch.no_grad():
        want = net.graph_trunk(_cpu(pb, net.config.node_feat_dim))
    err = (got - want).abs().max().item()
    assert torch.isfinite(got).all()
    assert err < TOL * max(1.0, want.abs().max().item()), f"max abs error {err}"
    assert ext.device_error_word(clear=True) == 0


def test_trunk_matches_reference_module_outputs():
    from hive_neuralnet_b200.hive_gpu import load_extension
    from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridTrunk
    g = dict(np.load(GOLD))
    ext = load_extension()
    torch.manual_seed(0)
    net = HiveHybridGNN().eval()
    pb = _batch(ext, g["states"])
    assert np.array_equal(pb.token_features.cpu().numpy(), g["token_features"])
    got = HybridTrunk(net)(pb).cpu().numpy()
    np.testing.assert_allclose(got, g["default/graph_summary"], atol=TOL, rtol=TOL)


@pytest.mark.parametrize("n", [1, 3, 37, 601])
def test_packed_trunk_equals_unpacked(n):
    # positions with at most 15 token slots in use share a 32-row slot in
    # pairs: the output is the one-position-per-slot output bit for bit,
    # for batches with an odd number of small positions and ragged passes
    from hive_neuralnet_b200.hive_gpu import load_extension
    from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridTrunk
    ext = load_extension()
    torch.manual_seed(5)
    net = HiveHybridGNN().eval()
    with torch.no_grad():
        net.graph_trunk.cls_token.normal_(0, 0.5)
    orc = O.oracle()
    st = np.concatenate([orc.generate_positions(81, 0, n, 12, 0), orc.generate_positions(82, 0, n, 150, 7)])
    rng = np.random.default_rng(n)
    st = st[rng.permutation(len(st))][:max(n, 2)]
    pb = _batch(ext, st)
    small = int((pb.token_mask[:, 15:].sum(1) == 0).sum().item())
    trunk = HybridTrunk(net)
    a = trunk(pb, packed=True)
    b = trunk(pb, packed=False)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32)), f"{small} small of {len(st)}"
    assert ext.device_error_word(clear=True) == 0
