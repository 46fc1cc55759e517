"""Training-side batch builders (FNNTrainer._build_forward_batch and the
hybrid replay bundle) on the kernels: inputs bit-exact against the oracle,
and a differentiable torch forward / backward runs on them."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_build_forward_batch_matches_oracle_and_trains():
    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.training import build_forward_batch
    orc = O.oracle()
    st = np.concatenate([orc.generate_positions(61, 0, 300, 60, 0), orc.generate_positions(62, 0, 300, 140, 7)])
    mo, no, fo = orc.legal_moves_features(st)
    roots = np.repeat(np.arange(len(st), dtype=np.int64), no)
    idx = np.concatenate([np.arange(k, dtype=np.int64) for k in no])
    so = orc.successor_features(st, mo, roots, idx)
    rf, sf, atr, na = build_forward_batch(torch.from_numpy(st).cuda(), len(st))
    assert np.array_equal(rf.cpu().numpy().view(np.uint32), fo.view(np.uint32))
    assert np.array_equal(sf.cpu().numpy().view(np.uint32), so.view(np.uint32))
    assert np.array_equal(atr.cpu().numpy(), roots) and np.array_equal(na.cpu().numpy(), no.astype(np.int64))
    net = HiveFNN().cuda()
    logits, values = net(rf, sf, atr, na)
    (logits.square().mean() + values.square().mean()).backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in net.parameters())


def test_build_hybrid_forward_batch_matches_oracle():
    from hive_neuralnet_b200.hybrid import HiveHybridGNN
    from hive_neuralnet_b200.training import build_hybrid_forward_batch
    orc = O.oracle()
    st = orc.generate_positions(63, 0, 256, 150, 7)
    mo, no, fo = orc.legal_moves_features(st)
    tf, tq, tr, tz, tm, gf, nt, mf = orc.hybrid_encode(st, mo, no)
    rf, sf, atr, na, pb, mfv = build_hybrid_forward_batch(torch.from_numpy(st).cuda(), len(st))
    valid = np.arange(256)[None, :] < no[:, None]
    assert np.array_equal(rf.cpu().numpy().view(np.uint32), fo.view(np.uint32))
    assert np.array_equal(pb.token_features.cpu().numpy().view(np.uint32), tf.view(np.uint32))
    assert np.array_equal(pb.num_tokens.cpu().numpy(), nt)
    assert np.array_equal(mfv.cpu().numpy().view(np.uint32), mf[valid].view(np.uint32))
    torch.manual_seed(0)
    net = HiveHybridGNN().cuda()
    pbn = type(pb)(pb.token_features[..., :net.config.node_feat_dim], pb.token_q.long(), pb.token_r.long(),
                   pb.token_z.long(), pb.token_mask, pb.global_features, pb.num_tokens)
    logits, values = net(rf, sf, atr, na, pbn, mfv)
    (logits.square().mean() + values.square().mean()).backward()
    assert logits.shape[0] == int(no.sum()) and values.shape == (len(st), 1)
