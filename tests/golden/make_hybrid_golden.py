"""Pin the hybrid FNN-transformer mirror to the REFERENCE module (run where
the reference tree exists).  Builds hive_fnn_transformer's HiveHybridGNN with
torch.manual_seed(0) for the default and `small` configs, records a SHA-256
of every parameter (creation order) and the network's fp32 outputs on the
piece tokens / move features / FNN features of 24 seeded positions (inputs
made by the oracle, which tests/test_oracle.py pins to the reference).

    python tests/golden/make_hybrid_golden.py
"""
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle.oracle import reference_dir  # noqa: E402

sys.path.insert(0, reference_dir())

from oracle import oracle as O  # noqa: E402
from hive_fnn_transformer.fnn_transformer_net import HiveHybridGNN, HybridGNNConfig  # noqa: E402  (reference)
from hive_fnn_transformer.graph_types import HybridPieceTensorBatch  # noqa: E402  (reference)


def inputs():
    orc = O.oracle()
    st = np.concatenate([orc.generate_positions(31, 0, 12, 60, 0), orc.generate_positions(32, 0, 12, 120, 7)])
    mo, no, fo = orc.legal_moves_features(st)
    tf, tq, tr, tz, tm, gf, nt, mf = orc.hybrid_encode(st, mo, no)
    roots = np.repeat(np.arange(len(st), dtype=np.int64), no)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in no])
    sf = orc.successor_features(st, mo, roots, idx)
    return dict(states=st, moves=mo, num_legal=no, root_features=fo, token_features=tf, token_q=tq, token_r=tr,
                token_z=tz, token_mask=tm, global_features=gf, num_tokens=nt, move_features=mf, succ_roots=roots,
                succ_moves=idx, succ_features=sf)


def param_digest(net) -> str:
    h = hashlib.sha256()
    for name, p in net.named_parameters():
        h.update(name.encode())
        h.update(p.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def main():
    x = inputs()
    out = dict(x)
    for name, cfg in (("default", HybridGNNConfig()), ("small", HybridGNNConfig.small())):
        torch.manual_seed(0)
        net = HiveHybridGNN(cfg).eval()
        d = cfg.node_feat_dim
        pb = HybridPieceTensorBatch(
            token_features=torch.from_numpy(x["token_features"][..., :d]), token_q=torch.from_numpy(x["token_q"]).long(),
            token_r=torch.from_numpy(x["token_r"]).long(), token_z=torch.from_numpy(x["token_z"]).long(),
            token_mask=torch.from_numpy(x["token_mask"]).bool(), global_features=torch.from_numpy(x["global_features"]),
            num_tokens=torch.from_numpy(x["num_tokens"]))
        n = x["num_legal"]
        valid = np.arange(256)[None, :] < n[:, None]
        with torch.no_grad():
            logits, values = net(torch.from_numpy(x["root_features"]), torch.from_numpy(x["succ_features"]),
                                 torch.from_numpy(x["succ_roots"]), torch.from_numpy(n.astype(np.int64)), pb,
                                 torch.from_numpy(x["move_features"][valid]))
            g = net.graph_trunk(pb)
        out[f"{name}/params_sha256"] = np.array(param_digest(net))
        out[f"{name}/param_count"] = np.array(net.count_parameters())
        out[f"{name}/logits"] = logits.numpy()
        out[f"{name}/values"] = values.numpy()
        out[f"{name}/graph_summary"] = g.numpy()
        print(name, net.count_parameters())
    np.savez_compressed(os.path.join(HERE, "hybrid_reference_seed0.npz"), **out)


if __name__ == "__main__":
    main()
