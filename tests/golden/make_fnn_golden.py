"""Pin the HiveFNN mirror to the REFERENCE module (run where the reference
tree exists): builds hive_fnn.fnn_network.HiveFNN from the reference with
torch.manual_seed(0) for each preset and records its state_dict and its
encode / value_head / score_actions outputs on seeded features.

    python tests/golden/make_fnn_golden.py
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle.oracle import reference_dir  # noqa: E402

sys.path.insert(0, reference_dir())

from hive_fnn.fnn_network import FNNConfig, HiveFNN  # noqa: E402  (the reference module)


def main():
    out = {}
    g = torch.Generator().manual_seed(123)
    feats = torch.rand((16, 122), generator=g) * 3.0
    succ = torch.rand((24, 122), generator=g) * 3.0
    atr = torch.randint(0, 16, (24,), generator=g)
    for name in ("small", "medium", "large"):
        torch.manual_seed(0)
        net = HiveFNN(getattr(FNNConfig, name)())
        sd = net.state_dict()
        for k, v in sd.items():
            out[f"{name}/{k}"] = v.numpy()
        with torch.no_grad():
            logits, values = net(feats, succ, atr, None)
        out[f"{name}/out_logits"] = logits.numpy()
        out[f"{name}/out_values"] = values.numpy()
        out[f"{name}/params"] = np.array(net.count_parameters())
    out["in/root"] = feats.numpy()
    out["in/succ"] = succ.numpy()
    out["in/action_to_root"] = atr.numpy()
    np.savez_compressed(os.path.join(HERE, "fnn_reference_seed0.npz"), **out)
    print({n: int(out[f"{n}/params"]) for n in ("small", "medium", "large")})


if __name__ == "__main__":
    main()
