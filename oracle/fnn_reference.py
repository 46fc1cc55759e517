"""fp32 PyTorch (CPU) restatement of the reference leaf evaluation.

TEST INFRASTRUCTURE ONLY (the checker for the fused FNN kernel).  Follows
hive_fnn/fnn_mcts_orchestrator.py:243-316 (_eval_states) step by step:
encode the roots and every legal successor (features from the oracle's
successor path, oracle/hive_oracle.c orc_successor_features_batch), value
head on the roots and on the successors, action tower on (root, successor)
pairs, scatter into [T, 256] with -1e30 padding, softmax, zero the padding,
child_q = -value(successor).
"""
from __future__ import annotations

import numpy as np
import torch


def eval_states_reference(net, root_features: np.ndarray, succ_features: np.ndarray,
                          num_legal: np.ndarray, max_legal: int = 256):
    total = root_features.shape[0]
    n64 = torch.from_numpy(num_legal.astype(np.int64))
    slot = torch.arange(max_legal).unsqueeze(0)
    valid = slot < n64.unsqueeze(1)
    action_to_root = torch.arange(total).unsqueeze(1).expand_as(valid)[valid]
    with torch.no_grad():
        rf = torch.from_numpy(root_features).float()
        sf = torch.from_numpy(succ_features).float()
        all_emb = net.encode(torch.cat([rf, sf], dim=0))
        root_emb, succ_emb = all_emb[:total], all_emb[total:]
        root_values = net.value_head(root_emb).squeeze(-1).float()
        child_values = net.value_head(succ_emb).squeeze(-1).float()
        logits = net.score_actions(root_emb[action_to_root], succ_emb).float()
    legal_logits = torch.full((total, max_legal), -1e30, dtype=torch.float32)
    legal_logits[valid] = logits
    priors = torch.softmax(legal_logits, dim=1).masked_fill(~valid, 0.0)
    child_q = torch.zeros((total, max_legal), dtype=torch.float32)
    child_q[valid] = -child_values
    raw = torch.zeros((total, max_legal), dtype=torch.float32)
    raw[valid] = logits
    return priors.numpy(), root_values.numpy(), child_q.numpy(), raw.numpy()
