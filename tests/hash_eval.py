"""Test helper: a leaf evaluator whose outputs are bit-identical on the CPU
and on a GPU.

It stands in for the network in search-parity tests, so that a search run by
the reference's own driver on the CPU and the same search run by this
package on a B200 see the same priors, values and child Q to the last bit:
the outputs are functions of the state bytes computed in int64 and scaled by
powers of two (exact in float32), with no transcendental or division whose
last ulp could differ between devices.

* h = sum over the 3424 state bytes of byte * w_j (fixed seeded weights);
* prior of legal slot i: w_i / 2^k with w_i = 1 + (a * i + b) mod 256
  (a odd, so the weights of one state are distinct: no ties in a top-k) and
  2^k the smallest power of two >= sum w (priors sum to at most 1);
* value: (h >> 14) mod 2049 - 1024, times 2^-10;
* child Q of slot i: (31 h + 977 i) mod 2049 - 1024, times 2^-10.
Tree sums of such values stay exact in float32 for any order of addition.
"""
from __future__ import annotations

import numpy as np
import torch

_W = torch.from_numpy(np.random.default_rng(777).integers(1, 1 << 20, 3424, dtype=np.int64))


def hash_eval(states: torch.Tensor, legal_moves: torch.Tensor, num_legal: torch.Tensor, total: int,
              root_features=None):
    """(priors [total, 256] f32, values [total] f32, child_q [total, 256] f32)."""
    dev = states.device
    st = states[:total].to(torch.int64)
    h = (st * _W.to(dev)).sum(dim=1)
    slot = torch.arange(256, device=dev, dtype=torch.int64).unsqueeze(0)
    valid = slot < num_legal[:total].to(torch.int64).unsqueeze(1)
    a = 2 * (h % 64) + 1
    b = (h // 64) % 256
    w = 1 + (a.unsqueeze(1) * slot + b.unsqueeze(1)) % 256
    w = torch.where(valid, w, torch.zeros_like(w))
    p = w.sum(dim=1).clamp(min=1) - 1  # smallest power of two >= the sum, by bit smearing
    for sh in (1, 2, 4, 8, 16, 32):
        p = p | (p >> sh)
    p = p + 1
    # a division by a power of two is exact however a device implements it
    priors = w.to(torch.float32) / p.to(torch.float32).unsqueeze(1)
    scale = torch.tensor(2.0 ** -10, dtype=torch.float32, device=dev)
    values = ((h // 16384) % 2049 - 1024).to(torch.float32) * scale
    cq = (((h.unsqueeze(1) * 31 + slot * 977) % 2049) - 1024).to(torch.float32) * scale
    cq = torch.where(valid, cq, torch.zeros_like(cq))
    return priors.contiguous(), values.contiguous(), cq.contiguous()
