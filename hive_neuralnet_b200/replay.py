"""Replay-sample exchange between self-play ranks.

Self-play games are sharded across GPUs with no collective on the hot path;
once per training iteration every rank's ``FNNTrainingExample`` list
(hive_fnn/fnn_replay_buffer.py:21-31) is gathered so that every rank holds
the whole iteration's samples.  The examples travel as one size-prefixed
byte buffer per rank through ``torch.distributed.all_gather`` (NCCL over
NVLink for CUDA tensors, gloo for CPU tensors): two collectives per
iteration, the buffer sizes and then the padded buffers.

Record layout (little-endian, 4-byte aligned):
  u16 n (policy length, <= 256) | u8 flags (bit 0 use_for_policy, bit 1
  use_for_value) | u8 0 | f32 value_target | f32 value_weight |
  f32 surprise_weight | 3424 state bytes | n x f32 policy target
"""
from __future__ import annotations

import struct

import numpy as np
import torch

from .orchestrator import FNNTrainingExample

STATE_BYTES = 3424
_HEAD = struct.Struct("<HBBfff")  # 16 bytes


def pack_examples(examples: list[FNNTrainingExample]) -> np.ndarray:
    """Serialise examples into one uint8 buffer."""
    parts = []
    for e in examples:
        sb = np.ascontiguousarray(e.state_bytes, dtype=np.uint8).reshape(-1)
        if sb.size != STATE_BYTES:
            raise ValueError(f"state_bytes: expected {STATE_BYTES} bytes, got {sb.size}")
        pol = np.ascontiguousarray(e.policy_target, dtype=np.float32).reshape(-1)
        if pol.size > 256:
            raise ValueError("policy_target longer than 256")
        flags = (1 if e.use_for_policy else 0) | (2 if e.use_for_value else 0)
        parts.append(np.frombuffer(_HEAD.pack(pol.size, flags, 0, float(e.value_target), float(e.value_weight),
                                              float(e.surprise_weight)), dtype=np.uint8))
        parts.append(sb)
        parts.append(pol.view(np.uint8))
    return np.concatenate(parts) if parts else np.zeros(0, np.uint8)


def unpack_examples(buf: np.ndarray) -> list[FNNTrainingExample]:
    """Inverse of :func:`pack_examples`."""
    buf = np.ascontiguousarray(buf, dtype=np.uint8).reshape(-1)
    out, off = [], 0
    while off < buf.size:
        if off + _HEAD.size + STATE_BYTES > buf.size:
            raise ValueError("truncated replay buffer")
        n, flags, _, v, vw, sw = _HEAD.unpack_from(buf, off)
        off += _HEAD.size
        sb = buf[off:off + STATE_BYTES].copy()
        off += STATE_BYTES
        if off + 4 * n > buf.size:
            raise ValueError("truncated replay buffer")
        pol = buf[off:off + 4 * n].copy().view(np.float32)
        off += 4 * n
        out.append(FNNTrainingExample(sb, pol, float(v), bool(flags & 1), bool(flags & 2), float(vw), float(sw)))
    return out


def gather_examples(examples: list[FNNTrainingExample], group=None,
                    device: torch.device | str | None = None) -> list[FNNTrainingExample]:
    """All-gather every rank's examples; returns them in rank order on every rank.
    ``device`` is where the buffers live for the collective (a CUDA device for
    NCCL, CPU for gloo); by default CUDA when the backend is NCCL."""
    import torch.distributed as dist
    if not dist.is_initialized():
        return list(examples)
    world = dist.get_world_size(group)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
            else torch.device("cpu")
    local = torch.from_numpy(pack_examples(examples)).to(device)
    size = torch.tensor([local.numel()], dtype=torch.int64, device=device)
    sizes = [torch.zeros_like(size) for _ in range(world)]
    dist.all_gather(sizes, size, group=group)
    sizes = [int(s.item()) for s in sizes]
    cap = max(max(sizes), 1)
    padded = torch.zeros((cap,), dtype=torch.uint8, device=device)
    padded[:local.numel()] = local
    bufs = [torch.empty((cap,), dtype=torch.uint8, device=device) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    out = []
    for b, n in zip(bufs, sizes):
        out.extend(unpack_examples(b[:n].cpu().numpy()))
    return out
