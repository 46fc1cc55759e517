"""FNN leaf evaluator: the reference's HiveFNN and a fused sm_100a evaluation.

``HiveFNN`` / ``FNNConfig`` keep the reference's module layout, parameter
names and presets (hive_fnn/fnn_network.py:24-176), so reference checkpoints
and seeded random initialisations load unchanged.  ``FusedFNNEvaluator``
replaces the reference's leaf evaluation
(``FNNMCTSOrchestrator._eval_states``, hive_fnn/fnn_mcts_orchestrator.py:243-316:
successor features -> encode -> value head -> action tower -> masked softmax)
with one kernel launch that never materialises successor features in HBM.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.nn as nn

from . import _lib

FEAT_DIM = 122
MAX_LEGAL = 256


@dataclass
class FNNConfig:
    """Same fields and presets as hive_fnn/fnn_network.py:24-44."""

    feat_dim: int = FEAT_DIM
    hidden_dim: int = 64
    embed_dim: int = 64
    action_hidden: int = 64

    @classmethod
    def small(cls) -> "FNNConfig":
        return cls(hidden_dim=8, embed_dim=8, action_hidden=8)

    @classmethod
    def medium(cls) -> "FNNConfig":
        return cls(hidden_dim=32, embed_dim=32, action_hidden=32)

    @classmethod
    def large(cls) -> "FNNConfig":
        return cls(hidden_dim=64, embed_dim=64, action_hidden=64)


class HiveFNN(nn.Module):
    """Module with the reference's layers, in the reference's creation order
    (so ``torch.manual_seed(s); HiveFNN()`` draws the same initial weights)."""

    def __init__(self, config: FNNConfig | None = None) -> None:
        super().__init__()
        self.config = config or FNNConfig.large()
        self.config.feat_dim = FEAT_DIM
        c = self.config
        self.fc1 = nn.Linear(c.feat_dim, c.hidden_dim)
        self.ln1 = nn.LayerNorm(c.hidden_dim)
        self.fc2 = nn.Linear(c.hidden_dim, c.embed_dim)
        self.value_fc = nn.Linear(c.embed_dim, 1)
        self.action_fc1 = nn.Linear(c.embed_dim * 2, c.action_hidden)
        self.action_fc2 = nn.Linear(c.action_hidden, 1)

    @staticmethod
    def _pad_loaded_weight(old: torch.Tensor, new_template: torch.Tensor, *, noise_scale: float = 1e-3):
        """A checkpoint's fc1 weight of another feature width: the overlap is
        copied, the rest drawn from N(0, noise_scale) (fnn_network.py:74-85)."""
        new = torch.empty_like(new_template)
        new.normal_(mean=0.0, std=noise_scale)
        rows, cols = min(old.shape[0], new.shape[0]), min(old.shape[1], new.shape[1])
        new[:rows, :cols] = old[:rows, :cols]
        return new

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        """fnn_network.py:87-94: checkpoints written with another feature width load."""
        state = dict(state_dict)
        cur = self.state_dict()
        key = "fc1.weight"
        if key in state and key in cur and state[key].shape != cur[key].shape:
            state[key] = self._pad_loaded_weight(state[key], cur[key])
        return super().load_state_dict(state, strict=strict, assign=assign)

    def encode(self, features: torch.Tensor) -> torch.Tensor:
        return self.fc2(self.ln1(torch.sigmoid(self.fc1(features))))

    def value_head(self, embed: torch.Tensor) -> torch.Tensor:
        return torch.tanh(self.value_fc(embed))

    def score_actions(self, root_embed: torch.Tensor, successor_embed: torch.Tensor) -> torch.Tensor:
        combined = torch.cat([root_embed, successor_embed], dim=1)
        return self.action_fc2(torch.sigmoid(self.action_fc1(combined))).squeeze(-1)

    def forward(self, root_features, successor_features, action_to_root, num_actions):
        root_emb = self.encode(root_features)
        root_values = self.value_head(root_emb)
        if action_to_root.shape[0] == 0:
            return root_features.new_zeros((0,)), root_values
        succ_emb = self.encode(successor_features)
        return self.score_actions(root_emb[action_to_root], succ_emb), root_values

    def count_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad)


def pack_weights(net: HiveFNN, device: torch.device | str = "cuda") -> torch.Tensor:
    """Pack the parameters (fp32) in the kernel's transposed layout:
    fc1.W^T, fc1.b, ln1.w, ln1.b, fc2.W^T, fc2.b, value.w, value.b,
    action_fc1.W^T, action_fc1.b, action_fc2.w, action_fc2.b."""
    with torch.no_grad():
        parts = [
            net.fc1.weight.t(), net.fc1.bias, net.ln1.weight, net.ln1.bias,
            net.fc2.weight.t(), net.fc2.bias,
            net.value_fc.weight.reshape(-1), net.value_fc.bias,
            net.action_fc1.weight.t(), net.action_fc1.bias,
            net.action_fc2.weight.reshape(-1), net.action_fc2.bias,
        ]
        flat = torch.cat([p.detach().float().contiguous().reshape(-1) for p in parts])
    return flat.to(device).contiguous()


# Batches up to this many leaves size the row workspace for 256 rows per leaf
# (about 2 GB at 16,384 leaves) instead of counting the rows: the count would
# be a device -> host read, one synchronisation per search wave.  The row
# kernels read the actual count from the device.
ROWS_BOUND_MAX_LEAVES = 16384


def _rows(num_legal: torch.Tensor, total: int) -> int:
    """Rows to size the row pipeline for: an upper bound (256 per leaf, no
    synchronisation) for batches up to ROWS_BOUND_MAX_LEAVES, else the exact
    sum of min(max(num_legal, 0), 256) (one device sync)."""
    if total <= ROWS_BOUND_MAX_LEAVES:
        return total * MAX_LEGAL
    return int(num_legal[:total].clamp(0, MAX_LEGAL).sum().item())


class _Workspace:
    """Device scratch that only grows (256-byte aligned from the caching allocator)."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, dev) -> torch.Tensor:
        if self.buf is None or self.buf.device != dev or self.buf.numel() < nbytes:
            self.buf = torch.empty((max(int(nbytes * 1.25), 256),), dtype=torch.uint8, device=dev)
        return self.buf


class FusedFNNEvaluator:
    """Leaf evaluation on the device.

    ``eval_states`` has the signature and outputs of the reference's
    ``FNNMCTSOrchestrator._eval_states``: (priors_per_legal [T,256],
    root_values [T], child_q_per_legal [T,256]).  It runs the row pipeline
    (``hv_fnn_eval_leaves_rows``: successor features of all leaves, then the
    network as a tiled fp32 GEMM over the successor rows); ``eval_states_fused``
    runs the single warp-per-leaf kernel (``hv_fnn_eval_leaves``), which needs
    no workspace."""

    def __init__(self, net: HiveFNN, device: torch.device | str = "cuda"):
        self.net = net
        self.device = torch.device(device)
        self.lib = _lib.load()
        c = net.config
        self.dims = (c.hidden_dim, c.embed_dim, c.action_hidden)
        self.ws = _Workspace()
        self.refresh()

    def refresh(self) -> None:
        """Re-pack the weights (call after the network was trained)."""
        self.weights = pack_weights(self.net, self.device)
        want = self.lib.hv_fnn_weights_size(*self.dims)
        if want != self.weights.numel():
            raise ValueError(f"packed {self.weights.numel()} floats, kernel expects {want}")

    def _outputs(self, states, legal_moves, num_legal, total, root_features, return_logits):
        dev = states.device
        priors = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        values = torch.empty((total,), dtype=torch.float32, device=dev)
        child_q = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        logits = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev) if return_logits else None
        for t, name, dt in ((states, "states", torch.uint8), (legal_moves, "legal_moves", torch.uint8),
                            (num_legal, "num_legal", torch.int32)):
            if t.dtype != dt or not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{name}: expected contiguous CUDA {dt}")
        if root_features is not None and (root_features.dtype != torch.float32 or not root_features.is_contiguous()):
            raise ValueError("root_features: expected contiguous float32")
        return priors, values, child_q, logits

    def eval_states(self, states: torch.Tensor, legal_moves: torch.Tensor, num_legal: torch.Tensor,
                    total: int, root_features: torch.Tensor | None = None, return_logits: bool = False):
        import ctypes
        priors, values, child_q, logits = self._outputs(states, legal_moves, num_legal, total, root_features,
                                                        return_logits)
        if total > 0:
            dev = states.device
            rows = _rows(num_legal, total)
            need = ctypes.c_size_t(0)
            _lib.check(self.lib.hv_leaf_rows_workspace_bytes(total, rows, 0, ctypes.addressof(need)), "workspace")
            ws = self.ws.get(need.value, dev)
            with torch.cuda.device(dev):
                _lib.check(self.lib.hv_fnn_eval_leaves_rows(
                    states.data_ptr(), legal_moves.data_ptr(), num_legal.data_ptr(),
                    None if root_features is None else root_features.data_ptr(), total, rows,
                    self.weights.data_ptr(), *self.dims, priors.data_ptr(), values.data_ptr(), child_q.data_ptr(),
                    None if logits is None else logits.data_ptr(), ws.data_ptr(), ws.numel(),
                    torch.cuda.current_stream(dev).cuda_stream), "fnn_eval_leaves_rows")
        return (priors, values, child_q, logits) if return_logits else (priors, values, child_q)

    def eval_states_fused(self, states: torch.Tensor, legal_moves: torch.Tensor, num_legal: torch.Tensor,
                          total: int, root_features: torch.Tensor | None = None, return_logits: bool = False):
        priors, values, child_q, logits = self._outputs(states, legal_moves, num_legal, total, root_features,
                                                        return_logits)
        if total > 0:
            dev = states.device
            with torch.cuda.device(dev):
                _lib.check(self.lib.hv_fnn_eval_leaves(
                    states.data_ptr(), legal_moves.data_ptr(), num_legal.data_ptr(),
                    None if root_features is None else root_features.data_ptr(), total,
                    self.weights.data_ptr(), *self.dims, priors.data_ptr(), values.data_ptr(),
                    child_q.data_ptr(), None if logits is None else logits.data_ptr(),
                    torch.cuda.current_stream(dev).cuda_stream), "fnn_eval_leaves")
        return (priors, values, child_q, logits) if return_logits else (priors, values, child_q)
