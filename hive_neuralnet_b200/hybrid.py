"""Hybrid FNN-transformer evaluator (the reference's ``hive_fnn_transformer``).

``HiveHybridGNN`` / ``HybridGNNConfig`` keep the reference's module tree,
parameter names, presets and creation order
(hive_fnn_transformer/fnn_transformer_net.py:30-371), so checkpoints and
seeded random initialisations load unchanged; the torch forward is the fp32
statement of the network that the sm_100a kernels are checked against.

``HybridEvaluator`` replaces ``HybridMCTSOrchestrator._eval_states``
(hive_fnn_transformer/fnn_transformer_mcts_orchestrator.py:42-169): piece
tokens -> relative transformer trunk (fp16 tcgen05 GEMMs and warp-MMA attention, fp32 accumulation)
-> value head; successor generation + FNN encode + hybrid action scoring +
masked softmax fused in one warp-per-leaf kernel.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from . import _lib
from .fnn import FEAT_DIM, MAX_LEGAL, FNNConfig, HiveFNN

BASE_NODE_FEAT_DIM = 26
ARTICULATION_NODE_FEAT_DIM = 27
GLOBAL_FEAT_DIM = 6
MAX_PIECE_TOKENS = 28
MOVE_FEAT_DIM = 31


@dataclass
class HybridGNNConfig:
    """Same fields, defaults and presets as fnn_transformer_net.py:30-74."""

    fnn_config: FNNConfig | None = None
    use_articulation_token_flag: bool = False
    graph_hidden_dim: int = 64
    graph_layers: int = 4
    graph_mlp_hidden: int = 96
    num_heads: int = 8
    max_piece_tokens: int = MAX_PIECE_TOKENS
    rel_coord_clip: int = 8
    rel_height_clip: int = 2
    value_hidden: int = 128
    move_feat_dim: int = MOVE_FEAT_DIM
    node_feat_dim: int = BASE_NODE_FEAT_DIM
    global_feat_dim: int = GLOBAL_FEAT_DIM

    def __post_init__(self) -> None:
        self.node_feat_dim = ARTICULATION_NODE_FEAT_DIM if self.use_articulation_token_flag else BASE_NODE_FEAT_DIM

    @classmethod
    def small(cls) -> "HybridGNNConfig":
        return cls(fnn_config=FNNConfig.medium(), graph_hidden_dim=64, graph_layers=4, graph_mlp_hidden=96,
                   value_hidden=96)

    @classmethod
    def large(cls) -> "HybridGNNConfig":
        return cls(fnn_config=FNNConfig.large(), use_articulation_token_flag=True, graph_hidden_dim=128,
                   graph_layers=8, graph_mlp_hidden=192, value_hidden=256)


@dataclass
class HybridPieceTensorBatch:
    """Padded piece tokens (hive_fnn_transformer/graph_types.py:17-37)."""

    token_features: torch.Tensor
    token_q: torch.Tensor
    token_r: torch.Tensor
    token_z: torch.Tensor
    token_mask: torch.Tensor
    global_features: torch.Tensor
    num_tokens: torch.Tensor


class RelativeSelfAttention(nn.Module):
    """Multi-head self-attention with learned (dq, dr, dz) offset biases per head."""

    def __init__(self, hidden_dim: int, num_heads: int, rel_coord_clip: int, rel_height_clip: int) -> None:
        super().__init__()
        if hidden_dim % num_heads:
            raise ValueError("hidden_dim must be divisible by num_heads")
        self.hidden_dim, self.num_heads = hidden_dim, num_heads
        self.head_dim = hidden_dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.rel_coord_clip, self.rel_height_clip = rel_coord_clip, rel_height_clip
        self.qkv = nn.Linear(hidden_dim, hidden_dim * 3)
        self.out_proj = nn.Linear(hidden_dim, hidden_dim)
        self.dq_bias = nn.Embedding(rel_coord_clip * 2 + 1, num_heads)
        self.dr_bias = nn.Embedding(rel_coord_clip * 2 + 1, num_heads)
        self.dz_bias = nn.Embedding(rel_height_clip * 2 + 1, num_heads)

    def forward(self, x, token_q, token_r, token_z, token_mask):
        b, n, _ = x.shape
        q, k, v = self.qkv(x).view(b, n, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        scores = (q @ k.transpose(-2, -1)) * self.scale

        def rel(t, clip):  # offset of key j from query i, clipped and shifted to an index
            return (t.unsqueeze(1) - t.unsqueeze(2)).clamp(-clip, clip) + clip

        bias = (self.dq_bias(rel(token_q, self.rel_coord_clip)) + self.dr_bias(rel(token_r, self.rel_coord_clip))
                + self.dz_bias(rel(token_z, self.rel_height_clip)))
        scores = scores + bias.permute(0, 3, 1, 2).to(scores.dtype)
        scores = scores.masked_fill(~token_mask[:, None, None, :], torch.finfo(scores.dtype).min)
        out = torch.softmax(scores, dim=-1) @ v
        return self.out_proj(out.transpose(1, 2).reshape(b, n, self.hidden_dim))


class RelativeTransformerBlock(nn.Module):
    """Pre-LayerNorm block: attention and a GELU MLP, each with a residual."""

    def __init__(self, hidden_dim, num_heads, ffn_hidden, rel_coord_clip, rel_height_clip) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(hidden_dim)
        self.attn = RelativeSelfAttention(hidden_dim, num_heads, rel_coord_clip, rel_height_clip)
        self.norm2 = nn.LayerNorm(hidden_dim)
        self.ffn = nn.Sequential(nn.Linear(hidden_dim, ffn_hidden), nn.GELU(), nn.Linear(ffn_hidden, hidden_dim))

    def forward(self, x, token_q, token_r, token_z, token_mask):
        x = x + self.attn(self.norm1(x), token_q, token_r, token_z, token_mask)
        return x + self.ffn(self.norm2(x))


class HybridRelativeTransformerTrunk(nn.Module):
    """CLS token + piece tokens through the blocks; returns the normalised CLS row."""

    def __init__(self, config: HybridGNNConfig) -> None:
        super().__init__()
        h = config.graph_hidden_dim
        self.max_piece_tokens = config.max_piece_tokens
        self.token_proj = nn.Linear(config.node_feat_dim, h)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, h))
        self.layers = nn.ModuleList([
            RelativeTransformerBlock(h, config.num_heads, config.graph_mlp_hidden, config.rel_coord_clip,
                                     config.rel_height_clip)
            for _ in range(config.graph_layers)])
        self.norm = nn.LayerNorm(h)
        self.out_dim = h

    def forward(self, pb: HybridPieceTensorBatch) -> torch.Tensor:
        mask_f = pb.token_mask.unsqueeze(-1).to(torch.float32)
        tokens = self.token_proj(pb.token_features) * mask_f.to(self.token_proj.weight.dtype)
        b = tokens.shape[0]
        x = torch.cat([self.cls_token.expand(b, -1, -1), tokens], dim=1)
        z = torch.zeros((b, 1), dtype=pb.token_q.dtype, device=tokens.device)
        tq, tr, tz = (torch.cat([z, t], dim=1) for t in (pb.token_q, pb.token_r, pb.token_z))
        tm = torch.cat([torch.ones((b, 1), dtype=torch.bool, device=tokens.device), pb.token_mask], dim=1)
        for layer in self.layers:
            x = layer(x, tq, tr, tz, tm)
            x = torch.cat([x[:, :1], x[:, 1:] * mask_f.to(x.dtype)], dim=1)
        return self.norm(x)[:, 0]


class HiveHybridGNN(nn.Module):
    """FNN successor features plus transformer-aware policy / value heads
    (fnn_transformer_net.py:212-371), same creation order as the reference."""

    model_version = "fnn_transformer"

    def __init__(self, config: HybridGNNConfig | None = None) -> None:
        super().__init__()
        self.config = config or HybridGNNConfig()
        fc = self.config.fnn_config or FNNConfig.large()
        fc.feat_dim = FEAT_DIM
        self.config.move_feat_dim = MOVE_FEAT_DIM
        self.fnn = HiveFNN(fc)
        self.graph_trunk = HybridRelativeTransformerTrunk(self.config)
        e, h = fc.embed_dim, self.graph_trunk.out_dim
        self.policy_graph_proj = nn.Linear(h, e)
        self.policy_move_proj = nn.Linear(self.config.move_feat_dim, e)
        self.policy_fc1 = nn.Linear(e * 4, fc.action_hidden)
        self.policy_fc2 = nn.Linear(fc.action_hidden, 1)
        self.value_head = nn.Sequential(nn.Linear(e + h + self.config.global_feat_dim, self.config.value_hidden),
                                        nn.ReLU(), nn.Linear(self.config.value_hidden, 1))

    @staticmethod
    def _resize_loaded_tensor(old: torch.Tensor, new_template: torch.Tensor, *, noise_scale: float = 1e-3):
        """Overlap of a checkpoint tensor of another shape copied into the live
        one; a resized floating tensor starts from N(0, noise_scale)
        (fnn_transformer_net.py:244-270)."""
        new = new_template.detach().clone()
        if old.dtype.is_floating_point and new.dtype.is_floating_point and old.shape != new.shape:
            new.normal_(mean=0.0, std=noise_scale)
        overlap = tuple(slice(0, min(a, b)) for a, b in zip(old.shape, new.shape))
        if overlap:
            new[overlap] = old[overlap].to(dtype=new.dtype, device=new.device)
        else:
            new.copy_(old.to(dtype=new.dtype, device=new.device))
        return new

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        """fnn_transformer_net.py:272-286: unknown keys dropped, missing keys
        keep the live initialisation, resized tensors keep their overlap."""
        state = dict(state_dict)
        cur = self.state_dict()
        for key in list(state.keys()):
            if key not in cur:
                state.pop(key)
        for key, t in cur.items():
            if key not in state:
                state[key] = t
            elif state[key].shape != t.shape:
                state[key] = self._resize_loaded_tensor(state[key], t)
        return super().load_state_dict(state, strict=strict, assign=assign)

    def load_fnn_policy_weights(self, fnn: HiveFNN) -> None:
        """fnn_transformer_net.py:359-365: the shared FNN encoder from a trained HiveFNN."""
        self.fnn.load_state_dict(fnn.state_dict())

    def score_hybrid_actions(self, root_emb, root_graph_emb, successor_emb, move_features):
        combined = torch.cat([root_emb, self.policy_graph_proj(root_graph_emb), successor_emb,
                              self.policy_move_proj(move_features)], dim=1)
        return self.policy_fc2(torch.sigmoid(self.policy_fc1(combined))).squeeze(-1)

    def policy_forward(self, root_features, successor_features, action_to_root, piece_batch, move_features):
        """fnn_transformer_net.py:329-347"""
        root_emb = self.fnn.encode(root_features)
        if action_to_root.shape[0] == 0:
            return root_features.new_zeros((0,))
        g = self.graph_trunk(piece_batch)
        return self.score_hybrid_actions(root_emb[action_to_root], g[action_to_root],
                                         self.fnn.encode(successor_features), move_features)

    def value_forward(self, root_features, piece_batch):
        root_emb = self.fnn.encode(root_features)
        g = self.graph_trunk(piece_batch)
        return torch.tanh(self.value_head(torch.cat([root_emb, g, piece_batch.global_features], dim=1)))

    def forward(self, root_features, successor_features, action_to_root, num_actions, piece_batch, move_features):
        root_emb = self.fnn.encode(root_features)
        g = self.graph_trunk(piece_batch)
        if action_to_root.shape[0] == 0:
            logits = root_features.new_zeros((0,))
        else:
            logits = self.score_hybrid_actions(root_emb[action_to_root], g[action_to_root],
                                               self.fnn.encode(successor_features), move_features)
        values = torch.tanh(self.value_head(torch.cat([root_emb, g, piece_batch.global_features], dim=1)))
        return logits, values

    def count_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad)


HiveFNNTransformer = HiveHybridGNN


# ---------------------------------------------------------------------------
# device weight images for the sm_100a kernels
# ---------------------------------------------------------------------------
TRUNK_HIDDEN, TRUNK_HEADS, TRUNK_FFN, TRUNK_LAYERS, TRUNK_KIN = 64, 8, 96, 4, 32


def _slabs(w: torch.Tensor, k_pad: int | None = None) -> torch.Tensor:
    """[N, K] row-major -> the kernels' K-major slab layout [K/8][N][8] (zero-padded K)."""
    n, k = w.shape
    kp = k_pad or k
    if kp != k:
        w = torch.cat([w, w.new_zeros((n, kp - k))], dim=1)
    return w.reshape(n, kp // 8, 8).permute(1, 0, 2).contiguous().reshape(-1)


def check_trunk_config(cfg: HybridGNNConfig) -> None:
    if (cfg.graph_hidden_dim, cfg.num_heads, cfg.graph_mlp_hidden, cfg.graph_layers) != (
            TRUNK_HIDDEN, TRUNK_HEADS, TRUNK_FFN, TRUNK_LAYERS):
        raise NotImplementedError("the sm_100a trunk kernel implements the default and `small` presets "
                                  "(hidden 64, 8 heads, MLP 96, 4 blocks)")
    if cfg.rel_coord_clip != 8 or cfg.rel_height_clip != 2:
        raise NotImplementedError("the sm_100a trunk kernel implements rel_coord_clip 8, rel_height_clip 2")


def pack_trunk(trunk: HybridRelativeTransformerTrunk, device) -> tuple[torch.Tensor, torch.Tensor]:
    """(fp16 weight image as int16 storage, fp32 parameters) in the layout of hv_trunk.cuh."""
    with torch.no_grad():
        img = [_slabs(trunk.token_proj.weight.float(), TRUNK_KIN)]
        par = [trunk.token_proj.bias, trunk.cls_token.reshape(-1), trunk.norm.weight, trunk.norm.bias]
        for blk in trunk.layers:
            a = blk.attn
            img += [_slabs(a.qkv.weight.float()), _slabs(a.out_proj.weight.float()),
                    _slabs(blk.ffn[0].weight.float()), _slabs(blk.ffn[2].weight.float())]
            par += [blk.norm1.weight, blk.norm1.bias, a.qkv.bias, a.out_proj.bias, blk.norm2.weight,
                    blk.norm2.bias, blk.ffn[0].bias, blk.ffn[2].bias, a.dq_bias.weight.reshape(-1),
                    a.dr_bias.weight.reshape(-1), a.dz_bias.weight.reshape(-1)]
        image = torch.cat(img).to(torch.float16).view(torch.int16).to(device).contiguous()
        params = torch.cat([p.detach().float().reshape(-1) for p in par]).to(device).contiguous()
    return image, params


class HybridTrunk:
    """The relative transformer trunk on the tensor cores: piece tokens -> graph summary [B, 64]."""

    def __init__(self, net: HiveHybridGNN, device="cuda"):
        check_trunk_config(net.config)
        self.net, self.device = net, torch.device(device)
        self.lib = _lib.load()
        self.refresh()

    def refresh(self) -> None:
        import ctypes
        self.image, self.params = pack_trunk(self.net.graph_trunk, self.device)
        ie, pf = ctypes.c_int(0), ctypes.c_int(0)
        _lib.check(self.lib.hv_hybrid_trunk_sizes(ctypes.addressof(ie), ctypes.addressof(pf)), "trunk sizes")
        if (ie.value, pf.value) != (self.image.numel(), self.params.numel()):
            raise ValueError(f"packed ({self.image.numel()}, {self.params.numel()}), kernel expects "
                             f"({ie.value}, {pf.value})")

    def __call__(self, pb: HybridPieceTensorBatch, packed: bool = False) -> torch.Tensor:
        """packed: positions with at most 15 token slots in use share the
        kernel's 32-row slots in pairs (hv_hybrid_trunk_packed); the same output."""
        import ctypes
        tf = pb.token_features
        B = tf.shape[0]
        out = torch.empty((B, TRUNK_HIDDEN), dtype=torch.float32, device=tf.device)
        if B == 0:
            return out
        if tf.shape[1:] != (MAX_PIECE_TOKENS, ARTICULATION_NODE_FEAT_DIM) or tf.dtype != torch.float32:
            raise ValueError("token_features: expected float32 [B, 28, 27] (the encoder's full rows)")
        tq, tr, tz = (t.to(torch.int32).contiguous() for t in (pb.token_q, pb.token_r, pb.token_z))
        tm = pb.token_mask.to(torch.uint8).contiguous()
        tf = tf.contiguous()
        stream = torch.cuda.current_stream(tf.device).cuda_stream
        args = (tf.data_ptr(), tq.data_ptr(), tr.data_ptr(), tz.data_ptr(), tm.data_ptr(), B,
                self.net.config.node_feat_dim, self.image.data_ptr(), self.params.data_ptr(), out.data_ptr())
        with torch.cuda.device(tf.device):
            if packed:
                need = ctypes.c_size_t(0)
                _lib.check(self.lib.hv_hybrid_trunk_packed_workspace_bytes(B, ctypes.addressof(need)), "trunk ws")
                ws = getattr(self, "_slot_ws", None)
                if ws is None or ws.device != tf.device or ws.numel() < need.value:
                    ws = self._slot_ws = torch.empty((int(need.value),), dtype=torch.uint8, device=tf.device)
                _lib.check(self.lib.hv_hybrid_trunk_packed(*args, ws.data_ptr(), ws.numel(), stream),
                           "hybrid_trunk_packed")
            else:
                _lib.check(self.lib.hv_hybrid_trunk(*args, stream), "hybrid_trunk")
        return out


def pack_heads(net: HiveHybridGNN, device) -> torch.Tensor:
    """fp32 policy / value head weights in the layout of hv_hybrid.cuh (hyb_offsets); the
    move-projection block of policy_fc1 is folded into a [A, 31] matrix on the host (float64)."""
    e = net.fnn.config.embed_dim
    with torch.no_grad():
        w1 = net.policy_fc1.weight.double()
        wm = w1[:, 3 * e:4 * e]
        fold = wm @ net.policy_move_proj.weight.double()          # [A, 31]
        b1 = net.policy_fc1.bias.double() + wm @ net.policy_move_proj.bias.double()
        parts = [net.policy_graph_proj.weight.t(), net.policy_graph_proj.bias, w1[:, :3 * e].t(), fold.t(), b1,
                 net.policy_fc2.weight.reshape(-1), net.policy_fc2.bias, net.value_head[0].weight.t(),
                 net.value_head[0].bias, net.value_head[2].weight.reshape(-1), net.value_head[2].bias]
        flat = torch.cat([p.detach().double().contiguous().reshape(-1) for p in parts]).float()
        # fp16 slab image for the tensor-core row kernel (hv_mlp_tc.cuh), 16-byte aligned
        fnn = net.fnn
        img = torch.cat([_slabs_b(fnn.fc1.weight.float(), 128), _slabs_b(fnn.fc2.weight.float(), 64),
                         _slabs_b(torch.cat([w1[:, 2 * e:3 * e].float(), fold.float()], dim=1), 96, split=e)])
        # the per-leaf root network (k_leaf_root_tc): encode, value layer in
        # three K blocks, graph projection, root half of the action layer
        vh1 = net.value_head[0].weight.float()  # [V, E + 64 + 6]
        g = net.graph_trunk.out_dim
        root = torch.cat([_slabs_b(fnn.fc1.weight.float(), 128), _slabs_b(fnn.fc2.weight.float(), 64),
                          _slabs_b(vh1[:, :e], 64, rows=128), _slabs_b(vh1[:, e:e + g], 64, rows=128),
                          _slabs_b(vh1[:, e + g:], 16, rows=128), _slabs_b(net.policy_graph_proj.weight.float(), 64),
                          _slabs_b(w1[:, :e].float(), 64), _slabs_b(w1[:, e:2 * e].float(), 64)])
        pad = (-flat.numel()) % 4
        flat = torch.cat([flat, flat.new_zeros(pad), img.view(torch.float32), root.view(torch.float32)])
    return flat.to(device).contiguous()


def _slabs_b(w: torch.Tensor, k_pad: int, split: int | None = None, rows: int = 64) -> torch.Tensor:
    """[N <= rows, K] fp32 weight -> fp16 B operand [rows x k_pad] in the K-major
    slab layout (element (n, k) at ((k / 8) * rows + n) * 8 + k % 8), zero padded.
    With ``split``, columns [split:] start at K = 64 (the [A1s | C] layout)."""
    out = torch.zeros(rows, k_pad, dtype=torch.float32)
    if split is None:
        out[:w.shape[0], :w.shape[1]] = w
    else:
        out[:w.shape[0], :split] = w[:, :split]
        out[:w.shape[0], 64:64 + w.shape[1] - split] = w[:, split:]
    return out.half().reshape(rows, k_pad // 8, 8).permute(1, 0, 2).contiguous().reshape(-1)



def _check_leaf_inputs(states, legal_moves, num_legal, root_features) -> None:
    """The library reads these buffers as packed arrays: reject any other
    dtype, layout or device before a pointer is passed."""
    for t, name, dt in ((states, "states", torch.uint8), (legal_moves, "legal_moves", torch.uint8),
                        (num_legal, "num_legal", torch.int32)):
        if t.dtype != dt or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name}: expected contiguous CUDA {dt}")
    if root_features is not None and (root_features.dtype != torch.float32 or not root_features.is_cuda
                                      or not root_features.is_contiguous()):
        raise ValueError("root_features: expected contiguous CUDA float32")

class HybridEvaluator:
    """Leaf evaluation of the hybrid network with the signature and outputs of the
    reference's ``HybridMCTSOrchestrator._eval_states``: (priors [T,256], values [T],
    child_q [T,256] = 0).  One C-ABI call (hv_hybrid_evaluate): piece tokens, trunk
    (tcgen05), fused heads; the tokens and summaries live in a cached workspace."""

    def __init__(self, net: HiveHybridGNN, device="cuda"):
        from .fnn import pack_weights
        from .hive_gpu import load_extension
        self.net, self.device = net, torch.device(device)
        self.lib = _lib.load()
        self.ext = load_extension()
        self.trunk = HybridTrunk(net, self.device)
        fc = net.fnn.config
        self.fdims = (fc.hidden_dim, fc.embed_dim, fc.action_hidden)
        self.vh = net.config.value_hidden
        self._pack_weights = pack_weights
        self.refresh()

    def refresh(self) -> None:
        """Re-pack every weight image (call after the network was trained)."""
        self.trunk.refresh()
        self.fnn_weights = self._pack_weights(self.net.fnn, self.device)
        self.head_weights = pack_heads(self.net, self.device)
        want = self.lib.hv_hybrid_head_weights_size(self.fdims[1], self.fdims[2], self.vh)
        if want != self.head_weights.numel():
            raise ValueError(f"packed {self.head_weights.numel()} head floats, kernel expects {want}")

    def _workspace(self, total: int, dev) -> torch.Tensor:
        import ctypes
        need = ctypes.c_size_t(0)
        _lib.check(self.lib.hv_hybrid_workspace_bytes(total, ctypes.addressof(need)), "hybrid workspace size")
        ws = getattr(self, "_ws", None)
        if ws is None or ws.device != dev or ws.numel() < need.value:
            self._ws = ws = torch.empty((max(need.value, 1),), dtype=torch.uint8, device=dev)
        return ws

    def eval_states(self, states, legal_moves, num_legal, total, root_features=None, return_logits=False):
        """The row pipeline (``hv_hybrid_evaluate_rows``): tokens, trunk, successor
        features and move features of all leaves, tiled fp32 heads over the rows."""
        import ctypes

        from .fnn import _rows
        dev = states.device
        priors = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        values = torch.empty((total,), dtype=torch.float32, device=dev)
        child_q = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        logits = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev) if return_logits else None
        if total == 0:
            return (priors, values, child_q, logits) if return_logits else (priors, values, child_q)
        for t, name, dt in ((states, "states", torch.uint8), (legal_moves, "legal_moves", torch.uint8),
                            (num_legal, "num_legal", torch.int32)):
            if t.dtype != dt or not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{name}: expected contiguous CUDA {dt}")
        if root_features is not None and (root_features.dtype != torch.float32 or not root_features.is_contiguous()):
            raise ValueError("root_features: expected contiguous float32")
        rows = _rows(num_legal, total)
        need = ctypes.c_size_t(0)
        _lib.check(self.lib.hv_leaf_rows_workspace_bytes(total, rows, 1, ctypes.addressof(need)), "workspace")
        if getattr(self, "_rows_ws", None) is None or self._rows_ws.device != dev or self._rows_ws.numel() < need.value:
            self._rows_ws = torch.empty((max(int(need.value * 1.25), 256),), dtype=torch.uint8, device=dev)
        ws = self._rows_ws
        with torch.cuda.device(dev):
            _lib.check(self.lib.hv_hybrid_evaluate_rows(
                states.data_ptr(), legal_moves.data_ptr(), num_legal.data_ptr(),
                None if root_features is None else root_features.data_ptr(), total, rows,
                self.net.config.node_feat_dim, self.trunk.image.data_ptr(), self.trunk.params.data_ptr(),
                self.fnn_weights.data_ptr(), *self.fdims, self.head_weights.data_ptr(), self.vh, priors.data_ptr(),
                values.data_ptr(), child_q.data_ptr(), None if logits is None else logits.data_ptr(), ws.data_ptr(),
                ws.numel(), torch.cuda.current_stream(dev).cuda_stream), "hybrid_evaluate_rows")
        return (priors, values, child_q, logits) if return_logits else (priors, values, child_q)

    def eval_states_fused(self, states, legal_moves, num_legal, total, root_features=None, return_logits=False):
        """The single-call warp-per-leaf evaluation (``hv_hybrid_evaluate``)."""
        dev = states.device
        priors = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        values = torch.empty((total,), dtype=torch.float32, device=dev)
        child_q = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        logits = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev) if return_logits else None
        if total == 0:
            return (priors, values, child_q, logits) if return_logits else (priors, values, child_q)
        _check_leaf_inputs(states, legal_moves, num_legal, root_features)
        ws = self._workspace(total, dev)
        with torch.cuda.device(dev):
            _lib.check(self.lib.hv_hybrid_evaluate(
                states.data_ptr(), legal_moves.data_ptr(), num_legal.data_ptr(),
                None if root_features is None else root_features.data_ptr(), total, self.net.config.node_feat_dim,
                self.trunk.image.data_ptr(), self.trunk.params.data_ptr(), self.fnn_weights.data_ptr(),
                *self.fdims, self.head_weights.data_ptr(), self.vh, priors.data_ptr(), values.data_ptr(),
                child_q.data_ptr(), None if logits is None else logits.data_ptr(), ws.data_ptr(), ws.numel(),
                torch.cuda.current_stream(dev).cuda_stream), "hybrid_evaluate")
        if return_logits:
            return priors, values, child_q, logits
        return priors, values, child_q

    def eval_states_noalloc(self, states, legal_moves, num_legal, total, root_features=None):
        """Same outputs as :meth:`eval_states` through ``hv_hybrid_evaluate_noalloc``: the
        library uses its fixed device scratch (at most 9137 positions per call) instead
        of this evaluator's workspace.  Calls on one device must not overlap."""
        dev = states.device
        priors = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        values = torch.empty((total,), dtype=torch.float32, device=dev)
        child_q = torch.empty((total, MAX_LEGAL), dtype=torch.float32, device=dev)
        if total == 0:
            return priors, values, child_q
        _check_leaf_inputs(states, legal_moves, num_legal, root_features)
        with torch.cuda.device(dev):
            _lib.check(self.lib.hv_hybrid_evaluate_noalloc(
                states.data_ptr(), legal_moves.data_ptr(), num_legal.data_ptr(),
                None if root_features is None else root_features.data_ptr(), total, self.net.config.node_feat_dim,
                self.trunk.image.data_ptr(), self.trunk.params.data_ptr(), self.fnn_weights.data_ptr(),
                *self.fdims, self.head_weights.data_ptr(), self.vh, priors.data_ptr(), values.data_ptr(),
                child_q.data_ptr(), None, torch.cuda.current_stream(dev).cuda_stream), "hybrid_evaluate_noalloc")
        return priors, values, child_q
