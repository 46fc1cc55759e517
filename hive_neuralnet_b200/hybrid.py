"""Hybrid FNN-transformer evaluator (the reference's ``hive_fnn_transformer``).

``HiveHybridGNN`` / ``HybridGNNConfig`` keep the reference's module tree,
parameter names, presets and creation order
(hive_fnn_transformer/fnn_transformer_net.py:30-371), so checkpoints and
seeded random initialisations load unchanged; the torch forward is the fp32
statement of the network that the sm_100a kernels are checked against.

``HybridEvaluator`` replaces ``HybridMCTSOrchestrator._eval_states``
(hive_fnn_transformer/fnn_transformer_mcts_orchestrator.py:42-169): piece
tokens -> relative transformer trunk (bf16 tcgen05 GEMMs, fp32 attention)
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

    def score_hybrid_actions(self, root_emb, root_graph_emb, successor_emb, move_features):
        combined = torch.cat([root_emb, self.policy_graph_proj(root_graph_emb), successor_emb,
                              self.policy_move_proj(move_features)], dim=1)
        return self.policy_fc2(torch.sigmoid(self.policy_fc1(combined))).squeeze(-1)

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
