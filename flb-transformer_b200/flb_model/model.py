"""FLB-Transformer built on this package's operators (additive attention, wavefront engine).

Same architecture, math and parameter names as models/FLB_Model.py of FLB-Transformer, so a
state_dict trained with either loads into the other:

  FLB_Attention_Layer (:9-62)  gates: lat' = lat * sigmoid(G_L fdbk + b_L), x' = x *
                               sigmoid(G_X lat' + b_X); the three tokens [x', lat', fdbk] are
                               projected to q, k, v ([B, H, 3, D/H]), combined by
                               fused_additive_attention with v_a [H, 1, D/H], projected by W_o
                               and added back to the unrefined tokens (x, lat, fdbk).
  FLB_Block (:64-96)           priors lat = P_lat LN(prev_lat), fdbk = P_fb LN(prev_fdbk); the
                               attention layer; aux = (lat_prior - h_lat)^2 + (fdbk_prior -
                               h_fdbk)^2 with the outputs detached. Four outputs = four ports.
  FLB_Transformer (:98-179)    embedding -> WavefrontEngine over a (layers, seq_len) grid with
                               dependencies top (port 0), left (port 1), bottom-left (port 2)
                               and 4 ports -> the top row's port-0 states -> linear head;
                               aux_loss = mean(aux grid) * aux_weight; next contexts = the last
                               column of ports 1 and 2.

The dropout modules exist for state compatibility and run where the reference runs them (the
attention layer's own dropout is not applied there either).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from kernels.additive_attention import fused_additive_attention
from wavefront.wavefront_api import WavefrontConfig
from wavefront.wavefront_engine import WavefrontEngine


class FLBAttentionLayer(nn.Module):
    def __init__(self, hidden_dim: int, num_heads: int = 8, dropout: float = 0.1):
        super().__init__()
        if hidden_dim % num_heads:
            raise ValueError(f"hidden_dim {hidden_dim} is not divisible by {num_heads} heads")
        self.hidden_dim, self.num_heads = hidden_dim, num_heads
        self.head_dim = hidden_dim // num_heads
        self.linear_gate_L = nn.Linear(hidden_dim, hidden_dim)
        self.linear_gate_X = nn.Linear(hidden_dim, hidden_dim)
        self.W_q = nn.Linear(hidden_dim, hidden_dim, bias=False)
        self.W_k = nn.Linear(hidden_dim, hidden_dim, bias=False)
        self.v_a = nn.Parameter(torch.randn(num_heads, 1, self.head_dim) * 0.02)
        self.W_v = nn.Linear(hidden_dim, hidden_dim, bias=False)
        self.W_o = nn.Linear(hidden_dim, hidden_dim, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x_token, lat_token, fdbk_token):
        n, _, dim = x_token.shape                      # each token [n, 1, dim]
        lat_ref = lat_token * torch.sigmoid(self.linear_gate_L(fdbk_token))
        x_ref = x_token * torch.sigmoid(self.linear_gate_X(lat_ref))
        seq = torch.cat([x_ref, lat_ref, fdbk_token], dim=1)       # [n, 3, dim]

        def heads(t):                                  # [n, 3, dim] -> [n, H, 3, dim/H]
            return t.view(n, 3, self.num_heads, self.head_dim).transpose(1, 2).contiguous()

        att = fused_additive_attention(heads(self.W_q(seq)), heads(self.W_k(seq)),
                                       heads(self.W_v(seq)), self.v_a)
        o = self.W_o(att.transpose(1, 2).contiguous().view(n, 3, dim))
        return o[:, 0:1] + x_token, o[:, 1:2] + lat_token, o[:, 2:3] + fdbk_token


class FLBBlock(nn.Module):
    """FLB_Block (models/FLB_Model.py:64-96). The reference fixes 8 attention heads (:73);
    num_heads (default 8) makes the head count a constructor argument."""

    def __init__(self, hidden_dim: int, dropout: float = 0.1, num_heads: int = 8):
        super().__init__()
        self.norm_lat = nn.LayerNorm(hidden_dim)
        self.norm_fdbk = nn.LayerNorm(hidden_dim)
        self.proj_lateral = nn.Linear(hidden_dim, hidden_dim, bias=False)
        self.proj_feedback = nn.Linear(hidden_dim, hidden_dim, bias=False)
        self.flb_attention = FLBAttentionLayer(hidden_dim, num_heads=num_heads, dropout=dropout)

    def forward(self, x_input, prev_lat, prev_fdbk):
        b, cells, dim = x_input.shape
        lat_prior = self.proj_lateral(self.norm_lat(prev_lat))
        fdbk_prior = self.proj_feedback(self.norm_fdbk(prev_fdbk))
        h_x, h_lat, h_fdbk = self.flb_attention(x_input.reshape(b * cells, 1, dim),
                                                lat_prior.reshape(b * cells, 1, dim),
                                                fdbk_prior.reshape(b * cells, 1, dim))
        aux = (lat_prior - h_lat.detach()) ** 2 + (fdbk_prior - h_fdbk.detach()) ** 2
        return h_x, h_lat, h_fdbk, aux


FLB_DEPENDENCIES = [((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)]


class FLBTransformer(nn.Module):
    def __init__(self, vocab_size: int, hidden_dim: int = 256, num_layers: int = 6,
                 seq_len: int = 128, batch_size: int = 32, dropout: float = 0.1,
                 aux_weight: float = 0.05, num_heads: int = 8):
        super().__init__()
        self.aux_weight = aux_weight
        self.embedding = nn.Embedding(vocab_size, hidden_dim)
        self.emb_dropout = nn.Dropout(dropout)
        self.out_dropout = nn.Dropout(dropout)
        self.config = WavefrontConfig(grid_shape=(num_layers, seq_len), batch_size=batch_size,
                                      dim=hidden_dim, dependencies=FLB_DEPENDENCIES, num_ports=4)
        self.layers = nn.ModuleList([FLBBlock(hidden_dim, dropout, num_heads)
                                     for _ in range(num_layers)])
        self.engine = WavefrontEngine(self.config, self.layers)
        self.head = nn.Linear(hidden_dim, vocab_size)

    def grids_to_outputs(self, grids):
        """(logits [batch, seq, vocab], aux_loss, (next_lat, next_fdbk)) from the engine's four
        port grids [cells, batch, dim]."""
        L, S = self.config.grid_shape
        B, D = self.config.batch_size, self.config.dim
        y, lat, fdbk, aux = (g.view(L, S, B, D) for g in grids)
        top = self.out_dropout(y[-1].transpose(0, 1))               # [batch, seq, dim]
        logits = self.head(top)
        aux_loss = aux.mean() * self.aux_weight
        return logits, aux_loss, (lat[:, -1], fdbk[:, -1])

    def forward(self, tokens, context=None, engine=None):
        """tokens [batch, seq_len] int64. `engine` optionally replaces self.engine (for example
        a GraphedWavefrontEngine captured from it)."""
        x = self.emb_dropout(self.embedding(tokens))
        states = {}
        if context is not None:
            states = {1: context[0], 2: context[1]}
        grids = (engine or self.engine)(x, states)
        return self.grids_to_outputs(grids)
