"""Attention layers — reference ``neural/transformer_layers.py:22-309``.

Multi-head attention with optional QK layer-norm (ViT-22B style), a pre-norm
block with optional cross-attention, encoder / decoder stacks and a
sinusoidal positional encoding.  On the GPU, unmasked attention runs on this
framework's column-attention kernel (``csrc/attention.cu``: one warp per
(column, head), online softmax in fp32, forward and backward, no score
matrix in memory); masked or biased attention and CPU tensors use
``torch.nn.functional.scaled_dot_product_attention``.  Self-attention
projects Q, K and V with one GEMM over the concatenated weights.  Parameter names (``q_proj`` / ``k_proj`` / ``v_proj`` /
``out_proj``, ``ln1`` / ``ln_cross`` / ``ln2`` / ``ffn``) match the reference so
its state dicts load unchanged.

In this model family attention is column-local (sequence = vertical levels
of one column, batch = columns), so no sequence sharding is involved.
"""

from __future__ import annotations

import math
from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class ColumnAttentionFn(torch.autograd.Function):
    """softmax(q kᵀ · scale) v over ``(G, S, D)`` tensors with the kernel pair of ``csrc/attention.cu``."""

    @staticmethod
    def forward(ctx, q, k, v, scale: float):
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("column attention")
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o, lse = ops.column_attention_fwd(q, k, v, float(scale))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale = float(scale)
        return o

    @staticmethod
    def backward(ctx, g):
        from tornado_gcm_b200.ops import _ext

        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _ext.require("column attention backward").column_attention_bwd(
            q, k, v, o, g.contiguous().to(o.dtype), lse, ctx.scale)
        return dq, dk, dv, None


def column_attention_supported(q: torch.Tensor, k: torch.Tensor) -> bool:
    """Shapes and dtypes the column-attention kernel takes."""
    from tornado_gcm_b200.ops import _ext

    D = q.shape[-1]
    return (q.is_cuda and _ext.available() and q.dtype in (torch.float32, torch.bfloat16) and k.dtype == q.dtype
            and D in (8, 16, 32, 64) and q.shape[-2] <= 128 and k.shape[-2] <= 128 and k.shape[-2] * D <= 7264)


def column_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """``(…, S, D)`` attention (no mask) on the column-attention kernel."""
    lead = q.shape[:-2]
    D = q.shape[-1]
    out = ColumnAttentionFn.apply(q.reshape(-1, q.shape[-2], D), k.reshape(-1, k.shape[-2], D),
                                  v.reshape(-1, v.shape[-2], D), 1.0 / math.sqrt(D))
    return out.reshape(lead + out.shape[-2:])


class MultiHeadAttention(nn.Module):
    def __init__(self, num_heads: int, in_features: int, qkv_features: Optional[int] = None,
                 out_features: Optional[int] = None, in_kv_features: Optional[int] = None, *,
                 normalize_qk: bool = False, use_bias: bool = True):
        super().__init__()
        self.num_heads = num_heads
        self.in_features = in_features
        self.qkv_features = qkv_features or in_features
        self.out_features = out_features or in_features
        self.in_kv_features = in_kv_features or in_features
        if self.qkv_features % num_heads:
            raise ValueError(f"qkv_features ({self.qkv_features}) must be divisible by num_heads ({num_heads})")
        self.head_dim = self.qkv_features // num_heads
        self.q_proj = nn.Linear(in_features, self.qkv_features, bias=use_bias)
        self.k_proj = nn.Linear(self.in_kv_features, self.qkv_features, bias=use_bias)
        self.v_proj = nn.Linear(self.in_kv_features, self.qkv_features, bias=use_bias)
        self.out_proj = nn.Linear(self.qkv_features, self.out_features, bias=use_bias)
        self.normalize_qk = normalize_qk
        if normalize_qk:
            self.q_ln = nn.LayerNorm(self.head_dim)
            self.k_ln = nn.LayerNorm(self.head_dim)
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.out_proj):
            nn.init.xavier_normal_(lin.weight)
            if lin.bias is not None:
                nn.init.zeros_(lin.bias)

    def _heads(self, t: torch.Tensor) -> torch.Tensor:
        # (..., seq, H*D) → (..., H, seq, D)
        return t.unflatten(-1, (self.num_heads, self.head_dim)).transpose(-3, -2)

    def _project(self, query, key, value):
        if key is None and value is None and self.in_kv_features == self.in_features:
            w = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], 0)
            b = None if self.q_proj.bias is None else torch.cat(
                [self.q_proj.bias, self.k_proj.bias, self.v_proj.bias], 0)
            return F.linear(query, w, b).chunk(3, dim=-1)
        key = query if key is None else key
        value = key if value is None else value
        return self.q_proj(query), self.k_proj(key), self.v_proj(value)

    def forward(self, query: torch.Tensor, key: Optional[torch.Tensor] = None, value: Optional[torch.Tensor] = None,
                attention_bias: Optional[torch.Tensor] = None, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``query (…, Sq, Din)``, ``key/value (…, Skv, Dkv)``; ``mask`` True = attend,
        broadcast over heads ``(…, Sq, Skv)``; ``attention_bias`` ``(…, H, Sq, Skv)``."""
        q, k, v = (self._heads(t) for t in self._project(query, key, value))
        if self.normalize_qk:
            q, k = self.q_ln(q), self.k_ln(k)
        if attention_bias is None and mask is None and column_attention_supported(q, k):
            out = column_attention(q, k, v.to(q.dtype))
            return self.out_proj(out.transpose(-3, -2).flatten(-2))
        attn_mask = None
        if attention_bias is not None:
            attn_mask = attention_bias.to(q.dtype)
        if mask is not None:
            m = mask.unsqueeze(-3)
            if attn_mask is None:
                attn_mask = m
            else:
                attn_mask = attn_mask.masked_fill(~m, float("-inf"))
        out = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask)
        return self.out_proj(out.transpose(-3, -2).flatten(-2))


class TransformerBlock(nn.Module):
    """Pre-norm block: self-attention, optional cross-attention, feed-forward."""

    def __init__(self, d_model: int, num_heads: int, d_ff: Optional[int] = None, activation: Callable = F.gelu,
                 normalize_qk: bool = False, cross_attention: bool = False, d_cross: Optional[int] = None,
                 use_bias: bool = True, dropout: float = 0.0):
        super().__init__()
        d_ff = d_ff or 4 * d_model
        self.ln1 = nn.LayerNorm(d_model)
        self.self_attn = MultiHeadAttention(num_heads, d_model, normalize_qk=normalize_qk, use_bias=use_bias)
        self.cross_attention = cross_attention
        if cross_attention:
            self.ln_cross = nn.LayerNorm(d_model)
            self.cross_attn = MultiHeadAttention(num_heads, d_model, in_kv_features=d_cross or d_model,
                                                 normalize_qk=normalize_qk, use_bias=use_bias)
        self.ln2 = nn.LayerNorm(d_model)
        act = nn.GELU() if activation is F.gelu else (nn.ReLU() if activation is F.relu else _Act(activation))
        self.ffn = nn.Sequential(nn.Linear(d_model, d_ff, bias=use_bias), act, nn.Dropout(dropout),
                                 nn.Linear(d_ff, d_model, bias=use_bias), nn.Dropout(dropout))
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor, context: Optional[torch.Tensor] = None, mask: Optional[torch.Tensor] = None,
                cross_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        x = x + self.dropout(self.self_attn(self.ln1(x), mask=mask))
        if self.cross_attention and context is not None:
            x = x + self.dropout(self.cross_attn(self.ln_cross(x), context, context, mask=cross_mask))
        return x + self.ffn(self.ln2(x))


class _Act(nn.Module):
    def __init__(self, fn: Callable):
        super().__init__()
        self.fn = fn

    def forward(self, x):
        return self.fn(x)


class TransformerEncoder(nn.Module):
    def __init__(self, d_model: int, num_heads: int, num_layers: int, d_ff: Optional[int] = None,
                 activation: Callable = F.gelu, normalize_qk: bool = False, dropout: float = 0.0):
        super().__init__()
        self.layers = nn.ModuleList([TransformerBlock(d_model, num_heads, d_ff, activation, normalize_qk,
                                                      dropout=dropout) for _ in range(num_layers)])
        self.final_ln = nn.LayerNorm(d_model)

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x, mask=mask)
        return self.final_ln(x)


class TransformerDecoder(nn.Module):
    def __init__(self, d_model: int, num_heads: int, num_layers: int, d_cross: Optional[int] = None,
                 d_ff: Optional[int] = None, activation: Callable = F.gelu, normalize_qk: bool = False,
                 dropout: float = 0.0):
        super().__init__()
        self.layers = nn.ModuleList([TransformerBlock(d_model, num_heads, d_ff, activation, normalize_qk,
                                                      cross_attention=True, d_cross=d_cross, dropout=dropout)
                                     for _ in range(num_layers)])
        self.final_ln = nn.LayerNorm(d_model)

    def forward(self, x: torch.Tensor, context: torch.Tensor, mask: Optional[torch.Tensor] = None,
                cross_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x, context=context, mask=mask, cross_mask=cross_mask)
        return self.final_ln(x)


class SinusoidalPositionalEncoding(nn.Module):
    """Adds ``sin/cos(pos · 10000^(-2i/d))`` to ``(…, seq, d)`` inputs."""

    def __init__(self, d_model: int, max_len: int = 10000):
        super().__init__()
        pos = torch.arange(max_len, dtype=torch.float64)[:, None]
        freq = torch.exp(torch.arange(0, d_model, 2, dtype=torch.float64) * (-math.log(10000.0) / d_model))
        pe = torch.zeros(max_len, d_model, dtype=torch.float64)
        pe[:, 0::2] = torch.sin(pos * freq)
        pe[:, 1::2] = torch.cos(pos * freq[: d_model // 2])
        self.register_buffer("pe", pe.float(), persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x + self.pe[: x.shape[-2]].to(x.dtype)


class ColumnTransformer(nn.Module):
    """Levels-as-sequence transformer for :class:`~tornado_gcm_b200.neural.towers.ColumnTransformerTower`.

    ``(columns, levels, features)`` → ``(columns, levels, out_features)``.
    """

    def __init__(self, in_features: int, out_features: int, d_model: int = 64, num_heads: int = 4,
                 num_layers: int = 2, normalize_qk: bool = True, max_levels: int = 256):
        super().__init__()
        self.embed = nn.Linear(in_features, d_model)
        self.pos = SinusoidalPositionalEncoding(d_model, max_levels)
        self.encoder = TransformerEncoder(d_model, num_heads, num_layers, normalize_qk=normalize_qk)
        self.head = nn.Linear(d_model, out_features)

    def forward(self, x: torch.Tensor, latents: Optional[torch.Tensor] = None,
                positional_encoding: Optional[torch.Tensor] = None) -> torch.Tensor:
        h = self.embed(x)
        h = h + positional_encoding.to(h.dtype) if positional_encoding is not None else self.pos(h)
        if latents is not None:
            h = h + latents.to(h.dtype)
        return self.head(self.encoder(h))
