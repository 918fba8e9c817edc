"""Native Llama building blocks whose ``state_dict`` matches HF Llama names.

The reference builds its modules from ``transformers``' ``LlamaDecoderLayer``
(``src/opendipaco/modules.py:18-98``). Here every layer is our own module so its
parameters can live in the flat, device-resident buffers the B200 executor uses,
while keeping the exact parameter names the checkpoint format needs::

    layers.{i}.self_attn.{q,k,v,o}_proj.weight
    layers.{i}.mlp.{gate,up,down}_proj.weight
    layers.{i}.{input,post_attention}_layernorm.weight
    embed_tokens.weight ; norm.weight ; lm_head.weight

Parameters are created in the same order as HF creates them (q, k, v, o, gate,
up, down, input norm, post norm) with PyTorch's default initialisers, so for a
given seed the bank is bit-identical to the reference's (no ``post_init`` runs
there either).

Forward math: on CPU tensors the modules compute with plain PyTorch ops (the
numerical oracle). On CUDA tensors they route to the sm_100a kernels in
:mod:`opendipaco_b200.ops` (GEMM, attention, RMSNorm, RoPE, fused cross-entropy)
and raise if the extension is missing.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..config import BackboneConfig


def rope_cos_sin(head_dim: int, theta: float, seqlen: int, device=None, offset: int = 0):
    """fp32 ``cos, sin`` tables ``[seqlen, head_dim]`` (rotate-half convention).

    ``inv_freq = theta^(-2i/d)``; the table is ``cat(freqs, freqs)`` like HF's
    default rope (``LlamaRotaryEmbedding.compute_default_rope_parameters``).
    """
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(offset, offset + seqlen, dtype=torch.float32)
    freqs = torch.outer(pos, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(device), emb.sin().to(device)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x``: [B, H, S, D]; ``cos/sin``: [S, D] fp32. Returns promoted dtype."""
    return x * cos + _rotate_half(x) * sin


def _use_kernels(t: torch.Tensor) -> bool:
    return t.is_cuda


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _use_kernels(x):
            from ..ops import autograd as A

            return A.rms_norm(x, self.weight, self.variance_epsilon)
        dt = x.dtype
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        return self.weight * h.to(dt)


class Attention(nn.Module):
    def __init__(self, bb: BackboneConfig):
        super().__init__()
        self.num_heads = bb.num_attention_heads
        self.num_kv = bb.kv_heads()
        self.head_dim = bb.hidden_size // bb.num_attention_heads
        self.rope_theta = bb.rope_theta
        self.q_proj = nn.Linear(bb.hidden_size, self.num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(bb.hidden_size, self.num_kv * self.head_dim, bias=False)
        self.v_proj = nn.Linear(bb.hidden_size, self.num_kv * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, bb.hidden_size, bias=False)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                pad_mask: torch.Tensor | None = None) -> torch.Tensor:
        if _use_kernels(x):
            from ..ops import autograd as A

            return A.attention_block(x, self, cos, sin, pad_mask)
        b, s, _ = x.shape
        q = self.q_proj(x).view(b, s, self.num_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(b, s, self.num_kv, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(b, s, self.num_kv, self.head_dim).transpose(1, 2)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        if self.num_kv != self.num_heads:
            rep = self.num_heads // self.num_kv
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
        mask = torch.ones(s, s, dtype=torch.bool, device=x.device).tril()
        if pad_mask is not None:  # key padding: [b, s] bool, True = real token
            mask = mask[None, None] & pad_mask[:, None, None, :]
        q, k, v = q.to(v.dtype), k.to(v.dtype), v
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        o = o.transpose(1, 2).reshape(b, s, self.num_heads * self.head_dim)
        return self.o_proj(o)


class MLP(nn.Module):
    def __init__(self, bb: BackboneConfig):
        super().__init__()
        self.gate_proj = nn.Linear(bb.hidden_size, bb.intermediate_size, bias=False)
        self.up_proj = nn.Linear(bb.hidden_size, bb.intermediate_size, bias=False)
        self.down_proj = nn.Linear(bb.intermediate_size, bb.hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _use_kernels(x):
            from ..ops import autograd as A

            return A.mlp_block(x, self)
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    """Pre-norm Llama block: x + attn(norm(x)); then + mlp(norm(.))."""

    def __init__(self, bb: BackboneConfig, layer_idx: int = 0):
        super().__init__()
        self.layer_idx = layer_idx
        self.self_attn = Attention(bb)
        self.mlp = MLP(bb)
        self.input_layernorm = RMSNorm(bb.hidden_size, eps=bb.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(bb.hidden_size, eps=bb.rms_norm_eps)

    def forward(self, x, cos, sin, pad_mask=None):
        h = x + self.self_attn(self.input_layernorm(x), cos, sin, pad_mask)
        return h + self.mlp(self.post_attention_layernorm(h))


class EmbeddingModule(nn.Module):
    """Token embedding (reference ``src/opendipaco/modules.py:42-48``)."""

    def __init__(self, bb: BackboneConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(bb.vocab_size, bb.hidden_size)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        if _use_kernels(ids):
            from ..ops import autograd as A

            return A.embedding(ids, self.embed_tokens.weight)
        return self.embed_tokens(ids)


class BlockModule(nn.Module):
    """A stack of decoder layers: one routing expert or one trunk block."""

    def __init__(self, bb: BackboneConfig, num_layers: int, layer_offset: int = 0):
        super().__init__()
        self.layers = nn.ModuleList(DecoderLayer(bb, layer_offset + i) for i in range(num_layers))

    def forward(self, x, cos, sin, pad_mask=None):
        for layer in self.layers:
            x = layer(x, cos, sin, pad_mask)
        return x


LevelModule = BlockModule


class HeadModule(nn.Module):
    """Final RMSNorm + untied LM head (reference ``src/opendipaco/modules.py:91-98``)."""

    def __init__(self, bb: BackboneConfig):
        super().__init__()
        self.norm = RMSNorm(bb.hidden_size, eps=bb.rms_norm_eps)
        self.lm_head = nn.Linear(bb.hidden_size, bb.vocab_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _use_kernels(x):
            from ..ops import autograd as A

            return A.linear(self.norm(x), self.lm_head.weight)
        return self.lm_head(self.norm(x))


def param_count_per_layer(bb: BackboneConfig) -> int:
    h, f, d = bb.hidden_size, bb.intermediate_size, bb.head_dim
    qkv = h * (bb.num_attention_heads + 2 * bb.kv_heads()) * d
    return qkv + bb.num_attention_heads * d * h + 3 * h * f + 2 * h


def flops_per_token(bb: BackboneConfig, num_layers: int, seq_len: int) -> float:
    """Training FLOPs per token (fwd + bwd = 3x fwd) of one path, causal attention."""
    h, d = bb.hidden_size, bb.head_dim
    per_layer = 2 * (param_count_per_layer(bb) - 2 * h)
    attn = 2 * 2 * bb.num_attention_heads * d * seq_len / 2  # QK^T and PV, causal half
    head = 2 * h * bb.vocab_size
    return 3.0 * (num_layers * (per_layer + attn) + head)


__all__ = [
    "RMSNorm", "Attention", "MLP", "DecoderLayer", "EmbeddingModule", "BlockModule",
    "LevelModule", "HeadModule", "rope_cos_sin", "apply_rope", "flops_per_token",
    "param_count_per_layer",
]
