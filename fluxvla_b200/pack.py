"""Weight packing for the fused GEMM epilogues (done once at load time).

The reference packs its Gemma weights for Triton in
fluxvla/models/backbones/llms/condition_gemma_inference.py:46-111 (fold
(1+w) into the weights, permute Q/K rows so rotate-half RoPE becomes
pairwise, transpose to [K,N]).  Here weights stay in the nn.Linear
[out, in] layout (K-major, what the tcgen05 descriptors read) and only the
output features are re-ordered so that the two values an epilogue combines
sit in adjacent packed rows:

* QKV + RoPE: per head, packed row 2i = dim i and 2i+1 = dim i + head_dim/2
  (the rotate-half partners), for the 8 query heads and the key head; the
  value head keeps its natural order.  Norm weights are NOT folded (the norm
  kernel applies (1+w) in f32 like GemmaRMSNorm._norm, condition_gemma.py:75).
* gate/up (GeGLU): packed row 2i = gate_proj row i, 2i+1 = up_proj row i.
"""
from __future__ import annotations

import torch


def pair_rows(w: torch.Tensor, head_dim: int) -> torch.Tensor:
    """[H*hd, K] -> rows re-ordered per head to (i, i+hd/2) pairs."""
    H = w.shape[0] // head_dim
    x = w.reshape(H, 2, head_dim // 2, -1)          # [H, half-sel, i, K]
    return x.permute(0, 2, 1, 3).reshape(w.shape)   # [H, i, half-sel, K]


def unpair_rows(w: torch.Tensor, head_dim: int) -> torch.Tensor:
    H = w.shape[0] // head_dim
    x = w.reshape(H, head_dim // 2, 2, -1)
    return x.permute(0, 2, 1, 3).reshape(w.shape)


def pack_qkv(q_w, k_w, v_w, head_dim: int) -> torch.Tensor:
    return torch.cat([pair_rows(q_w, head_dim), pair_rows(k_w, head_dim),
                      v_w], dim=0).contiguous()


def pack_geglu(gate_w, up_w) -> torch.Tensor:
    return torch.stack([gate_w, up_w], dim=1).reshape(
        2 * gate_w.shape[0], -1).contiguous()


def rope_table(max_pos: int, head_dim: int, theta: float = 10000.0,
               device='cpu') -> torch.Tensor:
    """[max_pos, head_dim/2, 2] f32 (cos, sin) of pos * theta^(-2i/d),
    computed as GemmaRotaryEmbedding does (condition_gemma.py:207-260)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64)
                           .float() / head_dim))
    f = torch.arange(max_pos, dtype=torch.int64).float()[:, None] * inv
    return torch.stack([f.cos(), f.sin()], dim=-1).contiguous().to(device)
