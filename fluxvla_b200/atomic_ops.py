"""Drop-in for the PI0 / PI0.5 operators of ``fluxvla/ops/atomic_ops.py``.

Every function keeps the reference's name, positional / keyword signature,
out-parameter convention (callers pass preallocated bf16 buffers, functions
return ``None`` except ``AttnMultiKey``, which returns a new tensor as the
reference does) and the reference's buffer layouts:

* weights as the reference's Triton packer leaves them
  (condition_gemma_inference.py:65-170, siglip_vit_inference.py:10): bf16
  ``[in_features, out_features]`` row-major, RMSNorm ``(1 + w)`` folded into
  the QKV / gate / up weights of the prefix LLM, Q / K output columns in
  the pairwise-RoPE order (column 2i = dim i, 2i+1 = dim i + head_dim/2);
* activations, residual streams and biases in bf16;
* the rotary table as ``[rows, head_dim]`` bf16 (cos, sin) pairs
  (pi05_flowmatching_inference.py:444-456), one row per token;
* q / k outputs with each rotary pair adjacent (the Triton kernels'
  ``tl.interleave``, attention_triton_ops.py:149-214).

The arithmetic runs in this library's kernels (``fvb_gemm``,
``fvb_norm_bf16``, ``fvb_attention``).  Their weight operand is K-major
(``[out, in]``, what the tcgen05 shared-memory descriptors read), so each
reference weight is transposed once, on first use, into a cache keyed by the
tensor's storage, shape and version; f32 copies of the bf16 biases are cached
the same way.  Input reshapes the reference wrapper itself does in torch
(the patch gather of ``conv2d_embed_res``) are done in torch here too.

Numerics differ from the reference only in rounding order: GEMMs accumulate
in f32 and round once, and q / k are rotated before (not after) rounding to
bf16.  The operators of the GR00T head (``mha_*``, ``ff_gelu``,
``dit_block_*``, ``vl_sa_block``, ``ada_layer_norm``, ``layer_norm_triton``)
and ``rms_matmul_scaled_qkv_rope`` (Eagle2 only) are outside this path.
"""
from __future__ import annotations

import math
import weakref
from typing import Dict, Tuple

import torch

from . import ops
from ._lib import (ACT_GELU_TANH, ACT_SILU, EPI_BF16, EPI_GEGLU,
                   EPI_QKV_ROPE, NORM_ADA_STYLE, NORM_LAYER, NORM_RMS)
from .pack import pack_geglu

BF16 = torch.bfloat16

_cache: Dict[Tuple, tuple] = {}
_pos: Dict[Tuple, torch.Tensor] = {}


def _owner(t: torch.Tensor) -> torch.Tensor:
    """The tensor that owns a view's memory (the view itself otherwise)."""
    return t._base if t._base is not None else t


def _key(tag, *ts):
    return (tag,) + tuple((id(_owner(t)), t.storage_offset(), tuple(t.shape),
                           tuple(t.stride()), t._version) for t in ts)


def _cached(tag, make, *ts):
    """Derived copy (transpose, f32 cast, packing) of caller tensors, kept
    while those tensors live and are unmodified.  Entries hold weak
    references to the owning tensors: a new tensor that happens to reuse a
    freed tensor's memory (or Python id) never hits an old entry, and
    entries of dead tensors are dropped."""
    k = _key(tag, *ts)
    e = _cache.get(k)
    if e is not None and all(r() is _owner(t) for r, t in zip(e[0], ts)):
        return e[1]
    for kk in [kk for kk, (refs, _) in _cache.items()
               if any(r() is None for r in refs)]:
        del _cache[kk]
    v = make()
    _cache[k] = ([weakref.ref(_owner(t)) for t in ts], v)
    return v


def clear_cache() -> None:
    """Drop the transposed-weight / f32-bias copies (e.g. after new weights
    were loaded into the same buffers without a version bump)."""
    _cache.clear()
    _pos.clear()
    _scratch_bufs.clear()


_scratch_bufs: Dict[Tuple, torch.Tensor] = {}


def _scratch(tag: str, rows: int, cols: int, device) -> torch.Tensor:
    """A zero-initialised bf16 staging buffer kept per (tag, shape, device):
    allocated on the first call of a shape only.  Callers overwrite the
    leading columns each call; padding columns stay zero."""
    k = (tag, rows, cols, str(device))
    t = _scratch_bufs.get(k)
    if t is None:
        t = torch.zeros(rows, cols, dtype=BF16, device=device)
        _scratch_bufs[k] = t
    return t


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def _wt(w: torch.Tensor) -> torch.Tensor:
    """Reference weight [K, N] -> [N, K8] bf16, K zero-padded to a multiple
    of 8 (the GEMM's row pitch rule)."""
    def make():
        k, n = w.shape
        t = torch.zeros(n, _pad8(k), dtype=BF16, device=w.device)
        t[:, :k] = w.t()
        return t
    return _cached('wt', make, w)


def _geglu_w(gate_w: torch.Tensor, up_w: torch.Tensor) -> torch.Tensor:
    """Separate [K, I] gate / up weights -> [2I, K] rows (gate_i, up_i)."""
    return _cached('geglu', lambda: pack_geglu(gate_w.t(), up_w.t()),
                   gate_w, up_w)


def _f32(b: torch.Tensor) -> torch.Tensor:
    return _cached('f32', lambda: b.reshape(-1).float().contiguous(), b)


def _rows(t: torch.Tensor, n: int) -> torch.Tensor:
    """[..., n] contiguous -> [rows, n] view."""
    return t.reshape(-1, n)


def _ln(x2, norm_w, norm_b, x_norm2, eps):
    ops.norm_bf16(NORM_LAYER, x2, x_norm2, w=norm_w.reshape(-1),
                  b=norm_b.reshape(-1), eps=eps)


def _linear(x2, w, out2, *, bias=None, act=0, res=None, gate_tok=None):
    """out2 = [res +] [gate_tok *] act(x2 @ w + bias), reference w [K, N]."""
    wt = _wt(w)
    k = x2.shape[1]
    if wt.shape[1] != k:  # K not a multiple of 8: pad the activation rows
        xp = _scratch('linear_x', x2.shape[0], wt.shape[1], x2.device)
        xp[:, :k].copy_(x2)
        x2 = xp
    ops.gemm(x2, wt, out2, epilogue=EPI_BF16, act=act,
             bias=None if bias is None else _f32(bias), res=res,
             gate_tok=gate_tok)


def _positions(n: int, device) -> torch.Tensor:
    """0..n-1 as int32 (the reference's rotary table has one row per token)."""
    k = (n, str(device))
    if k not in _pos:
        _pos[k] = torch.arange(n, dtype=torch.int32, device=device)
    return _pos[k]


def _qkv_rope(x2, weight_qkv, rope_weight, Q, K, V, head_dim, num_heads):
    seq = x2.shape[0]
    wt = _wt(weight_qkv)
    cs = rope_weight[:seq].float().reshape(seq, head_dim // 2, 2)
    ops.gemm(x2, wt, Q.reshape(seq, -1), epilogue=EPI_QKV_ROPE,
             k_out=K.reshape(seq, head_dim), v_out=V.reshape(seq, head_dim),
             n_heads=num_heads, head_dim=head_dim, rope_cs=cs,
             positions=_positions(seq, x2.device), rope_interleaved=True)


# ---------------------------------------------------------------------------
# Vision encoder ops (atomic_ops.py:34-111)
# ---------------------------------------------------------------------------

def conv2d_embed_res(images, patch_w, patch_b, pos_emb, out, grid_size,
                     patch_size, num_patches, vit_hidden):
    """atomic_ops.py:34 — patch embedding: out[v*P + p] = patch(v, p) @ W + b
    + pos_emb[p], patch vectors in (kh, kw, c) order."""
    nviews = images.shape[0]
    seq = num_patches * nviews
    feats = 3 * patch_size * patch_size
    x = images.view(nviews, grid_size, patch_size, grid_size, patch_size,
                    3).permute(0, 1, 3, 2, 4, 5).reshape(seq, feats)
    pos = _cached(('pos_rep', nviews), lambda: pos_emb.reshape(
        num_patches, vit_hidden).repeat(nviews, 1).contiguous(), pos_emb)
    _linear(x.contiguous(), patch_w, _rows(out, vit_hidden), bias=patch_b,
            res=pos)


def layer_norm_QKV_matmul_bias(x, norm_w, norm_b, qkv_w, qkv_b, out, x_norm,
                               num_patches, vit_hidden, vit_qkv_hidden):
    """atomic_ops.py:56 — LayerNorm (eps 1e-5, the Triton kernel's default)
    then out = x_norm @ W + b."""
    xn = _rows(x_norm, vit_hidden)
    _ln(_rows(x, vit_hidden), norm_w, norm_b, xn, 1e-5)
    _linear(xn, qkv_w, _rows(out, vit_qkv_hidden), bias=qkv_b)


def AttnMultiKey(QKV, num_patches, vit_num_heads, vit_head_dim, vit_hidden):
    """atomic_ops.py:65 — per-view multi-head self-attention over the fused
    QKV rows (SDPA, scale 1/sqrt(head_dim)); returns [views, patches,
    hidden]."""
    qkv = QKV.reshape(-1, num_patches, 3 * vit_hidden)
    nv = qkv.shape[0]
    out = torch.empty(nv, num_patches, vit_hidden, dtype=QKV.dtype,
                      device=QKV.device)
    q2 = qkv.reshape(-1, 3 * vit_hidden)
    W = vit_hidden
    ops.attention(ops.attn_args(
        q2, q2[:, W:], q2[:, 2 * W:], out.reshape(-1, W), n_q=num_patches,
        n_kv=num_patches, heads=vit_num_heads, group=1, head_dim=vit_head_dim,
        scale=1.0 / math.sqrt(vit_head_dim), q_row_stride=3 * W,
        q_head_stride=vit_head_dim, k_row_stride=3 * W,
        k_head_stride=vit_head_dim, v_row_stride=3 * W,
        v_head_stride=vit_head_dim, o_row_stride=W, o_head_stride=vit_head_dim,
        batch=nv, q_batch_rows=num_patches, kv_batch_rows=num_patches))
    return out


def matmul_bias_res(x, weight, bias, res, out, buf, num_patches, vit_hidden):
    """atomic_ops.py:79 — out = x @ W + b + res (cublasLt bias + residual)."""
    n = weight.shape[1]
    _linear(_rows(x, weight.shape[0]), weight, _rows(out, n), bias=bias,
            res=_rows(res, n))


def layer_norm_matmul_bias_gelu(x, norm_w, norm_b, weight, bias, out, x_norm,
                                num_patches, vit_hidden, vit_intermediate):
    """atomic_ops.py:83 — LayerNorm (eps 1e-5) then out = gelu_tanh(x_norm @
    W + b)."""
    xn = _rows(x_norm, vit_hidden)
    _ln(_rows(x, vit_hidden), norm_w, norm_b, xn, 1e-5)
    _linear(xn, weight, _rows(out, vit_intermediate), bias=bias,
            act=ACT_GELU_TANH)


def matmul_split_k_bias_res(x, weight, bias, res, out, buf, num_patches,
                            vit_intermediate, vit_hidden):
    """atomic_ops.py:107 — out = x @ W + b + res."""
    matmul_bias_res(x, weight, bias, res, out, buf, num_patches, vit_hidden)


def layer_norm_matmul_bias(x, norm_w, norm_b, proj_w, proj_b, out, x_norm,
                           num_patches, in_features, out_features, eps=1e-5):
    """atomic_ops.py:117 — LayerNorm(eps) then out = x_norm @ W + b."""
    x2 = _rows(x, in_features)
    xn = _rows(x_norm, in_features)[:x2.shape[0]]
    _ln(x2, norm_w, norm_b, xn, eps)
    _linear(xn, proj_w, _rows(out, out_features)[:x2.shape[0]], bias=proj_b)


# ---------------------------------------------------------------------------
# Gemma prefix / action expert ops (atomic_ops.py:155-385)
# ---------------------------------------------------------------------------

def rms_matmul_qkv_rope(x, weight_qkv, rope_weight, Q, K, V, x_norm,
                        hidden_dim, head_dim, num_kv_heads):
    """atomic_ops.py:155 — x_norm = x * rsqrt(mean(x^2) + 1e-6) (the (1+w)
    scale is folded into weight_qkv), then [q | k | v] = x_norm @ W with
    RoPE on q (num_kv_heads heads — the reference passes the query head
    count under this name) and k."""
    x2 = _rows(x, hidden_dim)
    xn = _rows(x_norm, hidden_dim)
    ops.norm_bf16(NORM_RMS, x2, xn, eps=1e-6)
    _qkv_rope(xn, weight_qkv, rope_weight, Q, K, V, head_dim, num_kv_heads)


def matmul_res(x, weight, out, in_features, out_features):
    """atomic_ops.py:172 — out += x @ W (bf16 residual, one rounding)."""
    o = _rows(out, out_features)
    _linear(_rows(x, in_features), weight, o, res=o)


def rms_matmul_gate(x, gate_w, up_w, out, x_norm, hidden_dim,
                    intermediate_dim):
    """atomic_ops.py:196 — RMS norm (no weight), then out =
    gelu_tanh(x_norm @ Wg) * (x_norm @ Wu)."""
    xn = _rows(x_norm, hidden_dim)
    ops.norm_bf16(NORM_RMS, _rows(x, hidden_dim), xn, eps=1e-6)
    matmul_gate(xn, gate_w, up_w, out, hidden_dim, intermediate_dim)


def matmul_attn_v(x, V, out, head_dim):
    """atomic_ops.py:209 — out = P @ V for probabilities x [queries, keys]
    and values V [keys, head_dim] (the reference's unfused attention; the
    fused path is ``fvb_attention``)."""
    q, keys = x.shape
    kp = _pad8(keys)
    vt = _scratch('attn_vt', head_dim, kp, x.device)
    vt[:, :keys].copy_(V.reshape(keys, head_dim).t())
    if kp != keys:
        xp = _scratch('attn_p', q, kp, x.device)
        xp[:, :keys].copy_(x)
        x = xp
    ops.gemm(x, vt, _rows(out, head_dim), epilogue=EPI_BF16)


def matmul_bias_silu(x, weight, bias, out, in_features, out_features):
    """atomic_ops.py:229 — out = silu(x @ W + b)."""
    x2 = _rows(x, in_features)
    _linear(x2, weight, _rows(out, out_features)[:x2.shape[0]], bias=bias,
            act=ACT_SILU)


def matmul_bias_small(x, weight, bias, out, in_features, out_features,
                      BLOCK_SIZE_N=32, BLOCK_SIZE_M=32, BLOCK_SIZE_K=32):
    """atomic_ops.py:249 — out = x @ W + b (block sizes are tuning knobs of
    the Triton kernel and have no effect here)."""
    x2 = _rows(x, in_features)
    _linear(x2, weight, _rows(out, out_features)[:x2.shape[0]], bias=bias)


def adarms_norm_style_proj(x, time_emb, mod_w, mod_b, x_normed, gate, style,
                           hidden_dim, style_dim):
    """atomic_ops.py:278 — style = time_emb @ Wmod + bmod over x's rows, then
    adaRMSNorm with (scale | shift | gate) of style row 0:
    x_normed = x * rsqrt(mean(x^2) + 1e-6) * (1 + scale) + shift, gate
    broadcast to every row (adarms_norm_kernel norm_triton_ops.py:355)."""
    x2 = _rows(x, hidden_dim)
    seq = x2.shape[0]
    st = _rows(style, style_dim)[:seq]
    _linear(_rows(time_emb, hidden_dim)[:seq], mod_w, st, bias=mod_b)
    ops.norm_bf16(NORM_ADA_STYLE, x2, _rows(x_normed, hidden_dim), style=st,
                  gate_out=_rows(gate, hidden_dim), eps=1e-6)


def matmul_qkv_rope(x_normed, weight_qkv, rope_weight, Q, K, V, hidden_dim,
                    head_dim, num_kv_heads):
    """atomic_ops.py:307 — [q | k | v] = x_normed @ W with RoPE on q and k."""
    _qkv_rope(_rows(x_normed, hidden_dim), weight_qkv, rope_weight, Q, K, V,
              head_dim, num_kv_heads)


def matmul_res_gate(x, weight, out, gate, in_features, out_features,
                    BLOCK_SIZE_N=32, BLOCK_SIZE_M=32, BLOCK_SIZE_K=128):
    """atomic_ops.py:343 — out += (x @ W) * gate, gate bf16 [rows, N]."""
    o = _rows(out, out_features)
    _linear(_rows(x, in_features), weight, o, res=o,
            gate_tok=_rows(gate, out_features)[:o.shape[0]])


def matmul_gate(x, gate_w, up_w, out, in_features, intermediate_dim):
    """atomic_ops.py:373 — out = gelu_tanh(x @ Wg) * (x @ Wu)."""
    ops.gemm(_rows(x, in_features), _geglu_w(gate_w, up_w),
             _rows(out, intermediate_dim), epilogue=EPI_GEGLU)


__all__ = [
    'AttnMultiKey', 'adarms_norm_style_proj', 'conv2d_embed_res',
    'layer_norm_matmul_bias', 'layer_norm_matmul_bias_gelu',
    'layer_norm_QKV_matmul_bias', 'matmul_attn_v', 'matmul_bias_res',
    'matmul_bias_silu', 'matmul_bias_small', 'matmul_gate',
    'matmul_qkv_rope', 'matmul_res', 'matmul_res_gate',
    'matmul_split_k_bias_res', 'rms_matmul_gate', 'rms_matmul_qkv_rope',
    'clear_cache']
