"""torch-facing wrappers over the C ABI (one call = one or two kernel launches
on the current torch CUDA stream).  Every wrapper takes caller-allocated
outputs, like the reference's fluxvla/ops/atomic_ops.py functions; nothing
here allocates device memory except where a docstring says so.

The per-op entry points that callers reach outside a CUDA graph (GEMM,
norms, softmax, small linear) go through the thin torch C++ extension
``fluxvla_b200._C`` (argument checks with TORCH_CHECK, the current stream,
no Python-side struct building); the others through the ctypes binding of
the same library.  Both are required: there is no fallback.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from ._lib import (ACT_NONE, EPI_BF16, EPI_F32_ACC, EPI_F32_STORE,
                   EPI_GEGLU, EPI_QKV_ROPE, AttnArgs, ExpertArgs, GemmArgs,
                   check)

BF16 = torch.bfloat16
F32 = torch.float32

_ext = None


def _C():
    """The torch extension (built next to the library by
    ``python -m fluxvla_b200.build``)."""
    global _ext
    if _ext is None:
        try:
            from . import _C as ext
        except ImportError as e:
            raise RuntimeError(
                'fluxvla_b200._C is missing: build it with `python -m '
                'fluxvla_b200.build` (there is no fallback path)') from e
        _ext = ext
    return _ext


def _ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _rowmajor(t: torch.Tensor, name: str, dtype) -> int:
    if t.dtype != dtype:
        raise TypeError(f'{name}: expected {dtype}, got {t.dtype}')
    if not t.is_cuda:
        raise ValueError(f'{name}: must be a CUDA tensor')
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f'{name}: expected a 2-D row-major view')
    return t.stride(0)


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *,
         epilogue: int = EPI_BF16, swap: bool = False, act: int = ACT_NONE,
         bias: Optional[torch.Tensor] = None,
         gate: Optional[torch.Tensor] = None, alpha: float = 1.0,
         split_k: int = 1, block_n: int = 0,
         row_add: Optional[torch.Tensor] = None, row_add_mod: int = 0,
         k_out: Optional[torch.Tensor] = None,
         v_out: Optional[torch.Tensor] = None, n_heads: int = 0,
         head_dim: int = 0, rope_cs: Optional[torch.Tensor] = None,
         positions: Optional[torch.Tensor] = None,
         workspace: Optional[torch.Tensor] = None,
         norm: Optional[tuple] = None, pair: bool = False,
         res: Optional[torch.Tensor] = None,
         gate_tok: Optional[torch.Tensor] = None,
         rope_interleaved: bool = False) -> None:
    """C[M,N] = A[M,K] @ B[N,K]^T with a fused epilogue (see fvb_gemm).
    split_k=0 picks the split automatically for swapped GEMMs; a swapped
    split GEMM with a non-additive epilogue needs ``workspace`` (a zeroed
    uint8 tensor of gemm_workspace_bytes(...), left zeroed by the call).
    ``norm=(mode, out_bf16, w, b, eps, sync)`` normalises the finished f32
    output rows into ``out_bf16`` in the same launch (``sync``: an int64
    device tensor, zero before first use).  ``res`` / ``gate_tok`` (bf16
    [m, n] row-major views) make the bf16 epilogue out = res + gate_tok *
    act(alpha*acc + bias); ``rope_interleaved`` stores rotated q / k with each
    rotary pair adjacent."""
    nm, nout, nw, nb, neps, nsync = norm if norm is not None else (
        0, None, None, None, 0.0, None)
    _C().gemm(a, b, out, epilogue, swap, act, bias, gate, alpha, split_k,
              block_n, row_add, row_add_mod, k_out, v_out, n_heads, head_dim,
              rope_cs, positions, workspace, pair, res, gate_tok,
              rope_interleaved, nm, nout, nw, nb, neps, nsync)


def gemm_workspace_bytes(m: int, n: int, swap: bool, epilogue: int) -> int:
    args = GemmArgs(m=m, n=n, swap=int(swap), epilogue=epilogue)
    return int(_lib.lib().fvb_gemm_workspace_bytes(C.byref(args)))


def attn_args(q, k, v, o, *, n_q, n_kv, heads, group, head_dim, scale,
              q_row_stride, q_head_stride, k_row_stride, k_head_stride,
              v_row_stride, v_head_stride, o_row_stride, o_head_stride,
              batch=1, q_batch_rows=0, kv_batch_rows=0, key_valid=None,
              n_prefix=None, q_block=None, k_block=None, kv_splits=1,
              workspace=None) -> AttnArgs:
    return AttnArgs(
        q=_ptr(q), q_row_stride=q_row_stride, q_head_stride=q_head_stride,
        k=_ptr(k), k_row_stride=k_row_stride, k_head_stride=k_head_stride,
        v=_ptr(v), v_row_stride=v_row_stride, v_head_stride=v_head_stride,
        o=_ptr(o), o_row_stride=o_row_stride, o_head_stride=o_head_stride,
        n_q=n_q, n_kv=n_kv, heads=heads, group=group, batch=batch,
        q_batch_rows=q_batch_rows, kv_batch_rows=kv_batch_rows,
        head_dim=head_dim, scale=scale, key_valid=_ptr(key_valid),
        n_prefix=n_kv if n_prefix is None else n_prefix,
        q_block=_ptr(q_block), k_block=_ptr(k_block), kv_splits=kv_splits,
        workspace=_ptr(workspace),
        workspace_bytes=0 if workspace is None else workspace.numel() *
        workspace.element_size())


def attention_workspace_bytes(args: AttnArgs) -> int:
    n = _lib.lib().fvb_attention_workspace_bytes(C.byref(args))
    if n < 0:
        check(1)
    return n


def attention(args: AttnArgs) -> None:
    """Fused attention; with kv_splits > 1 also launches the combine."""
    L = _lib.lib()
    check(L.fvb_attention(C.byref(args), _stream()))
    if args.kv_splits > 1:
        check(L.fvb_attention_combine(C.byref(args), _stream()))


def norm_bf16(mode: int, x: torch.Tensor, out: torch.Tensor, *, w=None,
              b=None, style=None, gate_out=None, eps: float = 1e-6) -> None:
    """Norm of bf16 rows (fvb_norm_bf16): NORM_RMS (no weight), NORM_LAYER
    (w, b bf16) or NORM_ADA_STYLE (style bf16 row: scale | shift | gate;
    the gate goes to gate_out for every row)."""
    _C().norm_bf16(mode, x, out, w, b, style, gate_out, eps)


def softmax_rows(logits: torch.Tensor, out: torch.Tensor, *, n_prefix: int,
                 valid_prefix: torch.Tensor) -> None:
    """bf16 out = softmax over the attended keys of f32 logits rows
    (fvb_softmax_rows); valid_prefix: int32 device tensor of one value."""
    _C().softmax_rows(logits, out, n_prefix, valid_prefix)


def norm(mode: int, x: torch.Tensor, out: torch.Tensor, *, w=None, b=None,
         mod=None, eps: float = 1e-6) -> None:
    _C().norm(mode, x, out, w, b, mod, eps)


def patchify(images_u8: torch.Tensor, patch: int, mean3, std3,
             out: torch.Tensor) -> None:
    """mean3 / std3: three host floats each."""
    V, H, W, _ = images_u8.shape
    m = (C.c_float * 3)(*[float(x) for x in mean3])
    s = (C.c_float * 3)(*[float(x) for x in std3])
    check(_lib.lib().fvb_patchify(_ptr(images_u8), V, H, W, patch,
                                  C.cast(m, C.c_void_p), C.cast(s, C.c_void_p),
                                  _ptr(out), out.stride(0), _stream()))


def patchify_f32(pixels: torch.Tensor, patch: int, out: torch.Tensor) -> None:
    """Normalised f32 pixels [views, 3, H, W] -> bf16 patch rows."""
    V, Cc, H, W = pixels.shape
    assert Cc == 3 and pixels.dtype == torch.float32 and pixels.is_contiguous()
    check(_lib.lib().fvb_patchify_f32(_ptr(pixels), V, H, W, patch,
                                      _ptr(out), out.stride(0), _stream()))


def resize_patchify(images_u8: torch.Tensor, size: int, patch: int, mean3,
                    std3, out: torch.Tensor) -> None:
    """uint8 [V,H,W,3] of any size -> OpenCV INTER_LINEAR resize to
    size x size -> normalise -> bf16 patch rows (as patchify)."""
    V, H, W, _ = images_u8.shape
    m = (C.c_float * 3)(*[float(x) for x in mean3])
    s = (C.c_float * 3)(*[float(x) for x in std3])
    check(_lib.lib().fvb_resize_patchify(_ptr(images_u8), V, H, W, size, patch,
                                         C.cast(m, C.c_void_p), C.cast(s, C.c_void_p),
                                         _ptr(out), out.stride(0), _stream()))


def embed_tokens(ids: torch.Tensor, table: torch.Tensor, scale: float,
                 out: torch.Tensor) -> None:
    check(_lib.lib().fvb_embed_tokens(_ptr(ids), ids.numel(), _ptr(table),
                                      table.shape[1], scale, _ptr(out),
                                      out.stride(0), _stream()))


def small_linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, *,
                 bias=None, act: int = ACT_NONE, mode: int = 0,
                 alpha: float = 1.0, k: Optional[int] = None) -> None:
    """y = act(x @ w[:, :k]^T + bias); mode 0 store f32, 1 store bf16,
    2 out += alpha*y (f32)."""
    _C().small_linear(x, w, out, bias, act, mode, alpha, k or 0)


def probe_wait_timeout(limit_s: float = 0.05) -> bool:
    """Run the bounded-wait failure probe; True if the wait gave up."""
    g = C.c_int(0)
    check(_lib.lib().fvb_probe_wait_timeout(int(limit_s * 1e9), C.byref(g), _stream()))
    return g.value == 1


def device_status(reset: bool = False) -> int:
    s = C.c_int(0)
    check(_lib.lib().fvb_get_device_status(C.byref(s), int(reset)))
    return s.value


def launch_count() -> int:
    return _lib.lib().fvb_launch_count()


def expert_args(*, n_layers, n_tok, width, mlp, heads, head_dim, n_prefix,
                w_qkv, w_o, w_gu, w_down, in_scale, post_scale, x, k_cache,
                v_cache, blocks, positions, rope_cs, rope_suffix=None, qkv_bias=None,
                gu_bias=None, o_gate=None, down_gate=None, key_valid=None,
                eps=1e-6, workspace=None) -> ExpertArgs:
    return ExpertArgs(
        n_layers=n_layers, n_tok=n_tok, width=width, mlp=mlp, heads=heads,
        head_dim=head_dim, n_prefix=n_prefix, w_qkv=_ptr(w_qkv),
        w_o=_ptr(w_o), w_gu=_ptr(w_gu), w_down=_ptr(w_down),
        in_scale=_ptr(in_scale), post_scale=_ptr(post_scale),
        qkv_bias=_ptr(qkv_bias), gu_bias=_ptr(gu_bias), o_gate=_ptr(o_gate),
        down_gate=_ptr(down_gate), eps=eps, x=_ptr(x),
        k_cache=_ptr(k_cache), v_cache=_ptr(v_cache),
        cache_rows=k_cache.shape[1], key_valid=_ptr(key_valid),
        blocks=_ptr(blocks), positions=_ptr(positions),
        rope_cs=_ptr(rope_cs), rope_suffix=_ptr(rope_suffix),
        workspace=_ptr(workspace),
        workspace_bytes=0 if workspace is None else
        workspace.numel() * workspace.element_size())


def expert_workspace_bytes(args: ExpertArgs) -> int:
    n = _lib.lib().fvb_expert_workspace_bytes(C.byref(args))
    if n < 0:
        check(1)
    return int(n)


def expert_step(args: ExpertArgs) -> None:
    """All expert layers of one denoise step (one cooperative launch)."""
    check(_lib.lib().fvb_expert_step(C.byref(args), _stream()))
