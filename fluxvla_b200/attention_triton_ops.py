"""Drop-in for the attention kernels that the reference's PI0.5 Triton path
launches directly (fluxvla/ops/triton/attention_triton_ops.py, called from
pi05_flowmatching_inference.py:100-129,212-245).

Each name is an object that accepts the Triton launch syntax
``kernel[grid](args..., BLOCK_SIZE_*=...)`` with the reference kernel's
argument list; the grid and block sizes are Triton tuning knobs and are
ignored.  Tensors stand where the reference passes pointers, as in a Triton
launch.  The work runs in this library's kernels:

* ``matmul_abT_scale`` (attention_triton_ops.py:6): out[M, N] =
  scale * q[M, K] @ k[N, K]^T, written densely with row stride N into the
  caller's f32 (or bf16) logits buffer — ``fvb_gemm`` (f32 accumulation;
  the reference rounds the logits to bf16 first);
* ``softmax_kernel_masklen`` (:81) and ``softmax_kernel_prefix_suffix``
  (:112): row softmax of those logits over the keys below the valid
  prefix length (read from device memory) plus, for the second, every
  suffix key — ``fvb_softmax_rows``.

The fused path (no logits in HBM) is ``fvb_attention``, which the
library's own engine uses.
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import EPI_BF16, EPI_F32_STORE


class _TritonStyle:
    """``kernel[grid](*args, **meta)`` -> ``fn(*args, **meta)``."""

    def __init__(self, fn):
        self.fn = fn
        self.__doc__ = fn.__doc__
        self.__name__ = fn.__name__

    def __getitem__(self, grid):
        return self.fn

    def __call__(self, *a, **k):
        raise TypeError(f'{self.__name__} is launched as {self.__name__}[grid](...)')


def _dense(t: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """The reference kernels address their buffers as flat row-major arrays
    of `cols` columns from the tensor's first element."""
    return t.reshape(-1)[:rows * cols].view(rows, cols)


def _matmul_abT_scale(q_ptr, k_ptr, out_ptr, M, N, K, scale_factor,
                      BLOCK_SIZE_M=32, BLOCK_SIZE_N=32, BLOCK_SIZE_K=64):
    """attention_triton_ops.py:6 — out = scale * q @ k^T."""
    q = _dense(q_ptr, M, K)
    k = _dense(k_ptr, N, K)
    out = _dense(out_ptr, M, N)
    if out.dtype == torch.float32:
        ops.gemm(q, k, out, epilogue=EPI_F32_STORE, alpha=float(scale_factor))
    else:
        ops.gemm(q, k, out, epilogue=EPI_BF16, alpha=float(scale_factor))


def _softmax_kernel_masklen(inp_ptr, queries, keys, valid_keys_len_ptr,
                            out_ptr, BLOCK_SIZE_M=4, BLOCK_SIZE=1024):
    """attention_triton_ops.py:81 — softmax over keys < valid length."""
    ops.softmax_rows(_dense(inp_ptr, queries, keys), _dense(out_ptr, queries, keys),
                     n_prefix=keys, valid_prefix=valid_keys_len_ptr)


def _softmax_kernel_prefix_suffix(inp_ptr, queries, keys_prefix, keys_suffix,
                                  valid_prefix_len_ptr, out_ptr,
                                  BLOCK_SIZE_M=4, BLOCK_SIZE=1024):
    """attention_triton_ops.py:112 — softmax over the valid prefix keys and
    every suffix key."""
    total = keys_prefix + keys_suffix
    ops.softmax_rows(_dense(inp_ptr, queries, total), _dense(out_ptr, queries, total),
                     n_prefix=keys_prefix, valid_prefix=valid_prefix_len_ptr)


matmul_abT_scale = _TritonStyle(_matmul_abT_scale)
softmax_kernel_masklen = _TritonStyle(_softmax_kernel_masklen)
softmax_kernel_prefix_suffix = _TritonStyle(_softmax_kernel_prefix_suffix)

__all__ = ['matmul_abT_scale', 'softmax_kernel_masklen',
           'softmax_kernel_prefix_suffix']
