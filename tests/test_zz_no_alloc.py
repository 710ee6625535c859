"""fvb_attention_noalloc: the allocation-free attention entry point.

It is for callers that cannot allocate device memory (fixed memory budgets,
allocators that forbid cudaMalloc after start-up, bindings that cannot pass a
device buffer); its key-split scratch lives in an array owned by the library.
This file is collected last so a failure here cannot hide other tests.

Checks, through the C ABI, that it matches fvb_attention + combine with a
caller workspace (same tolerance as the kernel tests) on two calls in a row
with different inputs (the shared scratch keeps the previous call's
contents), and that an oversized request is rejected.
"""
import ctypes as C

import pytest
import torch

from fluxvla_b200 import _lib, ops
from fluxvla_b200._lib import AttnArgs

pytestmark = pytest.mark.gpu
FVB_ERR_WORKSPACE = 5


def _noalloc():
    f = _lib.lib().fvb_attention_noalloc
    f.restype = C.c_int
    f.argtypes = [C.POINTER(AttnArgs), C.c_void_p]
    return f


def _close(out, ref, tol=1e-2):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale + tol * 0.1, f'max err {err} scale {scale}'


def _case(seed, S=51, E=816, H=8, hd=256, splits=14):
    torch.manual_seed(seed)
    dev = 'cuda'
    q = (torch.randn(S, H * hd, device=dev)).bfloat16()
    kc = torch.randn(E + S, hd, device=dev).bfloat16()
    vc = torch.randn(E + S, hd, device=dev).bfloat16()
    valid = torch.ones(E, dtype=torch.uint8, device=dev)
    valid[E - 10 - seed:] = 0
    blk = torch.tensor([1] + [2] * (S - 1), dtype=torch.int32, device=dev)
    o_ref = torch.empty(S, H * hd, device=dev, dtype=torch.bfloat16)
    o_new = torch.empty_like(o_ref)
    kw = dict(n_q=S, n_kv=E + S, heads=H, group=H, head_dim=hd,
              scale=hd ** -0.5, q_row_stride=H * hd, q_head_stride=hd,
              k_row_stride=hd, k_head_stride=0, v_row_stride=hd,
              v_head_stride=0, o_row_stride=H * hd, o_head_stride=hd,
              key_valid=valid, n_prefix=E, q_block=blk, k_block=blk,
              kv_splits=splits)
    a_ref = ops.attn_args(q, kc, vc, o_ref, **kw)
    ws = torch.empty(max(ops.attention_workspace_bytes(a_ref), 16),
                     dtype=torch.uint8, device=dev)
    a_ref = ops.attn_args(q, kc, vc, o_ref, workspace=ws, **kw)
    a_new = ops.attn_args(q, kc, vc, o_new, **kw)
    return a_ref, a_new, o_ref, o_new, (q, kc, vc, valid, blk, ws)


def test_noalloc_matches_workspace_path_twice():
    f = _noalloc()
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (0, 1):
        a_ref, a_new, o_ref, o_new, keep = _case(seed)
        ops.attention(a_ref)
        rc = f(C.byref(a_new), stream)
        assert rc == 0, _lib.lib().fvb_last_error().decode()
        torch.cuda.synchronize()
        _close(o_new, o_ref)
    assert ops.device_status() == 0


def test_noalloc_rejects_oversized_scratch():
    f = _noalloc()
    # 8 heads x 2048 query rows x 16 splits x 258 floats = 270 MB > 8 MiB
    a_ref, a_new, *_ = _case(2, S=2048, E=1024, splits=16)
    rc = f(C.byref(a_new), torch.cuda.current_stream().cuda_stream)
    assert rc == FVB_ERR_WORKSPACE
    assert 'limit' in _lib.lib().fvb_last_error().decode()
