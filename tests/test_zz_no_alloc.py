"""fvb_attention_noalloc: the allocation-free attention entry point.

It is for callers that cannot allocate device memory (fixed memory budgets,
allocators that forbid cudaMalloc after start-up, bindings that cannot pass a
device buffer); its key-split scratch lives in an array owned by the library.
This file is collected last so a failure here cannot hide other tests.

Checks, through the C ABI, on two calls in a row with different inputs (the
shared scratch keeps the previous call's contents):
  * the result against a plain PyTorch fp32 attention of the same inputs
    (the numerics) and against fvb_attention + combine with a caller
    workspace (the scratch addressing), for the expert's suffix-mask MQA
    shape (head_dim 256) and for the SigLIP shape (head_dim 72, 16 heads,
    two views as a batch with per-view row offsets);
  * that an oversized request is rejected.
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


def _mqa_case(seed, S=51, E=816, H=8, hd=256, splits=14):
    """Expert suffix attention: 8 query heads over one K/V head, prefix keys
    with a pad mask, suffix keys visible by block id."""
    torch.manual_seed(seed)
    dev = 'cuda'
    q = torch.randn(S, H * hd, device=dev).bfloat16()
    kc = torch.randn(E + S, hd, device=dev).bfloat16()
    vc = torch.randn(E + S, hd, device=dev).bfloat16()
    valid = torch.ones(E, dtype=torch.uint8, device=dev)
    valid[E - 10 - seed:] = 0
    blk = torch.tensor([1] + [2] * (S - 1), dtype=torch.int32, device=dev)
    kw = dict(n_q=S, n_kv=E + S, heads=H, group=H, head_dim=hd,
              scale=hd ** -0.5, q_row_stride=H * hd, q_head_stride=hd,
              k_row_stride=hd, k_head_stride=0, v_row_stride=hd,
              v_head_stride=0, o_row_stride=H * hd, o_head_stride=hd,
              key_valid=valid, n_prefix=E, q_block=blk, k_block=blk,
              kv_splits=splits)
    qf = q.float().view(S, H, hd).transpose(0, 1)           # [H, S, hd]
    s = qf @ kc.float().t() * hd ** -0.5                      # [H, S, E+S]
    vis = torch.zeros(S, E + S, dtype=torch.bool, device=dev)
    vis[:, :E] = valid.bool()[None]
    vis[:, E:] = blk[None, :] <= blk[:, None]
    s = s.masked_fill(~vis[None], float('-inf'))
    ref = (s.softmax(-1) @ vc.float()).transpose(0, 1).reshape(S, H * hd)
    return q, kc, vc, kw, ref, (valid, blk)


def _siglip_case(seed, views=2, T=256, H=16, hd=72, splits=3):
    """SigLIP attention: 16 heads of 72 dims, each view its own sequence,
    q / k / v column blocks of one [views*T, 3*1152] buffer."""
    torch.manual_seed(seed)
    dev = 'cuda'
    W = H * hd
    qkv = torch.randn(views * T, 3 * W, device=dev).bfloat16()
    q, k, v = qkv, qkv[:, W:], qkv[:, 2 * W:]
    kw = dict(n_q=T, n_kv=T, heads=H, group=1, head_dim=hd,
              scale=hd ** -0.5, q_row_stride=3 * W, q_head_stride=hd,
              k_row_stride=3 * W, k_head_stride=hd, v_row_stride=3 * W,
              v_head_stride=hd, o_row_stride=W, o_head_stride=hd,
              batch=views, q_batch_rows=T, kv_batch_rows=T, kv_splits=splits)
    x = qkv.float().view(views, T, 3, H, hd)
    qf, kf, vf = (x[:, :, i].transpose(1, 2) for i in range(3))  # [V,H,T,hd]
    p = (qf @ kf.transpose(-1, -2) * hd ** -0.5).softmax(-1)
    ref = (p @ vf).transpose(1, 2).reshape(views * T, W)
    return q, k, v, kw, ref, (qkv,)


@pytest.mark.parametrize('case', ['mqa_hd256', 'siglip_hd72_batch2'])
def test_noalloc_matches_torch_and_workspace_path_twice(case):
    f = _noalloc()
    stream = torch.cuda.current_stream().cuda_stream
    make = _mqa_case if case == 'mqa_hd256' else _siglip_case
    for seed in (0, 1):
        q, k, v, kw, ref, keep = make(seed)
        o_ws = torch.empty(ref.shape, device='cuda', dtype=torch.bfloat16)
        o_new = torch.empty_like(o_ws)
        a_ws = ops.attn_args(q, k, v, o_ws, **kw)
        ws = torch.empty(max(ops.attention_workspace_bytes(a_ws), 16),
                         dtype=torch.uint8, device='cuda')
        a_ws = ops.attn_args(q, k, v, o_ws, workspace=ws, **kw)
        a_new = ops.attn_args(q, k, v, o_new, **kw)
        ops.attention(a_ws)
        rc = f(C.byref(a_new), stream)
        assert rc == 0, _lib.lib().fvb_last_error().decode()
        torch.cuda.synchronize()
        _close(o_new, ref)        # numerics vs torch fp32
        _close(o_new, o_ws)       # same as the caller-workspace path
    assert ops.device_status() == 0


def test_noalloc_rejects_oversized_scratch():
    f = _noalloc()
    # 8 heads x 2048 query rows x 16 splits x 258 floats = 270 MB > 8 MiB
    q, k, v, kw, _, keep = _mqa_case(2, S=2048, E=1024, splits=16)
    o = torch.empty(2048, 8 * 256, device='cuda', dtype=torch.bfloat16)
    a_new = ops.attn_args(q, k, v, o, **kw)
    rc = f(C.byref(a_new), torch.cuda.current_stream().cuda_stream)
    assert rc == FVB_ERR_WORKSPACE
    assert 'limit' in _lib.lib().fvb_last_error().decode()
