"""Per-kernel numerics of the CUDA path against plain PyTorch fp32 references
of the same op (bf16 inputs upcast).  Tolerances: bf16 outputs 1e-2 abs +
1e-2 rel of the output scale; f32 outputs 2e-3 rel."""
import math

import pytest
import torch

from fluxvla_b200 import ops
from fluxvla_b200._lib import (ACT_GELU_TANH, ACT_NONE, ACT_SILU, EPI_BF16,
                               EPI_F32_ACC, EPI_F32_STORE, EPI_GEGLU,
                               EPI_QKV_ROPE, NORM_ADA_RMS, NORM_GEMMA_RMS,
                               NORM_LAYER)
from fluxvla_b200.pack import pack_geglu, pack_qkv, rope_table

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def close(out, ref, tol=1e-2):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale + tol * 0.1, f'max err {err} scale {scale}'


def rnd(*s, std=1.0, dtype=torch.bfloat16):
    return (torch.randn(*s, device=DEV) * std).to(dtype)


@pytest.mark.parametrize('m,n,k,bn', [(816, 2560, 2048, 128), (3, 40, 64, 0),
                                      (130, 300, 592, 64), (768, 4304, 1152, 256),
                                      (17, 2048, 4304, 128), (768, 3456, 1152, 192),
                                      (130, 300, 592, 192)])
@pytest.mark.parametrize('act', [ACT_NONE, ACT_GELU_TANH])
def test_gemm_bf16_bias_act(m, n, k, bn, act):
    torch.manual_seed(m + n)
    a, b = rnd(m, k), rnd(n, k, std=0.02)
    bias = torch.randn(n, device=DEV) * 0.1
    out = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    ops.gemm(a, b, out, epilogue=EPI_BF16, bias=bias, act=act, block_n=bn)
    ref = a.float() @ b.float().t() + bias
    if act == ACT_GELU_TANH:
        ref = torch.nn.functional.gelu(ref, approximate='tanh')
    torch.cuda.synchronize()
    close(out, ref)


@pytest.mark.parametrize('tokens', [1, 50, 51, 64])
@pytest.mark.parametrize('feat,k', [(1024, 1024), (2560, 1024), (32, 1024)])
def test_gemm_swap_bf16(tokens, feat, k):
    torch.manual_seed(tokens)
    w, x = rnd(feat, k, std=0.02), rnd(tokens, k)
    bias = torch.randn(feat, device=DEV) * 0.1
    out = torch.empty(tokens, feat, device=DEV, dtype=torch.bfloat16)
    ops.gemm(w, x, out, epilogue=EPI_BF16, swap=True, bias=bias,
             act=ACT_SILU)
    ref = torch.nn.functional.silu(x.float() @ w.float().t() + bias)
    torch.cuda.synchronize()
    close(out, ref)


@pytest.mark.parametrize('swap', [False, True])
@pytest.mark.parametrize('split', [1, 4])
def test_gemm_f32_acc_gate(swap, split):
    torch.manual_seed(3)
    T, F, K = (51, 1024, 4096) if swap else (816, 2048, 2048)
    x, w = rnd(T, K), rnd(F, K, std=0.02)
    res = torch.randn(T, F, device=DEV)
    gate = torch.randn(F, device=DEV)
    bias = torch.randn(F, device=DEV) * 0.1
    out = res.clone()
    if swap:
        ops.gemm(w, x, out, epilogue=EPI_F32_ACC, swap=True, gate=gate,
                 bias=bias, split_k=split, alpha=0.5)
    else:
        ops.gemm(x, w, out, epilogue=EPI_F32_ACC, gate=gate, bias=bias,
                 split_k=split, alpha=0.5)
    ref = res + 0.5 * gate * (x.float() @ w.float().t() + bias)
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize('m,n,k,bn,split', [(130, 300, 592, 128, 3),
                                            (3, 40, 64, 64, 1),
                                            (768, 1152, 4304, 128, 2),
                                            (768, 1152, 4304, 192, 4)])
def test_gemm_f32_acc_ragged(m, n, k, bn, split):
    """Ragged edge tiles of the TMA reduce-add epilogue (rows and columns
    past the end are clipped by the tensor map)."""
    torch.manual_seed(m + split)
    x, w = rnd(m, k), rnd(n, k, std=0.02)
    res = torch.randn(m, n, device=DEV)
    bias = torch.randn(n, device=DEV) * 0.1
    out = res.clone()
    ops.gemm(x, w, out, epilogue=EPI_F32_ACC, bias=bias, split_k=split,
             block_n=bn)
    ref = res + x.float() @ w.float().t() + bias
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize('epi', [EPI_BF16, EPI_F32_STORE, EPI_F32_ACC])
def test_gemm_unaligned_rows_write_back(epi):
    """Output rows that do not start on 16-byte boundaries take the per-row
    write-back instead of the TMA-store epilogue."""
    torch.manual_seed(epi)
    m, n, k = 200, 256, 256
    x, w = rnd(m, k), rnd(n, k, std=0.02)
    f32 = epi in (EPI_F32_STORE, EPI_F32_ACC)
    cols = n
    big = torch.randn(m, cols + 1, device=DEV)
    if not f32:
        big = big.bfloat16()
    out = big[:, :cols]
    before = out.clone()
    edge = big[:, cols].clone()
    ops.gemm(x, w, out, epilogue=epi)
    acc = x.float() @ w.float().t()
    if epi == EPI_F32_ACC:
        ref = before + acc
    else:
        ref = acc
    torch.cuda.synchronize()
    if f32:
        torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)
    else:
        close(out, ref)
    assert torch.equal(big[:, cols], edge)  # the column past the view is untouched


@pytest.mark.parametrize('mode,m,n,k,bn,split', [
    (NORM_GEMMA_RMS, 816, 2048, 2048, 256, 2),
    (NORM_LAYER, 768, 1152, 4304, 192, 4),
    (NORM_LAYER, 100, 1152, 256, 128, 1)])
def test_gemm_fused_residual_norm(mode, m, n, k, bn, split):
    """Residual GEMM with the next norm fused behind a grid-wide barrier:
    out += x w^T, then norm(out) -> bf16, twice on one sync counter."""
    torch.manual_seed(m + n)
    sync = torch.zeros(1, dtype=torch.int64, device=DEV)
    for it in range(2):
        x, w = rnd(m, k), rnd(n, k, std=0.02)
        res = torch.randn(m, n, device=DEV)
        nw, nb = rnd(n, std=0.5), rnd(n, std=0.5)
        out = res.clone()
        xn = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
        ops.gemm(x, w, out, epilogue=EPI_F32_ACC, split_k=split, block_n=bn,
                 norm=(mode, xn, nw, nb if mode == NORM_LAYER else None, 1e-6, sync))
        ref = res + x.float() @ w.float().t()
        torch.cuda.synchronize()
        torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)
        if mode == NORM_LAYER:
            yref = torch.nn.functional.layer_norm(ref, (n,), nw.float(), nb.float(), 1e-6)
        else:
            yref = ref * torch.rsqrt(ref.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + nw.float())
        close(xn, yref)


@pytest.mark.parametrize('swap', [False, True])
def test_gemm_f32_store_row_add(swap):
    torch.manual_seed(4)
    T, F, K = 768, 1152, 592
    x, w = rnd(T, K), rnd(F, K, std=0.02)
    pos = rnd(256, F, std=0.02)
    bias = torch.randn(F, device=DEV) * 0.1
    out = torch.empty(T, F, device=DEV)
    if swap:
        T = 50
        x = x[:T].contiguous()
        out = out[:T].contiguous()
        ops.gemm(w, x, out, epilogue=EPI_F32_STORE, swap=True, bias=bias,
                 row_add=pos, row_add_mod=256)
    else:
        ops.gemm(x, w, out, epilogue=EPI_F32_STORE, bias=bias, row_add=pos,
                 row_add_mod=256)
    ref = x.float() @ w.float().t() + bias + pos.float().repeat(3, 1)[:T]
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize('swap', [False, True])
def test_gemm_geglu(swap):
    torch.manual_seed(5)
    T, F, K = (51, 4096, 1024) if swap else (816, 16384, 2048)
    x = rnd(T, K)
    g, u = rnd(F, K, std=0.02), rnd(F, K, std=0.02)
    wp = pack_geglu(g, u)
    out = torch.empty(T, F, device=DEV, dtype=torch.bfloat16)
    if swap:
        ops.gemm(wp, x, out, epilogue=EPI_GEGLU, swap=True)
    else:
        ops.gemm(x, wp, out, epilogue=EPI_GEGLU)
    xf = x.float()
    ref = torch.nn.functional.gelu(xf @ g.float().t(), approximate='tanh') * (
        xf @ u.float().t())
    torch.cuda.synchronize()
    close(out, ref)


def _rope_ref(x, pos, hd):
    cs = rope_table(int(pos.max()) + 1, hd).to(x.device)
    c = cs[pos.long(), :, 0].repeat(1, 2)[:, None]
    s = cs[pos.long(), :, 1].repeat(1, 2)[:, None]
    x1, x2 = x[..., :hd // 2], x[..., hd // 2:]
    return x * c + torch.cat([-x2, x1], -1) * s


@pytest.mark.parametrize('swap', [False, True])
def test_gemm_qkv_rope(swap):
    torch.manual_seed(6)
    H, hd = 8, 256
    T, K = (51, 1024) if swap else (816, 2048)
    x = rnd(T, K)
    qw, kw, vw = rnd(H * hd, K, std=0.02), rnd(hd, K, std=0.02), rnd(
        hd, K, std=0.02)
    wp = pack_qkv(qw, kw, vw, hd)
    pos = (torch.arange(T, device=DEV) + (816 if swap else 0)).int()
    cs = rope_table(1024, hd, device=DEV)
    q = torch.empty(T, H * hd, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(T + 3, hd, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros(T + 3, hd, device=DEV, dtype=torch.bfloat16)
    kw_ = dict(epilogue=EPI_QKV_ROPE, k_out=kc[2:], v_out=vc[2:], n_heads=H,
               head_dim=hd, rope_cs=cs, positions=pos)
    if swap:
        ops.gemm(wp, x, q, swap=True, **kw_)
    else:
        ops.gemm(x, wp, q, **kw_)
    xf = x.float()
    qr = _rope_ref((xf @ qw.float().t()).view(T, H, hd), pos, hd)
    kr = _rope_ref((xf @ kw.float().t()).view(T, 1, hd), pos, hd)
    torch.cuda.synchronize()
    close(q.view(T, H, hd), qr)
    close(kc[2:2 + T], kr[:, 0])
    close(vc[2:2 + T], xf @ vw.float().t())
    assert kc[:2].abs().sum() == 0 and kc[2 + T:].abs().sum() == 0


def _attn_ref(q, k, v, mask, scale):
    # q [H, Sq, D], k/v [Skv, D], mask [Sq, Skv] bool
    s = (q.float() @ k.float().t()) * scale
    s = s.masked_fill(~mask[None], float('-inf'))
    return torch.softmax(s, -1) @ v.float()


@pytest.mark.parametrize('splits', [1, 7])
def test_attention_suffix_mask_mqa(splits):
    torch.manual_seed(7)
    H, hd, E, S = 8, 256, 816, 51
    q = rnd(S, H * hd)
    kc, vc = rnd(E + S, hd), rnd(E + S, hd)
    o = torch.empty(S, H * hd, device=DEV, dtype=torch.bfloat16)
    valid = torch.ones(E, dtype=torch.uint8, device=DEV)
    valid[800:] = 0
    blk = torch.tensor([1, 2] + [2] * 49, dtype=torch.int32, device=DEV)
    args = ops.attn_args(q, kc, vc, o, n_q=S, n_kv=E + S, heads=H, group=H,
                         head_dim=hd, scale=hd ** -0.5, q_row_stride=H * hd,
                         q_head_stride=hd, k_row_stride=hd, k_head_stride=0,
                         v_row_stride=hd, v_head_stride=0,
                         o_row_stride=H * hd, o_head_stride=hd,
                         key_valid=valid, n_prefix=E, q_block=blk,
                         k_block=blk, kv_splits=splits)
    ws = torch.empty(max(ops.attention_workspace_bytes(args), 16),
                     dtype=torch.uint8, device=DEV)
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    ops.attention(args)
    mask = torch.cat([valid.bool()[None].expand(S, E),
                      blk[None, :] <= blk[:, None]], 1)
    ref = _attn_ref(q.view(S, H, hd).transpose(0, 1), kc, vc, mask,
                    hd ** -0.5)
    torch.cuda.synchronize()
    close(o.view(S, H, hd).transpose(0, 1), ref)


def test_attention_prefix_bidirectional_and_causal():
    torch.manual_seed(8)
    H, hd, E = 8, 256, 816
    q = rnd(E, H * hd)
    kc, vc = rnd(E, hd), rnd(E, hd)
    o = torch.empty_like(q)
    valid = torch.ones(E, dtype=torch.uint8, device=DEV)
    valid[790:] = 0
    base = dict(n_q=E, n_kv=E, heads=H, group=H, head_dim=hd,
                scale=hd ** -0.5, q_row_stride=H * hd, q_head_stride=hd,
                k_row_stride=hd, k_head_stride=0, v_row_stride=hd,
                v_head_stride=0, o_row_stride=H * hd, o_head_stride=hd)
    ops.attention(ops.attn_args(q, kc, vc, o, key_valid=valid, **base))
    ref = _attn_ref(q.view(E, H, hd).transpose(0, 1), kc, vc,
                    valid.bool()[None].expand(E, E), hd ** -0.5)
    torch.cuda.synchronize()
    close(o.view(E, H, hd).transpose(0, 1), ref)
    ar = torch.arange(E, dtype=torch.int32, device=DEV)
    ops.attention(ops.attn_args(q, kc, vc, o, n_prefix=0, q_block=ar,
                                k_block=ar, **base))
    ref = _attn_ref(q.view(E, H, hd).transpose(0, 1), kc, vc,
                    torch.ones(E, E, dtype=torch.bool, device=DEV).tril(),
                    hd ** -0.5)
    torch.cuda.synchronize()
    close(o.view(E, H, hd).transpose(0, 1), ref)


@pytest.mark.parametrize('splits', [1, 2, 3])
@pytest.mark.parametrize('case', ['growing_logits', 'masked_head_blocks',
                                  'all_masked', 'gqa_ragged'])
def test_attention_tensor_core_prefix(case, splits):
    """The tcgen05 prefill attention (unsplit, no suffix blocks): logits that
    grow along the keys force the in-place O rescale; masked leading key
    blocks start rows with no reference max; a fully masked prompt gives
    zeros; 2 K/V heads with a ragged query count cover the flattened
    (head, row) tiling."""
    torch.manual_seed(10)
    hd = 256
    if case == 'gqa_ragged':
        H, G, E = 4, 2, 100
    else:
        H, G, E = 8, 8, 816
    KVH = H // G
    q = rnd(E, H * hd)
    k, v = rnd(E, KVH * hd), rnd(E, KVH * hd)
    valid = torch.ones(E, dtype=torch.uint8, device=DEV)
    if case == 'growing_logits':
        k = (k.float() * (1 + 0.05 * torch.arange(E, device=DEV))[:, None]).bfloat16()
    elif case == 'masked_head_blocks':
        valid[:200] = 0
        valid[700:] = 0
    elif case == 'all_masked':
        valid[:] = 0
    o = torch.full_like(q, 7.0)
    kw = dict(n_q=E, n_kv=E, heads=H, group=G, head_dim=hd,
              scale=hd ** -0.5, q_row_stride=H * hd, q_head_stride=hd,
              k_row_stride=KVH * hd, k_head_stride=hd, v_row_stride=KVH * hd,
              v_head_stride=hd, o_row_stride=H * hd, o_head_stride=hd,
              key_valid=valid, kv_splits=splits)
    args = ops.attn_args(q, k, v, o, **kw)
    ws = torch.empty(max(ops.attention_workspace_bytes(args), 16),
                     dtype=torch.uint8, device=DEV)
    ops.attention(ops.attn_args(q, k, v, o, workspace=ws, **kw))
    torch.cuda.synchronize()
    got = o.view(E, H, hd).transpose(0, 1)
    if case == 'all_masked':
        assert torch.equal(got.float(), torch.zeros_like(got.float()))
        return
    for kh in range(KVH):
        hs = slice(kh * G, (kh + 1) * G)
        ref = _attn_ref(q.view(E, H, hd).transpose(0, 1)[hs],
                        k[:, kh * hd:(kh + 1) * hd], v[:, kh * hd:(kh + 1) * hd],
                        valid.bool()[None].expand(E, E), hd ** -0.5)
        close(got[hs], ref)


def test_attention_siglip_hd72_views():
    torch.manual_seed(9)
    V, P, H, hd = 3, 256, 16, 72
    W = H * hd
    qkv = rnd(V * P, 3 * W)
    o = torch.empty(V * P, W, device=DEV, dtype=torch.bfloat16)
    args = ops.attn_args(qkv, qkv[:, W:], qkv[:, 2 * W:], o, n_q=P, n_kv=P,
                         heads=H, group=1, head_dim=hd, scale=hd ** -0.5,
                         q_row_stride=3 * W, q_head_stride=hd,
                         k_row_stride=3 * W, k_head_stride=hd,
                         v_row_stride=3 * W, v_head_stride=hd,
                         o_row_stride=W, o_head_stride=hd, batch=V,
                         q_batch_rows=P, kv_batch_rows=P)
    ops.attention(args)
    x = qkv.float().view(V, P, 3, H, hd)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), \
        x[:, :, 2].transpose(1, 2)
    ref = torch.softmax(q @ k.transpose(-1, -2) * hd ** -0.5, -1) @ v
    torch.cuda.synchronize()
    close(o.view(V, P, H, hd).transpose(1, 2), ref)


@pytest.mark.parametrize('mode', [NORM_GEMMA_RMS, NORM_ADA_RMS, NORM_LAYER])
@pytest.mark.parametrize('out_f32', [False, True])
@pytest.mark.parametrize('R,D', [(51, 1024), (816, 2048), (768, 1152), (70, 1000)])
def test_norm(mode, out_f32, R, D):
    torch.manual_seed(10)
    x = torch.randn(R, D, device=DEV) * 3 + 0.5
    w = rnd(D, std=0.02) + (1 if mode == NORM_LAYER else 0)
    b = rnd(D, std=0.02)
    mod = torch.randn(2 * D, device=DEV) * 0.1
    out = torch.empty(R, D, device=DEV,
                      dtype=torch.float32 if out_f32 else torch.bfloat16)
    ops.norm(mode, x, out, w=w, b=b, mod=mod, eps=1e-6)
    if mode == NORM_LAYER:
        ref = torch.nn.functional.layer_norm(x, (D,), w.float(), b.float(),
                                             1e-6)
    else:
        n = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-6)
        ref = n * (1 + w.float()) if mode == NORM_GEMMA_RMS else \
            n * (1 + mod[:D]) + mod[D:]
    torch.cuda.synchronize()
    close(out, ref, 1e-2 if not out_f32 else 1e-5)


def test_patchify_embed_small_linear():
    torch.manual_seed(11)
    img = torch.randint(0, 256, (3, 224, 224, 3), dtype=torch.uint8,
                        device=DEV)
    mean = torch.tensor([123.5, 116.0, 103.6], device=DEV)
    std = torch.tensor([58.3, 57.0, 57.3], device=DEV)
    out = torch.empty(768, 592, device=DEV, dtype=torch.bfloat16)
    ops.patchify(img, 14, mean.tolist(), std.tolist(), out)
    x = (img.float().permute(0, 3, 1, 2) - mean[:, None, None]) / (
        std[:, None, None] + 1e-8)
    ref = x.unfold(2, 14, 14).unfold(3, 14, 14)        # V,3,16,16,14,14
    ref = ref.permute(0, 2, 3, 1, 4, 5).reshape(768, 588)
    torch.cuda.synchronize()
    close(out[:, :588], ref)
    assert out[:, 588:].abs().sum() == 0
    # the same patch rows from already normalised f32 CHW pixels (the
    # reference model's `images` input)
    out2 = torch.full_like(out, 7.0)
    ops.patchify_f32(x.contiguous(), 14, out2)
    torch.cuda.synchronize()
    assert torch.equal(out2[:, :588], ref.bfloat16())
    assert out2[:, 588:].abs().sum() == 0

    table = rnd(1000, 64, std=0.02)
    ids = torch.randint(0, 1000, (7,), device=DEV)
    e = torch.zeros(9, 64, device=DEV)
    ops.embed_tokens(ids, table, 8.0, e[2:])
    torch.cuda.synchronize()
    torch.testing.assert_close(e[2:], table[ids].float() * 8.0)

    x = torch.randn(50, 1024, device=DEV)
    w = rnd(32, 1024, std=0.02)
    bias = torch.randn(32, device=DEV)
    acc = torch.randn(50, 32, device=DEV)
    ref = acc - 0.1 * (x @ w.float().t() + bias)
    ops.small_linear(x, w, acc, bias=bias, mode=2, alpha=-0.1)
    torch.cuda.synchronize()
    torch.testing.assert_close(acc, ref, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize('T,K,N,mode,act,xoff', [
    (50, 32, 1024, 1, ACT_NONE, 0),      # narrow K, bf16 out (action in-proj)
    (1, 32, 1024, 0, ACT_NONE, 0),       # state token
    (50, 1024, 32, 2, ACT_NONE, 0),      # wide K, x += alpha * y (out-proj)
    (7, 1024, 100, 0, ACT_SILU, 0),      # wide K, f32 out with activation
    (5, 40, 33, 0, ACT_NONE, 0),         # narrow K, ragged N
    (3, 300, 17, 0, ACT_GELU_TANH, 1)])  # generic path (K not a multiple of 256, unaligned x)
def test_small_linear_paths(T, K, N, mode, act, xoff):
    torch.manual_seed(T * K + N)
    xb = torch.randn(T, K + xoff, device=DEV)
    x = xb[:, xoff:]
    w = rnd(N, K, std=0.1)
    bias = torch.randn(N, device=DEV)
    y = x @ w.float().t() + bias
    if act == ACT_SILU:
        y = torch.nn.functional.silu(y)
    elif act == ACT_GELU_TANH:
        y = torch.nn.functional.gelu(y, approximate='tanh')
    if mode == 1:
        out = torch.empty(T, N, device=DEV, dtype=torch.bfloat16)
        ref = y
    elif mode == 2:
        out = torch.randn(T, N, device=DEV)
        ref = out + 0.25 * y
    else:
        out = torch.empty(T, N, device=DEV)
        ref = y
    ops.small_linear(x, w, out, bias=bias, mode=mode, alpha=0.25, act=act)
    torch.cuda.synchronize()
    if mode == 1:
        close(out, ref)
    else:
        torch.testing.assert_close(out, ref, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize('h,w,size,patch', [(256, 256, 224, 14), (480, 640, 224, 14),
                                            (20, 30, 28, 14), (61, 47, 56, 14),
                                            (224, 224, 224, 14), (96, 96, 48, 12)])
def test_resize_patchify_bit_exact(h, w, size, patch):
    """Device resize (OpenCV INTER_LINEAR) + normalise + patch rows equal the
    oracle's restatement bit for bit (uint8 resize, then the same f32
    normalise and bf16 rounding)."""
    import numpy as np
    from oracle.pi0_oracle import resize_linear_u8
    V = 3
    mean3, std3 = (0.485 * 255, 0.456 * 255, 0.406 * 255), (0.229 * 255, 0.224 * 255, 0.225 * 255)
    rng = np.random.default_rng(h * w)
    imgs = rng.integers(0, 256, (V, h, w, 3), dtype=np.uint8)
    g = size // patch
    K = 3 * patch * patch
    out = torch.full((V * g * g, K + 4), 9.0, device=DEV, dtype=torch.bfloat16)
    ops.resize_patchify(torch.from_numpy(imgs).to(DEV), size, patch, mean3, std3, out)
    r = torch.from_numpy(np.stack([resize_linear_u8(v, size, size) for v in imgs]))
    x = r.float().permute(0, 3, 1, 2)
    x = (x - torch.tensor(mean3)[:, None, None]) / (torch.tensor(std3)[:, None, None] + 1e-8)
    p = x.unfold(2, patch, patch).unfold(3, patch, patch)
    ref = p.permute(0, 2, 3, 1, 4, 5).reshape(V * g * g, K).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(out[:, :K].cpu(), ref)
    assert (out[:, K:].float() == 0).all()


@pytest.mark.parametrize('split', [0, 3, 16])
def test_gemm_swap_split_fixup(split):
    """Swapped split-K GEMMs with non-additive epilogues reduce their splits
    in the workspace; results match and the workspace is left zeroed."""
    torch.manual_seed(12)
    T, K, H, hd = 51, 1024, 8, 256
    x = rnd(T, K)
    ws = torch.zeros(ops.gemm_workspace_bytes(4096 * 2, T, True, EPI_GEGLU),
                     dtype=torch.uint8, device=DEV)
    # GeGLU
    g, u = rnd(4096, K, std=0.02), rnd(4096, K, std=0.02)
    out = torch.empty(T, 4096, device=DEV, dtype=torch.bfloat16)
    for _ in range(2):
        ops.gemm(pack_geglu(g, u), x, out, epilogue=EPI_GEGLU, swap=True,
                 split_k=split, workspace=ws)
    xf = x.float()
    ref = torch.nn.functional.gelu(xf @ g.float().t(), approximate='tanh') * (
        xf @ u.float().t())
    torch.cuda.synchronize()
    close(out, ref)
    assert ws.count_nonzero() == 0
    # SiLU with bias
    w = rnd(1024, K, std=0.02)
    bias = torch.randn(1024, device=DEV) * 0.1
    out = torch.empty(T, 1024, device=DEV, dtype=torch.bfloat16)
    ops.gemm(w, x, out, swap=True, bias=bias, act=ACT_SILU, split_k=split,
             workspace=ws)
    torch.cuda.synchronize()
    close(out, torch.nn.functional.silu(xf @ w.float().t() + bias))
    assert ws.count_nonzero() == 0
    # QKV + RoPE
    qw, kw, vw = rnd(H * hd, K, std=0.02), rnd(hd, K, std=0.02), rnd(
        hd, K, std=0.02)
    pos = (torch.arange(T, device=DEV) + 816).int()
    cs = rope_table(1024, hd, device=DEV)
    q = torch.empty(T, H * hd, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(T, hd, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros(T, hd, device=DEV, dtype=torch.bfloat16)
    ops.gemm(pack_qkv(qw, kw, vw, hd), x, q, swap=True, epilogue=EPI_QKV_ROPE,
             k_out=kc, v_out=vc, n_heads=H, head_dim=hd, rope_cs=cs,
             positions=pos, split_k=split, workspace=ws)
    torch.cuda.synchronize()
    close(q.view(T, H, hd), _rope_ref((xf @ qw.float().t()).view(T, H, hd), pos, hd))
    close(kc, _rope_ref((xf @ kw.float().t()).view(T, 1, hd), pos, hd)[:, 0])
    close(vc, xf @ vw.float().t())
    assert ws.count_nonzero() == 0


def test_gemm_split_without_workspace_is_rejected():
    x, w = rnd(51, 1024), rnd(1024, 1024, std=0.02)
    out = torch.empty(51, 1024, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match='workspace'):
        ops.gemm(w, x, out, swap=True, split_k=4)


def test_bounded_wait_gives_up_and_context_stays_usable():
    """Failure path without a GPU fault: a wait on an mbarrier that nothing
    arrives on runs out after its (short) limit, the kernel records
    FVB_ERR_DEVICE_TIMEOUT and returns, and the next kernels run normally."""
    from fluxvla_b200._lib import FVB_ERR_DEVICE_TIMEOUT
    ops.device_status(reset=True)
    assert ops.probe_wait_timeout(0.05)
    assert ops.device_status(reset=True) == FVB_ERR_DEVICE_TIMEOUT
    assert ops.device_status() == 0
    a, b = rnd(64, 64), rnd(64, 64)
    out = torch.empty(64, 64, device=DEV, dtype=torch.bfloat16)
    ops.gemm(a, b, out)
    torch.cuda.synchronize()
    close(out, a.float() @ b.float().t())
    assert ops.device_status() == 0


@pytest.mark.parametrize('F,T,K,epi,split', [
    (1024, 816, 512, EPI_GEGLU, 1),
    (640, 100, 256, EPI_GEGLU, 1),
    (512, 816, 1024, EPI_F32_ACC, 1),
    (384, 300, 2048, EPI_F32_ACC, 3)])
def test_gemm_pair_two_sm(F, T, K, epi, split):
    """Two-SM (cta_group::2) swapped GEMM: 256 weight rows x 208 tokens per
    CTA pair, each SM loading half of the token tile."""
    torch.manual_seed(F + T)
    w, x = rnd(F, K, std=0.02), rnd(T, K)
    acc = x.float() @ w.float().t()
    if epi == EPI_GEGLU:
        out = torch.empty(T, F // 2, device=DEV, dtype=torch.bfloat16)
        ops.gemm(w, x, out, epilogue=EPI_GEGLU, swap=True, pair=True)
        ref = torch.nn.functional.gelu(acc[:, 0::2], approximate='tanh') * acc[:, 1::2]
        torch.cuda.synchronize()
        close(out, ref)
    else:
        res = torch.randn(T, F, device=DEV)
        out = res.clone()
        ops.gemm(w, x, out, epilogue=EPI_F32_ACC, swap=True, pair=True, split_k=split)
        torch.cuda.synchronize()
        torch.testing.assert_close(out, res + acc, atol=2e-3, rtol=2e-3)
    assert ops.device_status() == 0
