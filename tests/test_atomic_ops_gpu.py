"""GPU parity of the atomic_ops drop-in: every operator of the reference's
PI0 / PI0.5 Triton path, called with the reference's buffer layouts
(bf16 activations, [in, out] weights, interleaved rotary tables), against a
float32 torch restatement of the reference kernel it replaces:

  conv2d_embed_res          matmul_small_bias_res_mod matmul_triton_ops.py:100
  layer_norm_*              layer_norm_small_kernel norm_triton_ops.py:90
  rms_matmul_*              rms_norm_kernel norm_triton_ops.py:317
  *_qkv_rope                matmul_n_2048_2560_qkv_rope / matmul_rope_qkv
                            attention_triton_ops.py:149,293
  matmul_res / _res_gate    matmul_small_res / _res_gate matmul_triton_ops.py:548,713
  matmul_gate               matmul_small_gate matmul_triton_ops.py:764
  matmul_bias_silu / _small matmul_small_bias_silu / _bias :590,12
  adarms_norm_style_proj    matmul_small_bias + adarms_norm_kernel norm_triton_ops.py:355
  matmul_bias_res           cublasLt bias + residual (matmul_bias_forward_cuda.cu)
  AttnMultiKey              torch SDPA (atomic_ops.py:65)

Tolerance: bf16 outputs within relative L2 1e-2 and max-abs 3e-2 of the
largest reference magnitude.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from fluxvla_b200 import atomic_ops as A

pytestmark = pytest.mark.gpu
dev = 'cuda'
bf = torch.bfloat16


def close(out, ref, name=''):
    out, ref = out.float(), ref.float()
    rel = ((out - ref).norm() / ref.norm().clamp_min(1e-12)).item()
    mx = (out - ref).abs().max().item()
    lim = 3e-2 * ref.abs().max().item()
    assert rel <= 1e-2 and mx <= lim, f'{name}: rel-l2 {rel:.3e} max-abs {mx:.3e} (lim {lim:.3e})'


def g(seed):
    return torch.Generator(device=dev).manual_seed(seed)


def rn(*shape, seed=0, scale=1.0):
    return (torch.randn(*shape, generator=g(seed), device=dev) * scale).to(bf)


def gelu_tanh(x):
    return 0.5 * x * (1 + torch.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))


def rms(x, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def ln(x, w, b, eps):
    m = x.mean(-1, keepdim=True)
    v = (x - m).pow(2).mean(-1, keepdim=True)
    return (x - m) * torch.rsqrt(v + eps) * w + b


def rope_interleaved(y, cs):
    """y [t, 2n] pairs (2i, 2i+1) rotated by cs [t, 2n] (cos, sin) pairs."""
    a, b = y[:, 0::2], y[:, 1::2]
    c, s = cs[:, 0::2], cs[:, 1::2]
    out = torch.empty_like(y)
    out[:, 0::2] = a * c - b * s
    out[:, 1::2] = b * c + a * s
    return out


def rope_table(rows, hd=256, start=0):
    pos = torch.arange(start, start + rows, device=dev, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd))
    ph = pos[:, None] * inv[None]
    return torch.stack([ph.cos(), ph.sin()], -1).reshape(rows, hd).to(bf)


# ---------------------------------------------------------------------------
# vision encoder ops (SigLIP So400m widths, 2 views)
# ---------------------------------------------------------------------------
NV, P, VH, VI, VHEADS, VHD = 2, 256, 1152, 4304, 16, 72


def test_conv2d_embed_res():
    imgs = rn(NV, 224, 224, 3, seed=1)
    w, b, pos = rn(588, VH, seed=2, scale=0.02), rn(VH, seed=3, scale=0.02), rn(P, VH, seed=4)
    out = torch.zeros(NV, P, VH, dtype=bf, device=dev)
    A.conv2d_embed_res(imgs, w, b, pos, out, 16, 14, P, VH)
    x = imgs.float().view(NV, 16, 14, 16, 14, 3).permute(0, 1, 3, 2, 4, 5).reshape(NV * P, 588)
    ref = x @ w.float() + b.float() + pos.float().repeat(NV, 1)
    close(out.reshape(-1, VH), ref, 'conv2d_embed_res')


def test_layer_norm_qkv_attention_and_residuals():
    x = rn(NV, P, VH, seed=5)
    nw, nb = rn(VH, seed=6, scale=0.1), rn(VH, seed=7, scale=0.1)
    qw, qb = rn(VH, 3 * VH, seed=8, scale=0.02), rn(3 * VH, seed=9, scale=0.02)
    qkv = torch.empty(NV, P, 3 * VH, dtype=bf, device=dev)
    xn = torch.empty(NV, P, VH, dtype=bf, device=dev)
    A.layer_norm_QKV_matmul_bias(x, nw, nb, qw, qb, qkv, xn, P, VH, 3 * VH)
    close(xn, ln(x.float(), nw.float(), nb.float(), 1e-5), 'layer_norm (eps 1e-5)')
    close(qkv.reshape(-1, 3 * VH), xn.float().reshape(-1, VH) @ qw.float() + qb.float(), 'qkv')

    attn = A.AttnMultiKey(qkv, P, VHEADS, VHD, VH)
    assert attn.shape == (NV, P, VH) and attn.dtype == bf
    t = qkv.float().view(NV, P, 3, VHEADS, VHD).permute(2, 0, 3, 1, 4)
    ref = F.scaled_dot_product_attention(t[0], t[1], t[2]).transpose(1, 2).reshape(NV, P, VH)
    close(attn, ref, 'AttnMultiKey')

    ow, ob = rn(VH, VH, seed=10, scale=0.02), rn(VH, seed=11, scale=0.02)
    res = x.clone()
    ref = attn.float().reshape(-1, VH) @ ow.float() + ob.float() + res.float().reshape(-1, VH)
    A.matmul_bias_res(attn, ow, ob, res, res, None, P, VH)  # in place, as the reference calls it
    close(res.reshape(-1, VH), ref, 'matmul_bias_res')

    uw, ub = rn(VH, VI, seed=12, scale=0.02), rn(VI, seed=13, scale=0.02)
    h = torch.empty(NV, P, VI, dtype=bf, device=dev)
    A.layer_norm_matmul_bias_gelu(res, nw, nb, uw, ub, h, xn, P, VH, VI)
    close(h.reshape(-1, VI), gelu_tanh(xn.float().reshape(-1, VH) @ uw.float() + ub.float()),
          'layer_norm_matmul_bias_gelu')

    dw, db = rn(VI, VH, seed=14, scale=0.02), rn(VH, seed=15, scale=0.02)
    ref = h.float().reshape(-1, VI) @ dw.float() + db.float() + res.float().reshape(-1, VH)
    A.matmul_split_k_bias_res(h, dw, db, res, res, None, P, VI, VH)
    close(res.reshape(-1, VH), ref, 'matmul_split_k_bias_res')


def test_layer_norm_matmul_bias_projector():
    x = rn(NV, P, VH, seed=16)
    nw, nb = rn(VH, seed=17, scale=0.1), rn(VH, seed=18, scale=0.1)
    pw, pb = rn(VH, 2048, seed=19, scale=0.02), rn(2048, seed=20, scale=0.02)
    out = torch.empty(NV * P, 2048, dtype=bf, device=dev)
    xn = torch.empty(NV, P, VH, dtype=bf, device=dev)
    A.layer_norm_matmul_bias(x, nw, nb, pw, pb, out, xn, num_patches=P,
                             in_features=VH, out_features=2048, eps=1e-5)
    close(xn, ln(x.float(), nw.float(), nb.float(), 1e-5), 'layer_norm')
    close(out, xn.float().reshape(-1, VH) @ pw.float() + pb.float(), 'projector')


# ---------------------------------------------------------------------------
# Gemma prefix ops (E rows, width 2048, 8 q heads + 1 kv head of 256)
# ---------------------------------------------------------------------------
E, LH, LI, HD, NH = 200, 2048, 16384, 256, 8


def test_rms_matmul_qkv_rope_and_attention_v():
    x = rn(E, LH, seed=21)
    w = rn(LH, (NH + 2) * HD, seed=22, scale=0.02)
    rope = rope_table(E)
    Q = torch.empty(E * NH, HD, dtype=bf, device=dev)
    Kc = torch.zeros(2, E + 64, HD, dtype=bf, device=dev)
    Vc = torch.zeros(2, E + 64, HD, dtype=bf, device=dev)
    xn = torch.empty(E, LH, dtype=bf, device=dev)
    A.rms_matmul_qkv_rope(x, w, rope, Q, Kc[1, :E], Vc[1, :E], xn,
                          hidden_dim=LH, head_dim=HD, num_kv_heads=NH)
    close(xn, rms(x.float()), 'rms_norm')
    y = xn.float() @ w.float()
    cs = rope.float()
    qref = torch.cat([rope_interleaved(y[:, h * HD:(h + 1) * HD], cs) for h in range(NH)], 1)
    close(Q.view(E, NH * HD), qref, 'q')
    close(Kc[1, :E], rope_interleaved(y[:, NH * HD:(NH + 1) * HD], cs), 'k')
    close(Vc[1, :E], y[:, (NH + 1) * HD:], 'v')
    assert Kc[0].abs().max() == 0 and Kc[1, E:].abs().max() == 0  # nothing else written

    p = torch.softmax(rn(E * NH, E, seed=23).float(), -1).to(bf)
    ctx = torch.empty(E * NH, HD, dtype=bf, device=dev)
    A.matmul_attn_v(p, Vc[1, :E], ctx, head_dim=HD)
    close(ctx, p.float() @ Vc[1, :E].float(), 'matmul_attn_v')


def test_matmul_res_and_rms_gate():
    x = rn(E, LH, seed=24)
    a = rn(E, LH, seed=25)
    ow = rn(LH, LH, seed=26, scale=0.02)
    ref = x.float() + a.float() @ ow.float()
    A.matmul_res(a, ow, x, in_features=LH, out_features=LH)
    close(x, ref, 'matmul_res')

    gw, uw = rn(LH, 4096, seed=27, scale=0.02), rn(LH, 4096, seed=28, scale=0.02)
    h = torch.empty(E, 4096, dtype=bf, device=dev)
    xn = torch.empty(E, LH, dtype=bf, device=dev)
    A.rms_matmul_gate(x, gw, uw, h, xn, hidden_dim=LH, intermediate_dim=4096)
    close(xn, rms(x.float()), 'rms_norm')
    ref = gelu_tanh(xn.float() @ gw.float()) * (xn.float() @ uw.float())
    close(h, ref, 'rms_matmul_gate')


# ---------------------------------------------------------------------------
# action expert ops (S suffix rows, width 1024, PI0.5 adaRMS)
# ---------------------------------------------------------------------------
S, DH, DI = 50, 1024, 4096


def test_time_mlp_action_in_and_out():
    te = rn(1, DH, seed=30)
    w1, b1 = rn(DH, DH, seed=31, scale=0.02), rn(DH, seed=32, scale=0.02)
    xb = torch.zeros(S, DH, dtype=bf, device=dev)
    A.matmul_bias_silu(te, w1, b1, xb, in_features=DH, out_features=DH)
    ref = F.silu(te.float() @ w1.float() + b1.float())
    close(xb[:1], ref, 'matmul_bias_silu (one row)')
    assert xb[1:].abs().max() == 0

    noise = rn(S, 32, seed=33)
    aw, ab = rn(32, DH, seed=34, scale=0.02), rn(DH, seed=35, scale=0.02)
    x = torch.empty(S, DH, dtype=bf, device=dev)
    A.matmul_bias_small(noise, aw, ab, x, in_features=32, out_features=DH,
                        BLOCK_SIZE_N=32, BLOCK_SIZE_M=32, BLOCK_SIZE_K=32)
    close(x, noise.float() @ aw.float() + ab.float(), 'action_in_proj')

    ow, ob = rn(DH, 32, seed=36, scale=0.02), rn(32, seed=37, scale=0.02)
    act = torch.empty(S, 32, dtype=bf, device=dev)
    A.matmul_bias_small(x, ow, ob, act, in_features=DH, out_features=32,
                        BLOCK_SIZE_N=16, BLOCK_SIZE_M=16, BLOCK_SIZE_K=256)
    close(act, x.float() @ ow.float() + ob.float(), 'action_out_proj')


def test_expert_layer_ops():
    x = rn(S, DH, seed=40)
    temb = rn(S, DH, seed=41)
    mw, mb = rn(DH, 3 * DH, seed=42, scale=0.02), rn(3 * DH, seed=43, scale=0.02)
    xn = torch.empty(S, DH, dtype=bf, device=dev)
    gate = torch.empty(S, DH, dtype=bf, device=dev)
    style = torch.empty(S, 3 * DH, dtype=bf, device=dev)
    A.adarms_norm_style_proj(x, temb, mw, mb, xn, gate, style, hidden_dim=DH,
                             style_dim=3 * DH)
    st_ref = temb.float() @ mw.float() + mb.float()
    close(style, st_ref, 'style')
    st = style[0].float()
    sc, sh, gt = st[:DH], st[DH:2 * DH], st[2 * DH:]
    close(xn, rms(x.float()) * (1 + sc) + sh, 'adarms x_normed')
    assert torch.equal(gate, style[0, 2 * DH:].expand(S, DH))

    qkv_w = rn(DH, (NH + 2) * HD, seed=44, scale=0.02)
    rope = rope_table(S, start=815)
    q = torch.empty(S * NH, HD, dtype=bf, device=dev)
    Kc = torch.zeros(816 + S, HD, dtype=bf, device=dev)
    Vc = torch.zeros(816 + S, HD, dtype=bf, device=dev)
    A.matmul_qkv_rope(xn, qkv_w, rope, q, Kc[816:], Vc[816:], hidden_dim=DH,
                      head_dim=HD, num_kv_heads=NH)
    y = xn.float() @ qkv_w.float()
    cs = rope.float()
    qref = torch.cat([rope_interleaved(y[:, h * HD:(h + 1) * HD], cs) for h in range(NH)], 1)
    close(q.view(S, NH * HD), qref, 'expert q')
    close(Kc[816:], rope_interleaved(y[:, NH * HD:(NH + 1) * HD], cs), 'expert k')
    close(Vc[816:], y[:, (NH + 1) * HD:], 'expert v')

    ow = rn(NH * HD, DH, seed=45, scale=0.02)
    ref = x.float() + (q.view(S, -1).float() @ ow.float()) * gate.float()
    A.matmul_res_gate(q.view(-1, NH * HD), ow, x, gate, in_features=NH * HD,
                      out_features=DH, BLOCK_SIZE_N=32, BLOCK_SIZE_M=32, BLOCK_SIZE_K=128)
    close(x, ref, 'matmul_res_gate')

    gw, uw = rn(DH, DI, seed=46, scale=0.02), rn(DH, DI, seed=47, scale=0.02)
    h = torch.empty(S, DI, dtype=bf, device=dev)
    A.matmul_gate(xn, gw, uw, h, in_features=DH, intermediate_dim=DI)
    close(h, gelu_tanh(xn.float() @ gw.float()) * (xn.float() @ uw.float()), 'matmul_gate')


def test_weight_cache_follows_in_place_updates():
    a = rn(64, 256, seed=50)
    w = rn(256, 128, seed=51, scale=0.02)
    out = torch.zeros(64, 128, dtype=bf, device=dev)
    b = torch.zeros(128, dtype=bf, device=dev)
    A.matmul_bias_small(a, w, b, out, 256, 128)
    close(out, a.float() @ w.float(), 'first weights')
    w.copy_(rn(256, 128, seed=52, scale=0.02))  # bumps the version
    A.matmul_bias_small(a, w, b, out, 256, 128)
    close(out, a.float() @ w.float(), 'updated weights')


# ---------------------------------------------------------------------------
# the unfused attention trio that pi05_flowmatching_inference.py launches
# directly (attention_triton_ops.py:5,81,111), with the Triton launch syntax
# ---------------------------------------------------------------------------
from fluxvla_b200 import attention_triton_ops as T  # noqa: E402


def masked_softmax_ref(lg, n_prefix, valid):
    keys = lg.shape[1]
    j = torch.arange(keys, device=dev)
    ok = (j >= n_prefix) | (j < min(max(valid, 0), n_prefix))
    return torch.softmax(torch.where(ok[None], lg, torch.full_like(lg, -2.3819763e38)), -1)


@pytest.mark.parametrize('valid', [E, 150, 0])
def test_prefix_attention_trio(valid):
    Q = rn(E * NH, HD, seed=60)
    Kc = rn(E, HD, seed=61)
    Vc = rn(E, HD, seed=62)
    logits = torch.zeros(E * NH, E, device=dev)
    probs = torch.zeros(E * NH, E, dtype=bf, device=dev)
    vlen = torch.tensor([valid], dtype=torch.int32, device=dev)
    T.matmul_abT_scale[(999,)](Q, Kc, logits, E * NH, E, HD, 1.0 / 16,
                               BLOCK_SIZE_M=32, BLOCK_SIZE_N=32, BLOCK_SIZE_K=64)
    lref = Q.float() @ Kc.float().t() / 16
    close(logits, lref, 'matmul_abT_scale')
    T.softmax_kernel_masklen[(1,)](logits, E * NH, E, vlen, probs, BLOCK_SIZE_M=4,
                                   BLOCK_SIZE=1024)
    close(probs, masked_softmax_ref(logits, E, valid), 'softmax_kernel_masklen')
    ctx = torch.empty(E * NH, HD, dtype=bf, device=dev)
    A.matmul_attn_v(probs, Vc, ctx, head_dim=HD)
    close(ctx, probs.float() @ Vc.float(), 'P.V')


def test_suffix_attention_trio():
    pre = 816
    Q = rn(S * NH, HD, seed=63)
    Kc = rn(pre + S, HD, seed=64)
    logits = torch.zeros(S * NH, pre + S, device=dev)
    probs = torch.zeros(S * NH, pre + S, dtype=bf, device=dev)
    vlen = torch.tensor([700], dtype=torch.int32, device=dev)
    T.matmul_abT_scale[(1,)](Q, Kc, logits, S * NH, pre + S, HD, 256 ** -0.5)
    close(logits, Q.float() @ Kc.float().t() / 16, 'matmul_abT_scale (ragged N)')
    T.softmax_kernel_prefix_suffix[(1,)](logits, S * NH, pre, S, vlen, probs)
    p = probs.float()
    close(p, masked_softmax_ref(logits, pre, 700), 'softmax_kernel_prefix_suffix')
    assert p[:, 700:pre].abs().max() == 0 and p[:, pre:].min() > 0
