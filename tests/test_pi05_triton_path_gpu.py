"""The reference's PI0.5 Triton pipeline run end to end on this library's
drop-ins: the call sequence of ``pi05_model``
(fluxvla/models/vlas/pi05_flowmatching_inference.py:22-312 — vision_encoder,
transformer_encoder, transformer_decoder), restated here step for step with
the reference's own operator names imported from
``fluxvla_b200.atomic_ops`` / ``fluxvla_b200.attention_triton_ops``, on
weights packed as the reference's ``prepare_triton()`` methods pack them
(siglip_vit_inference.py:10-100, condition_gemma_inference.py:46-170,
linear_projector_inference.py:8, pi05_flowmatching_inference.py:550-620)
and buffers laid out as its ``_init_buffers`` (:356-440).  The actions are
compared with the fp32 eager oracle.

Two documented reference discrepancies are resolved toward the eager model,
as the rest of this library does: the decoder's rotary rows start at the
eager suffix position (prefix length + i, pi0_flowmatching.py:817-819)
rather than the Triton path's one-off start (:458-461); everything else —
bf16 residual streams, bf16 x_t accumulation (pi05_flowmatching_inference.py:
310), LayerNorm eps 1e-5 — follows the Triton path.  Tolerances: (1) as the
reference design runs it, the north star's relative L2 1e-2 and a max-abs
within the rounding the bf16 x_t buffer itself adds, one bf16 unit in the
last place of the largest action per Euler step (steps * 2^-8 * max|x|);
(2) with only the Euler accumulation of x_t moved to f32, the north star's
max-abs 2e-2 and relative L2 1e-2 — the drop-ins add no error beyond it.
"""
import math

import pytest
import torch

from fluxvla_b200.atomic_ops import (AttnMultiKey, adarms_norm_style_proj,
                                     conv2d_embed_res, layer_norm_matmul_bias,
                                     layer_norm_matmul_bias_gelu,
                                     layer_norm_QKV_matmul_bias, matmul_attn_v,
                                     matmul_bias_res, matmul_bias_silu,
                                     matmul_bias_small, matmul_gate,
                                     matmul_qkv_rope, matmul_res,
                                     matmul_res_gate, matmul_split_k_bias_res,
                                     rms_matmul_gate, rms_matmul_qkv_rope)
from fluxvla_b200.attention_triton_ops import (matmul_abT_scale,
                                               softmax_kernel_masklen,
                                               softmax_kernel_prefix_suffix)
from fluxvla_b200.config import pi05_config
from fluxvla_b200.weights import make_weights
from oracle import pi0_oracle as O

pytestmark = pytest.mark.gpu
dev = 'cuda'
bf = torch.bfloat16


# ---------------------------------------------------------------------------
# weight packing of the reference's prepare_triton() methods
# ---------------------------------------------------------------------------
def _rope_format(w_q, w_k, hd, nq):
    """condition_gemma_inference.py:46-63: rotate-half partners adjacent."""
    k_in = w_q.shape[1]
    w_q = w_q.view(nq, 2, hd // 2, k_in).permute(0, 2, 1, 3).reshape(nq * hd, k_in)
    w_k = w_k.view(2, hd // 2, k_in).permute(1, 0, 2).reshape(hd, k_in)
    return w_q, w_k


def triton_weights(cfg, W, num_steps):
    f = {k: v.float().to(dev) for k, v in W.items()}
    out = {}

    def put(k, t):
        out[k] = t.contiguous().to(bf)

    # SigLIP (siglip_vit_inference.py:10-100)
    put('vision_patch_embedding_w',
        f['vision.patch_w'].permute(2, 3, 1, 0).reshape(-1, cfg.vis_width))
    put('vision_patch_embedding_b', f['vision.patch_b'])
    put('vision_position_embedding', f['vision.pos'])
    L = range(cfg.vis_layers)
    st = lambda fn: torch.stack([fn(f'vision.l{i}.') for i in L])  # noqa: E731
    put('vision_attn_qkv_w', st(lambda p: torch.cat([f[p + 'q_w'].t(), f[p + 'k_w'].t(),
                                                     f[p + 'v_w'].t()], 1)))
    put('vision_attn_qkv_b', st(lambda p: torch.cat([f[p + 'q_b'], f[p + 'k_b'], f[p + 'v_b']])))
    put('vision_attn_o_w', st(lambda p: f[p + 'o_w'].t()))
    put('vision_attn_o_b', st(lambda p: f[p + 'o_b']))
    put('vision_ffn_up_w', st(lambda p: f[p + 'fc1_w'].t()))
    put('vision_ffn_up_b', st(lambda p: f[p + 'fc1_b']))
    put('vision_ffn_down_w', st(lambda p: f[p + 'fc2_w'].t()))
    put('vision_ffn_down_b', st(lambda p: f[p + 'fc2_b']))
    put('vision_pre_attn_norm_w', st(lambda p: f[p + 'ln1_w']))
    put('vision_pre_attn_norm_b', st(lambda p: f[p + 'ln1_b']))
    put('vision_pre_ffn_norm_w', st(lambda p: f[p + 'ln2_w']))
    put('vision_pre_ffn_norm_b', st(lambda p: f[p + 'ln2_b']))
    put('vision_final_norm_w', f['vision.post_w'])
    put('vision_final_norm_b', f['vision.post_b'])
    # projector (linear_projector_inference.py:8)
    put('encoder_multi_modal_projector_w', f['proj_w'].t())
    put('encoder_multi_modal_projector_b', f['proj_b'])
    # Gemma prefix, role='llm' (condition_gemma_inference.py:68-111)
    hd, H = cfg.head_dim, cfg.heads
    qkv, o_w, g_w, u_w, d_w = [], [], [], [], []
    for i in range(cfg.llm_layers):
        p = f'llm.l{i}.'
        s = (1 + f[p + 'in_norm'])[None]
        q, k = _rope_format(f[p + 'q_w'] * s, f[p + 'k_w'] * s, hd, H)
        qkv.append(torch.cat([q.t(), k.t(), (f[p + 'v_w'] * s).t()], 1))
        o_w.append(f[p + 'o_w'].t())
        s2 = (1 + f[p + 'post_norm'])[None]
        g_w.append((f[p + 'gate_w'] * s2).t())
        u_w.append((f[p + 'up_w'] * s2).t())
        d_w.append(f[p + 'down_w'].t())
    for k, v in [('qkv', qkv), ('o', o_w), ('gate', g_w), ('up', u_w), ('down', d_w)]:
        put({'qkv': 'encoder_attn_qkv_w', 'o': 'encoder_attn_o_w',
             'gate': 'encoder_ffn_gate_w', 'up': 'encoder_ffn_up_w',
             'down': 'encoder_ffn_down_w'}[k], torch.stack(v))
    # action expert, role='expert' (condition_gemma_inference.py:113-170)
    qkv, o_w, g_w, u_w, d_w, am, ab, fm, fb = ([] for _ in range(9))
    for i in range(cfg.exp_layers):
        p = f'exp.l{i}.'
        q, k = _rope_format(f[p + 'q_w'], f[p + 'k_w'], hd, H)
        qkv.append(torch.cat([q.t(), k.t(), f[p + 'v_w'].t()], 1))
        o_w.append(f[p + 'o_w'].t())
        g_w.append(f[p + 'gate_w'].t())
        u_w.append(f[p + 'up_w'].t())
        d_w.append(f[p + 'down_w'].t())
        am.append(f[p + 'in_norm_dense_w'].t())
        ab.append(f[p + 'in_norm_dense_b'])
        fm.append(f[p + 'post_norm_dense_w'].t())
        fb.append(f[p + 'post_norm_dense_b'])
    for k, v in [('decoder_attn_qkv_w', qkv), ('decoder_attn_o_w', o_w),
                 ('decoder_ffn_gate_w', g_w), ('decoder_ffn_up_w', u_w),
                 ('decoder_ffn_down_w', d_w), ('decoder_pre_attn_norm_mod_w', am),
                 ('decoder_pre_attn_norm_mod_b', ab), ('decoder_pre_ffn_norm_mod_w', fm),
                 ('decoder_pre_ffn_norm_mod_b', fb)]:
        put(k, torch.stack(v))
    put('decoder_final_norm_mod_w', f['exp.norm_dense_w'].t())
    put('decoder_final_norm_mod_b', f['exp.norm_dense_b'])
    # action / time projections (pi05_flowmatching_inference.py:550-560)
    for ours, theirs in [('action_in', 'decoder_action_in_proj'),
                         ('action_out', 'decoder_action_out_proj'),
                         ('time_in', 'decoder_time_mlp_in'),
                         ('time_out', 'decoder_time_mlp_out')]:
        put(theirs + '_w', f[ours + '_w'].t())
        put(theirs + '_b', f[ours + '_b'])
    # _prepare_adarms_cond (:527-548): sin | cos of t*2pi/period, bf16
    frac = torch.linspace(0.0, 1.0, cfg.exp_width // 2, device=dev)
    period = 4e-3 * (4.0 / 4e-3) ** frac
    t = torch.tensor(1.0, device=dev)
    embs = []
    for _ in range(num_steps):
        x = t[None, None] * (1.0 / period)[None] * 2 * math.pi
        embs.append(torch.cat([torch.sin(x), torch.cos(x)], -1).to(bf))
        t = t + (-1.0 / num_steps)
    out['decoder_time_embeds'] = torch.cat(embs, 0)
    return out


# ---------------------------------------------------------------------------
# pi05_model (pi05_flowmatching_inference.py:22-312), restated
# ---------------------------------------------------------------------------
def vision_encoder(w, b, num_views, num_vit_layers):
    num_patches, vit_hidden, vit_intermediate = 256, 1152, 4304
    conv2d_embed_res(b['observation_images_normalized'], w['vision_patch_embedding_w'],
                     w['vision_patch_embedding_b'], w['vision_position_embedding'],
                     b['vision_x'], 16, 14, num_patches, vit_hidden)
    for i in range(num_vit_layers):
        layer_norm_QKV_matmul_bias(b['vision_x'], w['vision_pre_attn_norm_w'][i],
                                   w['vision_pre_attn_norm_b'][i], w['vision_attn_qkv_w'][i],
                                   w['vision_attn_qkv_b'][i], b['vision_QKV'],
                                   b['vision_x_norm'], num_patches, vit_hidden, 3 * vit_hidden)
        attn = AttnMultiKey(b['vision_QKV'], num_patches, 16, 72, vit_hidden)
        matmul_bias_res(attn, w['vision_attn_o_w'][i], w['vision_attn_o_b'][i], b['vision_x'],
                        b['vision_x'], None, num_patches, vit_hidden)
        layer_norm_matmul_bias_gelu(b['vision_x'], w['vision_pre_ffn_norm_w'][i],
                                    w['vision_pre_ffn_norm_b'][i], w['vision_ffn_up_w'][i],
                                    w['vision_ffn_up_b'][i], b['vision_hidden'],
                                    b['vision_x_norm'], num_patches, vit_hidden,
                                    vit_intermediate)
        matmul_split_k_bias_res(b['vision_hidden'], w['vision_ffn_down_w'][i],
                                w['vision_ffn_down_b'][i], b['vision_x'], b['vision_x'], None,
                                num_patches, vit_intermediate, vit_hidden)


def transformer_encoder(w, b, enc, num_encoder_layers):
    layer_norm_matmul_bias(b['vision_x'], w['vision_final_norm_w'], w['vision_final_norm_b'],
                           w['encoder_multi_modal_projector_w'],
                           w['encoder_multi_modal_projector_b'], b['encoder_x'],
                           b['vision_x_norm'], num_patches=256, in_features=1152,
                           out_features=2048, eps=1e-5)
    for i in range(num_encoder_layers):
        rms_matmul_qkv_rope(b['encoder_x'], w['encoder_attn_qkv_w'][i],
                            b['encoder_rope_weights'], b['encoder_Q'],
                            b['encoder_K'][i, :enc], b['encoder_V'][i, :enc],
                            b['encoder_x_norm'], hidden_dim=2048, head_dim=256,
                            num_kv_heads=8)
        if i != num_encoder_layers - 1:
            tq = b['encoder_Q'].shape[0]
            matmul_abT_scale[(1,)](b['encoder_Q'], b['encoder_K'][i, :enc],
                                   b['encoder_logits_buf'], tq, enc, 256, 1.0 / 16,
                                   BLOCK_SIZE_M=32, BLOCK_SIZE_N=32, BLOCK_SIZE_K=64)
            softmax_kernel_masklen[(1,)](b['encoder_logits_buf'], tq, enc,
                                         b['valid_encoder_len'], b['encoder_attn_buf'],
                                         BLOCK_SIZE_M=4, BLOCK_SIZE=1024)
            matmul_attn_v(b['encoder_attn_buf'], b['encoder_V'][i, :enc],
                          b['encoder_ctx_buf'], head_dim=256)
            matmul_res(b['encoder_ctx_buf'].view(-1, 2048), w['encoder_attn_o_w'][i],
                       b['encoder_x'], in_features=2048, out_features=2048)
            rms_matmul_gate(b['encoder_x'], w['encoder_ffn_gate_w'][i],
                            w['encoder_ffn_up_w'][i], b['encoder_hidden'],
                            b['encoder_x_norm'], hidden_dim=2048, intermediate_dim=16384)
            matmul_res(b['encoder_hidden'], w['encoder_ffn_down_w'][i], b['encoder_x'],
                       in_features=16384, out_features=2048)


def transformer_decoder(w, b, enc, num_decoder_layers, num_steps,
                        xt_f32=False):
    """xt_f32: keep the Euler accumulation of x_t in an f32 copy (the
    projections still read the bf16 buffer) instead of the reference
    design's bf16 ``add_`` (:310); isolates the drop-ins' own error."""
    xt = b['diffusion_noise'].float() if xt_f32 else None
    for step in range(num_steps):
        matmul_bias_silu(w['decoder_time_embeds'][step].view(1, -1),
                         w['decoder_time_mlp_in_w'], w['decoder_time_mlp_in_b'],
                         b['decoder_x_buf'], in_features=1024, out_features=1024)
        matmul_bias_silu(b['decoder_x_buf'], w['decoder_time_mlp_out_w'],
                         w['decoder_time_mlp_out_b'], b['decoder_time_emb'],
                         in_features=1024, out_features=1024)
        matmul_bias_small(b['diffusion_noise'], w['decoder_action_in_proj_w'],
                          w['decoder_action_in_proj_b'], b['decoder_x'], in_features=32,
                          out_features=1024, BLOCK_SIZE_N=32, BLOCK_SIZE_M=32,
                          BLOCK_SIZE_K=32)
        seq = b['decoder_x'].shape[0]
        for i in range(num_decoder_layers):
            adarms_norm_style_proj(b['decoder_x'], b['decoder_time_emb'],
                                   w['decoder_pre_attn_norm_mod_w'][i],
                                   w['decoder_pre_attn_norm_mod_b'][i], b['x_normed_buf'],
                                   b['gate_buf'], b['decoder_style'], hidden_dim=1024,
                                   style_dim=3072)
            matmul_qkv_rope(b['x_normed_buf'], w['decoder_attn_qkv_w'][i],
                            b['decoder_rope_weights'], b['decoder_q_buf'],
                            b['encoder_K'][i, enc:enc + seq], b['encoder_V'][i, enc:enc + seq],
                            hidden_dim=1024, head_dim=256, num_kv_heads=8)
            tq = b['decoder_q_buf'].shape[0]
            matmul_abT_scale[(1,)](b['decoder_q_buf'], b['encoder_K'][i, :enc + seq],
                                   b['decoder_logits_buf'], tq, enc + seq, 256, 256 ** -0.5,
                                   BLOCK_SIZE_M=32, BLOCK_SIZE_N=32, BLOCK_SIZE_K=64)
            softmax_kernel_prefix_suffix[(1,)](b['decoder_logits_buf'], tq, enc, seq,
                                               b['valid_encoder_len'], b['decoder_attn_buf'],
                                               BLOCK_SIZE_M=4, BLOCK_SIZE=1024)
            matmul_attn_v(b['decoder_attn_buf'], b['encoder_V'][i, :enc + seq],
                          b['decoder_q_buf'], head_dim=256)
            matmul_res_gate(b['decoder_q_buf'].view(-1, 2048), w['decoder_attn_o_w'][i],
                            b['decoder_x'], b['gate_buf'], in_features=2048,
                            out_features=1024, BLOCK_SIZE_N=32, BLOCK_SIZE_M=32,
                            BLOCK_SIZE_K=128)
            adarms_norm_style_proj(b['decoder_x'], b['decoder_time_emb'],
                                   w['decoder_pre_ffn_norm_mod_w'][i],
                                   w['decoder_pre_ffn_norm_mod_b'][i], b['x_normed_buf'],
                                   b['gate_buf'], b['decoder_style'], hidden_dim=1024,
                                   style_dim=3072)
            matmul_gate(b['x_normed_buf'], w['decoder_ffn_gate_w'][i], w['decoder_ffn_up_w'][i],
                        b['decoder_hidden'], in_features=1024, intermediate_dim=4096)
            matmul_res_gate(b['decoder_hidden'], w['decoder_ffn_down_w'][i], b['decoder_x'],
                            b['gate_buf'], in_features=4096, out_features=1024,
                            BLOCK_SIZE_N=16, BLOCK_SIZE_M=32, BLOCK_SIZE_K=256)
        adarms_norm_style_proj(b['decoder_x'], b['decoder_time_emb'],
                               w['decoder_final_norm_mod_w'], w['decoder_final_norm_mod_b'],
                               b['x_normed_buf'], b['gate_buf'], b['decoder_style'],
                               hidden_dim=1024, style_dim=3072)
        matmul_bias_small(b['x_normed_buf'], w['decoder_action_out_proj_w'],
                          w['decoder_action_out_proj_b'], b['decoder_action_buf'],
                          in_features=1024, out_features=32, BLOCK_SIZE_N=16,
                          BLOCK_SIZE_M=16, BLOCK_SIZE_K=256)
        if xt_f32:
            xt += b['decoder_action_buf'].float() * (-1.0 / num_steps)
            b['diffusion_noise'].copy_(xt)
        else:
            b['diffusion_noise'].add_(b['decoder_action_buf'], alpha=-1.0 / num_steps)
    return xt


def buffers(nv, enc, dec, layers):
    """_init_buffers, pi05_flowmatching_inference.py:356-440."""
    z = lambda *s, dt=bf: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
    return {
        'observation_images_normalized': z(nv, 224, 224, 3),
        'vision_x': z(nv, 256, 1152), 'vision_x_norm': z(nv, 256, 1152),
        'vision_QKV': z(nv, 256, 3456), 'vision_hidden': z(nv, 256, 4304),
        'encoder_rope_weights': z(enc, 256), 'encoder_x': z(enc, 2048),
        'encoder_x_norm': z(enc, 2048), 'encoder_K': z(layers, enc + dec, 256),
        'encoder_V': z(layers, enc + dec, 256), 'encoder_Q': z(enc * 8, 256),
        'encoder_hidden': z(enc, 16384),
        'valid_encoder_len': z(1, dt=torch.int32),
        'encoder_logits_buf': z(enc * 8, enc, dt=torch.float32),
        'encoder_attn_buf': z(enc * 8, enc), 'encoder_ctx_buf': z(enc * 8, 256),
        'decoder_rope_weights': z(dec, 256), 'decoder_x': z(dec, 1024),
        'decoder_x_buf': z(dec, 1024), 'decoder_action_buf': z(dec, 32),
        'decoder_time_emb': z(dec, 1024), 'decoder_style': z(dec, 3072),
        'decoder_q_buf': z(dec * 8, 256),
        'decoder_logits_buf': z(dec * 8, enc + dec, dt=torch.float32),
        'decoder_attn_buf': z(dec * 8, enc + dec), 'decoder_hidden': z(dec, 4096),
        'x_normed_buf': z(dec, 1024), 'gate_buf': z(dec, 1024),
        'diffusion_noise': z(dec, 32)}


def rope_rows(positions):
    """_init_rope_table (:444-456): bf16 (cos, sin) pairs per position."""
    inv = 1.0 / (10000 ** (torch.arange(0, 256, 2, dtype=torch.float32, device=dev) / 256))
    ph = inv[None, :] * positions[:, None].to(dev).float()
    return torch.cat([torch.cos(ph).to(bf)[:, :, None], torch.sin(ph).to(bf)[:, :, None]],
                     2).view(-1, 256)


def test_pi05_model_on_drop_in_ops():
    cfg = pi05_config(vis_layers=2, llm_layers=2, exp_layers=2, vocab=4096)
    n_tok, steps = 80, cfg.num_steps
    W = make_weights(cfg, 11)
    g = torch.Generator().manual_seed(12)
    imgs = torch.randint(0, 256, (cfg.n_views, 224, 224, 3), generator=g, dtype=torch.uint8)
    toks = torch.randint(0, cfg.vocab, (1, n_tok), generator=g)
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g).bfloat16().float()

    nv, dec = cfg.n_views, cfg.n_actions
    enc = nv * 256 + n_tok
    w = triton_weights(cfg, W, steps)
    b = buffers(nv, enc, dec, max(cfg.llm_layers, cfg.exp_layers))
    pix = O.normalize_images(imgs, [cfg.img_mean] * nv, [cfg.img_std] * nv)
    b['observation_images_normalized'].copy_(pix.permute(0, 2, 3, 1))
    emb = W['llm.embed'].float()[toks[0]] * math.sqrt(2048)
    b['encoder_x'][nv * 256:].copy_(emb)
    b['valid_encoder_len'].fill_(enc)
    b['encoder_rope_weights'].copy_(rope_rows(torch.arange(enc)))
    b['decoder_rope_weights'].copy_(rope_rows(torch.arange(enc, enc + dec)))
    b['diffusion_noise'].copy_(noise[0])

    vision_encoder(w, b, nv, cfg.vis_layers)
    transformer_encoder(w, b, enc, cfg.llm_layers)
    transformer_decoder(w, b, enc, cfg.exp_layers, steps)
    torch.cuda.synchronize()

    out = b['diffusion_noise'].float().cpu()
    # (1) against the fp32 eager oracle: the north star's relative L2, and a
    # max-abs bound of one bf16 ulp of the largest action per Euler step
    # (the reference design keeps x_t in bf16)
    ref = O.predict_action(cfg, W, imgs, toks, state, noise)[0]
    err = (out - ref).abs().max().item()
    rel = ((out - ref).norm() / ref.norm()).item()
    bound = steps * 2.0 ** -8 * ref.abs().max().item()
    assert rel <= 1e-2 and err <= bound, f'max-abs {err:.3e} (bound {bound:.3e}) rel-l2 {rel:.3e}'
    # (2) the same pipeline with x_t accumulated in f32: the drop-ins' own
    # error is within the north star (max-abs 2e-2, relative L2 1e-2)
    b['diffusion_noise'].copy_(noise[0])
    out32 = transformer_decoder(w, b, enc, cfg.exp_layers, steps,
                                xt_f32=True).cpu()
    torch.cuda.synchronize()
    err32 = (out32 - ref).abs().max().item()
    rel32 = ((out32 - ref).norm() / ref.norm()).item()
    assert err32 <= 2e-2 and rel32 <= 1e-2, f'max-abs {err32:.3e} rel-l2 {rel32:.3e}'


