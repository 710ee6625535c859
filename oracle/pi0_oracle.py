"""CPU fp32 restatement of FluxVLA's PI0 / PI0.5 eager inference path.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
path in ``fluxvla_b200``.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it; the
product path never does.

Every function restates the reference algorithm in plain torch fp32 on the CPU
and cites the reference file:line it follows (paths relative to the FluxVLA
project root).  The restatement is pinned against outputs of the reference's
own modules (imported through a small shim by ``tests/golden/make_golden.py``)
on seeded random weights: see ``tests/test_oracle_golden.py``.

Weights are passed as a flat ``dict[str, Tensor]`` (names documented in
``fluxvla_b200/weights.py``); tensors may be bf16, they are upcast per use.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch

Tensor = torch.Tensor
F32 = torch.float32


def _w(W: Dict[str, Tensor], name: str) -> Tensor:
    return W[name].to(F32)


def linear(x: Tensor, w: Tensor, b: Optional[Tensor] = None) -> Tensor:
    """nn.Linear: x @ w.T + b (fluxvla/models/projectors/linear_projector.py:37-52)."""
    y = x @ w.to(F32).t()
    if b is not None:
        y = y + b.to(F32)
    return y


def gelu_tanh(x: Tensor) -> Tensor:
    """ACT2FN['gelu_pytorch_tanh'] (condition_gemma.py:170, GemmaMLP.act_fn)."""
    return torch.nn.functional.gelu(x, approximate='tanh')


# ---------------------------------------------------------------------------
# Norms
# ---------------------------------------------------------------------------

def gemma_rms_norm(x: Tensor, w: Tensor, eps: float = 1e-6) -> Tensor:
    """GemmaRMSNorm plain branch: x*rsqrt(mean(x^2)+eps)*(1+w).

    fluxvla/models/backbones/llms/condition_gemma.py:75-116.
    """
    var = torch.mean(x * x, dim=-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * (1.0 + w.to(F32))


def gemma_ada_rms_norm(x: Tensor, cond: Tensor, dense_w: Tensor,
                       dense_b: Tensor, eps: float = 1e-6
                       ) -> Tuple[Tensor, Tensor]:
    """GemmaRMSNorm adaptive branch: modulation = dense(cond) split into
    (scale, shift, gate); out = norm(x)*(1+scale)+shift.

    fluxvla/models/backbones/llms/condition_gemma.py:118-147.
    ``cond`` is [B, cond_dim]; returns (normed [B,S,D], gate [B,1,D]).
    """
    var = torch.mean(x * x, dim=-1, keepdim=True)
    normed = x * torch.rsqrt(var + eps)
    mod = linear(cond, dense_w, dense_b)
    if mod.dim() == 2 and x.dim() == 3:
        mod = mod.unsqueeze(1)
    scale, shift, gate = torch.chunk(mod, 3, dim=-1)
    return normed * (1 + scale) + shift, gate


def layer_norm(x: Tensor, w: Tensor, b: Tensor, eps: float = 1e-6) -> Tensor:
    """nn.LayerNorm as used by HF SiglipEncoderLayer / post_layernorm
    (eps = vision_config.layer_norm_eps = 1e-6,
    configs/pi0/pi0_paligemma_libero_10_full_finetune.py:52)."""
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w.to(F32),
                                          b.to(F32), eps)


# ---------------------------------------------------------------------------
# RoPE (rotate-half), attention
# ---------------------------------------------------------------------------

def rope_cos_sin(pos: Tensor, head_dim: int, theta: float = 10000.0
                 ) -> Tuple[Tensor, Tensor]:
    """GemmaRotaryEmbedding default rope: inv_freq = theta^(-2i/d);
    emb = cat(freqs, freqs).

    fluxvla/models/backbones/llms/condition_gemma.py:207-260.
    ``pos`` is [B, S] (int); returns cos, sin [B, S, head_dim] fp32.
    """
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2,
                                             dtype=torch.int64).to(F32)
                                / head_dim))
    freqs = pos.to(F32)[..., None] * inv_freq
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: Tensor) -> Tensor:
    """condition_gemma.py:263-267."""
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """apply_rotary_pos_emb, condition_gemma.py:270-299 (x: [B,H,S,D],
    cos/sin: [B,S,D])."""
    return x * cos[:, None] + rotate_half(x) * sin[:, None]


def attention(q: Tensor, k: Tensor, v: Tensor, add_mask: Optional[Tensor],
              scale: float) -> Tensor:
    """eager_attention_forward, condition_gemma.py:340-365 (GQA via
    repeat_kv :302-317).  q [B,H,S,D]; k,v [B,Hkv,T,D]; add_mask [B,1,S,T]
    additive.  Returns [B,S,H*D]."""
    rep = q.shape[1] // k.shape[1]
    if rep > 1:
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    a = (q @ k.transpose(2, 3)) * scale
    if add_mask is not None:
        a = a + add_mask[..., :k.shape[2]]
    a = torch.softmax(a, dim=-1)
    o = a @ v
    return o.transpose(1, 2).reshape(q.shape[0], q.shape[2], -1)


def additive_mask(bool_mask: Tensor) -> Tensor:
    """_prepare_attention_masks_4d, pi0_flowmatching.py:522-527: 0 where
    allowed, finfo(bfloat16).min elsewhere; [B,S,T] -> [B,1,S,T]."""
    m = torch.zeros(bool_mask.shape, dtype=F32)
    m.masked_fill_(~bool_mask, torch.finfo(torch.bfloat16).min)
    return m[:, None]


def make_att_2d_masks(pad_masks: Tensor, att_masks: Tensor) -> Tensor:
    """fluxvla/engines/utils/model_utils.py:77-95."""
    cs = torch.cumsum(att_masks.to(torch.int64), dim=1)
    att_2d = cs[:, None, :] <= cs[:, :, None]
    pad_2d = pad_masks[:, None, :] & pad_masks[:, :, None]
    return att_2d & pad_2d


def sinusoidal_time(t: Tensor, dim: int, min_period: float = 4e-3,
                    max_period: float = 4.0) -> Tensor:
    """create_sinusoidal_pos_embedding, model_utils.py:40-68."""
    fraction = torch.linspace(0.0, 1.0, dim // 2, dtype=F32)
    period = min_period * (max_period / min_period) ** fraction
    scaling = 1.0 / period * 2 * math.pi
    x = t.to(F32)[..., None] * scaling
    return torch.cat([torch.sin(x), torch.cos(x)], dim=-1)


# ---------------------------------------------------------------------------
# Gemma decoder (ConditionGemmaModel)
# ---------------------------------------------------------------------------

def gemma_layer(x: Tensor, W: Dict[str, Tensor], p: str, cos: Tensor,
                sin: Tensor, add_mask: Optional[Tensor], num_heads: int,
                num_kv_heads: int, head_dim: int,
                past_kv: Optional[Tuple[Tensor, Tensor]] = None,
                adarms_cond: Optional[Tensor] = None,
                eps: float = 1e-6) -> Tuple[Tensor, Tuple[Tensor, Tensor]]:
    """GemmaDecoderLayer.forward, condition_gemma.py:600-662, with
    GemmaAttention.forward :488-535 (prefix cache concat :500-515) and
    GemmaMLP.forward :177-192.  Returns (x_out, (k, v)) where k, v are this
    layer's own (post-RoPE) keys/values [B,Hkv,S,D] (what
    ``DynamicCache.update`` stores when use_cache=True)."""
    B, S, _ = x.shape
    ada = adarms_cond is not None
    res = x
    if ada:
        h, gate = gemma_ada_rms_norm(x, adarms_cond, W[p + 'in_norm_dense_w'],
                                     W[p + 'in_norm_dense_b'], eps)
    else:
        h, gate = gemma_rms_norm(x, W[p + 'in_norm'], eps), None
    q = linear(h, W[p + 'q_w']).view(B, S, num_heads, head_dim).transpose(1, 2)
    k = linear(h, W[p + 'k_w']).view(B, S, num_kv_heads,
                                     head_dim).transpose(1, 2)
    v = linear(h, W[p + 'v_w']).view(B, S, num_kv_heads,
                                     head_dim).transpose(1, 2)
    q = apply_rope(q, cos, sin)
    k = apply_rope(k, cos, sin)
    own = (k, v)
    if past_kv is not None:
        k = torch.cat([past_kv[0].to(F32), k], dim=2)
        v = torch.cat([past_kv[1].to(F32), v], dim=2)
    o = attention(q, k, v, add_mask, head_dim ** -0.5)
    o = linear(o, W[p + 'o_w'])
    x = res + (o if gate is None else o * gate)
    res = x
    if ada:
        h, gate = gemma_ada_rms_norm(x, adarms_cond,
                                     W[p + 'post_norm_dense_w'],
                                     W[p + 'post_norm_dense_b'], eps)
    else:
        h, gate = gemma_rms_norm(x, W[p + 'post_norm'], eps), None
    m = linear(gelu_tanh(linear(h, W[p + 'gate_w'])) * linear(h, W[p + 'up_w']),
               W[p + 'down_w'])
    x = res + (m if gate is None else m * gate)
    return x, own


def gemma_model(x: Tensor, W: Dict[str, Tensor], p: str, n_layers: int,
                pos: Tensor, add_mask: Optional[Tensor], num_heads: int,
                num_kv_heads: int, head_dim: int,
                past_kv: Optional[List[Tuple[Tensor, Tensor]]] = None,
                adarms_cond: Optional[Tensor] = None, final_norm: bool = True
                ) -> Tuple[Tensor, List[Tuple[Tensor, Tensor]]]:
    """ConditionGemmaModel.forward, condition_gemma.py:833-994 (no
    embedding scaling inside; final norm :983, adaptive when use_adarms)."""
    cos, sin = rope_cos_sin(pos, head_dim)
    kv = []
    for i in range(n_layers):
        x, own = gemma_layer(x, W, f'{p}l{i}.', cos, sin, add_mask, num_heads,
                             num_kv_heads, head_dim,
                             None if past_kv is None else past_kv[i],
                             adarms_cond)
        kv.append(own)
    if final_norm:
        if adarms_cond is not None:
            x, _ = gemma_ada_rms_norm(x, adarms_cond, W[p + 'norm_dense_w'],
                                      W[p + 'norm_dense_b'])
        else:
            x = gemma_rms_norm(x, W[p + 'norm'])
    return x, kv


# ---------------------------------------------------------------------------
# SigLIP vision tower (HF SiglipVisionModel, vision_use_head=False)
# ---------------------------------------------------------------------------

def _resize_taps(dst: int, src: int, clamp_weights: bool):
    """Source taps and 11-bit fixed-point weights of one axis of OpenCV's
    INTER_LINEAR resize (the `cv2.resize` that ResizeImages calls,
    fluxvla/transforms/transform_images.py:103-106): f = (d+0.5)*scale-0.5
    with scale = 1/(dst/src) in float64, rounded to float32, s = floor(f), weights round((1-f')*2048), round(f'*2048)
    (half to even).  Along x a tap left of 0 or at/after the last column is
    clamped with its fraction set to 0; along y the fraction is kept and only
    the row indices are clamped."""
    import numpy as np
    d = np.arange(dst, dtype=np.float64)
    scale = 1.0 / (dst / src)  # OpenCV: 1 / (dst / src) in double
    f = ((d + 0.5) * scale - 0.5).astype(np.float32)
    s = np.floor(f).astype(np.int64)
    f = (f - s.astype(np.float32)).astype(np.float32)
    if clamp_weights:
        f[s < 0] = 0
        s[s < 0] = 0
        f[s >= src - 1] = 0
        s[s >= src - 1] = src - 1
    w0 = np.rint((np.float32(1.0) - f) * np.float32(2048)).astype(np.int64)
    w1 = np.rint(f * np.float32(2048)).astype(np.int64)
    return np.clip(s, 0, src - 1), np.clip(s + 1, 0, src - 1), w0, w1


def resize_linear_u8(img_hwc, height: int, width: int):
    """uint8 [H, W, C] -> uint8 [height, width, C] exactly as OpenCV's
    INTER_LINEAR: horizontal pass in int (S[x0]*a0 + S[x1]*a1), vertical
    pass in the fixed-point form of its vectorised kernel,
    (((r0>>4)*b0 >> 16) + ((r1>>4)*b1 >> 16) + 2) >> 2, saturated to
    [0, 255].  Pinned against cv2.resize by tests/golden (make_resize_golden)."""
    import numpy as np
    img = np.asarray(img_hwc)
    h, w = img.shape[:2]
    x0, x1, a0, a1 = _resize_taps(width, w, True)
    y0, y1, b0, b1 = _resize_taps(height, h, False)
    rows = (img[:, x0].astype(np.int64) * a0[None, :, None] +
            img[:, x1].astype(np.int64) * a1[None, :, None])
    v = (((rows[y0] >> 4) * b0[:, None, None]) >> 16) + \
        (((rows[y1] >> 4) * b1[:, None, None]) >> 16)
    return np.clip((v + 2) >> 2, 0, 255).astype(np.uint8)


def normalize_images(images_u8: Tensor, means, stds) -> Tensor:
    """NormalizeImages, fluxvla/transforms/transform_images.py:313-372:
    (x - mean) / (std + 1e-8) per channel.  Input uint8 HWC [V,H,W,3];
    output float [V,3,H,W] (the transform works on CHW arrays)."""
    x = images_u8.to(F32).permute(0, 3, 1, 2)
    m = torch.tensor(means, dtype=F32)[:, :, None, None]
    s = torch.tensor(stds, dtype=F32)[:, :, None, None]
    return (x - m) / (s + 1e-8)


def siglip_forward(pix: Tensor, W: Dict[str, Tensor], n_layers: int,
                   num_heads: int, patch: int = 14, eps: float = 1e-6
                   ) -> Tensor:
    """One view through HF SiglipVisionModel (transformers, called from
    fluxvla/models/backbones/visions/siglip_vit.py:107-126):
    SiglipVisionEmbeddings (conv patch + learned pos) -> pre-LN encoder
    layers (LN1 -> MHA with bias, scale hd^-0.5 -> +res -> LN2 ->
    fc1 -> gelu_tanh -> fc2 -> +res) -> post_layernorm.
    ``pix`` [B,3,H,W] -> [B, P, width]."""
    x = torch.nn.functional.conv2d(pix, _w(W, 'vision.patch_w'),
                                   _w(W, 'vision.patch_b'), stride=patch)
    x = x.flatten(2).transpose(1, 2) + _w(W, 'vision.pos')[None]
    B, P, D = x.shape
    hd = D // num_heads
    for i in range(n_layers):
        p = f'vision.l{i}.'
        h = layer_norm(x, W[p + 'ln1_w'], W[p + 'ln1_b'], eps)
        q = linear(h, W[p + 'q_w'], W[p + 'q_b']).view(B, P, num_heads,
                                                       hd).transpose(1, 2)
        k = linear(h, W[p + 'k_w'], W[p + 'k_b']).view(B, P, num_heads,
                                                       hd).transpose(1, 2)
        v = linear(h, W[p + 'v_w'], W[p + 'v_b']).view(B, P, num_heads,
                                                       hd).transpose(1, 2)
        o = attention(q, k, v, None, hd ** -0.5)
        x = x + linear(o, W[p + 'o_w'], W[p + 'o_b'])
        h = layer_norm(x, W[p + 'ln2_w'], W[p + 'ln2_b'], eps)
        x = x + linear(gelu_tanh(linear(h, W[p + 'fc1_w'], W[p + 'fc1_b'])),
                       W[p + 'fc2_w'], W[p + 'fc2_b'])
    return layer_norm(x, W['vision.post_w'], W['vision.post_b'], eps)


# ---------------------------------------------------------------------------
# PI0 / PI0.5 glue
# ---------------------------------------------------------------------------

def embed_prefix(cfg, W, pixel_values: Tensor, lang_tokens: Tensor,
                 img_masks: Tensor, lang_masks: Tensor):
    """PI0FlowMatching.embed_prefix, pi0_flowmatching.py:204-250.
    pixel_values [B, 3V, H, W] normalised; returns (embs, pad, att)."""
    B = pixel_values.shape[0]
    views = pixel_values.unflatten(1, (-1, 3))
    toks = [siglip_forward(views[:, i], W, cfg.vis_layers, cfg.vis_heads,
                           cfg.patch) for i in range(views.shape[1])]
    img = linear(torch.cat(toks, dim=1), W['proj_w'], W['proj_b'])
    per_view = img.shape[1] // views.shape[1]
    pad = [img_masks[:, i:i + 1].expand(B, per_view)
           for i in range(views.shape[1])]
    lang = W['llm.embed'][lang_tokens].to(F32) * math.sqrt(cfg.llm_width)
    embs = torch.cat([img, lang], dim=1)
    pad = torch.cat(pad + [lang_masks], dim=1)
    att = torch.zeros_like(pad)
    return embs, pad, att


def prefill(cfg, W, embs: Tensor, pad: Tensor, att: Tensor,
            n_layers: Optional[int] = None):
    """The prefix half of predict_action, pi0_flowmatching.py:722-742:
    bidirectional prefix mask, positions cumsum(pad)-1, use_cache=True.
    Returns the per-layer (k, v) list [B,1,E,D]."""
    m2 = make_att_2d_masks(pad, att)
    pos = torch.cumsum(pad.to(torch.int64), dim=1) - 1
    _, kv = gemma_model(embs, W, 'llm.', n_layers or cfg.llm_layers, pos,
                        additive_mask(m2), cfg.heads, 1, cfg.head_dim,
                        final_norm=False)
    return kv


def pi0_embed_suffix(cfg, W, state: Tensor, x_t: Tensor, t: Tensor):
    """PI0FlowMatching.embed_suffix, pi0_flowmatching.py:252-321."""
    B = x_t.shape[0]
    embs, att = [], []
    if cfg.has_state_token:
        embs.append(linear(state, W['state_proj_w'], W['state_proj_b'])[:, None])
        att += [1]
    temb = sinusoidal_time(t, cfg.exp_width)
    a = linear(x_t, W['action_in_w'], W['action_in_b'])
    temb = temb[:, None, :].expand_as(a)
    h = linear(torch.cat([a, temb], dim=2), W['action_time_in_w'],
               W['action_time_in_b'])
    h = torch.nn.functional.silu(h)
    embs.append(linear(h, W['action_time_out_w'], W['action_time_out_b']))
    att += [1] + [0] * (cfg.n_actions - 1)
    embs = torch.cat(embs, dim=1)
    pad = torch.ones(B, embs.shape[1], dtype=torch.bool)
    att = torch.tensor(att, dtype=torch.bool)[None].expand(B, -1)
    return embs, pad, att, None


def pi05_embed_suffix(cfg, W, state, x_t: Tensor, t: Tensor):
    """PI05FlowMatching.embed_suffix, pi05_flowmatching.py:68-127: no state
    token; time -> silu(time_mlp_in) -> silu(time_mlp_out) = adarms cond."""
    B = x_t.shape[0]
    temb = sinusoidal_time(t, cfg.exp_width)
    a = linear(x_t, W['action_in_w'], W['action_in_b'])
    temb = torch.nn.functional.silu(linear(temb, W['time_in_w'],
                                           W['time_in_b']))
    temb = torch.nn.functional.silu(linear(temb, W['time_out_w'],
                                           W['time_out_b']))
    pad = torch.ones(B, a.shape[1], dtype=torch.bool)
    att = torch.tensor([1] + [0] * (cfg.n_actions - 1),
                       dtype=torch.bool)[None].expand(B, -1)
    return a, pad, att, temb


def denoise_step(cfg, W, state, prefix_pad: Tensor, kv, x_t: Tensor,
                 t: Tensor, n_layers: Optional[int] = None) -> Tensor:
    """PI0FlowMatching.denoise_step, pi0_flowmatching.py:787-831."""
    embed = pi05_embed_suffix if cfg.adarms else pi0_embed_suffix
    embs, spad, satt, cond = embed(cfg, W, state, x_t, t)
    B, S = spad.shape
    E = prefix_pad.shape[1]
    full = torch.cat([prefix_pad[:, None, :].expand(B, S, E),
                      make_att_2d_masks(spad, satt)], dim=2)
    pos = prefix_pad.sum(-1, keepdim=True) + torch.cumsum(
        spad.to(torch.int64), dim=1) - 1
    out, _ = gemma_model(embs, W, 'exp.', n_layers or cfg.exp_layers, pos,
                         additive_mask(full), cfg.heads, 1, cfg.head_dim,
                         past_kv=kv, adarms_cond=cond)
    out = out[:, -cfg.n_actions:]
    return linear(out, W['action_out_w'], W['action_out_b'])


def euler_loop(cfg, W, state, prefix_pad, kv, noise: Tensor,
               n_layers: Optional[int] = None) -> Tensor:
    """_predict_action_plain, pi0_flowmatching.py:642-649 (t=1, dt=-1/steps,
    fp32 time accumulation, while t >= -dt/2)."""
    dt = torch.tensor(-1.0 / cfg.num_steps, dtype=F32)
    t = torch.tensor(1.0, dtype=F32)
    x = noise.clone().to(F32)
    B = x.shape[0]
    while t >= -dt / 2:
        v = denoise_step(cfg, W, state, prefix_pad, kv, x, t.expand(B),
                         n_layers)
        x += dt * v
        t += dt
    return x


def step_times(num_steps: int) -> List[float]:
    """The fp32 time values the Euler loop visits (pi0_flowmatching.py:643-649)."""
    dt = torch.tensor(-1.0 / num_steps, dtype=F32)
    t = torch.tensor(1.0, dtype=F32)
    out = []
    while t >= -dt / 2:
        out.append(float(t))
        t += dt
    return out


def predict_action(cfg, W, images_u8: Tensor, lang_tokens: Tensor,
                   state: Tensor, noise: Tensor,
                   img_masks: Optional[Tensor] = None,
                   lang_masks: Optional[Tensor] = None) -> Tensor:
    """PI0FlowMatching.predict_action, pi0_flowmatching.py:702-785 (plain
    Euler branch), batch 1, with the image normalisation of the serving
    transform in front.  images_u8 [V,H,W,3] uint8."""
    V = images_u8.shape[0]
    pix = normalize_images(images_u8, [cfg.img_mean] * V, [cfg.img_std] * V)
    pix = pix.reshape(1, 3 * V, *pix.shape[2:])
    if img_masks is None:
        img_masks = torch.ones(1, V, dtype=torch.bool)
    if lang_masks is None:
        lang_masks = torch.ones(lang_tokens.shape, dtype=torch.bool)
    embs, pad, att = embed_prefix(cfg, W, pix, lang_tokens, img_masks,
                                  lang_masks)
    kv = prefill(cfg, W, embs, pad, att)
    return euler_loop(cfg, W, state, pad, kv, noise)


def gemma_layer_causal(cfg, W, x: Tensor, p: str = 'llm.l0.') -> Tensor:
    """config[0]: one Gemma-2B decoder layer over x with the default causal
    mask (create_causal_mask when attention_mask is None,
    condition_gemma.py:930-937) and positions 0..S-1."""
    B, S, _ = x.shape
    pos = torch.arange(S)[None].expand(B, S)
    cos, sin = rope_cos_sin(pos, cfg.head_dim)
    causal = torch.ones(S, S, dtype=torch.bool).tril()[None].expand(B, S, S)
    out, _ = gemma_layer(x.to(F32), W, p, cos, sin, additive_mask(causal),
                         cfg.heads, 1, cfg.head_dim)
    return out
