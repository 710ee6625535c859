"""B200 inference engine for PI0 / PI0.5 (batch 1 per replica).

Mirrors the reference's accelerated PI0.5 class
(fluxvla/models/vlas/pi05_flowmatching_inference.py:329-656): weights are
packed once, every activation lives in a static device buffer, and the whole
request (SigLIP + Gemma prefix prefill writing the bf16 KV cache, then the
10-step flow-matching loop of the action expert) is one CUDA graph replayed
per call.  Every kernel comes from libfluxvla_b200.so; torch only allocates
the buffers and owns the stream/graph.

Algorithm (same math as the eager reference, PI0FlowMatching.predict_action,
fluxvla/models/vlas/pi0_flowmatching.py:702-831):
  prefix: patchify+normalise -> patch GEMM (+bias +pos) -> 27 SigLIP layers
          -> post-LN -> projector -> rows 0..767; token embeddings * sqrt(2048)
          -> rows 768..; 18 Gemma layers (RMSNorm -> QKV+RoPE GEMM writing the
          K/V cache -> attention -> o_proj+res -> RMSNorm -> GeGLU GEMM ->
          down+res); the last layer stops after its K/V (its output is unused).
  loop:   10 Euler steps of the expert (suffix = state token + 50 action
          tokens for PI0; 50 action tokens with adaRMSNorm for PI0.5).
Step-invariant work is hoisted to load time: the time-embedding half of
action_time_mlp_in (PI0) and the time MLP plus every adaRMS modulation
(PI0.5) depend only on the step index.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from . import ops
from ._lib import (ACT_GELU_TANH, ACT_NONE, ACT_SILU, EPI_BF16, EPI_F32_ACC,
                   EPI_F32_STORE, EPI_GEGLU, EPI_QKV_ROPE, NORM_ADA_RMS,
                   NORM_GEMMA_RMS, NORM_LAYER)
from .config import PI0Config
from .pack import pack_geglu, pack_qkv, rope_table

BF16, F32 = torch.bfloat16, torch.float32


def step_times(num_steps: int):
    """fp32 times visited by the Euler loop (pi0_flowmatching.py:642-649)."""
    dt = torch.tensor(-1.0 / num_steps, dtype=F32)
    t = torch.tensor(1.0, dtype=F32)
    out = []
    while t >= -dt / 2:
        out.append(float(t))
        t += dt
    return out, float(dt)


def sinusoid(ts, dim: int) -> torch.Tensor:
    """create_sinusoidal_pos_embedding (model_utils.py:40-68), fp32, CPU."""
    t = torch.tensor(ts, dtype=F32)
    fraction = torch.linspace(0.0, 1.0, dim // 2, dtype=F32)
    period = 4e-3 * (4.0 / 4e-3) ** fraction
    x = t[:, None] * (1.0 / period * 2 * math.pi)
    return torch.cat([torch.sin(x), torch.cos(x)], dim=-1)


class PI0EngineB200:
    """One replica of the PI0 / PI0.5 inference path on one GPU.

    Args:
        cfg: model dimensions (PI0Config; cfg.adarms selects PI0.5).
        weights: dict of bf16 tensors named as in fluxvla_b200.weights (CPU
            or GPU).  Parts that are absent are skipped: an engine without
            'vision'/'llm' weights runs the denoise loop on an externally
            supplied KV cache (``set_prefix_cache``).
        prefix_len: E, the number of prefix rows (views*256 + prompt tokens).
        device: CUDA device.
    """

    def __init__(self, cfg: PI0Config, weights: Dict[str, torch.Tensor],
                 prefix_len: int, device='cuda', attn_splits: int = 0,
                 loop_impl: str = 'mega', camera_hw: Optional[tuple] = None,
                 image_format: str = 'u8'):
        self.cfg = cfg
        # 'u8': uint8 HWC camera views, normalised on the device (fast
        # path); 'f32': the reference model's normalised float pixels
        # [1, 3*views, H, W] (after its NormalizeImages transform)
        assert image_format in ('u8', 'f32')
        self.image_format = image_format
        # camera frame size (H, W) of the uint8 views handed to
        # predict_action; frames not already image_size x image_size are
        # resized on the device (OpenCV INTER_LINEAR, fused with normalise
        # and the patch layout)
        self.camera_hw = tuple(camera_hw) if camera_hw else (cfg.image_size,
                                                            cfg.image_size)
        # 'mega': one persistent cooperative kernel per denoise step for all
        # expert layers (fvb_expert_step); 'ops': one launch per operator
        assert loop_impl in ('mega', 'ops')
        self.loop_impl = loop_impl
        self.dev = torch.device(device)
        self.E = prefix_len
        self.S = cfg.n_suffix
        self.A = cfg.n_actions
        self.has_vision = 'vision.patch_w' in weights
        self.has_llm = 'llm.l0.q_w' in weights
        self.graph = None
        self.launches_per_call = None
        d = self.dev
        W = {k: v.to(d) for k, v in weights.items()}
        self._pack(W)
        del W
        self._alloc()
        self._attn_splits = attn_splits or max(
            1, -(-(self.E + self.S) // 64))
        self._precompute_steps()

    # ------------------------------------------------------------------
    # weights
    # ------------------------------------------------------------------
    def _pack(self, W):
        cfg, hd = self.cfg, self.cfg.head_dim
        f32 = lambda t: t.float().contiguous()  # noqa: E731
        P: Dict[str, torch.Tensor] = {}
        if self.has_vision:
            pk = ((cfg.patch_k + 7) // 8) * 8
            pw = torch.zeros(cfg.vis_width, pk, dtype=BF16, device=self.dev)
            pw[:, :cfg.patch_k] = W['vision.patch_w'].reshape(
                cfg.vis_width, -1)
            P['patch_w'], P['patch_b'] = pw, f32(W['vision.patch_b'])
            P['pos'] = W['vision.pos'].contiguous()
            for i in range(cfg.vis_layers):
                p = f'vision.l{i}.'
                P[p + 'qkv_w'] = torch.cat(
                    [W[p + 'q_w'], W[p + 'k_w'], W[p + 'v_w']]).contiguous()
                P[p + 'qkv_b'] = f32(torch.cat(
                    [W[p + 'q_b'], W[p + 'k_b'], W[p + 'v_b']]))
                for n in ['ln1_w', 'ln1_b', 'ln2_w', 'ln2_b', 'o_w', 'fc1_w',
                          'fc2_w']:
                    P[p + n] = W[p + n].contiguous()
                for n in ['o_b', 'fc1_b', 'fc2_b']:
                    P[p + n] = f32(W[p + n])
            P['post_w'], P['post_b'] = W['vision.post_w'], W['vision.post_b']
            P['proj_w'], P['proj_b'] = W['proj_w'].contiguous(), f32(
                W['proj_b'])
        if self.has_llm:
            P['embed'] = W['llm.embed'].contiguous()
        for pre, n_layers, present in (('llm.', cfg.llm_layers, self.has_llm),
                                       ('exp.', cfg.exp_layers, True)):
            if not present:
                continue
            for i in range(n_layers):
                p = f'{pre}l{i}.'
                P[p + 'qkv'] = pack_qkv(W[p + 'q_w'], W[p + 'k_w'],
                                        W[p + 'v_w'], hd)
                P[p + 'o_w'] = W[p + 'o_w'].contiguous()
                P[p + 'gu'] = pack_geglu(W[p + 'gate_w'], W[p + 'up_w'])
                P[p + 'down_w'] = W[p + 'down_w'].contiguous()
                for n in ['in_norm', 'post_norm']:
                    if p + n in W:
                        P[p + n] = W[p + n].contiguous()
                    else:
                        P[p + n + '_dense_w'] = W[p + n + '_dense_w']
                        P[p + n + '_dense_b'] = f32(W[p + n + '_dense_b'])
            if pre + 'norm' in W:
                P[pre + 'norm'] = W[pre + 'norm']
            elif pre + 'norm_dense_w' in W:
                P[pre + 'norm_dense_w'] = W[pre + 'norm_dense_w']
                P[pre + 'norm_dense_b'] = f32(W[pre + 'norm_dense_b'])
        # layer-stacked expert weights (one tensor map per kind for the
        # persistent step kernel); the per-layer entries become views
        L = cfg.exp_layers
        for n in ['qkv', 'o_w', 'gu', 'down_w']:
            st = torch.cat([P[f'exp.l{i}.{n}'] for i in range(L)]).contiguous()
            rows = st.shape[0] // L
            P[f'exp.{n}_all'] = st
            for i in range(L):
                P[f'exp.l{i}.{n}'] = st[i * rows:(i + 1) * rows]
        for n in ['action_in', 'action_out', 'state_proj', 'action_time_in',
                  'action_time_out', 'time_in', 'time_out']:
            if n + '_w' in W:
                P[n + '_w'] = W[n + '_w'].contiguous()
                P[n + '_b'] = f32(W[n + '_b'])
        self.P = P

    # ------------------------------------------------------------------
    # static buffers
    # ------------------------------------------------------------------
    def _alloc(self):
        cfg, d, E, S = self.cfg, self.dev, self.E, self.S
        z = lambda *s, dt=BF16: torch.zeros(*s, dtype=dt, device=d)  # noqa
        hd, L = cfg.head_dim, cfg.exp_layers
        B = {}
        B['kc'] = z(L, E + S, hd)
        B['vc'] = z(L, E + S, hd)
        if self.has_vision:
            R = cfg.n_views * cfg.tokens_per_view
            Wv = cfg.vis_width
            B['images'] = z(cfg.n_views, self.camera_hw[0], self.camera_hw[1], 3,
                            dt=torch.uint8)
            if self.image_format == 'f32':
                B['pixels'] = z(cfg.n_views, 3, cfg.image_size,
                                cfg.image_size, dt=F32)
            B['patches'] = z(R, self.P['patch_w'].shape[1])
            B['v_res'] = z(R, Wv, dt=F32)
            B['v_xn'] = z(R, Wv)
            B['v_qkv'] = z(R, 3 * Wv)
            B['v_ao'] = z(R, Wv)
            B['v_h'] = z(R, cfg.vis_mlp)
        if self.has_llm:
            Wl = cfg.llm_width
            B['tokens'] = z(E, dt=torch.int64)
            B['l_res'] = z(E, Wl, dt=F32)
            B['l_xn'] = z(E, Wl)
            B['l_q'] = z(E, cfg.heads * hd)
            B['l_ao'] = z(E, cfg.heads * hd)
            B['l_h'] = z(E, cfg.llm_mlp)
        We = cfg.exp_width
        B['pos_prefix'] = z(E, dt=torch.int32)
        B['key_valid'] = z(E, dt=torch.uint8)
        B['pos_suffix'] = z(S, dt=torch.int32)
        att = ([1] if cfg.has_state_token else []) + [1] + [0] * (self.A - 1)
        B['blocks'] = torch.tensor(att, dtype=torch.int32).cumsum(0).to(
            torch.int32).to(d)
        B['state'] = z(1, cfg.state_dim, dt=F32)
        B['noise'] = z(self.A, cfg.action_dim, dt=F32)
        B['x_t'] = z(self.A, cfg.action_dim, dt=F32)
        B['state_emb'] = z(1, We, dt=F32)
        B['e_res'] = z(S, We, dt=F32)
        B['e_xn'] = z(S, We)
        B['e_q'] = z(S, cfg.heads * hd)
        B['e_ao'] = z(S, cfg.heads * hd)
        B['e_h'] = z(S, cfg.exp_mlp)
        B['a_emb'] = z(self.A, We)
        B['at_h'] = z(self.A, We)
        B['e_fin'] = z(S, We, dt=F32)
        # split-K workspace of the swapped loop GEMMs (zeroed once, left
        # zeroed by every GEMM): sized for the widest one (gate/up)
        ws = max(ops.gemm_workspace_bytes(2 * cfg.exp_mlp, S, True, EPI_GEGLU),
                 ops.gemm_workspace_bytes(cfg.heads * hd + 2 * hd, S, True,
                                          EPI_QKV_ROPE))
        B['gemm_ws'] = z(ws, dt=torch.uint8)
        # grid-barrier counter of the GEMMs with a fused norm (only grows)
        B['norm_sync'] = z(1, dt=torch.int64)
        # key-split partials of the prefix attention (f32 O + max/sum),
        # sized for up to 4 splits
        B['prefix_attn_ws'] = z(4 * cfg.heads * E * (hd + 2) * 4 + 16,
                                dt=torch.uint8)
        max_pos = E + S + 8
        B['rope'] = rope_table(max_pos, hd, device=d)
        B['rope_suffix'] = z(S, hd // 2, 2, dt=F32)
        self.B = B
        self.mean3 = list(cfg.img_mean)
        self.std3 = list(cfg.img_std)

    def _precompute_steps(self):
        """Hoist the step-invariant time conditioning out of the loop."""
        cfg, d, P = self.cfg, self.dev, self.P
        self.times, self.dt = step_times(cfg.num_steps)
        n = len(self.times)
        temb = sinusoid(self.times, cfg.exp_width).to(d)
        We = cfg.exp_width
        if not cfg.adarms:
            # b_k = W_time . temb_k + b, with W_time the second half of
            # action_time_mlp_in's input columns (pi0_flowmatching.py:297-299)
            self.step_bias = torch.empty(n, We, dtype=F32, device=d)
            ops.small_linear(temb, P['action_time_in_w'][:, We:],
                             self.step_bias, bias=P['action_time_in_b'])
            # action_in_proj is linear and feeds only the action half of
            # action_time_mlp_in, so the two compose into one K = 32
            # projection: h = silu(x_t Wc^T + bc + b_k) with
            # Wc = W_time_in[:, :We] W_in and bc = W_time_in[:, :We] b_in,
            # formed once in f32 (one launch per step instead of two)
            Wa = P['action_time_in_w'][:, :We].float()
            self.w_act_time = (Wa @ P['action_in_w'].float()).to(BF16)
            self.step_bias_c = self.step_bias + (
                Wa @ P['action_in_b'].float())[None]
        else:
            # cond_k = silu(W_out silu(W_in temb_k + b_in) + b_out)
            # (pi05_flowmatching.py:97-108); mod_k = dense(cond_k) per norm
            h = torch.empty(n, We, dtype=F32, device=d)
            cond = torch.empty(n, We, dtype=F32, device=d)
            ops.small_linear(temb, P['time_in_w'], h, bias=P['time_in_b'],
                             act=ACT_SILU)
            ops.small_linear(h, P['time_out_w'], cond, bias=P['time_out_b'],
                             act=ACT_SILU)
            self.mods = {}
            names = [f'exp.l{i}.{m}' for i in range(cfg.exp_layers)
                     for m in ('in_norm', 'post_norm')] + ['exp.norm']
            for nm in names:
                out = torch.empty(n, 3 * We, dtype=F32, device=d)
                ops.small_linear(cond, P[nm + '_dense_w'], out,
                                 bias=P[nm + '_dense_b'])
                self.mods[nm] = out
        self._build_step_tables()
        if d.type == 'cuda':
            torch.cuda.synchronize(d)

    def _build_step_tables(self):
        """Per-step inputs of the persistent expert kernel.  RMSNorm enters
        the GEMMs as x*(1+w) (rstd is applied by the consumer); adaRMSNorm as
        x*(1+scale) plus the step-constant W*shift (bias) and the residual
        gates (condition_gemma.py:118-147, 319-337)."""
        cfg, P, B, d = self.cfg, self.P, self.B, self.dev
        L, We = cfg.exp_layers, cfg.exp_width
        hd, H = cfg.head_dim, cfg.heads
        n = len(self.times)
        if not cfg.adarms:
            ins = torch.stack([1.0 + P[f'exp.l{i}.in_norm'].float()
                               for i in range(L)]).contiguous()
            posts = torch.stack([1.0 + P[f'exp.l{i}.post_norm'].float()
                                 for i in range(L)]).contiguous()
            self.step_tables = [dict(in_scale=ins, post_scale=posts)] * n
            return
        tabs = []
        shift_in = torch.stack([self.mods[f'exp.l{i}.in_norm'][:, We:2 * We]
                                for i in range(L)])        # [L, n, We]
        shift_post = torch.stack([self.mods[f'exp.l{i}.post_norm'][:, We:2 * We]
                                  for i in range(L)])
        qkv_b = torch.empty(L, n, (H + 2) * hd, dtype=F32, device=d)
        gu_b = torch.empty(L, n, 2 * cfg.exp_mlp, dtype=F32, device=d)
        for i in range(L):
            ops.small_linear(shift_in[i].contiguous(), P[f'exp.l{i}.qkv'],
                             qkv_b[i])
            ops.small_linear(shift_post[i].contiguous(), P[f'exp.l{i}.gu'],
                             gu_b[i])
        for k in range(n):
            tabs.append(dict(
                in_scale=torch.stack([1.0 + self.mods[f'exp.l{i}.in_norm'][k, :We]
                                      for i in range(L)]).contiguous(),
                post_scale=torch.stack([1.0 + self.mods[f'exp.l{i}.post_norm'][k, :We]
                                        for i in range(L)]).contiguous(),
                o_gate=torch.stack([self.mods[f'exp.l{i}.in_norm'][k, 2 * We:]
                                    for i in range(L)]).contiguous(),
                down_gate=torch.stack([self.mods[f'exp.l{i}.post_norm'][k, 2 * We:]
                                       for i in range(L)]).contiguous(),
                qkv_bias=qkv_b[:, k].contiguous(),
                gu_bias=gu_b[:, k].contiguous()))
        self.step_tables = tabs

    def _expert_args(self, k: int):
        cfg, P, B = self.cfg, self.P, self.B
        a = dict(n_layers=cfg.exp_layers, n_tok=self.S, width=cfg.exp_width,
                 mlp=cfg.exp_mlp, heads=cfg.heads, head_dim=cfg.head_dim,
                 n_prefix=self.E, w_qkv=P['exp.qkv_all'], w_o=P['exp.o_w_all'],
                 w_gu=P['exp.gu_all'], w_down=P['exp.down_w_all'],
                 x=B['e_res'], k_cache=B['kc'], v_cache=B['vc'],
                 key_valid=B['key_valid'], blocks=B['blocks'],
                 positions=B['pos_suffix'], rope_cs=B['rope'],
                 rope_suffix=B['rope_suffix'])
        a.update(self.step_tables[k])
        if 'expert_ws' not in B:
            nbytes = ops.expert_workspace_bytes(ops.expert_args(**a))
            B['expert_ws'] = torch.zeros(nbytes, dtype=torch.uint8,
                                         device=self.dev)
        a['workspace'] = B['expert_ws']
        return ops.expert_args(**a)

    # ------------------------------------------------------------------
    # prefix
    # ------------------------------------------------------------------
    def _vision(self):
        cfg, P, B, T = self.cfg, self.P, self.B, self.tiles
        Wv, R = cfg.vis_width, cfg.n_views * cfg.tokens_per_view
        hdv = Wv // cfg.vis_heads
        if self.image_format == 'f32':
            ops.patchify_f32(B['pixels'], cfg.patch, B['patches'])
        elif self.camera_hw == (cfg.image_size, cfg.image_size):
            ops.patchify(B['images'], cfg.patch, self.mean3, self.std3,
                         B['patches'])
        else:
            ops.resize_patchify(B['images'], cfg.image_size, cfg.patch,
                                self.mean3, self.std3, B['patches'])
        ops.gemm(B['patches'], P['patch_w'], B['v_res'], epilogue=EPI_F32_STORE,
                 bias=P['patch_b'], row_add=P['pos'],
                 row_add_mod=cfg.tokens_per_view)
        qkv = B['v_qkv']
        attn = ops.attn_args(
            qkv, qkv[:, Wv:], qkv[:, 2 * Wv:], B['v_ao'],
            n_q=cfg.tokens_per_view, n_kv=cfg.tokens_per_view,
            heads=cfg.vis_heads, group=1, head_dim=hdv, scale=hdv ** -0.5,
            q_row_stride=3 * Wv, q_head_stride=hdv, k_row_stride=3 * Wv,
            k_head_stride=hdv, v_row_stride=3 * Wv, v_head_stride=hdv,
            o_row_stride=Wv, o_head_stride=hdv, batch=cfg.n_views,
            q_batch_rows=cfg.tokens_per_view,
            kv_batch_rows=cfg.tokens_per_view)
        # the LayerNorm after each residual GEMM runs in that GEMM's launch
        # (fused norm behind a grid barrier); only the first one is separate
        ops.norm(NORM_LAYER, B['v_res'], B['v_xn'], w=P['vision.l0.ln1_w'],
                 b=P['vision.l0.ln1_b'])
        for i in range(cfg.vis_layers):
            p = f'vision.l{i}.'
            ops.gemm(B['v_xn'], P[p + 'qkv_w'], qkv, bias=P[p + 'qkv_b'],
                     block_n=T['vis_qkv'][0])
            ops.attention(attn)
            self._residual_gemm('vis_o', B['v_ao'], P[p + 'o_w'], B['v_res'],
                                dict(bias=P[p + 'o_b'], block_n=T['vis_o'][0],
                                     split_k=T['vis_o'][1]),
                                (NORM_LAYER, B['v_xn'], P[p + 'ln2_w'], P[p + 'ln2_b']))
            ops.gemm(B['v_xn'], P[p + 'fc1_w'], B['v_h'], bias=P[p + 'fc1_b'],
                     act=ACT_GELU_TANH, block_n=T['vis_fc1'][0])
            nxt = f'vision.l{i + 1}.ln1_' if i + 1 < cfg.vis_layers else 'post_'
            self._residual_gemm('vis_fc2', B['v_h'], P[p + 'fc2_w'], B['v_res'],
                                dict(bias=P[p + 'fc2_b'], block_n=T['vis_fc2'][0],
                                     split_k=T['vis_fc2'][1]),
                                (NORM_LAYER, B['v_xn'], P[nxt + 'w'], P[nxt + 'b']))
        ops.gemm(B['v_xn'], P['proj_w'], B['l_res'][:R], epilogue=EPI_F32_STORE,
                 bias=P['proj_b'])

    # residual GEMM call sites whose following norm runs in the GEMM's launch
    # (grid barrier + norm tail); the others launch the norm kernel after it.
    # None by default: measured on the full prefill (5.45 ms unfused vs
    # 5.71 ms with all four sites fused), the grid barrier holds every CTA
    # until the slowest tile is done, which costs more than the norm launch
    # whose start overlaps the GEMM's tail under programmatic dependent launch.
    fused_norm_sites = frozenset()
    # residual GEMM call sites run as two-SM pair tiles (swapped orientation,
    # 256 weight rows per CTA pair, fvb_gemm `pair`) with these K splits
    pair_sites = {}
    # key splits of the Gemma prefix attention (tcgen05 kernel + combine).
    # 1: measured on the full prefill, 2 splits (102 CTAs + the combine of
    # f32 partials) cost 0.2 ms more than 51 unsplit CTAs
    prefix_attn_splits = 1
    # (tile width, K splits) of the prefill GEMM call sites, measured on the
    # full prefill graph
    tiles = dict(vis_qkv=(192, 1), vis_o=(0, 2), vis_fc1=(192, 1),
                 vis_fc2=(192, 4), llm_qkv=(0, 1), llm_o=(256, 2),
                 llm_down=(256, 5))

    def _residual_gemm(self, site, a, w, res, kw, norm):
        """res += a @ w^T, then norm(res) -> bf16 (mode, out, w, b)."""
        mode, out, nw, nb = norm
        if site in self.pair_sites:
            ops.gemm(w, a, res, epilogue=EPI_F32_ACC, swap=True, pair=True,
                     split_k=self.pair_sites[site],
                     **{k: v for k, v in kw.items() if k not in ('block_n', 'split_k')})
            ops.norm(mode, res, out, w=nw, b=nb)
        elif site in self.fused_norm_sites:
            ops.gemm(a, w, res, epilogue=EPI_F32_ACC,
                     norm=(mode, out, nw, nb, 1e-6, self.B['norm_sync']), **kw)
        else:
            ops.gemm(a, w, res, epilogue=EPI_F32_ACC, **kw)
            ops.norm(mode, res, out, w=nw, b=nb)

    def _llm(self):
        cfg, P, B, E, T = self.cfg, self.P, self.B, self.E, self.tiles
        hd, H = cfg.head_dim, cfg.heads
        R = cfg.n_views * cfg.tokens_per_view if self.has_vision else 0
        ops.embed_tokens(B['tokens'][:E - R], P['embed'],
                         math.sqrt(cfg.llm_width), B['l_res'][R:])
        ops.norm(NORM_GEMMA_RMS, B['l_res'], B['l_xn'], w=P['llm.l0.in_norm'])
        for i in range(cfg.llm_layers):
            p = f'llm.l{i}.'
            kc, vc = B['kc'][i], B['vc'][i]
            ops.gemm(B['l_xn'], P[p + 'qkv'], B['l_q'], epilogue=EPI_QKV_ROPE,
                     block_n=T['llm_qkv'][0],
                     k_out=kc[:E], v_out=vc[:E], n_heads=H, head_dim=hd,
                     rope_cs=B['rope'], positions=B['pos_prefix'])
            if i == cfg.llm_layers - 1:
                break  # only the K/V of the last layer is consumed
            ops.attention(ops.attn_args(
                B['l_q'], kc, vc, B['l_ao'], n_q=E, n_kv=E, heads=H, group=H,
                head_dim=hd, scale=hd ** -0.5, q_row_stride=H * hd,
                q_head_stride=hd, k_row_stride=hd, k_head_stride=0,
                v_row_stride=hd, v_head_stride=0, o_row_stride=H * hd,
                o_head_stride=hd, key_valid=B['key_valid'], n_prefix=E,
                kv_splits=self.prefix_attn_splits, workspace=B['prefix_attn_ws']))
            self._residual_gemm('llm_o', B['l_ao'], P[p + 'o_w'], B['l_res'],
                                dict(block_n=T['llm_o'][0], split_k=T['llm_o'][1]),
                                (NORM_GEMMA_RMS, B['l_xn'], P[p + 'post_norm'], None))
            ops.gemm(B['l_xn'], P[p + 'gu'], B['l_h'], epilogue=EPI_GEGLU,
                     block_n=256)
            # the next layer's input norm rides on the down projection
            self._residual_gemm('llm_down', B['l_h'], P[p + 'down_w'], B['l_res'],
                                dict(block_n=T['llm_down'][0],
                                     split_k=T['llm_down'][1]),
                                (NORM_GEMMA_RMS, B['l_xn'],
                                 P[f'llm.l{i + 1}.in_norm'], None))

    def _state_token(self):
        if self.cfg.has_state_token:
            ops.small_linear(self.B['state'], self.P['state_proj_w'],
                             self.B['state_emb'], bias=self.P['state_proj_b'])

    # ------------------------------------------------------------------
    # denoise loop
    # ------------------------------------------------------------------
    def _expert_step(self, k: int):
        cfg, P, B, E, S, A = self.cfg, self.P, self.B, self.E, self.S, self.A
        hd, H, We = cfg.head_dim, cfg.heads, cfg.exp_width
        ada = cfg.adarms
        res = B['e_res']
        off = S - A  # 1 with the PI0 state token
        if ada:
            # suffix = action_in_proj(x_t) (pi05_flowmatching.py:95)
            ops.small_linear(B['x_t'], P['action_in_w'], res,
                             bias=P['action_in_b'])
        else:
            ops.small_linear(B['x_t'], self.w_act_time, B['at_h'],
                             bias=self.step_bias_c[k], act=ACT_SILU, mode=1)
            # K splits summed in the workspace, the last split stores
            ops.gemm(P['action_time_out_w'], B['at_h'], res[off:],
                     epilogue=EPI_F32_STORE, swap=True,
                     bias=P['action_time_out_b'], split_k=0,
                     workspace=B['gemm_ws'])
            if off:
                res[:off].copy_(B['state_emb'])
        if self.loop_impl == 'mega':
            ops.expert_step(self._expert_args(k))
        else:
            self._expert_layers_ops(k)
        fin = B['e_fin'][off:]
        if ada:
            ops.norm(NORM_ADA_RMS, res[off:], fin, mod=self.mods['exp.norm'][k])
        else:
            ops.norm(NORM_GEMMA_RMS, res[off:], fin, w=P['exp.norm'])
        # v_t = action_out_proj(out); x_t += dt * v_t (pi0_flowmatching.py:646)
        ops.small_linear(fin, P['action_out_w'], B['x_t'],
                         bias=P['action_out_b'], mode=2, alpha=self.dt)

    def _expert_layers_ops(self, k: int):
        """The expert layers with one launch per operator (reference path
        for the persistent kernel)."""
        cfg, P, B, E, S = self.cfg, self.P, self.B, self.E, self.S
        hd, H, We = cfg.head_dim, cfg.heads, cfg.exp_width
        ada = cfg.adarms
        res = B['e_res']
        def attn(kc, vc):
            return ops.attn_args(
                B['e_q'], kc, vc, B['e_ao'], n_q=S, n_kv=E + S, heads=H,
                group=H, head_dim=hd, scale=hd ** -0.5, q_row_stride=H * hd,
                q_head_stride=hd, k_row_stride=hd, k_head_stride=0,
                v_row_stride=hd, v_head_stride=0, o_row_stride=H * hd,
                o_head_stride=hd, key_valid=B['key_valid'], n_prefix=E,
                q_block=B['blocks'], k_block=B['blocks'],
                kv_splits=self._attn_splits, workspace=self.attn_ws)

        for i in range(cfg.exp_layers):
            p = f'exp.l{i}.'
            kc, vc = B['kc'][i], B['vc'][i]
            if ada:
                m_in = self.mods[p + 'in_norm'][k]
                m_post = self.mods[p + 'post_norm'][k]
                ops.norm(NORM_ADA_RMS, res, B['e_xn'], mod=m_in)
            else:
                ops.norm(NORM_GEMMA_RMS, res, B['e_xn'], w=P[p + 'in_norm'])
            ops.gemm(P[p + 'qkv'], B['e_xn'], B['e_q'], swap=True,
                     epilogue=EPI_QKV_ROPE, k_out=kc[E:], v_out=vc[E:],
                     n_heads=H, head_dim=hd, rope_cs=B['rope'],
                     positions=B['pos_suffix'])
            ops.attention(attn(kc, vc))
            ops.gemm(P[p + 'o_w'], B['e_ao'], res, swap=True,
                     epilogue=EPI_F32_ACC, split_k=0,
                     gate=m_in[2 * We:] if ada else None)
            if ada:
                ops.norm(NORM_ADA_RMS, res, B['e_xn'], mod=m_post)
            else:
                ops.norm(NORM_GEMMA_RMS, res, B['e_xn'], w=P[p + 'post_norm'])
            ops.gemm(P[p + 'gu'], B['e_xn'], B['e_h'], swap=True,
                     epilogue=EPI_GEGLU)
            ops.gemm(P[p + 'down_w'], B['e_h'], res, swap=True,
                     epilogue=EPI_F32_ACC, split_k=0,
                     gate=m_post[2 * We:] if ada else None)

    def _loop(self):
        self.B['x_t'].copy_(self.B['noise'])
        for k in range(len(self.times)):
            self._expert_step(k)

    # ------------------------------------------------------------------
    # public API
    # ------------------------------------------------------------------
    @property
    def attn_ws(self):
        if not hasattr(self, '_attn_ws'):
            cfg = self.cfg
            rows = cfg.heads * self.S
            n = self._attn_splits * rows * (cfg.head_dim + 2) * 4
            self._attn_ws = torch.empty(max(n, 16), dtype=torch.uint8,
                                        device=self.dev)
        return self._attn_ws

    def set_prefix_cache(self, k: torch.Tensor, v: torch.Tensor,
                         key_valid: Optional[torch.Tensor] = None):
        """Install an external prefix KV cache [L, E, hd] (loop-only mode)."""
        E = self.E
        self.B['kc'][:, :E].copy_(k)
        self.B['vc'][:, :E].copy_(v)
        kv = torch.ones(E, dtype=torch.uint8) if key_valid is None else \
            key_valid.to(torch.uint8).cpu()
        self._set_masks(kv)

    def _set_masks(self, key_valid_cpu: torch.Tensor):
        """Positions and key mask from the prefix pad mask
        (pi0_flowmatching.py:730 and :817-819)."""
        self._last_key_valid = key_valid_cpu.to(torch.bool).clone()
        kv = key_valid_cpu.to(torch.int64)
        pos = (torch.cumsum(kv, 0) - 1).clamp(min=0).to(torch.int32)
        self.B['key_valid'].copy_(kv.to(torch.uint8))
        self.B['pos_prefix'].copy_(pos)
        pos_suf = (int(kv.sum()) + torch.arange(self.S)).to(torch.int32)
        self.B['pos_suffix'].copy_(pos_suf)
        # rotary cos/sin of the suffix positions, gathered once per request
        self.B['rope_suffix'].copy_(
            self.B['rope'][pos_suf.to(self.B['rope'].device).long()])

    def load_inputs(self, images_u8=None, lang_tokens=None, lang_masks=None,
                    img_masks=None, state=None, noise=None):
        """Copy one request into the static input buffers (H2D)."""
        cfg, B = self.cfg, self.B
        if images_u8 is not None and self.image_format == 'f32':
            B['pixels'].copy_(images_u8.reshape(B['pixels'].shape),
                              non_blocking=True)
        elif images_u8 is not None:
            B['images'].copy_(images_u8.reshape(B['images'].shape),
                              non_blocking=True)
        if lang_tokens is not None:
            lt = lang_tokens.reshape(-1)
            B['tokens'][:lt.numel()].copy_(lt, non_blocking=True)
            R = cfg.n_views * cfg.tokens_per_view if self.has_vision else 0
            im = torch.ones(cfg.n_views, dtype=torch.bool) if img_masks is None \
                else img_masks.reshape(-1).bool().cpu()
            lm = torch.ones(lt.numel(), dtype=torch.bool) if lang_masks is None \
                else lang_masks.reshape(-1).bool().cpu()
            kv = torch.cat([im.repeat_interleave(cfg.tokens_per_view), lm])
            assert kv.numel() == self.E, (kv.numel(), self.E)
            # positions / key mask / suffix rotary rows depend only on the
            # padding pattern: rebuilt only when it changes
            last = getattr(self, '_last_key_valid', None)
            if last is None or not torch.equal(last, kv):
                self._set_masks(kv)
        if state is not None and cfg.has_state_token:
            B['state'].copy_(state.reshape(1, -1), non_blocking=True)
        if noise is not None:
            B['noise'].copy_(noise.reshape(self.A, -1), non_blocking=True)

    def run_prefix(self):
        if self.has_vision:
            self._vision()
        if self.has_llm:
            self._llm()
        self._state_token()

    def run(self, prefix: bool = True):
        """Enqueue one full request (prefix + loop) on the current stream."""
        if prefix:
            self.run_prefix()
        else:
            self._state_token()
        self._loop()

    def capture(self, prefix: bool = True):
        """Capture run() into one CUDA graph (after one eager warm-up)."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            n0 = ops.launch_count()
            self.run(prefix)
            self.launches_per_call = ops.launch_count() - n0
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.run(prefix)
        torch.cuda.synchronize(self.dev)
        self.graph = g
        self._graph_prefix = prefix

    def replay(self):
        self.graph.replay()

    @property
    def actions(self) -> torch.Tensor:
        return self.B['x_t']

    def predict_action(self, images=None, lang_tokens=None, states=None,
                       img_masks=None, lang_masks=None, noise=None):
        """PI0FlowMatching.predict_action semantics at batch 1: returns
        [1, n_actions, action_dim] float32 on the host."""
        if noise is None:
            noise = torch.randn(self.A, self.cfg.action_dim)
        self.load_inputs(images, lang_tokens, lang_masks, img_masks, states,
                         noise)
        if self.graph is None:
            self.capture(prefix=self.has_vision or self.has_llm)
        self.replay()
        # read back through a pinned buffer on the engine's stream
        if getattr(self, '_x_host', None) is None:
            self._x_host = torch.empty(self.B['x_t'].shape, dtype=self.B['x_t'].dtype,
                                       pin_memory=True)
        self._x_host.copy_(self.B['x_t'], non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        self.check_device_status()
        return self._x_host.clone().reshape(1, self.A, -1)

    def check_device_status(self):
        """Raise if a kernel of the last replay gave up a bounded wait.

        The kernels never trap: a wait that runs past its limit records
        FVB_ERR_DEVICE_TIMEOUT in the library's status word and returns, so
        that chunk's actions are invalid.  The status word is read after the
        chunk's synchronisation; on an error it is cleared, the engine's
        synchronisation state (the persistent step's barrier counter and
        abort flag, split-K workspaces) is zeroed so that the next chunk
        starts clean, and the error is raised."""
        st = ops.device_status()
        if st:
            ops.device_status(reset=True)
            self.reset_sync_state()
            raise RuntimeError(
                f'fluxvla_b200: device status {st} (a kernel wait gave up); '
                'the actions of this chunk are invalid, the engine has been '
                'reset for the next call')

    def reset_sync_state(self):
        """Zero every workspace that carries state between launches."""
        for k in ('expert_ws', 'gemm_ws', 'norm_sync', 'prefix_attn_ws'):
            if k in self.B:
                self.B[k].zero_()
        torch.cuda.synchronize(self.dev)
