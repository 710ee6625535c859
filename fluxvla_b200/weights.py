"""Seeded synthetic weights for the PI0 / PI0.5 architectures.

There is no network and no checkpoint, so every run uses random weights of
the real architecture: ~N(0, 0.02) for every linear weight, bias, embedding
and Gemma norm weight (Gemma norms scale by (1 + w), so their weights are
perturbations around 0), and 1 + N(0, 0.02) for SigLIP LayerNorm scales.
Values are rounded to bf16 (the inference dtype); the fp32 oracle upcasts the
same bf16 values, so both sides see identical weights.

Each tensor has its own generator seeded from (seed, crc32(name)), so any
subset can be generated independently and reproducibly on the CPU.

Names (shapes use the reference nn.Linear [out, in] convention):
  vision.patch_w [W,3,14,14], vision.patch_b [W], vision.pos [P,W]
  vision.l{i}.{ln1_w,ln1_b,q_w,q_b,k_w,k_b,v_w,v_b,o_w,o_b,ln2_w,ln2_b,
               fc1_w,fc1_b,fc2_w,fc2_b}, vision.post_w, vision.post_b
  proj_w [2048,W], proj_b
  llm.embed [vocab,2048]; llm.l{i}.{in_norm,q_w,k_w,v_w,o_w,post_norm,
                                   gate_w,up_w,down_w}; llm.norm
  exp.l{i}.{...same...}; exp.norm  (PI0.5: *_norm_dense_w/_b, norm_dense_w/_b)
  state_proj_w/b, action_in_w/b, action_out_w/b,
  action_time_in_w/b, action_time_out_w/b (PI0); time_in_w/b, time_out_w/b
  (PI0.5)
"""
from __future__ import annotations

import zlib
from typing import Dict, Iterable, List, Tuple

import torch

from .config import PI0Config

STD = 0.02


def weight_shapes(cfg: PI0Config, parts: Iterable[str] = ('vision', 'llm',
                                                          'exp', 'heads')
                  ) -> List[Tuple[str, tuple, str]]:
    """(name, shape, init) for every tensor; init is 'n' (N(0,.02)) or
    'ln' (1 + N(0,.02))."""
    out = []
    parts = set(parts)
    W, hd, H = cfg.vis_width, cfg.head_dim, cfg.heads
    if 'vision' in parts:
        out += [('vision.patch_w', (W, 3, cfg.patch, cfg.patch), 'n'),
                ('vision.patch_b', (W,), 'n'),
                ('vision.pos', (cfg.tokens_per_view, W), 'n')]
        for i in range(cfg.vis_layers):
            p = f'vision.l{i}.'
            out += [(p + 'ln1_w', (W,), 'ln'), (p + 'ln1_b', (W,), 'n')]
            for n in 'qkvo':
                out += [(p + n + '_w', (W, W), 'n'), (p + n + '_b', (W,), 'n')]
            out += [(p + 'ln2_w', (W,), 'ln'), (p + 'ln2_b', (W,), 'n'),
                    (p + 'fc1_w', (cfg.vis_mlp, W), 'n'),
                    (p + 'fc1_b', (cfg.vis_mlp,), 'n'),
                    (p + 'fc2_w', (W, cfg.vis_mlp), 'n'),
                    (p + 'fc2_b', (W,), 'n')]
        out += [('vision.post_w', (W,), 'ln'), ('vision.post_b', (W,), 'n'),
                ('proj_w', (cfg.llm_width, W), 'n'),
                ('proj_b', (cfg.llm_width,), 'n')]

    def gemma(prefix, layers, width, mlp, ada):
        o = []
        for i in range(layers):
            p = f'{prefix}l{i}.'
            if ada:
                o += [(p + 'in_norm_dense_w', (3 * width, width), 'n'),
                      (p + 'in_norm_dense_b', (3 * width,), 'n')]
            else:
                o += [(p + 'in_norm', (width,), 'n')]
            o += [(p + 'q_w', (H * hd, width), 'n'),
                  (p + 'k_w', (hd, width), 'n'),
                  (p + 'v_w', (hd, width), 'n'),
                  (p + 'o_w', (width, H * hd), 'n')]
            if ada:
                o += [(p + 'post_norm_dense_w', (3 * width, width), 'n'),
                      (p + 'post_norm_dense_b', (3 * width,), 'n')]
            else:
                o += [(p + 'post_norm', (width,), 'n')]
            o += [(p + 'gate_w', (mlp, width), 'n'),
                  (p + 'up_w', (mlp, width), 'n'),
                  (p + 'down_w', (width, mlp), 'n')]
        if ada:
            o += [(prefix + 'norm_dense_w', (3 * width, width), 'n'),
                  (prefix + 'norm_dense_b', (3 * width,), 'n')]
        else:
            o += [(prefix + 'norm', (width,), 'n')]
        return o

    if 'llm' in parts:
        out += [('llm.embed', (cfg.vocab, cfg.llm_width), 'n')]
        out += gemma('llm.', cfg.llm_layers, cfg.llm_width, cfg.llm_mlp,
                     False)
    if 'exp' in parts:
        out += gemma('exp.', cfg.exp_layers, cfg.exp_width, cfg.exp_mlp,
                     cfg.adarms)
    if 'heads' in parts:
        E, A = cfg.exp_width, cfg.action_dim
        out += [('action_in_w', (E, A), 'n'), ('action_in_b', (E,), 'n'),
                ('action_out_w', (A, E), 'n'), ('action_out_b', (A,), 'n')]
        if cfg.has_state_token:
            out += [('state_proj_w', (E, cfg.state_dim), 'n'),
                    ('state_proj_b', (E,), 'n')]
        if cfg.adarms:
            out += [('time_in_w', (E, E), 'n'), ('time_in_b', (E,), 'n'),
                    ('time_out_w', (E, E), 'n'), ('time_out_b', (E,), 'n')]
        else:
            out += [('action_time_in_w', (E, 2 * E), 'n'),
                    ('action_time_in_b', (E,), 'n'),
                    ('action_time_out_w', (E, E), 'n'),
                    ('action_time_out_b', (E,), 'n')]
    return out


def gen_tensor(name: str, shape: tuple, init: str, seed: int,
               device='cpu') -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1000003 + zlib.crc32(name.encode())) & (2**63 - 1))
    t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    t.mul_(STD)
    if init == 'ln':
        t.add_(1.0)
    return t.to(torch.bfloat16)


def make_weights(cfg: PI0Config, seed: int = 0,
                 parts: Iterable[str] = ('vision', 'llm', 'exp', 'heads'),
                 device='cpu') -> Dict[str, torch.Tensor]:
    return {n: gen_tensor(n, s, i, seed, device)
            for n, s, i in weight_shapes(cfg, parts)}


def make_weights_matching(cfg: PI0Config, seed: int, predicate,
                          parts: Iterable[str] = ('vision', 'llm', 'exp',
                                                  'heads'),
                          device='cpu') -> Dict[str, torch.Tensor]:
    """Only the tensors whose name satisfies ``predicate`` (same values as
    make_weights would give them)."""
    return {n: gen_tensor(n, s, i, seed, device)
            for n, s, i in weight_shapes(cfg, parts) if predicate(n)}
