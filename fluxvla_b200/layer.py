"""config[0]: one Gemma-2B decoder layer with the default causal mask.

The reference's single-layer workload runs ``GemmaDecoderLayer`` (via
ConditionGemmaModel) over x [1, S, 2048] with ``attention_mask=None``, i.e.
the causal mask of ``create_causal_mask`` (condition_gemma.py:930-937), and
positions 0..S-1: RMSNorm (1+w) -> q/k/v + RoPE -> causal MQA (8 query
heads, 1 KV head, head_dim 256) -> o_proj + residual -> RMSNorm -> gated
GELU-tanh MLP -> down + residual (condition_gemma.py:488-656).

``GemmaLayerB200`` runs it with the prefill kernels of the engine (the
QKV+RoPE GEMM epilogue, the split-over-keys attention with a block mask of
per-row ids 0..S-1, which is exactly the causal mask, the residual GEMMs
with f32 TMA reduce-add, the GeGLU GEMM) from static buffers, captured in
one CUDA graph.  The residual stream and the output are f32.
"""
from __future__ import annotations

from typing import Dict

import torch

from . import ops
from ._lib import EPI_F32_ACC, EPI_GEGLU, EPI_QKV_ROPE, NORM_GEMMA_RMS
from .config import PI0Config
from .pack import pack_geglu, pack_qkv, rope_table

BF16, F32 = torch.bfloat16, torch.float32


class GemmaLayerB200:
    """One Gemma decoder layer over S rows, causal, positions 0..S-1.

    weights: ``llm.l0.{in_norm,q_w,k_w,v_w,o_w,post_norm,gate_w,up_w,
    down_w}`` (nn.Linear [out, in] layout), any prefix ``p``."""

    def __init__(self, cfg: PI0Config, weights: Dict[str, torch.Tensor],
                 rows: int, device='cuda', p: str = 'llm.l0.',
                 attn_splits: int = 4):
        d = self.dev = torch.device(device)
        self.cfg, self.S = cfg, rows
        W = {k[len(p):]: v.to(d) for k, v in weights.items()
             if k.startswith(p)}
        hd, H, Wd = cfg.head_dim, cfg.heads, cfg.llm_width
        self.P = dict(qkv=pack_qkv(W['q_w'], W['k_w'], W['v_w'], hd),
                      o_w=W['o_w'].contiguous(),
                      gu=pack_geglu(W['gate_w'], W['up_w']),
                      down_w=W['down_w'].contiguous(),
                      in_norm=W['in_norm'].contiguous(),
                      post_norm=W['post_norm'].contiguous())
        z = lambda *s, dt=BF16: torch.zeros(*s, dtype=dt, device=d)  # noqa
        S = rows
        self.B = dict(x=z(S, Wd, dt=F32), xn=z(S, Wd), q=z(S, H * hd),
                      kc=z(S, hd), vc=z(S, hd), ao=z(S, H * hd),
                      h=z(S, cfg.llm_mlp),
                      pos=torch.arange(S, dtype=torch.int32, device=d),
                      rope=rope_table(S + 8, hd, device=d))
        kw = self._attn_kw(attn_splits)
        n = ops.attention_workspace_bytes(ops.attn_args(
            self.B['q'], self.B['kc'], self.B['vc'], self.B['ao'], **kw))
        self.B['attn_ws'] = z(max(n, 16), dt=torch.uint8)
        self.attn = ops.attn_args(self.B['q'], self.B['kc'], self.B['vc'],
                                  self.B['ao'], workspace=self.B['attn_ws'],
                                  **kw)
        self.graph = None
        self.launches_per_call = None

    def _attn_kw(self, splits):
        cfg, S, B = self.cfg, self.S, self.B
        hd, H = cfg.head_dim, cfg.heads
        # key j visible to query t iff pos_id[j] <= pos_id[t]: causal
        return dict(n_q=S, n_kv=S, heads=H, group=H, head_dim=hd,
                    scale=hd ** -0.5, q_row_stride=H * hd, q_head_stride=hd,
                    k_row_stride=hd, k_head_stride=0, v_row_stride=hd,
                    v_head_stride=0, o_row_stride=H * hd, o_head_stride=hd,
                    n_prefix=0, q_block=B['pos'], k_block=B['pos'],
                    kv_splits=splits)

    def run(self):
        """Enqueue the layer on the current stream (x updated in place)."""
        cfg, P, B = self.cfg, self.P, self.B
        ops.norm(NORM_GEMMA_RMS, B['x'], B['xn'], w=P['in_norm'])
        ops.gemm(B['xn'], P['qkv'], B['q'], epilogue=EPI_QKV_ROPE,
                 k_out=B['kc'], v_out=B['vc'], n_heads=cfg.heads,
                 head_dim=cfg.head_dim, rope_cs=B['rope'], positions=B['pos'])
        ops.attention(self.attn)
        ops.gemm(B['ao'], P['o_w'], B['x'], epilogue=EPI_F32_ACC,
                 block_n=256, split_k=2)
        ops.norm(NORM_GEMMA_RMS, B['x'], B['xn'], w=P['post_norm'])
        ops.gemm(B['xn'], P['gu'], B['h'], epilogue=EPI_GEGLU, block_n=256)
        ops.gemm(B['h'], P['down_w'], B['x'], epilogue=EPI_F32_ACC,
                 block_n=256, split_k=5)

    def capture(self):
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        saved = self.B['x'].clone()
        with torch.cuda.stream(s):
            n0 = ops.launch_count()
            self.run()
            self.launches_per_call = ops.launch_count() - n0
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.run()
        torch.cuda.synchronize(self.dev)
        self.B['x'].copy_(saved)
        self.graph = g

    def replay(self):
        self.graph.replay()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [1, S, width] (host or device) -> layer output [1, S, width]
        f32 on the host."""
        self.B['x'].copy_(x.reshape(self.S, -1), non_blocking=True)
        if self.graph is None:
            self.capture()
            self.B['x'].copy_(x.reshape(self.S, -1))
        self.replay()
        if getattr(self, '_host', None) is None:
            self._host = torch.empty(self.B['x'].shape, dtype=F32,
                                     pin_memory=True)
        self._host.copy_(self.B['x'], non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        st = ops.device_status()
        if st:
            ops.device_status(reset=True)
            raise RuntimeError(f'fluxvla_b200: device status {st}')
        return self._host.clone().reshape(1, self.S, -1)
