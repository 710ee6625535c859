"""Test-only torch emulation of the C ABI ops, for checking the engine's host
orchestration (buffer wiring, packing, masks, positions, step tables) on a
machine without a GPU.  It is monkeypatched over ``fluxvla_b200.ops`` inside
tests only; the product never imports it and has no CPU path.
"""
import torch
import torch.nn.functional as F

from fluxvla_b200._lib import (ACT_GELU_TANH, ACT_SILU, EPI_BF16,
                               EPI_F32_ACC, EPI_F32_STORE, EPI_GEGLU,
                               NORM_ADA_RMS, NORM_GEMMA_RMS, NORM_LAYER)

_count = [0]


def _act(x, act):
    if act == ACT_GELU_TANH:
        return F.gelu(x, approximate='tanh')
    if act == ACT_SILU:
        return F.silu(x)
    return x


def gemm(a, b, out, *, epilogue=EPI_BF16, swap=False, act=0, bias=None,
         gate=None, alpha=1.0, split_k=1, block_n=0, row_add=None,
         row_add_mod=0, k_out=None, v_out=None, n_heads=0, head_dim=0,
         rope_cs=None, positions=None, workspace=None, norm=None):
    _count[0] += 1
    acc = a.float() @ b.float().t()
    if swap:
        acc = acc.t()
    T, Fn = acc.shape
    if epilogue == EPI_BF16:
        y = alpha * acc + (bias if bias is not None else 0)
        out.copy_(_act(y, act).to(out.dtype))
    elif epilogue == EPI_F32_STORE:
        y = acc + (bias if bias is not None else 0)
        if row_add is not None:
            idx = torch.arange(T) % row_add_mod
            y = y + row_add.float()[idx]
        out.copy_(y)
    elif epilogue == EPI_F32_ACC:
        y = acc + (bias if bias is not None else 0)
        y = y * alpha
        if gate is not None:
            y = y * gate
        out.add_(y)
    elif epilogue == EPI_GEGLU:
        out.copy_((F.gelu(acc[:, 0::2], approximate='tanh') *
                   acc[:, 1::2]).to(out.dtype))
    else:
        hd, H, half = head_dim, n_heads, head_dim // 2
        pos = positions.long()
        c = rope_cs[pos, :, 0][:, None]
        s = rope_cs[pos, :, 1][:, None]
        qk = acc[:, :(H + 1) * hd].reshape(T, H + 1, half, 2)
        x1, x2 = qk[..., 0], qk[..., 1]
        r = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)
        out.copy_(r[:, :H].reshape(T, H * hd).to(out.dtype))
        k_out.copy_(r[:, H].to(k_out.dtype))
        v_out.copy_(acc[:, (H + 1) * hd:].to(v_out.dtype))
    if norm is not None:  # fused norm of the finished output, same launch
        mode, nout, nw, nb, eps, _sync = norm
        _norm_into(mode, out, nout, nw, nb, None, eps)


class _Args:

    def __init__(self, **kw):
        self.__dict__.update(kw)


def attn_args(q, k, v, o, **kw):
    d = dict(batch=1, q_batch_rows=0, kv_batch_rows=0, key_valid=None,
             n_prefix=None, q_block=None, k_block=None, kv_splits=1,
             workspace=None)
    d.update(kw)
    return _Args(q=q, k=k, v=v, o=o, **d)


def attention(a):
    _count[0] += 1
    hd, H = a.head_dim, a.heads
    batch, qbr, kbr = a.batch, a.q_batch_rows, a.kv_batch_rows
    for b in range(batch):
        for h in range(H):
            kvh = h // a.group

            def view(t, rs, hs, r0, n, head):
                base = t.storage_offset()
                st = t.untyped_storage()
                full = torch.empty(0, dtype=t.dtype).set_(st)
                idx = (base + (r0 + torch.arange(n))[:, None] * rs +
                       head * hs + torch.arange(hd)[None])
                return full, idx

            fq, iq = view(a.q, a.q_row_stride, a.q_head_stride, b * qbr,
                          a.n_q, h)
            kt, vt = a.k, a.v
            fk, ik = view(kt, a.k_row_stride, a.k_head_stride, b * kbr,
                          a.n_kv, kvh)
            fv, iv = view(vt, a.v_row_stride, a.v_head_stride, b * kbr,
                          a.n_kv, kvh)
            q, k, v = fq[iq].float(), fk[ik].float(), fv[iv].float()
            s = q @ k.t() * a.scale
            npre = a.n_prefix if a.n_prefix is not None else a.n_kv
            mask = torch.ones(a.n_q, a.n_kv, dtype=torch.bool)
            if a.key_valid is not None:
                mask[:, :npre] &= a.key_valid[:npre].bool()[None]
            if a.q_block is not None and npre < a.n_kv:
                kb = a.k_block[:a.n_kv - npre]
                mask[:, npre:] &= kb[None] <= a.q_block[:a.n_q, None]
            s = s.masked_fill(~mask, float('-inf'))
            o = torch.softmax(s, -1) @ v
            fo, io = view(a.o, a.o_row_stride, a.o_head_stride, b * qbr,
                          a.n_q, h)
            fo[io] = o.to(fo.dtype)


def attention_workspace_bytes(args):
    return 16


def gemm_workspace_bytes(m, n, swap, epilogue):
    return 16


def norm(mode, x, out, *, w=None, b=None, mod=None, eps=1e-6):
    _count[0] += 1
    _norm_into(mode, x, out, w, b, mod, eps)


def _norm_into(mode, x, out, w, b, mod, eps):
    D = x.shape[1]
    if mode == NORM_LAYER:
        y = F.layer_norm(x, (D,), w.float(), b.float(), eps)
    else:
        n = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)
        y = n * (1 + w.float()) if mode == NORM_GEMMA_RMS else \
            n * (1 + mod[:D]) + mod[D:2 * D]
    out.copy_(y.to(out.dtype))


def patchify(img, patch, mean3, std3, out):
    _count[0] += 1
    V = img.shape[0]
    m = torch.tensor(mean3)[:, None, None]
    s = torch.tensor(std3)[:, None, None]
    x = (img.float().permute(0, 3, 1, 2) - m) / (s + 1e-8)
    p = x.unfold(2, patch, patch).unfold(3, patch, patch)
    p = p.permute(0, 2, 3, 1, 4, 5).reshape(out.shape[0], -1)
    out.zero_()
    out[:, :p.shape[1]] = p.to(out.dtype)


def resize_patchify(img, size, patch, mean3, std3, out):
    from oracle.pi0_oracle import resize_linear_u8
    r = torch.stack([torch.from_numpy(resize_linear_u8(v.numpy(), size, size))
                     for v in img.cpu()])
    patchify(r, patch, mean3, std3, out)


def embed_tokens(ids, table, scale, out):
    _count[0] += 1
    out.copy_(table[ids.long()].float() * scale)


def small_linear(x, w, out, *, bias=None, act=0, mode=0, alpha=1.0, k=None):
    _count[0] += 1
    K = k or x.shape[1]
    y = x[:, :K].float() @ w[:, :K].float().t()
    if bias is not None:
        y = y + bias
    y = _act(y, act)
    if mode == 2:
        out.add_(alpha * y)
    else:
        out.copy_(y.to(out.dtype))


def expert_args(**kw):
    d = dict(qkv_bias=None, gu_bias=None, o_gate=None, down_gate=None,
             key_valid=None, eps=1e-6, workspace=None)
    d.update(kw)
    return _Args(**d)


def expert_workspace_bytes(args):
    return 16


def expert_step(a):
    """Same factorisation as the persistent kernel: GEMMs on x*(1+w), the
    per-token rstd applied by the consumer, adaRMS shift as W*shift bias."""
    _count[0] += 1
    L, S, W, hd, H = a.n_layers, a.n_tok, a.width, a.head_dim, a.heads
    E, half = a.n_prefix, a.head_dim // 2
    x = a.x
    pos = a.positions.long()
    c = a.rope_cs[pos, :, 0][:, None]
    s = a.rope_cs[pos, :, 1][:, None]
    blk = a.blocks[:S]
    qkv_rows = (H + 2) * hd
    for l in range(L):
        wq = a.w_qkv[l * qkv_rows:(l + 1) * qkv_rows].float()
        rs = torch.rsqrt((x * x).mean(-1, keepdim=True) + a.eps)
        acc = (x * a.in_scale[l]) @ wq.t() * rs
        if a.qkv_bias is not None:
            acc = acc + a.qkv_bias[l]
        qk = acc[:, :(H + 1) * hd].reshape(S, H + 1, half, 2)
        x1, x2 = qk[..., 0], qk[..., 1]
        r = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)
        q, k = r[:, :H], r[:, H]
        v = acc[:, (H + 1) * hd:]
        # the suffix keys / values land in the cache rows after the prefix
        a.k_cache[l, E:E + S] = k.bfloat16()
        a.v_cache[l, E:E + S] = v.bfloat16()
        kk = a.k_cache[l, :E + S].float()
        vv = a.v_cache[l, :E + S].float()
        mask = torch.ones(S, E + S, dtype=torch.bool)
        if a.key_valid is not None:
            mask[:, :E] &= a.key_valid[:E].bool()[None]
        mask[:, E:] &= blk[None] <= blk[:, None]
        att = torch.einsum('thd,kd->htk', q.bfloat16().float(), kk) * hd ** -0.5
        att = att.masked_fill(~mask[None], float('-inf')).softmax(-1)
        o = torch.einsum('htk,kd->thd', att, vv).reshape(S, H * hd)
        wo = a.w_o[l * W:(l + 1) * W].float()
        y = o.bfloat16().float() @ wo.t()
        x += y * (a.o_gate[l] if a.o_gate is not None else 1)
        rs = torch.rsqrt((x * x).mean(-1, keepdim=True) + a.eps)
        gu_rows = 2 * a.mlp
        wg = a.w_gu[l * gu_rows:(l + 1) * gu_rows].float()
        gu = (x * a.post_scale[l]) @ wg.t() * rs
        if a.gu_bias is not None:
            gu = gu + a.gu_bias[l]
        h = (F.gelu(gu[:, 0::2], approximate='tanh') * gu[:, 1::2]).bfloat16()
        wd = a.w_down[l * W:(l + 1) * W].float()
        y = h.float() @ wd.t()
        x += y * (a.down_gate[l] if a.down_gate is not None else 1)


def launch_count():
    return _count[0]


def install(monkeypatch):
    from fluxvla_b200 import engine, ops
    for name in ['gemm', 'attn_args', 'attention', 'attention_workspace_bytes',
                 'gemm_workspace_bytes', 'expert_args', 'expert_step',
                 'expert_workspace_bytes',
                 'norm', 'patchify', 'resize_patchify', 'embed_tokens',
                 'small_linear',
                 'launch_count']:
        monkeypatch.setattr(ops, name, globals()[name])
    monkeypatch.setattr(engine.torch.cuda, 'synchronize', lambda *a: None)
