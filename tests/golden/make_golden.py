"""Generate golden vectors from the reference FluxVLA eager modules.

Run where the reference sources are available, either as a source tree
named by ``$FLUXVLA_REF`` or as the pip-installed copy under ``baseline/_ref``:

    FLUXVLA_REF=<FluxVLA source tree> python tests/golden/make_golden.py [names]

The reference modules are loaded by file path behind the shim of
``oracle/ref_shim.py`` (stub registries, transformers-5.5 patches).
The reference modules then run unmodified, in fp32 on the CPU, on weights
from ``fluxvla_b200.weights.make_weights`` (loaded into their state dicts by
name), and their outputs are saved as small ``.pt`` fixtures next to this
script.  The tests compare the oracle (``oracle/pi0_oracle.py``) with these
fixtures; they never read the reference tree.
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from fluxvla_b200.config import PI0Config, pi05_config  # noqa: E402
from fluxvla_b200.weights import make_weights  # noqa: E402
from oracle.ref_shim import (_gemma_cfg, build_ref_model,  # noqa: E402
                             load_reference, load_weights, name_map)


# ---------------------------------------------------------------------------
# fixtures
# ---------------------------------------------------------------------------

def tiny_cfg(pi05=False):
    kw = dict(vis_layers=2, vis_width=32, vis_heads=2, vis_mlp=48, patch=14,
              image_size=28, n_views=2, llm_layers=2, llm_width=64,
              llm_mlp=96, vocab=97, heads=2, head_dim=16, exp_layers=2,
              exp_width=32, exp_mlp=64, n_actions=4, action_dim=8,
              state_dim=8, num_steps=10)
    return pi05_config(**kw) if pi05 else PI0Config(**kw)


def inputs(cfg, seed, n_tokens):
    g = torch.Generator().manual_seed(seed)
    imgs = torch.randint(0, 256, (cfg.n_views, cfg.image_size,
                                  cfg.image_size, 3), generator=g,
                         dtype=torch.uint8)
    toks = torch.randint(0, cfg.vocab, (1, n_tokens), generator=g)
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    return imgs, toks, state, noise


def gen_predict(ref, cfg, seed, n_tokens, lang_valid=None):
    W = make_weights(cfg, seed)
    model = build_ref_model(ref, cfg)
    load_weights(model, cfg, W)
    imgs, toks, state, noise = inputs(cfg, seed + 1, n_tokens)
    V = cfg.n_views
    # NormalizeImages (fluxvla/transforms/transform_images.py:339-360; that
    # module imports cv2/timm/torchvision, absent here, so its one-line
    # arithmetic is applied inline): (x - mean) / (std + 1e-8), CHW per view.
    x = imgs.float().permute(0, 3, 1, 2)
    mean = torch.tensor(cfg.img_mean)[:, None, None]
    std = torch.tensor(cfg.img_std)[:, None, None]
    pix = ((x - mean) / (std + 1e-8)).reshape(1, 3 * V, cfg.image_size,
                                                cfg.image_size)
    lang_masks = torch.ones(1, n_tokens, dtype=torch.bool)
    if lang_valid is not None:
        lang_masks[:, lang_valid:] = False
    img_masks = torch.ones(1, V, dtype=torch.bool)
    with torch.no_grad():
        embs, pad, att = model.embed_prefix(pix, toks, img_masks, lang_masks)
        out = model.predict_action(pix, toks, state, img_masks=img_masks,
                                   lang_masks=lang_masks, noise=noise.clone())
    return dict(cfg=vars(cfg), seed=seed, images=imgs, lang_tokens=toks,
                lang_masks=lang_masks, state=state, noise=noise,
                prefix_embs=embs, actions=out)


def gen_gemma_layer(ref, seed, S=16):
    """config[0] geometry (Gemma-2B layer, causal, positions 0..S-1)."""
    cfg = PI0Config(llm_layers=1)
    W = make_weights(cfg, seed, parts=('llm',))
    del W['llm.embed']
    g = ref.cg.ConditionGemmaModel(
        **{k: v for k, v in _gemma_cfg(cfg.llm_width, cfg.llm_mlp, 1, cfg,
                                       False).items() if k != 'type'})
    g = g.float().eval()
    g.config._attn_implementation = 'eager'
    sd = {}
    for ours, theirs in name_map(cfg).items():
        if ours.startswith('llm.') and ours != 'llm.embed':
            sd[theirs[len('llm_backbone.'):]] = W[ours].float()
    g.load_state_dict(sd, strict=False)
    x = torch.randn(1, S, cfg.llm_width,
                    generator=torch.Generator().manual_seed(seed + 7))
    with torch.no_grad():
        layer = g.layers[0]
        pos = torch.arange(S)[None]
        pe = g.rotary_emb(x, pos)
        causal = torch.full((S, S), torch.finfo(torch.float32).min).triu(1)
        out = layer(x, attention_mask=causal[None, None], position_ids=pos,
                    position_embeddings=pe)[0]
    return dict(seed=seed, x=x, out=out)


def real_width_cfg(pi05=False):
    """Production widths (SigLIP 1152 / head_dim 72 / MLP 4304, Gemma-2B 2048 /
    MLP 16384, expert 1024 / MLP 4096, 8 query heads of 256, 50 actions x 32)
    at one layer per tower, one 224x224 view and a 4096-token vocabulary, so
    that the reference runs in seconds on the CPU."""
    kw = dict(vis_layers=1, llm_layers=1, exp_layers=1, n_views=1,
              vocab=4096)
    return pi05_config(**kw) if pi05 else PI0Config(**kw)


def gen_predict_real_width(ref, pi05, seed, n_tokens):
    """predict_action at production widths: one SigLIP layer on one 256-token
    view, one Gemma-2B layer over the 256 + n_tokens prefix rows, ten Euler
    steps of one expert layer attending to that cached prefix.  Prefix
    embeddings are kept at every 16th row to keep the fixture small."""
    d = gen_predict(ref, real_width_cfg(pi05), seed, n_tokens)
    d['prefix_rows'] = torch.arange(0, d['prefix_embs'].shape[1], 16)
    d['prefix_embs'] = d['prefix_embs'][:, d['prefix_rows']].clone()
    return d


def main():
    ref = load_reference()
    torch.manual_seed(0)
    fixtures = {
        'pi0_tiny.pt': lambda: gen_predict(ref, tiny_cfg(False), 11, 5),
        'pi0_tiny_pad.pt': lambda: gen_predict(ref, tiny_cfg(False), 12, 6,
                                               lang_valid=3),
        'pi05_tiny.pt': lambda: gen_predict(ref, tiny_cfg(True), 13, 5),
        'gemma_layer_cfg0.pt': lambda: gen_gemma_layer(ref, 21),
        'pi0_real_width.pt': lambda: gen_predict_real_width(ref, False, 31,
                                                            16),
        'pi05_real_width.pt': lambda: gen_predict_real_width(ref, True, 32,
                                                             48),
    }
    for name in sys.argv[1:] or list(fixtures):
        torch.save(fixtures[name](), os.path.join(HERE, name))
        print('wrote', name)


if __name__ == '__main__':
    main()
