"""Generate golden vectors from the reference FluxVLA eager modules.

Run in a container that has the reference source tree (read-only) at
``$FLUXVLA_REF`` (default ``/root/reference``):

    python tests/golden/make_golden.py

The reference package cannot be imported as a whole here (its
``fluxvla/__init__`` pulls in jsonlines, mmengine, timm, wandb, ...), and the
installed transformers is 5.5 instead of the pinned 4.53.2
(requirements.txt:37).  So this script loads the reference *modules* it needs
by file path behind a small shim:

* stub ``fluxvla.engines`` registries whose ``register_module()`` is the
  identity and whose ``build_*_from_cfg`` instantiate the known classes;
* three transformers-5.5 compatibility patches used by condition_gemma.py:
  ``transformers.utils.LossKwargs`` (an empty TypedDict),
  ``ROPE_INIT_FUNCTIONS['default']`` (inv_freq = theta^(-2i/d)) and
  ``DynamicCache.__getitem__`` returning (keys, values) of a layer;
* a stub ``timm.models.vision_transformer`` (only referenced by the FSDP
  policy of siglip_vit.py).

The reference modules then run unmodified, in fp32 on the CPU, on weights
from ``fluxvla_b200.weights.make_weights`` (loaded into their state dicts by
name), and their outputs are saved as small ``.pt`` fixtures next to this
script.  The tests compare the oracle (``oracle/pi0_oracle.py``) with these
fixtures; they never read the reference tree.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types
import typing

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get('FLUXVLA_REF', '/root/reference')
sys.path.insert(0, REPO)

from fluxvla_b200.config import PI0Config, pi05_config  # noqa: E402
from fluxvla_b200.weights import make_weights  # noqa: E402


# ---------------------------------------------------------------------------
# shim
# ---------------------------------------------------------------------------

class _Registry:

    def __init__(self, name):
        self.name = name
        self.classes = {}

    def register_module(self, *a, **k):

        def deco(cls):
            self.classes[cls.__name__] = cls
            return cls

        if a and isinstance(a[0], type):
            return deco(a[0])
        return deco


def _install_shim():
    import transformers
    import transformers.utils as tu
    from transformers.cache_utils import DynamicCache
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    if not hasattr(tu, 'LossKwargs'):
        class LossKwargs(typing.TypedDict, total=False):
            pass
        tu.LossKwargs = LossKwargs

    def _default_rope(config, device=None, *a, **k):
        base = config.rope_theta if hasattr(config, 'rope_theta') else \
            config.rope_parameters['rope_theta']
        dim = getattr(config, 'head_dim', None) or (
            config.hidden_size // config.num_attention_heads)
        inv = 1.0 / (base**(torch.arange(0, dim, 2, dtype=torch.int64).to(
            device=device, dtype=torch.float) / dim))
        return inv, 1.0

    ROPE_INIT_FUNCTIONS.setdefault('default', _default_rope)
    if not hasattr(DynamicCache, '__getitem__'):
        DynamicCache.__getitem__ = lambda c, i: (c.layers[i].keys,
                                                 c.layers[i].values)

    timm = types.ModuleType('timm')
    timm_models = types.ModuleType('timm.models')
    vt = types.ModuleType('timm.models.vision_transformer')
    vt.Block = type('Block', (), {})
    vt.VisionTransformer = type('VisionTransformer', (), {})
    sys.modules.update({'timm': timm, 'timm.models': timm_models,
                        'timm.models.vision_transformer': vt})

    regs = {n: _Registry(n) for n in
            ['VLAS', 'LLM_BACKBONES', 'VISION_BACKBONES', 'PROJECTORS',
             'VLM_BACKBONES', 'HEADS']}

    def _builder(reg):

        def build(cfg):
            cfg = dict(cfg)
            t = cfg.pop('type')
            for r in regs.values():
                if t in r.classes:
                    return r.classes[t](**cfg)
            raise KeyError(t)

        return build

    pkgs = ['fluxvla', 'fluxvla.engines', 'fluxvla.engines.utils',
            'fluxvla.models', 'fluxvla.models.vlas', 'fluxvla.models.backbones',
            'fluxvla.models.backbones.llms', 'fluxvla.models.backbones.visions',
            'fluxvla.models.projectors']
    for p in pkgs:
        m = types.ModuleType(p)
        m.__path__ = [os.path.join(REF, *p.split('.'))]
        sys.modules[p] = m
    eng = sys.modules['fluxvla.engines']
    for n, r in regs.items():
        setattr(eng, n, r)
    for n in ['llm_backbone', 'projector', 'vision_backbone', 'vlm_backbone',
              'head']:
        setattr(eng, f'build_{n}_from_cfg', _builder(n))

    class _Overwatch:

        def __getattr__(self, k):
            return lambda *a, **kw: None

    eng.initialize_overwatch = lambda name: _Overwatch()
    ow = types.ModuleType('fluxvla.engines.utils.overwatch')
    ow.initialize_overwatch = eng.initialize_overwatch
    sys.modules['fluxvla.engines.utils.overwatch'] = ow
    losses = types.ModuleType('fluxvla.engines.losses')
    losses.reduce_action_bc_loss = lambda *a, **k: None
    sys.modules['fluxvla.engines.losses'] = losses
    return regs


def _load(modname, relpath):
    spec = importlib.util.spec_from_file_location(
        modname, os.path.join(REF, relpath))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[modname] = mod
    spec.loader.exec_module(mod)
    return mod


def load_reference():
    regs = _install_shim()
    mu = _load('fluxvla.engines.utils.model_utils',
               'fluxvla/engines/utils/model_utils.py')
    cg = _load('fluxvla.models.backbones.llms.condition_gemma',
               'fluxvla/models/backbones/llms/condition_gemma.py')
    _load('fluxvla.models.backbones.visions.configs',
          'fluxvla/models/backbones/visions/configs.py')
    _load('fluxvla.models.backbones.visions.base_vision',
          'fluxvla/models/backbones/visions/base_vision.py')
    _load('fluxvla.models.backbones.visions.siglip_vit',
          'fluxvla/models/backbones/visions/siglip_vit.py')
    _load('fluxvla.models.projectors.linear_projector',
          'fluxvla/models/projectors/linear_projector.py')
    _load('fluxvla.models.vlas.base_vla', 'fluxvla/models/vlas/base_vla.py')
    pi0 = _load('fluxvla.models.vlas.pi0_flowmatching',
                'fluxvla/models/vlas/pi0_flowmatching.py')
    pi05 = _load('fluxvla.models.vlas.pi05_flowmatching',
                 'fluxvla/models/vlas/pi05_flowmatching.py')
    return types.SimpleNamespace(mu=mu, cg=cg, pi0=pi0, pi05=pi05, regs=regs)


# ---------------------------------------------------------------------------
# model construction with our weights
# ---------------------------------------------------------------------------

def _gemma_cfg(width, mlp, layers, cfg, ada):
    return dict(type='ConditionGemmaModel', adarms_cond_dim=width if ada
                else None, head_dim=cfg.head_dim, hidden_size=width,
                intermediate_size=mlp, num_attention_heads=cfg.heads,
                num_hidden_layers=layers, num_key_value_heads=1,
                rms_norm_eps=1e-6, rope_theta=10000.0, use_adarms=ada,
                vocab_size=cfg.vocab, max_position_embeddings=8192)


def build_ref_model(ref, cfg: PI0Config):
    vis = dict(type='SigLIPViTBackbone', vision_backbone_id='siglip_224',
               vision_config=dict(
                   attention_dropout=0.0, hidden_act='gelu_pytorch_tanh',
                   hidden_size=cfg.vis_width, image_size=cfg.image_size,
                   intermediate_size=cfg.vis_mlp, layer_norm_eps=1e-6,
                   num_attention_heads=cfg.vis_heads, num_channels=3,
                   num_hidden_layers=cfg.vis_layers, patch_size=cfg.patch,
                   vision_use_head=False))
    E = cfg.exp_width
    kw = dict(
        llm_backbone=_gemma_cfg(cfg.llm_width, cfg.llm_mlp, cfg.llm_layers,
                                cfg, False),
        vision_backbone=vis,
        projector=dict(type='LinearProjector', in_dim=cfg.vis_width,
                       out_dim=cfg.llm_width),
        proj_width=E, n_action_steps=cfg.n_actions,
        action_in_proj=dict(type='LinearProjector', in_dim=cfg.action_dim,
                            out_dim=E),
        action_out_proj=dict(type='LinearProjector', in_dim=E,
                             out_dim=cfg.action_dim),
        max_action_dim=cfg.action_dim, num_steps=cfg.num_steps,
        llm_expert=_gemma_cfg(E, cfg.exp_mlp, cfg.exp_layers, cfg,
                              cfg.adarms),
        attention_implementation='eager')
    if cfg.adarms:
        kw.update(time_mlp_in=dict(type='LinearProjector', in_dim=E,
                                   out_dim=E),
                  time_mlp_out=dict(type='LinearProjector', in_dim=E,
                                    out_dim=E))
        model = ref.pi05.PI05FlowMatching(**kw)
    else:
        kw.update(state_proj=dict(type='LinearProjector',
                                  in_dim=cfg.state_dim, out_dim=E),
                  action_time_mlp_in=dict(type='LinearProjector',
                                          in_dim=2 * E, out_dim=E),
                  action_time_mlp_out=dict(type='LinearProjector', in_dim=E,
                                           out_dim=E))
        model = ref.pi0.PI0FlowMatching(**kw)
    return model.float().eval()


def name_map(cfg: PI0Config):
    """our weight name -> reference state_dict key (the product's map)."""
    from fluxvla_b200.loader import reference_name_map
    return reference_name_map(cfg)


def load_weights(model, cfg, W):
    sd = model.state_dict()
    nm = name_map(cfg)
    new = {}
    for ours, theirs in nm.items():
        assert theirs in sd, theirs
        assert sd[theirs].shape == W[ours].shape, (theirs, sd[theirs].shape,
                                                   W[ours].shape)
        new[theirs] = W[ours].float()
    missing = [k for k in sd if k not in new]
    # the reference keeps an unused copy of rotary inv_freq buffers only
    assert all('inv_freq' in k or 'position_ids' in k or
               'llm_expert.embed_tokens' in k for k in missing), \
        missing
    model.load_state_dict(new, strict=False)


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


def main():
    ref = load_reference()
    torch.manual_seed(0)
    fixtures = {
        'pi0_tiny.pt': gen_predict(ref, tiny_cfg(False), 11, 5),
        'pi0_tiny_pad.pt': gen_predict(ref, tiny_cfg(False), 12, 6,
                                       lang_valid=3),
        'pi05_tiny.pt': gen_predict(ref, tiny_cfg(True), 13, 5),
        'gemma_layer_cfg0.pt': gen_gemma_layer(ref, 21),
    }
    for name, d in fixtures.items():
        torch.save(d, os.path.join(HERE, name))
        print('wrote', name)


if __name__ == '__main__':
    main()
