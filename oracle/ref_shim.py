"""Load the reference FluxVLA eager modules (unmodified) behind a small shim.

Test and measurement infrastructure only: the golden-vector generator
(tests/golden/make_golden.py) and the reference arm of bench.py use it to run
the reference's own PI0 / PI0.5 eager path on the CPU.  The product
(fluxvla_b200/) never imports it.

The reference package cannot be imported as a whole (its ``fluxvla/__init__``
pulls in jsonlines, mmengine, timm, wandb, ...) and the installed
transformers is 5.5 instead of the pinned 4.53.2 (requirements.txt:37), so
the modules the path needs are loaded by file path after installing:

* stub ``fluxvla.engines`` registries whose ``register_module()`` is the
  identity and whose ``build_*_from_cfg`` instantiate the known classes;
* three transformers-5.5 compatibility patches used by condition_gemma.py:
  ``transformers.utils.LossKwargs`` (an empty TypedDict),
  ``ROPE_INIT_FUNCTIONS['default']`` (inv_freq = theta^(-2i/d)) and
  ``DynamicCache.__getitem__`` returning (keys, values) of a layer;
* a stub ``timm.models.vision_transformer`` (only referenced by the FSDP
  policy of siglip_vit.py).

Where the reference lives: ``reference_root()`` takes ``$FLUXVLA_REF`` (a
source tree) or else the pip-installed copy under ``baseline/_ref`` of this
repository; there is no other default.
"""
from __future__ import annotations

import contextlib
import importlib.util
import os
import sys
import types
import typing

import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

from fluxvla_b200.config import PI0Config  # noqa: E402


def reference_root():
    """Directory holding the reference ``fluxvla`` package, or None."""
    for cand in (os.environ.get('FLUXVLA_REF'),
                 os.path.join(REPO, 'baseline', '_ref')):
        if cand and os.path.isfile(os.path.join(
                cand, 'fluxvla', 'models', 'vlas', 'pi0_flowmatching.py')):
            return cand
    return None


REF = None  # set by load_reference()


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


def load_reference(root=None):
    global REF
    REF = root or reference_root()
    if REF is None:
        raise FileNotFoundError('reference FluxVLA sources not found: set '
                                '$FLUXVLA_REF or install baseline/_ref')
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



@contextlib.contextmanager
def no_param_init():
    """Skip the random initialisation of nn.Linear / nn.Embedding /
    nn.LayerNorm while a reference model is constructed (every parameter is
    overwritten by load_weights afterwards; initialising 3.5 B parameters
    would take minutes on the CPU)."""
    import torch.nn as nn
    saved = [(c, c.reset_parameters) for c in (nn.Linear, nn.Embedding,
                                                nn.LayerNorm)]
    try:
        for c, _ in saved:
            c.reset_parameters = lambda self: None
        yield
    finally:
        for c, f in saved:
            c.reset_parameters = f
