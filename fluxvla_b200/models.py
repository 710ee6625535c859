"""Model-level drop-ins: PI0FlowMatchingB200 / PI05FlowMatchingB200.

The reference runners call ``vla.predict_action(images, lang_tokens, states,
img_masks, lang_masks, noise)`` on a model built from its config
(fluxvla/models/vlas/pi0_flowmatching.py:702-785,
pi05_flowmatching.py:26-127; callers libero_eval_runner.py:308,
zmq_server.py:239).  The classes here subclass those eager classes, keep
their constructor, weights (``from_pretrained`` with its ``name_mapping``)
and every other method, and replace ``predict_action`` with the B200 engine:

* ``images``: the reference's normalised float pixels, a tensor
  [B, 3*views, H, W] or a list of per-view [B, 3, H, W] tensors; they are
  patchified on the device (``fvb_patchify_f32``).
* ``lang_tokens`` [B, L], ``states`` [B, S], optional ``img_masks``
  [B, views], ``lang_masks`` [B, L] and ``noise`` [B, n_actions, action_dim]
  (sampled N(0, 1) when absent, as ``sample_noise``).
* returns ``[B, n_actions, action_dim]`` float32 on the device of
  ``states``.  A batch runs request by request (one CUDA-graph replay each);
  the engine is built on first use for each (views, prompt length), from the
  module's own state dict (``weights_from_state_dict``, cast to bf16 once).

Not supported on this path (raises): a caller-supplied
``past_key_values`` and the real-time-chunking arguments (``prev_actions``
with ``prefix_len`` / ``rtc_config``); those callers keep the eager class.

``make_b200_class(base)`` derives the drop-in from any PI0 / PI0.5 eager
class object (e.g. one loaded by file path); when the reference package is
importable the two named classes are created at import and registered in
its ``VLAS`` registry.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from .config import PI0Config


def config_from_module(model, n_views: int) -> PI0Config:
    """PI0Config of an eager PI0 / PI0.5 model (its backbone configs)."""
    lc = model.llm_backbone.config
    ec = model.llm_expert.config
    vc = model.vision_backbone.vision.config
    ada = bool(getattr(ec, 'use_adarms', False))
    return PI0Config(
        vis_layers=vc.num_hidden_layers, vis_width=vc.hidden_size,
        vis_heads=vc.num_attention_heads, vis_mlp=vc.intermediate_size,
        patch=vc.patch_size, image_size=vc.image_size, n_views=n_views,
        llm_layers=lc.num_hidden_layers, llm_width=lc.hidden_size,
        llm_mlp=lc.intermediate_size, vocab=lc.vocab_size,
        heads=lc.num_attention_heads, head_dim=lc.head_dim,
        exp_layers=ec.num_hidden_layers, exp_width=ec.hidden_size,
        exp_mlp=ec.intermediate_size, n_actions=model.n_action_steps,
        action_dim=model.max_action_dim,
        state_dim=(model.state_proj.projector.in_features
                   if getattr(model, 'state_proj', None) is not None
                   else PI0Config.state_dim),
        num_steps=model.num_steps, has_state_token=not ada, adarms=ada)


class B200PredictMixin:
    """predict_action on the B200 engine (see module docstring)."""

    b200_device: str = 'cuda'

    def _b200_engine(self, n_views: int, n_tokens: int):
        from .engine import PI0EngineB200
        from .loader import weights_from_state_dict
        cache: Dict[Tuple[int, int], object] = self.__dict__.setdefault(
            '_b200_engines', {})
        key = (n_views, n_tokens)
        if key not in cache:
            cfg = config_from_module(self, n_views)
            sd = {k: v.detach() for k, v in self.state_dict().items()}
            W = weights_from_state_dict(sd, cfg, device=self.b200_device)
            cache[key] = PI0EngineB200(
                cfg, W, prefix_len=n_views * cfg.tokens_per_view + n_tokens,
                device=self.b200_device, image_format='f32')
        return cache[key]

    @torch.no_grad()
    def predict_action(self, images, lang_tokens, states, img_masks=None,
                       lang_masks=None, past_key_values=None, noise=None,
                       prev_actions=None, prefix_len: int = 0,
                       rtc_config: Optional[dict] = None, *args, **kwargs):
        if past_key_values is not None:
            raise NotImplementedError(
                'B200 predict_action computes its own prefix cache')
        if prev_actions is not None and prefix_len > 0 and rtc_config:
            raise NotImplementedError(
                'real-time chunking is not on the B200 path')
        if isinstance(images, (list, tuple)):
            images = torch.cat(list(images), dim=1)
        B = states.shape[0]
        V = images.shape[1] // 3
        L = lang_tokens.shape[1]
        eng = self._b200_engine(V, L)
        if noise is None:
            noise = torch.randn(B, eng.A, eng.cfg.action_dim,
                                device=states.device)
        outs = []
        for b in range(B):
            px = images[b].reshape(V, 3, *images.shape[2:]).float()
            outs.append(eng.predict_action(
                px.to(eng.dev).contiguous(), lang_tokens[b:b + 1],
                states[b:b + 1].float(),
                img_masks=None if img_masks is None else img_masks[b:b + 1],
                lang_masks=None if lang_masks is None else
                lang_masks[b:b + 1],
                noise=noise[b:b + 1].float()))
        return torch.cat(outs).to(states.device)


def make_b200_class(base, name: Optional[str] = None):
    """The drop-in subclass of an eager PI0 / PI0.5 class."""
    return type(name or base.__name__ + 'B200', (B200PredictMixin, base),
                {'__doc__': f'{base.__name__} with predict_action on the '
                            'B200 engine (fluxvla_b200.models).'})


def to_b200(model):
    """Turn an existing eager PI0 / PI0.5 instance into its drop-in (same
    module tree and weights, B200 predict_action)."""
    model.__class__ = make_b200_class(type(model))
    return model


try:  # the reference package, when it is importable as a package
    from fluxvla.engines import VLAS as _VLAS  # type: ignore
    from fluxvla.models.vlas.pi0_flowmatching import \
        PI0FlowMatching as _PI0  # type: ignore
    from fluxvla.models.vlas.pi05_flowmatching import \
        PI05FlowMatching as _PI05  # type: ignore
    PI0FlowMatchingB200 = _VLAS.register_module()(
        make_b200_class(_PI0, 'PI0FlowMatchingB200'))
    PI05FlowMatchingB200 = _VLAS.register_module()(
        make_b200_class(_PI05, 'PI05FlowMatchingB200'))
except Exception:  # noqa: BLE001 - not importable: make_b200_class/to_b200
    PI0FlowMatchingB200 = PI05FlowMatchingB200 = None
