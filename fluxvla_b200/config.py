"""Model dimensions of the PI0 / PI0.5 inference path.

Defaults follow the reference PI0 config
(configs/pi0/pi0_paligemma_libero_10_full_finetune.py:15-117): SigLIP
So400m/14 (27 layers, width 1152, MLP 4304, 16 heads), Gemma-2B prefix
(18 layers, width 2048, MLP 16384, 8 query heads, 1 KV head, head_dim 256) and
the Gemma action expert (18 layers, width 1024, MLP 4096).  The action-chunk
length is 50 (the benchmark workload) instead of the LIBERO config's 10.
"""
from __future__ import annotations

import dataclasses


@dataclasses.dataclass
class PI0Config:
    # vision tower
    vis_layers: int = 27
    vis_width: int = 1152
    vis_heads: int = 16
    vis_mlp: int = 4304
    patch: int = 14
    image_size: int = 224
    n_views: int = 3
    # Gemma prefix
    llm_layers: int = 18
    llm_width: int = 2048
    llm_mlp: int = 16384
    vocab: int = 257152
    # shared attention geometry (8 query heads, 1 KV head)
    heads: int = 8
    head_dim: int = 256
    # action expert
    exp_layers: int = 18
    exp_width: int = 1024
    exp_mlp: int = 4096
    # flow matching
    n_actions: int = 50
    action_dim: int = 32
    state_dim: int = 32
    num_steps: int = 10
    has_state_token: bool = True      # PI0: state_proj token; PI0.5: none
    adarms: bool = False              # PI0.5: adaRMSNorm expert
    # image normalisation (NormalizeImages,
    # configs/pi05/pi05_paligemma_libero_10_full_inference.py:263-268)
    img_mean: tuple = (123.515625, 116.04492188, 103.59375)
    img_std: tuple = (58.27148438, 57.02636719, 57.27539062)

    @property
    def tokens_per_view(self) -> int:
        return (self.image_size // self.patch) ** 2

    @property
    def n_suffix(self) -> int:
        return self.n_actions + (1 if self.has_state_token else 0)

    @property
    def patch_k(self) -> int:
        return 3 * self.patch * self.patch


def pi0_config(**kw) -> PI0Config:
    return PI0Config(**kw)


def pi05_config(**kw) -> PI0Config:
    kw.setdefault('has_state_token', False)
    kw.setdefault('adarms', True)
    return PI0Config(**kw)
