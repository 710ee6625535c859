"""PI0.5 prompt construction: state discretisation and the prompt string.

Restates the PI0.5 prompter of the reference
(fluxvla/transforms/prompters.py:290-314, after openpi's
``PaligemmaTokenizer.tokenize``):

* the state vector (already normalised to [-1, 1]) is zero-padded to
  ``max_state_dim`` (32);
* each entry is binned into 256 uniform bins over [-1, 1]: bin index =
  ``np.digitize(x, np.linspace(-1, 1, 257)[:-1]) - 1``, i.e. the number of
  left bin edges ``e_j = -1 + 2j/256`` (j = 0..255) that are <= x, minus one.
  Values below -1 give -1 and values >= 1 - 2/256 give 255, exactly as the
  reference (no clipping);
* the prompt is ``'Task: {task}, State: {s_0 s_1 ... s_31};\\nAction: '`` with
  the task text stripped, underscores and newlines replaced by spaces.

Turning the prompt into token ids needs the PaliGemma sentencepiece model,
which is not part of the reference tree; ``tokenize_prompt`` takes it as an
argument.  config[3] feeds the resulting 80 token ids (48 text + 32 state)
to ``PI0EngineB200.predict_action``, whose embedding gather runs on the GPU.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np

N_BINS = 256


def bin_edges(n_bins: int = N_BINS) -> np.ndarray:
    """Left edges of the n_bins uniform bins over [-1, 1] (float64, as
    np.linspace computes them)."""
    return np.linspace(-1.0, 1.0, n_bins + 1)[:-1]


def discretize_state(state: Sequence[float], max_state_dim: int = 32,
                     n_bins: int = N_BINS) -> np.ndarray:
    """Pad the state to max_state_dim and return its int64 bin indices."""
    s = np.asarray(state, dtype=np.float64).reshape(-1)
    if s.shape[0] > max_state_dim:
        raise ValueError(f'state has {s.shape[0]} entries, more than '
                         f'max_state_dim={max_state_dim}')
    padded = np.zeros(max_state_dim, dtype=np.float64)
    padded[:s.shape[0]] = s
    # count of edges <= x (right-closed search) minus one; NaN compares
    # false against every edge and lands past the last bin, like digitize
    edges = bin_edges(n_bins)
    idx = np.searchsorted(edges, padded, side='right').astype(np.int64) - 1
    idx[np.isnan(padded)] = n_bins - 1
    return idx


def format_prompt(task: str, state_bins: Sequence[int]) -> str:
    """The PI0.5 prompt string for a task description and state bins."""
    cleaned = task.strip().replace('_', ' ').replace('\n', ' ')
    state_str = ' '.join(str(int(b)) for b in state_bins)
    return f'Task: {cleaned}, State: {state_str};\nAction: '


def pi05_prompt(task: str, state: Optional[Sequence[float]],
                max_state_dim: int = 32) -> str:
    """Prompt of one PI0.5 request (state required, as in the reference)."""
    if state is None:
        raise ValueError('State is required for PI05')
    return format_prompt(task, discretize_state(state, max_state_dim))


def tokenize_prompt(prompt: str, sp_model, max_len: int,
                    add_bos: bool = True) -> tuple:
    """Token ids and pad mask of a prompt with a sentencepiece processor
    (``sp_model.encode(str) -> List[int]``); right-padded with 0 to max_len,
    truncated beyond it.  The PaliGemma tokenizer model must be supplied by
    the caller."""
    ids: List[int] = list(sp_model.encode(prompt))
    if add_bos:
        ids = [sp_model.bos_id()] + ids
    ids = ids[:max_len]
    mask = [True] * len(ids) + [False] * (max_len - len(ids))
    ids = ids + [0] * (max_len - len(ids))
    return np.asarray(ids, dtype=np.int64), np.asarray(mask, dtype=bool)
