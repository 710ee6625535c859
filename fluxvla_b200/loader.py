"""Weights from a FluxVLA PI0 / PI0.5 checkpoint.

The reference loads `model.safetensors` into its eager modules through
`BaseVLA.from_pretrained` (fluxvla/models/vlas/base_vla.py:190-288, with its
per-model `name_mapping`); the Triton inference classes then re-pack those
tensors (e.g. condition_gemma_inference.py:46-111).  Here the checkpoint's
state_dict names map straight onto this library's weight names (the tensors
keep the nn.Linear / conv / embedding shapes of the eager modules), are cast
to bf16 once, and `PI0EngineB200` packs them for the kernels.

`read_safetensors` parses the safetensors container itself (an 8-byte
little-endian header length, a JSON header of dtype / shape / byte offsets,
then the raw little-endian tensor bytes), so no third-party reader is
needed; sharded checkpoints with a `model.safetensors.index.json` are
followed file by file.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict, Iterable, Optional

import numpy as np
import torch

from .config import PI0Config
from .weights import weight_shapes

_DTYPES = {
    'F32': (np.float32, torch.float32),
    'F16': (np.float16, torch.float16),
    'BF16': (np.uint16, torch.bfloat16),  # reinterpreted after loading
    'F64': (np.float64, torch.float64),
    'I64': (np.int64, torch.int64),
    'I32': (np.int32, torch.int32),
    'U8': (np.uint8, torch.uint8),
}


def reference_name_map(cfg: PI0Config) -> Dict[str, str]:
    """This library's weight name -> the reference model's state_dict key
    (PI0FlowMatching / PI05FlowMatching module tree: vision_backbone.vision
    (HF SiglipVisionModel), projector, llm_backbone and llm_expert
    (ConditionGemmaModel), the action / state / time projectors)."""
    m = {'vision.patch_w':
         'vision_backbone.vision.vision_model.embeddings.patch_embedding.weight',
         'vision.patch_b':
         'vision_backbone.vision.vision_model.embeddings.patch_embedding.bias',
         'vision.pos': 'vision_backbone.vision.vision_model.embeddings.'
         'position_embedding.weight',
         'vision.post_w':
         'vision_backbone.vision.vision_model.post_layernorm.weight',
         'vision.post_b':
         'vision_backbone.vision.vision_model.post_layernorm.bias',
         'proj_w': 'projector.projector.weight',
         'proj_b': 'projector.projector.bias',
         'llm.embed': 'llm_backbone.embed_tokens.weight',
         'llm.norm': 'llm_backbone.norm.weight',
         'action_in_w': 'action_in_proj.projector.weight',
         'action_in_b': 'action_in_proj.projector.bias',
         'action_out_w': 'action_out_proj.projector.weight',
         'action_out_b': 'action_out_proj.projector.bias'}
    for i in range(cfg.vis_layers):
        s = f'vision_backbone.vision.vision_model.encoder.layers.{i}.'
        p = f'vision.l{i}.'
        for a, b in [('ln1', 'layer_norm1'), ('ln2', 'layer_norm2')]:
            m[p + a + '_w'] = s + b + '.weight'
            m[p + a + '_b'] = s + b + '.bias'
        for a, b in [('q', 'q_proj'), ('k', 'k_proj'), ('v', 'v_proj'),
                     ('o', 'out_proj')]:
            m[p + a + '_w'] = s + 'self_attn.' + b + '.weight'
            m[p + a + '_b'] = s + 'self_attn.' + b + '.bias'
        for a in ['fc1', 'fc2']:
            m[p + a + '_w'] = s + 'mlp.' + a + '.weight'
            m[p + a + '_b'] = s + 'mlp.' + a + '.bias'

    def gemma(ours, theirs, layers, ada):
        for i in range(layers):
            s, p = f'{theirs}.layers.{i}.', f'{ours}l{i}.'
            for a in 'qkvo':
                m[p + a + '_w'] = s + f'self_attn.{a}_proj.weight'
            for a in ['gate', 'up', 'down']:
                m[p + a + '_w'] = s + f'mlp.{a}_proj.weight'
            for a, b in [('in_norm', 'input_layernorm'),
                         ('post_norm', 'post_attention_layernorm')]:
                if ada:
                    m[p + a + '_dense_w'] = s + b + '.dense.weight'
                    m[p + a + '_dense_b'] = s + b + '.dense.bias'
                else:
                    m[p + a] = s + b + '.weight'
        if ada:
            m[ours + 'norm_dense_w'] = theirs + '.norm.dense.weight'
            m[ours + 'norm_dense_b'] = theirs + '.norm.dense.bias'
        else:
            m[ours + 'norm'] = theirs + '.norm.weight'

    gemma('llm.', 'llm_backbone', cfg.llm_layers, False)
    gemma('exp.', 'llm_expert', cfg.exp_layers, cfg.adarms)
    if cfg.adarms:
        for a in ['in', 'out']:
            m[f'time_{a}_w'] = f'time_mlp_{a}.projector.weight'
            m[f'time_{a}_b'] = f'time_mlp_{a}.projector.bias'
    else:
        m['state_proj_w'] = 'state_proj.projector.weight'
        m['state_proj_b'] = 'state_proj.projector.bias'
        for a in ['in', 'out']:
            m[f'action_time_{a}_w'] = f'action_time_mlp_{a}.projector.weight'
            m[f'action_time_{a}_b'] = f'action_time_mlp_{a}.projector.bias'
    return m


def _read_one(path: str, keys: Optional[set] = None) -> Dict[str, torch.Tensor]:
    with open(path, 'rb') as f:
        (n,) = struct.unpack('<Q', f.read(8))
        header = json.loads(f.read(n))
    base = 8 + n
    raw = np.memmap(path, dtype=np.uint8, mode='r')
    out = {}
    for name, info in header.items():
        if name == '__metadata__' or (keys is not None and name not in keys):
            continue
        dt = info['dtype']
        if dt not in _DTYPES:
            raise ValueError(f'{path}: {name}: unsupported dtype {dt}')
        npdt, tdt = _DTYPES[dt]
        a, b = info['data_offsets']
        arr = np.frombuffer(raw[base + a:base + b], dtype=npdt).reshape(info['shape'])
        t = torch.from_numpy(arr.copy())
        if dt == 'BF16':
            t = t.view(torch.bfloat16)
        out[name] = t
    return out


def _header(path: str) -> dict:
    with open(path, 'rb') as f:
        (n,) = struct.unpack('<Q', f.read(8))
        return json.loads(f.read(n))


def safetensors_index(path: str) -> Dict[str, str]:
    """tensor name -> file holding it, for a .safetensors file, a
    `*.safetensors.index.json` (its weight_map) or a directory (its
    model.safetensors.index.json, its model.safetensors, or else every
    .safetensors file in it, as BaseVLA.from_pretrained reads a directory,
    base_vla.py:199-207).  Only headers are read."""
    if os.path.isdir(path):
        idx = os.path.join(path, 'model.safetensors.index.json')
        one = os.path.join(path, 'model.safetensors')
        if os.path.exists(idx):
            path = idx
        elif os.path.exists(one):
            path = one
        else:
            out = {}
            for fn in sorted(os.listdir(path)):
                if fn.endswith('.safetensors'):
                    fp = os.path.join(path, fn)
                    out.update({k: fp for k in _header(fp)
                                if k != '__metadata__'})
            return out
    if path.endswith('.json'):
        with open(path) as f:
            wmap = json.load(f)['weight_map']
        root = os.path.dirname(path)
        return {k: os.path.join(root, fn) for k, fn in wmap.items()}
    return {k: path for k in _header(path) if k != '__metadata__'}


def read_safetensors(path: str, keys: Optional[Iterable[str]] = None
                     ) -> Dict[str, torch.Tensor]:
    """Tensors of a .safetensors file, of every shard listed by a
    `*.safetensors.index.json`, or of the checkpoint in a directory (see
    safetensors_index).  `keys` restricts the result (and the bytes read) to
    those names."""
    want = None if keys is None else set(keys)
    index = safetensors_index(path)
    files = sorted({fn for k, fn in index.items()
                    if want is None or k in want})
    out = {}
    for fn in files:
        out.update(_read_one(fn, want))
    return out


def write_safetensors(path: str, tensors: Dict[str, torch.Tensor]) -> None:
    """Minimal writer (f32 / f16 / bf16 / int tensors) for tests and tools."""
    rev = {tdt: name for name, (_, tdt) in _DTYPES.items()}
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        dt = rev[t.dtype]
        b = (t.view(torch.uint16) if t.dtype == torch.bfloat16 else t).numpy().tobytes()
        header[name] = {'dtype': dt, 'shape': list(t.shape),
                        'data_offsets': [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header).encode()
    hj += b' ' * (-len(hj) % 8)
    with open(path, 'wb') as f:
        f.write(struct.pack('<Q', len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def weights_from_state_dict(sd: Dict[str, torch.Tensor], cfg: PI0Config,
                            parts: Iterable[str] = ('vision', 'llm', 'exp', 'heads'),
                            strip_prefix: str = '',
                            device='cpu') -> Dict[str, torch.Tensor]:
    """Reference state_dict -> this library's bf16 weights for `parts`.
    Keys may carry a common prefix (e.g. 'vla.' or 'module.'), removed with
    `strip_prefix`.  Raises KeyError for missing tensors and ValueError for
    shape mismatches, naming every offending tensor."""
    if strip_prefix:
        sd = {k[len(strip_prefix):] if k.startswith(strip_prefix) else k: v
              for k, v in sd.items()}
    nm = reference_name_map(cfg)
    out, missing, bad = {}, [], []
    for name, shape, _ in weight_shapes(cfg, parts):
        key = nm[name]
        if key not in sd:
            missing.append(key)
            continue
        t = sd[key]
        if tuple(t.shape) != tuple(shape):
            bad.append(f'{key}: {tuple(t.shape)} != {tuple(shape)}')
            continue
        out[name] = t.to(device=device, dtype=torch.bfloat16)
    if missing:
        raise KeyError(f'{len(missing)} tensors missing from the checkpoint: '
                       f'{missing[:8]}{" ..." if len(missing) > 8 else ""}')
    if bad:
        raise ValueError('shape mismatch: ' + '; '.join(bad[:8]))
    return out


# The reference configs' checkpoint name mappings for openpi checkpoints
# (configs/pi0/pi0_paligemma_libero_10_full_finetune.py:106-118 and
# configs/pi05/pi05_paligemma_aloha+ur_4090_full_finetune.py:104-116): a
# substring of the model's parameter name -> its replacement in the
# checkpoint.  The entries are data that must equal the reference's to read
# the same files.
PI0_NAME_MAPPING = {
    'llm_backbone': 'paligemma_with_expert.paligemma.model.language_model',
    'vision_backbone.vision':
    'paligemma_with_expert.paligemma.model.vision_tower',
    'projector.projector':
    'paligemma_with_expert.paligemma.model.multi_modal_projector.linear',
    'llm_expert': 'paligemma_with_expert.gemma_expert.model',
    'action_time_mlp_in.projector': 'action_time_mlp_in',
    'action_time_mlp_out.projector': 'action_time_mlp_out',
    'state_proj.projector': 'state_proj',
    'action_in_proj.projector': 'action_in_proj',
    'action_out_proj.projector': 'action_out_proj',
    'llm_backbone.embed_tokens': 'paligemma_with_expert.paligemma.lm_head',
}
PI05_NAME_MAPPING = {
    k: v for k, v in PI0_NAME_MAPPING.items()
    if not k.startswith(('action_time_mlp', 'state_proj'))}
PI05_NAME_MAPPING.update({'time_mlp_in.projector': 'time_mlp_in',
                          'time_mlp_out.projector': 'time_mlp_out'})


def default_name_mapping(cfg: PI0Config) -> Dict[str, str]:
    return dict(PI05_NAME_MAPPING if cfg.adarms else PI0_NAME_MAPPING)


def mapped_key(model_name: str, name_mapping: Dict[str, str],
               available) -> Optional[str]:
    """The checkpoint key of one model parameter under a substring mapping,
    following BaseVLA.from_pretrained (base_vla.py:226-262): every mapping
    entry whose key occurs in the name proposes name.replace(key, value);
    the proposal present in the checkpoint wins; two present proposals are
    an error; none is a miss (None)."""
    hit = None
    for key, val in name_mapping.items():
        if key in model_name:
            cand = model_name.replace(key, val)
            if cand not in available:
                continue
            if hit is not None and hit != cand:
                raise ValueError(f"parameter '{model_name}' matched several "
                                 f"checkpoint keys: '{hit}', '{cand}'")
            hit = cand
    return hit


def read_checkpoint(path: str, keys: Optional[Iterable[str]] = None
                    ) -> Dict[str, torch.Tensor]:
    """Tensors of a checkpoint: safetensors file / sharded index /
    directory of .safetensors files, or a torch .pt / .pth file holding a
    state dict or {'model': state dict} (base_vla.py:190-222)."""
    if path.endswith(('.pt', '.pth')):
        ck = torch.load(path, map_location='cpu', weights_only=True)
        if isinstance(ck, dict) and 'model' in ck and isinstance(
                ck['model'], dict):
            ck = ck['model']
        if not isinstance(ck, dict):
            raise ValueError(f'{path}: not a state dict')
        if keys is not None:
            ks = set(keys)
            ck = {k: v for k, v in ck.items() if k in ks}
        return ck
    if path.endswith('.safetensors') or os.path.isdir(path) or \
            path.endswith('.json'):
        return read_safetensors(path, keys)
    raise ValueError(f'unsupported checkpoint format: {path}')


def checkpoint_keys(path: str) -> set:
    """Names of every tensor in a checkpoint (reads headers only for
    safetensors)."""
    if path.endswith(('.pt', '.pth')):
        return set(read_checkpoint(path).keys())
    return set(safetensors_index(path).keys())


def load_pretrained(path: str, cfg: PI0Config,
                    parts: Iterable[str] = ('vision', 'llm', 'exp', 'heads'),
                    strip_prefix: str = '', device='cpu',
                    name_mapping: Optional[Dict[str, str]] = None
                    ) -> Dict[str, torch.Tensor]:
    """Checkpoint (safetensors file / index / directory, or .pt / .pth) ->
    weights for PI0EngineB200.

    Without ``name_mapping`` the checkpoint carries the reference model's own
    state_dict names (optionally under ``strip_prefix``).  With one (e.g.
    ``default_name_mapping(cfg)`` for openpi ``pi0_base`` / ``pi05_base``
    checkpoints) each model name is translated as the reference's
    ``from_pretrained`` does; ``name_mapping='auto'`` picks the config's
    default mapping when the checkpoint uses openpi names."""
    nm = reference_name_map(cfg)
    names = [n for n, _, _ in weight_shapes(cfg, parts)]
    if name_mapping == 'auto':
        avail = checkpoint_keys(path)
        direct = sum((strip_prefix + nm[n]) in avail for n in names)
        name_mapping = None if direct == len(names) else \
            default_name_mapping(cfg)
    if not name_mapping:
        keys = [strip_prefix + nm[n] for n in names]
        sd = read_checkpoint(path, keys)
        return weights_from_state_dict(sd, cfg, parts, strip_prefix, device)
    avail = checkpoint_keys(path)
    want, missing = {}, []
    for n in names:
        k = mapped_key(nm[n], name_mapping, avail)
        if k is None:
            missing.append(nm[n])
        else:
            want[nm[n]] = k
    if missing:
        raise KeyError(f'{len(missing)} parameters not found in the '
                       f'checkpoint under the name mapping: {missing[:8]}'
                       f'{" ..." if len(missing) > 8 else ""}')
    raw = read_checkpoint(path, set(want.values()))
    sd = {ours: raw[theirs] for ours, theirs in want.items()}
    return weights_from_state_dict(sd, cfg, parts, '', device)
