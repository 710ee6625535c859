"""Checkpoint loading (fluxvla_b200.loader): the safetensors container, the
reference-name mapping for PI0 and PI0.5, sharded indexes, prefixes and the
errors for incomplete checkpoints.  CPU only."""
import json
import os

import pytest
import torch

from fluxvla_b200.config import PI0Config, pi05_config
from fluxvla_b200.loader import (load_pretrained, read_safetensors,
                                 reference_name_map, weights_from_state_dict,
                                 write_safetensors)
from fluxvla_b200.weights import make_weights, weight_shapes


def tiny(pi05=False):
    kw = dict(vis_layers=2, vis_width=32, vis_heads=2, vis_mlp=48, patch=14,
              image_size=28, n_views=2, llm_layers=2, llm_width=64,
              llm_mlp=96, vocab=97, heads=2, head_dim=16, exp_layers=2,
              exp_width=32, exp_mlp=64, n_actions=4, action_dim=8,
              state_dim=8, num_steps=10)
    return pi05_config(**kw) if pi05 else PI0Config(**kw)


def reference_state_dict(cfg, W, dtype=torch.float32, prefix=''):
    nm = reference_name_map(cfg)
    sd = {prefix + nm[k]: v.to(dtype) for k, v in W.items()}
    # tensors the reference keeps that this path does not use
    sd[prefix + 'llm_backbone.layers.0.self_attn.rotary_emb.inv_freq'] = torch.ones(4)
    return sd


@pytest.mark.parametrize('pi05', [False, True])
@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_round_trip_through_safetensors(tmp_path, pi05, dtype):
    cfg = tiny(pi05)
    W = make_weights(cfg, seed=3)
    path = str(tmp_path / 'model.safetensors')
    write_safetensors(path, reference_state_dict(cfg, W, dtype))
    got = load_pretrained(path, cfg)
    assert set(got) == set(W)
    for k, v in W.items():
        assert got[k].dtype == torch.bfloat16 and got[k].shape == v.shape
        assert torch.equal(got[k], v.to(dtype).to(torch.bfloat16)), k


def test_sharded_index_and_prefix(tmp_path):
    cfg = tiny()
    W = make_weights(cfg, seed=4)
    sd = reference_state_dict(cfg, W, prefix='vla.')
    keys = sorted(sd)
    half = len(keys) // 2
    shards = {'model-00001-of-00002.safetensors': keys[:half],
              'model-00002-of-00002.safetensors': keys[half:]}
    wmap = {}
    for fn, ks in shards.items():
        write_safetensors(str(tmp_path / fn), {k: sd[k] for k in ks})
        wmap.update({k: fn for k in ks})
    with open(tmp_path / 'model.safetensors.index.json', 'w') as f:
        json.dump({'metadata': {}, 'weight_map': wmap}, f)
    got = load_pretrained(str(tmp_path), cfg, strip_prefix='vla.')
    for k, v in W.items():
        assert torch.equal(got[k], v), k
    # only the expert part: only the expert's tensors are read
    exp = load_pretrained(str(tmp_path), cfg, parts=('exp',), strip_prefix='vla.')
    assert set(exp) == {n for n, _, _ in weight_shapes(cfg, ('exp',))}


def test_header_and_dtypes(tmp_path):
    t = {'a': torch.arange(6, dtype=torch.float32).reshape(2, 3),
         'b': torch.tensor([1.5, -2.25], dtype=torch.bfloat16),
         'c': torch.tensor([7, 8], dtype=torch.int64)}
    p = str(tmp_path / 'x.safetensors')
    write_safetensors(p, t)
    with open(p, 'rb') as f:
        n = int.from_bytes(f.read(8), 'little')
        hdr = json.loads(f.read(n))
    assert hdr['b']['dtype'] == 'BF16' and hdr['a']['shape'] == [2, 3]
    got = read_safetensors(p)
    for k in t:
        assert got[k].dtype == t[k].dtype and torch.equal(got[k], t[k])
    assert set(read_safetensors(p, keys=['c'])) == {'c'}


def test_missing_and_mismatched_tensors():
    cfg = tiny()
    W = make_weights(cfg, seed=5)
    sd = reference_state_dict(cfg, W)
    nm = reference_name_map(cfg)
    del sd[nm['llm.l1.down_w']]
    with pytest.raises(KeyError, match='down_proj'):
        weights_from_state_dict(sd, cfg)
    sd = reference_state_dict(cfg, W)
    sd[nm['proj_w']] = torch.zeros(3, 3)
    with pytest.raises(ValueError, match='projector'):
        weights_from_state_dict(sd, cfg)


def _openpi_state_dict(cfg, W, dtype=torch.float32):
    """The reference state dict renamed as an openpi checkpoint stores it
    (the inverse of the config's name_mapping), with the token embedding
    under the lm_head name only."""
    from fluxvla_b200.loader import default_name_mapping
    nm = reference_name_map(cfg)
    mp = default_name_mapping(cfg)
    sd = {}
    for ours, theirs in nm.items():
        if ours not in W:
            continue
        if theirs == 'llm_backbone.embed_tokens.weight':
            key = 'paligemma_with_expert.paligemma.lm_head.weight'
        else:
            key = theirs
            for k in sorted(mp, key=len, reverse=True):
                if k in theirs and k != 'llm_backbone.embed_tokens':
                    key = theirs.replace(k, mp[k])
                    break
        sd[key] = W[ours].to(dtype)
    return sd


@pytest.mark.parametrize('pi05', [False, True])
def test_openpi_names_through_name_mapping(tmp_path, pi05):
    cfg = tiny(pi05)
    W = make_weights(cfg, seed=5)
    sd = _openpi_state_dict(cfg, W)
    assert any(k.startswith('paligemma_with_expert.gemma_expert.model.')
               for k in sd)
    path = str(tmp_path / 'model.safetensors')
    write_safetensors(path, sd)
    from fluxvla_b200.loader import default_name_mapping
    for mapping in (default_name_mapping(cfg), 'auto'):
        got = load_pretrained(path, cfg, name_mapping=mapping)
        assert set(got) == set(W)
        for k in W:
            assert torch.equal(got[k], W[k].bfloat16()), k
    with pytest.raises(KeyError):
        load_pretrained(path, cfg)  # the model's own names are absent


@pytest.mark.parametrize('wrap', [False, True])
def test_torch_pt_checkpoint(tmp_path, wrap):
    cfg = tiny()
    W = make_weights(cfg, seed=6)
    sd = reference_state_dict(cfg, W)
    path = str(tmp_path / 'ckpt.pth')
    torch.save({'model': sd, 'step': 3} if wrap else sd, path)
    got = load_pretrained(path, cfg)
    for k in W:
        assert torch.equal(got[k], W[k].bfloat16()), k
    from fluxvla_b200.loader import default_name_mapping
    path2 = str(tmp_path / 'openpi.pt')
    torch.save(_openpi_state_dict(cfg, W), path2)
    got = load_pretrained(path2, cfg, name_mapping=default_name_mapping(cfg))
    assert torch.equal(got['exp.l0.q_w'], W['exp.l0.q_w'].bfloat16())


def test_directory_of_unindexed_shards(tmp_path):
    cfg = tiny()
    W = make_weights(cfg, seed=7)
    sd = reference_state_dict(cfg, W)
    ks = sorted(sd)
    write_safetensors(str(tmp_path / 'a.safetensors'),
                      {k: sd[k] for k in ks[::2]})
    write_safetensors(str(tmp_path / 'b.safetensors'),
                      {k: sd[k] for k in ks[1::2]})
    got = load_pretrained(str(tmp_path), cfg)
    for k in W:
        assert torch.equal(got[k], W[k].bfloat16()), k
