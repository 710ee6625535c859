"""Pin the CPU oracle against golden vectors produced by the reference's own
eager modules (tests/golden/make_golden.py)."""
import os

import torch

from fluxvla_b200.config import PI0Config
from fluxvla_b200.weights import make_weights
from oracle import pi0_oracle as O

G = os.path.join(os.path.dirname(__file__), 'golden')


def _load(name):
    return torch.load(os.path.join(G, name), weights_only=False)


def _predict(d):
    cfg = PI0Config(**d['cfg'])
    W = make_weights(cfg, d['seed'])
    lang_masks = d['lang_masks']
    out = O.predict_action(cfg, W, d['images'], d['lang_tokens'], d['state'],
                           d['noise'], lang_masks=lang_masks)
    return out


def test_pi0_tiny_matches_reference():
    d = _load('pi0_tiny.pt')
    out = _predict(d)
    torch.testing.assert_close(out, d['actions'], atol=2e-5, rtol=1e-4)


def test_pi0_tiny_padded_prompt_matches_reference():
    d = _load('pi0_tiny_pad.pt')
    out = _predict(d)
    torch.testing.assert_close(out, d['actions'], atol=2e-5, rtol=1e-4)


def test_pi05_tiny_matches_reference():
    d = _load('pi05_tiny.pt')
    out = _predict(d)
    torch.testing.assert_close(out, d['actions'], atol=2e-5, rtol=1e-4)


def test_prefix_embeddings_match_reference():
    d = _load('pi0_tiny.pt')
    cfg = PI0Config(**d['cfg'])
    W = make_weights(cfg, d['seed'])
    V = cfg.n_views
    pix = O.normalize_images(d['images'], [cfg.img_mean] * V,
                             [cfg.img_std] * V).reshape(1, 3 * V,
                                                        cfg.image_size,
                                                        cfg.image_size)
    embs, pad, att = O.embed_prefix(cfg, W, pix, d['lang_tokens'],
                                    torch.ones(1, V, dtype=torch.bool),
                                    d['lang_masks'])
    torch.testing.assert_close(embs, d['prefix_embs'], atol=1e-5, rtol=1e-5)


def test_gemma_layer_cfg0_geometry_matches_reference():
    d = _load('gemma_layer_cfg0.pt')
    cfg = PI0Config(llm_layers=1)
    W = make_weights(cfg, d['seed'], parts=('llm',))
    out = O.gemma_layer_causal(cfg, W, d['x'])
    torch.testing.assert_close(out, d['out'], atol=1e-4, rtol=1e-4)


def test_resize_matches_opencv_golden():
    """The oracle's INTER_LINEAR restatement against cv2.resize outputs
    (tests/golden/make_resize_golden.py): bit-exact uint8."""
    import os
    from tests.golden.make_resize_golden import source
    d = torch.load(os.path.join(os.path.dirname(__file__), 'golden', 'resize_u8.pt'))
    from oracle.pi0_oracle import resize_linear_u8
    for (seed, h, w, H, W) in d['cases']:
        got = resize_linear_u8(source(seed, h, w), H, W)
        assert torch.equal(torch.from_numpy(got), d['outputs'][(seed, h, w, H, W)]), (h, w, H, W)


def _predict_real_width(name, atol):
    d = _load(name)
    cfg = PI0Config(**d['cfg'])
    W = make_weights(cfg, d['seed'])
    out = _predict(d)
    torch.testing.assert_close(out, d['actions'], atol=atol, rtol=1e-4)
    V = cfg.n_views
    pix = O.normalize_images(d['images'], [cfg.img_mean] * V,
                             [cfg.img_std] * V).reshape(1, 3 * V,
                                                        cfg.image_size,
                                                        cfg.image_size)
    embs, _, _ = O.embed_prefix(cfg, W, pix, d['lang_tokens'],
                                torch.ones(1, V, dtype=torch.bool),
                                d['lang_masks'])
    torch.testing.assert_close(embs[:, d['prefix_rows']], d['prefix_embs'],
                               atol=1e-4, rtol=1e-4)


def test_pi0_real_width_matches_reference():
    """Production widths (SigLIP 1152/hd 72 on a 256-token view, Gemma-2B
    layer over 272 prefix rows, expert layer 1024 wide, 51 suffix rows):
    prefix embeddings and the 10-step actions of the reference's own eager
    PI0FlowMatching.predict_action."""
    _predict_real_width('pi0_real_width.pt', 1e-4)


def test_pi05_real_width_matches_reference():
    """As above for PI05FlowMatching (adaRMS expert, 304 prefix rows)."""
    _predict_real_width('pi05_real_width.pt', 1e-4)
