"""Model-level drop-ins (fluxvla_b200.models) against the reference's own
eager PI0FlowMatching / PI05FlowMatching, loaded by file path from the
installed reference (baseline/_ref or $FLUXVLA_REF) through the shim of
oracle/ref_shim.py.  Skipped when the reference is not installed.

CPU: the derived class keeps the eager class's interface and its config is
read from the module tree.  GPU: on the same seeded weights and inputs the
drop-in's predict_action (normalised float images [1, 3V, 224, 224]) matches
the eager model's own predict_action in fp32 on the CPU within the north-star
tolerance (max-abs 2e-2, relative L2 1e-2), at production widths with one
layer per tower and three views (816 prefix rows)."""
import pytest
import torch

from oracle import ref_shim

pytestmark = pytest.mark.skipif(ref_shim.reference_root() is None,
                                reason='reference not installed')

_REF = None


def _ref():
    global _REF
    if _REF is None:
        _REF = ref_shim.load_reference()
    return _REF


def _model(pi05, cfg=None, seed=41):
    from fluxvla_b200.config import PI0Config, pi05_config
    from fluxvla_b200.weights import make_weights
    kw = dict(vis_layers=1, llm_layers=1, exp_layers=1, vocab=4096)
    cfg = cfg or (pi05_config(**kw) if pi05 else PI0Config(**kw))
    ref = _ref()
    with ref_shim.no_param_init():
        m = ref_shim.build_ref_model(ref, cfg)
    ref_shim.load_weights(m, cfg, make_weights(cfg, seed))
    return m, cfg


@pytest.mark.parametrize('pi05', [False, True])
def test_dropin_class_and_config(pi05):
    from fluxvla_b200.models import config_from_module, make_b200_class
    m, cfg = _model(pi05)
    base = type(m)
    cls = make_b200_class(base)
    assert issubclass(cls, base) and cls.__name__ == base.__name__ + 'B200'
    got = config_from_module(m, cfg.n_views)
    assert got == cfg, (got, cfg)


def _inputs(cfg, seed, n_tok):
    g = torch.Generator().manual_seed(seed)
    u8 = torch.randint(0, 256, (cfg.n_views, 224, 224, 3), generator=g,
                       dtype=torch.uint8)
    mean = torch.tensor(cfg.img_mean)[:, None, None]
    std = torch.tensor(cfg.img_std)[:, None, None]
    pix = ((u8.float().permute(0, 3, 1, 2) - mean) / (std + 1e-8)).reshape(
        1, 3 * cfg.n_views, 224, 224)
    toks = torch.randint(0, cfg.vocab, (1, n_tok), generator=g)
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    return pix, toks, state, noise


@pytest.mark.gpu
@pytest.mark.parametrize('pi05', [False, True])
def test_dropin_matches_reference_predict_action(pi05):
    from fluxvla_b200.models import to_b200
    m, cfg = _model(pi05)
    n_tok = 80 if pi05 else 48
    pix, toks, state, noise = _inputs(cfg, 42, n_tok)
    lm = torch.ones(1, n_tok, dtype=torch.bool)
    lm[:, n_tok - 7:] = False
    im = torch.ones(1, cfg.n_views, dtype=torch.bool)
    with torch.no_grad():
        ref = m.predict_action(pix, toks, state, img_masks=im, lang_masks=lm,
                               noise=noise.clone())
    to_b200(m)
    out = m.predict_action(pix, toks, state, img_masks=im, lang_masks=lm,
                           noise=noise.clone())
    assert out.shape == ref.shape and out.dtype == torch.float32
    err = (out - ref).abs().max().item()
    rel = ((out - ref).norm() / ref.norm()).item()
    assert err <= 2e-2 and rel <= 1e-2, (err, rel)
    # a list of per-view tensors (the reference also accepts it) and a
    # batch of two requests
    out2 = m.predict_action(list(pix.repeat(2, 1, 1, 1).split(3, dim=1)),
                            toks.repeat(2, 1),
                            state.repeat(2, 1), img_masks=im.repeat(2, 1),
                            lang_masks=lm.repeat(2, 1),
                            noise=noise.repeat(2, 1, 1))
    assert out2.shape[0] == 2
    assert (out2[0] - out[0]).abs().max().item() < 1e-2
    assert (out2[1] - out[0]).abs().max().item() < 1e-2
