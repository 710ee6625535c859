"""Host-side logic of the engine on CPU: the orchestration (packing, buffer
wiring, masks, positions, hoisted step tables) is run with a torch emulation
of each C-ABI op (tests/emulated_ops.py) and compared with the oracle.  The
real kernels are covered by the -m gpu tests."""
import torch

from fluxvla_b200.config import PI0Config, pi05_config
from fluxvla_b200.engine import PI0EngineB200, sinusoid, step_times
from fluxvla_b200.weights import make_weights
from oracle import pi0_oracle as O
from tests import emulated_ops
from tests.golden.make_golden import tiny_cfg


def _tiny(pi05):
    kw = dict(vis_layers=2, vis_width=64, vis_heads=4, vis_mlp=96, patch=14,
              image_size=28, n_views=2, llm_layers=2, llm_width=64,
              llm_mlp=96, vocab=97, heads=2, head_dim=16, exp_layers=2,
              exp_width=32, exp_mlp=64, n_actions=4, action_dim=8,
              state_dim=8)
    return pi05_config(**kw) if pi05 else PI0Config(**kw)


def _run(monkeypatch, pi05, lang_valid=None):
    emulated_ops.install(monkeypatch)
    cfg = _tiny(pi05)
    W = make_weights(cfg, 9)
    g = torch.Generator().manual_seed(10)
    n_tok = 5
    imgs = torch.randint(0, 256, (cfg.n_views, 28, 28, 3), generator=g,
                         dtype=torch.uint8)
    toks = torch.randint(0, cfg.vocab, (1, n_tok), generator=g)
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    lm = torch.ones(1, n_tok, dtype=torch.bool)
    if lang_valid is not None:
        lm[:, lang_valid:] = False
    E = cfg.n_views * cfg.tokens_per_view + n_tok
    eng = PI0EngineB200(cfg, W, prefix_len=E, device='cpu')
    eng.load_inputs(imgs, toks, lm, None, state, noise)
    eng.run()
    ref = O.predict_action(cfg, W, imgs, toks, state, noise, lang_masks=lm)
    return eng.actions[None], ref


def test_engine_host_logic_pi0(monkeypatch):
    out, ref = _run(monkeypatch, False)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=1e-2)


def test_engine_host_logic_pi0_padded(monkeypatch):
    out, ref = _run(monkeypatch, False, lang_valid=2)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=1e-2)


def test_engine_host_logic_pi05(monkeypatch):
    out, ref = _run(monkeypatch, True)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=1e-2)


def test_step_times_and_sinusoid_match_oracle():
    ts, dt = step_times(10)
    assert ts == O.step_times(10) and len(ts) == 10
    assert dt == float(torch.tensor(-0.1, dtype=torch.float32))
    torch.testing.assert_close(sinusoid(ts, 64),
                               O.sinusoidal_time(torch.tensor(ts), 64))


def test_engine_resizes_camera_frames(monkeypatch):
    """Frames of another size go through the device resize (OpenCV
    INTER_LINEAR) and give the actions of the pre-resized frames."""
    import numpy as np
    emulated_ops.install(monkeypatch)
    cfg = _tiny(False)
    W = make_weights(cfg, 9)
    g = torch.Generator().manual_seed(11)
    n_tok = 5
    cam = torch.randint(0, 256, (cfg.n_views, 40, 33, 3), generator=g,
                        dtype=torch.uint8)
    toks = torch.randint(0, cfg.vocab, (1, n_tok), generator=g)
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    E = cfg.n_views * cfg.tokens_per_view + n_tok
    eng = PI0EngineB200(cfg, W, prefix_len=E, device='cpu', camera_hw=(40, 33))
    eng.load_inputs(cam, toks, None, None, state, noise)
    eng.run()
    out = eng.actions[None]
    small = torch.stack([torch.from_numpy(O.resize_linear_u8(v.numpy(), 28, 28))
                         for v in cam])
    ref = O.predict_action(cfg, W, small, toks, state, noise)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=1e-2)
