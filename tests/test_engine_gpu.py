"""End-to-end parity: the CUDA engine (through the C ABI) against the CPU
oracle on identical seeded inputs and random bf16 weights.

Tolerance (north star): actions within max-abs 2e-2 and relative L2 1e-2 of
the fp32 oracle.
"""
import pytest
import torch

from fluxvla_b200.config import PI0Config, pi05_config
from fluxvla_b200.engine import PI0EngineB200
from fluxvla_b200.weights import make_weights
from oracle import pi0_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2


def check_actions(out, ref):
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs().max().item()
    rel = ((out - ref).norm() / ref.norm()).item()
    assert err <= MAX_ABS and rel <= REL_L2, f'max-abs {err:.3e} rel-l2 {rel:.3e}'
    return err, rel


def request(cfg, seed, n_tokens):
    g = torch.Generator().manual_seed(seed)
    imgs = torch.randint(0, 256, (cfg.n_views, cfg.image_size, cfg.image_size,
                                  3), generator=g, dtype=torch.uint8)
    toks = torch.randint(0, cfg.vocab, (1, n_tokens), generator=g)
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    return imgs, toks, state, noise


@pytest.mark.parametrize('loop_impl', ['mega', 'ops'])
@pytest.mark.parametrize('pi05', [False, True])
def test_denoise_loop_external_cache(pi05, loop_impl):
    """config[1] geometry (expert width 1024, 816-row prefix cache ~N(0,1),
    51 or 50 suffix tokens, 10 Euler steps) at reduced depth."""
    kw = dict(exp_layers=3, llm_layers=3)
    cfg = pi05_config(**kw) if pi05 else PI0Config(**kw)
    W = make_weights(cfg, 1, parts=('exp', 'heads'))
    E = 816
    g = torch.Generator().manual_seed(2)
    kv = [(torch.randn(1, 1, E, cfg.head_dim, generator=g).bfloat16(),
           torch.randn(1, 1, E, cfg.head_dim, generator=g).bfloat16())
          for _ in range(cfg.exp_layers)]
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    eng = PI0EngineB200(cfg, W, prefix_len=E, loop_impl=loop_impl)
    eng.set_prefix_cache(torch.stack([k[0, 0] for k, _ in kv]),
                         torch.stack([v[0, 0] for _, v in kv]))
    eng.load_inputs(state=state, noise=noise)
    eng.run(prefix=False)
    torch.cuda.synchronize()
    out = eng.actions.cpu()[None]
    ref = O.euler_loop(cfg, W, state, torch.ones(1, E, dtype=torch.bool), kv,
                       noise)
    check_actions(out, ref)


@pytest.mark.parametrize('pi05', [False, True])
def test_full_pipeline_reduced_depth(pi05):
    """config[2]/[3] geometry (3 views 224x224, SigLIP So400m widths, Gemma-2B
    widths, 48 prompt tokens (+32 state tokens for PI0.5)) at 2 layers per
    tower, through the captured CUDA graph."""
    kw = dict(vis_layers=2, llm_layers=2, exp_layers=2, vocab=4096)
    cfg = pi05_config(**kw) if pi05 else PI0Config(**kw)
    n_tok = 80 if pi05 else 48
    W = make_weights(cfg, 3)
    imgs, toks, state, noise = request(cfg, 4, n_tok)
    eng = PI0EngineB200(cfg, W, prefix_len=768 + n_tok)
    out = eng.predict_action(imgs, toks, state, noise=noise)
    ref = O.predict_action(cfg, W, imgs, toks, state, noise)
    check_actions(out, ref)
    # a second replay of the graph also matches (split-K partial sums are
    # accumulated with f32 atomics, so replays agree to rounding, not bits)
    out2 = eng.predict_action(imgs, toks, state, noise=noise)
    check_actions(out2, ref)


def test_full_pipeline_padded_prompt():
    """Prompt padding: masked prefix keys and cumsum positions."""
    cfg = PI0Config(vis_layers=1, llm_layers=2, exp_layers=2, vocab=4096)
    W = make_weights(cfg, 5)
    imgs, toks, state, noise = request(cfg, 6, 48)
    lm = torch.ones(1, 48, dtype=torch.bool)
    lm[:, 30:] = False
    eng = PI0EngineB200(cfg, W, prefix_len=816)
    out = eng.predict_action(imgs, toks, state, lang_masks=lm, noise=noise)
    ref = O.predict_action(cfg, W, imgs, toks, state, noise, lang_masks=lm)
    check_actions(out, ref)


@pytest.mark.slow
def test_full_pi0_config2_full_depth():
    """config[2]: full PI0 (27 SigLIP + 18 Gemma + 18 expert layers)."""
    cfg = PI0Config()
    W = make_weights(cfg, 7)
    imgs, toks, state, noise = request(cfg, 8, 48)
    eng = PI0EngineB200(cfg, W, prefix_len=816)
    out = eng.predict_action(imgs, toks, state, noise=noise)
    ref = O.predict_action(cfg, W, imgs, toks, state, noise)
    check_actions(out, ref)


@pytest.mark.slow
def test_full_pi05_config3_full_depth():
    """config[3]: full PI0.5 (27 SigLIP + 18 Gemma + 18 adaRMS expert layers,
    848-row prefix = 3 views + 48 text + 32 state tokens, 50 action tokens)."""
    cfg = pi05_config()
    W = make_weights(cfg, 9)
    imgs, toks, state, noise = request(cfg, 10, 80)
    eng = PI0EngineB200(cfg, W, prefix_len=848)
    out = eng.predict_action(imgs, toks, state, noise=noise)
    ref = O.predict_action(cfg, W, imgs, toks, state, noise)
    check_actions(out, ref)


def _abort_word(eng):
    """The persistent step's abort flag inside the engine's workspace: the
    barrier block (320 words, 256-byte aligned) is the workspace's last
    piece and the flag is its word 288."""
    ws = eng.B['expert_ws']
    bar_bytes = (320 * 4 + 255) // 256 * 256
    off = ws.numel() - bar_bytes + 288 * 4
    return ws[off:off + 4]


def test_stale_abort_flag_is_reported_and_cleared():
    """Failure detection without a GPU fault: the abort flag a timed-out wait
    would leave behind is raised from the host; the next chunk must report
    FVB_ERR_DEVICE_TIMEOUT through predict_action (not return silent
    garbage), and the chunk after that must be clean again."""
    from fluxvla_b200 import ops
    cfg = PI0Config(exp_layers=2, llm_layers=2)
    W = make_weights(cfg, 1, parts=('exp', 'heads'))
    E = 816
    g = torch.Generator().manual_seed(3)
    k = torch.randn(cfg.exp_layers, E, cfg.head_dim, generator=g).bfloat16()
    v = torch.randn(cfg.exp_layers, E, cfg.head_dim, generator=g).bfloat16()
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    eng = PI0EngineB200(cfg, W, prefix_len=E)
    eng.set_prefix_cache(k.cuda(), v.cuda())
    ops.device_status(reset=True)
    clean = eng.predict_action(states=state, noise=noise)
    assert torch.isfinite(clean).all()
    _abort_word(eng).fill_(1)
    with pytest.raises(RuntimeError, match='device status 4'):
        eng.predict_action(states=state, noise=noise)
    assert ops.device_status() == 0
    again = eng.predict_action(states=state, noise=noise)
    assert (again - clean).abs().max().item() < 1e-2


def test_config0_gemma_layer_causal_816_rows():
    """config[0]: one Gemma-2B decoder layer, x [1, 816, 2048] ~N(0,1),
    causal mask, positions 0..815, through the prefill kernels (captured
    graph) against the fp32 oracle."""
    from fluxvla_b200.layer import GemmaLayerB200
    cfg = PI0Config(llm_layers=1)
    W = make_weights(cfg, 21, parts=('llm',))
    del W['llm.embed']
    x = torch.randn(1, 816, cfg.llm_width,
                    generator=torch.Generator().manual_seed(22))
    lay = GemmaLayerB200(cfg, W, 816)
    ref = O.gemma_layer_causal(cfg, W, x)

    def check(out):
        # hidden states of magnitude up to ~5 (not actions): max-abs within
        # 1 % of the output's scale and relative L2 1e-2; the layer's own
        # contribution (out - x) within 2 % relative L2
        err = (out - ref).abs().max().item()
        assert err <= 1e-2 * ref.abs().max().item(), err
        assert ((out - ref).norm() / ref.norm()).item() <= 1e-2
        d, dr = out - x, ref - x
        assert ((d - dr).norm() / dr.norm()).item() < 2e-2
    check(lay.forward(x))
    check(lay.forward(x))


@pytest.mark.parametrize('pi05', [False, True])
def test_masked_view_and_padded_prompt(pi05):
    """A camera view masked out (img_masks) and a right-padded prompt: the
    view's 256 keys and the pad tokens are invisible to every query and the
    positions follow cumsum(pad) - 1 (pi0_flowmatching.py:221-250,730)."""
    kw = dict(vis_layers=1, llm_layers=2, exp_layers=2, vocab=4096)
    cfg = pi05_config(**kw) if pi05 else PI0Config(**kw)
    n_tok = 80 if pi05 else 48
    W = make_weights(cfg, 13)
    imgs, toks, state, noise = request(cfg, 14, n_tok)
    im = torch.tensor([[True, False, True]])
    lm = torch.ones(1, n_tok, dtype=torch.bool)
    lm[:, n_tok - 11:] = False
    eng = PI0EngineB200(cfg, W, prefix_len=768 + n_tok)
    out = eng.predict_action(imgs, toks, state, img_masks=im, lang_masks=lm,
                             noise=noise)
    ref = O.predict_action(cfg, W, imgs, toks, state, noise, img_masks=im,
                           lang_masks=lm)
    check_actions(out, ref)
    # the same engine (graph) serves an unmasked request next
    out2 = eng.predict_action(imgs, toks, state, noise=noise)
    check_actions(out2, O.predict_action(cfg, W, imgs, toks, state, noise))


def test_camera_resize_path_end_to_end():
    """Camera frames of another size (480x640) resized on the device with
    OpenCV's INTER_LINEAR (fvb_resize_patchify) inside the captured graph,
    against the oracle on the same frames resized by its restatement."""
    import numpy as np
    cfg = PI0Config(vis_layers=1, llm_layers=1, exp_layers=1, vocab=4096)
    W = make_weights(cfg, 15)
    g = torch.Generator().manual_seed(16)
    frames = torch.randint(0, 256, (3, 480, 640, 3), generator=g,
                           dtype=torch.uint8)
    _, toks, state, noise = request(cfg, 17, 48)
    eng = PI0EngineB200(cfg, W, prefix_len=816, camera_hw=(480, 640))
    out = eng.predict_action(frames, toks, state, noise=noise)
    resized = torch.stack([torch.from_numpy(np.ascontiguousarray(
        O.resize_linear_u8(f.numpy(), 224, 224))) for f in frames])
    ref = O.predict_action(cfg, W, resized, toks, state, noise)
    check_actions(out, ref)
