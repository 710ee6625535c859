"""PI0.5 state discretisation and prompt string against the reference's
arithmetic (fluxvla/transforms/prompters.py:299-314), bit-exact."""
import numpy as np
import pytest

from fluxvla_b200.prompt import discretize_state, format_prompt, pi05_prompt


def _ref_bins(state, max_dim=32):
    padded = np.zeros(max_dim)
    padded[:state.shape[0]] = state
    return np.digitize(padded, bins=np.linspace(-1, 1, 256 + 1)[:-1]) - 1


@pytest.mark.parametrize('seed', range(5))
def test_bins_match_digitize_random(seed):
    rng = np.random.default_rng(seed)
    for n in (1, 7, 14, 32):
        s = rng.uniform(-1.2, 1.2, n)
        assert np.array_equal(discretize_state(s), _ref_bins(s))


def test_bins_match_digitize_on_edges():
    edges = np.linspace(-1, 1, 257)
    vals = np.concatenate([edges, np.nextafter(edges, -2),
                           np.nextafter(edges, 2), [-5.0, 5.0, 0.0, -0.0,
                                                    np.inf, -np.inf, np.nan]])
    for i in range(0, len(vals), 32):
        chunk = vals[i:i + 32]
        assert np.array_equal(discretize_state(chunk), _ref_bins(chunk)), i


def test_prompt_string():
    s = np.array([-1.0, 0.0, 0.999, 1.0])
    p = pi05_prompt('  pick_up the\nbowl ', s)
    bins = ' '.join(map(str, _ref_bins(s)))
    assert p == f'Task: pick up the bowl, State: {bins};\nAction: '
    assert format_prompt('x', [0, 255]) == 'Task: x, State: 0 255;\nAction: '


def test_state_required_and_length_checked():
    with pytest.raises(ValueError):
        pi05_prompt('t', None)
    with pytest.raises(ValueError):
        discretize_state(np.zeros(33))
