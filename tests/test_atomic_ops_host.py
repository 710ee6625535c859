"""The atomic_ops / attention_triton_ops drop-ins keep the reference's
operator names and signatures (fixture recorded from fluxvla/ops/atomic_ops.py by
tests/golden/make_atomic_ops_signatures.py)."""
import inspect
import json
import os

import pytest

from fluxvla_b200 import atomic_ops, attention_triton_ops

SIGS = json.load(open(os.path.join(os.path.dirname(__file__), 'golden',
                                   'atomic_ops_signatures.json')))


def test_fixture_covers_the_pi05_import_list():
    assert len([n for n in SIGS if not n.startswith('triton:')]) == 17
    assert len([n for n in SIGS if n.startswith('triton:')]) == 3


@pytest.mark.parametrize('name', sorted(SIGS))
def test_signature_matches_reference(name):
    if name.startswith('triton:'):
        # launched as kernel[grid](...): the launcher returns the function
        fn = getattr(attention_triton_ops, name[len('triton:'):])[(1,)]
        ref_file = 'attention_triton_ops.py'
    else:
        fn = getattr(atomic_ops, name)
        ref_file = 'atomic_ops.py'
    params = list(inspect.signature(fn).parameters.values())
    assert [p.name for p in params] == SIGS[name]['args']
    for p in params:
        if p.name in SIGS[name]['defaults']:
            assert p.default == SIGS[name]['defaults'][p.name], p.name
        else:
            assert p.default is inspect.Parameter.empty, p.name
    assert f'{ref_file}:{SIGS[name]["line"]}' in fn.__doc__


def test_triton_style_launchers_need_a_grid():
    k = attention_triton_ops.matmul_abT_scale
    assert k[(1,)] is k[(148, 1, 1)]  # the grid is a tuning knob, ignored
    with pytest.raises(TypeError):
        k(None, None, None, 1, 1, 1, 1.0)
