"""The C-ABI library loads without a GPU and exports every entry point that
include/fluxvla_b200.h declares (no compute calls)."""
import ctypes
import os
import re

import pytest

from fluxvla_b200 import _lib

HDR = os.path.join(os.path.dirname(os.path.dirname(__file__)), 'include',
                   'fluxvla_b200.h')


def declared():
    src = open(HDR).read()
    src = re.sub(r'/\*.*?\*/', '', src, flags=re.S)
    return sorted(set(re.findall(r'\b(fvb_\w+)\s*\(', src)))


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n


def test_python_binding_covers_abi():
    L = _lib.lib()
    assert L.fvb_version() == 1
    for n in declared():
        if n != 'fvb_attention_noalloc':
            assert n in _lib.EXPORTS, n


def test_invalid_arguments_return_errors_without_gpu():
    L = _lib.lib()
    args = _lib.GemmArgs()
    rc = L.fvb_gemm(ctypes.byref(args), None)
    assert rc == 1 and b'NULL' in L.fvb_last_error()


def test_torch_extension_loads_and_reports_errors():
    """fluxvla_b200._C (the thin torch extension over the C ABI) loads with
    the library, exposes the op entry points, raises ValueError for a bad
    argument and RuntimeError (with the library's message) for an error the
    C ABI returns — without a GPU."""
    import torch

    from fluxvla_b200 import ops
    ext = ops._C()
    for name in ('gemm', 'norm', 'norm_bf16', 'softmax_rows', 'small_linear'):
        assert callable(getattr(ext, name))
    with pytest.raises(RuntimeError, match='status is NULL'):
        ext.error_path_probe()
    with pytest.raises(ValueError, match='must be a CUDA tensor'):
        ops.norm(0, torch.zeros(2, 128), torch.zeros(2, 128))
    with pytest.raises(ValueError, match='expected'):
        ops.norm(0, torch.zeros(2, 128, dtype=torch.int32), torch.zeros(2, 128))
