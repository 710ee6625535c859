"""ctypes binding of libfluxvla_b200.so (the C ABI in include/fluxvla_b200.h).

The library is required: importing the ops without it raises, there is no
fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'libfluxvla_b200.so')

FVB_OK = 0
(FVB_ERR_INVALID_ARG, FVB_ERR_UNSUPPORTED, FVB_ERR_CUDA, FVB_ERR_DEVICE_TIMEOUT,
 FVB_ERR_WORKSPACE) = range(1, 6)
EPI_BF16, EPI_F32_STORE, EPI_F32_ACC, EPI_GEGLU, EPI_QKV_ROPE = range(5)
ACT_NONE, ACT_GELU_TANH, ACT_SILU = range(3)
NORM_GEMMA_RMS, NORM_ADA_RMS, NORM_LAYER, NORM_RMS, NORM_ADA_STYLE = range(5)


class GemmArgs(C.Structure):
    _fields_ = [('a', C.c_void_p), ('lda', C.c_int64), ('b', C.c_void_p),
                ('ldb', C.c_int64), ('m', C.c_int32), ('n', C.c_int32),
                ('k', C.c_int32), ('swap', C.c_int32),
                ('epilogue', C.c_int32), ('act', C.c_int32),
                ('split_k', C.c_int32), ('block_n', C.c_int32),
                ('out', C.c_void_p), ('ldo', C.c_int64),
                ('bias', C.c_void_p), ('gate', C.c_void_p),
                ('alpha', C.c_float), ('row_add', C.c_void_p),
                ('row_add_mod', C.c_int32), ('k_out', C.c_void_p),
                ('v_out', C.c_void_p), ('ld_kv', C.c_int64),
                ('n_heads', C.c_int32), ('head_dim', C.c_int32),
                ('rope_cs', C.c_void_p), ('positions', C.c_void_p),
                ('workspace', C.c_void_p), ('workspace_bytes', C.c_int64),
                ('norm_mode', C.c_int32), ('norm_out', C.c_void_p),
                ('ld_norm_out', C.c_int64), ('norm_w', C.c_void_p),
                ('norm_b', C.c_void_p), ('norm_eps', C.c_float),
                ('norm_sync', C.c_void_p), ('pair', C.c_int32),
                ('res', C.c_void_p), ('ld_res', C.c_int64),
                ('gate_tok', C.c_void_p), ('ld_gate_tok', C.c_int64),
                ('rope_interleaved', C.c_int32)]


class AttnArgs(C.Structure):
    _fields_ = [('q', C.c_void_p), ('q_row_stride', C.c_int64),
                ('q_head_stride', C.c_int64), ('k', C.c_void_p),
                ('k_row_stride', C.c_int64), ('k_head_stride', C.c_int64),
                ('v', C.c_void_p), ('v_row_stride', C.c_int64),
                ('v_head_stride', C.c_int64), ('o', C.c_void_p),
                ('o_row_stride', C.c_int64), ('o_head_stride', C.c_int64),
                ('n_q', C.c_int32), ('n_kv', C.c_int32),
                ('heads', C.c_int32), ('group', C.c_int32),
                ('batch', C.c_int32), ('q_batch_rows', C.c_int64),
                ('kv_batch_rows', C.c_int64), ('head_dim', C.c_int32),
                ('scale', C.c_float), ('key_valid', C.c_void_p),
                ('n_prefix', C.c_int32), ('q_block', C.c_void_p),
                ('k_block', C.c_void_p), ('kv_splits', C.c_int32),
                ('workspace', C.c_void_p), ('workspace_bytes', C.c_int64)]


class ExpertArgs(C.Structure):
    _fields_ = [('n_layers', C.c_int32), ('n_tok', C.c_int32),
                ('width', C.c_int32), ('mlp', C.c_int32),
                ('heads', C.c_int32), ('head_dim', C.c_int32),
                ('n_prefix', C.c_int32), ('w_qkv', C.c_void_p),
                ('w_o', C.c_void_p), ('w_gu', C.c_void_p),
                ('w_down', C.c_void_p), ('in_scale', C.c_void_p),
                ('post_scale', C.c_void_p), ('qkv_bias', C.c_void_p),
                ('gu_bias', C.c_void_p), ('o_gate', C.c_void_p),
                ('down_gate', C.c_void_p), ('eps', C.c_float),
                ('x', C.c_void_p), ('k_cache', C.c_void_p),
                ('v_cache', C.c_void_p), ('cache_rows', C.c_int64),
                ('key_valid', C.c_void_p), ('blocks', C.c_void_p),
                ('positions', C.c_void_p), ('rope_cs', C.c_void_p),
                ('rope_suffix', C.c_void_p),
                ('workspace', C.c_void_p), ('workspace_bytes', C.c_int64)]


EXPORTS = {
    'fvb_expert_step': (C.c_int, [C.POINTER(ExpertArgs), C.c_void_p]),
    'fvb_expert_workspace_bytes': (C.c_int64, [C.POINTER(ExpertArgs)]),
    'fvb_gemm': (C.c_int, [C.POINTER(GemmArgs), C.c_void_p]),
    'fvb_gemm_workspace_bytes': (C.c_int64, [C.POINTER(GemmArgs)]),
    'fvb_attention': (C.c_int, [C.POINTER(AttnArgs), C.c_void_p]),
    'fvb_attention_workspace_bytes': (C.c_int64, [C.POINTER(AttnArgs)]),
    'fvb_attention_combine': (C.c_int, [C.POINTER(AttnArgs), C.c_void_p]),
    'fvb_softmax_rows': (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32,
                                   C.c_int32, C.c_void_p, C.c_void_p, C.c_int64,
                                   C.c_void_p]),
    'fvb_norm_bf16': (C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_void_p,
                                C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                C.c_float, C.c_void_p]),
    'fvb_norm': (C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_void_p,
                           C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                           C.c_void_p]),
    'fvb_resize_patchify': (C.c_int, [C.c_void_p, C.c_int32, C.c_int32,
                                      C.c_int32, C.c_int32, C.c_int32,
                                      C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_int64, C.c_void_p]),
    'fvb_probe_wait_timeout': (C.c_int, [C.c_int64, C.c_void_p, C.c_void_p]),
    'fvb_patchify_f32': (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                   C.c_int32, C.c_void_p, C.c_int64, C.c_void_p]),
    'fvb_patchify': (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                               C.c_int32, C.c_void_p, C.c_void_p,
                               C.c_void_p, C.c_int64, C.c_void_p]),
    'fvb_embed_tokens': (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p,
                                   C.c_int32, C.c_float, C.c_void_p,
                                   C.c_int64, C.c_void_p]),
    'fvb_small_linear': (C.c_int, [C.c_void_p, C.c_int64, C.c_int32,
                                   C.c_int32, C.c_void_p, C.c_int64,
                                   C.c_int32, C.c_void_p, C.c_int32,
                                   C.c_int32, C.c_float, C.c_void_p,
                                   C.c_int64, C.c_void_p]),
    'fvb_gemm_trace_next': (C.c_int, []),
    'fvb_expert_trace_read': (C.c_int, [C.c_void_p, C.c_int32]),
    'fvb_gemm_trace_read': (C.c_int, [C.c_void_p, C.c_int32]),
    'fvb_get_device_status': (C.c_int, [C.POINTER(C.c_int), C.c_int]),
    'fvb_last_error': (C.c_char_p, []),
    'fvb_version': (C.c_int, []),
    'fvb_launch_count': (C.c_int64, []),
}

_lib = None


def lib():
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f'{LIB_PATH} is missing: build it with '
                '`python -m fluxvla_b200.build` (there is no fallback path)')
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in EXPORTS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class FVBError(RuntimeError):
    pass


def check(rc: int):
    if rc != FVB_OK:
        raise FVBError(f'fluxvla_b200 error {rc}: '
                       f'{lib().fvb_last_error().decode()}')
