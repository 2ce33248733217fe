"""ctypes binding of ``libkb200.so`` (declarations in ``include/kb200.h``).

The library is the product's only compute path.  If it is missing or fails
to load, :func:`lib` raises -- there is no CPU or eager fallback.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / 'libkb200.so'
_lock = threading.Lock()
_lib = None

KB200_OK = 0
ERRORS = {1: 'invalid argument', 2: 'misaligned pointer', 3: 'workspace', 4: 'launch failure',
          5: 'device wait timed out'}
ERRORS_BY_NAME = {'invalid': 1, 'align': 2, 'workspace': 3, 'launch': 4, 'timeout': 5}


class GdnArgs(ctypes.Structure):
    """Mirror of ``KB200GdnArgs`` (include/kb200.h)."""
    _fields_ = [
        ('q', ctypes.c_void_p), ('k', ctypes.c_void_p), ('v', ctypes.c_void_p),
        ('g', ctypes.c_void_p), ('beta', ctypes.c_void_p), ('initial_state', ctypes.c_void_p),
        ('o', ctypes.c_void_p), ('final_state', ctypes.c_void_p),
        ('cu_seqlens', ctypes.c_void_p), ('chunk_indices', ctypes.c_void_p),
        ('chunk_offsets', ctypes.c_void_p),
        ('B', ctypes.c_int64), ('T', ctypes.c_int64), ('H', ctypes.c_int64),
        ('K', ctypes.c_int64), ('V', ctypes.c_int64), ('N', ctypes.c_int64),
        ('num_chunks', ctypes.c_int64), ('scale', ctypes.c_float), ('use_qk_l2norm', ctypes.c_int),
    ]


class GdnPrologueArgs(ctypes.Structure):
    """Mirror of ``KB200GdnPrologueArgs`` (include/kb200.h)."""
    _fields_ = [
        ('xq', ctypes.c_void_p), ('xk', ctypes.c_void_p), ('xv', ctypes.c_void_p),
        ('ldq', ctypes.c_int64), ('ldk', ctypes.c_int64), ('ldv', ctypes.c_int64),
        ('wq', ctypes.c_void_p), ('wk', ctypes.c_void_p), ('wv', ctypes.c_void_p),
        ('bq', ctypes.c_void_p), ('bk', ctypes.c_void_p), ('bv', ctypes.c_void_p),
        ('q', ctypes.c_void_p), ('k', ctypes.c_void_p), ('v', ctypes.c_void_p),
        ('a', ctypes.c_void_p), ('b', ctypes.c_void_p),
        ('lda', ctypes.c_int64), ('ldb', ctypes.c_int64),
        ('A_log', ctypes.c_void_p), ('dt_bias', ctypes.c_void_p),
        ('g', ctypes.c_void_p), ('beta', ctypes.c_void_p),
        ('B', ctypes.c_int64), ('T', ctypes.c_int64), ('H', ctypes.c_int64),
        ('Cqk', ctypes.c_int64), ('Cv', ctypes.c_int64),
        ('W', ctypes.c_int), ('allow_neg_eigval', ctypes.c_int),
        ('cache_q', ctypes.c_void_p), ('cache_k', ctypes.c_void_p), ('cache_v', ctypes.c_void_p),
    ]


_ATTN_SIG = (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 5 +
             [ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p])

# name -> (restype, argtypes); every symbol include/kb200.h declares
SIGNATURES = {
    'kb200_abi_version': (ctypes.c_int, []),
    'kb200_last_error': (ctypes.c_char_p, []),
    'kb200_gdn_workspace_size': (ctypes.c_size_t, [ctypes.POINTER(GdnArgs)]),
    'kb200_gdn_launch_count': (ctypes.c_int, [ctypes.POINTER(GdnArgs)]),
    'kb200_gdn_chunk_fwd': (ctypes.c_int, [ctypes.POINTER(GdnArgs), ctypes.c_void_p,
                                           ctypes.c_size_t, ctypes.c_void_p]),
    'kb200_rmsnorm_rope': (ctypes.c_int, [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 6 +
                           [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p]),
    'kb200_gdn_status': (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    'kb200_wait_probe': (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    'kb200_read_error_word': (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    'kb200_gdn_noalloc_scratch_bytes': (ctypes.c_size_t, []),
    'kb200_gdn_chunk_fwd_noalloc': (ctypes.c_int, [ctypes.POINTER(GdnArgs), ctypes.c_void_p]),
    'kb200_attn_fp8_workspace_size': (ctypes.c_size_t, [ctypes.c_int64] * 4),
    'kb200_attn_fp8_fwd': _ATTN_SIG,
    'kb200_attn_fp8_quantize': _ATTN_SIG,
    'kb200_attn_fp8_attend': _ATTN_SIG,
    'kb200_attn_fp8_fwd_window': (_ATTN_SIG[0], _ATTN_SIG[1] + [ctypes.c_int64] * 2),
    'kb200_attn_fp8_attend_window': (_ATTN_SIG[0], _ATTN_SIG[1] + [ctypes.c_int64] * 2),
    'kb200_attn_fp8_status': (ctypes.c_int, [ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_void_p]),
    'kb200_gdn_prologue': (ctypes.c_int, [ctypes.POINTER(GdnPrologueArgs), ctypes.c_void_p]),
    'kb200_rmsnorm_gated': (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 4 +
                            [ctypes.c_float, ctypes.c_void_p]),
    'kb200_residual_ln_mod': (ctypes.c_int, [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 3 +
                              [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_float] + [ctypes.c_void_p] * 2),
}


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f'{_LIB_PATH} is missing: build it with `python -m kairos_sensenova_b200.build` '
                    '(there is no fallback implementation)')
            handle = ctypes.CDLL(str(_LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != KB200_OK:
        msg = lib().kb200_last_error().decode(errors='replace')
        kind = ERRORS.get(rc, f'error {rc}')
        if rc == 1:
            raise ValueError(f'{what}: {msg}')
        raise RuntimeError(f'{what} failed ({kind}): {msg}')
