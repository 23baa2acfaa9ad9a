"""Loader for libtreeattn_b200.so (the C ABI declared in include/treeattn_b200.h).

The library is built in-tree (``treeattn_b200/lib/``) by ``python -m treeattn_b200.build`` or
``__graft_entry__.build()``. There is no fallback: if the library is missing, every entry point raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, 'lib', 'libtreeattn_b200.so')

TA_OK, TA_ERR_ARG, TA_ERR_CUDA = 0, 1, 2
DTYPE_CODES = {'float32': 0, 'bfloat16': 1, 'float16': 2}

c_void_p, c_int, c_int64, c_float = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
P = c_void_p
I = c_int
L = c_int64
F = c_float

# name -> argtypes (every entry returns int unless listed in _RESTYPES)
SIGNATURES = {
    'ta_version': [],
    'ta_last_error': [],
    'ta_device_error': [P],
    'ta_level_nodes': [I, I, I],
    'ta_wait_probe': [L, P],
    'ta_build_levels': [P, I, I, I, I, I, L, L, L, I, I, I, I, P, L, L, P],
    'ta_build_log_levels': [P, I, I, I, I, I, L, L, L, I, I, I, I, P, L, L, P],
    'ta_gate_levels': [P, P, P, I, I, I, I, L, L, I, I, I, F, I, P],
    'ta_gate_append': [P, I, I, I, I, L, L, L, P, P, P, L, L, I, I, I, P, F, I, P],
    'ta_select': [P, I, I, I, I, I, L, L, L, P, L, L, P, L, L, I, I, I, I, I, P, P, P, P],
    'ta_finish': [P, P, P, P, P, P, L, I, I, I, I, P, P, P, P, P],
    'ta_seg_attn': [P, P, P, I, I, I, I, I, L, L, L, L, L, L, L, L, L, I, P, L, L, P, P, I, P, I, I, I, F,
                    P, L, L, L, P, P, P],
    'ta_prefill_attn': [P, P, P, I, I, I, I, I, L, L, L, L, L, L, L, L, L, I, P, L, L, P, P, I, P, I, I, I, F,
                        P, L, L, L, P, P, P],
    'ta_sparse_attn': [P, P, P, I, I, I, I, I, L, L, L, L, L, L, L, L, L, I, P, I, I, F, P, L, L, L, P, P],
    'ta_neighbor_pass': [P, I, I, I, I, I, L, L, L, P, L, L, P, L, L, I, I, P, P, P, I, I, I, F, I, I, I, P, P, P,
                         P],
    'ta_lane_search': [P, P, P, I, I, I, I, I, P, P, P, P],
    'ta_lane_order': [P, L, L, P, I, I, I, I, I, I, P, P, P, P, P],
    'ta_lane_order_noalloc': [P, L, L, P, I, I, I, I, I, I, P, P, P],
    'ta_lane_sums': [P, L, L, P, P, I, I, I, P, P, P, P],
    'ta_lane_insert': [P, P, P, I, I, I, P, P, P, P],
    'ta_lane_select': [P, P, P, I, I, I, I, I, I, I, I, I, I, F, I, P, P, P, P, P, P, P, P, P],
    'ta_forest_levels': [P, I, I, I, I, I, I, I, P, I, F, F, P, P],
    'ta_soft_gate': [P, P, I, L, I, I, F, F, P, P],
    'ta_forest_select': [P, I, I, I, I, I, L, L, L, P, P, I, I, P, I, I, P, P, P, P, P, P, P],
    'ta_sparse_attn_bwd': [P, P, P, P, P, P, I, I, I, I, I, I, P, I, I, F, P, P, P, P],
    'ta_gather_dot': [P, P, I, I, I, I, I, I, I, L, L, L, L, L, L, P, I, F, P, P],
    'ta_gather_dot_blocks': [P, P, I, I, I, I, I, L, L, L, L, L, P, I, I, I, F, P, P],
    'ta_dedupe': [P, P, P, L, I, P],
    'ta_append': [P, P, I, I, I, I, L, L, L, L, P, P, L, L, L, P, L, L, I, I, I, P, P],
    'ta_decode_step': [P, I, I, I, I, L, L, L, P, P, L, L, L, P, L, L, I, I, I, P, I, I, I, F, P, L, P, P, P, I,
                       P, P, P],
    'ta_decode_default_splits': [I, I, I, I],
    'ta_embed_ln': [P, P, I, P, P, I, I, I, I, P, F, P, P, P],
    'ta_add_ln': [P, P, I, I, I, P, F, P, P],
    'ta_gelu': [P, I, L, P],
    'ta_argmax_advance': [P, I, I, I, P, P, P],
    'ta_linear_supported': [I, I, I, I, I],
    'ta_linear_rows': [P, L, I, I, I, I, P, I, I, P, L, P, P, P, P, P],
    'ta_add_splits_ln': [P, P, I, I, I, I, P, F, P, P],
    'ta_argmax_finish': [P, I, I, I, P, P, P],
    'ta_block_tail_plan': [I, I, I, I, P, P],
    'ta_block_tail': [P, P, P, P, P, P, P, P, F, I, I, I, P, P, P, L, P, P],
}
_RESTYPES = {'ta_last_error': ctypes.c_char_p, 'ta_level_nodes': c_int64}

_lib = None


class TreeAttnError(RuntimeError):
    """A treeattn_b200 entry point rejected its arguments or failed to launch."""


def load():
    """Load the shared library (once). Raises TreeAttnError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise TreeAttnError('libtreeattn_b200.so not found at %s: build it with `python -m treeattn_b200.build` '
                            '(there is no CPU or Triton fallback)' % LIB_PATH)
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, c_int)
    _lib = lib
    return lib


def last_error():
    return load().ta_last_error().decode(errors='replace')


def call(name, *args):
    """Call an entry point and raise TreeAttnError on a non-zero status."""
    fn = getattr(load(), name)
    rc = fn(*args)
    if rc != TA_OK:
        kind = 'bad argument' if rc == TA_ERR_ARG else 'CUDA failure'
        raise TreeAttnError('%s: %s (%s)' % (name, last_error(), kind))
    return rc


def device_error():
    """Read and clear the device-side error record: (code, kernel, a, b). Synchronizes the device."""
    out = (ctypes.c_int * 4)()
    call('ta_device_error', ctypes.cast(out, c_void_p))
    return tuple(out)


def exported_symbols():
    return list(SIGNATURES)
