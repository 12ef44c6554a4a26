"""ctypes binding of the C ABI in ``include/slimkv_b200.h``.

The shared library ``libslimkv_b200.so`` is built in-tree by
``slimkv_b200.build``.  There is deliberately no fallback: if the library is
missing or fails to load, every entry point raises, so no CPU or eager path
can silently stand in for the CUDA kernels.
"""
import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get('SLIMKV_B200_LIB', _PKG / 'libslimkv_b200.so'))

SLIMKV_OK = 0
ERRORS = {1: 'invalid argument', 2: 'unsupported shape', 3: 'alignment', 4: 'workspace',
          5: 'CUDA error', 6: 'tensor map'}
DEVICE_TIMEOUT = 0x1
DEVICE_BAD_LENGTH = 0x2
DEVICE_MISALIGNED = 0x4

I64x3 = ctypes.c_int64 * 3
I64x2 = ctypes.c_int64 * 2


class AttentionArgs(ctypes.Structure):
    _fields_ = [
        ('q', ctypes.c_void_p), ('q_stride', I64x3),
        ('k', ctypes.c_void_p), ('k_stride', I64x3),
        ('v', ctypes.c_void_p), ('v_stride', I64x3),
        ('out', ctypes.c_void_p), ('out_stride', I64x3),
        ('lse', ctypes.c_void_p), ('cache_seqlens', ctypes.c_void_p),
        ('batch', ctypes.c_int), ('queries', ctypes.c_int), ('heads', ctypes.c_int),
        ('kv_heads', ctypes.c_int), ('keys', ctypes.c_int), ('head_dim', ctypes.c_int),
        ('value_dim', ctypes.c_int), ('scale', ctypes.c_float), ('causal', ctypes.c_int),
        ('num_splits', ctypes.c_int), ('lse_masked_positive', ctypes.c_int), ('out_fp32', ctypes.c_int),
    ]


class LatentDecodeArgs(ctypes.Structure):
    _fields_ = [
        ('batch', ctypes.c_int), ('length', ctypes.c_int), ('heads', ctypes.c_int),
        ('kv_heads', ctypes.c_int), ('head_dim', ctypes.c_int), ('rank_k', ctypes.c_int),
        ('rank_v', ctypes.c_int), ('scale', ctypes.c_float),
        ('q', ctypes.c_void_p), ('q_stride', I64x3),
        ('raw_k_rot', ctypes.c_void_p), ('raw_v', ctypes.c_void_p), ('raw_k_pre', ctypes.c_void_p),
        ('raw_stride_batch', ctypes.c_int64), ('raw_stride_token', ctypes.c_int64),
        ('raw_capacity', ctypes.c_int),
        ('lat_k', ctypes.c_void_p), ('lat_v', ctypes.c_void_p),
        ('lat_stride_batch', ctypes.c_int64), ('lat_stride_row', ctypes.c_int64),
        ('lat_capacity', ctypes.c_int),
        ('raw_len', ctypes.c_void_p), ('latent_len', ctypes.c_void_p),
        ('query_len', ctypes.c_void_p), ('qpos', ctypes.c_void_p),
        ('new_k', ctypes.c_void_p), ('new_v', ctypes.c_void_p), ('new_stride', ctypes.c_int64),
        ('new_lat_k', ctypes.c_void_p), ('new_lat_v', ctypes.c_void_p), ('new_lat_stride', ctypes.c_int64),
        ('uk', ctypes.c_void_p), ('uv', ctypes.c_void_p),
        ('uk_bias', ctypes.c_void_p), ('uv_bias', ctypes.c_void_p),
        ('cos', ctypes.c_void_p), ('sin', ctypes.c_void_p), ('rope_positions', ctypes.c_int),
        ('out', ctypes.c_void_p), ('out_stride', I64x2), ('out_fp32', ctypes.c_int),
        ('latent_len_max', ctypes.c_int), ('raw_len_max', ctypes.c_int),
        ('latent_splits', ctypes.c_int), ('raw_splits', ctypes.c_int),
        ('attn_event_begin', ctypes.c_void_p), ('attn_event_end', ctypes.c_void_p),
        ('lat_pages', ctypes.c_void_p), ('lat_page_stride', ctypes.c_int64), ('lat_slots', ctypes.c_int),
        ('lat_sink_elements', ctypes.c_int), ('lat_table', ctypes.c_void_p), ('lat_table_stride', ctypes.c_int64),
        ('lat_num_pages', ctypes.c_int),
        ('out_lse', ctypes.c_void_p), ('latent_shard', ctypes.c_int), ('wait_limit_ns', ctypes.c_uint64),
        ('raw_stride_head', ctypes.c_int64), ('plan', ctypes.c_void_p),
    ]


# Exported symbols and their ctypes signatures; the CPU test suite checks
# that the built library exports every one of them.
_P = ctypes.c_void_p
_I = ctypes.c_int
class BeaconPagesArgs(ctypes.Structure):
    """Mirror of ``slimkv_beacon_pages``."""
    _fields_ = [
        ('pages', ctypes.c_void_p), ('page_stride', ctypes.c_int64), ('slots', ctypes.c_int),
        ('rank_k', ctypes.c_int), ('rank_v', ctypes.c_int), ('sink_elements', ctypes.c_int),
        ('table', ctypes.c_void_p), ('table_stride', ctypes.c_int64), ('num_pages', ctypes.c_int),
    ]


class RawPagesArgs(ctypes.Structure):
    """Mirror of ``slimkv_raw_pages``."""
    _fields_ = [
        ('pages', ctypes.c_void_p), ('block_size', ctypes.c_int), ('kv_heads', ctypes.c_int),
        ('head_dim', ctypes.c_int), ('table', ctypes.c_void_p), ('table_stride', ctypes.c_int64),
        ('num_blocks', ctypes.c_int),
    ]


_L = ctypes.c_int64


class WindowProjectArgs(ctypes.Structure):
    """Mirror of ``slimkv_window_project_args``."""
    _fields_ = [
        ('batch', _I), ('rows', _I), ('hidden', _I),
        ('hidden_states', _P), ('hidden_stride_batch', _L), ('hidden_stride_row', _L),
        ('raw_rows', _P), ('raw_count', _I), ('beacon_rows', _P), ('beacon_count', _I),
        ('heads', _I), ('kv_heads', _I), ('head_dim', _I), ('rank_k', _I), ('rank_v', _I),
        ('w_q', _P), ('b_q', _P), ('w_k', _P), ('b_k', _P), ('w_v', _P), ('b_v', _P),
        ('w_bq', _P), ('b_bq', _P), ('w_k_down', _P), ('w_v_down', _P), ('w_k_up', _P), ('b_k_up', _P),
        ('w_v_up', _P), ('b_v_up', _P),
        ('query', _P), ('query_stride_batch', _L), ('query_stride_row', _L),
        ('key', _P), ('key_stride_batch', _L), ('key_stride_row', _L),
        ('value', _P), ('value_stride_batch', _L), ('value_stride_row', _L),
        ('key_latent', _P), ('key_latent_stride_batch', _L), ('key_latent_stride_row', _L),
        ('value_latent', _P), ('value_latent_stride_batch', _L), ('value_latent_stride_row', _L),
        ('latent_rows', _I), ('latent_start', _P), ('beacon_pages', ctypes.POINTER(BeaconPagesArgs)),
        ('beacon_start', _P),
        ('raw_start', _P), ('raw_first', _I), ('raw_key_cache', _P), ('raw_value_cache', _P),
        ('raw_cache_stride_batch', _L), ('raw_cache_stride_row', _L), ('raw_cache_rows', _I),
        ('raw_pages', ctypes.POINTER(RawPagesArgs)), ('write_sink', _I),
        ('workspace', _P), ('workspace_bytes', ctypes.c_size_t),
    ]


class ReconstructArgs(ctypes.Structure):
    """Mirror of ``slimkv_reconstruct_args``."""
    _fields_ = [
        ('batch', _I), ('rows', _I), ('kv_heads', _I), ('head_dim', _I), ('rank_k', _I), ('rank_v', _I),
        ('lat_k', _P), ('lat_v', _P), ('lat_stride_batch', _L), ('lat_stride_row', _L), ('lat_capacity', _I),
        ('w_k_up', _P), ('b_k_up', _P), ('w_v_up', _P), ('b_v_up', _P), ('key', _P), ('value', _P),
        ('out_stride_batch', _L), ('out_stride_row', _L), ('out_rows', _I), ('out_start', _P),
        ('workspace', _P), ('workspace_bytes', ctypes.c_size_t),
        ('row_count', _P),
    ]


class MergePartialsArgs(ctypes.Structure):
    """Mirror of ``slimkv_merge_partials_args``."""
    _fields_ = [
        ('parts', _I), ('rows', _I), ('dim', _I), ('part_out', _P), ('part_stride', _L),
        ('part_lse', _P), ('lse_part_stride', _L), ('out', _P), ('out_fp32', _I), ('out_lse', _P),
    ]


class PrefillAttentionArgs(ctypes.Structure):
    """Mirror of ``slimkv_prefill_attention_args``."""
    _fields_ = [
        ('batch', _I), ('kv_heads', _I), ('rows_per_token', _I), ('tokens', _I), ('dim_qk', _I), ('dim_v', _I),
        ('q', _P), ('q_stride', _L * 3), ('k', _P), ('v', _P), ('kv_stride', _L * 3), ('kv_capacity', _I),
        ('kv_len', _P), ('causal', _I), ('causal_offset', _I), ('scale', ctypes.c_float), ('out', _P),
        ('out_stride', _L * 3), ('lse', _P), ('lse_stride', _L * 2), ('wait_limit_ns', ctypes.c_uint64),
    ]


_PL = ctypes.POINTER(ctypes.c_int64)

SIGNATURES = {
    'slimkv_version': (_I, []),
    'slimkv_last_error': (ctypes.c_char_p, []),
    'slimkv_device_status': (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    'slimkv_attention_workspace_size': (ctypes.c_size_t, [ctypes.POINTER(AttentionArgs)]),
    'slimkv_attention_forward': (_I, [ctypes.POINTER(AttentionArgs), _P, ctypes.c_size_t, _P]),
    'slimkv_attention_forward_noalloc': (_I, [ctypes.POINTER(AttentionArgs), _P]),
    'slimkv_latent_decode_workspace_size': (ctypes.c_size_t, [ctypes.POINTER(LatentDecodeArgs)]),
    'slimkv_latent_decode': (_I, [ctypes.POINTER(LatentDecodeArgs), _P, ctypes.c_size_t, _P]),
    'slimkv_decode_plan_words': (ctypes.c_size_t, [ctypes.POINTER(LatentDecodeArgs)]),
    'slimkv_decode_plan': (_I, [ctypes.POINTER(LatentDecodeArgs), _P, _P]),
    'slimkv_rope_decode': (_I, [_P, ctypes.POINTER(ctypes.c_int64), _P, ctypes.POINTER(ctypes.c_int64), _P, _P,
                                _I, _P, ctypes.c_int64, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    'slimkv_decode_schedule': (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    'slimkv_beacon_pages_append': (_I, [ctypes.POINTER(BeaconPagesArgs), _I, _P, _I, _P, _L, _L, _P, _L, _L, _P]),
    'slimkv_beacon_pages_gather': (_I, [ctypes.POINTER(BeaconPagesArgs), _I, _P, _I, _P, _L, _L, _P, _L, _L, _P]),
    'slimkv_beacon_pages_sink': (_I, [ctypes.POINTER(BeaconPagesArgs), _I, _P, _P, _L, _I, _P]),
    'slimkv_raw_pages_write': (_I, [ctypes.POINTER(RawPagesArgs), _I, _P, _I, _P, _L, _L, _P, _L, _L, _P]),
    'slimkv_raw_pages_read': (_I, [ctypes.POINTER(RawPagesArgs), _I, _P, _P, _I, _P, _L, _L, _P, _L, _L, _P]),
    'slimkv_window_project_workspace_size': (ctypes.c_size_t, [ctypes.POINTER(WindowProjectArgs)]),
    'slimkv_window_project': (_I, [ctypes.POINTER(WindowProjectArgs), _P]),
    'slimkv_prefill_rope': (_I, [_P, _PL, _P, _PL, _P, _P, _I, _P, _L, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _PL,
                                 _P, _PL, _P]),
    'slimkv_rope_rows': (_I, [_P, _PL, _P, _PL, _P, _L, _P, _I, _I, _I, _I, _P, _P, _I, _P]),
    'slimkv_merge': (_I, [_P, ctypes.POINTER(ctypes.c_int64), _P, ctypes.POINTER(ctypes.c_int64), _P,
                          ctypes.POINTER(ctypes.c_int64), _P, ctypes.POINTER(ctypes.c_int64), _I, _I, _I,
                          _I, _P, _P]),
    'slimkv_merge_partials': (_I, [ctypes.POINTER(MergePartialsArgs), _P]),
    'slimkv_reconstruct_kv_workspace_size': (ctypes.c_size_t, [ctypes.POINTER(ReconstructArgs)]),
    'slimkv_reconstruct_kv': (_I, [ctypes.POINTER(ReconstructArgs), _P]),
    'slimkv_prefill_attention': (_I, [ctypes.POINTER(PrefillAttentionArgs), _P]),
    'slimkv_rms_norm': (_I, [_P, _L, _P, _P, _L, _I, _I, ctypes.c_float, _P]),
    'slimkv_silu_mul': (_I, [_P, _L, _P, _L, _I, _I, _P]),
}

_lib = None


def load():
    """Load the shared library once; raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f'{LIB_PATH} is missing; build it with `python -m slimkv_b200.build` '
                              '(no CPU fallback exists)')
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class SlimKVError(RuntimeError):
    pass


def check(rc):
    if rc != SLIMKV_OK:
        msg = load().slimkv_last_error().decode(errors='replace')
        raise SlimKVError(f'slimkv_b200: {ERRORS.get(rc, rc)}: {msg}')


def device_status(clear=False):
    value = ctypes.c_uint(0)
    check(load().slimkv_device_status(ctypes.byref(value), int(clear)))
    return value.value
