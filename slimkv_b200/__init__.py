"""B200-native (sm_100a) SlimKV decode-time latent attention.

The hot path of SlimKV decode — attention over the compressed cache of
low-rank Beacon K/V latents plus full-dimension sinks and raw tail — as
hand-written CUDA kernels behind a C ABI (``include/slimkv_b200.h``), with
thin torch bindings that mirror the reference's Python entry points:

* ``slimkv_b200.kernels``    — torch wrappers over the C ABI
* ``slimkv_b200.extension``  — drop-in ``slimkv_fa2_decode_320`` module
* ``slimkv_b200.fa2_decode`` — mirror of ``slimkv.llama3.fa2_decode``
* ``slimkv_b200.rope``       — RoPE tables built exactly like the reference
* ``slimkv_b200.schedule``   — Beacon decode schedule (per sequence)
* ``slimkv_b200.cache``      — native HBM cache layout and decode step
"""
__version__ = '0.1.0'


def library():
    """Load ``libslimkv_b200.so`` (raises if it has not been built)."""
    from . import _lib
    return _lib.load()
