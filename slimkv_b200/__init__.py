"""B200-native (sm_100a) SlimKV decode-time latent attention.

The hot path of SlimKV decode — attention over the compressed cache of
low-rank Beacon K/V latents plus full-dimension sinks and raw tail — as
hand-written CUDA kernels behind a C ABI (``include/slimkv_b200.h``), with
thin torch bindings that mirror the reference's Python entry points:

* ``slimkv_b200.kernels``    — torch wrappers over the C ABI
* ``slimkv_b200.fa2_decode`` — the reference's ``fa2_decode.decode`` contract
* ``slimkv_b200.extension``  — drop-in ``slimkv_fa2_decode_320`` module
* ``slimkv_b200.vllm``       — the vLLM plugin's page geometry and batched paged decode
* ``slimkv_b200.pages``      — GPU drop-in for the plugin's page classes
* ``slimkv_b200.runtime``    — CUDA-graph batched decode step of a SlimKV Llama
* ``slimkv_b200.prefill``    — prefill window projection and Beacon append
* ``slimkv_b200.prefill_attention`` — a prefill chunk's attention over its latent history
* ``slimkv_b200.reconstruct``— the reconstruct decode backend
* ``slimkv_b200.parallel``   — sequence split across GPUs, max-over-ranks timing
* ``slimkv_b200.tensor_parallel`` — decode split by KV head and by sequence across GPUs
* ``slimkv_b200.rope``       — RoPE tables built exactly like the reference
"""
__version__ = '0.2.0'


def library():
    """Load ``libslimkv_b200.so`` (raises if it has not been built)."""
    from . import _lib
    return _lib.load()
