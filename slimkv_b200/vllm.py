"""The vLLM plugin's paged-cache interface on the fused sm_100a decode.

The reference plugin (slimkv/vllm_plugin/) lets vLLM own two page sets per
layer — raw pages ``[blocks, 16, 2, Hkv, D]`` (pre-RoPE K/V by absolute raw
position) and compact Beacon pages ``[blocks, rows, Rk + Rv]`` (the sink token
in the root page, then one ``[k | v]`` latent row per slot) — and runs every
request on its own: ``restore_memory`` gathers its pages into the model's
Memory, the HF model runs, ``flush_memory`` scatters the new rows back
(``SlimKVLlamaForCausalLM._paged_forward``, vllm_plugin/model.py:114-142;
paged_model.py:7-83).

Here:

* :class:`RawPageBackend` / :class:`BeaconPageBackend` keep the reference
  backends' cache geometry (``get_kv_cache_shape``,
  ``get_kv_cache_stride_order``, ``indexes_kv_by_block_stride``;
  vllm_plugin/backend.py:45-95) and :func:`beacon_block_size` /
  :func:`storage_block_size` its page arithmetic (backend.py:13-29,
  108-131), so pages allocated for the reference are read here unchanged;
* :class:`PagedDecodeLayer` replaces the per-request restore / decode / flush
  loop for a decode step with one batched call per layer, driven by the
  plugin's metadata (``common_attn_metadata``: per-request block-table rows,
  ``query_start_loc``, ``seq_lens``): every request's Beacon schedule is
  derived on the device from its sequence length, the raw tail is read from
  the raw pages and rotated at its compressed positions, the fused decode
  reads the latent rows straight from the Beacon pages (appending this step's
  Beacon row into its page), and the new raw token is written to its raw page.

Everything runs on the device without host synchronisation, so a decode step
can be captured in a CUDA graph.
"""
import ctypes
import math

import torch

from . import _lib, kernels, pages as P


class RawPageBackend:
    """Geometry of the plugin's raw KV pages (``SLIMKV_RAW``)."""

    @staticmethod
    def get_name():
        return 'SLIMKV_RAW'

    @staticmethod
    def get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size, cache_dtype_str='auto'):
        return num_blocks, block_size, 2, num_kv_heads, head_size

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension=False):
        return (1, 0, 2, 3, 4, 5) if include_num_layers_dimension else (0, 1, 2, 3, 4)

    @classmethod
    def indexes_kv_by_block_stride(cls):
        return True


class BeaconPageBackend(RawPageBackend):
    """Geometry of the plugin's compact Beacon pages (``SLIMKV_BEACON``)."""

    @staticmethod
    def get_name():
        return 'SLIMKV_BEACON'

    @staticmethod
    def get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size, cache_dtype_str='auto'):
        return num_blocks, block_size, head_size

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension=False):
        return (1, 0, 2, 3) if include_num_layers_dimension else (0, 1, 2)


beacon_block_size = P.beacon_block_size


def storage_block_size(block_size, token_ratio, raw_width, head_size):
    """Rows of ``head_size`` elements a Beacon page stores
    (``BeaconSpec.storage_block_size``, backend.py:18-20): the slots plus the
    rows the sink token's K and V occupy."""
    return block_size // token_ratio + (2 * raw_width + head_size - 1) // head_size


class PagedDecodeLayer:
    """One layer's decode attention over vLLM pages, batched over requests.

    ``raw_pages`` ``[blocks, 16, 2, Hkv, D]`` and ``beacon_pages`` ``[blocks,
    rows, Rk + Rv]`` are the layer's engine-owned caches; ``layout`` the
    Beacon page layout (:class:`slimkv_b200.pages.BeaconPageLayout`); ``uk``
    / ``uv`` the up-projection weights (and optional biases); ``cos`` /
    ``sin`` the fp32 rotary tables.  ``window``, ``ratio`` and ``sink`` (0 or
    1, as the plugin's paged mode allows) are the Beacon configuration;
    ``max_batch`` sizes the device buffers.

    ``__call__(q, new_k, new_v, new_lat_k, new_lat_v, seq_lens, raw_table,
    beacon_table, out)`` runs one decode step: ``q [B, 2, H, D]`` pre-RoPE
    queries of the raw token and of the Beacon slot (used only by requests
    that insert a Beacon this step), ``new_k / new_v [B, Hkv*D]`` the raw
    token's pre-RoPE K/V, ``new_lat_k / new_lat_v [B, R]`` the Beacon slot's
    latents, ``seq_lens`` int32 ``[B]`` the tokens of each request including
    this step's (vLLM's ``seq_lens``), ``raw_table`` / ``beacon_table`` int32
    block-table rows ``[B, n]``; writes ``out [B, 2, H*D]``.
    """

    def __init__(self, raw_pages, beacon_pages, layout, uk, uv, cos, sin, *, window, ratio, sink, max_batch,
                 uk_bias=None, uv_bias=None, heads):
        if sink not in (0, 1):
            raise ValueError('Paged SlimKV keeps at most one sink token (vllm_plugin/model.py:49-58).')
        if window % ratio:
            raise ValueError('The window must hold whole Beacon groups.')
        self.raw_pages, self.beacon_pages, self.layout = raw_pages, beacon_pages, layout
        self.uk, self.uv, self.uk_bias, self.uv_bias = uk, uv, uk_bias, uv_bias
        self.cos, self.sin = cos, sin
        self.window, self.ratio, self.sink, self.heads = window, ratio, sink, heads
        dev = raw_pages.device
        self.kv_heads, self.head_dim = raw_pages.shape[3], raw_pages.shape[4]
        self.cap = (sink + window + 1 + 63) // 64 * 64
        B = max_batch
        i32 = dict(dtype=torch.int32, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        # Raw workspace: pre-RoPE rows read from the pages, rotated rows for the
        # fused decode (which appends this step's token), values.
        self.raw_pre = torch.zeros(B, self.cap, self.kv_heads, self.head_dim, **bf)
        self.raw_rot = torch.zeros_like(self.raw_pre)
        self.raw_v = torch.zeros_like(self.raw_pre)
        self.history, self.tail = torch.zeros(B, **i32), torch.zeros(B, **i32)
        self.raw_len, self.latent_len = torch.zeros(B, **i32), torch.zeros(B, **i32)
        self.query_len, self.qpos = torch.zeros(B, **i32), torch.zeros(B, 2, **i32)
        self.raw_start, self.raw_count = torch.zeros(B, **i32), torch.zeros(B, **i32)
        self.rot_count = torch.zeros(B, **i32)
        self.positions = torch.zeros(B, self.cap, **i32)
        self._token = torch.arange(self.cap, dtype=torch.int32, device=dev)

    def schedule(self, seq_lens):
        """The Beacon schedule of this step for each request (the per-request
        state ``restore_memory`` rebuilds from the processed-token count,
        paged_model.py:7-33, advanced by one raw token): ``processed = seq_len
        - 1`` tokens are in the pages."""
        B = seq_lens.numel()
        per_window = self.window // self.ratio
        processed = seq_lens.to(torch.int32) - 1
        torch.remainder(processed, self.window, out=self.tail[:B])
        torch.mul(torch.div(processed, self.window, rounding_mode='floor'), per_window, out=self.history[:B])
        torch.sub(processed, self.tail[:B], out=self.raw_start[:B])
        self.raw_count[:B].copy_(self.tail[:B])
        tail0 = self.tail[:B].clone()
        hist0 = self.history[:B].clone()
        # query_len / raw_len / latent_len / qpos from (history, tail); the
        # counters it advances are scratch copies.
        kernels.decode_schedule(self.history[:B], self.tail[:B], self.raw_len[:B], self.latent_len[:B],
                                self.query_len[:B], self.qpos[:B], self.sink, self.window, self.ratio)
        # Compressed positions of the rows to rotate: sink s -> s; raw token i
        # of the open window -> i + i // ratio + sink + history (fa2_decode.py:127-131).
        t = self._token[None].expand(B, -1)
        i = t - self.sink
        raw_pos = i + torch.div(i, self.ratio, rounding_mode='floor') + self.sink + hist0[:, None]
        torch.where(t < self.sink, t, raw_pos, out=self.positions[:B])
        torch.add(tail0, self.sink, out=self.rot_count[:B])
        return processed

    def __call__(self, q, new_k, new_v, new_lat_k, new_lat_v, seq_lens, raw_table, beacon_table, out):
        B = q.shape[0]
        processed = self.schedule(seq_lens)
        # Restore the raw rows: the sink from the root Beacon page, the open
        # window's raw tail from the raw pages (pre-RoPE).
        if self.sink:
            bp = P.BeaconPages(self.beacon_pages, self.layout)
            a = bp._args(P._table(beacon_table, self.beacon_pages.device))
            flat_k = self.raw_pre[:B, 0].reshape(B, -1)
            flat_v = self.raw_v[:B, 0].reshape(B, -1)
            _lib.check(_lib.load().slimkv_beacon_pages_sink(ctypes.byref(a), B, flat_k.data_ptr(), flat_v.data_ptr(),
                                                            flat_k.stride(0), 0, P._stream()))
        P.raw_read(self.raw_pages, raw_table, self.raw_start[:B], self.raw_count[:B], self.raw_pre[:B, self.sink:],
                   self.raw_v[:B, self.sink:])
        kernels.rope_rows(self.raw_pre[:B], self.positions[:B], self.cos, self.sin, counts=self.rot_count[:B],
                          out=self.raw_rot[:B])
        call = kernels.LatentDecodeCall(
            q=q, raw_k_rot=self.raw_rot[:B], raw_v=self.raw_v[:B], lat_pages=(self.beacon_pages, self.layout,
                                                                             beacon_table),
            raw_len=self.raw_len[:B], latent_len=self.latent_len[:B], query_len=self.query_len[:B],
            qpos=self.qpos[:B], uk=self.uk, uv=self.uv, uk_bias=self.uk_bias, uv_bias=self.uv_bias,
            cos=self.cos, sin=self.sin, out=out, new_k=new_k, new_v=new_v, new_lat_k=new_lat_k,
            new_lat_v=new_lat_v, scale=1.0 / math.sqrt(self.head_dim),
            latent_len_max=beacon_table.shape[1] * self.layout.slots, raw_len_max=self.cap)
        call()
        # Flush: this step's raw token to its raw page (pre-RoPE K, V);
        # the Beacon row went into its page inside the fused decode.
        P.raw_write(self.raw_pages, raw_table, processed, new_k.view(B, 1, self.kv_heads, self.head_dim),
                    new_v.view(B, 1, self.kv_heads, self.head_dim))
        return out
