"""Paged SlimKV cache IO on the GPU: drop-in for the vLLM plugin's page classes.

Mirrors ``slimkv/vllm_plugin/paged_cache.py:12-127`` - the same classes,
constructor checks, error messages and return shapes - with every copy done by
the library's CUDA kernels (``slimkv_beacon_pages_*`` / ``slimkv_raw_pages_*``)
instead of torch advanced indexing.  Page bytes are identical.  The batched
functions at the end serve several sequences (one block-table row each) per
launch.
"""
import ctypes
from dataclasses import dataclass

import torch

from . import _lib


@dataclass(frozen=True)
class BeaconPageLayout:
    """Compact Beacon page geometry (paged_cache.py:12-44): a page holds
    ``[2 * raw_width sink elements][slots x (key_rank + value_rank)]``."""
    raw_block_size: int
    token_ratio: int
    key_rank: int
    value_rank: int
    raw_width: int

    def __post_init__(self):
        if min(self.raw_block_size, self.token_ratio, self.key_rank,
               self.value_rank, self.raw_width) <= 0:
            raise ValueError('Cache dimensions must be positive.')
        if self.raw_block_size % self.token_ratio:
            raise ValueError('Raw block size must be divisible by the token ratio.')

    @property
    def slots(self):
        return self.raw_block_size // self.token_ratio

    @property
    def width(self):
        return self.key_rank + self.value_rank

    @property
    def sink_elements(self):
        return 2 * self.raw_width

    @property
    def page_elements(self):
        return self.sink_elements + self.slots * self.width

    @property
    def storage_rows(self):
        return (self.page_elements + self.width - 1) // self.width


def beacon_block_size(ratio, raw_width, max_width, raw_block=16):
    """Raw tokens one Beacon page covers in the vLLM backend
    (``create_page_layers``, slimkv/vllm_plugin/backend.py:108-118): the page
    has the bytes of a ``raw_block``-token raw page; after the sink it holds
    ``(elements - 2 * raw_width) // max_width`` slots of ``ratio`` raw tokens,
    rounded down to a multiple of ``raw_block``."""
    page_bytes = raw_block * 2 * raw_width * 2
    block = (((page_bytes // 2 - 2 * raw_width) // max_width) * ratio // raw_block) * raw_block
    if block < raw_block or block % ratio:
        raise ValueError('Cannot represent the selected token ratio in compact pages.')
    return block


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _table(block_table, device):
    t = torch.as_tensor(block_table).to(device=device, dtype=torch.int32)
    return t.reshape(-1, t.shape[-1]).contiguous() if t.dim() else t.reshape(1, 1)


def _cursor(values, device):
    return torch.as_tensor(values, dtype=torch.int32).reshape(-1).to(device)


def _require_cuda(t):
    if not t.is_cuda:
        raise RuntimeError('slimkv_b200 page IO runs on CUDA tensors')


class BeaconPages:
    """Read and append compact rows without owning or allocating KV pages."""

    def __init__(self, pages, layout):
        if pages.dtype != torch.bfloat16:
            raise ValueError('SlimKV pages must retain BF16 checkpoint precision.')
        self.pages = pages.flatten(1)
        if self.pages.data_ptr() != pages.data_ptr():
            raise ValueError('Each physical page must have contiguous feature storage.')
        if self.pages.shape[1] < layout.page_elements:
            raise ValueError('Physical page is too small for the declared ranks.')
        self.layout = layout

    def _args(self, table):
        _require_cuda(self.pages)
        a = _lib.BeaconPagesArgs()
        a.pages = self.pages.data_ptr()
        a.page_stride = self.pages.stride(0)
        a.slots = self.layout.slots
        a.rank_k, a.rank_v = self.layout.key_rank, self.layout.value_rank
        a.sink_elements = self.layout.sink_elements
        a.table, a.table_stride = table.data_ptr(), table.shape[-1]
        a.num_pages = self.pages.shape[0]
        return a

    def read(self, block_table, count):
        if count == 0:
            return None, None
        table = _table(block_table, self.pages.device)[:1]
        dev = self.pages.device
        k = torch.empty(1, 1, count, self.layout.key_rank, dtype=torch.bfloat16, device=dev)
        v = torch.empty(1, 1, count, self.layout.value_rank, dtype=torch.bfloat16, device=dev)
        n = _cursor([count], dev)
        a = self._args(table)
        _lib.check(_lib.load().slimkv_beacon_pages_gather(ctypes.byref(a), 1, n.data_ptr(), count, k.data_ptr(),
                                                          0, k.stride(2), v.data_ptr(), 0, v.stride(2), _stream()))
        return k, v

    def append(self, block_table, start, key, value):
        if key.dtype != self.pages.dtype or value.dtype != self.pages.dtype:
            raise ValueError('Cache writes must not change dtype.')
        if (key.ndim != 4 or value.ndim != 4 or key.shape[:2] != (1, 1)
                or value.shape[:3] != key.shape[:3]
                or key.shape[-1] != self.layout.key_rank
                or value.shape[-1] != self.layout.value_rank):
            raise ValueError('Expected independent B1 global-rank K/V tensors.')
        count = key.shape[2]
        if count == 0:
            return
        key = key if key.stride(-1) == 1 else key.contiguous()
        value = value if value.stride(-1) == 1 else value.contiguous()
        table = _table(block_table, self.pages.device)[:1]
        s = _cursor([start], self.pages.device)
        a = self._args(table)
        _lib.check(_lib.load().slimkv_beacon_pages_append(ctypes.byref(a), 1, s.data_ptr(), count, key.data_ptr(), 0,
                                                          key.stride(2), value.data_ptr(), 0, value.stride(2),
                                                          _stream()))

    def write_sink(self, root_block, key, value):
        if key.numel() + value.numel() != self.layout.sink_elements or key.dtype != self.pages.dtype \
                or value.dtype != self.pages.dtype or key.numel() != value.numel():
            raise ValueError('Sink cache must retain the original raw K/V dimensions.')
        k = key.reshape(1, -1).contiguous()
        v = value.reshape(1, -1).contiguous()
        table = _table([int(root_block)], self.pages.device)
        a = self._args(table)
        _lib.check(_lib.load().slimkv_beacon_pages_sink(ctypes.byref(a), 1, k.data_ptr(), v.data_ptr(), 0, 1,
                                                        _stream()))

    def read_sink(self, root_block, heads, head_dim):
        if heads * head_dim != self.layout.raw_width:
            raise ValueError('Sink head dimensions differ from the page layout.')
        dev = self.pages.device
        k = torch.empty(1, heads * head_dim, dtype=torch.bfloat16, device=dev)
        v = torch.empty_like(k)
        table = _table([int(root_block)], dev)
        a = self._args(table)
        _lib.check(_lib.load().slimkv_beacon_pages_sink(ctypes.byref(a), 1, k.data_ptr(), v.data_ptr(), 0, 0,
                                                        _stream()))
        return tuple(x.reshape(1, heads, 1, head_dim) for x in (k, v))


class RawPages:
    """Read current-window raw KV using absolute raw-token positions."""

    def __init__(self, pages):
        if pages.dtype != torch.bfloat16 or pages.ndim != 5 or pages.shape[2] != 2:
            raise ValueError('Expected BF16 pages in block/token/KV/head/dim order.')
        self.pages = pages
        self.block_size = pages.shape[1]

    def _args(self, table):
        _require_cuda(self.pages)
        if not self.pages.is_contiguous():
            raise ValueError('Raw pages must be contiguous.')
        a = _lib.RawPagesArgs()
        a.pages = self.pages.data_ptr()
        a.block_size, a.kv_heads, a.head_dim = self.block_size, self.pages.shape[3], self.pages.shape[4]
        a.table, a.table_stride = table.data_ptr(), table.shape[-1]
        a.num_blocks = self.pages.shape[0]
        return a

    def read(self, block_table, start, count):
        if count == 0:
            return None, None
        dev = self.pages.device
        heads, dim = self.pages.shape[3], self.pages.shape[4]
        k = torch.empty(1, count, heads, dim, dtype=torch.bfloat16, device=dev)
        v = torch.empty_like(k)
        table = _table(block_table, dev)[:1]
        s, n = _cursor([start], dev), _cursor([count], dev)
        a = self._args(table)
        _lib.check(_lib.load().slimkv_raw_pages_read(ctypes.byref(a), 1, s.data_ptr(), n.data_ptr(), count,
                                                     k.data_ptr(), 0, k.stride(1), v.data_ptr(), 0, v.stride(1),
                                                     _stream()))
        return tuple(x[0].transpose(0, 1)[None] for x in (k, v))

    def write(self, block_table, start, key, value):
        if key.dtype != self.pages.dtype or value.dtype != self.pages.dtype:
            raise ValueError('Raw cache writes must retain BF16 values.')
        rows_k = key[0].transpose(0, 1).contiguous()          # [T, H, D]
        rows_v = value[0].transpose(0, 1).contiguous()
        if rows_k.shape[1:] != self.pages.shape[3:] or rows_v.shape != rows_k.shape:
            raise ValueError('Raw cache dimensions differ from the engine allocation.')
        count = rows_k.shape[0]
        if count == 0:
            return
        table = _table(block_table, self.pages.device)[:1]
        s = _cursor([start], self.pages.device)
        a = self._args(table)
        _lib.check(_lib.load().slimkv_raw_pages_write(ctypes.byref(a), 1, s.data_ptr(), count, rows_k.data_ptr(), 0,
                                                      rows_k.stride(0), rows_v.data_ptr(), 0, rows_v.stride(0),
                                                      _stream()))


# ---- batched forms (one block-table row and cursor per sequence) -----------

def beacon_append(pages, layout, tables, start, key, value):
    """Append ``key/value [B, n, R]`` at logical rows ``start[b]..start[b]+n``
    of each sequence's Beacon pages (``tables [B, pages_per_seq]``)."""
    bp = BeaconPages(pages, layout)
    tables = _table(tables, bp.pages.device)
    a = bp._args(tables)
    s = _cursor(start, bp.pages.device)
    _lib.check(_lib.load().slimkv_beacon_pages_append(ctypes.byref(a), key.shape[0], s.data_ptr(), key.shape[1],
                                                      key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
                                                      value.stride(0), value.stride(1), _stream()))


def beacon_gather(pages, layout, tables, count, key, value):
    """Gather the first ``count[b]`` rows of each sequence into dense
    ``key/value [B, cap, R]``."""
    bp = BeaconPages(pages, layout)
    tables = _table(tables, bp.pages.device)
    a = bp._args(tables)
    n = _cursor(count, bp.pages.device)
    _lib.check(_lib.load().slimkv_beacon_pages_gather(ctypes.byref(a), key.shape[0], n.data_ptr(), key.shape[1],
                                                      key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
                                                      value.stride(0), value.stride(1), _stream()))


def raw_write(pages, tables, start, key, value):
    """Write ``key/value [B, n, Hkv, D]`` at raw positions ``start[b]..`` of
    each sequence's raw pages."""
    rp = RawPages(pages)
    tables = _table(tables, pages.device)
    a = rp._args(tables)
    s = _cursor(start, pages.device)
    _lib.check(_lib.load().slimkv_raw_pages_write(ctypes.byref(a), key.shape[0], s.data_ptr(), key.shape[1],
                                                  key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
                                                  value.stride(0), value.stride(1), _stream()))


def raw_read(pages, tables, start, count, key, value):
    """Read ``count[b]`` raw tokens from ``start[b]`` into ``key/value [B, cap, Hkv, D]``."""
    rp = RawPages(pages)
    tables = _table(tables, pages.device)
    a = rp._args(tables)
    s, n = _cursor(start, pages.device), _cursor(count, pages.device)
    _lib.check(_lib.load().slimkv_raw_pages_read(ctypes.byref(a), key.shape[0], s.data_ptr(), n.data_ptr(),
                                                 key.shape[1], key.data_ptr(), key.stride(0), key.stride(1),
                                                 value.data_ptr(), value.stride(0), value.stride(1), _stream()))
