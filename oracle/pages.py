"""Paged SlimKV cache addressing (oracle, test-only).  Bit-exact integer work."""
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class BeaconPageLayout:
    """Compact Beacon page geometry.

    Restates ``BeaconPageLayout`` (slimkv/vllm_plugin/paged_cache.py:12-44):
    a page holds ``[2*raw_width sink elements][slots x (key_rank+value_rank)]``
    bf16 values, ``slots = raw_block_size // token_ratio``.
    """
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


def beacon_page_slots(table, start, count, layout):
    """Physical page and first element of logical Beacons ``start..start+count``.

    Restates ``BeaconPages._indices`` (slimkv/vllm_plugin/paged_cache.py:55-62):
    logical Beacon ``n`` lives in page ``table[n // slots]`` at element
    ``sink_elements + (n % slots) * width`` of that page.
    """
    n = np.arange(start, start + count, dtype=np.int64)
    table = np.asarray(table, dtype=np.int64)
    return table[n // layout.slots], layout.sink_elements + (n % layout.slots) * layout.width


def raw_page_slots(table, start, count, block_size):
    """Physical block and row of absolute raw positions ``start..start+count``.

    Restates ``RawPages.read/write`` addressing
    (slimkv/vllm_plugin/paged_cache.py:111-127).
    """
    p = np.arange(start, start + count, dtype=np.int64)
    table = np.asarray(table, dtype=np.int64)
    return table[p // block_size], p % block_size


def beacon_block_size(ratio, raw_width, max_width, raw_block=16):
    """Raw tokens covered by one Beacon page of the vLLM backend.

    Restates ``create_page_layers`` (slimkv/vllm_plugin/backend.py:108-118):
    a Beacon page has the byte size of a raw page, ``raw_block * 2 *
    raw_width * 2`` bytes; after the sink it holds ``(elements - 2 *
    raw_width) // max_width`` slots, i.e. that many times ``ratio`` raw
    tokens, rounded down to a multiple of ``raw_block``.
    """
    page_bytes = raw_block * 2 * raw_width * 2
    block = (((page_bytes // 2 - 2 * raw_width) // max_width) * ratio // raw_block) * raw_block
    if block < raw_block or block % ratio:
        raise ValueError('Cannot represent the selected token ratio in compact pages.')
    return block


def beacon_pages_append(pages, table, start, key, value, layout):
    """Write latent rows into flat pages ``pages [num_pages, >= page_elements]``.

    Restates ``BeaconPages.append`` (slimkv/vllm_plugin/paged_cache.py:78-87):
    row ``i`` is ``cat(key[i], value[i])`` stored at its logical slot.
    """
    page, col = beacon_page_slots(table, start, key.shape[0], layout)
    rows = np.concatenate([key, value], axis=-1)
    for i in range(rows.shape[0]):
        pages[page[i], col[i]:col[i] + layout.width] = rows[i]


def beacon_pages_read(pages, table, count, layout):
    """Read the first ``count`` latent rows as ``(key [count, Rk], value [count, Rv])``."""
    page, col = beacon_page_slots(table, 0, count, layout)
    rows = np.stack([pages[page[i], col[i]:col[i] + layout.width] for i in range(count)]) \
        if count else np.zeros((0, layout.width), pages.dtype)
    return rows[:, :layout.key_rank], rows[:, layout.key_rank:]
