"""Beacon interleave and decode-step schedule (oracle, test-only).

Integer bookkeeping only; results must be bit-exact with the reference.
"""
import numpy as np


def interleave_roles(input_size, remainder, ratio):
    """Roles of one interleaved chunk and the new remainder.

    Restates the interleave rule of ``Memory._step``
    (slimkv/memory.py:491-567, indices 579-589): ``beacon_size = (input_size
    + remainder) // ratio`` Beacons are inserted into ``input_size`` raw
    tokens; in the interleaved sequence of length ``input_size +
    beacon_size`` position ``i`` is a Beacon iff ``beacon_size > 0`` and
    ``i % (ratio + 1) == ratio - remainder``.  Returns ``(roles, beacon_size,
    new_remainder)`` with ``roles`` int64 (0 raw, 1 Beacon).
    """
    beacon_size = (input_size + remainder) // ratio
    total = input_size + beacon_size
    roles = np.zeros(total, dtype=np.int64)
    if beacon_size > 0:
        i = np.arange(total)
        roles[i % (ratio + 1) == ratio - remainder] = 1
    return roles, beacon_size, (input_size + remainder) % ratio


def paged_restore_roles(processed, window, ratio):
    """Window roles rebuilt from a raw-token cursor.

    Restates ``restore_memory`` (slimkv/vllm_plugin/paged_model.py:7-52):
    with ``raw = processed % window`` raw tokens in the open window there are
    ``raw // ratio`` Beacons, one after every ``ratio`` raw tokens.  Returns
    ``(roles, raw_indices, history_count, beacon_count)``.
    """
    raw = processed % window
    history = processed // window * (window // ratio)
    beacons = processed // ratio
    count = raw + raw // ratio
    roles = np.zeros(count, dtype=np.int64)
    roles[ratio::ratio + 1] = 1
    return roles, np.nonzero(roles == 0)[0], history, beacons


class FastDecodeSchedule:
    """Length and role bookkeeping of one SlimKV ``LlamaMemory``.

    Mirrors, for the latent cache mode (interleaved Beacons, one
    non-overlapping window, single token ratio, no skip overrides):

    * prefill chunks: ``Memory._step`` interleave branch and window cursor
      (slimkv/memory.py:406-666) plus ``LlamaMemory.update_memory``
      (slimkv/llama3/memory.py:233-278);
    * decode steps: the fast path ``LlamaMemory._step``
      (slimkv/llama3/memory.py:101-162): ``size = (rem + 1) // ratio``,
      roles appended with the new Beacon last, the raw index of the new raw
      token is the number of roles before it, positions ``arange(past + 1 +
      size)``; the window completes when ``end >= start + window``.

    Lengths are per layer (all layers agree) in cache rows:
    ``sink``, ``history`` (completed-window latents), ``raw`` (open-window raw
    tokens) and ``window`` (open-window Beacon latents).
    """

    def __init__(self, window, ratio, sink):
        if window % ratio:
            raise ValueError('window must be divisible by ratio')
        self.window, self.ratio, self.sink_size = window, ratio, sink
        self.start = 0
        self.seq_len = 0
        self.end = 0
        self.is_full_window = True
        self.remainder = 0
        self.roles = np.zeros(0, dtype=np.int64)
        self.window_roles = None
        self.window_raw_indices = None
        self.sink = self.history = self.raw = self.win = 0

    @property
    def past_length(self):
        return self.sink + self.history + self.raw + self.win

    def _update(self, key_rows, new_raw, new_latents, full, roles):
        # LlamaMemory.update_memory (slimkv/llama3/memory.py:233-278): while no
        # history exists the sink is re-taken from the first rows of this
        # call's keys (257-262).
        if self.history == 0 and self.sink_size > 0:
            self.sink = min(self.sink_size, key_rows)
        if full:
            self.history += self.win + new_latents
            self.raw = 0
            self.win = 0
            self.window_roles = None
            self.window_raw_indices = None
        else:
            self.raw += new_raw
            self.win += new_latents
            self.window_roles = roles != 0
            self.window_raw_indices = np.nonzero(roles == 0)[0]

    def prefill(self, count):
        """Feed ``count`` prompt tokens; returns the per-window-chunk records."""
        self.seq_len += count
        records = []
        while self.end < self.seq_len:
            start = self.start
            end = start + self.window
            full = end <= self.seq_len
            if not full:
                end = self.seq_len
            input_size = end - self.end
            roles, size, self.remainder = interleave_roles(input_size, self.remainder, self.ratio)
            if self.is_full_window:
                self.roles = np.zeros(0, dtype=np.int64)
            self.roles = np.concatenate([self.roles, roles])
            past = self.past_length
            self.is_full_window = full
            self.start = start + self.window if full else start
            self.end = end
            records.append(dict(size=size, roles=self.roles.copy(), positions=past + len(roles),
                                full=full))
            self._update(input_size + size, input_size, size, full, self.roles)
        return records

    def decode(self):
        """One decode step of the fast path; returns its metadata record."""
        self.seq_len += 1
        start, end = self.start, self.seq_len
        full = end >= start + self.window
        if self.is_full_window:
            previous_roles, previous_raw = 0, 0
            self.roles = np.zeros(0, dtype=np.int64)
            raw_indices = np.zeros(0, dtype=np.int64)
        else:
            previous_roles = len(self.roles)
            raw_indices = (np.zeros(0, dtype=np.int64) if self.window_raw_indices is None
                           else self.window_raw_indices.copy())
            previous_raw = len(raw_indices)
        size = (self.remainder + 1) // self.ratio
        self.remainder = (self.remainder + 1) % self.ratio
        new = np.zeros(1 + size, dtype=np.int64)
        if size:
            new[-1] = 1
        self.roles = np.concatenate([self.roles[:previous_roles], new])
        raw_indices = np.concatenate([raw_indices[:previous_raw], [previous_roles]]).astype(np.int64)
        past = self.past_length
        record = dict(size=size, roles=self.roles.copy(), raw_indices=raw_indices.copy(),
                      positions=past + 1 + size, full=full,
                      sink=self.sink, history=self.history, raw=self.raw, window=self.win)
        self.is_full_window = full
        self.start = start + self.window if full else start
        self.end = end
        self._update(1, 1, size, full, self.roles)
        if not full:
            self.window_raw_indices = raw_indices
        return record
