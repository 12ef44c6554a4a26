"""Reconstruction decode backend: full-dimension Beacon K/V, then attention.

The reference's ``reconstruct`` decode backend (``reconstruction_attention``,
tools/benchmark/context_decode_runtime.py:298-344, built on
``ReconstructionCache.materialize``, slimkv/llama3/memory.py:26-48) rebuilds
every Beacon key and value from its latent with the up-projections each step
and runs ordinary grouped attention over the raw keys (RoPE'd) and the
reconstructed Beacon keys (no RoPE).  Here:

* ``slimkv_reconstruct_kv`` (tcgen05 GEMM, fp32 accumulation, one bf16
  rounding as a bf16 ``nn.Linear``) writes the Beacon rows of each sequence
  right after its raw rows in one ``[B, raw_capacity + latent_capacity, Hkv,
  D]`` key buffer (and the same for values), so
* one split-KV attention call per query row covers a sequence's keys as one
  contiguous range: the raw token's query sees every key except a Beacon
  inserted this step (the last key), the Beacon query sees all of them.

The latent path (:mod:`slimkv_b200.kernels` ``LatentDecodeCall``) computes
the same attention without rebuilding the keys; this backend exists for the
reference's reconstruct configurations and to compare the two.
"""
import ctypes
import math

import torch

from . import _lib
from .kernels import _bf16_cuda, _require, _stream, attention_forward


def reconstruct_kv(lat_k, lat_v, w_k_up, w_v_up, key, value, rows, b_k_up=None, b_v_up=None, out_start=None,
                   workspace=None, head_dim=None, row_count=None):
    """``key[b, out_start[b] + r] = bf16(lat_k[b, r] @ w_k_up.T + b_k_up)`` for
    ``r < rows`` and ``r < row_count[b]`` (and the same for values).
    ``lat_k / lat_v [B, cap, R]`` (rows contiguous, matching strides), ``key /
    value [B, out_rows, Hkv*D]`` with ``head_dim`` given (or ``[B, out_rows,
    Hkv, D]``) bf16, ``out_start`` and ``row_count`` int32 ``[B]`` on the
    device or ``None`` (0, and no per-sequence limit)."""
    _bf16_cuda(lat_k, lat_v, w_k_up, w_v_up, key, value)
    _require(lat_k.stride() == lat_v.stride() and lat_k.stride(-1) == 1 and lat_v.stride(-1) == 1,
             'latent caches [B, cap, R] need matching strides and contiguous rows')
    _require(key.stride() == value.stride() and key.stride(-1) == 1, 'key / value buffers need matching strides')
    batch = lat_k.shape[0]
    kvd = w_k_up.shape[0]
    _require(w_v_up.shape[0] == kvd and w_k_up.shape[1] == lat_k.shape[-1] and w_v_up.shape[1] == lat_v.shape[-1],
             'up-projection weights must be [Hkv*D, R]')
    flat_k = key.flatten(2) if key.dim() == 4 else key
    _require(flat_k.shape[-1] == kvd and flat_k.stride(-1) == 1, 'key rows must hold Hkv*D contiguous values')
    for b in (b_k_up, b_v_up):
        if b is not None:
            _bf16_cuda(b)
    for t, name in ((out_start, 'out_start'), (row_count, 'row_count')):
        if t is not None:
            _require(t.is_cuda and t.dtype == torch.int32 and t.numel() == batch and t.is_contiguous(),
                     f'{name} must be int32 [B] on the device')
    a = _lib.ReconstructArgs()
    a.batch, a.rows, a.rank_k, a.rank_v = batch, int(rows), lat_k.shape[-1], lat_v.shape[-1]
    a.head_dim = key.shape[-1] if key.dim() == 4 else int(head_dim or 0)
    _require(a.head_dim > 0 and kvd % a.head_dim == 0, 'head_dim must divide Hkv*D')
    a.kv_heads = kvd // a.head_dim
    a.lat_k, a.lat_v = lat_k.data_ptr(), lat_v.data_ptr()
    a.lat_stride_batch, a.lat_stride_row, a.lat_capacity = lat_k.stride(0), lat_k.stride(1), lat_k.shape[1]
    a.w_k_up, a.w_v_up = w_k_up.data_ptr(), w_v_up.data_ptr()
    a.b_k_up = 0 if b_k_up is None else b_k_up.data_ptr()
    a.b_v_up = 0 if b_v_up is None else b_v_up.data_ptr()
    a.key, a.value = key.data_ptr(), value.data_ptr()
    a.out_stride_batch, a.out_stride_row, a.out_rows = flat_k.stride(0), flat_k.stride(1), flat_k.shape[1]
    a.out_start = 0 if out_start is None else out_start.data_ptr()
    a.row_count = 0 if row_count is None else row_count.data_ptr()
    lib = _lib.load()
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    with torch.cuda.device(key.device):
        _lib.check(lib.slimkv_reconstruct_kv(ctypes.byref(a), _stream()))
    return key, value


class ReconstructDecode:
    """One layer's reconstruct-backend attention for fixed buffers.

    ``raw_k_rot / raw_v [B, raw_cap, Hkv, D]``: sinks, raw tail and this
    step's raw token, keys already rotated; ``lat_k / lat_v [B, lat_cap, R]``
    with this step's Beacon appended; ``raw_len / latent_len / query_len``
    int32 ``[B]`` on the device.  ``key_full / value_full`` (``[B, raw_cap +
    lat_cap, Hkv, D]``, shareable between layers) receive the raw rows and the
    reconstructed Beacon rows.  ``__call__(q_rot, out)``: ``q_rot [B, L, H, D]``
    (RoPE'd queries), ``out [B, L, H, D]`` bf16.
    """

    def __init__(self, *, raw_k_rot, raw_v, lat_k, lat_v, w_k_up, w_v_up, raw_len, latent_len, query_len,
                 key_full, value_full, b_k_up=None, b_v_up=None, scale=None, latent_rows=None):
        B, raw_cap, kv_heads, dim = raw_k_rot.shape
        _require(key_full.shape[0] == B and key_full.shape[1] >= raw_cap + lat_k.shape[1] and
                 key_full.shape[2:] == (kv_heads, dim), 'key_full must be [B, >= raw_cap + lat_cap, Hkv, D]')
        self.raw_k_rot, self.raw_v, self.lat_k, self.lat_v = raw_k_rot, raw_v, lat_k, lat_v
        self.w = (w_k_up, w_v_up, b_k_up, b_v_up)
        self.raw_len, self.latent_len, self.query_len = raw_len, latent_len, query_len
        self.key_full, self.value_full = key_full, value_full
        self.scale = scale if scale is not None else 1.0 / math.sqrt(dim)
        # Every row a sequence can hold; each sequence rebuilds only its
        # latent_len rows (the rest of the capacity is skipped on the device).
        self.rows = int(latent_rows if latent_rows is not None else lat_k.shape[1])
        self.raw_cap = raw_cap
        self.seq0 = torch.zeros(B, dtype=torch.int32, device=raw_len.device)
        self.seq1 = torch.zeros_like(self.seq0)

    def __call__(self, q_rot, out):
        w_k, w_v, b_k, b_v = self.w
        # Raw rows first (rotated keys as cached), Beacon rows right after them.
        self.key_full[:, :self.raw_cap].copy_(self.raw_k_rot)
        self.value_full[:, :self.raw_cap].copy_(self.raw_v)
        reconstruct_kv(self.lat_k, self.lat_v, w_k, w_v, self.key_full, self.value_full, self.rows, b_k, b_v,
                       out_start=self.raw_len, row_count=self.latent_len)
        total = self.raw_len + self.latent_len
        two = (self.query_len == 2).to(torch.int32)
        torch.sub(total, two, out=self.seq0)              # the raw token's query skips this step's Beacon
        torch.mul(total, two, out=self.seq1)              # the Beacon query sees every key
        for l in range(q_rot.shape[1]):
            attention_forward(q_rot[:, l:l + 1], self.key_full, self.value_full, self.scale,
                              cache_seqlens=self.seq0 if l == 0 else self.seq1, lse_masked_positive=False,
                              out=out[:, l:l + 1])
        return out
