"""Prefill window compression and Beacon append on the GPU.

Drop-in for the prefill side of the reference's latent-cache path:

* ``prepare_metadata`` / ``PrefillMetadata`` (slimkv/llama3/prefill_ops.py:
  9-36): the chunk's raw and Beacon row index lists;
* ``fused_prefill_rope`` (prefill_ops.py:48-74, kernel prefill_kernels.py:
  7-53): BF16-exact rotary of q and k with Beacon keys left unrotated;
* ``qkv_proj_with_beacon`` + ``_incremental_cache`` (slimkv/llama3/
  modeling_llama.py:1291-1367): every chunk row projected by the weights its
  role selects (raw rows: q/k/v_proj; Beacon rows: beacon_q_proj and the
  low-rank K/V down- and up-projections), the Beacon latents packed for the
  latent cache;
* the cache writes that follow (``Memory.update_memory``, slimkv/llama3/
  memory.py:233-278, and ``flush_memory``, slimkv/vllm_plugin/
  paged_model.py:55-83): Beacon latents into a dense latent cache or the
  vLLM plugin's Beacon pages, raw K/V rows into a dense raw cache or raw
  pages, the first raw token into the root page's sink.

All of it runs in ``slimkv_window_project`` (one tcgen05 launch for the
projections that read the hidden rows, one for the Beacon up-projection) and
``slimkv_prefill_rope``; there is no CPU fallback.
"""
import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .pages import BeaconPages, RawPages


@dataclass
class PrefillMetadata:
    """Same fields as the reference's ``PrefillMetadata`` (prefill_ops.py:9-14)."""
    raw_indices: torch.Tensor
    beacon_indices: torch.Tensor
    roles: torch.Tensor
    positions: Optional[torch.Tensor]
    replicas: bool


def window_roles(input_size, remainder, ratio):
    """Roles of one interleaved chunk (``Memory._step``, slimkv/memory.py:
    491-567, indices 579-589): ``(input_size + remainder) // ratio`` Beacons
    among ``input_size`` raw tokens, position ``i`` of the interleaved chunk a
    Beacon iff ``i % (ratio + 1) == ratio - remainder``.  Returns ``(roles
    int64 tensor (0 raw, 1 Beacon), beacon_count, new_remainder)`` on the CPU."""
    beacons = (input_size + remainder) // ratio
    i = torch.arange(input_size + beacons)
    roles = ((i % (ratio + 1)) == (ratio - remainder)).long() if beacons > 0 else torch.zeros_like(i)
    return roles, beacons, (input_size + remainder) % ratio


def metadata_from_roles(roles, chunk_rows, positions=None):
    """The index lists ``prepare_metadata`` builds (prefill_ops.py:31-36):
    the chunk is the last ``chunk_rows`` window roles; role 0 rows are raw,
    every other role is a Beacon row (2 = replica)."""
    current = roles[-chunk_rows:] if chunk_rows else roles[:0]
    return PrefillMetadata((current == 0).nonzero().flatten(), (current != 0).nonzero().flatten(), roles, positions,
                           bool((current == 2).any()))


@dataclass
class BeaconProjectionWeights:
    """nn.Linear weights ``[out, in]`` (bf16, CUDA) of one attention layer."""
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    bq: torch.Tensor
    k_down: torch.Tensor
    v_down: torch.Tensor
    k_up: torch.Tensor
    v_up: torch.Tensor
    q_bias: Optional[torch.Tensor] = None
    k_bias: Optional[torch.Tensor] = None
    v_bias: Optional[torch.Tensor] = None
    bq_bias: Optional[torch.Tensor] = None
    k_up_bias: Optional[torch.Tensor] = None
    v_up_bias: Optional[torch.Tensor] = None

    @classmethod
    def from_attention(cls, attn):
        """Weights of a reference ``LlamaAttention`` with low-rank Beacon K/V
        (modeling_llama.py:237-250, 369-381, 432-444)."""
        if getattr(attn.config, 'beacon_headwise_up_proj', False):
            raise NotImplementedError('headwise Beacon up-projections are not supported by slimkv_b200')
        shared = getattr(attn.config, 'beacon_shared_kv_down_proj', False)
        kd = attn.beacon_kv_down_proj if shared else attn.beacon_k_down_proj
        vd = attn.beacon_kv_down_proj if shared else attn.beacon_v_down_proj

        def w(m):
            return m.weight.detach()

        def b(m):
            return None if m.bias is None else m.bias.detach()

        return cls(q=w(attn.q_proj), k=w(attn.k_proj), v=w(attn.v_proj), bq=w(attn.beacon_q_proj), k_down=w(kd),
                   v_down=w(vd), k_up=w(attn.beacon_k_up_proj), v_up=w(attn.beacon_v_up_proj),
                   q_bias=b(attn.q_proj), k_bias=b(attn.k_proj), v_bias=b(attn.v_proj),
                   bq_bias=b(attn.beacon_q_proj), k_up_bias=b(attn.beacon_k_up_proj),
                   v_up_bias=b(attn.beacon_v_up_proj))


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def _weight(t, name, device):
    if t is None:
        return None
    if t.dtype != torch.bfloat16 or t.device != device:
        raise ValueError(f'{name} must be a bf16 tensor on {device}')
    return t.contiguous()


_WORKSPACE = {}


def _workspace(device, nbytes):
    """Split-K scratch per device, grown on demand.  Calls that share it run
    on one stream."""
    ws = _WORKSPACE.get(device)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACE[device] = ws
    return ws


def _i32(t, device):
    return None if t is None else torch.as_tensor(t).to(device=device, dtype=torch.int32).reshape(-1).contiguous()


def project_window(weights, hidden, metadata, heads, kv_heads, head_dim, *, query=True, key=True, value=True,
                   latents=True, latent_cache=None, lat_start=None, beacon=None, raw_start=None, raw_first=0,
                   raw_cache=None, raw=None, write_sink=False, split=True):
    """Project one interleaved chunk ``hidden [B, n, hidden]`` and append it.

    ``metadata`` gives the chunk's raw / Beacon row lists (``raw_indices``,
    ``beacon_indices``, shared by the batch).  Chunk outputs (pre-RoPE,
    ``[B, n, .]``) are returned for ``query`` / ``key`` / ``value``; Beacon
    latents as ``key_latents`` / ``value_latents`` ``[B, 1, n_beacon, R]``
    (``ReconstructionCacheUpdate`` packing for latent decode).  Cache targets:

    * ``latent_cache=(lat_k [B, cap, Rk], lat_v [B, cap, Rv])``: latents go
      to rows ``lat_start[b] + j`` instead of a per-chunk tensor;
    * ``beacon=(BeaconPages, block_tables [B, pages])``: latents appended at
      logical rows ``lat_start[b] + j`` (``BeaconPages.append``);
    * ``raw_cache=(k [B, cap, Hkv, D], v)`` or ``raw=(RawPages,
      block_tables)``: raw row ``i >= raw_first`` at position
      ``raw_start[b] + i`` (``RawPages.write``);
    * ``write_sink``: the raw token at position 0 into the root Beacon
      page's sink (``BeaconPages.write_sink``).

    ``split=False`` keeps every reduction in one CTA even when the call has
    fewer output tiles than SMs (no split-K workspace).
    """
    if metadata.replicas:
        raise NotImplementedError('replica Beacon rows (parallel windows) are not on the prefill fast path')
    if hidden.dtype != torch.bfloat16 or hidden.dim() != 3 or not hidden.is_cuda:
        raise ValueError('hidden must be a bf16 CUDA tensor [B, n, hidden]')
    dev = hidden.device
    if hidden.stride(-1) != 1:
        hidden = hidden.contiguous()
    B, n, hs = hidden.shape
    W = weights
    qd, kvd = heads * head_dim, kv_heads * head_dim
    rank_k, rank_v = W.k_down.shape[0], W.v_down.shape[0]
    raw_rows = _i32(metadata.raw_indices, dev)
    beacon_rows = _i32(metadata.beacon_indices, dev)
    nb = beacon_rows.numel()
    bf = dict(dtype=torch.bfloat16, device=dev)
    out = {}
    a = _lib.WindowProjectArgs()
    a.batch, a.rows, a.hidden = B, n, hs
    a.hidden_states, a.hidden_stride_batch, a.hidden_stride_row = hidden.data_ptr(), hidden.stride(0), hidden.stride(1)
    a.raw_rows, a.raw_count = raw_rows.data_ptr(), raw_rows.numel()
    a.beacon_rows, a.beacon_count = beacon_rows.data_ptr(), nb
    a.heads, a.kv_heads, a.head_dim, a.rank_k, a.rank_v = heads, kv_heads, head_dim, rank_k, rank_v
    keep = []
    for field, t in [('w_q', W.q), ('b_q', W.q_bias), ('w_k', W.k), ('b_k', W.k_bias), ('w_v', W.v),
                     ('b_v', W.v_bias), ('w_bq', W.bq), ('b_bq', W.bq_bias), ('w_k_down', W.k_down),
                     ('w_v_down', W.v_down), ('w_k_up', W.k_up), ('b_k_up', W.k_up_bias), ('w_v_up', W.v_up),
                     ('b_v_up', W.v_up_bias)]:
        t = _weight(t, field, dev)
        keep.append(t)
        setattr(a, field, _ptr(t))
    if query:
        out['query'] = torch.empty(B, n, qd, **bf)
        a.query, a.query_stride_batch, a.query_stride_row = out['query'].data_ptr(), n * qd, qd
    if key:
        out['key'] = torch.empty(B, n, kvd, **bf)
        a.key, a.key_stride_batch, a.key_stride_row = out['key'].data_ptr(), n * kvd, kvd
    if value:
        out['value'] = torch.empty(B, n, kvd, **bf)
        a.value, a.value_stride_batch, a.value_stride_row = out['value'].data_ptr(), n * kvd, kvd
    starts = {}
    if lat_start is not None:
        starts['lat'] = _i32(lat_start, dev)
        a.beacon_start = starts['lat'].data_ptr()
    if raw_start is not None:
        starts['raw'] = _i32(raw_start, dev)
        a.raw_start = starts['raw'].data_ptr()
    if latent_cache is not None:
        lk, lv = latent_cache
        if lat_start is None:
            raise ValueError('a latent cache needs lat_start')
        if lk.stride(-1) != 1 or lv.stride(-1) != 1 or lk.shape[1] != lv.shape[1]:
            raise ValueError('latent caches must be [B, cap, R] with contiguous rows')
        a.key_latent, a.key_latent_stride_batch, a.key_latent_stride_row = lk.data_ptr(), lk.stride(0), lk.stride(1)
        a.value_latent, a.value_latent_stride_batch, a.value_latent_stride_row = (lv.data_ptr(), lv.stride(0),
                                                                                 lv.stride(1))
        a.latent_rows = lk.shape[1]
        a.latent_start = starts['lat'].data_ptr()
    elif latents or (nb and (key or value)):
        lk = torch.empty(B, nb, rank_k, **bf)
        lv = torch.empty(B, nb, rank_v, **bf)
        a.key_latent, a.key_latent_stride_batch, a.key_latent_stride_row = lk.data_ptr(), nb * rank_k, rank_k
        a.value_latent, a.value_latent_stride_batch, a.value_latent_stride_row = lv.data_ptr(), nb * rank_v, rank_v
        a.latent_rows = nb
        if latents:
            out['key_latents'], out['value_latents'] = lk[:, None], lv[:, None]
        keep += [lk, lv]
    if beacon is not None:
        pages, tables = beacon
        if not isinstance(pages, BeaconPages):
            raise TypeError('beacon must be (BeaconPages, block_tables)')
        tbl = torch.as_tensor(tables).to(device=dev, dtype=torch.int32)
        tbl = tbl.reshape(-1, tbl.shape[-1]).contiguous()
        keep.append(tbl)
        bp = pages._args(tbl)
        a.beacon_pages = ctypes.pointer(bp)
    if raw_cache is not None:
        rk, rv = raw_cache
        if rk.shape != rv.shape or rk.stride() != rv.stride() or rk.shape[2] * rk.shape[3] != kvd or \
                rk.stride(2) != head_dim or rk.stride(3) != 1:
            raise ValueError('Raw cache dimensions differ from the engine allocation.')
        a.raw_key_cache, a.raw_value_cache = rk.data_ptr(), rv.data_ptr()
        a.raw_cache_stride_batch, a.raw_cache_stride_row, a.raw_cache_rows = rk.stride(0), rk.stride(1), rk.shape[1]
    if raw is not None:
        rpages, tables = raw
        if not isinstance(rpages, RawPages):
            raise TypeError('raw must be (RawPages, block_tables)')
        tbl = torch.as_tensor(tables).to(device=dev, dtype=torch.int32)
        tbl = tbl.reshape(-1, tbl.shape[-1]).contiguous()
        keep.append(tbl)
        rp = rpages._args(tbl)
        a.raw_pages = ctypes.pointer(rp)
    a.raw_first = raw_first
    a.write_sink = int(bool(write_sink))
    lib = _lib.load()
    need = lib.slimkv_window_project_workspace_size(ctypes.byref(a)) if split else 0
    if need:
        ws = _workspace(dev, need)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(_lib.load().slimkv_window_project(ctypes.byref(a), torch.cuda.current_stream(dev).cuda_stream))
    return out


def qkv_proj_with_beacon(attn, hidden_states, beacon_size, beacon_indices, return_latents=False, metadata=None):
    """Mirror of ``LlamaAttention.qkv_proj_with_beacon`` (modeling_llama.py:
    1291-1345) under prefill metadata.  Returns ``(query, key, value)`` as
    ``[B, n, .]`` and, with ``return_latents``, the Beacon rows' latents
    ``[B, n_beacon, R]`` (the rows ``_incremental_cache`` keeps).  Without
    ``metadata`` the chunk rows are the last ``n`` entries of
    ``beacon_indices``."""
    n = hidden_states.shape[1]
    if metadata is None:
        metadata = metadata_from_roles(beacon_indices.to(hidden_states.device), n)
    w = BeaconProjectionWeights.from_attention(attn)
    r = project_window(w, hidden_states, metadata, attn.num_heads, attn.num_key_value_heads, attn.head_dim,
                       latents=return_latents)
    base = (r['query'], r['key'], r['value'])
    if return_latents:
        return base + (r['key_latents'][:, 0], r['value_latents'][:, 0])
    return base


def fused_prefill_rope(q, k, rope, metadata, sink):
    """Drop-in for ``prefill_ops.fused_prefill_rope`` (prefill_ops.py:48-74).

    Returns ``(oq, ok)`` (``torch.empty_like`` layouts) or ``None`` for inputs
    the reference's fused kernel does not take (the caller then runs its own
    rotary).  ``rope`` is any object with ``cos_cached`` / ``sin_cached``
    tables ``[positions, D]``."""
    if (not q.is_cuda or not k.is_cuda or q.dtype != torch.bfloat16 or k.dtype != q.dtype
            or q.shape[-1] != k.shape[-1] or q.shape[-1] % 2
            or q.numel() >= 2 ** 31 or k.numel() >= 2 ** 31
            or metadata.positions is None or metadata.positions.shape != (q.shape[0], k.shape[2])
            or k.shape[2] > rope.cos_cached.shape[0]
            or metadata.roles.numel() > k.shape[2]
            or q.stride(-1) != 1 or k.stride(-1) != 1):
        return None
    dev = q.device
    cos = rope.cos_cached.to(device=dev, dtype=torch.float32).contiguous()
    sin = rope.sin_cached.to(device=dev, dtype=torch.float32).contiguous()
    pos = metadata.positions.to(device=dev, dtype=torch.int64)
    if pos.stride(-1) != 1:
        pos = pos.contiguous()
    roles = metadata.roles.to(device=dev, dtype=torch.int64).contiguous()
    oq, ok = torch.empty_like(q), torch.empty_like(k)
    B, H, Q, D = q.shape
    Hk, K = k.shape[1], k.shape[2]

    def st(t):
        return (ctypes.c_int64 * 3)(*t.stride()[:3])

    _lib.check(_lib.load().slimkv_prefill_rope(q.data_ptr(), st(q), k.data_ptr(), st(k), cos.data_ptr(),
                                               sin.data_ptr(), cos.shape[0], pos.data_ptr(), pos.stride(0),
                                               roles.data_ptr(), roles.numel(), int(sink), B, H, Hk, Q, K, D,
                                               oq.data_ptr(), st(oq), ok.data_ptr(), st(ok),
                                               torch.cuda.current_stream(dev).cuda_stream))
    return oq, ok
