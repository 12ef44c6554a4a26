"""Torch-tensor entry points over the C ABI (``include/slimkv_b200.h``).

Each wrapper checks devices, dtypes and shapes, sizes and allocates the
workspace from PyTorch's caching allocator (so calls can be captured in CUDA
graphs), and launches on the current CUDA stream.  There is no CPU path:
CPU tensors or a missing library raise.
"""
import ctypes
import math

import torch

from . import _lib


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _require(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _bf16_cuda(*tensors):
    for t in tensors:
        _require(t.is_cuda, 'CUDA tensors required')
        _require(t.dtype == torch.bfloat16, 'BF16 only')


def attention_forward(q, k, v, scale, causal=False, num_splits=0, cache_seqlens=None,
                      lse_masked_positive=True, out=None, lse=None):
    """Split-KV grouped decode attention over BSHD tensors.

    ``q [B, Q, H, D]``, ``k [B, N, Hkv, D]``, ``v [B, N, Hkv, Dv]`` bf16 with a
    contiguous last dimension; returns ``(out [B, Q, H, Dv] bf16, lse [B, H,
    Q] fp32)``.  Rows that see no key get zero output and ``lse = +inf`` when
    ``lse_masked_positive`` (the reference extension's convention) or
    ``-inf`` otherwise.
    """
    _bf16_cuda(q, k, v)
    _require(q.dim() == 4 and k.dim() == 4 and v.dim() == 4, 'BSHD tensors required')
    _require(q.stride(3) == 1 and k.stride(3) == 1 and v.stride(3) == 1, 'Last dimension must be contiguous')
    _require(q.device == k.device == v.device, 'Same device required')
    batch, queries, heads, dim = q.shape
    _require(k.shape[0] == batch and v.shape[:3] == k.shape[:3] and k.shape[3] == dim, 'Invalid K/V shape')
    if out is None:
        out = q.new_empty(batch, queries, heads, v.shape[3])
    _require(out.dtype in (torch.bfloat16, torch.float32) and out.is_cuda, 'out must be bf16 or fp32 on CUDA')
    if lse is None:
        lse = torch.empty(batch, heads, queries, device=q.device, dtype=torch.float32)
    if cache_seqlens is not None:
        _require(cache_seqlens.is_cuda and cache_seqlens.dtype == torch.int32 and cache_seqlens.is_contiguous()
                 and cache_seqlens.numel() == batch, 'One CUDA int32 cache length per sequence required')
    a = _lib.AttentionArgs()
    a.q, a.q_stride = q.data_ptr(), _lib.I64x3(*q.stride()[:3])
    a.k, a.k_stride = k.data_ptr(), _lib.I64x3(*k.stride()[:3])
    a.v, a.v_stride = v.data_ptr(), _lib.I64x3(*v.stride()[:3])
    a.out, a.out_stride = out.data_ptr(), _lib.I64x3(*out.stride()[:3])
    a.lse = lse.data_ptr()
    a.cache_seqlens = 0 if cache_seqlens is None else cache_seqlens.data_ptr()
    a.batch, a.queries, a.heads, a.kv_heads = batch, queries, heads, k.shape[2]
    a.keys, a.head_dim, a.value_dim = k.shape[1], dim, v.shape[3]
    a.scale, a.causal, a.num_splits = float(scale), int(bool(causal)), int(num_splits)
    a.lse_masked_positive = int(bool(lse_masked_positive))
    a.out_fp32 = int(out.dtype == torch.float32)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        size = lib.slimkv_attention_workspace_size(ctypes.byref(a))
        if size == 0:   # planning rejected the arguments; surface its error
            _lib.check(lib.slimkv_attention_forward(ctypes.byref(a), None, 0, _stream()))
        ws = torch.empty(size, dtype=torch.uint8, device=q.device)
        _lib.check(lib.slimkv_attention_forward(ctypes.byref(a), _ptr(ws), size, _stream()))
    return out, lse


def attention_forward_noalloc(q, k, v, scale, out, lse, causal=False, num_splits=0, cache_seqlens=None,
                              lse_masked_positive=True):
    """``attention_forward`` through the allocation-free entry point.

    For callers that cannot allocate device memory: the caller provides
    ``out`` and ``lse``, and the split scratch comes from the library's fixed
    16 MiB static buffer.  Calls on one device share that buffer, so they
    must not overlap on the GPU (keep them on one stream).
    """
    _bf16_cuda(q, k, v)
    _require(q.dim() == 4 and k.dim() == 4 and v.dim() == 4, 'BSHD tensors required')
    _require(q.stride(3) == 1 and k.stride(3) == 1 and v.stride(3) == 1, 'Last dimension must be contiguous')
    batch, queries, heads, dim = q.shape
    _require(out.dtype in (torch.bfloat16, torch.float32) and out.is_cuda, 'out must be bf16 or fp32 on CUDA')
    a = _lib.AttentionArgs()
    a.q, a.q_stride = q.data_ptr(), _lib.I64x3(*q.stride()[:3])
    a.k, a.k_stride = k.data_ptr(), _lib.I64x3(*k.stride()[:3])
    a.v, a.v_stride = v.data_ptr(), _lib.I64x3(*v.stride()[:3])
    a.out, a.out_stride = out.data_ptr(), _lib.I64x3(*out.stride()[:3])
    a.lse = lse.data_ptr()
    a.cache_seqlens = 0 if cache_seqlens is None else cache_seqlens.data_ptr()
    a.batch, a.queries, a.heads, a.kv_heads = batch, queries, heads, k.shape[2]
    a.keys, a.head_dim, a.value_dim = k.shape[1], dim, v.shape[3]
    a.scale, a.causal, a.num_splits = float(scale), int(bool(causal)), int(num_splits)
    a.lse_masked_positive = int(bool(lse_masked_positive))
    a.out_fp32 = int(out.dtype == torch.float32)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().slimkv_attention_forward_noalloc(ctypes.byref(a), _stream()))
    return out, lse


def rope_decode(q, k, cos, sin, query_positions, raw_indices, sink, history):
    """BF16-exact decode RoPE (``decode_ops.fused_rope`` contract).

    ``q [B, H, Q, D]`` is rotated at ``query_positions [B, Q]`` (int64); key
    ``s`` of ``k [B, Hkv, K, D]`` sits at ``s`` when ``s < sink``, at the
    first query position when it is the last key, and otherwise at
    ``raw_indices[s - sink] + sink + history``.  Returns contiguous copies.
    """
    _bf16_cuda(q, k)
    _require(cos.dtype == torch.float32 and sin.dtype == torch.float32 and cos.is_cuda, 'fp32 CUDA tables')
    _require(q.stride(3) == 1 and k.stride(3) == 1, 'Last dimension must be contiguous')
    _require(q.dim() == 4 and k.dim() == 4 and q.shape[0] == k.shape[0] and q.shape[3] == k.shape[3],
             'q [B, H, Q, D] and k [B, Hkv, K, D] must share B and D')
    _require(query_positions.shape == (q.shape[0], q.shape[2]), 'query positions must be [B, Q]')
    if k.shape[2] - 1 > sink:
        _require(raw_indices is not None and raw_indices.numel() >= k.shape[2] - 1 - sink,
                 'raw indices must cover the keys between the sinks and the current token')
    qpos = query_positions.to(torch.int64)
    _require(qpos.stride(1) == 1, 'query positions must be row-contiguous')
    raw = None if raw_indices is None else raw_indices.to(torch.int64).contiguous()
    oq, ok = torch.empty(q.shape, dtype=q.dtype, device=q.device), torch.empty(k.shape, dtype=k.dtype, device=k.device)
    st = (ctypes.c_int64 * 3)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(lib.slimkv_rope_decode(
            _ptr(q), st(*q.stride()[:3]), _ptr(k), st(*k.stride()[:3]), _ptr(cos), _ptr(sin), cos.shape[0],
            _ptr(qpos), qpos.stride(0), _ptr(raw), int(sink), int(history), q.shape[0], q.shape[1], k.shape[1],
            q.shape[2], k.shape[2], q.shape[3], _ptr(oq), _ptr(ok), _stream()))
    return oq, ok


def rope_rows(x, positions, cos, sin, counts=None, out=None):
    """BF16-exact RoPE of ``x [B, T, H, D]`` rows at ``positions [B, T]``
    (int32, per sequence), for ``t < counts[b]`` (``slimkv_rope_rows``);
    returns ``out`` (a new ``[B, T, H, D]`` tensor when not given)."""
    _bf16_cuda(x)
    _require(x.dim() == 4 and x.stride(3) == 1, 'x must be [B, T, H, D] with a contiguous last dimension')
    _require(positions.is_cuda and positions.dtype == torch.int32 and positions.stride(1) == 1 and
             positions.shape[0] == x.shape[0] and positions.shape[1] >= x.shape[1], 'int32 positions [B, >= T]')
    _require(cos.dtype == torch.float32 and cos.is_contiguous() and sin.is_contiguous(), 'fp32 tables')
    if counts is not None:
        _require(counts.is_cuda and counts.dtype == torch.int32 and counts.numel() == x.shape[0], 'int32 counts [B]')
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _require(out.shape == x.shape and out.stride(3) == 1 and out.data_ptr() != x.data_ptr(), 'distinct out')
    st = ctypes.c_int64 * 3
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().slimkv_rope_rows(
            _ptr(x), st(*x.stride()[:3]), _ptr(out), st(*out.stride()[:3]), _ptr(positions), positions.stride(0),
            _ptr(counts), x.shape[0], x.shape[1], x.shape[2], x.shape[3], _ptr(cos), _ptr(sin), cos.shape[0],
            _stream()))
    return out


def rms_norm(x, weight, eps, out=None):
    """``LlamaRMSNorm`` of the rows of ``x [..., hidden]`` (bf16, rows with a
    contiguous last dimension): ``weight * bf16(x * rsqrt(mean(x^2) + eps))``
    (``slimkv_rms_norm``; slimkv/llama3/modeling_llama.py:79-95)."""
    _bf16_cuda(x, weight)
    H = x.shape[-1]
    rows = x.view(-1, H)
    _require(rows.stride(1) == 1 and weight.is_contiguous() and weight.numel() == H, 'rows [N, hidden], weight [hidden]')
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    orows = out.view(-1, H)
    _require(orows.shape == rows.shape and orows.stride(1) == 1, 'out like x')
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().slimkv_rms_norm(_ptr(rows), rows.stride(0), _ptr(weight), _ptr(orows), orows.stride(0),
                                              rows.shape[0], H, float(eps), _stream()))
    return out


def silu_mul(gate_up, out=None):
    """``silu(gate) * up`` of rows ``gate_up [N, 2I]`` = ``[gate | up]`` (bf16),
    each product rounded as the bf16 modules round it (``slimkv_silu_mul``;
    ``LlamaMLP.forward``, modeling_llama.py:97-113).  Returns ``[N, I]``."""
    _bf16_cuda(gate_up)
    _require(gate_up.dim() == 2 and gate_up.stride(1) == 1 and gate_up.shape[1] % 2 == 0, 'gate_up [N, 2I]')
    n, inter = gate_up.shape[0], gate_up.shape[1] // 2
    if out is None:
        out = torch.empty((n, inter), dtype=gate_up.dtype, device=gate_up.device)
    _require(out.shape == (n, inter) and out.stride(1) == 1, 'out [N, I]')
    with torch.cuda.device(gate_up.device):
        _lib.check(_lib.load().slimkv_silu_mul(_ptr(gate_up), gate_up.stride(0), _ptr(out), out.stride(0), n, inter,
                                              _stream()))
    return out


def merge(raw, raw_lse, latent, latent_lse):
    """LSE merge of BHQD bf16 outputs (``decode_ops.fused_merge`` contract)."""
    _bf16_cuda(raw, latent)
    _require(raw.stride(3) == 1 and latent.stride(3) == 1, 'Last dimension must be contiguous')
    _require(raw_lse.dtype == torch.float32 and latent_lse.dtype == torch.float32, 'fp32 LSE required')
    out = torch.empty(raw.shape, dtype=raw.dtype, device=raw.device)
    st = (ctypes.c_int64 * 3)
    lib = _lib.load()
    with torch.cuda.device(raw.device):
        _lib.check(lib.slimkv_merge(_ptr(raw), st(*raw.stride()[:3]), _ptr(raw_lse), st(*raw_lse.stride()[:3]),
                                    _ptr(latent), st(*latent.stride()[:3]), _ptr(latent_lse),
                                    st(*latent_lse.stride()[:3]), raw.shape[0], raw.shape[1], raw.shape[2],
                                    raw.shape[3], _ptr(out), _stream()))
    return out


class LatentDecodeCall:
    """Prepared arguments of ``slimkv_latent_decode`` for fixed buffers.

    Built once per (layer, batch shape) by the decode runtime; ``__call__``
    re-launches with the same pointers, which is what a CUDA graph captures.
    """

    def __init__(self, *, q, raw_k_rot, raw_v, lat_k=None, lat_v=None, raw_len, latent_len, qpos, uk, uv, cos, sin,
                 out, query_len=None, raw_k_pre=None, new_k=None, new_v=None, new_lat_k=None, new_lat_v=None,
                 uk_bias=None, uv_bias=None, scale=None, latent_len_max=0, raw_len_max=0, latent_splits=0,
                 raw_splits=0, lat_pages=None, out_lse=None, latent_shard=False, wait_limit_ns=0, plan=None):
        """``lat_pages = (pages, layout, tables)`` replaces ``lat_k / lat_v``
        with the vLLM plugin's Beacon pages: ``pages [num_pages, >=
        layout.page_elements]`` bf16 (a ``pages.BeaconPageLayout`` layout) and
        ``tables [B, pages_per_seq]`` int32 block tables on the device.

        Sequence split: ``out_lse`` (fp32 ``[B, L, H]``, contiguous) receives
        each output row's log-sum-exp over this call's keys, so that shards of
        one sequence can be merged (:func:`merge_partials`);
        ``latent_shard=True`` marks a latent cache that does not hold this
        step's Beacon row (no causal latent mask, no ``new_lat_*``).

        ``wait_limit_ns`` bounds every pipeline wait of the attention kernel
        (0: 2 s); a wait that runs out sets ``SLIMKV_DEVICE_TIMEOUT`` in the
        device status word and the kernel returns early.

        ``plan``: an int32 device tensor that :meth:`compute_plan` (of this or
        another call with the same lengths) fills before this call runs; the
        call then skips planning and starts its attention early."""
        paged = lat_pages is not None
        _require(paged or (lat_k is not None and lat_v is not None), 'lat_k / lat_v or lat_pages required')
        _bf16_cuda(q, raw_k_rot, raw_v, uk, uv, *(() if paged else (lat_k, lat_v)))
        _require(out.is_cuda and out.dtype in (torch.bfloat16, torch.float32), 'out must be bf16 or fp32 on CUDA')
        batch, length, heads, dim = q.shape
        kv_heads = raw_k_rot.shape[2]
        _require(raw_k_rot.shape[0] == batch and raw_k_rot.shape[3] == dim, 'raw cache shape')
        _require(raw_k_rot.stride() == raw_v.stride() and raw_k_rot.stride(3) == 1 and
                 (raw_k_pre is None or raw_k_pre.stride() == raw_k_rot.stride()),
                 'raw caches [B, cap, Hkv, D] (token-major, or a head-major view) need matching strides')
        if not paged:
            _require(lat_k.stride() == lat_v.stride() and lat_k.stride(2) == 1 and lat_v.stride(2) == 1,
                     'latent caches [B, cap, R] need matching strides and contiguous rows')
        for t in (raw_len, latent_len, qpos) + (() if query_len is None else (query_len,)):
            _require(t.is_cuda and t.dtype == torch.int32 and t.is_contiguous(), 'int32 CUDA metadata')
        a = _lib.LatentDecodeArgs()
        a.batch, a.length, a.heads, a.kv_heads, a.head_dim = batch, length, heads, kv_heads, dim
        if paged:
            pages, layout, tables = lat_pages
            _bf16_cuda(pages)
            flat = pages.flatten(1)
            _require(flat.data_ptr() == pages.data_ptr() and flat.stride(1) == 1 and
                     flat.shape[1] >= layout.page_elements, 'pages must be [num_pages, >= page_elements] rows')
            _require(tables.is_cuda and tables.dtype == torch.int32 and tables.dim() == 2 and
                     tables.shape[0] == batch and tables.stride(1) == 1, 'block tables must be int32 [B, n] on CUDA')
            a.rank_k, a.rank_v = layout.key_rank, layout.value_rank
        else:
            a.rank_k, a.rank_v = lat_k.shape[2], lat_v.shape[2]
        _require(uk.shape == (kv_heads * dim, a.rank_k) and uv.shape == (kv_heads * dim, a.rank_v),
                 'up-projection weights must be [Hkv*D, R]')
        a.scale = float(scale if scale is not None else 1.0 / math.sqrt(dim))
        a.q, a.q_stride = q.data_ptr(), _lib.I64x3(*q.stride()[:3])
        a.raw_k_rot, a.raw_v = raw_k_rot.data_ptr(), raw_v.data_ptr()
        a.raw_k_pre = 0 if raw_k_pre is None else raw_k_pre.data_ptr()
        a.raw_stride_batch, a.raw_stride_token = raw_k_rot.stride(0), raw_k_rot.stride(1)
        a.raw_stride_head = raw_k_rot.stride(2)
        a.raw_capacity = raw_k_rot.shape[1]
        if paged:
            a.lat_k = a.lat_v = 0
            a.lat_pages, a.lat_page_stride = flat.data_ptr(), flat.stride(0)
            a.lat_slots, a.lat_sink_elements = layout.slots, layout.sink_elements
            a.lat_table, a.lat_table_stride = tables.data_ptr(), tables.stride(0)
            a.lat_num_pages = flat.shape[0]
            a.lat_capacity = tables.shape[1] * layout.slots
        else:
            a.lat_k, a.lat_v = lat_k.data_ptr(), lat_v.data_ptr()
            a.lat_stride_batch, a.lat_stride_row = lat_k.stride(0), lat_k.stride(1)
            a.lat_capacity = lat_k.shape[1]
        a.raw_len, a.latent_len, a.qpos = raw_len.data_ptr(), latent_len.data_ptr(), qpos.data_ptr()
        a.query_len = 0 if query_len is None else query_len.data_ptr()
        for name, t in (('new_k', new_k), ('new_v', new_v), ('new_lat_k', new_lat_k), ('new_lat_v', new_lat_v),
                        ('uk_bias', uk_bias), ('uv_bias', uv_bias)):
            if t is not None:
                _bf16_cuda(t)
                _require(t.stride(-1) == 1, f'{name} must have a contiguous last dimension')
                _require(t.dim() == 1 or t.shape[0] == batch, f'{name} must have one row per sequence')
            setattr(a, name, 0 if t is None else t.data_ptr())
        if new_k is not None:
            _require(new_k.shape[-1] == kv_heads * dim and new_k.stride() == new_v.stride(), 'new K/V rows')
            a.new_stride = new_k.stride(0)
        if new_lat_k is not None:
            _require(new_lat_k.shape[-1] == a.rank_k and new_lat_v.shape[-1] == a.rank_v
                     and new_lat_k.stride(0) == new_lat_v.stride(0), 'new latent rows')
            a.new_lat_stride = new_lat_k.stride(0)
        a.uk, a.uv = uk.data_ptr(), uv.data_ptr()
        _require(cos.dtype == torch.float32 and cos.is_contiguous() and sin.is_contiguous(), 'fp32 tables')
        a.cos, a.sin, a.rope_positions = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
        _require(out.shape == (batch, length, heads * dim) and out.stride(2) == 1, 'out must be [B, L, H*D]')
        a.out, a.out_stride = out.data_ptr(), _lib.I64x2(out.stride(0), out.stride(1))
        a.out_fp32 = int(out.dtype == torch.float32)
        a.latent_len_max, a.raw_len_max = int(latent_len_max), int(raw_len_max)
        a.latent_splits, a.raw_splits = int(latent_splits), int(raw_splits)
        if out_lse is not None:
            _require(out_lse.is_cuda and out_lse.dtype == torch.float32 and out_lse.is_contiguous() and
                     out_lse.shape == (batch, length, heads), 'out_lse must be contiguous fp32 [B, L, H]')
        a.out_lse = 0 if out_lse is None else out_lse.data_ptr()
        a.latent_shard = int(bool(latent_shard))
        a.wait_limit_ns = int(wait_limit_ns)
        if plan is not None:
            _require(plan.is_cuda and plan.dtype == torch.int32 and plan.is_contiguous(), 'plan: int32 CUDA tensor')
            a.plan = plan.data_ptr()
        self.args = a
        self.device = q.device
        self._keep = (q, raw_k_rot, raw_v, raw_k_pre, lat_k, lat_v, lat_pages, raw_len, latent_len, query_len, qpos,
                      new_k, new_v, new_lat_k, new_lat_v, uk, uv, uk_bias, uv_bias, cos, sin, out_lse, plan, out)
        lib = _lib.load()
        size = lib.slimkv_latent_decode_workspace_size(ctypes.byref(a))
        if size == 0:
            _lib.check(lib.slimkv_latent_decode(ctypes.byref(a), None, 0, None))
        self.workspace = torch.empty(size, dtype=torch.uint8, device=q.device)

    def plan_words(self):
        """int32 words of this call's step plan (``slimkv_decode_plan_words``)."""
        return int(_lib.load().slimkv_decode_plan_words(ctypes.byref(self.args)))

    def use_plan(self, plan):
        """Run with the step plan in ``plan`` (filled by :meth:`compute_plan`
        before each launch) instead of planning per call."""
        _require(plan.is_cuda and plan.dtype == torch.int32 and plan.numel() >= self.plan_words(), 'plan buffer')
        self.args.plan = plan.data_ptr()
        self._plan = plan

    def compute_plan(self, plan):
        """Fill ``plan`` (int32, >= :meth:`plan_words` words) with the step's
        work plan from this call's current device lengths
        (``slimkv_decode_plan``), on the current stream."""
        _require(plan.is_cuda and plan.dtype == torch.int32 and plan.numel() >= self.plan_words(), 'plan buffer')
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().slimkv_decode_plan(ctypes.byref(self.args), _ptr(plan), _stream()))
        return plan

    def __call__(self, attn_events=None):
        """Launch; ``attn_events`` = (begin, end) ``torch.cuda.Event`` pair
        (already recorded once, so that torch has created them) re-recorded
        around the attention kernel alone (not inside graph capture)."""
        lib = _lib.load()
        a = self.args
        if attn_events is not None:
            _require(all(e.cuda_event for e in attn_events), 'record the timing events once before passing them')
        a.attn_event_begin, a.attn_event_end = ((attn_events[0].cuda_event, attn_events[1].cuda_event)
                                                if attn_events is not None else (0, 0))
        try:
            with torch.cuda.device(self.device):
                _lib.check(lib.slimkv_latent_decode(ctypes.byref(a), _ptr(self.workspace),
                                                    self.workspace.numel(), _stream()))
        finally:
            a.attn_event_begin, a.attn_event_end = 0, 0
        return self._keep[-1]


def latent_decode(**kwargs):
    """One fused decode-attention step (see :class:`LatentDecodeCall`)."""
    return LatentDecodeCall(**kwargs)()


def merge_partials(part_out, part_lse, out, out_lse=None):
    """N-part LSE merge (``slimkv_merge_partials``): ``part_out [N, rows,
    dim]`` fp32 and ``part_lse [N, rows]`` fp32 (any part strides; rows and
    dim contiguous) into ``out [rows, dim]`` (bf16 or fp32, contiguous) and
    optionally ``out_lse [rows]``."""
    _require(part_out.is_cuda and part_out.dtype == torch.float32 and part_lse.dtype == torch.float32,
             'fp32 CUDA partials')
    parts, rows, dim = part_out.shape
    _require(part_out.stride(2) == 1 and part_out.stride(1) == dim and part_lse.shape == (parts, rows) and
             part_lse.stride(1) == 1, 'partials must be [N, rows, dim] / [N, rows] with contiguous rows')
    _require(out.is_contiguous() and out.numel() == rows * dim and out.dtype in (torch.bfloat16, torch.float32),
             'out must be contiguous [rows, dim] bf16 or fp32')
    if out_lse is not None:
        _require(out_lse.is_contiguous() and out_lse.numel() == rows and out_lse.dtype == torch.float32,
                 'out_lse must be contiguous fp32 [rows]')
    a = _lib.MergePartialsArgs(parts, rows, dim, part_out.data_ptr(), part_out.stride(0), part_lse.data_ptr(),
                               part_lse.stride(0), out.data_ptr(), int(out.dtype == torch.float32),
                               0 if out_lse is None else out_lse.data_ptr())
    with torch.cuda.device(out.device):
        _lib.check(_lib.load().slimkv_merge_partials(ctypes.byref(a), _stream()))
    return out


def decode_schedule(history, tail, raw_len, latent_len, query_len, qpos, sink, window, ratio):
    """Advance the per-sequence Beacon schedule on the device (in place).

    Writes this step's ``query_len``, ``raw_len``, ``latent_len`` and ``qpos
    [B, 2]`` from the counters ``history`` / ``tail`` and advances them.
    """
    for t in (history, tail, raw_len, latent_len, query_len, qpos):
        _require(t.is_cuda and t.dtype == torch.int32 and t.is_contiguous(), 'int32 CUDA counters')
    batch = history.numel()
    _require(qpos.shape == (batch, 2), 'qpos must be [B, 2]')
    _lib.check(_lib.load().slimkv_decode_schedule(batch, int(sink), int(window), int(ratio), _ptr(history),
                                                  _ptr(tail), _ptr(raw_len), _ptr(latent_len), _ptr(query_len),
                                                  _ptr(qpos), _stream()))
