"""Whole-model decode runtime over the native latent cache (B > 1, graphs).

A batched, CUDA-graph-captured decode step of a Llama-3.1-style SlimKV model
whose attention is the fused latent decode of ``libslimkv_b200.so``:

* per-sequence Beacon schedule advanced on the device every step
  (``slimkv_decode_schedule``, the per-sequence form of
  ``LlamaMemory._step``, slimkv/llama3/memory.py:101-162), so a replay
  needs no host work and sequences may sit at different window offsets;
* projections and the MLP are cuBLAS GEMMs issued by torch; the raw row uses
  ``q/k/v_proj`` and the Beacon row ``beacon_q_proj`` plus the K/V
  down-projections (slimkv/llama3/fa2_decode.py:89-99);
* every step carries two rows per sequence — the raw token and a Beacon slot
  that only sequences inserting a Beacon this step use (``query_len``), so
  the graph shape never changes.

Weights are random N(0, std) (no checkpoint is available offline); the cache
is filled with synthetic latents/keys of the magnitude that projections of
unit-variance hidden states produce.  This is the reference's static decode
(slimkv/llama3/static_decode.py:43-287) generalised to B > 1 and ragged
lengths.
"""
from dataclasses import dataclass, field

import torch

from . import kernels
from .rope import LLAMA3_SCALING, rope_tables


@dataclass
class LatentLlamaConfig:
    """Llama-3.1-8B geometry with SlimKV r4 ranks and t4 Beacons."""
    vocab: int = 128256
    hidden: int = 4096
    intermediate: int = 14336
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    rank_k: int = 320
    rank_v: int = 320
    window: int = 1024
    ratio: int = 4
    sink: int = 4
    rope_theta: float = 500000.0
    rope_scaling: dict = field(default_factory=lambda: dict(LLAMA3_SCALING))
    rope_positions: int = 131072
    rms_eps: float = 1e-5
    qkv_bias: bool = False        # q/k/v (and Beacon q / up-projection) biases, as in Qwen2


def qwen25_14b_r2():
    """Qwen2.5-14B geometry (48 layers, hidden 5120, 40 / 8 heads, q/k/v bias,
    RoPE theta 1e6 without scaling) with SlimKV r2 ranks (512 / 512) and t4
    Beacons."""
    return LatentLlamaConfig(vocab=152064, hidden=5120, intermediate=13824, layers=48, heads=40, kv_heads=8,
                             head_dim=128, rank_k=512, rank_v=512, ratio=4, rope_theta=1e6, rope_scaling=None,
                             rope_positions=262144, rms_eps=1e-6, qkv_bias=True)


class RandomWeights:
    """bf16 weights drawn from N(0, std) on the device (norm weights = 1)."""

    def __init__(self, cfg, device, seed=0, std=0.02):
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        H, I, kvd = cfg.hidden, cfg.intermediate, cfg.kv_heads * cfg.head_dim
        qd = cfg.heads * cfg.head_dim

        def w(*shape, scale=std):
            return torch.randn(*shape, generator=gen, device=device, dtype=torch.bfloat16).mul_(scale)

        self.embed = w(cfg.vocab, H)
        self.beacon_embed = w(1, H)
        self.final_norm = torch.ones(H, device=device, dtype=torch.bfloat16)
        self.lm_head = w(cfg.vocab, H)
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append(dict(
                norm1=torch.ones(H, device=device, dtype=torch.bfloat16),
                norm2=torch.ones(H, device=device, dtype=torch.bfloat16),
                w_raw=w(qd + 2 * kvd, H),                        # q_proj | k_proj | v_proj
                w_beacon=w(qd + cfg.rank_k + cfg.rank_v, H),     # beacon_q_proj | k_down | v_down
                w_o=w(H, qd),
                uk=w(kvd, cfg.rank_k),                           # beacon_k_up_proj.weight
                uv=w(kvd, cfg.rank_v),                           # beacon_v_up_proj.weight
                w_gate_up=w(2 * I, H),
                w_down=w(H, I)))
            if cfg.qkv_bias:
                # Biases of q/k/v_proj and beacon_q_proj (the K/V down-projections
                # have none) and of the up-projections (present with k/v bias).
                zeros = torch.zeros(cfg.rank_k + cfg.rank_v, device=device, dtype=torch.bfloat16)
                self.layers[-1].update(b_raw=w(qd + 2 * kvd, scale=0.1),
                                       b_beacon=torch.cat([w(qd, scale=0.1), zeros]),
                                       uk_bias=w(kvd, scale=0.1), uv_bias=w(kvd, scale=0.1))

    def nbytes(self):
        total = sum(t.numel() * 2 for t in (self.embed, self.beacon_embed, self.lm_head))
        return total + sum(t.numel() * 2 for layer in self.layers for t in layer.values())


class StateDictWeights:
    """Runtime weights from a SlimKV Llama state dict.

    Parameter names are the reference model's (``LlamaForCausalLM`` with
    Beacon projections, slimkv/llama3/modeling_llama.py:181-277 and 351-382):
    per layer ``self_attn.{q,k,v,o}_proj``, ``self_attn.beacon_q_proj``, the
    K/V down-projections (``beacon_{k,v}_down_proj`` or a shared
    ``beacon_kv_down_proj``), the up-projections ``beacon_{k,v}_up_proj``,
    ``mlp.{gate,up,down}_proj`` and the two RMSNorms, plus the raw and Beacon
    embeddings, the final norm and ``lm_head``.  The runtime's fused layout is
    built from them: ``[q | k | v]`` for the raw row, ``[beacon_q | k_down |
    v_down]`` for the Beacon row and ``[gate | up]``; biases are taken when the
    state dict has them (``cfg.qkv_bias``).  Values may be numpy arrays or
    tensors; they are stored as bf16 on ``device``."""

    def __init__(self, cfg, state_dict, device):
        def t(name):
            return torch.as_tensor(state_dict[name]).to(device=device, dtype=torch.bfloat16).contiguous()

        def opt(name):
            return t(name) if name in state_dict else None

        self.embed = t('model.embed_tokens.weight')
        self.beacon_embed = t('model.beacon_embed_tokens.weight')
        self.final_norm = t('model.norm.weight')
        self.lm_head = t('lm_head.weight')
        self.layers = []
        for i in range(cfg.layers):
            p = f'model.layers.{i}.'
            a = p + 'self_attn.'
            shared = a + 'beacon_kv_down_proj.weight' in state_dict
            kd = t(a + ('beacon_kv_down_proj.weight' if shared else 'beacon_k_down_proj.weight'))
            vd = kd if shared else t(a + 'beacon_v_down_proj.weight')
            layer = dict(
                norm1=t(p + 'input_layernorm.weight'), norm2=t(p + 'post_attention_layernorm.weight'),
                w_raw=torch.cat([t(a + 'q_proj.weight'), t(a + 'k_proj.weight'), t(a + 'v_proj.weight')]),
                w_beacon=torch.cat([t(a + 'beacon_q_proj.weight'), kd, vd]),
                w_o=t(a + 'o_proj.weight'), uk=t(a + 'beacon_k_up_proj.weight'), uv=t(a + 'beacon_v_up_proj.weight'),
                w_gate_up=torch.cat([t(p + 'mlp.gate_proj.weight'), t(p + 'mlp.up_proj.weight')]),
                w_down=t(p + 'mlp.down_proj.weight'))
            if cfg.qkv_bias:
                zeros = torch.zeros(cfg.rank_k + cfg.rank_v, device=device, dtype=torch.bfloat16)
                layer.update(b_raw=torch.cat([t(a + 'q_proj.bias'), t(a + 'k_proj.bias'), t(a + 'v_proj.bias')]),
                             b_beacon=torch.cat([t(a + 'beacon_q_proj.bias'), zeros]),
                             uk_bias=opt(a + 'beacon_k_up_proj.bias'), uv_bias=opt(a + 'beacon_v_up_proj.bias'))
            self.layers.append(layer)

    def nbytes(self):
        total = sum(t.numel() * 2 for t in (self.embed, self.beacon_embed, self.lm_head))
        return total + sum(t.numel() * 2 for layer in self.layers for t in layer.values() if t is not None)


class LatentDecodeRuntime:
    """Batched decode over per-sequence compressed caches.

    ``history[b]`` completed-window latents and ``tails[b]`` raw tokens of the
    open window per sequence (0 <= tail < window).  Caches are allocated for
    ``extra_windows`` more windows of growth.
    """

    def __init__(self, cfg, weights, history, tails, device, extra_windows=1, seed=1, fill_std=1.3, paged=False,
                 raw_pre=True, latent_splits=0, raw_splits=0, seq_split=None, backend='latent'):
        """``paged`` keeps each layer's latent cache in the vLLM plugin's Beacon
        pages (page size of a 16-token raw page, ``create_page_layers``,
        slimkv/vllm_plugin/backend.py:108-131), each sequence owning the pages
        its own length needs, in shuffled order; ``raw_pre=False`` drops the
        pre-RoPE copy of the raw keys (only the append writes it);
        ``latent_splits`` / ``raw_splits`` override the attention split plan
        (0: the library's choice).

        ``seq_split`` (a ``torch.distributed`` process group, or ``True`` for
        the default group) splits every sequence's completed-window latents
        over the group's ranks in contiguous 64-row shards
        (``parallel.shard_range``): rank ``r`` holds rows ``[start_r,
        end_r)``; the last rank also holds the open window, the Beacons this
        decode appends and the raw cache.  Each layer's fused decode then
        attends over the rank's shard (``latent_shard`` on all but the last
        rank) and writes fp32 partials that one NCCL all-gather and
        ``slimkv_merge_partials`` combine (``parallel.SequenceSplitMerge``).
        Everything else runs replicated, so every rank keeps identical
        hidden states.

        ``backend='reconstruct'`` runs the reference's reconstruct decode
        backend instead of the latent one (:mod:`slimkv_b200.reconstruct`):
        per layer the queries and the new raw key are rotated
        (``slimkv_rope_decode``), the new raw K/V and Beacon latents are
        appended, every Beacon key and value is rebuilt from its latent
        (``slimkv_reconstruct_kv``) into a full-dimension buffer shared by the
        layers, and split-KV attention runs over raw + rebuilt keys."""
        self.cfg, self.w, self.device = cfg, weights, device
        B = len(history)
        self.batch = B
        hist = torch.as_tensor(history, dtype=torch.int32)
        tail = torch.as_tensor(tails, dtype=torch.int32)
        if (tail < 0).any() or (tail >= cfg.window).any():
            raise ValueError('tails must lie in [0, window)')
        if cfg.sink > 1 and (hist == 0).any():
            raise ValueError('decode with more than one sink needs a completed first window')
        per_window = cfg.window // cfg.ratio
        if backend not in ('latent', 'reconstruct'):
            raise ValueError('backend must be latent or reconstruct')
        self.backend = backend
        self.split = None
        if backend == 'reconstruct' and (paged or (seq_split is not None and seq_split is not False)):
            raise ValueError('the reconstruct backend runs on the native layout without a sequence split')
        if seq_split is not None and seq_split is not False:
            import torch.distributed as dist
            from .parallel import shard_range
            group = None if seq_split is True else seq_split
            world, rank = dist.get_world_size(group), dist.get_rank(group)
            if paged:
                raise ValueError('the sequence split uses the native latent layout')
            bounds = [shard_range(int(h), world, rank, tile=64) for h in hist.tolist()]
            self.split = dict(group=group, world=world, rank=rank, last=rank == world - 1,
                              offset=torch.tensor([a for a, _ in bounds], dtype=torch.int32),
                              rows=torch.tensor([b - a for a, b in bounds], dtype=torch.int32))
        self.raw_capacity = (cfg.sink + cfg.window + 1 + 63) // 64 * 64
        if self.split is not None and not self.split['last']:
            self.raw_capacity = 64                   # no raw keys on a shard rank (raw_len 0)
            self.lat_capacity = max(64, (int(self.split['rows'].max()) + 63) // 64 * 64)
        else:
            first = 0 if self.split is None else int(self.split['offset'].min())
            self.lat_capacity = (int(hist.max()) - first + (1 + extra_windows) * per_window + 63) // 64 * 64
        kvd = cfg.kv_heads * cfg.head_dim
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)

        # Cache contents: N(0, fill_std^2) bf16.  Large caches repeat one
        # random block (cheap to fill; the values only set magnitudes).
        block = torch.randn(1 << 24, generator=gen, device=device, dtype=torch.bfloat16).mul_(fill_std)

        def fill(*shape):
            t = torch.empty(*shape, device=device, dtype=torch.bfloat16)
            flat = t.view(-1)
            for i in range(0, flat.numel(), block.numel()):
                n = min(block.numel(), flat.numel() - i)
                flat[i:i + n].copy_(block[:n])
            return t

        self.layout = None
        if paged:
            from .pages import BeaconPageLayout, beacon_block_size
            width = cfg.rank_k + cfg.rank_v
            self.layout = BeaconPageLayout(beacon_block_size(cfg.ratio, kvd, width), cfg.ratio, cfg.rank_k,
                                           cfg.rank_v, kvd)
            slots = self.layout.slots
            need = [(int(h) + (1 + extra_windows) * per_window + slots - 1) // slots for h in hist.tolist()]
            order = torch.randperm(sum(need), generator=torch.Generator().manual_seed(seed))
            tables = torch.zeros(B, max(need), dtype=torch.int32)
            at = 0
            for b, n in enumerate(need):
                tables[b, :n] = order[at:at + n].int()
                at += n
            self.tables = tables.to(device)
            self.num_pages = sum(need)
            self.lat_capacity = max(need) * slots
        # HBM layout (streaming order of the attention kernel): each (sequence,
        # KV head) holds its raw keys / values as one contiguous run of tokens
        # (head-major [B, Hkv, cap, D], seen as a [B, cap, Hkv, D] view), and
        # each sequence its latent K rows and latent V rows as two contiguous
        # planes ([B, 2, cap, R]: lat_k = plane 0, lat_v = plane 1), so every
        # 128-key tile the kernel fetches is one contiguous block of HBM.
        self.caches = []
        rmax = max(cfg.rank_k, cfg.rank_v)
        for _ in range(cfg.layers):
            def raw():
                return fill(B, cfg.kv_heads, self.raw_capacity, cfg.head_dim).transpose(1, 2)
            raw_k = raw()
            c = dict(raw_k_rot=raw_k, raw_k_pre=raw() if raw_pre else None, raw_v=raw())
            if raw_pre:
                c['raw_k_pre'].copy_(raw_k)
            if paged:
                c['pages'] = fill(self.num_pages, self.layout.page_elements)
            else:
                lat = fill(B, 2, self.lat_capacity, rmax)
                c.update(lat=lat, lat_k=lat[:, 0, :, :cfg.rank_k], lat_v=lat[:, 1, :, :cfg.rank_v])
            self.caches.append(c)
        # Per-sequence schedule counters and per-step metadata (device).
        i32 = dict(dtype=torch.int32, device=device)
        self.history = hist.to(device)
        self.tail = tail.to(device)
        self.raw_len = torch.zeros(B, **i32)
        self.latent_len = torch.zeros(B, **i32)
        self.query_len = torch.zeros(B, **i32)
        self.qpos = torch.zeros(B, 2, **i32)
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.rope_theta, cfg.rope_positions, cfg.rope_scaling, device)
        # Step buffers: two rows per sequence (raw token, Beacon slot).
        bf = dict(dtype=torch.bfloat16, device=device)
        H, qd = cfg.hidden, cfg.heads * cfg.head_dim
        self.width = qd + 2 * kvd
        self.tokens = torch.zeros(B, dtype=torch.int64, device=device)
        self.x = torch.zeros(B, 2, H, **bf)
        self.z = torch.zeros(B, 2, self.width, **bf)            # projection outputs per row
        self.attn = torch.zeros(B, 2, qd, **bf)
        self.h = torch.zeros(B, 2, H, **bf)                      # normalised rows
        self.gu = torch.zeros(2 * B, 2 * cfg.intermediate, **bf)
        self.act = torch.zeros(2 * B, cfg.intermediate, **bf)
        self.h_final = torch.zeros(B, H, **bf)
        self.logits = torch.zeros(B, cfg.vocab, dtype=torch.float32, device=device)
        z = self.z
        q = z[:, :, :qd].unflatten(-1, (cfg.heads, cfg.head_dim))          # [B, 2, H, D]
        # Every call covers the whole latent capacity: a sequence may grow up to
        # it during a run (the append checks the capacity on the device).
        lat_max = self.lat_capacity
        self.calls = []
        self.merges = []
        sp = self.split
        call_raw_len, call_lat_len = self.raw_len, self.latent_len
        if sp is not None:
            from .parallel import SequenceSplitMerge
            sp['offset'], sp['rows'] = sp['offset'].to(device), sp['rows'].to(device)
            # Shard-relative latent counts: fixed on shard ranks, the running
            # count minus the shard's first row on the last rank.
            sp['latent_len'] = sp['rows'].clone() if not sp['last'] else torch.zeros(B, **i32)
            call_lat_len = sp['latent_len']
            if not sp['last']:
                call_raw_len = torch.zeros(B, **i32)
        for c, layer in zip(self.caches, weights.layers):
            pages = (c['pages'], self.layout, self.tables) if paged else None
            shard = sp is not None and not sp['last']
            out, lse = self.attn, None
            if sp is not None:
                m = SequenceSplitMerge(B, 2, cfg.heads, cfg.head_dim, group=sp['group'], device=device,
                                       merged=self.attn)
                self.merges.append(m)
                out, lse = m.out, m.lse
            self.calls.append(kernels.LatentDecodeCall(
                q=q, raw_k_rot=c['raw_k_rot'], raw_v=c['raw_v'], raw_k_pre=c['raw_k_pre'],
                lat_k=c.get('lat_k'), lat_v=c.get('lat_v'), lat_pages=pages, raw_len=call_raw_len,
                latent_len=call_lat_len,
                query_len=self.query_len, qpos=self.qpos, uk=layer['uk'], uv=layer['uv'],
                uk_bias=layer.get('uk_bias'), uv_bias=layer.get('uv_bias'),
                cos=self.cos, sin=self.sin, out=out, out_lse=lse, latent_shard=shard,
                new_k=None if shard else z[:, 0, qd:qd + kvd], new_v=None if shard else z[:, 0, qd + kvd:qd + 2 * kvd],
                new_lat_k=None if shard else z[:, 1, qd:qd + cfg.rank_k],
                new_lat_v=None if shard else z[:, 1, qd + cfg.rank_k:qd + cfg.rank_k + cfg.rank_v],
                latent_len_max=lat_max, raw_len_max=self.raw_capacity,
                latent_splits=latent_splits, raw_splits=raw_splits))
        self.call_latent_len, self.call_raw_len = call_lat_len, call_raw_len
        # One work plan per step serves every layer (same lengths): computed
        # once after the schedule, it lets each layer's attention start while
        # its prologue finishes.
        self.plan = torch.zeros(max(self.calls[0].plan_words(), 1), **i32)
        for call in self.calls:
            call.use_plan(self.plan)
        self.recon = []
        if backend == 'reconstruct':
            from .reconstruct import ReconstructDecode
            full = (B, self.raw_capacity + self.lat_capacity, cfg.kv_heads, cfg.head_dim)
            self.key_full = torch.zeros(full, **bf)
            self.value_full = torch.zeros(full, **bf)
            self.batch_index = torch.arange(B, device=device)
            for c, layer in zip(self.caches, weights.layers):
                self.recon.append(ReconstructDecode(
                    raw_k_rot=c['raw_k_rot'], raw_v=c['raw_v'], lat_k=c['lat_k'], lat_v=c['lat_v'],
                    w_k_up=layer['uk'], w_v_up=layer['uv'], b_k_up=layer.get('uk_bias'), b_v_up=layer.get('uv_bias'),
                    raw_len=self.raw_len, latent_len=self.latent_len, query_len=self.query_len,
                    key_full=self.key_full, value_full=self.value_full))
        self.graph = None
        self.graph_host = None

    # ------------------------------------------------------------------
    def load_memory(self, layers, window_raw_indices=None):
        """Fill the caches from the reference's latent Memory after a prefill.

        ``layers[i]`` holds layer i's ``LlamaMemory`` activations
        (slimkv/llama3/memory.py:219-278), batch-major with every sequence at
        the history and tail this runtime was built with: ``sink_k/sink_v
        [B, Hkv, S, D]`` and ``raw_k/raw_v [B, Hkv, T, D]`` (pre-RoPE, as the
        reference stores them), ``hist_k/hist_v [B, N, R]`` (completed
        windows) and ``win_k/win_v [B, n, R]`` (the open window's Beacons).
        ``window_raw_indices`` (``[T]``) places the raw tail in the
        interleaved window; keys are rotated at ``index + S + N``
        (fa2_decode.py:127-131) with the BF16-exact rule of the fused decode
        and stored in the native token-major layout."""
        if self.layout is not None or self.split is not None:
            raise ValueError('load_memory fills the dense, unsplit latent layout')
        cfg, dev = self.cfg, self.device
        hist, tail = self.history.cpu(), self.tail.cpu()
        if not (hist == hist[0]).all() or not (tail == tail[0]).all():
            raise ValueError('load_memory needs every sequence at the same history and tail')
        N, T, S = int(hist[0]), int(tail[0]), cfg.sink
        n_win = T // cfg.ratio
        bf = dict(device=dev, dtype=torch.bfloat16)
        idx = None
        if T:
            if window_raw_indices is None or len(window_raw_indices) != T:
                raise ValueError('window_raw_indices must place every raw token of the open window')
            idx = torch.as_tensor(window_raw_indices, dtype=torch.int64, device=dev)
        B = self.batch
        def rows(st, name, n, width, heads=None):
            x = torch.as_tensor(st[name]).to(**bf)
            if x.numel() != B * (heads or 1) * n * width:
                raise ValueError(f'{name} must hold {B} x {heads or 1} x {n} x {width} values')
            return x.reshape(B, heads, n, width) if heads else x.reshape(B, n, width)

        for c, st in zip(self.caches, layers):
            parts = [('sink_k', 'sink_v', S)] + ([('raw_k', 'raw_v', T)] if T else [])
            keys = torch.cat([rows(st, k, n, cfg.head_dim, cfg.kv_heads) for k, _, n in parts], dim=2)
            values = torch.cat([rows(st, v, n, cfg.head_dim, cfg.kv_heads) for _, v, n in parts], dim=2)
            # The decode RoPE rotates key K-1 at the query position: append a
            # dummy row there and drop it.
            dummy = torch.zeros(B, cfg.kv_heads, 1, cfg.head_dim, **bf)
            q = torch.zeros(B, cfg.heads, 1, cfg.head_dim, **bf)
            qpos = torch.full((B, 1), S + N + T + n_win, dtype=torch.int64, device=dev)
            _, k_rot = kernels.rope_decode(q, torch.cat([keys, dummy], dim=2), self.cos, self.sin, qpos, idx, S, N)
            K = S + T
            c['raw_k_rot'][:, :K].copy_(k_rot[:, :, :K].transpose(1, 2))
            if c['raw_k_pre'] is not None:
                c['raw_k_pre'][:, :K].copy_(keys.transpose(1, 2))
            c['raw_v'][:, :K].copy_(values.transpose(1, 2))
            lat_k, lat_v = rows(st, 'hist_k', N, cfg.rank_k), rows(st, 'hist_v', N, cfg.rank_v)
            if n_win:
                lat_k = torch.cat([lat_k, rows(st, 'win_k', n_win, cfg.rank_k)], 1)
                lat_v = torch.cat([lat_v, rows(st, 'win_v', n_win, cfg.rank_v)], 1)
            c['lat_k'][:, :N + n_win].copy_(lat_k)
            c['lat_v'][:, :N + n_win].copy_(lat_v)

    def step_eager(self):
        """One decode step on the current stream (what the graph captures)."""
        cfg, w = self.cfg, self.w
        B, H = self.batch, cfg.hidden
        qd = cfg.heads * cfg.head_dim
        nb = qd + cfg.rank_k + cfg.rank_v
        kernels.decode_schedule(self.history, self.tail, self.raw_len, self.latent_len, self.query_len,
                                self.qpos, cfg.sink, cfg.window, cfg.ratio)
        sp = self.split
        if sp is not None and sp['last']:
            torch.sub(self.latent_len, sp['offset'], out=sp['latent_len'])
        if not self.recon:
            self.calls[0].compute_plan(self.plan)
        x = self.x
        x[:, 0].copy_(w.embed.index_select(0, self.tokens))
        x[:, 1].copy_(w.beacon_embed.expand(B, -1))
        x2d, h = x.view(2 * B, H), self.h
        for i, (layer, call) in enumerate(zip(w.layers, self.calls)):
            kernels.rms_norm(x, layer['norm1'], cfg.rms_eps, out=h)
            if cfg.qkv_bias:
                torch.addmm(layer['b_raw'], h[:, 0], layer['w_raw'].t(), out=self.z[:, 0])
                torch.addmm(layer['b_beacon'], h[:, 1], layer['w_beacon'].t(), out=self.z[:, 1, :nb])
            else:
                torch.mm(h[:, 0], layer['w_raw'].t(), out=self.z[:, 0])
                torch.mm(h[:, 1], layer['w_beacon'].t(), out=self.z[:, 1, :nb])
            if self.recon:
                self._reconstruct_attention(i)
            else:
                call()
            if self.merges:
                self.merges[i]()                     # all-gather of the partials + N-part merge -> self.attn
            # Residual adds in the GEMMs' accumulate (beta = 1, one bf16 rounding).
            x2d.addmm_(self.attn.view(2 * B, qd), layer['w_o'].t())
            kernels.rms_norm(x, layer['norm2'], cfg.rms_eps, out=h)
            torch.mm(h.view(2 * B, H), layer['w_gate_up'].t(), out=self.gu)
            kernels.silu_mul(self.gu, out=self.act)
            x2d.addmm_(self.act, layer['w_down'].t())
        final = kernels.rms_norm(x[:, 0], w.final_norm, cfg.rms_eps, out=self.h_final)
        # bf16 operands, the fp32 accumulator kept as the logits (no bf16
        # rounding of the output: same weight traffic, exact to the GEMM).
        torch.mm(final, w.lm_head.t(), torch.float32, out=self.logits)
        return self.logits

    def _reconstruct_attention(self, i):
        """One layer of the reconstruct backend (reconstruction_attention,
        tools/benchmark/context_decode_runtime.py:298-344): RoPE of the
        queries and of the new raw key, cache appends, Beacon K/V rebuilt from
        the latents, attention over raw + rebuilt keys into ``self.attn``."""
        cfg, c = self.cfg, self.caches[i]
        B, qd, kvd = self.batch, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        z = self.z
        q = z[:, :, :qd].unflatten(-1, (cfg.heads, cfg.head_dim)).transpose(1, 2)      # [B, H, 2, D]
        k_new = z[:, 0, qd:qd + kvd].unflatten(-1, (cfg.kv_heads, 1, cfg.head_dim))    # [B, Hkv, 1, D]
        q_rot, k_rot = kernels.rope_decode(q, k_new, self.cos, self.sin, self.qpos, None, 0, 0)
        row = (self.raw_len - 1).long()
        c['raw_k_rot'].index_put_((self.batch_index, row), k_rot[:, :, 0])
        c['raw_v'].index_put_((self.batch_index, row), z[:, 0, qd + kvd:qd + 2 * kvd].unflatten(-1, (cfg.kv_heads, cfg.head_dim)))
        if c['raw_k_pre'] is not None:
            c['raw_k_pre'].index_put_((self.batch_index, row), k_new[:, :, 0])
        # The Beacon latent pair of rows that insert one (others rewrite their last row unchanged).
        lrow = (self.latent_len - 1).clamp_min(0).long()
        insert = (self.query_len == 2)[:, None]
        for name, lo, hi in (('lat_k', qd, qd + cfg.rank_k), ('lat_v', qd + cfg.rank_k, qd + cfg.rank_k + cfg.rank_v)):
            new_lat = torch.where(insert, z[:, 1, lo:hi], c[name][self.batch_index, lrow])
            c[name].index_put_((self.batch_index, lrow), new_lat)
        self.recon[i](q_rot.transpose(1, 2), self.attn.view(B, 2, cfg.heads, cfg.head_dim))

    def capture(self, warmup=2):
        """Capture one decode step in a CUDA graph (warm-up steps advance the cache)."""
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.step_eager()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.step_eager()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        return self.graph

    def step(self):
        if self.graph is None:
            return self.step_eager()
        self.graph.replay()
        return self.logits

    def capture_host_io(self, host_tokens, host_next):
        """Capture a second graph for serving from host memory: this step's
        token ids copied in from ``host_tokens`` (pinned int64 [B]), the step,
        the greedy next tokens copied out to ``host_next`` (pinned int64 [B]),
        all in one replay (``step_host``)."""
        if not (host_tokens.is_pinned() and host_next.is_pinned() and host_tokens.numel() == self.batch and
                host_next.numel() == self.batch):
            raise ValueError('host_tokens / host_next must be pinned int64 [batch]')
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        self.graph_host = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph_host, stream=stream):
            self.tokens.copy_(host_tokens, non_blocking=True)
            self.step_eager()
            host_next.copy_(self.logits.argmax(-1), non_blocking=True)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        self._host_next = host_next
        return self.graph_host

    def step_host(self):
        """One decode step from and to host memory (``capture_host_io``):
        returns the pinned next-token buffer once it holds this step's tokens."""
        self.graph_host.replay()
        torch.cuda.current_stream(self.device).synchronize()
        return self._host_next

    def next_tokens(self):
        return self.logits.argmax(-1)

    # ------------------------------------------------------------------
    def attention_kernel_bytes(self):
        """Algorithmic HBM bytes of one attention launch (one layer, both
        branches): every latent K/V row (``N (Rk + Rv) 2``) and every raw
        key/value (``(S + T + 1) Hkv D 2`` each) of every sequence, read once
        (this rank's shard under a sequence split)."""
        cfg = self.cfg
        lat = self.call_latent_len.long().sum().item() * (cfg.rank_k + cfg.rank_v) * 2
        raw = self.call_raw_len.long().sum().item() * cfg.kv_heads * cfg.head_dim * 2 * 2
        return lat + raw

    def attention_bytes(self):
        """Algorithmic HBM bytes of this step's attention, summed over layers.

        Per layer and sequence: the latent K/V rows read (``N (Rk + Rv) 2``),
        the raw keys/values read (``S + T + 1`` tokens of ``Hkv D`` bf16 K and
        V), the query and output rows, plus the up-projection weights once.
        """
        cfg = self.cfg
        lat = self.call_latent_len.long().sum().item() * (cfg.rank_k + cfg.rank_v) * 2
        raw = self.call_raw_len.long().sum().item() * cfg.kv_heads * cfg.head_dim * 2 * 2
        rows = self.query_len.long().sum().item() * cfg.heads * cfg.head_dim * 2 * 2
        weights = cfg.kv_heads * cfg.head_dim * (cfg.rank_k + cfg.rank_v) * 2
        return cfg.layers * (lat + raw + rows + weights)
