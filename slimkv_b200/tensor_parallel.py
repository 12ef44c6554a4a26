"""Tensor-parallel decode: projections and MLP split by KV head, attention by sequence.

The partition the decode step takes over N GPUs of one node (one process per
GPU, NCCL): the weights that dominate a decode step at small batch are
split N ways, so that a fixed global batch gets faster with more GPUs.

* q/k/v and Beacon-q projections column-parallel by KV head (rank r owns KV
  heads ``[r Hkv/N, (r+1) Hkv/N)`` and their query heads); ``o_proj``,
  ``down_proj`` row-parallel with an NCCL all-reduce of fp32 partial sums;
  ``gate/up_proj`` column-parallel; ``lm_head`` split by vocabulary rows and
  all-gathered.
* The latents are shared by every KV head (one latent "head" per sequence),
  so splitting attention by head would make every rank read every latent.
  Attention is split by sequence instead: rank r holds the caches (all KV
  heads, latents and raw rows) of sequences ``[r B/N, (r+1) B/N)``.  One
  all-to-all per layer turns the head-split projection outputs into the
  sequence-split rows the fused decode reads, and one all-to-all turns its
  outputs back into the head-split rows of ``o_proj``.  The K/V
  down-projections (the Beacon latents) are small and replicated; each rank
  computes them for its own sequences.

Per layer: 2 all-to-alls and 2 all-reduces; per step one all-gather of the
logits.  The hidden state is replicated on every rank.
"""
import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import kernels
from .runtime import LatentDecodeRuntime


def shard_weights(cfg, weights, rank, world):
    """This rank's slices of a full set of runtime weights (``RandomWeights``
    / ``StateDictWeights`` layout): a list of per-layer dicts and the
    vocabulary slice of ``lm_head``."""
    D, H, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    if H % world or Hkv % world or cfg.intermediate % world or cfg.vocab % world:
        raise ValueError('heads, KV heads, intermediate size and vocabulary must divide by the ranks')
    qd, kvd = H * D, Hkv * D
    qs, ks, Is = qd // world, kvd // world, cfg.intermediate // world
    q = slice(rank * qs, (rank + 1) * qs)
    k = slice(qd + rank * ks, qd + (rank + 1) * ks)
    v = slice(qd + kvd + rank * ks, qd + kvd + (rank + 1) * ks)
    i0 = slice(rank * Is, (rank + 1) * Is)
    i1 = slice(cfg.intermediate + rank * Is, cfg.intermediate + (rank + 1) * Is)
    layers = []
    for L in weights.layers:
        s = dict(norm1=L['norm1'], norm2=L['norm2'],
                 w_raw=torch.cat([L['w_raw'][q], L['w_raw'][k], L['w_raw'][v]]).contiguous(),
                 w_bq=L['w_beacon'][q].contiguous(),
                 w_down_lat=L['w_beacon'][qd:qd + cfg.rank_k + cfg.rank_v].contiguous(),
                 w_o=L['w_o'][:, q].contiguous(),
                 w_gate_up=torch.cat([L['w_gate_up'][i0], L['w_gate_up'][i1]]).contiguous(),
                 w_down=L['w_down'][:, i0].contiguous())
        if cfg.qkv_bias:
            s.update(b_raw=torch.cat([L['b_raw'][q], L['b_raw'][k], L['b_raw'][v]]).contiguous(),
                     b_bq=L['b_beacon'][q].contiguous())
        layers.append(s)
    vs = cfg.vocab // world
    return layers, weights.lm_head[rank * vs:(rank + 1) * vs].contiguous()


def heads_to_sequences(send, recv, z, qs, ks, group=None):
    """All-to-all of the head-split projection outputs into sequence-split
    attention inputs.

    ``send [B, 2 qs + 2 ks]``: this rank's heads for every sequence, per row
    ``[q raw | k new | v new | q Beacon]`` (rows in sequence order, so rank s
    receives rows ``[s B/N, (s+1) B/N)``).  ``recv [N, B/N, same]`` receives
    each rank's heads for this rank's sequences.  ``z [B/N, 2, width]`` (the
    fused decode's projection buffer) gets every head: row 0 ``[q | k | v]``,
    row 1 ``[q Beacon | ...]`` (the Beacon latents are written separately)."""
    dist.all_to_all_single(recv, send, group=group)
    N, b = recv.shape[0], recv.shape[1]
    qd, kvd = N * qs, N * ks
    z[:, 0, :qd].view(b, N, qs).copy_(recv[:, :, :qs].permute(1, 0, 2))
    z[:, 0, qd:qd + kvd].view(b, N, ks).copy_(recv[:, :, qs:qs + ks].permute(1, 0, 2))
    z[:, 0, qd + kvd:qd + 2 * kvd].view(b, N, ks).copy_(recv[:, :, qs + ks:qs + 2 * ks].permute(1, 0, 2))
    z[:, 1, :qd].view(b, N, qs).copy_(recv[:, :, qs + 2 * ks:].permute(1, 0, 2))


def sequences_to_heads(attn, send, recv, group=None):
    """All-to-all of the sequence-split attention output ``attn [B/N, 2, H D]``
    into every sequence's rows for this rank's heads: ``recv [N, B/N, 2,
    H D / N]``, i.e. ``[B, 2, H D / N]`` in sequence order."""
    N, b, _, qs = send.shape
    send.copy_(attn.view(b, 2, N, qs).permute(2, 0, 1, 3))
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(N * b, 2, qs)


class TensorParallelDecode:
    """One rank of a tensor-parallel decode step over the global batch.

    ``history`` / ``tails`` describe all B sequences (B divisible by the
    ranks); this rank keeps the caches of its own B/N.  ``weights`` is the
    full model (sliced here; the attention's up-projections stay whole).
    ``group``: the process group (default: the world).  ``step()`` returns
    the fp32 logits ``[B, vocab]`` of every sequence on every rank."""

    def __init__(self, cfg, weights, history, tails, device, group=None, **runtime_kwargs):
        self.cfg, self.device, self.group = cfg, device, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        B = len(history)
        if B % self.world:
            raise ValueError('the global batch must divide by the ranks')
        self.batch, self.local = B, B // self.world
        lo = self.rank * self.local
        # Caches, schedule and fused decode calls of this rank's sequences.
        self.rt = LatentDecodeRuntime(cfg, weights, list(history)[lo:lo + self.local],
                                      list(tails)[lo:lo + self.local], device, **runtime_kwargs)
        if self.rt.recon or self.rt.split is not None:
            raise ValueError('tensor parallelism runs the latent backend without a sequence split')
        self.layers, self.lm_head = shard_weights(cfg, weights, self.rank, self.world)
        self.rt.w = None            # the local runtime's own (unsplit) step is not used
        self.embed, self.beacon_embed, self.final_norm = weights.embed, weights.beacon_embed, weights.final_norm
        D, H, Hkv, N, b = cfg.head_dim, cfg.heads, cfg.kv_heads, self.world, self.local
        self.qs, self.ks = H * D // N, Hkv * D // N
        P = 2 * self.qs + 2 * self.ks                    # per sequence: q raw | k | v | q Beacon
        bf = dict(dtype=torch.bfloat16, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        self.tokens = torch.zeros(B, dtype=torch.int64, device=device)
        self.x = torch.zeros(B, 2, cfg.hidden, **bf)
        self.send1 = torch.zeros(B, P, **bf)             # rows in sequence order = destination order
        self.recv1 = torch.zeros(N, b, P, **bf)          # [source head shard, my sequences, fields]
        self.lat = torch.zeros(b, cfg.rank_k + cfg.rank_v, **bf)
        self.send2 = torch.zeros(N, b, 2, self.qs, **bf)  # [destination head shard, my sequences, rows]
        self.recv2 = torch.zeros(N, b, 2, self.qs, **bf)  # [source sequence shard, ...] = [B, 2, my heads]
        self.part = torch.zeros(2 * B, cfg.hidden, **f32)
        vs = cfg.vocab // N
        self.logits_part = torch.zeros(B, vs, **f32)
        self.logits_all = torch.zeros(N, B, vs, **f32)
        self.logits = torch.zeros(B, cfg.vocab, **f32)
        self.graph = None

    def _attention_inputs(self, layer):
        """Head-split projections of every sequence -> this rank's sequences
        with every head, in the local runtime's projection buffer."""
        cfg, rt, N, b, qs, ks = self.cfg, self.rt, self.world, self.local, self.qs, self.ks
        h = F.rms_norm(self.x, (cfg.hidden,), layer['norm1'], cfg.rms_eps)
        raw = torch.addmm(layer['b_raw'], h[:, 0], layer['w_raw'].t()) if cfg.qkv_bias else h[:, 0] @ layer['w_raw'].t()
        bq = torch.addmm(layer['b_bq'], h[:, 1], layer['w_bq'].t()) if cfg.qkv_bias else h[:, 1] @ layer['w_bq'].t()
        self.send1[:, :qs + 2 * ks].copy_(raw)
        self.send1[:, qs + 2 * ks:].copy_(bq)
        heads_to_sequences(self.send1, self.recv1, rt.z, qs, ks, self.group)
        # The Beacon latents of this rank's sequences (replicated weights).
        lo = self.rank * b
        torch.mm(h[lo:lo + b, 1], layer['w_down_lat'].t(), out=self.lat)
        qd = cfg.heads * cfg.head_dim
        rt.z[:, 1, qd:qd + cfg.rank_k + cfg.rank_v].copy_(self.lat)

    def step_eager(self):
        """One decode step on the current stream (what the graph captures)."""
        cfg, rt, N, b, B = self.cfg, self.rt, self.world, self.local, self.batch
        H, I = cfg.hidden, cfg.intermediate // N
        kernels.decode_schedule(rt.history, rt.tail, rt.raw_len, rt.latent_len, rt.query_len, rt.qpos, cfg.sink,
                                cfg.window, cfg.ratio)
        rt.calls[0].compute_plan(rt.plan)
        x = self.x
        x[:, 0].copy_(self.embed.index_select(0, self.tokens))
        x[:, 1].copy_(self.beacon_embed.expand(B, -1))
        for layer, call in zip(self.layers, rt.calls):
            self._attention_inputs(layer)
            call()
            # This rank's sequences with every head -> every sequence with this
            # rank's heads, then the row-parallel o_proj and its all-reduce.
            rows = sequences_to_heads(rt.attn, self.send2, self.recv2, self.group)
            torch.mm(rows.view(2 * B, self.qs), layer['w_o'].t(), torch.float32, out=self.part)
            dist.all_reduce(self.part, group=self.group)
            x.add_(self.part.view(B, 2, H))
            h2 = F.rms_norm(x, (H,), layer['norm2'], cfg.rms_eps)
            gu = h2.view(2 * B, H) @ layer['w_gate_up'].t()
            act = F.silu(gu[:, :I]) * gu[:, I:]
            torch.mm(act, layer['w_down'].t(), torch.float32, out=self.part)
            dist.all_reduce(self.part, group=self.group)
            x.add_(self.part.view(B, 2, H))
        final = F.rms_norm(x[:, 0], (H,), self.final_norm, cfg.rms_eps)
        torch.mm(final, self.lm_head.t(), torch.float32, out=self.logits_part)
        dist.all_gather_into_tensor(self.logits_all, self.logits_part, group=self.group)
        self.logits.view(B, N, -1).copy_(self.logits_all.permute(1, 0, 2))
        return self.logits

    def capture(self, warmup=2):
        """Capture one decode step (with its collectives) in a CUDA graph."""
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

    def release(self):
        """Drop the captured graph (it holds NCCL work; release it before the
        process group is destroyed)."""
        self.graph = None
