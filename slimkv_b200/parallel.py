"""Multi-GPU plumbing of the decode path (one process per GPU).

Two ways the path scales:

* **Batch replicas** (the bench's weak scaling): every rank owns whole
  sequences; nothing crosses ranks on the data path.  Only the timing uses a
  collective (:func:`max_over_ranks`).
* **Sequence split** (one long sequence over several GPUs): each rank holds a
  contiguous shard of the sequence's keys (:func:`shard_range`), computes its
  partial attention output and log-sum-exp over that shard, and
  :func:`merge_sequence_split` combines the partials exactly - the LSE merge of
  ``merge_attention`` (slimkv/llama3/fa2_decode.py:57-66) generalised to N
  parts: ``T = logsumexp_r(lse_r)``, ``out = sum_r exp(lse_r - T) out_r``.
  The exchange is one all-gather of the LSEs (B*H*L floats) and one all-reduce
  of the weighted outputs, over NCCL (NVLink) on GPUs or gloo on CPU.

On GPUs the decode runtime uses :class:`SequenceSplitMerge`: the fused decode
of each rank writes its fp32 partial output and LSE straight into one packed
buffer, a single NCCL all-gather moves those buffers (the partials after the
V up-projection: ``B*L*H*(D+1)`` floats a rank, 20 KB a layer for one
Qwen2.5-14B sequence), and ``slimkv_merge_partials`` combines the N parts on
every rank.  The merge after the up-projection is exact because the
up-projection and its bias are linear and the merge weights sum to 1.
"""
import torch
import torch.distributed as dist


def shard_range(n_keys, world, rank, tile=128):
    """Contiguous key range ``[start, end)`` of ``rank``: whole ``tile``-key
    tiles spread evenly (the last rank takes the ragged end)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError('rank out of range')
    tiles = (max(int(n_keys), 0) + tile - 1) // tile
    start = min(n_keys, (rank * tiles // world) * tile)
    end = min(n_keys, ((rank + 1) * tiles // world) * tile)
    return start, end


def merge_sequence_split(out, lse, group=None):
    """Exact merge of per-rank partial attention.

    ``out [..., H, L, D]``-like tensor whose leading dims match ``lse``'s with
    one trailing feature dim (any layout where ``lse.unsqueeze(-1)``
    broadcasts against ``out``); ``lse`` is the natural-log sum of exp of this
    rank's scores, ``-inf`` for a rank without keys.  Returns ``(out, lse)`` of
    the whole sequence on every rank (fp32).  Rows without keys anywhere get
    zero output and ``-inf`` LSE.
    """
    out = out.float()
    lse = lse.float()
    world = dist.get_world_size(group)
    parts = [torch.empty_like(lse) for _ in range(world)]
    dist.all_gather(parts, lse.contiguous(), group=group)
    stack = torch.stack(parts)                                     # [world, ...]
    m = stack.max(dim=0).values
    finite = torch.isfinite(m)
    m_safe = torch.where(finite, m, torch.zeros_like(m))
    total = torch.where(finite, m_safe + torch.log(torch.exp(stack - m_safe).sum(dim=0)),
                        torch.full_like(m, float('-inf')))
    weight = torch.where(torch.isfinite(lse) & finite, torch.exp(lse - torch.where(finite, total, m_safe)),
                         torch.zeros_like(lse))
    merged = (out * weight.unsqueeze(-1)).contiguous()
    dist.all_reduce(merged, op=dist.ReduceOp.SUM, group=group)
    return merged, total


class SequenceSplitMerge:
    """One layer's cross-GPU exchange of a sequence split (graph-capturable).

    ``out`` (fp32 ``[B, L, H*D]``) and ``lse`` (fp32 ``[B, L, H]``) are views
    of this rank's packed send buffer, handed to the fused decode as its
    ``out`` / ``out_lse``; :meth:`__call__` all-gathers the packed buffers and
    merges them into ``merged`` (``[B, L, H*D]``, ``out_dtype``) with
    ``slimkv_merge_partials``.  Rows that no rank writes (unused Beacon
    slots) keep LSE ``-inf`` and merge to zeros.
    """

    def __init__(self, batch, length, heads, head_dim, group=None, device=None, out_dtype=torch.bfloat16,
                 merged=None):
        self.group = group
        self.world = dist.get_world_size(group)
        rows = batch * length * heads
        self.rows, self.dim = rows, head_dim
        self.lse_at = rows * head_dim
        width = self.lse_at + (rows + 3) // 4 * 4                    # float4-aligned part stride
        self.send = torch.zeros(width, dtype=torch.float32, device=device)
        self.send[self.lse_at:].fill_(float('-inf'))
        self.gather = torch.empty(self.world, width, dtype=torch.float32, device=device)
        self.out = self.send[:self.lse_at].view(batch, length, heads * head_dim)
        self.lse = self.send[self.lse_at:self.lse_at + rows].view(batch, length, heads)
        self.merged = merged if merged is not None else torch.empty(batch, length, heads * head_dim,
                                                                    dtype=out_dtype, device=device)

    def __call__(self):
        from . import kernels
        dist.all_gather_into_tensor(self.gather, self.send, group=self.group)
        kernels.merge_partials(self.gather[:, :self.lse_at].view(self.world, self.rows, self.dim),
                               self.gather[:, self.lse_at:self.lse_at + self.rows], self.merged)
        return self.merged


def max_over_ranks(value, device=None, group=None):
    """The largest ``value`` over all ranks (e.g. a step time, so that a
    multi-GPU time is the slowest rank's)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.item()
