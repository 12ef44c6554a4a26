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


def max_over_ranks(value, device=None, group=None):
    """The largest ``value`` over all ranks (e.g. a step time, so that a
    multi-GPU time is the slowest rank's)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.item()
