"""The two all-to-alls of the tensor-parallel decode, on two gloo ranks (CPU).

``heads_to_sequences`` must hand each rank, for its own sequences, the
projection rows of every head exactly as an unsplit projection lays them
out in the fused decode's buffer; ``sequences_to_heads`` must give each rank
every sequence's attention rows for its own heads.  Checked against the
unsplit tensors built from the same seed on every rank.
"""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank(rank, world, port, errors):
    os.environ['MASTER_ADDR'], os.environ['MASTER_PORT'] = '127.0.0.1', str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        from slimkv_b200.tensor_parallel import heads_to_sequences, sequences_to_heads
        B, H, Hkv, D = 6, 8, 4, 4
        qd, kvd, N = H * D, Hkv * D, world
        qs, ks, b = qd // N, kvd // N, B // N
        g = torch.Generator().manual_seed(0)
        q_raw, q_bcn = torch.randn(B, qd, generator=g), torch.randn(B, qd, generator=g)
        k_new, v_new = torch.randn(B, kvd, generator=g), torch.randn(B, kvd, generator=g)
        # This rank's head shard of every sequence, packed as the decode sends it.
        send = torch.cat([q_raw[:, rank * qs:(rank + 1) * qs], k_new[:, rank * ks:(rank + 1) * ks],
                          v_new[:, rank * ks:(rank + 1) * ks], q_bcn[:, rank * qs:(rank + 1) * qs]], 1).contiguous()
        recv = torch.zeros(N, b, send.shape[1])
        width = qd + 2 * kvd
        z = torch.full((b, 2, width), float('nan'))
        heads_to_sequences(send, recv, z, qs, ks)
        mine = slice(rank * b, (rank + 1) * b)
        assert torch.equal(z[:, 0], torch.cat([q_raw, k_new, v_new], 1)[mine])
        assert torch.equal(z[:, 1, :qd], q_bcn[mine])
        # Attention rows: this rank's sequences, every head -> every sequence, my heads.
        attn_all = torch.randn(B, 2, qd, generator=g)
        send2, recv2 = torch.zeros(N, b, 2, qs), torch.zeros(N, b, 2, qs)
        rows = sequences_to_heads(attn_all[mine].contiguous(), send2, recv2)
        assert torch.equal(rows, attn_all[:, :, rank * qs:(rank + 1) * qs])
    except Exception as e:                      # reported by the parent
        errors.put(f'rank {rank}: {e!r}')
    finally:
        dist.destroy_process_group()


def test_exchanges_on_two_gloo_ranks():
    ctx = mp.get_context('spawn')
    errors = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert errors.empty(), errors.get()
