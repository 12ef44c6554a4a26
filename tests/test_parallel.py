"""Multi-rank host logic on CPU (gloo, world size 2).

The sequence split: each rank computes the oracle's attention over its
contiguous key shard and ``merge_sequence_split`` must reproduce attention
over the whole sequence (the LSE merge of fa2_decode.py:57-66 over ranks),
both for plain attention and for the fused latent decode step (latent
history sharded, raw branch on the last rank, biases included).  Also the
max-over-ranks timing helper.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _run(fn, port, *args):
    mp.start_processes(_entry, args=(fn, port) + args, nprocs=WORLD, start_method='spawn', join=True)


def _entry(rank, fn, port, *args):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    from datetime import timedelta
    dist.init_process_group('gloo', rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        fn(rank, *args)
    finally:
        dist.destroy_process_group()


def _attention_split(rank):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden'))
    import oracle
    from cases import attention_case
    from slimkv_b200.parallel import merge_sequence_split, shard_range
    c = attention_case(31, 2, 2, 8, 2, 700, 64, 64, False)
    n = c['k'].shape[1]
    lo, hi = shard_range(n, WORLD, rank)
    out, lse = oracle.eager_attention(c['q'], c['k'][:, lo:hi], c['v'][:, lo:hi], c['scale'], False)
    out_t = torch.from_numpy(np.ascontiguousarray(out.transpose(0, 2, 1, 3)))      # [B, H, Q, D]
    merged, total = merge_sequence_split(out_t, torch.from_numpy(lse))
    ref, ref_lse = oracle.eager_attention(c['q'], c['k'], c['v'], c['scale'], False)
    np.testing.assert_allclose(merged.numpy(), ref.transpose(0, 2, 1, 3), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(total.numpy(), ref_lse, rtol=1e-6, atol=1e-6)


def _decode_split(rank, length):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden'))
    import oracle
    from oracle.decode import latent_decode_attention
    from cases import decode_case, LLAMA8B
    from slimkv_b200.parallel import merge_sequence_split, shard_range
    c = decode_case(41, batch=2, length=length, history=600, tail=70, heads=8, kv_heads=2, head_dim=32,
                    rk=48, rv=40, bias=True)
    cos, sin = oracle.rope_tables(32, LLAMA8B['theta'], 4096, LLAMA8B['scaling'])
    n_lat = c['lat_k'].shape[1]
    lo, hi = shard_range(n_lat, WORLD, rank)
    last = rank == WORLD - 1
    raw = slice(None) if last else slice(0, 0)       # the raw branch lives on the last rank
    r = latent_decode_attention(c['q'], c['raw_k'][:, raw], c['raw_v'][:, raw], c['lat_k'][:, lo:hi],
                                c['lat_v'][:, lo:hi], c['uk'], c['uv'], cos, sin, c['qpos'], c['kpos'][:, raw],
                                length - 1 if last else 0, uk_bias=c['bk'], uv_bias=c['bv'])
    b, l, h = c['q'].shape[:3]
    lse = np.logaddexp(r['raw_lse'], r['latent_lse']) if 'latent_lse' in r else r['raw_lse']   # [B, H, L]
    out = r['out'].reshape(b, l, h, -1).transpose(0, 2, 1, 3)                                  # [B, H, L, d]
    merged, _ = merge_sequence_split(torch.from_numpy(np.ascontiguousarray(out)), torch.from_numpy(lse))
    ref = latent_decode_attention(c['q'], c['raw_k'], c['raw_v'], c['lat_k'], c['lat_v'], c['uk'], c['uv'], cos,
                                  sin, c['qpos'], c['kpos'], length - 1, uk_bias=c['bk'], uv_bias=c['bv'])
    want = ref['out'].reshape(b, l, h, -1).transpose(0, 2, 1, 3)
    err = np.linalg.norm(merged.numpy() - want) / np.linalg.norm(want)
    assert err < 1e-6, err


def _max_over_ranks(rank):
    from slimkv_b200.parallel import max_over_ranks
    assert max_over_ranks(1.0 + rank) == float(WORLD)


def test_shard_range_covers_keys_once():
    from slimkv_b200.parallel import shard_range
    for n in (0, 1, 127, 128, 129, 1000, 8447):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(s % 128 == 0 for s, _ in spans if s < n)


def test_sequence_split_attention_matches_whole_sequence():
    _run(_attention_split, _free_port())


@pytest.mark.parametrize('length', [1, 2])
def test_sequence_split_latent_decode_matches_whole_sequence(length):
    _run(_decode_split, _free_port(), length)


def test_max_over_ranks():
    _run(_max_over_ranks, _free_port())
