"""Paged cache IO: the GPU page classes against the reference's page bytes.

``slimkv_b200.pages`` mirrors ``slimkv/vllm_plugin/paged_cache.py``; every
page write must be bit-exact with the reference (golden bytes written by the
reference's own classes, ``tests/golden/make_golden.py:gen_pages``) and with
the oracle's addressing for batched random cases.  Argument checks raise the
reference's errors before any launch.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from oracle.pages import BeaconPageLayout as OracleLayout, beacon_pages_append, raw_page_slots

GOLDEN = np.load(Path(__file__).parent / 'golden' / 'reference_golden.npz')


def _bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


# ---- host-side checks (no GPU) --------------------------------------------

def test_layout_matches_reference_geometry_and_errors():
    from slimkv_b200.pages import BeaconPageLayout
    a = BeaconPageLayout(192, 4, 320, 320, 1024)
    assert (a.slots, a.width, a.sink_elements, a.page_elements, a.storage_rows) == (48, 640, 2048, 32768, 52)
    with pytest.raises(ValueError, match='Cache dimensions must be positive.'):
        BeaconPageLayout(0, 4, 320, 320, 1024)
    with pytest.raises(ValueError, match='Raw block size must be divisible by the token ratio.'):
        BeaconPageLayout(10, 4, 320, 320, 1024)


def test_page_classes_reject_what_the_reference_rejects():
    from slimkv_b200.pages import BeaconPageLayout, BeaconPages, RawPages
    layout = BeaconPageLayout(4, 2, 3, 5, 4)
    with pytest.raises(ValueError, match='BF16 checkpoint precision'):
        BeaconPages(torch.zeros(3, layout.page_elements), layout)
    with pytest.raises(ValueError, match='contiguous feature storage'):
        BeaconPages(torch.zeros(3, 2, layout.page_elements, dtype=torch.bfloat16)[:, :, :-1], layout)
    with pytest.raises(ValueError, match='too small'):
        BeaconPages(torch.zeros(3, layout.page_elements - 1, dtype=torch.bfloat16), layout)
    pages = BeaconPages(torch.zeros(3, layout.page_elements, dtype=torch.bfloat16), layout)
    with pytest.raises(ValueError, match='must not change dtype'):
        pages.append(torch.tensor([0]), 0, torch.zeros(1, 1, 2, 3), torch.zeros(1, 1, 2, 5, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match='independent B1 global-rank'):
        pages.append(torch.tensor([0]), 0, torch.zeros(1, 1, 2, 4, dtype=torch.bfloat16),
                     torch.zeros(1, 1, 2, 5, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match='original raw K/V dimensions'):
        pages.write_sink(0, torch.zeros(3, dtype=torch.bfloat16), torch.zeros(4, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match='Sink head dimensions'):
        pages.read_sink(0, 3, 2)
    with pytest.raises(ValueError, match='block/token/KV/head/dim'):
        RawPages(torch.zeros(8, 4, 3, 2, 3, dtype=torch.bfloat16))
    raw = RawPages(torch.zeros(8, 4, 2, 2, 3, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match='retain BF16'):
        raw.write(torch.tensor([0]), 0, torch.zeros(1, 2, 3, 3), torch.zeros(1, 2, 3, 3, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match='differ from the engine allocation'):
        raw.write(torch.tensor([0]), 0, torch.zeros(1, 3, 3, 3, dtype=torch.bfloat16),
                  torch.zeros(1, 3, 3, 3, dtype=torch.bfloat16))


# ---- GPU: bit-exact page bytes --------------------------------------------

@pytest.mark.gpu
def test_beacon_pages_reproduce_reference_bytes():
    from slimkv_b200.pages import BeaconPageLayout, BeaconPages
    layout = BeaconPageLayout(4, 2, 3, 5, 4)
    backing = torch.full((12, layout.page_elements + 7), -13, dtype=torch.bfloat16, device='cuda')
    pages = BeaconPages(backing[:, :layout.page_elements], layout)
    for index, table in enumerate([torch.tensor([7, 2, 9]), torch.tensor([4, 1, 10])]):
        k = (torch.arange(18).reshape(1, 1, 6, 3) + index * 32).to(torch.bfloat16).cuda()
        v = (torch.arange(30).reshape(1, 1, 6, 5) + index * 32).to(torch.bfloat16).cuda()
        pages.append(table, 0, k[:, :, :3], v[:, :, :3])
        pages.append(table, 3, k[:, :, 3:], v[:, :, 3:])
        sink = torch.full((1, 1, 1, 4), index + 1, dtype=torch.bfloat16, device='cuda')
        pages.write_sink(table[0], sink, sink + 2)
        rk, rv = pages.read(table, 6)
        assert torch.equal(rk, k) and torch.equal(rv, v)
        sk, sv = pages.read_sink(table[0], 1, 4)
        assert torch.equal(sk, sink) and torch.equal(sv, sink + 2)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(backing), GOLDEN['pages_small'].view(np.uint16))

    layout = BeaconPageLayout(192, 4, 320, 320, 1024)
    backing = torch.zeros((9, layout.storage_rows, layout.width), dtype=torch.bfloat16, device='cuda')
    pages = BeaconPages(backing, layout)
    table = torch.tensor([5, 0, 8, 3, 6])
    k = torch.from_numpy(GOLDEN['pages_r4_kin']).view(torch.bfloat16).cuda()
    v = torch.from_numpy(GOLDEN['pages_r4_vin']).view(torch.bfloat16).cuda()
    pages.append(table, 0, k[:, :, :130], v[:, :, :130])
    pages.append(table, 130, k[:, :, 130:], v[:, :, 130:])
    rk, rv = pages.read(table, 200)
    assert torch.equal(rk, k) and torch.equal(rv, v)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(backing), GOLDEN['pages_r4'].view(np.uint16))


@pytest.mark.gpu
def test_raw_pages_reproduce_reference_bytes():
    from slimkv_b200.pages import RawPages
    raw = RawPages(torch.zeros(8, 4, 2, 2, 3, dtype=torch.bfloat16, device='cuda'))
    key = torch.arange(42).reshape(1, 2, 7, 3).to(torch.bfloat16).cuda()
    raw.write(torch.tensor([5, 2, 6, 1]), 5, key, -key)
    rk, rv = raw.read(torch.tensor([5, 2, 6, 1]), 5, 7)
    assert torch.equal(rk, key) and torch.equal(rv, -key)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(raw.pages), GOLDEN['raw_pages'].view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize('ranks,ratio', [((320, 320), 4), ((160, 160), 8), ((48, 40), 2)])
def test_batched_beacon_append_and_gather_match_oracle(ranks, ratio):
    from slimkv_b200 import pages as P
    rk, rv = ranks
    layout = P.BeaconPageLayout(16 * ratio * 3, ratio, rk, rv, 64)
    rng = np.random.default_rng(rk + ratio)
    B, n_pages, per_seq = 3, 40, 6
    # Sequences own disjoint pages, as an engine's block tables do.
    tables = rng.permutation(n_pages)[:B * per_seq].reshape(B, per_seq).astype(np.int32)
    start = rng.integers(0, layout.slots * 2, size=B).astype(np.int32)
    count = int(layout.slots * 3)
    k = oracle.round_bf16(rng.standard_normal((B, count, rk)).astype(np.float32))
    v = oracle.round_bf16(rng.standard_normal((B, count, rv)).astype(np.float32))
    backing = torch.zeros(n_pages, layout.page_elements + 16, dtype=torch.bfloat16, device='cuda')
    kt = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vt = torch.from_numpy(v).to(torch.bfloat16).cuda()
    P.beacon_append(backing, layout, torch.from_numpy(tables), start, kt, vt)
    want = np.zeros((n_pages, layout.page_elements + 16), np.float32)
    ol = OracleLayout(layout.raw_block_size, ratio, rk, rv, 64)
    for b in range(B):
        beacon_pages_append(want, tables[b], int(start[b]), k[b], v[b], ol)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(backing), oracle.bf16_bits(want))
    # gather back the first start + count rows of each sequence
    n = start + count
    gk = torch.zeros(B, int(n.max()), rk, dtype=torch.bfloat16, device='cuda')
    gv = torch.zeros(B, int(n.max()), rv, dtype=torch.bfloat16, device='cuda')
    P.beacon_gather(backing, layout, torch.from_numpy(tables), n, gk, gv)
    torch.cuda.synchronize()
    for b in range(B):
        assert torch.equal(gk[b, start[b]:n[b]].cpu(), kt[b].cpu())
        assert torch.equal(gv[b, start[b]:n[b]].cpu(), vt[b].cpu())


@pytest.mark.gpu
def test_batched_raw_write_and_read_match_oracle_addressing():
    from slimkv_b200 import pages as P
    rng = np.random.default_rng(5)
    B, blocks, per_seq, bs, H, D = 4, 64, 12, 16, 8, 128
    tables = rng.permutation(blocks)[:B * per_seq].reshape(B, per_seq).astype(np.int32)
    start = rng.integers(0, 60, size=B).astype(np.int32)
    count = 97
    k = torch.randn(B, count, H, D).to(torch.bfloat16).cuda()
    v = torch.randn(B, count, H, D).to(torch.bfloat16).cuda()
    pages = torch.zeros(blocks, bs, 2, H, D, dtype=torch.bfloat16, device='cuda')
    P.raw_write(pages, torch.from_numpy(tables), start, k, v)
    torch.cuda.synchronize()
    host = pages.cpu()
    for b in range(B):
        blk, row = raw_page_slots(tables[b], int(start[b]), count, bs)
        assert torch.equal(host[blk, row, 0], k[b].cpu()) and torch.equal(host[blk, row, 1], v[b].cpu())
    rk = torch.zeros_like(k)
    rv = torch.zeros_like(v)
    counts = np.array([count, 5, 0, 60], np.int32)
    P.raw_read(pages, torch.from_numpy(tables), start, counts, rk, rv)
    torch.cuda.synchronize()
    for b in range(B):
        assert torch.equal(rk[b, :counts[b]], k[b, :counts[b]]) and torch.equal(rv[b, :counts[b]], v[b, :counts[b]])
        assert (rk[b, counts[b]:] == 0).all()


@pytest.mark.gpu
def test_page_id_outside_the_allocation_is_reported_not_written():
    from slimkv_b200 import _lib, pages as P
    layout = P.BeaconPageLayout(16, 2, 8, 8, 8)
    backing = torch.zeros(4, layout.page_elements, dtype=torch.bfloat16, device='cuda')
    _lib.device_status(clear=True)
    k = torch.ones(1, 1, 3, 8, dtype=torch.bfloat16, device='cuda')
    P.BeaconPages(backing, layout).append(torch.tensor([9]), 0, k, k)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 2          # SLIMKV_DEVICE_BAD_LENGTH
    assert (backing == 0).all()
