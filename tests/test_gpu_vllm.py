"""The vLLM plugin's paged decode, batched over requests, on the fused decode.

``slimkv_b200.vllm.PagedDecodeLayer`` takes what the plugin's
``_paged_forward`` receives from vLLM (vllm_plugin/model.py:114-142): each
request's block-table rows for its raw and Beacon pages and its ``seq_lens``
entry, for one decode token per request.  Pages are filled through the GPU
drop-in of the plugin's page classes (``slimkv_b200.pages``, bit-exact with
the reference page bytes in ``tests/test_pages.py``), in shuffled blocks, with
requests at different window offsets (some insert a Beacon this step).

Checked against the oracle: the attention output of every request row (bf16
bar: norm-wise 3e-3 plus the reference GPU tolerance), and the page bytes the
step writes — the new raw token at its absolute raw position (pre-RoPE K and
V) and the new Beacon row at its slot — bit for bit; all other page bytes
unchanged.
"""
import numpy as np
import pytest
import torch

import oracle
from cases import LLAMA8B
from gpu_util import assert_attention_close, to_bf16

pytestmark = pytest.mark.gpu


def test_backends_keep_the_plugin_cache_geometry():
    from slimkv_b200 import vllm
    assert vllm.RawPageBackend.get_kv_cache_shape(10, 16, 8, 128) == (10, 16, 2, 8, 128)
    assert vllm.BeaconPageBackend.get_kv_cache_shape(10, 192, 1, 640) == (10, 192, 640)
    assert vllm.RawPageBackend.get_kv_cache_stride_order() == (0, 1, 2, 3, 4)
    assert vllm.BeaconPageBackend.get_kv_cache_stride_order(True) == (1, 0, 2, 3)
    assert (vllm.RawPageBackend.get_name(), vllm.BeaconPageBackend.get_name()) == ('SLIMKV_RAW', 'SLIMKV_BEACON')
    # r4 / t4 on Llama-3.1-8B: 192 raw tokens (48 slots) per page, two sink rows.
    assert vllm.beacon_block_size(4, 1024, 640) == 192
    assert vllm.storage_block_size(192, 4, 1024, 640) == 48 + 4


def test_paged_decode_layer_matches_oracle_and_page_bytes():
    from slimkv_b200 import pages as P, vllm, _lib
    dev = torch.device('cuda', 0)
    rng = np.random.default_rng(2027)
    Hkv, D, H, R, ratio, window, sink = 8, 128, 32, 320, 4, 1024, 1
    kvd = Hkv * D
    block = vllm.beacon_block_size(ratio, kvd, 2 * R)
    layout = P.BeaconPageLayout(block, ratio, R, R, kvd)
    # Tokens already in the pages per request (all past their first window).
    processed = np.array([1024 + 7, 2048 + 300, 3072 + 1019, 1024 + 3, 5000])
    B = len(processed)
    seq_lens = processed + 1
    raw_blocks = (seq_lens + 15) // 16
    beacon_rows = processed // ratio + 1
    beacon_blocks = (beacon_rows + layout.slots - 1) // layout.slots
    raw_perm = rng.permutation(int(raw_blocks.sum()) + 5)
    bcn_perm = rng.permutation(int(beacon_blocks.sum()) + 3)
    raw_table = np.zeros((B, raw_blocks.max()), np.int32)
    bcn_table = np.zeros((B, beacon_blocks.max()), np.int32)
    a = c = 0
    for b in range(B):
        raw_table[b, :raw_blocks[b]] = raw_perm[a:a + raw_blocks[b]]
        bcn_table[b, :beacon_blocks[b]] = bcn_perm[c:c + beacon_blocks[b]]
        a += raw_blocks[b]
        c += beacon_blocks[b]
    raw_pages = to_bf16(rng.standard_normal((len(raw_perm), 16, 2, Hkv, D), dtype=np.float32))
    bcn_pages = to_bf16(rng.standard_normal((len(bcn_perm), layout.storage_rows, 2 * R), dtype=np.float32))
    # Contents the requests wrote before this step: raw K/V of every token,
    # Beacon latents, the sink token in each root page.
    mag = 1.3
    raw_k = [oracle.round_bf16(rng.standard_normal((n, Hkv, D), dtype=np.float32) * mag) for n in processed]
    raw_v = [oracle.round_bf16(rng.standard_normal((n, Hkv, D), dtype=np.float32) * mag) for n in processed]
    lat_k = [oracle.round_bf16(rng.standard_normal((n // ratio, R), dtype=np.float32) * mag) for n in processed]
    lat_v = [oracle.round_bf16(rng.standard_normal((n // ratio, R), dtype=np.float32) * mag) for n in processed]
    rt_dev, bt_dev = torch.from_numpy(raw_table).to(dev), torch.from_numpy(bcn_table).to(dev)
    for b in range(B):
        P.raw_write(raw_pages, rt_dev[b:b + 1], [0], to_bf16(raw_k[b])[None], to_bf16(raw_v[b])[None])
        P.beacon_append(bcn_pages, layout, bt_dev[b:b + 1], [0], to_bf16(lat_k[b])[None], to_bf16(lat_v[b])[None])
        P.BeaconPages(bcn_pages, layout).write_sink(int(bcn_table[b, 0]), to_bf16(raw_k[b][0]), to_bf16(raw_v[b][0]))
    torch.cuda.synchronize()
    raw_before, bcn_before = raw_pages.clone(), bcn_pages.clone()

    uk = oracle.round_bf16(rng.standard_normal((kvd, R), dtype=np.float32) * 0.05)
    uv = oracle.round_bf16(rng.standard_normal((kvd, R), dtype=np.float32) * 0.05)
    q = oracle.round_bf16(rng.standard_normal((B, 2, H, D), dtype=np.float32) * mag)
    new_k = oracle.round_bf16(rng.standard_normal((B, kvd), dtype=np.float32) * mag)
    new_v = oracle.round_bf16(rng.standard_normal((B, kvd), dtype=np.float32) * mag)
    new_lat = oracle.round_bf16(rng.standard_normal((B, 2 * R), dtype=np.float32) * mag)
    cos, sin = oracle.rope_tables(D, LLAMA8B['theta'], 16384, LLAMA8B['scaling'])
    cos_t, sin_t = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    layer = vllm.PagedDecodeLayer(raw_pages, bcn_pages, layout, to_bf16(uk), to_bf16(uv), cos_t, sin_t,
                                  window=window, ratio=ratio, sink=sink, max_batch=8, heads=H)
    lat_t = to_bf16(new_lat)
    out = torch.zeros(B, 2, H * D, dtype=torch.bfloat16, device=dev)
    _lib.device_status(clear=True)
    layer(to_bf16(q), to_bf16(new_k), to_bf16(new_v), lat_t[:, :R], lat_t[:, R:],
          torch.from_numpy(seq_lens.astype(np.int32)).to(dev), rt_dev, bt_dev, out)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0

    raw_after, bcn_after = raw_pages.clone(), bcn_pages.clone()
    expect_raw, expect_bcn = raw_before.clone(), bcn_before.clone()
    for b in range(B):
        p = int(processed[b])
        T = p % window
        hist = p // window * (window // ratio)
        inserts = (T + 1) % ratio == 0
        L = 1 + inserts
        qpos = sink + hist + T + T // ratio
        # Oracle inputs: sink, the open window's raw tail, this token (pre-RoPE).
        rk = np.concatenate([raw_k[b][:1], raw_k[b][p - T:p], new_k[b].reshape(1, Hkv, D)])
        rv = np.concatenate([raw_v[b][:1], raw_v[b][p - T:p], new_v[b].reshape(1, Hkv, D)])
        i = np.arange(T)
        kpos = np.concatenate([[0], i + i // ratio + sink + hist, [qpos]])
        lk, lv = lat_k[b][:hist + T // ratio], lat_v[b][:hist + T // ratio]
        if inserts:
            lk = np.concatenate([lk, new_lat[b:b + 1, :R]])
            lv = np.concatenate([lv, new_lat[b:b + 1, R:]])
        ref = oracle.latent_decode_attention(q[b:b + 1, :L], rk[None], rv[None], lk[None], lv[None], uk, uv, cos,
                                             sin, np.array([[qpos, qpos + 1][:L]]), kpos[None], L - 1)['out']
        assert_attention_close(out[b:b + 1, :L], ref)
        # Page bytes this step writes: raw token p, and the Beacon row.
        blk, slot = raw_table[b, p // 16], p % 16
        expect_raw[blk, slot, 0] = to_bf16(new_k[b].reshape(Hkv, D))
        expect_raw[blk, slot, 1] = to_bf16(new_v[b].reshape(Hkv, D))
        if inserts:
            n = hist + T // ratio
            flat = expect_bcn.view(expect_bcn.shape[0], -1)
            page, off = bcn_table[b, n // layout.slots], layout.sink_elements + (n % layout.slots) * 2 * R
            flat[page, off:off + 2 * R] = lat_t[b]
    assert torch.equal(raw_after.view(torch.int16), expect_raw.view(torch.int16))
    assert torch.equal(bcn_after.view(torch.int16), expect_bcn.view(torch.int16))
