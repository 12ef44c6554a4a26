"""GPU parity of the fused latent decode step, RoPE and merge.

``slimkv_latent_decode`` (C ABI) is compared with the oracle's restatement
of ``fa2_decode.decode`` steps 3-8 on identical seeded bf16 inputs at the
Llama-3.1-8B geometry (H=32, Hkv=8, D=128) with small caches, and its cache
writes are checked bit-exactly.  Attention outputs use the parity bar of
norm-wise relative error 2e-3 plus the reference GPU validation's
element-wise tolerance (0.015); RoPE and cache writes must be bit-exact.
"""
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from oracle.decode import latent_decode_attention
from cases import decode_case, LLAMA8B
from gpu_util import assert_attention_close, assert_bits_equal, to_bf16

pytestmark = pytest.mark.gpu

_TABLES = {}


def tables(positions=16384):
    if positions not in _TABLES:
        cos, sin = oracle.rope_tables(128, LLAMA8B['theta'], positions, LLAMA8B['scaling'])
        _TABLES[positions] = (cos, sin, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda())
    return _TABLES[positions]


def run_fused(c, query_len, extra_cap=3, pre=True, fp32=False, stale=0.0, paged=False, wait_limit_ns=0,
              positions=16384, step_plan=False):
    """Stage the caches without this step's entries, run the fused step.

    Cache rows past each sequence's staged length hold ``stale``.  With
    ``paged`` the latent cache lives in Beacon pages (vLLM plugin layout,
    48 slots per page, disjoint shuffled block tables) instead.  With
    ``step_plan`` the work plan is computed first by ``compute_plan`` (as the
    runtime does once per step) and the call starts its attention early.
    """
    from slimkv_b200 import kernels
    cos, sin, cos_t, sin_t = tables(positions)
    B, L, H, D = c['q'].shape
    Hkv, rk, rv = c['kv_heads'], c['rk'], c['rv']
    n_raw, n_lat = c['n_raw'], c['n_lat']
    raw_cap = int(n_raw.max()) + extra_cap
    lat_cap = int(n_lat.max()) + extra_cap
    raw_k = np.full((B, raw_cap, Hkv, D), stale, np.float32)
    raw_v = np.full_like(raw_k, stale)
    lat_k = np.full((B, lat_cap, rk), stale, np.float32)
    lat_v = np.full((B, lat_cap, rv), stale, np.float32)
    new_k = np.zeros((B, Hkv * D), np.float32)
    new_v = np.zeros_like(new_k)
    new_lk = np.zeros((B, rk), np.float32)
    new_lv = np.zeros((B, rv), np.float32)
    for b in range(B):
        r = int(n_raw[b]) - 1                        # row of the current token
        raw_k[b, :r] = oracle.rope_bf16(c['raw_k'][b, :r], cos, sin, c['kpos'][b, :r, None])
        raw_v[b, :r] = c['raw_v'][b, :r]
        new_k[b] = c['raw_k'][b, r].reshape(-1)
        new_v[b] = c['raw_v'][b, r].reshape(-1)
        n = int(n_lat[b]) - (1 if query_len[b] == 2 else 0)
        lat_k[b, :n] = c['lat_k'][b, :n]
        lat_v[b, :n] = c['lat_v'][b, :n]
        if query_len[b] == 2:
            new_lk[b] = c['lat_k'][b, n]
            new_lv[b] = c['lat_v'][b, n]
    # New latents arrive as column views of one down-projection output row.
    new_l = to_bf16(np.concatenate([new_lk, new_lv], axis=-1))
    new_latents = dict(new_lat_k=new_l[:, :rk], new_lat_v=new_l[:, rk:])
    # Native latent layout: one [B, cap, Rk + Rv] buffer, K and V as column views.
    lat = to_bf16(np.concatenate([lat_k, lat_v], axis=-1))
    t = dict(q=to_bf16(c['q']), raw_k_rot=to_bf16(raw_k), raw_v=to_bf16(raw_v), lat_k=lat[..., :rk],
             lat_v=lat[..., rk:], uk=to_bf16(c['uk']), uv=to_bf16(c['uv']), cos=cos_t, sin=sin_t,
             raw_len=torch.tensor(n_raw, dtype=torch.int32, device='cuda'),
             latent_len=torch.tensor(n_lat, dtype=torch.int32, device='cuda'),
             query_len=torch.tensor(query_len, dtype=torch.int32, device='cuda'),
             qpos=torch.tensor(c['qpos'], dtype=torch.int32, device='cuda'),
             new_k=to_bf16(new_k), new_v=to_bf16(new_v), **new_latents,
             out=torch.zeros(B, L, H * D, dtype=torch.float32 if fp32 else torch.bfloat16, device='cuda'))
    if pre:
        t['raw_k_pre'] = torch.zeros_like(t['raw_k_rot'])
    if c['bk'] is not None:
        t['uk_bias'], t['uv_bias'] = to_bf16(c['bk']), to_bf16(c['bv'])
    if paged:
        from slimkv_b200 import pages as P
        layout = P.BeaconPageLayout(192, 4, rk, rv, Hkv * D)
        per_seq = (lat_cap + layout.slots - 1) // layout.slots
        n_pages = B * per_seq + 3
        order = np.random.default_rng(B * lat_cap).permutation(n_pages)[:B * per_seq]
        block_tables = torch.from_numpy(order.reshape(B, per_seq).astype(np.int32)).cuda()
        backing = torch.full((n_pages, layout.page_elements + 8), stale, dtype=torch.bfloat16, device='cuda')
        P.beacon_append(backing, layout, block_tables, np.zeros(B, np.int32), t['lat_k'], t['lat_v'])
        t['lat_pages'] = (backing, layout, block_tables)
        t['lat_k_dense'], t['lat_v_dense'] = t.pop('lat_k'), t.pop('lat_v')
    call = kernels.LatentDecodeCall(**{k: v for k, v in t.items() if not k.endswith('_dense')},
                                    wait_limit_ns=wait_limit_ns)
    if step_plan:
        plan = torch.zeros(call.plan_words(), dtype=torch.int32, device='cuda')
        call.use_plan(plan)
        call.compute_plan(plan)
    call()
    torch.cuda.synchronize()
    if paged:
        # The appended Beacon rows, read back from the pages.
        backing, layout, block_tables = t['lat_pages']
        gk, gv = torch.zeros_like(t['lat_k_dense']), torch.zeros_like(t['lat_v_dense'])
        P.beacon_gather(backing, layout, block_tables, np.full(B, lat_cap, np.int32), gk, gv)
        torch.cuda.synchronize()
        t['lat_k'], t['lat_v'] = gk, gv
    return t


def oracle_rows(c, query_len, positions=16384):
    """Per-row oracle results (each row with its own query length)."""
    cos, sin, _, _ = tables(positions)
    outs = []
    for b in range(c['q'].shape[0]):
        L = int(query_len[b])
        nr, nl = int(c['n_raw'][b]), int(c['n_lat'][b])
        r = latent_decode_attention(c['q'][b:b + 1, :L], c['raw_k'][b:b + 1, :nr], c['raw_v'][b:b + 1, :nr],
                                    c['lat_k'][b:b + 1, :nl], c['lat_v'][b:b + 1, :nl], c['uk'], c['uv'], cos, sin,
                                    c['qpos'][b:b + 1, :L], c['kpos'][b:b + 1, :nr], L - 1,
                                    uk_bias=c['bk'], uv_bias=c['bv'])
        outs.append(r)
    return outs


def check(c, query_len, t, positions=16384):
    refs = oracle_rows(c, query_len, positions)
    errs = []
    for b, r in enumerate(refs):
        L = int(query_len[b])
        errs.append(assert_attention_close(t['out'][b:b + 1, :L], r['out']))
        # Cache writes: rotated / pre-RoPE current key, value, new latents.
        row = int(c['n_raw'][b]) - 1
        assert_bits_equal(t['raw_k_rot'][b, row], r['k_rot'][0, row])
        assert_bits_equal(t['raw_v'][b, row], c['raw_v'][b, row])
        if 'raw_k_pre' in t:
            assert_bits_equal(t['raw_k_pre'][b, row], c['raw_k'][b, row])
        if L == 2:
            n = int(c['n_lat'][b]) - 1
            assert_bits_equal(t['lat_k'][b, n], c['lat_k'][b, n])
            assert_bits_equal(t['lat_v'][b, n], c['lat_v'][b, n])
    return max(errs)


def test_a_wait_that_runs_out_reports_timeout_and_the_context_stays_usable():
    """Every pipeline wait of the attention kernel is bounded.  With a bound
    of 1 ns the waits run out while copies are still in flight (the producer
    finds its rings full at once): the kernel must set
    SLIMKV_DEVICE_TIMEOUT, drain its copies and MMAs, free its tensor memory
    and return — no fault, no hang — and the next call, with the default
    bound, must match the oracle on the same context."""
    from slimkv_b200 import _lib
    c = decode_case(91, batch=3, length=2, history=2048, tail=300, ragged=True)
    query_len = np.array([2, 1, 2])
    _lib.device_status(clear=True)
    run_fused(c, query_len, wait_limit_ns=1)
    assert _lib.device_status(clear=True) & _lib.DEVICE_TIMEOUT
    t = run_fused(c, query_len)
    assert _lib.device_status(clear=True) == 0
    check(c, query_len, t)


@pytest.mark.parametrize('stale', [float('nan'), float('inf')])
def test_stale_cache_rows_past_the_length_are_ignored(stale):
    """Rows past each length may hold anything (NaN, inf) and must not leak."""
    c = decode_case(71, batch=3, length=2, history=300, tail=39, ragged=True)
    query_len = np.array([2, 1, 2])
    for fp32 in (False, True):
        t = run_fused(c, query_len, extra_cap=200, fp32=fp32, stale=stale)
        assert torch.isfinite(t['out'].float()).all()
        check(c, query_len, t)


@pytest.mark.parametrize('length,history,tail,bias', [(1, 300, 37, False), (2, 500, 39, True), (2, 129, 1023, False)])
def test_fused_decode_reads_the_latent_cache_from_pages(length, history, tail, bias):
    """The latent branch streams Beacon pages through block tables; the
    inserted Beacon row is appended into its page."""
    c = decode_case(300 + history, batch=3, length=length, history=history, tail=tail, bias=bias, ragged=True)
    query_len = np.full(3, length)
    check(c, query_len, run_fused(c, query_len, paged=True))
    check(c, query_len, run_fused(c, query_len, paged=True, fp32=True, stale=float('nan')))


@pytest.mark.parametrize('length,history,tail,rank,bias,ragged', [
    (1, 300, 37, 320, False, False),
    (2, 300, 39, 320, False, False),
    (1, 1024, 0, 320, False, False),
    (2, 200, 3, 320, True, False),
    (1, 513, 700, 160, False, True),
    (2, 129, 1023, 320, False, True),
    (1, 64, 5, 256, True, True),
    (2, 2048, 511, 320, False, True),
])
def test_fused_decode_matches_oracle(length, history, tail, rank, bias, ragged):
    c = decode_case(100 + history + tail, batch=3, length=length, history=history, tail=tail, rk=rank, rv=rank,
                    bias=bias, ragged=ragged)
    query_len = np.full(3, length)
    check(c, query_len, run_fused(c, query_len))
    check(c, query_len, run_fused(c, query_len, fp32=True))


@pytest.mark.parametrize('length,heads,rank,ragged', [
    (1, 40, 512, True), (2, 40, 512, False), (2, 32, 384, True), (1, 40, 320, False), (2, 40, 160, True),
    (2, 40, 384, True), (1, 40, 256, True)])
def test_qwen_geometry_and_wide_latents(length, heads, rank, ragged):
    """40 query heads over 8 KV heads (Qwen2.5-14B) and latent ranks up to 512
    (r2), with up-projection biases.  An even number of 64-column V chunks
    (ranks 256, 384, 512) runs the tensor-memory kernel's 40-head layout (one
    query per latent CTA, V chunks cycling through a 4-slot ring); odd ones
    (160, 320) and 32 heads above rank 320 the split-KV route."""
    c = decode_case(500 + rank + length, batch=3, length=length, history=700, tail=300, heads=heads, kv_heads=8,
                    rk=rank, rv=rank, bias=True, ragged=ragged)
    query_len = np.full(3, length)
    check(c, query_len, run_fused(c, query_len))
    check(c, query_len, run_fused(c, query_len, fp32=True))


@pytest.mark.parametrize('paged', [False, True])
def test_wide_layout_mixed_queries_stale_rows_and_early_start(paged):
    """The 40-head layout at rank 512: sequences with and without a Beacon in
    one batch (each query its own latent segment, the merge combining both
    segments' pieces), NaN in the cache rows past every length (cleared by the
    P.V warp in the partial last tile), dense or paged latents; a step plan
    with the early attention start gives the same bits."""
    c = decode_case(2140, batch=7, length=2, history=900, tail=300, heads=40, kv_heads=8, rk=512, rv=512,
                    bias=True, ragged=True)
    query_len = np.array([2, 1, 1, 2, 1, 2, 2])
    c['n_lat'] = c['n_lat'] - (query_len == 1)
    a = run_fused(c, query_len, extra_cap=150, fp32=True, paged=paged, stale=float('nan'))
    assert torch.isfinite(a['out']).all()
    check(c, query_len, a)
    b = run_fused(c, query_len, extra_cap=150, fp32=True, paged=paged, stale=float('nan'), step_plan=True)
    for key in ('out', 'lat_k', 'lat_v'):
        x, y = a[key], b[key]
        assert torch.equal(torch.nan_to_num(x.float(), nan=7.0), torch.nan_to_num(y.float(), nan=7.0)), key


@pytest.mark.parametrize('paged', [False, True])
def test_large_ragged_batch_splits_every_sequence_by_its_length(paged):
    """More sequences than SMs / 3 with latent lengths from 1 to ~4.6k rows:
    each sequence gets its own number of bounded splits (the work list the
    prologue writes), and the merge combines exactly those."""
    c = decode_case(77, batch=60, length=2, history=4096, tail=900, rk=160, rv=160, ragged=True)
    query_len = np.array([1 + (b % 3 == 0) for b in range(60)])
    c['n_lat'] = c['n_lat'] - (query_len == 1)
    c['n_lat'][3] = 1                                  # only this step's Beacon
    c['n_lat'][4] = 0 if query_len[4] == 1 else 1      # no latent at all when no Beacon is inserted
    c['n_lat'][5] = 129                                # one row past a tile
    check(c, query_len, run_fused(c, query_len, paged=paged))


@pytest.mark.parametrize('length', [1, 2])
def test_paged_decode_is_bit_identical_to_dense(length):
    """Same inputs, latent cache in Beacon pages or dense: the same bits."""
    c = decode_case(5, batch=3, length=length, history=2176, tail=1000, rk=160, rv=160, ratio=8)
    query_len = np.full(3, length)
    dense = run_fused(c, query_len, fp32=True)
    paged = run_fused(c, query_len, fp32=True, paged=True)
    assert torch.equal(dense['out'], paged['out'])


@pytest.mark.parametrize('paged', [False, True])
def test_step_plan_and_early_attention_are_bit_identical(paged):
    """A plan computed before the call (the runtime's one per step) and the
    attention launch that overlaps the prologue give the same outputs and
    cache writes, bit for bit, as per-call planning."""
    c = decode_case(2101, batch=9, length=2, history=700, tail=300, ragged=True, bias=True)
    query_len = np.array([2, 1, 2, 1, 1, 2, 1, 2, 1])
    a = run_fused(c, query_len, fp32=True, paged=paged)
    b = run_fused(c, query_len, fp32=True, paged=paged, step_plan=True)
    for key in ('out', 'raw_k_rot', 'raw_v', 'raw_k_pre', 'lat_k', 'lat_v'):
        assert torch.equal(a[key].view(torch.int32) if a[key].dtype == torch.float32 else a[key].view(torch.int16),
                           b[key].view(torch.int32) if b[key].dtype == torch.float32 else b[key].view(torch.int16)), key
    check(c, query_len, b)


def test_mixed_query_lengths_in_one_batch():
    """Only some rows insert a Beacon this step (per-row query_len)."""
    c = decode_case(7, batch=4, length=2, history=400, tail=19)
    query_len = np.array([2, 1, 2, 1])
    c['n_lat'] = c['n_lat'] - (query_len == 1)           # rows without a Beacon have one latent fewer
    check(c, query_len, run_fused(c, query_len))
    check(c, query_len, run_fused(c, query_len, fp32=True))


def test_distinct_key_and_value_ranks():
    c = decode_case(9, batch=2, length=2, history=300, tail=11, rk=160, rv=192)
    query_len = np.full(2, 2)
    check(c, query_len, run_fused(c, query_len))


def test_no_history_only_window_latents():
    """First open window: no completed history, a handful of window latents."""
    c = decode_case(11, batch=2, length=1, history=0, tail=12, sink=1)
    query_len = np.full(2, 1)
    check(c, query_len, run_fused(c, query_len))


def test_rope_decode_is_bit_exact_against_reference_bits():
    from slimkv_b200 import kernels
    golden = np.load(Path(__file__).parent / 'golden' / 'reference_golden.npz')
    cos, sin = oracle.rope_tables(128, LLAMA8B['theta'], LLAMA8B['max_positions'], LLAMA8B['scaling'])
    cos_t, sin_t = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    q = torch.from_numpy(golden['rope_q_in']).cuda().view(torch.bfloat16)       # [2, 32, 2, 128]
    k = torch.from_numpy(golden['rope_k_in']).cuda().view(torch.bfloat16)       # [2, 8, 70, 128]
    pos = torch.from_numpy(golden['rope_pos']).cuda()                          # [2, 70]
    # Express the reference's free positions through the decode contract:
    # no sink, raw indices = positions[:-1] for row 0 (history 0).
    qo, _ = kernels.rope_decode(q, k, cos_t, sin_t, pos[:, -2:].contiguous(), pos[0, :-1], 0, 0)
    assert np.array_equal(qo.view(torch.int16).cpu().numpy(), golden['rope_q_out'])
    _, ko = kernels.rope_decode(q[:1], k[:1], cos_t, sin_t, pos[:1, -1:].expand(1, 2).contiguous(), pos[0, :-1], 0, 0)
    assert np.array_equal(ko.view(torch.int16).cpu().numpy(), golden['rope_k_out'][:1])


def test_rope_decode_with_sinks_and_history_matches_oracle():
    from slimkv_b200 import kernels
    cos, sin, cos_t, sin_t = tables()
    rng = np.random.default_rng(5)
    B, H, Hkv, Q, K, S, hist = 2, 32, 8, 2, 51, 4, 384
    q = oracle.round_bf16(rng.standard_normal((B, H, Q, 128), dtype=np.float32) * 2)
    k = oracle.round_bf16(rng.standard_normal((B, Hkv, K, 128), dtype=np.float32) * 2)
    raw_idx = np.arange(K - S - 1) * 2
    first = hist + S + 2 * raw_idx.size
    qpos = np.tile(np.arange(first, first + Q), (B, 1))
    qo, ko = kernels.rope_decode(to_bf16(q), to_bf16(k), cos_t, sin_t, torch.from_numpy(qpos).cuda(),
                                 torch.from_numpy(raw_idx).cuda(), S, hist)
    kpos = oracle.raw_key_positions(S, raw_idx, hist, first)
    assert_bits_equal(qo, oracle.rope_bf16(q, cos, sin, qpos[:, None, :]))
    assert_bits_equal(ko, oracle.rope_bf16(k, cos, sin, np.tile(kpos, (B, 1))[:, None, :]))


def test_merge_matches_oracle():
    from slimkv_b200 import kernels
    rng = np.random.default_rng(21)
    raw = oracle.round_bf16(rng.standard_normal((2, 32, 2, 128), dtype=np.float32))
    lat = oracle.round_bf16(rng.standard_normal((2, 32, 2, 128), dtype=np.float32))
    rl = rng.standard_normal((2, 32, 2), dtype=np.float32) * 4
    ll = rng.standard_normal((2, 32, 2), dtype=np.float32) * 4
    ll[..., 0] = -np.inf
    out = kernels.merge(to_bf16(raw), torch.from_numpy(rl).cuda(), to_bf16(lat), torch.from_numpy(ll).cuda())
    ref = oracle.merge_attention(raw, rl, lat, ll)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=1e-3, rtol=8e-3)
    assert_bits_equal(out[:, :, 0], raw[:, :, 0])


def run_sharded(c, query_len, starts, paged=False):
    """Sequence split emulated on one GPU.

    The caches are staged and this step's entries appended by one whole
    fused step (``run_fused``); then shard ``k`` attends over latent rows
    ``[starts[k], starts[k+1])`` of every sequence (the last shard: to the
    sequence's end, with the raw branch and the causal Beacon row; the
    others: ``latent_shard`` and no raw keys), each writing its output and
    log-sum-exp, and ``merge_partials`` combines the N partials as the
    all-gather of a real split would hand them over.  Returns the whole
    step's caches/outputs, the merged output and LSE, and the partials.
    """
    from slimkv_b200 import kernels
    t = run_fused(c, query_len, fp32=True, paged=paged)
    _, _, cos_t, sin_t = tables()
    B, L, H, D = c['q'].shape
    N = len(starts)
    common = dict(q=t['q'], raw_k_rot=t['raw_k_rot'], raw_v=t['raw_v'], uk=t['uk'], uv=t['uv'], cos=cos_t,
                  sin=sin_t, qpos=t['qpos'], query_len=t['query_len'], uk_bias=t.get('uk_bias'),
                  uv_bias=t.get('uv_bias'))
    outs = torch.zeros(N, B, L, H * D, dtype=torch.float32, device='cuda')
    lses = torch.full((N, B, L, H), float('-inf'), dtype=torch.float32, device='cuda')
    for k in range(N):
        s, last = starts[k], k == N - 1
        e = None if last else starts[k + 1]
        lat_len = c['n_lat'] - s if last else np.full(B, e - s)
        if paged:
            backing, layout, block_tables = t['lat_pages']
            assert s % layout.slots == 0 and (last or e % layout.slots == 0)
            lat = dict(lat_pages=(backing, layout,
                                  block_tables[:, s // layout.slots:None if last else e // layout.slots]))
        else:
            lat = dict(lat_k=t['lat_k'][:, s:e], lat_v=t['lat_v'][:, s:e])
        kernels.latent_decode(**common, **lat, latent_len=torch.tensor(lat_len, dtype=torch.int32, device='cuda'),
                              raw_len=t['raw_len'] if last else torch.zeros(B, dtype=torch.int32, device='cuda'),
                              out=outs[k], out_lse=lses[k], latent_shard=not last)
    merged = torch.empty(B, L, H * D, dtype=torch.float32, device='cuda')
    merged_lse = torch.empty(B, L, H, dtype=torch.float32, device='cuda')
    kernels.merge_partials(outs.view(N, B * L * H, D), lses.view(N, B * L * H), merged, merged_lse)
    torch.cuda.synchronize()
    return t, merged, merged_lse, outs, lses


def check_sharded(c, query_len, starts, paged=False):
    t, merged, merged_lse, _, _ = run_sharded(c, query_len, starts, paged)
    _, whole, whole_lse, _, _ = run_sharded(c, query_len, [0], paged)
    for b, r in enumerate(oracle_rows(c, query_len)):
        L = int(query_len[b])
        assert_attention_close(merged[b:b + 1, :L], r['out'])
        lse = np.logaddexp(r['raw_lse'], r['latent_lse'])[0].T            # [L, H]
        for got in (merged_lse, whole_lse):
            np.testing.assert_allclose(got[b, :L].cpu().numpy(), lse, atol=2e-3, rtol=1e-4)
        # The merge of shards is the same attention as the unsplit call, up
        # to the rounding of probabilities against a different running max.
        a, w = merged[b, :L].double(), whole[b, :L].double()
        assert ((a - w).norm() / w.norm()).item() < 1e-3
        assert torch.equal(whole[b, :L], t['out'][b, :L])


@pytest.mark.parametrize('paged', [False, True])
@pytest.mark.parametrize('starts', [[0, 384], [0, 96, 384, 720]])
def test_sequence_split_shards_merge_to_the_whole_step(starts, paged):
    """Latent shards of each sequence (the last one with the raw branch and
    this step's Beacon) merged with the N-part LSE merge equal the unsplit
    fused step and the oracle; rows that insert a Beacon and rows that do not
    are mixed, with up-projection biases."""
    c = decode_case(41, batch=3, length=2, history=1500, tail=300, bias=True, ragged=True)
    query_len = np.array([2, 1, 2])
    c['n_lat'] = c['n_lat'] - (query_len == 1)
    check_sharded(c, query_len, starts, paged)


@pytest.mark.parametrize('length', [1, 2])
def test_sequence_split_qwen_geometry(length):
    """40 heads, rank 512 (the split-KV route with 32-key tiles): shards of a
    long latent history merge to the unsplit step."""
    c = decode_case(43, batch=2, length=length, history=2000, tail=200, heads=40, rk=512, rv=512, bias=True)
    query_len = np.full(2, length)
    check_sharded(c, query_len, [0, 640, 1280])


@pytest.mark.parametrize('parts,dim,out_fp32', [(1, 128, True), (3, 128, False), (8, 96, True), (40, 320, True),
                                                (64, 64, False)])
def test_merge_partials_matches_numpy(parts, dim, out_fp32):
    """The N-part LSE merge against a float64 numpy restatement, with parts
    and whole rows that have no keys (-inf)."""
    from slimkv_b200 import kernels
    rng = np.random.default_rng(parts * 1000 + dim)
    rows = 37
    out = rng.standard_normal((parts, rows, dim)).astype(np.float32)
    lse = (rng.standard_normal((parts, rows)) * 6).astype(np.float32)
    lse[rng.random((parts, rows)) < 0.3] = -np.inf
    lse[:, 5] = -np.inf                                  # a row without keys anywhere
    m = lse.max(0)
    finite = np.isfinite(m)
    total = np.where(finite, np.log(np.exp(lse.astype(np.float64) - np.where(finite, m, 0)).sum(0)) + m, -np.inf)
    w = np.where(np.isfinite(lse), np.exp(lse - np.where(finite, total, 0)), 0.0)
    want = (w[..., None] * out).sum(0)
    # Part strides wider than a part, as in an all-gather of [outputs | lses].
    packed = np.zeros((parts, rows * dim + (rows + 3) // 4 * 4 + 4), np.float32)
    packed[:, :rows * dim] = out.reshape(parts, -1)
    packed[:, rows * dim:rows * dim + rows] = lse
    dev = torch.from_numpy(packed).cuda()
    got = torch.empty(rows, dim, dtype=torch.float32 if out_fp32 else torch.bfloat16, device='cuda')
    got_lse = torch.empty(rows, dtype=torch.float32, device='cuda')
    kernels.merge_partials(dev[:, :rows * dim].view(parts, rows, dim), dev[:, rows * dim:rows * dim + rows], got,
                           got_lse)
    torch.cuda.synchronize()
    tol = 1e-5 if out_fp32 else 8e-3
    np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=tol, atol=tol)
    np.testing.assert_allclose(got_lse.cpu().numpy(), total, rtol=1e-6, atol=1e-5)
    assert np.all(got.float().cpu().numpy()[5] == 0)
