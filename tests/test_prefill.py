"""Prefill window compression and Beacon append.

CPU: the oracle against the reference's own outputs (``tests/golden/
make_golden.py:gen_prefill``: ``qkv_proj_with_beacon`` + ``_incremental_cache``
on a bf16 module, ``_apply_rotary_with_beacon``) and the host-side argument
checks of the C ABI.  GPU: ``slimkv_window_project`` / ``slimkv_prefill_rope``
against the golden outputs and the oracle - row roles, index lists, page and
cache bytes bit-exact; projections within one bf16 ulp of the correctly
rounded result (the reference's own bf16 GEMMs differ from it the same way),
or within fp32-accumulation noise where a dot product cancels.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from oracle.bf16 import bf16_bits, from_bf16_bits
from oracle.pages import BeaconPageLayout as OracleLayout

GOLD = np.load(Path(__file__).parent / 'golden' / 'prefill_golden.npz')
TAGS = ['first', 'second', 'nobeacon', 'long']
HEADS, KV_HEADS, HEAD_DIM = 4, 2, 32


def _f(key):
    return from_bf16_bits(GOLD[key].view(np.uint16))


def _weights():
    w = {}
    for name in ['q', 'k', 'v', 'bq', 'k_down', 'v_down', 'k_up', 'v_up']:
        w[name] = _f(f'prefill_w_{name}')
        bias = f'prefill_w_{name}_bias'
        if bias in GOLD:
            w[name + '_bias'] = _f(bias)
    return w


def ulps(a_bits, b_bits):
    """Distance in bf16 units in the last place between two bit arrays."""
    def ordered(x):
        x = np.asarray(x, np.uint16).astype(np.int32)
        return np.where(x & 0x8000, 0x8000 - (x & 0x7FFF), x + 0x8000)
    return np.abs(ordered(a_bits) - ordered(b_bits))


def assert_within_one_ulp(got_bits, want_bits, max_frac=0.05, atol_frac=1e-5):
    """Every element within one bf16 ulp of the correctly rounded value, or -
    where the dot product cancels to a value far below its terms - within an
    absolute ``atol_frac * max|want|`` (fp32 accumulation over K terms);
    at most ``max_frac`` of the elements may differ at all."""
    d = ulps(got_bits, want_bits)
    got, want = from_bf16_bits(got_bits), from_bf16_bits(want_bits)
    atol = atol_frac * np.abs(want).max()
    far = (d > 1) & (np.abs(got - want) > atol)
    assert not far.any(), \
        f'{far.sum()} elements beyond one ulp and {atol:.2e}, first at {np.argwhere(far)[:3].tolist()}'
    assert (d > 0).mean() <= max_frac, f'{(d > 0).mean():.3%} of elements differ'


# ---- oracle vs the reference (CPU) -----------------------------------------

@pytest.mark.parametrize('tag', TAGS)
def test_oracle_metadata_matches_reference(tag):
    roles = GOLD[f'prefill_{tag}_roles']
    n = GOLD[f'prefill_{tag}_hidden'].shape[1]
    raw, beacon, replicas = oracle.prefill_metadata(roles, n)
    assert np.array_equal(raw, GOLD[f'prefill_{tag}_raw_indices'])
    assert not replicas
    assert len(raw) + len(beacon) == n


@pytest.mark.parametrize('tag', TAGS)
def test_oracle_projection_matches_reference(tag):
    r = oracle.project_with_beacon(_f(f'prefill_{tag}_hidden'), GOLD[f'prefill_{tag}_roles'], _weights())
    for name in ['query', 'key', 'value']:
        assert_within_one_ulp(bf16_bits(r[name]), GOLD[f'prefill_{tag}_{name}'].view(np.uint16))
    if f'prefill_{tag}_key_latents' in GOLD:
        assert_within_one_ulp(bf16_bits(r['key_latent']), GOLD[f'prefill_{tag}_key_latents'].view(np.uint16)[:, 0])
        assert_within_one_ulp(bf16_bits(r['value_latent']),
                              GOLD[f'prefill_{tag}_value_latents'].view(np.uint16)[:, 0])
    else:
        assert r['key_latent'].shape[1] == 0


@pytest.mark.parametrize('tag', ['a', 'b', 'c'])
def test_oracle_prefill_rope_matches_reference_bits(tag):
    p = f'prope_{tag}_'
    qo, ko = oracle.prefill_rope(_f(p + 'q'), _f(p + 'k'), GOLD['prope_cos'], GOLD['prope_sin'], GOLD[p + 'pos'],
                                 GOLD[p + 'roles'], int(GOLD[p + 'sink']))
    assert np.array_equal(bf16_bits(qo), GOLD[p + 'qo'].view(np.uint16))
    assert np.array_equal(bf16_bits(ko), GOLD[p + 'ko'].view(np.uint16))


def test_oracle_rejects_replicas():
    with pytest.raises(ValueError, match='replica'):
        oracle.project_with_beacon(np.zeros((1, 5, 8), np.float32), np.array([0, 0, 0, 0, 2]), _weights())


# ---- host-side checks (no GPU) ---------------------------------------------

def test_window_project_rejects_bad_arguments_before_launch():
    from slimkv_b200 import _lib
    lib = _lib.load()

    def args(**kw):
        a = _lib.WindowProjectArgs()
        a.batch, a.rows, a.hidden = 1, 8, 64
        a.heads, a.kv_heads, a.head_dim, a.rank_k, a.rank_v = 4, 2, 16, 8, 8
        a.hidden_states, a.hidden_stride_batch, a.hidden_stride_row = 1 << 20, 512, 64
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    for kw, code in [(dict(raw_count=9), 1), (dict(hidden=60), 3), (dict(hidden_stride_row=65), 3),
                     (dict(raw_count=2), 1), (dict(heads=0), 1),
                     (dict(raw_key_cache=1 << 20, raw_start=1 << 20), 1),
                     (dict(write_sink=1, raw_start=1 << 20), 1)]:
        assert lib.slimkv_window_project(ctypes.byref(args(**kw)), None) == code, kw
    assert lib.slimkv_window_project(ctypes.byref(args(batch=0)), None) == 0
    st = (ctypes.c_int64 * 3)(0, 0, 0)
    assert lib.slimkv_prefill_rope(1, st, 1, st, 1, 1, 16, 1, 4, None, 0, 0, 1, 4, 2, 5, 4, 32, 1, st, 1, st,
                                   None) == 1    # more queries than keys


def test_prefill_wrappers_follow_reference_contracts():
    from slimkv_b200 import prefill
    roles = torch.tensor([0, 0, 0, 0, 2])
    meta = prefill.metadata_from_roles(roles, 5)
    assert meta.replicas and meta.beacon_indices.tolist() == [4]
    with pytest.raises(NotImplementedError, match='replica'):
        prefill.project_window(None, torch.zeros(1, 5, 8), meta, 1, 1, 8)
    # CPU tensors are not the fused kernel's inputs: the reference returns None.
    rope = type('R', (), {'cos_cached': torch.zeros(8, 8), 'sin_cached': torch.zeros(8, 8)})()
    q = torch.zeros(1, 2, 3, 8, dtype=torch.bfloat16)
    assert prefill.fused_prefill_rope(q, q, rope, meta, 0) is None

    class Cfg:
        beacon_headwise_up_proj = True

    with pytest.raises(NotImplementedError, match='headwise'):
        prefill.BeaconProjectionWeights.from_attention(type('A', (), {'config': Cfg()})())


# ---- GPU ----------------------------------------------------------------------

def _gpu_weights():
    from slimkv_b200.prefill import BeaconProjectionWeights
    w = {k: torch.from_numpy(v).to('cuda', torch.bfloat16) for k, v in _weights().items()}
    return BeaconProjectionWeights(**w)


def _bits(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize('tag', TAGS)
def test_window_projection_matches_reference(tag):
    from slimkv_b200 import _lib, prefill
    _lib.device_status(clear=True)
    hidden = torch.from_numpy(GOLD[f'prefill_{tag}_hidden']).view(torch.bfloat16).cuda()
    roles = torch.from_numpy(GOLD[f'prefill_{tag}_roles']).cuda()
    meta = prefill.metadata_from_roles(roles, hidden.shape[1])
    assert torch.equal(meta.raw_indices.cpu(), torch.from_numpy(GOLD[f'prefill_{tag}_raw_indices']))
    r = prefill.project_window(_gpu_weights(), hidden, meta, HEADS, KV_HEADS, HEAD_DIM)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    for name in ['query', 'key', 'value']:
        assert_within_one_ulp(_bits(r[name]), GOLD[f'prefill_{tag}_{name}'].view(np.uint16))
    if f'prefill_{tag}_key_latents' in GOLD:
        assert_within_one_ulp(_bits(r['key_latents']), GOLD[f'prefill_{tag}_key_latents'].view(np.uint16))
        assert_within_one_ulp(_bits(r['value_latents']), GOLD[f'prefill_{tag}_value_latents'].view(np.uint16))


def _llama_case(seed, batch, raw_tokens, remainder, ratio=4, rank_k=320, rank_v=320, bias=False):
    """Llama-3.1-8B layer geometry, random N(0, 0.02) weights, N(0, 1) hidden."""
    g = torch.Generator(device='cuda')
    g.manual_seed(seed)

    def w(*shape, std=0.02):
        return (torch.randn(*shape, generator=g, device='cuda') * std).to(torch.bfloat16)

    from slimkv_b200.prefill import BeaconProjectionWeights
    H, qd, kvd = 4096, 4096, 1024
    weights = BeaconProjectionWeights(
        q=w(qd, H), k=w(kvd, H), v=w(kvd, H), bq=w(qd, H), k_down=w(rank_k, H), v_down=w(rank_v, H),
        k_up=w(kvd, rank_k, std=0.05), v_up=w(kvd, rank_v, std=0.05),
        q_bias=w(qd, std=0.5) if bias else None, k_bias=w(kvd, std=0.5) if bias else None,
        v_bias=w(kvd, std=0.5) if bias else None, bq_bias=w(qd, std=0.5) if bias else None,
        k_up_bias=w(kvd, std=0.5) if bias else None, v_up_bias=w(kvd, std=0.5) if bias else None)
    roles, _, _ = oracle.interleave_roles(raw_tokens, remainder, ratio)
    hidden = w(batch, len(roles), H, std=1.0)
    return weights, hidden, roles


def _np_weights(W):
    d = {}
    for name in ['q', 'k', 'v', 'bq', 'k_down', 'v_down', 'k_up', 'v_up']:
        d[name] = getattr(W, name).float().cpu().numpy()
        b = getattr(W, name + '_bias', None)
        if b is not None:
            d[name + '_bias'] = b.float().cpu().numpy()
    return d


@pytest.mark.gpu
@pytest.mark.parametrize('raw_tokens,remainder,bias', [(120, 0, False), (131, 3, True)])
def test_window_projection_llama_geometry_matches_oracle(raw_tokens, remainder, bias):
    from slimkv_b200 import _lib, prefill
    W, hidden, roles = _llama_case(3 + raw_tokens, 2, raw_tokens, remainder, bias=bias)
    meta = prefill.metadata_from_roles(torch.from_numpy(roles).cuda(), len(roles))
    _lib.device_status(clear=True)
    r = prefill.project_window(W, hidden, meta, 32, 8, 128)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    h, w = hidden.float().cpu().numpy(), _np_weights(W)
    want = oracle.project_with_beacon(h, roles, w)
    assert_within_one_ulp(_bits(r['key_latents'][:, 0]), bf16_bits(want['key_latent']))
    assert_within_one_ulp(_bits(r['value_latents'][:, 0]), bf16_bits(want['value_latent']))
    # Beacon keys/values are up-projected from the kernel's own bf16 latents (a
    # one-ulp latent difference moves them by more than one ulp).
    lat = (r['key_latents'][:, 0].float().cpu().numpy(), r['value_latents'][:, 0].float().cpu().numpy())
    want = oracle.project_with_beacon(h, roles, w, latents=lat)
    for name in ['query', 'key', 'value']:
        assert_within_one_ulp(_bits(r[name]), bf16_bits(want[name]))


@pytest.mark.gpu
@pytest.mark.parametrize('query', [True, False])
def test_split_reduction_matches_single_cta_deterministically(query):
    """Few output tiles: each reduction is split over several CTAs whose fp32
    partial tiles are summed in slice order by a second kernel; results stay
    within one ulp of the unsplit launch and repeat bit for bit."""
    from slimkv_b200 import _lib, prefill
    W, hidden, roles = _llama_case(23, 1, 96, 1, bias=True)
    meta = prefill.metadata_from_roles(torch.from_numpy(roles).cuda(), len(roles))
    _lib.device_status(clear=True)
    split = prefill.project_window(W, hidden, meta, 32, 8, 128, query=query)
    single = prefill.project_window(W, hidden, meta, 32, 8, 128, query=query, split=False)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    names = ['key', 'value', 'key_latents', 'value_latents'] + (['query'] if query else [])
    raw = meta.raw_indices
    for name in names:
        # Beacon keys/values are up-projected from latents that may differ in
        # the last bit between the two summation orders: compare raw rows.
        a, b = (split[name][:, raw], single[name][:, raw]) if name in ('key', 'value') else (split[name], single[name])
        assert_within_one_ulp(_bits(a), _bits(b))
    for _ in range(3):
        again = prefill.project_window(W, hidden, meta, 32, 8, 128, query=query)
        torch.cuda.synchronize()
        for name in names:
            assert torch.equal(again[name], split[name])


@pytest.mark.gpu
def test_window_append_writes_pages_like_flush_memory():
    """Latents into Beacon pages, kept raw rows into raw pages and the first raw
    token into the root page's sink: bytes equal to the oracle's flush of the
    kernel's own dense outputs."""
    from slimkv_b200 import _lib, prefill
    from slimkv_b200.pages import BeaconPageLayout, BeaconPages, RawPages
    W, hidden, roles = _llama_case(11, 3, 200, 0, rank_k=320, rank_v=320)
    B, n = hidden.shape[:2]
    meta = prefill.metadata_from_roles(torch.from_numpy(roles).cuda(), n)
    layout = BeaconPageLayout(192, 4, 320, 320, 1024)
    rng = np.random.default_rng(3)
    n_pages, per_seq = 24, 6
    btab = rng.permutation(n_pages)[:B * per_seq].reshape(B, per_seq).astype(np.int32)
    rtab = rng.permutation(96)[:B * 26].reshape(B, 26).astype(np.int32)
    bpages = torch.zeros(n_pages, layout.page_elements, dtype=torch.bfloat16, device='cuda')
    rpages = torch.zeros(96, 16, 2, 8, 128, dtype=torch.bfloat16, device='cuda')
    lat_start = np.array([0, 48, 5], np.int32)
    raw_start = np.array([0, 192, 20], np.int32)
    raw_first = 150
    _lib.device_status(clear=True)
    r = prefill.project_window(W, hidden, meta, 32, 8, 128, query=False, lat_start=lat_start,
                               beacon=(BeaconPages(bpages, layout), btab), raw_start=raw_start, raw_first=raw_first,
                               raw=(RawPages(rpages), rtab), write_sink=True)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    key, value = r['key'].float().cpu().numpy(), r['value'].float().cpu().numpy()
    lk, lv = r['key_latents'][:, 0].float().cpu().numpy(), r['value_latents'][:, 0].float().cpu().numpy()
    want_b = np.zeros((n_pages, layout.page_elements), np.float32)
    want_r = np.zeros((96, 16, 2, 1024), np.float32)
    ol = OracleLayout(192, 4, 320, 320, 1024)
    raw_idx = meta.raw_indices.cpu().numpy()
    for b in range(B):
        oracle.flush_chunk(want_b, want_r, btab[b], rtab[b], ol, 16, key[b], value[b], lk[b], lv[b], raw_idx,
                           int(lat_start[b]), int(raw_start[b]), raw_first, True)
    assert np.array_equal(_bits(bpages), bf16_bits(want_b))
    assert np.array_equal(_bits(rpages).reshape(96, 16, 2, 1024), bf16_bits(want_r))
    # the sink exists only for the sequence whose chunk starts at raw position 0
    assert (want_b[btab[0][0], :2048] != 0).any() and not (want_b[btab[1][0], :2048] != 0).any()


@pytest.mark.gpu
def test_window_append_into_dense_caches_at_cursors():
    """HF-style dense caches: latents at lat_start[b] + j of the latent cache
    and raw rows at raw_start[b] + i of the raw cache; the up-projected Beacon
    keys read the latents back from the cache rows just written."""
    from slimkv_b200 import _lib, prefill
    W, hidden, roles = _llama_case(17, 2, 64, 2)
    B, n = hidden.shape[:2]
    meta = prefill.metadata_from_roles(torch.from_numpy(roles).cuda(), n)
    lat = torch.full((B, 80, 640), -7.0, dtype=torch.bfloat16, device='cuda')
    rk = torch.full((B, 96, 8, 128), -7.0, dtype=torch.bfloat16, device='cuda')
    rv = torch.full_like(rk, -7.0)
    lat_start, raw_start = [3, 40], [10, 0]
    _lib.device_status(clear=True)
    r = prefill.project_window(W, hidden, meta, 32, 8, 128, latents=False, latent_cache=(lat[..., :320],
                               lat[..., 320:]), lat_start=lat_start, raw_start=raw_start, raw_cache=(rk, rv))
    ref = prefill.project_window(W, hidden, meta, 32, 8, 128)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    nb, raw_idx = meta.beacon_indices.numel(), meta.raw_indices
    for b in range(B):
        s = lat_start[b]
        assert torch.equal(lat[b, s:s + nb, :320], ref['key_latents'][b, 0])
        assert torch.equal(lat[b, s:s + nb, 320:], ref['value_latents'][b, 0])
        assert (lat[b, :s] == -7).all() and (lat[b, s + nb:] == -7).all()
        t = raw_start[b]
        assert torch.equal(rk[b, t:t + raw_idx.numel()].flatten(1), ref['key'][b, raw_idx])
        assert torch.equal(rv[b, t:t + raw_idx.numel()].flatten(1), ref['value'][b, raw_idx])
        assert (rk[b, t + raw_idx.numel():] == -7).all()
    for name in ['query', 'key', 'value']:
        assert torch.equal(r[name], ref[name])


@pytest.mark.gpu
def test_window_projection_reports_bad_rows_without_writing():
    from slimkv_b200 import _lib, prefill
    W, hidden, roles = _llama_case(5, 1, 8, 0)
    meta = prefill.metadata_from_roles(torch.from_numpy(roles).cuda(), hidden.shape[1])
    meta.raw_indices = meta.raw_indices.clone()
    meta.raw_indices[0] = 999                          # outside the chunk
    lat = torch.zeros(1, 4, 640, dtype=torch.bfloat16, device='cuda')
    rk = torch.zeros(1, 16, 8, 128, dtype=torch.bfloat16, device='cuda')
    _lib.device_status(clear=True)
    # 2 Beacons with 1 latent row left at the cursor; raw row 0 indexes outside the chunk.
    prefill.project_window(W, hidden, meta, 32, 8, 128, query=False, value=False, latents=False,
                           latent_cache=(lat[..., :320], lat[..., 320:]), lat_start=[3], raw_start=[0],
                           raw_cache=(rk, rk.clone()))
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == _lib.DEVICE_BAD_LENGTH
    assert (lat[0, :3] == 0).all() and (lat[0, 3] != 0).any()
    assert (rk[0, 0] == 0).all() and (rk[0, 1:8] != 0).any(dim=-1).all() and (rk[0, 8:] == 0).all()


@pytest.mark.gpu
@pytest.mark.parametrize('tag,transposed', [('a', True), ('b', True), ('c', False)])
def test_prefill_rope_reproduces_reference_bits(tag, transposed):
    from slimkv_b200 import prefill
    p = f'prope_{tag}_'
    q = torch.from_numpy(GOLD[p + 'q']).view(torch.bfloat16).cuda()
    k = torch.from_numpy(GOLD[p + 'k']).view(torch.bfloat16).cuda()
    if transposed:     # the reference test's [B, S, H, D] storage seen as [B, H, S, D]
        q = q.transpose(1, 2).contiguous().transpose(1, 2)
        k = k.transpose(1, 2).contiguous().transpose(1, 2)
    rope = type('R', (), {'cos_cached': torch.from_numpy(GOLD['prope_cos']).cuda(),
                          'sin_cached': torch.from_numpy(GOLD['prope_sin']).cuda()})()
    meta = prefill.PrefillMetadata(None, None, torch.from_numpy(GOLD[p + 'roles']).cuda(),
                                   torch.from_numpy(GOLD[p + 'pos']).cuda(), True)
    qo, ko = prefill.fused_prefill_rope(q, k, rope, meta, int(GOLD[p + 'sink']))
    torch.cuda.synchronize()
    assert qo.stride() == q.stride() and ko.stride() == k.stride()
    assert np.array_equal(_bits(qo), GOLD[p + 'qo'].view(np.uint16))
    assert np.array_equal(_bits(ko), GOLD[p + 'ko'].view(np.uint16))


@pytest.mark.gpu
def test_prefill_rope_llama_window_matches_oracle():
    from slimkv_b200 import prefill
    from slimkv_b200.rope import LLAMA3_SCALING, rope_tables
    cos, sin = rope_tables(128, 500000.0, 8192, LLAMA3_SCALING, 'cuda')
    rng = np.random.default_rng(9)
    roles, _, _ = oracle.interleave_roles(1024, 0, 4)
    Q, K = len(roles), len(roles) + 4 + 512
    q = torch.randn(2, 32, Q, 128, device='cuda').to(torch.bfloat16)
    k = torch.randn(2, 8, K, 128, device='cuda').to(torch.bfloat16)
    pos = torch.arange(K, device='cuda')[None].expand(2, -1) + torch.tensor([[0], [700]], device='cuda')
    rope = type('R', (), {'cos_cached': cos, 'sin_cached': sin})()
    meta = prefill.PrefillMetadata(None, None, torch.from_numpy(roles).cuda(), pos, False)
    qo, ko = prefill.fused_prefill_rope(q, k, rope, meta, 4)
    torch.cuda.synchronize()
    wq, wk = oracle.prefill_rope(q.float().cpu().numpy(), k.float().cpu().numpy(), cos.cpu().numpy(),
                                 sin.cpu().numpy(), pos.cpu().numpy(), roles, 4)
    assert np.array_equal(_bits(qo), bf16_bits(wq))
    assert np.array_equal(_bits(ko), bf16_bits(wk))


def test_window_roles_match_the_oracle_interleave():
    """The product's role list (bench and callers) is the reference's interleave rule."""
    from oracle.schedule import interleave_roles
    from slimkv_b200.prefill import window_roles
    for size, rem, ratio in [(1024, 0, 4), (1000, 3, 4), (7, 1, 8), (3, 0, 4), (4096, 2, 8)]:
        roles, nb, new_rem = window_roles(size, rem, ratio)
        want, wnb, wrem = interleave_roles(size, rem, ratio)
        assert np.array_equal(roles.numpy(), want) and nb == wnb and new_rem == wrem
