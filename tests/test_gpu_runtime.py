"""Whole-step decode runtime: the latent cache in the vLLM plugin's Beacon pages.

The paged runtime (per-sequence shuffled block tables, the backend's page
size rule) must follow the dense runtime given the same cache contents,
through steps that insert a Beacon row (appended into a page) and steps that
do not.  The attention step itself is bit-identical between the layouts
(``test_gpu_decode.py``); the logits also pass through cuBLAS GEMMs, so they
are held to the bf16-logit bar (2e-2 absolute).
"""
import pytest
import torch


@pytest.mark.gpu
def test_paged_runtime_matches_dense_runtime():
    from slimkv_b200 import pages as P
    from slimkv_b200.runtime import LatentDecodeRuntime, LatentLlamaConfig, RandomWeights
    dev = torch.device('cuda', 0)
    cfg = LatentLlamaConfig(layers=2, vocab=512, hidden=1024, intermediate=2048, rank_k=160, rank_v=160, ratio=8)
    w = RandomWeights(cfg, dev, seed=3)
    per_window = cfg.window // cfg.ratio
    history, tails = [per_window * 3, per_window * 17, per_window], [5, 1000, 7]
    dense = LatentDecodeRuntime(cfg, w, history, tails, dev)
    paged = LatentDecodeRuntime(cfg, w, history, tails, dev, paged=True)
    assert paged.layout.slots == 96                     # 768 raw tokens per 64 KB page at r8 / t8
    for cd, cp in zip(dense.caches, paged.caches):
        for name in ('raw_k_rot', 'raw_k_pre', 'raw_v'):
            cp[name].copy_(cd[name])
        for b, h in enumerate(history):
            n = h + per_window                           # history + the open window's rows
            P.beacon_append(cp['pages'], paged.layout, paged.tables[b:b + 1], [0], cd['lat_k'][b:b + 1, :n],
                            cd['lat_v'][b:b + 1, :n])
    tokens = torch.tensor([3, 77, 500], device=dev)
    inserted = 0
    for _ in range(3):
        dense.tokens.copy_(tokens)
        paged.tokens.copy_(tokens)
        ld, lp = dense.step_eager().clone(), paged.step_eager().clone()
        torch.cuda.synchronize()
        assert torch.isfinite(ld).all()
        assert (ld - lp).abs().max().item() <= 2e-2
        inserted += int((paged.query_len == 2).sum())
        tokens = ld.argmax(-1)
    assert inserted >= 2                                # Beacon rows went into pages on some steps


@pytest.mark.gpu
def test_qwen_geometry_runtime_steps():
    """Qwen2.5-14B geometry (40 / 8 heads, q/k/v and up-projection biases,
    r2 ranks 512) through whole runtime steps on the split-KV route."""
    from slimkv_b200.runtime import LatentDecodeRuntime, RandomWeights, qwen25_14b_r2
    from slimkv_b200 import _lib
    dev = torch.device('cuda', 0)
    cfg = qwen25_14b_r2()
    cfg.layers, cfg.vocab, cfg.hidden, cfg.intermediate = 2, 512, 1024, 2048
    w = RandomWeights(cfg, dev, seed=5)
    per_window = cfg.window // cfg.ratio
    rt = LatentDecodeRuntime(cfg, w, [per_window * 5, per_window * 2], [3, 700], dev, raw_pre=False)
    _lib.device_status(clear=True)
    tokens = torch.tensor([11, 400], device=dev)
    for _ in range(5):                                  # the first row inserts a Beacon at step 1
        rt.tokens.copy_(tokens)
        logits = rt.step_eager()
        torch.cuda.synchronize()
        assert torch.isfinite(logits).all()
        tokens = logits.argmax(-1)
    assert _lib.device_status(clear=True) == 0


@pytest.mark.gpu
@pytest.mark.parametrize('geometry', ['llama', 'qwen'])
def test_reconstruct_backend_runtime_follows_latent_backend(geometry):
    """The reconstruct backend (Beacon K/V rebuilt each step, then attention)
    against the latent backend on the same caches, through steps that insert
    Beacons and graph replays, and after one sequence has grown past every
    length seen at construction (the rebuild covers each sequence's current
    latent count, up to the capacity).  One layer, so both backends see
    identical attention inputs each step: the attention rows differ only by
    the bf16 rounding of the rebuilt keys and values (norm-wise 1e-2); the
    caches the backends append must stay bit-identical, and the second query
    row of a sequence that inserts no Beacon (zero keys) comes out zero."""
    from slimkv_b200 import _lib
    from slimkv_b200.runtime import LatentDecodeRuntime, LatentLlamaConfig, RandomWeights, qwen25_14b_r2
    dev = torch.device('cuda', 0)
    if geometry == 'llama':
        cfg = LatentLlamaConfig(layers=1, vocab=512, hidden=1024, intermediate=2048)
    else:
        cfg = qwen25_14b_r2()
        cfg.layers, cfg.vocab, cfg.hidden, cfg.intermediate = 1, 512, 1024, 2048
    w = RandomWeights(cfg, dev, seed=9)
    per_window = cfg.window // cfg.ratio
    history, tails = [per_window * 4, per_window * 9, per_window], [1013, 300, 7]
    lat = LatentDecodeRuntime(cfg, w, history, tails, dev, extra_windows=2)
    rec = LatentDecodeRuntime(cfg, w, history, tails, dev, extra_windows=2, backend='reconstruct')
    for cl, cr in zip(lat.caches, rec.caches):
        for name in ('raw_k_rot', 'raw_k_pre', 'raw_v', 'lat'):
            cr[name].copy_(cl[name])
    tokens = torch.tensor([3, 77, 500], device=dev)
    inserted = 0

    def compare(a, b):
        torch.cuda.synchronize()
        for bb, q in enumerate(lat.query_len.tolist()):
            for l in range(q):
                x, y = lat.attn[bb, l].double(), rec.attn[bb, l].double()
                assert ((x - y).norm() / x.norm()).item() < 1e-2
            if q == 1:
                assert torch.count_nonzero(rec.attn[bb, 1]).item() == 0
        d = (a.float() - b.float()).abs()
        assert d.mean().item() < 5e-3 and d.max().item() <= 0.125
        for cl, cr in zip(lat.caches, rec.caches):
            for name in ('raw_k_rot', 'raw_k_pre', 'raw_v', 'lat'):
                assert torch.equal(cl[name], cr[name]), name

    for _ in range(6):
        lat.tokens.copy_(tokens)
        rec.tokens.copy_(tokens)
        compare(lat.step_eager().clone(), rec.step_eager().clone())
        inserted += int((lat.query_len == 2).sum())
        tokens = lat.next_tokens().clone()
    for rt in (lat, rec):
        rt.tokens.copy_(tokens)
        rt.capture(warmup=1)
    for _ in range(2):
        compare(lat.step().clone(), rec.step().clone())
        tokens = lat.next_tokens().clone()
        lat.tokens.copy_(tokens)
        rec.tokens.copy_(tokens)
    # Sequence 2 jumps to 11 windows of history: more latents than the
    # longest sequence at construction plus a window (within the capacity).
    grown = per_window * 11
    assert grown + per_window > max(history) + per_window + 64
    for rt in (lat, rec):
        rt.history[2] = grown
    for _ in range(2):
        compare(lat.step().clone(), rec.step().clone())
        assert int(lat.latent_len[2].item()) > max(history) + per_window + 64
        tokens = lat.next_tokens().clone()
        lat.tokens.copy_(tokens)
        rec.tokens.copy_(tokens)
    assert _lib.device_status(clear=True) == 0
    assert inserted >= 2


@pytest.mark.gpu
def test_host_io_graph_matches_device_steps():
    """``capture_host_io`` / ``step_host``: token ids in from pinned host memory,
    the step, greedy tokens out, one replay — the same tokens and logits as
    the device-resident graph steps of a twin runtime."""
    from slimkv_b200.runtime import LatentDecodeRuntime, LatentLlamaConfig, RandomWeights
    dev = torch.device('cuda', 0)
    cfg = LatentLlamaConfig(layers=2, vocab=512, hidden=1024, intermediate=2048)
    w = RandomWeights(cfg, dev, seed=11)
    per_window = cfg.window // cfg.ratio
    history, tails = [per_window * 3, per_window], [5, 1000]
    a = LatentDecodeRuntime(cfg, w, history, tails, dev)
    b = LatentDecodeRuntime(cfg, w, history, tails, dev)
    start = torch.tensor([7, 300], dtype=torch.int64)
    for rt in (a, b):
        rt.tokens.copy_(start.to(dev))
        rt.capture(warmup=1)
    host_in = start.clone().pin_memory()
    host_out = torch.empty(2, dtype=torch.int64).pin_memory()
    b.capture_host_io(host_in, host_out)
    tokens = start.to(dev)
    for _ in range(4):
        a.tokens.copy_(tokens)
        logits = a.step().clone()
        tokens = a.next_tokens()
        got = b.step_host()
        assert torch.equal(got.cuda(), tokens)
        assert torch.equal(b.logits, logits)
        host_in.copy_(got)
