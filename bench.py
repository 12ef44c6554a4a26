#!/usr/bin/env python
"""Decode benchmark: Llama-3.1-8B-r4 t4f4, 32k context, batch 16 per GPU.

a full 32-layer decode step of a Llama-3.1-8B-geometry
SlimKV model (random N(0, 0.02) bf16 weights, latent ranks 320/320, Beacon
ratio 4, 4 sinks) over batch 16, every sequence with 32 completed 1024-token
windows (8192 Beacon latents) and a raw tail of U{0..1023} tokens.  One
"step" decodes one raw token per sequence (plus a Beacon row where the
schedule inserts one) through all 32 layers, CUDA-graph captured.

Prints one JSON line: ``value`` = decode tokens/s over all ranks (device
time, inputs resident), ``e2e`` = the same through the public runtime API
with per-step host->device token upload and device->host read of the
sampled tokens, ``roofline`` for the fused latent attention step (HBM bytes
per launch / CUDA-event time), ``cpu_baseline`` = one whole decode step of
the reference's own CPU path on this host's cores.

``prefill`` (one window of one layer) times the
role-selected window projection with the Beacon-page append against the
reference's own recipe run through torch/cuBLAS on the same GPU; its
roofline is tensor-bound (useful FLOPs / time vs the measured bf16 peak).

``--impl reference`` times the reference's own eager decode
(``fa2_decode.decode`` with ``eager_forward``, imported from the package
installed under ``baseline/_ref``) with its Llama modules, whole 32-layer
steps on the host's cores, on the same workload and metric; without that
install it times the numpy restatement in ``oracle/cpu_decode.py``.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'decode tokens/s and latent-attn HBM GB/s (% of peak), Llama-3.1-8B-r4 t4f4 32k ctx'
UNIT = 'tokens/s'
BATCH = 16
HISTORY = 8192          # 32 completed windows x 256 Beacon latents
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser(description=__doc__.split('\n')[0])
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--impl', default='slimkv_b200', choices=['slimkv_b200', 'reference'])
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-prefill', action='store_true', help='skip the config-4 prefill window measurement')
    p.add_argument('--prefill-only', action='store_true',
                   help='only the config-4 prefill window measurement (profiling runs)')
    p.add_argument('--config', type=int, default=2, choices=[2, 3, 5],
                   help='2 (default): the metric\'s config; 3: batched paged decode, r8, B=256, ragged contexts; '
                        '5: Qwen2.5-14B geometry, r2, 131072-token contexts, 32 sequences per GPU')
    p.add_argument('--tp', action='store_true',
                   help='config 2 at a fixed global batch of 16 over the N ranks: projections and MLP split by KV '
                        'head, attention split by sequence (all-to-all), strong scaling')
    p.add_argument('--seq-split', action='store_true',
                   help='with --config 5: the batch-1 524288-token sequence, its latents split over the N ranks '
                        '(cross-GPU LSE merge over NCCL every layer)')
    p.add_argument('--reconstruct', action='store_true',
                   help='with --config 5: the reference\'s reconstruct decode backend (Beacon K/V rebuilt from the '
                        'latents every step, then attention) instead of the latent backend')
    p.add_argument('--kernel-only', action='store_true',
                   help='one layer of the same workload: time the attention kernel alone (profiling runs)')
    return p.parse_args()


C3_BATCH = 256
C3_METRIC = 'decode tokens/s and latent-attn HBM GB/s, paged vLLM-plugin layout, Llama-3.1-8B-r8 t8f8, ' \
            'B=256, ctx U[2048,131072]'


def config3(n, ctx):
    return {'workload': 'Llama-3.1-8B-r8 t8f8 batched paged decode step (BASELINE config 3), latent path',
            'global_batch': C3_BATCH * n, 'batch_per_gpu': C3_BATCH,
            'context': f'U[2048, 131072] seeded (mean {int(ctx.mean())}, max {int(ctx.max())})',
            'latent_rank': '160/160', 'ratio': 8, 'sinks': 4, 'layers': 32,
            'latent_cache': 'Beacon pages of the vLLM plugin (96 slots = 768 raw tokens per 64 KB page), '
                            'shuffled per-sequence block tables; raw tail in the native rotated layout',
            'parallelism': f'dp{n} (independent replicas, no data-path collective)',
            'l2': 'each step reads ~60 GB (weights + caches) >> 126 MB L2; no flush needed'}


C5_BATCH = 32
C5_METRIC = 'decode tokens/s and latent-attn HBM GB/s, Qwen2.5-14B-r2 t4 latent path, 131072-token contexts'


def config5(n):
    return {'workload': 'Qwen2.5-14B geometry r2 t4 decode step (BASELINE config 5, batch-64 run as 32 sequences '
                        'per GPU), latent path',
            'global_batch': C5_BATCH * n, 'batch_per_gpu': C5_BATCH, 'context': '131072 + raw tail U{0..1023}',
            'beacon_latents': 32768, 'latent_rank': '512/512', 'heads': '40 / 8 KV', 'sinks': 4, 'layers': 48,
            'parallelism': f'dp{n} (independent replicas; 64 sequences = 2 GPUs)',
            'l2': 'each step reads ~140 GB (weights + caches) >> 126 MB L2; no flush needed'}


C5S_CONTEXT = 524288
C5S_METRIC = 'decode tokens/s of one 524288-token sequence split over N GPUs (cross-GPU LSE merge), ' \
             'Qwen2.5-14B-r2 t4 latent path'


def config5s(n, tail):
    return {'workload': 'Qwen2.5-14B geometry r2 t4 decode step of one 524288-token sequence (BASELINE config 5, '
                        'batch-1 run), latents sequence-split over the GPUs',
            'global_batch': 1, 'context': f'{C5S_CONTEXT} + raw tail {tail}', 'beacon_latents': C5S_CONTEXT // 4,
            'latent_rank': '512/512', 'heads': '40 / 8 KV', 'sinks': 4, 'layers': 48,
            'parallelism': f'sequence split over {n} GPU(s): contiguous 64-row latent shards, raw tail and new '
                           'Beacons on the last rank, one NCCL all-gather of fp32 partials + N-part LSE merge per '
                           'layer; projections / MLP replicated' if n > 1 else 'one GPU, no split',
            'l2': 'each step reads ~43 GB (weights + latents) >> 126 MB L2; no flush needed'}


def config(n):
    return {'workload': 'Llama-3.1-8B-r4 t4f4 decode step (BASELINE config 2), latent path',
            'global_batch': BATCH * n, 'batch_per_gpu': BATCH, 'context': '32768 + raw tail U{0..1023}',
            'beacon_latents': HISTORY, 'latent_rank': '320/320', 'sinks': 4, 'layers': 32,
            'parallelism': f'dp{n} (independent replicas, no data-path collective)',
            'l2': 'each step reads ~23 GB (weights + caches) >> 126 MB L2; no flush needed'}


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.QUERY}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.flush()
        self.file.seek(0)
        sm, mx, reasons = [], 0.0, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.file.read().strip().splitlines():
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == 'active':
                    reasons.add(name)
        os.unlink(self.file.name)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': mx, 'reasons': sorted(reasons), 'samples': len(sm)}


def peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d['hbm_gbs']), 'measured'
    return FALLBACK_HBM_GBS, 'fallback'


def tensor_peak():
    """Dense bf16 TFLOP/s to divide by: the measured cuBLAS burst figure."""
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)['bf16_tflops']), 'measured (MEASURED_PEAKS.json bf16_tflops, burst)'
    return 1590.0, 'fallback 1590 TFLOP/s'


def traffic_per_launch(kernel_bytes):
    """ncu DRAM bytes (read + write) of one attention launch, from the
    committed capture of the same kernel on one layer of this workload,
    scaled to this run's algorithmic bytes per launch (traffic grows with the
    latent / raw rows streamed)."""
    path = os.path.join(ROOT, 'profiles', 'decode_tc_kernel_c2_traffic.json')
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    return (d['dram_read_bytes'] + d['dram_write_bytes']) * kernel_bytes / d['algorithmic_bytes']


REF_DIR = os.path.join(ROOT, 'baseline', '_ref')


def _cpu_model():
    try:
        with open('/proc/cpuinfo') as f:
            for line in f:
                if line.startswith('model name'):
                    return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


def _reference_package():
    """Import the reference package installed under ``baseline/_ref`` (``pip
    install --no-deps --target``).  It imports two packages at load time that
    this path never uses (``pytz`` for a version check, ``accelerate`` for a
    type); minimal stand-ins are written to a temporary directory when they
    are absent.  Returns the modules, or raises ImportError."""
    import importlib.util
    if not os.path.isdir(os.path.join(REF_DIR, 'slimkv')):
        raise ImportError('baseline/_ref holds no installed slimkv package')
    stubs = tempfile.mkdtemp(prefix='slimkv_stubs_')
    if importlib.util.find_spec('pytz') is None:
        os.makedirs(os.path.join(stubs, 'pytz'))
        with open(os.path.join(stubs, 'pytz', '__init__.py'), 'w') as f:
            f.write('__version__ = "2024.1"\n')
    if importlib.util.find_spec('accelerate') is None:
        os.makedirs(os.path.join(stubs, 'accelerate'))
        with open(os.path.join(stubs, 'accelerate', '__init__.py'), 'w') as f:
            f.write('__version__ = "1.0.0"\nclass Accelerator:\n    pass\n')
    sys.path[:0] = [stubs, REF_DIR]
    from slimkv.llama3 import fa2_decode
    from slimkv.llama3.configuration_llama import LlamaConfig
    from slimkv.llama3.latent_decode import eager_forward
    from slimkv.llama3.memory import ReconstructionCache
    from slimkv.llama3.modeling_llama import LlamaAttention, LlamaMLP, LlamaRMSNorm
    return dict(fa2_decode=fa2_decode, LlamaConfig=LlamaConfig, eager_forward=eager_forward,
                ReconstructionCache=ReconstructionCache, LlamaAttention=LlamaAttention, LlamaMLP=LlamaMLP,
                LlamaRMSNorm=LlamaRMSNorm)


class ReferenceDecodeStep:
    """One decode step of the workload through the reference's own modules
    on the CPU: per layer ``LlamaRMSNorm``, ``fa2_decode.decode(...,
    forward=eager_forward)`` (the reference's eager latent decode with its
    ``o_proj``), the residual, ``LlamaRMSNorm`` and ``LlamaMLP``; then the
    final norm and the vocabulary projection of the raw rows.  fp32, the
    reference's CPU dtype.  The reference batches only equal-length caches,
    so each sequence (its own raw tail) is its own ``decode`` call; norms and
    MLP run on the whole batch.  One layer's weights serve all 32 layers
    (32 distinct fp32 layers do not fit host memory); every layer's
    arithmetic runs.  Caches: N(0, 1.3^2), weights the modules' own init."""

    LAYERS, VOCAB, HIDDEN, SINK, RANK, KV_HEADS, HEAD_DIM = 32, 128256, 4096, 4, 320, 8, 128

    def __init__(self, m, batch, history, seed=1234):
        import numpy as np
        import torch
        self.m, self.torch = m, torch
        R, Hkv, D, S = self.RANK, self.KV_HEADS, self.HEAD_DIM, self.SINK
        cfg = m['LlamaConfig'](
            vocab_size=self.VOCAB, hidden_size=self.HIDDEN, intermediate_size=14336, num_hidden_layers=self.LAYERS,
            num_attention_heads=32, num_key_value_heads=Hkv, max_position_embeddings=131072, rope_theta=500000.0,
            rope_scaling=dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                              original_max_position_embeddings=8192, rope_type='llama3'),
            beacon_param=['q', 'k', 'v'], beacon_window=1024, beacon_stride=1024, beacon_ratio=[4],
            beacon_ratio_mix='sequence', beacon_sink_size=S, beacon_skip_rope_for_beacon_k=True,
            beacon_k_compression='lowrank_svd', beacon_v_compression='lowrank_svd',
            beacon_k_latent_head_dim_list=[R // Hkv] * self.LAYERS,
            beacon_v_latent_head_dim_list=[R // Hkv] * self.LAYERS, beacon_decode_backend='latent',
            torch_dtype=torch.float32)
        cfg._attn_implementation = 'eager'
        with torch.no_grad():
            self.attn = m['LlamaAttention'](cfg, layer_idx=0).eval()
            self.mlp = m['LlamaMLP'](cfg).eval()
            self.norm1, self.norm2, self.norm_f = (m['LlamaRMSNorm'](self.HIDDEN) for _ in range(3))
            self.lm_head = torch.empty(self.VOCAB, self.HIDDEN).normal_(0, 0.02)
        gen = torch.Generator().manual_seed(seed)
        tails = np.random.default_rng(seed).integers(0, 1024, size=batch)     # the GPU arm's tails
        self.seqs = []
        for t in map(int, tails):
            nw = t // 4
            rnd = lambda *shape: torch.randn(*shape, generator=gen) * 1.3
            raw_idx = torch.arange(t) + torch.arange(t) // 4 if t else None
            win_roles = torch.zeros(t + nw, dtype=torch.bool)
            win_roles[4::5] = True
            size = int((t + 1) % 4 == 0)
            roles = torch.zeros(t + nw + 1 + size, dtype=torch.long)
            roles[:t + nw] = win_roles.long()
            roles[-1] = size

            def cache(kind):
                return m['ReconstructionCache'](rnd(1, Hkv, S, D), rnd(1, 1, history, R),
                                                rnd(1, Hkv, t, D) if t else None, rnd(1, 1, nw, R) if nw else None,
                                                win_roles if t else None, Hkv, D, kind, raw_idx)
            positions = torch.arange(S + history + t + nw + 1 + size)[None]
            self.seqs.append((cache('k'), cache('v'), size, roles, positions))
        self.x = torch.randn(batch, 2, self.HIDDEN, generator=gen)

    def layer(self, x):
        fa2 = self.m['fa2_decode']
        y = x.clone()
        for b, (pk, pv, size, roles, positions) in enumerate(self.seqs):
            h = self.norm1(x[b:b + 1, :size + 1])
            out, _, _ = fa2.decode(self.attn, h, positions, (pk, pv, size, roles), forward=self.m['eager_forward'])
            y[b:b + 1, :size + 1] += out
        return y + self.mlp(self.norm2(y))

    def step(self, layers=None):
        with self.torch.inference_mode():
            x = self.x
            for _ in range(layers or self.LAYERS):
                x = self.layer(x)
            return self.norm_f(x[:, 0]) @ self.lm_head.T


def _reference_or_port(batch):
    """(runner, kind, description): the reference's own decode step when its
    package is installed under baseline/_ref, else the numpy restatement
    (pinned to the reference's decode goldens)."""
    try:
        ref = ReferenceDecodeStep(_reference_package(), batch, HISTORY)
        return ref, 'reference', ('reference SlimKV (baseline/_ref) fa2_decode.decode(forward=eager_forward) + '
                                  'LlamaRMSNorm/LlamaMLP modules, fp32 torch on CPU')
    except ImportError as e:
        return None, 'port', f'numpy restatement of the reference decode ({e})'


def cpu_baseline(batch):
    import torch
    ref, kind, what = _reference_or_port(batch)
    if ref is None:
        from oracle.cpu_decode import time_decode_step
        seconds, threads, sample = time_decode_step(batch=batch, history=HISTORY)
        return {'value': batch / seconds, 'unit': UNIT, 'cores': threads, 'kind': 'port', 'sample': sample,
                'cpu': _cpu_model()}
    ref.step(layers=1)                                    # warm-up
    t0 = time.perf_counter()
    ref.step()
    seconds = time.perf_counter() - t0
    return {'value': batch / seconds, 'unit': UNIT, 'cores': torch.get_num_threads(), 'kind': kind,
            'sample': f'one whole decode step (32 layers + vocab projection), batch {batch}; {what}',
            'cpu': _cpu_model()}


def run_reference(args):
    """The reference arm: the reference's own CPU decode on this host, the
    same workload and metric, whole steps (W warm-up, K timed)."""
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    import torch
    ref, kind, what = _reference_or_port(BATCH)
    if ref is None:
        from oracle.cpu_decode import CpuDecodeLayer, _rms
        import numpy as np
        rng = np.random.default_rng(1234)
        layer, lengths = CpuDecodeLayer.synthetic(HISTORY, rng.integers(0, 1024, size=BATCH))
        x0 = rng.standard_normal((BATCH, 2, 4096), dtype=np.float32)
        head = rng.standard_normal((128256, 4096), dtype=np.float32) * np.float32(0.02)

        def step():
            x = x0
            for _ in range(32):
                x = layer.forward(x, lengths)
            return _rms(x[:, 0]) @ head.T
        threads = len(os.sched_getaffinity(0))
    else:
        step = ref.step
        threads = torch.get_num_threads()
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = BATCH * args.steps / total
    sample = f'{args.steps} whole decode steps (32 layers + vocab projection) of batch {BATCH}; {what}'
    print(json.dumps({
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': 1000.0 * total / args.steps,
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': config(1),
        'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': threads, 'kind': kind, 'sample': sample,
                         'cpu': _cpu_model()},
        'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
        'note': 'CPU: the reference GPU decode kernel builds only for sm_90/sm_120; rank 0 alone runs under '
                'torchrun'}), flush=True)


PREFILL_BATCH = 4
PREFILL_WINDOW = 1024


def prefill_window_step(device, steps, warmup):
    """BASELINE config 4, one window of one layer: B=4 sequences x 1280
    interleaved rows (1024 raw tokens + 256 Beacons), Llama-3.1-8B r4 layer
    (hidden 4096, 32/8 heads, ranks 320/320), hidden rows N(0, 1), random
    N(0, 0.02) weights.  Times (CUDA graphs, device time) the role-selected
    projection with the Beacon-page append (``slimkv_window_project``), the
    append alone (Beacon latents -> pages) and the reference's recipe on the
    same GPU through torch/cuBLAS: every row through both weight sets,
    torch.where, index_select and the page write by advanced indexing
    (modeling_llama.py:1291-1367, paged_cache.py:78-87)."""
    import torch
    from slimkv_b200 import prefill, _lib
    from slimkv_b200.pages import BeaconPageLayout, BeaconPages
    g = torch.Generator(device=device)
    g.manual_seed(4)
    H, qd, kvd, R, B = 4096, 4096, 1024, 320, PREFILL_BATCH

    def w(*shape, std=0.02):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    W = prefill.BeaconProjectionWeights(q=w(qd, H), k=w(kvd, H), v=w(kvd, H), bq=w(qd, H), k_down=w(R, H),
                                        v_down=w(R, H), k_up=w(kvd, R), v_up=w(kvd, R))
    roles, _, _ = prefill.window_roles(PREFILL_WINDOW, 0, 4)
    n = len(roles)
    hidden = w(B, n, H, std=1.0)
    meta = prefill.metadata_from_roles(roles.to(device), n)
    meta.raw_indices, meta.beacon_indices = meta.raw_indices.int(), meta.beacon_indices.int()
    layout = BeaconPageLayout(192, 4, R, R, kvd)
    per_seq = 32 * 1024 // 192 + 2                        # a 32k prompt's Beacon pages
    pages = torch.zeros(B * per_seq, layout.page_elements, dtype=torch.bfloat16, device=device)
    tables = torch.arange(B * per_seq, dtype=torch.int32, device=device).reshape(B, per_seq)
    lat_start = torch.full((B,), 7 * 256, dtype=torch.int32, device=device)    # the 8th window of the prompt
    bp = BeaconPages(pages, layout)
    nb = meta.beacon_indices.numel()

    def ours():
        return prefill.project_window(W, hidden, meta, 32, 8, 128, lat_start=lat_start, beacon=(bp, tables))

    def append_only():
        prefill.project_window(W, hidden, meta, 32, 8, 128, query=False, key=False, value=False, latents=False,
                               lat_start=lat_start, beacon=(bp, tables))

    role_raw = (meta.roles == 0)[:, None]
    cols = torch.arange(layout.width, device=device)

    def recipe():
        q = torch.where(role_raw, hidden @ W.q.t(), hidden @ W.bq.t())
        lk, lv = hidden @ W.k_down.t(), hidden @ W.v_down.t()
        k = torch.where(role_raw, hidden @ W.k.t(), lk @ W.k_up.t())
        v = torch.where(role_raw, hidden @ W.v.t(), lv @ W.v_up.t())
        sk, sv = lk.index_select(1, meta.beacon_indices), lv.index_select(1, meta.beacon_indices)
        for b in range(B):
            logical = torch.arange(7 * 256, 7 * 256 + nb, device=device)
            page = tables[b].long()[logical // layout.slots]
            col = layout.sink_elements + (logical % layout.slots)[:, None] * layout.width + cols[None]
            pages[page[:, None], col] = torch.cat([sk[b], sv[b]], dim=-1)
        return q, k, v

    def graph_us(fn):
        fn()
        torch.cuda.synchronize()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(max(warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps * 1000.0

    _lib.device_status(clear=True)
    t_ours, t_append, t_ref = graph_us(ours), graph_us(append_only), graph_us(recipe)
    status = _lib.device_status(clear=True)
    raw_rows, beacon_rows = B * PREFILL_WINDOW, B * nb
    flops = 2 * H * (raw_rows * (qd + 2 * kvd) + beacon_rows * (qd + 2 * R)) + 2 * beacon_rows * 2 * R * kvd
    append_flops = 2 * H * beacon_rows * 2 * R
    append_bytes = beacon_rows * H * 2 + 2 * R * H * 2 + beacon_rows * 2 * R * 2
    return {'workload': 'BASELINE config 4 window step, one layer: B=4 x (1024 raw + 256 Beacon) interleaved rows, '
                        'Llama-3.1-8B r4 (hidden 4096, heads 32/8, ranks 320/320), Beacon pages 192 raw tokens',
            'us_per_window_layer': t_ours, 'raw_tokens_per_s_per_layer': raw_rows / (t_ours / 1e6),
            'tflops': flops / (t_ours / 1e6) / 1e12, 'flops_per_window_layer': flops,
            'append_only_us': t_append, 'append_only_gbs': append_bytes / (t_append / 1e6) / 1e9,
            'append_only_bytes': append_bytes, 'append_only_tflops': append_flops / (t_append / 1e6) / 1e12,
            'reference_recipe_gpu_us': t_ref, 'speedup_vs_reference_recipe': t_ref / t_ours,
            'kernels': 'project_kernel (tcgen05, gathered rows) + finalize_kernel when split', 'device_status': status}


def prefill_chunk_attention(device, steps, warmup):
    """BASELINE config 4, the attention of one layer at the last 4096-token
    chunk of the 32768-token prompts: B=4 x 5120 chunk rows (4 windows of
    1024 raw + 256 Beacon rows), 4 sinks, 7168 history Beacon latents (ranks
    320), Llama-3.1-8B heads (32 / 8, dim 128).  Times (CUDA graphs) the
    absorbed-history attention (``prefill_attention.latent_history_attention``:
    two ``slimkv_prefill_attention`` launches, the absorb and up-projection
    GEMMs, the LSE merge), the materialised recipe on this library's kernels
    and the reference's recipe on the same GPU through torch: the history up-
    projected by ``nn.Linear`` each chunk, concatenated with the sinks and the
    chunk, then a causal (bottom-right) scaled-dot-product attention."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention.bias import causal_lower_right
    from slimkv_b200 import _lib
    from slimkv_b200 import prefill_attention as PA
    g = torch.Generator(device=device)
    g.manual_seed(44)
    B, T, P, N, H, Hkv, D, R = PREFILL_BATCH, 5120, 4, 7168, 32, 8, 128, 320
    bf = lambda *s, std=1.0: (torch.randn(*s, generator=g, device=device) * std).to(torch.bfloat16)
    q, k_cur, v_cur = bf(B, T, H, D), bf(B, T, Hkv, D), bf(B, T, Hkv, D)
    sink_k, sink_v = bf(B, P, Hkv, D), bf(B, P, Hkv, D)
    lat = bf(B, N, 2 * R, std=1.3)
    lat_k, lat_v = lat[..., :R], lat[..., R:]
    uk, uv = bf(Hkv * D, R, std=0.05), bf(Hkv * D, R, std=0.05)
    lat_len = torch.full((B,), N, dtype=torch.int32, device=device)
    scale = 1.0 / math.sqrt(D)
    mask = causal_lower_right(T, P + N + T)

    def absorbed():
        return PA.latent_history_attention(q, sink_k, sink_v, lat_k, lat_v, lat_len, uk, uv, k_cur, v_cur, scale)

    def materialized():
        return PA.materialized_history_attention(q, sink_k, sink_v, lat_k, lat_v, N, uk, uv, k_cur, v_cur, scale)

    def recipe():
        hk = (lat_k @ uk.t()).view(B, N, Hkv, D)
        hv = (lat_v @ uv.t()).view(B, N, Hkv, D)
        keys = torch.cat([sink_k, hk, k_cur], 1).transpose(1, 2)
        vals = torch.cat([sink_v, hv, v_cur], 1).transpose(1, 2)
        return F.scaled_dot_product_attention(q.transpose(1, 2), keys, vals, attn_mask=mask, scale=scale,
                                              enable_gqa=True)

    def graph_us(fn):
        fn()
        torch.cuda.synchronize()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(max(warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps * 1000.0

    # The two kernel launches alone (inputs as latent_history_attention makes them).
    q_lat = torch.einsum('btgjd,gdr->btgjr', q.view(B, T, Hkv, H // Hkv, D), uk.view(Hkv, D, R)).reshape(B, T, H, R)
    keys_k, keys_v = torch.cat([sink_k, k_cur], 1), torch.cat([sink_v, v_cur], 1)
    chunk_len = torch.full((B,), P + T, dtype=torch.int32, device=device)

    def history_kernel():
        return PA.attention(q_lat, lat_k.unsqueeze(2), lat_v.unsqueeze(2), lat_len, scale, H)

    def chunk_kernel():
        return PA.attention(q, keys_k, keys_v, chunk_len, scale, H // Hkv, causal=True, causal_offset=P)

    _lib.device_status(clear=True)
    t_hist_k, t_chunk_k = graph_us(history_kernel), graph_us(chunk_kernel)
    t_abs, t_mat = graph_us(absorbed), graph_us(materialized)
    try:
        t_ref = graph_us(recipe)
    except RuntimeError as e:                                  # no SDPA backend for this mask on this build
        t_ref = None
        ref_error = str(e).splitlines()[0]
    status = _lib.device_status(clear=True)
    # FLOPs: 2 per multiply-add of S and of P.V (causal chunk part: the visible half).
    chunk_keys = B * H * (T * P + T * (T + 1) // 2)
    hist_pairs = B * H * T * N
    f_hist_abs = 2 * hist_pairs * 2 * R
    f_hist_mat = 2 * hist_pairs * 2 * D
    f_chunk = 2 * chunk_keys * 2 * D
    out = {'workload': 'BASELINE config 4 prefill attention, one layer at the last chunk: B=4 x 5120 rows '
                       '(4096 raw + 1024 Beacon), 4 sinks, 7168 history latents (ranks 320), heads 32/8 dim 128',
           'absorbed_us': t_abs, 'absorbed_tflops': (f_hist_abs + f_chunk) / (t_abs / 1e6) / 1e12,
           'absorbed_flops': f_hist_abs + f_chunk,
           'materialized_us': t_mat, 'materialized_tflops': (f_hist_mat + f_chunk) / (t_mat / 1e6) / 1e12,
           'materialized_flops': f_hist_mat + f_chunk,
           'history_kernel_us': t_hist_k, 'history_kernel_tflops': f_hist_abs / (t_hist_k / 1e6) / 1e12,
           'chunk_kernel_us': t_chunk_k, 'chunk_kernel_tflops': f_chunk / (t_chunk_k / 1e6) / 1e12,
           'reference_recipe_gpu_us': t_ref,
           'kernels': 'prefill_attention_kernel (tcgen05, twice) + cuBLAS absorb / up-projection + merge_kernel; '
                      'materialized: project_kernel (reconstruct) + prefill_attention_kernel',
           'device_status': status}
    if t_ref is None:
        out['reference_recipe_error'] = ref_error
    else:
        out['speedup_vs_reference_recipe'] = t_ref / min(t_abs, t_mat)
    return out


def attention_kernel_time(rt, reps):
    """Average device time of the attention launch (both branches) alone:
    CUDA events recorded by the library right around that kernel, on the
    launching stream, over `reps` launches cycling through the layers."""
    import torch
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for b, e in events:         # creates the CUDA events (torch makes them lazily); the library re-records them
        b.record()
        e.record()
    torch.cuda.synchronize()
    for i in range(reps):
        rt.calls[i % len(rt.calls)](attn_events=events[i])
    torch.cuda.synchronize()
    return sum(b.elapsed_time(e) for b, e in events) / reps


def reconstruct_roofline(rt, reps):
    """The reconstruct backend per layer: the whole attention step (RoPE,
    appends, Beacon K/V rebuild, attention) and the rebuild alone
    (``slimkv_reconstruct_kv``: 2 x rows x R x Hkv*D x 2 FLOPs for K and V),
    CUDA events on the launching stream, cycling through the layers."""
    import torch
    from slimkv_b200.reconstruct import reconstruct_kv
    cfg = rt.cfg
    ev = lambda: torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a0, a1 = ev(), ev()
    a0.record()
    for i in range(reps * cfg.layers):
        rt._reconstruct_attention(i % cfg.layers)
    a1.record()
    torch.cuda.synchronize()
    step_us = a0.elapsed_time(a1) / (reps * cfg.layers) * 1000.0
    r0, r1 = ev(), ev()
    r0.record()
    for i in range(reps * cfg.layers):
        d = rt.recon[i % cfg.layers]
        w_k, w_v, b_k, b_v = d.w
        reconstruct_kv(d.lat_k, d.lat_v, w_k, w_v, d.key_full, d.value_full, d.rows, b_k, b_v, out_start=d.raw_len,
                       row_count=d.latent_len)
    r1.record()
    torch.cuda.synchronize()
    rebuild_us = r0.elapsed_time(r1) / (reps * cfg.layers) * 1000.0
    rows = int(rt.latent_len.sum().item())
    kvd = cfg.kv_heads * cfg.head_dim
    flops = 2.0 * rows * kvd * (cfg.rank_k + cfg.rank_v)
    tflops = flops / (rebuild_us / 1e6) / 1e12
    peak, source = tensor_peak()
    return {'step_per_layer_us': step_us, 'rebuild_per_layer_us': rebuild_us, 'rebuilt_rows_per_layer': rows,
            'rebuild_flops_per_layer': flops,
            'roofline': {'bound': 'tensor', 'achieved': tflops, 'peak': peak, 'unit': 'TFLOP/s',
                         'frac': tflops / peak, 'peak_source': source, 'traffic': None,
                         'kernel': 'project_kernel (Beacon K/V rebuild, tcgen05)',
                         'flops_per_launch': flops, 'us_per_launch': rebuild_us}}


def own_launches_per_step(rt):
    """Kernels of this repository's library (names in the ``slimkv``
    namespace) that one eager decode step launches, counted by the CUDA
    profiler (torch/cuBLAS kernels excluded).  Run after the timed region;
    the step advances the cache like any other."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        rt.step_eager()
        torch.cuda.synchronize()
    n = sum(1 for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA and 'slimkv' in e.name)
    if n == 0:
        # The profiler saw no kernel at all (its CUDA activity tracing is
        # unavailable, e.g. under another profiler): the step's launches by
        # construction — schedule and plan, then prologue, attention and merge
        # per layer.
        n = 2 + 3 * rt.cfg.layers
    return n


def kernel_only(args):
    """One layer of the bench workload (same batch, history, tails; config 2,
    or config 3 / 5 with ``--config``): the fused decode call
    repeated; prints the attention kernel's time.  Small device footprint,
    for ncu captures of the dominant kernel."""
    import numpy as np
    import torch
    from slimkv_b200 import _lib
    from slimkv_b200.runtime import LatentDecodeRuntime, LatentLlamaConfig, RandomWeights
    device = torch.device('cuda', 0)
    rng = np.random.default_rng(1234)
    if args.config == 5:
        import dataclasses
        from slimkv_b200.runtime import qwen25_14b_r2
        cfg = dataclasses.replace(qwen25_14b_r2(), layers=1, vocab=1024)
        batch = C5_BATCH
        history = [131072 // cfg.window * (cfg.window // cfg.ratio)] * batch
        extra = dict(raw_pre=False)
    elif args.config == 3:
        cfg = LatentLlamaConfig(rank_k=160, rank_v=160, ratio=8, layers=1, vocab=1024)
        batch = C3_BATCH
        ctx = rng.integers(2048, 131072 + 1, size=batch)
        history = (ctx // cfg.window) * (cfg.window // cfg.ratio)
        extra = dict(paged=True, raw_pre=False)
    else:
        cfg = LatentLlamaConfig(layers=1, vocab=1024)
        batch = BATCH
        history = [HISTORY] * batch
        extra = {}
    weights = RandomWeights(cfg, device, seed=0)
    tails = ctx % cfg.window if args.config == 3 else rng.integers(0, cfg.window, size=batch)
    rt = LatentDecodeRuntime(cfg, weights, history, tails, device, extra_windows=1, **extra)
    rt.tokens.copy_(torch.from_numpy(rng.integers(0, cfg.vocab, size=batch)).to(device))
    rt.step_eager()
    for _ in range(max(args.warmup, 1)):
        rt.calls[0]()
    ms = attention_kernel_time(rt, max(args.steps, 1))
    nbytes = rt.attention_kernel_bytes()
    print(json.dumps({'kernel_only': True, 'attention_us': ms * 1e3, 'bytes_per_launch': nbytes,
                      'achieved_gbs': nbytes / (ms / 1e3) / 1e9, 'device_status': _lib.device_status(clear=True)}),
          flush=True)


TP_METRIC = 'decode tokens/s, Llama-3.1-8B-r4 t4f4 32k ctx, global batch 16 over N GPUs (KV-head tensor parallel)'


def tensor_parallel_bench(args):
    """Strong scaling of config 2: global batch 16, weights split by KV head,
    attention split by sequence (`slimkv_b200.tensor_parallel`).  Also times
    the step's collectives alone (2 all-to-alls + 2 all-reduces per layer and
    the logits all-gather, same buffers, CUDA graph) as the communication
    floor of the step."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from slimkv_b200.parallel import max_over_ranks
    from slimkv_b200.runtime import LatentLlamaConfig, RandomWeights
    from slimkv_b200.tensor_parallel import TensorParallelDecode
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        dist.init_process_group('nccl', timeout=timedelta(seconds=300))
    else:
        import socket
        with socket.socket() as sock:
            sock.bind(('127.0.0.1', 0))
            port = sock.getsockname()[1]
        dist.init_process_group('nccl', init_method=f'tcp://127.0.0.1:{port}', rank=0, world_size=1,
                                timeout=timedelta(seconds=300))
    torch.cuda.set_device(local)
    device = torch.device('cuda', local)
    rng = np.random.default_rng(1234)                      # the same global batch on every rank
    cfg = LatentLlamaConfig()
    weights = RandomWeights(cfg, device, seed=0)
    tails = rng.integers(0, cfg.window, size=BATCH)
    tp = TensorParallelDecode(cfg, weights, [HISTORY] * BATCH, tails, device, extra_windows=1)
    del weights
    torch.cuda.empty_cache()
    tp.tokens.copy_(torch.from_numpy(rng.integers(0, cfg.vocab, size=BATCH)).to(device))
    tp.capture(warmup=2)
    for _ in range(max(args.warmup, 3)):
        tp.step()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(args.steps):
        tp.step()
    s1.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    dist.barrier()
    ms = max_over_ranks(s0.elapsed_time(s1) / args.steps, device=device)
    # End to end: host tokens in, sampled tokens out, every step.
    host_in = torch.from_numpy(rng.integers(0, cfg.vocab, size=BATCH)).pin_memory()
    host_out = torch.empty(BATCH, dtype=torch.int64).pin_memory()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        tp.tokens.copy_(host_in, non_blocking=True)
        logits = tp.step()
        host_out.copy_(logits.argmax(-1), non_blocking=True)
        torch.cuda.current_stream().synchronize()
        host_in.copy_(host_out)
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, device=device)
    # The collectives alone, captured like the step.
    comm = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))

    def collectives():
        for _ in range(cfg.layers):
            dist.all_to_all_single(tp.recv1, tp.send1)
            dist.all_to_all_single(tp.recv2, tp.send2)
            dist.all_reduce(tp.part)
            dist.all_reduce(tp.part)
        dist.all_gather_into_tensor(tp.logits_all, tp.logits_part)
    with torch.cuda.stream(stream):
        collectives()
    torch.cuda.current_stream(device).wait_stream(stream)
    with torch.cuda.graph(comm, stream=stream):
        collectives()
    torch.cuda.current_stream(device).wait_stream(stream)
    for _ in range(3):
        comm.replay()
    torch.cuda.synchronize()
    dist.barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(args.steps):
        comm.replay()
    c1.record()
    torch.cuda.synchronize()
    dist.barrier()
    comm_ms = max_over_ranks(c0.elapsed_time(c1) / args.steps, device=device)
    per_layer_bytes = (tp.send1.numel() + tp.send2.numel()) * 2 + 2 * tp.part.numel() * 4
    result = {
        'metric': TP_METRIC, 'value': BATCH / (ms / 1000.0), 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
        'warmup': max(args.warmup, 3), 'ms_per_step': ms, 'higher_is_better': True, 'scaling': 'strong',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (random N(0,0.02) weights, synthetic cache)',
        'config': {'workload': 'Llama-3.1-8B-r4 t4f4 decode step (BASELINE config 2), latent path',
                   'global_batch': BATCH, 'batch_per_gpu': BATCH // world, 'context': '32768 + raw tail U{0..1023}',
                   'beacon_latents': HISTORY, 'layers': 32,
                   'parallelism': f'tp{world}: q/k/v/o, Beacon q and MLP split by KV head (all-reduce), attention '
                                  f'split by sequence (all-to-all), lm_head by vocabulary (all-gather)',
                   'l2': 'each step reads > 2 GB per GPU >> 126 MB L2; no flush needed'},
        'e2e': {'value': BATCH / (e2e_ms / 1000.0), 'unit': UNIT, 'h2d_bytes_per_step': BATCH * 8,
                'd2h_bytes_per_step': BATCH * 8, 'ms_per_step': e2e_ms},
        'communication': {'ms_per_step_collectives_alone': comm_ms, 'collectives_per_step': 4 * cfg.layers + 1,
                          'bytes_sent_per_rank_per_layer': per_layer_bytes},
        'gpu_launches': args.steps * own_launches_per_step(tp),
        'clocks': clock_info,
    }
    comm = None
    tp.release()
    if dist.get_rank() == 0:
        print(json.dumps(result), flush=True)
    dist.destroy_process_group()


def main():
    args = parse()
    if args.tp:
        return tensor_parallel_bench(args)
    if args.impl == 'reference':
        return run_reference(args)
    if args.kernel_only:
        return kernel_only(args)
    if args.prefill_only:
        import torch
        device = torch.device('cuda', 0)
        print(json.dumps({'prefill_only': True, **prefill_window_step(device, max(args.steps, 1), args.warmup),
                          'chunk_attention': prefill_chunk_attention(device, max(args.steps, 1), args.warmup)}),
              flush=True)
        return
    import numpy as np
    import torch
    import torch.distributed as dist
    from slimkv_b200 import _lib
    from slimkv_b200.runtime import LatentDecodeRuntime, LatentLlamaConfig, RandomWeights

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        from datetime import timedelta
        dist.init_process_group('nccl', timeout=timedelta(seconds=300))
    torch.cuda.set_device(local)
    device = torch.device('cuda', local)
    # A sequence split decodes one sequence on every rank: same inputs everywhere.
    split = args.seq_split and args.config == 5
    rng = np.random.default_rng(1234 if split else 1234 + rank)
    if split:
        from slimkv_b200.runtime import qwen25_14b_r2
        cfg = qwen25_14b_r2()
        weights = RandomWeights(cfg, device, seed=0)
        batch = 1
        tails = rng.integers(0, cfg.window, size=batch)
        history = [C5S_CONTEXT // cfg.window * (cfg.window // cfg.ratio)]
        rt = LatentDecodeRuntime(cfg, weights, history, tails, device, extra_windows=1, raw_pre=False,
                                 seq_split=True if world > 1 else None)
        metric, workload = C5S_METRIC, config5s(world, int(tails[0]))
    elif args.config == 3:
        # Config 3: r8 ranks, one Beacon per 8 raw tokens, contexts U[2048, 131072].
        cfg = LatentLlamaConfig(rank_k=160, rank_v=160, ratio=8)
        weights = RandomWeights(cfg, device, seed=0)
        batch = C3_BATCH
        ctx = rng.integers(2048, 131072 + 1, size=batch)
        history = (ctx // cfg.window) * (cfg.window // cfg.ratio)
        tails = ctx % cfg.window
        rt = LatentDecodeRuntime(cfg, weights, history, tails, device, extra_windows=1, paged=True, raw_pre=False)
        metric, workload = C3_METRIC, config3(world, ctx)
    elif args.config == 5:
        from slimkv_b200.runtime import qwen25_14b_r2
        cfg = qwen25_14b_r2()
        weights = RandomWeights(cfg, device, seed=0)
        batch = C5_BATCH
        tails = rng.integers(0, cfg.window, size=batch)
        history = [131072 // cfg.window * (cfg.window // cfg.ratio)] * batch
        backend = 'reconstruct' if args.reconstruct else 'latent'
        rt = LatentDecodeRuntime(cfg, weights, history, tails, device, extra_windows=1, raw_pre=False,
                                 backend=backend)
        metric, workload = C5_METRIC, config5(world)
        if args.reconstruct:
            metric = metric.replace('latent path', 'reconstruct path')
            workload['workload'] = workload['workload'].replace('latent path', 'reconstruct backend (Beacon K/V '
                                                                'rebuilt from latents every step, then attention)')
    else:
        cfg = LatentLlamaConfig()
        weights = RandomWeights(cfg, device, seed=0)
        batch = BATCH
        tails = rng.integers(0, cfg.window, size=BATCH)
        rt = LatentDecodeRuntime(cfg, weights, [HISTORY] * BATCH, tails, device, extra_windows=1)
        metric, workload = METRIC, config(world)
    rt.tokens.copy_(torch.from_numpy(rng.integers(0, cfg.vocab, size=batch)).to(device))
    rt.capture(warmup=2)
    for _ in range(max(args.warmup, 3)):
        rt.step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    from slimkv_b200.parallel import max_over_ranks as _max_over_ranks

    def max_over_ranks(x):
        return _max_over_ranks(x, device=device)

    # ---- device-resident timed region -------------------------------------
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    attn_bytes = 0
    start.record()
    for _ in range(args.steps):
        rt.step()
    end.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    jobs = 1 if split else world                 # a split decodes the same sequence on every rank
    value = jobs * batch / (ms / 1000.0)

    # ---- end to end through the runtime API: host tokens in, host tokens out -
    host_in = torch.from_numpy(rng.integers(0, cfg.vocab, size=batch)).pin_memory()
    host_out = torch.empty(batch, dtype=torch.int64).pin_memory()
    rt.capture_host_io(host_in, host_out)               # token copy in, step, greedy tokens out: one replay
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        host_in.copy_(rt.step_host())                   # the next step needs these tokens
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    merge_us = None
    if rt.merges:
        # The cross-GPU exchange alone: all-gather of the fp32 partials + the
        # N-part merge kernel, cycling through the layers' buffers.
        barrier()
        torch.cuda.synchronize()
        m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        m0.record()
        for i in range(cfg.layers * 4):
            rt.merges[i % cfg.layers]()
        m1.record()
        torch.cuda.synchronize()
        merge_us = max_over_ranks(m0.elapsed_time(m1) / (cfg.layers * 4)) * 1000.0

    recon = None
    if rt.recon:
        recon = reconstruct_roofline(rt, max(args.steps, 4))
    # ---- roofline of the dominant kernel: the attention launch (latent + raw
    # branches) timed alone with CUDA events on its stream; the whole fused
    # step per layer (prologue + attention + merge) is reported beside it.
    reps = max(args.steps, 8) * 4
    kernel_bytes = rt.attention_kernel_bytes()
    attn_ms = attention_kernel_time(rt, reps)
    if split:
        attn_ms = max_over_ranks(attn_ms)
    achieved = kernel_bytes / (attn_ms / 1000.0) / 1e9
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for i in range(reps):
        rt.calls[i % cfg.layers]()
    a1.record()
    torch.cuda.synchronize()
    layer_ms = a0.elapsed_time(a1) / reps
    layer_bytes = rt.attention_bytes() / cfg.layers
    peak, peak_kind = peaks()
    status = _lib.device_status(clear=True)
    rt.graph = None
    rt.graph_host = None
    prefill = None
    if not args.no_prefill and args.config == 2:
        prefill = prefill_window_step(device, max(args.steps, 10), args.warmup)
        prefill['us_per_window_layer'] = max_over_ranks(prefill['us_per_window_layer'])
        tf_peak = tensor_peak()
        prefill['roofline'] = {'bound': 'tensor', 'achieved': prefill['tflops'], 'peak': tf_peak[0],
                               'unit': 'TFLOP/s', 'frac': prefill['tflops'] / tf_peak[0], 'peak_source': tf_peak[1]}

    result = {
        'metric': metric, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
        'warmup': max(args.warmup, 3), 'ms_per_step': ms, 'higher_is_better': True,
        'scaling': 'strong' if split else 'weak',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (random N(0,0.02) weights, synthetic cache)',
        'config': workload,
        'e2e': {'value': jobs * batch / (e2e_ms / 1000.0), 'unit': UNIT, 'h2d_bytes_per_step': batch * 8,
                'd2h_bytes_per_step': batch * 8, 'ms_per_step': e2e_ms},
        'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s', 'frac': achieved / peak,
                     'peak_source': f'{peak_kind} (MEASURED_PEAKS.json hbm_gbs)' if peak_kind == 'measured'
                     else 'fallback 6650 GB/s',
                     'traffic': traffic_per_launch(kernel_bytes) if args.config == 2 else None, 'kernel': ('decode_tc_kernel' if args.config != 5 else 'decode_tc_kernel<wide> (40 heads, ranks 512)') +
                     ' (latent + raw branches, one launch per layer)', 'bytes_per_launch': kernel_bytes, 'us_per_launch': attn_ms * 1000.0,
                     'fused_step_per_layer': {'us': layer_ms * 1000.0, 'bytes': layer_bytes,
                                              'gbs': layer_bytes / (layer_ms / 1000.0) / 1e9}},
        'gpu_launches': args.steps * own_launches_per_step(rt),
        'clocks': clock_info, 'device_status': status,
    }
    if prefill is not None:
        result['prefill'] = prefill
    if recon is not None:
        # The reconstruct backend's dominant kernel is the Beacon K/V rebuild
        # (tensor-bound); the latent fused step above is the comparison.
        result['reconstruct'] = recon
        result['roofline'] = recon.pop('roofline')
        result['latent_backend_fused_step_per_layer_us'] = layer_ms * 1000.0
    if split:
        result['sequence_split'] = {
            'ranks': world, 'latent_rows_this_rank': int(rt.call_latent_len.sum().item()),
            'attention_us_per_layer_max_over_ranks': attn_ms * 1000.0,
            'merge_us_per_layer_max_over_ranks': merge_us,
            'exchange_bytes_per_rank_per_layer': rt.merges[0].send.numel() * 4 if rt.merges else 0}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config == 2:
        result['cpu_baseline'] = cpu_baseline(BATCH)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
