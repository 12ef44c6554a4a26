"""Multi-step decode of the native runtime against the reference model's logits.

``tests/golden/make_golden.py`` (``gen_model_decode``) ran the reference's
own SlimKV ``LlamaForCausalLM`` — two layers with the Llama-3.1-8B attention
geometry (32 / 8 heads, head_dim 128, r4 ranks 320 / 320), a 64-token Beacon
window, ratio 4, four sinks, seeded bf16-representable weights
(``cases.tiny_model_weights``) — through a 212-token prefill and 60
single-token decode steps in fp32, recording its memory after the prefill and
the logits of every decode step.  The decode crosses one window rollover and
inserts a Beacon every fourth step.

Here the runtime (``slimkv_b200.runtime``: the device Beacon schedule, cuBLAS
projections and MLP in bf16, and the fused sm_100a latent decode per layer)
is loaded with the same weights (``StateDictWeights``) and the reference's
post-prefill memory (``load_memory``) and fed the same tokens.  Every step's
bf16 logits must be within 2e-2 absolute of the reference's fp32 logits —
the logits bar of ``BASELINE.json`` — eagerly and under CUDA-graph replay.
"""
import numpy as np
import pytest
import torch

GOLDEN = 'tests/golden/reference_golden.npz'


def _runtime(dev):
    from cases import LLAMA8B, TINY_MODEL, tiny_model_weights
    from slimkv_b200.runtime import LatentDecodeRuntime, LatentLlamaConfig, StateDictWeights
    s = TINY_MODEL
    cfg = LatentLlamaConfig(vocab=s['vocab'], hidden=s['hidden'], intermediate=s['intermediate'], layers=s['layers'],
                            heads=s['heads'], kv_heads=s['kv_heads'], head_dim=s['head_dim'], rank_k=s['rank'],
                            rank_v=s['rank'], window=s['window'], ratio=s['ratio'], sink=s['sink'],
                            rope_theta=s['theta'], rope_scaling=dict(LLAMA8B['scaling']), rope_positions=4096,
                            rms_eps=s['rms_eps'])
    weights = StateDictWeights(cfg, tiny_model_weights(), dev)
    golden = np.load(GOLDEN)
    per_window = s['window'] // s['ratio']
    history = (s['prefill'] // s['window']) * per_window
    tail = s['prefill'] % s['window']
    rt = LatentDecodeRuntime(cfg, weights, [history], [tail], dev, extra_windows=2)
    layers = [{k: golden[f'model_l{i}_{k}'] for k in ('sink_k', 'sink_v', 'hist_k', 'hist_v', 'raw_k', 'raw_v',
                                                       'win_k', 'win_v')} for i in range(cfg.layers)]
    rt.load_memory(layers, golden['model_window_raw_indices'])
    return rt, golden


@pytest.mark.gpu
@pytest.mark.parametrize('graph', [False, True])
def test_runtime_logits_match_reference_model(graph):
    from cases import tiny_model_tokens
    from slimkv_b200 import _lib
    dev = torch.device('cuda', 0)
    rt, golden = _runtime(dev)
    want = golden['model_logits']
    _, steps = tiny_model_tokens()
    _lib.device_status(clear=True)
    if graph:
        # Capturing runs warm-up steps that advance the cache: rebuild the
        # state afterwards, then replay from the recorded post-prefill memory.
        rt.capture(warmup=1)
        rt2, _ = _runtime(dev)
        for c2, c in zip(rt2.caches, rt.caches):
            for k in ('raw_k_rot', 'raw_k_pre', 'raw_v', 'lat'):
                c[k].copy_(c2[k])
        rt.history.copy_(rt2.history)
        rt.tail.copy_(rt2.tail)
        del rt2
    worst, inserted = 0.0, 0
    for i, tok in enumerate(steps):
        rt.tokens.fill_(int(tok))
        logits = rt.step().clone()
        torch.cuda.synchronize()
        inserted += int(rt.query_len[0].item() == 2)
        err = (logits[0].cpu().numpy() - want[i]).__abs__().max()
        worst = max(worst, err)
        assert err <= 2e-2, f'step {i}: max |logits - reference| = {err:.3e}'
    assert _lib.device_status(clear=True) == 0
    assert inserted == 15                                  # one Beacon every fourth raw token
    assert int(rt.history[0].item()) == 64                 # the open window closed during the run
    print(f'graph={graph}: worst logit error {worst:.3e} over {len(steps)} steps')
