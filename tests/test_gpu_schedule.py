"""Device decode schedule vs the oracle's restatement of ``LlamaMemory._step``.

Each sequence starts from its own prompt length (ragged window offsets); for
every step the device metadata (query length, raw keys, latents, query
position) must equal the oracle's schedule exactly, across window rollovers.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('window,ratio,sink', [(1024, 4, 4), (16, 4, 1), (64, 8, 2)])
def test_device_schedule_matches_oracle(window, ratio, sink):
    from slimkv_b200 import kernels
    rng = np.random.default_rng(window + ratio)
    B = 6
    windows = rng.integers(1, 4, size=B)
    tails = rng.integers(0, window, size=B)
    prompts = windows * window + tails
    per_window = window // ratio
    scheds = []
    for n in prompts:
        s = oracle.FastDecodeSchedule(window, ratio, sink)
        s.prefill(int(n))
        scheds.append(s)
    dev = torch.device('cuda')
    i32 = lambda x: torch.tensor(np.asarray(x), dtype=torch.int32, device=dev)
    history = i32([s.history for s in scheds])
    tail = i32([s.raw for s in scheds])
    assert np.array_equal(history.cpu().numpy(), windows * per_window)
    raw_len, latent_len, query_len = (torch.zeros(B, dtype=torch.int32, device=dev) for _ in range(3))
    qpos = torch.zeros(B, 2, dtype=torch.int32, device=dev)
    steps = 3 * window + 7
    got = []
    for _ in range(steps):
        kernels.decode_schedule(history, tail, raw_len, latent_len, query_len, qpos, sink, window, ratio)
        got.append(torch.stack([query_len, raw_len, latent_len, qpos[:, 0], qpos[:, 1]]).cpu())
    got = torch.stack(got).numpy()
    for i in range(steps):
        for b, s in enumerate(scheds):
            r = s.decode()
            size = r['size']
            want = (1 + size, r['sink'] + r['raw'] + 1, r['history'] + r['window'] + size,
                    r['positions'] - 1 - size, r['positions'] - size)
            assert tuple(got[i, :, b]) == want, (i, b, tuple(got[i, :, b]), want)
