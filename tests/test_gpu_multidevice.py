"""GPU, two devices in one process: every kernel's opt-in to large shared memory is made per device. The same process
runs the NVFP4 GEMV, the attention and the allocation-free attention on device 0 and then on device 1, each against
the same call on device 0 (bit-identical: the kernels are deterministic). Skipped with fewer than two GPUs."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _need_two():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def test_kernels_run_on_a_second_device_in_the_same_process(cuda, xtg):
    import torch
    _need_two()
    rng = np.random.default_rng(11)
    n, k, slots, heads, kvh = 640, 1024, 1024, 8, 2
    codes = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    scales = rng.integers(0x30, 0x40, (n, k // 16), dtype=np.uint8)
    x = rng.standard_normal((8, k)).astype(np.float32)
    att = dict(q=rng.standard_normal((8, heads, 128)).astype(np.float32),
               k=rng.standard_normal((8, kvh, 128)).astype(np.float32),
               v=rng.standard_normal((8, kvh, 128)).astype(np.float32),
               k_codes=rng.integers(0, 256, kvh * slots * 128, dtype=np.uint8),
               v_codes=rng.integers(0, 256, kvh * slots * 128, dtype=np.uint8),
               k_scales=rng.uniform(0.005, 0.02, (kvh, slots)).astype(np.float32),
               v_scales=rng.uniform(0.005, 0.02, (kvh, slots)).astype(np.float32))
    results = []
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            t = {key: torch.from_numpy(val).cuda() for key, val in att.items()}
            lin = xtg.Linear([(torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda(), 1.0)], k)
            y = lin(torch.from_numpy(x).cuda())[0]
            a = xtg.attention(pos0=slots - 8, window=0, scale=1 / math.sqrt(128), splits=6, **t)
            b = xtg.attention_noalloc(pos0=slots - 8, window=0, scale=1 / math.sqrt(128), splits=6, **t)
            torch.cuda.synchronize()
            results.append((y.cpu().numpy(), a.cpu().numpy(), b.cpu().numpy()))
            lin.close()
    for r in results[1:]:
        for got, want in zip(r, results[0]):
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
