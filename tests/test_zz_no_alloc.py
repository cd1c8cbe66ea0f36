"""GPU: xtg_cuda_attention_noalloc (split partials in the library's fixed scratch, nothing allocated) against
xtg_cuda_attention (per-call allocation) on the same inputs, within the attention tolerance of the other GPU tests:
    |noalloc - attention| <= 2e-3 * max(|attention|, rms(attention)).
Collected last, so that it also runs after every other test in one process."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 2e-3


def close_rel(got, ref, tol=TOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = math.sqrt((ref ** 2).mean())
    worst = (np.abs(got - ref) / np.maximum(np.abs(ref), rms)).max()
    return bool(np.all(np.abs(got - ref) <= tol * np.maximum(np.abs(ref), rms))), worst


def make_case(torch, seed, slots, ring, heads=24, kvh=6, n_q=8):
    """Random int8 codes and positive scales in the library's cache layout (any bytes are valid codes), queries and
    this call's keys / values; a ring gets the slot -> position table of its most recent `slots` positions."""
    rng = np.random.default_rng(seed)
    d = 128
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    kc = t(rng.integers(0, 256, kvh * slots * d, dtype=np.uint8))
    vc = t(rng.integers(0, 256, kvh * slots * d, dtype=np.uint8))
    ks = t(rng.uniform(0.005, 0.02, (kvh, slots)).astype(np.float32))
    vs = t(rng.uniform(0.005, 0.02, (kvh, slots)).astype(np.float32))
    q = t(rng.standard_normal((n_q, heads, d)).astype(np.float32))
    k = t(rng.standard_normal((n_q, kvh, d)).astype(np.float32))
    v = t(rng.standard_normal((n_q, kvh, d)).astype(np.float32))
    if ring:
        pos0 = 8192 + 37
        rp = np.array([pos0 - 1 - ((pos0 - 1 - s) % slots) for s in range(slots)], np.int32)
        return dict(q=q, k=k, v=v, k_codes=kc, v_codes=vc, k_scales=ks, v_scales=vs, pos0=pos0, window=1024,
                    scale=1 / math.sqrt(d), ring_pos=t(rp))
    return dict(q=q, k=k, v=v, k_codes=kc, v_codes=vc, k_scales=ks, v_scales=vs, pos0=slots - 8, window=0,
                scale=1 / math.sqrt(d))


def test_noalloc_matches_attention_on_consecutive_calls(cuda, xtg):
    import torch
    # a global cache over 144 head-split pairs, then a ring over 48 pairs: the second call starts from the first
    # call's scratch contents
    cases = [(make_case(torch, 1, 4096, False), 24), (make_case(torch, 2, 1088, True), 8)]
    for case, splits in cases:
        ref = xtg.attention(splits=splits, **case).cpu().numpy()
        got = xtg.attention_noalloc(splits=splits, **case)
        torch.cuda.synchronize()
        ok, worst = close_rel(got.cpu().numpy(), ref)
        assert ok, (splits, worst)


def test_noalloc_rejects_more_pairs_than_its_scratch(cuda, xtg):
    import torch
    case = make_case(torch, 3, 4096, False)
    with pytest.raises(xtg.XtgError, match="256"):
        xtg.attention_noalloc(splits=43, **case)   # 6 KV heads x 43 splits = 258 pairs
