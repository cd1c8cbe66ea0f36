"""CPU: the sampling path's checker and host logic.

* The oracle's top-k and Sampler::sample restatements are pinned to the reference's own argmax, top_logprobs and
  Sampler(seed).sample (tests/golden/sampling.npz, made by tests/golden/make_golden.py from engine/src/sampler.cpp
  compiled here), each draw given as the first uniform value of that seed's engine.
* xtg_cuda_sample_candidates (host code of the library, no device work) decides from k candidates exactly as the
  reference does from the whole row, or answers -2 where the candidates cannot decide.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import make_golden as G  # noqa: E402
import oracle  # noqa: E402

FIX = np.load(os.path.join(ROOT, "tests", "golden", "sampling.npz"))


def _total(row, temperature):
    """The device's normaliser: float exp((l - max) / T), summed in double."""
    inv_t = np.float32(1.0) / np.float32(temperature if temperature > 0 else 1.0)
    return float(np.sum(np.exp((row - row.max()) * inv_t).astype(np.float32).astype(np.float64)))


def _needs_full_row(row, k, t, tk, tp, mp):
    """Where the reference's Sampler::sample reaches past the k most likely entries: no filter (a draw over the
    whole row in index order), or a top_p / min_p filter whose kept mass or entries run past the sorted head."""
    if t <= 0 or (0 < tk <= k):
        return False
    if tk == 0 and tp >= 1.0 and mp <= 0.0:
        return True
    inv_t = np.float32(1.0) / np.float32(t)
    w = np.sort(np.exp((row - row.max()) * inv_t).astype(np.float32))[::-1].astype(np.float64)
    total = w.sum()
    head = w[:k]
    past_top_p = tp < 1.0 and head.sum() < total * tp
    past_min_p = mp > 0.0 and np.count_nonzero(w >= mp * w[0]) >= k
    return len(row) > k and (past_top_p or past_min_p)


@pytest.mark.parametrize("vocab", G.SAMPLING_VOCABS)
def test_oracle_topk_and_argmax_pinned(vocab):
    x = G.sampling_inputs(vocab)
    for r in range(G.SAMPLING_ROWS):
        idx, val = oracle.topk(x[r], G.SAMPLING_TOPK)
        np.testing.assert_array_equal(idx, FIX[f"v{vocab}_top_idx"][r])
        lse = float(x[r].max()) + np.log(np.sum(np.exp((x[r] - x[r].max()).astype(np.float64))))
        np.testing.assert_allclose(val - lse, FIX[f"v{vocab}_top_lp"][r], rtol=0, atol=2e-5)
        assert idx[0] == FIX[f"v{vocab}_argmax"][r]


@pytest.mark.parametrize("vocab", G.SAMPLING_VOCABS)
def test_oracle_sample_pinned(vocab):
    x = G.sampling_inputs(vocab)
    tok, us = FIX[f"v{vocab}_tokens"], FIX[f"v{vocab}_u"]
    for r in range(G.SAMPLING_ROWS):
        for pi, (t, k, tp, mp) in enumerate(G.SAMPLING_PARAMS):
            for d in range(G.SAMPLING_DRAWS):
                assert oracle.sample(x[r], t, k, tp, mp, us[r, pi, d]) == tok[r, pi, d], (vocab, r, pi, d)


@pytest.mark.parametrize("vocab", G.SAMPLING_VOCABS)
def test_sample_candidates_matches_reference(xtg, vocab):
    x = G.sampling_inputs(vocab)
    tok, us = FIX[f"v{vocab}_tokens"], FIX[f"v{vocab}_u"]
    k = min(vocab, 1024)
    decided = undecided = 0
    for r in range(G.SAMPLING_ROWS):
        idx, val = oracle.topk(x[r], k)
        for pi, (t, tk, tp, mp) in enumerate(G.SAMPLING_PARAMS):
            total = _total(x[r], t)
            for d in range(G.SAMPLING_DRAWS):
                got = xtg.sample_candidates(idx, val, float(x[r].max()), total, vocab, t, tk, tp, mp, us[r, pi, d])
                if got == -2:
                    undecided += 1
                    assert _needs_full_row(x[r], k, t, tk, tp, mp), (vocab, r, pi, d)
                else:
                    decided += 1
                    assert got == tok[r, pi, d], (vocab, r, pi, d, got, tok[r, pi, d])
    assert decided > 0 and undecided >= G.SAMPLING_ROWS * G.SAMPLING_DRAWS   # the no-filter setting at least


def test_sample_candidates_needs_enough_candidates(xtg):
    x = G.sampling_inputs(4096)[0]
    idx, val = oracle.topk(x, 16)
    total = _total(x, 1.0)
    mx = float(x.max())
    assert xtg.sample_candidates(idx, val, mx, total, 4096, 1.0, 40, 1.0, 0.0, 0.3) == -2    # top_k above k
    assert xtg.sample_candidates(idx, val, mx, total, 4096, 1.0, 0, 0.9, 0.0, 0.3) == -2     # top_p: k < 1024
    assert xtg.sample_candidates(idx, val, mx, total, 4096, 0.0, 0, 1.0, 0.0, 0.3) == idx[0]  # greedy
    assert xtg.sample_candidates(idx, val, mx, total, 4096, 1.0, 8, 1.0, 0.0, 1.5) == -1     # u outside [0, 1)
    assert xtg.sample_candidates(idx, val, mx, total, 4096, 1.0, 8, 1.0, 0.0, 0.0) == idx[0]
