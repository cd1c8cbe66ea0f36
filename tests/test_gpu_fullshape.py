"""GPU: the benchmarked step itself against the oracle, at its full shape.

BASELINE config 3 is the synthetic Dory-3072 step: hidden 3072, 24 q / 6 KV heads of 128, FFN 9216, vocab 131072,
4 + 40 x 2 + 4 sublayers (11 global and 33 sliding attention sublayers, 44 MLP), 1088-slot rings over a window of
1024, RoPE theta 1e4 (sliding) / 1e7 (global), the 8K tier with 8184 positions prefilled. The session that bench.py
times (CUDA graph, programmatic dependent launch) runs one 8-row verify step; the oracle's restatement of
DorySession::sublayer / forward (packs/dory/dory.cpp:467-578) runs the same step on the same seeded weights and
caches. The gate is north_star's: identical argmax and max |d logit| <= 5e-2 for every row. The same shape then
checks verify against sequential decoding (the 8 rows one at a time after a rewind) and the device argmax.

The oracle needs a minute or two of host time on the GPU box's cores (3.35 GB of weights generated and quantised,
one step over them); the module builds it once."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
LOGIT_TOL = 5e-2
PREFILL = 8184
TOKENS = [17, 4242, 99, 131071, 5, 70000, 123, 2048]


@pytest.fixture(scope="module")
def oracle_logits(xtg):
    ref = O.SynthDory(dict(xtg.DORY_3072), ctx=8192, n_prefill=PREFILL)
    try:
        return ref.step(TOKENS)
    finally:
        ref.close()


@pytest.fixture(scope="module")
def session(cuda, xtg):
    s = xtg.Session(dict(xtg.DORY_3072), context=8192)
    s.prefill_synthetic(PREFILL)
    yield s
    s.close()


def rows(out, n):
    return np.stack([out[i] for i in range(n)])


def test_config3_step_matches_oracle(session, oracle_logits):
    got = rows(session.forward(TOKENS, want=2), 8)
    diff = np.abs(got - oracle_logits).max()
    assert np.array_equal(got.argmax(1), oracle_logits.argmax(1)), (got.argmax(1), oracle_logits.argmax(1))
    assert diff <= LOGIT_TOL, diff
    assert session.argmax(8) == list(oracle_logits.argmax(1))
    assert session.pos() == PREFILL + 8


def test_config3_verify_matches_sequential(session, oracle_logits):
    """The 8 rows one step at a time from the same state give the verify step's logits (the rings, the global
    caches and the positions of one-row steps against one eight-row step)."""
    assert session.rewind(PREFILL)
    seq = np.stack([session.forward([t], want=1)[0] for t in TOKENS])
    assert np.array_equal(seq.argmax(1), oracle_logits.argmax(1))
    assert np.abs(seq - oracle_logits).max() <= LOGIT_TOL


def test_config3_bench_replay_matches_oracle(session, oracle_logits):
    """xtg_cuda_bench replays the same step graph that the bench times: its argmax is the oracle's."""
    assert session.rewind(PREFILL)
    session.bench(TOKENS, 2)
    assert session.argmax(8) == list(oracle_logits.argmax(1))


# ---- the real Dory 4B's shape: head_dim 256, 16 q / 4 KV heads, hidden 2560, FFN 7168 ----

# every width and the 8K tier; 12 sublayers of the 112, a global and a sliding attention sublayer in the loop
DORY_4B_CUT = dict(n_in=2, n_rec=4, n_out=2, loops=2, global_every=2)


@pytest.fixture(scope="module")
def dory4b(cuda, xtg):
    """(session, oracle logits) for one 8-row step of the Dory 4B shape (synthetic weights, 1088-slot rings, vocab
    131072) over 8184 prefilled positions."""
    cfg = dict(xtg.DORY_4B, **DORY_4B_CUT)
    ref = O.SynthDory(cfg, ctx=8192, n_prefill=PREFILL)
    try:
        want = ref.step(TOKENS)
    finally:
        ref.close()
    s = xtg.Session(cfg, context=8192)
    s.prefill_synthetic(PREFILL)
    yield s, want
    s.close()


def test_dory4b_step_matches_oracle(dory4b):
    s, want = dory4b
    got = rows(s.forward(TOKENS, want=2), 8)
    assert np.array_equal(got.argmax(1), want.argmax(1)), (got.argmax(1), want.argmax(1))
    assert np.abs(got - want).max() <= LOGIT_TOL, np.abs(got - want).max()
    assert s.info()["kv_bytes"] > 0 and s.pos() == PREFILL + 8


def test_dory4b_verify_matches_sequential(dory4b):
    s, want = dory4b
    assert s.rewind(PREFILL)
    seq = np.stack([s.forward([t], want=1)[0] for t in TOKENS])
    assert np.array_equal(seq.argmax(1), want.argmax(1))
    assert np.abs(seq - want).max() <= LOGIT_TOL
