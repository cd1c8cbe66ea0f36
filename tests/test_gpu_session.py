"""GPU: the session behind the C ABI (xtg_cuda_open / forward / rewind / snapshot / restore / grow / debug_cache)
against the oracle's step (packs/dory/dory.cpp:467-578 order) and the NPU plugin's state rules
(npu/xtg_npu.cpp:346-447): full-step parity (identical argmax, max |d logit| <= 5e-2), verify vs sequential
agreement, rewind / snapshot / restore / tier moves, and the error paths (-1 with the state unchanged)."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
LOGIT_TOL = 5e-2


@pytest.fixture(scope="module")
def cfg(xtg):
    return dict(xtg.SMALL)


def logits_of(out, n):
    return np.stack([out[i] for i in range(n)])


@pytest.mark.parametrize("layers", [dict(n_in=1, n_rec=0, n_out=0, loops=0), dict(n_in=2, n_rec=0, n_out=0, loops=0),
                                    dict(n_in=2, n_rec=2, n_out=0, loops=1), dict(n_in=0, n_rec=4, n_out=2, loops=2)])
def test_partial_models_match_oracle(cuda, xtg, cfg, layers):
    """One attention sublayer; attention + MLP; a loop; loops without input layers: each against the oracle."""
    c = dict(cfg, **layers)
    toks = [5, 17, 900, 3, 44, 1023, 0, 256]
    ref = O.SynthDory(c, ctx=256, n_prefill=70)
    with xtg.Session(c, context=256) as s:
        s.prefill_synthetic(70)
        got = logits_of(s.forward(toks, want=2), 8)
    want = ref.step(toks)
    ref.close()
    assert np.array_equal(got.argmax(1), want.argmax(1))
    assert np.abs(got - want).max() <= LOGIT_TOL, np.abs(got - want).max()


def test_steps_match_oracle(cuda, xtg, cfg):
    steps = [[5, 17, 900, 3, 44, 1023, 0, 256], [8, 9, 10, 11, 12, 13, 14, 15], [600, 601, 2], [4095]]
    ref = O.SynthDory(cfg, ctx=512, n_prefill=100)
    with xtg.Session(cfg, context=512) as s:
        s.prefill_synthetic(100)
        for toks in steps:
            got = logits_of(s.forward(toks, want=2), len(toks))
            want = ref.step(toks)
            assert np.array_equal(got.argmax(1), want.argmax(1))
            assert np.abs(got - want).max() <= LOGIT_TOL, np.abs(got - want).max()
            assert s.argmax(8) == list(want.argmax(1))
        assert s.pos() == ref.n_past == 100 + 8 + 8 + 3 + 1
        # the prefilled part of the caches is the oracle's, byte for byte; the new rows decode close to it
        for inst in (0, 1):
            kc, vc, ks, vs, ring = ref.cache(inst)
            dk = s.debug_cache(inst, 0).transpose(2, 0, 1)   # [slots][h][d]
            dv = s.debug_cache(inst, 1).transpose(1, 0, 2)
            dks = s.debug_cache(inst, 2).T
            if not ring:
                assert np.array_equal(dk[:100], kc[:100]) and np.array_equal(dv[:100], vc[:100])
                assert np.array_equal(dks[:100], ks[:100])
                new = slice(100, 120)
                kd = dk[new].view(np.int8).astype(np.float32) * dks[new][..., None]
                kr = kc[new].view(np.int8).astype(np.float32) * ks[new][..., None]
                assert np.abs(kd - kr).max() < 0.05


def test_verify_matches_sequential(cuda, xtg, cfg):
    toks = [31, 32, 33, 34, 35, 36, 37, 38]
    with xtg.Session(cfg, context=512) as a, xtg.Session(cfg, context=512) as b:
        a.prefill_synthetic(200)
        b.prefill_synthetic(200)
        va = logits_of(a.forward(toks, want=2), 8)
        vb = np.stack([b.forward([t], want=1)[0] for t in toks])
        assert np.array_equal(va.argmax(1), vb.argmax(1))
        assert np.abs(va - vb).max() <= LOGIT_TOL


def test_forward_is_deterministic_and_rewind_replays(cuda, xtg, cfg):
    with xtg.Session(cfg, context=512) as s:
        s.prefill_synthetic(150)
        a = logits_of(s.forward([1, 2, 3, 4, 5, 6, 7, 8], want=2), 8)
        assert s.rewind(150)
        b = logits_of(s.forward([1, 2, 3, 4, 5, 6, 7, 8], want=2), 8)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_rewind_rules(cuda, xtg, cfg):
    ring, window = cfg["ring"], cfg["window"]
    with xtg.Session(cfg, context=512) as s:
        s.prefill_synthetic(300)
        for _ in range(3):
            s.forward([7] * 8, want=0)
        n = s.pos()
        assert not s.rewind(n + 1) and s.pos() == n
        assert not s.rewind(-1) and s.pos() == n
        lowest = n - ring + window - 1   # the ring still holds window - 1 positions before it
        assert not s.rewind(lowest - 1) and s.pos() == n
        assert s.rewind(lowest) and s.pos() == lowest
        assert s.rewind(lowest)


def test_snapshot_restore(cuda, xtg, cfg):
    with xtg.Session(cfg, context=512, snapshots=2) as s:
        assert s.snapshot_slots() == 2 and s.snapshot_pos(0) == -1 and s.snapshot_pos(5) == -1
        assert not s.restore(0)
        s.prefill_synthetic(120)
        s.forward([9] * 8, want=0)
        s.snapshot(1)
        p = s.pos()
        assert s.snapshot_pos(1) == p
        after = logits_of(s.forward(list(range(40, 48)), want=2), 8)
        for _ in range(20):   # far past the ring's slack: only the snapshot brings position p back
            s.forward([3] * 8, want=0)
        assert not s.rewind(p)
        assert s.restore(1) and s.pos() == p
        again = logits_of(s.forward(list(range(40, 48)), want=2), 8)
        assert np.array_equal(after.view(np.uint32), again.view(np.uint32))
        # a forward below a snapshot's position drops it
        s.snapshot(0)
        q = s.pos()
        assert s.rewind(q - 4)
        s.forward([1], want=0)
        assert s.snapshot_pos(0) == -1


def test_grow_moves_tier_bit_exactly(cuda, xtg, cfg):
    toks1, toks2 = list(range(100, 108)), list(range(200, 208))
    with xtg.Session(cfg, context=256) as small, xtg.Session(cfg, context=1024) as big:
        small.prefill_synthetic(180)
        big.prefill_synthetic(180)
        small.forward(toks1, want=0)
        big.forward(toks1, want=0)
        with pytest.raises(xtg.XtgError):
            small.grow("128")                    # cannot hold pos(): the session keeps its tier
        assert small.info()["context"] == 256
        small.grow("1k")
        assert small.info()["context"] == 1024 and small.pos() == big.pos()
        a = logits_of(small.forward(toks2, want=2), 8)
        b = logits_of(big.forward(toks2, want=2), 8)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        g_small = small.debug_cache(1, 0)
        g_big = big.debug_cache(1, 0)
        assert np.array_equal(g_small[:, :, :204], g_big[:, :, :204])


def test_tiers_fit_up_and_down(cuda, xtg, cfg):
    """Tiers over a real session (NpuModel::fit, npu.cpp:181-198): a prompt past the first tier moves the session up
    before the forward, logits bit-identical to a session opened at the large tier; after a restore to a short
    prefix (a snapshot taken at 64 positions, kept across the move) the next forward moves it down again, still
    bit-identical."""
    prompt = [(7 * i + 3) % cfg["vocab"] for i in range(300)]
    nxt = list(range(40, 48))
    with xtg.Session(cfg, context=256) as s, xtg.Session(cfg, context=1024) as big:
        t = s.tiers([256, 512, 1024])
        a0 = logits_of(t.forward(prompt[:64], want=2), 64)
        b0 = logits_of(big.forward(prompt[:64], want=2), 64)
        s.snapshot(0)
        big.snapshot(0)
        a = np.concatenate([a0, logits_of(t.forward(prompt[64:], want=2), 236)])
        b = np.concatenate([b0, logits_of(big.forward(prompt[64:], want=2), 236)])
        assert t.moves == [512] and s.info()["context"] == 512
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert s.snapshot_pos(0) == 64 and s.restore(0) and big.restore(0)
        assert s.pos() == 64
        a = logits_of(t.forward(nxt, want=2), 8)
        b = logits_of(big.forward(nxt, want=2), 8)
        assert t.moves == [512, 256] and s.info()["context"] == 256
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_head_dim_256_matches_oracle(cuda, xtg, cfg):
    """The real Dory 4B's head shape (head_dim 256, 4 q heads per KV head) at the small widths: verify steps against
    the oracle (the q|k|v preparation kernel after the projection, the 256-dim attention and combine), then a tier
    move and a snapshot restore bit-exact, and verify against sequential decoding."""
    c = dict(cfg, head_dim=256, seed=21)
    steps = [[5, 17, 900, 3, 44, 1023, 0, 256], [8, 9, 10], [4000, 1, 2, 3, 4, 5, 6, 7]]
    ref = O.SynthDory(c, ctx=256, n_prefill=150)
    with xtg.Session(c, context=256) as s, xtg.Session(c, context=512) as big:
        s.prefill_synthetic(150)
        big.prefill_synthetic(150)
        for toks in steps:
            got = logits_of(s.forward(toks, want=2), len(toks))
            want = ref.step(toks)
            assert np.array_equal(got.argmax(1), want.argmax(1))
            assert np.abs(got - want).max() <= LOGIT_TOL, np.abs(got - want).max()
            big.forward(toks, want=0)
        s.snapshot(0)
        s.grow("512")
        a = logits_of(s.forward([7, 8, 9], want=2), 3)
        b = logits_of(big.forward([7, 8, 9], want=2), 3)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        p = s.snapshot_pos(0)
        assert s.restore(0) and s.pos() == p
        seq = np.stack([s.forward([t], want=1)[0] for t in [7, 8, 9]])
        assert np.array_equal(seq.argmax(1), a.argmax(1)) and np.abs(seq - a).max() <= LOGIT_TOL
    ref.close()


def test_error_paths_leave_state_unchanged(cuda, xtg, cfg):
    with xtg.Session(cfg, context=128) as s:
        s.prefill_synthetic(100)
        with pytest.raises(xtg.XtgError, match="out of range"):
            s.forward([1, cfg["vocab"]], want=0)
        assert s.pos() == 100
        with pytest.raises(xtg.XtgError, match="context full"):
            s.forward([1] * 29, want=0)
        assert s.pos() == 100
        s.forward([1] * 28, want=0)
        assert s.pos() == 128
        assert s.debug_cache(999, 0) is None
        info = s.info()
        assert info["decode_ar"] == 8 and info["ring_slots"] == cfg["ring"] and info["sliding_window"] == cfg["window"]
    with pytest.raises(xtg.XtgError):
        xtg.Session(cfg, context=100)            # not a multiple of 64
    with pytest.raises(xtg.XtgError):
        xtg.Session(dict(cfg, head_dim=64))      # the kernels are written for head_dim 128


def test_topk_and_sampling_from_the_step(cuda, xtg, cfg):
    """xtg_cuda_topk on the last step's logits equals the oracle's top-k of the logits the callback returned, and a
    draw from the candidates equals Sampler::sample's (restated) on the whole row wherever the candidates decide."""
    toks = [5, 17, 900, 3, 44, 1023, 0, 256]
    with xtg.Session(cfg, context=256) as s:
        s.prefill_synthetic(70)
        out = logits_of(s.forward(toks, want=2), 8)
        assert s.argmax(8) == [int(np.argmax(r)) for r in out]
        for k, temp in ((1, 1.0), (64, 0.8), (1024, 1.0)):
            idx, val, mx, tot = s.topk(k, temp)
            assert idx.shape == (8, k)
            for r in range(8):
                ri, rv = O.topk(out[r], k)
                np.testing.assert_array_equal(idx[r], ri)
                np.testing.assert_array_equal(val[r], rv)
                assert mx[r] == out[r].max()
        idx, val, mx, tot = s.topk(1024, 0.8)
        decided = 0
        for r in range(8):
            for (tk, tp, mp) in ((40, 1.0, 0.0), (0, 0.9, 0.0), (0, 1.0, 0.05), (20, 0.8, 0.01)):
                for u in (0.0, 0.13, 0.5, 0.77, 0.999):
                    got = xtg.sample_candidates(idx[r], val[r], mx[r], tot[r], cfg["vocab"], 0.8, tk, tp, mp, u)
                    if got != -2:
                        decided += 1
                        assert got == O.sample(out[r], 0.8, tk, tp, mp, u)
        assert decided > 0
        with pytest.raises(xtg.XtgError):
            s.topk(0)


def test_sessions_over_shared_weights(cuda, xtg, cfg):
    """xtg_cuda_open_shared: sessions over one weight set (one shared from another, with its own tier) stepping at
    the same time from their own threads give the logits of an independent session bit for bit, and keep the
    weights after the owner is closed."""
    import threading
    steps = [[5, 17, 900, 3, 44, 1023, 0, 256], [9, 10]]
    with xtg.Session(cfg, context=256) as ref:
        ref.prefill_synthetic(70)
        want = [logits_of(ref.forward(t, want=2), len(t)) for t in steps]
    a = xtg.Session(cfg, context=256)
    b = xtg.Session.shared(a, context=256)
    c = xtg.Session.shared(b, context=512)
    try:
        assert b.info()["weight_bytes"] == c.info()["weight_bytes"] == a.info()["weight_bytes"]
        assert c.info()["context"] == 512
        for s in (a, b, c):
            s.prefill_synthetic(70)
        got = {}

        def run(name, s):
            got[name] = logits_of(s.forward(steps[0], want=2), 8)

        th = [threading.Thread(target=run, args=(n, s)) for n, s in (("a", a), ("b", b), ("c", c))]
        for t in th:
            t.start()
        for t in th:
            t.join()
        for n in "abc":
            np.testing.assert_array_equal(got[n], want[0], err_msg=n)
        a.close()   # the owner goes first: b and c still hold the weights
        for s in (b, c):
            np.testing.assert_array_equal(logits_of(s.forward(steps[1], want=2), 2), want[1])
    finally:
        for s in (a, b, c):
            s.close()
    with pytest.raises(xtg.XtgError):
        with xtg.Session(cfg, context=256) as o:
            xtg.Session.shared(o, context=256, kv_world=2, kv_rank=0, nccl_id="00" * 128)


def test_forward_batch_matches_one_by_one(cuda, xtg, cfg):
    """xtg_cuda_forward_batch over sessions with different token counts (one of them two steps, one none) gives
    each session's logits of a forward of its own, bit for bit, and advances each position; a refused call (a
    session twice, a token out of range) changes nothing."""
    lists = [[5, 17, 900, 3, 44, 1023, 0, 256], [8, 9, 10], list(range(100, 111)), []]
    with xtg.Session(cfg, context=256) as owner:
        owner.prefill_synthetic(70)
        # batch=0: verify steps of each session's own graph (8 rows at a time), all in flight at once in the batch
        # call (the batched step and the prompt chunks are tested below)
        singles = [xtg.Session.shared(owner, context=256, batch=0) for _ in lists]
        batch = [xtg.Session.shared(owner, context=256, batch=0) for _ in lists]
        try:
            want = []
            for s, t in zip(singles, lists):
                s.prefill_synthetic(70)
                want.append(s.forward(t, want=2) if t else {})
            for s in batch:
                s.prefill_synthetic(70)
            # the session given no tokens keeps a snapshot past its position (as a forward of nothing does)
            batch[3].forward([1] * 8, want=0)
            batch[3].snapshot(0)
            assert batch[3].rewind(70) and batch[3].snapshot_pos(0) == 78
            with pytest.raises(xtg.XtgError):
                xtg.forward_batch([batch[0], batch[0]], [lists[0], lists[1]])
            with pytest.raises(xtg.XtgError):
                xtg.forward_batch(batch[:2], [lists[0], [cfg["vocab"]]])
            assert [s.pos() for s in batch] == [70] * len(batch)
            got = xtg.forward_batch(batch, lists, want=2)
            for i, t in enumerate(lists):
                assert sorted(got[i]) == sorted(want[i]) == list(range(len(t)))
                for r in want[i]:
                    np.testing.assert_array_equal(got[i][r], want[i][r], err_msg=f"session {i} row {r}")
                assert batch[i].pos() == 70 + len(t)
            assert batch[3].snapshot_pos(0) == 78
        finally:
            for s in singles + batch:
                s.close()


@pytest.mark.parametrize("hd", [128, 256])
def test_forward_batch_batched_step(cuda, xtg, cfg, hd):
    """xtg_cuda_forward_batch over sessions that share one weight set runs them as one batched step (every projection
    one tcgen05 GEMM over all their rows): nine sessions (a group of 8 and a group of 1) at different positions, with
    different token counts (one of two rounds, one of none), each within the step tolerance of a forward of its own
    (identical argmax), the first also against the oracle; positions advance, and a second call after rewinds gives
    the same logits again. At head_dim 128 and 256 (the real Dory 4B's)."""
    cfg = dict(cfg, head_dim=hd)
    lists = [[5, 17, 900, 3, 44, 1023, 0, 256], [8, 9, 10], list(range(100, 111)), [], [4095], [1, 2, 3, 4],
             [700] * 8, [9, 8, 7, 6, 5], [11, 12]]
    pre = [70, 90, 64, 100, 75, 128, 81, 99, 70]
    with xtg.Session(cfg, context=512) as owner:
        sess = [xtg.Session.shared(owner, context=512) for _ in lists]
        singles = [xtg.Session.shared(owner, context=512) for _ in lists]
        try:
            for s, p in zip(sess + singles, pre + pre):
                s.prefill_synthetic(p)
            want = [s.forward(t, want=2) if t else {} for s, t in zip(singles, lists)]
            got = xtg.forward_batch(sess, lists, want=2)
            for i, t in enumerate(lists):
                assert sorted(got[i]) == list(range(len(t)))
                assert sess[i].pos() == pre[i] + len(t)
                if not t:
                    continue
                g, w = logits_of(got[i], len(t)), logits_of(want[i], len(t))
                assert np.array_equal(g.argmax(1), w.argmax(1)), i
                assert np.abs(g - w).max() <= LOGIT_TOL, (i, np.abs(g - w).max())
            ref = O.SynthDory(cfg, ctx=512, n_prefill=pre[0])
            oracle = ref.step(lists[0])
            ref.close()
            g0 = logits_of(got[0], 8)
            assert np.array_equal(g0.argmax(1), oracle.argmax(1))
            assert np.abs(g0 - oracle).max() <= LOGIT_TOL
            assert sess[0].argmax(8) == list(oracle.argmax(1))
            for s, p in zip(sess, pre):
                assert s.rewind(p)
            again = xtg.forward_batch(sess, lists, want=2)
            for i, t in enumerate(lists):
                for r in range(len(t)):
                    np.testing.assert_array_equal(again[i][r], got[i][r], err_msg=f"session {i} row {r}")
        finally:
            for s in sess + singles:
                s.close()


@pytest.mark.parametrize("hd,window", [(128, 64), (256, 64), (128, 24)])
def test_prompt_chunks_match_oracle_and_verify_steps(cuda, xtg, cfg, hd, window):
    """A forward of more than decode_rows tokens runs prompt chunks of up to 64 rows through the batched step, with
    the arithmetic of the reference's multi-row attention (packs/dory/dory.cpp:825-929 attend_rows,
    engine/src/kv.cpp:166-286): every row attends the cache below the chunk's first position and the chunk's own rows
    up to itself, unquantized. 100 tokens (a chunk of 64, one of 36) within the step tolerance of the oracle run on
    the same chunks (identical argmax); the same tokens as the session's 8-row verify steps (batch=0) against the
    oracle stepped 8 rows at a time; the position and the next verify step agree too. At head_dim 128 and 256, and
    with a window of 24 (the same 128-slot ring), where a chunk's later rows no longer see its first ones."""
    cfg = dict(cfg, head_dim=hd, window=window)
    toks = [(37 * i + 11) % cfg["vocab"] for i in range(100)]
    wants, nxts = {}, {}
    for name, cuts in (("chunks", (0, 64, 100)), ("steps", tuple(range(0, 100, 8)) + (100,))):
        ref = O.SynthDory(cfg, ctx=512, n_prefill=70)
        wants[name] = np.concatenate([ref.step(toks[o:e]) for o, e in zip(cuts, cuts[1:])])
        nxts[name] = ref.step([5, 6, 7, 8])
        ref.close()
    with xtg.Session(cfg, context=512) as a, xtg.Session(cfg, context=512, batch=0) as b:
        assert a.info()["prefill_ar"] == 64
        a.prefill_synthetic(70)
        b.prefill_synthetic(70)
        ga = logits_of(a.forward(toks, want=2), 100)
        gb = logits_of(b.forward(toks, want=2), 100)
        assert a.pos() == b.pos() == 170
        for got, want in ((ga, wants["chunks"]), (gb, wants["steps"])):
            assert np.array_equal(got.argmax(1), want.argmax(1))
            assert np.abs(got - want).max() <= LOGIT_TOL, np.abs(got - want).max()
        assert a.argmax(8)[:4] == list(wants["chunks"][96:].argmax(1))
        last = a.forward(toks[:1], want=1)   # one more row: a single verify step after the chunks
        assert sorted(last) == [0]
        assert a.rewind(170) and b.rewind(170)   # the oracle's state: 170 positions
        na = logits_of(a.forward([5, 6, 7, 8], want=2), 4)
        nb = logits_of(b.forward([5, 6, 7, 8], want=2), 4)
        for got, want in ((na, nxts["chunks"]), (nb, nxts["steps"])):
            assert np.array_equal(got.argmax(1), want.argmax(1))
            assert np.abs(got - want).max() <= LOGIT_TOL
        assert a.pos() == 174
