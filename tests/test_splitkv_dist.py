"""CPU: the batch-1 split-KV decomposition across processes, run as two gloo ranks on 127.0.0.1.

The step's global-layer attention over GPUs works like this: the cache's 64-slot chunks are cut into
splits_total = splits x world parts (part s covers chunks [n s / S, n (s + 1) / S)), process r computes parts
r splits .. (r + 1) splits - 1, merges them into one (max m, sum l, o relative to m) per query row and head, the
processes exchange those, every process merges them in rank order, and the step's own keys are added last. Here the
same steps in numpy, with the exchange as a gloo all-gather, must give the oracle's attention over the whole cache --
including a rank whose parts are all empty (a short cache)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HEADS, KVH, D, NQ = 4, 2, 128, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(pos0, seed=5):
    import oracle
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((NQ, HEADS, D)).astype(np.float32)
    k = rng.standard_normal((NQ, KVH, D)).astype(np.float32)
    v = rng.standard_normal((NQ, KVH, D)).astype(np.float32)
    kc, ks = oracle.kv_encode(oracle.KV_I8, rng.standard_normal((pos0 * KVH, D)).astype(np.float32))
    vc, vs = oracle.kv_encode(oracle.KV_I8, rng.standard_normal((pos0 * KVH, D)).astype(np.float32))
    return q, k, v, kc.reshape(pos0, KVH, D), vc.reshape(pos0, KVH, D), ks.reshape(pos0, KVH), vs.reshape(pos0, KVH)


def _rank_part(q, ck, cv, pos0, scale, rank, world, splits):
    """This rank's merged cached part: m [NQ, HEADS], l [NQ, HEADS], o [NQ, HEADS, D] (o relative to m)."""
    keys = ck.astype(np.float32)
    vals = cv.astype(np.float32)
    nchunks, stot = (pos0 + 63) // 64, splits * world
    m = np.full((NQ, HEADS), -np.inf, np.float32)
    l = np.zeros((NQ, HEADS), np.float32)
    o = np.zeros((NQ, HEADS, D), np.float32)
    group = HEADS // KVH
    for sidx in range(rank * splits, (rank + 1) * splits):
        cb, ce = nchunks * sidx // stot, nchunks * (sidx + 1) // stot
        lo, hi = 64 * cb, min(64 * ce, pos0)
        if hi <= lo:
            continue
        for h in range(HEADS):
            kh = h // group
            s = q[:, h, :] @ keys[lo:hi, kh, :].T * scale                      # [NQ, keys]
            ms = s.max(axis=1)
            p = np.exp(s - ms[:, None])
            ls, os_ = p.sum(axis=1), p @ vals[lo:hi, kh, :]
            mn = np.maximum(m[:, h], ms)
            wa = np.where(m[:, h] == -np.inf, 0.0, np.exp(m[:, h] - mn))
            wb = np.exp(ms - mn)
            l[:, h] = l[:, h] * wa + ls * wb
            o[:, h] = o[:, h] * wa[:, None] + os_ * wb[:, None]
            m[:, h] = mn
    return m, l, o


def _merge_and_finish(parts, q, k, v, scale):
    """Rank-order merge of the processes' parts, then the step's own keys j <= i (unquantized)."""
    ms = np.stack([p[0] for p in parts])
    M = ms.max(axis=0)
    w = np.where(ms == -np.inf, 0.0, np.exp(ms - M[None]))
    L = sum(w[r] * parts[r][1] for r in range(len(parts)))
    O = sum(w[r][..., None] * parts[r][2] for r in range(len(parts)))
    out = np.zeros((NQ, HEADS, D), np.float32)
    group = HEADS // KVH
    for i in range(NQ):
        for h in range(HEADS):
            kh = h // group
            own = np.array([q[i, h] @ k[j, kh] * scale for j in range(i + 1)])
            mall = max(own.max(), M[i, h])
            cs = 0.0 if M[i, h] == -np.inf else np.exp(M[i, h] - mall)
            pj = np.exp(own - mall)
            num = O[i, h] * cs + (pj[:, None] * v[: i + 1, kh]).sum(axis=0)
            out[i, h] = num / (L[i, h] * cs + pj.sum())
    return out


def _rank(rank, world, port, pos0, splits, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, kc, vc, ks, vs = _inputs(pos0)
        import oracle
        ck = oracle.kv_decode(oracle.KV_I8, kc, ks)
        cv = oracle.kv_decode(oracle.KV_I8, vc, vs)
        scale = 1.0 / np.sqrt(D)
        m, l, o = _rank_part(q, ck, cv, pos0, scale, rank, world, splits)
        mine = torch.from_numpy(np.concatenate([m.ravel(), l.ravel(), o.ravel()]))
        got = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(got, mine)
        nm = NQ * HEADS
        parts = [(g[:nm].numpy().reshape(NQ, HEADS), g[nm:2 * nm].numpy().reshape(NQ, HEADS),
                  g[2 * nm:].numpy().reshape(NQ, HEADS, D)) for g in got]
        out[rank] = (_merge_and_finish(parts, q, k, v, scale), bool(np.all(m == -np.inf)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pos0,splits", [(1000, 3), (64, 2)])
def test_split_kv_decomposition_matches_oracle(pos0, splits):
    import oracle
    world = 2
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank, args=(world, _free_port(), pos0, splits, out), nprocs=world, join=True)
        res = dict(out)
    q, k, v, kc, vc, ks, vs = _inputs(pos0)
    ref = oracle.attention(q, k, v, kc, vc, ks, vs, pos0, 0, 1.0 / np.sqrt(D))
    for rank in range(world):
        np.testing.assert_allclose(res[rank][0], ref, rtol=2e-5, atol=2e-5)
    np.testing.assert_array_equal(res[0][0], res[1][0])   # every process the same bits
    if pos0 == 64:   # one chunk: parts 0..2 of 4 are empty, so rank 0 contributes nothing
        assert res[0][1] and not res[1][1]
