"""GPU (2 or more): the batch-1 long-context step with the global caches' chunks split across processes, one GPU
each, and the attention partials of the global layers joined by an NCCL all-gather before the log-sum-exp combine.

Every process holds the whole model and every cache and runs the whole step; only the chunk range each global-layer
attention reads differs. Two exchanges: the default one inside the combine kernel (each process merges its own
splits, then the processes' partials meet over NVLink as sequence-numbered words) and an ncclAllGather of every
split's partial. With the same total number of splits as one process, the all-gather gives that process's logits bit
for bit and the peer exchange moves them by rounding only; every process computes the same bits either way. The
single-process step itself is pinned to the oracle by the session tests. A process that steps alone makes its
peers' words never arrive: the bounded wait gives up with an error instead of hanging."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
N_PAST = 20000
CONTEXT = 32768
TOKENS = [7, 4001, 123]


def _product():
    if "xtier_go_b200" in sys.modules:
        return sys.modules["xtier_go_b200"]
    pkg = os.path.join(ROOT, "xtier-go_b200")
    spec = importlib.util.spec_from_file_location("xtier_go_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xtier_go_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def _run(xtg, device, **opts):
    with xtg.Session(model=xtg.SMALL, context=CONTEXT, device=device, **opts) as s:
        info = s.info()
        s.prefill_synthetic(N_PAST)
        logits = s.forward(TOKENS, want=2)
        return info, logits, s.argmax(len(TOKENS))


def _alone(xtg, rank, world, nccl_id, barrier):
    """Every process steps once, then rank 1 steps alone: its combine waits for partials that never come and must
    give up after kv_wait_ms with an error (the context stays usable), not hang."""
    with xtg.Session(model=xtg.SMALL, context=4096, device=rank, kv_world=world, kv_rank=rank, nccl_id=nccl_id,
                     kv_wait_ms=300) as s:
        s.prefill_synthetic(2000)
        s.forward(TOKENS[:1], want=0)
        msg = None
        if rank == 1:
            try:
                s.forward(TOKENS[:1], want=0)
            except xtg.XtgError as e:
                msg = str(e)
        barrier.wait()   # the others keep their buffers mapped until rank 1 is done
        return msg


def _rank(rank, world, ids, barrier, out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"   # plain peer copies: no NVLink multicast objects bound to a process
    import torch   # loads the NCCL the parent's unique ids came from, which the library then binds
    torch.cuda.set_device(rank)
    xtg = _product()
    split = dict(kv_world=world, kv_rank=rank)
    same = _run(xtg, rank, nccl_id=ids[0], splits_global=128 // world, **split)
    dflt = _run(xtg, rank, nccl_id=ids[1], **split)
    nccl = _run(xtg, rank, nccl_id=ids[2], splits_global=128 // world, kv_exchange="nccl", **split)
    alone = _alone(xtg, rank, world, ids[3], barrier)
    out[rank] = (same, dflt, nccl, alone)


@pytest.mark.gpu
@pytest.mark.timeout(600)
@pytest.mark.parametrize("world", [2, 4])
def test_split_kv_across_gpus(cuda, xtg, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"split-KV across processes needs {world} GPUs")
    ids = [bytes(torch.cuda.nccl.unique_id()).hex() for _ in range(4)]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_rank, args=(world, ids, mgr.Barrier(world), out), nprocs=world, join=True,
                           start_method="spawn")
        res = dict(out)
    one_same = _run(xtg, 0, splits_global=128)
    one_dflt = _run(xtg, 0)

    for rank in range(world):
        (info, logits, am), (dinfo, dlogits, dam), (ninfo, nlogits, nam), alone = res[rank]
        assert info["kv_world"] == world and info["kv_rank"] == rank and info["splits_global"] == 128 // world
        assert info["kv_exchange"] == "peer" and ninfo["kv_exchange"] == "nccl" and info["global_layers"] > 0
        assert dinfo["splits_global"] * world <= 256
        # the same 128 chunk ranges as one process: through the all-gather every split's partial meets in the same
        # combine, so the logits are identical; the peer exchange merges each process's splits first, then the
        # processes' partials (rounding only)
        assert sorted(logits) == sorted(one_same[1]) == sorted(nlogits)
        for r in logits:
            np.testing.assert_array_equal(nlogits[r], one_same[1][r])
            d = np.abs(logits[r] - one_same[1][r]).max()
            assert d <= 5e-2, (rank, r, d)
        assert am == one_same[2] == nam
        assert (alone is None) if rank != 1 else ("timed out" in alone), alone
        # default split counts: rounding only
        for r in dlogits:
            d = np.abs(dlogits[r] - one_dflt[1][r]).max()
            assert d <= 5e-2, (rank, r, d)
        assert dam == one_dflt[2]
    # every process computes the same bits (the partials are merged in rank order everywhere)
    for k in range(3):
        for r in res[0][k][1]:
            for rank in range(1, world):
                np.testing.assert_array_equal(res[0][k][1][r], res[rank][k][1][r])
