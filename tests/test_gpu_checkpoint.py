"""GPU: sessions opened from a Dory checkpoint (xtg_cuda_open on a ModelOpt W4A16_NVFP4 directory) against the
oracle's checkpoint model, itself pinned to the reference's Dory pack (tests/test_checkpoint.py), and against the
reference pack directly where oracle/_ref is built. Parity bar: identical argmax, max |d logit| <= 5e-2."""

import numpy as np
import pytest

import oracle as O
from tests import dory_ckpt

pytestmark = pytest.mark.gpu
LOGIT_TOL = 5e-2
STEPS = [[5, 17, 4095, 0, 99, 1234, 7, 3000], [1, 2, 3], [4000, 12, 9, 77, 3, 3, 3, 1], [42]]


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("dory_small_gpu")
    cfg, tensors = dory_ckpt.write_checkpoint(str(d), seed=2)
    return str(d), cfg, tensors


def rows(out, n):
    return np.stack([out[i] for i in range(n)])


def check(got, want):
    assert np.array_equal(got.argmax(1), want.argmax(1))
    assert np.abs(got - want).max() <= LOGIT_TOL, np.abs(got - want).max()


@pytest.mark.parametrize("head", ["bf16", "nvfp4"])
def test_checkpoint_steps_match_oracle(cuda, xtg, ckpt, head):
    """Verify steps from an empty cache, FP8 KV: the BF16 lm_head kernel (head.cu) or the head quantized at load."""
    d, cfg, tensors = ckpt
    ora = O.CheckpointDory(cfg, tensors, ctx=1024, n_prefill=0, head=head, kv_dtype=O.KV_FP8)
    with xtg.Session(path=d, context=1024, kv_dtype="fp8", head=head) as s:
        info = s.info()
        assert info["source"] == "checkpoint" and info["head"] == head and info["loops"] == 2
        for toks in STEPS:
            check(rows(s.forward(toks, want=2), len(toks)), ora.step(toks))
        assert s.pos() == ora.n_past
    ora.close()


def test_checkpoint_matches_reference_pack(cuda, xtg, ckpt):
    """The same steps against the reference's own DoryModel / DorySession on the checkpoint files."""
    if O.ref() is None:
        pytest.skip("oracle/_ref (the reference's own kernels) is not built")
    d, _, _ = ckpt
    ref = O.RefDory(d, kv_dtype="fp8", context=1024)
    with xtg.Session(path=d, context=1024, kv_dtype="fp8") as s:
        for toks in STEPS:
            check(rows(s.forward(toks, want=2), len(toks)), ref.forward(toks))
    ref.close()


@pytest.mark.parametrize("loops", [1, 3])
def test_checkpoint_loops_option(cuda, xtg, ckpt, loops):
    """loops other than the checkpoint's n_recurrent_loops: the recurrent sublayers' one weight copy read `loops`
    times, a KV instance per loop; int8 KV prefilled past the ring."""
    d, cfg, tensors = ckpt
    ora = O.CheckpointDory(cfg, tensors, ctx=1024, n_prefill=300, loops=loops)
    with xtg.Session(path=d, context=1024, loops=loops) as s:
        s.prefill_synthetic(300)
        assert s.info()["loops"] == loops
        for toks in STEPS[:2]:
            check(rows(s.forward(toks, want=2), len(toks)), ora.step(toks))
    ora.close()


def test_checkpoint_prompt_chunks(cuda, xtg, ckpt):
    """A 40-token prompt with the NVFP4 head runs as one batched prompt chunk (8-row groups over the session's caches,
    the BF16 embedding in the batched step); the oracle runs the same 40 rows as one chunk (each row attends the
    chunk's rows up to itself unquantized, as attend_rows does)."""
    d, cfg, tensors = ckpt
    toks = [(37 * i + 11) % 4096 for i in range(40)]
    ora = O.CheckpointDory(cfg, tensors, ctx=1024, n_prefill=0, head="nvfp4")
    want = ora.step(toks)
    with xtg.Session(path=d, context=1024, head="nvfp4") as s:
        assert s.info()["prefill_ar"] == 64
        got = rows(s.forward(toks, want=2), 40)
        check(got, want)
        nxt = [3, 4, 5]
        check(rows(s.forward(nxt, want=2), 3), ora.step(nxt))
    ora.close()


def test_checkpoint_bf16_head_keeps_verify_steps(cuda, xtg, ckpt):
    """With the BF16 head, prompts run as 8-row verify steps (the batched step's head is NVFP4)."""
    d, cfg, tensors = ckpt
    with xtg.Session(path=d, context=1024) as s:
        assert s.info()["prefill_ar"] == 8
        toks = [(13 * i + 1) % 4096 for i in range(20)]
        got = rows(s.forward(toks, want=2), 20)
    ora = O.CheckpointDory(cfg, tensors, ctx=1024, n_prefill=0)
    want = np.concatenate([ora.step(toks[i:i + 8]) for i in range(0, 20, 8)])
    ora.close()
    check(got, want)


@pytest.mark.parametrize("head", ["bf16", "nvfp4"])
def test_checkpoint_head_dim_256(cuda, xtg, tmp_path, head):
    """A head_dim-256 checkpoint (the real Dory 4B's head shape, GQA 4): verify steps against the oracle's checkpoint
    model and the reference's own Dory pack; with the NVFP4 head the 20-token prompt runs as a 64-row chunk of the
    batched step, with the BF16 head as 8-row steps."""
    cfg, tensors = dory_ckpt.write_checkpoint(str(tmp_path), dory_ckpt.small_config(head_dim=256), seed=4)
    ora = O.CheckpointDory(cfg, tensors, ctx=1024, n_prefill=0, head=head, kv_dtype=O.KV_FP8)
    ref = O.RefDory(str(tmp_path), kv_dtype="fp8", context=1024) if O.ref() is not None else None
    with xtg.Session(path=str(tmp_path), context=1024, kv_dtype="fp8", head=head) as s:
        assert s.info()["prefill_ar"] == (64 if head == "nvfp4" else 8)
        for toks in STEPS + [[(11 * i + 5) % 4096 for i in range(20)]]:
            got = rows(s.forward(toks, want=2), len(toks))
            if head == "nvfp4" or len(toks) <= 8:   # one chunk of the batched step, or one verify step
                want = ora.step(toks)
            else:
                want = np.concatenate([ora.step(toks[i:i + 8]) for i in range(0, len(toks), 8)])
            check(got, want)
            if ref is not None and head == "bf16" and len(toks) <= 8:
                check(got, ref.forward(toks))
    ora.close()
    if ref is not None:
        ref.close()


@pytest.mark.parametrize("vocab,hidden,m", [(131072, 3072, 8), (4099, 512, 3), (200, 5120, 1)])
def test_head_bf16_kernel(cuda, xtg, vocab, hidden, m):
    """xtg_cuda_head_bf16 at the Dory-3072 head shape and ragged ones against a float64 torch reference of
    matmul_bf16 x logit scale: |d logit| <= 1e-3 (x is carried as bf16 hi + lo, ~16 bits), argmax a true maximum."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(vocab + hidden + m)
    w = (torch.randn(vocab, hidden, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(m, hidden, generator=g, device="cuda")
    x = x / x.norm(dim=1, keepdim=True)   # the residual stream is unit-norm
    ls = torch.rand(vocab, generator=g, device="cuda") * 100 + 100
    logits, am = xtg.head_bf16(x, w, ls)
    ref = (x.double() @ w.double().t()) * ls.double()
    assert (logits.double() - ref).abs().max().item() <= 1e-3
    top = ref.max(dim=1).values
    picked = ref.gather(1, am.long().view(-1, 1)).view(-1)
    assert torch.all(picked >= top - 1e-3)
    assert torch.equal(am.long(), logits.argmax(dim=1))
