"""CPU: the C-ABI library builds, loads, and exports every entry point include/xtg_cuda.h declares; the session API
mirrors npu/xtg_npu.h's (same names after the prefix, same arities); open fails cleanly (NULL + message) without a
usable GPU. No compute call is made here."""
import ctypes as C
import re

import pytest

NPU_ABI = {  # npu/xtg_npu.h:23-47, name -> number of parameters
    "open": 4, "info": 3, "forward": 8, "pos": 1, "rewind": 2, "snapshot_slots": 1, "snapshot_pos": 2,
    "snapshot": 2, "restore": 2, "grow": 4, "debug_cache": 5, "close": 1,
}


def test_every_declared_symbol_is_exported(xtg):
    L = xtg.lib()
    declared = xtg.declared_symbols()
    assert len(declared) >= 24
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing


def test_session_abi_mirrors_npu_plugin(xtg):
    text = open(xtg.HEADER).read()
    for name, nargs in NPU_ABI.items():
        m = re.search(r"XTG_CUDA_API\s+[\w\*\s]+?\bxtg_cuda_%s\s*\(([^)]*)\)" % name, text)
        assert m, name
        args = [a for a in m.group(1).split(",") if a.strip()]
        assert len(args) == nargs, (name, args)


def test_open_without_gpu_reports_an_error(xtg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU tests cover open")
    err = C.create_string_buffer(512)
    h = xtg.lib().xtg_cuda_open(b"synthetic", b"{}", err, len(err))
    assert not h
    assert err.value


def test_open_rejects_unknown_models_and_bad_options(xtg):
    L = xtg.lib()
    err = C.create_string_buffer(512)
    assert not L.xtg_cuda_open(b"/no/such/model", b"{}", err, len(err))   # a checkpoint directory without files
    assert b"no config.json" in err.value
    assert not L.xtg_cuda_open(b"", b"{}", err, len(err))
    assert b"synthetic" in err.value
    assert not L.xtg_cuda_open(b"synthetic", b"{\"kv_dtype\": \"bf16\"", err, len(err))
    assert err.value


@pytest.mark.parametrize("entry", ["xtg_cuda_attention", "xtg_cuda_attention_noalloc"])
def test_attention_rejects_unaligned_pointers_before_any_device_work(xtg, entry):
    """The cache is read by 16-byte bulk copies, q, k, v and out by 16-byte loads and stores: a pointer off a 16-byte
    boundary is an error at the call (checked on the host, so this runs without a GPU), never a GPU fault."""
    good, bad = 4096, 4096 + 4
    for field in ("q", "k", "v", "out", "k_codes", "v_codes", "k_scales", "v_scales"):
        ptrs = dict(q=good, k=good, v=good, out=good, k_codes=good, v_codes=good, k_scales=good, v_scales=good)
        ptrs[field] = bad
        a = xtg.AttnArgs(8, 100, 24, 6, 128, 0, 0.1, ptrs["q"], ptrs["k"], ptrs["v"], ptrs["k_codes"],
                         ptrs["v_codes"], ptrs["k_scales"], ptrs["v_scales"], 128, 0, None, 0, ptrs["out"])
        err = C.create_string_buffer(512)
        rc = getattr(xtg.lib(), entry)(C.byref(a), 4, None, err, len(err))
        assert rc == -1 and b"16-byte" in err.value, (field, err.value)


@pytest.mark.parametrize("entry", ["xtg_cuda_attention", "xtg_cuda_attention_noalloc"])
@pytest.mark.parametrize("kv_heads", [0, -2])
def test_attention_rejects_no_kv_heads_before_any_device_work(xtg, entry, kv_heads):
    """q heads are grouped over the KV heads (heads % kv_heads): kv_heads < 1 is an error at the call, checked on the
    host before any division or allocation (this runs without a GPU)."""
    good = 4096
    a = xtg.AttnArgs(8, 100, 24, kv_heads, 128, 0, 0.1, good, good, good, good, good, good, good, 128, 0, None, 0,
                     good)
    err = C.create_string_buffer(512)
    rc = getattr(xtg.lib(), entry)(C.byref(a), 4, None, err, len(err))
    assert rc == -1 and b"KV head" in err.value, err.value


@pytest.mark.parametrize("options,needle", [
    (b'{"model": {"head_dim": 64}}', b"head_dim must be 128 or 256"),
    (b'{"model": {"head_dim": 256}, "kv_world": 2, "kv_rank": 0, "nccl_id": "' + b"0" * 256 + b'"}',
     b"takes head_dim 128"),
])
def test_open_checks_head_dim_before_any_device_work(xtg, options, needle):
    """head_dim 128 or 256 (the real Dory 4B's); split-KV across GPUs at 128 only: refused from the options alone."""
    err = C.create_string_buffer(512)
    assert not xtg.lib().xtg_cuda_open(b"synthetic", options, err, len(err))
    assert needle in err.value, err.value


@pytest.mark.parametrize("entry", ["xtg_cuda_attention", "xtg_cuda_attention_noalloc"])
def test_attention_rejects_other_head_dims_before_any_device_work(xtg, entry):
    good = 4096
    a = xtg.AttnArgs(8, 100, 16, 4, 192, 0, 0.1, good, good, good, good, good, good, good, 128, 0, None, 0, good)
    err = C.create_string_buffer(512)
    rc = getattr(xtg.lib(), entry)(C.byref(a), 4, None, err, len(err))
    assert rc == -1 and b"head_dim 128 or 256" in err.value, err.value
