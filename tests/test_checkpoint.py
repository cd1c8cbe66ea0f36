"""CPU: Dory checkpoints (ModelOpt W4A16_NVFP4: config.json + model.safetensors, the layout packs/dory/dory.cpp:77-134
and 316-439 reads). The oracle's checkpoint model is pinned to the reference's own Dory pack (DoryModel / DorySession,
compiled into oracle/_ref) on the same files; xtg_cuda_open reads and checks the files before any device work, so
its error paths run here."""
import ctypes as C
import json
import os

import numpy as np
import pytest

import oracle as O
from tests import dory_ckpt

TOKS = [5, 17, 4095, 0, 99, 1234, 7, 3000]


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("dory_small")
    cfg, tensors = dory_ckpt.write_checkpoint(str(d), seed=1)
    return str(d), cfg, tensors


@pytest.mark.parametrize("loops", [None, 1])
def test_oracle_checkpoint_matches_reference_pack(ckpt, loops):
    """CheckpointDory (weight sharing across loops, scale folding, BF16 embedding and head, layer_types order) against
    the reference's DoryModel on the same checkpoint: 8 rows, then 3 more, FP8 KV."""
    if O.ref() is None:
        pytest.skip("oracle/_ref (the reference's own kernels) is not built")
    d, cfg, tensors = ckpt
    extra = {} if loops is None else {"loops": loops}
    ref = O.RefDory(d, kv_dtype="fp8", context=1024, **extra)
    ora = O.CheckpointDory(cfg, tensors, ctx=1024, n_prefill=0, loops=loops, kv_dtype=O.KV_FP8)
    try:
        for toks in (TOKS, [1, 2, 3]):
            want = ref.forward(toks)
            got = ora.step(toks)
            assert np.array_equal(got.argmax(1), want.argmax(1))
            assert np.abs(got - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
        assert ora.n_past == ref.n_past == 11
    finally:
        ref.close()
        ora.close()


def test_oracle_checkpoint_head_dim_256_matches_reference_pack(tmp_path):
    """The real Dory 4B's head shape (head_dim 256, 4 q heads per KV head) on a small checkpoint: CheckpointDory
    against the reference's DoryModel, 8 rows then 3, FP8 KV."""
    if O.ref() is None:
        pytest.skip("oracle/_ref (the reference's own kernels) is not built")
    cfg, tensors = dory_ckpt.write_checkpoint(str(tmp_path), dory_ckpt.small_config(head_dim=256), seed=3)
    ref = O.RefDory(str(tmp_path), kv_dtype="fp8", context=1024)
    ora = O.CheckpointDory(cfg, tensors, ctx=1024, n_prefill=0, kv_dtype=O.KV_FP8)
    try:
        for toks in (TOKS, [1, 2, 3]):
            want = ref.forward(toks)
            got = ora.step(toks)
            assert np.array_equal(got.argmax(1), want.argmax(1))
            assert np.abs(got - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
    finally:
        ref.close()
        ora.close()


def _open(xtg, path, options=b"{}"):
    err = C.create_string_buffer(1024)
    h = xtg.lib().xtg_cuda_open(os.fsencode(path), options, err, len(err))
    if h:
        xtg.lib().xtg_cuda_close(h)
    return h, err.value.decode()


def _variant(tmp_path, base, name, config=None, safetensors=None):
    d = tmp_path / name
    d.mkdir()
    cfg = dict(base[1])
    if config:
        cfg.update(config)
    (d / "config.json").write_text(json.dumps(cfg))
    src = os.path.join(base[0], "model.safetensors")
    data = open(src, "rb").read() if safetensors is None else safetensors(open(src, "rb").read())
    (d / "model.safetensors").write_bytes(data)
    return str(d)


@pytest.mark.parametrize("name,config,needle", [
    ("not_dory", {"model_type": "llama"}, "not a Dory checkpoint"),
    ("w4a4", {"quantization_config": {"quant_algo": "NVFP4"}}, "W4A16_NVFP4"),
    ("tied", {"tie_word_embeddings": True}, "untied"),
    ("bias", {"attention_bias": True}, "no biases"),
    ("short_types", {"layer_types": dory_ckpt.SMALL_LAYER_TYPES[:-1]}, "layer_types has 7"),
    ("bad_type", {"layer_types": ["conv"] + dory_ckpt.SMALL_LAYER_TYPES[1:]}, "unknown layer type conv"),
    ("counts", {"n_output_layers": 3}, "input + recurrent + output"),
    ("no_theta", {"rope_parameters": {"sliding_attention": {"rope_theta": 1e4}}}, "no rope_theta"),
    ("partial_rope", {"rope_parameters": {"sliding_attention": {"rope_theta": 1e4, "partial_rotary_factor": 0.5},
                                          "full_attention": {"rope_theta": 1e7}}}, "full-width RoPE"),
    ("head_dim", {"head_dim": 64}, "head_dim must be 128 or 256"),
])
def test_open_rejects_bad_configs(xtg, ckpt, tmp_path, name, config, needle):
    h, msg = _open(xtg, _variant(tmp_path, ckpt, name, config=config))
    assert not h and needle in msg, msg


@pytest.mark.parametrize("name,mangle,needle", [
    ("short", lambda b: b[:4], "shorter than its header length"),
    ("huge_header", lambda b: (1 << 40).to_bytes(8, "little") + b[8:], "bad safetensors header length"),
    ("not_json", lambda b: b[:8] + b"x" + b[9:], "JSON"),
    ("past_end", lambda b: b[: len(b) - 64], "outside the file"),
])
def test_open_rejects_bad_safetensors(xtg, ckpt, tmp_path, name, mangle, needle):
    h, msg = _open(xtg, _variant(tmp_path, ckpt, name, safetensors=mangle))
    assert not h and needle in msg, msg


@pytest.mark.parametrize("options,needle", [
    (b'{"model": {"hidden": 512}}', "brings its own shape"),
    (b'{"kv_mode": "last_loop"}', "only per_loop"),
    (b'{"head": "fp8"}', "bf16 | nvfp4"),
    (b'{"loops": 5}', "loops: 1..4"),
    (b'{"context": 131072}', "max_position_embeddings"),
])
def test_open_rejects_bad_options(xtg, ckpt, options, needle):
    d, cfg, _ = ckpt
    h, msg = _open(xtg, d, options)
    assert not h and needle in msg, msg


def test_open_missing_directory(xtg, tmp_path):
    h, msg = _open(xtg, str(tmp_path / "nowhere"))
    assert not h and "no config.json" in msg
