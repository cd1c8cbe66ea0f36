"""Test fixture: small Dory checkpoints in the ModelOpt W4A16_NVFP4 layout packs/dory/dory.cpp reads (config.json and
model.safetensors; config keys dory.cpp:77-134, tensor names and dtypes dory.cpp:321-392 and 417-428).

The weights are seeded normal bf16 values quantized by the oracle's NVFP4 quantizer. The stored scale vectors are
drawn so that, once folded as dory.cpp:326-364 folds them, they land in the synthetic model's ranges."""
import json
import os

import numpy as np

from oracle import quantize_nvfp4

# every sublayer kind in the input, recurrent and output blocks, not in the synthetic model's alternation
SMALL_LAYER_TYPES = ["sliding_attention", "mlp", "mlp", "full_attention", "sliding_attention", "mlp",
                     "full_attention", "mlp"]


def small_config(**kw):
    c = {
        "model_type": "dory", "hidden_size": 512, "intermediate_size": 1024, "num_attention_heads": 8,
        "num_key_value_heads": 2, "head_dim": 128, "vocab_size": 4096, "num_hidden_layers": 8,
        "n_input_layers": 2, "n_recurrent_layers": 4, "n_output_layers": 2, "n_recurrent_loops": 2,
        "recurrent_kv_cache_mode": "per_loop", "sliding_window": 64, "max_position_embeddings": 65536,
        "initializer_range": 0.02, "ngpt_alpha_init": 0.05, "attention_output_gate_logit_scale_init": None,
        "attention_bias": False, "mlp_bias": False, "hidden_act": "silu", "tie_word_embeddings": False,
        "layer_types": list(SMALL_LAYER_TYPES),
        "rope_parameters": {"sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
                            "full_attention": {"rope_type": "default", "rope_theta": 10000000.0}},
        "quantization_config": {"quant_algo": "W4A16_NVFP4", "group_size": 16},
    }
    c.update(kw)
    return c


def bf16_bits(x):
    """f32 -> bf16 bits, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def make_tensors(config, seed=0):
    """name -> (safetensors dtype, array) for config's shapes."""
    rng = np.random.default_rng(seed)
    H, F, V = config["hidden_size"], config["intermediate_size"], config["vocab_size"]
    d, heads, kvh = config["head_dim"], config["num_attention_heads"], config["num_key_value_heads"]
    Q, KV = heads * d, kvh * d
    init = np.float32(config["initializer_range"])
    t = {}

    def weight(name, n, k):
        w = bf16_bits(rng.standard_normal((n, k), np.float32) * np.float32(0.02))
        codes, scales, g = quantize_nvfp4(w)
        t[name + ".weight"] = ("U8", codes)
        t[name + ".weight_scale"] = ("F8_E4M3", scales)
        t[name + ".weight_scale_2"] = ("F32", np.array(g, np.float32))

    def vec(name, n, lo, hi):
        t[name] = ("BF16", bf16_bits(rng.uniform(lo, hi, n).astype(np.float32)))

    # raw ranges: folded lr = |s| alpha_init / init in [0.05, 0.2]; qscale = (s sqrt(d) / init)^2 in ~[48, 80];
    # gscale = (s sqrt(gate_init) / init)^2 in ~[25, 75]; suv * sqrt(H) in ~[25, 75]; logit scale / init in [100, 200]
    a = float(config["ngpt_alpha_init"]) / float(init)
    gate_init = config.get("attention_output_gate_logit_scale_init") or float(np.sqrt(np.float32(H)))
    for l, kind in enumerate(config["layer_types"]):
        p = f"backbone.layers.{l}."
        if kind == "mlp":
            weight(p + "mixer.gate_proj", F, H)
            weight(p + "mixer.up_proj", F, H)
            weight(p + "mixer.down_proj", H, F)
            vec(p + "mixer.suv_gate", F, 25 / np.sqrt(H), 75 / np.sqrt(H))
            vec(p + "mixer.suv_up", F, 25 / np.sqrt(H), 75 / np.sqrt(H))
            vec(p + "mlp_alpha", H, 0.05 / a, 0.2 / a)
        else:
            for n, rows in (("q_proj", Q), ("k_proj", KV), ("v_proj", KV), ("g_proj", Q)):
                weight(p + "mixer." + n, rows, H)
            weight(p + "mixer.o_proj", H, Q)
            qf = float(np.sqrt(d)) / float(init)
            gf = float(np.sqrt(gate_init)) / float(init)
            vec(p + "mixer.sqk", Q, np.sqrt(48) / qf, np.sqrt(80) / qf)
            vec(p + "mixer.s_gate", Q, 5 / gf, np.sqrt(75) / gf)
            vec(p + "attn_alpha", H, 0.05 / a, 0.2 / a)
    t["backbone.embeddings.weight"] = ("BF16", bf16_bits(rng.standard_normal((V, H), np.float32) * np.float32(0.02)))
    t["lm_head.weight"] = ("BF16", bf16_bits(rng.standard_normal((V, H), np.float32) * np.float32(0.02)))
    vec("lm_head.logit_scale", V, 100 * float(init), 200 * float(init))
    return t


def write_safetensors(path, tensors):
    """tensors: name -> (dtype, array): the 8-byte header length, the JSON header (padded to 8 bytes), the data."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        dt, a = tensors[name]
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(np.shape(a)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_checkpoint(directory, config=None, seed=0, tensors=None):
    """A checkpoint directory; returns (config, {name: array})."""
    config = config or small_config()
    tensors = tensors or make_tensors(config, seed)
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config, f)
    write_safetensors(os.path.join(directory, "model.safetensors"), tensors)
    return config, {k: v for k, (_, v) in tensors.items()}
