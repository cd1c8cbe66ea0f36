"""Generates the golden fixtures in this directory by running XTier Go's OWN CPU kernels (oracle/_ref/libxtgref.so,
compiled from the reference sources by `make -C oracle ref`) on seeded inputs.

    python tests/golden/make_golden.py        # needs oracle/_ref (the reference tree present)

Inputs are regenerated from the seeded generators of the oracle (xo_gen_*), so a fixture holds only the case
parameters and the reference's outputs. Cases follow the reference's own tests/kernels_test.cpp:
  e4m3.npz         f32 -> E4M3 codes over a grid with ties and saturation (fp.cpp:30-49), the 256-code decode table
  nvfp4.npz        matmul_nvfp4 (kernels.cpp:84-138): kernels_test.cpp:57-87's recipe (two fused weights 70x256 and
                   33x256, random codes, scales 0x20..0x4f, global 0.37, m in 1, 2, 7) and a quantized N(0, 0.02)
                   96x512 weight at m in 1, 8
  attention.npz    attention (kv.cpp:166-286) over an FP8 KvCache, the 7 cases of kernels_test.cpp:139-141
  elementwise.npz  justnorm, slerp_residual, rope, swiglu_scaled (kernels.cpp:169-234)
  step_fp8.npz     three steps (8, 8, 3 rows) of a tiny synthetic Dory from an empty state, run with the reference's
                   kernels in DorySession::sublayer / run_chunk order with FP8 KvCaches (ring = window + 16 slots)
  sampling.npz     argmax, top_logprobs and Sampler(seed).sample (sampler.cpp:8-94) on seeded logits rows with ties
                   (vocab 4096 and 131072) under the filter settings of SAMPLING_PARAMS, with the first uniform draw
                   of each seed's engine

    python tests/golden/make_golden.py sampling   # only sampling.npz
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402

f32p, u8p = O.f32p, O.u8p

# ---- shared case definitions (the tests regenerate the inputs from these) ----
SEED = 42
NVFP4_FUSED = dict(n=(70, 33), k=256, ms=(1, 2, 7), global_=0.37)
NVFP4_QUANT = dict(n=96, k=512, ms=(1, 8))
ATTN_CASES = [  # cached, n_q, window (kernels_test.cpp:139-141); heads 8, kv heads 2, d 64, scale 0.7
    (300, 1, 0), (5000, 1, 0), (300, 1, 64), (100, 37, 0), (100, 37, 16), (0, 20, 0), (900, 3, 128)]
ATTN_SHAPE = dict(heads=8, kv_heads=2, d=64, scale=0.7)
TINY = dict(hidden=256, ffn=512, heads=4, kv_heads=2, head_dim=128, vocab=1024, n_in=2, n_rec=4, n_out=2, loops=2,
            window=16, ring=32, global_every=2, theta_sliding=1e4, theta_global=1e7, weight_std=0.02,
            lr_lo=0.05, lr_hi=0.2, qs_lo=48.0, qs_hi=80.0, gs_lo=25.0, gs_hi=75.0, suv_lo=25.0, suv_hi=75.0,
            ls_lo=100.0, ls_hi=200.0, kvs_lo=0.0008, kvs_hi=0.0016, seed=7)
STEP_TOKENS = [[5, 17, 900, 3, 44, 1023, 0, 256], [8, 9, 10, 11, 12, 13, 14, 15], [600, 601, 2]]


def fused_inputs():
    """kernels_test.cpp:43-55's random weights, drawn from the oracle's generator: codes any byte, scales
    0x20 + (r % 0x30), global 0.37; x ~ U(-1, 1)."""
    k = NVFP4_FUSED["k"]
    ws = []
    for i, n in enumerate(NVFP4_FUSED["n"]):
        codes = (O.gen_int8(SEED, 10 + 4 * i, n * k // 2).view(np.uint8)).reshape(n, k // 2).copy()
        sb = np.array([O.lib().xo_rand_bits(SEED, 11 + 4 * i, j) % 0x30 for j in range(n * k // 16)], np.uint8)
        scales = (0x20 + sb).reshape(n, k // 16).astype(np.uint8)
        ws.append((codes, scales, NVFP4_FUSED["global_"]))
    x = O.gen_uniform(SEED, 20, -1.0, 1.0, max(NVFP4_FUSED["ms"]) * k).reshape(-1, k)
    return ws, x


def quant_inputs():
    n, k = NVFP4_QUANT["n"], NVFP4_QUANT["k"]
    raw, codes, scales, g = O.synth_weight(SEED, 30, n, k)
    x = O.bf16_to_f32(O.gen_normal_bf16(SEED, 31, 1.0, max(NVFP4_QUANT["ms"]) * k)).reshape(-1, k)
    return (codes, scales, g), x


def attention_inputs(ci):
    cached, n_q, window = ATTN_CASES[ci]
    h, kvh, d = ATTN_SHAPE["heads"], ATTN_SHAPE["kv_heads"], ATTN_SHAPE["d"]
    total = cached + n_q
    K = O.gen_uniform(SEED, 100 + 8 * ci, -1.0, 1.0, total * kvh * d).reshape(total, kvh, d)
    V = O.gen_uniform(SEED, 101 + 8 * ci, -1.0, 1.0, total * kvh * d).reshape(total, kvh, d)
    q = O.gen_uniform(SEED, 102 + 8 * ci, -1.0, 1.0, n_q * h * d).reshape(n_q, h, d)
    return K, V, q


def elementwise_inputs():
    x = O.gen_uniform(SEED, 200, -1.0, 1.0, 8 * 384).reshape(8, 384)
    o = O.gen_uniform(SEED, 201, -1.0, 1.0, 8 * 384).reshape(8, 384)
    lr = O.gen_uniform(SEED, 202, 0.05, 0.2, 384)
    qr = O.gen_uniform(SEED, 203, -1.0, 1.0, 3 * 6 * 128).reshape(3, 6, 128)
    g = O.gen_uniform(SEED, 204, -2.0, 2.0, 4 * 512).reshape(4, 512)
    u = O.gen_uniform(SEED, 205, -2.0, 2.0, 4 * 512).reshape(4, 512)
    sg = O.gen_uniform(SEED, 206, 0.5, 2.0, 512)
    su = O.gen_uniform(SEED, 207, 0.5, 2.0, 512)
    return x, o, lr, qr, g, u, sg, su


def e4m3_grid():
    L = O.lib()
    table = O.e4m3_table()
    finite = table[np.isfinite(table)]
    mids = []
    pos = np.unique(finite[finite >= 0])
    for a, b in zip(pos[:-1], pos[1:]):
        mids += [(a + b) / 2, np.nextafter(np.float32((a + b) / 2), np.float32(0)),
                 np.nextafter(np.float32((a + b) / 2), np.float32(1e9))]
    extra = [447.9, 448.0, 449.0, 464.0, 465.0, 1000.0, 1e30, np.inf, 1e-12, 2.0 ** -10, 2.0 ** -11]
    g = np.concatenate([finite, np.float32(mids), np.float32(extra)]).astype(np.float32)
    g = np.concatenate([g, -g])
    g = np.concatenate([g, O.gen_uniform(SEED, 1, -500.0, 500.0, 4096),
                        O.gen_uniform(SEED, 2, -0.03, 0.03, 4096)]).astype(np.float32)
    del L
    return g


class XrSublayer(C.Structure):
    _fields_ = [("kind", C.c_int), ("codes", u8p * 5), ("scales", u8p * 5), ("globals", C.c_float * 5),
                ("lr", f32p), ("qscale", f32p), ("gscale", f32p), ("sg", f32p), ("su", f32p), ("theta", C.c_float),
                ("window", C.c_int), ("cache", C.c_void_p)]


class XrShape(C.Structure):
    _fields_ = [("hidden", C.c_int), ("ffn", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int)]


def reference_steps(cfg, steps, threads=4):
    """The tiny synthetic model stepped with the reference's kernels (oracle/_ref), FP8 KvCaches."""
    R = O.ref()
    R.xr_sublayer.argtypes = [C.c_void_p, C.POINTER(XrShape), C.POINTER(XrSublayer), f32p, C.c_int, C.c_int64,
                              C.c_int, f32p]
    R.xr_head.argtypes = [C.c_void_p, u8p, u8p, C.c_float, C.c_int, C.c_int, f32p, C.c_int, f32p, f32p]
    model = O.SynthDory(cfg, ctx=64, n_prefill=0, kv_dtype=O.KV_FP8)
    M = model.model.contents
    pool = R.xr_pool_new(threads)
    H, F, Q = cfg["hidden"], cfg["ffn"], cfg["heads"] * cfg["head_dim"]
    shape = XrShape(H, F, cfg["heads"], cfg["kv_heads"], cfg["head_dim"])
    kinds = O.kinds(cfg)
    caches = []
    subs = []
    for e, kind in enumerate(kinds):
        L = M.layers[e]
        s = XrSublayer()
        s.kind = kind
        for j in range(5):
            s.codes[j] = L.w[j].codes
            s.scales[j] = L.w[j].scales
            s.globals[j] = L.w[j].global_
        s.lr, s.qscale, s.gscale, s.sg, s.su = L.lr, L.qscale, L.gscale, L.sg, L.su
        s.theta = L.theta
        s.window = cfg["window"] if kind == 1 else 0
        if kind:
            c = R.xr_kv_new(cfg["kv_heads"], cfg["head_dim"], 64, cfg["ring"] if kind == 1 else 0, 1)
            caches.append(c)
            s.cache = c
        subs.append(s)
    codes, scales, g = model.weight(-1, 0)
    ls = np.ctypeslib.as_array(M.logit_scale, shape=(cfg["vocab"],)).copy()
    c_head = np.ascontiguousarray(codes)
    s_head = np.ascontiguousarray(scales)
    out = []
    pos = 0
    for toks in steps:
        m = len(toks)
        x = np.zeros((m, H), np.float32)   # the tied head's rows, decoded by the reference's nvfp4_row
        for r, t in enumerate(toks):
            R.xr_nvfp4_row(O.ptr(c_head, u8p), O.ptr(s_head, u8p), g, cfg["vocab"], H, t, O.ptr(x[r], f32p))
        work = np.zeros(m * (4 * H + 3 * Q + 2 * F) + 64, np.float32)
        e = 0
        for _ in range(cfg["n_in"]):
            assert R.xr_sublayer(pool, C.byref(shape), C.byref(subs[e]), O.ptr(x, f32p), m, pos, 1,
                                 O.ptr(work, f32p)) == 0, R.xr_last_error()
            e += 1
        inp = x.copy()
        state = x.copy()
        for _ in range(cfg["loops"]):
            x = np.ascontiguousarray(state + inp, np.float32)
            R.xr_justnorm(O.ptr(x, f32p), m, H)
            for _ in range(cfg["n_rec"]):
                assert R.xr_sublayer(pool, C.byref(shape), C.byref(subs[e]), O.ptr(x, f32p), m, pos, 1,
                                     O.ptr(work, f32p)) == 0, R.xr_last_error()
                e += 1
            state = x.copy()
            R.xr_justnorm(O.ptr(state, f32p), m, H)
        x = state.copy()
        for _ in range(cfg["n_out"]):
            assert R.xr_sublayer(pool, C.byref(shape), C.byref(subs[e]), O.ptr(x, f32p), m, pos, 1,
                                 O.ptr(work, f32p)) == 0, R.xr_last_error()
            e += 1
        logits = np.zeros((m, cfg["vocab"]), np.float32)
        assert R.xr_head(pool, O.ptr(c_head, u8p), O.ptr(s_head, u8p), g, cfg["vocab"], H, O.ptr(x, f32p), m,
                         O.ptr(ls, f32p), O.ptr(logits, f32p)) == 0
        out.append(logits)
        pos += m
    for c in caches:
        R.xr_kv_free(c)
    R.xr_pool_free(pool)
    model.close()
    return out


SAMPLING_VOCABS = (4096, 131072)
SAMPLING_ROWS = 4
SAMPLING_DRAWS = 12
SAMPLING_TOPK = 64
# (temperature, top_k, top_p, min_p)
SAMPLING_PARAMS = [(0.0, 0, 1.0, 0.0), (0.7, 40, 1.0, 0.0), (1.0, 0, 0.9, 0.0), (0.8, 0, 1.0, 0.05),
                   (1.2, 50, 0.95, 0.02), (1.0, 0, 1.0, 0.0), (0.6, 0, 0.5, 0.1), (0.05, 0, 0.99, 0.0)]


def sampling_inputs(vocab):
    """Logits rows N(0, 3^2) with ties: row 1 repeats its max ten times, row 2 rounds every 7th entry to 0.1, row 3
    is rounded to 0.5 throughout (many equal values)."""
    rng = np.random.default_rng(9 + vocab)
    x = (rng.standard_normal((SAMPLING_ROWS, vocab)) * 3.0).astype(np.float32)
    x[1, 100:110] = x[1].max()
    x[2, ::7] = np.round(x[2, ::7], 1)
    x[3] = np.round(x[3] * 2.0) / 2.0
    return x


def sampling_fixture(R):
    res = {}
    for vocab in SAMPLING_VOCABS:
        x = sampling_inputs(vocab)
        am = np.array([R.xr_argmax(O.ptr(np.ascontiguousarray(r), f32p), vocab) for r in x], np.int32)
        lp = np.zeros((SAMPLING_ROWS, SAMPLING_TOPK), np.float32)
        ix = np.zeros((SAMPLING_ROWS, SAMPLING_TOPK), np.int32)
        tok = np.zeros((SAMPLING_ROWS, len(SAMPLING_PARAMS), SAMPLING_DRAWS), np.int32)
        us = np.zeros((SAMPLING_ROWS, len(SAMPLING_PARAMS), SAMPLING_DRAWS), np.float64)
        for r in range(SAMPLING_ROWS):
            row = np.ascontiguousarray(x[r])
            assert R.xr_top_logprobs(O.ptr(row, f32p), vocab, SAMPLING_TOPK, O.ptr(lp[r], f32p),
                                     ix[r].ctypes.data_as(O.i32p)) == 0
            for pi, (t, k, tp, mp) in enumerate(SAMPLING_PARAMS):
                for d in range(SAMPLING_DRAWS):
                    u = C.c_double()
                    tok[r, pi, d] = R.xr_sample(O.ptr(row, f32p), vocab, t, k, tp, mp, 1000 + 17 * d, C.byref(u))
                    us[r, pi, d] = u.value
        res[f"v{vocab}_argmax"] = am
        res[f"v{vocab}_top_lp"] = lp
        res[f"v{vocab}_top_idx"] = ix
        res[f"v{vocab}_tokens"] = tok
        res[f"v{vocab}_u"] = us
    np.savez_compressed(os.path.join(HERE, "sampling.npz"), **res)


def main():
    R = O.ref()
    assert R is not None, "oracle/_ref/libxtgref.so missing: run `make -C oracle ref` with the reference present"
    if sys.argv[1:] == ["sampling"]:
        sampling_fixture(R)
        print("sampling.npz written to", HERE)
        return
    pool = R.xr_pool_new(4)
    # e4m3
    grid = e4m3_grid()
    codes = np.array([R.xr_f32_to_e4m3(float(v)) for v in grid], np.uint8)
    table = np.array([R.xr_e4m3_to_f32(b) for b in range(256)], np.float32)
    np.savez_compressed(os.path.join(HERE, "e4m3.npz"), grid=grid, codes=codes, table=table)
    # nvfp4
    ws, x = fused_inputs()
    res = {}
    for m in NVFP4_FUSED["ms"]:
        ya, yb = O.ref_matmul_nvfp4(pool, ws, x[:m])
        res[f"fused_m{m}_a"] = ya
        res[f"fused_m{m}_b"] = yb
    w, xq = quant_inputs()
    for m in NVFP4_QUANT["ms"]:
        res[f"quant_m{m}"] = O.ref_matmul_nvfp4(pool, [w], xq[:m])[0]
    np.savez_compressed(os.path.join(HERE, "nvfp4.npz"), **res)
    # attention over FP8 KvCaches
    res = {}
    h, kvh, d = ATTN_SHAPE["heads"], ATTN_SHAPE["kv_heads"], ATTN_SHAPE["d"]
    for ci, (cached, n_q, window) in enumerate(ATTN_CASES):
        K, V, q = attention_inputs(ci)
        total = cached + n_q
        cache = R.xr_kv_new(kvh, d, total + 8, window if window > 0 else 0, 1)
        for p in range(0, cached, 50):
            n = min(50, cached - p)
            kk = np.ascontiguousarray(K[p:p + n])
            vv = np.ascontiguousarray(V[p:p + n])
            assert R.xr_kv_store(cache, p, n, O.ptr(kk, f32p), O.ptr(vv, f32p)) == 0
        out = np.zeros((n_q, h, d), np.float32)
        kn = np.ascontiguousarray(K[cached:])
        vn = np.ascontiguousarray(V[cached:])
        qq = np.ascontiguousarray(q)
        assert R.xr_attention(pool, n_q, cached, h, kvh, d, window, ATTN_SHAPE["scale"], O.ptr(qq, f32p),
                              O.ptr(kn, f32p), O.ptr(vn, f32p), cache, O.ptr(out, f32p)) == 0
        res[f"case{ci}"] = out
        R.xr_kv_free(cache)
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **res)
    # elementwise
    x, o, lr, qr, g, u, sg, su = elementwise_inputs()
    jn = x.copy()
    R.xr_justnorm(O.ptr(jn, f32p), 8, 384)
    sl = x.copy()
    R.xr_slerp_residual(O.ptr(sl, f32p), O.ptr(o, f32p), O.ptr(lr, f32p), 8, 384)
    rp = qr.copy()
    R.xr_rope(O.ptr(rp, f32p), 3, 6, 128, 8190, 1e6)
    sw = g.copy()
    R.xr_swiglu_scaled(O.ptr(sw, f32p), O.ptr(u, f32p), O.ptr(sg, f32p), O.ptr(su, f32p), 4, 512)
    np.savez_compressed(os.path.join(HERE, "elementwise.npz"), justnorm=jn, slerp=sl, rope=rp, swiglu=sw)
    # step
    logits = reference_steps(TINY, STEP_TOKENS)
    np.savez_compressed(os.path.join(HERE, "step_fp8.npz"), **{f"step{i}": l for i, l in enumerate(logits)})
    sampling_fixture(R)
    R.xr_pool_free(pool)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
