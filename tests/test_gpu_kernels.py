"""GPU: the sm_100a kernels against the oracle (CPU restatement, itself pinned to the reference's outputs).

Bars: integer / byte work bit-exact (generators, quantizer, int8 / FP8 KV encode); NVFP4
GEMV and attention within 2e-3 relative error per output, floored by the outputs' RMS:
    |gpu - oracle| <= 2e-3 * max(|oracle|, rms(oracle)).
"""
import math
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as G  # noqa: E402
import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 2e-3


def close_rel(got, ref, tol=TOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = math.sqrt((ref ** 2).mean())
    bound = tol * np.maximum(np.abs(ref), rms)
    worst = (np.abs(got - ref) / np.maximum(np.abs(ref), rms)).max()
    return bool(np.all(np.abs(got - ref) <= bound)), worst


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---- generators and the quantizer: bit-exact ----

def test_generators_bit_exact(cuda, xtg, torch_mod):
    torch = torch_mod
    n = 1 << 20
    g = torch.empty(n, dtype=torch.int16, device="cuda")
    xtg.gen(0, 3, 1234, 0.02, 0.0, g)
    assert np.array_equal(g.cpu().numpy().view(np.uint16), O.gen_normal_bf16(3, 1234, 0.02, n))
    u = torch.empty(n, dtype=torch.float32, device="cuda")
    xtg.gen(1, 3, 77, 0.005, 0.02, u)
    assert np.array_equal(u.cpu().numpy().view(np.uint32), O.gen_uniform(3, 77, 0.005, 0.02, n).view(np.uint32))
    i8 = torch.empty(n, dtype=torch.int8, device="cuda")
    xtg.gen(2, 5, 9, 0, 0, i8)
    assert np.array_equal(i8.cpu().numpy(), O.gen_int8(5, 9, n))


@pytest.mark.parametrize("n,k", [(96, 512), (9216, 3072), (3072, 9216), (70, 256)])
def test_quantizer_bit_exact(cuda, xtg, torch_mod, n, k):
    torch = torch_mod
    raw, codes, scales, g = O.synth_weight(0, 30 + n, n, k)
    dc, ds, dg = xtg.quantize_nvfp4(dev(torch, raw.view(np.int16)))
    assert np.array_equal(dc.cpu().numpy(), codes)
    assert np.array_equal(ds.cpu().numpy(), scales)
    assert np.float32(dg.item()) == np.float32(g)


# ---- the NVFP4 GEMV (matmul_nvfp4) ----

def run_linear(xtg, torch, weights, x):
    k = x.shape[1]
    dw = [(dev(torch, c), dev(torch, s), g) for c, s, g in weights]
    L = xtg.Linear(dw, k)
    ys = L(dev(torch, x.astype(np.float32)))
    out = [y.cpu().numpy() for y in ys]
    L.close()
    return out


def test_gemv_reference_recipe(cuda, xtg, torch_mod):
    """kernels_test.cpp:57-87's case (two fused weights 70x256 and 33x256, m in 1, 2, 7) against the reference's own
    outputs (golden) and the oracle."""
    gold = np.load(os.path.join(HERE, "golden", "nvfp4.npz"))
    ws, x = G.fused_inputs()
    for m in G.NVFP4_FUSED["ms"]:
        ya, yb = run_linear(xtg, torch_mod, ws, x[:m])
        ok, worst = close_rel(np.concatenate([ya.ravel(), yb.ravel()]),
                              np.concatenate([gold[f"fused_m{m}_a"].ravel(), gold[f"fused_m{m}_b"].ravel()]))
        assert ok, (m, worst)


@pytest.mark.parametrize("n,k", [(9216, 3072), (3072, 9216)])
@pytest.mark.parametrize("m", [1, 8])
def test_gemv_config0(cuda, xtg, torch_mod, n, k, m):
    """W ~ N(0, 0.02) quantized, x bf16 ~ N(0, 1)."""
    raw, codes, scales, g = O.synth_weight(0, 7000 + n, n, k)
    x = O.bf16_to_f32(O.gen_normal_bf16(0, 7100 + k, 1.0, 8 * k)).reshape(8, k)[:m]
    got = run_linear(xtg, torch_mod, [(codes, scales, g)], x)[0]
    ref = O.matmul_nvfp4([(codes, scales, g)], x)[0]
    ok, worst = close_rel(got, ref)
    assert ok, worst


@pytest.mark.parametrize("m", [1, 8])
def test_gemv_config1_projection_set(cuda, xtg, torch_mod, m):
    """QKV (4608, fused), QKVG (7680), O, gate+up (fused), down; hidden 3072."""
    H, F, Q, KV = 3072, 9216, 3072, 768
    x = O.bf16_to_f32(O.gen_normal_bf16(1, 7200, 1.0, 8 * F)).reshape(8, F)
    sets = {
        "qkvg": ([(Q, H), (KV, H), (KV, H), (Q, H)], H),
        "o": ([(H, Q)], Q),
        "gate_up": ([(F, H), (F, H)], H),
        "down": ([(H, F)], F),
    }
    for name, (shapes, k) in sets.items():
        ws = [O.synth_weight(1, 7300 + 16 * i + len(name), n, kk)[1:] for i, (n, kk) in enumerate(shapes)]
        got = run_linear(xtg, torch_mod, ws, x[:m, :k])
        ref = O.matmul_nvfp4(ws, x[:m, :k])
        ok, worst = close_rel(np.concatenate([g_.ravel() for g_ in got]), np.concatenate([r.ravel() for r in ref]))
        assert ok, (name, worst)


def test_gemv_ragged_shapes(cuda, xtg, torch_mod):
    """Rows not a multiple of 16 and inputs not a multiple of 64 (padding), fused with uneven weights."""
    k = 336
    ws = [O.synth_weight(2, 7400 + i, n, k)[1:] for i, n in enumerate((1, 17, 100))]
    x = O.gen_uniform(2, 7500, -1.0, 1.0, 5 * k).reshape(5, k)
    got = run_linear(xtg, torch_mod, ws, x)
    ref = O.matmul_nvfp4(ws, x)
    ok, worst = close_rel(np.concatenate([g_.ravel() for g_ in got]), np.concatenate([r.ravel() for r in ref]))
    assert ok, worst


def test_gemv_deterministic(cuda, xtg, torch_mod):
    torch = torch_mod
    raw, codes, scales, g = O.synth_weight(4, 7600, 3072, 9216)
    x = dev(torch, O.gen_uniform(4, 7601, -1.0, 1.0, 8 * 9216).reshape(8, 9216))
    L = xtg.Linear([(dev(torch, codes), dev(torch, scales), g)], 9216)
    a = L(x)[0].cpu().numpy()
    b = L(x)[0].cpu().numpy()
    L.close()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ---- the tensor-core GEMM (matmul_nvfp4's m > 2 path: prefill chunks, batches) ----

@pytest.mark.parametrize("m", [9, 33, 70])
def test_gemm_ragged_shapes(cuda, xtg, torch_mod, m):
    """Rows past a tile of 32, inputs not a multiple of 64 (padding), fused uneven weights; against the oracle."""
    k = 336
    ws = [O.synth_weight(2, 7700 + i, n, k)[1:] for i, n in enumerate((1, 17, 100, 130))]
    x = O.gen_uniform(2, 7800 + m, -1.0, 1.0, m * k).reshape(m, k)
    got = run_linear(xtg, torch_mod, ws, x)
    ref = O.matmul_nvfp4(ws, x)
    ok, worst = close_rel(np.concatenate([g_.ravel() for g_ in got]), np.concatenate([r.ravel() for r in ref]))
    assert ok, worst


def test_gemm_config1_m512(cuda, xtg, torch_mod):
    """BASELINE config 1 at M = 512 (a prefill chunk on tcgen05): the full projection set runs on the GPU; the oracle
    checks the first and last 128 output rows of every weight (the scalar oracle at full size takes minutes)."""
    H, F, Q, KV, M = 3072, 9216, 3072, 768, 512
    x = O.bf16_to_f32(O.gen_normal_bf16(1, 7900, 1.0, M * F)).reshape(M, F)
    sets = {
        "qkvg": ([(Q, H), (KV, H), (KV, H), (Q, H)], H),
        "o": ([(H, Q)], Q),
        "gate_up": ([(F, H), (F, H)], H),
        "down": ([(H, F)], F),
    }
    for name, (shapes, k) in sets.items():
        ws = [O.synth_weight(1, 8000 + 16 * i + len(name), n, kk)[1:] for i, (n, kk) in enumerate(shapes)]
        got = run_linear(xtg, torch_mod, ws, x[:, :k])
        for (codes, scales, g), y in zip(ws, got):
            n = codes.shape[0]
            for lo in (0, n - 128):
                sub = [(codes[lo:lo + 128], scales[lo:lo + 128], g)]
                ref = O.matmul_nvfp4(sub, x[:, :k])[0]
                ok, worst = close_rel(y[:, lo:lo + 128], ref)
                assert ok, (name, lo, worst)


def test_gemm_deterministic(cuda, xtg, torch_mod):
    torch = torch_mod
    raw, codes, scales, g = O.synth_weight(4, 8100, 1024, 3072)
    x = dev(torch, O.gen_uniform(4, 8101, -1.0, 1.0, 200 * 3072).reshape(200, 3072))
    L = xtg.Linear([(dev(torch, codes), dev(torch, scales), g)], 3072)
    a = L(x)[0].cpu().numpy()
    b = L(x)[0].cpu().numpy()
    L.close()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ---- attention ----

def swz_k(s64):
    return (s64 ^ (s64 >> 3)) & 7


def k_index(kvh, slots, D=128):
    """Flat position of element (h, s, d) of K in the library's layout (include/xtg_cuda.h), shape [h][s][d]: each
    128-dim half of a row swizzled in 16-byte units."""
    h, sl, d = np.meshgrid(np.arange(kvh), np.arange(slots), np.arange(D), indexing="ij")
    return (h * slots + sl) * D + 128 * (d >> 7) + 16 * (((d >> 4) & 7) ^ swz_k(sl & 63)) + (d & 15)


def v_index(kvh, slots, D=128):
    """Flat position of element (h, d, s) of V, shape [h][d][s]."""
    h, d, sl = np.meshgrid(np.arange(kvh), np.arange(D), np.arange(slots), indexing="ij")
    return ((h * (slots // 64) + sl // 64) * D + d) * 64 + 16 * (((sl & 63) >> 4) ^ ((d >> 1) & 3)) + (sl & 15)


def cache_to_device(torch, codes_k, codes_v, ks, vs):
    """Oracle layout [slots][kv_heads][D] / [slots][kv_heads] -> the library's K and V layouts and scales
    [h][slots]."""
    slots, kvh, D = codes_k.shape
    kc = np.zeros(kvh * slots * D, np.uint8)
    vc = np.zeros_like(kc)
    kc[k_index(kvh, slots, D)] = codes_k.transpose(1, 0, 2)
    vc[v_index(kvh, slots, D)] = codes_v.transpose(1, 2, 0)
    return dev(torch, kc), dev(torch, vc), dev(torch, np.ascontiguousarray(ks.T)), dev(torch, np.ascontiguousarray(vs.T))


def rope_rows(x, pos0, theta):
    x = np.ascontiguousarray(x, np.float32).copy()
    L = O.lib()
    L.xo_rope(O.ptr(x, O.f32p), x.shape[0], x.shape[1], x.shape[2], pos0, theta)
    return x


def config2_inputs(seed, slots, n_q, ring, heads=24, kvh=6, d=128):
    ck = O.gen_int8(seed, 1, slots * kvh * d).view(np.uint8).reshape(slots, kvh, d)
    cv = O.gen_int8(seed, 2, slots * kvh * d).view(np.uint8).reshape(slots, kvh, d)
    ks = O.gen_uniform(seed, 3, 0.005, 0.02, slots * kvh).reshape(slots, kvh)
    vs = O.gen_uniform(seed, 4, 0.005, 0.02, slots * kvh).reshape(slots, kvh)
    q = O.bf16_to_f32(O.gen_normal_bf16(seed, 5, 1.0, n_q * heads * d)).reshape(n_q, heads, d)
    k = O.bf16_to_f32(O.gen_normal_bf16(seed, 6, 1.0, n_q * kvh * d)).reshape(n_q, kvh, d)
    v = O.bf16_to_f32(O.gen_normal_bf16(seed, 7, 1.0, n_q * kvh * d)).reshape(n_q, kvh, d)
    return ck, cv, ks, vs, q, k, v


@pytest.mark.parametrize("L", [4096, 8192, 32768])
def test_attention_config2_global(cuda, xtg, torch_mod, L):
    """BASELINE config 2, global layer: 8 rows at p = L - 8 over L - 8 cached positions (slot = position)."""
    torch = torch_mod
    pos0, n_q = L - 8, 8
    ck, cv, ks, vs, q, k, v = config2_inputs(20 + L, L, n_q, False)
    q = rope_rows(q, pos0, 1e6)
    k = rope_rows(k, pos0, 1e6)
    scale = 1.0 / math.sqrt(128)
    ref = O.attention(q, k, v, ck, cv, ks, vs, pos0, 0, scale)
    kc, vc, kss, vss = cache_to_device(torch, ck, cv, ks, vs)
    for splits in (1, 24):
        got = xtg.attention(dev(torch, q), dev(torch, k), dev(torch, v), kc, vc, kss, vss, pos0, 0, scale,
                            splits=splits).cpu().numpy()
        ok, worst = close_rel(got, ref)
        assert ok, (splits, worst)


def test_attention_config2_sliding_ring(cuda, xtg, torch_mod):
    """BASELINE config 2, sliding layer: a 1088-slot ring holding the most recent 1088 positions in rotated slot
    order, window 1024; the mask comes from the slot -> position table."""
    torch = torch_mod
    ring, window, n_q = 1088, 1024, 8
    pos0 = 8192 - 8 + 37
    ck, cv, ks, vs, q, k, v = config2_inputs(99, ring, n_q, True)
    ring_pos = np.array([pos0 - 1 - ((pos0 - 1 - s) % ring) for s in range(ring)], np.int64)
    q = rope_rows(q, pos0, 1e6)
    k = rope_rows(k, pos0, 1e6)
    scale = 1.0 / math.sqrt(128)
    ref = O.attention(q, k, v, ck, cv, ks, vs, pos0, window, scale, ring_pos=ring_pos)
    kc, vc, kss, vss = cache_to_device(torch, ck, cv, ks, vs)
    rp = dev(torch, ring_pos.astype(np.int32))
    for splits in (1, 8, 17):
        got = xtg.attention(dev(torch, q), dev(torch, k), dev(torch, v), kc, vc, kss, vss, pos0, window, scale,
                            ring_pos=rp, splits=splits).cpu().numpy()
        ok, worst = close_rel(got, ref)
        assert ok, (splits, worst)


@pytest.mark.parametrize("dtype", [O.KV_I8, O.KV_FP8])
@pytest.mark.parametrize("case", [(300, 1, 0), (5000, 1, 0), (300, 1, 64), (100, 7, 0), (100, 8, 16), (0, 8, 0),
                                  (900, 3, 128), (64, 1, 0), (1, 2, 0)])
def test_attention_reference_cases(cuda, xtg, torch_mod, dtype, case):
    """kernels_test.cpp:139-141's cases (cached, n_q, window) with head_dim 128, 8 q / 2 KV heads, scale 0.7; n_q
    capped at the 8 rows of a verify step. Window cases run as a ring of window + 64 slots holding the latest
    positions, with stale slots marked -1."""
    torch = torch_mod
    cached, n_q, window = case
    heads, kvh, d = 8, 2, 128
    total = cached + n_q
    K = O.gen_uniform(31, 1, -1.0, 1.0, total * kvh * d).reshape(total, kvh, d)
    V = O.gen_uniform(31, 2, -1.0, 1.0, total * kvh * d).reshape(total, kvh, d)
    q = O.gen_uniform(31, 3, -1.0, 1.0, n_q * heads * d).reshape(n_q, heads, d)
    ring = window > 0
    slots = (window + 64 + 63) // 64 * 64 if ring else max(64, (total + 63) // 64 * 64)
    ck = np.zeros((slots, kvh, d), np.uint8)
    cv = np.zeros_like(ck)
    ks = np.zeros((slots, kvh), np.float32)
    vs = np.zeros_like(ks)
    rp = np.full(slots, -1, np.int64)
    for p in range(cached):
        s = p % slots
        (ck[s], ks[s]), (cv[s], vs[s]) = O.kv_encode(dtype, K[p]), O.kv_encode(dtype, V[p])
        rp[s] = p
    ref = O.attention(q, K[cached:], V[cached:], ck, cv, ks, vs, cached, window, 0.7,
                      ring_pos=rp if ring else None, dtype=dtype)
    kc, vc, kss, vss = cache_to_device(torch, ck, cv, ks, vs)
    got = xtg.attention(dev(torch, q), dev(torch, K[cached:]), dev(torch, V[cached:]), kc, vc, kss, vss, cached,
                        window, 0.7, ring_pos=dev(torch, rp.astype(np.int32)) if ring else None, dtype=dtype,
                        splits=3).cpu().numpy()
    ok, worst = close_rel(got, ref)
    assert ok, worst


@pytest.mark.parametrize("ring", [False, True])
def test_attention_head_dim_256(cuda, xtg, torch_mod, ring):
    """The real Dory 4B's attention shape: head_dim 256, 16 q / 4 KV heads; a global cache of 4096 positions and a
    1088-slot rotated ring (window 1024), int8 codes, at several splits, against the oracle."""
    torch = torch_mod
    n_q = 8
    slots = 1088 if ring else 4096
    pos0 = 5000 if ring else 4088
    ck, cv, ks, vs, q, k, v = config2_inputs(7 + ring, slots, n_q, ring, heads=16, kvh=4, d=256)
    q = rope_rows(q, pos0, 1e4)
    k = rope_rows(k, pos0, 1e4)
    scale = 1.0 / math.sqrt(256)
    rp = np.array([pos0 - 1 - ((pos0 - 1 - s) % slots) for s in range(slots)], np.int64) if ring else None
    window = 1024 if ring else 0
    ref = O.attention(q, k, v, ck, cv, ks, vs, pos0, window, scale, ring_pos=rp)
    kc, vc, kss, vss = cache_to_device(torch, ck, cv, ks, vs)
    for splits in ((1, 17) if ring else (1, 5, 37)):
        got = xtg.attention(dev(torch, q), dev(torch, k), dev(torch, v), kc, vc, kss, vss, pos0, window, scale,
                            ring_pos=dev(torch, rp.astype(np.int32)) if ring else None, splits=splits).cpu().numpy()
        ok, worst = close_rel(got, ref)
        assert ok, (splits, worst)


# ---- KV store: bit-exact encode ----

@pytest.mark.parametrize("dtype", [O.KV_I8, O.KV_FP8])
@pytest.mark.parametrize("ring", [False, True])
def test_kv_store_bit_exact(cuda, xtg, torch_mod, dtype, ring):
    torch = torch_mod
    kvh, slots, n, pos = 3, 128, 70 if not ring else 200, 30
    k = O.gen_uniform(41, 1, -3.0, 3.0, n * kvh * 128).reshape(n, kvh, 128)
    v = O.gen_uniform(41, 2, -0.2, 0.2, n * kvh * 128).reshape(n, kvh, 128)
    k[5, 1] = 0.0
    kc = torch.zeros(kvh * slots * 128, dtype=torch.uint8, device="cuda")
    vc = torch.zeros(kvh * slots * 128, dtype=torch.uint8, device="cuda")
    kss = torch.zeros((kvh, slots), dtype=torch.float32, device="cuda")
    vss = torch.zeros((kvh, slots), dtype=torch.float32, device="cuda")
    xtg.kv_store(dev(torch, k), dev(torch, v), pos, slots, ring, dtype, kc, vc, kss, vss)
    kc, vc, kss, vss = kc.cpu().numpy(), vc.cpu().numpy(), kss.cpu().numpy(), vss.cpu().numpy()
    kc = kc[k_index(kvh, slots)]          # [h][s][d]
    vc = vc[v_index(kvh, slots)]          # [h][d][s]
    first = pos + n - slots if ring and n > slots else pos
    for p in range(first, pos + n):
        s = p % slots if ring else p
        for h in range(kvh):
            c, sc = O.kv_encode(dtype, k[p - pos, h][None])
            assert np.array_equal(kc[h, s], c[0]) and kss[h, s] == sc[0]
            c, sc = O.kv_encode(dtype, v[p - pos, h][None])
            assert np.array_equal(vc[h, :, s], c[0]) and vss[h, s] == sc[0]


# ---- top-k candidates of the sampler (engine/src/sampler.cpp): bit-exact indices and values ----

def _total_f32_exp(row, temperature):
    inv_t = np.float32(1.0) / np.float32(temperature)
    return float(np.sum(np.exp((row - row.max()) * inv_t).astype(np.float32).astype(np.float64)))


@pytest.mark.parametrize("vocab", G.SAMPLING_VOCABS)
def test_topk_rows_match_oracle(cuda, xtg, torch_mod, vocab):
    """The fixture's rows (ties: a repeated max, rounded entries, a row of half-integers) at k from 1 to 1024."""
    torch = torch_mod
    x = G.sampling_inputs(vocab)
    t = torch.from_numpy(x).cuda()
    for k in (1, 5, 64, 1024):
        for temp in (1.0, 0.7):
            idx, val, mx, tot = xtg.topk(t, k, temp)
            torch.cuda.synchronize()
            idx, val, mx, tot = idx.cpu().numpy(), val.cpu().numpy(), mx.cpu().numpy(), tot.cpu().numpy()
            for r in range(G.SAMPLING_ROWS):
                ri, rv = O.topk(x[r], k)
                np.testing.assert_array_equal(idx[r], ri, err_msg=f"k={k} row {r}")
                np.testing.assert_array_equal(val[r], rv)
                assert mx[r] == x[r].max()
                assert abs(tot[r] - _total_f32_exp(x[r], temp)) <= 1e-6 * tot[r]


@pytest.mark.parametrize("vocab,k", [(7, 7), (1000, 1000), (1001, 3), (4099, 1024), (131071, 100)])
def test_topk_rows_ragged(cuda, xtg, torch_mod, vocab, k):
    """Rows that do not fill the cluster's entries (scalar loads, entries past the row), k up to the whole row."""
    torch = torch_mod
    rng = np.random.default_rng(vocab)
    x = np.round(rng.standard_normal((3, vocab)) * 4).astype(np.float32)   # many ties
    idx, val, mx, tot = xtg.topk(torch.from_numpy(x).cuda(), k, 1.0)
    torch.cuda.synchronize()
    for r in range(3):
        ri, rv = O.topk(x[r], k)
        np.testing.assert_array_equal(idx[r].cpu().numpy(), ri)
        np.testing.assert_array_equal(val[r].cpu().numpy(), rv)
        assert abs(tot[r].item() - _total_f32_exp(x[r], 1.0)) <= 1e-6 * tot[r].item()


def test_topk_rejects_bad_k(cuda, xtg, torch_mod):
    t = torch_mod.zeros(2, 100, device="cuda")
    for k in (0, 101, 1025):
        with pytest.raises(xtg.XtgError):
            xtg.topk(t, k)


def test_topk_rows_unaligned_pointer(cuda, xtg, torch_mod):
    """Rows starting one float past a 16-byte boundary (a caller's sub-view) take the scalar loads."""
    torch = torch_mod
    rng = np.random.default_rng(11)
    x = rng.standard_normal((2, 4096)).astype(np.float32)
    buf = torch.zeros(2 * 4096 + 1, device="cuda")
    buf[1:] = torch.from_numpy(x.reshape(-1)).cuda()
    view = buf[1:].view(2, 4096)
    assert view.data_ptr() % 16 == 4
    idx, val, mx, tot = xtg.topk(view, 64, 1.0)
    torch.cuda.synchronize()
    for r in range(2):
        ri, rv = O.topk(x[r], 64)
        np.testing.assert_array_equal(idx[r].cpu().numpy(), ri)
        np.testing.assert_array_equal(val[r].cpu().numpy(), rv)
