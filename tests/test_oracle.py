"""CPU: the oracle (C restatement) pinned against the reference's own outputs (tests/golden, produced by the
reference's compiled kernels) and the known answers of the reference's tests/kernels_test.cpp."""
import math
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as G  # noqa: E402  (case definitions; the reference itself is not run here)
import oracle as O  # noqa: E402

GOLD = os.path.join(HERE, "golden")


def gold(name):
    return np.load(os.path.join(GOLD, name))


# ---- number formats: kernels_test.cpp:30-41 ----

def test_e4m3_known_answers():
    L = O.lib()
    assert L.xo_e4m3_to_f32(0x38) == 1.0
    assert L.xo_e4m3_to_f32(0x7E) == 448.0
    assert L.xo_e4m3_to_f32(0x01) == math.ldexp(1.0, -9)
    assert math.isnan(L.xo_e4m3_to_f32(0x7F))
    for c in range(256):
        if (c & 0x7F) == 0x7F:
            continue
        assert L.xo_f32_to_e4m3(L.xo_e4m3_to_f32(c)) == c
    assert L.xo_f32_to_e4m3(1000.0) == 0x7E and L.xo_f32_to_e4m3(-1000.0) == 0xFE
    assert L.xo_f32_to_bf16(1.0) == 0x3F80 and L.xo_bf16_to_f32(0x3F80) == 1.0


def test_e4m3_matches_reference_grid():
    g = gold("e4m3.npz")
    L = O.lib()
    got = np.array([L.xo_f32_to_e4m3(float(v)) for v in g["grid"]], np.uint8)
    np.testing.assert_array_equal(got, g["codes"])
    table = O.e4m3_table()
    ref = g["table"]
    fin = np.isfinite(ref)
    np.testing.assert_array_equal(table[fin], ref[fin])
    assert np.all(np.isnan(table[~fin]))


# ---- NVFP4: kernels_test.cpp:57-87 and the reference's own outputs ----

def rms_err(y, ref):
    ref = np.asarray(ref, np.float64)
    return np.abs(np.asarray(y, np.float64) - ref).max() / math.sqrt((ref ** 2).mean())


def test_nvfp4_matmul_matches_reference_and_double():
    g = gold("nvfp4.npz")
    ws, x = G.fused_inputs()
    for m in G.NVFP4_FUSED["ms"]:
        ya, yb = O.matmul_nvfp4(ws, x[:m])
        # the reference's outputs
        assert rms_err(ya, g[f"fused_m{m}_a"]) < 2e-6
        assert rms_err(yb, g[f"fused_m{m}_b"]) < 2e-6
        # kernels_test's bar: against a double dot over the decoded rows, < 2e-5 of the output RMS
        ex = [x[:m].astype(np.float64) @ O.dequant_nvfp4(*w).T for w in ws]
        allref = np.concatenate([e.ravel() for e in ex])
        allgot = np.concatenate([ya.ravel(), yb.ravel()])
        assert rms_err(allgot, allref) < 2e-5
    w, xq = G.quant_inputs()
    for m in G.NVFP4_QUANT["ms"]:
        y = O.matmul_nvfp4([w], xq[:m])[0]
        assert rms_err(y, g[f"quant_m{m}"]) < 2e-6


def test_nvfp4_row_decode_matches_dequant():
    codes, scales, g = G.quant_inputs()[0]
    L = O.lib()
    import ctypes as C
    w = O.Nvfp4(O.ptr(codes, O.u8p), O.ptr(scales, O.u8p), g, codes.shape[0], codes.shape[1] * 2)
    row = np.zeros(codes.shape[1] * 2, np.float32)
    for r in (0, 17, 95):
        L.xo_nvfp4_row(C.byref(w), r, O.ptr(row, O.f32p))
        np.testing.assert_allclose(row, O.dequant_nvfp4(codes, scales, g)[r], rtol=2e-7)


def test_quantizer_properties():
    """The restated quantizer (no reference counterpart): every code decodes to the nearest representable value
    of w / (scale * global) (ties to the even code), scales are the E4M3 encode of amax / (6 * global)."""
    raw, codes, scales, g = O.synth_weight(3, 99, 64, 256)
    w = O.bf16_to_f32(raw).reshape(64, 256)
    assert g == np.float32(np.abs(w).max()) / np.float32(2688.0)
    table = O.e4m3_table()
    L = O.lib()
    six_g = np.float32(6.0) * np.float32(g)
    for r in range(0, 64, 7):
        for grp in range(16):
            blk = w[r, grp * 16:(grp + 1) * 16]
            sc = np.float32(np.abs(blk).max()) / six_g
            assert scales[r, grp] == L.xo_f32_to_e4m3(float(sc))
            denom = np.float32(table[scales[r, grp]]) * np.float32(g)
            q = blk / denom
            c = np.stack([codes[r, grp * 8:(grp + 1) * 8] & 15, codes[r, grp * 8:(grp + 1) * 8] >> 4], -1).ravel()
            vals = O.E2M1[c]
            mags = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float32)
            for qi, vi in zip(q, vals):
                d = np.abs(mags - min(abs(qi), 6.0))
                assert abs(vi) in mags[d == d.min()]
    # the whole dequantized tensor stays within half a step of the block's grid
    err = np.abs(O.dequant_nvfp4(codes, scales, g) - w).max()
    assert err <= np.abs(w).max() / 6.0


# ---- attention: kernels_test.cpp:104-183 ----

@pytest.mark.parametrize("ci", range(len(G.ATTN_CASES)))
def test_attention_fp8_matches_reference(ci):
    cached, n_q, window = G.ATTN_CASES[ci]
    h, kvh, d = G.ATTN_SHAPE["heads"], G.ATTN_SHAPE["kv_heads"], G.ATTN_SHAPE["d"]
    K, V, q = G.attention_inputs(ci)
    total = cached + n_q
    # the restated FP8 encode of the cached rows (the reference's KvCache::store rule); a window cache is a ring of
    # `window` slots there, which the slot -> position table reproduces
    slots = window if window > 0 else total + 8
    ck = np.zeros((slots, kvh, d), np.uint8)
    cv = np.zeros_like(ck)
    cks = np.zeros((slots, kvh), np.float32)
    cvs = np.zeros_like(cks)
    ring_pos = np.full(slots, -1, np.int64) if window > 0 else None
    for p in range(cached):
        s = p % slots
        kc, ks = O.kv_encode(O.KV_FP8, K[p])
        vc, vs = O.kv_encode(O.KV_FP8, V[p])
        ck[s], cks[s], cv[s], cvs[s] = kc, ks, vc, vs
        if ring_pos is not None:
            ring_pos[s] = p
    out = O.attention(q, K[cached:], V[cached:], ck, cv, cks, cvs, cached, window, G.ATTN_SHAPE["scale"],
                      ring_pos=ring_pos, dtype=O.KV_FP8)
    ref = gold("attention.npz")[f"case{ci}"]
    assert np.abs(out - ref).max() < 2e-5


def test_fp8_kv_encode_bit_exact_with_reference():
    """The FP8 KV rows the restatement writes are the reference KvCache's bytes (kv.cpp:94-108)."""
    R = O.ref()
    if R is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    x = O.gen_uniform(5, 1, -2.0, 2.0, 200 * 64).reshape(200, 64)
    c = R.xr_kv_new(1, 64, 200, 0, 1)
    xx = np.ascontiguousarray(x)
    assert R.xr_kv_store(c, 0, 200, O.ptr(xx, O.f32p), O.ptr(xx, O.f32p)) == 0
    kb = np.zeros((200, 64), np.float32)
    vb = np.zeros_like(kb)
    R.xr_kv_load(c, 0, 0, 200, O.ptr(kb, O.f32p), O.ptr(vb, O.f32p))
    R.xr_kv_free(c)
    codes, scales = O.kv_encode(O.KV_FP8, x)
    np.testing.assert_array_equal(O.kv_decode(O.KV_FP8, codes, scales), kb)


def test_fp8_ring_keeps_last_positions():
    """kernels_test.cpp:185-193: an FP8 ring of 64 keeps the last 64 of 3000 positions (error < 0.07 of 0.3)."""
    k = O.gen_uniform(6, 1, -0.3, 0.3, 3000 * 64).reshape(3000, 64)
    codes, scales = O.kv_encode(O.KV_FP8, k[2936:])
    back = O.kv_decode(O.KV_FP8, codes, scales)
    assert np.abs(back - k[2936:]).max() / 0.3 < 0.07


def test_int8_kv_encode_rule():
    x = O.gen_uniform(8, 1, -3.0, 3.0, 50 * 128).reshape(50, 128)
    x[7] = 0.0
    codes, scales = O.kv_encode(O.KV_I8, x)
    c = codes.view(np.int8).astype(np.int32)
    assert np.abs(c).max() <= 127
    amax = np.abs(x).max(1)
    expect = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    np.testing.assert_array_equal(scales, expect)
    np.testing.assert_array_equal(c, np.clip(np.rint(x * (np.float32(1.0) / expect[:, None])), -127, 127))


# ---- elementwise: kernels.cpp:169-234 ----

def test_elementwise_match_reference():
    g = gold("elementwise.npz")
    x, o, lr, qr, gg, u, sg, su = G.elementwise_inputs()
    L = O.lib()
    jn = x.copy()
    L.xo_justnorm(O.ptr(jn, O.f32p), 8, 384)
    np.testing.assert_allclose(jn, g["justnorm"], rtol=0, atol=2e-7)
    sl = x.copy()
    L.xo_slerp_residual(O.ptr(sl, O.f32p), O.ptr(o, O.f32p), O.ptr(lr, O.f32p), 8, 384)
    np.testing.assert_allclose(sl, g["slerp"], rtol=0, atol=2e-7)
    rp = qr.copy()
    L.xo_rope(O.ptr(rp, O.f32p), 3, 6, 128, 8190, 1e6)
    np.testing.assert_allclose(rp, g["rope"], rtol=0, atol=2e-6)
    sw = gg.copy()
    L.xo_swiglu_scaled(O.ptr(sw, O.f32p), O.ptr(u, O.f32p), O.ptr(sg, O.f32p), O.ptr(su, O.f32p), 4, 512)
    np.testing.assert_allclose(sw, g["swiglu"], rtol=2e-6, atol=1e-6)


# ---- the step: the reference's kernels in DorySession order (FP8 caches) ----

def test_step_matches_reference_kernels():
    g = gold("step_fp8.npz")
    m = O.SynthDory(G.TINY, ctx=64, n_prefill=0, kv_dtype=O.KV_FP8)
    for i, toks in enumerate(G.STEP_TOKENS):
        got = m.step(toks)
        ref = g[f"step{i}"]
        assert np.abs(got - ref).max() < 2e-3, (i, np.abs(got - ref).max())
        assert np.array_equal(got.argmax(1), ref.argmax(1))
    m.close()


# ---- ring / masks / rewind: npu/xtg_npu.cpp:236-258, 362-369 ----

def test_masks_and_rewind_semantics():
    ring, window, ctx = 24, 16, 64
    ring_pos = np.full(ring, -1, np.int64)
    n_past = 0
    for step in range(6):
        rows = [8, 8, 3, 8, 5, 8][step]
        mask, wmask = O.fill_masks(8, rows, n_past, ctx, ring, window, ring_pos)
        for i in range(8):
            if i >= rows:
                assert mask[i].sum() == 1 and mask[i, ctx + i] == 1
                assert wmask[i].sum() == 1 and wmask[i, ring + i] == 1
                continue
            p = n_past + i
            assert mask[i, :n_past].all() and not mask[i, n_past:ctx].any()
            assert mask[i, ctx:ctx + i + 1].all() and not mask[i, ctx + i + 1:].any()
            for s in range(ring):
                q = ring_pos[s]
                assert wmask[i, s] == (0 <= q < n_past and p - q < window)
        for r in range(rows):
            ring_pos[(n_past + r) % ring] = n_past + r
        n_past += rows
    # the ring holds positions n_past - ring .. n_past - 1: rewinds that keep the window are allowed
    assert O.rewind_ok(n_past, n_past, window, ring_pos)
    # the lowest position still held is n_past - ring; `to` needs to - window + 1 .. to - 1
    lowest_ok = n_past - ring + window - 1
    assert O.rewind_ok(lowest_ok, n_past, window, ring_pos)
    assert not O.rewind_ok(lowest_ok - 1, n_past, window, ring_pos)
    assert not O.rewind_ok(n_past + 1, n_past, window, ring_pos)
    assert not O.rewind_ok(-1, n_past, window, ring_pos)
