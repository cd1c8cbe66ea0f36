"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers.

* ``lib()``: the C restatement of the Dory verify step (``oracle/libxtg_oracle.so``, built from ``xtg_oracle.c``).
* ``ref()``: XTier Go's own CPU kernels compiled from the reference sources (``oracle/_ref/libxtgref.so``, built by
  ``make -C oracle ref`` where the reference tree is present); ``None`` when that build is absent.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and reference legs may import this
package, and only as the checker or the timed CPU baseline; the product (``libxtg_cuda.so``) never calls it.
"""
import ctypes as C
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libxtg_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libxtgref.so")

_lib = None
_ref = None

f32p = C.POINTER(C.c_float)
u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)
i8p = C.POINTER(C.c_int8)
i32p = C.POINTER(C.c_int32)
i64p = C.POINTER(C.c_int64)


def ptr(a, t):
    return a.ctypes.data_as(t)


class Nvfp4(C.Structure):
    _fields_ = [("codes", u8p), ("scales", u8p), ("global_", C.c_float), ("n_out", C.c_int), ("k", C.c_int)]


class Cache(C.Structure):
    _fields_ = [("dtype", C.c_int), ("ring", C.c_int), ("slots", C.c_int64), ("k", u8p), ("v", u8p),
                ("ks", f32p), ("vs", f32p)]


class Attn(C.Structure):
    _fields_ = [("n_q", C.c_int), ("pos0", C.c_int64), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("window", C.c_int), ("scale", C.c_float), ("q", f32p), ("k", f32p),
                ("v", f32p), ("cache", C.POINTER(Cache)), ("ring_pos", i64p), ("out", f32p)]


class Layer(C.Structure):
    _fields_ = [("kind", C.c_int), ("w", Nvfp4 * 5), ("lr", f32p), ("qscale", f32p), ("gscale", f32p),
                ("sg", f32p), ("su", f32p), ("theta", C.c_float), ("cache", C.c_int)]


class Model(C.Structure):
    _fields_ = [("hidden", C.c_int), ("ffn", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("vocab", C.c_int), ("window", C.c_int), ("n_in", C.c_int),
                ("n_rec", C.c_int), ("n_out", C.c_int), ("loops", C.c_int), ("layers", C.POINTER(Layer)),
                ("head", Nvfp4), ("logit_scale", f32p), ("embed_bf16", u16p), ("head_bf16", u16p)]


class State(C.Structure):
    _fields_ = [("caches", C.POINTER(Cache)), ("n_caches", C.c_int), ("ring_pos", i64p), ("ring", C.c_int),
                ("n_past", C.c_int64)]


SYNTH_FIELDS = [("hidden", C.c_int), ("ffn", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("vocab", C.c_int), ("n_in", C.c_int), ("n_rec", C.c_int),
                ("n_out", C.c_int), ("loops", C.c_int), ("window", C.c_int), ("ring", C.c_int),
                ("global_every", C.c_int), ("theta_sliding", C.c_float), ("theta_global", C.c_float),
                ("weight_std", C.c_float), ("lr_lo", C.c_float), ("lr_hi", C.c_float), ("qs_lo", C.c_float),
                ("qs_hi", C.c_float), ("gs_lo", C.c_float), ("gs_hi", C.c_float), ("suv_lo", C.c_float),
                ("suv_hi", C.c_float), ("ls_lo", C.c_float), ("ls_hi", C.c_float), ("kvs_lo", C.c_float),
                ("kvs_hi", C.c_float), ("seed", C.c_uint64)]


class SynthCfg(C.Structure):
    _fields_ = SYNTH_FIELDS


def build():
    """Compile the restatement (plain gcc); the reference build is ``make -C oracle ref``."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        L.xo_e4m3_to_f32.restype = C.c_float
        L.xo_e4m3_to_f32.argtypes = [C.c_uint8]
        L.xo_f32_to_e4m3.restype = C.c_uint8
        L.xo_f32_to_e4m3.argtypes = [C.c_float]
        L.xo_f32_to_bf16.restype = C.c_uint16
        L.xo_f32_to_bf16.argtypes = [C.c_float]
        L.xo_bf16_to_f32.restype = C.c_float
        L.xo_bf16_to_f32.argtypes = [C.c_uint16]
        L.xo_rand_bits.restype = C.c_uint64
        L.xo_rand_bits.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
        L.xo_gen_normal_bf16.argtypes = [C.c_uint64, C.c_uint64, C.c_float, u16p, C.c_int64]
        L.xo_gen_uniform.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_float, f32p, C.c_int64]
        L.xo_gen_int8.argtypes = [C.c_uint64, C.c_uint64, i8p, C.c_int64]
        L.xo_quantize_nvfp4.argtypes = [u16p, C.c_int, C.c_int, u8p, u8p, f32p]
        L.xo_nvfp4_row.argtypes = [C.POINTER(Nvfp4), C.c_int, f32p]
        L.xo_matmul_nvfp4.argtypes = [C.POINTER(Nvfp4), C.c_int, f32p, C.c_int, C.POINTER(f32p)]
        L.xo_justnorm.argtypes = [f32p, C.c_int, C.c_int]
        L.xo_slerp_residual.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int]
        L.xo_rope.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_int64, C.c_float]
        L.xo_swiglu_scaled.argtypes = [f32p, f32p, f32p, f32p, C.c_int, C.c_int]
        L.xo_kv_encode.argtypes = [C.c_int, f32p, C.c_int, u8p, f32p]
        L.xo_kv_decode.restype = C.c_float
        L.xo_kv_decode.argtypes = [C.c_int, C.c_uint8, C.c_float]
        L.xo_attention.argtypes = [C.POINTER(Attn)]
        L.xo_fill_masks.argtypes = [C.c_int, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int, i64p, u8p, u8p]
        L.xo_rewind_ok.restype = C.c_int
        L.xo_rewind_ok.argtypes = [C.c_int64, C.c_int64, C.c_int, C.c_int, i64p]
        L.xo_step_work_floats.restype = C.c_int64
        L.xo_step_work_floats.argtypes = [C.POINTER(Model), C.c_int]
        L.xo_step.argtypes = [C.POINTER(Model), C.POINTER(State), i32p, C.c_int, f32p, f32p]
        L.xo_argmax.restype = C.c_int
        L.xo_argmax.argtypes = [f32p, C.c_int]
        L.xo_synth_n_evals.restype = C.c_int
        L.xo_synth_n_evals.argtypes = [C.POINTER(SynthCfg)]
        L.xo_synth_kind.restype = C.c_int
        L.xo_synth_kind.argtypes = [C.POINTER(SynthCfg), C.c_int]
        L.xo_synth_model_new.restype = C.POINTER(Model)
        L.xo_synth_model_new.argtypes = [C.POINTER(SynthCfg)]
        L.xo_synth_model_free.argtypes = [C.POINTER(Model)]
        L.xo_synth_state_new.restype = C.POINTER(State)
        L.xo_synth_state_new.argtypes = [C.POINTER(Model), C.POINTER(SynthCfg), C.c_int64, C.c_int, C.c_int64]
        L.xo_synth_state_free.argtypes = [C.POINTER(State)]
        _lib = L
    return _lib


def ref():
    """The reference's own kernels, or None where oracle/_ref was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        R = C.CDLL(REF_SO)
        R.xr_last_error.restype = C.c_char_p
        R.xr_pool_new.restype = C.c_void_p
        R.xr_pool_new.argtypes = [C.c_int]
        R.xr_pool_free.argtypes = [C.c_void_p]
        R.xr_e4m3_to_f32.restype = C.c_float
        R.xr_e4m3_to_f32.argtypes = [C.c_uint8]
        R.xr_f32_to_e4m3.restype = C.c_uint8
        R.xr_f32_to_e4m3.argtypes = [C.c_float]
        R.xr_f32_to_bf16.restype = C.c_uint16
        R.xr_f32_to_bf16.argtypes = [C.c_float]
        R.xr_bf16_to_f32.restype = C.c_float
        R.xr_bf16_to_f32.argtypes = [C.c_uint16]
        R.xr_nvfp4_row.argtypes = [u8p, u8p, C.c_float, C.c_int, C.c_int, C.c_int, f32p]
        R.xr_matmul_nvfp4.restype = C.c_int
        R.xr_matmul_nvfp4.argtypes = [C.c_void_p, C.c_int, C.POINTER(u8p), C.POINTER(u8p), f32p, i32p, C.c_int,
                                      f32p, C.c_int, C.POINTER(f32p)]
        R.xr_justnorm.argtypes = [f32p, C.c_int, C.c_int]
        R.xr_slerp_residual.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int]
        R.xr_rope.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_int64, C.c_float]
        R.xr_swiglu_scaled.argtypes = [f32p, f32p, f32p, f32p, C.c_int, C.c_int]
        R.xr_kv_new.restype = C.c_void_p
        R.xr_kv_new.argtypes = [C.c_int, C.c_int, C.c_int64, C.c_int, C.c_int]
        R.xr_kv_free.argtypes = [C.c_void_p]
        R.xr_kv_store.restype = C.c_int
        R.xr_kv_store.argtypes = [C.c_void_p, C.c_int64, C.c_int, f32p, f32p]
        R.xr_kv_load.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, f32p, f32p]
        R.xr_attention.restype = C.c_int
        R.xr_attention.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                   f32p, f32p, f32p, C.c_void_p, f32p]
        R.xr_sublayer.restype = C.c_int
        R.xr_head.restype = C.c_int
        R.xr_argmax.restype = C.c_int
        R.xr_argmax.argtypes = [f32p, C.c_int]
        R.xr_top_logprobs.restype = C.c_int
        R.xr_top_logprobs.argtypes = [f32p, C.c_int, C.c_int, f32p, i32p]
        R.xr_sample.restype = C.c_int
        R.xr_sample.argtypes = [f32p, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float, C.c_uint64,
                                C.POINTER(C.c_double)]
        R.xr_dory_load.restype = C.c_void_p
        R.xr_dory_load.argtypes = [C.c_char_p, C.c_char_p, C.c_void_p]
        R.xr_dory_free.argtypes = [C.c_void_p]
        R.xr_dory_vocab.restype = C.c_int
        R.xr_dory_vocab.argtypes = [C.c_void_p]
        R.xr_dory_session.restype = C.c_void_p
        R.xr_dory_session.argtypes = [C.c_void_p]
        R.xr_dory_session_free.argtypes = [C.c_void_p]
        R.xr_dory_n_past.restype = C.c_int64
        R.xr_dory_n_past.argtypes = [C.c_void_p]
        R.xr_dory_rewind.restype = C.c_int
        R.xr_dory_rewind.argtypes = [C.c_void_p, C.c_int64]
        R.xr_dory_forward.restype = C.c_int
        R.xr_dory_forward.argtypes = [C.c_void_p, i32p, C.c_int, C.c_int, f32p]
        _ref = R
    return _ref


class RefDory:
    """The reference's own Dory pack (packs/dory/dory.cpp, CPU backend) on a checkpoint directory: DoryModel's
    loader and a DorySession, forward with every row's logits."""

    def __init__(self, directory, threads=0, **options):
        R = ref()
        if R is None:
            raise RuntimeError("oracle/_ref is not built")
        self.R = R
        self.pool = R.xr_pool_new(threads or (os.cpu_count() or 1))
        opts = dict(backend="cpu")
        opts.update(options)
        self.model = R.xr_dory_load(os.fsencode(directory), json.dumps(opts).encode(), self.pool)
        if not self.model:
            R.xr_pool_free(self.pool)
            raise RuntimeError(R.xr_last_error().decode())
        self.vocab = R.xr_dory_vocab(self.model)
        self.s = R.xr_dory_session(self.model)
        if not self.s:
            raise RuntimeError(R.xr_last_error().decode())

    @property
    def n_past(self):
        return self.R.xr_dory_n_past(self.s)

    def forward(self, tokens):
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros((len(toks), self.vocab), np.float32)
        if self.R.xr_dory_forward(self.s, ptr(toks, i32p), len(toks), self.vocab, ptr(out, f32p)) != 0:
            raise RuntimeError(self.R.xr_last_error().decode())
        return out

    def rewind(self, n):
        return self.R.xr_dory_rewind(self.s, n) == 0

    def close(self):
        if getattr(self, "s", None):
            self.R.xr_dory_session_free(self.s)
            self.s = None
        if getattr(self, "model", None):
            self.R.xr_dory_free(self.model)
            self.model = None
        if getattr(self, "pool", None):
            self.R.xr_pool_free(self.pool)
            self.pool = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ----------------------------------------------------------------------------------------------------------------
# numpy conveniences over the restatement
# ----------------------------------------------------------------------------------------------------------------

def gen_normal_bf16(seed, stream, std, n):
    out = np.empty(n, np.uint16)
    lib().xo_gen_normal_bf16(seed, stream, std, ptr(out, u16p), n)
    return out


def gen_uniform(seed, stream, lo, hi, n):
    out = np.empty(n, np.float32)
    lib().xo_gen_uniform(seed, stream, lo, hi, ptr(out, f32p), n)
    return out


def gen_int8(seed, stream, n):
    out = np.empty(n, np.int8)
    lib().xo_gen_int8(seed, stream, ptr(out, i8p), n)
    return out


def bf16_to_f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    L = lib()
    flat = x.reshape(-1)
    o = out.reshape(-1)
    for i in range(flat.size):
        o[i] = L.xo_f32_to_bf16(float(flat[i]))
    return out


def e4m3_table():
    L = lib()
    return np.array([L.xo_e4m3_to_f32(b) for b in range(256)], np.float32)


E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], np.float32)


def quantize_nvfp4(w_bf16):
    """bf16 [n, k] -> (codes u8 [n, k/2], scales u8 [n, k/16], global f32)."""
    w = np.ascontiguousarray(w_bf16, np.uint16)
    n, k = w.shape
    codes = np.empty((n, k // 2), np.uint8)
    scales = np.empty((n, k // 16), np.uint8)
    g = np.zeros(1, np.float32)
    lib().xo_quantize_nvfp4(ptr(w, u16p), n, k, ptr(codes, u8p), ptr(scales, u8p), ptr(g, f32p))
    return codes, scales, float(g[0])


def dequant_nvfp4(codes, scales, global_):
    """The decoded weight [n, k] in float64 (exact products)."""
    n, half = codes.shape
    c = np.stack([codes & 15, codes >> 4], axis=-1).reshape(n, half * 2)
    s = e4m3_table()[scales].astype(np.float64)
    return E2M1[c].astype(np.float64) * np.repeat(s, 16, axis=1) * np.float64(np.float32(global_))


def synth_weight(seed, stream, n, k, std=0.02):
    raw = gen_normal_bf16(seed, stream, std, n * k).reshape(n, k)
    return (raw,) + quantize_nvfp4(raw)


def matmul_nvfp4(weights, x):
    """The restated matmul_nvfp4: weights = [(codes, scales, global)], x f32 [m, k] -> list of [m, n_i]."""
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    nw = len(weights)
    ws = (Nvfp4 * nw)()
    ys = [np.zeros((m, w[0].shape[0]), np.float32) for w in weights]
    keep = []
    for i, (codes, scales, g) in enumerate(weights):
        codes = np.ascontiguousarray(codes)
        scales = np.ascontiguousarray(scales)
        keep += [codes, scales]
        ws[i] = Nvfp4(ptr(codes, u8p), ptr(scales, u8p), g, codes.shape[0], k)
    yp = (f32p * nw)(*[ptr(y, f32p) for y in ys])
    lib().xo_matmul_nvfp4(ws, nw, ptr(x, f32p), m, yp)
    return ys


def ref_matmul_nvfp4(pool, weights, x):
    """The reference's own matmul_nvfp4 (oracle/_ref) on the same bytes."""
    R = ref()
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    nw = len(weights)
    keep = []
    codes_p = (u8p * nw)()
    scales_p = (u8p * nw)()
    globals_ = np.array([w[2] for w in weights], np.float32)
    n_out = np.array([w[0].shape[0] for w in weights], np.int32)
    ys = [np.zeros((m, w[0].shape[0]), np.float32) for w in weights]
    for i, (codes, scales, _) in enumerate(weights):
        codes = np.ascontiguousarray(codes)
        scales = np.ascontiguousarray(scales)
        keep += [codes, scales]
        codes_p[i] = ptr(codes, u8p)
        scales_p[i] = ptr(scales, u8p)
    yp = (f32p * nw)(*[ptr(y, f32p) for y in ys])
    rc = R.xr_matmul_nvfp4(pool, nw, codes_p, scales_p, ptr(globals_, f32p), ptr(n_out, i32p), k, ptr(x, f32p), m,
                           yp)
    assert rc == 0, R.xr_last_error()
    return ys


def kv_encode(dtype, x):
    """Rows x [n, d] -> (codes u8 [n, d], scales f32 [n])."""
    x = np.ascontiguousarray(x, np.float32)
    n, d = x.shape
    codes = np.empty((n, d), np.uint8)
    scales = np.empty(n, np.float32)
    L = lib()
    for r in range(n):
        L.xo_kv_encode(dtype, ptr(x[r], f32p), d, codes[r].ctypes.data_as(u8p),
                       scales[r:].ctypes.data_as(f32p))
    return codes, scales


KV_I8, KV_FP8 = 0, 1


def kv_decode(dtype, codes, scales):
    if dtype == KV_I8:
        return codes.view(np.int8).astype(np.float32) * scales[..., None]
    return e4m3_table()[codes] * scales[..., None]


def attention(q, k, v, cache_k, cache_v, cache_ks, cache_vs, pos0, window, scale, ring_pos=None, dtype=KV_I8):
    """Restated attention. q [n_q, heads, d]; k, v [n_q, kv_heads, d]; cache_* [slots, kv_heads, d] codes and
    [slots, kv_heads] scales; ring_pos: slot -> position for a ring (None: a global cache, slot = position)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    n_q, heads, d = q.shape
    kvh = k.shape[1]
    ck = np.ascontiguousarray(cache_k, np.uint8)
    cv = np.ascontiguousarray(cache_v, np.uint8)
    cks = np.ascontiguousarray(cache_ks, np.float32)
    cvs = np.ascontiguousarray(cache_vs, np.float32)
    slots = ck.shape[0]
    rp = np.ascontiguousarray(ring_pos if ring_pos is not None else np.zeros(1), np.int64)
    c = Cache(dtype, 1 if ring_pos is not None else 0, slots, ptr(ck, u8p), ptr(cv, u8p), ptr(cks, f32p),
              ptr(cvs, f32p))
    out = np.zeros_like(q)
    a = Attn(n_q, pos0, heads, kvh, d, window, scale, ptr(q, f32p), ptr(k, f32p), ptr(v, f32p), C.pointer(c),
             ptr(rp, i64p), ptr(out, f32p))
    lib().xo_attention(C.byref(a))
    return out


def fill_masks(ar, rows, n_past, ctx, ring, window, ring_pos):
    rp = np.ascontiguousarray(ring_pos, np.int64)
    mask = np.zeros((ar, ctx + ar), np.uint8)
    wmask = np.zeros((ar, ring + ar), np.uint8)
    lib().xo_fill_masks(ar, rows, n_past, ctx, ring, window, ptr(rp, i64p), ptr(mask, u8p), ptr(wmask, u8p))
    return mask, wmask


def rewind_ok(to, n_past, window, ring_pos):
    rp = np.ascontiguousarray(ring_pos, np.int64)
    return bool(lib().xo_rewind_ok(to, n_past, window, len(rp), ptr(rp, i64p)))


# ----------------------------------------------------------------------------------------------------------------
# The synthetic model on the CPU
# ----------------------------------------------------------------------------------------------------------------

def synth_cfg(**kw):
    c = SynthCfg()
    for name, _ in SYNTH_FIELDS:
        setattr(c, name, kw[name])
    return c


class SynthDory:
    """The seeded synthetic Dory model plus one KV state, stepped by the restatement."""

    def __init__(self, cfg: dict, ctx: int, n_prefill: int, kv_dtype=KV_I8):
        self.cfg = dict(cfg)
        self.c = synth_cfg(**cfg)
        L = lib()
        self.model = L.xo_synth_model_new(C.byref(self.c))
        self.state = L.xo_synth_state_new(self.model, C.byref(self.c), ctx, kv_dtype, n_prefill)

    def close(self):
        L = lib()
        if self.state:
            L.xo_synth_state_free(self.state)
            self.state = None
        if self.model:
            L.xo_synth_model_free(self.model)
            self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def n_past(self):
        return self.state.contents.n_past

    def ring_pos(self):
        s = self.state.contents
        return np.ctypeslib.as_array(s.ring_pos, shape=(s.ring,)).copy()

    def step(self, tokens):
        L = lib()
        toks = np.ascontiguousarray(tokens, np.int32)
        m = len(toks)
        logits = np.zeros((m, self.cfg["vocab"]), np.float32)
        work = np.zeros(L.xo_step_work_floats(self.model, m), np.float32)
        L.xo_step(self.model, self.state, ptr(toks, i32p), m, ptr(logits, f32p), ptr(work, f32p))
        return logits

    def weight(self, e, j):
        """(codes, scales, global) of evaluation e's weight j (head: e = -1)."""
        M = self.model.contents
        w = M.head if e < 0 else M.layers[e].w[j]
        n, k = w.n_out, w.k
        codes = np.ctypeslib.as_array(w.codes, shape=(n * (k // 2),)).reshape(n, k // 2).copy()
        scales = np.ctypeslib.as_array(w.scales, shape=(n * (k // 16),)).reshape(n, k // 16).copy()
        return codes, scales, float(w.global_)

    def cache(self, i):
        """(k codes, v codes, k scales, v scales, ring) of KV instance i, [slots, kv_heads, d] / [slots, kv_heads]."""
        s = self.state.contents
        c = s.caches[i]
        kvh, d = self.cfg["kv_heads"], self.cfg["head_dim"]
        n = c.slots
        k = np.ctypeslib.as_array(c.k, shape=(n * kvh * d,)).reshape(n, kvh, d).copy()
        v = np.ctypeslib.as_array(c.v, shape=(n * kvh * d,)).reshape(n, kvh, d).copy()
        ks = np.ctypeslib.as_array(c.ks, shape=(n * kvh,)).reshape(n, kvh).copy()
        vs = np.ctypeslib.as_array(c.vs, shape=(n * kvh,)).reshape(n, kvh).copy()
        return k, v, ks, vs, bool(c.ring)


class CheckpointDory(SynthDory):
    """A Dory checkpoint's tensors stepped by the restatement: the model packs/dory/dory.cpp:316-439 builds from
    config.json and model.safetensors (recurrent sublayers' weights shared by every loop, the stored scales folded as
    dory.cpp:326-364 folds them), with the BF16 embedding table and either the BF16 lm_head (head "bf16") or its
    NVFP4 quantization (head "nvfp4", the device loader's option). The KV state is seeded as the synthetic model's.

    config: config.json as a dict; tensors: name -> array (U8 codes, F8_E4M3 scales as uint8, F32 globals, BF16 as
    uint16 bits), as the checkpoint stores them."""

    def __init__(self, config: dict, tensors: dict, ctx: int, n_prefill: int, loops=None, head="bf16",
                 kv_dtype=KV_I8, ring=None, seed=3, kvs_lo=0.0008, kvs_hi=0.0016):
        c = config
        H, F = c["hidden_size"], c["intermediate_size"]
        heads, kvh, d = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        V = c["vocab_size"]
        n_in, n_rec, n_out = c["n_input_layers"], c["n_recurrent_layers"], c["n_output_layers"]
        loops = c.get("n_recurrent_loops", 1) if loops is None else loops
        kinds_ = [{"mlp": 0, "sliding_attention": 1, "full_attention": 2}[t] for t in c["layer_types"]]
        window = c.get("sliding_window", 0) if 1 in kinds_ else 64
        ring = window + 64 if ring is None else ring
        f32 = np.float32
        init_range = f32(c["initializer_range"])
        alpha_scale = f32(c["ngpt_alpha_init"]) / init_range
        sqk_factor = np.sqrt(f32(d)) / init_range
        gate_init = c.get("attention_output_gate_logit_scale_init")
        gate_init = np.sqrt(f32(H)) if gate_init is None else f32(gate_init)
        gate_factor = np.sqrt(f32(gate_init)) / init_range
        suv_factor = np.sqrt(f32(H))
        rope = c["rope_parameters"]
        theta = {1: f32(rope.get("sliding_attention", {}).get("rope_theta", 0)),
                 2: f32(rope.get("full_attention", {}).get("rope_theta", 0))}
        keep = []

        def arr(a, dt):
            a = np.ascontiguousarray(a, dt)
            keep.append(a)
            return a

        def bf16(name):
            return bf16_to_f32(tensors[name]).astype(f32)

        def nvfp4(name):
            w = Nvfp4()
            codes = arr(tensors[name + ".weight"], np.uint8)
            scales = arr(tensors[name + ".weight_scale"], np.uint8)
            w.codes, w.scales = ptr(codes, u8p), ptr(scales, u8p)
            w.global_ = float(np.asarray(tensors[name + ".weight_scale_2"], f32).reshape(()))
            w.n_out, w.k = codes.shape[0], codes.shape[1] * 2
            return w

        phys = list(range(n_in)) + [n_in + r for _ in range(loops) for r in range(n_rec)] + \
            [n_in + n_rec + r for r in range(n_out)]
        layers = (Layer * len(phys))()
        built = {}
        n_attn = 0
        for e, l in enumerate(phys):
            L = layers[e]
            k = kinds_[l]
            L.kind = k
            p = f"backbone.layers.{l}."
            if l not in built:
                lr = arr(np.abs(bf16(p + ("mlp_alpha" if k == 0 else "attn_alpha")) * alpha_scale), f32)
                if k == 0:
                    ws = [nvfp4(p + "mixer." + n) for n in ("gate_proj", "up_proj", "down_proj")]
                    vec = dict(sg=arr(bf16(p + "mixer.suv_gate") * suv_factor, f32),
                               su=arr(bf16(p + "mixer.suv_up") * suv_factor, f32))
                else:
                    ws = [nvfp4(p + "mixer." + n) for n in ("q_proj", "k_proj", "v_proj", "g_proj", "o_proj")]
                    qs, gs = bf16(p + "mixer.sqk"), bf16(p + "mixer.s_gate")
                    vec = dict(qscale=arr((qs * sqk_factor) * (qs * sqk_factor), f32),
                               gscale=arr((gs * gate_factor) * (gs * gate_factor), f32))
                built[l] = (ws, lr, vec)
            ws, lr, vec = built[l]
            for j, w in enumerate(ws):
                L.w[j] = w
            L.lr = ptr(lr, f32p)
            for name, a in vec.items():
                setattr(L, name, ptr(a, f32p))
            if k != 0:
                L.theta = float(theta[k])
                L.cache = n_attn
                n_attn += 1
        M = Model()
        M.hidden, M.ffn, M.heads, M.kv_heads, M.head_dim, M.vocab = H, F, heads, kvh, d, V
        M.window, M.n_in, M.n_rec, M.n_out, M.loops = window, n_in, n_rec, n_out, loops
        M.layers = C.cast(layers, C.POINTER(Layer))
        M.logit_scale = ptr(arr(bf16("lm_head.logit_scale") / init_range, f32), f32p)
        M.embed_bf16 = ptr(arr(tensors["backbone.embeddings.weight"], np.uint16), u16p)
        lm = arr(tensors["lm_head.weight"], np.uint16)
        if head == "bf16":
            M.head_bf16 = ptr(lm, u16p)
        else:   # the loader's quantizer (bit-exact with this one)
            codes, scales, g = quantize_nvfp4(lm)
            hw = Nvfp4()
            hw.codes, hw.scales = ptr(arr(codes, np.uint8), u8p), ptr(arr(scales, np.uint8), u8p)
            hw.global_, hw.n_out, hw.k = g, V, H
            M.head = hw
        self._keep = (keep, layers, M)
        self.cfg = dict(hidden=H, ffn=F, heads=heads, kv_heads=kvh, head_dim=d, vocab=V, n_in=n_in, n_rec=n_rec,
                        n_out=n_out, loops=loops, window=window, ring=ring, global_every=0, theta_sliding=1e4,
                        theta_global=1e4, weight_std=0.02, lr_lo=0, lr_hi=1, qs_lo=0, qs_hi=1, gs_lo=0, gs_hi=1,
                        suv_lo=0, suv_hi=1, ls_lo=0, ls_hi=1, kvs_lo=kvs_lo, kvs_hi=kvs_hi, seed=seed)
        self.c = synth_cfg(**self.cfg)
        self.model = C.pointer(M)
        self.state = lib().xo_synth_state_new(self.model, C.byref(self.c), ctx, kv_dtype, n_prefill)

    def close(self):
        if self.state:
            lib().xo_synth_state_free(self.state)
            self.state = None
        self.model = None


def kinds(cfg: dict):
    c = synth_cfg(**cfg)
    L = lib()
    return [L.xo_synth_kind(C.byref(c), e) for e in range(L.xo_synth_n_evals(C.byref(c)))]


def topk(logits, k):
    """The k most likely entries of a row, most likely first: more_likely (engine/src/sampler.cpp:26-28), value
    descending, ties to the lowest index; as top_logprobs' partial_sort (sampler.cpp:30-40) orders them."""
    logits = np.asarray(logits, np.float32)
    order = np.lexsort((np.arange(len(logits)), -logits.astype(np.float64)))
    return order[:k].astype(np.int32), logits[order[:k]]


def sample(logits, temperature, top_k, top_p, min_p, u):
    """Sampler::sample (engine/src/sampler.cpp:41-94) restated with the draw given: u in [0, 1) stands for
    uniform_real_distribution<double>(0, total) (value = u * total). Where the reference's partial_sort leaves the
    tail past its sorted head in an unspecified order, this sorts the whole row; callers compare only where the
    sorted head decides."""
    logits = np.asarray(logits, np.float32)
    n = len(logits)
    if temperature <= 0.0:
        return int(np.argmax(logits))                       # argmax: the first index of the maximum
    mx = logits.max()
    inv_t = np.float32(1.0) / np.float32(temperature)
    w = np.exp((logits - mx) * inv_t).astype(np.float32)   # float weights, as std::exp(float)
    total = float(np.sum(w.astype(np.float64)))
    idx = np.arange(n)
    keep = n
    if 0 < top_k < n:
        order = np.lexsort((idx, -w.astype(np.float64)))
        keep = top_k
        total = float(np.sum(w[order[:keep]].astype(np.float64)))
    elif top_p < 1.0 or min_p > 0.0:
        order = np.lexsort((idx, -w.astype(np.float64)))
    else:
        order = idx                                         # no filter: the row in index order
    cw = w[order]
    if min_p > 0.0:
        floor = np.float32(min_p) * cw[0]
        k = 0
        t = 0.0
        while k < keep and cw[k] >= floor:
            t += float(cw[k])
            k += 1
        keep = max(1, k)
        total = t if k else float(cw[0])
    if top_p < 1.0:
        target = total * float(np.float32(top_p))
        cum = 0.0
        k = 0
        while k < keep:
            cum += float(cw[k])
            k += 1
            if cum >= target:
                break
        keep = max(1, k)
        total = cum
    r = u * total
    cum = 0.0
    for i in range(keep):
        cum += float(cw[i])
        if r < cum:
            return int(order[i])
    return int(order[keep - 1])

