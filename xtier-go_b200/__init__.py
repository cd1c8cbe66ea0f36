"""xtier-go_b200: ctypes bindings of libxtg_cuda.so (include/xtg_cuda.h), the B200 backend of the Dory verify step.

`Session` mirrors the NPU plugin's session API of XTier Go (npu/xtg_npu.h: open / info / forward / pos / rewind /
snapshot_slots / snapshot_pos / snapshot / restore / grow / debug_cache / close) with the same argument meaning and
error behaviour: a failed call raises `XtgError` carrying the library's message where the C ABI returns -1. The
kernel-level functions take torch CUDA tensors (device memory and streams only; the arithmetic runs in the
library's sm_100a kernels). Importing this module never falls back to anything: if the library is missing it raises.
"""
import ctypes as C
import json
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libxtg_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "xtg_cuda.h")

_lib = None


class XtgError(RuntimeError):
    pass


def build():
    """Compile libxtg_cuda.so for sm_100a in-tree (nvcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


LOGITS_FN = C.CFUNCTYPE(None, C.c_int, C.POINTER(C.c_float), C.c_void_p)


class AttnArgs(C.Structure):
    _fields_ = [("n_q", C.c_int), ("pos0", C.c_int64), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("window", C.c_int), ("scale", C.c_float), ("q", C.c_void_p),
                ("k", C.c_void_p), ("v", C.c_void_p), ("k_codes", C.c_void_p), ("v_codes", C.c_void_p),
                ("k_scales", C.c_void_p), ("v_scales", C.c_void_p), ("slots", C.c_int64), ("ring", C.c_int),
                ("ring_pos", C.c_void_p), ("dtype", C.c_int), ("out", C.c_void_p)]


class Sampling(C.Structure):
    """xtg_cuda_sampling: Sampler::sample's parameters."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("min_p", C.c_float)]


def lib():
    """The loaded library; raises if it was not built (no silent fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise XtgError(f"{LIB} is missing: build it with xtier-go_b200's Makefile (__graft_entry__.build())")
        L = C.CDLL(LIB)
        E = C.c_char_p
        L.xtg_cuda_open.restype = C.c_void_p
        L.xtg_cuda_open.argtypes = [C.c_char_p, C.c_char_p, E, C.c_int]
        L.xtg_cuda_open_shared.restype = C.c_void_p
        L.xtg_cuda_open_shared.argtypes = [C.c_void_p, C.c_char_p, E, C.c_int]
        L.xtg_cuda_info.restype = C.c_int
        L.xtg_cuda_info.argtypes = [C.c_void_p, C.c_char_p, C.c_int]
        L.xtg_cuda_forward.restype = C.c_int
        L.xtg_cuda_forward.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, LOGITS_FN, C.c_void_p,
                                       E, C.c_int]
        L.xtg_cuda_forward_batch.restype = C.c_int
        L.xtg_cuda_forward_batch.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.POINTER(C.POINTER(C.c_int32)),
                                             C.POINTER(C.c_int), C.c_int, LOGITS_FN, C.c_void_p, E, C.c_int]
        L.xtg_cuda_pos.restype = C.c_int64
        L.xtg_cuda_pos.argtypes = [C.c_void_p]
        L.xtg_cuda_rewind.restype = C.c_int
        L.xtg_cuda_rewind.argtypes = [C.c_void_p, C.c_int64]
        L.xtg_cuda_snapshot_slots.restype = C.c_int
        L.xtg_cuda_snapshot_slots.argtypes = [C.c_void_p]
        L.xtg_cuda_snapshot_pos.restype = C.c_int64
        L.xtg_cuda_snapshot_pos.argtypes = [C.c_void_p, C.c_int]
        L.xtg_cuda_snapshot.restype = None
        L.xtg_cuda_snapshot.argtypes = [C.c_void_p, C.c_int]
        L.xtg_cuda_restore.restype = C.c_int
        L.xtg_cuda_restore.argtypes = [C.c_void_p, C.c_int]
        L.xtg_cuda_grow.restype = C.c_int
        L.xtg_cuda_grow.argtypes = [C.c_void_p, C.c_char_p, E, C.c_int]
        L.xtg_cuda_debug_cache.restype = C.c_int64
        L.xtg_cuda_debug_cache.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int64]
        L.xtg_cuda_close.restype = None
        L.xtg_cuda_close.argtypes = [C.c_void_p]
        L.xtg_cuda_argmax.restype = C.c_int
        L.xtg_cuda_argmax.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int]
        L.xtg_cuda_topk.restype = C.c_int
        L.xtg_cuda_topk.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    E, C.c_int]
        L.xtg_cuda_topk_rows.restype = C.c_int
        L.xtg_cuda_topk_rows.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_void_p, E, C.c_int]
        L.xtg_cuda_head_bf16.restype = C.c_int
        L.xtg_cuda_head_bf16.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p, E, C.c_int]
        L.xtg_cuda_sample_candidates.restype = C.c_int
        L.xtg_cuda_sample_candidates.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_int,
                                                 C.POINTER(Sampling), C.c_double]
        L.xtg_cuda_prefill_synthetic.restype = C.c_int
        L.xtg_cuda_prefill_synthetic.argtypes = [C.c_void_p, C.c_int64, E, C.c_int]
        L.xtg_cuda_bench.restype = C.c_int
        L.xtg_cuda_bench.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.c_int,
                                     C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_int64), E, C.c_int]
        L.xtg_cuda_step_bytes.restype = C.c_int64
        L.xtg_cuda_step_bytes.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.xtg_cuda_linear_new.restype = C.c_void_p
        L.xtg_cuda_linear_new.argtypes = [C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                          C.POINTER(C.c_float), C.POINTER(C.c_int), C.c_int, E, C.c_int]
        L.xtg_cuda_linear_forward.restype = C.c_int
        L.xtg_cuda_linear_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_void_p), C.c_void_p, E,
                                              C.c_int]
        L.xtg_cuda_linear_bytes.restype = C.c_int64
        L.xtg_cuda_linear_bytes.argtypes = [C.c_void_p]
        L.xtg_cuda_linear_free.restype = None
        L.xtg_cuda_linear_free.argtypes = [C.c_void_p]
        L.xtg_cuda_quantize_nvfp4.restype = C.c_int
        L.xtg_cuda_quantize_nvfp4.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                              C.c_void_p, E, C.c_int]
        L.xtg_cuda_attention.restype = C.c_int
        L.xtg_cuda_attention.argtypes = [C.POINTER(AttnArgs), C.c_int, C.c_void_p, E, C.c_int]
        L.xtg_cuda_attention_noalloc.restype = C.c_int
        L.xtg_cuda_attention_noalloc.argtypes = [C.POINTER(AttnArgs), C.c_int, C.c_void_p, E, C.c_int]
        L.xtg_cuda_kv_store.restype = C.c_int
        L.xtg_cuda_kv_store.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int64, C.c_int,
                                        C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, E,
                                        C.c_int]
        L.xtg_cuda_gen.restype = C.c_int
        L.xtg_cuda_gen.argtypes = [C.c_int, C.c_uint64, C.c_uint64, C.c_float, C.c_float, C.c_void_p, C.c_int64,
                                   C.c_void_p, E, C.c_int]
        _lib = L
    return _lib


def declared_symbols():
    """Every function include/xtg_cuda.h declares."""
    import re
    text = open(HEADER).read()
    return sorted(set(re.findall(r"XTG_CUDA_API\s+[\w\*\s]+?\b(xtg_cuda_\w+)\s*\(", text)))


def _err():
    return C.create_string_buffer(1024)


def _check(rc, err):
    if rc != 0:
        raise XtgError(err.value.decode(errors="replace"))


# ----------------------------------------------------------------------------------------------------------------
# Synthetic model shapes
# ----------------------------------------------------------------------------------------------------------------

# BASELINE's Dory-shaped synthetic model (hidden 3072, 24 q / 6 KV heads of 128, FFN 9216, vocab 131072, 4 + 40 x 2 +
# 4 sublayers, every 4th attention sublayer global, 1088-slot rings over a window of 1024). The unit-norm-ish KV
# prefill scales keep the random cached keys at the model's own key norm.
DORY_3072 = dict(hidden=3072, ffn=9216, heads=24, kv_heads=6, head_dim=128, vocab=131072, n_in=4, n_rec=40, n_out=4,
                 loops=2, window=1024, ring=1088, global_every=4, theta_sliding=1e4, theta_global=1e7,
                 weight_std=0.02, lr_lo=0.05, lr_hi=0.2, qs_lo=48.0, qs_hi=80.0, gs_lo=25.0, gs_hi=75.0,
                 suv_lo=25.0, suv_hi=75.0, ls_lo=100.0, ls_hi=200.0, kvs_lo=0.0008, kvs_hi=0.0016, seed=3)

# The real Dory 4B's shape (head_dim 256, GQA 4, 16 + 40 x 2 + 16 sublayers) with the synthetic model's seeded weights
# and sublayer alternation.
DORY_4B = dict(DORY_3072, hidden=2560, ffn=7168, heads=16, kv_heads=4, head_dim=256, n_in=16, n_rec=40, n_out=16,
               seed=5)

# A small model with the same structure for parity tests that a CPU oracle finishes in seconds.
SMALL = dict(DORY_3072, hidden=512, ffn=1024, heads=8, kv_heads=2, vocab=4096, n_in=2, n_rec=4, n_out=2, loops=2,
             window=64, ring=128, global_every=2, seed=11)


# ----------------------------------------------------------------------------------------------------------------
# The session
# ----------------------------------------------------------------------------------------------------------------

class Session:
    """One xtg_cuda handle (npu/xtg_npu.h's session): weights, KV instances, ring table, snapshots."""

    def __init__(self, model=None, context=8192, kv_dtype="int8", snapshots=2, decode_rows=8, device=0, graph=True,
                 pdl=True, path=None, **extra):
        """The synthetic model of shape `model` (default DORY_3072), or (path) the Dory checkpoint in that directory
        (config.json + model.safetensors, ModelOpt W4A16_NVFP4); extra options as xtg_cuda_open takes them (for a
        checkpoint: loops, kv_mode, ring, head "bf16" | "nvfp4")."""
        opts = dict(context=context, kv_dtype=kv_dtype, snapshots=snapshots, decode_rows=decode_rows, device=device,
                    graph=int(graph), pdl=int(pdl))
        if path is None:
            opts["model"] = dict(model or DORY_3072)
        opts.update(extra)
        self.options = opts
        self.path = path
        if path is None:
            self.model = opts["model"]
        else:
            with open(os.path.join(path, "config.json")) as f:
                cfg = json.load(f)
            self.model = dict(hidden=cfg["hidden_size"], ffn=cfg["intermediate_size"],
                              heads=cfg["num_attention_heads"], kv_heads=cfg["num_key_value_heads"],
                              head_dim=cfg["head_dim"], vocab=cfg["vocab_size"])
        err = _err()
        src = b"synthetic" if path is None else os.fsencode(path)
        self.h = lib().xtg_cuda_open(src, json.dumps(opts).encode(), err, len(err))
        if not self.h:
            raise XtgError(err.value.decode(errors="replace"))

    @classmethod
    def shared(cls, owner, context=8192, kv_dtype="int8", snapshots=2, decode_rows=8, graph=True, pdl=True, **extra):
        """xtg_cuda_open_shared: another session over owner's weights (its own caches, stream and graph)."""
        self = cls.__new__(cls)
        opts = dict(context=context, kv_dtype=kv_dtype, snapshots=snapshots, decode_rows=decode_rows,
                    graph=int(graph), pdl=int(pdl))
        opts.update(extra)
        self.options = dict(owner.options, **opts)
        self.model = owner.model
        err = _err()
        self.h = lib().xtg_cuda_open_shared(owner.h, json.dumps(opts).encode(), err, len(err))
        if not self.h:
            raise XtgError(err.value.decode(errors="replace"))
        return self

    def close(self):
        if getattr(self, "h", None):
            lib().xtg_cuda_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def info(self):
        buf = C.create_string_buffer(4096)
        n = lib().xtg_cuda_info(self.h, buf, len(buf))
        if n < 0:
            raise XtgError("info: buffer too small")
        return json.loads(buf.value.decode())

    def forward(self, tokens, want=2):
        """Run the tokens; returns {row: logits (numpy f32 [vocab])} for the rows asked for (want 0 / 1 / 2)."""
        import numpy as np
        toks = (C.c_int32 * len(tokens))(*[int(t) for t in tokens])
        out = {}
        vocab = self.model["vocab"]
        rows = np.empty((len(tokens) if want == 2 else min(1, want), vocab), np.float32) if want else None
        nbytes = vocab * 4

        def cb(row, ptr, user):   # the row is valid only during the call: one copy into the result array
            dst = rows[row if want == 2 else 0]
            C.memmove(dst.ctypes.data, ptr, nbytes)
            out[row] = dst

        fn = LOGITS_FN(cb)
        err = _err()
        _check(lib().xtg_cuda_forward(self.h, toks, len(tokens), want, fn, None, err, len(err)), err)
        return out

    def pos(self):
        return lib().xtg_cuda_pos(self.h)

    def rewind(self, n):
        return lib().xtg_cuda_rewind(self.h, n) == 0

    def snapshot_slots(self):
        return lib().xtg_cuda_snapshot_slots(self.h)

    def snapshot_pos(self, slot):
        return lib().xtg_cuda_snapshot_pos(self.h, slot)

    def snapshot(self, slot):
        lib().xtg_cuda_snapshot(self.h, slot)

    def restore(self, slot):
        return lib().xtg_cuda_restore(self.h, slot) == 0

    def grow(self, tier):
        err = _err()
        _check(lib().xtg_cuda_grow(self.h, str(tier).encode(), err, len(err)), err)

    def tiers(self, contexts):
        """The session over a list of context tiers (Tiers below); the session's own context must be the first."""
        return Tiers(self, contexts)

    def debug_cache(self, instance, value):
        """K codes [kv_heads][128][slots] (0), V codes [kv_heads][slots][128] (1), K / V scales [kv_heads][slots]
        (2 / 3) as numpy arrays; None for no such instance."""
        import numpy as np
        n = lib().xtg_cuda_debug_cache(self.h, instance, value, None, 0)
        if n < 0:
            return None
        buf = np.empty(n, np.uint8)
        got = lib().xtg_cuda_debug_cache(self.h, instance, value, buf.ctypes.data, n)
        if got != n:
            raise XtgError("debug_cache failed")
        kvh = self.model["kv_heads"]
        if value >= 2:
            f = buf.view(np.float32)
            return f.reshape(kvh, -1)
        slots = n // (kvh * 128)
        return buf.reshape(kvh, 128, slots) if value == 0 else buf.reshape(kvh, slots, 128)

    def argmax(self, n=8):
        out = (C.c_int32 * n)()
        k = lib().xtg_cuda_argmax(self.h, out, n)
        if k < 0:
            raise XtgError("argmax: no step yet")
        return list(out[:k])

    def topk(self, k, temperature=1.0):
        """xtg_cuda_topk: the last step's rows' k most likely entries (idx, logit [rows][k]), row max, total."""
        import numpy as np
        idx = np.empty((8, k), np.int32)
        val = np.empty((8, k), np.float32)
        mx = np.empty(8, np.float32)
        tot = np.empty(8, np.float64)
        err = _err()
        rows = lib().xtg_cuda_topk(self.h, k, temperature, idx.ctypes.data, val.ctypes.data, mx.ctypes.data,
                                   tot.ctypes.data, err, len(err))
        if rows < 0:
            raise XtgError(err.value.decode(errors="replace"))
        return idx.reshape(-1)[:rows * k].reshape(rows, k), val.reshape(-1)[:rows * k].reshape(rows, k), \
            mx[:rows], tot[:rows]

    def prefill_synthetic(self, n_past):
        err = _err()
        _check(lib().xtg_cuda_prefill_synthetic(self.h, n_past, err, len(err)), err)

    def bench(self, tokens, steps, profile=False):
        toks = (C.c_int32 * len(tokens))(*[int(t) for t in tokens])
        ms = C.c_double()
        cms = (C.c_double * 4)()
        cl = (C.c_int64 * 4)()
        err = _err()
        _check(lib().xtg_cuda_bench(self.h, toks, len(tokens), steps, 1 if profile else 0, C.byref(ms), cms, cl, err,
                                    len(err)), err)
        return ms.value, list(cms), list(cl)

    def step_bytes(self, what=0, m=8):
        return lib().xtg_cuda_step_bytes(self.h, what, m)


class Tiers:
    """A session over context tiers, as packs/dory/npu.cpp's NpuModel keeps its .pte buckets (npu.cpp:142-160) and
    NpuSession::forward fits each chunk (npu.cpp:266-270). fit(need) moves the session to the smallest tier with
    room for `need` positions (npu.cpp:181-198): up when a request outgrows the current tier, down when a shorter
    conversation follows, never below the positions already held. A tier here is a context length given to
    xtg_cuda_grow in place of a .pte path; the caches are reallocated and the held positions copied on the device."""

    def __init__(self, session, contexts):
        ctx = [int(c) for c in contexts]
        if not ctx:
            raise XtgError("tiers: no context tiers")
        for a, b in zip(ctx, ctx[1:]):
            if b <= a:
                raise XtgError(f"tiers: {b} after {a}: list the tiers by context")
        have = session.info()["context"]
        if have != ctx[0]:
            raise XtgError(f"tiers: the session holds {have} positions, the first tier {ctx[0]}")
        self.session = session
        self.contexts = ctx
        self.cur = 0
        self.moves = []

    @property
    def context(self):
        return self.contexts[-1]

    def fit(self, need):
        to = 0
        while to < len(self.contexts) and self.contexts[to] < need:
            to += 1
        if to == len(self.contexts):
            raise XtgError(f"context full: {need} positions (the largest tier holds {self.contexts[-1]})")
        if to == self.cur or self.session.pos() > self.contexts[to]:
            return
        self.session.grow(self.contexts[to])
        self.cur = to
        self.moves.append(self.contexts[to])

    def forward(self, tokens, want=2):
        """The session's forward after fitting n_past + len(tokens); the rows as Session.forward returns them."""
        if len(self.contexts) > 1:
            self.fit(self.session.pos() + len(tokens))
        return self.session.forward(tokens, want)


# ----------------------------------------------------------------------------------------------------------------
# Kernel level (torch CUDA tensors as device memory)
# ----------------------------------------------------------------------------------------------------------------

def forward_batch(sessions, token_lists, want=2):
    """xtg_cuda_forward_batch: every session's steps in flight together from this thread; returns one
    {row: logits} dict per session (rows numbered within each session)."""
    import numpy as np
    nh = len(sessions)
    hs = (C.c_void_p * nh)(*[s.h for s in sessions])
    arrs = [(C.c_int32 * max(1, len(t)))(*[int(v) for v in t]) for t in token_lists]
    toks = (C.POINTER(C.c_int32) * nh)(*[C.cast(a, C.POINTER(C.c_int32)) for a in arrs])
    ns = (C.c_int * nh)(*[len(t) for t in token_lists])
    base = np.cumsum([0] + [len(t) for t in token_lists])
    vocabs = [s.model["vocab"] for s in sessions]   # the sessions may serve different models
    out = [dict() for _ in range(nh)]

    def cb(row, ptr, user):
        i = int(np.searchsorted(base, row, side="right")) - 1
        vocab = vocabs[i]
        dst = np.empty(vocab, np.float32)
        C.memmove(dst.ctypes.data, ptr, vocab * 4)
        out[i][row - int(base[i])] = dst

    fn = LOGITS_FN(cb)
    err = _err()
    _check(lib().xtg_cuda_forward_batch(hs, nh, toks, ns, want, fn, None, err, len(err)), err)
    return out


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class Linear:
    """matmul_nvfp4's fused weights on the device (xtg_cuda_linear_*)."""

    def __init__(self, weights, k):
        """weights: [(codes uint8 CUDA [n, k/2], scales uint8 CUDA [n, k/16], global float)]"""
        nw = len(weights)
        self._keep = weights
        codes = (C.c_void_p * nw)(*[w[0].data_ptr() for w in weights])
        scales = (C.c_void_p * nw)(*[w[1].data_ptr() for w in weights])
        globals_ = (C.c_float * nw)(*[float(w[2]) for w in weights])
        n_out = (C.c_int * nw)(*[int(w[0].shape[0]) for w in weights])
        self.n_out = [int(w[0].shape[0]) for w in weights]
        self.k = k
        err = _err()
        self.h = lib().xtg_cuda_linear_new(nw, codes, scales, globals_, n_out, k, err, len(err))
        if not self.h:
            raise XtgError(err.value.decode(errors="replace"))

    def __call__(self, x, ys=None):
        import torch
        m = x.shape[0]
        if ys is None:
            ys = [torch.empty((m, n), dtype=torch.float32, device=x.device) for n in self.n_out]
        yp = (C.c_void_p * len(ys))(*[y.data_ptr() for y in ys])
        err = _err()
        _check(lib().xtg_cuda_linear_forward(self.h, _ptr(x), m, yp, _stream(), err, len(err)), err)
        return ys

    def bytes(self):
        return lib().xtg_cuda_linear_bytes(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().xtg_cuda_linear_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def quantize_nvfp4(w_bf16):
    """bf16 bits (int16/uint16 CUDA tensor [n, k]) -> (codes, scales, global tensor)."""
    import torch
    n, k = w_bf16.shape
    codes = torch.empty((n, k // 2), dtype=torch.uint8, device=w_bf16.device)
    scales = torch.empty((n, k // 16), dtype=torch.uint8, device=w_bf16.device)
    g = torch.empty(1, dtype=torch.float32, device=w_bf16.device)
    err = _err()
    _check(lib().xtg_cuda_quantize_nvfp4(_ptr(w_bf16), n, k, _ptr(codes), _ptr(scales), _ptr(g), _stream(), err,
                                         len(err)), err)
    return codes, scales, g


def attention(q, k, v, k_codes, v_codes, k_scales, v_scales, pos0, window, scale, ring_pos=None, dtype=0, splits=4):
    """xtg_cuda_attention: q [n_q][heads][128], k / v [n_q][kv_heads][128] f32; cache in this library's layout."""
    import torch
    n_q, heads, d = q.shape
    kvh = k.shape[1]
    out = torch.empty_like(q)
    a = AttnArgs(n_q, pos0, heads, kvh, d, window, scale, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                 k_codes.data_ptr(), v_codes.data_ptr(), k_scales.data_ptr(), v_scales.data_ptr(),
                 k_scales.shape[1], 1 if ring_pos is not None else 0,
                 ring_pos.data_ptr() if ring_pos is not None else None, dtype, out.data_ptr())
    err = _err()
    _check(lib().xtg_cuda_attention(C.byref(a), splits, _stream(), err, len(err)), err)
    return out


def attention_noalloc(q, k, v, k_codes, v_codes, k_scales, v_scales, pos0, window, scale, ring_pos=None, dtype=0,
                      splits=4, out=None):
    """xtg_cuda_attention_noalloc: attention() with the split partials in the library's fixed scratch (nothing
    allocated by the library; kv_heads x splits <= 256). Enqueued on the current stream, not waited for."""
    import torch
    n_q, heads, d = q.shape
    kvh = k.shape[1]
    if out is None:
        out = torch.empty_like(q)
    a = AttnArgs(n_q, pos0, heads, kvh, d, window, scale, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                 k_codes.data_ptr(), v_codes.data_ptr(), k_scales.data_ptr(), v_scales.data_ptr(),
                 k_scales.shape[1], 1 if ring_pos is not None else 0,
                 ring_pos.data_ptr() if ring_pos is not None else None, dtype, out.data_ptr())
    err = _err()
    _check(lib().xtg_cuda_attention_noalloc(C.byref(a), splits, _stream(), err, len(err)), err)
    return out


def head_bf16(x, w, logit_scale, logits=True):
    """xtg_cuda_head_bf16 on torch CUDA tensors: x [m][hidden] f32, w [vocab][hidden] bf16 (or int16 bits),
    logit_scale [vocab] f32 -> (logits [m][vocab] or None, argmax [m] int32)."""
    import torch
    m, hidden = x.shape
    vocab = w.shape[0]
    out = torch.empty((m, vocab), dtype=torch.float32, device=x.device) if logits else None
    am = torch.empty(m, dtype=torch.int32, device=x.device)
    err = _err()
    _check(lib().xtg_cuda_head_bf16(x.data_ptr(), m, w.data_ptr(), vocab, hidden, logit_scale.data_ptr(),
                                    out.data_ptr() if logits else None, am.data_ptr(), _stream(), err, len(err)), err)
    return out, am


def topk(logits, k, temperature=1.0):
    """xtg_cuda_topk_rows on a torch CUDA tensor [rows][vocab] f32: (idx, logit [rows][k], row_max, total)."""
    import torch
    rows, vocab = logits.shape
    dev = logits.device
    idx = torch.empty(rows, k, dtype=torch.int32, device=dev)
    val = torch.empty(rows, k, dtype=torch.float32, device=dev)
    mx = torch.empty(rows, dtype=torch.float32, device=dev)
    tot = torch.empty(rows, dtype=torch.float64, device=dev)
    err = _err()
    _check(lib().xtg_cuda_topk_rows(logits.data_ptr(), rows, vocab, k, temperature, idx.data_ptr(), val.data_ptr(),
                                    mx.data_ptr(), tot.data_ptr(), _stream(), err, len(err)), err)
    return idx, val, mx, tot


def sample_candidates(idx, logit, row_max, total, vocab, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, u=0.5):
    """xtg_cuda_sample_candidates (host only): Sampler::sample over one row's candidates; -2 when they cannot
    decide (the caller samples from the full row)."""
    import numpy as np
    idx = np.ascontiguousarray(idx, np.int32)
    logit = np.ascontiguousarray(logit, np.float32)
    p = Sampling(temperature, top_k, top_p, min_p)
    return lib().xtg_cuda_sample_candidates(idx.ctypes.data, logit.ctypes.data, len(idx), float(row_max),
                                            float(total), vocab, C.byref(p), u)


def kv_store(k, v, pos, slots, ring, dtype, k_codes, v_codes, k_scales, v_scales):
    n, kvh, _ = k.shape
    err = _err()
    _check(lib().xtg_cuda_kv_store(_ptr(k), _ptr(v), pos, n, kvh, slots, 1 if ring else 0, dtype, _ptr(k_codes),
                                   _ptr(v_codes), _ptr(k_scales), _ptr(v_scales), _stream(), err, len(err)), err)


def gen(what, seed, stream_id, a, b, out):
    err = _err()
    _check(lib().xtg_cuda_gen(what, seed, stream_id, a, b, _ptr(out), out.numel(), _stream(), err, len(err)), err)
    return out
