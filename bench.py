"""Benchmark of the Dory verify step on B200s, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...    (one rank per GPU, NCCL only for the barrier / max)

A step is one 8-row verify step of the synthetic Dory-3072 model (4 + 40 x 2 + 4 sublayers, NVFP4 weights with
g_proj and a tied NVFP4 head, int8 KV, 8K tier with 8184 positions prefilled): 3.35 GB streamed per step, far
larger than the 126 MB L2, so no flush is needed between steps. Every rank runs its own independent sequence
(weak scaling, no collective on the data path). `value` is rows verified per second over all ranks with the inputs
resident (CUDA events on the session's stream, max over ranks); `e2e` is the same through the C ABI forward()
with host token buffers and every row's logits copied back (wall clock around the call).

--impl reference times XTier Go's own CPU kernels (oracle/_ref/libxtgref.so, compiled from the reference sources)
on the same config: whole steps (88 sublayers in DorySession order and the whole head) on all host cores, with the
reference's FP8 KvCache and its 1040-slot rings (it has no int8 cache).
"""
import argparse
import ctypes as C
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
METRIC = "decode tok/s per B200 (NVFP4 Dory-shape, 8K ctx) and % of HBM roofline"
UNIT = "tok/s"
TOKENS = [17, 4242, 99, 131071, 5, 70000, 123, 2048]
PREFILL = 8184
TOPK = 64
FALLBACK_HBM = 6650.0


def package():
    pkg = os.path.join(ROOT, "xtier-go_b200")
    spec = importlib.util.spec_from_file_location("xtier_go_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xtier_go_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM, "fallback"


def peaks_bf16():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"])
    return 1590.0


def ncu_traffic():
    """dram bytes per GEMV launch from the committed ncu summary (profiles/), or None."""
    p = os.path.join(ROOT, "profiles", "gemv_nvfp4_dory3072.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1]))
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------------------------------
# the reference's CPU implementation (oracle/_ref): whole steps
# ------------------------------------------------------------------------------------------------------------------

class ReferenceStep:
    """The config-3 verify step on XTier Go's own CPU kernels (oracle/_ref/libxtgref.so, compiled from the reference
    sources), in DorySession::forward / run_chunk / sublayer order (packs/dory/dory.cpp:467-578): the tied head's
    rows (nvfp4_row), 4 + 40 x 2 + 4 sublayers (matmul_nvfp4, rope, justnorm, attention, KvCache::store, swiglu_scaled,
    slerp_residual) with the loop norms between them, then the NVFP4 head. Weights: the seeded synthetic Dory (the
    oracle builds them; the reference kernels read the same NVFP4 bytes). Caches: the reference's FP8 KvCache (it has
    no int8 one), a global cache per global sublayer holding 8184 positions and a ring of window + 16 = 1040 slots
    (the reference's own ring size) per sliding sublayer holding its last 1040. Every step runs at the same position
    (a verify step after a rewind)."""

    def __init__(self, model, threads, prefill=PREFILL):
        import numpy as np
        import oracle as O
        sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
        from make_golden import XrShape, XrSublayer  # the ctypes mirrors of ref_shim.cpp's structs
        R = O.ref()
        if R is None:
            raise RuntimeError("oracle/_ref/libxtgref.so is not built")
        self.O, self.R, self.np = O, R, np
        R.xr_sublayer.argtypes = [C.c_void_p, C.POINTER(XrShape), C.POINTER(XrSublayer), O.f32p, C.c_int, C.c_int64,
                                  C.c_int, O.f32p]
        R.xr_head.argtypes = [C.c_void_p, O.u8p, O.u8p, C.c_float, C.c_int, C.c_int, O.f32p, C.c_int, O.f32p,
                              O.f32p]
        self.cfg = cfg = dict(model)
        self.pos = prefill
        self.ring = cfg["window"] + 16
        self.synth = O.SynthDory(cfg, ctx=64, n_prefill=0, kv_dtype=O.KV_FP8)
        M = self.synth.model.contents
        self.pool = R.xr_pool_new(threads)
        H, F, Q, kvh, d = cfg["hidden"], cfg["ffn"], cfg["heads"] * cfg["head_dim"], cfg["kv_heads"], cfg["head_dim"]
        self.shape = XrShape(H, F, cfg["heads"], kvh, d)
        self.kinds = O.kinds(cfg)
        self.caches, self.subs = [], []
        for e, kind in enumerate(self.kinds):
            L = M.layers[e]
            sub = XrSublayer()
            sub.kind = kind
            for j in range(5):
                sub.codes[j] = L.w[j].codes
                sub.scales[j] = L.w[j].scales
                sub.globals[j] = L.w[j].global_
            sub.lr, sub.qscale, sub.gscale, sub.sg, sub.su = L.lr, L.qscale, L.gscale, L.sg, L.su
            sub.theta = L.theta
            sub.window = cfg["window"] if kind == 1 else 0
            if kind:
                c = R.xr_kv_new(kvh, d, 8192, self.ring if kind == 1 else 0, 1)
                first = 0 if kind == 2 else prefill - self.ring
                for p in range(first, prefill, 512):
                    n = min(512, prefill - p)
                    kk = O.gen_uniform(cfg["seed"], 600000 + 2 * e, -0.1, 0.1, n * kvh * d)
                    vv = O.gen_uniform(cfg["seed"], 600001 + 2 * e, -0.1, 0.1, n * kvh * d)
                    assert R.xr_kv_store(c, p, n, O.ptr(kk, O.f32p), O.ptr(vv, O.f32p)) == 0, R.xr_last_error()
                self.caches.append(c)
                sub.cache = c
            self.subs.append(sub)
        codes, scales, self.g_head = self.synth.weight(-1, 0)
        self.c_head, self.s_head = np.ascontiguousarray(codes), np.ascontiguousarray(scales)
        self.ls = np.ctypeslib.as_array(M.logit_scale, shape=(cfg["vocab"],)).copy()
        self.work = np.zeros(8 * (4 * H + 3 * Q + 2 * F) + 64, np.float32)
        self.logits = np.zeros((8, cfg["vocab"]), np.float32)

    def step(self, tokens):
        O, R, np, cfg = self.O, self.R, self.np, self.cfg
        H, m, f32p, u8p = cfg["hidden"], len(tokens), O.f32p, O.u8p
        x = np.zeros((m, H), np.float32)
        for r, t in enumerate(tokens):
            R.xr_nvfp4_row(O.ptr(self.c_head, u8p), O.ptr(self.s_head, u8p), self.g_head, cfg["vocab"], H, t,
                           O.ptr(x[r], f32p))
        e = 0

        def sub(x):
            nonlocal e
            assert R.xr_sublayer(self.pool, C.byref(self.shape), C.byref(self.subs[e]), O.ptr(x, f32p), m,
                                 self.pos, 1, O.ptr(self.work, f32p)) == 0, R.xr_last_error()
            e += 1

        for _ in range(cfg["n_in"]):
            sub(x)
        inp, state = x.copy(), x.copy()
        for _ in range(cfg["loops"]):
            x = np.ascontiguousarray(state + inp, np.float32)
            R.xr_justnorm(O.ptr(x, f32p), m, H)
            for _ in range(cfg["n_rec"]):
                sub(x)
            state = x.copy()
            R.xr_justnorm(O.ptr(state, f32p), m, H)
        x = state.copy()
        for _ in range(cfg["n_out"]):
            sub(x)
        assert R.xr_head(self.pool, O.ptr(self.c_head, u8p), O.ptr(self.s_head, u8p), self.g_head, cfg["vocab"], H,
                         O.ptr(x, f32p), m, O.ptr(self.ls, f32p), O.ptr(self.logits, f32p)) == 0
        return self.logits[:m]

    def close(self):
        for c in self.caches:
            self.R.xr_kv_free(c)
        self.caches = []
        if self.pool:
            self.R.xr_pool_free(self.pool)
            self.pool = None
        self.synth.close()


def reference_steps(model, threads, steps, warmup):
    """Seconds per whole reference step (the mean over `steps` timed steps after `warmup`), and the setup time."""
    t0 = time.perf_counter()
    ref = ReferenceStep(model, threads)
    setup = time.perf_counter() - t0
    try:
        for _ in range(warmup):
            ref.step(TOKENS)
        t0 = time.perf_counter()
        for _ in range(steps):
            ref.step(TOKENS)
        step_s = (time.perf_counter() - t0) / steps
    finally:
        ref.close()
    return step_s, setup


def reference_config(n):
    c = config_block(n)
    c.update(kv_dtype="fp8 (the reference's KvCache has no int8 form)", ring_slots=1040,
             ring_note="the reference's own ring: window 1024 + 16 slots")
    return c


def run_reference(args, rank):
    if rank != 0:
        return
    x = package()
    model = dict(x.DORY_3072)
    threads = os.cpu_count() or 1
    steps, warmup = max(1, args.steps), max(0, args.warmup)
    step_s, setup = reference_steps(model, threads, steps, warmup)
    value = 8.0 / step_s
    sample = (f"whole config-3 steps: {steps} timed after {warmup} warm-up, each the 88 sublayers and the whole "
              f"NVFP4 head on the reference's kernels (8 rows at position 8184, FP8 KvCaches, 1040-slot rings); "
              f"setup {setup:.1f} s untimed")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 activations, NVFP4 weights, fp8 KV",
            "data": "synthetic", "config": reference_config(args.gpus),
            "steps_per_s": 1.0 / step_s, "rows_per_s": value,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_block(n):
    return {"workload": "config3: synthetic Dory-3072 NVFP4 8-row verify step, 8K tier, 8184 positions prefilled, "
                        "batch 1 per GPU",
            "model": "Dory-3072 synthetic (hidden 3072, 24q/6kv x 128, ffn 9216, vocab 131072, 4+40x2+4, g_proj, "
                     "tied NVFP4 head)",
            "global_batch": n, "seq_len": 8192, "rows_per_step": 8, "kv_dtype": "int8",
            "l2": "inputs larger than L2 (3.35 GB streamed per step)",
            "parallelism": f"replicas x{n} (independent sequences, no collective)"}


# ------------------------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------------------------

def dist_barrier(dist, device="cuda"):
    """Every rank here (a no-op without a process group), then the device idle."""
    import torch
    if dist is not None:
        dist.barrier()
    if device == "cuda":
        torch.cuda.synchronize()


def max_over_ranks(v, dist, device="cuda"):
    """The slowest rank's time: every rank gets the max (an all-reduce; NCCL on GPUs, gloo in the CPU tests)."""
    import torch
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v, dist, device="cuda"):
    """The sum over every rank (an all-reduce; NCCL on GPUs, gloo in the CPU tests)."""
    import torch
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


GEMM_SETS = [("qkvg", [3072, 768, 768, 3072], 3072), ("o", [3072], 3072), ("gate_up", [9216, 9216], 3072),
             ("down", [3072], 9216)]


def gemm_block(x, device, m=512, reps=6):
    """BASELINE config 1 at M = 512 (a prefill chunk) through the library's linear API on the tcgen05 GEMM: each
    projection set of the sublayer with seeded random NVFP4 weights (3 copies rotated), x ~ N(0, 1). Device time of
    the GEMM kernel and of the activation digitizer from the CUDA activity timeline; FLOPs = 2 M N K. The FP4 MMA work
    is 4x that (4 activation digits); its peak is taken as 4x the measured dense bf16 GEMM peak."""
    import re
    import torch
    from torch.profiler import profile, ProfilerActivity
    g = torch.Generator(device=device)
    g.manual_seed(1)
    out = {}
    for name, outs, k in GEMM_SETS:
        lins = []
        for _ in range(3):
            ws = [(torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=device, generator=g),
                   torch.randint(0x30, 0x40, (n, k // 16), dtype=torch.uint8, device=device, generator=g), 1.0)
                  for n in outs]
            lins.append(x.Linear(ws, k))
        xin = torch.randn(m, k, device=device, generator=g)
        ys = [torch.empty(m, n, device=device) for n in outs]
        for it in range(6):
            lins[it % 3](xin, ys)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for it in range(reps):
                lins[it % 3](xin, ys)
            torch.cuda.synchronize()
        tot = {}
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                mm = re.search(r"(\w+_kernel)", ev.name)
                if mm:
                    d = tot.setdefault(mm.group(1), [0, 0.0])
                    d[0] += 1
                    d[1] += ev.device_time_total
        gemm_us = tot["gemm_kernel"][1] / tot["gemm_kernel"][0]
        dig_us = tot["act_digitize_kernel"][1] / tot["act_digitize_kernel"][0]
        flops = 2.0 * m * sum(outs) * k
        out[name] = {"n": sum(outs), "k": k, "gemm_us": gemm_us, "digitize_us": dig_us,
                     "tflops": flops / gemm_us / 1e6, "tflops_with_digitize": flops / (gemm_us + dig_us) / 1e6}
        for l_ in lins:
            l_.close()
    return out


def head_block(x, device, m=8, reps=20):
    """The lm_head at the Dory-3072 shape (vocab 131072 x 3072, 8 rows): the NVFP4 head on the GEMV (226 MB, the
    synthetic model's) beside a checkpoint's BF16 head (805 MB, the reference's matmul_bf16, head.cu). Seeded random
    weights, one copy each (both larger than L2); device time per launch from the CUDA activity timeline; algorithmic
    bytes = the weight bytes + x in f32 + logits in f32."""
    import torch
    from torch.profiler import profile, ProfilerActivity
    V, H = 131072, 3072
    g = torch.Generator(device=device)
    g.manual_seed(5)
    peak, peak_kind = peaks()
    xin = torch.randn(m, H, device=device, generator=g)
    xin = xin / xin.norm(dim=1, keepdim=True)
    codes = torch.randint(0, 256, (V, H // 2), dtype=torch.uint8, device=device, generator=g)
    scales = torch.randint(0x30, 0x40, (V, H // 16), dtype=torch.uint8, device=device, generator=g)
    lin = x.Linear([(codes, scales, 1.0)], H)
    ys = [torch.empty(m, V, device=device)]
    w = (torch.randn(V, H, device=device, generator=g) * 0.02).to(torch.bfloat16)
    ls = torch.rand(V, device=device, generator=g) * 100 + 100
    for _ in range(3):
        lin(xin, ys)
        x.head_bf16(xin, w, ls)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            lin(xin, ys)
            x.head_bf16(xin, w, ls)
        torch.cuda.synchronize()
    kt = kernel_times(prof)
    io = m * H * 4 + m * V * 4
    out = {}
    for name, kern, wb in (("nvfp4", "gemv_kernel", V * H // 2 + V * H // 16 + 4), ("bf16", "head_bf16_kernel", V * H * 2)):
        us = kt[kern]
        out[name] = {"us": us, "algorithmic_bytes": wb + io, "gbs": (wb + io) / us / 1e3,
                     "frac": (wb + io) / us / 1e3 / peak, "peak": peak, "peak_kind": peak_kind}
    lin.close()
    return out


def kernel_times(prof):
    """Mean device time (us) per kernel name (the `*_kernel` symbol) from a torch.profiler CUDA timeline."""
    import re
    import torch
    tot = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            mm = re.search(r"(\w+_kernel)", ev.name)
            if mm:
                d = tot.setdefault(mm.group(1), [0, 0.0])
                d[0] += 1
                d[1] += ev.device_time_total
    return {k: v[1] / v[0] for k, v in tot.items()}


def config0_block(x, device, copies=16, reps=32):
    """one NVFP4 GEMV at M = 1 through the linear API, 9216 x 3072 and 3072 x 9216, 16 weight
    copies rotated (> L2). Device time of the GEMV kernel (the activation digitizer listed apart); algorithmic bytes
    = NVFP4 codes + scales + global + x in bf16 + y in f32."""
    import torch
    from torch.profiler import profile, ProfilerActivity
    g = torch.Generator(device=device)
    g.manual_seed(0)
    peak, peak_kind = peaks()
    out = {}
    for n, k, alg in ((9216, 3072, 15968260), (3072, 9216, 15955972)):
        lins = [x.Linear([(torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=device, generator=g),
                           torch.randint(0x30, 0x40, (n, k // 16), dtype=torch.uint8, device=device, generator=g),
                           1.0)], k) for _ in range(copies)]
        xin = torch.randn(1, k, device=device, generator=g)
        ys = [torch.empty(1, n, device=device)]
        for it in range(copies):
            lins[it](xin, ys)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for it in range(reps):
                lins[it % copies](xin, ys)
            torch.cuda.synchronize()
        t = kernel_times(prof)
        us = t["gemv_kernel"]
        out[f"{n}x{k}"] = {"gemv_us": us, "digitize_us": t.get("digitize_rows_kernel"), "algorithmic_bytes": alg,
                           "gbs": alg / us / 1e3, "frac": alg / us / 1e3 / peak, "peak": peak, "peak_kind": peak_kind}
        for l_ in lins:
            l_.close()
    return out


def config2_block(x, device, reps=6):
    """decode attention for 8 rows x 24 q heads over an int8 KV cache (6 KV heads, head_dim 128),
    codes U[-127, 127], scales U(0.005, 0.02), q ~ N(0, 1) unit-normed per head: global layers at L = 4096, 8192,
    32768 (p = L - 8) with the step's 49 splits, and a sliding layer (1088-slot ring in rotated order, window 1024,
    17 splits). Device time of the attention kernel plus the split combine; bytes = L * 1584 + 147,456 (q and out)."""
    import torch
    from torch.profiler import profile, ProfilerActivity
    g = torch.Generator(device=device)
    g.manual_seed(2)
    peak, peak_kind = peaks()
    kvh, heads = 6, 24

    def rows(n, h):
        t = torch.randn(8, h, 128, device=device, generator=g)
        return t / t.norm(dim=-1, keepdim=True)

    out = {}
    for name, slots, pos0, window, ring, splits in (("global_4096", 4096, 4088, 0, False, 49),
                                                  ("global_8192", 8192, 8184, 0, False, 49),
                                                  ("global_32768", 32768, 32760, 0, False, 49),
                                                  ("sliding_1088", 1088, 40000, 1024, True, 17)):
        q, k, v = rows(8, heads), rows(8, kvh), rows(8, kvh)
        kc = torch.randint(-127, 128, (kvh * slots * 128,), dtype=torch.int8, device=device, generator=g)
        vc = torch.randint(-127, 128, (kvh * slots * 128,), dtype=torch.int8, device=device, generator=g)
        ks = torch.rand(kvh, slots, device=device, generator=g) * 0.015 + 0.005
        vs = torch.rand(kvh, slots, device=device, generator=g) * 0.015 + 0.005
        rp = None
        if ring:   # the most recent 1088 positions, slot = position % 1088 (rotated order)
            p = torch.arange(pos0 - slots, pos0, device=device, dtype=torch.int32)
            rp = torch.empty(slots, dtype=torch.int32, device=device)
            rp[p % slots] = p
        args = (q, k, v, kc.view(torch.uint8), vc.view(torch.uint8), ks, vs, pos0, window, 1.0 / 128 ** 0.5 * 8)
        for _ in range(3):
            x.attention(*args, ring_pos=rp, splits=splits)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(reps):
                x.attention(*args, ring_pos=rp, splits=splits)
            torch.cuda.synchronize()
        t = kernel_times(prof)
        us = t["attention_kernel"] + t["attn_combine_kernel"]
        alg = slots * 1584 + 147456
        out[name] = {"attention_us": t["attention_kernel"], "combine_us": t["attn_combine_kernel"],
                     "algorithmic_bytes": alg, "gbs": alg / us / 1e3, "frac": alg / us / 1e3 / peak}
    return out


def split_kv_block(x, rank, world, local_rank, dist, steps, warmup, context=32768):
    """The batch-1 long-context step split across the N processes: one sequence at 32K context, every process holding
    the whole model and every cache, each attending 1/N of the global caches' chunks, the attention partials joined
    inside the combine kernel (each process's merged partial stored into every peer's slots over NVLink as words
    carrying the step's sequence number) or, for comparison, by an NCCL all-gather between the kernels. Against the
    same step on one GPU (every rank runs that alone too). Times are the max over ranks."""
    import torch
    model = dict(x.DORY_3072)
    out = {"context": context, "n_past": context - 8}
    for name, exch in (("one_gpu", None), ("split_kv", "peer"), ("split_kv_nccl", "nccl")):
        opts = {}
        if exch:
            ids = [bytes(torch.cuda.nccl.unique_id()).hex() if rank == 0 else None]
            dist.broadcast_object_list(ids, src=0)
            opts = dict(kv_world=world, kv_rank=rank, nccl_id=ids[0], kv_exchange=exch)
        s = x.Session(model, context=context, device=local_rank, **opts)
        try:
            s.prefill_synthetic(context - 8)
            s.bench(TOKENS, max(1, warmup))
            dist_barrier(dist)
            ms, _, _ = s.bench(TOKENS, steps)
            dist_barrier(dist)
            out[name + "_ms_per_step"] = max_over_ranks(ms, dist)
            if exch:
                out[name + "_argmax_matches_one_gpu"] = s.argmax(8) == out["_argmax"]
                out["splits_global_per_gpu"] = s.info()["splits_global"]
            else:
                out["_argmax"] = s.argmax(8)
        finally:
            s.close()
    out.pop("_argmax")
    out["speedup"] = out["one_gpu_ms_per_step"] / out["split_kv_ms_per_step"]
    out["tok_s"] = 8.0 / (out["split_kv_ms_per_step"] / 1e3)
    return out


def topk_block(x, device, vocab, reps=20):
    """Device time of the sampler-candidate kernel (xtg_cuda_topk_rows) on 8 rows of logits at k = 64 and 1024:
    one read of the rows (8 x vocab x 4 bytes) against the HBM roofline."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(5)
    logits = torch.randn(8, vocab, device=device, generator=g) * 3
    peak, _ = peaks()
    out = {}
    for k in (TOPK, 1024):
        for _ in range(3):
            x.topk(logits, k)
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            x.topk(logits, k)
        e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        alg = 8 * vocab * 4
        out[f"k{k}"] = {"us": us, "algorithmic_bytes": alg, "gbs": alg / us / 1e3, "frac": alg / us / 1e3 / peak}
    return out


def shared_sessions_block(x, s, dist, steps, sessions=4):
    """Config 4's layout on each GPU: `sessions` independent sequences over one weight set (the first is the bench's
    session, the others opened with xtg_cuda_open_shared, each at 8184 positions), each stepping in its own thread on
    its own stream and graph. Rows per second by wall clock around all of them (max over ranks)."""
    import threading
    others = [x.Session.shared(s, context=8192) for _ in range(sessions - 1)]
    try:
        every = [s] + others
        for o in others:
            o.prefill_synthetic(PREFILL)
        for o in every:
            o.bench(TOKENS, 3)
        dist_barrier(dist)
        th = [threading.Thread(target=o.bench, args=(TOKENS, steps)) for o in every]
        t0 = time.perf_counter()
        for t in th:
            t.start()
        for t in th:
            t.join()
        wall = time.perf_counter() - t0
        dist_barrier(dist)
        wall = max_over_ranks(wall, dist)
        e2e = e2e_tk = None
        if dist is None:   # one process: the end-to-end legs (measured on 1 GPU only)
            # end to end from one thread (a server's engine thread): xtg_cuda_forward_batch with host tokens in and every
            # row's logits out, then each session's rewind
            lists = [TOKENS] * sessions
            for _ in range(2):
                x.forward_batch(every, lists, want=2)
                for o in every:
                    o.rewind(PREFILL)
            t0 = time.perf_counter()
            for _ in range(steps):
                x.forward_batch(every, lists, want=2)
                for o in every:
                    o.rewind(PREFILL)
            e2e = time.perf_counter() - t0
            # the same with the sampler's 64 candidates per row instead of whole rows (xtg_cuda_topk per session)
            for _ in range(2):
                x.forward_batch(every, lists, want=0)
                for o in every:
                    o.topk(TOPK)
                    o.rewind(PREFILL)
            t0 = time.perf_counter()
            for _ in range(steps):
                x.forward_batch(every, lists, want=0)
                for o in every:
                    o.topk(TOPK)
                    o.rewind(PREFILL)
            e2e_tk = time.perf_counter() - t0
    finally:
        for o in others:
            o.close()
    return {"sessions_per_gpu": sessions, "steps_each": steps, "wall_s": wall,
            "rows_per_s_per_gpu": sessions * 8 * steps / wall,
            "e2e_forward_batch_rows_per_s_per_gpu": sessions * 8 * steps / e2e if e2e else None,
            "e2e_forward_batch_topk_rows_per_s_per_gpu": sessions * 8 * steps / e2e_tk if e2e_tk else None,
            "e2e_d2h_bytes_per_round": sessions * 8 * 131072 * 4}


def acceptance_draws(n, seed=4):
    """BASELINE config 4's seeded acceptance: tokens accepted per verify step, uniform in 1..4 (numpy PCG64, seed 4)."""
    import numpy as np
    return np.random.default_rng(seed).integers(1, 5, n)


def rates(world, ms_per_step):
    """Steps, verify rows and accepted tokens per second for the whole job (accepted: the mean of 256 seeded draws
    of 1..4 tokens per step, as config 4 drives its rewinds)."""
    steps = world / (ms_per_step / 1e3)
    acc = float(acceptance_draws(256).mean())
    return {"steps_per_s": steps, "rows_per_s": 8.0 * steps, "accepted_tok_per_s": acc * steps,
            "accepted_per_step": acc}


def config4_draws(rank, world, steps, seqs_total):
    """This rank's share of config 4's seeded acceptances: sequences rank * per_gpu .. (rank + 1) * per_gpu - 1 of the
    [steps][seqs_total] draws (the same draws whatever the partition)."""
    per_gpu = seqs_total // world
    return acceptance_draws(steps * seqs_total).reshape(steps, seqs_total)[:, rank * per_gpu:(rank + 1) * per_gpu]


def config4_block(x, rank, world, local_rank, dist, steps=256, seqs_total=64, context=32768, prefill=30000):
    """64 independent sequences of the config-3 model at the 32K tier, each prefilled to 30000
    positions, partitioned over the N GPUs (64 / N per GPU, no collective on the data path). 256 verify rounds: every
    sequence verifies 8 rows (xtg_cuda_forward_batch: the sessions step as batched steps of up to 8 sequences, each
    projection one tcgen05 GEMM over their rows), its 8 argmax tokens are read back, and a seeded acceptance of 1..4
    tokens (numpy PCG64, seed 4, one draw per sequence and round) drives its rewind to base + accepted. Wall clock around
    the rounds, max over ranks."""
    per_gpu = seqs_total // world
    model = dict(x.DORY_3072)
    acc = config4_draws(rank, world, steps, seqs_total)
    owner = x.Session(model, context=context, device=local_rank)
    sessions = [owner] + [x.Session.shared(owner, context=context) for _ in range(per_gpu - 1)]
    try:
        for s in sessions:
            s.prefill_synthetic(prefill)
        lists = [TOKENS] * per_gpu
        for _ in range(2):   # warm-up (the batched graphs are captured here)
            x.forward_batch(sessions, lists, want=0)
            for s in sessions:
                s.argmax(8)
                s.rewind(prefill)
        dist_barrier(dist)
        base = [prefill] * per_gpu
        t0 = time.perf_counter()
        for st in range(steps):
            x.forward_batch(sessions, lists, want=0)
            for j, s in enumerate(sessions):
                s.argmax(8)
                base[j] += int(acc[st, j])
                assert s.rewind(base[j])
        wall = time.perf_counter() - t0
        dist_barrier(dist)
        wall = max_over_ranks(wall, dist)
        accepted = sum_over_ranks(float(acc.sum()), dist)   # every rank's own draws
        kv = sessions[0].step_bytes(2, 8)   # one sequence's KV read per round at its last position
        weights = sessions[0].step_bytes(1, 8)
        groups = (per_gpu + 7) // 8
    finally:
        for s in sessions:
            s.close()
    rows = 8.0 * per_gpu * steps / wall
    peak, peak_kind = peaks()
    bytes_round = groups * weights + per_gpu * kv
    return {"sequences": seqs_total, "per_gpu": per_gpu, "context": context, "prefill": prefill, "steps": steps,
            "wall_s": wall, "rows_per_s_per_gpu": rows, "job_rows_per_s": rows * world,
            "accepted_tok_per_s_per_gpu": accepted / world / wall, "job_accepted_tok_per_s": accepted / wall,
            "mean_accepted_per_round": float(acc.mean()), "ms_per_round": wall / steps * 1e3,
            "batched_groups_per_gpu": groups,
            "roofline": {"bound": "hbm", "bytes_per_round_per_gpu": bytes_round,
                         "note": "weights once per batched group of 8 + every sequence's KV (at its final position)",
                         "achieved": bytes_round / (wall / steps) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": bytes_round / (wall / steps) / 1e9 / peak, "peak_kind": peak_kind},
            "e2e": {"h2d_bytes_per_round": per_gpu * 48, "d2h_bytes_per_round": per_gpu * 8 * 4,
                    "note": "the rounds above are end to end: host tokens in, each session's argmax read back"}}


def prefill_block(x, local_rank, n_tokens=4096, reps=3):
    """Prompt processing on the config-3 model (8K tier, from position 0): xtg_cuda_forward of n_tokens tokens without
    logits, in prompt chunks of 64 rows through the batched step (every projection one tcgen05 GEMM over the chunk),
    against the same tokens in 8-row verify steps (batch=0). Wall clock per call (best of reps)."""
    model = dict(x.DORY_3072)
    toks = [(37 * i + 11) % model["vocab"] for i in range(n_tokens)]
    out = {"tokens": n_tokens}
    for name, batch in (("chunks64", 1), ("verify8", 0)):
        s = x.Session(model, context=8192, device=local_rank, batch=batch)
        try:
            best = None
            for _ in range(reps + 1):
                s.rewind(0)
                t0 = time.perf_counter()
                s.forward(toks, want=0)
                dt = time.perf_counter() - t0
                best = dt if best is None else min(best, dt)
            out[name + "_s"] = best
            out[name + "_tok_per_s"] = n_tokens / best
        finally:
            s.close()
    out["speedup"] = out["verify8_s"] / out["chunks64_s"]
    return out


def dory4b_block(x, local_rank, steps, warmup):
    """The real Dory 4B's shape (hidden 2560, 16 q / 4 KV heads of 256, FFN 7168, vocab 131072, 16 + 40 x 2 + 16
    sublayers; synthetic weights): the 8-row verify step at the 8K tier over 8184 prefilled positions, graph replays
    timed with CUDA events as the headline step is, with its own step roofline."""
    s = x.Session(dict(x.DORY_4B), context=8192, device=local_rank)
    try:
        s.prefill_synthetic(PREFILL)
        s.bench(TOKENS, max(1, warmup))
        ms, _, _ = s.bench(TOKENS, steps)
        pms, cms, cl = s.bench(TOKENS, 3, profile=True)
        step_bytes = s.step_bytes(0, 8)
        gemv_bytes = s.step_bytes(1, 8)
        peak, peak_kind = peaks()
        return {"ms_per_step": ms, "rows_per_s": 8.0 / (ms / 1e3), "rates": rates(1, ms),
                "launches_per_step": int(sum(cl)),
                "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (ms / 1e3) / 1e9,
                                  "frac": step_bytes / (ms / 1e3) / 1e9 / peak, "peak": peak, "peak_kind": peak_kind},
                "gemv_roofline": {"achieved_gbs": gemv_bytes / (cms[0] / 1e3) / 1e9,
                                  "frac": gemv_bytes / (cms[0] / 1e3) / 1e9 / peak},
                "kernel_ms_per_step": {"gemv": cms[0], "attention": cms[1], "combine": cms[2], "small": cms[3],
                                       "eager_total": pms},
                "splits_global": s.info().get("splits_global")}
    finally:
        s.close()


def job_rows_per_s(world, ms_per_step):
    """Whole-job throughput: every rank verifies 8 rows of its own sequence per step (weak scaling)."""
    return world * 8.0 / (ms_per_step / 1e3)


def run_ours(args, rank, world, local_rank, dist):
    import torch
    x = package()
    torch.cuda.set_device(local_rank)
    model = dict(x.DORY_3072)
    s = x.Session(model, context=8192, device=local_rank)
    s.prefill_synthetic(PREFILL)

    def barrier():
        dist_barrier(dist)

    # warm-up (graph capture included), then the timed device region
    s.bench(TOKENS, max(1, args.warmup))
    barrier()
    with Clocks(local_rank) as clk:
        ms, _, _ = s.bench(TOKENS, args.steps)
    barrier()
    ms = max_over_ranks(ms, dist)
    value = job_rows_per_s(world, ms)
    # end to end through the C ABI: host token buffer in, every row's logits out, the rewind a verify step does
    for _ in range(2):
        s.forward(TOKENS, want=2)
        s.rewind(PREFILL)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s.forward(TOKENS, want=2)
        s.rewind(PREFILL)
    e2e_s = (time.perf_counter() - t0) / args.steps
    barrier()
    e2e_s = max_over_ranks(e2e_s, dist)
    # the same, reading back the sampler's 64 most likely candidates per row (xtg_cuda_topk) instead of whole rows
    for _ in range(2):
        s.forward(TOKENS, want=0)
        s.topk(TOPK)
        s.rewind(PREFILL)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s.forward(TOKENS, want=0)
        s.topk(TOPK)
        s.rewind(PREFILL)
    e2e_topk_s = (time.perf_counter() - t0) / args.steps
    barrier()
    e2e_topk_s = max_over_ranks(e2e_topk_s, dist)
    # per-kernel-class device time (eager launches with events), for the roofline of the dominant kernel
    pms, cms, cl = s.bench(TOKENS, 3, profile=True)
    gemv_bytes = s.step_bytes(1, 8)
    step_bytes = s.step_bytes(0, 8)
    peak, peak_kind = peaks()
    gemv_launches = max(1, cl[0])
    achieved = gemv_bytes / (cms[0] / 1e3) / 1e9
    traffic = ncu_traffic()
    info = s.info()
    shared = shared_sessions_block(x, s, dist, args.steps)
    s.close()
    cfg4 = None if args.no_config4 else config4_block(x, rank, world, local_rank, dist, steps=args.config4_steps)
    pre = prefill_block(x, local_rank) if world == 1 else None
    topk_t = topk_block(x, f"cuda:{local_rank}", model["vocab"]) if world == 1 else None
    gemm = gemm_block(x, f"cuda:{local_rank}") if (world == 1 and not args.no_gemm) else None
    cfg0 = config0_block(x, f"cuda:{local_rank}") if (world == 1 and not args.no_gemm) else None
    cfg2 = config2_block(x, f"cuda:{local_rank}") if (world == 1 and not args.no_gemm) else None
    heads = head_block(x, f"cuda:{local_rank}") if (world == 1 and not args.no_gemm) else None
    d4b = dory4b_block(x, local_rank, args.steps, args.warmup) if world == 1 else None
    # the batch-1 split over GPUs: measured where its 2-GPU tests run (--split-kv-max raises the bound)
    skv = (split_kv_block(x, rank, world, local_rank, dist, args.steps, args.warmup)
           if 1 < world <= args.split_kv_max else None)
    if rank != 0:
        return
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "nvfp4 weights x e2m1-digit activations (4 block-scaled digits) on tcgen05, f32 accumulate; int8 KV",
            "data": "synthetic (seeded random-init weights, random prefilled KV)", "config": config_block(world),
            "value_counts": "verify rows per second (8 per step); accepted tokens per second are in `rates`",
            "rates": rates(world, ms),
            "e2e": {"value": world * 8.0 / e2e_s, "unit": UNIT, "h2d_bytes_per_step": 48,
                    "d2h_bytes_per_step": 8 * model["vocab"] * 4, "ms_per_step": e2e_s * 1e3},
            "e2e_topk": {"value": world * 8.0 / e2e_topk_s, "unit": UNIT, "h2d_bytes_per_step": 48,
                         "d2h_bytes_per_step": 8 * TOPK * 8 + 8 * 12, "ms_per_step": e2e_topk_s * 1e3,
                         "note": f"forward without logits, then xtg_cuda_topk(k={TOPK}): the sampler's candidates"},
            "roofline": {"bound": "hbm", "kernel": "gemv_nvfp4 (all NVFP4 GEMVs of the step)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "algorithmic_bytes_per_launch": gemv_bytes / gemv_launches,
                         "launch_ms": cms[0] / gemv_launches},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (ms / 1e3) / 1e9,
                              "frac": step_bytes / (ms / 1e3) / 1e9 / peak, "peak": peak},
            "kernel_ms_per_step": {"gemv": cms[0], "attention": cms[1], "combine": cms[2], "small": cms[3],
                                   "eager_total": pms},
            "gpu_launches": int(sum(cl)) * args.steps,
            "clocks": clk.summary(),
            "library": {"splits_global": info.get("splits_global"), "splits_ring": info.get("splits_ring"),
                        "graph": info.get("graph"), "pdl": info.get("pdl")}}
    if topk_t:
        line["topk"] = topk_t
    line["config4_shared_sessions"] = {
        "config": "4 independent sequences per GPU over one weight set (xtg_cuda_open_shared), 8K tier, each "
                  "stepping concurrently on its own stream; wall clock", **shared,
        "job_rows_per_s": world * shared["rows_per_s_per_gpu"], "vs_one_session": shared["rows_per_s_per_gpu"] / (value / world)}
    if cfg4:
        line["config4"] = {"config": "config4: 64 sequences of the config-3 model at the 32K tier (30000 prefilled), "
                                     "partitioned over the GPUs, 8-row verify rounds through xtg_cuda_forward_batch "
                                     "(batched steps of up to 8 sequences), argmax read back, seeded 1..4 acceptance "
                                     "driving rewinds; wall clock, max over ranks", **cfg4}
    if pre:
        line["prefill"] = {"config": "prompt of 4096 tokens on the config-3 model (8K tier) from position 0, no logits: "
                                     "64-row prompt chunks (tcgen05 GEMM, batched step) vs 8-row verify steps; wall "
                                     "clock, best of 3", **pre}
    if cfg0:
        line["config0_gemv"] = {"config": "config0: one NVFP4 GEMV, M = 1, 16 weight copies rotated", **cfg0}
    if cfg2:
        line["config2_attention"] = {"config": "config2: 8-row decode attention, int8 KV, attention + split combine",
                                     **cfg2}
    if heads:
        line["lm_head"] = {"config": "lm_head at vocab 131072 x 3072, 8 rows: NVFP4 on the GEMV (the synthetic model's "
                                     "head) and a checkpoint's BF16 head (head.cu, mma.sync over bf16 hi + lo rows)",
                           **heads}
    if d4b:
        line["dory4b"] = {"config": "the real Dory 4B shape (hidden 2560, 16 q / 4 KV heads of head_dim 256, FFN 7168, "
                                    "vocab 131072, 16 + 40 x 2 + 16 sublayers) with synthetic weights, 8K tier, "
                                    "8184 prefilled, 8-row verify step, graph replays", **d4b}
    if skv:
        line["batch1_split_kv"] = {"config": "batch-1 verify step (8 rows) at 32K context, the global caches' chunks "
                                             "split over the GPUs, partials exchanged over NVLink inside the combine "
                                             "kernel (split_kv) or by ncclAllGather (split_kv_nccl)", **skv}
    if gemm:
        tot_flops = sum(2.0 * 512 * v["n"] * v["k"] for v in gemm.values())
        tot_us = sum(v["gemm_us"] for v in gemm.values())
        bf16 = peaks_bf16()
        line["prefill_gemm"] = {
            "config": "config1 projection set at M=512 (QKVG 7680, O 3072, gate+up 18432, down 3072x9216), tcgen05 "
                      "mxf4nvf4, activations as 4 E2M1 digits", "per_projection": gemm,
            "total_gemm_us": tot_us, "tflops": tot_flops / tot_us / 1e6,
            "roofline": {"bound": "tensor", "achieved_fp4_mma_tflops": 4 * tot_flops / tot_us / 1e6,
                         "peak": 4 * bf16, "unit": "TFLOP/s", "frac": 4 * tot_flops / tot_us / 1e6 / (4 * bf16),
                         "peak_kind": "4x measured bf16 dense (burst)",
                         "note": "frac counts the FP4 MMA work (4 digits per activation); the useful 2 M N K "
                                 "against the same FP4 dense peak and against the measured bf16 peak:",
                         "useful_tflops": tot_flops / tot_us / 1e6,
                         "useful_frac_of_fp4_peak": tot_flops / tot_us / 1e6 / (4 * bf16),
                         "useful_frac_of_bf16_peak": tot_flops / tot_us / 1e6 / bf16}}
    if world == 1 and not args.no_cpu_baseline:
        try:
            step_s, setup = reference_steps(model, os.cpu_count() or 1, 2, 1)
            line["cpu_baseline"] = {"value": 8.0 / step_s, "unit": UNIT, "cores": os.cpu_count() or 1,
                                    "kind": "reference",
                                    "sample": "2 whole config-3 steps after 1 warm-up on the reference's kernels "
                                              "(FP8 KvCaches, 1040-slot rings: the reference has no int8 cache)"}
        except Exception as e:  # the baseline is reported, never the target
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "reference",
                                    "sample": f"unavailable: {e}"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true", help="skip the config-1 M=512 prefill GEMM measurement")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 batched serving measurement")
    ap.add_argument("--config4-steps", type=int, default=256, help="verify rounds of the config-4 measurement")
    ap.add_argument("--split-kv-max", type=int, default=8,
                    help="largest world size at which the batch-1 split-KV step is measured (N > 1)")
    ap.add_argument("--ncu-steps", type=int, default=0,
                    help="profiling driver: run this many eager steps (no graph, no JSON) for ncu, then exit")
    ap.add_argument("--ncu-model", default="full", choices=["full", "small"],
                    help="small: the same shapes with 2 + 2 + 2 sublayers (about 0.5 GB on the device)")
    ap.add_argument("--ncu-gemm", type=int, default=0,
                    help="profiling driver: run the config-1 gate+up GEMM at M=512 this many times, then exit")
    ap.add_argument("--ncu-batch", type=int, default=0,
                    help="profiling driver: this many batched rounds of 8 sequences (8K tier), then exit")
    ap.add_argument("--ncu-head", type=int, default=0,
                    help="profiling driver: the BF16 lm_head (vocab 131072 x 3072, 8 rows) this many times, then exit")
    ap.add_argument("--ncu-attn", type=int, default=0,
                    help="profiling driver: config-2 global attention (int8 KV, L = 32768, 49 splits) this many "
                         "times, then exit")
    ap.add_argument("--ncu-attn-len", type=int, default=32768, help="cached positions of --ncu-attn (a multiple of 64)")
    args = ap.parse_args()
    if args.ncu_attn:
        import torch
        x = package()
        g = torch.Generator(device="cuda").manual_seed(2)
        kvh, heads, slots = 6, 24, args.ncu_attn_len
        q, k, v = (torch.nn.functional.normalize(torch.randn(8, h, 128, device="cuda", generator=g), dim=-1)
                   for h in (heads, kvh, kvh))
        kc = torch.randint(-127, 128, (kvh * slots * 128,), dtype=torch.int8, device="cuda", generator=g)
        vc = torch.randint(-127, 128, (kvh * slots * 128,), dtype=torch.int8, device="cuda", generator=g)
        ks = torch.rand(kvh, slots, device="cuda", generator=g) * 0.015 + 0.005
        vs = torch.rand(kvh, slots, device="cuda", generator=g) * 0.015 + 0.005
        for _ in range(args.ncu_attn):
            x.attention(q, k, v, kc.view(torch.uint8), vc.view(torch.uint8), ks, vs, slots - 8, 0,
                        1.0 / 128 ** 0.5 * 8, splits=49)
        torch.cuda.synchronize()
        return
    if args.ncu_gemm:
        import torch
        x = package()
        g = torch.Generator(device="cuda")
        g.manual_seed(1)
        k = 3072
        ws = [(torch.randint(0, 256, (9216, k // 2), dtype=torch.uint8, device="cuda", generator=g),
               torch.randint(0x30, 0x40, (9216, k // 16), dtype=torch.uint8, device="cuda", generator=g), 1.0)
              for _ in range(2)]
        lin = x.Linear(ws, k)
        xin = torch.randn(512, k, device="cuda", generator=g)
        for _ in range(args.ncu_gemm):
            lin(xin)
        torch.cuda.synchronize()
        lin.close()
        return
    if args.ncu_head:
        import torch
        x = package()
        g = torch.Generator(device="cuda").manual_seed(5)
        w = (torch.randn(131072, 3072, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        xin = torch.randn(8, 3072, device="cuda", generator=g)
        ls = torch.rand(131072, device="cuda", generator=g) * 100 + 100
        for _ in range(args.ncu_head):
            x.head_bf16(xin, w, ls)
        torch.cuda.synchronize()
        return
    if args.ncu_batch:
        x = package()
        model = dict(x.DORY_3072)
        if args.ncu_model == "small":
            model.update(n_in=2, n_rec=2, n_out=2, loops=1)
        owner = x.Session(model, context=8192)
        sess = [owner] + [x.Session.shared(owner, context=8192) for _ in range(7)]
        for s_ in sess:
            s_.prefill_synthetic(PREFILL)
        for _ in range(args.ncu_batch):
            x.forward_batch(sess, [TOKENS] * 8, want=0)
            for s_ in sess:
                s_.rewind(PREFILL)
        for s_ in sess:
            s_.close()
        return
    if args.ncu_steps:
        x = package()
        model = dict(x.DORY_3072)
        if args.ncu_model == "small":
            model.update(n_in=2, n_rec=2, n_out=2, loops=1)
        s = x.Session(model, context=8192, graph=False)
        s.prefill_synthetic(PREFILL)
        s.bench(TOKENS, args.ncu_steps)
        s.close()
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        # the collectives here are a barrier, a max and the split-KV step's small all-gather: plain peer copies
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        dist = tdist
    try:
        run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
