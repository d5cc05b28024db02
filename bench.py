"""Benchmark of the region hot path on B200: Qwen3-4B-4bit prefill-128 + 1 decode.

One step = one request as the reference's workload defines it
(models/workloads/qwen3_4b_prefill_128.yaml; autotuner_runtime/inference.py:
131-156): from an empty KV cache, prefill 128 prompt tokens, pick the next
token, run one decode step, pick again. Every region runs through the bundle's
wrappers (try_call -> libmt.so), strict mode on (a fallback raises). The
request is captured once in a CUDA graph and replayed.

  value  prompt tokens/s (128 / request time) with tokens already on the
         device, CUDA events around K replays, max over ranks, x ranks
         (independent replicas: the path does not shard).
  e2e    the same metric through the public call with host buffers: pinned
         host tokens -> device, replay, read back the two picked tokens and
         the logprob, every step.
  roofline  the dominant kernel (tcgen05 prefill qmm, all 144 launches of
         the request's prefill) timed on its own stream with CUDA events:
         algorithmic FLOPs / time vs the measured bf16 peak.
  cpu_baseline  the oracle restatement (C, OpenMP, all host threads) on one
         decoder layer of the same request, extrapolated to the full request.

--impl reference times the CPU implementation of the path (the oracle port;
the reference's own path is MLX on Apple GPUs, unavailable here) on the same
metric. --mode kernels prints per-region kernel timings (profiling entry).
--config llama3_8b_tp times the Llama-3-8B 8-bit prefill forward (batch 8 x
2048), tensor-parallel over the torchrun ranks with NCCL (run_llama_tp).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Qwen3-4B-4bit prefill-128 tok/s per GPU, % of HBM/TC roofline, vs MLX CPU"
PROMPT = 128
REFERENCE_WALL_CAP_S = 150


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sms.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for name, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sms)}


# ------------------------------------------------------------------ peaks
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ distributed
def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ workload
def qmm_launches(cfg, M):
    """(name, M, N, K, kind) of the prefill qmm launches of one layer."""
    h, q, kv, f = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.ffn
    return [("qkv", M, q + 2 * kv, h), ("o_proj", M, h, q), ("gate_up", M, 2 * f, h), ("down", M, h, f)]


def request_flops(cfg, prompt=PROMPT):
    per_layer = sum(2 * M * N * K for _, M, N, K in qmm_launches(cfg, prompt))
    return per_layer * cfg.layers


def packed_weight_bytes(cfg):
    h, q, kv, f = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.ffn
    params = (h * (q + 2 * kv) + q * h + 3 * h * f) * cfg.layers
    per_param = cfg.bits / 8 + 2 * 2 / cfg.group  # packed bits + bf16 scale and bias per group
    return params * per_param, cfg.vocab * h * per_param


class Request:
    """The applied model, its cache and a captured CUDA graph of one request."""

    def __init__(self, cfg, seed=0):
        import torch

        from metal_autotune_b200.autotuner_runtime.apply import apply
        from metal_autotune_b200.targets import qwen3
        os.environ["MT_STRICT_REGIONS"] = "1"
        self.torch = torch
        self.cfg = cfg
        t0 = time.time()
        model = qwen3.build(cfg, seed=seed, device="cuda")
        torch.cuda.synchronize()
        log(f"built random Qwen3 ({cfg.layers} layers) in {time.time() - t0:.1f}s")
        bundle = ROOT / "metal_autotune_b200" / "bundles" / ("qwen3_4b" if cfg.layers == 36 else "qwen3_tiny")
        self.model = apply(model, bundle)
        self.cache = qwen3.KVCache(cfg, device="cuda")
        from metal_autotune_b200 import workload
        self.tokens = workload.seeded_tokens((PROMPT,), 0, cfg.vocab, seed=seed)
        self.host_tokens = self.tokens.cpu().pin_memory()
        self.host_out = torch.empty(3, dtype=torch.int32).pin_memory()
        self.qwen3 = qwen3
        self.launches_per_step = None

    def eager(self):
        return self.qwen3.request(self.model, self.tokens, self.cache)

    def capture(self):
        torch = self.torch
        from metal_autotune_b200 import lib
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.eager()
            self.eager()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        before = lib.CALLS[0]
        with torch.cuda.graph(self.graph):
            self.out = self.eager()
            # the three results in one buffer, so e2e reads them back with one copy
            self.res_dev = torch.cat([self.out[0].view(1), self.out[1].view(1),
                                      self.out[2].view(torch.int32).view(1)])
        self.launches_per_step = lib.CALLS[0] - before

    def replay(self):
        self.graph.replay()

    def e2e_step(self):
        """Public-API request with host buffers: H2D tokens, run, D2H result."""
        torch = self.torch
        self.tokens.copy_(self.host_tokens, non_blocking=True)
        self.graph.replay()
        self.host_out.copy_(self.res_dev, non_blocking=True)


def time_region(fn, steps, world):
    import torch
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end)


def qmm_roofline(req, peaks, reps=20):
    """Time the request's prefill qmm launches (the dominant kernel) alone."""
    import torch

    from metal_autotune_b200 import lib
    cfg = req.cfg
    layers = req.model.wrapped.layers
    x = {"qkv": torch.randn(PROMPT, cfg.hidden, device="cuda").to(torch.bfloat16),
         "o": torch.randn(PROMPT, cfg.heads * cfg.head_dim, device="cuda").to(torch.bfloat16),
         "down": torch.randn(PROMPT, cfg.ffn, device="cuda").to(torch.bfloat16)}
    res = torch.randn(PROMPT, cfg.hidden, device="cuda").to(torch.bfloat16)
    outs = {}

    def run_all():
        for L in layers:
            W = L._w
            outs["qkv"] = lib.quantized_matmul_multi(x["qkv"], [W["qkv"][0:3], W["qkv"][3:6], W["qkv"][6:9]])
            outs["o"] = lib.quantized_matmul(x["o"], *W["o"], residual=res)
            outs["gu"] = lib.quantized_matmul_swiglu(x["qkv"], *W["gate_up"])
            outs["d"] = lib.quantized_matmul(x["down"], *W["down"], residual=res)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run_all()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            run_all()
        g.replay()
        s.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(s)
        for _ in range(reps):
            g.replay()
        end.record(s)
        s.synchronize()
    ms = start.elapsed_time(end) / reps
    launches = 4 * len(layers)
    flops = request_flops(cfg)
    achieved = flops / (ms / 1e3) / 1e12
    peak = peaks["bf16_tflops"]
    return {"bound": "tensor", "kernel": "qmm_tc_kernel (prefill qkv/o/gate_up/down, 144 launches)",
            "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "peak_source": f"{peaks['source']} bf16_tflops (burst)", "ms_all_launches": round(ms, 4),
            "us_per_launch": round(ms * 1e3 / launches, 2), "traffic": None}


# ------------------------------------------------------------------ CPU side
def cpu_layer_sample(cfg, seed=0):
    """Numpy copies of one random layer for the oracle (same generator as the model)."""
    import numpy as np
    import torch

    from metal_autotune_b200 import workload
    g = torch.Generator(device="cpu").manual_seed(seed)
    h, q, kv, ff = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.ffn
    W = {}
    for name, (nn_, kk) in dict(q=(q, h), k=(kv, h), v=(kv, h), o=(h, q), g=(ff, h), u=(ff, h), d=(h, ff)).items():
        wq, s, b = workload.random_quantized(nn_, kk, group=cfg.group, bits=cfg.bits, generator=g, device="cpu")
        W[name] = (wq.numpy().view(np.uint32), s.float().numpy(), b.float().numpy())
    return W


def cpu_request_seconds(cfg, threads):
    """Oracle time of one decoder layer's prefill + decode (all regions),
    extrapolated to the request (x layers) plus the lm_head rows."""
    import numpy as np

    from oracle import ref as R
    os.environ["OMP_NUM_THREADS"] = str(threads)
    R.lib()
    W = cpu_layer_sample(cfg)
    rng = np.random.default_rng(0)
    h = R.round_to(rng.standard_normal((PROMPT, cfg.hidden)).astype(np.float32), "bfloat16")
    ones_h = np.ones(cfg.hidden, np.float32)
    ones_d = np.ones(cfg.head_dim, np.float32)

    def layer(x, kc, vc, off):
        T = x.shape[0]
        qm = lambda a, w: R.quantized_matmul(a, *w, cfg.group, cfg.bits)
        xn = R.rms_norm(x, ones_h, cfg.eps)
        q, k, v = qm(xn, W["q"]), qm(xn, W["k"]), qm(xn, W["v"])
        qh, kc, vc = R.qk_norm_rope_cache(q, k, v, ones_d, ones_d, cfg.eps, kc, vc, cfg.heads, cfg.kv_heads,
                                          off, cfg.rope_theta)
        o = R.sdpa(qh[None], kc[None, :, :off + T], vc[None, :, :off + T], 1 / math.sqrt(cfg.head_dim), True, off)
        o = o[0].transpose(1, 0, 2).reshape(T, -1)
        h2 = R.add(qm(o, W["o"]), x)
        xn2 = R.rms_norm(h2, ones_h, cfg.eps)
        return R.add(qm(R.swiglu(qm(xn2, W["g"]), qm(xn2, W["u"])), W["d"]), h2)

    kc = np.zeros((cfg.kv_heads, cfg.max_len, cfg.head_dim), np.float32)
    vc = np.zeros_like(kc)
    t0 = time.perf_counter()
    layer(h, kc, vc, 0)
    layer(h[-1:], kc, vc, PROMPT)
    t_layer = time.perf_counter() - t0
    # lm_head: two rows against the tied embedding (vocab x hidden), timed on a slice and scaled
    rows = 8192
    wq, s, b = W["g"]  # any packed matrix of width `hidden` stands in for the embedding rows
    reps = max(1, rows // wq.shape[0])
    t1 = time.perf_counter()
    for _ in range(reps):
        R.qmv(h[-1:], wq, s, b, cfg.group, cfg.bits)
    t_head = (time.perf_counter() - t1) / (reps * wq.shape[0]) * cfg.vocab * 2
    return t_layer * cfg.layers + t_head, t_layer


def cpu_baseline(cfg, threads):
    secs, t_layer = cpu_request_seconds(cfg, threads)
    return {"value": round(PROMPT / secs, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"oracle C restatement (OpenMP {threads} threads) of 1 of {cfg.layers} decoder layers of "
                       f"the request (prefill 128 + decode 1, all regions) = {t_layer:.2f}s, x{cfg.layers} "
                       "+ lm_head rows timed on a slice; MLX CPU unavailable on this box")}


def run_reference(args, cfg):
    rank, world, _ = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    vals = []
    t_start = time.time()
    for _ in range(max(1, args.steps)):
        secs, t_layer = cpu_request_seconds(cfg, threads)
        vals.append(PROMPT / secs)
        if time.time() - t_start > REFERENCE_WALL_CAP_S:
            break
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(PROMPT / v * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "qwen3_4b_prefill_128+decode_1", "model": "Qwen3-4B 4-bit g64 (random init)",
                       "prompt_tokens": PROMPT, "decode_tokens": 1, "batch": 1, "parallelism": "host cores"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"each step: 1 of {cfg.layers} decoder layers (prefill 128 + decode 1) "
                                       f"timed, extrapolated x{cfg.layers}; median of {len(vals)} steps (of "
                                       f"{args.steps} requested; wall cap {REFERENCE_WALL_CAP_S}s); the "
                                       "reference's own path is MLX on an Apple GPU (unavailable on this box), "
                                       "so the oracle port is timed"},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ kernels mode
def run_kernels(args, cfg):
    """Each prefill/decode region kernel at the config's shapes, timed alone."""
    import torch

    from metal_autotune_b200 import lib, workload
    peaks = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(0)
    rows = []
    only = set(args.only.split(",")) if args.only else None

    def bench(name, fn, flops=0.0, nbytes=0.0, reps=args.steps):
        if only and name not in only:
            return
        # launches are captured in a CUDA graph so host-side call overhead is not timed
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            for _ in range(max(args.warmup, 1)):
                fn()
            st.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                for _ in range(reps):
                    fn()
            g.replay()
            st.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(st)
            g.replay()
            e.record(st)
            st.synchronize()
        us = s.elapsed_time(e) * 1e3 / reps
        r = {"kernel": name, "us": round(us, 2)}
        if flops:
            r["tflops"] = round(flops / us / 1e6, 2)
            r["frac_tc"] = round(r["tflops"] / peaks["bf16_tflops"], 4)
        if nbytes:
            r["gbs"] = round(nbytes / us / 1e3, 1)
            r["frac_hbm"] = round(r["gbs"] / peaks["hbm_gbs"], 4)
        rows.append(r)
        print(json.dumps(r), flush=True)

    h, q, kv, ff = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.ffn
    W = {k: workload.random_quantized(n_, k_, generator=g) for k, (n_, k_) in
         dict(q=(q, h), k=(kv, h), v=(kv, h), o=(h, q), g=(ff, h), u=(ff, h), d=(h, ff)).items()}
    bpp = cfg.bits / 8 + 4 / cfg.group
    for M in (PROMPT, 1):
        xh = torch.randn(M, h, device="cuda").to(torch.bfloat16)
        xq = torch.randn(M, q, device="cuda").to(torch.bfloat16)
        xf = torch.randn(M, ff, device="cuda").to(torch.bfloat16)
        res = torch.randn(M, h, device="cuda").to(torch.bfloat16)
        tag = "prefill" if M > 1 else "decode"
        bench(f"{tag}_qkv", lambda: lib.quantized_matmul_multi(xh, [W["q"], W["k"], W["v"]]),
              2 * M * (q + 2 * kv) * h, (q + 2 * kv) * h * bpp)
        bench(f"{tag}_o_proj", lambda: lib.quantized_matmul(xq, *W["o"], residual=res), 2 * M * h * q, h * q * bpp)
        bench(f"{tag}_gate_up", lambda: lib.quantized_matmul_swiglu(xh, *W["g"], *W["u"]), 4 * M * ff * h,
              2 * ff * h * bpp)
        bench(f"{tag}_down", lambda: lib.quantized_matmul(xf, *W["d"], residual=res), 2 * M * h * ff, h * ff * bpp)
        nw = torch.ones(h, device="cuda", dtype=torch.bfloat16)
        bench(f"{tag}_rms_norm", lambda: lib.rms_norm(xh, nw, 1e-6), 0, 2 * M * h * 2)
        if M <= 4:
            # the decode cuts with the RMSNorm fused into the matmul's staging of x
            bench(f"{tag}_norm_qkv", lambda: lib.rms_norm_quantized_matmul_multi(xh, nw, 1e-6, [W["q"], W["k"], W["v"]]),
                  2 * M * (q + 2 * kv) * h, (q + 2 * kv) * h * bpp)
            bench(f"{tag}_norm_gate_up", lambda: lib.rms_norm_quantized_matmul_swiglu(xh, nw, 1e-6, *W["g"], *W["u"]),
                  4 * M * ff * h, 2 * ff * h * bpp)
    # attention regions: prefill prologue + sdpa (two launches), decode fused prologue + attention
    D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    kc = torch.randn(Hkv, cfg.max_len, D, device="cuda").to(torch.bfloat16)
    vc = torch.randn(Hkv, cfg.max_len, D, device="cuda").to(torch.bfloat16)
    qn = torch.ones(D, device="cuda", dtype=torch.bfloat16)
    sc = 1.0 / math.sqrt(D)
    qp = torch.randn(PROMPT, Hq * D, device="cuda").to(torch.bfloat16)
    kp = torch.randn(PROMPT, Hkv * D, device="cuda").to(torch.bfloat16)
    vp = torch.randn(PROMPT, Hkv * D, device="cuda").to(torch.bfloat16)
    qh = torch.empty(Hq, PROMPT, D, device="cuda", dtype=torch.bfloat16)
    bench("prefill_qk_norm_rope_cache", lambda: lib.qk_norm_rope_cache(
        qp, kp, vp, qn, qn, cfg.eps, qh, kc, vc, n_heads=Hq, n_kv_heads=Hkv, offset=0, rope_base=cfg.rope_theta),
        0, 2 * PROMPT * (Hq + 3 * Hkv) * D * 2)
    bench("prefill_sdpa", lambda: lib.sdpa(qh[None], kc[None, :, :PROMPT], vc[None, :, :PROMPT], scale=sc,
                                           causal=True, q_offset=0, out_layout="blhd"),
          2 * Hq * PROMPT * PROMPT * D, 0)
    bench("decode_attention", lambda: lib.qk_norm_rope_sdpa_decode(
        qp[:1], kp[:1], vp[:1], qn, qn, cfg.eps, kc, vc, n_heads=Hq, n_kv_heads=Hkv, offset=PROMPT,
        rope_base=cfg.rope_theta, scale=sc), 0, 2 * (PROMPT + 1) * Hkv * D * 2)
    # mlx-whisper encoder conv stem (fp16, 8 x 3000 frames): conv1 128 -> 1280 (k3 s1),
    # conv2 1280 -> 1280 (k3 s2), each with its bias and GELU
    xw = torch.randn(8, 3000, 128, device="cuda").to(torch.float16)
    w1 = (torch.randn(1280, 3, 128, device="cuda") / 20).to(torch.float16)
    w2 = (torch.randn(1280, 3, 1280, device="cuda") / 60).to(torch.float16)
    bw = torch.zeros(1280, device="cuda", dtype=torch.float16)
    h1 = lib.conv1d(xw, w1, bw, stride=1, padding=1, act=1)
    bench("whisper_conv1", lambda: lib.conv1d(xw, w1, bw, stride=1, padding=1, act=1), 2 * 8 * 3000 * 1280 * 3 * 128,
          8 * 3000 * (128 + 1280) * 2)
    bench("whisper_conv2", lambda: lib.conv1d(h1, w2, bw, stride=2, padding=1, act=1), 2 * 8 * 1500 * 1280 * 3 * 1280,
          8 * (3000 + 1500) * 1280 * 2)
    # the elementwise and normalisation regions at the other targets' sizes (HBM-bound)
    xl = torch.randn(8 * 2048, 4096, device="cuda").to(torch.bfloat16)
    wl = torch.ones(4096, device="cuda", dtype=torch.bfloat16)
    bench("llama_rms_norm", lambda: lib.rms_norm(xl, wl, 1e-5), 0, 2 * xl.numel() * 2)
    xr = torch.randn(8, 32, 2048, 128, device="cuda").to(torch.bfloat16)
    bench("llama_rope", lambda: lib.rope(xr, 128, base=5e5, offset=0), 0, 2 * xr.numel() * 2)
    gl = torch.randn(8 * 2048, 14336, device="cuda").to(torch.bfloat16)
    ul = torch.randn(8 * 2048, 14336, device="cuda").to(torch.bfloat16)
    bench("llama_swiglu", lambda: lib.swiglu(gl, ul), 0, 3 * gl.numel() * 2)
    del gl, ul
    xln = torch.randn(8 * 1500, 1280, device="cuda").to(torch.float16)
    wln = torch.ones(1280, device="cuda", dtype=torch.float16)
    bln = torch.zeros(1280, device="cuda", dtype=torch.float16)
    bench("whisper_layer_norm", lambda: lib.layer_norm(xln, wln, bln, 1e-5), 0, 2 * xln.numel() * 2)
    # Mamba-370m layer at 512 steps (d_inner 2048, d_state 16, fp16): depthwise causal conv + selective scan
    Lm, Dm, NSm = 512, 2048, 16
    xm_ = torch.randn(Lm, Dm, device="cuda").to(torch.float16)
    dtm = torch.randn(Lm, Dm, device="cuda").to(torch.float16)
    zm = torch.randn(Lm, Dm, device="cuda").to(torch.float16)
    Bm_ = torch.randn(Lm, NSm, device="cuda").to(torch.float16)
    Cm_ = torch.randn(Lm, NSm, device="cuda").to(torch.float16)
    Am = -torch.arange(1, NSm + 1, device="cuda", dtype=torch.float32).repeat(Dm, 1)
    dtb = torch.zeros(Dm, device="cuda")
    Dv = torch.ones(Dm, device="cuda")
    cw = (torch.randn(Dm, 4, device="cuda") / 2).to(torch.float16)
    bench("mamba_conv1d", lambda: lib.causal_conv1d(xm_, cw, None), 0, 2 * Lm * Dm * 2)
    bench("mamba_scan", lambda: lib.mamba_scan(xm_, dtm, dtb, Am, Bm_, Cm_, Dv, zm), 0,
          (4 * Lm * Dm + 2 * Lm * NSm) * 2)
    # output-diff reduction of the verification ladder on Llama-size hidden states ([8, 2048, 4096] bf16)
    da = torch.randn(8 * 2048 * 4096, device="cuda").to(torch.bfloat16)
    db = (da.float() + 1e-3).to(torch.bfloat16)
    st_ = torch.zeros(C.sizeof(lib.DiffStats), dtype=torch.uint8, device="cuda")
    bench("diff_reduce", lambda: lib.diff_reduce(da, db, rtol=1e-2, atol=1e-2, stats=st_), 0, 2 * da.numel() * 2)
    # attention at the other targets' sizes: mlx-whisper encoder (8 clips, 20 heads, 1500 frames,
    # head_dim 64, non-causal) and Llama-3-8B prefill (8 x 2048 tokens, 32/8 heads, causal)
    qw_ = torch.randn(8, 20, 1500, 64, device="cuda").to(torch.float16)
    bench("whisper_sdpa", lambda: lib.sdpa(qw_, qw_, qw_, scale=0.125, causal=False), 4 * 8 * 20 * 1500 * 1500 * 64, 0)
    ql_ = torch.randn(8, 32, 2048, 128, device="cuda").to(torch.bfloat16)
    kl_ = torch.randn(8, 8, 2048, 128, device="cuda").to(torch.bfloat16)
    bench("llama_sdpa", lambda: lib.sdpa(ql_, kl_, kl_, scale=1.0 / math.sqrt(128), causal=True),
          2 * 8 * 32 * 2048 * 2048 * 128, 0)
    # Llama-3-8B 8-bit projections at batch 8 x 2048 (tp = 1): the prefill qmm at large M
    if not only or any(k.startswith("llama_qmm") for k in only):
        TL = 8 * 2048
        xl_ = torch.randn(TL, 4096, device="cuda").to(torch.bfloat16)
        gl_, ul_ = (workload.random_quantized(14336, 4096, bits=8, generator=g) for _ in range(2))
        dl_ = workload.random_quantized(4096, 14336, bits=8, generator=g)
        al_ = torch.empty(TL, 14336, device="cuda", dtype=torch.bfloat16)
        yl_ = torch.empty(TL, 4096, device="cuda", dtype=torch.bfloat16)
        bench("llama_qmm_gate_up_swiglu", lambda: lib.quantized_matmul_swiglu(xl_, *gl_, *ul_, bits=8, out=al_),
              2 * TL * 2 * 14336 * 4096, 0)
        bench("llama_qmm_down", lambda: lib.quantized_matmul(al_, *dl_, bits=8, out=yl_), 2 * TL * 4096 * 14336, 0)
    # mlx-whisper encoder MLP (fp16, 8 clips x 1500 frames): fc1 1280 -> 5120 + GELU, fc2 5120 -> 1280
    xm = torch.randn(8 * 1500, 1280, device="cuda").to(torch.float16)
    f1 = (torch.randn(5120, 1280, device="cuda") / 36).to(torch.float16)
    f2 = (torch.randn(1280, 5120, device="cuda") / 72).to(torch.float16)
    b1 = torch.zeros(5120, device="cuda", dtype=torch.float16)
    hm = lib.linear(xm, f1, b1, act=1)
    bench("whisper_fc1_gelu", lambda: lib.linear(xm, f1, b1, act=1), 2 * 12000 * 5120 * 1280,
          (12000 * (1280 + 5120) + 5120 * 1280) * 2)
    bench("whisper_fc2", lambda: lib.linear(hm, f2, bw, act=0), 2 * 12000 * 1280 * 5120,
          (12000 * (1280 + 5120) + 5120 * 1280) * 2)
    print(json.dumps({"kernels": rows, "peaks": peaks}), flush=True)
    return 0


# ------------------------------------------------------------------ main
LLAMA_B, LLAMA_L = 8, 2048


def run_llama_tp(args):
    """Llama-3-8B 8-bit, batch 8 x prefill 2048, tensor-parallel over the
    ranks (one shard per GPU, NCCL all-reduce after o_proj and down).

      value  prompt tokens/s of the whole job (8 x 2048 / forward time),
             CUDA events around K forwards, max over ranks
      e2e    the same with pinned host tokens copied in and rank 0's
             last-position logits read back every forward
      roofline  the whole forward per GPU: its algorithmic FLOPs / tp over
             the forward time, against the sustained bf16 peak; plus the
             gate/up qmm+SwiGLU (the largest kernel) timed alone."""
    import torch

    from metal_autotune_b200 import build, lib, workload
    from metal_autotune_b200.targets import llama_tp
    build.build_library()
    rank, world, local = dist_setup()
    cfg = llama_tp.LLAMA3_8B if args.config == "llama3_8b_tp" else llama_tp.TINY
    B, L = (LLAMA_B, LLAMA_L) if cfg.layers == 32 else (2, 128)
    comm = llama_tp.ProcessGroupComm() if world > 1 else llama_tp.LocalComm()
    t0 = time.time()
    model = llama_tp.LlamaTP(cfg, world, [rank], comm, seed=0, device="cuda")
    torch.cuda.synchronize()
    log(f"rank {rank}: built Llama shard {rank}/{world} ({cfg.layers} layers) in {time.time() - t0:.1f}s, "
        f"{torch.cuda.memory_allocated() / 2**30:.1f} GiB")
    tokens = workload.seeded_tokens((B, L), 0, cfg.vocab, seed=0)
    host_tokens = tokens.cpu().pin_memory()
    host_logits = torch.empty(B, cfg.vocab, dtype=torch.bfloat16).pin_memory()
    out = {}

    def step():
        out["logits"] = model(tokens)

    def e2e_step():
        tokens.copy_(host_tokens, non_blocking=True)
        out["logits"] = model(tokens)
        host_logits.copy_(out["logits"], non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    calls0 = lib.CALLS[0]
    with ClockSampler(local) as clk:
        ms_total = time_region(step, args.steps, world)
        ms_e2e_total = time_region(e2e_step, args.steps, world)
    launches = lib.CALLS[0] - calls0
    ms = max_over_ranks(ms_total / args.steps, world)
    ms_e2e = max_over_ranks(ms_e2e_total / args.steps, world)
    status = lib.device_status(clear=True)
    if status != 0:
        raise RuntimeError(f"device status {status:#x}: a kernel's bounded wait expired")
    if not bool(torch.isfinite(out["logits"].float()).all()):
        raise RuntimeError("non-finite logits")

    # the largest kernel alone: gate/up qmm + SwiGLU of layer 0 on this shard
    peaks = measured_peaks()
    sl = model.shards[0].layers[0]
    xn = torch.randn(B * L, cfg.hidden, device="cuda", dtype=torch.bfloat16)
    act = torch.empty(B * L, sl.gate[0].shape[0], device="cuda", dtype=torch.bfloat16)
    run = lambda: lib.quantized_matmul_swiglu(xn, *sl.gate, *sl.up, group_size=cfg.group, bits=cfg.bits, out=act)
    for _ in range(3):
        run()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(10):
        run()
    ev[1].record()
    torch.cuda.synchronize()
    k_ms = ev[0].elapsed_time(ev[1]) / 10
    k_flops = 2 * B * L * 2 * sl.gate[0].shape[0] * cfg.hidden
    fwd_flops = llama_tp.forward_flops(cfg, B, L)
    sustained = peaks["bf16_tflops_sustained"] or peaks["bf16_tflops"]
    achieved = fwd_flops / world / (ms / 1e3) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": sustained, "unit": "TFLOP/s",
            "frac": round(achieved / sustained, 4), "traffic": None, "peak_source": f"{peaks['source']} sustained",
            "what": "whole forward per GPU (algorithmic FLOPs / tp / forward time)",
            "forward_tflop": round(fwd_flops / 1e12, 3),
            "gate_up_swiglu": {"ms": round(k_ms, 4), "tflops": round(k_flops / (k_ms / 1e3) / 1e12, 2),
                               "frac_of_burst": round(k_flops / (k_ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4),
                               "M": B * L, "N": 2 * sl.gate[0].shape[0], "K": cfg.hidden}}
    if rank != 0:
        barrier(world)
        return 0
    line = {
        "metric": "Llama-3-8B-8bit prefill tok/s (batch 8 x 2048), tensor-parallel",
        "value": round(B * L / (ms / 1e3), 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "llama3_8b_prefill_8x2048" if cfg.layers == 32 else "llama_tiny",
                   "model": "Llama-3-8B 8-bit affine g64, random init" if cfg.layers == 32 else "tiny Llama",
                   "batch": B, "prompt_tokens": L, "parallelism": f"tp{world}",
                   "collective": "NCCL all-reduce (bf16) after o_proj and down, all-gather of lm_head rows",
                   "l2": "inputs larger than L2 (8.5 GB of packed weights per forward / tp)"},
        "e2e": {"value": round(B * L / (ms_e2e / 1e3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": B * L * 4, "d2h_bytes_per_step": B * cfg.vocab * 2},
        "roofline": roof, "clocks": clk.summary(), "gpu_launches": launches,
        "gpu_launches_note": "libmt entry-point calls in the timed region; a blocked prefill qmm call issues "
                             "one launch per L2-sized block, so kernel launches are at least this many",
    }
    barrier(world)
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="default 300 (Qwen3 request), 5 (Llama forward)")
    ap.add_argument("--warmup", type=int, default=None, help="default 10 (Qwen3 request), 3 (Llama forward)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="qwen3_4b", choices=["qwen3_4b", "qwen3_tiny", "llama3_8b_tp", "llama_tiny_tp"],
                    help="llama*_tp: Llama-3-8B 8-bit prefill 8 x 2048, tensor-parallel over the ranks")
    ap.add_argument("--mode", default="request", choices=["request", "kernels"])
    ap.add_argument("--only", default="", help="kernels mode: comma-separated kernel names")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--launch-list", action="store_true",
                    help="replay the request W + K times, the K inside an NVTX range 'request', and exit "
                         "(for ncu --nvtx --nvtx-include request/)")
    args = ap.parse_args()
    llama = args.config.startswith("llama")
    if args.steps is None:
        args.steps = 5 if llama else 300
    if args.warmup is None:
        args.warmup = 3 if llama else 10
    if args.warmup < 3 and args.mode == "request":
        args.warmup = 3

    if args.config.startswith("llama"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the Llama TP line has no CPU arm; the default "
                              "Qwen3 line carries the reference arm"}), flush=True)
            return 0
        return run_llama_tp(args)
    from metal_autotune_b200.targets import qwen3
    cfg = qwen3.QWEN3_4B if args.config == "qwen3_4b" else qwen3.TINY

    if args.impl == "reference":
        return run_reference(args, cfg)

    import torch

    from metal_autotune_b200 import build, lib
    build.build_library()
    rank, world, local = dist_setup()
    if args.mode == "kernels":
        return run_kernels(args, cfg)

    req = Request(cfg)
    req.capture()
    for _ in range(args.warmup):
        req.replay()
    torch.cuda.synchronize()
    if args.launch_list:
        torch.cuda.nvtx.range_push("request")
        for _ in range(args.steps):
            req.replay()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        log(f"launch list: {args.steps} request(s) of {req.launches_per_step} launches")
        return 0
    with ClockSampler(local) as clk:
        ms_total = time_region(req.replay, args.steps, world)
        ms_e2e_total = time_region(req.e2e_step, args.steps, world)
    ms = max_over_ranks(ms_total / args.steps, world)
    ms_e2e = max_over_ranks(ms_e2e_total / args.steps, world)
    status = lib.device_status(clear=True)
    if status != 0:
        raise RuntimeError(f"device status {status:#x}: a kernel's bounded wait expired")
    peaks = measured_peaks()
    roof = qmm_roofline(req, peaks)
    wbytes, ebytes = packed_weight_bytes(cfg)
    roof["request_floor_ms"] = round(max(request_flops(cfg) / (peaks["bf16_tflops"] * 1e12),
                                         (2 * wbytes + ebytes) / (peaks["hbm_gbs"] * 1e9)) * 1e3, 4)
    prof = ROOT / "profiles" / "qmm_tc_prefill_qwen3_4b.traffic.json"
    if prof.exists():
        roof["traffic"] = json.loads(prof.read_text()).get("bytes_per_launch")
        roof["traffic_note"] = json.loads(prof.read_text()).get("note")
    if rank != 0:
        barrier(world)
        return 0
    line = {
        "metric": METRIC, "value": round(PROMPT * world / (ms / 1e3), 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "qwen3_4b_prefill_128+decode_1" if cfg.layers == 36 else "qwen3_tiny",
                   "model": f"Qwen3-{'4B' if cfg.layers == 36 else 'tiny'} 4-bit affine g64, random init",
                   "prompt_tokens": PROMPT, "decode_tokens": 1, "batch": 1,
                   "l2": "inputs larger than L2 (2.3 GB packed weights per request)",
                   "parallelism": f"replicas x{world}", "graph": "one CUDA graph per request"},
        "e2e": {"value": round(PROMPT * world / (ms_e2e / 1e3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": PROMPT * 4, "d2h_bytes_per_step": 12},
        "roofline": roof, "clocks": clk.summary(),
        "gpu_launches": int(req.launches_per_step * args.steps * 2),
        "launches_per_step": req.launches_per_step,
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(cfg, os.cpu_count() or 1)
    barrier(world)
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        del req
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
