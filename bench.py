"""Benchmark of the region hot path on B200: Qwen3-4B-4bit prefill-128 + 1 decode.

One step = one request as the reference's workload defines it
(models/workloads/qwen3_4b_prefill_128.yaml; autotuner_runtime/inference.py:
131-156): from an empty KV cache, prefill 128 prompt tokens, pick the next
token, run one decode step, pick again. Every region runs through the bundle's
wrappers (try_call -> libmt.so), strict mode on (a fallback raises). The
request is captured once in a CUDA graph and replayed. Timed regions go
through the timing harness (autotuner_runtime.measure: CUDA events on the
launching stream, device synchronised on both sides).

  value  prompt tokens/s (128 / request time) with tokens already on the
         device, CUDA events around K replays, max over ranks, x ranks
         (independent replicas: the path does not shard).
  e2e    the same metric through the public call with host buffers: pinned
         host tokens -> device, replay, read back the two picked tokens and
         the logprob, every step.
  roofline  the dominant kernel (tcgen05 prefill qmm, all 144 launches of
         the request's prefill) timed on its own stream with CUDA events:
         algorithmic FLOPs / time vs the measured bf16 peak.
  cpu_baseline  the oracle restatement (C, OpenMP, all host threads) running
         one whole request (36 layers, prefill 128 + decode 1, lm_head) on
         this model's own weights, copied to the host.
  llama_tp  the Llama-3-8B 8-bit prefill forward (batch 8 x 2048),
         tensor-parallel over the same ranks (tp = N, NCCL all-reduce after
         o_proj and down): ms per forward, whole-job tok/s, per-GPU TFLOP/s
         and the share of the forward the all-reduces take alone.

--impl reference times the CPU implementation of the path (the oracle port;
the reference's own path is MLX on Apple GPUs, unavailable here): whole
requests on the same weights, as many as fit a wall-clock cap. --mode
kernels prints per-region kernel timings (profiling entry). --config
llama3_8b_tp prints the Llama line alone.
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
    """nvidia-smi samples every 50 ms while the measurement runs. The caller
    marks the timed region (mark_start/mark_end); the summary gives the
    median SM clock and the throttle reasons over the whole sampled window
    (the timed region plus the untimed replays around it) and how many
    samples fell inside the timed region itself."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, period_ms: int = 50):
        self.idx = device_index
        self.period_ms = period_ms
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.timed = [None, None]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def wait_first_sample(self, timeout_s: float = 5.0):
        """Block until nvidia-smi has reported once: it takes a few hundred
        ms to start, longer than a short timed region (5 tensor-parallel
        forwards at tp 8 take under 0.5 s)."""
        t_end = time.time() + timeout_s
        while self.proc is not None and not self.lines and time.time() < t_end:
            time.sleep(0.01)

    def mark_start(self):
        self.timed[0] = time.time()

    def mark_end(self):
        self.timed[1] = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sms, mx, reasons, inside = [], None, set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        t0, t1 = self.timed
        for ts, ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 10:
                continue
            try:
                sm = float(p[2])
                mx = float(p[3])
            except ValueError:
                continue
            sms.append(sm)
            if t0 is not None and t1 is not None and t0 - self.period_ms / 1e3 <= ts <= t1 + self.period_ms / 1e3:
                inside += 1
            for name, v in zip(names, p[6:10]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sms), "samples_in_timed_region": inside,
                "period_ms": self.period_ms,
                "window": "the timed region plus untimed replays of the same step around it"}


def soak(fn, seconds: float):
    """Untimed repetitions of fn for about `seconds` (clock samples around the timed region)."""
    import torch
    t_end = time.time() + seconds
    while time.time() < t_end:
        for _ in range(8):
            fn()
        torch.cuda.synchronize()


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
        before = lib.kernel_launches()
        with torch.cuda.graph(self.graph):
            self.out = self.eager()
            # the three results in one buffer, so e2e reads them back with one copy
            self.res_dev = torch.cat([self.out[0].view(1), self.out[1].view(1),
                                      self.out[2].view(torch.int32).view(1)])
        self.launches_per_step = lib.kernel_launches() - before

    def replay(self):
        self.graph.replay()

    def e2e_step(self):
        """Public-API request with host buffers: H2D tokens, run, D2H result."""
        torch = self.torch
        self.tokens.copy_(self.host_tokens, non_blocking=True)
        self.graph.replay()
        self.host_out.copy_(self.res_dev, non_blocking=True)


def time_region(fn, steps, world, stream=None):
    """Device milliseconds of `steps` calls of fn (autotuner_runtime.measure:
    CUDA events on the launching stream, synchronised on both sides), between
    barriers of all ranks."""
    from metal_autotune_b200.autotuner_runtime import measure
    barrier(world)
    ms = measure.time_steps(fn, steps, stream)
    barrier(world)
    return ms


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
        from metal_autotune_b200.autotuner_runtime import measure
        ms = measure.time_steps(g.replay, reps, stream=s) / reps
    launches = 4 * len(layers)
    flops = request_flops(cfg)
    achieved = flops / (ms / 1e3) / 1e12
    peak = peaks["bf16_tflops"]
    return {"bound": "tensor", "kernel": "qmm_tc_kernel (prefill qkv/o/gate_up/down, 144 launches)",
            "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "peak_source": f"{peaks['source']} bf16_tflops (burst)", "ms_all_launches": round(ms, 4),
            "us_per_launch": round(ms * 1e3 / launches, 2), "traffic": None}


# ------------------------------------------------------------------ CPU side
def qwen3_config_record(cfg, world):
    """The `config` of the Qwen3 line, identical in both arms."""
    return {"workload": "qwen3_4b_prefill_128+decode_1" if cfg.layers == 36 else "qwen3_tiny",
            "model": f"Qwen3-{'4B' if cfg.layers == 36 else 'tiny'} 4-bit affine g64, random init (seed 0)",
            "prompt_tokens": PROMPT, "decode_tokens": 1, "batch": 1,
            "l2": "inputs larger than L2 (2.3 GB packed weights per request)",
            "parallelism": f"replicas x{world}"}


def host_weights(model):
    """The oracle's host copy of a Qwen3 model's weights (bf16 values as fp32)."""
    from oracle import qwen3_ref
    return qwen3_ref.model_weights(model)


def cpu_request(cfg, weights, tokens_np, threads, force_token0=None):
    """One whole request on the oracle (C, OpenMP `threads`): prefill, pick,
    one decode step, pick, all 36 layers and the lm_head. Returns (seconds,
    RequestResult)."""
    os.environ["OMP_NUM_THREADS"] = str(threads)
    from oracle import qwen3_ref
    from oracle import ref as R
    R.lib()
    t0 = time.perf_counter()
    res = qwen3_ref.request(cfg, weights, tokens_np, force_token0=force_token0)
    return time.perf_counter() - t0, res


def cpu_baseline(cfg, model, tokens, threads, gpu=None):
    """The oracle timed on one whole request of this model (its weights copied
    to the host): about 20 s of CPU work on 16 cores. With gpu = (first pick,
    second pick, decode logits) of the GPU request, the oracle decodes the
    GPU's first pick and the two decode logits rows are compared."""
    import numpy as np
    w = host_weights(model)
    secs, res = cpu_request(cfg, w, tokens.cpu().numpy(), threads,
                            force_token0=None if gpu is None else int(gpu[0]))
    out = {"value": round(PROMPT / secs, 3), "unit": "tok/s", "cores": threads, "kind": "port",
           "sample": (f"one whole request (prefill {PROMPT} + decode 1, all {cfg.layers} layers and the lm_head) "
                      f"of this model's weights on the oracle C restatement, OpenMP {threads} threads: "
                      f"{secs:.2f} s; MLX CPU unavailable on this box")}
    if gpu is not None:
        t0, t1, lg = gpu
        ref = res.decode_logits.astype(np.float64)
        got = np.asarray(lg, np.float64).reshape(-1)
        diff = np.abs(got - ref)
        out["check"] = {"first_pick_equal": int(t0) == res.token0,
                        "decode_logits_rel_l2": float(np.linalg.norm(got - ref) / np.linalg.norm(ref)),
                        "decode_logits_max_abs_over_max": float(diff.max() / np.abs(ref).max()),
                        "second_pick_gap_to_oracle_max": float(ref.max() - ref[int(t1)]),
                        "second_pick_within_2x_max_abs": bool(ref.max() - ref[int(t1)] <= 2 * diff.max())}
    return out


def run_reference(args, cfg):
    """The CPU implementation of the path (the oracle port; the reference's own
    path is MLX on an Apple GPU, unavailable on this box), on the same seeded
    weights and prompt as the GPU arm, whole requests on all host threads.
    Rank 0 alone runs it; other ranks exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch

    from metal_autotune_b200 import workload
    from metal_autotune_b200.targets import qwen3
    threads = os.cpu_count() or 1
    # the same seeded weights as the GPU arm: generated where that arm generates them, then copied out
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    model = qwen3.build(cfg, seed=0, device=dev)
    weights = host_weights(model)
    del model
    if dev == "cuda":
        torch.cuda.empty_cache()
    tokens = workload.seeded_tokens((PROMPT,), 0, cfg.vocab, seed=0, device="cpu").numpy()
    secs, times = [], []
    t_start = time.time()
    for _ in range(max(1, args.steps)):
        dt, _ = cpu_request(cfg, weights, tokens, threads)
        times.append(dt)
        if time.time() - t_start + dt > REFERENCE_WALL_CAP_S:
            break
    ms = statistics.median(times) * 1e3
    v = PROMPT / (ms / 1e3)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": len(times), "steps_requested": args.steps, "warmup": 0, "warmup_requested": args.warmup,
            "ms_per_step": round(ms, 3), "ms_per_step_all": [round(t * 1e3, 1) for t in times],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": qwen3_config_record(cfg, args.gpus),
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"each step one whole request (prefill {PROMPT} + decode 1, all "
                                       f"{cfg.layers} layers and the lm_head) on the oracle C restatement, "
                                       f"OpenMP {threads} threads; {len(times)} of {args.steps} requested steps "
                                       f"measured (wall cap {REFERENCE_WALL_CAP_S} s); no warm-up (no caches "
                                       "or compilation to warm); the reference's own path is MLX on an Apple "
                                       "GPU (unavailable on this box), so the oracle port is timed"},
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


def llama_tp_record(cfg, B, L, steps, warmup, rank, world, local, overlap=True):
    """Llama-3-8B 8-bit prefill forward (batch B x L), tensor-parallel over the
    `world` ranks (one shard per GPU, NCCL all-reduce after o_proj and down).
    Every rank takes the same collective steps; times are max over ranks.

      ms / tok_s    the forward (CUDA events around `steps` forwards)
      e2e           the same with pinned host tokens copied in and the gathered
                    last-position logits read back every forward
      per_gpu_tflops  algorithmic FLOPs / tp / forward time, vs the sustained peak
      allreduce     the forward's 2 x layers all-reduces of [B*L, hidden] bf16
                    timed alone (same sizes, same communicator): their share
                    of the forward
      gate_up_swiglu  the largest kernel alone (layer 0's shard)"""
    import torch

    from metal_autotune_b200 import lib, workload
    from metal_autotune_b200.targets import llama_tp
    comm = llama_tp.ProcessGroupComm() if world > 1 else llama_tp.LocalComm()
    t0 = time.time()
    model = llama_tp.LlamaTP(cfg, world, [rank], comm, seed=0, device="cuda", overlap=overlap)
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

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    calls0 = lib.kernel_launches()
    with ClockSampler(local) as clk:
        clk.wait_first_sample()
        clk.mark_start()
        ms_total = time_region(step, steps, world)
        clk.mark_end()
        ms_e2e_total = time_region(e2e_step, steps, world)
    launches = lib.kernel_launches() - calls0
    ms = max_over_ranks(ms_total / steps, world)
    ms_e2e = max_over_ranks(ms_e2e_total / steps, world)
    status = lib.device_status(clear=True)
    if status != 0:
        raise RuntimeError(f"device status {status:#x}: a kernel's bounded wait expired")
    if not bool(torch.isfinite(out["logits"].float()).all()):
        raise RuntimeError("non-finite logits")

    # the forward's all-reduces alone: 2 per layer of the [B*L, hidden] bf16 partial
    ar_ms = 0.0
    if world > 1:
        buf = torch.randn(B * L, cfg.hidden, device="cuda").to(torch.bfloat16)
        n_ar = 2 * cfg.layers
        for _ in range(2):
            comm.all_reduce([buf])
        ar_ms = max_over_ranks(time_region(lambda: [comm.all_reduce([buf]) for _ in range(n_ar)], 1, world), world)
        del buf

    # the largest kernel alone: gate/up qmm + SwiGLU of layer 0 on this shard
    from metal_autotune_b200.autotuner_runtime import measure
    peaks = measured_peaks()
    sl = model.shards[0].layers[0]
    xn = torch.randn(B * L, cfg.hidden, device="cuda", dtype=torch.bfloat16)
    act = torch.empty(B * L, sl.gate[0].shape[0], device="cuda", dtype=torch.bfloat16)
    run = lambda: lib.quantized_matmul_swiglu(xn, *sl.gate, *sl.up, group_size=cfg.group, bits=cfg.bits, out=act)
    for _ in range(3):
        run()
    k_ms = measure.time_steps(run, 10) / 10
    k_flops = 2 * B * L * 2 * sl.gate[0].shape[0] * cfg.hidden
    fwd_flops = llama_tp.forward_flops(cfg, B, L)
    sustained = peaks["bf16_tflops_sustained"] or peaks["bf16_tflops"]
    achieved = fwd_flops / world / (ms / 1e3) / 1e12
    rec = {"tp": world, "nccl_ranks": world if world > 1 else 0, "ms_per_forward": round(ms, 4),
           "allreduce_overlap": bool(overlap and world > 1),
           "steps": steps, "warmup": warmup, "tok_s": round(B * L / (ms / 1e3), 2),
           "e2e_tok_s": round(B * L / (ms_e2e / 1e3), 2),
           "e2e_bytes": {"h2d_per_step": B * L * 4, "d2h_per_step": B * cfg.vocab * 2},
           "forward_tflop": round(fwd_flops / 1e12, 3), "per_gpu_tflops": round(achieved, 2),
           "frac_of_sustained": round(achieved / sustained, 4),
           "peak": {"value": sustained, "unit": "TFLOP/s", "source": f"{peaks['source']} sustained bf16"},
           "allreduce": {"calls_per_forward": 2 * cfg.layers if world > 1 else 0,
                         "bytes_each": B * L * cfg.hidden * 2, "ms_alone": round(ar_ms, 4),
                         "share_of_forward": round(ar_ms / ms, 4),
                         "what": "NCCL bf16 all-reduce of the row-parallel partial after o_proj and down"},
           "gate_up_swiglu": {"ms": round(k_ms, 4), "tflops": round(k_flops / (k_ms / 1e3) / 1e12, 2),
                              "frac_of_burst": round(k_flops / (k_ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4),
                              "M": B * L, "N": 2 * sl.gate[0].shape[0], "K": cfg.hidden},
           "clocks": clk.summary(), "gpu_launches": launches,
           "config": {"workload": "llama3_8b_prefill_8x2048" if cfg.layers == 32 else "llama_tiny",
                      "model": "Llama-3-8B 8-bit affine g64, random init (seed 0)" if cfg.layers == 32
                      else "tiny Llama", "batch": B, "prompt_tokens": L, "parallelism": f"tp{world}",
                      "scaling": "strong"}}
    del model, out
    torch.cuda.empty_cache()
    return rec


def llama_launch_list(cfg, B, L, steps, warmup, rank, world):
    """W forwards, then K inside the NVTX range 'forward' (for ncu --nvtx
    --nvtx-include forward/), and exit."""
    import torch

    from metal_autotune_b200 import workload
    from metal_autotune_b200.targets import llama_tp
    comm = llama_tp.ProcessGroupComm() if world > 1 else llama_tp.LocalComm()
    model = llama_tp.LlamaTP(cfg, world, [rank], comm, seed=0, device="cuda")
    tokens = workload.seeded_tokens((B, L), 0, cfg.vocab, seed=0)
    for _ in range(warmup):
        model(tokens)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("forward")
    for _ in range(steps):
        model(tokens)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    log(f"launch list: {steps} forward(s)")
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def run_llama_tp(args):
    """The Llama-3-8B tensor-parallel forward as its own JSON line."""
    from metal_autotune_b200 import build
    from metal_autotune_b200.targets import llama_tp
    build.build_library()
    rank, world, local = dist_setup()
    cfg = llama_tp.LLAMA3_8B if args.config == "llama3_8b_tp" else llama_tp.TINY
    B, L = (LLAMA_B, LLAMA_L) if cfg.layers == 32 else (2, 128)
    if args.launch_list:
        return llama_launch_list(cfg, B, L, args.steps, args.warmup, rank, world)
    rec = llama_tp_record(cfg, B, L, args.steps, args.warmup, rank, world, local, overlap=not args.no_overlap)
    if rank == 0:
        line = {"metric": "Llama-3-8B-8bit prefill tok/s (batch 8 x 2048), tensor-parallel",
                "value": rec["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": rec["ms_per_forward"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": rec["config"],
                "e2e": {"value": rec["e2e_tok_s"], "unit": "tok/s",
                        "h2d_bytes_per_step": rec["e2e_bytes"]["h2d_per_step"],
                        "d2h_bytes_per_step": rec["e2e_bytes"]["d2h_per_step"]},
                "roofline": {"bound": "tensor", "achieved": rec["per_gpu_tflops"], "peak": rec["peak"]["value"],
                             "unit": "TFLOP/s", "frac": rec["frac_of_sustained"], "traffic": None,
                             "what": "whole forward per GPU (algorithmic FLOPs / tp / forward time)"},
                "clocks": rec["clocks"], "gpu_launches": rec["gpu_launches"], "llama_tp": rec}
    barrier(world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------ other targets
WHISPER_BATCH, MAMBA_TOKENS = 8, 512


FORWARDS_PER_GRAPH = {"mlp": 16}  # launch-bound targets: forwards per timed graph replay


class ModelStep:
    """A bundle-applied target, its seeded device input and pinned host
    copies, one forward captured in a CUDA graph."""

    def __init__(self, kind: str, tiny: bool = False, backend: str = "replay"):
        import torch

        from metal_autotune_b200 import lib, workload
        from metal_autotune_b200.autotuner_runtime.apply import apply
        os.environ["MT_STRICT_REGIONS"] = "1"
        self.torch, self.kind = torch, kind
        bdir = ROOT / "metal_autotune_b200" / "bundles"
        sfx = "_graph" if backend == "graph" else ""
        if backend == "graph" and kind == "mamba":
            raise SystemExit("the graph backend has no Mamba bundle (the replay bundle serves it)")
        if kind == "whisper":
            from metal_autotune_b200.targets import whisper
            self.cfg = whisper.TINY if tiny else whisper.WHISPER_TURBO
            model = whisper.build(self.cfg, seed=0)
            g = torch.Generator(device="cuda").manual_seed(0)
            self.x = torch.randn(WHISPER_BATCH, self.cfg.frames, self.cfg.n_mels, generator=g,
                                 device="cuda").to(torch.float16)
            self.model = apply(model, bdir / (("whisper_tiny" if tiny else "whisper_turbo") + sfx))
            self.flops = whisper.encoder_flops(self.cfg, WHISPER_BATCH)
            self.units = WHISPER_BATCH * self.cfg.frames
        elif kind == "mamba":
            from metal_autotune_b200.targets import mamba
            self.cfg = mamba.TINY if tiny else mamba.MAMBA_370M
            model = mamba.build(self.cfg, seed=0)
            self.x = workload.seeded_tokens((MAMBA_TOKENS,), 0, self.cfg.vocab, seed=0)
            self.model = apply(model, bdir / ("mamba_tiny" if tiny else "mamba_370m"))
            self.flops = mamba.prefill_flops(self.cfg, MAMBA_TOKENS)
            self.units = MAMBA_TOKENS
        else:
            from metal_autotune_b200.targets import tiny_mlp
            self.cfg = tiny_mlp.TINY_MLP
            model, self.x = tiny_mlp.build(self.cfg)
            self.model = apply(model, bdir / ("tiny_mlp" + sfx))
            self.flops = tiny_mlp.flops(self.cfg)
            self.units = 1
        self.raw = model
        self.host_x = self.x.cpu().pin_memory()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.model(self.x)
            self.model(self.x)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        before = lib.kernel_launches()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            out = self.model(self.x)
        self.launches_per_step = lib.kernel_launches() - before
        self.out = out[0] if isinstance(out, tuple) else out  # the pick for Mamba, the activations otherwise
        self.host_out = torch.empty_like(self.out, device="cpu").pin_memory()
        # A forward of a few microseconds replays faster on the GPU than the host can launch graphs, so
        # `replay` runs FORWARDS_PER_GRAPH complete forwards captured back to back in one graph (each
        # recomputed from the input), timing the device; e2e_step keeps one forward per call.
        self.per_replay = FORWARDS_PER_GRAPH.get(kind, 1)
        self.multi = None
        if self.per_replay > 1:
            self.multi = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.multi):
                for _ in range(self.per_replay):
                    self.model(self.x)

    def replay(self):
        (self.multi or self.graph).replay()

    def e2e_step(self):
        self.x.copy_(self.host_x, non_blocking=True)
        self.graph.replay()
        self.host_out.copy_(self.out, non_blocking=True)


def model_cpu_baseline(step, threads):
    """The oracle on a bounded sample of the same workload, on all host threads."""
    import numpy as np
    os.environ["OMP_NUM_THREADS"] = str(threads)
    from oracle import ref as R
    R.lib()
    if step.kind == "whisper":
        from oracle import whisper_ref
        cfg = step.cfg
        W = whisper_ref.encoder_weights(step.raw, n_blocks=1)
        mel = step.x[:1].float().cpu().numpy()
        t0 = time.perf_counter()
        x = whisper_ref.stem(cfg, W, mel)
        t_stem = time.perf_counter() - t0
        t0 = time.perf_counter()
        whisper_ref.block(cfg, W.blocks[0], x)
        t_block = time.perf_counter() - t0
        secs = WHISPER_BATCH * (t_stem + cfg.n_layer * t_block)
        sample = (f"the stem ({t_stem:.2f} s) and one block ({t_block:.2f} s) of one clip on the oracle C "
                  f"restatement, OpenMP {threads} threads, scaled to {WHISPER_BATCH} clips x {cfg.n_layer} blocks")
        return {"value": round(step.units / secs, 3), "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": sample}
    if step.kind == "mamba":
        from oracle import mamba_ref
        W = mamba_ref.model_weights(step.raw)
        t0 = time.perf_counter()
        mamba_ref.prefill(step.cfg, W, step.x.cpu().numpy())
        secs = time.perf_counter() - t0
        return {"value": round(MAMBA_TOKENS / secs, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"the whole prefill ({step.cfg.n_layer} layers, {MAMBA_TOKENS} tokens, lm_head) on the "
                          f"oracle C restatement, OpenMP {threads} threads: {secs:.2f} s"}
    m = step.raw
    xs = step.x.cpu().numpy()
    w1, b1 = m.l1.weight.cpu().numpy(), m.l1.bias.cpu().numpy()
    w2, b2 = m.l2.weight.cpu().numpy(), m.l2.bias.cpu().numpy()
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 2.0:
        R.gelu_mlp(xs, w1, b1, w2, b2)
        n += 1
    us = (time.perf_counter() - t0) / n * 1e6
    return {"value": round(us, 2), "unit": "us", "cores": threads, "kind": "port",
            "sample": f"{n} forwards of the oracle C restatement (OpenMP {threads} threads) in 2 s"}


MODEL_LINES = {
    "whisper_turbo": ("whisper", "Whisper-large-v3-turbo encoder mel frames/s (batch 8 x 3000 frames)", "frames/s",
                      True),
    "whisper_tiny": ("whisper", "Whisper encoder (tiny) mel frames/s", "frames/s", True),
    "mamba_370m": ("mamba", "Mamba-370m prefill tok/s (512 tokens)", "tok/s", True),
    "mamba_tiny": ("mamba", "Mamba (tiny) prefill tok/s", "tok/s", True),
    "tiny_mlp": ("mlp", "tiny GELU-MLP forward latency (x [32,256] fp32, 256->1024->256)", "us", False),
}


def run_model_line(args):
    """One bench line for the Whisper encoder, Mamba-370m or the tiny MLP:
    value = the target's units per second (or the forward's latency for the
    tiny MLP), CUDA events around K graph replays; e2e the same with the
    input copied from pinned host memory and the output read back; roofline
    the whole forward's algorithmic FLOPs against the measured bf16/fp16
    tensor peak."""
    import torch

    from metal_autotune_b200 import build, lib
    kind, metric, unit, higher = MODEL_LINES[args.config]
    build.build_library()
    rank, world, local = dist_setup()
    tiny = args.config.endswith("_tiny")
    if args.impl == "reference":
        if rank != 0:
            return 0
        step = ModelStep(kind, tiny)
        cb = model_cpu_baseline(step, os.cpu_count() or 1)
        v = cb["value"]
        ms = (1e3 / (v / step.units)) if higher else v / 1e3
        print(json.dumps({"impl": "reference", "metric": metric, "value": v, "unit": unit, "n_gpus": args.gpus,
                          "steps": 1, "warmup": 0, "ms_per_step": round(ms, 4), "higher_is_better": higher,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f32" if kind == "mlp" else "f16",
                          "data": "synthetic", "config": {"workload": args.config}, "cpu_baseline": cb,
                          "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return 0
    step = ModelStep(kind, tiny, args.backend)
    for _ in range(args.warmup):
        step.replay()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        clk.wait_first_sample()
        soak(step.replay, 0.3)
        clk.mark_start()
        ms_total = time_region(step.replay, args.steps, world)
        clk.mark_end()
        ms_e2e_total = time_region(step.e2e_step, args.steps, world)
        soak(step.replay, 0.3)
    ms = max_over_ranks(ms_total / (args.steps * step.per_replay), world)  # per forward
    ms_e2e = max_over_ranks(ms_e2e_total / args.steps, world)
    status = lib.device_status(clear=True)
    if status != 0:
        raise RuntimeError(f"device status {status:#x}: a kernel's bounded wait expired")
    peaks = measured_peaks()
    achieved = step.flops / (ms / 1e3) / 1e12
    val = (lambda t: round(step.units * world / (t / 1e3), 2)) if higher else (lambda t: round(t * 1e3, 3))
    line = {"metric": metric, "value": val(ms), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": higher, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32" if kind == "mlp" else "f16", "data": "synthetic",
            "config": {"workload": args.config, "parallelism": f"replicas x{world}",
                       "graph": ("one CUDA graph per forward" if step.per_replay == 1 else
                                 f"{step.per_replay} forwards per timed CUDA graph (value: device time per forward); "
                                 "e2e one forward per call"),
                       "backend": args.backend,
                       "l2": "inputs larger than L2" if kind != "mlp" else "fits L2 (launch-bound, 1.3 MB)"},
            "e2e": {"value": val(ms_e2e), "unit": unit, "h2d_bytes_per_step": step.host_x.numel()
                    * step.host_x.element_size(), "d2h_bytes_per_step": step.host_out.numel()
                    * step.host_out.element_size()},
            "roofline": {"bound": "tensor" if kind != "mlp" else "launch", "achieved": round(achieved, 3),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops"], 5), "traffic": None,
                         "what": "whole forward: algorithmic FLOPs / forward time vs the measured bf16 burst peak",
                         "forward_gflop": round(step.flops / 1e9, 3)},
            "clocks": clk.summary(),
            "gpu_launches": int(step.launches_per_step * args.steps * (step.per_replay + 1)),
            "launches_per_step": step.launches_per_step}
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = model_cpu_baseline(step, os.cpu_count() or 1)
    barrier(world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="default 300 (Qwen3 request), 5 (Llama forward), 20 (the other targets)")
    ap.add_argument("--warmup", type=int, default=None, help="default 10 (Qwen3 request), 3 (Llama forward)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="qwen3_4b",
                    choices=["qwen3_4b", "qwen3_tiny", "llama3_8b_tp", "llama_tiny_tp", *MODEL_LINES],
                    help="llama*_tp: Llama-3-8B 8-bit prefill 8 x 2048, tensor-parallel over the ranks; "
                         "whisper_turbo / mamba_370m / tiny_mlp: the other targets' own lines")
    ap.add_argument("--mode", default="request", choices=["request", "kernels"])
    ap.add_argument("--backend", default="replay", choices=["replay", "graph"],
                    help="whisper / tiny_mlp lines: the replay bundle (hand-written wrappers) or the graph bundle "
                         "(traced graph with the regions substituted)")
    ap.add_argument("--only", default="", help="kernels mode: comma-separated kernel names")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-llama-tp", action="store_true",
                    help="skip the Llama-3-8B tensor-parallel record of the default line")
    ap.add_argument("--llama-steps", type=int, default=5, help="timed forwards of the Llama record")
    ap.add_argument("--no-overlap", action="store_true",
                    help="Llama TP: all-reduces between the blocks instead of overlapped with the other micro-batch")
    ap.add_argument("--launch-list", action="store_true",
                    help="replay the request W + K times, the K inside an NVTX range 'request' ('forward' for "
                         "the Llama line), and exit (for ncu --nvtx --nvtx-include request/)")
    args = ap.parse_args()
    llama = args.config.startswith("llama")
    if args.steps is None:
        args.steps = 5 if llama else 20 if args.config in MODEL_LINES else 300
    if args.warmup is None:
        args.warmup = 3 if llama else 10
    if args.warmup < 3 and args.mode == "request":
        args.warmup = 3

    if args.config in MODEL_LINES:
        return run_model_line(args)
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
        clk.wait_first_sample()
        soak(req.replay, 0.5)
        clk.mark_start()
        ms_total = time_region(req.replay, args.steps, world)
        clk.mark_end()
        ms_e2e_total = time_region(req.e2e_step, args.steps, world)
        soak(req.replay, 0.5)
    ms = max_over_ranks(ms_total / args.steps, world)
    ms_e2e = max_over_ranks(ms_e2e_total / args.steps, world)
    status = lib.device_status(clear=True)
    if status != 0:
        raise RuntimeError(f"device status {status:#x}: a kernel's bounded wait expired")
    gpu_picks = [int(x) for x in req.host_out[:2].tolist()]
    gpu_decode_logits = req.model.last_logits.float().cpu().numpy()
    peaks = measured_peaks()
    roof = qmm_roofline(req, peaks)
    wbytes, ebytes = packed_weight_bytes(cfg)
    roof["request_floor_ms"] = round(max(request_flops(cfg) / (peaks["bf16_tflops"] * 1e12),
                                         (2 * wbytes + ebytes) / (peaks["hbm_gbs"] * 1e9)) * 1e3, 4)
    prof = ROOT / "profiles" / "qmm_tc_prefill_qwen3_4b.traffic.json"
    if prof.exists():
        roof["traffic"] = json.loads(prof.read_text()).get("bytes_per_launch")
        roof["traffic_note"] = json.loads(prof.read_text()).get("note")
    line = {
        "metric": METRIC, "value": round(PROMPT * world / (ms / 1e3), 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": qwen3_config_record(cfg, world),
        "graph": "one CUDA graph per request",
        "e2e": {"value": round(PROMPT * world / (ms_e2e / 1e3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": PROMPT * 4, "d2h_bytes_per_step": 12},
        "roofline": roof, "clocks": clk.summary(),
        "gpu_launches": int(req.launches_per_step * args.steps * 2),
        "launches_per_step": req.launches_per_step,
    }
    if not args.no_cpu_baseline and world == 1 and rank == 0:
        line["cpu_baseline"] = cpu_baseline(cfg, req.model, req.tokens, os.cpu_count() or 1,
                                            (gpu_picks[0], gpu_picks[1], gpu_decode_logits))
    if not args.no_llama_tp and cfg.layers == 36:
        # every rank builds its shard and takes the same collective steps
        from metal_autotune_b200.targets import llama_tp
        del req
        torch.cuda.empty_cache()
        line["llama_tp"] = llama_tp_record(llama_tp.LLAMA3_8B, LLAMA_B, LLAMA_L, args.llama_steps, 3, rank, world,
                                           local, overlap=not args.no_overlap)
    barrier(world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
