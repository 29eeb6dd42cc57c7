#!/usr/bin/env python
"""Decode throughput of the Qwen2.5-7B-shape int8 decoder on B200 (batch 1).

One step = one greedy decode token through all 28 layers and the LM head at a 512-token context,
int8 per-output-channel weights (uniform codes in [-127, 127], fp16 scales U[1e-3, 2e-2], seed 2),
fp16 KV cache. Weights are 7.07 GB per step, far larger than the 126 MB L2, so no flush is needed.

  value   device-resident decode: each step's input token is the previous step's on-device argmax,
          K steps replay one cached CUDA graph; timed with CUDA events on the model's stream.
  e2e     the same decode through the public C-ABI call (LlmModel.Decode): per step the token id and
          position go host->device and the full vocab logits come back device->host, argmax on the host.
  roofline  the dominant kernel by device time (the k-split int8 GEMV of q/k/v, o_proj and down), each
          projection launched on its own over rotating weight copies (more than L2) and timed with events;
          by_launch adds each projection and the bulk GEMV's gate/up (with ncu DRAM traffic).
  cpu_baseline  the CPU oracle port (C, fp32 AVX2 FMA, OpenMP) of the same decoder and weights on the
          host cores at the same 512-token context (all threads, plus a single-thread figure); the legs
          below carry the same port on their own configuration (config 4: one layer, extrapolated).
  step_roofline  all bytes of a step (weights + KV) over the step time.
  prefill_s  a warm prefill of the 512-token prompt (one 512-row tcgen05 GEMM per projection).
  bs16    16 sequences decoded together (device-resident batched greedy, tcgen05 integer GEMM).
  cfg0 / cfg1 / cfg3  the other BASELINE configurations on this GPU (N = 1 only): the config-0 GEMV
          and GEMM, Qwen2.5-0.5B fp16 decode, and the Gated DeltaNet layer (decode bs1 / bs8, 4096-token
          prefill).
  tp      config 4 (Llama-3-70B shape, bf16) decoded tensor-parallel over all N ranks of the job (N = 1:
          the whole model on one GPU), with the all-reduce path and its measured per-call time.

--impl reference runs the reference's CPU path (the oracle port; the reference's own C# + Level Zero
code cannot run here) on all host threads and prints the same metric.
Multi-GPU (torchrun): config 2 fits one GPU, so N ranks run N independent replicas (weak scaling; no
collective on its data path); the timed region is bracketed by barriers and the max time over ranks is
reported. The `tp` leg is the tensor-parallel measurement at every N. --workload cfg4 runs that leg alone
(cfg3 the DeltaNet layer alone); --profile-case runs small cases for ncu captures.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (Qwen2.5-7B Int8, bs1)"
CFG2 = dict(hidden_size=3584, intermediate_size=18944, num_layers=28, num_attention_heads=28, num_key_value_heads=4,
            head_dim=128, vocab_size=152064, max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6,
            tie_word_embeddings=0, attention_bias=1, q8_group=0)
ORC2 = dict(hidden=3584, inter=18944, layers=28, heads=28, kv_heads=4, head_dim=128, vocab=152064, max_pos=32768,
            eps=1e-6, theta=1e6, tie=0, bias=1, qk_norm=0, rope_type=0, rope_factor=1.0, rope_original_max=0,
            rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0)
SEED = 2
# Config 4: Llama-3-70B shape, bf16, llama3 RoPE scaling, tensor-parallel over the torchrun ranks.
CFG4 = dict(hidden_size=8192, intermediate_size=28672, num_layers=80, num_attention_heads=64, num_key_value_heads=8,
            head_dim=128, vocab_size=128256, max_position_embeddings=131072, rms_norm_eps=1e-5, rope_theta=5e5,
            tie_word_embeddings=0, attention_bias=0, rope_type=3, rope_factor=8.0, rope_low_freq_factor=1.0,
            rope_high_freq_factor=4.0, rope_original_max_position=8192)
CFG4_PROMPT = 2048
BS16 = 16  # the metric's second batch size (decode at batch 1 and batch 16)
CONTEXT = 512


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def tflops_peak() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"])
        except Exception:
            pass
    return 1590.0


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons read every 20 ms through NVML (the library nvidia-smi
    reports from; reads only) on a host thread, each sample time-stamped so that only samples taken
    inside the timed region count. Falls back to `nvidia-smi -lms` when NVML is unavailable."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples: list[tuple[float, float, float, int]] = []  # (t, sm MHz, max MHz, reason bits)
        self.stop_flag = threading.Event()
        self.thread = None
        self.proc = None
        self.window = (0.0, float("inf"))

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def loop():
                while not self.stop_flag.is_set():
                    try:
                        sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        bits = int(get_reasons(h))
                        self.samples.append((time.monotonic(), sm, mx, bits))
                    except Exception:
                        pass
                    self.stop_flag.wait(0.02)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
        except Exception:
            self._start_smi()

    def _start_smi(self):
        fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={fields}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        bits = list(self.REASONS.values())

        def read():
            for line in self.proc.stdout:
                r = [c.strip() for c in line.split(",")]
                try:
                    b = sum(bit for bit, v in zip(bits, r[2:6]) if v.lower().startswith("active"))
                    self.samples.append((time.monotonic(), float(r[0]), float(r[1]), b))
                except (ValueError, IndexError):
                    continue

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def mark(self, t0: float, t1: float):
        """The timed region, in time.monotonic() seconds."""
        self.window = (t0, t1)

    def stop(self) -> dict:
        self.stop_flag.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        t0, t1 = self.window
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside and self.samples:  # region shorter than one sample: take the nearest after its start
            after = [s for s in self.samples if s[0] >= t0]
            inside = after[:1]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock samples"], "samples": 0}
        reasons = sorted(name for name, bit in self.REASONS.items() if any(s[3] & bit for s in inside))
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": max(s[2] for s in inside),
                "reasons": reasons, "samples": len(inside)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------------------------------------
# CPU: the oracle port of the same decoder
# ------------------------------------------------------------------------------------------------

class CpuDecoder:
    """The oracle port of the config-2 decoder on the host cores, for timing: the same int8 weights
    (seed 2) with projections accumulated in fp32 fused multiply-adds on AVX2 (orc_gemm_fast; the checker
    build accumulates in double), and a 512-token context whose K/V rows are filled with seeded values
    (the context's values do not change the work of a decode step), so steps run at the GPU arm's
    positions 512 and on."""

    def __init__(self, max_steps: int):
        from oracle import oracle as orc

        self.orc = orc
        self.om = orc.OracleModel(dict(ORC2, wdtype=orc.I8, group=0, kv_dtype=orc.F16), CONTEXT + max_steps + 8)
        self.om.init_synthetic(SEED, 0.02, 1e-3, 2e-2)
        self.om.set_fast(True)
        rng = np.random.default_rng(SEED + 100)
        kvd = ORC2["kv_heads"] * ORC2["head_dim"]
        for layer in range(ORC2["layers"]):
            k = rng.standard_normal((CONTEXT, kvd)).astype(np.float32)
            v = rng.standard_normal((CONTEXT, kvd)).astype(np.float32)
            self.om.write_kv(layer, 0, k, v)
        self.pos = CONTEXT
        self.tok = int(rng.integers(0, 152064))

    def sample(self, budget_s: float, max_steps: int, threads: int) -> dict:
        self.orc.set_num_threads(threads)
        t0 = time.perf_counter()
        lg = self.om.step(self.tok, self.pos)  # one untimed step sizes the sample
        self.tok, self.pos = int(np.argmax(lg)), self.pos + 1
        first = time.perf_counter() - t0
        steps = max(1, min(max_steps, int(budget_s / max(first, 1e-3))))
        p0 = self.pos
        t0 = time.perf_counter()
        for _ in range(steps):
            lg = self.om.step(self.tok, self.pos)
            self.tok, self.pos = int(np.argmax(lg)), self.pos + 1
        dt = time.perf_counter() - t0
        return {"value": steps / dt, "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{steps} greedy decode steps of the full 28-layer config-2 decoder (same int8 weights, "
                          f"seed {SEED}) at positions {p0}..{p0 + steps - 1} of a {CONTEXT}-token context; C oracle, "
                          f"OpenMP over output rows, int8 x f32 products accumulated in fp32 FMA (AVX2)"}

    def close(self):
        self.om.close()


def cpu_baseline(budget_s: float) -> dict:
    """All host threads, plus a single-thread figure, on a bounded sample."""
    threads = os.cpu_count() or 1
    dec = CpuDecoder(64)
    allc = dec.sample(budget_s * 0.6, 32, threads)
    one = dec.sample(budget_s * 0.4, 8, 1)
    dec.close()
    allc["single_thread"] = {"value": one["value"], "unit": "tok/s", "cores": 1, "sample": one["sample"]}
    return allc


def _timed_steps(fn, budget_s: float, max_reps: int) -> tuple[int, float]:
    """One untimed call sizes the sample; then as many calls as fit the budget (at least one)."""
    t0 = time.perf_counter()
    fn()
    first = time.perf_counter() - t0
    reps = max(1, min(max_reps, int(budget_s / max(first, 1e-4))))
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    return reps, time.perf_counter() - t0


def cpu_legs(budget_s: float) -> dict:
    """The oracle port on the host cores (all threads, fp32-accumulate timing build) for the other BASELINE
    configurations, each a bounded sample: config 0 (the int8 GEMV and its M = 128 GEMM), config 1 (decode
    of the fp16 Qwen2.5-0.5B shape at a 128-token context), config 3 (one Gated DeltaNet layer's decode
    step: projections, conv, recurrence, gated norm, out_proj; bf16 weights) and config 4 (one bf16 decoder
    layer of the Llama-3-70B shape at a 2048-token context, extrapolated to 80 layers plus the LM head by
    bytes)."""
    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    orc.set_num_threads(threads)
    each = budget_s / 4
    out = {}
    rng = np.random.default_rng(0)
    # Config 0.
    n, k = 4864, 896
    q = rng.integers(-127, 128, (n, k)).astype(np.int8)
    sc = orc.f16_bits(rng.uniform(1e-3, 2e-2, n).astype(np.float32))
    x1 = rng.standard_normal((1, k)).astype(np.float32)
    x128 = rng.standard_normal((128, k)).astype(np.float32)
    r1, t1 = _timed_steps(lambda: orc.gemm_fast(x1, q, orc.I8, sc, k), each / 2, 20000)
    r2, t2 = _timed_steps(lambda: orc.gemm_fast(x128, q, orc.I8, sc, k), each / 2, 2000)
    b1, b128 = n * k + 2 * n + 2 * k + 2 * n, n * k + 2 * n + 128 * (2 * k + 2 * n)
    out["cfg0"] = {"gemv_us": round(t1 / r1 * 1e6, 2), "gemv_gbs": round(b1 * r1 / t1 / 1e9, 2),
                   "gemm_m128_us": round(t2 / r2 * 1e6, 2), "gemm_m128_tflops": round(2 * 128 * n * k * r2 / t2 / 1e12, 4),
                   "cores": threads, "kind": "port",
                   "sample": f"{r1} GEMVs and {r2} M = 128 GEMMs of the int8 [4864, 896] weights (per-channel scales)"}
    # Config 1.
    c1 = dict(hidden=896, inter=4864, layers=24, heads=14, kv_heads=2, head_dim=64, vocab=151936, max_pos=32768,
              eps=1e-6, theta=1e6, tie=1, bias=1, qk_norm=0, rope_type=0, rope_factor=1.0, rope_original_max=0,
              rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0,
              wdtype=orc.F16, group=0, kv_dtype=orc.F16)
    om = orc.OracleModel(c1, 160)
    om.init_synthetic(1, 0.02)
    om.set_fast(True)
    for layer in range(24):
        om.write_kv(layer, 0, rng.standard_normal((128, 128)).astype(np.float32),
                    rng.standard_normal((128, 128)).astype(np.float32))
    st = {"pos": 128, "tok": 1}

    def step1():
        lg = om.step(st["tok"], st["pos"])
        st["tok"], st["pos"] = int(np.argmax(lg)), min(st["pos"] + 1, 150)

    r, t = _timed_steps(step1, each, 20)
    om.close()
    out["cfg1"] = {"value": round(r / t, 2), "unit": "tok/s", "cores": threads, "kind": "port",
                   "sample": f"{r} greedy decode steps of the 24-layer fp16 decoder at a 128-token context"}
    # Config 3: a one-layer hybrid oracle whose only layer is the Gated DeltaNet layer (tiny MLP, vocab and
    # embedding so that the layer dominates).
    H, HK, HV, DK, DV = 2048, 16, 32, 128, 128
    c3 = dict(hidden=H, inter=16, layers=1, heads=16, kv_heads=16, head_dim=128, vocab=16, max_pos=4096, eps=1e-6,
              theta=1e6, tie=0, bias=0, qk_norm=0, rope_type=0, rope_factor=1.0, rope_low=1.0, rope_high=4.0,
              rope_beta_fast=32.0, rope_beta_slow=1.0, wdtype=orc.BF16, group=0, kv_dtype=orc.F32, linear_mask=1,
              lin_k_heads=HK, lin_v_heads=HV, lin_k_dim=DK, lin_v_dim=DV, lin_conv=4, attn_gate=0, norm_offset=0.0)
    om = orc.OracleModel(c3, 4096)
    cd, vd = 2 * HK * DK + HV * DV, HV * DV
    for name, shape in (("in_proj_qkv.weight", (cd, H)), ("in_proj_z.weight", (vd, H)), ("in_proj_b.weight", (HV, H)),
                        ("in_proj_a.weight", (HV, H)), ("out_proj.weight", (H, vd)), ("conv1d.weight", (cd, 4)),
                        ("A_log", (HV,)), ("dt_bias", (HV,))):
        om.set_tensor("model.layers.0.linear_attn." + name, (rng.standard_normal(shape) * 0.02).astype(np.float32))
    om.set_fast(True)
    st = {"pos": 0}

    def step3():
        om.step(1, st["pos"])
        st["pos"] += 1

    r, t = _timed_steps(step3, each, 256)
    om.close()
    out["cfg3"] = {"us_per_step": round(t / r * 1e6, 1), "cores": threads, "kind": "port",
                   "sample": f"{r} decode steps of one Gated DeltaNet layer (16 / 32 heads of 128, bf16 projections, "
                             f"fp32 state), bs1"}
    # Config 4: one bf16 layer at the Llama-3-70B width, extrapolated.
    c4 = dict(hidden=8192, inter=28672, layers=1, heads=64, kv_heads=8, head_dim=128, vocab=16, max_pos=131072,
              eps=1e-5, theta=5e5, tie=0, bias=0, qk_norm=0, rope_type=3, rope_factor=8.0, rope_original_max=8192,
              rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0,
              wdtype=orc.BF16, group=0, kv_dtype=orc.BF16)
    om = orc.OracleModel(c4, 2100)
    om.init_synthetic(4, 0.02)
    om.set_fast(True)
    om.write_kv(0, 0, rng.standard_normal((2048, 1024)).astype(np.float32),
                rng.standard_normal((2048, 1024)).astype(np.float32))
    st = {"pos": 2048}

    def step4():
        om.step(1, st["pos"])
        st["pos"] = min(st["pos"] + 1, 2090)

    r, t = _timed_steps(step4, each, 20)
    om.close()
    layer_bytes = 2 * (8192 * (8192 + 2 * 1024) + 8192 * 8192 + 3 * 8192 * 28672)
    head_bytes = 2 * 128256 * 8192
    step_s = t / r * (80 + head_bytes / layer_bytes)
    out["cfg4"] = {"value": round(1.0 / step_s, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                   "extrapolated": True, "layer_ms": round(t / r * 1e3, 2),
                   "sample": f"{r} decode steps of one bf16 Llama-3-70B-width layer at a 2048-token context, scaled "
                             f"to 80 layers plus the LM head by their weight bytes"}
    return out


def run_reference(args) -> int:
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    # Each step is one full decode step on the CPU at the GPU arm's context; the timed sample is bounded
    # so the run ends within minutes.
    dec = CpuDecoder(max(args.steps, 8) + max(args.warmup, 1) + 4)
    warm = dec.sample(budget_s=5.0, max_steps=max(1, min(args.warmup, 2)), threads=threads)
    res = dec.sample(budget_s=60.0, max_steps=args.steps, threads=threads)
    dec.close()
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / res["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "config 2: Qwen2.5-7B-shape int8 decode, bs1, 512-token context", "batch": 1,
                       "seq_len": CONTEXT, "parallelism": "cpu"},
            "cpu_baseline": res,
            "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's own path (C# + LevelZero.NET on an Intel GPU) cannot run here; this arm times "
                    "the CPU restatement of its op sequence (oracle/, fp32-accumulate timing build), warmup "
                    f"{warm['value']:.3f} tok/s"}
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------------------------------------
# GPU
# ------------------------------------------------------------------------------------------------

def _time_projection(lz, dev, suite, stream_ptr, torch, n: int, k: int, epi: int, norm: bool, bias: bool,
                     blocked: bool, copies: int, reps: int = 25) -> tuple[float, int]:
    """One config-2 decode projection (int8, one f16 scale per row, one activation row) launched on its
    own through l0b_linear_fused, cycling over `copies` weight copies (more than L2 holds) so every launch
    streams its weights from HBM; CUDA events on the library's stream. Returns (average ms per launch,
    algorithmic bytes per launch: weights + scales + x (+ norm weight, bias) + output (read and written
    for the residual add))."""
    rng = np.random.default_rng(5 + n + k)
    q = rng.integers(-127, 128, (n, k), dtype=np.int8)
    if blocked:
        q = lz.block_int8(q)
    s = rng.uniform(1e-3, 2e-2, n).astype(np.float16)
    ws = [lz.SharedBuffer.from_array(dev, q) for _ in range(copies)]
    sb = lz.SharedBuffer.from_array(dev, s)
    x = lz.SharedBuffer.from_array(dev, rng.standard_normal(k).astype(np.float32))
    nw = lz.SharedBuffer.from_array(dev, np.ones(k, np.float32)) if norm else None
    bb = lz.SharedBuffer.from_array(dev, np.zeros(n, np.float32)) if bias else None
    out_cols = n // 2 if epi == suite.EPI_SWIGLU else n
    out = lz.SharedBuffer.from_array(dev, np.zeros(out_cols, np.float32))
    flag = epi | (suite.EPI_BLOCKED_WEIGHTS if blocked else 0)
    stream = torch.cuda.ExternalStream(stream_ptr)

    def launch(i):
        suite.linear_fused(dev, 1, n, k, x, ws[i % copies], sb, k, nw, 1e-6, flag, bb, out)

    for i in range(2 * copies):
        launch(i)
    dev.Synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps * copies):
        launch(i)
    e1.record(stream)
    e1.synchronize()
    avg_ms = e0.elapsed_time(e1) / (reps * copies)
    for b in ws + [sb, x, nw, bb, out]:
        if b is not None:
            b.Dispose()
    nbytes = n * k + 2 * n + 4 * k + (4 * k if norm else 0) + (4 * n if bias else 0) + \
        4 * out_cols * (2 if epi == suite.EPI_ACCUM else 1)
    return avg_ms, nbytes


def _traffic(name: str):
    tf = ROOT / "profiles" / name
    if tf.exists():
        return json.loads(tf.read_text()).get("dram_bytes_per_launch")
    return None


def dominant_kernel_roofline(lz, dev, suite, stream_ptr, torch, peak: float, peak_kind: str, bulk: bool = True) -> dict:
    """The step's dominant kernel by device time (profiles/decode_step_cfg2_launches.md: gemv_ksplit_kernel,
    50% of the bs1 step -- q/k/v, o_proj and down of every layer -- ahead of gemv_bulk_kernel, 39%: gate/up
    and the LM head). Each config-2 projection runs on its own over rotating weight copies (more than L2);
    `achieved` is the k-split kernel's average launch over one layer's mix (one q/k/v, one o_proj, one
    down): their algorithmic bytes over their summed durations. `by_launch` gives each projection, and the
    bulk kernel's gate/up, on its own with the DRAM traffic of its ncu capture where one exists."""
    H, I, QKV = 3584, 18944, 4608
    cases = {
        # name: (n, k, epilogue, norm, bias, blocked, copies)
        "qkv": (QKV, H, suite.EPI_STORE, True, True, True, 12),
        "o_proj": (H, H, suite.EPI_ACCUM, False, False, True, 16),
        "down": (H, I, suite.EPI_ACCUM, False, False, True, 4),
        "gate_up": (2 * I, H, suite.EPI_SWIGLU, True, False, False, 4),
    }
    by = {}
    for name, (n, k, epi, norm, bias, blocked, copies) in cases.items():
        ms, nbytes = _time_projection(lz, dev, suite, stream_ptr, torch, n, k, epi, norm, bias, blocked, copies)
        gbs = nbytes / (ms * 1e-3) / 1e9
        by[name] = {"kernel": ("gemv_bulk_kernel" if bulk else "gemv_mma_kernel<int8>") if name == "gate_up" else
                    "gemv_ksplit_kernel",
                    "shape": f"int8 [{n}, {k}]" + (" blocked" if blocked else " row-major"),
                    "avg_us": round(ms * 1e3, 2), "algorithmic_bytes": nbytes, "achieved": round(gbs, 1),
                    "frac": round(gbs / peak, 4)}
    by["down"]["traffic"] = _traffic("gemv_ksplit_i8_down_cfg2.traffic.json")
    by["gate_up"]["traffic"] = _traffic("gemv_i8_swiglu_cfg2.traffic.json") if bulk else None
    mix = ("qkv", "o_proj", "down")
    nbytes = sum(by[c]["algorithmic_bytes"] for c in mix)
    us = sum(by[c]["avg_us"] for c in mix)
    achieved = nbytes / (us * 1e-6) / 1e9
    name = ("gemv_ksplit_kernel (int8 blocked [N/16][K/512][16][512]; one 512-k block of a group of row tiles per "
            "CTA, bulk copies, integer mma.sync m16n8k32 on int8 digits, exact int64 row sums): q/k/v + o_proj + "
            "down of one layer")
    return {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
            "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
            "traffic_note": "measured per launch for the down projection only (by_launch.down.traffic)",
            "algorithmic_bytes": nbytes // 3, "avg_us": round(us / 3, 2), "by_launch": by}


def measure_cfg0(lz, dev, suite, stream_ptr, torch, peak: float, peak_kind: str, tflops_peak: float) -> dict:
    """Config 0: the single linear op y = x W^T with W int8 [4864, 896] (codes uniform in [-127, 127],
    fp16 per-row scales U[1e-3, 2e-2]) and x from N(0, 1) (fp16 values, f32 storage), seed 0: one row
    (decode GEMV, l0b_linear) and 128 rows (prefill GEMM on the tcgen05 kernel, l0b_linear_tc), each over
    40 rotating weight copies (174 MB > L2), CUDA events."""
    N, K, copies = 4864, 896, 40
    rng = np.random.default_rng(0)
    stream = torch.cuda.ExternalStream(stream_ptr)
    qs = [lz.SharedBuffer.from_array(dev, rng.integers(-127, 128, (N, K), dtype=np.int8)) for _ in range(copies)]
    ss = [lz.SharedBuffer.from_array(dev, rng.uniform(1e-3, 2e-2, N).astype(np.float16)) for _ in range(copies)]
    out = {}
    lib = lz.load_library()
    for M in (1, 128):
        x = lz.SharedBuffer.from_array(dev, rng.standard_normal((M, K)).astype(np.float16).astype(np.float32))
        y = lz.SharedBuffer(dev, lz.F32, M * N)

        def run(i):
            if M == 1:
                suite.linear(dev, 1, N, K, x, qs[i % copies], ss[i % copies], K, None, y)
            else:
                lz.check(lib.l0b_linear_tc_scaled(suite.handle, dev.handle, M, N, K, x.handle, qs[i % copies].handle,
                                                  ss[i % copies].handle, K, None, 0.0, 0, None, y.handle))

        for i in range(2 * copies):
            run(i)
        dev.Synchronize()
        reps = 10 * copies
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            run(i)
        e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) / reps * 1e3
        byt = N * K + N * 2 + M * K * 4 + M * N * 4
        flops = 2.0 * M * N * K
        r = {"us_per_call": round(us, 3), "algorithmic_bytes": byt, "achieved_gbs": round(byt / us / 1e3, 1),
             "hbm_frac": round(byt / us / 1e3 / peak, 4), "tflops": round(flops / us / 1e6, 2)}
        if M > 1:
            r["tensor_frac"] = round(flops / us / 1e6 / tflops_peak, 4)
        out["gemv_m1" if M == 1 else "gemm_m128"] = r
        x.Dispose()
        y.Dispose()
    for b in qs + ss:
        b.Dispose()
    out["note"] = (f"peak {peak} GB/s ({peak_kind}) and {tflops_peak} TFLOP/s bf16 (measured burst); the 4.4 MB "
                   "weight of one call fits L2, so the copies rotate; M=1 on the register-streamed tensor-core GEMV, "
                   "M=128 on tcgen05 kind::i8 with the activation digit cast included")
    return out


def measure_cfg1(lz, dev, suite, stream_ptr, torch, peak: float, steps: int, warmup: int) -> dict:
    """Config 1: Qwen2.5-0.5B shape, fp16 weights N(0, 0.02) seed 1 (tied embeddings), 128-token prompt,
    device-resident greedy decode at bs1 timed with CUDA events."""
    stream = torch.cuda.ExternalStream(stream_ptr)
    cfg = dict(hidden_size=896, intermediate_size=4864, num_layers=24, num_attention_heads=14, num_key_value_heads=2,
               head_dim=64, vocab_size=151936, max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6,
               tie_word_embeddings=1, attention_bias=1)
    prompt = np.random.default_rng(1).integers(0, 151936, 128).astype(np.int32)
    with lz.LlmModel(dev, suite, lz.model_config(kv_dtype=lz.F16, **cfg), 128 + warmup + steps + 8, "float16") as m:
        m.init_synthetic(1, 0.02)
        t0 = time.perf_counter()
        m.Prefill(prompt)
        prefill_s = time.perf_counter() - t0
        m.decode_greedy_device(warmup)
        dev.Synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.decode_greedy_device(steps)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        proj = m.ProjectionBytes
    pos_mid = 128 + warmup + steps / 2
    step_bytes = proj + 24 * 2 * 128 * 2 * pos_mid  # fp16 KV: 2 kv heads x 64 = 128 wide, K and V
    return {"workload": "config 1: Qwen2.5-0.5B-shape fp16 decode, bs1, 128-token prompt", "value": round(
        steps / (ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(ms / steps, 4), "prefill_s": round(prefill_s, 3),
        "bytes_per_step": int(step_bytes), "achieved_gbs": round(step_bytes / (ms / steps * 1e-3) / 1e9, 1),
        "frac": round(step_bytes / (ms / steps * 1e-3) / 1e9 / peak, 4)}


def measure_cfg3(lz, dev, suite, stream_ptr, torch, warmup: int) -> dict:
    """Config 3: one Gated DeltaNet layer (Qwen3.5 shape, bf16 projections) driven through the library's
    ops as LlmDecoderLayer.MixLinear calls them: in_proj (q, k, v | z) and (b | a) projections, causal
    conv + SiLU, the gated delta recurrence with its gated RMSNorm, out_proj. Decode: one token per
    step for bs sequences (the four in-projections one shared launch, conv and recurrence each one launch
    over all rows), one recorded command list per step. Prefill: 4096 tokens, projections on the tcgen05
    GEMM, the recurrence chunked."""
    H, HK, HV, DK, DV, KC, T = 2048, 16, 32, 128, 128, 4, 4096
    CONV = 2 * HK * DK + HV * DV
    ZD = HV * DV
    lib = lz.load_library()
    stream = torch.cuda.ExternalStream(stream_ptr)
    rng = np.random.default_rng(3)
    owned = []

    def bf16(shape, std):
        w = torch.from_numpy((rng.standard_normal(shape) * std).astype(np.float32)).to(torch.bfloat16)
        owned.append(lz.SharedBuffer.from_array(dev, w.view(torch.int16).numpy().view(np.uint16), lz.BF16))
        return owned[-1]

    def f32(a):
        owned.append(lz.SharedBuffer.from_array(dev, np.ascontiguousarray(a, np.float32)))
        return owned[-1]

    def f32n(n):
        owned.append(lz.SharedBuffer(dev, lz.F32, n))
        return owned[-1]

    # The in-projections [qkv; z; b; a] stacked in one matrix (ProjectShared: one launch streams it once);
    # views of it serve the per-projection prefill GEMMs.
    IN_ROWS = [CONV, ZD, HV, HV]
    w_in = bf16((sum(IN_ROWS), H), 0.02)
    offs = np.cumsum([0] + IN_ROWS) * H
    w_qkv, w_z, w_b, w_a = (w_in.View(int(offs[i]), IN_ROWS[i] * H) for i in range(4))
    owned.extend([w_qkv, w_z, w_b, w_a])
    w_o = bf16((H, ZD), 0.02)
    conv_w = f32(rng.standard_normal((CONV, KC)) * 0.3)
    a_log = f32(np.log(rng.uniform(1, 16, HV)))
    dt_bias = f32(rng.standard_normal(HV) * 0.1)
    norm_w = f32(1 + 0.1 * rng.standard_normal(DV))

    def layer_buffers(rows):
        return dict(x=f32(rng.standard_normal((rows, H))), qkv=f32n(rows * CONV), z=f32n(rows * ZD), b=f32n(rows * HV),
                    a=f32n(rows * HV), conv=f32n(rows * CONV), o=f32n(rows * ZD), y=f32n(rows * H))

    def timed(fn, reps):
        for _ in range(warmup):
            fn()
        dev.Synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    results = {}
    for bs in (1, 8):
        buf = layer_buffers(bs)
        # Every sequence's recurrent state and conv window, batched: one launch each for all sequences.
        states = f32n(bs * HV * DK * DV)
        conv_states = f32n(bs * CONV * (KC - 1))

        def step():
            dev.BeginRecording()
            suite.linear_shared(dev, bs, H, buf["x"], w_in, None, 0, IN_ROWS,
                                [buf["qkv"], buf["z"], buf["b"], buf["a"]])
            suite.CausalConv.ExecuteBatch(dev, buf["qkv"], conv_states, conv_w, buf["conv"], CONV, KC, bs)
            suite.GatedDelta.ExecuteBatch(dev, buf["conv"], buf["z"], buf["b"], buf["a"], a_log, dt_bias, norm_w,
                                          states, buf["o"], HK, HV, DK, DV, bs, 1e-6)
            suite.linear(dev, bs, H, ZD, buf["o"], w_o, None, 0, None, buf["y"])
            dev.EndRecording()

        ms = timed(step, 256 if bs == 1 else 64)
        proj = (CONV + ZD + 2 * HV) * H * 2 + H * ZD * 2
        step_bytes = proj + bs * (2 * HV * DK * DV * 4 + 2 * CONV * (KC - 1) * 4)
        results[f"bs{bs}"] = {"us_per_step": round(ms * 1e3, 2), "tok_s": round(bs / (ms / 1e3), 1),
                              "bytes_per_step": step_bytes, "achieved_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1)}
    # Prefill: 4096 tokens of one sequence.
    pre = layer_buffers(T)
    state = f32n(HV * DK * DV)
    conv_state = f32n(CONV * (KC - 1))
    phases = {}

    def tc(m, n, k, x, w, out):
        lz.check(lib.l0b_linear_tc(suite.handle, dev.handle, m, n, k, x.handle, w.handle, None, 0.0, 0, None,
                                   out.handle))

    phases["projections_in"] = timed(lambda: (tc(T, CONV, H, pre["x"], w_qkv, pre["qkv"]),
                                              tc(T, ZD, H, pre["x"], w_z, pre["z"]),
                                              tc(T, HV, H, pre["x"], w_b, pre["b"]),
                                              tc(T, HV, H, pre["x"], w_a, pre["a"])), 3)
    phases["causal_conv"] = timed(lambda: suite.CausalConv.Execute(dev, pre["qkv"], conv_state, conv_w, pre["conv"],
                                                                   CONV, KC, T), 3)
    phases["gated_delta"] = timed(lambda: suite.GatedDelta.ExecuteGrouped(
        dev, pre["conv"], pre["z"], pre["b"], pre["a"], a_log, dt_bias, norm_w, state, pre["o"], HK, HV, DK, DV, T,
        1e-6), 3)
    phases["out_proj"] = timed(lambda: tc(T, H, ZD, pre["o"], w_o, pre["y"]), 3)
    total = sum(phases.values())
    for bb in reversed(owned):  # views before the buffer they view
        bb.Dispose()
    return {"decode": results, "prefill_4096_ms": {k: round(v, 3) for k, v in phases.items()} | {"total": round(total, 3)},
            "config": "config 3: Gated DeltaNet layer alone, hidden 2048, 16 key / 32 value heads of 128, conv 4, "
                      "fp32 state [32,128,128] per sequence; bf16 weights 67 MB per step (below L2: decode figures "
                      "are L2-assisted)"}


def run_cfg3_deltanet(args) -> int:
    """Config 3 on its own (bench.py --workload cfg3)."""
    import ctypes as C

    import torch

    from l0llm_b200 import levelzero as lz

    dev = lz.ComputeDevice(0)
    suite = lz.LlmKernelSuite.Create(dev)
    sp = C.c_void_p()
    lz.check(lz.load_library().l0b_device_stream(dev.handle, C.byref(sp)))
    r = measure_cfg3(lz, dev, suite, sp.value, torch, args.warmup)
    suite.Dispose()
    dev.Dispose()
    bs1 = r["decode"]["bs1"]
    line = {"metric": "Gated DeltaNet layer decode tok/s (Qwen3.5 shape, bf16, bs1)", "value": bs1["tok_s"],
            "unit": "tok/s", "n_gpus": 1, "steps": 256, "warmup": args.warmup,
            "ms_per_step": round(bs1["us_per_step"] / 1e3, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": r["config"]}, "decode": r["decode"], "prefill_4096_ms": r["prefill_4096_ms"]}
    print(json.dumps(line))
    return 0


def measure_cfg4_tp(lz, dev, suite, stream_ptr, torch, dist, world: int, rank: int, local: int, steps: int,
                    warmup: int, batch: int = 1) -> dict:
    """Config 4 (Llama-3-70B shape, bf16, llama3 RoPE) decoded tensor-parallel over the `world` ranks of the
    job (world = 1: the whole 139 GB model on one GPU, the scaling anchor): q/k/v, gate/up and lm_head
    column-split, o_proj/down row-split with an all-reduce after each, KV heads split. A 2048-token prompt,
    then `warmup` + `steps` device-resident greedy steps at bs1; CUDA events on the model stream, max
    over ranks. Every rank takes the same collective steps; returns the result on every rank. batch > 1
    (BASELINE config 4's batch 32): the prompt is prefilled once and forked on the device into `batch`
    sequences, which then decode together (one graph per step)."""
    stream = torch.cuda.ExternalStream(stream_ptr)
    comm = None
    if world > 1:
        box = [lz.Communicator.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm = lz.Communicator(dev, box[0], world, rank)
    uses_peer = comm is not None and comm.UsesPeerAllReduce
    fused = lz.Communicator.fused_allreduce()
    cfg = lz.model_config(kv_dtype=lz.BF16, tp_size=world, tp_rank=rank, max_batch=batch, **CFG4)
    model = lz.LlmModel(dev, suite, cfg, CFG4_PROMPT + 2 * warmup + steps + 16, "bfloat16", comm=comm)
    model.init_synthetic(4, 0.02)
    prompt = np.random.default_rng(4).integers(0, CFG4["vocab_size"], CFG4_PROMPT).astype(np.int32)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    t0 = time.perf_counter()
    model.Prefill(prompt)
    barrier()
    prefill_s = time.perf_counter() - t0
    for sq in range(1, batch):
        model.ForkSequence(0, sq, 0)

    def decode(n):
        return model.decode_greedy_device(n) if batch == 1 else model.decode_greedy_device_batch(n, batch)

    decode(warmup)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    toks = decode(steps)
    e1.record(stream)
    e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    proj = model.ProjectionBytes
    t = torch.tensor([ms, prefill_s], dtype=torch.float64, device="cuda")
    agree = True
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        same = torch.tensor(toks.astype(np.int64), device="cuda")
        ref = same.clone()
        dist.broadcast(ref, src=0)
        agree = bool((same == ref).all())
    ms, prefill_s = float(t[0]), float(t[1])
    model.Dispose()
    ar_us = None
    if comm is not None:
        # The step's collective on its own: 2 x layers all-reduces of one hidden row per token, timed
        # back to back with CUDA events on the model stream (max over ranks), for the all-reduce share.
        # They are queued behind a ~50 ms device sleep so the events time the GPU, not the host's
        # per-call launch cost.
        n_ar = 2 * CFG4["num_layers"]
        with lz.SharedBuffer(dev, lz.F32, CFG4["hidden_size"]) as hb:
            for _ in range(20):
                comm.AllReduce(hb)
            barrier()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                torch.cuda._sleep(100_000_000)
            a0.record(stream)
            for _ in range(n_ar):
                comm.AllReduce(hb)
            a1.record(stream)
            a1.synchronize()
            barrier()
            ta = torch.tensor([a0.elapsed_time(a1) * 1e3 / n_ar], dtype=torch.float64, device="cuda")
            dist.all_reduce(ta, op=dist.ReduceOp.MAX)
            ar_us = float(ta[0])
        comm.Dispose()  # releases the device's captured graphs first
    return {"workload": f"config 4: Llama-3-70B-shape bf16 (80 layers, hidden 8192, 64/8 heads, inter 28672, vocab "
                        f"128256, llama3 RoPE), TP{world}, bs{batch}, {CFG4_PROMPT}-token prompt",
            "value": round(batch * steps / (ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(ms / steps, 4),
            "scaling": "strong", "parallelism": f"tp{world}", "prefill_s": round(prefill_s, 3),
            "per_rank_weight_gbs": round(proj / (ms / steps * 1e-3) / 1e9, 1),
            "weight_bytes_per_rank": int(proj), "ranks_agree_on_tokens": agree, "steps": steps, "warmup": warmup,
            "allreduce": ("peer memory, folded into the row-split GEMVs" if uses_peer and fused else "peer memory")
            if uses_peer else ("nccl" if world > 1 else "none"),
            "allreduce_us": None if ar_us is None else round(ar_us, 2),
            "allreduce_share": None if ar_us is None else
            round(2 * CFG4["num_layers"] * ar_us / (ms / steps * 1e3), 3)}


def run_cfg4_tp(args) -> int:
    """Config 4 on its own (bench.py --workload cfg4, under torchrun for N > 1)."""
    world, rank, local = dist_env()
    import ctypes as C
    import datetime

    import torch
    import torch.distributed as dist

    from l0llm_b200 import levelzero as lz

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    dev = lz.ComputeDevice(local)
    suite = lz.LlmKernelSuite.Create(dev)
    sp = C.c_void_p()
    lz.check(lz.load_library().l0b_device_stream(dev.handle, C.byref(sp)))
    sampler = ClockSampler(local)
    sampler.start()
    t_begin = time.monotonic()
    r = measure_cfg4_tp(lz, dev, suite, sp.value, torch, dist, world, rank, local, args.steps, args.warmup,
                        batch=args.tp_batch)
    sampler.mark(t_begin, time.monotonic())
    clocks = sampler.stop()
    suite.Dispose()
    dev.Dispose()
    if rank == 0:
        line = {
            "metric": f"decode tok/s (Llama-3-70B bf16, TP, bs{args.tp_batch})", "value": r["value"], "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": r["workload"], "global_batch": args.tp_batch, "seq_len": CFG4_PROMPT,
                       "parallelism": r["parallelism"],
                       "l2": "inputs larger than L2: every rank streams its weight shard each step"},
            "per_rank_weight_gbs": r["per_rank_weight_gbs"], "clocks": clocks, "prefill_s": r["prefill_s"],
            "ranks_agree_on_tokens": r["ranks_agree_on_tokens"], "allreduce": r["allreduce"],
            "allreduce_us": r["allreduce_us"], "allreduce_share": r["allreduce_share"]}
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_profile_case(case: str) -> int:
    """Small, self-contained launches for ncu captures (the commands in profiles/ run these).

    decode-bs1 / decode-bs16: the config-2 model (int8, seed 2) after its prompt(s) and three warm-up
    steps; one more decode step runs inside the NVTX range "step" (capture with --nvtx-include "step/").
    gemm-gateup-16: the config-2 gate/up projection (int8 [37888, 3584], SwiGLU) at 16 activation rows on
    the tensor-core GEMM, 3 rotating weight copies (408 MB > L2), 6 warm-up launches then 30 timed.
    attention-512: Attention.Execute at the config-2 head shape (hd 128, 28 query / 4 KV heads, f32
    caches of 4096 rows, 512 live positions), 5 warm-up launches then 50 timed.
    gemm-gateup-512: the gate/up projection of gemm-gateup-16 at 512 activation rows (a prefill chunk).
    attention-tp8: decode attention at one config-4 TP8 rank's heads (8 query / 1 KV head, hd 128, bf16
    caches, 2112 positions): the tensor-core kernel in 16-CTA clusters, 5 warm-up launches then 50 timed.
    decode-bs1-1layer: config 2 cut to one layer, one decode step inside the NVTX range "step".
    decode-cfg4-tp8-shard: one config-4 TP8 rank's shard shapes as a single-GPU model (no all-reduces),
    20 timed device-resident greedy steps after a 2048-token prompt, then one step inside "step".
    """
    import ctypes as C

    import torch

    from l0llm_b200 import levelzero as lz

    dev = lz.ComputeDevice(0)
    suite = lz.LlmKernelSuite.Create(dev)
    sp = C.c_void_p()
    lz.check(lz.load_library().l0b_device_stream(dev.handle, C.byref(sp)))
    rng = np.random.default_rng(SEED)
    if case == "decode-cfg4-tp8-shard":
        # One rank's share of config 4 at TP8 as a single-GPU model: 8 query heads, 1 KV head, intermediate
        # 3584, vocab 16032 give exactly the shard shapes (q/k/v [1280, 8192], o_proj [8192, 1024],
        # gate/up [7168, 8192], down [8192, 3584], lm_head [16032, 8192]), without the all-reduces.
        cfg = dict(CFG4, num_attention_heads=8, num_key_value_heads=1, intermediate_size=3584, vocab_size=16032)
        stream = torch.cuda.ExternalStream(sp.value)
        with lz.LlmModel(dev, suite, lz.model_config(kv_dtype=lz.BF16, **cfg), 2048 + 64, "bfloat16") as model:
            model.init_synthetic(4, 0.02)
            model.Prefill(rng.integers(0, cfg["vocab_size"], 2048).astype(np.int32))
            model.decode_greedy_device(5)
            dev.Synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            model.decode_greedy_device(20)
            e1.record(stream)
            e1.synchronize()
            torch.cuda.nvtx.range_push("step")
            model.decode_greedy_device(1)
            dev.Synchronize()
            torch.cuda.nvtx.range_pop()
            print(json.dumps({"profile_case": case, "ms_per_step": round(e0.elapsed_time(e1) / 20, 4),
                              "weight_bytes": model.ProjectionBytes}))
    elif case in ("decode-bs1", "decode-bs16"):
        batch = 1 if case == "decode-bs1" else BS16
        mc = lz.model_config(kv_dtype=lz.F16, max_batch=batch, **CFG2)
        with lz.LlmModel(dev, suite, mc, CONTEXT + 64, "int8") as model:
            model.init_synthetic(SEED, 0.02, 1e-3, 2e-2)
            for sq in range(batch):
                model.PrefillSequence(sq, rng.integers(0, CFG2["vocab_size"], CONTEXT).astype(np.int32),
                                      want_logits=False)
            step = (lambda n: model.decode_greedy_device(n)) if batch == 1 else \
                (lambda n: model.decode_greedy_device_batch(n, batch))
            step(3)
            dev.Synchronize()
            torch.cuda.nvtx.range_push("step")
            step(1)
            dev.Synchronize()
            torch.cuda.nvtx.range_pop()
        print(json.dumps({"profile_case": case, "ok": True}))
    elif case in ("gemm-gateup-16", "gemm-gateup-512"):
        H, I, copies = CFG2["hidden_size"], CFG2["intermediate_size"], 3
        M = BS16 if case == "gemm-gateup-16" else 512
        N = 2 * I
        qs = [lz.SharedBuffer.from_array(dev, rng.integers(-127, 128, (N, H), dtype=np.int8)) for _ in range(copies)]
        ss = [lz.SharedBuffer.from_array(dev, rng.uniform(1e-3, 2e-2, N).astype(np.float16)) for _ in range(copies)]
        x = lz.SharedBuffer.from_array(dev, rng.standard_normal(M * H).astype(np.float32))
        out = lz.SharedBuffer(dev, lz.F32, M * I)
        L = lz.load_library()

        def run(i):
            lz.check(L.l0b_linear_tc_scaled(suite.handle, dev.handle, M, N, H, x.handle, qs[i % copies].handle,
                                            ss[i % copies].handle, H, None, 0.0, 2 | 0x100, None, out.handle))

        for i in range(6):
            run(i)
        stream = torch.cuda.ExternalStream(sp.value)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dev.Synchronize()
        e0.record(stream)
        for i in range(30):
            run(i)
        e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) / 30 * 1e3
        print(json.dumps({"profile_case": case, "us_per_call_with_cast": round(us, 2),
                          "weight_gbs": round(N * H / us / 1e3, 1)}))
        for b in qs + ss + [x, out]:
            b.Dispose()
    elif case == "attention-tp8":
        # Decode attention at one config-4 TP8 rank's shape: 8 query heads on 1 KV head, bf16 caches,
        # position 2111 (the 2048-token prompt plus decode steps), tensor-core kernel in 16-CTA clusters.
        hd, nh, nkv, seq = 128, 8, 1, 2112
        bits = lambda a: torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        q = lz.SharedBuffer.from_array(dev, rng.standard_normal(nh * hd).astype(np.float32))
        kc = lz.SharedBuffer.from_array(dev, bits(rng.standard_normal(seq * nkv * hd).astype(np.float32)), lz.BF16)
        vc = lz.SharedBuffer.from_array(dev, bits(rng.standard_normal(seq * nkv * hd).astype(np.float32)), lz.BF16)
        out = lz.SharedBuffer(dev, lz.F32, nh * hd)
        for _ in range(5):
            suite.Attention.Execute(dev, q, kc, vc, out, hd, nh, nkv, seq, seq)
        stream = torch.cuda.ExternalStream(sp.value)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dev.Synchronize()
        with torch.cuda.stream(stream):
            torch.cuda._sleep(50_000_000)  # the launches queue behind it: the events time the GPU
        e0.record(stream)
        for _ in range(50):
            suite.Attention.Execute(dev, q, kc, vc, out, hd, nh, nkv, seq, seq)
        e1.record(stream)
        e1.synchronize()
        print(json.dumps({"profile_case": case, "us_per_call": round(e0.elapsed_time(e1) / 50 * 1e3, 2)}))
        for b in (q, kc, vc, out):
            b.Dispose()
    elif case == "decode-bs1-1layer":
        # Config 2 cut to one decoder layer (same shapes and int8 layout, ~3 GB on the device): a small
        # case for full captures of the per-layer kernels; one step inside the NVTX range "step".
        mc = lz.model_config(kv_dtype=lz.F16, **dict(CFG2, num_layers=1))
        with lz.LlmModel(dev, suite, mc, CONTEXT + 64, "int8") as model:
            model.init_synthetic(SEED, 0.02, 1e-3, 2e-2)
            model.Prefill(rng.integers(0, CFG2["vocab_size"], CONTEXT).astype(np.int32))
            model.decode_greedy_device(3)
            dev.Synchronize()
            torch.cuda.nvtx.range_push("step")
            model.decode_greedy_device(1)
            dev.Synchronize()
            torch.cuda.nvtx.range_pop()
        print(json.dumps({"profile_case": case, "ok": True}))
    elif case == "attention-512":
        hd, nh, nkv, seq, max_seq = 128, 28, 4, 512, 4096
        q = lz.SharedBuffer.from_array(dev, rng.standard_normal(nh * hd).astype(np.float32))
        kc = lz.SharedBuffer.from_array(dev, rng.standard_normal(max_seq * nkv * hd).astype(np.float32))
        vc = lz.SharedBuffer.from_array(dev, rng.standard_normal(max_seq * nkv * hd).astype(np.float32))
        out = lz.SharedBuffer(dev, lz.F32, nh * hd)
        for _ in range(5):
            suite.Attention.Execute(dev, q, kc, vc, out, hd, nh, nkv, seq, max_seq)
        stream = torch.cuda.ExternalStream(sp.value)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dev.Synchronize()
        e0.record(stream)
        for _ in range(50):
            suite.Attention.Execute(dev, q, kc, vc, out, hd, nh, nkv, seq, max_seq)
        e1.record(stream)
        e1.synchronize()
        print(json.dumps({"profile_case": case, "us_per_call": round(e0.elapsed_time(e1) / 50 * 1e3, 2)}))
        for b in (q, kc, vc, out):
            b.Dispose()
    else:
        raise SystemExit(f"unknown profile case {case}")
    suite.Dispose()
    dev.Dispose()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-only", action="store_true",
                    help="only the dominant-kernel roofline loop (small device footprint, for ncu captures)")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg3", "cfg4"],
                    help="cfg2: the headline (Qwen2.5-7B int8, one GPU, replicas over N); cfg3: the Gated DeltaNet "
                         "layer alone (bf16, one GPU); cfg4: Llama-3-70B bf16 tensor-parallel over the N ranks")
    ap.add_argument("--no-bulk-gemv", action="store_true",
                    help="one-row projections on the register-streamed GEMV only (l0b_set_gemv_bulk(0))")
    ap.add_argument("--no-legs", action="store_true", help="skip the config 0 / 1 / 3 legs of the bench line")
    ap.add_argument("--nccl-only", action="store_true",
                    help="tensor-parallel all-reduces on NCCL only (no peer-memory all-reduce)")
    ap.add_argument("--pair-allreduce", action="store_true",
                    help="row-split GEMV + separate all-reduce kernel instead of the all-reduce folded into the GEMV")
    ap.add_argument("--no-tp", action="store_true", help="skip the config 4 tensor-parallel leg (tp)")
    ap.add_argument("--tp-batch", type=int, default=1,
                    help="--workload cfg4 only: sequences decoded together (BASELINE config 4 also runs 32), one "
                         "prompt prefilled and forked on the device")
    ap.add_argument("--profile-case", choices=["decode-bs1", "decode-bs16", "gemm-gateup-16", "attention-512",
                                               "decode-cfg4-tp8-shard", "gemm-gateup-512", "attention-tp8",
                                               "decode-bs1-1layer"],
                    help="run one small case for an ncu capture instead of the benchmark")
    args = ap.parse_args()
    if args.no_bulk_gemv:
        from l0llm_b200 import levelzero as lz

        lz.load_library().l0b_set_gemv_bulk(0)
    if args.nccl_only:
        from l0llm_b200 import levelzero as lz

        lz.Communicator.set_peer_allreduce(False)
    if args.pair_allreduce:
        from l0llm_b200 import levelzero as lz

        lz.Communicator.set_fused_allreduce(False)
    if args.profile_case:
        return run_profile_case(args.profile_case)
    if args.impl == "reference":
        return run_reference(args)
    args.warmup = max(3, args.warmup)
    if args.workload == "cfg4":
        return run_cfg4_tp(args)
    if args.workload == "cfg3":
        return run_cfg3_deltanet(args)
    if args.kernel_only:
        import ctypes as C

        import torch

        from l0llm_b200 import levelzero as lz

        dev = lz.ComputeDevice(0)
        suite = lz.LlmKernelSuite.Create(dev)
        sp = C.c_void_p()
        lz.check(lz.load_library().l0b_device_stream(dev.handle, C.byref(sp)))
        peak, kind = peaks()
        print(json.dumps(dominant_kernel_roofline(lz, dev, suite, sp.value, torch, peak, kind,
                                                  bulk=not args.no_bulk_gemv)))
        suite.Dispose()
        dev.Dispose()
        return 0

    world, rank, local = dist_env()
    import torch

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        pg = dist

    from l0llm_b200 import levelzero as lz

    peak, peak_kind = peaks()
    dev = lz.ComputeDevice(local)
    suite = lz.LlmKernelSuite.Create(dev)
    import ctypes as C

    sp = C.c_void_p()
    lz.check(lz.load_library().l0b_device_stream(dev.handle, C.byref(sp)))
    stream = torch.cuda.ExternalStream(sp.value)

    # Sequence 0 carries the bs1 measurement (warm-up, timed steps, end-to-end steps), then all BS16
    # sequences decode together; the cache holds every step of sequence 0.
    max_seq = CONTEXT + 2 * args.warmup + 3 * args.steps + 16
    mc = lz.model_config(kv_dtype=lz.F16, max_batch=BS16, **CFG2)
    model = lz.LlmModel(dev, suite, mc, max_seq, "int8")
    model.init_synthetic(SEED, 0.02, 1e-3, 2e-2)
    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, 152064, CONTEXT).astype(np.int32)
    # prefill_s: a warm prefill (the first one also pays one-time kernel loading and plan setup).
    model.Prefill(prompt)
    model.ResetSequence()
    t0 = time.perf_counter()
    model.Prefill(prompt)
    prefill_s = time.perf_counter() - t0
    proj_bytes = model.ProjectionBytes

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    # Warm-up (graph capture happens here), then the timed device-resident decode. The clock sampler
    # runs from before the warm-up and keeps only the samples taken inside the timed region.
    sampler = ClockSampler(local)
    sampler.start()
    model.decode_greedy_device(args.warmup)
    pos_start = model.Position
    launches0 = lz.kernel_launch_count()
    barrier()
    t_begin = time.monotonic()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    model.decode_greedy_device(args.steps)
    e1.record(stream)
    e1.synchronize()
    sampler.mark(t_begin, time.monotonic())
    barrier()
    ms = e0.elapsed_time(e1)
    launches = lz.kernel_launch_count() - launches0
    clocks = sampler.stop()

    # End to end through the public call: token/position in, full logits out, argmax on the host.
    logits = np.zeros(model.vocab, np.float32)
    tok = int(np.argmax(model.Decode(1, logits)))
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        model.Decode(tok, logits)
        tok = int(np.argmax(logits))
    f1.record(stream)
    f1.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1)

    # Batch 16: the other sequences get their own 512-token prompts, then device-resident greedy
    # decoding of all 16 at their own positions (one CUDA graph per step).
    for sq in range(1, BS16):
        model.PrefillSequence(sq, rng.integers(0, 152064, CONTEXT).astype(np.int32), want_logits=False)
    model.decode_greedy_device_batch(args.warmup, BS16)
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    model.decode_greedy_device_batch(args.steps, BS16)
    g1.record(stream)
    g1.synchronize()
    barrier()
    bs16_ms = g0.elapsed_time(g1)

    roof = dominant_kernel_roofline(lz, dev, suite, sp.value, torch, peak, peak_kind, bulk=not args.no_bulk_gemv)

    if pg is not None:
        t = torch.tensor([ms, e2e_ms, bs16_ms], dtype=torch.float64, device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, e2e_ms, bs16_ms = float(t[0]), float(t[1]), float(t[2])
    proj_bytes_cfg2 = model.ProjectionBytes
    model.Dispose()

    # The other BASELINE configurations (one GPU, rank 0 of a single-rank run) and config 4 tensor-parallel
    # over all ranks of the job.
    legs = {}
    if world == 1 and not args.no_legs:
        tf_peak = tflops_peak()
        legs["cfg0"] = measure_cfg0(lz, dev, suite, sp.value, torch, peak, peak_kind, tf_peak)
        legs["cfg1"] = measure_cfg1(lz, dev, suite, sp.value, torch, peak, args.steps, args.warmup)
        legs["cfg3"] = measure_cfg3(lz, dev, suite, sp.value, torch, args.warmup)
    tp = None
    if not args.no_tp:
        barrier()
        tp = measure_cfg4_tp(lz, dev, suite, sp.value, torch, pg, world, rank, local, args.steps, args.warmup)

    tokens = world * args.steps
    value = tokens / (ms / 1e3)
    e2e = tokens / (e2e_ms / 1e3)
    kv_bytes = 28 * 2 * 512 * 2 * (pos_start + args.steps / 2)
    step_bytes = proj_bytes_cfg2 + kv_bytes
    step_gbs = step_bytes / (ms / args.steps * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(budget_s=25.0)
        # The same CPU port beside each of the other configurations' GPU legs (bounded samples).
        try:
            cl = cpu_legs(budget_s=20.0)
        except Exception as e:  # a baseline that failed is reported, not fatal to the GPU line
            cl = {k: {"error": f"{type(e).__name__}: {e}"} for k in ("cfg0", "cfg1", "cfg3", "cfg4")}
        for key in ("cfg0", "cfg1", "cfg3"):
            if key in legs:
                legs[key]["cpu_baseline"] = cl[key]
        if tp is not None:
            tp["cpu_baseline"] = cl["cfg4"]
    suite.Dispose()
    dev.Dispose()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "config 2: Qwen2.5-7B-shape int8 decode, bs1, 512-token context, fp16 KV",
                       "model": "Qwen2.5-7B-shape (28 layers, hidden 3584, 28/4 heads, inter 18944, vocab 152064)",
                       "global_batch": world, "seq_len": CONTEXT, "weights": "int8 per-channel, fp16 scales",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: 7.07 GB of weights streamed per step"},
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4 * 152064},
            "roofline": roof,
            "step_roofline": {"bytes_per_step": int(step_bytes), "achieved_gbs": round(step_gbs, 1), "peak": peak,
                              "frac": round(step_gbs / peak, 4), "roofline_tok_s": round(peak * 1e9 / step_bytes, 1)},
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "prefill_s": round(prefill_s, 3),
            "bs16": {"value": round(world * BS16 * args.steps / (bs16_ms / 1e3), 1), "unit": "tok/s",
                     "ms_per_step": round(bs16_ms / args.steps, 4), "sequences": BS16 * world,
                     "context": f"{CONTEXT}-token prompts, positions {CONTEXT}..{CONTEXT + args.warmup + args.steps}"},
        }
        line.update(legs)
        if tp is not None:
            line["tp"] = tp
        print(json.dumps(line))
    if pg is not None:
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
