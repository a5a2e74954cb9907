#!/usr/bin/env python3
"""Benchmarks of the decode hot path.

Default workload (--workload decode): batch-1 greedy
decoding of the synthetic Qwen3.8-27B Q4_K_M model - a seeded GGUF with the
upstream loader's exact tensor names, shapes, metadata and layer pattern, its
quantized weights drawn as in config 0 (q38b200.gguf, dist "config0"); a
128-token random prompt is prefilled, then tokens are generated greedily at a
4096-token context.  A step is one decoded token (all 64 layers, the LM head
and the argmax), run as one replay of the captured decode graph with the next
token fed back on the device.

  value   decoded tokens/s summed over ranks (each rank runs its own replica:
          weak scaling); weights (15.5 GB) stream from HBM every step.
  e2e     the same metric through the upstream-named public API with host
          buffers: q38_model_forward_token per step (token and position to the
          device, the 248,320 fp32 logits back to pinned host memory) and the
          argmax taken on the host, as the upstream CLI's loop does.
  roofline  algorithmic bytes of one step (every weight read once, the
          DeltaNet state read and written, KV rows read) / time per step.
  mtp     speculative decoding (q38_model_speculative_greedy) on the same model.

--workload matvec: one Q4_K x Q8_K matvec 17408 x 5120,
value in GB/s of algorithmic bytes, weights rotating over distinct copies;
--qtype IQ1_M / IQ2_S (and --shape 5120x17408) give BASELINE config 1.

`--impl reference` times the upstream engine's own CPU implementation of the
workload (built from its sources into oracle/_ref/) on this host's cores.
"""
import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen3.8-27b-in-c_b200", "python"))

import numpy as np  # noqa: E402

METRIC = "decode tok/s (Q4_K_M, bs1, MTP on/off); quant matvec HBM GB/s vs 8 TB/s peak"
UNIT = "GB/s"        # matvec workload
DECODE_UNIT = "tok/s"
Q4_K = 12
# The matvec case (set_matvec_case): BASELINE config 0 by default, config 1
# with --qtype IQ1_M / IQ2_S (IQ2_M's main type) and either shape.
QTYPE = Q4_K
ROWS, WIDTH = 17408, 5120
W_BYTES = X_BYTES = Y_BYTES = STEP_BYTES = 0
COPIES = 8                                      # >= 139 MB of weights > 126 MB L2
NOMINAL_HBM_GBS = 8000.0
WORKLOAD = ""
MATVEC_TYPES = {"Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16,
                "IQ2_XS": 17, "IQ3_XXS": 18, "IQ1_S": 19, "IQ3_S": 21, "IQ2_S": 22,
                "IQ4_XS": 23, "IQ1_M": 29}
CONFIG1_TYPES = (19, 22, 29)   # the IQ1_M/IQ2_M mixes of BASELINE config 1


def set_matvec_case(qtype_name="Q4_K", shape="17408x5120"):
    """Weight type and [rows x width] of the matvec workload; the algorithmic
    bytes are the GGUF weight bytes, the Q8_K activation and the fp32 output."""
    global QTYPE, ROWS, WIDTH, W_BYTES, X_BYTES, Y_BYTES, STEP_BYTES, WORKLOAD
    from q38b200 import synth
    QTYPE = MATVEC_TYPES[qtype_name]
    ROWS, WIDTH = (int(v) for v in shape.split("x"))
    elements, nbytes = synth.BLOCK[QTYPE]
    W_BYTES = ROWS * (WIDTH // elements) * nbytes       # Q4_K 17408x5120: 50,135,040
    X_BYTES = WIDTH // 256 * 292                         # Q8_K activation
    Y_BYTES = ROWS * 4
    STEP_BYTES = W_BYTES + X_BYTES + Y_BYTES
    config = "config0" if QTYPE == Q4_K else "config1" if QTYPE in CONFIG1_TYPES else "matvec"
    WORKLOAD = f"{config}: {qtype_name} {ROWS}x{WIDTH} x Q8_K matvec, bs1"


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as handle:
            data = json.load(handle)
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def read_traffic():
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "q4k_gemv_17408x5120.md")
    if QTYPE != Q4_K or (ROWS, WIDTH) != (17408, 5120) or not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("dram_bytes_per_launch:"):
            return int(line.split(":")[1].strip().replace(",", ""))
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x0000000000000002: "applications_clocks_setting",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._handle, self._nvml.NVML_CLOCK_SM))
                mask = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self._nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def cpu_reference_gemv(seconds=3.0, min_calls=20):
    """Time the upstream CPU kernel on this host (all cores, OpenMP)."""
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    os.environ.setdefault("OMP_PROC_BIND", "close")
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from q38b200 import synth
    weights = synth.quant_tensor(QTYPE, ROWS, WIDTH, seed=0)
    x = synth.activations(1, WIDTH, seed=1)
    copies = [weights] + [weights.copy() for _ in range(COPIES - 1)]
    if O.reference_available():
        impl, kind = O.Reference(), "reference"
        threads = int(os.environ["OMP_NUM_THREADS"])
    else:
        impl, kind = O.Oracle(), "port"
        threads = 1
    q8k = impl.quantize_q8_k(x)
    times = []
    start = time.perf_counter()
    i = 0
    while (time.perf_counter() - start < seconds or len(times) < min_calls) and len(times) < 10000:
        w = copies[i % COPIES]
        t0 = time.perf_counter()
        impl.gemm_q8_k(QTYPE, w, ROWS, WIDTH, q8k)
        times.append(time.perf_counter() - t0)
        i += 1
        if kind == "port" and time.perf_counter() - start > seconds:
            break
    med = statistics.median(times)
    return {"value": STEP_BYTES / med / 1e9, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{len(times)} full {WORKLOAD.split(': ')[1].split(' x')[0]} matvecs rotating {COPIES} weight copies; "
                      f"median {med * 1e3:.3f} ms"}


def run_matvec_reference(args, rank):
    if rank != 0:
        return
    base = cpu_reference_gemv(seconds=max(2.0, 0.02 * args.steps))
    line = {"metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference", "dtype": "int8xint8->int32,f32",
            "data": "synthetic", "scaling": "weak",
            "config": {"workload": WORKLOAD, "l2": f"rotating {COPIES} weight copies"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "vs_baseline": None}
    print(json.dumps(line), flush=True)


def capture(fn, count):
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(count):
            fn(i)
    return g


def run_matvec(args, rank, world, dist):
    import torch
    import q38b200 as q38
    from q38b200 import synth

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    weights = synth.quant_tensor(QTYPE, ROWS, WIDTH, seed=0)
    x_host = synth.activations(1, WIDTH, seed=1)
    tensors = [q38.DeviceTensor(QTYPE, WIDTH, ROWS, weights, layout=q38.LAYOUT_TILED)
               for _ in range(COPIES)]
    x_dev = torch.from_numpy(x_host).cuda()
    act = q38.quantize_q8_k(x_dev)
    out = torch.empty((1, ROWS), dtype=torch.float32, device="cuda")

    def step(i):
        q38.gemm_q8_k(tensors[i % COPIES], act, 1, out=out)

    # Uncaptured first call: sets kernel attributes and caches the plan.
    step(0)
    torch.cuda.synchronize()
    if args.profile:
        # Plain launches for ncu: warmup + steps, nothing else on the device.
        for i in range(args.warmup + args.steps):
            step(i)
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"profile_run": WORKLOAD, "launches": 1 + args.warmup + args.steps}), flush=True)
        return
    chunk = 64
    full_graph = capture(step, chunk)
    rem = args.steps % chunk
    rem_graph = capture(step, rem) if rem else None
    warm_graph = capture(step, args.warmup)

    warm_graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps // chunk):
            full_graph.replay()
        if rem_graph:
            rem_graph.replay()
        end.record()
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_per_step = max_ms / args.steps
    value = STEP_BYTES * args.steps * world / (max_ms / 1e3) / 1e9
    per_gpu = STEP_BYTES / (ms_per_step / 1e3) / 1e9

    # End-to-end through the C ABI with host buffers.
    x_pinned = torch.from_numpy(x_host).pin_memory()
    y_pinned = torch.empty((1, ROWS), dtype=torch.float32).pin_memory()
    e2e_steps = min(args.steps, 2000)

    def e2e_step(i):
        x_dev.copy_(x_pinned, non_blocking=True)
        q38.quantize_q8_k(x_dev, out=act)
        q38.gemm_q8_k(tensors[i % COPIES], act, 1, out=out)
        y_pinned.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(max(3, args.warmup)):
        e2e_step(i)
    if dist:
        dist.barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(e2e_steps):
        e2e_step(i)
    e2.record()
    torch.cuda.synchronize()
    t2 = torch.tensor([s2.elapsed_time(e2)], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_value = STEP_BYTES * e2e_steps * world / (float(t2.item()) / 1e3) / 1e9

    status = q38.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}: a kernel abandoned a bounded wait")

    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    cpu = cpu_reference_gemv(seconds=3.0) if world == 1 else None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xint8->int32,f32", "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "rows": ROWS, "width": WIDTH, "batch": 1,
                   "algorithmic_bytes_per_step": STEP_BYTES,
                   "l2": f"inputs larger than L2: {COPIES} rotating weight copies ({COPIES * W_BYTES / 1e6:.0f} MB)",
                   "parallelism": f"replica per GPU x{world}"},
        "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                     "peak_source": peak_kind, "frac_of_nominal_8tbs": per_gpu / NOMINAL_HBM_GBS,
                     "traffic": read_traffic(), "timing": "CUDA events over graph-replayed launches"},
        "e2e": {"value": e2e_value, "unit": UNIT, "steps": e2e_steps,
                "h2d_bytes_per_step": WIDTH * 4, "d2h_bytes_per_step": ROWS * 4},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# config 3: full-model greedy decode
# ---------------------------------------------------------------------------
PROMPT_TOKENS = 128
CONTEXT = 4096
VOCAB = 248320
MODEL_SEED = 0
MIX = "Q4_K_M"   # --mix: the model's type mix (gguf.MIXES); IQ1_M is config 4's IQ1_M-typed variant
DECODE_WORKLOAD = ""


def set_decode_mix(mix="Q4_K_M"):
    global MIX, DECODE_WORKLOAD
    MIX = mix
    config = "config3" if mix == "Q4_K_M" else "config4 IQ1_M-typed variant"
    DECODE_WORKLOAD = (f"{config}: synthetic Qwen3.8-27B {mix} GGUF (upstream loader contract, config-0 weight "
                       "draws), 128-token random prompt, greedy decode bs1, ctx 4096, MTP off")


def decode_model_path(rank, dist):
    """The synthetic model file, written once per machine (rank 0 first)."""
    from q38b200 import gguf
    path = gguf.cached_model_path(seed=MODEL_SEED, mtp=True, dist="config0", mix=MIX) if rank == 0 else None
    if dist:
        dist.barrier()
    if path is None:
        path = gguf.cached_model_path(seed=MODEL_SEED, mtp=True, dist="config0", mix=MIX)
    return path


def decode_weight_bytes():
    """Weight bytes one decode step reads: every tensor of the 64 target layers,
    the output norm and LM head, and one embedding row (the MTP layer is not
    part of a target step)."""
    from q38b200 import gguf, synth
    total = 0
    for name, shape, qtype in gguf.tensor_specs(mtp=False, mix=MIX):
        elements, nbytes = synth.BLOCK[qtype]
        size = int(np.prod(shape)) // elements * nbytes
        if name == "token_embd.weight":
            size = shape[0] // elements * nbytes
        total += size
    return total


STATE_BYTES = 48 * 48 * 128 * 128 * 4 * 2        # DeltaNet state, read and written
CONV_BYTES = 48 * 10240 * 4 * 4                  # conv ring: 3 taps read, 1 written
KV_ROW_BYTES = 16 * 1024 * 4 * 2                 # K and V rows of the 16 attention layers


def decode_step_bytes(position):
    """Algorithmic bytes of the decode step at `position`: weights + recurrent
    state + the KV rows it scans (positions 0..position) and writes."""
    return decode_weight_bytes() + STATE_BYTES + CONV_BYTES + KV_ROW_BYTES * (position + 2)


def read_step_traffic():
    path = os.path.join(ROOT, "profiles", "decode_step_config3.md")
    if MIX != "Q4_K_M" or not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("dram_bytes_per_step:"):
            return int(line.split(":")[1].strip().replace(",", ""))
    return None


def cpu_reference_decode(path, tokens, prompt):
    """Greedy decode with the upstream Q38Model on this host's cores: the
    prompt is prefilled (untimed), then `tokens` forward_token + argmax steps
    are timed."""
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    os.environ.setdefault("OMP_PROC_BIND", "close")
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not O.reference_available():
        return None
    ref = O.ReferenceModel(path, CONTEXT)
    token = int(np.argmax(ref.prefill(prompt)))
    t0 = time.perf_counter()
    for _ in range(tokens):
        token = int(np.argmax(ref.forward_token(token)))
    elapsed = time.perf_counter() - t0
    ref.close()
    return {"value": tokens / elapsed, "unit": DECODE_UNIT, "cores": int(os.environ["OMP_NUM_THREADS"]),
            "kind": "reference",
            "sample": f"upstream q38_model_forward_token + argmax, {tokens} greedy tokens after a "
                      f"{len(prompt)}-token prefill; {elapsed / tokens * 1e3:.1f} ms/token"}


def decode_prompt():
    return np.random.default_rng(1234).integers(0, VOCAB, PROMPT_TOKENS).tolist()


def run_decode_reference(args, rank, world, dist):
    path = decode_model_path(rank, dist)
    if rank != 0:
        return
    tokens = max(4, min(args.steps, 32))
    base = cpu_reference_decode(path, tokens, decode_prompt())
    if base is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libq38ref.so is not built"}), flush=True)
        return
    line = {"metric": METRIC, "value": base["value"], "unit": DECODE_UNIT, "n_gpus": args.gpus,
            "steps": tokens, "warmup": args.warmup, "ms_per_step": 1e3 / base["value"],
            "higher_is_better": True, "impl": "reference", "dtype": "int8xint8->int32,f32",
            "data": "synthetic (seeded)", "scaling": "weak",
            "config": {"workload": DECODE_WORKLOAD, "prompt": PROMPT_TOKENS, "context": CONTEXT},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": DECODE_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "vs_baseline": None}
    print(json.dumps(line), flush=True)


def run_decode(args, rank, world, dist):
    import torch
    from q38b200.model import Model

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    path = decode_model_path(rank, dist)
    m = Model(path, CONTEXT)
    stream = torch.cuda.ExternalStream(m.stream)
    prompt = decode_prompt()
    kernels = m.step_kernels

    def fresh():
        m.reset()
        return int(np.argmax(m.prefill(prompt)))

    def timed(fn):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        out = fn()
        end.record(stream)
        end.synchronize()
        return start.elapsed_time(end), out

    if args.profile:
        # For ncu (--profile-from-start off): W warm steps, then exactly one
        # decode step (one graph replay) between profiler start and stop.
        token = fresh()
        token = m.generate_greedy(token, args.warmup)[-1]
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        m.generate_greedy(token, 1)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        m.close()
        if rank == 0:
            print(json.dumps({"profile_run": DECODE_WORKLOAD, "profiled_steps": 1, "kernels_per_step": kernels}),
                  flush=True)
        return

    # W untimed warm-up steps, then exactly K timed steps in runs that fit the
    # context (a reset and a fresh prefill between runs are not timed).
    token = fresh()
    token = m.generate_greedy(token, args.warmup)[-1]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    elapsed_ms, step_bytes, left = 0.0, 0, args.steps
    with ClockSampler(local) as clocks:
        while left:
            if CONTEXT - m.position < 2:
                token = fresh()
            n = min(left, CONTEXT - m.position - 1)
            pos0 = m.position
            ms, toks = timed(lambda: m.generate_greedy(token, n))
            elapsed_ms += ms
            step_bytes += sum(decode_step_bytes(pos0 + i) for i in range(n))
            token = toks[-1]
            left -= n
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_per_step = max_ms / args.steps
    value = args.steps * world / (max_ms / 1e3)
    bytes_per_step = step_bytes / args.steps
    achieved = bytes_per_step / (ms_per_step / 1e3) / 1e9

    # End to end: the upstream-named API with host buffers, argmax on the host.
    token = fresh()
    for _ in range(3):
        token = int(np.argmax(m.forward_token(token)))
    e2e_steps = min(args.steps, 64)

    def e2e_loop():
        tok = token
        for _ in range(e2e_steps):
            tok = int(np.argmax(m.forward_token(tok)))
        return tok

    e2e_ms, _ = timed(e2e_loop)
    t2 = torch.tensor([e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_value = e2e_steps * world / (float(t2.item()) / 1e3)

    # MTP on: speculative greedy decoding at draft depths 1 and 3 (the
    # upstream's spec bench sweeps depths 1..4, qwen38_spec_bench.c:108-119).
    mtp = {}
    for drafts in (1, 3):
        m.reset()
        m.enable_mtp()
        token = int(np.argmax(m.prefill(prompt)))
        m.speculative_greedy(token, 0xFFFFFFFF, drafts)  # captures the draft and verification graphs
        m.reset()
        m.enable_mtp()
        token = int(np.argmax(m.prefill(prompt)))
        target = 48

        def spec_loop():
            tok, produced, calls = token, 0, 0
            while produced < target:
                accepted, _ = m.speculative_greedy(tok, 0xFFFFFFFF, drafts)
                produced += len(accepted)
                calls += 1
                tok = accepted[-1]
            return produced, calls

        mtp_ms, (produced, calls) = timed(spec_loop)
        mtp[f"depth_{drafts}"] = {"value": produced * world / (mtp_ms / 1e3), "unit": DECODE_UNIT,
                                  "draft_count": drafts, "tokens": produced, "calls": calls,
                                  "tokens_per_call": produced / calls, "ms_per_call": mtp_ms / calls}
    m.close()

    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    cpu = cpu_reference_decode(path, 16, prompt) if world == 1 else None
    line = {
        "metric": METRIC, "value": value, "unit": DECODE_UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xint8->int32,f32", "data": "synthetic (seeded GGUF, config-0 draws)",
        "config": {"workload": DECODE_WORKLOAD, "prompt": PROMPT_TOKENS, "context": CONTEXT, "batch": 1,
                   "mtp": "off", "weights_bytes_per_step": decode_weight_bytes(),
                   "l2": f"inputs larger than L2: {decode_weight_bytes() / 1e9:.1f} GB of weights stream every step",
                   "parallelism": f"replica per GPU x{world}"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS,
                     "traffic": read_step_traffic(), "algorithmic_bytes_per_step": bytes_per_step,
                     "unit_of_launch": "one decode step (one graph replay)",
                     "timing": "CUDA events on the model stream around K graph replays"},
        "e2e": {"value": e2e_value, "unit": DECODE_UNIT, "steps": e2e_steps, "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": VOCAB * 4, "api": "q38_model_forward_token + host argmax"},
        "mtp": dict(mtp, note="random-weight MTP head: drafts are almost never accepted, so each call yields "
                              "one token and costs the drafts plus a verification of depth tokens"),
        "gpu_launches": kernels * args.steps,
        "kernels_per_step": kernels,
        "clocks": clocks.summary(),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None)
    parser.add_argument("--warmup", type=int, default=None)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--workload", choices=("decode", "matvec"), default="decode")
    parser.add_argument("--qtype", choices=sorted(MATVEC_TYPES), default="Q4_K",
                        help="matvec workload: weight type (IQ1_M and IQ2_S give BASELINE config 1)")
    parser.add_argument("--shape", choices=("17408x5120", "5120x17408"), default="17408x5120",
                        help="matvec workload: rows x width")
    parser.add_argument("--profile", action="store_true",
                        help="plain launches only, for ncu: matvec - warmup + steps launches; decode - one decode "
                             "step between cudaProfilerStart/Stop; prints no bench line")
    parser.add_argument("--mix", choices=("Q4_K_M", "IQ1_M"), default="Q4_K_M",
                        help="decode workload: the model's type mix (IQ1_M: BASELINE config 4's IQ1_M-typed variant)")
    args = parser.parse_args()
    set_matvec_case(args.qtype, args.shape)
    set_decode_mix(args.mix)
    decode = args.workload == "decode"
    if args.steps is None:
        args.steps = 256 if decode else 20000
    if args.warmup is None:
        args.warmup = 3 if decode else 20
    assert args.warmup >= 3, "at least 3 warm-up steps"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as torch_dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        torch_dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        dist = torch_dist
    try:
        if args.impl == "reference":
            if decode:
                run_decode_reference(args, rank, world, dist)
            else:
                run_matvec_reference(args, rank)
        elif decode:
            run_decode(args, rank, world, dist)
        else:
            run_matvec(args, rank, world, dist)
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
