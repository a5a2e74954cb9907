#!/usr/bin/env python3
"""Benchmarks of the decode hot path.

Default workload (--workload decode): batch-1 greedy
decoding of the synthetic Qwen3.8-27B Q4_K_M model - a seeded GGUF with the
upstream loader's exact tensor names, shapes, metadata and layer pattern, its
quantized weights drawn as in config 0 (q38b200.gguf, dist "config0"); a
128-token random prompt is prefilled, then tokens are generated greedily.  A
step is one decoded token (all 64 layers, the LM head and the argmax), run as
one replay of the captured decode graph with the next token fed back on the
device.

  value   decoded tokens/s of the job; weights (15.5 GB) stream from HBM every
          step.  At N = 1 one GPU decodes; at N > 1 (torchrun) every rank holds
          one tensor-parallel shard of the same model and the N GPUs decode one
          sequence together (strong scaling).
  e2e     the same metric through the upstream-named public API with host
          buffers: q38_model_forward_token per step (token and position to the
          device, the 248,320 fp32 logits back to pinned host memory) and the
          argmax taken on the host, as the upstream CLI's loop does.
  roofline  algorithmic bytes of one step (every weight read once, the
          DeltaNet state read and written, KV rows read) / time per step.
  mtp     speculative decoding (q38_model_speculative_greedy) at draft depths
          1..4, and the cost of one verification pass of n tokens.
  subrecords (N = 1): the other BASELINE configs, each with its own CUDA-event
          timing, roofline and CPU baseline - config 0 and config 1 matvecs,
          the config 2 verification block at M = 1, 2, 4, 8, and config 4's
          4096-token prefill (time to first token) followed by 512 decode
          tokens.

--workload matvec / verify / prefill runs one of those alone (--qtype IQ1_M /
IQ2_S and --shape 5120x17408 select the matvec case).

`--impl reference` times the upstream engine's own CPU implementation of the
workload (built from its sources into oracle/_ref/) on this host's cores.
"""
import argparse
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
GBS = "GB/s"
TOKS = "tok/s"
NOMINAL_HBM_GBS = 8000.0
COPIES = 8                                      # rotating weight copies: >= 139 MB > 126 MB L2
MATVEC_TYPES = {"Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16,
                "IQ2_XS": 17, "IQ3_XXS": 18, "IQ1_S": 19, "IQ3_S": 21, "IQ2_S": 22,
                "IQ4_XS": 23, "IQ1_M": 29}
CONFIG1_TYPES = (19, 22, 29)   # the IQ1_M/IQ2_M mixes of BASELINE config 1
Q4_K, Q6_K = 12, 14


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as handle:
            data = json.load(handle)
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def roofline(achieved_gbs, extra=None):
    peak, kind = measured_peaks()
    out = {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": GBS, "frac": achieved_gbs / peak,
           "peak_source": kind, "frac_of_nominal_8tbs": achieved_gbs / NOMINAL_HBM_GBS,
           # DRAM bytes need a profiler capture; per-kernel ncu figures are in
           # the profiles directory, not measured in this run
           "traffic": None}
    out.update(extra or {})
    return out


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


def cpu_setup():
    """OpenMP on every host core, and the upstream build this host runs best."""
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    os.environ.setdefault("OMP_PROC_BIND", "close")
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    lib, flags = O.baseline_reference_lib()
    return O, lib, flags, int(os.environ["OMP_NUM_THREADS"])


def capture(fn, count):
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(count):
            fn(i)
    return g


def timed_graph(step, launches, warmup, chunk=64):
    """CUDA-event time (ms) of `launches` calls of step(i), replayed from
    captured graphs of `chunk` calls after `warmup` untimed ones."""
    import torch
    step(0)  # uncaptured first call: kernel attributes and plans
    torch.cuda.synchronize()
    full = capture(step, chunk)
    rem = launches % chunk
    rem_graph = capture(step, rem) if rem else None
    warm = capture(step, max(3, warmup))
    warm.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(launches // chunk):
        full.replay()
    if rem_graph:
        rem_graph.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end)


# ---------------------------------------------------------------------------
# configs 0 and 1: one quantized matvec
# ---------------------------------------------------------------------------
def matvec_case(qtype_name, shape):
    from q38b200 import synth
    qtype = MATVEC_TYPES[qtype_name]
    rows, width = (int(v) for v in shape.split("x"))
    elements, nbytes = synth.BLOCK[qtype]
    w_bytes = rows * (width // elements) * nbytes       # Q4_K 17408x5120: 50,135,040
    step_bytes = w_bytes + width // 256 * 292 + rows * 4  # + Q8_K activation + fp32 output
    config = "config0" if qtype == Q4_K else "config1" if qtype in CONFIG1_TYPES else "matvec"
    return {"qtype": qtype, "qtype_name": qtype_name, "rows": rows, "width": width, "w_bytes": w_bytes,
            "step_bytes": step_bytes,
            "workload": f"{config}: {qtype_name} {rows}x{width} x Q8_K matvec, bs1"}


def cpu_matvec(case, seconds=3.0, min_calls=20):
    """The upstream CPU kernel (q38_tensor_gemv_q8_k) on this host's cores."""
    from q38b200 import synth
    O, lib, flags, threads = cpu_setup()
    weights = synth.quant_tensor(case["qtype"], case["rows"], case["width"], seed=0)
    x = synth.activations(1, case["width"], seed=1)
    copies = [weights] + [weights.copy() for _ in range(COPIES - 1)]
    if os.path.exists(lib):
        impl, kind = O.Reference(lib), "reference"
    else:
        impl, kind, threads, flags = O.Oracle(), "port", 1, "project C restatement, scalar"
    q8k = impl.quantize_q8_k(x)
    for i in range(3):  # warm-up
        impl.gemm_q8_k(case["qtype"], copies[i], case["rows"], case["width"], q8k)
    times, start, i = [], time.perf_counter(), 0
    while (time.perf_counter() - start < seconds or len(times) < min_calls) and len(times) < 10000:
        t0 = time.perf_counter()
        impl.gemm_q8_k(case["qtype"], copies[i % COPIES], case["rows"], case["width"], q8k)
        times.append(time.perf_counter() - t0)
        i += 1
        if kind == "port" and time.perf_counter() - start > seconds:
            break
    med = statistics.median(times)
    return {"value": case["step_bytes"] / med / 1e9, "unit": GBS, "cores": threads, "kind": kind,
            "sample": f"{len(times)} {case['qtype_name']} {case['rows']}x{case['width']} matvecs rotating "
                      f"{COPIES} weight copies, median {med * 1e3:.3f} ms; {flags}"}


def measure_matvec(case, launches=4000, warmup=20, e2e_steps=1000, with_cpu=True):
    """Device matvec: graph-replayed launches over COPIES rotating weight
    copies (> L2), then end to end through the C ABI with host buffers."""
    import torch
    import q38b200 as q38
    from q38b200 import synth
    rows, width, qtype = case["rows"], case["width"], case["qtype"]
    weights = synth.quant_tensor(qtype, rows, width, seed=0)
    x_host = synth.activations(1, width, seed=1)
    tensors = [q38.DeviceTensor(qtype, width, rows, weights, layout=q38.LAYOUT_TILED) for _ in range(COPIES)]
    x_dev = torch.from_numpy(x_host).cuda()
    act = q38.quantize_q8_k(x_dev)
    out = torch.empty((1, rows), dtype=torch.float32, device="cuda")

    def step(i):
        q38.gemm_q8_k(tensors[i % COPIES], act, 1, out=out)

    with ClockSampler(torch.cuda.current_device()) as clocks:
        ms = timed_graph(step, launches, warmup)
    us = ms * 1e3 / launches
    gbs = case["step_bytes"] / (us * 1e-6) / 1e9

    x_pinned = torch.from_numpy(x_host).pin_memory()
    y_pinned = torch.empty((1, rows), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        x_dev.copy_(x_pinned, non_blocking=True)
        q38.quantize_q8_k(x_dev, out=act)
        q38.gemm_q8_k(tensors[i % COPIES], act, 1, out=out)
        y_pinned.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(3):
        e2e_step(i)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(e2e_steps):
        e2e_step(i)
    e2.record()
    torch.cuda.synchronize()
    e2e_gbs = case["step_bytes"] * e2e_steps / (s2.elapsed_time(e2) / 1e3) / 1e9
    if q38.device_status() != 0:
        raise RuntimeError("device status: a kernel abandoned a bounded wait")
    rec = {"workload": case["workload"], "value": gbs, "unit": GBS, "us_per_launch": us, "launches": launches,
           "warmup": warmup, "higher_is_better": True,
           "algorithmic_bytes_per_launch": case["step_bytes"],
           "l2": f"inputs larger than L2: {COPIES} rotating weight copies ({COPIES * case['w_bytes'] / 1e6:.0f} MB)",
           "roofline": roofline(gbs, {"timing": "CUDA events over graph-replayed launches"}),
           "e2e": {"value": e2e_gbs, "unit": GBS, "steps": e2e_steps, "h2d_bytes_per_step": width * 4,
                   "d2h_bytes_per_step": rows * 4,
                   "api": "q38cu_quantize_q8_k + q38cu_tensor_gemv_q8_k, host x in, host y out"},
           "gpu_launches": launches, "clocks": clocks.summary()}
    if with_cpu:
        rec["cpu_baseline"] = cpu_matvec(case)
    for t in tensors:
        t.free()
    return rec


# ---------------------------------------------------------------------------
# config 2: the verification block of one decoder layer at M = 1, 2, 4, 8
# ---------------------------------------------------------------------------
# One full-attention layer's projections in the Q4_K_M mix:
# (name, rows, width, type)
VERIFY_PROJS = [("attn_q", 12288, 5120, Q4_K), ("attn_k", 1024, 5120, Q4_K), ("attn_v", 1024, 5120, Q6_K),
                ("attn_output", 5120, 6144, Q4_K), ("ffn_gate", 17408, 5120, Q4_K),
                ("ffn_up", 17408, 5120, Q4_K), ("ffn_down", 5120, 17408, Q6_K)]
VERIFY_MS = (1, 2, 4, 8)


def verify_bytes(m):
    from q38b200 import synth
    total = 0
    for _, rows, width, qtype in VERIFY_PROJS:
        total += rows * (width // 256) * synth.BLOCK[qtype][1] + m * (width // 256) * 292 + m * rows * 4
    return total


def cpu_verify(reps=3):
    from q38b200 import synth
    O, lib, flags, threads = cpu_setup()
    if not os.path.exists(lib):
        return None
    ref = O.Reference(lib)
    mats = [(qtype, rows, width, synth.quant_tensor(qtype, rows, width, seed=100 + i))
            for i, (_, rows, width, qtype) in enumerate(VERIFY_PROJS)]
    per_m = {}
    for m in VERIFY_MS:
        acts = {w: ref.quantize_q8_k(synth.activations(m, w, seed=m)) for w in (5120, 6144, 17408)}
        for qtype, rows, width, data in mats:  # warm-up
            ref.gemm_q8_k(qtype, data, rows, width, acts[width])
        times = []
        for _ in range(reps):
            t0 = time.perf_counter()
            for qtype, rows, width, data in mats:
                ref.gemm_q8_k(qtype, data, rows, width, acts[width])
            times.append(time.perf_counter() - t0)
        per_m[m] = statistics.median(times) * 1e3
    return {"value": verify_bytes(8) / (per_m[8] / 1e3) / 1e9, "unit": GBS, "cores": threads, "kind": "reference",
            "ms_per_pass": per_m,
            "sample": f"upstream q38_tensor_gemm_q8_k over the 7 projections, median of {reps} passes per M; {flags}"}


def measure_verify(passes=200, warmup=5, with_cpu=True):
    """The seven projections of one full-attention layer applied to M token
    rows through the kernel-level C ABI (q38cu_tensor_gemm_q8_k, the batched
    launch verification uses), two rotating device copies of the layer
    (2 x 234 MB > L2)."""
    import torch
    import q38b200 as q38
    from q38b200 import synth
    copies = 2
    layer = []
    for i, (_, rows, width, qtype) in enumerate(VERIFY_PROJS):
        host = synth.quant_tensor(qtype, rows, width, seed=100 + i)
        layer.append([q38.DeviceTensor(qtype, width, rows, host, layout=q38.LAYOUT_TILED) for _ in range(copies)])
    per_m = {}
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for m in VERIFY_MS:
            acts = {w: q38.quantize_q8_k(torch.from_numpy(synth.activations(m, w, seed=m)).cuda())
                    for w in (5120, 6144, 17408)}
            outs = [torch.empty((m, rows), dtype=torch.float32, device="cuda") for _, rows, _, _ in VERIFY_PROJS]

            def step(i):
                for k, (_, rows, width, _) in enumerate(VERIFY_PROJS):
                    q38.gemm_q8_k(layer[k][i % copies], acts[width], m, out=outs[k])

            ms = timed_graph(step, passes, warmup, chunk=20) / passes
            gbs = verify_bytes(m) / (ms / 1e3) / 1e9
            per_m[m] = {"ms_per_pass": ms, "value": gbs, "unit": GBS, "algorithmic_bytes": verify_bytes(m),
                        "frac": gbs / measured_peaks()[0]}
    if q38.device_status() != 0:
        raise RuntimeError("device status: a kernel abandoned a bounded wait")
    rec = {"workload": "config2: one full-attention layer's projections (q 5120->12288, k/v 5120->1024, "
                       "o 6144->5120, gate/up 5120->17408, down 17408->5120; Q4_K, Q6_K for v and down) "
                       "on M = 1, 2, 4, 8 token rows of N(0,1) activations as Q8_K",
           "value": per_m[8]["value"], "unit": GBS, "higher_is_better": True, "per_m": per_m,
           "m8_over_m1": per_m[8]["ms_per_pass"] / per_m[1]["ms_per_pass"],
           "l2": "inputs larger than L2: two rotating copies of the layer (2 x 234 MB)",
           "roofline": roofline(per_m[8]["value"], {"unit_of_launch": "one pass of the 7 projections at M = 8",
                                                    "timing": "CUDA events over graph-replayed passes"}),
           "note": "attention over the 2048-position KV cache is in the decode step (config 3), not here",
           "gpu_launches": passes * len(VERIFY_PROJS) * len(VERIFY_MS), "clocks": clocks.summary()}
    if with_cpu:
        cpu = cpu_verify()
        if cpu:
            rec["cpu_baseline"] = cpu
    for copies_k in layer:
        for t in copies_k:
            t.free()
    return rec


# ---------------------------------------------------------------------------
# configs 3 and 4: the synthetic model
# ---------------------------------------------------------------------------
PROMPT_TOKENS = 128
PREFILL_TOKENS = 4096
PREFILL_DECODE = 512
PREFILL_WARMUP = 128  # a warm-up prompt long enough for the tensor-core prefill path
CONTEXT = PREFILL_TOKENS + PREFILL_DECODE   # config 3's 4096-token window fits inside
VOCAB = 248320
MODEL_SEED = 0
STATE_BYTES = 48 * 48 * 128 * 128 * 4 * 2        # DeltaNet state, read and written
CONV_BYTES = 48 * 10240 * 4 * 4                  # conv ring: 3 taps read, 1 written
KV_ROW_BYTES = 16 * 1024 * 4 * 2                 # K and V rows of the 16 attention layers (fp32)


def decode_workload(mix):
    config = "config3" if mix == "Q4_K_M" else "config4 IQ1_M-typed variant"
    return (f"{config}: synthetic Qwen3.8-27B {mix} GGUF (upstream loader contract, config-0 weight "
            "draws), 128-token random prompt, greedy decode bs1, ctx 4096, MTP off")


def decode_config(mix, world):
    """The config dict both arms print."""
    return {"workload": decode_workload(mix), "prompt": PROMPT_TOKENS, "context": 4096, "batch": 1, "mtp": "off",
            "context_capacity": CONTEXT, "weights_bytes_per_step": decode_weight_bytes(mix),
            "l2": "inputs larger than L2: 15.5 GB of weights stream every step",
            "parallelism": "single GPU" if world == 1 else f"tensor parallel x{world}"}


def model_path(mix, rank, dist):
    """The synthetic model file, written once per machine (rank 0 first)."""
    from q38b200 import gguf
    path = gguf.cached_model_path(seed=MODEL_SEED, mtp=True, dist="config0", mix=mix) if rank == 0 else None
    if dist:
        dist.barrier()
    if path is None:
        path = gguf.cached_model_path(seed=MODEL_SEED, mtp=True, dist="config0", mix=mix)
    return path


def decode_weight_bytes(mix):
    """Weight bytes one decode step reads: every tensor of the 64 target layers,
    the output norm and LM head, and one embedding row (the MTP layer is not
    part of a target step)."""
    from q38b200 import gguf, synth
    total = 0
    for name, shape, qtype in gguf.tensor_specs(mtp=False, mix=mix):
        elements, nbytes = synth.BLOCK[qtype]
        size = int(np.prod(shape)) // elements * nbytes
        if name == "token_embd.weight":
            size = shape[0] // elements * nbytes
        total += size
    return total


def decode_step_bytes(mix, position):
    """Algorithmic bytes of the decode step at `position`: weights + recurrent
    state + the KV rows it scans (positions 0..position) and writes."""
    return decode_weight_bytes(mix) + STATE_BYTES + CONV_BYTES + KV_ROW_BYTES * (position + 2)


def decode_prompt(n=PROMPT_TOKENS, seed=1234):
    return np.random.default_rng(seed).integers(0, VOCAB, n).tolist()


def cpu_decode(path, tokens, prompt, warmup=2):
    """Greedy decode with the upstream Q38Model on this host's cores: the
    prompt is prefilled and `warmup` tokens decoded (untimed), then `tokens`
    forward_token + argmax steps are timed."""
    O, lib, flags, threads = cpu_setup()
    if not os.path.exists(lib):
        return None
    ref = O.ReferenceModel(path, CONTEXT, lib_path=lib)
    token = int(np.argmax(ref.prefill(prompt)))
    for _ in range(warmup):
        token = int(np.argmax(ref.forward_token(token)))
    t0 = time.perf_counter()
    for _ in range(tokens):
        token = int(np.argmax(ref.forward_token(token)))
    elapsed = time.perf_counter() - t0
    ref.close()
    return {"value": tokens / elapsed, "unit": TOKS, "cores": threads, "kind": "reference",
            "sample": f"upstream q38_model_forward_token + argmax, {tokens} greedy tokens after a "
                      f"{len(prompt)}-token prefill and {warmup} untimed tokens; "
                      f"{elapsed / tokens * 1e3:.1f} ms/token; {flags}"}


def cpu_prefill(path, tokens=32):
    """The upstream layer-major prefill (q38_model_prefill) of a `tokens`-long
    random prompt on this host's cores: a bounded sample of config 4's
    4096-token prefill, reported as prompt tokens/s."""
    O, lib, flags, threads = cpu_setup()
    if not os.path.exists(lib):
        return None
    ref = O.ReferenceModel(path, CONTEXT, lib_path=lib)
    ref.prefill(decode_prompt(4, seed=7))  # warm-up (pages, threads)
    ref.reset()
    t0 = time.perf_counter()
    ref.prefill(decode_prompt(tokens, seed=4096))
    elapsed = time.perf_counter() - t0
    ref.close()
    return {"value": tokens / elapsed, "unit": TOKS, "cores": threads, "kind": "reference",
            "sample": f"upstream q38_model_prefill of a {tokens}-token random prompt (a bounded sample of the "
                      f"4096-token prompt), {elapsed:.2f} s; {flags}"}


def run_decode_reference(args, rank, world, dist):
    path = model_path(args.mix, rank, dist)
    if rank != 0:
        return
    tokens = max(4, min(args.steps, 32))
    base = cpu_decode(path, tokens, decode_prompt(), warmup=min(args.warmup, 3))
    if base is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libq38ref.so is not built"}), flush=True)
        return
    line = {"metric": METRIC, "value": base["value"], "unit": TOKS, "n_gpus": args.gpus,
            "steps": tokens, "warmup": args.warmup, "ms_per_step": 1e3 / base["value"],
            "higher_is_better": True, "impl": "reference", "dtype": "int8xint8->int32,f32",
            "data": "synthetic (seeded GGUF, config-0 draws)", "scaling": "strong" if world > 1 else "weak",
            "config": decode_config(args.mix, world),
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": TOKS, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "vs_baseline": None}
    print(json.dumps(line), flush=True)


def run_matvec_reference(args, rank):
    if rank != 0:
        return
    case = matvec_case(args.qtype, args.shape)
    base = cpu_matvec(case, seconds=max(2.0, 0.02 * args.steps))
    line = {"metric": METRIC, "value": base["value"], "unit": GBS, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference", "dtype": "int8xint8->int32,f32",
            "data": "synthetic", "scaling": "weak",
            "config": {"workload": case["workload"], "l2": f"rotating {COPIES} weight copies"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": GBS, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "vs_baseline": None}
    print(json.dumps(line), flush=True)


def measure_prefill(m, path, stream, with_cpu=True):
    """Config 4 on one GPU: time to first token of a 4096-token random prompt
    through q38_model_prefill (ids from host memory, last-token logits back to
    host memory), then 512 greedy decode tokens at positions 4096..4607."""
    import torch
    prompt = decode_prompt(PREFILL_TOKENS, seed=4096)
    m.reset()
    # warm-up on the same (tensor-core) path: kernels loaded, buffers and plans made
    m.prefill(decode_prompt(PREFILL_WARMUP, seed=3))
    m.reset()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        start.record(stream)
        logits = m.prefill(prompt)
        end.record(stream)
        end.synchronize()
    ttft_ms = start.elapsed_time(end)
    token = int(np.argmax(logits))
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    m.generate_greedy(token, PREFILL_DECODE)
    e2.record(stream)
    e2.synchronize()
    decode_ms = s2.elapsed_time(e2)
    rec = {"workload": "config4: 4096-token random-id prompt prefilled on the synthetic Q4_K_M model "
                       "(q38_model_prefill), then 512 greedy decode tokens",
           "value": PREFILL_TOKENS / (ttft_ms / 1e3), "unit": "prompt tok/s", "ttft_ms": ttft_ms,
           "higher_is_better": True,
           "decode_after_prefill": {"value": PREFILL_DECODE / (decode_ms / 1e3), "unit": TOKS,
                                    "positions": f"{PREFILL_TOKENS}..{PREFILL_TOKENS + PREFILL_DECODE - 1}"},
           "timing": "CUDA events on the model stream; the prefill call includes the ids upload and the "
                     "last token's logits download",
           "clocks": clocks.summary()}
    if with_cpu:
        cpu = cpu_prefill(path)
        if cpu:
            rec["cpu_baseline"] = cpu
    return rec


def verify_pass_costs(m, stream):
    """Time of one batched target pass of n tokens (the verification of n
    drafts: q38_model_prefill of n tokens is the same launch sequence) at
    position 128, n = 1..8; independent of the MTP head's acceptance."""
    import torch
    out = {}
    for n in range(1, 9):
        m.reset()
        m.prefill(decode_prompt())
        m.prefill(decode_prompt(n, seed=n))  # warm-up of this chunk size
        m.reset()
        m.prefill(decode_prompt())
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        m.prefill(decode_prompt(n, seed=n))
        end.record(stream)
        end.synchronize()
        out[n] = start.elapsed_time(end)
    return out


def guarded(fn):
    """A sub-record, or the reason it could not be measured (the headline
    line is printed either way)."""
    try:
        return fn()
    except Exception as exc:  # noqa: BLE001 - reported in the line
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}


def run_decode(args, rank, world, dist):
    import torch
    from q38b200.model import Model

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    path = model_path(args.mix, rank, dist)
    if world > 1:
        # one tensor-parallel shard per GPU; rank 0 makes the communicator id
        from q38b200.model import nccl_unique_id
        box = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        m = Model(path, CONTEXT, rank=rank, world=world, nccl_id=box[0])
    else:
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
            print(json.dumps({"profile_run": decode_workload(args.mix), "profiled_steps": 1,
                              "kernels_per_step": kernels}), flush=True)
        return

    # W untimed warm-up steps, then exactly K timed steps (runs stay inside
    # the 4096-token window of config 3; a reset and a fresh prefill between
    # runs are not timed).
    token = fresh()
    token = m.generate_greedy(token, args.warmup)[-1]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    elapsed_ms, step_bytes, left = 0.0, 0, args.steps
    with ClockSampler(local) as clocks:
        while left:
            if 4096 - m.position < 2:
                token = fresh()
            n = min(left, 4096 - m.position - 1)
            pos0 = m.position
            ms, toks = timed(lambda: m.generate_greedy(token, n))
            elapsed_ms += ms
            step_bytes += sum(decode_step_bytes(args.mix, pos0 + i) for i in range(n))
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
    value = args.steps / (max_ms / 1e3)
    bytes_per_step = step_bytes / args.steps
    achieved = bytes_per_step / world / (ms_per_step / 1e3) / 1e9

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
    e2e_value = e2e_steps / (float(t2.item()) / 1e3)

    mtp = None
    subrecords = {}
    if 1 < world <= 2 and not args.no_subrecords:
        # config 4's prefill on the shards (tensor-core GEMMs, all-reduce after
        # the row-parallel ones; the model takes that path up to 2 GPUs); every
        # rank makes the same calls; rank 0's timing
        subrecords["prefill_config4"] = guarded(lambda: measure_prefill(m, path, stream, with_cpu=False))
    if world == 1 and not args.no_subrecords:
        # the acceptance-independent cost of verifying n drafts, and config
        # 4's prefill (both before MTP is enabled: with MTP on, a prefill also
        # runs the MTP head's catch-up)
        verify_ms = verify_pass_costs(m, stream)
        subrecords["prefill_config4"] = guarded(lambda: measure_prefill(m, path, stream))
        # MTP on: speculative greedy decoding at draft depths 1..4 (the
        # upstream's spec bench sweep, qwen38_spec_bench.c:108-119).
        mtp = {"verify_pass_ms": verify_ms}
        for drafts in (1, 2, 3, 4):
            m.reset()
            m.enable_mtp()
            token = int(np.argmax(m.prefill(prompt)))
            m.speculative_greedy(token, 0xFFFFFFFF, drafts)  # captures the draft and verification graphs
            m.reset()
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
            mtp[f"depth_{drafts}"] = {"value": produced / (mtp_ms / 1e3), "unit": TOKS, "draft_count": drafts,
                                      "tokens": produced, "calls": calls, "tokens_per_call": produced / calls,
                                      "ms_per_call": mtp_ms / calls}
        mtp["note"] = ("random-weight MTP head: drafts are almost never accepted, so each call yields one token "
                       "and costs the drafts plus a verification of depth tokens")
    m.close()
    if world == 1 and not args.no_subrecords:
        subrecords["matvec_config0"] = guarded(lambda: measure_matvec(matvec_case("Q4_K", "17408x5120")))
        for q in ("IQ1_M", "IQ2_S"):
            for shape in ("17408x5120", "5120x17408"):
                subrecords[f"matvec_config1_{q}_{shape}"] = guarded(
                    lambda q=q, shape=shape: measure_matvec(matvec_case(q, shape), launches=2000, e2e_steps=200))
        subrecords["verify_config2"] = guarded(measure_verify)

    if rank != 0:
        return
    cpu = cpu_decode(path, 16, prompt) if world == 1 else None
    line = {
        "metric": METRIC, "value": value, "unit": TOKS, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "int8xint8->int32,f32", "data": "synthetic (seeded GGUF, config-0 draws)",
        "config": decode_config(args.mix, world),
        "roofline": roofline(achieved, {"algorithmic_bytes_per_step": bytes_per_step,
                                        "unit_of_launch": "one decode step (one graph replay)",
                                        "per_gpu": "algorithmic bytes / N per GPU" if world > 1 else "one GPU",
                                        "timing": "CUDA events on the model stream around K graph replays"}),
        "e2e": {"value": e2e_value, "unit": TOKS, "steps": e2e_steps, "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": VOCAB * 4, "api": "q38_model_forward_token + host argmax"},
        "gpu_launches": kernels * args.steps,
        "kernels_per_step": kernels,
        "clocks": clocks.summary(),
    }
    if mtp:
        line["mtp"] = mtp
    if cpu:
        line["cpu_baseline"] = cpu
    if subrecords:
        line["subrecords"] = subrecords
    print(json.dumps(line), flush=True)


def run_single(args, rank, world):
    """--workload matvec / verify / prefill alone (one GPU)."""
    import torch
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    if args.workload == "matvec":
        case = matvec_case(args.qtype, args.shape)
        if args.profile:
            import q38b200 as q38
            from q38b200 import synth
            w = synth.quant_tensor(case["qtype"], case["rows"], case["width"], seed=0)
            ts = [q38.DeviceTensor(case["qtype"], case["width"], case["rows"], w, layout=q38.LAYOUT_TILED)
                  for _ in range(COPIES)]
            act = q38.quantize_q8_k(torch.from_numpy(synth.activations(1, case["width"], seed=1)).cuda())
            out = torch.empty((1, case["rows"]), dtype=torch.float32, device="cuda")
            for i in range(args.warmup + args.steps):
                q38.gemm_q8_k(ts[i % COPIES], act, 1, out=out)
            torch.cuda.synchronize()
            print(json.dumps({"profile_run": case["workload"], "launches": args.warmup + args.steps}), flush=True)
            return
        rec = measure_matvec(case, launches=args.steps, warmup=args.warmup, with_cpu=world == 1)
    elif args.workload == "verify":
        rec = measure_verify(passes=args.steps, warmup=args.warmup)
    else:
        from q38b200.model import Model
        path = model_path(args.mix, rank, None)
        m = Model(path, CONTEXT)
        if args.profile:
            # one 4096-token prefill after a warm-up prefill, nothing else (for a launch list)
            m.prefill(decode_prompt(PREFILL_WARMUP, seed=3))
            m.reset()
            m.prefill(decode_prompt(PREFILL_TOKENS, seed=4096))
            torch.cuda.synchronize()
            m.close()
            print(json.dumps({"profile_run": "config4 prefill", "tokens": PREFILL_TOKENS}), flush=True)
            return
        rec = measure_prefill(m, path, torch.cuda.ExternalStream(m.stream))
        m.close()
    if rank != 0:
        return
    line = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->int32,f32", "data": "synthetic (seeded)",
            "config": {"workload": rec.pop("workload")}}
    line.update(rec)
    print(json.dumps(line), flush=True)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None)
    parser.add_argument("--warmup", type=int, default=None)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--workload", choices=("decode", "matvec", "verify", "prefill"), default="decode")
    parser.add_argument("--qtype", choices=sorted(MATVEC_TYPES), default="Q4_K",
                        help="matvec workload: weight type (IQ1_M and IQ2_S give BASELINE config 1)")
    parser.add_argument("--shape", choices=("17408x5120", "5120x17408"), default="17408x5120",
                        help="matvec workload: rows x width")
    parser.add_argument("--profile", action="store_true",
                        help="plain launches only, for ncu: matvec - warmup + steps launches; decode - one decode "
                             "step between cudaProfilerStart/Stop; prints no bench line")
    parser.add_argument("--mix", choices=("Q4_K_M", "IQ1_M"), default="Q4_K_M",
                        help="decode workload: the model's type mix (IQ1_M: BASELINE config 4's IQ1_M-typed variant)")
    parser.add_argument("--no-subrecords", action="store_true",
                        help="decode workload: the headline line only (no MTP sweep and no other configs)")
    args = parser.parse_args()
    decode = args.workload == "decode"
    if args.steps is None:
        args.steps = {"decode": 256, "matvec": 20000, "verify": 200, "prefill": 1}[args.workload]
    if args.warmup is None:
        args.warmup = 3 if args.workload in ("decode", "prefill") else 20
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
            elif args.workload == "matvec":
                run_matvec_reference(args, rank)
            elif rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference arm covers the decode and "
                                  "matvec workloads; the other configs carry their CPU baseline inline"}))
        elif decode:
            run_decode(args, rank, world, dist)
        else:
            run_single(args, rank, world)
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
