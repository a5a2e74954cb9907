"""In-graph launch timeline of the decode step of the synthetic model.

    PYTHONPATH=qwen3.8-27b-in-c_b200/python python -m q38b200.timeline

Opens the model with Q38CU_TRACE=1 (every kernel of the captured decode graph
keeps %globaltimer stamps of its CTAs, include/q38cuda_model.h), prefills 128
random tokens, decodes, and prints per kernel kind its cost inside the graph
(previous kernel's last CTA end to its own last CTA end) and, for the
weight-streaming GEMVs, the phases after the grid-dependency release.  Kernel
labels follow the decode step's launch order (q38_model.cu: enqueue_layer).
"""
import collections
import os

import numpy as np

from . import gguf


def labels():
    out = []
    for l in range(64):
        if (l + 1) % 4 == 0:
            out += [f"L{l}.qk", f"L{l}.v", f"L{l}.attn", f"L{l}.o"]
        else:
            out += [f"L{l}.qkvz", f"L{l}.delta", f"L{l}.out"]
        out += [f"L{l}.gate_up", f"L{l}.down{'6' if l % 2 == 0 else '4'}"]
    return out + ["head", "argmax"]


def kind(name):
    return name.split(".", 1)[1] if "." in name else name


def main(count=6):
    os.environ["Q38CU_TRACE"] = "1"
    import torch
    from .model import Model
    torch.cuda.set_device(0)
    m = Model(gguf.cached_model_path(seed=0, mtp=True, dist="config0"), 4096)
    prompt = np.random.default_rng(1234).integers(0, 248320, 128).tolist()
    tok = int(np.argmax(m.prefill(prompt)))
    tok = m.generate_greedy(tok, 4)[-1]
    m.trace()
    records = []
    for _ in range(count):
        tok = m.generate_greedy(tok, 1)[-1]
        records.append(m.trace().astype(np.int64))
    names = labels()
    n = len(records[0])
    assert n == len(names), (n, len(names))
    total = np.median([r[-1, 2] - r[0, 0] for r in records])
    print(f"step (first CTA start -> last CTA end): {total / 1e3:.1f} us over {n} traced kernels (median of {count} steps)")
    inc = collections.defaultdict(list)
    for i in range(n):
        inc[kind(names[i])].append(np.median([r[i, 2] - (r[i - 1, 2] if i else r[0, 0]) for r in records]))
    print("| kind | launches | us per step | us per launch |")
    print("|---|---:|---:|---:|")
    for k, v in sorted(inc.items(), key=lambda kv: -sum(kv[1])):
        print(f"| {k} | {len(v)} | {sum(v) / 1e3:.1f} | {np.mean(v) / 1e3:.2f} |")
    print()
    print("| GEMV kind | ready->staged | staged->decoded | decoded->end | prev end->ready |")
    print("|---|---:|---:|---:|---:|")
    ph = collections.defaultdict(list)
    for i in range(n):
        for r in records:
            if r[i, 3] == 0 or r[i, 4] == 0:
                continue
            prev = r[i - 1, 2] if i else r[0, 0]
            ph[kind(names[i])].append([r[i, 3] - r[i, 1], r[i, 4] - r[i, 3], r[i, 2] - r[i, 4], r[i, 1] - prev])
    for k, v in ph.items():
        md = np.median(np.array(v), axis=0) / 1e3
        print(f"| {k} | " + " | ".join(f"{x:.2f}" for x in md) + " |")
    # Fused RMSNorm prologues: the earliest CTA's steps (fields 1, 9, 8, 10, 7),
    # the spread to the last CTA staged (field 3) and the spread of the CTAs'
    # returns from the grid-dependency wait (fields 1, 6).
    print()
    print("| RMSNorm GEMV kind | ready->x loaded | ->sum known | ->warp 0 quantized | ->first staged "
          "| first->last staged | first->last ready |")
    print("|---|---:|---:|---:|---:|---:|---:|")
    sub = collections.defaultdict(list)
    for i in range(n):
        for r in records:
            if r[i, 3] == 0 or r[i, 4] == 0 or r[i, 9] in (0, -1) or r[i, 9] < r[i, 1]:
                continue
            sub[kind(names[i])].append([r[i, 9] - r[i, 1], r[i, 8] - r[i, 9], r[i, 10] - r[i, 8],
                                        r[i, 7] - r[i, 10], r[i, 3] - r[i, 7], r[i, 6] - r[i, 1]])
    for k, v in sub.items():
        md = np.median(np.array(v), axis=0) / 1e3
        print(f"| {k} | " + " | ".join(f"{x:.2f}" for x in md) + " |")
    m.close()


if __name__ == "__main__":
    main()
