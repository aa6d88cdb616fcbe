"""Times the reference's own sampling step on the CPU (baseline measurement only).

Runs `TinyGPT.generate` of the reference's python_ref/model.py:199-227 for one
token on fixed config-4-shaped logits (a stub model hands the logits back), so
the timed work is the reference's sampling block python_ref/model.py:213-224:
temperature, top-k threshold, softmax and torch.multinomial on torch-CPU.  The
reference takes one scalar top_k per call; the median of config 4's per-row
range (512) stands in for it.  Needs the reference tree (this container only):

    python oracle/time_python_ref.py --reference <tree> [--rows 512] [--threads N]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "tests", "golden"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--rows", type=int, default=512)
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    import torch
    from make_golden import load_python_ref
    from tinygpt_b200 import workloads as W
    torch.set_num_threads(args.threads)
    mod = load_python_ref(args.reference)
    w = W.make(4, seed=1, batch=args.rows)
    L = torch.from_numpy(W.bf16_bits_to_f32(w["logits"]))

    class Stub:
        cfg = types.SimpleNamespace(context_length=8)

        def eval(self):
            return self

        def __call__(self, idx):
            return L.unsqueeze(1), None

    g = torch.Generator().manual_seed(0)
    idx = torch.zeros((args.rows, 1), dtype=torch.long)
    mod.TinyGPT.generate(Stub(), idx, 1, temperature=0.8, top_k=512, generator=g)  # warm
    t0 = time.perf_counter()
    for _ in range(args.reps):
        mod.TinyGPT.generate(Stub(), idx, 1, temperature=0.8, top_k=512, generator=g)
    dt = (time.perf_counter() - t0) / args.reps
    print(json.dumps({"what": "python_ref TinyGPT.generate sampling step, torch-CPU",
                      "rows": args.rows, "vocab": W.CONFIGS[4]["vocab"], "threads": torch.get_num_threads(),
                      "cpu_count": os.cpu_count(), "s_per_step": dt, "rows_per_s": args.rows / dt}))


if __name__ == "__main__":
    main()
