"""Write tests/golden/c_abi_case.bin, the input and expected output of the C
ABI test (tests/c/abi_check.c): a small config-4-shaped batch (bf16 logits,
top-k / top-p / temperature per row, repetition penalty over a history) and
the ids and probabilities the CPU oracle gives for it.

Layout (little-endian): int32 dtype, vocab, batch, history_stride; logits
[batch, vocab] (2 bytes per element for bf16); tg_row_params [batch] (32 B);
int32 history [batch, history_stride]; int32 history_len [batch]; float
uniforms [batch]; int32 expected ids [batch]; float expected probs [batch].

Usage: python tests/golden/make_c_fixture.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle  # noqa: E402
from tinygpt_b200 import workloads as W  # noqa: E402


def main() -> None:
    oracle.build()
    w = W.make(4, seed=12, batch=12, vocab=5003)
    x = np.ascontiguousarray(w["logits"])
    assert x.dtype == np.uint16
    B, V = x.shape
    hist = np.ascontiguousarray(w["history"], dtype=np.int32)
    ids, probs = oracle.sample(x, w["params"], hist, w["history_len"], None, None, w["uniforms"])
    with open(os.path.join(HERE, "c_abi_case.bin"), "wb") as f:
        f.write(np.array([1, V, B, hist.shape[1]], np.int32).tobytes())
        f.write(x.tobytes())
        f.write(np.ascontiguousarray(w["params"]).tobytes())
        f.write(hist.tobytes())
        f.write(np.ascontiguousarray(w["history_len"], dtype=np.int32).tobytes())
        f.write(np.ascontiguousarray(w["uniforms"], dtype=np.float32).tobytes())
        f.write(ids.astype(np.int32).tobytes())
        f.write(probs.astype(np.float32).tobytes())
    print("wrote", os.path.join(HERE, "c_abi_case.bin"), B, V)


if __name__ == "__main__":
    main()
