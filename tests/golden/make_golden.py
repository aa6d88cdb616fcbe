"""Generate the golden fixtures in tests/golden/ (run here, where the reference
tree is mounted; the fixtures travel, the reference does not).

  ref_python_ref.npz  probabilities the reference's own TinyGPT.generate
                      (python_ref/model.py:199-227) hands to torch.multinomial,
                      captured on chosen logits through a stub model.
  ref_wasm.npz        ids the reference's own C++ tg_generate
                      (wasm/src/model.cpp:473-522, via oracle/_ref/libtgref.so)
                      samples from chosen logits, with the canonical uniforms its
                      std::mt19937 stream produced.
  ref_python_ref_configs.npz
                      the same capture at the configurations' shapes: V=50257
                      (config 1: T 0.8, top-k 40, five ids boosted +8), V=32000
                      bf16 with a Zipf bias and no top-k (config 2's T 0.7), and
                      V=128256 bf16 with a Zipf bias (config 4's T and top-k
                      range, bf16 ties at the threshold).
  oracle_cases.npz    oracle outputs (ids, probs) for seeded workloads of the
                      five configurations, regenerated from their seeds in tests.

Usage: python tests/golden/make_golden.py --reference <sarthak-fleet/tinygpt tree>
(or set TG_REFERENCE_ROOT)
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from tinygpt_b200 import workloads as W  # noqa: E402

# (config, seed, batch) cases whose oracle outputs are frozen in oracle_cases.npz
ORACLE_CASES = [(1, 0, 1), (1, 1, 1), (2, 0, 16), (3, 0, 8), (4, 0, 16), (4, 1, 16)]
SPEC_CASES = [(5, 0, 4)]


def load_python_ref(ref_root: str):
    path = os.path.join(ref_root, "python_ref", "model.py")
    spec = importlib.util.spec_from_file_location("tinygpt_ref_model", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def python_ref_probs(mod, logits: np.ndarray, temperature: float, top_k):
    """Run the reference's TinyGPT.generate for one token on fixed logits and
    return the probability rows it passes to torch.multinomial."""
    import torch
    L = torch.from_numpy(logits)

    class Stub:
        cfg = types.SimpleNamespace(context_length=8)

        def eval(self):
            return self

        def __call__(self, idx):
            return L.unsqueeze(1), None

    captured = {}
    orig = torch.multinomial

    def spy(probs, num_samples, *a, **k):
        captured["p"] = probs.detach().clone()
        return orig(probs, num_samples, *a, **k)

    torch.multinomial = spy
    try:
        g = torch.Generator().manual_seed(0)
        mod.TinyGPT.generate(Stub(), torch.zeros((L.shape[0], 1), dtype=torch.long), 1,
                             temperature=temperature, top_k=top_k, generator=g)
    finally:
        torch.multinomial = orig
    return captured["p"].numpy().astype(np.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TG_REFERENCE_ROOT"),
                    required="TG_REFERENCE_ROOT" not in os.environ)
    args = ap.parse_args()
    oracle.build()
    g = W.rng(20261201)

    # ---- python_ref pins ---------------------------------------------------------
    mod = load_python_ref(args.reference)
    cases = []
    for i, (V, T, k) in enumerate([(1000, 0.8, 40), (1000, 1.0, None), (5000, 0.7, 50),
                                   (5000, 1.3, 1), (300, 0.5, 299), (2048, 0.9, 100)]):
        x = g.normal(0.0, 3.0, size=(4, V)).astype(np.float32)
        if i == 5:  # bf16-valued logits: many exact ties at the top-k threshold
            x = W.bf16_bits_to_f32(W.to_bf16_bits(x))
        pr = python_ref_probs(mod, x, T, k)
        cases.append(dict(logits=x, T=np.float32(T), k=np.int32(0 if k is None else k), probs=pr))
    np.savez_compressed(os.path.join(HERE, "ref_python_ref.npz"),
                        n=len(cases), **{f"{key}_{i}": c[key] for i, c in enumerate(cases) for key in c})

    # ---- wasm tg_generate pins ----------------------------------------------------
    ref = oracle.ref_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libtgref.so missing: run make -C oracle")
    rows, Ts, ks, seeds, ids, us = [], [], [], [], [], []
    steps = 64
    for i in range(24):
        V = 256 if i % 3 else 97
        x = np.zeros(256, np.float32)
        x[:V] = g.normal(0.0, 2.0, size=V).astype(np.float32)
        T = float(g.choice([0.0, 0.5, 0.8, 1.0, 1.5]))
        k = int(g.choice([0, 1, 5, 40, V - 1]))
        seed = int(g.integers(1, 2**31))
        out = np.zeros(steps, np.uint8)
        n = ref.tgref_generate_fixed_logits(x.ctypes.data, V, T, k, seed, steps, out.ctypes.data)
        assert n == steps, n
        u = np.zeros(steps, np.float32)
        ref.tgref_canonical_uniforms(seed, steps, u.ctypes.data)
        rows.append(x); Ts.append(T); ks.append(k); seeds.append(seed)
        ids.append(out.astype(np.int32)); us.append(u)
        rows[-1] = np.concatenate([x[:V], np.full(256 - V, np.nan, np.float32)])
    np.savez_compressed(os.path.join(HERE, "ref_wasm.npz"), logits=np.stack(rows),
                        T=np.array(Ts, np.float32), k=np.array(ks, np.int32),
                        seed=np.array(seeds, np.int64), ids=np.stack(ids), u=np.stack(us))

    # ---- oracle outputs for seeded workloads ----------------------------------------
    out = {}
    for c, seed, B in ORACLE_CASES:
        w = W.make(c, seed=seed, batch=B)
        i, p = oracle.sample(w["logits"], w["params"], w.get("history"), w.get("history_len"),
                             w.get("mask_table"), w.get("state_id"), w["uniforms"])
        out[f"ids_{c}_{seed}_{B}"] = i
        out[f"probs_{c}_{seed}_{B}"] = p
    for c, seed, B in SPEC_CASES:
        w = W.make(c, seed=seed, batch=B)
        o, n = oracle.spec_verify(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                  w["u_accept"], w["u_draw"])
        out[f"spec_ids_{c}_{seed}_{B}"] = o
        out[f"spec_n_{c}_{seed}_{B}"] = n
    np.savez_compressed(os.path.join(HERE, "oracle_cases.npz"), **out)
    python_ref_config_pins(mod)
    print("golden fixtures written to", HERE)


def zipf_bias(g, V: int) -> np.ndarray:
    """-1.1 * ln(rank) over a random permutation of the ids (the bias of
    configs 2 and 4, tinygpt_b200.workloads)."""
    perm = g.permutation(V)
    bias = np.empty(V, np.float32)
    bias[perm] = (-1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))).astype(np.float32)
    return bias


def python_ref_config_pins(mod) -> None:
    """python_ref's probabilities at the configurations' shapes (a few rows each)."""
    g = W.rng(20261202)
    cases = []
    # config 1: V=50257 fp32, N(0, 3^2) + 8 on five ids, T 0.8, top-k 40
    x = g.normal(0.0, 3.0, size=(2, 50257)).astype(np.float32)
    for r in range(2):
        x[r, g.choice(50257, 5, replace=False)] += 8.0
    cases.append(dict(name="config1", logits=x, T=0.8, k=40, bf16=False))
    # config 2 shape: V=32000 bf16, N(0, 2.5^2) + Zipf bias, T 0.7, no top-k
    x = np.stack([g.normal(0.0, 2.5, size=32000).astype(np.float32) + zipf_bias(g, 32000) for _ in range(2)])
    cases.append(dict(name="config2", logits=W.bf16_bits_to_f32(W.to_bf16_bits(x)), T=0.7, k=None, bf16=True))
    # config 4 shape: V=128256 bf16, N(0, 3^2) + Zipf bias; k and T at both ends of config 4's ranges
    for T, k in ((0.3, 1), (0.9, 50), (1.2, 1024)):
        x = (g.normal(0.0, 3.0, size=128256).astype(np.float32) + zipf_bias(g, 128256))[None]
        cases.append(dict(name=f"config4_T{T}_k{k}", logits=W.bf16_bits_to_f32(W.to_bf16_bits(x)), T=T, k=k,
                          bf16=True))
    out = {"n": len(cases)}
    for i, c in enumerate(cases):
        pr = python_ref_probs(mod, c["logits"], c["T"], c["k"])
        out[f"name_{i}"] = np.array(c["name"])
        out[f"logits_{i}"] = W.to_bf16_bits(c["logits"]) if c["bf16"] else c["logits"]
        out[f"bf16_{i}"] = np.int32(c["bf16"])
        out[f"T_{i}"] = np.float32(c["T"])
        out[f"k_{i}"] = np.int32(0 if c["k"] is None else c["k"])
        out[f"probs_{i}"] = pr
    np.savez_compressed(os.path.join(HERE, "ref_python_ref_configs.npz"), **out)


if __name__ == "__main__":
    main()
