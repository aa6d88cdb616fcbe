"""The oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from python_ref and the C++ tg_generate), and the
oracle's arithmetic against libm.  CPU only."""
import os

import numpy as np
import pytest

from tinygpt_b200 import workloads as W

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def params1(T, k, top_p=1.0, min_p=0.0, rep=1.0, pres=0.0, freq=0.0):
    from oracle.oracle import ROW_PARAMS_DTYPE
    p = np.zeros(1, ROW_PARAMS_DTYPE)
    p["temperature"], p["top_k"], p["top_p"], p["min_p"] = T, k, top_p, min_p
    p["repetition_penalty"], p["presence_penalty"], p["frequency_penalty"] = rep, pres, freq
    return p[0]


def test_exp_within_one_ulp_of_libm(oracle_mod):
    xs = np.concatenate([np.linspace(-87.0, 0.0, 300001, dtype=np.float32),
                         -np.logspace(-30, 1.9, 20001).astype(np.float32)])
    got = np.array([oracle_mod.exp32(float(x)) for x in xs[::3]], np.float64)
    ref = np.exp(xs[::3].astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert (np.abs(got - ref) / ulp).max() < 1.0
    assert oracle_mod.exp32(0.0) == 1.0
    assert oracle_mod.qmass(0.0) == 1 << 44
    assert oracle_mod.qmass(-40.0) == 0 and oracle_mod.qmass(float("-inf")) == 0


# Probabilities are q / S with q = trunc(e * 2^44) and S >= 2^44, so each one
# carries an absolute error below 2^-44 from the fixed-point masses: the 1e-5
# relative bound holds for every probability >= 2^-44 / 1e-5 (5.7e-9); below
# that floor a probability is compared to within two quanta and counted.
P_FLOOR = 2.0 ** -44 / 1e-5


def _check_python_ref(oracle_mod, x, T, k, pref, what, report):
    _, _, _, st, q = oracle_mod.sample_row_detail(x, params1(T, k))
    keep = (st & 1).astype(bool)
    assert np.array_equal(keep, pref > 0), f"{what}: top-k support differs"
    p = q.astype(np.float64) / q.sum(dtype=np.float64)
    pr = pref.astype(np.float64)
    big = pr >= P_FLOOR
    rel = np.abs(p[big] - pr[big]) / pr[big]
    assert rel.max(initial=0.0) <= 1e-5, f"{what}: relative error {rel.max()}"
    small = keep & ~big
    assert (np.abs(p[small] - pr[small]) <= 2.0 ** -43).all(), f"{what}: error below the quantum floor"
    report[0] += int(big.sum())
    report[1] += int(small.sum())
    report[2] = max(report[2], float(rel.max(initial=0.0)))


def test_python_ref_distribution_pinned(oracle_mod, pin_report):
    """Support exactly and probabilities within 1e-5 relative of the reference's
    softmax after top-k (python_ref/model.py:213-224)."""
    z = np.load(os.path.join(GOLD, "ref_python_ref.npz"))
    acc = [0, 0, 0.0]
    for i in range(int(z["n"])):
        x, T, k, pref = z[f"logits_{i}"], float(z[f"T_{i}"]), int(z[f"k_{i}"]), z[f"probs_{i}"]
        for r in range(x.shape[0]):
            _check_python_ref(oracle_mod, x[r], T, k, pref[r], f"python_ref case {i} row {r}", acc)
    pin_report.append(f"python_ref small cases: {acc[0]} probabilities within 1e-5 relative (max {acc[2]:.2e}), "
                      f"{acc[1]} below {P_FLOOR:.1e} within 2^-43")


def test_python_ref_pinned_at_config_shapes(oracle_mod, pin_report):
    """The same pin at the configurations' vocabularies: V=50257 (config 1),
    32000 and 128256 with bf16 ties at the top-k threshold."""
    z = np.load(os.path.join(GOLD, "ref_python_ref_configs.npz"))
    acc = [0, 0, 0.0]
    for i in range(int(z["n"])):
        x = z[f"logits_{i}"]
        if int(z[f"bf16_{i}"]):
            x = W.bf16_bits_to_f32(x)
        T, k, pref = float(z[f"T_{i}"]), int(z[f"k_{i}"]), z[f"probs_{i}"]
        for r in range(x.shape[0]):
            _check_python_ref(oracle_mod, x[r], T, k, pref[r], f"python_ref {z[f'name_{i}']} row {r}", acc)
    pin_report.append(f"python_ref config shapes: {acc[0]} probabilities within 1e-5 relative (max {acc[2]:.2e}), "
                      f"{acc[1]} below {P_FLOOR:.1e} within 2^-43")


def test_wasm_tg_generate_draws_pinned(oracle_mod, pin_report):
    """Same ids as the reference's C++ tg_generate for the same logits and the
    same uniform stream.  Its fp32 running sums and the exact masses here differ
    by rounding, so a draw whose point lies within 1e-6 (relative to the total)
    of a cumulative boundary is exempt; exempt draws are counted and reported."""
    z = np.load(os.path.join(GOLD, "ref_wasm.npz"))
    checked = exempt = 0
    for r in range(z["logits"].shape[0]):
        row = z["logits"][r]
        V = int(np.isfinite(row).sum())
        x = row[:V].astype(np.float32)
        T, k = float(z["T"][r]), int(z["k"][r])
        for s in range(z["ids"].shape[1]):
            u = float(z["u"][r, s]) if T > 0 else 0.0
            i, prob, _, st, q = oracle_mod.sample_row_detail(x, params1(T, k), u=u)
            want = int(z["ids"][r, s])
            if T > 0:
                S = int(q[(st & 2).astype(bool)].sum())
                cdf = np.cumsum(np.where((st & 2).astype(bool), q, 0)).astype(np.float64)
                if np.min(np.abs(cdf - u * S)) < 1e-6 * S:
                    exempt += 1
                    pin_report.append(f"wasm row {r} step {s}: draw point within 1e-6 of a boundary "
                                      f"(oracle {i}, reference {want})")
                    continue
            checked += 1
            assert i == want, f"row {r} step {s}: oracle {i} reference {want}"
    pin_report.append(f"wasm tg_generate: {checked} draws equal, {exempt} exempt")
    assert checked > 1000 and exempt < 0.01 * checked


def test_oracle_cases_frozen(oracle_mod):
    """The oracle still reproduces its committed outputs (regression pin)."""
    z = np.load(os.path.join(GOLD, "oracle_cases.npz"))
    from tests.golden.make_golden import ORACLE_CASES, SPEC_CASES
    for c, seed, B in ORACLE_CASES:
        w = W.make(c, seed=seed, batch=B)
        i, p = oracle_mod.sample(w["logits"], w["params"], w.get("history"), w.get("history_len"),
                                 w.get("mask_table"), w.get("state_id"), w["uniforms"])
        assert np.array_equal(i, z[f"ids_{c}_{seed}_{B}"])
        assert np.array_equal(p, z[f"probs_{c}_{seed}_{B}"])
    for c, seed, B in SPEC_CASES:
        w = W.make(c, seed=seed, batch=B)
        o, n = oracle_mod.spec_verify(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                      w["u_accept"], w["u_draw"])
        assert np.array_equal(o, z[f"spec_ids_{c}_{seed}_{B}"])
        assert np.array_equal(n, z[f"spec_n_{c}_{seed}_{B}"])


def test_greedy_is_first_argmax_and_masks(oracle_mod):
    x = np.array([1.0, 3.0, 3.0, -2.0, 3.0], np.float32)
    i, p, *_ = oracle_mod.sample_row_detail(x, params1(0.0, 0))
    assert i == 1 and p == 1.0
    m = np.array([0b10101], np.uint32)  # tokens 0, 2, 4 allowed
    i, *_ = oracle_mod.sample_row_detail(x, params1(0.0, 0), mask=m)
    assert i == 2
    i, *_ = oracle_mod.sample_row_detail(x, params1(0.7, 0), mask=np.zeros(1, np.uint32))
    assert i == -1


def test_penalties_follow_ctrl_and_openai_rules(oracle_mod):
    x = np.array([2.0, -2.0, 1.0, 0.5], np.float32)
    hist = np.array([0, 1, 1, 7, -3], np.int32)  # ids outside the vocab are ignored
    _, _, y, _, _ = oracle_mod.sample_row_detail(x, params1(0.0, 0, rep=2.0), history=hist)
    assert np.array_equal(y, np.array([1.0, -4.0, 1.0, 0.5], np.float32))
    _, _, y, _, _ = oracle_mod.sample_row_detail(x, params1(0.0, 0, pres=0.5, freq=0.25), history=hist)
    assert np.array_equal(y, np.array([2.0 - 0.75, -2.0 - 1.0, 1.0, 0.5], np.float32))


def test_top_p_min_p_prefix(oracle_mod):
    x = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float64)).astype(np.float32)
    _, _, _, st, _ = oracle_mod.sample_row_detail(x, params1(1.0, 0, top_p=0.7))
    assert list((st >> 1) & 1) == [1, 1, 0, 0]
    _, _, _, st, _ = oracle_mod.sample_row_detail(x, params1(1.0, 0, min_p=0.35))
    assert list((st >> 1) & 1) == [1, 1, 0, 0]
    _, _, _, st, _ = oracle_mod.sample_row_detail(x, params1(1.0, 0, top_p=0.0))
    assert list((st >> 1) & 1) == [1, 0, 0, 0]
