"""CUDA sampling path vs the oracle: token ids AND probabilities bit-exact
(the arithmetic is defined op by op, so no tolerance is needed)."""
import numpy as np
import pytest

from tinygpt_b200 import workloads as W
from tests.gpu_helpers import assert_same

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("config,seed", [(1, 0), (1, 1), (2, 0), (2, 1), (3, 0), (3, 1), (4, 0), (4, 1)])
def test_config_parity_full_size(oracle_mod, sampler_factory, config, seed):
    w = W.make(config, seed=seed)
    s = sampler_factory(w["vocab"])
    assert_same(oracle_mod, s, w, what=f"config {config} seed {seed}")


def test_config1_steps(oracle_mod, sampler_factory):
    """Many steps of the single-row GPT-2 configuration (fresh uniform each step)."""
    w = W.make(1, seed=3)
    s = sampler_factory(w["vocab"])
    g = W.rng(7)
    for _ in range(50):
        w["uniforms"] = g.random(1, dtype=np.float32)
        assert_same(oracle_mod, s, w, what="config1 step")


def _base(B, V, seed, dtype="f32", scale=3.0):
    g = W.rng(seed)
    x = g.normal(0, scale, size=(B, V)).astype(np.float32)
    if dtype == "bf16":
        x = W.to_bf16_bits(x)
    p = np.zeros(B, W.ROW_PARAMS_DTYPE)
    p["temperature"] = 0.8
    p["top_p"] = 1.0
    return dict(logits=x, params=p, uniforms=g.random(B, dtype=np.float32), vocab=V), g


@pytest.mark.parametrize("V", [1, 7, 256, 1000, 3072, 3073, 50257, 128256])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_vocab_sizes_and_modes(oracle_mod, sampler_factory, V, dtype):
    B = 64
    w, g = _base(B, V, V * 7 + (dtype == "bf16"), dtype)
    p = w["params"]
    p["temperature"] = np.where(np.arange(B) % 4 == 0, 0.0, g.uniform(0.2, 2.0, B))
    p["top_k"] = g.choice([0, 1, 2, 40, 1024, 2000, V - 1, V, V + 5], size=B)
    p["top_p"] = g.choice([1.0, 0.9, 0.5, 0.0, 1e-4], size=B)
    p["min_p"] = g.choice([0.0, 0.0, 0.05, 1.0, 2.0], size=B)
    assert_same(oracle_mod, sampler_factory(V), w, what=f"V={V} {dtype}")


@pytest.mark.parametrize("stride_pad", [1, 3, 8])
def test_unaligned_row_stride(oracle_mod, sampler_factory, stride_pad):
    V = 5003
    for dtype in ("f32", "bf16"):
        w, g = _base(16, V, stride_pad, dtype)
        w["params"]["top_k"] = 50
        assert_same(oracle_mod, sampler_factory(V), w, stride=V + stride_pad, what="stride")


def _sorted_w():
    V = 128256
    B = 8
    base = np.linspace(-10, 10, V, dtype=np.float32)
    x = np.stack([base if b % 2 == 0 else base[::-1].copy() for b in range(B)])
    p = np.zeros(B, W.ROW_PARAMS_DTYPE)
    p["temperature"] = [0.0, 0.0, 0.9, 0.9, 0.5, 0.5, 1.0, 1.0]
    p["top_k"] = [0, 0, 10, 10, 1000, 1000, 3, 3]
    p["top_p"] = [1.0, 1.0, 0.9, 0.9, 0.5, 0.5, 1.0, 1.0]
    return dict(logits=x, params=p, uniforms=W.rng(1).random(B, dtype=np.float32))


def test_sorted_rows_force_full_row_path(oracle_mod, sampler_factory):
    """Ascending / descending rows defeat the sampled threshold: the candidate
    list overflows or comes up short and the full-row path must take over."""
    assert_same(oracle_mod, sampler_factory(128256), _sorted_w(), what="sorted")


def _ties_w():
    V = 128256
    B = 12
    x = np.zeros((B, V), np.float32)
    x[4:8, ::3] = 1.0
    x[8:, :] = W.bf16_bits_to_f32(W.to_bf16_bits(W.rng(3).normal(0, 0.05, size=(4, V)).astype(np.float32)))
    p = np.zeros(B, W.ROW_PARAMS_DTYPE)
    p["temperature"] = [0.0, 1.0, 1.0, 1.0] * 3
    p["top_k"] = [0, 5, 0, 100] * 3
    p["top_p"] = [1.0, 0.3, 0.5, 0.9] * 3
    return dict(logits=x, params=p, uniforms=W.rng(2).random(B, dtype=np.float32))


def test_ties_everywhere(oracle_mod, sampler_factory):
    """Constant rows and two-level rows: top-k keeps all ties, top-p orders
    ties by id, greedy returns the first maximum."""
    assert_same(oracle_mod, sampler_factory(128256), _ties_w(), what="ties")


def _pen_w():
    V = 32000
    B = 32
    w, g = _base(B, V, 11, "bf16")
    p = w["params"]
    p["temperature"] = np.where(np.arange(B) % 3 == 0, 0.0, 0.9)
    p["top_k"] = g.choice([0, 20, 500], size=B)
    p["repetition_penalty"] = g.choice([1.0, 1.3, 0.8, 5.0], size=B)
    p["presence_penalty"] = g.choice([0.0, 0.5, -1.0], size=B)
    p["frequency_penalty"] = g.choice([0.0, 0.3, -0.2], size=B)
    hist = g.integers(-5, V + 5, size=(B, 300)).astype(np.int32)
    # make the penalised tokens matter: history holds the row's top tokens
    lg = W.bf16_bits_to_f32(w["logits"])
    top = np.argsort(-lg, axis=1)[:, :40].astype(np.int32)
    hist[:, :120] = np.repeat(top, 3, axis=1)
    w["history"] = hist
    w["history_len"] = g.integers(0, 301, size=B).astype(np.int32)
    w["history_len"][0] = 300
    return w


def test_penalties_edge_cases(oracle_mod, sampler_factory):
    assert_same(oracle_mod, sampler_factory(32000), _pen_w(), what="penalties")


def _tile(w, rows):
    """The workload's rows repeated to `rows` rows (other uniforms per copy)."""
    B = w["params"].shape[0]
    reps = (rows + B - 1) // B
    out = {}
    for k, v in w.items():
        if isinstance(v, np.ndarray) and k != "mask_table" and v.shape[:1] == (B,):
            out[k] = np.concatenate([v] * reps)[:rows].copy()
        else:
            out[k] = v
    out["uniforms"] = W.rng(rows).random(rows, dtype=np.float32)
    return out


@pytest.mark.parametrize("rows", [3, 160])
@pytest.mark.parametrize("make", ["sorted", "ties", "penalties", "masks"])
def test_edge_workloads_other_kernel_widths(oracle_mod, sampler_factory, make, rows):
    """The edge workloads above run on the 1024-thread kernel (8-148 rows);
    fewer and more rows take the 256-thread kernel."""
    w = {"sorted": _sorted_w, "ties": _ties_w, "penalties": _pen_w, "masks": _masks_w}[make]()
    V = w["logits"].shape[1]
    assert_same(oracle_mod, sampler_factory(V), _tile(w, rows), what=f"{make} x{rows}")


def _masks_w():
    V = 128256
    B = 16
    w, g = _base(B, V, 5, "f32")
    Wd = (V + 31) // 32
    bits = np.zeros((4, Wd * 32), bool)
    bits[1, :V] = g.random(V) < 0.001
    bits[2, 12345] = True
    bits[3, :V] = True
    w["mask_table"] = W.pack_mask(bits)
    w["state_id"] = np.array([0, 1, 2, 3, -1] * 3 + [1], np.int32)
    w["params"]["temperature"] = np.where(np.arange(B) % 2 == 0, 0.0, 1.0)
    w["params"]["top_k"] = np.where(np.arange(B) % 4 == 1, 50, 0)
    return w


def test_masks_and_bad_states(oracle_mod, sampler_factory):
    V = 128256
    B = 16
    w, g = _base(B, V, 5, "f32")
    Wd = (V + 31) // 32
    bits = np.zeros((4, Wd * 32), bool)
    bits[1, :V] = g.random(V) < 0.001
    bits[2, 12345] = True
    bits[3, :V] = True
    w["mask_table"] = W.pack_mask(bits)
    w["state_id"] = np.array([0, 1, 2, 3, -1] * 3 + [1], np.int32)
    w["params"]["temperature"] = np.where(np.arange(B) % 2 == 0, 0.0, 1.0)
    w["params"]["top_k"] = np.where(np.arange(B) % 4 == 1, 50, 0)
    s = sampler_factory(V)
    gi, _ = assert_same(oracle_mod, s, w, what="masks")
    assert (gi[w["state_id"] == 0] == -1).all()
    assert (gi[w["state_id"] == 2] == 12345).all()
    s.device_status()  # clear
    w["state_id"] = np.array([7] + [0] * (B - 1), np.int32)
    gi, _ = assert_same(oracle_mod, s, w, what="bad state")
    assert gi[0] == -1 and s.device_status() & 1


def test_uniform_edges(oracle_mod, sampler_factory):
    V = 128256
    B = 8
    w, g = _base(B, V, 9, "bf16")
    w["params"]["top_k"] = 100
    w["uniforms"] = np.array([0.0, np.nextafter(1.0, 0.0), np.nan, -1.0, 1.0, 0.5, 1e-30, 0.999],
                             np.float32)
    assert_same(oracle_mod, sampler_factory(V), w, what="uniforms")


def test_host_entry_point_matches_device_entry_point(oracle_mod, sampler_factory):
    w = W.make(4, seed=5, batch=64)
    s = sampler_factory(w["vocab"])
    hi, hp = s.sample_host(w["logits"], w["params"], history=w["history"],
                           history_len=w["history_len"], uniforms=w["uniforms"], want_probs=True)
    oi, op = oracle_mod.sample(w["logits"], w["params"], w["history"], w["history_len"], None,
                               None, w["uniforms"])
    assert np.array_equal(hi, oi) and np.array_equal(hp.view(np.uint32), op.view(np.uint32))


@pytest.mark.parametrize("scale", [0.05, 0.3, 3.0])
def test_no_topk_truncation_modes(oracle_mod, sampler_factory, scale):
    """Rows without top-k but with top-p and/or min-p: the candidate list holds
    the largest values only, the rest contributes its mass; flat rows make the
    top-p prefix run past the list (full-row path) unless min-p stops it."""
    V = 32000
    B = 48
    w, g = _base(B, V, int(scale * 100) + 7, "bf16", scale=scale)
    p = w["params"]
    p["temperature"] = g.choice([0.5, 1.0, 2.0], size=B)
    p["top_k"] = 0
    p["top_p"] = g.choice([1.0, 0.99, 0.9, 0.5], size=B)
    p["min_p"] = g.choice([0.0, 0.05, 0.5, 0.9], size=B)
    w["history"] = g.integers(0, V, size=(B, 64)).astype(np.int32)
    w["history_len"] = np.full(B, 64, np.int32)
    p["presence_penalty"] = 0.4
    p["frequency_penalty"] = 0.2
    assert_same(oracle_mod, sampler_factory(V), w, what=f"no-topk scale={scale}")


def _nok_w(V, B, seed, dtype):
    """Rows without top-k that reach the full-row stages: no truncation at all,
    top-p cuts beyond any candidate list (flat rows, p close to 1), p = 0,
    min-p, ties, penalties raising and lowering values, masked rows."""
    w, g = _base(B, V, seed, dtype, scale=1.0)
    x = W.bf16_bits_to_f32(w["logits"]) if dtype == "bf16" else w["logits"]
    x = x.copy()
    x[0] = 0.0                                  # one constant row
    x[1, ::7] = 2.0                             # two levels
    x[2] *= 0.05                                # nearly flat
    if B > 3:
        x[3] = np.linspace(-8, 8, V, dtype=np.float32)  # sorted
    w["logits"] = W.to_bf16_bits(x) if dtype == "bf16" else x
    p = w["params"]
    p["top_k"] = 0
    p["temperature"] = g.choice([0.5, 1.0, 2.0], size=B)
    p["top_p"] = g.choice([1.0, 0.9999, 0.99, 0.95, 0.5, 0.0], size=B)
    p["min_p"] = g.choice([0.0, 0.0, 0.05], size=B)
    p["repetition_penalty"] = g.choice([1.0, 1.3], size=B)
    p["presence_penalty"] = g.choice([0.0, 0.5, -0.7], size=B)
    hist = g.integers(0, V, size=(B, 64)).astype(np.int32)
    w["history"] = hist
    w["history_len"] = g.integers(0, 65, size=B).astype(np.int32)
    Wd = (V + 31) // 32
    bits = g.random((3, Wd * 32)) < np.array([[0.5], [0.02], [1.0]])
    bits[:, V:] = False
    w["mask_table"] = W.pack_mask(bits)
    w["state_id"] = g.integers(-1, 3, size=B).astype(np.int32)
    return w


@pytest.mark.parametrize("V,dtype,B", [(128256, "bf16", 16), (128256, "f32", 3), (50021, "f32", 160),
                                        (50021, "bf16", 16)])
def test_full_row_stages_without_topk(oracle_mod, sampler_factory, V, dtype, B):
    w = _nok_w(V, B, V + B, dtype)
    s = sampler_factory(V)
    s.path_counters()
    assert_same(oracle_mod, s, w, what=f"no-top-k full rows V={V} {dtype} B={B}")
    assert s.path_counters()["full_row"] > 0


def test_config4_batch_8192(oracle_mod, sampler_factory):
    """Config 4 at its larger batch ("batch 2048 (also
    8192)"): four streaming / finishing launch pairs of 2048 rows each."""
    w = W.make(4, seed=7, batch=8192)
    s = sampler_factory(w["vocab"], max_batch=8192)
    assert_same(oracle_mod, s, w, what="config 4 B=8192")


@pytest.mark.parametrize("make", ["sorted", "ties", "penalties", "masks"])
def test_edge_workloads_two_kernel_mode(oracle_mod, sampler_factory, make):
    """The edge workloads at 1100 rows: the two-kernel mode (streaming kernel
    with its in-kernel threshold retries, warp-group finisher, fallback kernel
    for the rows the finisher leaves)."""
    w = {"sorted": _sorted_w, "ties": _ties_w, "penalties": _pen_w, "masks": _masks_w}[make]()
    V = w["logits"].shape[1]
    s = sampler_factory(V)
    s.path_counters()
    assert_same(oracle_mod, s, _tile(w, 1100), what=f"{make} x1100 two-kernel")
    c = s.path_counters()
    assert c["candidate"] + c["full_row"] >= 1100
