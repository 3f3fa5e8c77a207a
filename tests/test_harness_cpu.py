"""Harness, registry and reference hooks on CPU (no GPU): the shape of the
reference's tests/metalbench/test_bench_smoke.py plus hook-vs-oracle parity."""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle.ops as O
from metalbench_b200 import harness as Hm

REPO = Path(__file__).resolve().parents[1]


def test_bench_cli_usage():
    p = subprocess.run([str(REPO / "bench")], capture_output=True, text=True)
    assert p.returncode == 64 and "usage" in p.stderr
    p = subprocess.run([str(REPO / "bench"), "--help"], capture_output=True, text=True)
    assert p.returncode == 0 and "usage" in p.stdout


def test_registry_entries_well_formed():
    reg = Hm.registry_all()
    for name in ("sqr_mm", "transpose_2d", "transpose_batched_bf16", "conv2d",
                 "llama_decoder_layer", "llama_decoder_layer_decode", "gemm_bf16"):
        assert name in reg, name
    for name, e in reg.items():
        n = len(e["input_bindings"])
        assert len(e["input_shapes"]) == n == len(e["input_dtypes"]) == len(e["input_init"]), name
        assert e["kernel"] and e["output_dtype"] in ("f32", "bf16")
        b = Hm.Baseline(name)
        assert b.hook_path.exists()


def test_inputs_are_seeded_and_typed():
    b = Hm.Baseline("conv2d")
    x1, w1 = b.make_inputs()
    x2, _ = b.make_inputs()
    assert x1.dtype == np.uint16 and x1.shape == (32, 56, 56, 64)
    assert np.array_equal(x1, x2)
    w = Hm.bf16_bits_to_f32(w1)
    assert abs(float(w.std()) - (2.0 / 576) ** 0.5) < 0.01  # He-normal


def _hook(name, **kw):
    Hm.ensure_mlx()
    b = Hm.Baseline(name)
    mod = Hm._exec_file(b.hook_path, f"_t_{name}")
    return mod.Model(**kw)


def test_hooks_match_oracle_common():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((33, 17)).astype(np.float32)
    B = rng.standard_normal((17, 9)).astype(np.float32)
    np.testing.assert_allclose(_hook("sqr_mm").forward(A, B), O.sqr_mm(A, B), rtol=1e-5, atol=1e-5)
    T = rng.standard_normal((3, 5, 7)).astype(np.float32)
    assert np.array_equal(_hook("transpose_2d").forward(T), O.transpose_2d(T))
    assert np.array_equal(_hook("transpose_2d").forward(A), A.T)
    x = rng.standard_normal((2, 6, 5, 8)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 8)).astype(np.float32)
    m = _hook("conv2d", in_channels=8, out_channels=4, kernel_size=3, stride=1, padding=1)
    np.testing.assert_allclose(m.forward(x, w), O.conv2d_nhwc(x, w, padding=1), rtol=1e-5,
                               atol=1e-4)


@pytest.mark.parametrize("causal,past", [(False, 0), (True, 0), (True, 5)])
def test_decoder_hook_matches_oracle(causal, past):
    rng = np.random.default_rng(1)
    B, S, D, H, Hkv, FF = 2, 6, 64, 4, 2, 96
    r = lambda *s: (rng.standard_normal(s) * 0.2).astype(np.float32)
    W = [r(D, D + 2 * Hkv * 16), r(D, D), r(D, 2 * FF), r(FF, D)]
    x = rng.standard_normal((B, S, D)).astype(np.float32)
    kp = vp = None
    if past:
        kp, vp = r(B, Hkv, past, 16), r(B, Hkv, past, 16)
    m = _hook("llama_decoder_layer", S=S, D=D, H=H, H_kv=Hkv, FF=FF, base=500000.0,
              causal=causal)
    got = m.forward(x, *W, kp, vp) if past else m.forward(x, *W)
    ref = O.decoder_layer(x, *W, H=H, H_kv=Hkv, base=500000.0, causal=causal, k_past=kp,
                          v_past=vp)
    np.testing.assert_allclose(got, ref, rtol=2e-4, atol=2e-4)


def test_decoder_hook_reference_defaults_match_golden():
    """Default arguments reproduce the reference hook (golden fixture)."""
    d = np.load(REPO / "tests" / "golden" / "llama_decoder_layer.npz")
    got = _hook("llama_decoder_layer").forward(*[d[f"in{i}"] for i in range(5)])
    assert np.abs(got - d["out"]).max() / np.abs(d["out"]).max() < 1e-5


def test_compare_gate():
    a = np.arange(1000, dtype=np.float32)
    b = a.copy()
    b[:5] += 1.0  # 0.5 % off
    r = Hm.compare(a, b, rtol=0.0, atol=0.1)
    # the reference verdict needs every element; the 99 % gate is reported beside it
    assert r["frac_within_tol"] == pytest.approx(0.995) and not r["correct"] and r["gate_99"]
    assert not r["all_within"] and r["atol_needed"] == pytest.approx(1.0)
    assert not Hm.compare(a, b, rtol=0, atol=0)["gate_99"]  # bit-exact entries need 100 %
    assert Hm.compare(a, b, rtol=0.0, atol=1.0)["correct"]
    b[:20] += 1.0
    assert not Hm.compare(a, b, rtol=0.0, atol=0.1)["gate_99"]


def test_update_session_keeps_best_and_skips_incorrect(tmp_path, monkeypatch):
    monkeypatch.setattr(Hm, "SESSION_PATH", tmp_path / "session.json")
    res = {"correct": True, "chip": {"bucket": "b200"}, "kernel": "transpose_2d",
           "kernel_timing": {"median_ms": 1.0}, "metrics": {"stability": 1.0, "speedup": 2.0},
           "outputs": [{"max_err": 0.0, "frac_within_tol": 1.0}]}
    assert Hm.update_session("transpose_2d", res, "speed", 10)[0]
    res["kernel_timing"]["median_ms"] = 2.0
    assert not Hm.update_session("transpose_2d", res, "speed", 10)[0]
    res["kernel_timing"]["median_ms"] = 0.5
    assert Hm.update_session("transpose_2d", res, "speed", 10)[0]
    s = json.loads((tmp_path / "session.json").read_text())
    assert s["b200"]["transpose_2d"]["best_time_ms"] == 0.5
    assert "transpose" in s["b200"]["transpose_2d"]["metal_source"]
    res["correct"] = False
    assert Hm.update_session("transpose_2d", res, "speed", 10) == (False, "skipped (incorrect)")


def test_grade_targets():
    m = {"speedup": 2.0, "gflops": 1000.0, "gbps": 5.0, "stability": 0.5}
    assert Hm.grade(m, "balanced") == pytest.approx(0.5 * 2 + 0.3 * 1 + 0.2 * 0.5)
    assert Hm.grade(m, "memory") == 5.0


@pytest.mark.parametrize("name,nin", [("rms_norm_linear", 2), ("fused_add_rms_norm", 2),
                                      ("rope_embedding", 1), ("swiglu", 3),
                                      ("scaled_dot_product", 3), ("fused_qkv_projection", 2),
                                      ("rect_mm", 2), ("batch_mm", 2), ("llama_attention", 3), ("sqr_mm", 2),
                                      ("transformer_block", 5), ("mha_attention", 5),
                                      ("transpose_2d", 1)])
def test_our_hooks_reproduce_reference_hooks(name, nin):
    """Each hook under mlx/kernels/ (default arguments) reproduces the golden
    output of the reference's own hook on the same inputs."""
    d = np.load(REPO / "tests" / "golden" / f"{name}.npz")
    got = np.asarray(_hook(name).forward(*[d[f"in{i}"] for i in range(nin)]))
    scale = max(1.0, float(np.abs(d["out"]).max()))
    assert got.shape == d["out"].shape
    assert np.abs(got - d["out"]).max() <= 1e-4 * scale, name
