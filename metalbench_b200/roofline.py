"""Roofline classification for B200 (replaces the reference's per-M-chip table,
mlx/scripts/roofline.py:12-82, with the same classify / format_line interface).

Peaks come from MEASURED_PEAKS.json at the repository root when present (a
STREAM-style copy and a cuBLAS bf16 GEMM measured on this pool's B200s);
otherwise the nominal figures below are used and labelled "nominal".
"""
from __future__ import annotations

import json
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]

NOMINAL = {"hbm_gbs": 7700.0, "bf16_tflops": 2250.0, "tf32_tflops": 1100.0}


def peaks() -> dict:
    p = dict(NOMINAL, source="nominal")
    try:
        m = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        p.update(hbm_gbs=float(m["hbm_gbs"]), bf16_tflops=float(m["bf16_tflops"]),
                 source="measured (MEASURED_PEAKS.json)")
        # tf32 dense is half the bf16 rate on B200; scale the measured bf16 figure
        p["tf32_tflops"] = p["bf16_tflops"] / 2.0
    except Exception:
        pass
    return p


def compute_peak_tflops(roof: str, pk: dict) -> float:
    """Tensor peak a kernel is held to: bf16 dense, or the effective fp32 rate of
    3xTF32 (three tf32 products per fp32 product)."""
    if roof == "tensor_tf32x3":
        return pk["tf32_tflops"] / 3.0
    return pk["bf16_tflops"]


def classify(roof: str, flops: float, bytes_: float, median_ms: float) -> dict:
    pk = peaks()
    sec = median_ms / 1e3
    tf = compute_peak_tflops(roof, pk)
    gflops = flops / sec / 1e9 if sec > 0 else 0.0
    gbps = bytes_ / sec / 1e9 if sec > 0 else 0.0
    ridge = tf * 1e3 / pk["hbm_gbs"]
    intensity = flops / bytes_ if bytes_ > 0 else 0.0
    sol_c = gflops / (tf * 1e3) if tf else 0.0
    sol_m = gbps / pk["hbm_gbs"]
    t_c = flops / (tf * 1e12) if tf else 0.0
    t_m = bytes_ / (pk["hbm_gbs"] * 1e9)
    if flops == 0 or roof == "hbm":
        cls, sol = "memory-bound", sol_m
    elif roof == "ridge":
        cls = "balanced (ridge)"
        sol = max(t_c, t_m) / sec if sec > 0 else 0.0  # time at the roof / time taken
    elif intensity > ridge:
        cls, sol = "compute-bound", sol_c
    else:
        cls, sol = "memory-bound", sol_m
    if median_ms < 0.02:
        cls += " (latency-dominated <20us)"
    return dict(classification=cls, sol=sol, sol_compute=sol_c, sol_memory=sol_m,
                intensity=intensity, ridge=ridge, gflops=gflops, gbps=gbps,
                peak={"hbm_gbs": pk["hbm_gbs"], "tensor_tflops": tf, "source": pk["source"]})


def format_line(m: dict) -> str:
    return (f"  roofline    : {m['classification']}  sol={m['sol'] * 100:.0f}%  "
            f"intensity={m['intensity']:.1f} vs ridge {m['ridge']:.1f}  "
            f"[peaks {m['peak']['source']}: {m['peak']['hbm_gbs']:.0f} GB/s, "
            f"{m['peak']['tensor_tflops']:.0f} TFLOP/s]")
