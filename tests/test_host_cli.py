"""mb200_host: the drop-in for the reference's metalbench_host subprocess
protocol (manifest JSON in, one JSON line out, outputs written to files)."""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
HOST = REPO / "metalbench_b200" / "mb200_host"


@pytest.fixture(scope="module")
def host():
    if not HOST.exists():
        from metalbench_b200 import build
        build.build()
    return HOST


def test_host_requires_manifest(host):
    p = subprocess.run([str(host)], capture_output=True, text=True)
    assert p.returncode == 1 and "missing --manifest" in p.stderr


def test_host_rejects_bad_json(host, tmp_path):
    m = tmp_path / "m.json"
    m.write_text("{not json")
    p = subprocess.run([str(host), "--manifest", str(m)], capture_output=True, text=True)
    assert p.returncode == 1 and "parse" in p.stderr


@pytest.mark.gpu
def test_host_runs_reference_manifest(host, tmp_path):
    """A manifest in the reference's format (mlx_helpers.build_manifest), naming
    the Metal function transpose_2d_f32."""
    a = np.random.default_rng(1).uniform(-1, 1, (1024, 2048)).astype(np.float32)
    a.tofile(tmp_path / "in_0.bin")
    manifest = {
        "function": "transpose_2d_f32", "metallib": "unused",
        "buffers": [
            {"binding": 0, "role": "input", "path": str(tmp_path / "in_0.bin")},
            {"binding": 1, "role": "output", "path": str(tmp_path / "out_1.bin"),
             "size": a.nbytes},
            {"binding": 2, "role": "scalar", "dtype": "u32", "value": 1024},
            {"binding": 3, "role": "scalar", "dtype": "u32", "value": 2048}],
        "grid": [131072, 1, 1], "threadgroup": [256, 1, 1], "warmup": 2, "iters": 5,
        "profile": False}
    (tmp_path / "m.json").write_text(json.dumps(manifest))
    p = subprocess.run([str(host), "--manifest", str(tmp_path / "m.json")], capture_output=True,
                       text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    line = json.loads(p.stdout.strip().splitlines()[-1])
    for k in ("chip", "metal_device", "tg_static_mem_bytes", "pso_max_threads_per_tg", "min_ms",
              "median_ms", "mean_ms", "iters", "available_counter_sets", "profiling"):
        assert k in line
    assert line["iters"] == 5 and line["chip"]["bucket"] == "b200"
    out = np.fromfile(tmp_path / "out_1.bin", dtype=np.float32).reshape(2048, 1024)
    assert out.tobytes() == np.ascontiguousarray(a.T).tobytes()
