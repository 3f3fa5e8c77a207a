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


def _manifest_for(tmp_path, function, inputs, out_shape, scalars):
    """The manifest exactly as the reference's mlx_helpers.build_manifest
    (mlx/scripts/mlx_helpers.py:290-335) builds it: f32 input files, the
    output at binding len(inputs) with its byte size, u32/f32 scalars."""
    bufs = []
    for i, x in enumerate(inputs):
        p = tmp_path / f"in_{i}.bin"
        np.ascontiguousarray(x, dtype=np.float32).tofile(p)
        bufs.append({"binding": i, "role": "input", "path": str(p)})
    outp = tmp_path / f"out_{len(inputs)}.bin"
    bufs.append({"binding": len(inputs), "role": "output", "path": str(outp),
                 "size": int(np.prod(out_shape)) * 4})
    for b, dt, v in scalars:
        bufs.append({"binding": b, "role": "scalar", "dtype": dt, "value": v})
    m = {"function": function, "metallib": "unused", "buffers": bufs, "grid": [65536, 1, 1],
         "threadgroup": [1024, 1, 1], "warmup": 1, "iters": 3, "profile": False}
    (tmp_path / "m.json").write_text(json.dumps(m))
    return tmp_path / "m.json", outp


def _run_manifest(host, mpath, outp, out_shape):
    p = subprocess.run([str(host), "--manifest", str(mpath)], capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stderr
    json.loads(p.stdout.strip().splitlines()[-1])
    return np.fromfile(outp, dtype=np.float32).reshape(out_shape)


@pytest.mark.gpu
def test_host_runs_reference_conv2d_f32_manifest(host, tmp_path):
    """The reference's conv2d entry (common/registry.py:469-477): fp32, pad 0,
    scalars N,H,W,Cin,Cout,KH,KW,stride at bindings 3..10, rtol = atol = 1e-3
    on every element. Checked on the committed golden (made by the reference
    hook) and at the registry's own shape (8,64,64,64) * (128,3,3,64)."""
    import oracle.ops as O
    g = np.load(REPO / "tests" / "golden" / "conv2d.npz")
    x, w, want = g["in0"], g["in1"], g["out"]
    N, H, W, C = x.shape
    Co = w.shape[0]
    sc = [(3 + i, "u32", v) for i, v in enumerate((N, H, W, C, Co, 3, 3, 1))]
    m, o = _manifest_for(tmp_path, "conv2d_f32", [x, w], want.shape, sc)
    got = _run_manifest(host, m, o, want.shape)
    assert np.all(np.abs(got - want) <= 1e-3 + 1e-3 * np.abs(want))
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8, 64, 64, 64), dtype=np.float32)
    w = rng.standard_normal((128, 3, 3, 64), dtype=np.float32)
    sc = [(3 + i, "u32", v) for i, v in enumerate((8, 64, 64, 64, 128, 3, 3, 1))]
    m, o = _manifest_for(tmp_path, "conv2d_f32", [x, w], (8, 62, 62, 128), sc)
    got = _run_manifest(host, m, o, (8, 62, 62, 128))
    want = O.conv2d_nhwc(x, w, padding=0, acc=np.float64)
    assert np.all(np.abs(got - want) <= 1e-3 + 1e-3 * np.abs(want))


@pytest.mark.gpu
def test_host_runs_reference_llama_decoder_f32_manifest(host, tmp_path):
    """The reference's llama_decoder_layer entry (full/registry.py:87-104):
    fp32, S 64, D 128, H 4 / H_kv 2 (head_dim 32), FF 256, rtol = atol = 1e-2
    on every element against the float64 oracle, and against the golden the
    reference hook produced up to that golden's own fp32 error."""
    g = np.load(REPO / "tests" / "golden" / "llama_decoder_layer.npz")
    ins = [g[f"in{i}"] for i in range(5)]
    want = g["out"]
    sc = [(6, "u32", 64), (7, "u32", 128), (8, "u32", 4), (9, "u32", 2), (10, "u32", 256),
          (11, "f32", 10000.0), (12, "f32", 1e-5)]
    m, o = _manifest_for(tmp_path, "llama_decoder_layer_f32", ins, want.shape, sc)
    got = _run_manifest(host, m, o, want.shape)
    import oracle.ops as O
    from _f32check import check_against_fp32_golden
    exact = O.decoder_layer(ins[0], *ins[1:], H=4, H_kv=2, base=10000.0, acc=np.float64)
    check_against_fp32_golden(got, want, exact, 1e-2)
