"""best_times.md / LINK.md rendering and certify's kernel discovery (the
reference's scripts/render_best_times.py, scripts/render_link_md.py and
certify:20-43), on a synthetic session.json; no GPU."""
import json
import subprocess
from pathlib import Path

from metalbench_b200 import leaderboard as lb

REPO = Path(__file__).resolve().parents[1]


def _session(tmp_path):
    s = {"apple-m2": {"sqr_mm": {"best_time_ms": 1.25, "speedup_vs_mlx": 2.0}},
         "b200": {"sqr_mm": {"best_time_ms": 0.119, "speedup_vs_mlx": 100.0, "roofline_sol": 0.57},
                  "conv2d": {"best_time_ms": 0.021, "speedup_vs_mlx": 0.0}}}
    p = tmp_path / "session.json"
    p.write_text(json.dumps(s))
    return p


def test_best_times_has_every_registry_kernel_and_a_b200_column(tmp_path):
    out = lb.render_best_times(tmp_path / "bt.md", _session(tmp_path))
    text = out.read_text()
    assert "| kernel | set | M1 | M2 | M3 | M4 | M5 | B200 | B200 SoL |" in text
    row = next(line for line in text.splitlines() if line.startswith("| `sqr_mm`"))
    assert row == "| `sqr_mm` | common | — | 1.250 (2.00×) | — | — | — | 0.119 (100.00×) | 57 % |"
    conv = next(line for line in text.splitlines() if line.startswith("| `conv2d`"))
    assert "0.021" not in conv  # no speedup recorded -> "—", as in the reference
    from metalbench_b200 import harness
    for name in harness.registry_all():
        assert f"| `{name}` |" in text


def test_link_md_links_b200_kernels_to_their_cuda_sources(tmp_path):
    text = lb.render_link_md(tmp_path / "LINK.md", _session(tmp_path)).read_text()
    assert "## apple-m1 _(no data)_" in text and "## b200" in text
    b200 = text.split("## b200")[1]
    assert "- [sqr_mm](metalbench_b200/csrc/gemm.cu)" in b200
    for line in b200.splitlines():
        if line.startswith("- ["):
            for target in line.split("(")[1:]:
                assert (REPO / target.split(")")[0]).exists(), line


def test_kernels_for_maps_changes_to_registry_names():
    assert lb.kernels_for(["metalbench_b200/csrc/conv2d.cu"]) == ["conv2d"]
    assert lb.kernels_for(["metalbench_b200/csrc/f32_paths.cu"]) == ["conv2d_f32",
                                                                      "llama_decoder_layer_f32"]
    assert "swiglu" in lb.kernels_for(["mlx/kernels/standard/swiglu.py"])
    assert {"sqr_mm", "rect_mm", "batch_mm"} <= set(lb.kernels_for(["metalbench_b200/csrc/gemm.cu"]))
    from metalbench_b200 import harness
    assert set(lb.kernels_for(["metalbench_b200/csrc/common.cuh"])) == set(harness.registry_all())
    for v in harness.registry_all().values():
        assert lb.sources_for(v["kernel"]), v["kernel"]


def test_certify_script_parses():
    assert subprocess.run(["bash", "-n", str(REPO / "certify")]).returncode == 0


def test_certify_parses_the_harness_report(capsys):
    """certify extracts time, speedup, GFLOPS and GB/s from the report lines
    with awk field positions (the reference's certify:66-71); pin them on a
    report printed from a synthetic result."""
    from metalbench_b200 import harness as Hm
    res = {"task": "sqr_mm", "correct": True, "solo": None, "reference_impl": "mlx-compat",
           "reference_cpu_threads": 16, "tg_static_mem_bytes": 197752,
           "pso_max_threads_per_tg": 256,
           "chip": {"name": "NVIDIA B200", "type": "b200", "cpu_cores": 16, "gpu_cores": 148,
                    "ram_bytes": 2e11},
           "outputs": [{"max_err": 4.3e-4, "frac_within_tol": 1.0}],
           "kernel_timing": {"median_ms": 0.115, "min_ms": 0.113, "mean_ms": 0.116, "iters": 200},
           "reference_timing": {"median_ms": 12.0, "min_ms": 11.9, "mean_ms": 12.1, "iters": 5},
           "metrics": {"speedup": 104.3, "gflops": 149389.1, "gbps": 437.7,
                       "arith_intensity": 341.3, "stability": 0.99}}
    Hm.print_report(res, "speed", 104.3)
    out = capsys.readouterr().out
    script = r"""
      ms=$(awk '/^  kernel  /   { gsub(/ms/,"",$3); print $3; exit }' <<<"$OUT")
      sp=$(awk '/^  speedup/    { gsub(/×/,"",$3); print $3; exit }' <<<"$OUT")
      gf=$(awk '/^  compute/    { print $3; exit }' <<<"$OUT")
      gb=$(awk '/^  bandwidth/  { print $3; exit }' <<<"$OUT")
      grep -q "correctness : ✓ correct" <<<"$OUT" && echo "$ms $sp $gf $gb"
    """
    r = subprocess.run(["bash", "-c", script], env={"OUT": out, "PATH": "/usr/bin:/bin"},
                       capture_output=True, text=True)
    assert r.stdout.split() == ["0.115", "104.30", "149389.1", "437.7"], (r.stdout, out)
