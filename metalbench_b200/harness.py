"""MetalBench harness on B200: dispatch a kernel, time it, grade it.

    python mlx/scripts/harness.py <name> [--target speed|compute|memory|stable|balanced]
                                         [--iters N] [--warmup N] [--seed S]
                                         [--save] [--no-session] [--mlx-only | --metal-only]

Same flow, report lines, result files and exit code as the reference harness
(mlx/scripts/harness.py:52-508): seeded inputs -> native dispatch (here
libmb200's mb_run, in-process through ctypes, instead of the metalbench_host
subprocess) -> outputs compared with the MLX hook run on the CPU ->
speed / compute / memory / stable / balanced scores ->
results/<bucket>/<name>.json and session.json. Additions for B200: the
verdict is the reference's own (every element within atol + rtol*|b|); the
fraction of elements inside the tolerance is reported beside it together
with the north-star gate (>= 99 % of elements, ``gate_99``), bf16
inputs/outputs, a B200 roofline line, and the CPU core count of the
reference leg. The reference leg is real MLX when importable, else the numpy
MLX stand-in (labelled mlx-compat(numpy)).
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime as _dt
import importlib.util
import json
import os
import platform
import sys
import time
from pathlib import Path

import numpy as np

from . import _lib
from . import clocks, roofline

REPO_ROOT = Path(__file__).resolve().parents[1]
HOOK_ROOT = REPO_ROOT / "mlx" / "kernels"
CSRC = Path(__file__).resolve().parent / "csrc"
RESULTS_ROOT = REPO_ROOT / "results"
SESSION_PATH = REPO_ROOT / "session.json"
SETS = ("common", "standard", "full")
GATE_FRACTION = 0.99

DTYPE_NP = {"f32": np.float32, "bf16": np.uint16, "i32": np.int32, "u32": np.uint32}
DTYPE_BYTES = {"f32": 4, "bf16": 2, "i32": 4, "u32": 4, "f16": 2}

# kernel name -> CUDA sources that implement it (stored in session.json the way
# the reference stores the winning .metal source)
KERNEL_SOURCES = {
    "sqr_mm": ["gemm.cu", "gemm_core.cuh", "gemm_epi.cuh"],
    "gemm_bf16": ["gemm.cu", "gemm_core.cuh", "gemm_epi.cuh", "gemm_launch.cuh"],
    "transpose_2d": ["transpose.cu"],
    "transpose_batched": ["transpose.cu"],
    "conv2d": ["conv2d.cu", "gemm_core.cuh", "gemm_epi.cuh"],
    "llama_decoder_layer": ["decoder.cu", "decoder_epi.cuh", "attention.cu", "gemm_core.cuh"],
}


# ---------------------------------------------------------------------------
# bf16 helpers (numpy has no bf16: raw uint16 bit patterns)
# ---------------------------------------------------------------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# MLX (real or the numpy stand-in)
# ---------------------------------------------------------------------------
def ensure_mlx() -> str:
    try:
        import mlx.core  # noqa: F401
        mod = sys.modules["mlx"]
        if "mlx_compat" not in str(getattr(mod, "__file__", "")):
            return "mlx"
        return "mlx-compat(numpy)"
    except ImportError:
        # The repository's own mlx/ directory (the hook files) may have been
        # picked up as a namespace package; drop it before using the stand-in.
        for k in [k for k in sys.modules if k == "mlx" or k.startswith("mlx.")]:
            del sys.modules[k]
        sys.path.insert(0, str(Path(__file__).resolve().parent / "mlx_compat"))
        import mlx.core  # noqa: F401
        return "mlx-compat(numpy)"


# ---------------------------------------------------------------------------
# chip / device info (setup.cpp:116-136 equivalent through mb_device_info)
# ---------------------------------------------------------------------------
def chip_info() -> dict:
    d = _lib.MbDevice()
    try:
        _lib.call("mb_init", int(os.environ.get("LOCAL_RANK", "0")), 0, 1, None, 0)
        _lib.call("mb_device_info", C.byref(d))
        name, typ, bucket = d.name.decode(), d.type.decode(), d.bucket.decode()
    except Exception as e:  # no GPU: still describe the host
        name, typ, bucket = f"no GPU ({e})", "unknown", "unknown"
    return {"type": typ, "name": name, "bucket": bucket, "cpu_cores": os.cpu_count() or 0,
            "gpu_cores": d.sm_count, "ram_bytes": int(os.sysconf("SC_PAGE_SIZE") *
                                                      os.sysconf("SC_PHYS_PAGES")),
            "hbm_bytes": int(d.hbm_bytes), "cc": f"{d.cc_major}.{d.cc_minor}",
            "host": platform.node()}


# ---------------------------------------------------------------------------
# registry + hook loading (mlx_helpers.load_baseline equivalent)
# ---------------------------------------------------------------------------
def _exec_file(path: Path, modname: str):
    spec = importlib.util.spec_from_file_location(modname, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def registry_all() -> dict:
    out = {}
    for s in SETS:
        p = HOOK_ROOT / s / "registry.py"
        if p.exists():
            for k, v in _exec_file(p, f"_mb_registry_{s}").REGISTRY.items():
                out[k] = dict(v, set=s)
    return out


class Baseline:
    def __init__(self, name: str):
        reg = registry_all()
        if name not in reg:
            raise KeyError(f"no registry entry for '{name}' (known: {sorted(reg)})")
        self.name = name
        self.spec = reg[name]
        hook = self.spec.get("hook", name)
        path = HOOK_ROOT / self.spec["set"] / f"{hook}.py"
        if not path.exists():
            raise FileNotFoundError(f"hook not found: {path}")
        self.hook_path = path
        self._module = None

    @property
    def rtol(self):
        return float(self.spec.get("rtol", 1e-4))

    @property
    def atol(self):
        return float(self.spec.get("atol", 1e-5))

    def model(self):
        if self._module is None:
            ensure_mlx()
            self._module = _exec_file(self.hook_path, f"_mb_hook_{self.name}")
        return self._module.Model(**self.spec.get("model_kwargs", {}))

    def make_inputs(self, seed: int | None = None) -> list[np.ndarray]:
        """Seeded inputs per the registry (bf16 as uint16 bit patterns)."""
        seed = self.spec.get("seed", 0) if seed is None else seed
        rng = np.random.default_rng(seed)
        out = []
        for shape, dt, (dist, scale) in zip(self.spec["input_shapes"], self.spec["input_dtypes"],
                                            self.spec["input_init"]):
            if dist == "normal":
                a = rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
            elif dist == "uniform":
                a = rng.uniform(-scale, scale, shape).astype(np.float32)
            else:
                raise ValueError(f"unknown input distribution {dist}")
            out.append(f32_to_bf16_bits(a) if dt == "bf16" else a.astype(DTYPE_NP[dt]))
        return out

    def as_f32(self, inputs):
        return [bf16_bits_to_f32(x) if dt == "bf16" else x
                for x, dt in zip(inputs, self.spec["input_dtypes"])]

    def reference(self, inputs_f32):
        import mlx.core as mx
        out = self.model().forward(*[mx.array(x) for x in inputs_f32])
        mx.eval(out)
        return np.asarray(out, dtype=np.float32)


# ---------------------------------------------------------------------------
# native dispatch (replaces _run_host + metal/scripts/main.mm)
# ---------------------------------------------------------------------------
def run_kernel(b: Baseline, inputs: list[np.ndarray], warmup: int, iters: int,
               flush_l2: bool = False, profile: bool = False):
    """mb_run with host buffers: inputs uploaded, output copied back. Returns
    (timing dict in the reference's host JSON shape, output array)."""
    sp = b.spec
    out = np.empty(sp["output_shape"], dtype=DTYPE_NP[sp["output_dtype"]])
    out_binding = sp.get("output_binding", len(sp["input_bindings"]))
    if sp["kernel"] == "llama_decoder_layer":
        out_binding = 5
    bufs = (_lib.MbBuf * (len(inputs) + 1))()
    for i, (bind, x, dt) in enumerate(zip(sp["input_bindings"], inputs, sp["input_dtypes"])):
        x = np.ascontiguousarray(x)
        inputs[i] = x
        bufs[i] = _lib.MbBuf(bind, _lib.ROLE_INPUT, _lib.DTYPE[dt], 0, x.ctypes.data, x.nbytes)
    bufs[len(inputs)] = _lib.MbBuf(out_binding, _lib.ROLE_OUTPUT, _lib.DTYPE[sp["output_dtype"]],
                                   0, out.ctypes.data, out.nbytes)
    scal = sp.get("scalars", [])
    sc = (_lib.MbScalar * max(1, len(scal)))()
    for i, s in enumerate(scal):
        sc[i].binding, sc[i].dtype = s["binding"], _lib.DTYPE[s["dtype"]]
        if s["dtype"] == "f32":
            sc[i].v.f = float(s["value"])
        elif s["dtype"] == "i32":
            sc[i].v.i = int(s["value"])
        else:
            sc[i].v.u = int(s["value"])
    cfg = dict(sp.get("config", {}))
    if flush_l2:
        cfg["flush_l2"] = True
    if profile:
        cfg["profile"] = True
    t = _lib.MbTiming()
    dev = int(os.environ.get("LOCAL_RANK", "0"))
    _lib.call("mb_init", dev, 0, 1, None, 0)
    # SM clocks and throttle reasons sampled (NVML, read only) while mb_run
    # runs: a per-kernel number counts only with its clock record
    sampler = clocks.NvmlSampler(dev)
    sampler.start()
    try:
        _lib.call("mb_run", sp["kernel"].encode(), bufs, len(inputs) + 1, sc, len(scal),
                  json.dumps(cfg).encode(), warmup, iters, C.byref(t))
    finally:
        sampler.stop()
    timing = {"min_ms": t.min_ms, "median_ms": t.median_ms, "mean_ms": t.mean_ms,
              "iters": t.iters, "h2d_ms": t.h2d_ms, "d2h_ms": t.d2h_ms}
    extra = {"tg_static_mem_bytes": t.smem_bytes, "pso_max_threads_per_tg": t.threads_per_cta,
             "metal_device": None, "clocks": sampler.summary(),
             "profiling": {"counters_available": False, "enabled": bool(profile),
                           "profile_ms": t.profile_ms if profile else None,
                           "nvtx_range": f"mb_profile:{sp['kernel']}",
                           "timed_nvtx_range": f"mb_timed:{sp['kernel']}"}}
    return timing, extra, out


def time_reference(fn, warmup: int, iters: int) -> dict:
    """Wall-clock min/median/mean of fn() (mlx/scripts/timing.py:31-72 rules)."""
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        times.append((time.perf_counter() - t0) * 1000.0)
    times.sort()
    return {"min_ms": times[0], "median_ms": times[len(times) // 2],
            "mean_ms": sum(times) / len(times), "iters": iters}


def compare(actual: np.ndarray, expected: np.ndarray, rtol: float, atol: float) -> dict:
    """The reference gate all(|a-b| <= atol + rtol*|b|) (harness.py:26-33):
    correct = every element inside it. Reported beside it: the fraction of
    elements inside, ``gate_99`` (that fraction >= 99 %, the north-star
    gate) and ``atol_needed``, the smallest atol that would pass every
    element at this rtol."""
    a = np.asarray(actual, dtype=np.float64)
    b = np.asarray(expected, dtype=np.float64)
    if a.shape != b.shape:
        return {"all_within": False, "frac_within_tol": 0.0, "max_err": float("inf"),
                "correct": False, "gate_99": False, "atol_needed": float("inf")}
    if a.size == 0:
        return {"all_within": True, "frac_within_tol": 1.0, "max_err": 0.0, "correct": True,
                "gate_99": True, "atol_needed": 0.0}
    diff = np.abs(a - b)
    ok = (diff <= atol + rtol * np.abs(b)) & ~np.isnan(a)
    frac = float(ok.mean())
    need = 1.0 if (rtol == 0 and atol == 0) else GATE_FRACTION
    nan = bool(np.isnan(a).any())
    return {"all_within": bool(ok.all()), "frac_within_tol": frac,
            "max_err": float(np.nanmax(diff)), "correct": bool(ok.all()),
            "gate_99": frac >= need, "err_std": float(np.nanstd(a - b)),
            "atol_needed": float("inf") if nan else float(max(0.0, (diff - rtol * np.abs(b)).max()))}


def evaluate(name: str, *, seed=None, warmup=10, iters=200, solo=None, ref_warmup=None,
             ref_iters=None, flush_l2=False, profile=False):
    b = Baseline(name)
    sp = b.spec
    inputs = b.make_inputs(seed)
    chip = chip_info()
    ref_label = ensure_mlx()
    rw = sp.get("ref_warmup", 2) if ref_warmup is None else ref_warmup
    ri = sp.get("ref_iters", 10) if ref_iters is None else ref_iters
    flops, nbytes = float(sp.get("flops", 0)), float(sp.get("bytes", 0))
    result = {"task": name, "chip": chip, "reference_impl": ref_label,
              "reference_cpu_threads": os.cpu_count(), "kernel": sp["kernel"]}

    k_t = extra = out = None
    if solo != "mlx":
        k_t, extra, out = run_kernel(b, inputs, warmup, iters, flush_l2=flush_l2, profile=profile)
        result.update(extra)
        result["kernel_timing"] = k_t
    r_t = ref = None
    if solo != "metal":
        inputs_f32 = b.as_f32(inputs)
        t0 = time.perf_counter()
        ref = b.reference(inputs_f32)
        first_ms = (time.perf_counter() - t0) * 1000.0
        if rw == 0 and ri == 1:  # expensive references: the checked call is the timed one
            r_t = {"min_ms": first_ms, "median_ms": first_ms, "mean_ms": first_ms, "iters": 1}
        else:
            r_t = time_reference(lambda: b.reference(inputs_f32), rw, ri)
        result["reference_timing"] = r_t

    m = {}
    outputs = []
    correct = True
    if out is not None and ref is not None:
        got = bf16_bits_to_f32(out) if sp["output_dtype"] == "bf16" else out.astype(np.float32)
        cmp = compare(got, ref.reshape(got.shape), b.rtol, b.atol)
        outputs.append(dict(binding=len(sp["input_bindings"]), **cmp))
        result["ref_abs_max"] = float(np.abs(ref).max()) if ref.size else 0.0
        correct = cmp["correct"]
    t_main = k_t if k_t is not None else r_t
    sec = t_main["median_ms"] / 1000.0
    if sec > 0:
        if flops:
            m["gflops"] = flops / sec / 1e9
        if nbytes:
            m["gbps"] = nbytes / sec / 1e9
        if flops and nbytes:
            m["arith_intensity"] = flops / nbytes
    if k_t is not None and r_t is not None and k_t["median_ms"] > 0:
        m["speedup"] = r_t["median_ms"] / k_t["median_ms"]
    m["stability"] = max(0.0, 1.0 - abs(t_main["median_ms"] - t_main["mean_ms"]) /
                         t_main["mean_ms"]) if t_main["mean_ms"] > 0 else 0.0
    if k_t is not None:
        rl = roofline.classify(sp.get("roof", "hbm"), flops, nbytes, k_t["median_ms"])
        result["roofline"] = rl
    result.update(correct=correct, metrics=m, outputs=outputs)
    if solo:
        result["solo"] = solo
    return result


# ---------------------------------------------------------------------------
# grading, leaderboard, report (harness.py:176-333 semantics)
# ---------------------------------------------------------------------------
TARGETS = {
    "speed": lambda m: m.get("speedup", 0.0),
    "compute": lambda m: m.get("gflops", 0.0),
    "memory": lambda m: m.get("gbps", 0.0),
    "stable": lambda m: m.get("stability", 0.0),
    "balanced": lambda m: (0.5 * m.get("speedup", 0.0) + 0.3 * (m.get("gflops", 0.0) / 1000.0)
                           + 0.2 * m.get("stability", 0.0)),
}


def grade(metrics: dict, target: str) -> float:
    if target not in TARGETS:
        raise SystemExit(f"unknown target '{target}'; pick {list(TARGETS)}")
    return float(TARGETS[target](metrics))


def kernel_source(kernel: str) -> tuple[str, str]:
    files = KERNEL_SOURCES.get(kernel, [])
    text = "".join(f"// ===== {f} =====\n{(CSRC / f).read_text()}\n" for f in files
                   if (CSRC / f).exists())
    rel = ",".join(f"metalbench_b200/csrc/{f}" for f in files)
    return rel, text


def git_sha() -> str | None:
    try:
        import subprocess
        return subprocess.run(["git", "-C", str(REPO_ROOT), "rev-parse", "HEAD"],
                              capture_output=True, text=True, timeout=5).stdout.strip() or None
    except Exception:
        return None


def update_session(name: str, result: dict, target: str, iters: int):
    """session.json[bucket][name] keeps the best (lowest kernel median) correct
    run with the CUDA source that produced it (harness.py:196-247)."""
    if not result.get("correct"):
        return False, "skipped (incorrect)"
    if (result.get("clocks") or {}).get("rejected"):
        return False, "skipped (clock record rejected: throttled or clocks pinned low)"
    bucket = result["chip"]["bucket"]
    new_ms = result["kernel_timing"]["median_ms"]
    session = {}
    if SESSION_PATH.exists():
        try:
            session = json.loads(SESSION_PATH.read_text())
        except Exception:
            session = {}
    sec = session.setdefault(bucket, {})
    prev = sec.get(name)
    prev_ms = prev["best_time_ms"] if prev else None
    if prev_ms is not None and new_ms >= prev_ms:
        return False, f"current best {prev_ms:.3f} ms holds (this run {new_ms:.3f} ms)"
    rel, text = kernel_source(result["kernel"])
    m = result["metrics"]
    sec[name] = {
        "best_time_ms": new_ms, "speedup_vs_mlx": m.get("speedup"), "gflops": m.get("gflops"),
        "gbps": m.get("gbps"), "arith_intensity": m.get("arith_intensity"),
        "stability": m["stability"], "tg_static_mem_bytes": result.get("tg_static_mem_bytes"),
        "pso_max_threads_per_tg": result.get("pso_max_threads_per_tg"), "iters": iters,
        "target": target, "max_err": max((o["max_err"] for o in result["outputs"]), default=0.0),
        "frac_within_tol": min((o["frac_within_tol"] for o in result["outputs"]), default=1.0),
        "roofline_sol": result.get("roofline", {}).get("sol"),
        "reference_impl": result.get("reference_impl"),
        "clocks": result.get("clocks"),
        "metal_source_path": rel, "metal_source": text, "git_sha": git_sha(),
        "updated_at": _dt.datetime.now(_dt.timezone.utc).isoformat(timespec="seconds"),
    }
    SESSION_PATH.write_text(json.dumps(session, indent=2) + "\n")
    delta = "" if prev_ms is None else f" (was {prev_ms:.3f} ms, Δ {prev_ms - new_ms:+.3f})"
    return True, f"new best {new_ms:.3f} ms{delta}"


def print_report(result: dict, target: str, score: float) -> None:
    chip, m = result["chip"], result["metrics"]
    k_t, r_t = result.get("kernel_timing"), result.get("reference_timing")
    outs = result.get("outputs", [])
    line = "─" * 72
    ref_name = result.get("reference_impl", "mlx")
    print(line)
    solo = result.get("solo")
    head = f"  {result['task']}    " + (f"[{'MLX' if solo == 'mlx' else 'kernel'} only]" if solo
                                      else f"target={target}   score={score:.3f}")
    print(head)
    print(line)
    print(f"  device      : {chip['name']} ({chip['type']})  {chip['cpu_cores']} CPU / "
          f"{chip['gpu_cores']} SM / {chip['ram_bytes'] / 1e9:.0f} GB")
    if k_t is not None and result.get("tg_static_mem_bytes") is not None:
        print(f"  occupancy   : smem/CTA={result['tg_static_mem_bytes'] / 1024:.0f}KB  "
              f"threads/CTA={result['pso_max_threads_per_tg']}")
    print()
    if not solo:
        status = "✓ correct " if result["correct"] else "✗ INCORRECT"
        max_err = max((o["max_err"] for o in outs), default=0.0)
        frac = min((o["frac_within_tol"] for o in outs), default=1.0)
        print(f"  correctness : {status}    max_err={max_err:.3e}  within_tol={frac * 100:.3f}%")
        g99 = all(o.get("gate_99", True) for o in outs)
        print(f"  gate_99     : {'✓' if g99 else '✗'} (>= 99 % of elements within tolerance)")
        print(f"  speedup     : {m.get('speedup', 0):.2f}× vs MLX ({ref_name}, "
              f"{result.get('reference_cpu_threads')} CPU threads)")
    if k_t is not None:
        print(f"  kernel      : {k_t['median_ms']:.3f} ms  (min {k_t['min_ms']:.3f}, "
              f"mean {k_t['mean_ms']:.3f}, n={k_t['iters']})")
    if r_t is not None:
        print(f"  mlx ref     : {r_t['median_ms']:.3f} ms  (min {r_t['min_ms']:.3f}, "
              f"mean {r_t['mean_ms']:.3f}, n={r_t['iters']})")
    if "gflops" in m:
        print(f"  compute     : {m['gflops']:.1f} GFLOPS")
    if "gbps" in m:
        print(f"  bandwidth   : {m['gbps']:.1f} GB/s")
    if "arith_intensity" in m:
        print(f"  arith int.  : {m['arith_intensity']:.1f} FLOPs/byte")
    print(f"  stability   : {m['stability']:.2f}  (1.0 = perfectly consistent)")
    if "roofline" in result:
        print(roofline.format_line(result["roofline"]))
    ck = result.get("clocks")
    if ck:
        verdict = ("REJECTED (throttled or clocks pinned low)" if ck.get("rejected")
                   else "ok" if ck.get("rejected") is False else "no samples")
        sm = f"{ck['sm_mhz']:.0f}" if ck.get("sm_mhz") else "?"
        print(f"  clocks      : SM {sm} / {ck.get('sm_max_mhz') or 0:.0f} MHz  "
              f"reasons={','.join(ck.get('reasons', [])) or '-'}  n={ck.get('samples', 0)}  "
              f"[{verdict}]")
    pf = result.get("profiling", {})
    if pf.get("enabled"):
        print(f"  profile     : 1 extra dispatch {pf.get('profile_ms', 0):.3f} ms in NVTX range "
              f"'{pf['nvtx_range']}' (ncu --nvtx --nvtx-include \"{pf['nvtx_range']}/\")")
    if not solo:
        print()
        print(f"  {'target':>10s}   {'score':>10s}")
        print(f"  {'-' * 10}   {'-' * 10}")
        for t in TARGETS:
            print(f"  {t:>10s}   {grade(m, t):10.3f}")
    print(line)


def update_best_times_md() -> None:
    """Regenerate best_times.md and LINK.md from session.json (all chip buckets;
    scripts/render_best_times.py and render_link_md.py in the reference)."""
    from metalbench_b200 import leaderboard
    leaderboard.render_best_times()
    leaderboard.render_link_md()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="metalbench-harness")
    ap.add_argument("name", nargs="?")
    ap.add_argument("--_update_md", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--list", action="store_true", help="list registry entries")
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--ref-warmup", type=int, default=None)
    ap.add_argument("--ref-iters", type=int, default=None)
    ap.add_argument("--flush-l2", action="store_true", help="write 2x L2 between timed launches")
    ap.add_argument("--profile", action="store_true",
                    help="one extra dispatch inside an NVTX range for an outside profiler (ncu)")
    ap.add_argument("--save", action="store_true")
    ap.add_argument("--no-session", action="store_true")
    ap.add_argument("--target", default="speed", choices=list(TARGETS))
    solo = ap.add_mutually_exclusive_group()
    solo.add_argument("--mlx-only", action="store_true")
    solo.add_argument("--metal-only", "--kernel-only", dest="metal_only", action="store_true")
    args = ap.parse_args(argv)
    if args._update_md:
        update_best_times_md()
        return 0
    if args.list:
        for n, v in sorted(registry_all().items()):
            print(f"{v['set']:9s} {n:28s} kernel={v['kernel']}")
        return 0
    if not args.name:
        ap.error("kernel name required (or use --all from the bench script)")
    solo_mode = "mlx" if args.mlx_only else ("metal" if args.metal_only else None)
    result = evaluate(args.name, seed=args.seed, warmup=args.warmup, iters=args.iters,
                      solo=solo_mode, ref_warmup=args.ref_warmup, ref_iters=args.ref_iters,
                      flush_l2=args.flush_l2, profile=args.profile)
    score = grade(result["metrics"], args.target)
    result["target"], result["score"] = args.target, score
    print(f"[chip] {result['chip']['type']:>8s}  '{result['chip']['name']}'  "
          f"cpu={result['chip']['cpu_cores']}  sm={result['chip']['gpu_cores']}",
          file=sys.stderr)
    print_report(result, args.target, score)
    if solo_mode:
        return 0
    if args.save:
        out_dir = RESULTS_ROOT / result["chip"]["bucket"]
        out_dir.mkdir(parents=True, exist_ok=True)
        p = out_dir / f"{args.name}.json"
        p.write_text(json.dumps(result, indent=2, default=float))
        print(f"saved → {p.relative_to(REPO_ROOT)}", file=sys.stderr)
    if not args.no_session:
        updated, why = update_session(args.name, result, args.target, args.iters)
        prefix = "updated session.json" if updated else "session.json unchanged"
        print(f"{prefix} [{result['chip']['bucket']}/{args.name}]: {why}", file=sys.stderr)
    return 0 if result["correct"] else 1


if __name__ == "__main__":
    sys.exit(main())
