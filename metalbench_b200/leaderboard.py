"""Leaderboard files regenerated from session.json: best_times.md and LINK.md.

B200 counterparts of the reference's scripts/render_best_times.py (one row per
registry kernel, one column per chip: best time and speedup vs MLX) and
scripts/render_link_md.py (per chip, a link to the source of every kernel).
The reference enumerates kernels from metal/kernels/<set>/ and hard-codes the
chips apple-m1..m5; here the kernels are the registry entries of
mlx/kernels/<set>/registry.py, the chips are apple-m1..m5 followed by every
other bucket present in session.json (b200), and a kernel's source is the
libmb200 CUDA file that implements it.

    python -m metalbench_b200.leaderboard            # both files
    python -m metalbench_b200.leaderboard best-times
    python -m metalbench_b200.leaderboard link-md
    python -m metalbench_b200.leaderboard kernels-for FILE...   # registry names a change touches
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
APPLE_CHIPS = ["apple-m1", "apple-m2", "apple-m3", "apple-m4", "apple-m5"]
SETS = ("common", "standard", "full")

CSRC = "metalbench_b200/csrc"
# libmb200 kernel (registry "kernel" field) -> the CUDA sources implementing it
KERNEL_SOURCES = {
    "transpose_2d": ["transpose.cu"],
    "transpose_batched": ["transpose.cu"],
    "sqr_mm": ["gemm.cu", "gemm_core.cuh", "gemm_epi.cuh"],
    "batch_mm": ["gemm.cu", "gemm_core.cuh", "gemm_epi.cuh"],
    "gemm_bf16": ["gemm.cu", "gemm_core.cuh", "gemm_epi.cuh", "gemm_launch.cuh"],
    "conv2d": ["conv2d.cu", "gemm_core.cuh"],
    "llama_decoder_layer": ["decoder.cu", "decoder_epi.cuh", "attention.cu", "tp.cu",
                            "gemm_core.cuh", "gemm_launch.cuh"],
    "rms_norm_linear": ["fused_ops.cu", "decoder.cu", "gemm_core.cuh"],
    "fused_add_rms_norm": ["fused_ops.cu"],
    "rope_embedding": ["fused_ops.cu"],
    "swiglu": ["fused_ops.cu", "decoder_epi.cuh", "gemm_core.cuh"],
    "scaled_dot_product": ["fused_ops.cu", "attention.cu"],
    "llama_attention": ["fused_ops.cu", "attention.cu", "gemm.cu"],
    "mha_attention": ["fused_ops.cu", "attention.cu", "gemm.cu"],
    "transformer_block": ["fused_ops.cu", "attention.cu", "gemm.cu", "gemm_epi.cuh"],
}
# registry entries whose buffers take another path of the same mb_run kernel
# (the fp32 entries of the reference: conv2d_f32, llama_decoder_layer_f32)
DTYPE_SOURCES = {"f32": {"conv2d": ["f32_paths.cu", "gemm.cu", "gemm_core.cuh"],
                         "llama_decoder_layer": ["f32_paths.cu", "gemm.cu", "gemm_core.cuh"]}}
# files every kernel depends on
SHARED_SOURCES = ["common.cuh", "abi.cu", "registry.cu", "kernels.h"]


def _registry() -> dict:
    from metalbench_b200 import harness
    return harness.registry_all()


def _kernels(reg: dict) -> list[tuple[str, str]]:
    return [(v["set"], n) for s in SETS for n, v in sorted(reg.items()) if v["set"] == s]


def _session(path: Path | None = None) -> dict:
    p = path or REPO / "session.json"
    return json.loads(p.read_text()) if p.exists() else {}


def _chips(session: dict) -> list[str]:
    return APPLE_CHIPS + sorted(c for c in session if c not in APPLE_CHIPS)


def render_best_times(out: Path | None = None, session: Path | None = None) -> Path:
    reg, s = _registry(), _session(session)
    chips = _chips(s)

    def entry(chip: str, name: str) -> dict:
        return s.get(chip, {}).get(name) or {}

    def num(v) -> bool:
        return isinstance(v, (int, float)) and not isinstance(v, bool)

    # "<best ms> (<speedup>×)" per chip, the cell format best_times.md readers
    # parse; an entry without a positive speedup has no comparable time
    def cell(chip: str, name: str) -> str:
        e = entry(chip, name)
        t, x = e.get("best_time_ms"), e.get("speedup_vs_mlx")
        return f"{t:.3f} ({x:.2f}×)" if num(t) and num(x) and x > 0 else "—"

    def sol(chip: str, name: str) -> str:
        v = entry(chip, name).get("roofline_sol")
        return f"{v * 100:.0f} %" if num(v) else "—"

    extra = [c for c in chips if c not in APPLE_CHIPS]
    head = ["kernel", "set"] + [c.replace("apple-", "").upper() for c in chips] + \
           [f"{c.upper()} SoL" for c in extra]
    lines = [
        "# MetalBench Best Times",
        "",
        "Best kernel time in ms (speedup vs MLX) per chip; SoL = fraction of the chip's",
        "roofline. `—` = not benchmarked on that chip.",
        "Generated from `session.json` by `python -m metalbench_b200.leaderboard`. Do not hand-edit.",
        "",
        "| " + " | ".join(head) + " |",
        "|" + "---|" * len(head),
    ]
    kernels = _kernels(reg)
    for setname, name in kernels:
        cells = [cell(c, name) for c in chips] + [sol(c, name) for c in extra]
        lines.append(f"| `{name}` | {setname} | " + " | ".join(cells) + " |")
    covered = ", ".join(f"{c} ({len(s.get(c, {}))})" for c in chips if s.get(c))
    lines += ["", f"_{len(kernels)} kernels total. Chips covered: {covered or 'none'}._"]
    out = out or REPO / "best_times.md"
    out.write_text("\n".join(lines) + "\n")
    return out


def sources_for(kernel: str) -> list[str]:
    return [f"{CSRC}/{f}" for f in KERNEL_SOURCES.get(kernel, [])]


def render_link_md(out: Path | None = None, session: Path | None = None) -> Path:
    reg, s = _registry(), _session(session)
    kernels = _kernels(reg)
    chips = _chips(s)
    lines = [
        "# LINK.md",
        "",
        f"Per-chip kernel source links — {len(kernels)} kernels × {len(chips)} chips.",
        "Chips without benchmark data show kernels as plain text (no link). The Apple",
        "chips' Metal sources live in the reference repository; b200 links point at the",
        "CUDA files of libmb200 that implement each registry entry.",
        "",
        "Generated from `session.json` and the registry by `python -m metalbench_b200.leaderboard`.",
        "Do not hand-edit.",
        "",
    ]
    for chip in chips:
        has_data = bool(s.get(chip))
        lines.append(f"## {chip}" + ("" if has_data else " _(no data)_"))
        lines.append("")
        for _, name in kernels:
            srcs = sources_for(reg[name]["kernel"]) if has_data and chip not in APPLE_CHIPS else []
            if srcs:
                lines.append(f"- [{name}]({srcs[0]})" +
                             "".join(f" · [{Path(p).name}]({p})" for p in srcs[1:]))
            else:
                lines.append(f"- `{name}`")
        lines.append("")
    out = out or REPO / "LINK.md"
    out.write_text("\n".join(lines))
    return out


def kernels_for(paths: list[str]) -> list[str]:
    """Registry names whose implementation a change to `paths` touches (the
    kernel discovery of the reference's certify, for CUDA sources and hooks)."""
    reg = _registry()
    names = set()
    for p in paths:
        fname = Path(p).name
        if p.startswith("mlx/kernels/") and fname.endswith(".py") and fname != "registry.py":
            stem = fname[:-3]
            names.update(n for n, v in reg.items() if v.get("hook", n) == stem)
        elif p.startswith(CSRC + "/"):
            if fname in SHARED_SOURCES:
                names.update(reg)
            for n, v in reg.items():
                dt = (v.get("input_dtypes") or ["f32"])[0]
                srcs = DTYPE_SOURCES.get(dt, {}).get(v["kernel"]) or KERNEL_SOURCES.get(v["kernel"], [])
                if fname in srcs:
                    names.add(n)
    return sorted(names)


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    what = argv[0] if argv else "all"
    if what == "kernels-for":
        print("\n".join(kernels_for(argv[1:])))
        return 0
    if what in ("all", "best-times"):
        print(f"[leaderboard] wrote {render_best_times().relative_to(REPO)}", file=sys.stderr)
    if what in ("all", "link-md"):
        print(f"[leaderboard] wrote {render_link_md().relative_to(REPO)}", file=sys.stderr)
    if what not in ("all", "best-times", "link-md"):
        print(__doc__, file=sys.stderr)
        return 64
    return 0


if __name__ == "__main__":
    sys.exit(main())
