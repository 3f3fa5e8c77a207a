"""Generate golden fixtures by executing the REFERENCE's own hook files.

Run in the build container (where the read-only reference checkout exists):

    python tests/golden/gen_golden.py [--reference PATH]

MLX is not installed here, so ``metalbench_b200/mlx_compat`` (a numpy
implementation of the MLX ops the hooks use) is put on ``sys.path`` as ``mlx``. The script then
loads each hook (``mlx/kernels/<set>/<name>.py``) from the reference checkout,
builds its ``Model`` exactly as the reference harness does
(mlx/scripts/mlx_helpers.py:219-257: ``Model()`` with default arguments and one
N(0,1) float32 input per registry input shape) and stores inputs and outputs
in ``tests/golden/<name>.npz``. The fixtures are what pins ``oracle.ops``;
nothing at test time reads the reference checkout.
"""
from __future__ import annotations

import argparse
import os
import hashlib
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

# (name, set, registry input shapes, seed). Shapes are the reference registry
# shapes (common/registry.py:129,165-179,469-477; full/registry.py:87-104),
# shrunk where the reference shape would make the fixture large.
CASES = [
    ("sqr_mm", "common", [(64, 64), (64, 64)], 0),
    ("transpose_2d", "common", [(48, 80)], 1),
    ("conv2d", "common", [(2, 10, 12, 64), (128, 3, 3, 64)], 2),
    ("llama_decoder_layer", "full",
     [(64, 128), (128, 128 + 2 * 2 * 32), (128, 128), (128, 2 * 256), (256, 128)], 3),
    # standard set at the reference registry shapes (shrunk where large)
    # (mlx/kernels/standard/registry.py:26-42, 103-132, 280-292, 324-337, 382-396)
    ("rms_norm_linear", "standard", [(32, 1024), (48, 1024)], 5),
    ("fused_add_rms_norm", "standard", [(16, 1024), (16, 1024)], 5),
    ("rope_embedding", "standard", [(128, 64)], 5),
    ("swiglu", "standard", [(32, 64), (64, 96), (64, 96)], 5),
    ("scaled_dot_product", "standard", [(40, 128), (40, 128), (40, 128)], 5),
    ("fused_qkv_projection", "standard", [(16, 64), (64, 48)], 5),
    ("rect_mm", "common", [(32, 96), (96, 40)], 5),
    ("batch_mm", "common", [(3, 16, 24), (3, 24, 20)], 5),
    ("llama_attention", "standard", [(64, 128), (128, 256), (128, 128)], 5),
    ("transformer_block", "full", [(64, 128), (128, 384), (128, 128), (128, 256), (256, 128)], 5),
    ("mha_attention", "full", [(32, 128)] + [(128, 128)] * 4, 5),
]


def _load_hook(ref: Path, kset: str, name: str):
    path = ref / "mlx" / "kernels" / kset / f"{name}.py"
    spec = importlib.util.spec_from_file_location(f"_ref_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, hashlib.sha256(path.read_bytes()).hexdigest()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MB_REFERENCE_TREE"),
                    help="checkout of the reference repository (or set MB_REFERENCE_TREE)")
    args = ap.parse_args(argv)
    if not args.reference:
        ap.error("--reference (or MB_REFERENCE_TREE) is required")
    ref = Path(args.reference)
    try:
        import mlx.core  # noqa: F401
        print("[golden] using real mlx", file=sys.stderr)
    except ImportError:
        sys.path.insert(0, str(REPO / "metalbench_b200" / "mlx_compat"))
        print("[golden] mlx absent: using metalbench_b200/mlx_compat", file=sys.stderr)
    import mlx.core as mx

    for name, kset, shapes, seed in CASES:
        mod, digest = _load_hook(ref, kset, name)
        rng = np.random.default_rng(seed)
        inputs = [rng.standard_normal(s).astype(np.float32) for s in shapes]
        model = mod.Model()
        out = np.asarray(model.forward(*[mx.array(x) for x in inputs]), dtype=np.float32)
        blob = {f"in{i}": x for i, x in enumerate(inputs)}
        blob["out"] = out
        blob["hook_sha256"] = np.array(digest)
        blob["seed"] = np.array(seed)
        np.savez_compressed(HERE / f"{name}.npz", **blob)
        print(f"[golden] {name}: inputs {shapes} -> out {out.shape}", file=sys.stderr)


if __name__ == "__main__":
    main()
