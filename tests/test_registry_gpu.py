"""Accuracy sweep over every registry entry, the shape of the reference's
tests/metalbench/test_bench_accuracy_all.py:16-54 (which runs
`./bench k --no-save -- --iters 5 --warmup 2` per kernel and requires
`correctness : ✓` and max_err <= 0.05): harness.evaluate on the B200, the
kernel against the reference hook on the same seeded inputs, the >= 99 %
gate, and max_err <= max(0.05, 1e-4 * max|reference|) for the fp32 entries
(bf16 entries carry the bf16 rounding of outputs up to ~|8|, so their bound
is the gate)."""
import pytest

from metalbench_b200 import harness as Hm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(Hm.registry_all()))
def test_registry_entry_is_correct(name):
    r = Hm.evaluate(name, warmup=2, iters=5, ref_warmup=0, ref_iters=1)
    print(name, [(o["frac_within_tol"], o["max_err"], o["atol_needed"], o["err_std"])
                 for o in r["outputs"]])
    assert r["correct"], (name, r["outputs"])
    if Hm.registry_all()[name]["output_dtype"] == "f32":
        # the reference suite's max_err <= 0.05, scaled for outputs in the
        # thousands (llama_decoder_layer_f32 with N(0,1) weights: rms ~1400,
        # where the fp32 reference itself is 0.1-0.4 off the float64 result)
        bound = max(0.05, 1e-4 * r["ref_abs_max"])
        assert max(o["max_err"] for o in r["outputs"]) <= bound, (name, r["outputs"], bound)
