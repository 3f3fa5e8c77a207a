"""Accuracy sweep over every registry entry, the shape of the reference's
tests/metalbench/test_bench_accuracy_all.py:16-54 (which runs
`./bench k --no-save -- --iters 5 --warmup 2` per kernel and requires
`correctness : ✓` and max_err <= 0.05): harness.evaluate on the B200, the
kernel against the reference hook on the same seeded inputs, the >= 99 %
gate, and max_err <= 0.05 for the fp32 entries (bf16 entries carry the
bf16 rounding of outputs up to ~|8|, so their bound is the gate)."""
import pytest

from metalbench_b200 import harness as Hm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(Hm.registry_all()))
def test_registry_entry_is_correct(name):
    r = Hm.evaluate(name, warmup=2, iters=5, ref_warmup=0, ref_iters=1)
    assert r["correct"], (name, r["outputs"])
    if Hm.registry_all()[name]["output_dtype"] == "f32":
        assert max(o["max_err"] for o in r["outputs"]) <= 0.05, (name, r["outputs"])
