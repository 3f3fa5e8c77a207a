"""The CPU oracle against the golden fixtures made by executing the reference's
own hook files (tests/golden/gen_golden.py), plus known-answer checks."""
from pathlib import Path

import numpy as np
import pytest

import oracle.ops as O

GOLD = Path(__file__).resolve().parent / "golden"


def _load(name):
    return np.load(GOLD / f"{name}.npz")


def test_sqr_mm_matches_reference_hook():
    d = _load("sqr_mm")
    got = O.sqr_mm(d["in0"], d["in1"])
    np.testing.assert_allclose(got, d["out"], rtol=1e-5, atol=1e-4)


def test_transpose_matches_reference_hook_bit_exact():
    d = _load("transpose_2d")
    got = O.transpose_2d(d["in0"])
    assert got.tobytes() == d["out"].tobytes()


def test_conv2d_matches_reference_hook():
    d = _load("conv2d")
    got = O.conv2d_nhwc(d["in0"], d["in1"], stride=1, padding=0, acc=np.float64)
    np.testing.assert_allclose(got, d["out"], rtol=1e-5, atol=1e-3)


def test_decoder_layer_matches_reference_hook():
    d = _load("llama_decoder_layer")
    got = O.decoder_layer(d["in0"], d["in1"], d["in2"], d["in3"], d["in4"], H=4, H_kv=2,
                          base=10000.0, eps=1e-5, acc=np.float64)
    rel = np.abs(got - d["out"]).max() / np.abs(d["out"]).max()
    assert rel < 2e-4  # golden is the hook run in fp32; ours in fp64


def test_bf16_round_trip_and_rounding():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38, 0.0], dtype=np.float32)
    b = O.f32_to_bf16(x)
    back = O.bf16_to_f32(b)
    assert back[0] == 1.0 and back[3] == -2.5 and back[5] == 0.0
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: round to even -> 1.0
    assert back[1] == 1.0
    # 1 + 1.5*2^-8 rounds up to 1 + 2^-7
    assert back[2] == np.float32(1.0078125)
    assert np.all(O.bf16_to_f32(O.f32_to_bf16(back)) == back)


def test_conv2d_padding_known_answer():
    # 1x3x3x1 ones, 3x3 ones kernel, pad 1: counts of in-bounds neighbours.
    x = np.ones((1, 3, 3, 1), np.float32)
    w = np.ones((1, 3, 3, 1), np.float32)
    y = O.conv2d_nhwc(x, w, padding=1)[0, :, :, 0]
    np.testing.assert_array_equal(y, [[4, 6, 4], [6, 9, 6], [4, 6, 4]])


def test_rope_pairs_and_positions():
    # Position 0 is the identity; pair (0,1) with omega_0 = 1 rotates by pos.
    t = np.zeros((1, 2, 4), np.float64)
    t[0, :, 0] = 1.0
    out = O.rope(t, np.array([0, 1]), base=10000.0)
    np.testing.assert_allclose(out[0, 0], [1, 0, 0, 0])
    np.testing.assert_allclose(out[0, 1, :2], [np.cos(1.0), np.sin(1.0)], atol=1e-12)


def test_gqa_head_mapping():
    # With G=2, query heads 0,1 read kv head 0; 2,3 read kv head 1 (mx.repeat).
    k = np.arange(2)[None, :, None, None] * np.ones((1, 2, 3, 4))
    r = np.repeat(k, 2, axis=1)
    assert [r[0, h, 0, 0] for h in range(4)] == [0, 0, 1, 1]


@pytest.mark.parametrize("S,L", [(1, 5), (3, 4)])
def test_decode_with_cache_equals_full_causal(S, L):
    """Prefill L tokens, then run S new tokens against the cache: equal to a
    causal forward over all L+S tokens (size-independent property)."""
    rng = np.random.default_rng(7)
    D, H, Hkv, FF = 32, 4, 2, 48
    x = rng.standard_normal((2, L + S, D))
    Wqkv = rng.standard_normal((D, D + 2 * Hkv * (D // H))) * 0.2
    Wo = rng.standard_normal((D, D)) * 0.2
    Wgu = rng.standard_normal((D, 2 * FF)) * 0.2
    Wd = rng.standard_normal((FF, D)) * 0.2
    kw = dict(H=H, H_kv=Hkv, base=500000.0, causal=True, acc=np.float64)
    full = O.decoder_layer(x, Wqkv, Wo, Wgu, Wd, **kw)
    y0, k0, v0 = O.decoder_layer(x[:, :L], Wqkv, Wo, Wgu, Wd, return_kv=True, **kw)
    y1 = O.decoder_layer(x[:, L:], Wqkv, Wo, Wgu, Wd, k_past=k0, v_past=v0, **kw)
    np.testing.assert_allclose(y0, full[:, :L], rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(y1, full[:, L:], rtol=1e-9, atol=1e-9)


def test_allclose_report_fraction():
    a = np.array([1.0, 2.0, 3.0, 4.0])
    b = np.array([1.0, 2.0, 3.5, 4.0])
    r = O.allclose_report(a, b, rtol=0.0, atol=0.1)
    assert not r["all"] and r["frac_within_tol"] == 0.75 and r["max_err"] == 0.5


@pytest.mark.parametrize("name,fn", [
    ("rms_norm_linear", lambda d: O.rms_norm_linear(d["in0"], d["in1"])),
    ("fused_add_rms_norm", lambda d: O.fused_add_rms_norm(d["in0"], d["in1"])),
    ("rope_embedding", lambda d: O.rope_full(d["in0"])),
    ("swiglu", lambda d: O.swiglu(d["in0"], d["in1"], d["in2"])),
    ("scaled_dot_product", lambda d: O.sdpa(d["in0"], d["in1"], d["in2"])),
    ("fused_qkv_projection", lambda d: O.sqr_mm(d["in0"], d["in1"])),
    ("rect_mm", lambda d: O.sqr_mm(d["in0"], d["in1"])),
    ("batch_mm", lambda d: O.sqr_mm(d["in0"], d["in1"])),
    ("llama_attention", lambda d: O.llama_attention(d["in0"], d["in1"], d["in2"], H=4, H_kv=2)),
    ("transformer_block", lambda d: O.transformer_block(*[d[f"in{i}"] for i in range(5)], H=4)),
    ("mha_attention", lambda d: O.mha_attention(*[d[f"in{i}"] for i in range(5)], H=4)),
])
def test_standard_set_oracle_matches_reference_hooks(name, fn):
    d = _load(name)
    got = fn(d)
    scale = max(1.0, float(np.abs(d["out"]).max()))
    assert np.abs(got - d["out"]).max() <= 1e-4 * scale, name
