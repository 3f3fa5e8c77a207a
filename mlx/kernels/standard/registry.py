"""Standard-set registry entries served by the B200 backend (format: see
mlx/kernels/common/registry.py). The reference's entries
(mlx/kernels/standard/registry.py:26-42, 103-132, 280-292, 324-337, 382-396)
are fp32 at toy sizes; here they are the bf16 sub-steps of the decoder at the
BASELINE decoder's sizes (d_model 4096, FFN 14336, head_dim 128).
"""
M, D, FF, NQKV, S_ATT = 8192, 4096, 14336, 6144, 4096
REGISTRY = {}


def _u32(binding, value):
    return dict(binding=binding, dtype="u32", value=value)


REGISTRY["rms_norm_linear"] = dict(
    kernel="rms_norm_linear", metal_function="rms_norm_linear_f32",
    input_bindings=(0, 1), input_shapes=[(M, D), (D, D)], input_dtypes=["bf16", "bf16"],
    input_init=[("normal", 1.0), ("normal", 0.02)], output_shape=(M, D), output_dtype="bf16",
    scalars=[_u32(3, M), _u32(4, D), _u32(5, D), dict(binding=6, dtype="f32", value=1e-5)],
    model_kwargs=dict(dim=D, out_dim=D, eps=1e-5),
    rtol=2e-2, atol=2e-2, seed=3, flops=2 * M * D * D + 3 * M * D,
    bytes=2 * (2 * M * D + D * D), roof="tensor_bf16", ref_warmup=0, ref_iters=2)

REGISTRY["fused_add_rms_norm"] = dict(
    kernel="fused_add_rms_norm", metal_function="fused_add_rms_norm_f32",
    input_bindings=(0, 1), input_shapes=[(M, D), (M, D)], input_dtypes=["bf16", "bf16"],
    input_init=[("normal", 1.0), ("normal", 1.0)], output_shape=(M, D), output_dtype="bf16",
    scalars=[_u32(3, D), dict(binding=4, dtype="f32", value=1e-5)],
    model_kwargs=dict(dim=D, eps=1e-5),
    rtol=2e-2, atol=2e-2, seed=3, flops=6 * M * D, bytes=3 * M * D * 2,
    roof="hbm", ref_warmup=1, ref_iters=3)

REGISTRY["rope_embedding"] = dict(
    kernel="rope_embedding", metal_function="rope_embedding_f32",
    input_bindings=(0,), input_shapes=[(M, D)], input_dtypes=["bf16"],
    input_init=[("normal", 1.0)], output_shape=(M, D), output_dtype="bf16",
    scalars=[_u32(2, M), _u32(3, D), dict(binding=4, dtype="f32", value=10000.0)],
    model_kwargs=dict(base=10000.0),
    rtol=2e-2, atol=2e-2, seed=3, flops=6 * M * D // 2, bytes=2 * M * D * 2,
    roof="hbm", ref_warmup=1, ref_iters=3)

REGISTRY["swiglu"] = dict(
    kernel="swiglu", metal_function="swiglu_f32",
    input_bindings=(0, 1, 2), input_shapes=[(M, D), (D, FF), (D, FF)],
    input_dtypes=["bf16"] * 3, input_init=[("normal", 1.0), ("normal", 0.02), ("normal", 0.02)],
    output_shape=(M, FF), output_dtype="bf16",
    scalars=[_u32(4, M), _u32(5, D), _u32(6, FF)],
    rtol=2e-2, atol=2e-2, seed=3, flops=4 * M * D * FF + 5 * M * FF,
    bytes=2 * (M * D + 2 * D * FF + M * FF), roof="tensor_bf16", ref_warmup=0, ref_iters=1)

REGISTRY["fused_qkv_projection"] = dict(
    kernel="gemm_bf16", metal_function="fused_qkv_projection_f32",
    input_bindings=(0, 1), input_shapes=[(M, D), (D, NQKV)], input_dtypes=["bf16", "bf16"],
    input_init=[("normal", 1.0), ("normal", 0.02)], output_shape=(M, NQKV), output_dtype="bf16",
    scalars=[_u32(3, M), _u32(4, NQKV), _u32(5, D)], config={"b_layout": 1},
    rtol=2e-2, atol=2e-2, seed=3, flops=2 * M * D * NQKV, bytes=2 * (M * D + D * NQKV + M * NQKV),
    roof="tensor_bf16", ref_warmup=0, ref_iters=2)

REGISTRY["scaled_dot_product"] = dict(
    kernel="scaled_dot_product", metal_function="scaled_dot_product_f32",
    input_bindings=(0, 1, 2), input_shapes=[(S_ATT, 128)] * 3, input_dtypes=["bf16"] * 3,
    input_init=[("normal", 1.0)] * 3, output_shape=(S_ATT, 128), output_dtype="bf16",
    scalars=[_u32(4, S_ATT), _u32(5, 128)], model_kwargs=dict(d_head=128),
    rtol=2e-2, atol=2e-2, seed=3, flops=4 * S_ATT * S_ATT * 128,
    bytes=4 * S_ATT * 128 * 2, roof="tensor_bf16", ref_warmup=1, ref_iters=3)

# llama_attention (reference standard/registry.py:398-413: S 64, D 128, 4/2
# heads of 32, fp32) at the BASELINE decoder's attention shape: S 4096,
# d_model 4096, 32 query / 8 kv heads of 128, bf16.
LA_S, LA_D, LA_H, LA_HKV = 4096, 4096, 32, 8
LA_N = LA_D + 2 * LA_HKV * 128
REGISTRY["llama_attention"] = dict(
    kernel="llama_attention", metal_function="llama_attention_f32",
    input_bindings=(0, 1, 2), input_shapes=[(LA_S, LA_D), (LA_D, LA_N), (LA_D, LA_D)],
    input_dtypes=["bf16"] * 3, input_init=[("normal", 1.0), ("normal", 0.02), ("normal", 0.02)],
    output_shape=(LA_S, LA_D), output_dtype="bf16",
    scalars=[_u32(4, LA_S), _u32(5, LA_D), _u32(6, LA_H), _u32(7, LA_HKV),
             dict(binding=8, dtype="f32", value=10000.0)],
    model_kwargs=dict(S=LA_S, D=LA_D, H=LA_H, H_kv=LA_HKV, base=10000.0),
    rtol=2e-2, atol=2e-2, seed=3,
    flops=2 * LA_S * LA_D * LA_N + 4 * LA_H * LA_S * LA_S * 128 + 2 * LA_S * LA_D * LA_D,
    bytes=2 * (2 * LA_S * LA_D + LA_D * LA_N + LA_D * LA_D), roof="tensor_bf16",
    ref_warmup=0, ref_iters=1)
