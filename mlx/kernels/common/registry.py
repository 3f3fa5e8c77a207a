"""Common-set registry entries served by the B200 backend.

Keys kept from the reference registry (mlx/kernels/common/registry.py:44-61,
129, 165-179, 469-477): metal_function (the reference kernel symbol),
input_bindings, input_shapes, output_shape, rtol, atol, scalars (binding, dtype,
value), flops, bytes. B200 keys:
  kernel        libmb200 mb_run name
  input_dtypes  "f32" | "bf16" per input (bf16 travels as raw uint16)
  input_init    (distribution, scale) per input: "normal" N(0, scale^2) or
                "uniform" U[-scale, scale)
  output_dtype  dtype of the output buffer
  seed          generator seed
  model_kwargs  constructor arguments of the hook's Model
  config        extra mb_run keys (flat JSON)
  roof          "tensor_bf16" | "tensor_tf32x3" | "hbm" | "ridge" (roofline class)
  ref_warmup / ref_iters  default timing of the CPU reference leg
"""
N_SQ = 2048
REGISTRY = {}

REGISTRY["sqr_mm"] = dict(
    kernel="sqr_mm", metal_function="sqr_matmul_f32",
    input_bindings=(0, 1), input_shapes=[(N_SQ, N_SQ), (N_SQ, N_SQ)],
    input_dtypes=["f32", "f32"], input_init=[("normal", 1.0), ("normal", 1.0)],
    output_shape=(N_SQ, N_SQ), output_dtype="f32",
    scalars=[dict(binding=3, dtype="u32", value=N_SQ), dict(binding=4, dtype="u32", value=N_SQ),
             dict(binding=5, dtype="u32", value=N_SQ)],
    rtol=1e-4, atol=1e-3, seed=0,
    flops=2 * N_SQ ** 3, bytes=3 * N_SQ * N_SQ * 4,
    roof="tensor_tf32x3", ref_warmup=2, ref_iters=10)

REGISTRY["transpose_2d"] = dict(
    kernel="transpose_2d", metal_function="transpose_2d_f32",
    input_bindings=(0,), input_shapes=[(8192, 8192)], input_dtypes=["f32"],
    input_init=[("uniform", 1.0)], output_shape=(8192, 8192), output_dtype="f32",
    scalars=[dict(binding=2, dtype="u32", value=8192), dict(binding=3, dtype="u32", value=8192)],
    rtol=0, atol=0, seed=1, flops=0, bytes=2 * 8192 * 8192 * 4,
    roof="hbm", ref_warmup=2, ref_iters=10)

REGISTRY["transpose_batched_bf16"] = dict(
    kernel="transpose_batched", metal_function="transpose_2d_f32",
    input_bindings=(0,), input_shapes=[(64, 1024, 1024)], input_dtypes=["bf16"],
    input_init=[("uniform", 1.0)], output_shape=(64, 1024, 1024), output_dtype="bf16",
    scalars=[dict(binding=2, dtype="u32", value=64), dict(binding=3, dtype="u32", value=1024),
             dict(binding=4, dtype="u32", value=1024)],
    rtol=0, atol=0, seed=1, flops=0, bytes=2 * 64 * 1024 * 1024 * 2,
    hook="transpose_2d", roof="hbm", ref_warmup=2, ref_iters=10)

_CONV = (32, 56, 56, 64, 64, 3)  # N, H, W, Cin, Cout, K
REGISTRY["conv2d"] = dict(
    kernel="conv2d", metal_function="conv2d_f32",
    input_bindings=(0, 1),
    input_shapes=[(32, 56, 56, 64), (64, 3, 3, 64)], input_dtypes=["bf16", "bf16"],
    input_init=[("normal", 1.0), ("normal", (2.0 / (9 * 64)) ** 0.5)],
    output_shape=(32, 56, 56, 64), output_dtype="bf16",
    scalars=[dict(binding=b, dtype="u32", value=v) for b, v in
             zip(range(3, 11), (32, 56, 56, 64, 64, 3, 3, 1))],
    config={"padding": 1}, model_kwargs=dict(in_channels=64, out_channels=64, kernel_size=3,
                                             stride=1, padding=1),
    rtol=2e-2, atol=2e-2, seed=2,
    flops=2 * 32 * 56 * 56 * 64 * 64 * 9, bytes=2 * (32 * 56 * 56 * 64 * 2 + 64 * 9 * 64),
    roof="ridge", ref_warmup=1, ref_iters=3)

# The reference's own conv2d entry (common/registry.py:469-477), served
# unchanged next to the BASELINE one: fp32, x (8,64,64,64) * w (128,3,3,64),
# pad 0, N(0,1) inputs (mlx_helpers.py:236-251), rtol = atol = 1e-3.
REGISTRY["conv2d_f32"] = dict(
    kernel="conv2d", metal_function="conv2d_f32", hook="conv2d",
    input_bindings=(0, 1), input_shapes=[(8, 64, 64, 64), (128, 3, 3, 64)],
    input_dtypes=["f32", "f32"], input_init=[("normal", 1.0), ("normal", 1.0)],
    output_shape=(8, 62, 62, 128), output_dtype="f32",
    scalars=[dict(binding=b, dtype="u32", value=v) for b, v in
             zip(range(3, 11), (8, 64, 64, 64, 128, 3, 3, 1))],
    model_kwargs=dict(in_channels=64, out_channels=128, kernel_size=3, stride=1),
    rtol=1e-3, atol=1e-3, seed=0,
    flops=8 * 128 * 62 * 62 * 64 * 9 * 2, bytes=4 * (8 * 64 * 64 * 64 + 128 * 3 * 3 * 64 + 8 * 128 * 62 * 62),
    roof="tensor_tf32x3", ref_warmup=1, ref_iters=3)

REGISTRY["gemm_bf16"] = dict(
    kernel="gemm_bf16", metal_function="rect_matmul_f32",
    input_bindings=(0, 1), input_shapes=[(4096, 4096), (4096, 4096)],
    input_dtypes=["bf16", "bf16"], input_init=[("normal", 1.0), ("normal", 1.0)],
    output_shape=(4096, 4096), output_dtype="bf16",
    scalars=[dict(binding=3, dtype="u32", value=4096), dict(binding=4, dtype="u32", value=4096),
             dict(binding=5, dtype="u32", value=4096)],
    config={"b_layout": 1}, hook="sqr_mm",
    rtol=2e-2, atol=2.0, seed=4, flops=2 * 4096 ** 3, bytes=3 * 4096 * 4096 * 2,
    roof="tensor_bf16", ref_warmup=1, ref_iters=3)

REGISTRY["rect_mm"] = dict(
    kernel="sqr_mm", metal_function="rect_matmul_f32",
    input_bindings=(0, 1), input_shapes=[(1024, 4096), (4096, 2048)],
    input_dtypes=["f32", "f32"], input_init=[("normal", 1.0), ("normal", 1.0)],
    output_shape=(1024, 2048), output_dtype="f32",
    scalars=[dict(binding=3, dtype="u32", value=1024), dict(binding=4, dtype="u32", value=2048),
             dict(binding=5, dtype="u32", value=4096)],
    rtol=1e-4, atol=1e-3, seed=0, flops=2 * 1024 * 2048 * 4096,
    bytes=4 * (1024 * 4096 + 4096 * 2048 + 1024 * 2048),
    roof="tensor_tf32x3", ref_warmup=1, ref_iters=5)

# batched_matmul helper semantics (common/registry.py:61-77): A [B,M,K], B [B,K,N];
# the reference's own shape (131): 128 x (128x256 @ 256x512)
REGISTRY["batch_mm"] = dict(
    kernel="batch_mm", metal_function="batch_matmul_f32",
    input_bindings=(0, 1), input_shapes=[(128, 128, 256), (128, 256, 512)],
    input_dtypes=["f32", "f32"], input_init=[("normal", 1.0), ("normal", 1.0)],
    output_shape=(128, 128, 512), output_dtype="f32",
    scalars=[dict(binding=3, dtype="u32", value=128), dict(binding=4, dtype="u32", value=512),
             dict(binding=5, dtype="u32", value=256)],
    rtol=1e-4, atol=1e-3, seed=0, flops=128 * 2 * 128 * 512 * 256,
    bytes=128 * 4 * (128 * 256 + 256 * 512 + 128 * 512),
    roof="tensor_tf32x3", ref_warmup=1, ref_iters=5)
