"""CPU oracle for the MetalBench-B200 hot path.

TEST INFRASTRUCTURE ONLY. This package is the checker: the parity tests, the
smoke check and the CPU-baseline leg of ``bench.py`` call it. The product path
(``metalbench_b200`` and ``libmb200.so``) never imports it.

``oracle.ops`` restates, in numpy, the ``Model.forward`` of the four reference
hooks on the hot path:

* ``mlx/kernels/common/sqr_mm.py:10-11``        C = A @ B
* ``mlx/kernels/common/transpose_2d.py:10-11``  B = A^T
* ``mlx/kernels/common/conv2d.py:7-12``         NHWC x OHWI cross-correlation
* ``mlx/kernels/full/llama_decoder_layer.py:24-64`` the LLaMA decoder layer

``tests/golden/gen_golden.py`` executes the reference's own hook files (not
this restatement) through ``metalbench_b200/mlx_compat`` (a numpy stand-in for
the MLX ops they use) and commits their outputs as fixtures; the restatement
is pinned against those fixtures (tests/test_oracle.py).

Parity status: pinned against the reference hook code executed through the
numpy MLX stand-in. MLX itself (a third-party dependency, ``mlx>=0.18.0`` in the
reference's requirements.txt:1) is absent here, so the shim's op semantics are
restated from MLX's published API, not run.
"""
