"""CPU oracle for the quantized DiT-block hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the ``ltxq`` package
and its CUDA library) imports, links or executes anything under ``oracle/``.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use it, and only as the checker / the timed CPU baseline.

The oracle is a numpy restatement of the reference's MLX op composition for
the path (LTX_2_MLX/kernels/fused_ops.py, model/transformer/transformer.py,
model/transformer/feed_forward.py, model/transformer/attention.py,
loader/transformer_cache.py) and for its callers: the model's preprocess and
output heads, RoPE tables and latent positions, the denoise step and loops,
schedules, guiders, steppers, latent layouts and the noiser (``denoise``,
``rope``, ``latents``; model/transformer/model.py, rope.py,
timestep_embedding.py, components/, pipelines/av_pipeline.py).  MLX itself (the third-party dependency that
holds ``mx.quantize`` / ``mx.quantized_matmul`` / ``mx.fast.rms_norm``,
``mlx>=0.31.2`` per the reference's pyproject.toml:35) is not installable
here, so:

* pinned: the FP8 E4M3 known-answer vector of the reference's own test
  (tests/test_transformer_cache.py:64-95: byte 0x38 -> 1.0, x2.0 -> 2.0) and
  the structure/thresholds of tests/test_fused_ops.py;
* parity unpinned: the exact numerics of MLX's affine quantize, its
  quantized_matmul rounding and nn.gelu_approx.  The oracle restates MLX's
  published algorithms (documented per function) and the GPU path is held
  bit-exact / within tolerance against this restatement.
"""
