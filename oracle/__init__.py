"""CPU oracle for the nnunet-mlx inference hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch-CPU float32 (and NumPy), what the
reference (MedMLX/nnunet-mlx v0.9.0) computes on its inference path:

* ``oracle.network``        -- PlainConvUNet / ResidualEncoderUNet forward over the
                               converted (MLX channels-last) weight layout;
* ``oracle.sliding_window`` -- tile offsets, Gaussian importance map, minimum
                               padding, mirrored prediction, Gaussian-weighted
                               accumulation, fold averaging and label reduction.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and only as the checker or as the timed CPU
baseline.  The product path (``nnunet_mlx_b200``) never imports it and fails
loudly when its CUDA extension is missing.

Pinning: the geometry helpers are checked against golden vectors produced by
importing the reference's own host code (``tests/golden/make_golden.py``).
The network restatement cannot be pinned against the reference's outputs
because the reference network only runs on MLX/Metal (Apple silicon); it is
built from the same torch primitives (``conv3d``, ``instance_norm``,
``leaky_relu``, ``conv_transpose3d``) as the reference's own test oracle
(reference ``tests/nnunet_reference/oracle/network.py:62-88``), so its network
parity is "partial": pinned by construction and by the published tolerance,
not by recorded reference logits.
"""
