"""CPU oracle for the DiffusorRT denoising-decode hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy, the reference algorithms the B200 path must reproduce:

* ``oracle.selector`` — the unmask scoring and choice functions of
  ``python/src/edllm/backends/diffusion_runtime.py`` (raw max-prob, negative entropy with
  temperature / top-p, top-k and threshold choices, MASK exclusion);
* ``oracle.policy`` — the plan/select rules of the BD3 fixed-quota, block-threshold and
  entropy-count commit policies and the generic decode loop (same file);
* ``oracle.forward`` — the transformer forward under the reference's MLX precision contract
  (``python/src/edllm/backends/mlx_ops.py`` / ``mlx_forward.py``) and the float64 executable
  spec (``python/src/edllm/graph/numpyref.py``);
* ``oracle.synth`` — the seeded synthetic weight generator the native library uses, so the
  oracle sees bit-identical weights.

Parity is pinned against golden vectors produced by the reference itself (``tests/golden``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm may import
this package, and only as the checker or the timed CPU baseline. The product package
``diffusorrt_b200`` never imports it and has no CPU fallback.
"""
