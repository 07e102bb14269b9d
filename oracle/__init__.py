"""CPU oracle for the optimizer-step / mixed-precision hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy, the arithmetic of the reference implementation
(renderityai/NamiTorch, pure Python over NumPy/CuPy) for the functions on the hot path:

* ``oracle.adamw``  — Adam / AdamW updates (namitorch/optim/adam.py, namitorch/optim/_common.py)
* ``oracle.amp``    — GradScaler unscale / finite check / dynamic loss-scale update (namitorch/amp.py)
* ``oracle.clip``   — total gradient norm and clipping (namitorch/optim/clip_grad.py)
* ``oracle.xent``   — cross-entropy forward and backward (namitorch/nn/functional.py,
                      namitorch/_backend.py, namitorch/autograd.py)
* ``oracle.casts``  — round-to-nearest-even float32 -> bfloat16 / float16

Each function cites the reference lines it follows. The restatement is pinned against the
reference itself: ``tests/golden/make_golden.py`` runs the reference's own code in the
development container and records checksums and values, and the CPU test suite checks this
package against those fixtures.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline / reference arm
may import this package, and only as the checker or as the timed CPU baseline. The CUDA
product path (``namitorch_b200``) never imports, calls or falls back to it.
"""

__all__ = ["adamw", "amp", "clip", "xent", "casts"]
