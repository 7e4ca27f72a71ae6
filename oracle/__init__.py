"""CPU oracle for the RFSN compressed-KV decode path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / ``--impl reference`` legs may import this
package, and only as the checker (or the timed CPU baseline), never as the
thing measured on the GPU path.  The product package ``apple_b200`` never
imports it and has no CPU fallback.

* ``restate`` — numpy restatement of the reference algorithm (quantization.py,
  attention.py, cache.py, storage.py, rfsn_v10_mlx_ane_complete.py), each
  function citing the reference lines it follows, plus the extensions the
  B200 build adds (GQA, batch, recent-hot policy, top-k sparse residual).
  Pinned against golden fixtures produced by the reference itself.
* ``ref_loader`` + ``mlx_shim`` — run the unmodified reference on torch-CPU to
  produce those fixtures (only where the reference sources are present).
"""
