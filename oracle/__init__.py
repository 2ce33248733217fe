"""CPU oracle for the Kairos hybrid-attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
package.  Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
/ ``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or as the timed CPU baseline, never as the thing measured on the GPU.

Contents
--------
``gdn``        chunked gated delta rule (FLA v0.4.0 vendored in the reference
               under ``kairos/third_party/fla``) restated in plain torch CPU
               code, plus the token recurrence of
               ``fla/ops/gated_delta_product/naive.py:4-36``.
``attention``  softmax attention reference (the reference's own
               ``F.scaled_dot_product_attention`` fallback,
               ``kairos/modules/dits/kairos_dit.py:269-276``) and the per-head
               e4m3 quantisation that the FP8 kernel performs.
``layers``     the GatedDeltaNet prologue/epilogue element-wise math and the
               Ulysses all-to-all re-partition as index arithmetic.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own code in
the build container (the naive recurrence by file path, and the reference's
Triton chunk kernels under ``TRITON_INTERPRET=1``) and commits the outputs as
fixtures; ``tests/test_oracle.py`` checks this oracle against them.
"""
