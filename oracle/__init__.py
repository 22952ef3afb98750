"""CPU oracle for the VDN hot path. TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithms of ec-jt/vdn that the
B200 kernels replace: the block-32 E4M3/E8M0 MXFP8 quantiser and its
SWIZZLE_32_4_4 scale layout, the dequantised MXFP8 GEMM, and the frame-wise
bidirectional delta-rule linear-attention branch (VDA).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` (plus ``bench.py --impl reference``) may import it, and only as
the checker or the timed CPU baseline.  The product package ``vdn_b200`` never
imports it; a missing CUDA extension makes the product raise, it never routes
here.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own CPU
code (``quantize_cpu``, ``BidirectionalLinearBranch._readout``,
``VdnDelta.factor_apply``, ``_run_scans``, ``gather_linear_state``) on seeded
inputs and stores inputs and outputs under ``tests/golden/``; the ``-m "not
gpu"`` tests check this oracle against those fixtures and against the
reference's own known-answer vectors.
"""
