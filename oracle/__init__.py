"""TEST INFRASTRUCTURE ONLY — the CPU oracle of the HFFN sparse FFN hot path.

Nothing in ``hffn_b200`` imports, calls or links anything here. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use this package, and there only as the checker or as
the timed CPU baseline, never as the product path.

Contents:
- ``forward64``: float64 forward (``runtime/common/ffn/hffn_ffn_layers/reference.py:21-38`` of the reference);
- ``train64``: float64 forward + every backward group and the AdamW closed form
  (``runtime/gpu/nvidia/ffn/training/train_step.py:56-91``), plus the MSE loss of the training benchmark;
- ``layout``: the integer layouts (output-major down edges, transposed supports), numpy stable sorts
  (``runtime/gpu/nvidia/common/kernels/hffn_cuda/runtime.py:55-67``, ``runtime/gpu/nvidia/ffn/training/
  train_runtime.py:39-56``);
- ``x86ref``: ctypes binding of the reference's own x86 AVX2 inference kernel, compiled from the reference
  sources by ``oracle/Makefile`` into ``oracle/_ref/`` (``runtime/cpu/x86/ffn/inference/hffn/compact.py:107-217``).

Pinning: ``tests/test_oracle_golden.py`` checks ``forward64`` and ``train64`` against golden outputs that
``tests/golden/make_golden.py`` produced by running the reference's own Python oracles, and checks the generator
against the reference's pinned SHA-256 fingerprints; the x86 kernel is checked against ``forward64``.
"""
