"""CPU oracle for the chestnut frame path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference's hot path
(Alice7371/chestnut-on-pc, ``run_pinned2.py`` ``run_frame``) so that the CUDA
engine can be checked against it.  Only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` leg of ``bench.py`` may import it; the engine never
calls into it and has no CPU fallback.

Pinning status:
  * WMMA tile semantics (``wmma.py``) are pinned by the reference's own
    known-answer probes (``consumer_probe.py:142-171``, ``ffma_probe.py:112-139``,
    ``mma_probe.py:86-105``), restated as golden vectors in ``tests/golden``.
  * image2d border semantics (``border.py``) are pinned by the OpenCL sampler
    probe (``research/probe_sampler.py:12-23``) restated as a known-answer case.
  * queue semantics (``queues.py``) restate ``compile_modeld.py:166-221``.
  * the synthetic 39M / 1B models (``model.py``) have no reference output: the
    reference's pickles and its pinned tinygrad are absent, so model-level
    parity is UNPINNED -- it is defined by this restatement.
"""
