"""CPU oracle for the B200 decode hot path -- TEST INFRASTRUCTURE ONLY.

Plain numpy / torch-CPU restatements of the reference's algorithms for the four ops on the
path (device LRU expert cache, fused SiLU-mul -> FP8 quant, FP8 block-scaled lm_head, W4
group-128 lm_head). Every function cites the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import this package, and only as the checker or the timed CPU
baseline. The product package never imports it: its ops fail loudly when the CUDA
extension is missing instead of falling back here.
"""
