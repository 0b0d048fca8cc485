"""CPU oracle for the Switch Attention GQA prefill path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference implementation
(YushengZhao/SwitchAttentionKernels) computes on its hot path:

* ``indices``  -- routing-mask compaction and capacity buckets
  (``swiattn_gqa_prefill_varlen.py:271-322``), in numpy;
* ``metadata`` -- the per-row key bounds of the varlen metadata
  (consumed at ``swiattn_gqa_prefill_varlen.py:97-99,134-151,186-196``), in numpy;
* ``attention`` -- the two branch kernels (``swiattn_gqa_prefill.py:69-214``,
  ``swiattn_gqa_prefill_varlen.py:103-249``) as an FP32 torch computation, plus
  a tile-by-tile restatement of the kernel loop for small cases.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker (or, for the CPU
baseline, as the timed CPU restatement).  The product package never imports it.

Pinning.  The index compaction, capacity buckets, dispatch decisions and
validation errors are pinned against the reference's own Python code, executed
on the CPU by ``tests/golden/make_golden.py`` (fixtures in ``tests/golden``).
The attention numerics are **parity unpinned**: the reference kernels are
TileLang programs that only lower for Hopper (``T.wgmma_gemm``), so no output
of the reference kernel exists to compare with; the attention oracle follows
the kernel source line by line instead (citations in ``attention.py``).
"""
