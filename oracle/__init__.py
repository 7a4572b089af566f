"""CPU oracle for the FLUX transformer step — TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it. The product path
(``selas_b200``) never imports it and has no CPU fallback.

* ``oracle.flux_ref`` restates selas's eager PyTorch block math (``selas/models/flux.py``) on the CPU,
  in fp32 or in the bf16 compute dtype, plus the runner/prologue needed to replay a whole denoise run.
* ``oracle.nf4_ref`` restates the bitsandbytes-compatible NF4 codec of ``selas/codecs.py`` in numpy.

Both are pinned against golden vectors produced by the reference itself (``tests/golden/``).
"""
