"""CPU oracle for the decode-attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this package:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may use it, and only as the checker
or as the timed CPU baseline, never as the thing that is measured or shipped.

Contents
--------
``attention``  fp32 PyTorch (CPU) restatements of the reference's own oracles:
               dense GQA decode, StreamingLLM sink+window decode, the compacted
               cache builder, the slot validity rule, and the KIVI quantized
               attention oracle.
``kivi``       numpy restatement of the KIVI 2-bit quantizers (bit-exact with
               the reference's Triton kernels run under TRITON_INTERPRET=1),
               the unpack/dequant reference, ``build_quantized_kv_cache`` and a
               pure-Python model of the streaming (append) KIVI cache.

Parity pinning
--------------
The restatements are pinned against outputs of the reference itself, produced
in a container that has the reference checked out by
``tests/golden/make_golden.py`` (Triton interpreter on CPU) and committed as
fixtures under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks every
fixture.  The ring-buffer / append semantics have no reference counterpart;
they are pinned indirectly: at group-aligned phases the streaming cache state
must equal ``build_quantized_kv_cache`` of the same window (bit-exact) and the
attention output must equal the reference oracle's.
"""
