"""CPU oracle for the int4/int2 linear hot path. TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the reference algorithms of
``onecomp_runtime`` (kizuna-intelligence/onecompression-runtime) that the B200
kernels must reproduce:

* ``oracle.gptq``  -- AutoGPTQ v1/v2 unpack + dequant (``quant_utils.py:12-69``)
  and the qweight packer (``layers/fused_int4_linear.py:76-91``);
* ``oracle.rtn``   -- RTN uint8-nibble dequant (``quant_utils.py:72-103``), the packed
  embedding lookup (``layers/packed_linear.py:93-104``) and the conv codecs' RTN encoder
  (``layers/packed_conv.py:63-90``);
* ``oracle.dsv4``  -- DSV4 int4/int2 byte-packed dequant
  (``layers/dsv4_packed_linear.py:22-56``);
* ``oracle.eager`` -- the eager linear (``backend.py:246-264`` + ``F.linear``)
  and the MoE convention used by the grouped-expert path;
* ``oracle.fp``    -- IEEE-754 bf16/fp16 rounding helpers (round to nearest even).

Pinning: every function here is checked bit-for-bit (dequant) or within the
stated tolerance (GEMM) against golden vectors produced by running the
reference itself (``tests/golden/make_golden.py``, fixtures in
``tests/golden/*.npz``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline. The product path
(``onecompression-runtime_b200/onecomp_runtime``) never imports it.
"""
