"""CPU oracle for the quantfun2 DiT hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``quantfun2_b200`` imports this package; it is
used by ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
arm of ``bench.py`` as the checker and CPU baseline, never as the measured or
shipped path.

Parity status per module:
  ops.py        RoPE / RMSNorm / softmax restatements of src/kernels/__init__.py,
                PINNED against golden vectors produced by the reference's own eager
                bodies (tests/golden/make_golden.py imports the reference).
  sage.py       SageAttention-style INT8/FP8 quantization and attention.  The
                reference calls the third-party `sageattention` package (unpinned
                version, absent from the reference tree), so this restatement of the
                published algorithm is PARITY UNPINNED against it; the float output
                is checked against the reference's own SDPA branch
                (src/models/common/attn.py:123-130) within a stated tolerance.
"""
