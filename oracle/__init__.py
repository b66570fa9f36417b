"""CPU oracle of the tensor-parallel RMSNorm -- TEST INFRASTRUCTURE ONLY.

Restates, on the CPU, the arithmetic of the reference (haowen-han/RmsnormTP):

* ``tp_rmsnorm.py``  -- numpy restatement of the AllReduce TP RMSNorm
  (bench_rmsnorm_tp.py:16-22 / test_rmsnorm_tp.py:15-26) and of the fused
  kernel's formula (csrc/rmsnorm_tp.cu:72-96, :143-170). It is the parity
  checker of the CUDA path.
* ``torch_port.py`` -- the same AllReduce path on torch CPU tensors, for every
  rank of a group in one process (the CPU baseline that bench.py times) or
  across gloo ranks (the multi-process tests).

Parity is pinned: tests/golden/ holds vectors produced by running the
reference's own ``reference_tp_rmsnorm`` under gloo on CPU
(tests/golden/make_golden.py), and tests/test_oracle_golden.py checks both
restatements against them.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
``--impl reference`` legs may import this package, and only as the checker or
the CPU baseline -- never as the thing measured on the GPU path, which has no
CPU fallback.
"""
