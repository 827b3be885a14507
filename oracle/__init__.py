"""CPU oracle for the sparse decode-attention path.  TEST INFRASTRUCTURE ONLY.

* ``oracle.exact``: ctypes bindings of exact.c (the reference algorithm in the
  CUDA kernels' arithmetic order; GPU results must equal it bit for bit).
* ``oracle.torch_ref``: the reference's torch operator sequence (device-agnostic).
* ``oracle.synth``: seeded synthetic inputs.
* ``oracle.refgather``: the reference's own OpenMP ``gather_kv`` compiled from its
  sources into oracle/_ref/ (hi/cpu_kv_gather.cpp, hi/cpu_kv_run_gather.cpp).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may use
this package, and only as the checker or the timed CPU baseline.
"""
