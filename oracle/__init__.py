"""CPU oracle for the NVFP4 fused-MoE layer: TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference
arm may import, call or link anything in this package, and only as the checker or the
timed CPU baseline. The product path (``ftb``) never routes through it: the product fails
loudly when its CUDA library is missing.

Modules (the seeded synthetic generator the tests feed them lives in the product package,
``ftb.synth``, because bench.py and the tests generate device-side inputs with it):
  moe_oracle   numpy restatement of the reference's op order (per-route NVFP4 GEMV with
               per-word partials, bf16 stage roundings, SwiGLU, routed-weight down GEMV,
               fixed-order combine, shared-expert add), the router, and the permutation.
  cpu_moe      ctypes binding of cpu_moe.cpp, the OpenMP/AVX-512 C++ restatement that is
               both a second oracle and the timed CPU baseline.

Parity pins: golden vectors under ``tests/golden/`` were produced by the reference's own
Triton kernels (``fused_route.py``, ``nvfp4_marlin_swiglu.py``, the ``_e2m1_to_*`` helpers of
``kernel_triton_nvfp4_fused_moe.patch``) run by Triton's CPU interpreter; the generating
script is ``tests/golden/make_golden.py``.
"""
