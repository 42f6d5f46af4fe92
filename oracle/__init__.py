"""CPU oracle for FERRY's per-MoE-layer hot path.

TEST INFRASTRUCTURE ONLY.  This package restates the reference algorithms on
the CPU so that the CUDA kernels of ``ferry_b200`` can be checked against them.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
(``cpu_baseline`` and ``--impl reference``) may import it; the product path never does, and fails loudly when
its CUDA library is missing instead of falling back here.

Contents
  planner      ctypes binding of ferry_oracle.c: _demand, _admission_capacity,
               greedy_quota, build_lut, load_balanced_assignment, _choose_slot,
               plan_layer (FERRY and RANDOM), layer_slots, build_layout.
  metadata     GateHistory and the RouteGather history-row rule.
  expert_ops   torch-CPU restatement of ferry_expert_ops (pack_dispatch,
               unpack_dispatch, execute_experts, reduce_partials,
               scatter_returned) and of the MoE-hook routers.
  layer        one MoE layer over R emulated ranks, end to end on the CPU
               (the CPU baseline and the --impl reference arm of bench.py).
  dist_layer   the same layer across gloo processes with real collectives.
  build_ref    builds the reference's own expert_ops extension into _ref/.

Parity pin: tests/golden/ holds vectors produced by running the reference's
own numba/numpy code (tests/golden/make_golden.py); the integer algorithms are
checked bit-exactly against them.  The floating-point expert math has no
reference golden vectors (the reference's ops are CUDA-only); it follows the
reference's ATen op order and rounding points, and on a GPU box it is also
compared with the reference's own extension built by oracle/build_ref.py.
"""
