"""CPU oracle for the paged decode path -- TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py` (its CPU-baseline leg,
the reference arm, and the TP parity check run after the timed region) may
import this package, and only as the checker (or the timed CPU baseline).
The product (`torch_spyre_b200`) never imports it and has no CPU fallback.

Contents
  paged_attention  the reference's CPU eager decode path: paged gather, then
                   stock torch CPU SDPA in fp32 (the truth the reference's own
                   harness compares against, tests/inductor/utils_inductor.py:
                   620-703), plus an explicit restatement of the reference's
                   SDPA decomposition (torch_spyre/_inductor/decompositions.py:
                   549-596) as a second check.
  stick_layout     restatement of SpyreTensorLayout's tiling and stride map
                   (torch_spyre/csrc/spyre_tensor_impl.cpp:46-175) and of the
                   host<->device element map the DMA descriptors encode
                   (docs/source/user_guide/tensors_and_layouts.md "DMA
                   Encoding"; torch_spyre/csrc/spyre_mem.cpp:176-440).
  kv_relayout      numpy restatement of the KV append (overwrite_cpu,
                   torch_spyre/_inductor/customops.py:298-308; index_copy_) and
                   of the row-major <-> paged stick relayout, bit-exact.
  tp_step          the head-sharded TP step: decode of all heads, then the
                   full o_proj in fp32 (= the SUM all-reduce of the per-rank
                   partials, spyre_ccl.cpp:470-494).

Parity pinning: the layout restatement is checked against the reference's
golden layout vectors (tests/tensor/test_tensor_layout.py:39-104, 193-280); the
attention oracle is stock torch 2.11 CPU SDPA -- the same version the reference
pins -- checked against committed fixtures in tests/golden/ generated from the
reference's own decode test inputs (test_inductor_ops.py:2651-2678).
"""
