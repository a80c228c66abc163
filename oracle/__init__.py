"""CPU oracle for the cooperative-matrix GEMM / flash-attention path — TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference
legs may import this package, and only as the checker (or the timed CPU stand-in for the
reference's own CPU path). Nothing in ``lava.jl_b200/`` imports it; the product path fails
loudly without its CUDA library.

PARITY UNPINNED. Lava.jl (the reference) is a Julia→SPIR-V compiler whose arithmetic runs
inside a Vulkan driver or lavapipe; neither Julia nor a graphics stack exists on this
machine or the GPU box, and the reference's tests hold no numeric golden vectors for this
path (they are structural SPIR-V checks). The modules here restate the reference's
documented semantics, each function citing the Lava.jl file:line it follows, and are
pinned against:

* the reference's own definitions that are executable by reading: ``dot4x8``
  (``src/vocabulary/vocabulary.jl:31-35``), ``tensor_clampbits``
  (``src/vocabulary/tensor.jl:83-85``), the clamp-mode enum values
  (``src/vocabulary/tensor.jl:46-51``) and the ``CoopMatReduce`` masks
  (``src/vocabulary/coopmat.jl:292-297``), with known answers worked by hand;
* exact integer / rational arithmetic (pure-Python loops) on small cases, which the
  float64 restatement must reproduce bit for bit.

Modules: ``vocab`` (element-level restatement of the vocabulary), ``gemm`` (tiled coopmat
GEMM following ``test/glsl/coopmat2_gemm_regs.comp:53-83`` plus a fast float64/int64
matmul), ``attention`` (softmax attention by definition, blockwise online form),
``inputs`` (the seeded generators of the benchmark configs). Integer products are exact
(int64 accumulation).
"""
