"""larder_b200: Larder's attention / Gated-DeltaNet hot path as hand-written B200 (sm_100a) CUDA kernels.

The kernels live in liblarder_b200.so behind a plain C ABI (include/larder_b200.h). The Python modules here mirror
the reference's module surface so its callers pick them up as a drop-in:

  chunkattn  -- chunked / wide-cut causal prefill attention and the patched scaled_dot_product_attention
  foldattn   -- folded GQA multi-row (verify) attention on the split-KV decode kernel
  gdn_cuda   -- the Gated-DeltaNet recurrence (chunked prefill and recurrent decode) and gated_delta_update
  ops        -- the torch-level wrappers of every C-ABI entry point
  sharded    -- multi-GPU: sequence-sharded prefill, KV-range-sharded decode merged over NCCL
"""
from . import _lib, ops  # noqa: F401

__all__ = ["ops"]
