"""dspine_b200 -- B200-native (sm_100a) draft-block verification for DSpine speculative decoding.

The CUDA kernels live in csrc/ and are compiled into _lib/libdspine_b200.so (C ABI declared in
include/dspine_b200.h).  Host modules:
  verify        fused verification from logits (dsv_verify_logits, dsv_verify_logits_noalloc)
  lmhead        fused LM head + top-k + logsumexp, vocab-parallel TPHead (one all-gather)
  accept        greedy capped accept, standalone accept-compact
  sampling.rejection / sampling.random / sampling.tp_head / verification.sps /
  kernels.dspine / layers.fp8.coarse / layers.fp8.gather
                the reference's operators at the reference's module paths (sglang_dspine.*),
                same signatures and argument errors, backed by the CUDA kernels.
"""

__version__ = "0.1.0"
