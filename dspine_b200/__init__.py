"""dspine_b200 -- B200-native (sm_100a) draft-block verification for DSpine speculative decoding.

The CUDA kernels live in csrc/ and are compiled into _lib/libdspine_b200.so (C ABI declared in
include/dspine_b200.h).  Host modules mirror the reference package ``sglang_dspine`` at the same
module paths (sampling.rejection, sampling.sparse.accept, kernels.dspine, verification.caps,
verification.sps, sampling.tp_head, sampling.random, runtime.worker) so that the reference's
plugin hooks can call them unchanged.  ``verify.verify_logits`` is the fused entry point.
"""

__version__ = "0.1.0"
