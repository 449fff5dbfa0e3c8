"""B200-native (sm_100a) implementation of ReCaVSR's DiT hot path.

Drop-in modules mirroring the reference operator surface:
  recavsr_b200.kernels.local_attention  (paired_attention, sdpa_attention)
  recavsr_b200.kernels.native_norm      (native_layer_norm, native_rms_norm)
  recavsr_b200.runtime.nvfp4 / fp8      (quantizers, GEMMs, NVFP4Linear / FP8Linear)
  recavsr_b200.runtime.cache / rope     (FixedKVCache router, RollingRoPE)
plus the fused block executor recavsr_b200.runtime.block. All compute runs in
librecavsr_b200.so (include/recavsr_b200.h); PyTorch provides memory and streams.
"""

__version__ = "0.1.0"
