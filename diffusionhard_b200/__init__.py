"""B200-native (sm_100a) MDLM denoising hot path: W8A8 DDiT tensor engine,
rotary bidirectional attention with prefix K/V reuse, fused int8 output head
with Philox-Gumbel noisy argmax, and the candidate-cache ddpm_cache loop.

The compute lives in ``lib/libdh_b200.so`` (C ABI: ``include/dh_b200.h``);
this package is the host-side orchestration behind the reference's sampler
protocol.
"""

__version__ = "0.1.0"
