"""kquant_b200: B200-native EXL3/QSRT trellis weight encoder.

Drop-in backend for kquant's ``exl3_encoder_backend`` plugin API, on
hand-written sm_100a CUDA kernels reached through a C ABI
(``include/kq_b200.h``).
"""

__all__ = ["codebooks", "exl3_encoder_backend", "exl3_loader", "ldlq", "sqg_quantizer"]
__version__ = "0.1.0"
