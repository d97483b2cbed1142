"""B200-native TurboAdam: packed-state optimizer step on hand-written sm_100a
kernels behind a C ABI (include/turboadam_b200.h)."""
from .optimizer import TurboAdam, TurboAdamCommError

__version__ = "0.1.0"

__all__ = ["TurboAdam", "TurboAdamCommError"]
