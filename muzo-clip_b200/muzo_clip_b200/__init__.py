"""muzo_clip_b200 — MuZO-Clip's optimizer hot path on NVIDIA B200 (sm_100a).

Drop-in for the reference package ``muzo_clip``: the same public names, signatures and returned
statistics, backed by the native library ``libmuzo_b200.so`` (C ABI in include/muzo_b200.h).
"""

from .muzo_optimizer import MuZOClipOptimizer
from .newton_schulz import zeropower_via_newtonschulz5
from .parameter_filter import select_muzo_parameters
from .prng import iter_param_blocks, make_zo_noise_like
from .qk_clip import use_qk_capture_attention

__all__ = [
    "MuZOClipOptimizer",
    "iter_param_blocks",
    "make_zo_noise_like",
    "select_muzo_parameters",
    "use_qk_capture_attention",
    "zeropower_via_newtonschulz5",
]
