"""anima_attn -- B200-native attention for the Anima 2B DiT denoiser.

sm_100a kernels (tcgen05 / TMEM / TMA flash-attention forward, fused per-head
RMSNorm + 3D RoPE prologue) in libanima_attn.so, behind the reference runtime's
C ABI (include/anima_rt.h) and a device-pointer ABI (include/anima_attn.h).

Import from the repository root with the distribution folder on sys.path:

    sys.path.insert(0, "<repo>/anima-on-android_b200")
    import anima_attn
"""
from . import _lib
from ._lib import AnimaError, last_error
from .ops import apply_rope, attention, attention_core, device_info, prologue, sdpa, status, version
from .rope import rope_freqs_3d

__all__ = ["AnimaError", "apply_rope", "attention", "attention_core", "device_info", "last_error",
           "prologue", "rope_freqs_3d", "sdpa", "status", "version", "_lib"]
