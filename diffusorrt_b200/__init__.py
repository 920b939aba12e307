"""diffusorrt_b200 — B200-native (sm_100a) denoising-decode engine for block-diffusion and
masked-diffusion language models, a drop-in device-session provider for the DiffusorRT SDK.

    from diffusorrt_b200 import Runtime
    with Runtime(model_config=..., synthetic_seed=0) as rt, rt.session({...}) as s:
        s.start_device(...); s.propose_device(...); s.commit_device(...)

The compute path is the native library libdiffusorrt_b200.so (hand-written tcgen05 / TMA
kernels); see include/diffusorrt_b200.h for its C ABI.
"""
from .runtime import Runtime, Session, WindowResult  # noqa: F401

__all__ = ["Runtime", "Session", "WindowResult"]
