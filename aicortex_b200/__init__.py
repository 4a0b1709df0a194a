"""B200 (sm_100a) implementation of the AICortex inference hot path.

The compute lives in libaicortex_b200.so (CUDA kernels + C ABI declared in
include/aicortex.h); this package binds it with ctypes and mirrors the
reference's layer classes. Importing the package fails if the library is not
built: there is no fallback path.
"""
from ._lib import AIC_CONV_FAST, AIC_CONV_ORDERED, AIC_CONV_SIMT, AIC_MAMBA_EXACT, AIC_MAMBA_TENSOR, AicError, lib  # noqa: F401  (fails loudly when the .so is missing)
from .layers import (ConvBlock, ConvLayer, Cortex, Critic, MambaBlock, MambaLayer, audio_frontend, empty_f,  # noqa: F401
                     gap, gap_f16, grad_clip_factor, pack_f32, residual_add, residual_backward, screen_frontend,
                     set_actions, sgd_update, stem_pack)

__all__ = ["AIC_CONV_FAST", "AIC_CONV_ORDERED", "AIC_CONV_SIMT", "AIC_MAMBA_EXACT", "AIC_MAMBA_TENSOR", "AicError", "ConvBlock", "ConvLayer", "Cortex", "Critic", "MambaBlock", "MambaLayer", "audio_frontend", "empty_f", "gap",
           "gap_f16", "grad_clip_factor", "pack_f32", "residual_add", "residual_backward", "screen_frontend",
           "set_actions", "sgd_update", "stem_pack"]
