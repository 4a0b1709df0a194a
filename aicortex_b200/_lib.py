"""ctypes binding of include/aicortex.h (libaicortex_b200.so).

The library is the product: there is no Python or CPU fallback. Importing
this module fails loudly when the shared library has not been built.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libaicortex_b200.so"

AIC_OK = 0
AIC_ERR_INVALID = 1
AIC_ERR_UNSUPPORTED = 2
AIC_ERR_CUDA = 3
AIC_ERR_STATE = 4
AIC_ERR_IO = 5
AIC_MAX_BLOCKS = 16
AIC_CONV_ORDERED = 0
AIC_CONV_FAST = 1
AIC_CONV_SIMT = 2
AIC_MAMBA_TENSOR = 0
AIC_MAMBA_EXACT = 1


class AicError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"aicortex status {status}: {message}")
        self.status = status


class ConvLayerDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("in_channels", "out_channels", "kernel_size", "stride", "dim_in", "dim_out",
                                        "disable_activation")]


class ConvBlockDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("in_channels", "mid_channels", "out_channels", "stride", "dim_in", "dim_out",
                                        "dw_kernel")] + [("survival_probability", C.c_float),
                                                         ("residual_factor", C.c_float)]


class MambaLayerDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("d_model", "d_state", "out_channels", "activation")]


class MambaBlockDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("d_model", "d_state", "out_channels", "activation")] + [
        ("survival_probability", C.c_float), ("residual_factor", C.c_float)]


class CriticDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("in_channels", "units", "dim_in")]


class CortexDesc(C.Structure):
    _fields_ = [("planes", C.c_int), ("stem_channels", C.c_int), ("dim", C.c_int), ("n_blocks", C.c_int),
                ("blocks", ConvBlockDesc * AIC_MAX_BLOCKS), ("d_model", C.c_int), ("d_state", C.c_int),
                ("n_units", C.c_int), ("unit_residual_factor", C.c_float), ("actor_out", C.c_int),
                ("actor_activation", C.c_int), ("critic_units", C.c_int), ("chunk_frames", C.c_int)]


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int
F32 = C.c_float
SZ = C.POINTER(C.c_size_t)
PI64 = C.POINTER(C.c_int64)
PP = C.POINTER(C.c_void_p)

# name -> argtypes (restype is always aic_status = int)
_SIGS = {
    "aic_device_error_sync": [C.POINTER(C.c_int)],
    "aic_pack_f32": [P, I64, P, P, I32, I32, P],
    "aic_stem_pack": [P, I64, I32, I32, I32, P, P, P],
    "aic_residual_add": [P, P, P, P, P, P, I64, I32, F32, I32, P],
    "aic_gap": [P, P, I64, I32, I32, P, P, P, P],
    "aic_gap_f16": [P, P, I64, I32, I32, P, P],
    "aic_screen_frontend": [P, P, I32, I32, I32, C.c_uint32, F32, F32, P],
    "aic_set_actions": [P, I64, I32, P, P],
    "aic_selftest_rcp": [P, P, P],
    "aic_audio_workspace_bytes": [SZ],
    "aic_audio_frontend": [P, P, I32, I32, P, P],
    "aic_conv_layer_create": [C.POINTER(ConvLayerDesc), PP],
    "aic_conv_layer_sizes": [P, PI64, PI64, SZ],
    "aic_conv_layer_bind": [P, P],
    "aic_conv_layer_param_ptrs": [P, PP, PP, PP],
    "aic_conv_layer_load_weights": [P, P, P, P],
    "aic_conv_layer_load_file_sync": [P, C.c_char_p, P],
    "aic_conv_layer_forward": [P, P, P, P, P, I64, P],
    "aic_conv_layer_forward_exact": [P, P, P, P, P, I64, P],
    "aic_conv_layer_set_mode": [P, I32],
    "aic_conv_layer_destroy": [P],
    "aic_conv_block_create": [C.POINTER(ConvBlockDesc), PP],
    "aic_conv_block_layer": [P, I32, PP],
    "aic_conv_block_param_bytes": [P, SZ],
    "aic_conv_block_bind": [P, P],
    "aic_conv_block_workspace_bytes": [P, I64, SZ],
    "aic_conv_block_load_dir_sync": [P, C.c_char_p, P],
    "aic_conv_block_forward": [P, P, P, P, P, I64, I32, I32, P, P],
    "aic_conv_block_destroy": [P],
    "aic_selftest_wait_timeout": [I32, P, P],
    "aic_grad_clip_partials": [I64, PI64],
    "aic_grad_clip_factor": [P, I64, P, P, P],
    "aic_sgd_update": [P, P, I64, P, F32, F32, P],
    "aic_residual_backward": [P, P, I64, F32, F32, P],
    "aic_conv_layer_train_bytes": [P, SZ],
    "aic_conv_layer_train_bind": [P, P, P, F32, F32, P],
    "aic_conv_layer_backward": [P, P, P, P, P, P],
    "aic_conv_layer_train_views": [P, PP, PP, PP, PP],
    "aic_mamba_layer_train_bytes": [P, SZ],
    "aic_mamba_layer_train_bind": [P, P, P, F32, F32, P],
    "aic_mamba_layer_backward": [P, P, P, P, P, P],
    "aic_mamba_layer_train_views": [P, PP, PP, PP, PP],
    "aic_critic_train_bytes": [P, SZ],
    "aic_critic_train_bind": [P, P, F32, F32],
    "aic_critic_backward": [P, P, F32, P],
    "aic_critic_train_views": [P, PP, PP, PP],
    "aic_mamba_layer_create": [C.POINTER(MambaLayerDesc), PP],
    "aic_mamba_layer_sizes": [P, PI64, PI64, SZ],
    "aic_mamba_layer_bind": [P, P],
    "aic_mamba_layer_param_ptrs": [P, PP, PP, PP],
    "aic_mamba_layer_load_weights": [P, P, P, P],
    "aic_mamba_layer_load_file_sync": [P, C.c_char_p, P],
    "aic_mamba_layer_state_bytes": [P, I32, SZ],
    "aic_mamba_layer_bind_state": [P, P, I32],
    "aic_mamba_layer_trace_bytes": [P, I32, P],
    "aic_mamba_layer_bind_traces": [P, P, I32],
    "aic_mamba_layer_reset_state": [P, P],
    "aic_mamba_layer_workspace_bytes": [P, I64, SZ],
    "aic_mamba_layer_forward": [P, P, P, P, I32, I32, P, P],
    "aic_mamba_layer_outproj": [P, P, P, I64, P],
    "aic_mamba_layer_set_mode": [P, I32],
    "aic_mamba_layer_scan": [P, P, P, P, I32, I32, I32, P],
    "aic_mamba_layer_outproj_split": [P, P, P, I64, P],
    "aic_mamba_layer_forward_noalloc": [P, P, P, P, I32, I32, P],
    "aic_mamba_layer_destroy": [P],
    "aic_mamba_block_create": [C.POINTER(MambaBlockDesc), PP],
    "aic_mamba_block_layer": [P, I32, PP],
    "aic_mamba_block_param_bytes": [P, SZ],
    "aic_mamba_block_bind": [P, P],
    "aic_mamba_block_state_bytes": [P, I32, SZ],
    "aic_mamba_block_bind_state": [P, P, I32],
    "aic_mamba_block_trace_bytes": [P, I32, P],
    "aic_mamba_block_bind_traces": [P, P, I32],
    "aic_mamba_block_reset_state": [P, P],
    "aic_mamba_block_workspace_bytes": [P, I64, SZ],
    "aic_mamba_block_load_dir_sync": [P, C.c_char_p, P],
    "aic_mamba_block_forward": [P, P, P, P, I32, I32, I32, I32, I32, P, P],
    "aic_mamba_block_set_mode": [P, I32],
    "aic_mamba_block_destroy": [P],
    "aic_critic_create": [C.POINTER(CriticDesc), PP],
    "aic_critic_param_bytes": [P, SZ],
    "aic_critic_bind": [P, P],
    "aic_critic_load_weights": [P, P, P, P, P],
    "aic_critic_load_file_sync": [P, C.c_char_p, P],
    "aic_critic_state_bytes": [P, I32, SZ],
    "aic_critic_bind_state": [P, P, I32],
    "aic_critic_trace_bytes": [P, I32, P],
    "aic_critic_bind_traces": [P, P, I32],
    "aic_critic_reset_state": [P, P],
    "aic_critic_workspace_bytes": [P, I64, SZ],
    "aic_critic_forward": [P, P, P, P, I32, I32, P, P],
    "aic_critic_forward_pooled": [P, P, P, I32, I32, P, P],
    "aic_critic_destroy": [P],
    "aic_cortex_create": [C.POINTER(CortexDesc), PP],
    "aic_cortex_block": [P, I32, PP],
    "aic_cortex_unit": [P, I32, PP],
    "aic_cortex_actor": [P, PP],
    "aic_cortex_critic": [P, PP],
    "aic_cortex_param_bytes": [P, SZ],
    "aic_cortex_bind": [P, P],
    "aic_cortex_state_bytes": [P, I32, SZ],
    "aic_cortex_bind_state": [P, P, I32],
    "aic_cortex_reset_state": [P, P],
    "aic_cortex_workspace_bytes": [P, I32, I32, SZ],
    "aic_cortex_forward": [P, P, I32, I32, P, P, P, P, P, P],
    "aic_cortex_host_workspace_bytes": [P, I32, I32, SZ],
    "aic_cortex_forward_host": [P, P, I32, I32, P, P, P, P],
    "aic_cortex_set_exact": [P, I32],
    "aic_cortex_set_conv_mode": [P, I32],
    "aic_cortex_set_mamba_mode": [P, I32],
    "aic_cortex_last_launches": [P, PI64],
    "aic_cortex_profile_enable": [P, I32],
    "aic_cortex_profile_count": [P, C.POINTER(C.c_int)],
    "aic_cortex_profile_get": [P, I32, C.c_char_p, C.POINTER(C.c_double), PI64, C.POINTER(C.c_double),
                               C.POINTER(C.c_double)],
    "aic_cortex_profile_reset": [P],
    "aic_cortex_destroy": [P],
}


def _load() -> C.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(f"{_LIB_PATH.name} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
                          "(the CUDA extension is required, there is no fallback path)")
    lib = C.CDLL(str(_LIB_PATH))
    lib.aic_last_error.restype = C.c_char_p
    lib.aic_last_error.argtypes = []
    lib.aic_abi_version.restype = C.c_int
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = C.c_int
    return lib


lib = _load()
SYMBOLS = ("aic_last_error", "aic_abi_version", *_SIGS)


def call(name: str, *args) -> None:
    """Call an aic_* function and raise AicError on a non-zero status."""
    status = getattr(lib, name)(*args)
    if status != AIC_OK:
        raise AicError(status, lib.aic_last_error().decode(errors="replace"))
