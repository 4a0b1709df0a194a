"""C-ABI checks that need no GPU: the library loads, exports every symbol
declared in include/aicortex.h, validates descriptors the way the reference
constructors constrain them, and reports errors as status codes."""
import ctypes as C
import re
import subprocess

import pytest

from conftest import ROOT

from aicortex_b200 import _lib
from aicortex_b200._lib import (AIC_ERR_INVALID, AIC_ERR_IO, AIC_ERR_STATE, AIC_ERR_UNSUPPORTED, AIC_OK,
                                ConvBlockDesc, ConvLayerDesc, CriticDesc, MambaLayerDesc, lib)

HEADER = ROOT / "include" / "aicortex.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"AIC_API\s+[\w\s\*]+?\b(aic_\w+)\s*\(", text)))


def test_header_symbols_exported():
    names = declared_symbols()
    assert len(names) > 60
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib._LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # everything the ctypes layer binds is declared in the header
    assert set(_lib.SYMBOLS) <= set(names)


def test_only_aic_symbols_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib._LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    text_syms = [line.split()[-1] for line in out.splitlines() if " T " in line]
    assert all(s.startswith("aic_") for s in text_syms), [s for s in text_syms if not s.startswith("aic_")][:10]


def _create_conv(desc):
    h = C.c_void_p()
    st = lib.aic_conv_layer_create(C.byref(desc), C.byref(h))
    return st, h


def test_conv_layer_validation_and_sizes():
    st, h = _create_conv(ConvLayerDesc(64, 128, 1, 1, 16, 16, 0))
    assert st == AIC_OK
    we, be, pb = C.c_int64(), C.c_int64(), C.c_size_t()
    assert lib.aic_conv_layer_sizes(h, C.byref(we), C.byref(be), C.byref(pb)) == AIC_OK
    assert we.value == 64 * 128 and be.value == 128
    assert pb.value >= 64 * 128 // 2 + 64 * 128 // 32 + 128 * 4
    assert lib.aic_conv_layer_destroy(h) == AIC_OK
    # depthwise weight count is k*k*C (conv_layer.h:51)
    st, h = _create_conv(ConvLayerDesc(96, 96, 7, 2, 16, 8, 1))
    assert st == AIC_OK
    assert lib.aic_conv_layer_sizes(h, C.byref(we), None, None) == AIC_OK and we.value == 49 * 96
    lib.aic_conv_layer_destroy(h)
    # the reference throws for these kernel sizes (conv_layer.h:114,129)
    assert _create_conv(ConvLayerDesc(64, 64, 9, 1, 16, 16, 1))[0] == AIC_ERR_UNSUPPORTED
    assert _create_conv(ConvLayerDesc(64, 64, 6, 6, 36, 6, 1))[0] == AIC_ERR_UNSUPPORTED
    # channel counts must be whole 32-groups
    assert _create_conv(ConvLayerDesc(48, 64, 1, 1, 16, 16, 0))[0] == AIC_ERR_INVALID
    assert b"32" in lib.aic_last_error()
    # the reference kernels index with & (dim_out - 1)
    assert _create_conv(ConvLayerDesc(64, 64, 3, 2, 12, 6, 1))[0] == AIC_ERR_INVALID


def test_mamba_layer_validation():
    h = C.c_void_p()
    # d_state 16 cannot be expressed by the reference kernel (d_state >> 5 == 0)
    assert lib.aic_mamba_layer_create(C.byref(MambaLayerDesc(256, 16, 256, 1)), C.byref(h)) == AIC_ERR_UNSUPPORTED
    assert lib.aic_mamba_layer_create(C.byref(MambaLayerDesc(192, 32, 256, 1)), C.byref(h)) == AIC_ERR_INVALID
    assert lib.aic_mamba_layer_create(C.byref(MambaLayerDesc(256, 512, 256, 1)), C.byref(h)) == AIC_OK
    we = C.c_int64()
    assert lib.aic_mamba_layer_sizes(h, C.byref(we), None, None) == AIC_OK
    assert we.value == 512 * (2 + 32 + 4 * 512 + 256)  # mamba_layer.h:58
    # forward before any state is bound is a state error, not a crash
    assert lib.aic_mamba_layer_forward(h, None, None, None, 1, 1, None, None) == AIC_ERR_STATE
    lib.aic_mamba_layer_destroy(h)


def test_block_and_critic_validation():
    h = C.c_void_p()
    assert lib.aic_conv_block_create(C.byref(ConvBlockDesc(64, 256, 128, 2, 32, 16, 3, 1.0, 0.75)), C.byref(h)) == AIC_OK
    layer = C.c_void_p()
    assert lib.aic_conv_block_layer(h, 3, C.byref(layer)) == AIC_OK
    we = C.c_int64()
    lib.aic_conv_layer_sizes(layer, C.byref(we), None, None)
    assert we.value == 128 * 4 * 64  # 2x2 stride-2 shortcut (conv_block.h:55)
    assert lib.aic_conv_block_layer(h, 4, C.byref(layer)) == AIC_ERR_INVALID
    lib.aic_conv_block_destroy(h)
    assert lib.aic_conv_block_create(C.byref(ConvBlockDesc(64, 256, 128, 2, 32, 16, 3, 0.0, 0.75)),
                                     C.byref(h)) == AIC_ERR_INVALID
    assert lib.aic_critic_create(C.byref(CriticDesc(32, 100, 256)), C.byref(h)) == AIC_ERR_INVALID
    assert lib.aic_critic_create(C.byref(CriticDesc(32, 128, 256)), C.byref(h)) == AIC_OK
    lib.aic_critic_destroy(h)


def test_null_handles_and_misaligned_binds():
    assert lib.aic_conv_layer_forward(None, None, None, None, None, 1, None) == AIC_ERR_INVALID
    st, h = _create_conv(ConvLayerDesc(64, 64, 1, 1, 8, 8, 0))
    assert lib.aic_conv_layer_bind(h, C.c_void_p(0x1000 + 8)) == AIC_ERR_INVALID
    # forward on an unbound layer is a state error
    assert lib.aic_conv_layer_forward(h, None, None, None, None, 1, None) == AIC_ERR_STATE
    lib.aic_conv_layer_destroy(h)


def test_checkpoint_file_errors(tmp_path):
    """Missing and truncated layer files (conv_layer.h:31-44) fail with AIC_ERR_IO
    before any device work."""
    st, h = _create_conv(ConvLayerDesc(64, 64, 1, 1, 8, 8, 0))
    # binding records the pointer only; the device is not touched on these paths
    assert lib.aic_conv_layer_bind(h, C.c_void_p(0x100000)) == AIC_OK
    assert lib.aic_conv_layer_load_file_sync(h, str(tmp_path / "missing.bin").encode(), None) == AIC_ERR_IO
    short = tmp_path / "short.bin"
    short.write_bytes(b"\0" * (4 * (64 * 64 + 64) - 4))
    assert lib.aic_conv_layer_load_file_sync(h, str(short).encode(), None) == AIC_ERR_IO
    assert b"short read" in lib.aic_last_error()
    lib.aic_conv_layer_destroy(h)


def test_cortex_desc_chaining():
    from aicortex_b200 import workloads as W
    d = W.cortex_desc()
    h = C.c_void_p()
    assert lib.aic_cortex_create(C.byref(d), C.byref(h)) == AIC_OK
    nb = C.c_size_t()
    assert lib.aic_cortex_workspace_bytes(h, 4, 3, C.byref(nb)) == AIC_OK and nb.value > 0
    lib.aic_cortex_destroy(h)
    d.blocks[1].in_channels = 96  # does not chain with block 0's 64 outputs
    assert lib.aic_cortex_create(C.byref(d), C.byref(h)) == AIC_ERR_INVALID
    assert b"chain" in lib.aic_last_error()


@pytest.mark.parametrize("n", [31, -32])
def test_pack_rejects_bad_sizes(n):
    assert lib.aic_pack_f32(None, n, None, None, 0, 0, None) == AIC_ERR_INVALID


def test_dropin_header_and_driver_compile(tmp_path):
    """include/aicortex_layers.hpp (the reference's layer classes over the C
    ABI) and the test driver that uses it compile and link against the
    library; running it needs a GPU (tests/test_dropin_gpu.py)."""
    import shutil
    import subprocess
    from conftest import ROOT
    if shutil.which("g++") is None:
        pytest.skip("no g++")
    exe = tmp_path / "dropin_main"
    cmd = ["g++", "-std=c++17", "-O0", "-Wall", "-Werror", "-Wno-unused-parameter", "-DAIC_LAYERS_D_MODEL=256",
           "-DAIC_LAYERS_D_STATE=128", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
           str(ROOT / "tests" / "dropin" / "dropin_main.cpp"), "-L", str(ROOT / "aicortex_b200"), "-laicortex_b200",
           "-L", "/usr/local/cuda/lib64", "-lcudart", "-o", str(exe)]
    subprocess.run(cmd, check=True)
    assert exe.exists()
