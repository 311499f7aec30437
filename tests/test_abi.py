"""CPU tests of the drop-in boundary: the library builds for sm_100a, loads,
exports every symbol include/swamp_gpu.h declares, and validates arguments on
the host before touching a device (no compute calls here)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "swamp_gpu.h")


@pytest.fixture(scope="module")
def lib():
    import build_lib
    import swamp_gpu
    build_lib.build()
    return swamp_gpu.load_library()


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"SG_API\s+(?:const\s+char\s*\*\s*|int\s+)(sg_\w+)\s*\(", src)))


def test_header_declares_the_expected_api():
    import swamp_gpu
    assert declared_symbols() == sorted(swamp_gpu.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    so = os.path.join(ROOT, "llamanyon.rs_b200", "libswamp_gpu.so")
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (sg_\w+)", out))
    for sym in declared_symbols():
        assert sym in exported, sym
        assert getattr(lib, sym) is not None


def test_library_is_built_for_sm100a():
    import build_lib
    flags = " ".join(build_lib.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags and "-lineinfo" in flags


def test_header_compiles_as_c():
    src = '#include "swamp_gpu.h"\nint main(void){ sg_weight_t w = 0; (void)w; return SG_OK; }\n'
    path = "/tmp/sg_header_check.c"
    open(path, "w").write(src)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-c", path,
                    "-o", "/tmp/sg_header_check.o"], check=True)


def test_calls_before_init_are_rejected_on_the_host(lib):
    import swamp_gpu
    assert lib.sg_linear(None, None, None, 1, 0) == swamp_gpu.SG_OK - 6  # SG_ERR_NOT_INITIALIZED
    assert b"sg_init" in lib.sg_last_error()
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 144)()
    assert lib.sg_weight_register(buf, 12, 1, 256, 0, ctypes.byref(h)) == -6
    assert lib.sg_dequant_f32(None, None, 0) == -6
    assert lib.sg_fused_gemv_q4k(None, None, None, 1, 256) == -1  # null pointers (fused_gemv_q4k.rs:808)
    assert lib.sg_fused_gemv_q4k(buf, buf, buf, 1, 100) == -1     # n_cols % 256 (fused_gemv_q4k.rs:811)


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="host has a GPU")
def test_no_cpu_fallback_without_gpu(lib):
    """sg_init must fail loudly when no sm_100 device exists."""
    rc = lib.sg_init(1)
    assert rc != 0
    msg = lib.sg_last_error().decode()
    assert "CPU fallback" in msg or "CUDA" in msg or "device" in msg


def test_host_alloc_argument_checks(lib):
    """sg_host_alloc: a null out pointer is rejected, zero bytes give NULL
    with no CUDA call, and freeing NULL is a no-op."""
    assert lib.sg_host_alloc(16, None) == -1
    p = ctypes.c_void_p(1)
    assert lib.sg_host_alloc(0, ctypes.byref(p)) == 0 and p.value is None
    assert lib.sg_host_free(None) == 0


def test_binding_checks_output_arrays_on_the_host(lib):
    """linear / linear_multi reject an output array of the wrong shape,
    dtype or row layout (and a wrong count) before calling the library."""
    import numpy as np
    import swamp_gpu as sg
    g = sg.SwampGpu()
    W = sg.Weight(g, None, 12, 8, 256, 0)
    x = np.zeros((2, 256), np.float32)
    for bad in (np.zeros((2, 9), np.float32), np.zeros((2, 8), np.float64), np.zeros((8, 2), np.float32).T):
        with pytest.raises(sg.SwampGpuError) as e:
            g.linear(W, x, out=bad)
        assert e.value.code == -1
    with pytest.raises(sg.SwampGpuError) as e:
        g.linear_multi([W, W], x[0], outs=[np.zeros(8, np.float32)])
    assert e.value.code == -1
    with pytest.raises(sg.SwampGpuError) as e:  # a valid call reaches the library, which rejects the handle
        g.linear(W, x, out=np.zeros((2, 8), np.float32))
    assert e.value.code in (-6, -1)  # not initialised, or (after an init in this process) a null handle
