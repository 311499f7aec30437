import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "llamanyon.rs_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

SEED = 0x5EED1A11


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA path through the C ABI")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    orc.build()
    return orc


@pytest.fixture(scope="session")
def gpu():
    """The library on cuda:0. A GPU test without a usable GPU fails (no fallback)."""
    import swamp_gpu
    import build_lib as libbuild
    libbuild.build()
    lib = swamp_gpu.SwampGpu()
    lib.init(1)
    yield lib
    lib.shutdown()


PARITY_LOG = []  # (test, gated worst ratio, strict max, strict 99.9th percentile, share of strict > 1e-3, elements)


def reference_gate(y, ref, l2dot, rtol=1e-3):
    """Per-element parity bound used by every GEMV/GEMM test:

        |y - ref| <= rtol * max(|ref|, ||w_r .* x_b||_2)

    ref is the reference's f32 result (scalar Q4_K kernel / engine Q4_0
    route); ||w.*x||_2 is the natural magnitude of the dot product (a sum of
    K terms of random sign has |ref| of about that size), so elements whose
    true value cancels to ~0 are judged against the scale of their terms
    instead of an arbitrarily small |ref|. Returns the worst ratio.

    Beside it the north star's strict metric, max |y - ref| / |ref| per
    element (ref != 0), is recorded with its 99.9th percentile and the share
    of elements above rtol; the session summary prints them per test."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = np.maximum(np.abs(ref), np.asarray(l2dot, np.float64))
    denom = np.where(denom == 0, 1.0, denom)
    ratio = np.abs(y - ref) / denom
    worst = float(ratio.max()) if ratio.size else 0.0
    nz = ref != 0
    strict = np.abs(y - ref)[nz] / np.abs(ref)[nz]
    if strict.size:
        PARITY_LOG.append((os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0], worst, float(strict.max()),
                           float(np.quantile(strict, 0.999)), float(np.mean(strict > rtol)), int(strict.size)))
    assert np.all(np.isfinite(y)), "non-finite outputs"
    assert worst <= rtol, f"parity bound exceeded: max |y-ref|/max(|ref|,||w.*x||) = {worst:.3e} > {rtol}"
    return worst


def pytest_terminal_summary(terminalreporter):
    if not PARITY_LOG:
        return
    tr = terminalreporter
    tr.section("parity: gated bound and the strict per-element relative error")
    tr.write_line(f"{'test':<90} {'gate':>9} {'strict max':>11} {'strict p99.9':>12} {'>1e-3':>8} {'elements':>9}")
    for name, worst, smax, sq, frac, n in PARITY_LOG:
        tr.write_line(f"{name[-90:]:<90} {worst:9.2e} {smax:11.2e} {sq:12.2e} {frac:8.1e} {n:9d}")
    allmax = max(r[1] for r in PARITY_LOG)
    tr.write_line(f"worst gated ratio over {len(PARITY_LOG)} checks: {allmax:.3e}")


def reference_outputs(orc, dtype, w, x, n_rows, n_cols):
    """(ref f32 [B,N], l2dot [B,N]) from the oracle."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    ref = orc.reference_linear(dtype, w, x, n_rows, n_cols)
    l2 = np.stack([orc.gemv_f64(dtype, w, x[b], n_rows, n_cols)[2] for b in range(x.shape[0])])
    return ref, l2


def reference_outputs_batch(orc, dtype, w, x, n_rows, n_cols):
    """reference_outputs for whole full-size tensors, in seconds: ref is the
    engine's batched route (forward_linear_batch, linear.rs:176-239) on all
    host threads -- for Q4_0 the same dequantized-row dots as the per-token
    route, bit for bit; for Q4_K fused_gemv_q4k_batched's scalar order
    (fused_gemv_q4k.rs:650-698), the kernel the reference runs at prefill --
    and ||w.*x||_2 comes from the dequantized rows in f64 with numpy."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    ref = orc.forward_linear_batch(dtype, w, x, n_rows, n_cols, os.cpu_count() or 1)
    W = orc.dequantize(dtype, w, n_rows * n_cols).reshape(n_rows, n_cols)
    x2 = x.astype(np.float64) ** 2
    l2 = np.empty((x.shape[0], n_rows))
    for r0 in range(0, n_rows, 2048):
        wc = W[r0:r0 + 2048].astype(np.float64)
        l2[:, r0:r0 + 2048] = np.sqrt(x2 @ (wc * wc).T)
    return ref, l2
