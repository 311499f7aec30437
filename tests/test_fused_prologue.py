"""RMSNorm and SiLU-mul run inside the decode GEMV's operand build
(sg_rmsnorm_linear_multi_device, sg_silu_mul_linear_device) against the
separate calls (sg_rmsnorm_device / sg_silu_mul_device, then the linear) and
against the oracle's engine sequence (swamp-engine ops.rs:188-214 rmsnorm,
silu and mul_in_place, then forward_linear, linear.rs:14-90).

The fused rows equal the separate op's bit for bit (same arithmetic, and
RMSNorm's summation order replayed), but the GEMV adds the rows that several
CTAs share with atomic adds in any order, so two runs may differ in the last
bits: fused and separate outputs are compared to 1e-6 of the output scale,
and both to the oracle with the parity gate. Batches above the decode range
(40) take the unfused route inside the library.
"""
import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

pytestmark = pytest.mark.gpu
Q40, Q4K = 2, 12
EPS = 1e-5


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _close(a, b):
    scale = float(np.abs(b).max()) + 1e-30
    assert float(np.abs(a - b).max()) <= 1e-6 * scale


@pytest.mark.parametrize("batch", [1, 3, 16, 32, 40])
@pytest.mark.parametrize("dtype,k", [(Q40, 4096), (Q40, 2080), (Q4K, 4096), (Q4K, 1280)])
def test_rmsnorm_linear_multi(gpu, oracle, dtype, k, batch):
    import torch
    import swamp_gpu as sg
    ops = sg.LayerOps(gpu)
    rows = (600, 136)
    raws = [oracle.gen_weight(dtype, SEED, 700 + i, n, k) for i, n in enumerate(rows)]
    Ws = [gpu.register(w, dtype, n, k) for w, n in zip(raws, rows)]
    try:
        x = oracle.gen_x(SEED, 710 + batch, (batch, k)) * np.float32(3)
        nw = (1 + 0.1 * oracle.gen_x(SEED, 711, (k,))).astype(np.float32)
        xd, nwd = _t(x), _t(nw)
        fused = [torch.full((batch, n), float("nan"), device="cuda") for n in rows]
        gpu.rmsnorm_linear_multi_device(Ws, xd.data_ptr(), k, nwd.data_ptr(), EPS, [t.data_ptr() for t in fused],
                                        list(rows), batch)
        xn = torch.empty_like(xd)
        ops.rmsnorm(xd.data_ptr(), k, nwd.data_ptr(), xn.data_ptr(), k, k, batch, EPS)
        sep = [torch.empty(batch, n, device="cuda") for n in rows]
        gpu.linear_multi_device(Ws, xn.data_ptr(), k, [t.data_ptr() for t in sep], list(rows), batch)
        torch.cuda.synchronize()
        gpu.synchronize()
        assert torch.equal(xd.cpu(), torch.from_numpy(x))  # x is not modified
        xn_ref = np.stack([oracle.rmsnorm(x[b], nw, EPS) for b in range(batch)])
        for w, n, f, s in zip(raws, rows, fused, sep):
            f, s = f.cpu().numpy(), s.cpu().numpy()
            _close(f, s)
            ref, l2 = reference_outputs(oracle, dtype, w, xn_ref, n, k)
            reference_gate(f, ref, l2)
    finally:
        for W in Ws:
            W.free()


@pytest.mark.parametrize("batch", [1, 2, 9, 32, 40])
@pytest.mark.parametrize("dtype,k", [(Q40, 11008), (Q4K, 14336), (Q40, 96)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_silu_mul_linear(gpu, oracle, dtype, k, batch, accumulate):
    import torch
    import swamp_gpu as sg
    ops = sg.LayerOps(gpu)
    n = 520
    raw = oracle.gen_weight(dtype, SEED, 720, n, k)
    W = gpu.register(raw, dtype, n, k)
    try:
        ld = k + 8  # strided rows, like the [gate | up] buffer
        gu = np.zeros((batch, 2 * ld), np.float32)
        gu[:, :k] = oracle.gen_x(SEED, 721 + batch, (batch, k)) * np.float32(2)
        gu[:, ld:ld + k] = oracle.gen_x(SEED, 722 + batch, (batch, k))
        gud = _t(gu)
        g_ptr, u_ptr = gud.data_ptr(), gud.data_ptr() + ld * 4
        y0 = oracle.gen_x(SEED, 723, (batch, n))
        flags = sg.SG_FLAG_ACCUMULATE if accumulate else 0
        fused = _t(y0) if accumulate else torch.full((batch, n), float("nan"), device="cuda")
        gpu.silu_mul_linear_device(W, g_ptr, 2 * ld, u_ptr, 2 * ld, fused.data_ptr(), n, batch, flags=flags)
        torch.cuda.synchronize()
        assert torch.equal(gud.cpu(), torch.from_numpy(gu))  # g and u are not modified
        g2 = gud.clone()
        ops.silu_mul(g2.data_ptr(), 2 * ld, g2.data_ptr() + ld * 4, 2 * ld, k, batch)
        sep = _t(y0) if accumulate else torch.empty(batch, n, device="cuda")
        gpu.linear_device(W, g2.data_ptr(), 2 * ld, sep.data_ptr(), n, batch, flags=flags)
        torch.cuda.synchronize()
        gpu.synchronize()
        f, s = fused.cpu().numpy(), sep.cpu().numpy()
        _close(f, s)
        h = np.stack([oracle.silu_mul(gu[b, :k], gu[b, ld:ld + k]) for b in range(batch)])
        ref, l2 = reference_outputs(oracle, dtype, raw, h, n, k)
        if accumulate:
            ref = ref + y0
        reference_gate(f, ref, l2 + (np.abs(y0) if accumulate else 0))
    finally:
        W.free()


def test_bad_arguments(gpu, oracle):
    import torch
    import swamp_gpu as sg
    k = 256
    W = gpu.register(oracle.gen_weight(Q4K, SEED, 730, 8, k), Q4K, 8, k)
    try:
        x = torch.zeros(1, k, device="cuda")
        y = torch.zeros(1, 8, device="cuda")
        with pytest.raises(sg.SwampGpuError):
            gpu.rmsnorm_linear_multi_device([W], x.data_ptr(), k, 0, EPS, [y.data_ptr()], [8], 1)
        with pytest.raises(sg.SwampGpuError):
            gpu.silu_mul_linear_device(W, x.data_ptr(), k, 0, k, y.data_ptr(), 8, 1)
        with pytest.raises(sg.SwampGpuError):
            gpu.silu_mul_linear_device(W, x.data_ptr(), k, x.data_ptr(), k - 1, y.data_ptr(), 8, 1)
    finally:
        W.free()
