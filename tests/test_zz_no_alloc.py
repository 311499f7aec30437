"""sg_linear_device_noalloc through the C ABI: same results as
sg_linear_device and within the parity bound of the oracle's restatement of
the reference, two calls in a row, prefill batches rejected with a clear
error, and no device memory taken by the calls themselves.

Collected last (file name) so it also runs after every other GPU test; it
needs nothing from them and passes alone."""
import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

pytestmark = pytest.mark.gpu

Q40, Q4K = 2, 12
SG_ERR_UNSUPPORTED = -5


@pytest.mark.parametrize("dtype,n,k,batch", [(Q40, 300, 4096, 1), (Q40, 200, 11008, 4), (Q4K, 256, 4096, 16),
                                             (Q4K, 130, 14336, 3), (Q40, 64, 16384, 8),
                                             (Q4K, 40, 32768 + 256, 2)])
def test_noalloc_matches_device_entry(gpu, oracle, dtype, n, k, batch):
    torch = pytest.importorskip("torch")
    w = oracle.gen_weight(dtype, SEED, 90, n, k)
    W = gpu.register(w, dtype, n, k)
    try:
        x = torch.from_numpy(oracle.gen_x(SEED, 91, (batch, k))).cuda()
        y_ref = torch.empty(batch, n, device="cuda")
        gpu.linear_device(W, x.data_ptr(), k, y_ref.data_ptr(), n, batch)
        torch.cuda.synchronize()
        ref = y_ref.cpu().numpy()
        scale = np.abs(ref).max() + 1e-30
        x_host = x.cpu().numpy()
        orc, l2 = reference_outputs(oracle, dtype, w, x_host, n, k)
        for _ in range(2):  # two calls in a row on the shared scratch
            y = torch.full((batch, n), float("nan"), device="cuda")
            gpu.linear_device_noalloc(W, x.data_ptr(), k, y.data_ptr(), n, batch)
            torch.cuda.synchronize()
            got = y.cpu().numpy()
            assert np.all(np.isfinite(got))
            assert np.max(np.abs(got - ref)) <= 1e-6 * scale
            reference_gate(got, orc, l2)
    finally:
        W.free()


def test_noalloc_takes_no_device_memory(gpu, oracle):
    torch = pytest.importorskip("torch")
    n, k, batch = 512, 4096, 4
    W = gpu.register(oracle.gen_weight(Q40, SEED, 92, n, k), Q40, n, k)
    try:
        x = torch.from_numpy(oracle.gen_x(SEED, 93, (batch, k))).cuda()
        y = torch.empty(batch, n, device="cuda")
        gpu.linear_device_noalloc(W, x.data_ptr(), k, y.data_ptr(), n, batch)  # first call: one-time setup
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(5):
            gpu.linear_device_noalloc(W, x.data_ptr(), k, y.data_ptr(), n, batch)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0
    finally:
        W.free()


def test_noalloc_rejects_wide_tensor_at_batch_16(gpu, oracle):
    """From 3 tokens on the fixed workspace holds activation images (32768
    columns at 16 tokens); a wider tensor is refused with the limit in the
    message, while batch 2 (no images) still runs."""
    torch = pytest.importorskip("torch")
    import swamp_gpu as sg
    k = 32768 + 256
    W = gpu.register(oracle.gen_weight(Q4K, SEED, 95, 8, k), Q4K, 8, k)
    try:
        x = torch.zeros(16, k, device="cuda")
        y = torch.zeros(16, 8, device="cuda")
        with pytest.raises(sg.SwampGpuError) as e:
            gpu.linear_device_noalloc(W, x.data_ptr(), k, y.data_ptr(), 8, 16)
        assert e.value.code == SG_ERR_UNSUPPORTED and "32768" in str(e.value)
        gpu.linear_device_noalloc(W, x.data_ptr(), k, y.data_ptr(), 8, 2)
        torch.cuda.synchronize()
        assert torch.all(y[:2] == 0)
    finally:
        W.free()


def test_noalloc_rejects_prefill_batch(gpu, oracle):
    torch = pytest.importorskip("torch")
    import swamp_gpu as sg
    k = 4096
    W = gpu.register(oracle.gen_weight(Q4K, SEED, 94, 8, k), Q4K, 8, k)
    try:
        x17 = torch.zeros(17, k, device="cuda")
        y17 = torch.zeros(17, 8, device="cuda")
        with pytest.raises(sg.SwampGpuError) as e:
            gpu.linear_device_noalloc(W, x17.data_ptr(), k, y17.data_ptr(), 8, 17)
        assert e.value.code == SG_ERR_UNSUPPORTED and "1..16" in str(e.value)
    finally:
        W.free()
