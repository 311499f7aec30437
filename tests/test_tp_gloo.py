"""Tensor-parallel host logic on CPU: the library's shard plan (sg_tp_shard,
the same function sg_weight_register uses) and the column/row decomposition
of forward_linear over world_size-2 gloo ranks.

Column split (Q/K/V/gate/up) gives each rank a run of output rows; row split
(O/down) gives each rank whole blocks of every row and sums the partial
outputs with an all-reduce. Each rank computes its slice with the oracle (the
reference's CPU route) on exactly the bytes the library would upload to its
GPU; the gathered / reduced result must pass the parity gate against the
untouched tensor (tensor-parallel parity: the same values up to the f32 sum order)."""
import os
import socket
import sys

import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
Q40, Q4K = 2, 12
COL, ROW = 1, 2


def _lib():
    sys.path.insert(0, os.path.join(ROOT, "llamanyon.rs_b200"))
    import swamp_gpu as sg
    try:
        return sg.SwampGpu()
    except sg.SwampGpuError as e:
        pytest.skip(f"library not built: {e}")


@pytest.mark.parametrize("dtype,n,k", [(Q40, 4096, 4096), (Q40, 4096, 11008), (Q40, 11008, 4096),
                                       (Q4K, 14336, 4096), (Q4K, 4096, 14336), (Q40, 8192, 28672),
                                       (Q4K, 1024, 4096), (Q40, 7, 96)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_plan_partitions(dtype, n, k, world):
    """Every mode's slices are disjoint, cover the tensor, and cut on whole blocks."""
    lib = _lib()
    bs = 32 if dtype == Q40 else 256
    for mode in (0, COL, ROW):
        if mode == ROW and k // bs < world or mode == COL and n < world:
            continue
        rows_seen, cols_seen = [], []
        for r in range(world):
            r0, nr, c0, nc = lib.tp_shard(dtype, n, k, mode, world, r)
            assert nr > 0 and nc > 0
            assert c0 % bs == 0 and nc % bs == 0
            rows_seen.append((r0, nr))
            cols_seen.append((c0, nc))
        if mode == COL:
            assert rows_seen[0][0] == 0 and sum(x[1] for x in rows_seen) == n
            assert all(a[0] + a[1] == b[0] for a, b in zip(rows_seen, rows_seen[1:]))
            assert all(c == (0, k) for c in cols_seen)
        elif mode == ROW:
            assert cols_seen[0][0] == 0 and sum(x[1] for x in cols_seen) == k
            assert all(a[0] + a[1] == b[0] for a, b in zip(cols_seen, cols_seen[1:]))
            assert all(r == (0, n) for r in rows_seen)
        else:
            assert all(r == (0, n) for r in rows_seen) and all(c == (0, k) for c in cols_seen)


def test_shard_plan_rejects():
    import swamp_gpu as sg
    lib = _lib()
    bad = [
        (Q40, 64, 64, ROW, 4, 0),    # 2 blocks < 4 ranks
        (Q40, 3, 64, COL, 4, 0),     # 3 rows < 4 ranks
        (Q40, 64, 48, 0, 1, 0),      # K not a block multiple
        (Q4K, 64, 512, 3, 2, 0),     # bad mode
        (Q40, 64, 64, COL, 2, 2),    # rank out of range
        (8, 64, 64, 0, 1, 0),        # Q8_0: not on this path
    ]
    for args in bad:
        with pytest.raises(sg.SwampGpuError):
            lib.tp_shard(*args)


def _slice_rows(w, dtype, n, k, r0, nr):
    rb = (k // (32 if dtype == Q40 else 256)) * (18 if dtype == Q40 else 144)
    return np.ascontiguousarray(w.reshape(n, rb)[r0:r0 + nr]).reshape(-1)


def _slice_cols(w, dtype, n, k, c0, nc):
    bs, bb = (32, 18) if dtype == Q40 else (256, 144)
    rb = (k // bs) * bb
    return np.ascontiguousarray(w.reshape(n, rb)[:, c0 // bs * bb:(c0 + nc) // bs * bb]).reshape(-1)


def _rank_main(rank, world, port, dtype, n, k, mode, outdir):
    import torch.distributed as dist
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, HERE)
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = _lib()
        w = oracle.gen_weight(dtype, SEED, 40 + mode, n, k, n_threads=1)
        x = oracle.gen_x(SEED, 41, (k,))
        r0, nr, c0, nc = lib.tp_shard(dtype, n, k, mode, world, rank)
        if mode == COL:
            part = oracle.forward_linear(dtype, _slice_rows(w, dtype, n, k, r0, nr), x, nr, k, 1)
            parts = [None] * world
            dist.all_gather_object(parts, (r0, part))
            y = np.zeros(n, np.float32)
            for a, p in parts:
                y[a:a + len(p)] = p
        else:
            part = oracle.forward_linear(dtype, _slice_cols(w, dtype, n, k, c0, nc), x[c0:c0 + nc], n, nc, 1)
            t = torch.from_numpy(part.copy())
            dist.all_reduce(t)
            y = t.numpy()
        if rank == 0:
            np.save(os.path.join(outdir, "y.npy"), y)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("dtype,n,k,mode", [(Q40, 256, 1024, COL), (Q40, 256, 1024, ROW),
                                            (Q4K, 192, 1024, COL), (Q4K, 192, 1024, ROW),
                                            (Q40, 130, 352, ROW)])
def test_tp_world2_gloo(tmp_path, oracle, dtype, n, k, mode):
    import torch.multiprocessing as mp
    _lib()
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), dtype, n, k, mode, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    y = np.load(tmp_path / "y.npy")
    w = oracle.gen_weight(dtype, SEED, 40 + mode, n, k, n_threads=1)
    x = oracle.gen_x(SEED, 41, (k,))
    ref, l2 = reference_outputs(oracle, dtype, w, x, n, k)
    reference_gate(y, ref[0], l2[0])
    if mode == COL:  # row slices are computed exactly as the whole tensor's rows
        assert np.array_equal(y, oracle.forward_linear(dtype, w, x, n, k, 1))
