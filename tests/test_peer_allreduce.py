"""The row-split all-reduce over NVLink peer memory (sg_allreduce_device, used
by every row-split linear in one-process-per-GPU mode; the one-shot and the
two-shot kernel) against exact sums and NCCL, on 2 GPUs as 2 processes.
Skipped when fewer than 2 GPUs are visible: ranks whose kernels wait for one
another must each have their own GPU.

Exactness: the inputs are small integers, so every order of summation gives
the same float and the result must equal the integer sum exactly.
"""
import os
import socket
import sys

import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
COUNTS = (1, 3, 2048, 2049, 8192 + 4, 4096 * 8, (1 << 19), (1 << 19) + 16)  # the last above the peer cap: NCCL


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, outdir, two_shot="0"):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "llamanyon.rs_b200"), HERE):
        sys.path.insert(0, p)
    import swamp_gpu as sg
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), SG_PEER_ALLREDUCE="1",
                      SG_AR_TWO_SHOT=two_shot)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    g = sg.SwampGpu()
    out = {}
    try:
        uid = g.get_unique_id() if rank == 0 else bytes(128)
        t = torch.frombuffer(bytearray(uid), dtype=torch.uint8).cuda()
        dist.broadcast(t, 0)
        g.init_rank(rank, world, bytes(t.cpu().numpy().tobytes()), rank)
        out["path"] = g.allreduce_path()
        st = torch.cuda.Stream()
        # 1. exact integer sums, repeated (epoch and slot parity cycling)
        ok = True
        for rep in range(3):
            for n in COUNTS:
                base = torch.arange(n, device="cuda", dtype=torch.float32).remainder_(1000)
                buf = base * (rank + 1) + rep
                with torch.cuda.stream(st):
                    g.allreduce_device(buf.data_ptr(), n, st.cuda_stream)
                st.synchronize()
                want = base * sum(r + 1 for r in range(world)) + rep * world
                ok = ok and bool(torch.equal(buf, want))
        out["exact"] = ok
        # 2. a CUDA graph replayed with new data each time
        n = 40960
        buf = torch.zeros(n, device="cuda")
        with torch.cuda.stream(st):
            g.allreduce_device(buf.data_ptr(), n, st.cuda_stream)  # first use outside capture
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                g.allreduce_device(buf.data_ptr(), n, st.cuda_stream)
            gok = True
            for rep in range(7):
                buf.fill_(float(rank * 10 + rep))
                graph.replay()
                st.synchronize()
                gok = gok and bool(torch.all(buf == float(sum(r * 10 + rep for r in range(world)))))
            del graph
        out["graph"] = gok
        # 3. row-split linears through the device entry point, against the oracle
        errs = []
        for dtype, nr, k, b in ((2, 4096, 11008, 1), (12, 4096, 14336, 4), (12, 1000, 2048, 40)):
            w = oracle.gen_weight(dtype, SEED, 70 + b, nr, k)
            x = oracle.gen_x(SEED, 71 + b, (b, k))
            W = g.register(w, dtype, nr, k, sg.SG_TP_ROW)
            _, _, c0, nc = g.tp_shard(dtype, nr, k, sg.SG_TP_ROW, world, rank)
            xd = torch.from_numpy(np.ascontiguousarray(x[:, c0:c0 + nc])).cuda()
            yd = torch.full((b, nr), float("nan"), device="cuda")
            with torch.cuda.stream(st):
                g.linear_device(W, xd.data_ptr(), nc, yd.data_ptr(), nr, b, stream=st.cuda_stream)
            st.synchronize()
            g.synchronize()
            if rank == 0:
                ref, l2 = reference_outputs(oracle, dtype, w, x, nr, k)
                errs.append(reference_gate(yd.cpu().numpy(), ref, l2))
            W.free()
        out["linear_worst"] = max(errs) if errs else 0.0
        g.synchronize()
        torch.cuda.synchronize()
    finally:
        dist.barrier()  # no rank frees its receive buffer while a peer may still use it
        g.shutdown()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        import json
        with open(os.path.join(outdir, "out.json"), "w") as f:
            json.dump(out, f)


@pytest.mark.gpu
@pytest.mark.parametrize("two_shot", ["0", "1"])
def test_peer_allreduce_two_gpus(tmp_path, two_shot):
    """two_shot "1" (SG_AR_TWO_SHOT=1) sends every call through the
    reduce-scatter + all-gather kernel, which by default only large vectors
    on 4 or more ranks take."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (one per rank)")
    import json
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), two_shot), nprocs=2, join=True,
                       start_method="spawn")
    out = json.load(open(tmp_path / "out.json"))
    assert out["path"] == "peer"
    assert out["exact"] and out["graph"]
    assert out["linear_worst"] <= 1e-3
