"""A bounded device wait that runs out, on 2 GPUs as 2 processes.

The peer all-reduce (sg_allreduce_device with SG_PEER_ALLREDUCE=1) waits on
flags that the other rank raises. Here rank 1 skips one call on the host,
between steps, with nothing of its own in flight: rank 0's kernel waits for
a flag that nothing sets. With SG_WAIT_NS=50 ms in the environment the wait
gives up, the kernel records the error and returns, and rank 0's
sg_synchronize reports SG_ERR_DEVICE_FAULT instead of the GPU hanging. Both
ranks then shut down and initialise again (their epoch counters no longer
agree), and a clean call gives exact sums. No GPU is faulted, trapped or
hung: the failure is made on the host, and NVLS is off.

Skipped below 2 GPUs: ranks whose kernels wait for one another must each
have their own GPU.
"""
import json
import os
import socket
import sys
import time

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SG_ERR_DEVICE_FAULT = -7


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    sys.path.insert(0, os.path.join(ROOT, "llamanyon.rs_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), SG_PEER_ALLREDUCE="1",
                      SG_WAIT_NS="50000000", NCCL_NVLS_ENABLE="0")
    import swamp_gpu as sg
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    g = sg.SwampGpu()
    out = {}

    def init():
        ids = [g.get_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, 0)
        g.init_rank(rank, world, ids[0], rank)

    def exact_call(n, rep):
        buf = torch.full((n,), float(rank + 1 + rep), device="cuda")
        g.allreduce_device(buf.data_ptr(), n)
        g.synchronize()
        return bool(torch.all(buf == float(sum(r + 1 + rep for r in range(world)))))

    n = 4096
    init()
    out["path"] = g.allreduce_path()
    out["before"] = exact_call(n, 0)
    dist.barrier()
    # rank 1 skips this step on the host; rank 0's wait for its flag runs out
    if rank == 0:
        buf = torch.ones(n, device="cuda")
        t0 = time.perf_counter()
        g.allreduce_device(buf.data_ptr(), n)
        try:
            g.synchronize()
            out["code"] = 0
        except sg.SwampGpuError as e:
            out["code"] = e.code
            out["message"] = str(e)
        out["seconds"] = time.perf_counter() - t0
    dist.barrier()
    g.shutdown()
    dist.barrier()
    init()
    out["after"] = exact_call(n, 1) and exact_call(n, 2)
    g.synchronize()
    dist.barrier()
    g.shutdown()
    dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(outdir, f"w{rank}.json"), "w") as f:
        json.dump(out, f)


@pytest.mark.gpu
def test_peer_wait_runs_out_and_recovers(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (one per rank)")
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    o0 = json.load(open(tmp_path / "w0.json"))
    o1 = json.load(open(tmp_path / "w1.json"))
    assert o0["path"] == "peer" and o1["path"] == "peer"
    assert o0["before"] and o1["before"]
    assert o0["code"] == SG_ERR_DEVICE_FAULT, o0
    assert o0["seconds"] < 10.0  # the 50 ms limit, not the built-in 4 s
    assert o0["after"] and o1["after"]
