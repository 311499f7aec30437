"""Tensor parallelism on 2 GPUs.

One process per GPU (sg_init_rank, as bench.py under torchrun uses it):
column-split (Q/K/V/gate/up style) and row-split (O/down style) linears at
decode and prefill batch sizes, through the device entry points (and the
one with no device allocation) and the host-pointer ones (ordinary and
page-locked host rows), against the CPU oracle; row split with SG_FLAG_ACCUMULATE on
a replicated y (the residual stream). Then the tensor-parallel decoder
(llamanyon.rs_b200/decoder.py, stacked=False) against the oracle's engine
loop, and one configs[4]-width layer (d 8192, FFN 28672, Q4_0).

One process driving both GPUs (sg_init(2), ncclCommInitAll), as the
single-process Rust engine would: column and row split through sg_linear.

The one-process-per-GPU linears run on both all-reduce paths: the default
peer kernel over NVLink (sg_peer.cuh) and ncclAllReduce (SG_PEER_ALLREDUCE=0);
the decoder and the configs[4]-width layer on the default. sg_init(2) always
uses NCCL. Skipped below 2 GPUs (ranks whose collectives wait for one another
must each have their own GPU).
"""
import json
import os
import socket
import sys

import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
Q40, Q4K = 2, 12
SMALL = dict(n_layers=2, d=512, n_heads=8, n_kv_heads=2, ffn=1024, vocab=1000, context_len=64, max_seq=64)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _paths():
    for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "llamanyon.rs_b200"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)


def _rank(rank, world, port, outdir, part, path="peer"):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    _paths()
    if path == "nccl":
        os.environ["SG_PEER_ALLREDUCE"] = "0"
    else:
        os.environ.pop("SG_PEER_ALLREDUCE", None)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import swamp_gpu as sg
    import oracle
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    g = sg.SwampGpu()
    out = {"checks": []}
    try:
        uid = g.get_unique_id() if rank == 0 else bytes(128)
        t = torch.frombuffer(bytearray(uid), dtype=torch.uint8).cuda()
        dist.broadcast(t, 0)
        g.init_rank(rank, world, bytes(t.cpu().numpy().tobytes()), rank)
        out["path"] = g.allreduce_path()
        if part == "linears":
            _linears(g, sg, oracle, torch, rank, world, out)
        else:
            _decoder(g, sg, oracle, torch, dist, rank, world, out, part)
        g.synchronize()
        torch.cuda.synchronize()
    finally:
        dist.barrier()
        g.shutdown()
        dist.barrier()
        dist.destroy_process_group()
    with open(os.path.join(outdir, f"out{rank}.json"), "w") as f:
        json.dump(out, f)


def _gate(out, name, y, ref, l2):
    out["checks"].append([name, reference_gate(y, ref, l2)])


def _linears(g, sg, oracle, torch, rank, world, out):
    st = torch.cuda.Stream()
    for dtype in (Q40, Q4K):
        nr, k = 1000, 2048
        w = oracle.gen_weight(dtype, SEED, 80 + dtype, nr, k)
        for b in (1, 16, 40):
            x = oracle.gen_x(SEED, 81 + b, (b, k))
            ref, l2 = reference_outputs(oracle, dtype, w, x, nr, k)
            # column split: this rank's rows
            W = g.register(w, dtype, nr, k, sg.SG_TP_COLUMN)
            r0, rows, _, _ = g.tp_shard(dtype, nr, k, sg.SG_TP_COLUMN, world, rank)
            xd = torch.from_numpy(x).cuda()
            yd = torch.full((b, rows + 3), float("nan"), device="cuda")
            with torch.cuda.stream(st):
                g.linear_device(W, xd.data_ptr(), k, yd.data_ptr(), rows + 3, b, stream=st.cuda_stream)
            st.synchronize()
            g.synchronize()
            assert torch.isnan(yd[:, rows:]).all()
            _gate(out, f"column dt{dtype} b{b} device", yd[:, :rows].cpu().numpy(), ref[:, r0:r0 + rows],
                  l2[:, r0:r0 + rows])
            yh = g.linear(W, x)  # host pointers: this rank's rows of the whole output
            _gate(out, f"column dt{dtype} b{b} host", yh[:, r0:r0 + rows], ref[:, r0:r0 + rows], l2[:, r0:r0 + rows])
            # page-locked rows: x and this rank's rows of out move by DMA
            xp = g.host_array((b, k))
            xp[:] = x
            yp = g.host_array((b, nr))
            yp[:] = np.nan
            g.linear(W, xp, out=yp)
            assert np.isnan(yp[:, :r0]).all() and np.isnan(yp[:, r0 + rows:]).all()
            _gate(out, f"column dt{dtype} b{b} pinned", yp[:, r0:r0 + rows], ref[:, r0:r0 + rows],
                  l2[:, r0:r0 + rows])
            W.free()
            # row split: this rank's K slice, all-reduced outputs
            W = g.register(w, dtype, nr, k, sg.SG_TP_ROW)
            _, _, c0, nc = g.tp_shard(dtype, nr, k, sg.SG_TP_ROW, world, rank)
            xs = torch.from_numpy(np.ascontiguousarray(x[:, c0:c0 + nc])).cuda()
            yd = torch.full((b, nr), float("nan"), device="cuda")
            with torch.cuda.stream(st):
                g.linear_device(W, xs.data_ptr(), nc, yd.data_ptr(), nr, b, stream=st.cuda_stream)
            st.synchronize()
            g.synchronize()
            _gate(out, f"row dt{dtype} b{b} device", yd.cpu().numpy(), ref, l2)
            if b <= 16:  # the entry point with no device allocation, same all-reduce
                yd = torch.full((b, nr), float("nan"), device="cuda")
                with torch.cuda.stream(st):
                    g.linear_device_noalloc(W, xs.data_ptr(), nc, yd.data_ptr(), nr, b, stream=st.cuda_stream)
                st.synchronize()
                g.synchronize()
                _gate(out, f"row dt{dtype} b{b} noalloc", yd.cpu().numpy(), ref, l2)
            # row split onto a replicated y (the residual stream): y0 counted once
            y0 = np.linspace(-2, 2, b * nr).astype(np.float32).reshape(b, nr)
            yd = torch.from_numpy(y0.copy()).cuda()
            with torch.cuda.stream(st):
                g.linear_device(W, xs.data_ptr(), nc, yd.data_ptr(), nr, b, stream=st.cuda_stream,
                                flags=sg.SG_FLAG_ACCUMULATE)
            st.synchronize()
            g.synchronize()
            _gate(out, f"row+acc dt{dtype} b{b} device", yd.cpu().numpy() - y0, ref, l2)
            yh = g.linear(W, x)
            _gate(out, f"row dt{dtype} b{b} host", yh, ref, l2)
            yp[:] = np.nan
            g.linear(W, xp, out=yp)
            _gate(out, f"row dt{dtype} b{b} pinned", yp, ref, l2)
            W.free()


def _decoder(g, sg, oracle, torch, dist, rank, world, out, part):
    import decoder as dec
    from test_decoder import OracleModel
    if part == "decoder":
        cases = [(dtype, SMALL, 2, 9, 3) for dtype in (Q40, Q4K)]
    else:  # one configs[4]-width layer
        cases = [(Q40, dict(n_layers=1, d=8192, n_heads=64, n_kv_heads=8, ffn=28672, vocab=512, context_len=64,
                            max_seq=64), 1, 3, 2)]
    for dtype, cfgd, n_seqs, plen, n_new in cases:
        cfg = dec.DecoderConfig(dtype=dtype, **cfgd)
        model = dec.SynthModel(g, cfg, SEED, stacked=False)
        D = dec.Decoder(g, model, n_seqs=n_seqs, max_rows=n_seqs * plen)
        rng = np.random.default_rng(SEED + 3)
        prompts = rng.integers(0, cfg.vocab, size=(n_seqs, plen))
        logs = []
        rows = D.set_rows(prompts.reshape(-1), np.tile(np.arange(plen), n_seqs), np.repeat(np.arange(n_seqs), plen))
        D.forward(rows, prefill=(n_seqs, plen, plen, 1))
        torch.cuda.synchronize()
        g.synchronize()
        logs.append(D.logits[:rows].cpu().numpy())
        # feed the device's own picks back; the oracle follows the same tokens
        cur = [int(t) for t in D.next[:rows].cpu().numpy().reshape(n_seqs, plen)[:, -1]]
        toks = [list(cur)]
        for step in range(n_new):
            D.set_rows(cur, [plen + step] * n_seqs, list(range(n_seqs)))
            D.forward(n_seqs, decode=True)
            torch.cuda.synchronize()
            g.synchronize()
            logs.append(D.logits[:n_seqs].cpu().numpy())
            cur = [int(t) for t in D.next[:n_seqs].cpu().numpy()]
            toks.append(list(cur))
        D.free()
        model.free()
        if rank == 0:
            refs = [OracleModel(oracle, cfg, SEED) for _ in range(n_seqs)]
            worst = 0.0
            for s in range(n_seqs):
                for t in range(plen):
                    ref, _ = refs[s].step(int(prompts[s, t]), t)
                    got = logs[0][s * plen + t]
                    worst = max(worst, float(np.abs(got - ref).max()) / float(np.abs(ref).max()))
            for step in range(n_new):
                for s in range(n_seqs):
                    ref, _ = refs[s].step(toks[step][s], plen + step)
                    got = logs[step + 1][s]
                    worst = max(worst, float(np.abs(got - ref).max()) / float(np.abs(ref).max()))
            out["checks"].append([f"decoder dt{dtype} d{cfg.d} tp{world}", worst])


def _spawn(tmp_path, part, path="peer"):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (one per rank)")
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), part, path), nprocs=2, join=True,
                       start_method="spawn")
    return [json.load(open(tmp_path / f"out{r}.json")) for r in range(2)]


@pytest.mark.gpu
@pytest.mark.parametrize("path", ["peer", "nccl"])
def test_tp_linears_two_ranks(tmp_path, path):
    outs = _spawn(tmp_path, "linears", path)
    for o in outs:
        assert o["path"] == path
        names = [c[0] for c in o["checks"]]
        # 5 checks per (dtype, batch), 2 with page-locked host rows, the
        # no-allocation entry point at batch 1 and 16
        assert len(names) == 2 * 3 * 7 + 2 * 2
        assert max(c[1] for c in o["checks"]) <= 1e-3


@pytest.mark.gpu
def test_tp_decoder_two_ranks(tmp_path):
    """Logits of the TP2 decoder within 2e-3 * max |logit| of the oracle's
    engine loop at every prefill position and decode step."""
    outs = _spawn(tmp_path, "decoder")
    checks = outs[0]["checks"]
    assert len(checks) == 2
    assert max(c[1] for c in checks) <= 2e-3, checks


@pytest.mark.gpu
def test_tp_configs4_width_layer_two_ranks(tmp_path):
    """One d=8192 / FFN 28672 Q4_0 layer at TP2 against the oracle."""
    outs = _spawn(tmp_path, "wide")
    checks = outs[0]["checks"]
    assert len(checks) == 1
    assert checks[0][1] <= 2e-3, checks


def _single_process(outdir):
    _paths()
    import swamp_gpu as sg
    import oracle
    g = sg.SwampGpu()
    g.init(2)
    out = {"checks": []}
    try:
        for dtype in (Q40, Q4K):
            nr, k = 700, 1024
            w = oracle.gen_weight(dtype, SEED, 90 + dtype, nr, k)
            for b in (1, 16, 40):
                x = oracle.gen_x(SEED, 91 + b, (b, k))
                ref, l2 = reference_outputs(oracle, dtype, w, x, nr, k)
                for mode, name in ((sg.SG_TP_COLUMN, "column"), (sg.SG_TP_ROW, "row")):
                    W = g.register(w, dtype, nr, k, mode)
                    _gate(out, f"{name} dt{dtype} b{b}", g.linear(W, x), ref, l2)
                    W.free()
        g.synchronize()
    finally:
        g.shutdown()
    with open(os.path.join(outdir, "single.json"), "w") as f:
        json.dump(out, f)


@pytest.mark.gpu
def test_tp_single_process_two_gpus(tmp_path):
    """sg_init(2): one process drives both GPUs (NCCL communicator from
    ncclCommInitAll, grouped all-reduce), host-pointer calls."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    p = mp.get_context("spawn").Process(target=_single_process, args=(str(tmp_path),))
    p.start()
    p.join(600)
    assert p.exitcode == 0
    out = json.load(open(tmp_path / "single.json"))
    assert len(out["checks"]) == 2 * 3 * 2
    assert max(c[1] for c in out["checks"]) <= 1e-3
