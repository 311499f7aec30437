"""A device-resident decoder forward over the C ABI of libswamp_gpu.so.

Host-side mirror of swamp-engine's inference loop (executor.rs:403-550 for
one decode step, executor.rs:48-190 for the batched prompt prefill) in which
every tensor stays in GPU memory: the embedding row, RMSNorm, the quantized
Q/K/V, O, gate/up and down linears, RoPE with the KV-cache store, attention,
SiLU-mul, the residual adds (folded into the O and down linears with
SG_FLAG_ACCUMULATE), the final norm, the output head and the greedy pick.
A Rust engine makes the same calls through the FFI; torch here only owns
device buffers and streams.

Rows are query tokens: one per sequence in a decode step, all prompt
positions in a prefill. Each row carries (token, position, sequence) in
device int32 arrays, so a step captured in a CUDA graph replays with new
positions. Several sequences share the batch (the benchmark's batch 8) with
their own KV-cache slots.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import swamp_gpu as sg

ROLES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


@dataclass
class DecoderConfig:
    """Llama-style architecture (swamp-engine/src/model.rs config fields)."""
    n_layers: int
    d: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    dtype: int = sg.SG_DTYPE_Q4_K
    eps: float = 1e-5          # executor.rs:272
    context_len: int = 2048    # RoPE table length (ops.rs:20, executor.rs:207)
    max_seq: int = 2048        # KV-cache positions (executor.rs:320)

    @property
    def head_dim(self) -> int:
        return self.d // self.n_heads

    def shape(self, role: str):
        """(n_rows N, n_cols K) of a linear (shape[1], shape[0] in GGUF)."""
        kv = self.n_kv_heads * self.head_dim
        return {"attn_q": (self.d, self.d), "attn_k": (kv, self.d), "attn_v": (kv, self.d),
                "attn_output": (self.d, self.d), "ffn_gate": (self.ffn, self.d), "ffn_up": (self.ffn, self.d),
                "ffn_down": (self.d, self.ffn), "output": (self.vocab, self.d),
                "token_embd": (self.vocab, self.d)}[role]


def tensor_id(role: str, layer: int = -1) -> int:
    """Synthetic-generator id of a model tensor (weights and norm vectors)."""
    if layer < 0:
        return {"token_embd": 1, "output": 2, "output_norm": 3}[role]
    names = ROLES + ("attn_norm", "ffn_norm")
    return 1000 * (layer + 1) + names.index(role)


def norm_vector(gpu: sg.SwampGpu, seed: int, tid: int, n: int) -> np.ndarray:
    """Synthetic RMSNorm weight: 1 + 0.1 * N(0,1), rounded to f32."""
    return (1.0 + 0.1 * gpu.synth_x(seed, tid, (n,)).astype(np.float64)).astype(np.float32)


class SynthModel:
    """Random-init weights of the architecture, generated on the device.

    Single GPU (stacked=True): Q, K and V of a layer are registered as one
    tensor of d + 2 * kv rows (their GGUF rows one after the other), and gate
    and up as one of 2 * ffn rows: each pair of projections that reads the
    same x is one linear call, one prefill GEMM instead of three or two. The
    values are exactly those of the separate tensors.

    Tensor parallel (stacked=False, the job's world from gpu.topology()):
    Q, K, V, gate and up are column-split (each rank holds its heads' rows and
    its FFN slice, generated on the device from the same seeds, so the model
    is the same at every degree) and called as one multi-tensor linear; O and
    down are row-split over the same head / FFN slices, their partial sums
    all-reduced into the replicated residual stream (executor.rs:436-505 with
    the layout of linear.rs:31-45 generalised to ranks)."""

    def __init__(self, gpu: sg.SwampGpu, cfg: DecoderConfig, seed: int, stacked: bool = True):
        import torch
        self.cfg, self.seed = cfg, seed
        _, self.world, _ = gpu.topology()
        self.stacked = stacked and self.world == 1
        W = self.world
        if cfg.n_heads % W or cfg.n_kv_heads % W or cfg.ffn % W:
            raise ValueError(f"heads {cfg.n_heads}/{cfg.n_kv_heads} and ffn {cfg.ffn} must split over {W} ranks")
        self.layers = []
        for l in range(cfg.n_layers):
            def stacked_t(roles):
                blocks = [gpu.synth_blocks(cfg.dtype, seed, tensor_id(r, l), *cfg.shape(r)) for r in roles]
                rows = sum(cfg.shape(r)[0] for r in roles)
                return gpu.register(np.concatenate(blocks), cfg.dtype, rows, cfg.d)

            def synth(role, mode):
                return gpu.synth_weight(cfg.dtype, seed, tensor_id(role, l), *cfg.shape(role), mode)
            if self.stacked:
                self.layers.append({
                    "qkv": stacked_t(("attn_q", "attn_k", "attn_v")),
                    "attn_output": synth("attn_output", sg.SG_TP_REPLICATE),
                    "gate_up": stacked_t(("ffn_gate", "ffn_up")),
                    "ffn_down": synth("ffn_down", sg.SG_TP_REPLICATE),
                })
            else:
                self.layers.append({
                    "q": synth("attn_q", sg.SG_TP_COLUMN), "k": synth("attn_k", sg.SG_TP_COLUMN),
                    "v": synth("attn_v", sg.SG_TP_COLUMN),
                    "attn_output": synth("attn_output", sg.SG_TP_ROW),
                    "gate": synth("ffn_gate", sg.SG_TP_COLUMN), "up": synth("ffn_up", sg.SG_TP_COLUMN),
                    "ffn_down": synth("ffn_down", sg.SG_TP_ROW),
                })
        self.token_embd = gpu.synth_weight(cfg.dtype, seed, tensor_id("token_embd"), *cfg.shape("token_embd"))
        self.output = gpu.synth_weight(cfg.dtype, seed, tensor_id("output"), *cfg.shape("output"))
        dev = torch.device("cuda")
        self.attn_norm = torch.from_numpy(np.stack(
            [norm_vector(gpu, seed, tensor_id("attn_norm", l), cfg.d) for l in range(cfg.n_layers)])).to(dev)
        self.ffn_norm = torch.from_numpy(np.stack(
            [norm_vector(gpu, seed, tensor_id("ffn_norm", l), cfg.d) for l in range(cfg.n_layers)])).to(dev)
        self.output_norm = torch.from_numpy(norm_vector(gpu, seed, tensor_id("output_norm"), cfg.d)).to(dev)

    def weight_bytes(self) -> int:
        """GGUF bytes of every quantized tensor one decode step reads on one
        rank (the layers' shards and the replicated output head; the
        embedding table contributes one row per token, not counted)."""
        c = self.cfg
        tot = sum(sg.row_bytes(c.dtype, c.shape(r)[1]) * c.shape(r)[0] for r in ROLES) * c.n_layers // self.world
        return tot + sg.row_bytes(c.dtype, c.d) * c.vocab

    def free(self):
        for lw in self.layers:
            for w in lw.values():
                w.free()
        self.token_embd.free()
        self.output.free()


class Decoder:
    """Buffers and the forward pass for up to max_rows query rows."""

    def __init__(self, gpu: sg.SwampGpu, model: SynthModel, n_seqs: int, max_rows: int,
                 fuse_norm: bool = False, fuse_silu: bool = True):
        """fuse_norm / fuse_silu: RMSNorm / SiLU-mul run inside the following
        linear's operand build (sg_rmsnorm_linear_multi_device /
        sg_silu_mul_linear_device, the same rows as the separate calls);
        False runs the engine's two calls. Measured on configs[3] at batch 1:
        the SiLU fusion saves 1.4% of a decode step, the RMSNorm fusion costs
        0.7% (each prep CTA re-reads its token's row for the norm), so only
        the former is on by default."""
        import torch
        self.torch = torch
        self.fuse_norm, self.fuse_silu = fuse_norm, fuse_silu
        self.gpu, self.m, self.cfg = gpu, model, model.cfg
        self.ops = sg.LayerOps(gpu)
        c = self.cfg
        W = model.world
        # this rank's heads, KV heads and FFN slice
        self.n_heads, self.n_kv, self.ffn = c.n_heads // W, c.n_kv_heads // W, c.ffn // W
        self.rope = sg.Rope(gpu, c.head_dim, c.context_len)
        self.cache = sg.KvCache(gpu, c.n_layers, self.n_kv, c.head_dim, c.max_seq, n_seqs)
        self.max_rows = max_rows
        dev = torch.device("cuda")
        f = dict(device=dev, dtype=torch.float32)
        dq, kv = self.n_heads * c.head_dim, self.n_kv * c.head_dim
        self.dq = dq
        self.x = torch.zeros(max_rows, c.d, **f)
        self.xn = torch.zeros(max_rows, c.d, **f)
        self.qkv = torch.zeros(max_rows, dq + 2 * kv, **f)  # [q | k | v] per row
        self.q, self.k, self.v = self.qkv[:, :dq], self.qkv[:, dq:dq + kv], self.qkv[:, dq + kv:]
        self.att = torch.zeros(max_rows, dq, **f)
        self.gu = torch.zeros(max_rows, 2 * self.ffn, **f)  # [gate | up] per row
        self.gate, self.up = self.gu[:, :self.ffn], self.gu[:, self.ffn:]
        self.logits = torch.zeros(max_rows, c.vocab, **f)
        i32 = dict(device=dev, dtype=torch.int32)
        self.tokens = torch.zeros(max_rows, **i32)
        self.pos = torch.zeros(max_rows, **i32)
        self.seq = torch.zeros(max_rows, **i32)
        self.next = torch.zeros(max_rows, **i32)

    def set_rows(self, tokens, pos, seq):
        """Copy a batch's (token, position, sequence) rows to the device."""
        n = len(tokens)
        assert n <= self.max_rows
        t = self.torch
        self.tokens[:n].copy_(t.as_tensor(np.asarray(tokens, np.int32)))
        self.pos[:n].copy_(t.as_tensor(np.asarray(pos, np.int32)))
        self.seq[:n].copy_(t.as_tensor(np.asarray(seq, np.int32)))
        return n

    def forward(self, rows: int, stream: int | None = None, logits_rows: slice | None = None,
                decode: bool = False, prefill: tuple | None = None):
        """One forward pass of `rows` rows: logits (and the greedy pick in
        `next`) for the rows in logits_rows (default: all). decode=True for
        a step of one row per sequence: RoPE, the cache store and attention
        then run as one kernel per layer. prefill=(n_seqs, n_tokens,
        row_stride_seq, row_stride_pos) for a prompt pass whose rows are
        positions 0..n_tokens-1 of sequences 0..n_seqs-1 at those row
        strides: attention then serves blocks of positions per CTA."""
        use_pf = prefill is not None and self.cfg.head_dim in (64, 128)
        c, o, g = self.cfg, self.ops, self.gpu
        p = lambda t: t.data_ptr()
        D, DQ, KV, F = c.d, self.dq, self.n_kv * c.head_dim, self.ffn
        H = self.n_heads
        LQ, LG = DQ + 2 * KV, 2 * F  # row strides of [q | k | v] and [gate | up]
        ACC = sg.SG_FLAG_ACCUMULATE
        o.embed(self.m.token_embd, p(self.tokens), rows, p(self.x), D, stream)
        def norm_linear(norm, ws, ys, ld):
            """ys = W rmsnorm(x): fused (the norm runs inside the GEMV's operand
            build) or as the engine's two calls."""
            if self.fuse_norm:
                g.rmsnorm_linear_multi_device(ws, p(self.x), D, p(norm), c.eps, ys, [ld] * len(ws), rows,
                                              stream=stream)
            else:
                o.rmsnorm(p(self.x), D, p(norm), p(self.xn), D, D, rows, c.eps, stream)
                g.linear_multi_device(ws, p(self.xn), D, ys, [ld] * len(ws), rows, stream=stream)

        for l, lw in enumerate(self.m.layers):
            if self.m.stacked:
                norm_linear(self.m.attn_norm[l], [lw["qkv"]], [p(self.qkv)], LQ)
            else:
                norm_linear(self.m.attn_norm[l], [lw["q"], lw["k"], lw["v"]], [p(self.q), p(self.k), p(self.v)], LQ)
            if decode:
                o.rope_attention(self.rope, self.cache, l, p(self.q), LQ, p(self.k), LQ, p(self.v), LQ, p(self.att),
                                 DQ, p(self.pos), p(self.seq), rows, H, stream)
            else:
                o.rope_kv(self.rope, self.cache, l, p(self.q), LQ, p(self.k), LQ, p(self.v), LQ, p(self.pos),
                          p(self.seq), rows, H, stream)
                if use_pf:
                    o.attention_prefill(self.cache, l, p(self.q), LQ, p(self.att), DQ, *prefill, H, stream)
                else:
                    o.attention(self.cache, l, p(self.q), LQ, p(self.att), DQ, p(self.pos), None, p(self.seq), rows,
                                H, stream)
            # O: row-split over this rank's heads; the all-reduce adds every
            # rank's part (and the residual, once) into x
            g.linear_device(lw["attn_output"], p(self.att), DQ, p(self.x), D, rows, stream=stream, flags=ACC)
            if self.m.stacked:
                norm_linear(self.m.ffn_norm[l], [lw["gate_up"]], [p(self.gu)], LG)
            else:
                norm_linear(self.m.ffn_norm[l], [lw["gate"], lw["up"]], [p(self.gate), p(self.up)], LG)
            if self.fuse_silu:
                g.silu_mul_linear_device(lw["ffn_down"], p(self.gate), LG, p(self.up), LG, p(self.x), D, rows,
                                         stream=stream, flags=ACC)
            else:
                o.silu_mul(p(self.gate), LG, p(self.up), LG, F, rows, stream)
                g.linear_device(lw["ffn_down"], p(self.gate), LG, p(self.x), D, rows, stream=stream, flags=ACC)
        r0, r1 = (0, rows) if logits_rows is None else (logits_rows.start, logits_rows.stop)
        n = r1 - r0
        o.rmsnorm(p(self.x[r0]), D, p(self.m.output_norm), p(self.xn), D, D, n, c.eps, stream)
        g.linear_device(self.m.output, p(self.xn), D, p(self.logits), c.vocab, n, stream=stream)
        o.argmax(p(self.logits), c.vocab, c.vocab, n, p(self.next), stream)
        return n

    def advance(self, rows: int):
        """Greedy decoding: the next step's token is this step's pick, one
        position further (torch ops on the current stream)."""
        self.tokens[:rows].copy_(self.next[:rows])
        self.pos[:rows].add_(1)

    def free(self):
        self.rope.free()
        self.cache.free()


def main(argv=None):
    """Greedy generation with a random-init Llama-3-8B-shaped Q4_K model:
    python llamanyon.rs_b200/decoder.py --layers 32 --batch 1 --prompt 512 --new 16
    (one eager prefill pass, then eager decode steps; prints the device time
    per decode step and the first sequence's tokens)."""
    import argparse
    import time

    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--new", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0x5EED1A11)
    a = ap.parse_args(argv)
    gpu = sg.SwampGpu()
    gpu.init(1)
    cfg = DecoderConfig(n_layers=a.layers, d=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=128256,
                        max_seq=max(2048, a.prompt + a.new))
    model = SynthModel(gpu, cfg, a.seed)
    B, P = a.batch, a.prompt
    D = Decoder(gpu, model, n_seqs=B, max_rows=B * P)
    prompts = np.random.default_rng(a.seed).integers(0, cfg.vocab, size=(B, P))
    # rows in (position, sequence) order: the last B rows are the last position
    rows = D.set_rows(prompts.T.reshape(-1), np.repeat(np.arange(P), B), np.tile(np.arange(B), P))
    D.forward(rows, logits_rows=slice(rows - B, rows), prefill=(B, P, 1, B))
    out = [D.next[:B].cpu().tolist()]
    D.tokens[:B].copy_(D.next[:B])
    D.pos[:B].fill_(P)
    D.seq[:B].copy_(torch.arange(B, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(a.new - 1):
        D.forward(B, decode=True)
        D.advance(B)
        out.append(D.tokens[:B].cpu().tolist())
    torch.cuda.synchronize()
    gpu.synchronize()
    el = time.perf_counter() - t0
    print(f"decode: {el * 1e3 / max(1, a.new - 1):.3f} ms per step (eager, host-launched), "
          f"sequence 0: {[t[0] for t in out]}")
    D.free()
    model.free()
    gpu.shutdown()
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
