"""A whole decoder on the device (llamanyon.rs_b200/decoder.py) against the
oracle's restatement of swamp-engine's inference loop (executor.rs:403-550:
embed, per layer rmsnorm, Q/K/V, RoPE, cache save, attention, O + residual,
rmsnorm, gate/up, SiLU-mul, down + residual; final rmsnorm, output head,
greedy pick).

Tolerance: logits within 2e-3 * max |logit| of the oracle's; the greedy
token must agree wherever the oracle's top two logits differ by more than
1e-2 * max |logit| (closer calls are within the tolerance either way). The
oracle's tokens are fed back to both sides so that the sequences stay
aligned.
"""
import numpy as np
import pytest

from conftest import SEED

CFG = dict(n_layers=2, d=256, n_heads=4, n_kv_heads=2, ffn=512, vocab=1000, context_len=64, max_seq=64)


class OracleModel:
    """The reference forward on the host, one token at a time."""

    def __init__(self, oracle, cfg, seed):
        from decoder import ROLES, tensor_id
        self.o, self.c = oracle, cfg
        gen = lambda role, l=-1: oracle.gen_weight(cfg.dtype, seed, tensor_id(role, l), *cfg.shape(role))
        self.w = [{r: gen(r, l) for r in ROLES} for l in range(cfg.n_layers)]
        self.out_w = gen("output")
        emb = gen("token_embd")
        self.embd = oracle.dequantize(cfg.dtype, emb, cfg.vocab * cfg.d).reshape(cfg.vocab, cfg.d)
        nv = lambda tid: (1.0 + 0.1 * oracle.gen_x(seed, tid, (cfg.d,)).astype(np.float64)).astype(np.float32)
        self.attn_norm = [nv(tensor_id("attn_norm", l)) for l in range(cfg.n_layers)]
        self.ffn_norm = [nv(tensor_id("ffn_norm", l)) for l in range(cfg.n_layers)]
        self.output_norm = nv(tensor_id("output_norm"))
        self.lut = oracle.rope_lut(cfg.head_dim, cfg.context_len)
        hd, nkv = cfg.head_dim, cfg.n_kv_heads
        self.kc = np.zeros((cfg.n_layers, nkv, cfg.max_seq, hd), np.float32)
        self.vc = np.zeros_like(self.kc)

    def lin(self, role, layer, x):
        c = self.c
        n, k = c.shape(role)
        w = self.out_w if role == "output" else self.w[layer][role]
        return self.o.forward_linear(c.dtype, w, x, n, k, 4)

    def step(self, tok, pos):
        o, c = self.o, self.c
        hd = c.head_dim
        x = self.embd[tok].copy()
        for l in range(c.n_layers):
            xn = o.rmsnorm(x, self.attn_norm[l], c.eps)
            q, k, v = self.lin("attn_q", l, xn), self.lin("attn_k", l, xn), self.lin("attn_v", l, xn)
            q, k = o.rope_apply(q, k, pos, c.n_heads, c.n_kv_heads, hd, c.context_len, self.lut)
            self.kc[l, :, pos] = k.reshape(c.n_kv_heads, hd)
            self.vc[l, :, pos] = v.reshape(c.n_kv_heads, hd)
            att = o.attention(q, self.kc[l], self.vc[l], pos + 1, pos, c.n_heads, c.n_kv_heads, hd)
            x = o.add(x, self.lin("attn_output", l, att))
            xn = o.rmsnorm(x, self.ffn_norm[l], c.eps)
            g = o.silu_mul(self.lin("ffn_gate", l, xn), self.lin("ffn_up", l, xn))
            x = o.add(x, self.lin("ffn_down", l, g))
        xn = o.rmsnorm(x, self.output_norm, c.eps)
        logits = self.lin("output", -1, xn)
        return logits, o.argmax(logits)


def _check_logits(got, ref, tok_got, tok_ref):
    scale = float(np.abs(ref).max())
    err = float(np.abs(got - ref).max())
    assert err <= 2e-3 * scale, (err, scale)
    top = np.sort(ref)[-2:]
    if top[1] - top[0] > 1e-2 * scale:
        assert tok_got == tok_ref


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [12, 2])
def test_decoder_prefill_then_greedy_decode(gpu, oracle, dtype):
    import torch
    import decoder as dec
    cfg = dec.DecoderConfig(dtype=dtype, **CFG)
    model = dec.SynthModel(gpu, cfg, SEED)
    n_seqs, plen, n_new = 2, 18, 4  # 36 prefill rows: the prefill GEMM; then 2-row decode GEMVs
    D = dec.Decoder(gpu, model, n_seqs=n_seqs, max_rows=n_seqs * plen)
    try:
        rng = np.random.default_rng(SEED)
        prompts = rng.integers(0, cfg.vocab, size=(n_seqs, plen))
        refs = [OracleModel(oracle, cfg, SEED) for _ in range(n_seqs)]
        rows = D.set_rows(prompts.reshape(-1), np.tile(np.arange(plen), n_seqs), np.repeat(np.arange(n_seqs), plen))
        D.forward(rows, prefill=(n_seqs, plen, plen, 1))  # rows in (sequence, position) order
        torch.cuda.synchronize()
        gpu.synchronize()
        logits = D.logits[:rows].cpu().numpy()
        picks = D.next[:rows].cpu().numpy()
        cur = []
        for s in range(n_seqs):
            for t in range(plen):
                ref, tok = refs[s].step(int(prompts[s, t]), t)
                r = s * plen + t
                _check_logits(logits[r], ref, int(picks[r]), tok)
            cur.append(tok)
        for step in range(n_new):
            pos = plen + step
            D.set_rows(cur, [pos] * n_seqs, list(range(n_seqs)))
            D.forward(n_seqs, decode=True)  # one row per sequence: the fused decode attention
            torch.cuda.synchronize()
            gpu.synchronize()
            logits = D.logits[:n_seqs].cpu().numpy()
            picks = D.next[:n_seqs].cpu().numpy()
            nxt = []
            for s in range(n_seqs):
                ref, tok = refs[s].step(cur[s], pos)
                _check_logits(logits[s], ref, int(picks[s]), tok)
                nxt.append(tok)
            cur = nxt
    finally:
        D.free()
        model.free()


@pytest.mark.gpu
def test_decoder_graph_replay_matches_eager(gpu, oracle):
    """A decode step captured in a CUDA graph (fused decode attention),
    replayed with the device-side advance (token <- pick, position + 1),
    gives the eager two-call steps' tokens."""
    import torch
    import decoder as dec
    cfg = dec.DecoderConfig(**CFG)
    model = dec.SynthModel(gpu, cfg, SEED)
    D = dec.Decoder(gpu, model, n_seqs=2, max_rows=2)
    try:
        def run(graph):
            D.set_rows([5, 900], [0, 0], [0, 1])
            out = []
            if not graph:
                for _ in range(6):
                    D.forward(2)
                    out.append(D.next[:2].cpu().tolist())
                    D.advance(2)
                return out
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                D.forward(2, stream=st.cuda_stream, decode=True)  # eager first use (workspaces)
                D.set_rows([5, 900], [0, 0], [0, 1])
                st.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st):
                    D.forward(2, stream=st.cuda_stream, decode=True)
                    D.advance(2)
                for _ in range(6):
                    g.replay()
                    st.synchronize()
                    out.append([int(t) for t in D.tokens[:2].cpu().tolist()])
            return out
        eager = run(False)
        graph = run(True)
        assert graph == eager
    finally:
        D.free()
        model.free()


# configs[3]'s layer at full width (Llama-3-8B: d 4096, 32 query / 8 KV heads
# of 128, FFN 14336, Q4_K), one layer and a small vocabulary.
CFG3_LAYER = dict(n_layers=1, d=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=512, context_len=64, max_seq=64)


class WideOracleModel(OracleModel):
    """OracleModel with forward_linear on every host thread (the row split
    leaves each row's result unchanged)."""

    def lin(self, role, layer, x):
        import os
        c = self.c
        n, k = c.shape(role)
        w = self.out_w if role == "output" else self.w[layer][role]
        return self.o.forward_linear(c.dtype, w, x, n, k, os.cpu_count() or 4)


@pytest.mark.gpu
def test_decoder_configs3_full_width_layer(gpu, oracle):
    """One configs[3]-width layer: a 40-row prefill (2 sequences of 20, the
    prefill GEMM) and 3 two-row decode steps (the decode GEMV and fused decode
    attention), logits and greedy tokens against the oracle's engine loop."""
    import torch
    import decoder as dec
    cfg = dec.DecoderConfig(dtype=12, **CFG3_LAYER)
    model = dec.SynthModel(gpu, cfg, SEED)
    n_seqs, plen, n_new = 2, 20, 3
    D = dec.Decoder(gpu, model, n_seqs=n_seqs, max_rows=n_seqs * plen)
    try:
        rng = np.random.default_rng(SEED + 3)
        prompts = rng.integers(0, cfg.vocab, size=(n_seqs, plen))
        refs = [WideOracleModel(oracle, cfg, SEED) for _ in range(n_seqs)]
        rows = D.set_rows(prompts.reshape(-1), np.tile(np.arange(plen), n_seqs), np.repeat(np.arange(n_seqs), plen))
        D.forward(rows, prefill=(n_seqs, plen, plen, 1))
        torch.cuda.synchronize()
        gpu.synchronize()
        logits = D.logits[:rows].cpu().numpy()
        picks = D.next[:rows].cpu().numpy()
        cur = []
        for s in range(n_seqs):
            for t in range(plen):
                ref, tok = refs[s].step(int(prompts[s, t]), t)
                _check_logits(logits[s * plen + t], ref, int(picks[s * plen + t]), tok)
            cur.append(tok)
        for step in range(n_new):
            pos = plen + step
            D.set_rows(cur, [pos] * n_seqs, list(range(n_seqs)))
            D.forward(n_seqs, decode=True)
            torch.cuda.synchronize()
            gpu.synchronize()
            logits = D.logits[:n_seqs].cpu().numpy()
            picks = D.next[:n_seqs].cpu().numpy()
            nxt = []
            for s in range(n_seqs):
                ref, tok = refs[s].step(cur[s], pos)
                _check_logits(logits[s], ref, int(picks[s]), tok)
                nxt.append(tok)
            cur = nxt
    finally:
        D.free()
        model.free()
