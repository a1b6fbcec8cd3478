"""Minimal tensor-parallel Qwen3 decoder that drives the attention hot path in
context (config 5: Qwen3-32B greedy decode after an 8192-token prompt).

This is the caller of the path, not a product of its own: the projections,
norms and MLP are plain torch / cuBLAS, the collectives are NCCL; the fused
Q/K RMSNorm + RoPE + KV write and the prefill / decode attention are this
library's kernels, called exactly where the reference engine calls its cuTile
kernels (src/model.rs:4031-4219 prefill ops, 3494-3790 decode graph).

Layout (Megatron-style, TP = world size):
  - QKV and gate/up projections column-parallel (local heads, local
    intermediate), o_proj and down_proj row-parallel, each followed by an
    NCCL all-reduce (sum) of [tokens, hidden];
  - embedding replicated, lm_head vocab-parallel: each rank takes the argmax
    of its vocab slice and the (max, index) pairs are all-gathered;
  - per-layer KV cache [H_kv/TP][max_seq][128] (the reference layout, local
    heads); decode position in device memory, incremented inside the graph.
Weights are random N(0, 0.02) (norm weights 1 + N(0, 0.02)); there is no
checkpoint in this environment.
"""
import math
import time
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import attn


@dataclass
class Qwen3Shape:
    layers: int = 64
    hidden: int = 5120
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 25600
    vocab: int = 151936
    eps: float = 1e-6
    theta: float = 1.0e6


def _rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


class Qwen3TP:
    def __init__(self, shape, max_seq, rank=0, world=1, group=None, device=None, seed=6,
                 fused_allreduce=True):
        self.c = c = shape
        self.rank, self.world, self.group = rank, world, group
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        assert c.heads % world == 0 and c.kv_heads % world == 0 and c.inter % world == 0
        self.hq, self.hkv, self.it = c.heads // world, c.kv_heads // world, c.inter // world
        self.vshard = (c.vocab + world - 1) // world
        self.max_seq = max_seq
        g = torch.Generator(device=self.dev).manual_seed(seed * 1000 + rank)
        D, H = c.head_dim, c.hidden

        def w(*shape):
            return (torch.randn(*shape, device=self.dev, generator=g) * 0.02).half()

        def nw(n):
            return (1.0 + 0.02 * torch.randn(n, device=self.dev, generator=g)).half()

        self.embed = w(c.vocab, H) if rank == 0 else torch.empty(c.vocab, H, device=self.dev, dtype=torch.float16)
        if world > 1:
            torch.distributed.broadcast(self.embed, 0, group=group)
        self.lm_head = w(self.vshard, H)
        self.final_norm = nw(H)
        self.layers = []
        for _ in range(c.layers):
            L = dict(
                in_norm=nw(H), post_norm=nw(H), q_norm=nw(D), k_norm=nw(D),
                w_qkv=w((self.hq + 2 * self.hkv) * D, H),
                w_o=w(H, self.hq * D),
                w_gu=w(2 * self.it, H),
                w_down=w(H, self.it),
                k_cache=torch.zeros(self.hkv, max_seq, D, device=self.dev, dtype=torch.float16),
                v_cache=torch.zeros(self.hkv, max_seq, D, device=self.dev, dtype=torch.float16),
            )
            self.layers.append(L)
        self.rope = attn.rope_table(c.theta, max_seq, self.dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.tok = torch.zeros(1, dtype=torch.int64, device=self.dev)
        nks = attn.decode_workspace_bytes(1, max_seq, self.hq, self.hkv, max_seq)
        self.ws = torch.empty(max(16, nks), dtype=torch.uint8, device=self.dev)
        # Decode o_proj / down_proj (TP > 1), the faster of each measured on
        # B200 at TP = 2: o_proj as one grout kernel (GEMV + all-reduce over
        # NVLink peer memory + residual), down_proj as a cuBLAS GEMV followed
        # by the grout all-reduce + residual.  NCCL when disabled.
        self.comm = None
        if fused_allreduce and world > 1:
            from .tp import TPComm
            self.comm = TPComm(rank, world, H, group, self.dev)
        # decode-step buffers (fixed addresses for graph replay)
        self.q1 = torch.empty(1, self.hq, D, device=self.dev, dtype=torch.float16)
        self.o1 = torch.empty_like(self.q1)

    # ---------------------------------------------------------------- helpers
    def _allreduce(self, x):
        if self.world > 1:
            torch.distributed.all_reduce(x, group=self.group)
        return x

    def _argmax(self, x):
        logits = F.linear(x, self.lm_head).float()           # [1, vshard]
        v, i = logits.max(-1)
        i = i + self.rank * self.vshard
        if self.world > 1:
            pair = torch.stack([v, i.float()], -1).reshape(-1)    # [2]
            allp = torch.empty(2 * self.world, device=self.dev, dtype=torch.float32)
            torch.distributed.all_gather_into_tensor(allp, pair, group=self.group)
            allp = allp.view(self.world, 2)
            best = allp[:, 0].argmax().view(1)
            return allp[:, 1].gather(0, best).long()
        return i.view(1)

    # ---------------------------------------------------------------- prefill
    def prefill(self, tokens):
        """Run the prompt (eager, like the reference's StepGraph prefill):
        returns the first generated token id (device tensor [1])."""
        c, D = self.c, self.c.head_dim
        S = tokens.numel()
        x = self.embed[tokens]                                   # [S, H]
        for L in self.layers:
            h = _rms(x, L["in_norm"], c.eps)
            qkv = F.linear(h, L["w_qkv"])                        # [S, (hq+2hkv)*D]
            q = qkv[:, : self.hq * D].reshape(S, self.hq, D).contiguous()
            k = qkv[:, self.hq * D:(self.hq + self.hkv) * D].reshape(S, self.hkv, D).contiguous()
            v = qkv[:, (self.hq + self.hkv) * D:].reshape(S, self.hkv, D).contiguous()
            q_out = torch.empty_like(q)
            attn.qk_norm_rope_kv_prefill(q, k, v, L["q_norm"], L["k_norm"], self.rope, q_out,
                                         L["k_cache"], L["v_cache"], 0, c.eps)
            o = torch.empty_like(q_out)
            attn.attention_prefill(q_out, L["k_cache"], L["v_cache"], o, 0)
            x = x + self._allreduce(F.linear(o.view(S, -1), L["w_o"]))
            h = _rms(x, L["post_norm"], c.eps)
            gu = F.linear(h, L["w_gu"])
            a = F.silu(gu[:, : self.it]) * gu[:, self.it:]
            x = x + self._allreduce(F.linear(a, L["w_down"]))
        h = _rms(x[-1:], self.final_norm, c.eps)
        self.pos.fill_(S)
        self.tok.copy_(self._argmax(h))
        return self.tok

    # ---------------------------------------------------------------- decode
    def _decode_layers(self, x, attention_only=False):
        c, D = self.c, self.c.head_dim
        for L in self.layers:
            h = _rms(x, L["in_norm"], c.eps) if not attention_only else x
            qkv = F.linear(h, L["w_qkv"]) if not attention_only else self._qkv_dummy
            attn.qk_norm_rope_kv_decode(qkv, L["q_norm"], L["k_norm"], self.rope, self.q1,
                                        L["k_cache"], L["v_cache"], self.pos, self.hq, self.hkv,
                                        c.eps)
            attn.attention_decode(self.q1, L["k_cache"], L["v_cache"], self.pos, self.o1,
                                  self.max_seq, workspace=self.ws)
            if attention_only:
                continue
            if self.comm is not None:
                # o_proj: GEMV + all-reduce + residual in one grout kernel
                x1 = torch.empty_like(x)
                self.comm.gemv_allreduce(L["w_o"], self.o1, x1, residual=x)
                x = x1
            else:
                x = x + self._allreduce(F.linear(self.o1.view(1, -1), L["w_o"]))
            h = _rms(x, L["post_norm"], c.eps)
            gu = F.linear(h, L["w_gu"])
            a = (F.silu(gu[:, : self.it]) * gu[:, self.it:]).contiguous()
            if self.comm is not None:
                x2 = torch.empty_like(x)
                self.comm.allreduce(F.linear(a, L["w_down"]), x2, residual=x)
                x = x2
            else:
                x = x + self._allreduce(F.linear(a, L["w_down"]))
        return x

    def _decode_step(self):
        x = self.embed[self.tok]                                 # [1, H]
        x = self._decode_layers(x)
        h = _rms(x, self.final_norm, self.c.eps)
        self.tok.copy_(self._argmax(h))
        self.pos.add_(1)

    def capture(self):
        """Record one decode step (all layers + argmax + position += 1) into
        a CUDA graph, and a second graph with only the attention-path calls
        of the 64 layers (for the attention share of the step)."""
        self._qkv_dummy = torch.zeros(1, (self.hq + 2 * self.hkv) * self.c.head_dim,
                                      device=self.dev, dtype=torch.float16)
        saved = (self.pos.clone(), self.tok.clone())
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._decode_step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.pos.copy_(saved[0])
        self.tok.copy_(saved[1])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._decode_step()
        self.attn_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.attn_graph):
            self._decode_layers(None, attention_only=True)
        torch.cuda.synchronize()
        self.pos.copy_(saved[0])
        self.tok.copy_(saved[1])

    def decode(self, n_tokens, host_tokens=True):
        """Greedy decode by graph replay; like the reference's launch_step
        (src/model.rs:466-506) each step reads the token back to the host."""
        out = []
        for _ in range(n_tokens):
            self.graph.replay()
            if host_tokens:
                out.append(int(self.tok.item()))
        return out


def run_config5(rank=0, world=1, group=None, prompt_len=8192, gen_tokens=256, shape=None,
                barrier=None, fused_allreduce=True):
    """Config 5 measurement on this rank: returns a dict (rank 0 meaningful)."""
    c = shape or Qwen3Shape()
    dev = torch.device("cuda", torch.cuda.current_device())
    max_seq = prompt_len + gen_tokens
    t0 = time.perf_counter()
    m = Qwen3TP(c, max_seq, rank, world, group, dev, fused_allreduce=fused_allreduce)
    torch.cuda.synchronize()
    t_init = time.perf_counter() - t0
    g = torch.Generator(device=dev).manual_seed(6)
    tokens = torch.randint(0, c.vocab, (prompt_len,), device=dev, generator=g)
    # prefill (timed on device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if barrier:
        barrier()
    e0.record()
    m.prefill(tokens)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    m.capture()
    # warm-up replays then reset the position and caches written by them
    pos0, tok0 = m.pos.clone(), m.tok.clone()
    m.decode(3, host_tokens=False)
    torch.cuda.synchronize()
    m.pos.copy_(pos0)
    m.tok.copy_(tok0)
    if barrier:
        barrier()
    torch.cuda.synchronize()
    e0.record()
    toks = m.decode(gen_tokens)
    e1.record()
    torch.cuda.synchronize()
    decode_ms = e0.elapsed_time(e1)
    # attention share: the attention-path graph alone, replayed at the last
    # cache position (kv_len = max_seq)
    m.pos.fill_(max_seq - 1)
    ts = []
    for _ in range(5):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        m.attn_graph.replay()
        a1.record()
        torch.cuda.synchronize()
        ts.append(a0.elapsed_time(a1))
    attn_ms = sorted(ts)[len(ts) // 2]
    attn.check_device_error()
    return {"prefill_ms": prefill_ms, "decode_ms": decode_ms, "gen_tokens": gen_tokens,
            "tok_s": gen_tokens / (decode_ms * 1e-3), "step_ms": decode_ms / gen_tokens,
            "attn_ms_per_step": attn_ms, "init_s": t_init, "first_tokens": toks[:4],
            "allreduce": "grout NVLink P2P (o_proj fused GEMV+all-reduce, down_proj cuBLAS GEMV + all-reduce)" if m.comm is not None
                         else ("none" if world == 1 else "NCCL")}
