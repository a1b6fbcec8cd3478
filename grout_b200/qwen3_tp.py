"""Minimal tensor-parallel Qwen3 decoder that drives the attention hot path in
context (config 5: Qwen3-32B greedy decode after an 8192-token prompt).

This is the caller of the path, not a product of its own: the decode GEMVs
and the prefill o_proj / MLP GEMMs are cuBLAS, the NCCL collectives (or this
library's NVLink all-reduce) are the exchange; this library supplies the
attention path — the prefill QKV projection with the norm/RoPE/KV write as its
epilogue, prefill attention, and the decode step's fused norm/RoPE/KV write +
split-K attention in one kernel — and the residual add + RMSNorm and SiLU
product kernels around it, called where the reference engine calls its cuTile
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


# Weight identities for the block generator: (tensor id, layer, block).
_EMBED, _LM_HEAD, _FINAL_NORM = 0, 1, 2
_IN_NORM, _POST_NORM, _Q_NORM, _K_NORM = 10, 11, 12, 13
_WQ, _WK, _WV, _WO, _GATE, _UP, _DOWN = 14, 15, 16, 17, 18, 19, 20
CHUNKS = 8  # intermediate / vocab blocks; every TP degree divides it


def _block_seed(seed, tid, layer, block):
    h = seed & ((1 << 61) - 1)
    for v in (tid, layer, block):
        h = (h * 1000003 + v + 1) % ((1 << 61) - 1)
    return h


class Qwen3TP:
    """One rank of a tensor-parallel Qwen3 decoder.

    Every weight is generated block by block from (seed, tensor, layer,
    block): a query or KV head's projection rows, a head's o_proj columns,
    one of CHUNKS slices of the intermediate or vocab dimension.  A rank
    generates only the blocks it owns, so rank r of TP = N holds exactly the
    slice of the TP = 1 tensors that the Megatron layout gives it, and every
    TP degree is the same network."""

    def __init__(self, shape, max_seq, rank=0, world=1, group=None, device=None, seed=6,
                 fused_allreduce=True):
        self.c = c = shape
        self.rank, self.world, self.group = rank, world, group
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        assert c.heads % world == 0 and c.kv_heads % world == 0 and CHUNKS % world == 0
        assert c.inter % CHUNKS == 0 and c.vocab % CHUNKS == 0
        self.hq, self.hkv, self.it = c.heads // world, c.kv_heads // world, c.inter // world
        self.vshard = c.vocab // world
        self.max_seq = max_seq
        D, H = c.head_dim, c.hidden
        cpr = CHUNKS // world  # intermediate / vocab chunks per rank
        ich, vch = c.inter // CHUNKS, c.vocab // CHUNKS

        def gen(tid, layer, block):
            return torch.Generator(device=self.dev).manual_seed(_block_seed(seed, tid, layer, block))

        def w(shape_, tid, layer, block):
            return (torch.randn(*shape_, device=self.dev, generator=gen(tid, layer, block)) * 0.02).half()

        def nw(n, tid, layer):
            return (1.0 + 0.02 * torch.randn(n, device=self.dev, generator=gen(tid, layer, 0))).half()

        def rows(tid, layer, blocks, nrows, ncols):
            return torch.cat([w((nrows, ncols), tid, layer, b) for b in blocks], 0)

        self.embed = rows(_EMBED, 0, range(CHUNKS), vch, H)  # replicated
        self.lm_head = rows(_LM_HEAD, 0, range(rank * cpr, (rank + 1) * cpr), vch, H)
        self.final_norm = nw(H, _FINAL_NORM, 0)
        qh = range(rank * self.hq, (rank + 1) * self.hq)
        kh = range(rank * self.hkv, (rank + 1) * self.hkv)
        ch = range(rank * cpr, (rank + 1) * cpr)
        self.layers = []
        for li in range(c.layers):
            L = dict(
                in_norm=nw(H, _IN_NORM, li), post_norm=nw(H, _POST_NORM, li),
                q_norm=nw(D, _Q_NORM, li), k_norm=nw(D, _K_NORM, li),
                w_qkv=torch.cat([rows(_WQ, li, qh, D, H), rows(_WK, li, kh, D, H),
                                 rows(_WV, li, kh, D, H)], 0),
                w_o=torch.cat([w((H, D), _WO, li, h) for h in qh], 1),
                w_gu=torch.cat([rows(_GATE, li, ch, ich, H), rows(_UP, li, ch, ich, H)], 0),
                w_down=torch.cat([w((H, ich), _DOWN, li, b) for b in ch], 1),
                k_cache=torch.zeros(self.hkv, max_seq, D, device=self.dev, dtype=torch.float16),
                v_cache=torch.zeros(self.hkv, max_seq, D, device=self.dev, dtype=torch.float16),
            )
            self.layers.append(L)
        self.rope = attn.rope_table(c.theta, max_seq, self.dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.tok = torch.zeros(1, dtype=torch.int64, device=self.dev)
        # final-norm hidden state of the last step (written inside the graph)
        self.h_last = torch.zeros(1, H, device=self.dev, dtype=torch.float16)
        nks = attn.decode_workspace_bytes(1, max_seq, self.hq, self.hkv, max_seq)
        self.ws = torch.empty(max(16, nks), dtype=torch.uint8, device=self.dev)
        # Decode o_proj / down_proj (TP > 1): a cuBLAS GEMV followed by the
        # grout all-reduce + residual over NVLink peer memory, the faster form
        # measured on B200 at TP = 2 (the fused GEMV + all-reduce kernel's
        # GEMV streams at about half of cuBLAS's rate).  NCCL when disabled.
        self.comm = None
        if fused_allreduce and world > 1:
            from .tp import TPComm
            self.comm = TPComm(rank, world, H, group, self.dev)
        # decode-step buffers (fixed addresses for graph replay)
        self.q1 = torch.empty(1, self.hq, D, device=self.dev, dtype=torch.float16)
        self.o1 = torch.empty_like(self.q1)
        # layer-0 activations of the last eager prefill / decode step, kept
        # when trace is set (prefill/decode consistency checks)
        self.trace = None

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

    # ------------------------------------------------------------- residual
    def _norm(self, x, w, pending=None):
        """(normed, residual stream): rmsnorm(x + pending) * w in one kernel,
        the stream updated to x + pending when a partial is pending (the
        reference's add_rms_norm, src/kernels.rs:4449-4600)."""
        h = torch.empty_like(x)
        if pending is None:
            attn.add_rms_norm(x, w, h, self.c.eps)
            return h, x
        xn = torch.empty_like(x)
        attn.add_rms_norm(pending, w, h, self.c.eps, residual=x, residual_out=xn)
        return h, xn

    def _mlp_in(self, h, L):
        gu = F.linear(h, L["w_gu"])
        a = torch.empty(h.shape[0], self.it, device=self.dev, dtype=torch.float16)
        attn.silu_mul(gu, a)
        return a

    # ---------------------------------------------------------------- prefill
    def prefill(self, tokens):
        """Run the prompt (eager, like the reference's StepGraph prefill):
        returns the first generated token id (device tensor [1])."""
        c, D = self.c, self.c.head_dim
        S = tokens.numel()
        x = self.embed[tokens]                                   # [S, H]
        pending = None
        for L in self.layers:
            h, x = self._norm(x, L["in_norm"], pending)
            # QKV projection with the norm/RoPE/KV write as its epilogue
            q_out = torch.empty(S, self.hq, D, device=self.dev, dtype=torch.float16)
            tracing = self.trace is not None and L is self.layers[0]
            qkv = (torch.empty(S, (self.hq + 2 * self.hkv) * D, device=self.dev,
                               dtype=torch.float16) if tracing else None)
            attn.qkv_proj_norm_rope_kv_prefill(h, L["w_qkv"], L["q_norm"], L["k_norm"], self.rope,
                                               q_out, L["k_cache"], L["v_cache"], 0, c.eps,
                                               qkv_out=qkv)
            o = torch.empty_like(q_out)
            attn.attention_prefill(q_out, L["k_cache"], L["v_cache"], o, 0)
            if tracing:
                self.trace["prefill"] = (qkv, o.clone())
            p = self._allreduce(F.linear(o.view(S, -1), L["w_o"]))
            h, x = self._norm(x, L["post_norm"], p)
            pending = self._allreduce(F.linear(self._mlp_in(h, L), L["w_down"]))
        h, _ = self._norm(x[-1:].contiguous(), self.final_norm, pending[-1:].contiguous())
        self.h_last.copy_(h)
        self.pos.fill_(S)
        self.tok.copy_(self._argmax(h))
        return self.tok

    # ---------------------------------------------------------------- decode
    def _attention(self, qkv, L):
        """The decode step's fused Q/K norm + RoPE + KV write and split-K
        attention, one kernel (grout_attn_decode_fused)."""
        attn.attention_decode_fused(qkv, L["q_norm"], L["k_norm"], self.rope, L["k_cache"],
                                    L["v_cache"], self.pos, self.o1, self.max_seq, self.c.eps,
                                    workspace=self.ws)

    def _proj(self, w, x):
        """Decode GEMV [1, n] = w x (cuBLAS)."""
        return F.linear(x.view(1, -1), w)

    def _decode_layers(self, x, attention_only=False, mark=lambda name: None):
        """All layers of one decode step.  mark(name) is called after each
        stage (the per-stage breakdown records a timing event there)."""
        if attention_only:
            for L in self.layers:
                self._attention(self._qkv_dummy, L)
            return None
        pending = None   # a partial still to be added to x (NCCL path)
        for L in self.layers:
            h, x = self._norm(x, L["in_norm"], pending)
            mark("add_rms_norm")
            qkv = self._proj(L["w_qkv"], h)
            mark("qkv_gemv")
            self._attention(qkv, L)
            mark("attention")
            if self.trace is not None and L is self.layers[0]:
                self.trace["decode"] = (qkv.clone(), self.o1.clone())
            if self.comm is not None:
                # o_proj: cuBLAS GEMV, then the grout all-reduce + residual
                po = self._proj(L["w_o"], self.o1)
                mark("o_proj_gemv")
                x1 = torch.empty_like(x)
                self.comm.allreduce(po, x1, residual=x)
                mark("o_proj_allreduce")
                h, x = self._norm(x1, L["post_norm"])
            else:
                p = self._allreduce(self._proj(L["w_o"], self.o1))
                mark("o_proj_gemv" + ("_nccl_allreduce" if self.world > 1 else ""))
                h, x = self._norm(x, L["post_norm"], p)
            mark("add_rms_norm")
            gu = self._proj(L["w_gu"], h)
            mark("gate_up_gemv")
            a = torch.empty(1, self.it, device=self.dev, dtype=torch.float16)
            attn.silu_mul(gu, a)
            mark("silu_mul")
            d = self._proj(L["w_down"], a)
            mark("down_gemv")
            if self.comm is not None:
                # down_proj: cuBLAS GEMV, then the grout all-reduce + residual
                # (faster than the fused kernel at this shape, see tp_allreduce.cu)
                x2 = torch.empty_like(x)
                self.comm.allreduce(d, x2, residual=x)
                x, pending = x2, None
                mark("down_allreduce")
            else:
                pending = self._allreduce(d)
                if self.world > 1:
                    mark("down_nccl_allreduce")
        return x, pending

    def _decode_step(self, mark=lambda name: None):
        x = self.embed[self.tok]                                 # [1, H]
        mark("embed")
        x, pending = self._decode_layers(x, mark=mark)
        h, _ = self._norm(x, self.final_norm, pending)
        self.h_last.copy_(h)
        self.tok.copy_(self._argmax(h))
        self.pos.add_(1)
        mark("final_norm_lm_head_argmax")

    def breakdown(self):
        """Device time per stage of one decode step, summed over the layers
        (ms): the step recorded into a separate graph with a timing event
        after every stage.  Position and token are restored afterwards."""
        saved = (self.pos.clone(), self.tok.clone())
        marks = []

        def mark(name):
            e = torch.cuda.Event(enable_timing=True, external=True)
            e.record()
            marks.append((name, e))

        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            mark("start")
            self._decode_step(mark)
        g.replay()
        torch.cuda.synchronize()
        out = {}
        for (_, e0), (name, e1) in zip(marks, marks[1:]):
            out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
        self.pos.copy_(saved[0])
        self.tok.copy_(saved[1])
        del g
        return {k: round(v, 4) for k, v in out.items()}

    def step_eager(self):
        """One decode step without the graph (same ops); returns the token."""
        self._decode_step()
        return int(self.tok.item())

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
    # prefill (timed on device).  A first, untimed pass over the same prompt
    # loads every kernel module and sets up cuBLAS for these shapes; the
    # timed pass rewrites the same caches.
    m.prefill(tokens)
    torch.cuda.synchronize()
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
    m.pos.fill_(max_seq - 1)
    stages = m.breakdown()
    attn.check_device_error()
    return {"prefill_ms": prefill_ms, "decode_ms": decode_ms, "gen_tokens": gen_tokens,
            "tok_s": gen_tokens / (decode_ms * 1e-3), "step_ms": decode_ms / gen_tokens,
            "attn_ms_per_step": attn_ms, "init_s": t_init, "first_tokens": toks[:4],
            "stage_ms_per_step": stages,
            "allreduce": "grout NVLink P2P all-reduce + residual after cuBLAS GEMVs (o_proj, down_proj)" if m.comm is not None
                         else ("none" if world == 1 else "NCCL")}
