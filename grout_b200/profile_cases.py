"""Small, self-contained workloads for single-kernel ncu captures.

Each case runs one public entry point twice at a benchmark shape on ``cuda:0`` and
checks the device error word, so that ``ncu -k <kernel> -s 1 -c 1`` captures one warm
launch.  Usage: ``python -m grout_b200.profile_cases qkv_proj``.
"""
import sys

import torch

import grout_b200 as g


def qkv_proj() -> None:
    """Qwen3-32B prefill QKV projection + fused norm/RoPE/KV write, S = 4096."""
    g.init(0)
    S, hidden, hq, hkv, D = 4096, 5120, 64, 8, 128
    N = (hq + 2 * hkv) * D
    dev = torch.device("cuda", 0)
    x = torch.randn(S, hidden, device=dev).half()
    w = (torch.randn(N, hidden, device=dev) * 0.02).half()
    ones = torch.ones(D, dtype=torch.float16, device=dev)
    table = g.rope_table(1e6, S, dev)
    q_out = torch.empty(S, hq, D, dtype=torch.float16, device=dev)
    kc = torch.zeros(hkv, S, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    for _ in range(2):
        g.qkv_proj_norm_rope_kv_prefill(x, w, ones, ones, table, q_out, kc, vc, 0, 1e-6)
    torch.cuda.synchronize()
    g.check_device_error()
    print("ok")


CASES = {"qkv_proj": qkv_proj}

if __name__ == "__main__":
    CASES[sys.argv[1]]()
