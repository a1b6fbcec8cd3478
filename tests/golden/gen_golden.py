"""Writes the golden vectors in tests/golden/golden.npz.

An independent restatement (numpy float32/float64 and Python's libm, no code
shared with oracle/ or grout_b200/) of the reference math, on small seeded
inputs:
  - build_inv_freq (src/model.rs:7295-7306) and the RoPE angle table;
  - the fused Q/K RMSNorm + RoPE + KV write (src/kernels.rs:5012-5166) with
    the summation order the CUDA kernel and the C++ oracle share (8 lanes of
    8 lo + 8 hi elements, lane sum ((t0+t1)+(t2+t3))+((t4+t5)+(t6+t7)), xor
    butterfly 4,2,1);
  - causal GQA prefill attention and GQA decode attention, in float64
    (the "ideal" result the f16 kernels are held to within tolerance);
  - the reference's microbench KAT pattern (attention_microbench.rs:203-214).
The reference itself (Rust + cuTile) cannot run here, so these vectors pin
the oracle to a second restatement, not to reference outputs.

    python tests/golden/gen_golden.py
"""
import math
import os

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
D = 128


def splitmix_normal(seed, n):
    # same generator family as the product inputs, restated here
    g = np.uint64(0x9E3779B97F4A7C15)
    idx = np.arange(1, 2 * ((n + 1) // 2) + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + idx * g
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = ((z >> np.uint64(11)).astype(np.float64) + 0.5) / 2.0**53
    u1, u2 = u[0::2], u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(u.shape[0])
    out[0::2] = r * np.cos(2 * np.pi * u2)
    out[1::2] = r * np.sin(2 * np.pi * u2)
    return out[:n].astype(np.float32).astype(np.float16)


def inv_freq_f32pow(theta):
    # powf in f32: evaluate in double and round (glibc powf is correctly
    # rounded in practice for these arguments)
    out = []
    for i in range(0, D, 2):
        p = np.float32(np.float32(i) / np.float32(D))
        pw = np.float32(math.pow(float(np.float32(theta)), float(p)))
        out.append(np.float32(1.0) / pw)
    return np.array(out, dtype=np.float32)


def rope_table(inv, max_seq):
    t = np.empty((max_seq, 2, D // 2), dtype=np.float32)
    for pos in range(max_seq):
        for i in range(D // 2):
            ang = np.float32(np.float32(pos) * inv[i])
            t[pos, 0, i] = np.float32(math.cos(float(ang)))
            t[pos, 1, i] = np.float32(math.sin(float(ang)))
    return t


def norm_rope_row(x16, w16, cs, sn, eps):
    x = x16.astype(np.float32)
    w = w16.astype(np.float32)
    lo, hi = x[:64].reshape(8, 8), x[64:].reshape(8, 8)
    t = lo * lo + hi * hi                       # float32 elementwise
    s = ((t[:, 0] + t[:, 1]) + (t[:, 2] + t[:, 3])) + ((t[:, 4] + t[:, 5]) + (t[:, 6] + t[:, 7]))
    for off in (4, 2, 1):
        s = s + s[np.arange(8) ^ off]
    ss = s[0]
    inv = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(128.0)) + np.float32(eps))
    nlo = (x[:64] * inv) * w[:64]
    nhi = (x[64:] * inv) * w[64:]
    ylo = nlo * cs - nhi * sn
    yhi = nhi * cs + nlo * sn
    return np.concatenate([ylo, yhi]).astype(np.float16)


def attn_f64(qrow, K, V, scale):
    s = (K.astype(np.float64) @ qrow.astype(np.float64)) * scale
    p = np.exp(s - s.max())
    return (p @ V.astype(np.float64)) / p.sum()


def main():
    g = {}
    # ---- inv_freq / table
    theta = 1.0e6
    inv = inv_freq_f32pow(theta)
    g["inv_freq"] = inv
    max_seq = 16
    table = rope_table(inv, max_seq)
    g["rope_table"] = table
    # ---- fused norm/rope prefill: S=8, Hq=4, Hkv=2, pos0=3
    S, hq, hkv, pos0, eps = 8, 4, 2, 3, 1e-6
    q = splitmix_normal(1, S * hq * D).reshape(S, hq, D)
    k = splitmix_normal(2, S * hkv * D).reshape(S, hkv, D)
    v = splitmix_normal(3, S * hkv * D).reshape(S, hkv, D)
    qw = (1.0 + 0.02 * splitmix_normal(4, D).astype(np.float64)).astype(np.float32).astype(np.float16)
    kw = (1.0 + 0.02 * splitmix_normal(7, D).astype(np.float64)).astype(np.float32).astype(np.float16)
    q_out = np.zeros_like(q)
    kc = np.zeros((hkv, max_seq, D), np.float16)
    vc = np.zeros((hkv, max_seq, D), np.float16)
    for s in range(S):
        cs, sn = table[pos0 + s, 0], table[pos0 + s, 1]
        for h in range(hq):
            q_out[s, h] = norm_rope_row(q[s, h], qw, cs, sn, eps)
        for h in range(hkv):
            kc[h, pos0 + s] = norm_rope_row(k[s, h], kw, cs, sn, eps)
            vc[h, pos0 + s] = v[s, h]
    g.update(nr_q=q, nr_k=k, nr_v=v, nr_qw=qw, nr_kw=kw, nr_q_out=q_out, nr_k_cache=kc,
             nr_v_cache=vc)
    # ---- causal prefill, cache layout, P=5: S=40, Hq=4, Hkv=2, max_seq=48
    S, hq, hkv, P, ms = 40, 4, 2, 5, 48
    G = hq // hkv
    pq = splitmix_normal(11, S * hq * D).reshape(S, hq, D)
    pk = splitmix_normal(12, hkv * ms * D).reshape(hkv, ms, D)
    pv = splitmix_normal(13, hkv * ms * D).reshape(hkv, ms, D)
    scale = 1.0 / math.sqrt(D)
    po = np.zeros((S, hq, D), np.float64)
    for m in range(S):
        for h in range(hq):
            n = P + m + 1
            po[m, h] = attn_f64(pq[m, h], pk[h // G, :n], pv[h // G, :n], scale)
    g.update(pf_q=pq, pf_k=pk, pf_v=pv, pf_out=po, pf_pos0=np.int32(P))
    # ---- decode: B=2, Hq=8, Hkv=2, positions [37, 80], max_seq=96
    B, hq, hkv, ms = 2, 8, 2, 96
    G = hq // hkv
    pos = np.array([37, 80], np.uint32)
    dq = splitmix_normal(21, B * hq * D).reshape(B, hq, D)
    dk = splitmix_normal(22, B * hkv * ms * D).reshape(B, hkv, ms, D)
    dv = splitmix_normal(23, B * hkv * ms * D).reshape(B, hkv, ms, D)
    do = np.zeros((B, hq, D), np.float64)
    for b in range(B):
        for h in range(hq):
            n = int(pos[b]) + 1
            do[b, h] = attn_f64(dq[b, h], dk[b, h // G, :n], dv[b, h // G, :n], scale)
    g.update(dc_q=dq, dc_k=dk, dc_v=dv, dc_out=do, dc_pos=pos)
    # ---- reference KAT pattern (attention_microbench.rs:203-214), salts 1..3
    for salt in (1, 2, 3):
        i = np.arange(4096, dtype=np.int64)
        raw = ((i * 37 + salt * 17) % 101).astype(np.float32)
        g[f"pattern_{salt}"] = ((raw - np.float32(50.0)) / np.float32(80.0)).astype(np.float16)
    np.savez_compressed(OUT, **g)
    print("wrote", OUT, sum(a.nbytes for a in g.values()), "bytes")


if __name__ == "__main__":
    main()
