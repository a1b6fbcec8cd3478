// CPU oracle for the grout attention hot path — TEST INFRASTRUCTURE ONLY.
//
// This file restates, in plain C++ on the host, the arithmetic of the
// reference (rtburger/grout) kernels that the CUDA library replaces.  It is
// the checker used by tests/, by __graft_entry__.smoke() and by the
// cpu_baseline / --impl reference legs of bench.py.  The product path
// (grout_b200/) never links or calls it.
//
// Parity status: UNPINNED against the reference's own outputs.  The
// reference is Rust + cuTile (tileiras) and cannot be built or run in this
// environment, and its repository holds no stored expected outputs for any
// attention, RoPE or norm kernel.  What is pinned: (1) the reference's
// attention KAT generator (pattern_value, attention_microbench.rs:203-214)
// and its f32 cpu_reference (attention_microbench.rs:665-702), which
// oracle_attn_prefill_naive restates line for line; (2) analytic
// known-answer cases in tests/; (3) golden vectors in tests/golden/ written
// by an independent numpy restatement (tests/golden/gen_golden.py).
//
// Every function names the reference file:line it follows.  Build:
// oracle/build.py (g++ -O3 -march=x86-64-v2 -fopenmp -ffp-contract=off).
// -ffp-contract=off matters: the bit-exact fused norm/RoPE oracle must not
// be contracted into FMAs.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <algorithm>
#include <omp.h>

typedef uint16_t u16;

// ---------------------------------------------------------------- f16 <-> f32
// IEEE binary16 conversions, round-to-nearest-even, with subnormals, inf and
// NaN handled.  Written from the format definition.
static inline float h2f(u16 h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: value = man * 2^-24
      float f = (float)man * 5.9604644775390625e-8f;
      uint32_t fb;
      std::memcpy(&fb, &f, 4);
      bits = sign | fb;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

static inline u16 f2h(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) {  // inf / nan
    return (u16)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477ff000u) {  // >= 65520 rounds to inf
    return (u16)(sign | 0x7c00u);
  }
  if (ax < 0x38800000u) {  // below 2^-14: subnormal or zero in f16
    // value in units of 2^-24, rounded to nearest even
    float a;
    std::memcpy(&a, &ax, 4);
    float scaled = a * 16777216.0f;  // exact (power of two)
    float r = std::nearbyint(scaled); // default rounding mode: nearest-even
    return (u16)(sign | (uint32_t)r);
  }
  uint32_t e = (ax >> 23) - 112u;
  uint32_t m = ax & 0x7fffffu;
  uint32_t h = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
  return (u16)(sign | h);
}

static inline float round_f16(float f) { return h2f(f2h(f)); }

extern "C" {

void oracle_f32_to_f16(const float* in, u16* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2h(in[i]);
}
void oracle_f16_to_f32(const u16* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = h2f(in[i]);
}

// Reference KAT generator: attention_microbench.rs:203-214
//   raw = ((i*37 + salt*17) % 101); value = (raw - 50) / 80, rounded to f16.
void oracle_pattern(int64_t len, int64_t salt, u16* out) {
  for (int64_t i = 0; i < len; ++i) {
    float raw = (float)((uint64_t)(i * 37 + salt * 17) % 101);
    out[i] = f2h((raw - 50.0f) / 80.0f);
  }
}

// build_inv_freq: src/model.rs:7295-7306
//   for i in (0..D).step_by(2): inv.push(1.0f32 / theta.powf(i as f32 / D as f32))
void oracle_inv_freq(float theta, int32_t head_dim, float* out) {
  for (int32_t i = 0; i < head_dim; i += 2) {
    float p = (float)i / (float)head_dim;
    out[i / 2] = 1.0f / powf(theta, p);
  }
}

// RoPE angle table.  The reference evaluates theta = f32(pos) * inv_freq[i]
// in f32 (src/kernels.rs:5076-5079) and then cos/sin of that f32 angle.  The
// table holds cos/sin of exactly that f32 angle, evaluated in double and
// rounded once to f32.  Layout: [max_seq][2][half] (cos row then sin row).
void oracle_rope_table(const float* inv_freq, int32_t half, int32_t max_seq, float* table) {
  for (int32_t pos = 0; pos < max_seq; ++pos) {
    for (int32_t i = 0; i < half; ++i) {
      float theta = (float)pos * inv_freq[i];
      table[(int64_t)pos * 2 * half + i] = (float)std::cos((double)theta);
      table[(int64_t)pos * 2 * half + half + i] = (float)std::sin((double)theta);
    }
  }
}

// One head row of the fused norm + RoPE, D = 128.
// Math: src/kernels.rs:5012-5084 (prefill) / 5294-5420 (decode):
//   ss  = sum(x_lo^2 + x_hi^2);  inv = rsqrt(ss / D + eps)
//   n   = (x * inv) * w
//   y_lo = n_lo*cos - n_hi*sin ;  y_hi = n_hi*cos + n_lo*sin ; one f16 rounding
// Summation order (our contract, shared with the CUDA kernel): 8 lanes, lane
// j owns x[8j..8j+8) and x[64+8j..64+8j+8); t_e = lo_e^2 + hi_e^2;
// lane sum = ((t0+t1)+(t2+t3)) + ((t4+t5)+(t6+t7)); then a xor-butterfly over
// the 8 lanes with offsets 4,2,1.  rsqrt is evaluated as 1/sqrt with IEEE
// rounding; ss / 128 is exact scaling.
static void norm_rope_row(const u16* x, const u16* w, const float* cs, const float* sn,
                          float eps, u16* y) {
  float xf[128];
  for (int i = 0; i < 128; ++i) xf[i] = h2f(x[i]);
  float s[8];
  for (int j = 0; j < 8; ++j) {
    float t[8];
    for (int e = 0; e < 8; ++e) {
      int i = 8 * j + e;
      float a = xf[i] * xf[i];
      float b = xf[64 + i] * xf[64 + i];
      t[e] = a + b;
    }
    float u0 = t[0] + t[1], u1 = t[2] + t[3], u2 = t[4] + t[5], u3 = t[6] + t[7];
    float v0 = u0 + u1, v1 = u2 + u3;
    s[j] = v0 + v1;
  }
  for (int off = 4; off >= 1; off >>= 1) {
    float s2[8];
    for (int j = 0; j < 8; ++j) s2[j] = s[j] + s[j ^ off];
    std::memcpy(s, s2, sizeof(s));
  }
  float ss = s[0];
  float mean = ss / 128.0f;
  float arg = mean + eps;
  float inv = 1.0f / std::sqrt(arg);
  for (int i = 0; i < 64; ++i) {
    float nlo = (xf[i] * inv) * h2f(w[i]);
    float nhi = (xf[64 + i] * inv) * h2f(w[64 + i]);
    float a = nlo * cs[i];
    float b = nhi * sn[i];
    float c = nhi * cs[i];
    float d = nlo * sn[i];
    y[i] = f2h(a - b);
    y[64 + i] = f2h(c + d);
  }
}

// qk_norm_rope_kv_prefill_raw_f16: src/kernels.rs:4845-5168
//   q [S, Hq, D] (row stride q_row_stride), k/v [S, Hkv, D] (kv_row_stride)
//   q_out [S, Hq, D] (q_row_stride), caches [Hkv, max_seq, D] with head
//   stride cache_head_stride; row s goes to cache position pos0 + s.
void oracle_qk_norm_rope_kv_prefill(const u16* q, const u16* k, const u16* v,
                                    int64_t q_row_stride, int64_t kv_row_stride,
                                    const u16* q_w, const u16* k_w, const float* table,
                                    u16* q_out, u16* k_cache, u16* v_cache,
                                    int64_t cache_head_stride, int32_t pos0, int32_t seq_len,
                                    int32_t hq, int32_t hkv, float eps) {
  const int D = 128, H = 64;
#pragma omp parallel for schedule(static)
  for (int32_t s = 0; s < seq_len; ++s) {
    int32_t pos = pos0 + s;
    const float* cs = table + (int64_t)pos * 2 * H;
    const float* sn = cs + H;
    for (int32_t h = 0; h < hq; ++h)
      norm_rope_row(q + s * q_row_stride + h * D, q_w, cs, sn, eps,
                    q_out + s * q_row_stride + h * D);
    for (int32_t h = 0; h < hkv; ++h) {
      norm_rope_row(k + s * kv_row_stride + h * D, k_w, cs, sn, eps,
                    k_cache + h * cache_head_stride + (int64_t)pos * D);
      std::memcpy(v_cache + h * cache_head_stride + (int64_t)pos * D,
                  v + s * kv_row_stride + h * D, D * sizeof(u16));
    }
  }
}

// qk_norm_rope_kv_decode_raw_f16: src/kernels.rs:5180-5452, generalised to a
// batch: qkv [B][(Hq + 2Hkv) * D] = [Q | K | V] per sequence, position[b]
// from device memory in the kernel; q_out [B][Hq][D]; caches per sequence at
// base + b * cache_batch_stride.
void oracle_qk_norm_rope_kv_decode(const u16* qkv, const u16* q_w, const u16* k_w,
                                   const float* table, u16* q_out, u16* k_cache,
                                   u16* v_cache, int64_t cache_batch_stride,
                                   int64_t cache_head_stride, const uint32_t* position,
                                   int32_t batch, int32_t hq, int32_t hkv, float eps) {
  const int D = 128, H = 64;
  const int64_t row = (int64_t)(hq + 2 * hkv) * D;
  for (int32_t b = 0; b < batch; ++b) {
    int64_t pos = position[b];
    const float* cs = table + pos * 2 * H;
    const float* sn = cs + H;
    const u16* base = qkv + b * row;
    for (int32_t h = 0; h < hq; ++h)
      norm_rope_row(base + h * D, q_w, cs, sn, eps, q_out + ((int64_t)b * hq + h) * D);
    for (int32_t h = 0; h < hkv; ++h) {
      norm_rope_row(base + (int64_t)(hq + h) * D, k_w, cs, sn, eps,
                    k_cache + b * cache_batch_stride + h * cache_head_stride + pos * D);
      std::memcpy(v_cache + b * cache_batch_stride + h * cache_head_stride + pos * D,
                  base + (int64_t)(hq + hkv + h) * D, D * sizeof(u16));
    }
  }
}

// The reference's own f32 CPU attention: attention_microbench.rs:665-702.
// q [S, Hq, D], k/v [Hkv, S, D]; natural exp; out f32 [S, Hq, D].
void oracle_attn_prefill_naive(const float* q, const float* k, const float* v, float* out,
                               int32_t q_len, int32_t q_heads, int32_t kv_heads,
                               int32_t head_dim) {
  int qgs = q_heads / kv_heads;
  float scale = 1.0f / std::sqrt((float)head_dim);
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (int m = 0; m < q_len; ++m) {
    for (int qh = 0; qh < q_heads; ++qh) {
      int kvh = qh / qgs;
      std::vector<float> scores(m + 1);
      float max_score = -INFINITY;
      for (int n = 0; n <= m; ++n) {
        float dot = 0.0f;
        for (int d = 0; d < head_dim; ++d)
          dot += q[((int64_t)m * q_heads + qh) * head_dim + d] *
                 k[((int64_t)kvh * q_len + n) * head_dim + d];
        scores[n] = dot * scale;
        max_score = std::max(max_score, scores[n]);
      }
      float denom = 0.0f;
      for (auto& s : scores) {
        s = std::exp(s - max_score);
        denom += s;
      }
      for (int d = 0; d < head_dim; ++d) {
        float acc = 0.0f;
        for (int n = 0; n <= m; ++n)
          acc += scores[n] / denom * v[((int64_t)kvh * q_len + n) * head_dim + d];
        out[((int64_t)m * q_heads + qh) * head_dim + d] = acc;
      }
    }
  }
}

// Causal GQA prefill with the rounding points of fmha_prefill_causal
// (src/kernels.rs:2570-2725): scores in f32, log2-domain softmax
// (s2 = scale / ln 2), P rounded to f16 before the PV product, acc in f32,
// out = f16(acc / max(l, 1e-8)).  Row m of sequence b (query position
// pos0[b] + m) sees keys n <= pos0[b] + m and n < kv_len = pos0[b] + S_b.
// The softmax is taken against the row's final max (single pass), which is
// the same function as the tiled online form up to f16 rounding of P.
//
// Layout (general strides, elements):
//   q/out: row r of sequence b at (cu_q[b] + r) * q_row_stride + h * D
//   k/v:   key n of sequence b, kv head h at
//          b * kv_batch_stride + (kv_start[b] + n) * kv_row_stride + h * kv_head_stride
// ideal != 0: f64 scores/softmax, no f16 rounding of P (the f64 ideal).
// rows_step > 1 evaluates only every rows_step-th query row (bounded CPU
// timing sample); skipped rows are left untouched.
void oracle_attn_prefill(const u16* q, const u16* k, const u16* v, u16* out,
                         const int32_t* cu_q, const int32_t* pos0, const int32_t* kv_start,
                         int32_t batch, int32_t hq, int32_t hkv, int64_t q_row_stride,
                         int64_t kv_batch_stride, int64_t kv_row_stride,
                         int64_t kv_head_stride, float scale, int32_t ideal,
                         int32_t rows_step) {
  const int D = 128;
  const int G = hq / hkv;
  const float s2 = scale / std::log(2.0f);
  if (rows_step < 1) rows_step = 1;
  for (int32_t b = 0; b < batch; ++b) {
    const int32_t S = cu_q[b + 1] - cu_q[b];
    const int32_t P = pos0 ? pos0[b] : 0;
    const int64_t ks = kv_start ? kv_start[b] : 0;
    const int32_t kv_len = P + S;
    const int32_t nrows = (S + rows_step - 1) / rows_step;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int32_t ri = 0; ri < nrows; ++ri) {
      for (int32_t h = 0; h < hq; ++h) {
        const int32_t m = ri * rows_step;
        const int32_t kvh = h / G;
        const u16* qrow = q + (int64_t)(cu_q[b] + m) * q_row_stride + (int64_t)h * D;
        const int32_t nvis = std::min(P + m + 1, kv_len);
        float qf[D];
        for (int d = 0; d < D; ++d) qf[d] = h2f(qrow[d]);
        const u16* kb = k + b * kv_batch_stride + ks * kv_row_stride + kvh * kv_head_stride;
        const u16* vb = v + b * kv_batch_stride + ks * kv_row_stride + kvh * kv_head_stride;
        u16* orow = out + (int64_t)(cu_q[b] + m) * q_row_stride + (int64_t)h * D;
        if (ideal) {
          std::vector<double> sc(nvis);
          double mx = -INFINITY;
          for (int32_t n = 0; n < nvis; ++n) {
            const u16* kr = kb + (int64_t)n * kv_row_stride;
            double dot = 0.0;
            for (int d = 0; d < D; ++d) dot += (double)qf[d] * (double)h2f(kr[d]);
            sc[n] = dot * (double)scale;
            mx = std::max(mx, sc[n]);
          }
          double l = 0.0;
          std::vector<double> acc(D, 0.0);
          for (int32_t n = 0; n < nvis; ++n) {
            double p = std::exp(sc[n] - mx);
            l += p;
            const u16* vr = vb + (int64_t)n * kv_row_stride;
            for (int d = 0; d < D; ++d) acc[d] += p * (double)h2f(vr[d]);
          }
          for (int d = 0; d < D; ++d) orow[d] = f2h((float)(acc[d] / l));
        } else {
          std::vector<float> sc(nvis);
          float mx = -1.0e30f;
          for (int32_t n = 0; n < nvis; ++n) {
            const u16* kr = kb + (int64_t)n * kv_row_stride;
            float dot = 0.0f;
            for (int d = 0; d < D; ++d) dot += qf[d] * h2f(kr[d]);
            sc[n] = dot;
            mx = std::max(mx, dot * s2);
          }
          float l = 0.0f;
          float acc[D];
          for (int d = 0; d < D; ++d) acc[d] = 0.0f;
          for (int32_t n = 0; n < nvis; ++n) {
            float p = std::exp2(sc[n] * s2 - mx);
            l += p;
            float ph = round_f16(p);
            const u16* vr = vb + (int64_t)n * kv_row_stride;
            for (int d = 0; d < D; ++d) acc[d] += ph * h2f(vr[d]);
          }
          float ls = std::max(l, 1.0e-8f);
          for (int d = 0; d < D; ++d) orow[d] = f2h(acc[d] / ls);
        }
      }
    }
  }
}

// Split-K GQA decode with the reference's rounding points:
// fmha_decode_gqa_split (src/kernels.rs:4016-4185) + splitk_reduce_merge
// (src/kernels.rs:4201-4304), generalised to a batch.
//   q [B, Hq, D]; key n of sequence b, kv head h at
//   b * kv_batch_stride + h * kv_head_stride + n * D.  kv_len = position[b] + 1.
//   qk_scale is applied as given (the reference passes f16(1/sqrt(D)),
//   src/model.rs:3177); scores scaled by qk_scale / ln 2 after the dot
//   product; keys >= kv_len get -1e30 added before scaling (4113-4119);
//   l starts as a [BN] vector of ones (4074); per-split O is normalised and
//   rounded to f16 (4171-4179), lse = m + log2(max(sum l, 1e-8)) (4182);
//   merge weights 2^(lse_s - max) / max(sum, 1e-8), out rounded to f16.
// nks = number of splits, bn = tile size.  ideal != 0: f64 softmax over all
// keys, no intermediate rounding (nks/bn ignored).
void oracle_attn_decode(const u16* q, const u16* k, const u16* v, u16* out,
                        const uint32_t* position, int32_t batch, int32_t hq, int32_t hkv,
                        int64_t kv_batch_stride, int64_t kv_head_stride, float qk_scale,
                        int32_t nks, int32_t bn, int32_t ideal) {
  const int D = 128;
  const int G = hq / hkv;
  const float ln2 = std::log(2.0f);
  const float s2 = qk_scale / ln2;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int32_t b = 0; b < batch; ++b) {
    for (int32_t h = 0; h < hq; ++h) {
      const int32_t kvh = h / G;
      const int32_t s_kv = (int32_t)position[b] + 1;
      const u16* qr = q + ((int64_t)b * hq + h) * D;
      const u16* kb = k + b * kv_batch_stride + kvh * kv_head_stride;
      const u16* vb = v + b * kv_batch_stride + kvh * kv_head_stride;
      u16* orow = out + ((int64_t)b * hq + h) * D;
      float qf[D];
      for (int d = 0; d < D; ++d) qf[d] = h2f(qr[d]);
      if (ideal) {
        std::vector<double> sc(s_kv);
        double mx = -INFINITY;
        for (int32_t n = 0; n < s_kv; ++n) {
          double dot = 0.0;
          for (int d = 0; d < D; ++d) dot += (double)qf[d] * (double)h2f(kb[(int64_t)n * D + d]);
          sc[n] = dot * (double)qk_scale;
          mx = std::max(mx, sc[n]);
        }
        double l = 0.0;
        std::vector<double> acc(D, 0.0);
        for (int32_t n = 0; n < s_kv; ++n) {
          double p = std::exp(sc[n] - mx);
          l += p;
          for (int d = 0; d < D; ++d) acc[d] += p * (double)h2f(vb[(int64_t)n * D + d]);
        }
        for (int d = 0; d < D; ++d) orow[d] = f2h((float)(acc[d] / l));
        continue;
      }
      const int32_t tiles = (s_kv + bn - 1) / bn;
      const int32_t tps = (tiles + nks - 1) / nks;
      std::vector<float> o_split((size_t)nks * D);
      std::vector<float> lse(nks);
      std::vector<float> lvec(bn);
      std::vector<float> qk(bn);
      for (int32_t sp = 0; sp < nks; ++sp) {
        const int32_t t0 = sp * tps;
        const int32_t t1 = std::min(t0 + tps, tiles);
        float m = -1.0e30f;
        std::fill(lvec.begin(), lvec.end(), 1.0f);
        float acc[D];
        for (int d = 0; d < D; ++d) acc[d] = 0.0f;
        for (int32_t j = t0; j < t1; ++j) {
          float tmax = -INFINITY;
          for (int32_t i = 0; i < bn; ++i) {
            const int32_t n = j * bn + i;
            float dot = 0.0f;
            if (n < s_kv)
              for (int d = 0; d < D; ++d) dot += qf[d] * h2f(kb[(int64_t)n * D + d]);
            if (j == tiles - 1 && n >= s_kv) dot = dot + -1.0e30f;
            qk[i] = dot * s2;
            tmax = std::max(tmax, qk[i]);
          }
          const float mij = std::max(m, tmax);
          const float alpha = std::exp2(m - mij);
          for (int d = 0; d < D; ++d) acc[d] *= alpha;
          for (int32_t i = 0; i < bn; ++i) {
            const int32_t n = j * bn + i;
            const float p = std::exp2(qk[i] - mij);
            lvec[i] = lvec[i] * alpha + p;
            const float ph = round_f16(p);
            if (n < s_kv)
              for (int d = 0; d < D; ++d) acc[d] += ph * h2f(vb[(int64_t)n * D + d]);
          }
          m = mij;
        }
        float lsum = 0.0f;
        for (int32_t i = 0; i < bn; ++i) lsum += lvec[i];
        const float lsafe = std::max(lsum, 1.0e-8f);
        for (int d = 0; d < D; ++d) o_split[(size_t)sp * D + d] = round_f16(acc[d] / lsafe);
        lse[sp] = m + std::log2(lsafe);
      }
      float lmax = -INFINITY;
      for (int32_t sp = 0; sp < nks; ++sp) lmax = std::max(lmax, lse[sp]);
      std::vector<float> w(nks);
      float wsum = 0.0f;
      for (int32_t sp = 0; sp < nks; ++sp) {
        w[sp] = std::exp2(lse[sp] - lmax);
        wsum += w[sp];
      }
      wsum = std::max(wsum, 1.0e-8f);
      for (int d = 0; d < D; ++d) {
        float o = 0.0f;
        for (int32_t sp = 0; sp < nks; ++sp) o += o_split[(size_t)sp * D + d] * (w[sp] / wsum);
        orow[d] = f2h(o);
      }
    }
  }
}

int32_t oracle_num_threads(void) { return omp_get_max_threads(); }
void oracle_set_num_threads(int32_t n) { omp_set_num_threads(n); }

}  // extern "C"
