// The per-row arithmetic of the fused Q/K RMSNorm + RoPE write, shared by the
// standalone kernel (norm_rope.cu) and the fused decode kernel (decode.cu) so
// that both produce the same bits by construction.
//
// One octet (8 lanes) holds a 128-element head row: lane j of the octet owns
// the RoPE pairs i = 8j..8j+7, i.e. x[8j..8j+8) ("lo") and x[64+8j..64+8j+8)
// ("hi"), so rotate-half needs no shuffle and every access is 16 bytes.  The
// arithmetic is pinned so that the CPU oracle reproduces it bit for bit: no
// FMA contraction (explicit _rn intrinsics), a fixed sum order (lane sum
// ((t0+t1)+(t2+t3))+((t4+t5)+(t6+t7)), then an xor butterfly 4,2,1 over the
// octet), rsqrt as a correctly rounded reciprocal of a correctly rounded
// sqrt, and cos/sin read from a table of correctly rounded values of the
// reference's f32 angle f32(pos) * inv_freq[i] (src/kernels.rs:5012-5084).
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

namespace grout {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 v = __half22float2(h);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Lane j's cos (cs) and sin (sn) values of table row `trow` ([2][64] f32).
__device__ __forceinline__ void load_cos_sin(const float* trow, int j, float (&cs)[8],
                                             float (&sn)[8]) {
  const float4 c0 = __ldg(reinterpret_cast<const float4*>(trow + 8 * j));
  const float4 c1 = __ldg(reinterpret_cast<const float4*>(trow + 8 * j + 4));
  const float4 s0 = __ldg(reinterpret_cast<const float4*>(trow + 64 + 8 * j));
  const float4 s1 = __ldg(reinterpret_cast<const float4*>(trow + 64 + 8 * j + 4));
  cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
  cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
  sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
  sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
}

// RMSNorm of the octet's row (x = [xl | xh] as lane j's 16-byte chunks),
// scaled by the norm weight (wl, wh), rotated by (cs, sn) and rounded to f16
// once.  `mask` is the octet's lane mask for the butterfly.
__device__ __forceinline__ void octet_norm_rope(const uint4& xl, const uint4& xh,
                                                const float (&wl)[8], const float (&wh)[8],
                                                const float (&cs)[8], const float (&sn)[8],
                                                float eps, unsigned mask, uint4& out_lo,
                                                uint4& out_hi) {
  float lo[8], hi[8];
  unpack8(xl, lo);
  unpack8(xh, hi);
  float t[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) t[e] = __fadd_rn(__fmul_rn(lo[e], lo[e]), __fmul_rn(hi[e], hi[e]));
  float ss = __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3])),
                       __fadd_rn(__fadd_rn(t[4], t[5]), __fadd_rn(t[6], t[7])));
#pragma unroll
  for (int off = 4; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(mask, ss, off, 8));
  // ss / 128 is an exact power-of-two scaling; the correctly rounded
  // reciprocal equals the IEEE quotient 1.0f / x.
  const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(ss, 0.0078125f), eps)));
  float ylo[8], yhi[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float nlo = __fmul_rn(__fmul_rn(lo[e], inv), wl[e]);
    const float nhi = __fmul_rn(__fmul_rn(hi[e], inv), wh[e]);
    ylo[e] = __fsub_rn(__fmul_rn(nlo, cs[e]), __fmul_rn(nhi, sn[e]));
    yhi[e] = __fadd_rn(__fmul_rn(nhi, cs[e]), __fmul_rn(nlo, sn[e]));
  }
  out_lo = pack8(ylo);
  out_hi = pack8(yhi);
}

}  // namespace grout
