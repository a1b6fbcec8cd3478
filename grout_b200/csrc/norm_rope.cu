// Fused per-head RMSNorm + RoPE + KV-cache write (prefill and decode).
//
// Replaces qk_norm_rope_kv_prefill_raw_f16 / qk_norm_rope_kv_decode_raw_f16
// (reference src/kernels.rs:4845-5168, 5180-5452).  HBM-bound: every byte of
// q/k/v is read once and every output byte written once.
//
// Mapping: one half-warp (16 lanes) per 128-element head row.  Lane j owns
// the RoPE pairs i = 4j..4j+3, i.e. x[4j..4j+4) ("lo") and x[64+4j..64+4j+4)
// ("hi"), so rotate-half needs no shuffle and each half-warp load instruction
// covers two 128-byte segments.  The arithmetic is pinned so that the CPU
// oracle reproduces it bit for bit: no FMA contraction (explicit _rn
// intrinsics), a fixed sum order (lane sum (t0+t1)+(t2+t3), then a
// xor-butterfly 8,4,2,1), rsqrt as 1/sqrt with IEEE rounding, and cos/sin
// read from a table of correctly rounded values of the reference's f32 angle.
#include "internal.h"
#include "ptx.cuh"

namespace grout {

__device__ __forceinline__ void ld_half4(const __half* p, float (&f)[4]) {
  uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  __half2 a = *reinterpret_cast<__half2*>(&u.x);
  __half2 b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  f[0] = fa.x; f[1] = fa.y; f[2] = fb.x; f[3] = fb.y;
}

__device__ __forceinline__ void st_half4(__half* p, const float (&f)[4]) {
  __half2 a = __halves2half2(__float2half_rn(f[0]), __float2half_rn(f[1]));
  __half2 b = __halves2half2(__float2half_rn(f[2]), __float2half_rn(f[3]));
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(const NormRopeArgs a) {
  const int j = threadIdx.x & 15;  // lane within the half-warp
  const unsigned mask = 0xFFFFu << (threadIdx.x & 16);
  const int heads = a.hq + a.hkv;
  const int64_t ntask = (int64_t)a.rows * heads;
  const int64_t step = ((int64_t)gridDim.x * blockDim.x) >> 4;
  for (int64_t task = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4; task < ntask;
       task += step) {
    const int s = (int)(task / heads);
    const int hh = (int)(task - (int64_t)s * heads);
    const bool is_q = hh < a.hq;
    const int kh = hh - a.hq;
    const __half* src;
    const __half* vsrc = nullptr;
    __half* dst;
    __half* vdst = nullptr;
    int64_t pos;
    if (a.decode) {
      pos = a.d_position[s];
      if (pos >= a.max_seq) {
        if (j == 0 && hh == 0 && a.err) atomicCAS(a.err, 0, DEV_ERR_POSITION);
        continue;
      }
      const __half* row = a.q + (int64_t)s * a.q_row_stride;
      src = row + (int64_t)hh * kHeadDim;
      if (is_q) {
        dst = a.q_out + ((int64_t)s * a.hq + hh) * kHeadDim;
      } else {
        const int64_t off = (int64_t)s * a.cache_batch_stride + kh * a.cache_head_stride + pos * kHeadDim;
        dst = a.k_cache + off;
        vdst = a.v_cache + off;
        vsrc = row + (int64_t)(a.hq + a.hkv + kh) * kHeadDim;
      }
    } else {
      pos = (int64_t)a.pos0 + s;
      if (is_q) {
        src = a.q + (int64_t)s * a.q_row_stride + (int64_t)hh * kHeadDim;
        dst = a.q_out + (int64_t)s * a.q_row_stride + (int64_t)hh * kHeadDim;
      } else {
        src = a.k + (int64_t)s * a.kv_row_stride + (int64_t)kh * kHeadDim;
        vsrc = a.v + (int64_t)s * a.kv_row_stride + (int64_t)kh * kHeadDim;
        const int64_t off = kh * a.cache_head_stride + pos * kHeadDim;
        dst = a.k_cache + off;
        vdst = a.v_cache + off;
      }
    }
    // V: verbatim copy, issued first so it overlaps the norm math.
    if (vsrc) {
      const uint2 v0 = __ldg(reinterpret_cast<const uint2*>(vsrc + 4 * j));
      const uint2 v1 = __ldg(reinterpret_cast<const uint2*>(vsrc + 64 + 4 * j));
      *reinterpret_cast<uint2*>(vdst + 4 * j) = v0;
      *reinterpret_cast<uint2*>(vdst + 64 + 4 * j) = v1;
    }
    float lo[4], hi[4], wl[4], wh[4];
    ld_half4(src + 4 * j, lo);
    ld_half4(src + 64 + 4 * j, hi);
    const __half* w = is_q ? a.q_w : a.k_w;
    ld_half4(w + 4 * j, wl);
    ld_half4(w + 64 + 4 * j, wh);
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(a.table + pos * kHeadDim + 4 * j));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(a.table + pos * kHeadDim + 64 + 4 * j));
    const float cs[4] = {c4.x, c4.y, c4.z, c4.w};
    const float sn[4] = {s4.x, s4.y, s4.z, s4.w};

    float t[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) t[e] = __fadd_rn(__fmul_rn(lo[e], lo[e]), __fmul_rn(hi[e], hi[e]));
    float ss = __fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3]));
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(mask, ss, off, 16));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps)));

    float ylo[4], yhi[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float nlo = __fmul_rn(__fmul_rn(lo[e], inv), wl[e]);
      const float nhi = __fmul_rn(__fmul_rn(hi[e], inv), wh[e]);
      ylo[e] = __fsub_rn(__fmul_rn(nlo, cs[e]), __fmul_rn(nhi, sn[e]));
      yhi[e] = __fadd_rn(__fmul_rn(nhi, cs[e]), __fmul_rn(nlo, sn[e]));
    }
    st_half4(dst + 4 * j, ylo);
    st_half4(dst + 64 + 4 * j, yhi);
  }
}

cudaError_t launch_qk_norm_rope_kv(const NormRopeArgs& a, int num_sms, cudaStream_t s) {
  const int64_t ntask = (int64_t)a.rows * (a.hq + a.hkv);
  if (ntask == 0) return cudaSuccess;
  const int per_block = 256 / 16;
  int64_t blocks = (ntask + per_block - 1) / per_block;
  const int64_t cap = (int64_t)num_sms * 8;  // 8 resident 256-thread blocks per SM
  if (blocks > cap) blocks = cap;
  qk_norm_rope_kv_kernel<<<(unsigned)blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace grout
