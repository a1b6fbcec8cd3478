// Fused per-head RMSNorm + RoPE + KV-cache write (prefill and decode).
//
// Replaces qk_norm_rope_kv_prefill_raw_f16 / qk_norm_rope_kv_decode_raw_f16
// (reference src/kernels.rs:4845-5168, 5180-5452).  HBM-bound: every byte of
// q/k/v is read once and every output byte written once.
//
// Mapping: one octet (8 lanes) per 128-element head row, so a warp works on
// four rows at once, in a grid-stride loop over (token, head) rows; the row
// arithmetic (norm_rope.cuh) is pinned so that the CPU oracle reproduces it
// bit for bit.  Two restructurings measured slower on B200 (both timed
// against this kernel in the same GPU call, config 2, S = 4096): a warp per
// (token, 16-row slab) with the weights in registers, 38.9 vs 34.8 us, and
// octets that keep one head and walk over tokens, 41.0 vs 32.8-34.8 us —
// fewer instructions, but fewer rows in flight per SM.
#include "internal.h"
#include "norm_rope.cuh"
#include "ptx.cuh"

namespace grout {

// kPaged: K/V rows go to a page pool (page_table); the contiguous
// instantiation carries no page lookup.
template <bool kPaged>
__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(const NormRopeArgs a) {
  const int j = threadIdx.x & 7;  // lane within the octet
  const unsigned mask = 0xFFu << (threadIdx.x & 24);
  const uint32_t heads = (uint32_t)(a.hq + a.hkv);
  const uint32_t ntask = (uint32_t)a.rows * heads;
  const uint32_t step = (gridDim.x * blockDim.x) >> 3;
  for (uint32_t task = (blockIdx.x * blockDim.x + threadIdx.x) >> 3; task < ntask; task += step) {
    const uint32_t s = task / heads;
    const int hh = (int)(task - s * heads);
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
        int64_t off = (int64_t)s * a.cache_batch_stride + kh * a.cache_head_stride + pos * kHeadDim;
        if (kPaged) {
          const int64_t pg = pos / a.page_size;
          const int32_t page = a.page_table[(int64_t)s * a.table_stride + pg];
          if (page < 0 || page >= a.num_pages) {
            if (j == 0 && a.err) atomicCAS(a.err, 0, DEV_ERR_PAGE);
            continue;
          }
          off = ((int64_t)page * a.hkv + kh) * a.page_size * kHeadDim + (pos - pg * a.page_size) * kHeadDim;
        }
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
        int64_t off = kh * a.cache_head_stride + pos * kHeadDim;
        if (kPaged) {
          const int64_t pg = pos / a.page_size;
          const int32_t page = a.page_table[pg];
          if (page < 0 || page >= a.num_pages) {
            if (j == 0 && a.err) atomicCAS(a.err, 0, DEV_ERR_PAGE);
            continue;
          }
          off = ((int64_t)page * a.hkv + kh) * a.page_size * kHeadDim + (pos - pg * a.page_size) * kHeadDim;
        }
        dst = a.k_cache + off;
        vdst = a.v_cache + off;
      }
    }
    // Issue every load of the row first.
    const uint4 xl = ldg16(src + 8 * j);
    const uint4 xh = ldg16(src + 64 + 8 * j);
    uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
    if (vsrc) {
      v0 = ldg16(vsrc + 8 * j);
      v1 = ldg16(vsrc + 64 + 8 * j);
    }
    const __half* w = is_q ? a.q_w : a.k_w;
    const uint4 wl4 = ldg16(w + 8 * j);
    const uint4 wh4 = ldg16(w + 64 + 8 * j);
    const float* trow = a.table + pos * kHeadDim;
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(trow + 8 * j));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(trow + 8 * j + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(trow + 64 + 8 * j));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(trow + 64 + 8 * j + 4));
    if (vsrc) {  // V: verbatim copy
      *reinterpret_cast<uint4*>(vdst + 8 * j) = v0;
      *reinterpret_cast<uint4*>(vdst + 64 + 8 * j) = v1;
    }
    float wl[8], wh[8];
    unpack8(wl4, wl);
    unpack8(wh4, wh);
    const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    uint4 ylo, yhi;
    octet_norm_rope(xl, xh, wl, wh, cs, sn, a.eps, mask, ylo, yhi);
    *reinterpret_cast<uint4*>(dst + 8 * j) = ylo;
    *reinterpret_cast<uint4*>(dst + 64 + 8 * j) = yhi;
  }
}

cudaError_t launch_qk_norm_rope_kv(const NormRopeArgs& a, int num_sms, cudaStream_t s) {
  const int64_t ntask = (int64_t)a.rows * (a.hq + a.hkv);
  if (ntask == 0) return cudaSuccess;
  const int per_block = 256 / 8;
  int64_t blocks = (ntask + per_block - 1) / per_block;
  const int64_t cap = (int64_t)num_sms * 8;  // 8 resident 256-thread blocks per SM
  if (blocks > cap) blocks = cap;
  if (a.page_table)
    qk_norm_rope_kv_kernel<true><<<(unsigned)blocks, 256, 0, s>>>(a);
  else
    qk_norm_rope_kv_kernel<false><<<(unsigned)blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace grout
