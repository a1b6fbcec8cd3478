// Fused per-head RMSNorm + RoPE + KV-cache write (prefill and decode).
//
// Replaces qk_norm_rope_kv_prefill_raw_f16 / qk_norm_rope_kv_decode_raw_f16
// (reference src/kernels.rs:4845-5168, 5180-5452).  HBM-bound: every byte of
// q/k/v is read once and every output byte written once.
//
// Mapping: one octet (8 lanes) per 128-element head row (norm_rope.cuh holds
// the row arithmetic, pinned so that the CPU oracle reproduces it bit for
// bit); a warp takes 16 rows of one token at a time.
#include "internal.h"
#include "norm_rope.cuh"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kSlabRows = 16;  // head rows of one token per warp task (4 per octet)

// Row layout of one token: rows [0, hq) are Q heads (normalised with q_w),
// [hq, hq + hkv) K heads (k_w), [hq + hkv, hq + 2 hkv) V heads (copied).
//
// A warp task is (token, slab of 16 rows); octet o of the warp takes rows
// slab*16 + 4i + o, i < 4, issuing all four rows' loads before any math.  The
// norm weights live in registers for the whole kernel and the token's cos/sin
// row is loaded once per task, so per row only the row itself is read.
// kPaged: K/V rows go to a page pool (page_table); the contiguous
// instantiation carries no page lookup.
template <bool kPaged>
__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(const NormRopeArgs a) {
  const int j = threadIdx.x & 7;  // lane within the octet
  const int octet = (threadIdx.x >> 3) & 3;
  const unsigned mask = 0xFFu << (threadIdx.x & 24);
  const int R = a.hq + 2 * a.hkv;
  const int slabs = (R + kSlabRows - 1) / kSlabRows;
  const uint32_t ntask = (uint32_t)a.rows * (uint32_t)slabs;
  const uint32_t warps = (gridDim.x * blockDim.x) >> 5;

  float qwl[8], qwh[8], kwl[8], kwh[8];
  unpack8(ldg16(a.q_w + 8 * j), qwl);
  unpack8(ldg16(a.q_w + 64 + 8 * j), qwh);
  unpack8(ldg16(a.k_w + 8 * j), kwl);
  unpack8(ldg16(a.k_w + 64 + 8 * j), kwh);

  for (uint32_t task = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; task < ntask; task += warps) {
    const uint32_t s = task / (uint32_t)slabs;
    const int r0 = (int)(task - s * (uint32_t)slabs) * kSlabRows;
    int64_t pos;
    const __half* qsrc;      // this token's Q / K / V head-0 rows
    const __half* ksrc;
    const __half* vsrc;
    __half* qdst;
    int64_t kv_off;          // element offset of this token's K/V row of head 0
    int64_t kv_head_stride;  // elements between KV heads in the cache
    if (a.decode) {
      pos = a.d_position[s];
      if (pos >= a.max_seq) {
        if (r0 == 0 && (threadIdx.x & 31) == 0 && a.err) atomicCAS(a.err, 0, DEV_ERR_POSITION);
        continue;
      }
      qsrc = a.q + (int64_t)s * a.q_row_stride;
      ksrc = qsrc + (int64_t)a.hq * kHeadDim;
      vsrc = ksrc + (int64_t)a.hkv * kHeadDim;
      qdst = a.q_out + (int64_t)s * a.hq * kHeadDim;
      kv_off = (int64_t)s * a.cache_batch_stride + pos * kHeadDim;
    } else {
      pos = (int64_t)a.pos0 + s;
      qsrc = a.q + (int64_t)s * a.q_row_stride;
      ksrc = a.k + (int64_t)s * a.kv_row_stride;
      vsrc = a.v + (int64_t)s * a.kv_row_stride;
      qdst = a.q_out + (int64_t)s * a.q_row_stride;
      kv_off = pos * kHeadDim;
    }
    kv_head_stride = a.cache_head_stride;
    bool kv_ok = true;
    if (kPaged) {
      const int64_t pg = pos / a.page_size;
      const int32_t page = a.page_table[(a.decode ? (int64_t)s * a.table_stride : 0) + pg];
      kv_ok = page >= 0 && page < a.num_pages;
      kv_off = (int64_t)page * a.hkv * a.page_size * kHeadDim + (pos - pg * a.page_size) * kHeadDim;
      kv_head_stride = (int64_t)a.page_size * kHeadDim;
      if (!kv_ok && r0 + kSlabRows > a.hq && (threadIdx.x & 31) == 0 && a.err)
        atomicCAS(a.err, 0, DEV_ERR_PAGE);
    }
    // Issue every load of the slab first.
    uint4 xl[4], xh[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = r0 + 4 * i + octet;
      const __half* src = r < a.hq ? qsrc + (int64_t)r * kHeadDim
                        : r < a.hq + a.hkv ? ksrc + (int64_t)(r - a.hq) * kHeadDim
                                           : vsrc + (int64_t)(r - a.hq - a.hkv) * kHeadDim;
      if (r < R) {
        xl[i] = ldg16(src + 8 * j);
        xh[i] = ldg16(src + 64 + 8 * j);
      }
    }
    float cs[8], sn[8];
    if (r0 < a.hq + a.hkv) load_cos_sin(a.table + pos * kHeadDim, j, cs, sn);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = r0 + 4 * i + octet;
      if (r >= R) continue;
      if (r >= a.hq + a.hkv) {  // V: verbatim copy
        if (!kv_ok) continue;
        __half* dst = a.v_cache + kv_off + (int64_t)(r - a.hq - a.hkv) * kv_head_stride;
        *reinterpret_cast<uint4*>(dst + 8 * j) = xl[i];
        *reinterpret_cast<uint4*>(dst + 64 + 8 * j) = xh[i];
        continue;
      }
      const bool is_q = r < a.hq;
      uint4 ylo, yhi;
      octet_norm_rope(xl[i], xh[i], is_q ? qwl : kwl, is_q ? qwh : kwh, cs, sn, a.eps, mask, ylo,
                      yhi);
      __half* dst = is_q ? qdst + (int64_t)r * kHeadDim
                         : a.k_cache + kv_off + (int64_t)(r - a.hq) * kv_head_stride;
      if (!is_q && !kv_ok) continue;
      *reinterpret_cast<uint4*>(dst + 8 * j) = ylo;
      *reinterpret_cast<uint4*>(dst + 64 + 8 * j) = yhi;
    }
  }
}

}  // namespace

cudaError_t launch_qk_norm_rope_kv(const NormRopeArgs& a, int num_sms, cudaStream_t s) {
  const int R = a.hq + 2 * a.hkv;
  const int64_t ntask = (int64_t)a.rows * ((R + kSlabRows - 1) / kSlabRows);
  if (ntask == 0) return cudaSuccess;
  const int per_block = 256 / 32;
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
