// Weight streaming for the decode GEMVs (y = W x, one token): a CTA owns a
// contiguous block of rows of W, which is one contiguous byte range, and
// streams it through a shared-memory ring with untiled bulk copies
// (cp.async.bulk, 16 KB per copy, completion on mbarriers, never multicast).
// One producer warp issues the copies; each of kWarps consumer warps owns
// every kWarps-th row of the block and dots the parts of its rows in each
// piece with x held in shared memory, lanes striding over 16-byte chunks; a
// row's lane sums stay in registers across pieces and are reduced once, at
// the row's end.  Every sum runs in a fixed order, the result is
// deterministic.  The caller sums the warps' per-row slots (only the owner
// warp's slot of a row is non-zero).
//
// Measured on B200 (one rank, L2 flushed): a 5120 x 12800 block at 0.52 of
// the copy-measured HBM rate, cuBLAS's GEMV 0.75; a mapping that spreads
// every piece over all warps (reducing per 256 weights, or per row change)
// reached only 0.36-0.43: the consumers' shuffles, not the copies, set the
// rate (a copy-only probe of the same ring streams at 6.9 TB/s).
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace grout {

constexpr int kGemvPiece = 16384;  // bytes per bulk copy
constexpr int kGemvMaxStages = 12;  // up to 192 KB in flight per CTA
constexpr int kGemvMinK = 256;

__device__ __forceinline__ float gemv_dot8(const uint4& wv, const uint4& xv) {
  const __half2* wh = reinterpret_cast<const __half2*>(&wv);
  const __half2* xh = reinterpret_cast<const __half2*>(&xv);
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 a = __half22float2(wh[e]);
    const float2 b = __half22float2(xh[e]);
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
  }
  return acc;
}

// Barrier words: bars[0, nst) "piece landed" (count 1, transaction bytes),
// bars[kGemvMaxStages, kGemvMaxStages + nst) "slot free" (count kWarps).
__device__ __forceinline__ void gemv_init_bars(uint64_t* bars, int consumer_warps, int nst) {
  for (int i = 0; i < nst; ++i) {
    mbar_init(smem_u32(&bars[i]), 1);
    mbar_init(smem_u32(&bars[kGemvMaxStages + i]), consumer_warps);
  }
  fence_mbar_init();
}

// Called by every thread of the CTA's consumer warps (warp < kWarps) and of
// the producer warp (warp == kWarps).  w_blk: the first weight of the block
// (16-byte aligned), nrows * k weights; ring: nst <= kGemvMaxStages slots of
// kGemvPiece bytes.  red: [kWarps][red_stride] f32,
// zeroed by the caller; xs: x [k] f16 in shared memory.  Returns false if a
// bounded wait gave up (recorded in *err as 0x100 + site).
template <int kWarps>
__device__ __forceinline__ bool gemv_stream_rows(const __half* w_blk, int nrows, int k,
                                                 const __half* xs, uint8_t* ring, uint64_t* bars,
                                                 int nst, float* red, int red_stride, int* err,
                                                 int site, volatile int* abort) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t blk_bytes = (int64_t)nrows * k * 2;
  const int npieces = (int)((blk_bytes + kGemvPiece - 1) / kGemvPiece);
  const uint8_t* src = reinterpret_cast<const uint8_t*>(w_blk);
  bool ok = true;
  if (warp == kWarps) {
    if (lane == 0) {
      for (int p = 0; p < npieces; ++p) {
        const int st = p % nst;
        if (p >= nst &&
            !mbar_wait(smem_u32(&bars[kGemvMaxStages + st]), ((p / nst) - 1) & 1, err, site,
                       abort)) {
          ok = false;
          break;
        }
        const uint32_t bytes =
            (uint32_t)min((int64_t)kGemvPiece, blk_bytes - (int64_t)p * kGemvPiece);
        mbar_arrive_expect_tx(smem_u32(&bars[st]), bytes);
        bulk_load(smem_u32(ring + st * kGemvPiece), src + (int64_t)p * kGemvPiece, bytes,
                  smem_u32(&bars[st]));
      }
    }
    return ok;
  }
  // Warp w owns rows w, w + kWarps, ... of the block.  Every warp walks all
  // pieces in order — waits for each, adds the chunks of its rows that lie
  // in it, and releases it — so a slot is refilled once all warps are past
  // it.
  constexpr int kPieceChunks = kGemvPiece / 16;
  const int cpr = k / 8;  // 16-byte chunks per row
  const int total = nrows * cpr;  // < 2^31: a CTA's block is at most tens of MB
  float* my_red = red + warp * red_stride;
  int r = warp;
  float acc = 0.f;
  for (int p = 0; p < npieces; ++p) {
    const int st = p % nst;
    if (!mbar_wait(smem_u32(&bars[st]), (p / nst) & 1, err, site + 1, abort)) {
      ok = false;
      break;
    }
    const int c0 = p * kPieceChunks;
    const int c1 = min(c0 + kPieceChunks, total);
    const uint8_t* buf = ring + st * kGemvPiece;
    while (r < nrows) {
      const int rs = r * cpr, re = rs + cpr;
      if (rs >= c1) break;  // the row starts in a later piece
      const int lo = max(rs, c0), hi = min(re, c1);
      // four chunks per lane in flight (independent sums), then the rest
      int c = lo + lane;
      float a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (; c + 96 < hi; c += 128) {
        uint4 wv[4], xv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          wv[u] = *reinterpret_cast<const uint4*>(buf + (c + 32 * u - c0) * 16);
          xv[u] = *reinterpret_cast<const uint4*>(xs + (c + 32 * u - rs) * 8);
        }
        acc += gemv_dot8(wv[0], xv[0]);
        a1 += gemv_dot8(wv[1], xv[1]);
        a2 += gemv_dot8(wv[2], xv[2]);
        a3 += gemv_dot8(wv[3], xv[3]);
      }
      for (; c < hi; c += 32)
        acc += gemv_dot8(*reinterpret_cast<const uint4*>(buf + (c - c0) * 16),
                         *reinterpret_cast<const uint4*>(xs + (c - rs) * 8));
      acc += (a1 + a2) + a3;
      if (re > c1) break;  // the row goes on in the next piece
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane == 0) my_red[r] = acc;
      acc = 0.f;
      r += kWarps;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&bars[kGemvMaxStages + st]));
  }
  return ok;
}

}  // namespace grout
