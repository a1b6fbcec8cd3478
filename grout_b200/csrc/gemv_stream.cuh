// Weight streaming for the decode GEMVs (y = W x, one token): a CTA owns a
// contiguous block of rows of W, which is one contiguous byte range, and
// streams it through a shared-memory ring with untiled bulk copies
// (cp.async.bulk, 16 KB per copy, completion on mbarriers, never multicast).
// One producer warp issues the copies; kWarps consumer warps take 32
// consecutive 16-byte chunks (256 weights) at a time and dot them with x held
// in shared memory.  256 consecutive weights touch at most two rows when the
// row length k >= 256, so a warp splits its sum into those two rows and one
// lane adds them to the warp's own per-row slots — every sum runs in a fixed
// order, the result is deterministic.  The caller sums the warps' slots.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace grout {

constexpr int kGemvPiece = 16384;  // bytes per bulk copy
constexpr int kGemvStages = 6;     // ~96 KB in flight per CTA
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

// Barrier words: bars[0, kGemvStages) "piece landed" (count 1, transaction
// bytes), bars[kGemvStages, 2 kGemvStages) "slot free" (count kWarps).
__device__ __forceinline__ void gemv_init_bars(uint64_t* bars, int consumer_warps) {
  for (int i = 0; i < kGemvStages; ++i) {
    mbar_init(smem_u32(&bars[i]), 1);
    mbar_init(smem_u32(&bars[kGemvStages + i]), consumer_warps);
  }
  fence_mbar_init();
}

// Called by every thread of the CTA's consumer warps (warp < kWarps) and of
// the producer warp (warp == kWarps).  w_blk: the first weight of the block
// (16-byte aligned), nrows * k weights.  red: [kWarps][red_stride] f32,
// zeroed by the caller; xs: x [k] f16 in shared memory.  Returns false if a
// bounded wait gave up (recorded in *err as 0x100 + site).
template <int kWarps>
__device__ __forceinline__ bool gemv_stream_rows(const __half* w_blk, int nrows, int k,
                                                 const __half* xs, uint8_t* ring, uint64_t* bars,
                                                 float* red, int red_stride, int* err, int site,
                                                 volatile int* abort) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t blk_bytes = (int64_t)nrows * k * 2;
  const int npieces = (int)((blk_bytes + kGemvPiece - 1) / kGemvPiece);
  const uint8_t* src = reinterpret_cast<const uint8_t*>(w_blk);
  bool ok = true;
  if (warp == kWarps) {
    if (lane == 0) {
      for (int p = 0; p < npieces; ++p) {
        const int st = p % kGemvStages;
        if (p >= kGemvStages &&
            !mbar_wait(smem_u32(&bars[kGemvStages + st]), ((p / kGemvStages) - 1) & 1, err, site,
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
  constexpr int kConsumers = kWarps * 32;
  constexpr int kIter = (kGemvPiece / 16 + kConsumers - 1) / kConsumers;  // chunks per thread
  constexpr int kPieceW = kGemvPiece / 2;                                    // weights per piece
  float* my_red = red + warp * red_stride;
  // (row, col) of this thread's chunk i in the current piece, advanced by
  // one piece (kPieceW weights = q rows + rem) per step: no division in the
  // loop.
  const int q = kPieceW / k, rem = kPieceW - q * k;
  int row[kIter], col[kIter];
#pragma unroll
  for (int i = 0; i < kIter; ++i) {
    const int e = (threadIdx.x + i * kConsumers) * 8;
    row[i] = e / k;
    col[i] = e - row[i] * k;
  }
  for (int p = 0; p < npieces; ++p) {
    const int st = p % kGemvStages;
    if (!mbar_wait(smem_u32(&bars[st]), (p / kGemvStages) & 1, err, site + 1, abort)) {
      ok = false;
      break;
    }
    const int chunks = (int)(min((int64_t)kGemvPiece, blk_bytes - (int64_t)p * kGemvPiece) / 16);
    const uint8_t* buf = ring + st * kGemvPiece;
#pragma unroll
    for (int i = 0; i < kIter; ++i) {
      if (i * kConsumers < chunks) {  // block-uniform: whole chunk groups only
        const int c = threadIdx.x + i * kConsumers;
        const bool valid = c < chunks;
        // Past the end of the block (last piece only) a lane takes the last
        // row, which the valid lanes of its group reach: a group still
        // spans at most two rows.
        const int r = valid ? row[i] : nrows - 1;
        const float v = valid ? gemv_dot8(*reinterpret_cast<const uint4*>(buf + c * 16),
                                          *reinterpret_cast<const uint4*>(xs + col[i]))
                              : 0.f;
        const int row0 = __shfl_sync(0xffffffffu, r, 0);
        const int row1 = __shfl_sync(0xffffffffu, r, 31);
        float v0 = r == row0 ? v : 0.f;
        float v1 = r == row0 ? 0.f : v;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          v0 += __shfl_xor_sync(0xffffffffu, v0, off);
          v1 += __shfl_xor_sync(0xffffffffu, v1, off);
        }
        if (lane == 0) {
          my_red[row0] += v0;
          if (row1 != row0) my_red[row1] += v1;
        }
      }
      row[i] += q;
      col[i] += rem;
      if (col[i] >= k) {
        col[i] -= k;
        ++row[i];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&bars[kGemvStages + st]));
  }
  return ok;
}

}  // namespace grout
