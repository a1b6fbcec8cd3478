// Split-K GQA decode attention + LSE merge.
//
// Replaces fmha_decode_gqa_split + splitk_reduce_merge (reference
// src/kernels.rs:4016-4304), generalised to a batch of sequences.
//
// HBM-bound streaming kernel.  One CTA per (split, kv head, sequence).
//   - warp 4 (producer): TMA tile loads (128B swizzle, no multicast) of 64-key
//     K and V tiles into a 3-stage shared-memory ring, completion on mbarriers;
//   - warps 0-3 (consumers): each takes 16 of the 64 keys of a stage.  All G
//     query heads of the GQA group share every K/V byte read.  S^T = K Q^T and
//     O^T += V^T P^T run on mma.sync m16n8k16 with the group on N (8 columns:
//     G <= 8 heads): the keys/head_dim sit on M, so no MMA row is padding for
//     G = 8.  P goes from the S^T accumulator to the B operand of the PV MMA
//     with one movmatrix transpose per 8x8 block.  Online softmax in log2
//     space with quad-shuffle row maxima.
//   - the four warps' (m, l, O) are merged through shared memory; with one
//     split the CTA writes the f16 output directly, otherwise the normalised
//     split output (f32) and its log2-sum-exp go to the caller's workspace
//     and a small merge kernel combines the splits.
// Numerics follow the reference's decode: scores scaled by qk_scale / ln 2
// after the dot product, keys >= kv_len masked, P rounded to f16 for the PV
// product, f32 accumulation.  Differences: split outputs are kept in f32
// instead of f16 (one rounding fewer).
#include "internal.h"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kKeys = 64;                  // keys per stage
constexpr int kStages = 3;
constexpr int kBoxBytes = kKeys * 128;     // one 64-column box of one tile
constexpr int kTileBytes = 2 * kBoxBytes;  // 64 keys x 128 dims x f16
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kThreads = 160;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;

struct RedSmem {
  float o[4][128][9];  // padded: the per-dimension merge reads are conflict-free
  float m[4][8];
  float l[4][8];
};
static_assert(sizeof(RedSmem) <= kStages * kStageBytes, "reduction area must fit in the ring");

__global__ void __launch_bounds__(kThreads, 2)
    decode_split_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kStages);

  const int split = blockIdx.x;
  const int kh = blockIdx.y;
  const int b = blockIdx.z;
  const int G = a.hq / a.hkv;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int kv_len = (int)a.d_position[b] + 1;
  const int n_tiles = (kv_len + kKeys - 1) / kKeys;
  const int tps = (n_tiles + a.nks - 1) / a.nks;
  const int t0 = split * tps;
  const int t1 = min(t0 + tps, n_tiles);
  const int nt = t1 - t0;
  const int64_t head0 = (int64_t)b * a.hq + (int64_t)kh * G;

  if (nt <= 0) {  // empty split (only when nks > 1): weight 0 in the merge
    if (threadIdx.x < 128) {
      for (int g = 0; g < G; ++g) {
        a.part_o[((head0 + g) * a.nks + split) * 128 + threadIdx.x] = 0.0f;
        if (threadIdx.x == 0) a.part_lse[(head0 + g) * a.nks + split] = -INFINITY;
      }
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&bars[i]), 1);
      mbar_init(smem_u32(&bars[kStages + i]), 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // Consumer state lives at function scope so it survives the CTA barrier
  // that frees the ring for the cross-warp merge.
  const int g = lane >> 2;  // MMA row group: key (S^T) / dim (O^T) offset; head for Q
  const int t = lane & 3;   // MMA column pair: heads 2t, 2t+1
  float m0 = -1.0e30f, m1 = -1.0e30f, l0 = 0.f, l1 = 0.f;
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      for (int it = 0; it < nt; ++it) {
        const int st = it % kStages;
        const int r = it / kStages;
        if (r > 0 && !mbar_wait(smem_u32(&bars[kStages + st]), (r - 1) & 1, a.err, 1, abort_flag))
          break;
        const uint32_t full = smem_u32(&bars[st]);
        mbar_arrive_expect_tx(full, kStageBytes);
        const uint32_t kb = smem_u32(smem + st * kStageBytes);
        const uint32_t vb = kb + kTileBytes;
        int row = (t0 + it) * kKeys;
        int outer = b;  // sequence (contiguous caches) or page (paged pool)
        if (a.page_table) {
          // a 64-key tile never straddles a page (page_size % 64 == 0)
          const int pg = row / a.page_size;
          outer = __ldg(a.page_table + (int64_t)b * a.table_stride + pg);
          row -= pg * a.page_size;
          // an entry outside the pool reads the TMA fill (zeros): report it
          if ((outer < 0 || outer >= a.num_pages) && a.err) atomicCAS(a.err, 0, DEV_ERR_PAGE);
        }
        tma_load_4d(kb, &tm_k, full, 0, row, kh, outer);
        tma_load_4d(kb + kBoxBytes, &tm_k, full, 64, row, kh, outer);
        tma_load_4d(vb, &tm_v, full, 0, row, kh, outer);
        tma_load_4d(vb + kBoxBytes, &tm_v, full, 64, row, kh, outer);
      }
    }
  } else {
    // ----------------------------------------------------------- consumers
    uint32_t qb[8][2];
    {
      const __half* qp = a.q + (head0 + g) * 128;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        if (g < G) {
          qb[kk][0] = __ldg(reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * t));
          qb[kk][1] = __ldg(reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * t + 8));
        } else {
          qb[kk][0] = 0u;
          qb[kk][1] = 0u;
        }
      }
    }
    const float sl2 = a.scale_log2;
    const int a_row = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int a_chs = lane >> 4;
    const int v_row = 16 * warp + (lane & 7) + ((lane >> 4) & 1) * 8;
    const int v_chs = (lane >> 3) & 1;

    for (int it = 0; it < nt; ++it) {
      const int st = it % kStages;
      if (!mbar_wait(smem_u32(&bars[st]), (it / kStages) & 1, a.err, 2, abort_flag)) break;
      const uint32_t kb = smem_u32(smem + st * kStageBytes);
      const uint32_t vb = kb + kTileBytes;

      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int c = 2 * kk + a_chs;
        const uint32_t addr =
            kb + (c >> 3) * kBoxBytes + a_row * 128 + (((c & 7) ^ (a_row & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(addr, a0, a1, a2, a3);
        mma16816(sc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
      // sc: [0],[1] key g (heads 2t, 2t+1); [2],[3] key g+8.
      float s0 = sc[0] * sl2, s1 = sc[1] * sl2, s2 = sc[2] * sl2, s3 = sc[3] * sl2;
      const int kbase = (t0 + it) * kKeys + 16 * warp;
      if (kbase + 16 > kv_len) {
        if (kbase + g >= kv_len) s0 = s1 = -INFINITY;
        if (kbase + g + 8 >= kv_len) s2 = s3 = -INFINITY;
      }
      float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = ex2(m0 - mn0), al1 = ex2(m1 - mn1);
      const float p0 = ex2(s0 - mn0), p1 = ex2(s1 - mn1);
      const float p2 = ex2(s2 - mn0), p3 = ex2(s3 - mn1);
      l0 = l0 * al0 + (p0 + p2);
      l1 = l1 * al1 + (p1 + p3);
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
      }
      const uint32_t pb0 = movm_t(pack_half2(p0, p1));
      const uint32_t pb1 = movm_t(pack_half2(p2, p3));
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int c = 2 * mt + v_chs;
        const uint32_t addr =
            vb + (c >> 3) * kBoxBytes + v_row * 128 + (((c & 7) ^ (v_row & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(addr, a0, a1, a2, a3);
        mma16816(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[kStages + st]));
    }
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
  }
  __syncthreads();  // every stage consumed: the ring becomes the merge area
  if (*abort_flag) return;

  RedSmem* red = reinterpret_cast<RedSmem*>(smem);
  if (warp < 4) {
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      red->o[warp][16 * mt + g][2 * t] = o[mt][0];
      red->o[warp][16 * mt + g][2 * t + 1] = o[mt][1];
      red->o[warp][16 * mt + g + 8][2 * t] = o[mt][2];
      red->o[warp][16 * mt + g + 8][2 * t + 1] = o[mt][3];
    }
    if (g == 0) {
      red->m[warp][2 * t] = m0;
      red->m[warp][2 * t + 1] = m1;
      red->l[warp][2 * t] = l0;
      red->l[warp][2 * t + 1] = l1;
    }
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const int d = threadIdx.x;
    for (int hd = 0; hd < G; ++hd) {
      float M = red->m[0][hd];
#pragma unroll
      for (int w = 1; w < 4; ++w) M = fmaxf(M, red->m[w][hd]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float sc = ex2(red->m[w][hd] - M);
        L += red->l[w][hd] * sc;
        O += red->o[w][d][hd] * sc;
      }
      const float res = O / L;
      if (a.nks == 1) {
        a.out[(head0 + hd) * 128 + d] = __float2half_rn(res);
      } else {
        a.part_o[((head0 + hd) * a.nks + split) * 128 + d] = res;
        if (d == 0) a.part_lse[(head0 + hd) * a.nks + split] = M + __log2f(L);
      }
    }
  }
}

// Merge of the split outputs (splitk_reduce_merge, src/kernels.rs:4201-4304):
// w_s = 2^(lse_s - max) / sum, out = sum_s w_s * O_s, rounded to f16.
// One CTA per (sequence, query head), one thread per head dimension.
__global__ void __launch_bounds__(128) decode_merge_kernel(const DecodeArgs a) {
  const int64_t row = blockIdx.x;
  const int d = threadIdx.x;
  const float* lse = a.part_lse + row * a.nks;
  float M = -INFINITY;
  for (int s = 0; s < a.nks; ++s) M = fmaxf(M, lse[s]);
  float W = 0.f, O = 0.f;
  for (int s = 0; s < a.nks; ++s) {
    const float w = ex2(lse[s] - M);
    W += w;
    O += w * a.part_o[(row * a.nks + s) * 128 + d];
  }
  a.out[row * 128 + d] = __float2half_rn(O / W);
}

}  // namespace

cudaError_t decode_set_attributes() {
  return cudaFuncSetAttribute(decode_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSmemBytes);
}

cudaError_t launch_decode(const DecodeArgs& a, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                          cudaStream_t s) {
  dim3 grid(a.nks, a.hkv, a.batch);
  decode_split_kernel<<<grid, kThreads, kSmemBytes, s>>>(tm_k, tm_v, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || a.nks == 1) return e;
  decode_merge_kernel<<<(unsigned)((int64_t)a.batch * a.hq), 128, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace grout
