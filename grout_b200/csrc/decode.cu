// Split-K GQA decode attention + LSE merge, optionally fused with the decode
// step's Q/K RMSNorm + RoPE + KV-cache write.
//
// Replaces fmha_decode_gqa_split + splitk_reduce_merge (reference
// src/kernels.rs:4016-4304), generalised to a batch of sequences; the fused
// form also replaces qk_norm_rope_kv_decode_raw_f16 (src/kernels.rs:
// 5180-5452), which the reference launches right before it in the decode
// graph (src/model.rs:3494ff, 3728-3771).
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
//     split the CTA writes the f16 output directly.  With several splits each
//     CTA produces its normalised split output (f32) and log2-sum-exp, and
//       * kCluster: the splits of one (kv head, sequence) form one thread-block
//         cluster (<= 16 CTAs) and merge through distributed shared memory —
//         no workspace and no second launch;
//       * otherwise: the split outputs go to the caller's workspace and a
//         small merge kernel combines them.
//     Both merges run the same arithmetic in the same order, so the two forms
//     give identical bits.
//   - kFused: before streaming, each CTA normalises and rotates its G query
//     rows itself from the QKV row (the same octet arithmetic as the
//     standalone fused kernel, norm_rope.cuh, so the bits are the same); the
//     CTA whose split holds the new position also writes that position's K
//     (normalised, rotated) and V rows into the cache, and its producer loads
//     the tile holding them only after those stores are visible to TMA.
// Numerics follow the reference's decode: scores scaled by qk_scale / ln 2
// after the dot product, keys >= kv_len masked, P rounded to f16 for the PV
// product, f32 accumulation.  Differences: split outputs are kept in f32
// instead of f16 (one rounding fewer).
//
// Range checks on the device: a position >= max_seq records device error
// 0x200 and the sequence's output is zero (no cache access); a page-table
// entry outside [0, num_pages) records 0x201, its tile is loaded from page 0
// instead and masked out of the softmax.
#include "internal.h"
#include "norm_rope.cuh"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kKeys = 64;                  // keys per stage
constexpr int kStages = 3;
constexpr int kBoxBytes = kKeys * 128;     // one 64-column box of one tile
constexpr int kTileBytes = 2 * kBoxBytes;  // 64 keys x 128 dims x f16
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kThreads = 160;
constexpr int kRingBytes = kStages * kStageBytes;
// after the ring: full/empty/ready barriers, abort flag, per-stage tile masks,
// then the fused path's query rows [8][128] f16
constexpr int kCtlBytes = 128;
constexpr int kQsBytes = 8 * 128 * 2;
constexpr int kSmemBytes = kRingBytes + 1024 + kCtlBytes + kQsBytes;

struct RedSmem {
  float o[4][128][9];  // padded: the per-dimension merge reads are conflict-free
  float m[4][8];
  float l[4][8];
};
// A CTA's final split result, read by the other CTAs of its cluster.
struct FinSmem {
  float o[8][128];
  float lse[8];
};
constexpr int kFinOffset = 20480;
static_assert(sizeof(RedSmem) <= kFinOffset, "reduction area overlaps the split result");
static_assert(kFinOffset + sizeof(FinSmem) <= kRingBytes, "merge areas must fit in the ring");

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// The merge of split results (splitk_reduce_merge, src/kernels.rs:4201-4304):
// w_s = 2^(lse_s - max) / sum, out = sum_s w_s * O_s, rounded to f16.  An
// all-empty row (every lse = -inf: a sequence skipped by the range check)
// gives 0.  get(s) returns (lse_s, O_s[d]).
template <typename Get>
__device__ __forceinline__ __half merge_splits(int nks, Get get) {
  float M = -INFINITY;
  for (int s = 0; s < nks; ++s) M = fmaxf(M, get(s, true));
  if (M == -INFINITY) return __float2half_rn(0.f);
  float W = 0.f, O = 0.f;
  for (int s = 0; s < nks; ++s) {
    const float w = ex2(get(s, true) - M);
    W += w;
    O += w * get(s, false);
  }
  return __float2half_rn(O / W);
}

template <bool kPaged, bool kCluster, bool kFused>
__global__ void __launch_bounds__(kThreads, 2)
    decode_split_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRingBytes);  // full[3], empty[3], ready
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kStages + 1);
  volatile int* tile_mask = abort_flag + 1;                          // [kStages]
  __half* qs = reinterpret_cast<__half*>(smem + kRingBytes + kCtlBytes);  // [8][128]
  const uint32_t ready_bar = smem_u32(&bars[2 * kStages]);

  const int split = blockIdx.x;
  const int kh = blockIdx.y;
  const int b = blockIdx.z;
  const int G = a.hq / a.hkv;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const uint32_t pos = a.d_position[b];
  const bool pos_ok = pos < (uint32_t)a.max_seq;
  if (!pos_ok && split == 0 && kh == 0 && threadIdx.x == 0 && a.err)
    atomicCAS(a.err, 0, DEV_ERR_POSITION);
  const int kv_len = pos_ok ? (int)pos + 1 : 0;
  const int n_tiles = (kv_len + kKeys - 1) / kKeys;
  const int tps = (n_tiles + a.nks - 1) / a.nks;
  const int t0 = split * tps;
  const int t1 = min(t0 + tps, n_tiles);
  const int nt = max(0, t1 - t0);
  const int64_t head0 = (int64_t)b * a.hq + (int64_t)kh * G;
  // kFused: this CTA's split holds the new position's tile
  const int new_tile = (int)(pos / kKeys);
  const bool owner = kFused && pos_ok && new_tile >= t0 && new_tile < t1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&bars[i]), 1);
      mbar_init(smem_u32(&bars[kStages + i]), 4);
    }
    mbar_init(ready_bar, 1);
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
    if (lane == 0 && nt > 0) {
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      for (int it = 0; it < nt; ++it) {
        const int st = it % kStages;
        const int r = it / kStages;
        if (r > 0 && !mbar_wait(smem_u32(&bars[kStages + st]), (r - 1) & 1, a.err, 1, abort_flag))
          break;
        const int tile = t0 + it;
        if (owner && tile == new_tile) {
          // the new K/V row must be in memory (and visible to TMA) first
          if (!mbar_wait(ready_bar, 0, a.err, 3, abort_flag)) break;
          fence_proxy_async_global();
        }
        int row = tile * kKeys;
        int outer = b;  // sequence (contiguous caches) or page (paged pool)
        int masked = 0;
        if (kPaged) {
          // a 64-key tile never straddles a page (page_size % 64 == 0)
          const int pg = row / a.page_size;
          outer = __ldg(a.page_table + (int64_t)b * a.table_stride + pg);
          row -= pg * a.page_size;
          if (outer < 0 || outer >= a.num_pages) {
            // never hand TMA an out-of-pool coordinate: load page 0, mask it
            if (a.err) atomicCAS(a.err, 0, DEV_ERR_PAGE);
            outer = 0;
            masked = 1;
          }
        }
        tile_mask[st] = masked;
        const uint32_t full = smem_u32(&bars[st]);
        mbar_arrive_expect_tx(full, kStageBytes);
        const uint32_t kb = smem_u32(smem + st * kStageBytes);
        const uint32_t vb = kb + kTileBytes;
        tma_load_4d(kb, &tm_k, full, 0, row, kh, outer);
        tma_load_4d(kb + kBoxBytes, &tm_k, full, 64, row, kh, outer);
        tma_load_4d(vb, &tm_v, full, 0, row, kh, outer);
        tma_load_4d(vb + kBoxBytes, &tm_v, full, 64, row, kh, outer);
      }
    }
  } else {
    // ----------------------------------------------------------- consumers
    uint32_t qb[8][2];
    if (kFused) {
      // Octet o of the four consumer warps: o < G normalises query row
      // (head0 + o); in the owner CTA octet 8 writes the new K row and
      // octet 9 copies the new V row into the cache.
      const int oc = threadIdx.x >> 3;
      const int j = threadIdx.x & 7;
      const unsigned mask = 0xFFu << (threadIdx.x & 24);
      const __half* row = a.qkv + (int64_t)b * a.qkv_row_stride;
      if (pos_ok && (oc < G || (owner && oc < 10))) {
        const bool is_v = oc == 9;
        const __half* src = oc < G ? row + (head0 - (int64_t)b * a.hq + oc) * 128
                          : row + (int64_t)(a.hq + (is_v ? a.hkv : 0) + kh) * 128;
        const uint4 xl = ldg16(src + 8 * j), xh = ldg16(src + 64 + 8 * j);
        int64_t off = 0;  // cache element offset of (kh, pos) for the K/V rows
        bool kv_ok = true;
        if (oc >= G) {
          if (kPaged) {
            const int64_t pg = pos / a.page_size;
            const int32_t page = a.page_table[(int64_t)b * a.table_stride + pg];
            kv_ok = page >= 0 && page < a.num_pages;
            if (!kv_ok && j == 0 && a.err) atomicCAS(a.err, 0, DEV_ERR_PAGE);
            off = ((int64_t)page * a.hkv + kh) * a.page_size * 128 + (pos - pg * a.page_size) * 128;
          } else {
            off = (int64_t)b * a.cache_batch_stride + (int64_t)kh * a.cache_head_stride +
                  (int64_t)pos * 128;
          }
        }
        if (is_v) {
          if (kv_ok) {
            *reinterpret_cast<uint4*>(a.v_cache + off + 8 * j) = xl;
            *reinterpret_cast<uint4*>(a.v_cache + off + 64 + 8 * j) = xh;
          }
        } else {
          float wl[8], wh[8], cs[8], sn[8];
          const __half* w = oc < G ? a.q_w : a.k_w;
          unpack8(ldg16(w + 8 * j), wl);
          unpack8(ldg16(w + 64 + 8 * j), wh);
          load_cos_sin(a.table + (int64_t)pos * 128, j, cs, sn);
          uint4 ylo, yhi;
          octet_norm_rope(xl, xh, wl, wh, cs, sn, a.eps, mask, ylo, yhi);
          if (oc < G) {
            *reinterpret_cast<uint4*>(qs + oc * 128 + 8 * j) = ylo;
            *reinterpret_cast<uint4*>(qs + oc * 128 + 64 + 8 * j) = yhi;
            if (a.q_out && split == 0) {
              __half* qo = a.q_out + (head0 + oc) * 128;
              *reinterpret_cast<uint4*>(qo + 8 * j) = ylo;
              *reinterpret_cast<uint4*>(qo + 64 + 8 * j) = yhi;
            }
          } else if (kv_ok) {
            *reinterpret_cast<uint4*>(a.k_cache + off + 8 * j) = ylo;
            *reinterpret_cast<uint4*>(a.k_cache + off + 64 + 8 * j) = yhi;
          }
        }
        if (oc >= G) fence_proxy_async_global();  // cache stores -> later TMA reads
      }
      named_bar_sync(1, 128);  // the query rows are in shared memory
      if (owner && threadIdx.x == 0) mbar_arrive(ready_bar);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        if (g < G) {
          qb[kk][0] = *reinterpret_cast<const uint32_t*>(qs + g * 128 + 16 * kk + 2 * t);
          qb[kk][1] = *reinterpret_cast<const uint32_t*>(qs + g * 128 + 16 * kk + 2 * t + 8);
        } else {
          qb[kk][0] = 0u;
          qb[kk][1] = 0u;
        }
      }
    } else {
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
      if (kPaged && tile_mask[st]) {
        s0 = s1 = s2 = s3 = -INFINITY;
      } else if (kbase + 16 > kv_len) {
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
  // This split's result is valid unless it is empty or a wait gave up; an
  // invalid split contributes weight 0 to the merge.
  const bool valid = nt > 0 && !*abort_flag;

  RedSmem* red = reinterpret_cast<RedSmem*>(smem);
  FinSmem* fin = reinterpret_cast<FinSmem*>(smem + kFinOffset);
  if (valid && warp < 4) {
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
      float res = 0.f, lse = -INFINITY;
      if (valid) {
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
        if (L > 0.f) {  // L == 0: every key of the split was masked
          res = O / L;
          lse = M + __log2f(L);
        }
      }
      if (a.nks == 1) {
        if (valid || !pos_ok) a.out[(head0 + hd) * 128 + d] = __float2half_rn(res);
      } else if (kCluster) {
        fin->o[hd][d] = res;
        if (d == 0) fin->lse[hd] = lse;
      } else {
        a.part_o[((head0 + hd) * a.nks + split) * 128 + d] = res;
        if (d == 0) a.part_lse[(head0 + hd) * a.nks + split] = lse;
      }
    }
  }
  if (kCluster && a.nks > 1) {
    // Every CTA of the cluster reaches both barriers (no early exit above),
    // so the cluster cannot deadlock; the second keeps each CTA's shared
    // memory alive until the others have read it.
    cluster_sync_all();
    const uint32_t me = cluster_ctarank();
    if (threadIdx.x < 128) {
      const int d = threadIdx.x;
      for (int hd = (int)me; hd < G; hd += a.nks) {
        a.out[(head0 + hd) * 128 + d] = merge_splits(a.nks, [&](int s, bool want_lse) {
          return want_lse ? ld_dsmem_f32(&fin->lse[hd], (uint32_t)s)
                          : ld_dsmem_f32(&fin->o[hd][d], (uint32_t)s);
        });
      }
    }
    cluster_sync_all();
  }
}

// Workspace merge, one CTA per (sequence, query head), one thread per dim.
__global__ void __launch_bounds__(128) decode_merge_kernel(const DecodeArgs a) {
  const int64_t row = blockIdx.x;
  const int d = threadIdx.x;
  const float* lse = a.part_lse + row * a.nks;
  const float* po = a.part_o + row * a.nks * 128 + d;
  a.out[row * 128 + d] = merge_splits(a.nks, [&](int s, bool want_lse) {
    return want_lse ? lse[s] : po[s * 128];
  });
}

template <bool kPaged, bool kCluster, bool kFused>
cudaError_t set_attrs() {
  auto k = decode_split_kernel<kPaged, kCluster, kFused>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e == cudaSuccess && kCluster)
    e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

template <bool kPaged, bool kCluster, bool kFused>
cudaError_t launch_split(const DecodeArgs& a, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                         cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nks, a.hkv, a.batch);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  if (kCluster) {
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = a.nks;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, decode_split_kernel<kPaged, kCluster, kFused>, tm_k, tm_v, a);
}

template <bool kPaged, bool kFused>
cudaError_t launch_variant(const DecodeArgs& a, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                           cudaStream_t s) {
  const bool cluster = a.nks > 1 && a.cluster;
  cudaError_t e = cluster ? launch_split<kPaged, true, kFused>(a, tm_k, tm_v, s)
                          : launch_split<kPaged, false, kFused>(a, tm_k, tm_v, s);
  if (e != cudaSuccess || a.nks == 1 || cluster) return e;
  decode_merge_kernel<<<(unsigned)((int64_t)a.batch * a.hq), 128, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t decode_set_attributes() {
  cudaError_t e = cudaSuccess;
  const cudaError_t es[] = {
      set_attrs<false, false, false>(), set_attrs<false, true, false>(),
      set_attrs<true, false, false>(),  set_attrs<true, true, false>(),
      set_attrs<false, false, true>(),  set_attrs<false, true, true>(),
      set_attrs<true, false, true>(),   set_attrs<true, true, true>()};
  for (cudaError_t x : es)
    if (x != cudaSuccess) e = x;
  return e;
}

cudaError_t launch_decode(const DecodeArgs& a, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                          cudaStream_t s) {
  const bool paged = a.page_table != nullptr, fused = a.qkv != nullptr;
  if (paged)
    return fused ? launch_variant<true, true>(a, tm_k, tm_v, s)
                 : launch_variant<true, false>(a, tm_k, tm_v, s);
  return fused ? launch_variant<false, true>(a, tm_k, tm_v, s)
               : launch_variant<false, false>(a, tm_k, tm_v, s);
}

}  // namespace grout
