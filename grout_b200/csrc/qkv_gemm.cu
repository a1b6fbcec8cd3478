// QKV projection (prefill) with the fused Q/K RMSNorm + RoPE + KV-cache
// write as its epilogue.
//
// Replaces the QKV MatMulSlice of a prefill chunk (reference src/model.rs:
// 4076-4098, a cuBLAS GEMM writing an f16 [S][(Hq+2Hkv)*128] activation)
// followed by qk_norm_rope_kv_prefill_raw_f16 (src/kernels.rs:4845-5168):
// the activation never goes to memory.  The accumulator of every output
// element is rounded to f16 first (the reference's GEMM output type), then
// the epilogue applies exactly the fused kernel's arithmetic (norm_rope.cu:
// same operation order, same sum tree), so its results equal the fused
// kernel's on the same f16 QKV bit for bit.
//
// Persistent kernel, one CTA per SM, 256 threads; a tile is 128 tokens x
// 256 output features (two heads: 128-wide tiles re-read X too often and
// left the mainloop L2-bandwidth-bound at ~1.1 PFLOP/s):
//   warps 0-3  epilogue: thread r owns token row r of the tile, i.e. whole
//              head vectors (one head at a time), so the RMS sum and the
//              rotate-half pairs (i, i+64) stay inside the thread
//   warp 4     TMA producer: 64-column K blocks of X [128 tokens] and
//              W [256 output features] into a 4-stage ring (48 KB stages)
//   warp 5     MMA issuer (warp-uniform loop, one elected lane):
//              tcgen05.mma M=128 N=256 K=16, f32 accumulators in TMEM
//   warps 6-7  idle (complete the second warpgroup)
// Two TMEM accumulators (2 x 256 columns) alternate between tiles, so the
// epilogue of one tile overlaps the MMAs of the next.  Tiles are visited in
// groups of kGroupM token blocks per feature column, so the X and W blocks
// in use at once stay L2-resident.
#include "internal.h"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kBM = 128;            // tokens per tile
constexpr int kBN = 256;            // output features per tile (two heads)
constexpr int kBK = 64;             // K per stage (one 128-byte swizzled box)
constexpr int kStages = 4;
constexpr int kBoxBytes = 128 * kBK * 2;      // 16 KB: X box (128 rows)
constexpr int kStageBytes = 3 * kBoxBytes;    // X box + W box (256 rows)
constexpr int kThreads = 256;
constexpr int kGroupM = 16;
constexpr int kOffBar = kStages * kStageBytes;
constexpr int kSmemBytes = kOffBar + 256 + 1024;

constexpr int kBarFull = 0;                     // + stage
constexpr int kBarEmpty = kBarFull + kStages;   // + stage
constexpr int kBarAccFull = kBarEmpty + kStages;  // + buffer (commit)
constexpr int kBarAccEmpty = kBarAccFull + 2;     // + buffer (4 epilogue warps)
constexpr int kNumBars = kBarAccEmpty + 2;

// SW128 K-major descriptor words (same encoding as the attention kernel):
// low = address >> 4 | (16 >> 4) << 16, high = SBO 1024 >> 4 | v1 | SW128.
constexpr uint32_t kDescLbo = (16u >> 4) << 16;
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);

__device__ __forceinline__ void mma_ss_words(uint32_t d, uint32_t alo, uint32_t blo, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 da, db; setp.ne.u32 p, %4, 0;"
      " mov.b64 da, {%1, %5}; mov.b64 db, {%2, %5};"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p; }" ::"r"(d),
      "r"(alo), "r"(blo), "r"(idesc), "r"(acc), "n"(kDescHi)
      : "memory");
}

__device__ __forceinline__ void tile_of(int t, int m_tiles, int n_tiles, int& m, int& n) {
  const int per_group = kGroupM * n_tiles;
  const int g = t / per_group;
  const int rem = t - g * per_group;
  const int gm = min(kGroupM, m_tiles - g * kGroupM);
  n = rem / gm;
  m = g * kGroupM + (rem - n * gm);
}

// One head row of the epilogue: 128 f16-rounded values in x (lo = x[0..63],
// hi = x[64..127]); norm + RoPE with the fused kernel's operation order.
__device__ __forceinline__ void norm_rope_row(const float (&x)[128], const __half* w,
                                              const float* trow, float eps, __half* dst) {
  // sum of squares: lane-j partial over pairs 8j..8j+7, then the xor
  // butterfly 4, 2, 1 of the octet, done here in one thread
  float s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      t[e] = __fadd_rn(__fmul_rn(x[8 * j + e], x[8 * j + e]),
                       __fmul_rn(x[64 + 8 * j + e], x[64 + 8 * j + e]));
    s[j] = __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3])),
                     __fadd_rn(__fadd_rn(t[4], t[5]), __fadd_rn(t[6], t[7])));
  }
  float u[8], v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) u[j] = __fadd_rn(s[j], s[j ^ 4]);
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(u[j], u[j ^ 2]);
  const float ss = __fadd_rn(v[0], v[1]);
  const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(ss, 0.0078125f), eps)));
#pragma unroll
  for (int c = 0; c < 8; ++c) {  // pairs 8c .. 8c+7
    const uint4 wl4 = __ldg(reinterpret_cast<const uint4*>(w + 8 * c));
    const uint4 wh4 = __ldg(reinterpret_cast<const uint4*>(w + 64 + 8 * c));
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(trow + 8 * c));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(trow + 8 * c + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(trow + 64 + 8 * c));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(trow + 64 + 8 * c + 4));
    const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const __half2* wl = reinterpret_cast<const __half2*>(&wl4);
    const __half2* wh = reinterpret_cast<const __half2*>(&wh4);
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int e2 = 0; e2 < 4; ++e2) {
      const float2 wlf = __half22float2(wl[e2]);
      const float2 whf = __half22float2(wh[e2]);
      float ylo[2], yhi[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int e = 2 * e2 + q;
        const float wle = q ? wlf.y : wlf.x, whe = q ? whf.y : whf.x;
        const float nlo = __fmul_rn(__fmul_rn(x[8 * c + e], inv), wle);
        const float nhi = __fmul_rn(__fmul_rn(x[64 + 8 * c + e], inv), whe);
        ylo[q] = __fsub_rn(__fmul_rn(nlo, cs[e]), __fmul_rn(nhi, sn[e]));
        yhi[q] = __fadd_rn(__fmul_rn(nhi, cs[e]), __fmul_rn(nlo, sn[e]));
      }
      lo[e2] = pack_half2(ylo[0], ylo[1]);
      hi[e2] = pack_half2(yhi[0], yhi[1]);
    }
    *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(dst + 64 + 8 * c) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    qkv_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                    const QkvGemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = a.hq + 2 * a.hkv;
  const int m_tiles = (a.rows + kBM - 1) / kBM;
  const int n_tiles = (heads + 1) / 2;
  const int n_tile_total = m_tiles * n_tiles;
  const int kblocks = a.hidden / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(smem_u32(&bars[i]), (i >= kBarAccEmpty) ? 4 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tile_total && ok; t += gridDim.x) {
        int m, n;
        tile_of(t, m_tiles, n_tiles, m, n);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int st = it % kStages;
          if (it >= kStages &&
              !mbar_wait(smem_u32(&bars[kBarEmpty + st]), ((it / kStages) & 1) ^ 1u, a.err, 70,
                         abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&bars[kBarFull + st]);
          mbar_arrive_expect_tx(full, kStageBytes);
          const uint32_t dst = smem_base + st * kStageBytes;
          tma_load_3d(dst, &tm_x, full, kb * kBK, m * kBM, 0);
          tma_load_3d(dst + kBoxBytes, &tm_w, full, kb * kBK, n * kBN, 0);
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------- MMA issue
    const bool leader = elect_one();
    constexpr uint32_t idesc = idesc_f16_f32(kBM, kBN, 0, 0);
    const uint32_t base16 = smem_base >> 4;
    int it = 0, tcount = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tile_total && ok; t += gridDim.x, ++tcount) {
      const int buf = tcount & 1;
      // the epilogue must have drained this accumulator (two tiles ago)
      if (tcount >= 2 &&
          !mbar_wait(smem_u32(&bars[kBarAccEmpty + buf]), ((tcount >> 1) - 1) & 1, a.err, 71,
                     abort_flag))
        break;
      tc_fence_after();
      const uint32_t d = tmem + buf * kBN;
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int st = it % kStages;
        if (!mbar_wait(smem_u32(&bars[kBarFull + st]), (it / kStages) & 1, a.err, 72, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t xlo = base16 + (st * kStageBytes) / 16 + kDescLbo;
        const uint32_t wlo = base16 + (st * kStageBytes + kBoxBytes) / 16 + kDescLbo;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_ss_words(d, xlo + kk * 2, wlo + kk * 2, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(smem_u32(&bars[kBarEmpty + st]));
        }
        __syncwarp();
      }
      if (!ok) break;
      if (leader) tc_commit(smem_u32(&bars[kBarAccFull + buf]));
      __syncwarp();
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------- epilogue
    const int row = warp * 32 + lane;  // TMEM lane == token row of the tile
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    int tcount = 0;
    for (int t = blockIdx.x; t < n_tile_total; t += gridDim.x, ++tcount) {
      int m, n;
      tile_of(t, m_tiles, n_tiles, m, n);
      const int buf = tcount & 1;
      if (!mbar_wait(smem_u32(&bars[kBarAccFull + buf]), (tcount >> 1) & 1, a.err, 73, abort_flag))
        break;
      tc_fence_after();
      const int tok = m * kBM + row;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        const int head = 2 * n + hh;
        float x[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + buf * kBN + hh * 128 + c * 32, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)  // the reference's GEMM output is f16
            x[c * 32 + i] = __half2float(__float2half_rn(__uint_as_float(r[i])));
        }
        if (hh == 1) {  // the accumulator is in registers: hand it back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bars[kBarAccEmpty + buf]));
        }
        if (tok >= a.rows || head >= heads) continue;
        if (a.qkv_out) {  // optional: the f16 QKV activation itself
          __half* q = a.qkv_out + (int64_t)tok * a.qkv_row_stride + (int64_t)head * 128;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            uint4 u;
            u.x = pack_half2(x[8 * c + 0], x[8 * c + 1]);
            u.y = pack_half2(x[8 * c + 2], x[8 * c + 3]);
            u.z = pack_half2(x[8 * c + 4], x[8 * c + 5]);
            u.w = pack_half2(x[8 * c + 6], x[8 * c + 7]);
            *reinterpret_cast<uint4*>(q + 8 * c) = u;
          }
        }
        const int64_t pos = (int64_t)a.pos0 + tok;
        if (head < a.hq) {
          norm_rope_row(x, a.q_w, a.table + pos * 128, a.eps,
                        a.q_out + (int64_t)tok * a.q_out_row_stride + (int64_t)head * 128);
        } else if (head < a.hq + a.hkv) {
          const int kh = head - a.hq;
          norm_rope_row(x, a.k_w, a.table + pos * 128, a.eps,
                        a.k_cache + (int64_t)kh * a.cache_head_stride + pos * 128);
        } else {  // V: the f16 row, verbatim
          const int kh = head - a.hq - a.hkv;
          __half* dst = a.v_cache + (int64_t)kh * a.cache_head_stride + pos * 128;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            uint4 u;
            u.x = pack_half2(x[8 * c + 0], x[8 * c + 1]);
            u.y = pack_half2(x[8 * c + 2], x[8 * c + 3]);
            u.z = pack_half2(x[8 * c + 4], x[8 * c + 5]);
            u.w = pack_half2(x[8 * c + 6], x[8 * c + 7]);
            *reinterpret_cast<uint4*>(dst + 8 * c) = u;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t qkv_gemm_set_attributes() {
  return cudaFuncSetAttribute(qkv_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSmemBytes);
}

cudaError_t launch_qkv_gemm(const QkvGemmArgs& a, const CUtensorMap& tm_x, const CUtensorMap& tm_w,
                            int num_sms, cudaStream_t s) {
  const long long tiles = (long long)((a.rows + kBM - 1) / kBM) * ((a.hq + 2 * a.hkv + 1) / 2);
  if (tiles == 0) return cudaSuccess;
  const int grid = (int)(tiles < num_sms ? tiles : num_sms);
  qkv_gemm_kernel<<<grid, kThreads, kSmemBytes, s>>>(tm_x, tm_w, a);
  return cudaGetLastError();
}

}  // namespace grout
