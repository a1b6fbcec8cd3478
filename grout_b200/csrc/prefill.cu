// Causal GQA prefill attention on the 5th-generation tensor cores.
//
// Replaces fmha_prefill_causal / fmha_prefill_gqa_lpt (reference
// src/kernels.rs:2570-2725, 2943-3298) and flash_attn_causal_seq_f16
// (2462-2557): O = softmax(scale * Q K^T + causal mask) V per query head,
// f16 in, f32 accumulate, P rounded to f16 before the PV product, f16 out.
//
// Persistent kernel: one CTA per SM walks a list of work items; an item is
// two 128-row query tiles of one (sequence, head), streaming 128-key K/V
// tiles.  Warp roles (512 threads, 4 warpgroups):
//   warps 0-3   softmax for query tile 0 (one thread per query row = TMEM lane)
//   warps 4-7   softmax for query tile 1
//   warps 8-11  output: read the finished O_t out of TMEM (warp 8 + q owns
//               TMEM lanes 32q..), free it for the next item, normalise by
//               the row sums and store the rows
//   warp 12     TMA producer: Q_0, K_0, Q_1, V_0, K_1, ... of each item into
//               two query buffers and a 4-slot K/V ring
//   warp 13     MMA issuer: the whole warp runs the issue loop (so its
//               descriptors stay warp-uniform) and one elected lane issues
//               every tcgen05.mma and tcgen05.commit.  This warp shares its
//               SM sub-partition with two busy softmax warps, so each MMA is
//               kept to a few instructions: descriptors are precomputed low
//               words advanced by constant adds.
//   warps 14-15 idle (they complete the fourth warpgroup)
// Tensor memory (512 columns, f32): S0 [0,128) S1 [128,256) O0 [256,384)
// O1 [384,512).  P_t (f16 pairs) overwrites the first 64 columns of S_t and
// feeds the PV MMA straight from TMEM (A operand in TMEM, V from shared
// memory), so P never touches shared memory.
// Per KV tile j the MMA warp issues PV0(j), QK0(j+1), PV1(j), QK1(j+1):
// the next S of one query tile is computed while the other tile's softmax
// runs.  Because tcgen05 operations of one thread complete in issue order,
// "S_t(j+1) ready" also means "PV_t(j) done", which is what the softmax
// warps need before they rescale O_t in place.  Each tile flows straight
// into the next item (QK_t of item n+1 follows the last PV_t of item n, and
// each query buffer is reloaded as soon as its tile's last QK has run), so
// the half-period offset between the two tiles survives item boundaries and
// the output of one item overlaps the start of the next.
#include "internal.h"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kBM = 128;          // query rows per tile (= TMEM lanes)
constexpr int kBN = 128;          // keys per KV tile
constexpr int kSlots = 4;         // K/V ring slots
constexpr int kTile = 128 * 128 * 2;  // bytes of one 128x128 f16 tile (two 64-col boxes)
constexpr int kBox = kTile / 2;
constexpr int kThreads = 512;     // 4 warpgroups, one persistent CTA per SM
// Register split (setmaxnreg): launched at 128 per thread (512 x 128 =
// 65536); the two softmax warpgroups rise to 192, the output and issue
// warpgroups drop to 64: 2 x 128 x 192 + 2 x 128 x 64 = 65536.
constexpr int kRegsOther = 64;
constexpr int kRegsSoftmax = 192;
constexpr int kOffQ = 0;                       // 2 query tiles
constexpr int kOffKV = 2 * kTile;              // ring
constexpr int kOffBar = kOffKV + kSlots * kTile;
constexpr int kOffL = kOffBar + 512;           // row sums, then row maxima: [2][item parity][tile][row]
// Schedule of a ragged batch: sequence lengths, sequences by descending
// length, and per query-tile pair the first compacted item index.
constexpr int kSchedMaxBatch = 1024;
constexpr int kSchedMaxPairs = 1024;
constexpr int kSchedMaxRounds = 1536;  // items per CTA the precomputed list holds
constexpr int kOffSched = kOffL + 2 * 2 * 2 * 128 * 4;
constexpr int kSmemBytes =
    kOffSched + (2 * kSchedMaxBatch + kSchedMaxPairs + 1 + kSchedMaxRounds) * 4 + 1024;

// barrier indices (phases run on across the work items of a CTA)
constexpr int kBarQ = 0;                      // + tile: Q_t landed (TMA)
constexpr int kBarQfree = 2;                  // + tile: last QK_t of the item done (commit)
constexpr int kBarFull = 4;                   // + slot
constexpr int kBarEmpty = kBarFull + kSlots;  // + slot
constexpr int kBarS = kBarEmpty + kSlots;     // + tile (commit)
constexpr int kBarP = kBarS + 2;              // + tile (4 softmax warps)
constexpr int kBarOfull = kBarP + 2;          // + tile: O_t of the item final (commit)
constexpr int kBarOempty = kBarOfull + 2;     // + tile: O_t read out (4 output warps)
constexpr int kBarL = kBarOempty + 2;         // + tile: row sums written (4 softmax warps)
constexpr int kNumBars = kBarL + 2;

// ---- packed f32x2 arithmetic (sm_100a): two softmax elements per instruction
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x (x <= 0) for a pair, on the FMA/ALU pipes, used for a share of the
// softmax exponentials so the MUFU unit is not the only path.  Range
// reduction x = n + f, n = round(x) via the 1.5*2^23 magic constant,
// f in [-1/2, 1/2]; 2^f by a degree-3 polynomial fitted for minimum relative
// error (max 7.6e-5, below the f16 rounding P gets next); 2^n added into the
// exponent field.  Inputs below -125 clamp to ~2^-125 (P rounds to 0 in
// f16); the clamp keeps n + exponent(p) >= 1, so the sum never reaches the
// sign bit (p can be slightly below 1 when f < 0).
__device__ __forceinline__ void ex2_poly2(uint64_t x2, float& r0, float& r1) {
  float x0, x1;
  f2unpack(x2, x0, x1);
  x2 = f2pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t2 = fadd2(x2, f2pack(12582912.0f, 12582912.0f));
  const uint64_t n2 = fadd2(t2, f2pack(-12582912.0f, -12582912.0f));
  const uint64_t f2 = ffma2(n2, f2pack(-1.0f, -1.0f), x2);
  uint64_t p2 = ffma2(f2pack(0.05517090484f, 0.05517090484f), f2,
                      f2pack(0.24260953069f, 0.24260953069f));
  p2 = ffma2(p2, f2, f2pack(0.69326096773f, 0.69326096773f));
  p2 = ffma2(p2, f2, f2pack(0.99992817640f, 0.99992817640f));
  float p0, p1, t0, t1;
  f2unpack(p2, p0, p1);
  f2unpack(t2, t0, t1);
  r0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  r1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Element pairs (of the 16 per 32-column chunk) whose exponentials run on
// ex2_poly2: one in four, so MUFU carries 3/4 of the exponentials.
__device__ __forceinline__ constexpr bool poly_pair(int i) { return (i & 3) == 3; }

// Online-softmax rescaling threshold (log2 units): the reference max a row
// exponentiates against moves only when the row max grows by more than this,
// so P stays <= 2^8 and O is rescaled rarely.
constexpr float kRescaleThreshold = 8.0f;

__device__ __forceinline__ int ring_slot(int i) { return i % kSlots; }
__device__ __forceinline__ uint32_t ring_parity(int i) { return (uint32_t)((i / kSlots) & 1); }

// Low/high words of the SW128 shared-memory descriptor (matches
// smem_desc_sw128): low = start address >> 4 | LBO >> 4 << 16;
// high = SBO (1024) >> 4 | version 1 << 14 | layout SW128 (2) << 29.
constexpr uint32_t kDescLboK = (16u >> 4) << 16;
constexpr uint32_t kDescLboV = ((uint32_t)kBox >> 4) << 16;
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
static_assert(((uint64_t)kDescHi << 32) == ((uint64_t)(1024u >> 4) << 32 | 1ull << 46 | 2ull << 61),
              "descriptor high word");
__device__ __forceinline__ void mma_ss_lo(uint32_t d, uint32_t alo, uint32_t blo, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 da, db; setp.ne.u32 p, %4, 0;"
      " mov.b64 da, {%1, %5}; mov.b64 db, {%2, %5};"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p; }" ::"r"(d),
      "r"(alo), "r"(blo), "r"(idesc), "r"(acc), "n"(kDescHi)
      : "memory");
}
__device__ __forceinline__ void mma_ts_lo(uint32_t d, uint32_t a_tmem, uint32_t blo, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 db; setp.ne.u32 p, %4, 0;"
      " mov.b64 db, {%2, %5};"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %3, p; }" ::"r"(d),
      "r"(a_tmem), "r"(blo), "r"(idesc), "r"(acc), "n"(kDescHi)
      : "memory");
}

// One work item = two 128-row query tiles of one (sequence, head); items are
// numbered longest-first (query-tile pair descending, then head, then
// sequence).  In round r CTA c takes entry r * gridDim.x + c of the schedule,
// or r * gridDim.x + gridDim.x - 1 - c in odd rounds: the snake order evens
// out the causal work per CTA (a plain stride leaves the first CTAs ~12%
// more).  For a ragged batch the schedule skips the empty items (see
// item_of in prefill_kernel).
struct Item {
  int h, b, q0, S, P, ks, q_start, n_kv, n_kv0;
  int lo;   // first KV tile of this item (split-K: its range starts here)
  int nch;  // split-K: number of non-empty splits of this (pair, head, sequence)
};
template <bool kSplit>
__device__ __forceinline__ bool decode_item(const PrefillArgs& a, int idx, int n_pairs, Item& it) {
  int split = 0;
  if (kSplit) {
    split = idx % a.nsplit;
    idx /= a.nsplit;
  }
  const int per = a.hq * a.batch;
  const int pair = n_pairs - 1 - idx / per;
  const int rem = idx - (idx / per) * per;
  it.h = rem % a.hq;
  it.b = rem / a.hq;
  if (a.cu_q) {
    it.q_start = a.cu_q[it.b];
    it.S = a.cu_q[it.b + 1] - it.q_start;
  } else {
    it.q_start = 0;
    it.S = a.single_len;
  }
  it.P = a.pos0 ? a.pos0[it.b] : a.single_pos0;
  it.ks = a.kv_start ? a.kv_start[it.b] : 0;
  it.q0 = pair * 2 * kBM;
  if (it.q0 >= it.S) return false;  // ragged batch: this sequence is shorter
  const int rows_hi = min(it.q0 + 2 * kBM, it.S);
  it.n_kv = (it.P + rows_hi + kBN - 1) / kBN;
  // query tile 0 (rows q0 .. q0+127) never sees keys beyond P + q0 + 127
  it.n_kv0 = (it.P + min(it.q0 + kBM, it.S) + kBN - 1) / kBN;
  it.lo = 0;
  it.nch = 1;
  if (kSplit) {
    // Split [0, n_kv0) into chunks of tps tiles; the last chunk also takes
    // tile 1's extra tile, so both tiles have work in every chunk.
    const int tps = (it.n_kv0 + a.nsplit - 1) / a.nsplit;
    it.nch = (it.n_kv0 + tps - 1) / tps;
    const int lo = split * tps;
    if (lo >= it.n_kv0) return false;  // fewer chunks than splits
    const int hi0 = min(it.n_kv0, lo + tps);
    it.lo = lo;
    it.n_kv = hi0 == it.n_kv0 ? it.n_kv - lo : hi0 - lo;
    it.n_kv0 = hi0 - lo;
  }
  return true;
}

// The compacted schedule of a ragged batch (see prefill_kernel), built by the
// whole CTA into shared memory: sched = [len | ord | beg | list], list[r] =
// this CTA's item in round r.  Returns the number of rounds.
template <bool kSplit>
__device__ __forceinline__ int build_schedule(const PrefillArgs& a, int n_pairs, int n_items,
                                           int* sched) {
  int* s_len = sched;
  int* s_ord = s_len + kSchedMaxBatch;
  int* s_beg = s_ord + kSchedMaxBatch;
  int* s_list = s_beg + kSchedMaxPairs + 1;
  for (int b = threadIdx.x; b < a.batch; b += blockDim.x) s_len[b] = a.cu_q[b + 1] - a.cu_q[b];
  __syncthreads();
  for (int b = threadIdx.x; b < a.batch; b += blockDim.x) {
    const int lb = s_len[b];
    int rank = 0;
    for (int c = 0; c < a.batch; ++c) rank += (s_len[c] > lb) || (s_len[c] == lb && c < b);
    s_ord[rank] = b;
  }
  for (int rp = threadIdx.x; rp < n_pairs; rp += blockDim.x) {
    const int q0 = (n_pairs - 1 - rp) * 2 * kBM;
    int cnt = 0;
    for (int b = 0; b < a.batch; ++b) cnt += s_len[b] > q0;
    s_beg[rp + 1] = cnt * a.hq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s_beg[0] = 0;
    for (int rp = 1; rp <= n_pairs; ++rp) s_beg[rp] += s_beg[rp - 1];
  }
  __syncthreads();
  const int n_sched = s_beg[n_pairs] * (kSplit ? a.nsplit : 1);
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  const int rounds = min((n_sched + G - 1) / G, kSchedMaxRounds);
  for (int r = threadIdx.x; r < rounds; r += blockDim.x) {
    const int k = r * G + ((r & 1) ? G - 1 - c : c);
    int idx = n_items;
    if (k < n_sched) {
      const int ki = kSplit ? k / a.nsplit : k;
      int lo = 0, hi = n_pairs;  // largest rp with s_beg[rp] <= ki
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_beg[mid] <= ki) lo = mid;
        else hi = mid;
      }
      const int m = ki - s_beg[lo];
      idx = lo * (a.hq * a.batch) + s_ord[m / a.hq] * a.hq + m % a.hq;
      if (kSplit) idx = idx * a.nsplit + k % a.nsplit;
    }
    s_list[r] = idx;
  }
  return rounds;  // the list is published by the caller's next __syncthreads
}

// kPaged: K/V from a page pool; kSplit: split-K partial output; kCompact: a
// ragged batch scheduled over its non-empty items.  The plain instantiation
// carries none of them.
template <bool kPaged, bool kSplit, bool kCompact>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* lbuf = reinterpret_cast<float*>(smem + kOffL);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_pairs = (a.max_q_len + 2 * kBM - 1) / (2 * kBM);
  const int n_items = n_pairs * a.hq * a.batch * (kSplit ? a.nsplit : 1);
  // A ragged batch leaves holes in the (pair, sequence, head) numbering: a
  // short sequence has no items at high pair indices.  Striding over the
  // numbering with the holes left in gives some CTAs far more work than
  // others (the CTA-to-item map is fixed), so for a batch the CTAs stride
  // over the compacted list instead — the non-empty items only, still
  // longest first: pairs descending, then sequences by descending length,
  // then heads.  s_beg[rp] is the first compacted index of pair
  // n_pairs - 1 - rp; sequences holding that pair are the first ones of
  // s_ord.  Item indices handed to decode_item stay the plain numbering.
  int* s_len = reinterpret_cast<int*>(smem + kOffSched);
  const int* s_list = s_len + 2 * kSchedMaxBatch + kSchedMaxPairs + 1;  // this CTA's item per round
  const int n_rounds = kCompact ? build_schedule<kSplit>(a, n_pairs, n_items, s_len) : 0;
  // Item of this CTA in round r (n_items once the schedule is exhausted).
  auto item_of = [&](int r) -> int {
    if (kCompact) return r < n_rounds ? s_list[r] : n_items;
    return r * (int)gridDim.x + ((r & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      uint32_t cnt = 1;
      if ((i >= kBarP && i < kBarP + 2) || (i >= kBarOempty && i < kBarOempty + 2) ||
          (i >= kBarL && i < kBarL + 2))
        cnt = 4;  // one arrival per warp of a warpgroup
      mbar_init(smem_u32(&bars[i]), cnt);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 13) {
    tmem_alloc(smem_u32(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t smem_base = smem_u32(smem);

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
  if (warp == 12) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      int ring = 0, nq = 0;
      bool ok = true;
      for (int r = 0, idx; ok && (idx = item_of(r)) < n_items; ++r) {
        Item it;
        if (!decode_item<kSplit>(a, idx, n_pairs, it)) continue;
        const int kh = it.h / (a.hq / a.hkv);
        const int kvb = a.kv_batched ? it.b : 0;
        // Q_0, K_0, Q_1, then the rest: each tile's query buffer is refilled
        // as soon as that tile's last QK of the previous item has run.
        auto load_q = [&](int t) -> bool {
          if (nq > 0 &&
              !mbar_wait(smem_u32(&bars[kBarQfree + t]), (nq - 1) & 1, a.err, 11 + t, abort_flag))
            return false;
          const uint32_t bq = smem_u32(&bars[kBarQ + t]);
          mbar_arrive_expect_tx(bq, kTile);
          const uint32_t dst = smem_base + kOffQ + t * kTile;
          const int row = it.q_start + it.q0 + t * kBM;
          tma_load_3d(dst, &tm_q, bq, 0, it.h, row);
          tma_load_3d(dst + kBox, &tm_q, bq, 64, it.h, row);
          return true;
        };
        if (!load_q(0)) break;
        for (int i = 0; i < 2 * it.n_kv; ++i, ++ring) {
          if (i == 1 && !load_q(1)) {
            ok = false;
            break;
          }
          const int slot = ring_slot(ring);
          if (ring >= kSlots &&
              !mbar_wait(smem_u32(&bars[kBarEmpty + slot]), ring_parity(ring) ^ 1u, a.err, 10,
                         abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&bars[kBarFull + slot]);
          mbar_arrive_expect_tx(full, kTile);
          const CUtensorMap* map = (i & 1) ? &tm_v : &tm_k;
          const uint32_t dst = smem_base + kOffKV + slot * kTile;
          const int row = it.ks + (it.lo + (i >> 1)) * kBN;
          if (kPaged) {
            // two 64-key halves, each inside one page (page_size % 64 == 0);
            // a half past the sequence's last key reads page 0 (masked) and
            // leaves the table untouched
            const int32_t* trow = a.page_table + (int64_t)it.b * a.table_stride;
            const int kv_len = it.P + it.S;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int key = (it.lo + (i >> 1)) * kBN + hh * 64;
              int page = 0, r = 0;
              if (key < kv_len) {
                const int pg = key / a.page_size;
                page = __ldg(trow + pg);
                r = key - pg * a.page_size;
                if ((page < 0 || page >= a.num_pages) && a.err) atomicCAS(a.err, 0, DEV_ERR_PAGE);
              }
              tma_load_4d(dst + hh * (kBox / 2), map, full, 0, r, kh, page);
              tma_load_4d(dst + kBox + hh * (kBox / 2), map, full, 64, r, kh, page);
            }
          } else if (a.kv_batched) {
            tma_load_4d(dst, map, full, 0, row, kh, kvb);
            tma_load_4d(dst + kBox, map, full, 64, row, kh, kvb);
          } else {
            tma_load_3d(dst, map, full, 0, row, kh);
            tma_load_3d(dst + kBox, map, full, 64, row, kh);
          }
        }
        ++nq;
      }
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------- MMA issue
    // The whole warp runs the issue loop (warp-uniform descriptors); one
    // elected lane issues every MMA and commit.  Per KV tile j of an item:
    // PV0(j), QK0(j+1), PV1(j), QK1(j+1); the first QKs of the next item
    // follow the last PVs of this one, and its first PV_t waits until the
    // output warps have read O_t of this item out of TMEM.
    const bool leader = elect_one();
    constexpr uint32_t idesc_qk = idesc_f16_f32(kBM, kBN, 0, 0);
    constexpr uint32_t idesc_pv = idesc_f16_f32(kBM, 128, 0, 1);
    const uint32_t base16 = smem_base >> 4;
    auto qk = [&](int t, int slot) {
      const uint32_t qlo = base16 + (kOffQ + t * kTile) / 16 + kDescLboK;
      const uint32_t klo = base16 + (kOffKV + slot * kTile) / 16 + kDescLboK;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = ((kk >> 2) * kBox + (kk & 3) * 32) / 16;
        if (leader) mma_ss_lo(tmem + t * 128, qlo + off, klo + off, idesc_qk, kk > 0 ? 1u : 0u);
      }
    };
    auto pv = [&](int t, int slot, bool acc) {
      const uint32_t vlo = base16 + (kOffKV + slot * kTile) / 16 + kDescLboV;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        if (leader) mma_ts_lo(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, vlo + kk * (2048 / 16), idesc_pv,
                              (acc || kk > 0) ? 1u : 0u);
      }
    };
    // Each tile runs on into the next item: right after tile t's last PV of
    // item n the warp issues QK_t of item n + 1, so the two tiles keep their
    // half-period offset across item boundaries.
    auto next_valid = [&](int& rr, Item& itm) -> bool {
      for (int idx; (idx = item_of(rr)) < n_items; ++rr)
        if (decode_item<kSplit>(a, idx, n_pairs, itm)) return true;
      return false;
    };
    int ring = 0, nq = 0, pc0 = 0, pc1 = 0;
    int rr = 0;
    Item cur;
    bool has = next_valid(rr, cur);
    bool ok = true;
    if (has) {
      ok = mbar_wait(smem_u32(&bars[kBarQ + 0]), 0, a.err, 20, abort_flag) &&
           mbar_wait(smem_u32(&bars[kBarFull + ring_slot(ring)]), ring_parity(ring), a.err, 21, abort_flag);
      if (ok) {
        tc_fence_after();
        qk(0, ring_slot(ring));
        if (leader) tc_commit(smem_u32(&bars[kBarS + 0]));
        if (cur.n_kv0 == 1 && leader) tc_commit(smem_u32(&bars[kBarQfree + 0]));
        ok = mbar_wait(smem_u32(&bars[kBarQ + 1]), 0, a.err, 28, abort_flag);
      }
      if (ok) {
        tc_fence_after();
        qk(1, ring_slot(ring));
        if (leader) tc_commit(smem_u32(&bars[kBarS + 1]));
        if (leader) tc_commit(smem_u32(&bars[kBarEmpty + ring_slot(ring)]));
        if (cur.n_kv == 1 && leader) tc_commit(smem_u32(&bars[kBarQfree + 1]));
      }
    }
    while (has && ok) {
      int rn = rr + 1;
      Item nx;
      const bool hn = next_valid(rn, nx);
      const int n_kv = cur.n_kv, n_kv0 = cur.n_kv0;
      const int nring = ring + 2 * n_kv;  // K_0 of the next item
      for (int j = 0; j < n_kv; ++j) {
        const int iv = ring + 2 * j + 1, ik = ring + 2 * j + 2;
        const bool next = j + 1 < n_kv;
        ok = mbar_wait(smem_u32(&bars[kBarFull + ring_slot(iv)]), ring_parity(iv), a.err, 22, abort_flag);
        // K(j+1) only needs the slot K(j-1) released, so it is awaited
        // here, before P0(j), keeping the wait off the PV0 -> QK0 path.
        if (ok && next)
          ok = mbar_wait(smem_u32(&bars[kBarFull + ring_slot(ik)]), ring_parity(ik), a.err, 24, abort_flag);
        if (!ok) break;
        if (j < n_kv0) {
          ok = mbar_wait(smem_u32(&bars[kBarP + 0]), pc0 & 1, a.err, 23, abort_flag);
          if (ok && j == 0 && nq > 0)
            ok = mbar_wait(smem_u32(&bars[kBarOempty + 0]), (nq - 1) & 1, a.err, 26, abort_flag);
          if (!ok) break;
          ++pc0;
          tc_fence_after();
          pv(0, ring_slot(iv), j > 0);
          if (j == n_kv0 - 1 && leader) tc_commit(smem_u32(&bars[kBarOfull + 0]));
        }
        if (j + 1 < n_kv0) {
          tc_fence_after();
          qk(0, ring_slot(ik));
          if (leader) tc_commit(smem_u32(&bars[kBarS + 0]));
          if (j + 1 == n_kv0 - 1 && leader) tc_commit(smem_u32(&bars[kBarQfree + 0]));
        } else if (j + 1 == n_kv0 && hn) {
          // tile 0 is done with this item: start the next one
          ok = mbar_wait(smem_u32(&bars[kBarQ + 0]), (nq + 1) & 1, a.err, 20, abort_flag) &&
               mbar_wait(smem_u32(&bars[kBarFull + ring_slot(nring)]), ring_parity(nring), a.err, 21,
                         abort_flag);
          if (!ok) break;
          tc_fence_after();
          qk(0, ring_slot(nring));
          if (leader) tc_commit(smem_u32(&bars[kBarS + 0]));
          if (nx.n_kv0 == 1 && leader) tc_commit(smem_u32(&bars[kBarQfree + 0]));
        }
        ok = mbar_wait(smem_u32(&bars[kBarP + 1]), pc1 & 1, a.err, 25, abort_flag);
        if (ok && j == 0 && nq > 0)
          ok = mbar_wait(smem_u32(&bars[kBarOempty + 1]), (nq - 1) & 1, a.err, 27, abort_flag);
        if (!ok) break;
        ++pc1;
        tc_fence_after();
        pv(1, ring_slot(iv), j > 0);
        if (leader) tc_commit(smem_u32(&bars[kBarEmpty + ring_slot(iv)]));
        if (!next && leader) tc_commit(smem_u32(&bars[kBarOfull + 1]));
        if (next) {
          qk(1, ring_slot(ik));
          if (leader) tc_commit(smem_u32(&bars[kBarS + 1]));
          if (leader) tc_commit(smem_u32(&bars[kBarEmpty + ring_slot(ik)]));
          if (j + 1 == n_kv - 1 && leader) tc_commit(smem_u32(&bars[kBarQfree + 1]));
        } else if (hn) {
          // tile 1 is done with this item: start the next one (K_0 of it
          // was awaited when tile 0 started it)
          ok = mbar_wait(smem_u32(&bars[kBarQ + 1]), (nq + 1) & 1, a.err, 28, abort_flag);
          if (!ok) break;
          tc_fence_after();
          qk(1, ring_slot(nring));
          if (leader) tc_commit(smem_u32(&bars[kBarS + 1]));
          if (leader) tc_commit(smem_u32(&bars[kBarEmpty + ring_slot(nring)]));
          if (nx.n_kv == 1 && leader) tc_commit(smem_u32(&bars[kBarQfree + 1]));
        }
      }
      if (!ok) break;
      ring = nring;
      ++nq;
      cur = nx;
      rr = rn;
      has = hn;
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------ output
    // Warp 8 + q reads TMEM lanes 32q.. (query rows) of O_t once the MMA
    // warp reports it final, frees O_t for the next item, and writes the
    // normalised rows.
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    int nq = 0;
    bool ok = true;
    for (int r = 0, idx; ok && (idx = item_of(r)) < n_items; ++r) {
      Item it;
      if (!decode_item<kSplit>(a, idx, n_pairs, it)) continue;
#pragma unroll 1
      for (int t = 0; t < 2; ++t) {
        ok = mbar_wait(smem_u32(&bars[kBarOfull + t]), nq & 1, a.err, 40 + t, abort_flag);
        ok = ok && mbar_wait(smem_u32(&bars[kBarL + t]), nq & 1, a.err, 42 + t, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const float l_row = lbuf[((nq & 1) * 2 + t) * 128 + row];
        const float inv_l = 1.0f / fmaxf(l_row, 1.0e-8f);
        const int row_q = it.q0 + t * kBM + row;
        const bool valid = row_q < it.S;
        // split-K: this item's unnormalised rows and (m, l) go to the workspace
        float* prow = kSplit ? a.part + ((size_t)idx * 2 + t) * kPrefillPartFloats : nullptr;
        if (prow && valid) {
          prow[128 * 128 + row] = lbuf[512 + ((nq & 1) * 2 + t) * 128 + row];
          prow[128 * 129 + row] = l_row;
        }
        __half* orow = a.out + (int64_t)(it.q_start + row_q) * a.q_row_stride + (int64_t)it.h * 128;
        const uint32_t tO = tmem + 256 + t * 128 + lane_off;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tO + c * 32, r);
          tc_wait_ld();
          if (c == 3) {  // all of O_t is in registers now: release it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars[kBarOempty + t]));
          }
          if (prow && valid) {
            float4* dst = reinterpret_cast<float4*>(prow + row * 128 + c * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          } else if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 u;
              u.x = pack_half2(__uint_as_float(r[8 * v + 0]) * inv_l, __uint_as_float(r[8 * v + 1]) * inv_l);
              u.y = pack_half2(__uint_as_float(r[8 * v + 2]) * inv_l, __uint_as_float(r[8 * v + 3]) * inv_l);
              u.z = pack_half2(__uint_as_float(r[8 * v + 4]) * inv_l, __uint_as_float(r[8 * v + 5]) * inv_l);
              u.w = pack_half2(__uint_as_float(r[8 * v + 6]) * inv_l, __uint_as_float(r[8 * v + 7]) * inv_l);
              dst[v] = u;
            }
          }
        }
      }
      ++nq;
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // --------------------------------------------------------------- softmax
    const int t = warp >> 2;          // query tile
    const int row = threadIdx.x & 127;  // TMEM lane == query row within the tile
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_off;
    const uint32_t tO = tmem + 256 + t * 128 + lane_off;
    const float sl2 = a.scale_log2;
    int sc = 0, nq = 0;
    bool ok = true;
    for (int r = 0, idx; ok && (idx = item_of(r)) < n_items; ++r) {
      Item it;
      if (!decode_item<kSplit>(a, idx, n_pairs, it)) continue;
      const int row_q = it.q0 + t * kBM + row;
      const int kv_len = it.P + it.S;
      const int key_lim = min(it.P + row_q, kv_len - 1);  // last visible key
      const int n_t = t == 0 ? it.n_kv0 : it.n_kv;
      float m_run = -INFINITY, l = 0.f;  // m_run: the max P is exponentiated against
      for (int j = 0; j < n_t; ++j) {
        ok = mbar_wait(smem_u32(&bars[kBarS + t]), sc & 1, a.err, 30 + t, abort_flag);
        if (!ok) break;
        ++sc;
        tc_fence_after();
        uint32_t r[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, r[c]);
        tc_wait_ld();
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[c][i]);
        const int lim = key_lim - (it.lo + j) * kBN;
        if (lim < kBN - 1) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > lim) s[c] = -INFINITY;
        }
        float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
        float mx2 = fmaxf(s[4], s[5]), mx3 = fmaxf(s[6], s[7]);
#pragma unroll
        for (int c = 8; c < 128; c += 8) {
          mx0 = fmax3(mx0, s[c], s[c + 1]);
          mx1 = fmax3(mx1, s[c + 2], s[c + 3]);
          mx2 = fmax3(mx2, s[c + 4], s[c + 5]);
          mx3 = fmax3(mx3, s[c + 6], s[c + 7]);
        }
        const float mx_s = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
        float alpha = 1.0f;
        float m_new = m_run;
        if (mx_s > m_run + kRescaleThreshold) {
          m_new = mx_s;
          alpha = ex2(m_run - m_new);
        }
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const uint64_t sl2x2 = f2pack(sl2, sl2);
        const uint64_t negm2 = f2pack(-m_use, -m_use);
        uint64_t rsum = f2pack(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint64_t x2 = ffma2(f2pack(s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1]), sl2x2, negm2);
            float p0, p1;
            if (poly_pair(i)) {
              ex2_poly2(x2, p0, p1);
            } else {
              float x0, x1;
              f2unpack(x2, x0, x1);
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            rsum = fadd2(rsum, f2pack(p0, p1));
            pk[i] = pack_half2(p0, p1);
          }
          asm volatile(
              "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "
              "%10, %11, %12, %13, %14, %15, %16};" ::"r"(tS + c * 16),
              "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]),
              "r"(pk[7]), "r"(pk[8]), "r"(pk[9]), "r"(pk[10]), "r"(pk[11]), "r"(pk[12]),
              "r"(pk[13]), "r"(pk[14]), "r"(pk[15])
              : "memory");
        }
        float rs0, rs1;
        f2unpack(rsum, rs0, rs1);
        l = l * alpha + (rs0 + rs1);
        // Rescale O_t only when some row of the warp moved its reference max
        // (PV_t(j-1) has completed: it was issued before the QK that produced
        // this S).
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars[kBarP + t]));
        m_run = m_new;
      }
      if (!ok) break;
      // Row sums for the output warps.  The output warps must have taken
      // the previous item's sums (O_t of that item read out) first, so the
      // row-sum barrier never runs two phases ahead of its reader.
      if (nq > 0) {
        ok = mbar_wait(smem_u32(&bars[kBarOempty + t]), (nq - 1) & 1, a.err, 32 + t, abort_flag);
        if (!ok) break;
      }
      lbuf[((nq & 1) * 2 + t) * 128 + row] = l;
      lbuf[512 + ((nq & 1) * 2 + t) * 128 + row] = m_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[kBarL + t]));
      ++nq;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Split-K merge (prefill_splitk_reduce_merge, src/kernels.rs:3302-3759):
// per query row, M = max_s m_s, w_s = 2^(m_s - M),
// out = sum_s w_s O_s / max(sum_s w_s l_s, 1e-8), rounded to f16.
// One CTA per (item, query tile), decoded once; warp w takes rows w, w+32,
// w+64, w+96 and lane l dimensions 4l..4l+3, every split's loads issued
// together (the split loop is unrolled to kMaxSplits).
constexpr int kMaxSplits = 8;
__global__ void __launch_bounds__(1024) prefill_merge_kernel(const PrefillArgs a) {
  __shared__ int s_nch, s_rows;
  __shared__ int64_t s_out_row, s_h;
  const int t = blockIdx.x & 1;
  const int base = blockIdx.x >> 1;  // item index without the split
  if (threadIdx.x == 0) {
    const int n_pairs = (a.max_q_len + 2 * kBM - 1) / (2 * kBM);
    Item it;
    int nch = 0;
    if (decode_item<true>(a, base * a.nsplit, n_pairs, it)) {
      nch = it.nch;
      s_rows = min(kBM, it.S - (it.q0 + t * kBM));
      s_out_row = it.q_start + it.q0 + t * kBM;
      s_h = it.h;
    }
    s_nch = nch;
  }
  __syncthreads();
  const int nch = s_nch;
  if (nch == 0 || s_rows <= 0) return;  // empty item (ragged batch) or tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* p0 = a.part + ((size_t)base * a.nsplit * 2 + t) * kPrefillPartFloats;
  const size_t sstride = (size_t)2 * kPrefillPartFloats;  // next split, same item and tile
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp + 32 * i;
    if (r >= s_rows) break;
    float m[kMaxSplits], l[kMaxSplits];
    float4 o[kMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp) {
      if (sp < nch) {
        const float* ps = p0 + sp * sstride;
        m[sp] = ps[128 * 128 + r];
        l[sp] = ps[128 * 129 + r];
        o[sp] = reinterpret_cast<const float4*>(ps + r * 128)[lane];
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp)
      if (sp < nch) M = fmaxf(M, m[sp]);
    float W = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp) {
      if (sp < nch) {
        const float w = ex2(m[sp] - M);
        W += w * l[sp];
        acc.x += w * o[sp].x;
        acc.y += w * o[sp].y;
        acc.z += w * o[sp].z;
        acc.w += w * o[sp].w;
      }
    }
    const float inv = 1.0f / fmaxf(W, 1.0e-8f);
    uint2 u;
    u.x = pack_half2(acc.x * inv, acc.y * inv);
    u.y = pack_half2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(a.out + (s_out_row + r) * a.q_row_stride + s_h * 128 + 4 * lane) = u;
  }
}

}  // namespace

cudaError_t prefill_set_attributes() {
  for (auto k : {prefill_kernel<false, false, false>, prefill_kernel<true, false, false>,
                 prefill_kernel<false, true, false>, prefill_kernel<true, true, false>,
                 prefill_kernel<false, false, true>, prefill_kernel<true, false, true>,
                 prefill_kernel<false, true, true>, prefill_kernel<true, true, true>}) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_prefill(const PrefillArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                           const CUtensorMap& tm_v, cudaStream_t s) {
  const int n_pairs = (a.max_q_len + 2 * kBM - 1) / (2 * kBM);
  if (a.nsplit < 1 || a.nsplit > kMaxSplits || (a.nsplit > 1 && !a.part)) return cudaErrorInvalidValue;
  const long long n_items = (long long)n_pairs * a.hq * a.batch * a.nsplit;
  if (n_items == 0) return cudaSuccess;
  static int num_sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (num_sms[dev] == 0) {
    cudaError_t e = cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  const int grid = (int)(n_items < num_sms[dev] ? n_items : num_sms[dev]);
  const bool paged = a.page_table != nullptr, split = a.nsplit > 1;
  // The compacted schedule pays off when a pair index holds fewer items than
  // two rounds of CTAs (the holes then skew whole rounds): measured on B200
  // at config 4's batch, per-rank shard time 383-412 vs 500-528 us at 8
  // ranks (4 query heads), 1398-1410 vs 1508-1550 us at 2; with 32 query
  // heads (512 items per pair) the plain order is 2.5 % faster.
  const bool compact = a.cu_q != nullptr && a.batch > 1 && a.batch <= kSchedMaxBatch &&
                       n_pairs <= kSchedMaxPairs && (n_items + grid - 1) / grid <= kSchedMaxRounds &&
                       a.hq * a.batch < 2 * grid;
#define GROUT_PREFILL_LAUNCH(P, SP, C) \
  prefill_kernel<P, SP, C><<<grid, kThreads, kSmemBytes, s>>>(tm_q, tm_k, tm_v, a)
  if (compact) {
    if (paged && split) GROUT_PREFILL_LAUNCH(true, true, true);
    else if (paged) GROUT_PREFILL_LAUNCH(true, false, true);
    else if (split) GROUT_PREFILL_LAUNCH(false, true, true);
    else GROUT_PREFILL_LAUNCH(false, false, true);
  } else {
    if (paged && split) GROUT_PREFILL_LAUNCH(true, true, false);
    else if (paged) GROUT_PREFILL_LAUNCH(true, false, false);
    else if (split) GROUT_PREFILL_LAUNCH(false, true, false);
    else GROUT_PREFILL_LAUNCH(false, false, false);
  }
#undef GROUT_PREFILL_LAUNCH
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || a.nsplit <= 1) return e;
  prefill_merge_kernel<<<(unsigned)(n_items / a.nsplit * 2), 1024, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace grout
