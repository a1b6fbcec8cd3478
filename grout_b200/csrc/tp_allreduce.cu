// Tensor-parallel GEMV fused with its all-reduce, over NVLink peer memory.
//
// y = residual + sum_over_ranks(W_r x_r): the row-parallel o_proj / down_proj
// of a tensor-parallel decode step followed by the all-reduce the reference
// would need (it is single-GPU; the split is the Megatron layout of config 5).
// One kernel per call on every rank:
//   1. CTA i computes rows [i*R, (i+1)*R) of its partial W_r x_r in f32.
//      Those rows are one contiguous block of W; a producer warp streams it
//      through a 6-stage shared-memory ring with bulk copies (16 KB each,
//      completion on mbarriers, ~96 KB in flight per SM), and 16 consumer
//      warps take 32 consecutive 16-byte chunks (256 weights) at a time
//      against x in shared memory.  256 consecutive weights touch at most
//      two rows (K >= 256), so a warp splits its sum into those two rows and
//      one lane adds them to the warp's own per-row slots: every sum runs in
//      a fixed order, the partial is deterministic;
//   2. it stores that slice into slot [epoch & 1][rank] of every peer's
//      receive buffer (plain stores through the CUDA-IPC mapping over NVLink;
//      no TMA, no multicast) and, after a CTA barrier, raises flag
//      [rank][i] = epoch + 1 in every peer with a system-scope release store;
//   3. it waits — bounded by a 2 s limit, after which it records a device
//      error and writes nothing — for flag [p][i] >= epoch + 1 (wrap-aware)
//      from every peer p, then sums the partials in rank order 0..world-1 (identical
//      bits on every rank), adds the residual and writes f16.
// The epoch is a per-CTA counter in this rank's own buffer, advanced by the
// kernel, so one launch recorded in a CUDA graph replays correctly.  Receive
// slots alternate with the epoch parity: a rank can only reach call n+2 after
// every peer has raised its call-(n+1) flags, i.e. after the peer finished
// reading call n's slot.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/grout_attn.h"
#include "internal.h"
#include "gemv_stream.cuh"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kMaxWorld = 8;
constexpr int kCtas = 148;        // CTAs per call (one per SM on B200)
constexpr int kConsumers = 512;   // threads computing the GEMV
constexpr int kWarps = kConsumers / 32;
constexpr int kThreads = kConsumers + 32;  // + the bulk-copy producer warp
constexpr int kMaxRowsPerCta = 56;  // hidden <= 148 * 56
constexpr int kMaxK = 16384;      // x held in shared memory
constexpr int kRingStages = 11;  // with x (32 KB) and the static state: < 227 KB
constexpr int kGemvSmem = kMaxK * 2 + kRingStages * kGemvPiece;  // x | ring

// Per-rank buffer layout (bytes): recv [2][world][hidden] f32 | flags
// [world][kCtas] u32 | epoch [kCtas] u32 | broken u32 (set once any wait of
// this rank timed out: the ranks are out of step, later calls fail at once).
__host__ __device__ inline size_t recv_bytes(int world, int hidden) {
  return (size_t)2 * world * hidden * 4;
}
__host__ __device__ inline size_t flags_off(int world, int hidden) { return recv_bytes(world, hidden); }
__host__ __device__ inline size_t epoch_off(int world, int hidden) {
  return flags_off(world, hidden) + (size_t)world * kCtas * 4;
}
__host__ __device__ inline size_t broken_off(int world, int hidden) {
  return epoch_off(world, hidden) + (size_t)kCtas * 4;
}
__host__ __device__ inline size_t total_bytes(int world, int hidden) {
  return broken_off(world, hidden) + 16;
}

struct PeerPtrs {
  unsigned char* base[kMaxWorld];  // every rank's buffer as mapped in this process
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) gemv_allreduce_kernel(
    const PeerPtrs peers, const int rank, const int world, const int hidden, const int k,
    const __half* __restrict__ w, const __half* __restrict__ x,
    const __half* __restrict__ residual, __half* __restrict__ out, int* err) {
  extern __shared__ __align__(128) uint8_t gsmem[];  // x [kMaxK] f16 | ring (GEMV only)
  __half* xs = reinterpret_cast<__half*>(gsmem);
  uint8_t* ring = gsmem + kMaxK * 2;
  __shared__ __align__(8) uint64_t bars[2 * kGemvMaxStages];  // full, empty
  __shared__ int s_abort;
  __shared__ unsigned s_epoch;
  __shared__ int s_ok;
  const int cta = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = (hidden + kCtas - 1) / kCtas;
  const int r0 = min(hidden, cta * rows), r1 = min(hidden, r0 + rows);
  const int nrows = r1 - r0;

  unsigned char* mine = peers.base[rank];
  unsigned* epoch_p = reinterpret_cast<unsigned*>(mine + epoch_off(world, hidden)) + cta;
  volatile unsigned* broken = reinterpret_cast<unsigned*>(mine + broken_off(world, hidden));
  __shared__ float red[kWarps][kMaxRowsPerCta];
  if (threadIdx.x == 0) {
    s_epoch = *epoch_p;
    s_ok = *broken == 0u;
    s_abort = 0;
    if (!s_ok && err) atomicCAS(err, 0, DEV_ERR_TIMEOUT_BASE + 61);
    if (w) gemv_init_bars(bars, kWarps, kRingStages);
  }
  for (int i = threadIdx.x; i < kWarps * kMaxRowsPerCta; i += blockDim.x) (&red[0][0])[i] = 0.f;
  if (w && threadIdx.x < kConsumers)
    for (int i = threadIdx.x * 8; i < k; i += kConsumers * 8)
      *reinterpret_cast<uint4*>(&xs[i]) = __ldg(reinterpret_cast<const uint4*>(x + i));
  __syncthreads();
  if (!s_ok) return;  // an earlier call lost step with the peers
  const unsigned epoch = s_epoch + 1;
  const int slot = epoch & 1;

  // 1. partial rows: the CTA's block of W (nrows * k weights, contiguous)
  //    through the bulk-copy ring (gemv_stream.cuh).
  if (w) {
    gemv_stream_rows<kWarps>(w + (int64_t)r0 * k, nrows, k, xs, ring, bars, kRingStages, &red[0][0],
                             kMaxRowsPerCta, err, 62, (volatile int*)&s_abort);
  } else if (warp == 0) {  // exchange only: the partial is given (x[hidden])
    for (int i = lane; i < nrows; i += 32) red[0][i] = __half2float(x[r0 + i]);
  }
  __syncthreads();
  if (s_abort) {  // a ring wait gave up (recorded): leave the peers to time out
    if (threadIdx.x == 0) *broken = 1u;
    return;
  }
  // The CTA's slice of partials goes into slot [slot][rank] of every rank's
  // receive buffer.
  if (threadIdx.x < nrows) {
    float v = 0.f;
    for (int ww = 0; ww < kWarps; ++ww) v += red[ww][threadIdx.x];
    for (int p = 0; p < world; ++p) {
      float* recv = reinterpret_cast<float*>(peers.base[p]) + ((size_t)slot * world + rank) * hidden;
      recv[r0 + threadIdx.x] = v;
    }
  }
  // The CTA barrier orders every thread's partial stores before the flag
  // stores below; st.release.sys makes them visible to a peer that reads the
  // flag with ld.acquire.sys (release is cumulative over the barrier).
  __syncthreads();
  // 2. flags: every peer may now read our slice
  if (threadIdx.x < world) {
    const int p = threadIdx.x;
    unsigned* flag = reinterpret_cast<unsigned*>(peers.base[p] + flags_off(world, hidden)) +
                     rank * kCtas + cta;
    st_release_sys(flag, epoch);
  }
  // 3. wait for every peer's slice of these rows (bounded)
  if (threadIdx.x == 0) {
    s_ok = 1;
    const unsigned* flags = reinterpret_cast<const unsigned*>(mine + flags_off(world, hidden));
    const uint64_t t0 = globaltimer();
    for (int p = 0; p < world; ++p) {
      const unsigned* f = flags + p * kCtas + cta;
      uint32_t spins = 0;
      // A peer may already have finished this call and raised its flag for
      // the next one (epoch + 1) before this thread looks: any value at or
      // past this call's epoch (wrap-aware) means the slice is in place.
      // The slot that peer writes next is the other parity, so this call's
      // slot is still intact.
      while ((int)(ld_acquire_sys(f) - epoch) < 0) {
        if ((++spins & 255u) == 0 && globaltimer() - t0 > kWaitTimeoutNs) {
          s_ok = 0;
          *broken = 1u;
          if (err) atomicCAS(err, 0, DEV_ERR_TIMEOUT_BASE + 60);
          break;
        }
      }
      if (!s_ok) break;
    }
    *epoch_p = epoch;
  }
  __syncthreads();
  if (!s_ok) return;
  const float* recv = reinterpret_cast<const float*>(mine) + (size_t)slot * world * hidden;
  for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    float y = 0.f;
    for (int p = 0; p < world; ++p) y += __ldcg(recv + (size_t)p * hidden + r);
    if (residual) y += __half2float(residual[r]);
    out[r] = __float2half_rn(y);
  }
}

}  // namespace
}  // namespace grout

struct grout_tp_comm {
  int rank = -1, world = 0, hidden = 0, device = 0;
  grout::PeerPtrs peers{};
  bool opened[grout::kMaxWorld] = {};
  void* local = nullptr;  // this rank's exchange buffer (cudaMalloc, offset 0)
  int* err = nullptr;
};

using namespace grout;

namespace {
grout_status tp_fail(grout_status st, const char* what, cudaError_t e) {
  char m[200];
  snprintf(m, sizeof(m), "%s: %s", what, e == cudaSuccess ? "" : cudaGetErrorString(e));
  set_last_error(m);
  return st;
}
}  // namespace

extern "C" {

grout_status grout_tp_comm_create(int32_t world, int32_t hidden, grout_tp_comm** comm,
                                  void* handle_out) {
  if (!comm || !handle_out) return tp_fail(GROUT_ERR_INVALID_ARG, "null pointer argument", cudaSuccess);
  if (world < 1 || world > kMaxWorld || hidden <= 0 || hidden % 8 ||
      hidden > kCtas * kMaxRowsPerCta)
    return tp_fail(GROUT_ERR_INVALID_ARG,
                   "tp comm: need 1 <= world <= 8, hidden % 8 == 0, hidden <= 8288", cudaSuccess);
  grout_tp_comm* c = new grout_tp_comm();
  c->world = world;
  c->hidden = hidden;
  cudaGetDevice(&c->device);
  // The buffer is the library's own allocation so that its IPC handle maps
  // exactly this address in the peers (a sub-allocation of a caching
  // allocator would map the enclosing block instead).
  cudaError_t e = cudaMalloc(&c->local, total_bytes(world, hidden));
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, total_bytes(world, hidden));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return tp_fail(GROUT_ERR_CUDA, "tp comm setup", e);
  }
  static_assert(sizeof(h) == GROUT_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  c->err = device_error_word();
  e = cudaFuncSetAttribute(gemv_allreduce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kGemvSmem);
  if (e != cudaSuccess) {
    cudaFree(c->local);
    delete c;
    return tp_fail(GROUT_ERR_CUDA, "tp comm setup", e);
  }
  *comm = c;
  return GROUT_OK;
}

grout_status grout_tp_comm_connect(grout_tp_comm* c, int32_t rank, const void* all_handles) {
  if (!c || (c->world > 1 && !all_handles))
    return tp_fail(GROUT_ERR_INVALID_ARG, "null pointer argument", cudaSuccess);
  if (rank < 0 || rank >= c->world || c->rank >= 0)
    return tp_fail(GROUT_ERR_INVALID_ARG, "tp comm: bad rank or already connected", cudaSuccess);
  for (int p = 0; p < c->world; ++p) {
    if (p == rank) {
      c->peers.base[p] = static_cast<unsigned char*>(c->local);
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(all_handles) + (size_t)p * GROUT_IPC_HANDLE_BYTES,
                sizeof(h));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < p; ++q)
        if (c->opened[q]) {
          cudaIpcCloseMemHandle(c->peers.base[q]);
          c->opened[q] = false;
        }
      return tp_fail(GROUT_ERR_CUDA, "cudaIpcOpenMemHandle", e);
    }
    c->peers.base[p] = static_cast<unsigned char*>(ptr);
    c->opened[p] = true;
  }
  c->rank = rank;
  return GROUT_OK;
}

void grout_tp_comm_destroy(grout_tp_comm* c) {
  if (!c) return;
  for (int p = 0; p < c->world; ++p)
    if (c->opened[p]) cudaIpcCloseMemHandle(c->peers.base[p]);
  if (c->local) cudaFree(c->local);
  delete c;
}

grout_status grout_gemv_allreduce(grout_tp_comm* c, const void* w, int32_t k, const void* x,
                                  const void* residual, void* out, grout_stream_t stream) {
  if (!c || !w || !x || !out) return tp_fail(GROUT_ERR_INVALID_ARG, "null pointer argument", cudaSuccess);
  if (c->rank < 0) return tp_fail(GROUT_ERR_INVALID_ARG, "tp comm not connected", cudaSuccess);
  if (k < kGemvMinK || k % 8 || k > kMaxK)
    return tp_fail(GROUT_ERR_INVALID_ARG,
                   "gemv_allreduce: k must be a multiple of 8 in [256, 16384]", cudaSuccess);
  const void* ptrs[] = {w, x, out};
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15)
      return tp_fail(GROUT_ERR_INVALID_ARG, "gemv_allreduce: pointers must be 16-byte aligned",
                     cudaSuccess);
  gemv_allreduce_kernel<<<kCtas, kThreads, kGemvSmem, reinterpret_cast<cudaStream_t>(stream)>>>(
      c->peers, c->rank, c->world, c->hidden, k, static_cast<const __half*>(w),
      static_cast<const __half*>(x), static_cast<const __half*>(residual),
      static_cast<__half*>(out), c->err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tp_fail(GROUT_ERR_CUDA, "gemv_allreduce launch", e);
  return GROUT_OK;
}

grout_status grout_allreduce_residual(grout_tp_comm* c, const void* partial, const void* residual,
                                      void* out, grout_stream_t stream) {
  if (!c || !partial || !out)
    return tp_fail(GROUT_ERR_INVALID_ARG, "null pointer argument", cudaSuccess);
  if (c->rank < 0) return tp_fail(GROUT_ERR_INVALID_ARG, "tp comm not connected", cudaSuccess);
  gemv_allreduce_kernel<<<kCtas, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      c->peers, c->rank, c->world, c->hidden, 0, nullptr, static_cast<const __half*>(partial),
      static_cast<const __half*>(residual), static_cast<__half*>(out), c->err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tp_fail(GROUT_ERR_CUDA, "allreduce launch", e);
  return GROUT_OK;
}

}  // extern "C"
