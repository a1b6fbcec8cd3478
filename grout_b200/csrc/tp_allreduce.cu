// Tensor-parallel GEMV fused with its all-reduce, over NVLink peer memory.
//
// y = residual + sum_over_ranks(W_r x_r): the row-parallel o_proj / down_proj
// of a tensor-parallel decode step followed by the all-reduce the reference
// would need (it is single-GPU; the split is the Megatron layout of config 5).
// One kernel per call on every rank:
//   1. CTA i computes rows [i*R, (i+1)*R) of its partial W_r x_r in f32
//      (each warp a K slice of eight rows at a time, 16-byte weight loads
//      software-pipelined one step ahead, x in shared memory);
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
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kMaxWorld = 8;
constexpr int kCtas = 148;        // CTAs per call (one per SM on B200)
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxRowsPerCta = 56;  // hidden <= 148 * 56
constexpr int kMaxK = 16384;      // x held in shared memory

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
  __shared__ __align__(16) __half xs[kMaxK];
  __shared__ unsigned s_epoch;
  __shared__ int s_ok;
  const int cta = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = (hidden + kCtas - 1) / kCtas;
  const int r0 = min(hidden, cta * rows), r1 = min(hidden, r0 + rows);

  unsigned char* mine = peers.base[rank];
  unsigned* epoch_p = reinterpret_cast<unsigned*>(mine + epoch_off(world, hidden)) + cta;
  volatile unsigned* broken = reinterpret_cast<unsigned*>(mine + broken_off(world, hidden));
  if (threadIdx.x == 0) {
    s_epoch = *epoch_p;
    s_ok = *broken == 0u;
    if (!s_ok && err) atomicCAS(err, 0, DEV_ERR_TIMEOUT_BASE + 61);
  }
  __syncthreads();
  if (!s_ok) return;  // an earlier call lost step with the peers
  if (w)
    for (int i = threadIdx.x * 8; i < k; i += blockDim.x * 8)
      *reinterpret_cast<uint4*>(&xs[i]) = __ldg(reinterpret_cast<const uint4*>(x + i));
  __syncthreads();
  const unsigned epoch = s_epoch + 1;
  const int slot = epoch & 1;

  // 1. partial rows.  Warp w covers the K slice [k0, k1) of every row of
  //    this CTA, eight rows per group; each lane holds one 16-byte chunk of
  //    the eight rows, and the loads of the next (group, chunk) are issued
  //    before the current one is consumed, so round trips overlap.  Warp
  //    partials meet in shared memory and are summed in a fixed order.
  __shared__ float red[kWarps][kMaxRowsPerCta];
  const int nwarps = blockDim.x >> 5;
  const int kw = ((k + nwarps - 1) / nwarps + 255) / 256 * 256;
  const int k0 = warp * kw, k1 = min(k, k0 + kw);
  const int nrows = r1 - r0;
  const int ngroups = (nrows + 7) / 8;
  const int nchunks = w ? max(0, (k1 - k0 + 255) / 256) : 0;
  const int total = ngroups * nchunks;
  auto load = [&](int it, uint4 (&wv)[8]) {
    const int g = it / nchunks, ch = it - g * nchunks;
    const int c = k0 + ch * 256 + lane * 8;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = r0 + g * 8 + u;
      if (c < k1 && r < r1) wv[u] = __ldg(reinterpret_cast<const uint4*>(w + (int64_t)r * k + c));
      else wv[u] = make_uint4(0, 0, 0, 0);
    }
  };
  uint4 cur[8], nxt[8];
  float acc[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) acc[u] = 0.f;
  if (total > 0) load(0, cur);
  for (int it = 0; it < total; ++it) {
    if (it + 1 < total) load(it + 1, nxt);
    const int g = it / nchunks, ch = it - g * nchunks;
    const int c = k0 + ch * 256 + lane * 8;
    if (c < k1) {
      const uint4 xv = *reinterpret_cast<const uint4*>(&xs[c]);
      const __half2* xh = reinterpret_cast<const __half2*>(&xv);
      float xf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 b = __half22float2(xh[e]);
        xf[2 * e] = b.x;
        xf[2 * e + 1] = b.y;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const __half2* wh = reinterpret_cast<const __half2*>(&cur[u]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a = __half22float2(wh[e]);
          acc[u] = fmaf(a.x, xf[2 * e], acc[u]);
          acc[u] = fmaf(a.y, xf[2 * e + 1], acc[u]);
        }
      }
    }
    if (ch == nchunks - 1) {  // group done: warp-reduce its eight rows
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float v = acc[u];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0 && g * 8 + u < nrows) red[warp][g * 8 + u] = v;
        acc[u] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) cur[u] = nxt[u];
  }
  if (!w) {  // exchange only: warp 0 holds the given partial (x[hidden])
    for (int i = lane; i < nrows; i += 32) red[warp][i] = warp == 0 ? __half2float(x[r0 + i]) : 0.f;
  } else if (nchunks == 0 && lane == 0) {  // this warp's K slice is empty
    for (int i = 0; i < nrows; ++i) red[warp][i] = 0.f;
  }
  __syncthreads();
  // The CTA's slice of partials goes into slot [slot][rank] of every rank's
  // receive buffer.
  if (threadIdx.x < nrows) {
    float v = 0.f;
    for (int ww = 0; ww < nwarps; ++ww) v += red[ww][threadIdx.x];
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
  if (k <= 0 || k % 8 || k > kMaxK)
    return tp_fail(GROUT_ERR_INVALID_ARG,
                   "gemv_allreduce: k must be a positive multiple of 8, at most 16384", cudaSuccess);
  const void* ptrs[] = {w, x, out};
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15)
      return tp_fail(GROUT_ERR_INVALID_ARG, "gemv_allreduce: pointers must be 16-byte aligned",
                     cudaSuccess);
  gemv_allreduce_kernel<<<kCtas, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
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
