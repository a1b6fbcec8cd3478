// Tensor-parallel GEMV fused with its all-reduce, over NVLink peer memory.
//
// y = residual + sum_over_ranks(W_r x_r): the row-parallel o_proj / down_proj
// of a tensor-parallel decode step followed by the all-reduce the reference
// would need (it is single-GPU; the split is the Megatron layout of config 5).
// One kernel per call on every rank:
//   1. CTA i computes rows [i*R, (i+1)*R) of its partial W_r x_r in f32
//      (one warp per row, 16-byte coalesced weight loads, x in shared memory);
//   2. it stores that slice into slot [epoch & 1][rank] of every peer's
//      receive buffer (plain stores through the CUDA-IPC mapping over NVLink;
//      no TMA, no multicast), fences at system scope and raises flag
//      [rank][i] = epoch + 1 in every peer;
//   3. it waits — bounded by a 2 s limit, after which it records a device
//      error and writes nothing — for flag [p][i] == epoch + 1 from every
//      peer p, then sums the partials in rank order 0..world-1 (identical
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
constexpr int kCtas = 128;        // CTAs per call (all resident: one per SM at most)
constexpr int kThreads = 256;
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
  const int r0 = cta * rows, r1 = min(hidden, r0 + rows);

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
  for (int i = threadIdx.x * 8; i < k; i += kThreads * 8)
    *reinterpret_cast<uint4*>(&xs[i]) = __ldg(reinterpret_cast<const uint4*>(x + i));
  __syncthreads();
  const unsigned epoch = s_epoch + 1;
  const int slot = epoch & 1;

  // 1-2. partial rows, stored into every rank's receive slot [slot][rank]
  for (int r = r0 + warp; r < r1; r += kThreads / 32) {
    const __half* wr = w + (int64_t)r * k;
    float acc = 0.f;
    for (int c = lane * 8; c < k; c += 32 * 8) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wr + c));
      const uint4 xv = *reinterpret_cast<const uint4*>(&xs[c]);
      const __half2* wh = reinterpret_cast<const __half2*>(&wv);
      const __half2* xh = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = __half22float2(wh[e]);
        const float2 b = __half22float2(xh[e]);
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) {
      for (int p = 0; p < world; ++p) {
        float* recv = reinterpret_cast<float*>(peers.base[p]) + ((size_t)slot * world + rank) * hidden;
        recv[r] = acc;
      }
    }
  }
  if (lane == 0) __threadfence_system();  // this warp's remote stores before the flags
  __syncthreads();
  // 2. flags: after a system-scope fence every peer may read our slice
  if (threadIdx.x < world) {
    __threadfence_system();
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
      while (ld_acquire_sys(f) != epoch) {
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
  for (int r = r0 + threadIdx.x; r < r1; r += kThreads) {
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
  if (world < 1 || world > kMaxWorld || hidden <= 0 || hidden % 8)
    return tp_fail(GROUT_ERR_INVALID_ARG, "tp comm: need 1 <= world <= 8 and hidden % 8 == 0",
                   cudaSuccess);
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

}  // extern "C"
