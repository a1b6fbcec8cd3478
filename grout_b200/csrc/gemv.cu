// Decode GEMV, y = W x (+ residual), for the projections around the
// attention path of a decode step (QKV, o_proj, gate/up, down_proj at batch
// 1).  The reference runs these as cuBLAS GEMVs (src/cublas.rs:434-470,
// recorded in its decode graph src/model.rs:3248-3260); at batch 1 they are
// pure weight streams, so each CTA streams its contiguous block of rows with
// bulk copies through a shared-memory ring (gemv_stream.cuh) — ~96 KB in
// flight per SM — and the warps' per-row sums meet in shared memory in a
// fixed order.
#include "internal.h"
#include "gemv_stream.cuh"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32 + 32;  // consumers + the bulk-copy producer warp
constexpr int kMaxRows = 512;               // rows per CTA (red slots per warp)

__global__ void __launch_bounds__(kThreads) gemv_kernel(const __half* __restrict__ w, int n, int k,
                                                        const __half* __restrict__ x,
                                                        const __half* __restrict__ residual,
                                                        __half* __restrict__ y, int rows_per_cta,
                                                        int* err) {
  extern __shared__ __align__(128) uint8_t gsmem[];  // x [k] f16 | ring | red [kWarps][rows]
  __half* xs = reinterpret_cast<__half*>(gsmem);
  const int xbytes = (k * 2 + 127) / 128 * 128;
  uint8_t* ring = gsmem + xbytes;
  float* red = reinterpret_cast<float*>(ring + kGemvStages * kGemvPiece);
  __shared__ __align__(8) uint64_t bars[2 * kGemvStages];
  __shared__ int s_abort;
  const int r0 = min(n, (int)blockIdx.x * rows_per_cta);
  const int r1 = min(n, r0 + rows_per_cta);
  const int nrows = r1 - r0;
  if (nrows <= 0) return;
  if (threadIdx.x == 0) {
    s_abort = 0;
    gemv_init_bars(bars, kWarps);
  }
  for (int i = threadIdx.x; i < kWarps * rows_per_cta; i += blockDim.x) red[i] = 0.f;
  for (int i = threadIdx.x * 8; i < k; i += blockDim.x * 8)
    *reinterpret_cast<uint4*>(&xs[i]) = __ldg(reinterpret_cast<const uint4*>(x + i));
  __syncthreads();
  gemv_stream_rows<kWarps>(w + (int64_t)r0 * k, nrows, k, xs, ring, bars, red, rows_per_cta, err,
                           70, (volatile int*)&s_abort);
  __syncthreads();
  if (s_abort) return;  // recorded: the rows are left unwritten
  for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
    float v = 0.f;
#pragma unroll 4
    for (int ww = 0; ww < kWarps; ++ww) v += red[ww * rows_per_cta + r];
    if (residual) v += __half2float(residual[r0 + r]);
    y[r0 + r] = __float2half_rn(v);
  }
}

int smem_bytes(int k, int rows_per_cta) {
  return (k * 2 + 127) / 128 * 128 + kGemvStages * kGemvPiece + kWarps * rows_per_cta * 4;
}

}  // namespace

int gemv_max_k() { return 32768; }

cudaError_t gemv_set_attributes() {
  return cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              smem_bytes(gemv_max_k(), kMaxRows));
}

cudaError_t launch_gemv(const __half* w, int n, int k, const __half* x, const __half* residual,
                        __half* y, int num_sms, int* err, cudaStream_t s) {
  int ctas = num_sms;
  if ((n + ctas - 1) / ctas > kMaxRows) ctas = (n + kMaxRows - 1) / kMaxRows;
  if (ctas > n) ctas = n;
  const int rows = (n + ctas - 1) / ctas;
  ctas = (n + rows - 1) / rows;
  gemv_kernel<<<ctas, kThreads, smem_bytes(k, rows), s>>>(w, n, k, x, residual, y, rows, err);
  return cudaGetLastError();
}

}  // namespace grout
