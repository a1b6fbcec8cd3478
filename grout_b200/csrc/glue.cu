// Decode-graph neighbours of the attention path: the fused residual add +
// RMSNorm and the SiLU-gated product that sit between the attention and MLP
// GEMVs of every layer.  They replace the reference's add_rms_norm_f16 /
// add_rms_norm_decode_raw_f16 / rms_norm_f16 (src/kernels.rs:4449-4600,
// 1530ff) and silu_mul_2d_f16 (src/kernels.rs:1497-1526), which its decode
// graph records per layer (src/model.rs:3264-3354).  Memory-bound and tiny at
// decode (one 5120-wide row): what they save is launches — one kernel each
// where an unfused torch expression launches several.
#include "internal.h"
#include "norm_rope.cuh"
#include "ptx.cuh"

namespace grout {
namespace {

constexpr int kRmsThreads = 512;
constexpr int kRmsChunks = 4;  // 16-byte chunks per thread: n <= 512 * 4 * 8 = 16384

// One CTA per row.  combined = x (+ residual) in f32; residual_out =
// f16(combined); out = f16((combined * inv) * w) with inv = rsqrt(sum(c^2) / n
// + eps), the reference's order of operations.
__global__ void __launch_bounds__(kRmsThreads) add_rms_norm_kernel(
    const __half* __restrict__ x, const __half* __restrict__ residual,
    const __half* __restrict__ w, __half* __restrict__ out, __half* __restrict__ residual_out,
    int n, float eps) {
  __shared__ float warp_sums[kRmsThreads / 32];
  const int64_t row = blockIdx.x;
  const __half* xr = x + row * n;
  const __half* rr = residual ? residual + row * n : nullptr;
  float c[kRmsChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRmsChunks; ++i) {
    const int col = (i * kRmsThreads + threadIdx.x) * 8;
    if (col < n) {
      unpack8(ldg16(xr + col), c[i]);
      if (rr) {
        float r[8];
        unpack8(ldg16(rr + col), r);
#pragma unroll
        for (int e = 0; e < 8; ++e) c[i][e] = r[e] + c[i][e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(c[i][e], c[i][e], ss);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kRmsThreads / 32; ++i) tot += warp_sums[i];
  const float inv = rsqrtf(tot / (float)n + eps);
#pragma unroll
  for (int i = 0; i < kRmsChunks; ++i) {
    const int col = (i * kRmsThreads + threadIdx.x) * 8;
    if (col < n) {
      float wf[8], y[8];
      unpack8(ldg16(w + col), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = c[i][e] * inv * wf[e];
      *reinterpret_cast<uint4*>(out + row * n + col) = pack8(y);
      if (residual_out) *reinterpret_cast<uint4*>(residual_out + row * n + col) = pack8(c[i]);
    }
  }
}

// gate_up [rows][2n] (gate | up) -> out [rows][n]: silu(g) * u =
// (g / (1 + exp(-g))) * u, f32 math, one f16 rounding.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __half* __restrict__ gate_up,
                                                       __half* __restrict__ out, int rows, int n) {
  const int64_t chunks = (int64_t)rows * (n / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (n / 8);
    const int col = (int)(i - r * (n / 8)) * 8;
    float g[8], u[8], y[8];
    unpack8(ldg16(gate_up + r * 2 * n + col), g);
    unpack8(ldg16(gate_up + r * 2 * n + n + col), u);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = (1.0f / (1.0f + expf(-g[e]))) * g[e] * u[e];
    *reinterpret_cast<uint4*>(out + r * n + col) = pack8(y);
  }
}

}  // namespace

cudaError_t launch_add_rms_norm(const __half* x, const __half* residual, const __half* w,
                                __half* out, __half* residual_out, int rows, int n, float eps,
                                cudaStream_t s) {
  add_rms_norm_kernel<<<rows, kRmsThreads, 0, s>>>(x, residual, w, out, residual_out, n, eps);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const __half* gate_up, __half* out, int rows, int n, int num_sms,
                            cudaStream_t s) {
  const int64_t chunks = (int64_t)rows * (n / 8);
  int64_t blocks = (chunks + 255) / 256;
  if (blocks > (int64_t)num_sms * 8) blocks = (int64_t)num_sms * 8;
  silu_mul_kernel<<<(unsigned)blocks, 256, 0, s>>>(gate_up, out, rows, n);
  return cudaGetLastError();
}

}  // namespace grout
