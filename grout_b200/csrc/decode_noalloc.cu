// Allocation-free variant of the split-K decode entry point.
//
// Some callers cannot hand this library a workspace: an engine whose device
// memory is entirely owned by a planner that has no slot for it, a host that
// reaches the library only through a narrow FFI with no device allocator, or
// code that is already inside a stream capture where a cudaMalloc would be
// illegal.  For them, grout_attn_decode_noalloc keeps the split-K scratch in a
// fixed array in this module's global memory instead of a caller buffer.
//
// The array is a file-scope __device__ object: every GPU that loads this
// library holds kNoAllocScratchBytes (512 KiB) of it until the process exits.  In host
// code its name is only a host-side stand-in, so the kernels receive the
// device address obtained with cudaGetSymbolAddress, once per device, with
// that device current.
//
// Sharing: every call on a device uses the same array.  Calls whose kernels
// can overlap on the GPU (different streams without ordering between them)
// race on it; calls on one stream, or otherwise ordered, are safe.  The array
// keeps the previous call's contents; the decode kernel writes every scratch
// entry it later reads (empty or skipped splits write 0 and -inf), so nothing
// needs clearing between calls.
#include <cstdio>
#include <mutex>

#include "../../include/grout_attn.h"
#include "internal.h"

namespace {

// 512 KiB per device.  Decode needs split-K scratch only when one KV head
// and sequence get more than 16 splits (up to 16 merge inside a cluster),
// i.e. for few (sequence, KV head) pairs over long contexts: the automatic
// split count then keeps about one CTA per SM, so the scratch is about
// SMs * G * 129 * 4 bytes (611 KB at G = 8 on 148 SMs) or less when the
// context caps the splits.  Shapes above the limit are rejected.
constexpr size_t kNoAllocScratchBytes = 512u << 10;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDev = 64;
void* g_scratch_addr[kMaxDev] = {};
std::mutex g_scratch_mu;

}  // namespace

extern "C" {

size_t grout_attn_decode_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

grout_status grout_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       int64_t cache_batch_stride, int64_t cache_head_stride,
                                       const uint32_t* d_position, void* out, int32_t batch,
                                       int32_t max_kv_len, const grout_attn_dims* dims,
                                       grout_stream_t stream) {
  if (!dims)  // let the regular entry point report the argument error
    return grout_attn_decode(q, k_cache, v_cache, cache_batch_stride, cache_head_stride,
                             d_position, out, batch, max_kv_len, dims, nullptr, 0, stream);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    char msg[160];
    std::snprintf(msg, sizeof(msg), "no usable current device (%s)", cudaGetErrorString(e));
    grout::set_last_error(msg);
    return GROUT_ERR_CUDA;
  }
  void* scratch = nullptr;
  {
    // First call on this device: resolve the scratch array's device address
    // (this device must be current).  Later calls reuse it.
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        char msg[160];
        std::snprintf(msg, sizeof(msg), "cudaGetSymbolAddress(scratch) failed on device %d: %s",
                      dev, cudaGetErrorString(e));
        grout::set_last_error(msg);
        return GROUT_ERR_CUDA;
      }
      g_scratch_addr[dev] = p;
    }
    scratch = g_scratch_addr[dev];
  }
  const size_t need = grout_attn_decode_workspace_bytes(batch, max_kv_len, dims);
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "decode needs %zu bytes of split-K scratch (batch %d, max_kv_len %d); the "
                  "allocation-free entry point holds at most %zu bytes: use grout_attn_decode "
                  "with a caller workspace",
                  need, batch, max_kv_len, kNoAllocScratchBytes);
    grout::set_last_error(msg);
    return GROUT_ERR_INVALID_ARG;
  }
  return grout_attn_decode(q, k_cache, v_cache, cache_batch_stride, cache_head_stride, d_position,
                           out, batch, max_kv_len, dims, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
