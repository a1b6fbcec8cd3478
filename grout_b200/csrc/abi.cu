// C ABI of the attention hot path (include/grout_attn.h): host-side
// validation, split selection, TMA descriptor encoding and launches.
//
// The checks mirror the reference's pre-launch `ensure!`s in
// execute_qk_norm_rope_kv_prefill_op_ctx (src/model.rs:4771-4822) and
// attend_seq_arc_into_ctx_with_position (src/model.rs:6864-6937): every
// shape/range problem is reported before any device work.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/grout_attn.h"
#include "internal.h"

namespace grout {
namespace {

thread_local std::string g_last_error;

grout_status fail(grout_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

#define CUDA_TRY(expr)                                                                        \
  do {                                                                                       \
    cudaError_t e_ = (expr);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      return fail(GROUT_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_));           \
  } while (0)

// Device error word: one int per device, in this module's global memory.
__device__ int g_device_error;

constexpr int kMaxDevices = 64;
struct DeviceState {
  bool ready = false;
  int* err = nullptr;
  int num_sms = 0;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

grout_status current_state(DeviceState** out) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(GROUT_ERR_UNSUPPORTED, "device id %d", dev);
  if (!g_dev[dev].ready) {
    grout_status st = grout_attn_init(dev);
    if (st != GROUT_OK) return st;
  }
  *out = &g_dev[dev];
  return GROUT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

grout_status check_dims(const grout_attn_dims* d, int max_group) {
  if (!d) return fail(GROUT_ERR_INVALID_ARG, "dims is null");
  if (d->head_dim != 128)
    return fail(GROUT_ERR_UNSUPPORTED, "head_dim must be 128, got %d", d->head_dim);
  if (d->num_q_heads <= 0 || d->num_kv_heads <= 0 || d->num_q_heads % d->num_kv_heads != 0)
    return fail(GROUT_ERR_INVALID_ARG, "num_q_heads=%d must be a positive multiple of num_kv_heads=%d",
                d->num_q_heads, d->num_kv_heads);
  if (max_group > 0 && d->num_q_heads / d->num_kv_heads > max_group)
    return fail(GROUT_ERR_UNSUPPORTED, "GQA group %d > %d", d->num_q_heads / d->num_kv_heads,
                max_group);
  if (d->max_seq <= 0) return fail(GROUT_ERR_INVALID_ARG, "max_seq=%d must be positive", d->max_seq);
  return GROUT_OK;
}

float qk_scale(const grout_attn_dims* d) {
  return d->qk_scale > 0.f ? d->qk_scale : 1.0f / std::sqrt((float)d->head_dim);
}

grout_status encode_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                        const uint64_t* strides_elems, const uint32_t* box, const char* what) {
  if (!g_encode) return fail(GROUT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t gd[5];
  cuuint64_t gs[4];
  cuuint32_t bx[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (dims[i] == 0 || dims[i] > (1ull << 32))
      return fail(GROUT_ERR_INVALID_ARG, "%s: tensor dim %d = %llu out of range", what, i,
                  (unsigned long long)dims[i]);
  }
  for (int i = 0; i + 1 < rank; ++i) {
    gs[i] = strides_elems[i] * 2;
    if (gs[i] % 16 != 0 || gs[i] >= (1ull << 40))
      return fail(GROUT_ERR_INVALID_ARG, "%s: stride %d (%llu bytes) must be a multiple of 16",
                  what, i, (unsigned long long)gs[i]);
  }
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank,
                        const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GROUT_ERR_CUDA, "%s: cuTensorMapEncodeTiled error %d", what, (int)r);
  return GROUT_OK;
}

// Split count for decode: about one CTA per SM in total (measured on B200:
// longer splits stream better than many short ones, and every extra split
// costs a partial write and its share of the merge), never fewer than 256
// keys per split.  Counts just above the cluster limit come down to it when
// the launch still covers most SMs, so the splits merge inside a cluster
// (no workspace, no merge launch).
int choose_splits(int32_t batch, int32_t max_kv_len, int32_t hkv, int num_sms) {
  const int keys = 64;
  const int tiles = (max_kv_len + keys - 1) / keys;
  const int64_t units = (int64_t)batch * hkv;
  int64_t nks = (num_sms + units - 1) / units;
  const int64_t hi = std::max(1, tiles / 4);
  if (nks > hi) nks = hi;
  if (nks > kDecodeMaxClusterSplits && units * kDecodeMaxClusterSplits >= (num_sms * 5) / 8)
    nks = kDecodeMaxClusterSplits;
  if (nks < 1) nks = 1;
  if (nks > 1024) nks = 1024;
  return (int)nks;
}

}  // namespace

void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

int* device_error_word() {
  DeviceState* ds;
  return current_state(&ds) == GROUT_OK ? ds->err : nullptr;
}

}  // namespace grout

using namespace grout;

extern "C" {

const char* grout_attn_last_error(void) { return g_last_error.c_str(); }
const char* grout_attn_version(void) { return "grout_attn 0.1.0 (sm_100a)"; }

grout_status grout_attn_init(int32_t device) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (device < 0 || device >= kMaxDevices) return fail(GROUT_ERR_INVALID_ARG, "device %d", device);
  if (g_dev[device].ready) return GROUT_OK;
  int prev = 0;
  CUDA_TRY(cudaGetDevice(&prev));
  CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) {
    cudaSetDevice(prev);
    return fail(GROUT_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    CUDA_TRY(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                              cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) {
      cudaSetDevice(prev);
      return fail(GROUT_ERR_CUDA, "cuTensorMapEncodeTiled not found");
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  CUDA_TRY(decode_set_attributes());
  CUDA_TRY(prefill_set_attributes());
  CUDA_TRY(qkv_gemm_set_attributes());
  void* err = nullptr;
  CUDA_TRY(cudaGetSymbolAddress(&err, g_device_error));
  CUDA_TRY(cudaMemset(err, 0, sizeof(int)));
  CUDA_TRY(cudaDeviceSynchronize());
  g_dev[device].err = static_cast<int*>(err);
  g_dev[device].num_sms = prop.multiProcessorCount;
  g_dev[device].ready = true;
  CUDA_TRY(cudaSetDevice(prev));
  return GROUT_OK;
}

grout_status grout_attn_check_device_error(int32_t* code) {
  DeviceState* ds;
  grout_status st = current_state(&ds);
  if (st != GROUT_OK) return st;
  CUDA_TRY(cudaDeviceSynchronize());
  int v = 0;
  CUDA_TRY(cudaMemcpy(&v, ds->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) CUDA_TRY(cudaMemset(ds->err, 0, sizeof(int)));
  if (code) *code = v;
  return v == 0 ? GROUT_OK : fail(GROUT_ERR_DEVICE, "device error 0x%x", v);
}

void grout_inv_freq_host(float theta, int32_t head_dim, float* out) {
  for (int32_t i = 0; i < head_dim; i += 2) {
    const float p = (float)i / (float)head_dim;
    out[i / 2] = 1.0f / powf(theta, p);
  }
}

size_t grout_rope_table_bytes(int32_t max_seq, int32_t head_dim) {
  if (max_seq <= 0 || head_dim <= 0) return 0;
  return (size_t)max_seq * (size_t)head_dim * sizeof(float);
}

grout_status grout_rope_table_init(float* d_table, const float* inv_freq_host, int32_t head_dim,
                                   int32_t max_seq, grout_stream_t stream) {
  if (!d_table || !inv_freq_host) return fail(GROUT_ERR_INVALID_ARG, "null pointer");
  if (head_dim != 128) return fail(GROUT_ERR_UNSUPPORTED, "head_dim must be 128");
  if (max_seq <= 0) return fail(GROUT_ERR_INVALID_ARG, "max_seq must be positive");
  if (!aligned16(d_table)) return fail(GROUT_ERR_INVALID_ARG, "table must be 16-byte aligned");
  const int half = head_dim / 2;
  std::vector<float> host((size_t)max_seq * head_dim);
  for (int32_t pos = 0; pos < max_seq; ++pos) {
    float* row = host.data() + (size_t)pos * head_dim;
    for (int i = 0; i < half; ++i) {
      const float angle = (float)pos * inv_freq_host[i];
      row[i] = (float)std::cos((double)angle);
      row[half + i] = (float)std::sin((double)angle);
    }
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaMemcpyAsync(d_table, host.data(), host.size() * sizeof(float),
                           cudaMemcpyHostToDevice, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  return GROUT_OK;
}

grout_status grout_qk_norm_rope_kv_prefill(const void* q, const void* k, const void* v,
                                           int64_t q_row_stride, int64_t kv_row_stride,
                                           const void* q_norm_w, const void* k_norm_w,
                                           const float* rope_table, void* q_out, void* k_cache,
                                           void* v_cache, int64_t cache_head_stride,
                                           int32_t position_start, int32_t seq_len,
                                           const grout_attn_dims* dims, grout_stream_t stream) {
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (seq_len == 0 && position_start >= 0 && position_start <= dims->max_seq) return GROUT_OK;
  const void* ptrs[] = {q, k, v, q_norm_w, k_norm_w, rope_table, q_out, k_cache, v_cache};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  if (seq_len < 0 || position_start < 0)
    return fail(GROUT_ERR_INVALID_ARG, "seq_len=%d position_start=%d", seq_len, position_start);
  if ((int64_t)position_start + seq_len > dims->max_seq)
    return fail(GROUT_ERR_INVALID_ARG, "fused qk/rope/kv range [%d..%lld) exceeds max_seq %d",
                position_start, (long long)position_start + seq_len, dims->max_seq);
  if (q_row_stride < (int64_t)dims->num_q_heads * 128 || q_row_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "q_row_stride=%lld", (long long)q_row_stride);
  if (kv_row_stride < (int64_t)dims->num_kv_heads * 128 || kv_row_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "kv_row_stride=%lld", (long long)kv_row_stride);
  if (cache_head_stride < (int64_t)dims->max_seq * 128 || cache_head_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "cache_head_stride=%lld", (long long)cache_head_stride);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  NormRopeArgs a{};
  a.q = static_cast<const __half*>(q);
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.q_row_stride = q_row_stride;
  a.kv_row_stride = kv_row_stride;
  a.q_w = static_cast<const __half*>(q_norm_w);
  a.k_w = static_cast<const __half*>(k_norm_w);
  a.table = rope_table;
  a.q_out = static_cast<__half*>(q_out);
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.cache_head_stride = cache_head_stride;
  a.pos0 = position_start;
  a.rows = seq_len;
  a.hq = dims->num_q_heads;
  a.hkv = dims->num_kv_heads;
  a.max_seq = dims->max_seq;
  a.eps = dims->rms_eps;
  a.decode = 0;
  a.err = ds->err;
  CUDA_TRY(launch_qk_norm_rope_kv(a, ds->num_sms, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

grout_status grout_qk_norm_rope_kv_decode(const void* qkv, const void* q_norm_w,
                                          const void* k_norm_w, const float* rope_table,
                                          void* q_out, void* k_cache, void* v_cache,
                                          int64_t cache_batch_stride, int64_t cache_head_stride,
                                          const uint32_t* d_position, int32_t batch,
                                          const grout_attn_dims* dims, grout_stream_t stream) {
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (batch == 0) return GROUT_OK;
  const void* ptrs[] = {qkv, q_norm_w, k_norm_w, rope_table, q_out, k_cache, v_cache, d_position};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p) && p != d_position)
      return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  if (batch < 0) return fail(GROUT_ERR_INVALID_ARG, "batch=%d", batch);
  if (cache_head_stride < (int64_t)dims->max_seq * 128 || cache_head_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "cache_head_stride=%lld", (long long)cache_head_stride);
  if (batch > 1 && (cache_batch_stride < cache_head_stride * dims->num_kv_heads || cache_batch_stride % 8))
    return fail(GROUT_ERR_INVALID_ARG, "cache_batch_stride=%lld", (long long)cache_batch_stride);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  NormRopeArgs a{};
  a.q = static_cast<const __half*>(qkv);
  a.q_row_stride = (int64_t)(dims->num_q_heads + 2 * dims->num_kv_heads) * 128;
  a.q_w = static_cast<const __half*>(q_norm_w);
  a.k_w = static_cast<const __half*>(k_norm_w);
  a.table = rope_table;
  a.q_out = static_cast<__half*>(q_out);
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.cache_batch_stride = cache_batch_stride;
  a.cache_head_stride = cache_head_stride;
  a.d_position = d_position;
  a.rows = batch;
  a.hq = dims->num_q_heads;
  a.hkv = dims->num_kv_heads;
  a.max_seq = dims->max_seq;
  a.eps = dims->rms_eps;
  a.decode = 1;
  a.err = ds->err;
  CUDA_TRY(launch_qk_norm_rope_kv(a, ds->num_sms, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

static grout_status prefill_common(const grout_prefill_varlen_args* p, int32_t single_len,
                                   int32_t single_pos0, const grout_attn_dims* dims,
                                   grout_stream_t stream, int32_t nsplit = 1,
                                   void* workspace = nullptr, size_t workspace_bytes = 0) {
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (p->batch == 0 || p->max_q_len == 0) return GROUT_OK;
  if (!p->q || !p->out || !p->k || !p->v) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
  const void* ptrs[] = {p->q, p->out, p->k, p->v};
  for (const void* x : ptrs)
    if (!aligned16(x)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", x);
  if (p->batch < 0 || p->max_q_len < 0)
    return fail(GROUT_ERR_INVALID_ARG, "batch=%d max_q_len=%d", p->batch, p->max_q_len);
  if (p->batch == 0 || p->max_q_len == 0) return GROUT_OK;
  const int64_t hq = dims->num_q_heads, hkv = dims->num_kv_heads;
  if (p->q_row_stride < hq * 128 || p->q_row_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "q_row_stride=%lld", (long long)p->q_row_stride);
  if (p->q_rows <= 0 || p->kv_rows <= 0)
    return fail(GROUT_ERR_INVALID_ARG, "q_rows=%lld kv_rows=%lld", (long long)p->q_rows,
                (long long)p->kv_rows);
  if (p->kv_row_stride <= 0 || p->kv_head_stride <= 0 || p->kv_batch_stride < 0 ||
      p->kv_row_stride % 8 || p->kv_head_stride % 8 || p->kv_batch_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "bad kv strides row=%lld head=%lld batch=%lld",
                (long long)p->kv_row_stride, (long long)p->kv_head_stride,
                (long long)p->kv_batch_stride);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;

  CUtensorMap tq, tk, tv;
  {
    const uint64_t dq[3] = {128, (uint64_t)hq, (uint64_t)p->q_rows};
    const uint64_t sq[2] = {128, (uint64_t)p->q_row_stride};
    const uint32_t bq[3] = {64, 1, 128};
    st = encode_map(&tq, p->q, 3, dq, sq, bq, "q");
    if (st != GROUT_OK) return st;
  }
  const bool batched = p->kv_batch_stride > 0 && p->batch > 1;
  {
    const uint64_t dk[4] = {128, (uint64_t)p->kv_rows, (uint64_t)hkv, (uint64_t)p->batch};
    const uint64_t sk[3] = {(uint64_t)p->kv_row_stride, (uint64_t)p->kv_head_stride,
                            (uint64_t)p->kv_batch_stride};
    const uint32_t bk[4] = {64, 128, 1, 1};
    const int rank = batched ? 4 : 3;
    st = encode_map(&tk, p->k, rank, dk, sk, bk, "k");
    if (st != GROUT_OK) return st;
    st = encode_map(&tv, p->v, rank, dk, sk, bk, "v");
    if (st != GROUT_OK) return st;
  }
  PrefillArgs a{};
  a.out = static_cast<__half*>(p->out);
  a.q_row_stride = p->q_row_stride;
  a.cu_q = p->cu_seqlens_q;
  a.pos0 = p->position_start;
  a.kv_start = p->kv_start;
  a.batch = p->batch;
  a.max_q_len = p->max_q_len;
  a.hq = (int32_t)hq;
  a.hkv = (int32_t)hkv;
  a.kv_batched = batched ? 1 : 0;
  a.single_len = single_len;
  a.single_pos0 = single_pos0;
  a.scale_log2 = qk_scale(dims) / logf(2.0f);
  a.err = ds->err;
  a.nsplit = nsplit;
  if (nsplit > 1) {
    const size_t need = grout_attn_prefill_splitk_workspace_bytes(p->batch, p->max_q_len,
                                                                  (int32_t)hq, nsplit);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
      return fail(GROUT_ERR_INVALID_ARG, "workspace of %zu bytes (16-byte aligned) required, got %zu",
                  need, workspace ? workspace_bytes : (size_t)0);
    a.part = static_cast<float*>(workspace);
  }
  CUDA_TRY(launch_prefill(a, tq, tk, tv, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

int32_t grout_attn_prefill_splits(int32_t batch, int32_t max_q_len, const grout_attn_dims* dims) {
  if (!dims || batch <= 0 || max_q_len <= 0 || dims->num_q_heads <= 0) return 1;
  DeviceState* ds;
  int sms = 148;
  if (current_state(&ds) == GROUT_OK) sms = ds->num_sms;
  const int64_t items = (int64_t)((max_q_len + 255) / 256) * dims->num_q_heads * batch;
  if (items >= sms) return 1;
  // enough items to cover the SMs, and chunks of at least four KV tiles
  int32_t n = (int32_t)((sms + items - 1) / items);
  const int32_t tiles = (max_q_len + 127) / 128;
  n = std::min(n, std::max(1, tiles / 4));
  return std::max(1, std::min(n, 8));
}

size_t grout_attn_prefill_splitk_workspace_bytes(int32_t batch, int32_t max_q_len,
                                                 int32_t num_q_heads, int32_t num_splits) {
  if (batch <= 0 || max_q_len <= 0 || num_q_heads <= 0 || num_splits <= 1) return 0;
  const size_t base_items = (size_t)((max_q_len + 255) / 256) * num_q_heads * batch;
  return base_items * num_splits * 2 * kPrefillPartFloats * sizeof(float);
}

grout_status grout_attn_prefill_splitk(const grout_prefill_varlen_args* args, int32_t num_splits,
                                       const grout_attn_dims* dims, void* workspace,
                                       size_t workspace_bytes, grout_stream_t stream) {
  if (!args) return fail(GROUT_ERR_INVALID_ARG, "args is null");
  if (num_splits < 1 || num_splits > 8)
    return fail(GROUT_ERR_INVALID_ARG, "num_splits=%d must be in [1, 8]", num_splits);
  if (!args->cu_seqlens_q && args->batch != 1)
    return fail(GROUT_ERR_INVALID_ARG, "cu_seqlens_q is null with batch=%d", args->batch);
  // position_start is per sequence on the device; single sequences without
  // cu_seqlens use position 0 (pass position_start for an offset)
  return prefill_common(args, args->cu_seqlens_q ? 0 : args->max_q_len, 0, dims, stream,
                        num_splits, workspace, workspace_bytes);
}

grout_status grout_attn_prefill(const void* q, const void* k_cache, const void* v_cache,
                                void* out, int64_t cache_head_stride, int32_t position_start,
                                int32_t seq_len, const grout_attn_dims* dims,
                                grout_stream_t stream) {
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (seq_len < 0 || position_start < 0)
    return fail(GROUT_ERR_INVALID_ARG, "seq_len=%d position_start=%d", seq_len, position_start);
  if ((int64_t)position_start + seq_len > dims->max_seq)
    return fail(GROUT_ERR_INVALID_ARG, "attention range [%d..%lld) exceeds max_seq %d",
                position_start, (long long)position_start + seq_len, dims->max_seq);
  if (cache_head_stride < (int64_t)dims->max_seq * 128)
    return fail(GROUT_ERR_INVALID_ARG, "cache_head_stride=%lld", (long long)cache_head_stride);
  if (seq_len == 0) return GROUT_OK;
  grout_prefill_varlen_args p{};
  p.q = q;
  p.out = out;
  p.q_row_stride = (int64_t)dims->num_q_heads * 128;
  p.q_rows = seq_len;
  p.k = k_cache;
  p.v = v_cache;
  p.kv_batch_stride = 0;
  p.kv_row_stride = 128;
  p.kv_head_stride = cache_head_stride;
  p.kv_rows = dims->max_seq;
  p.batch = 1;
  p.max_q_len = seq_len;
  return prefill_common(&p, seq_len, position_start, dims, stream);
}

grout_status grout_attn_prefill_varlen(const grout_prefill_varlen_args* args,
                                       const grout_attn_dims* dims, grout_stream_t stream) {
  if (!args) return fail(GROUT_ERR_INVALID_ARG, "args is null");
  if (!args->cu_seqlens_q) return fail(GROUT_ERR_INVALID_ARG, "cu_seqlens_q is null");
  return prefill_common(args, 0, 0, dims, stream);
}

int32_t grout_attn_decode_splits(int32_t batch, int32_t max_kv_len, const grout_attn_dims* dims) {
  if (!dims || batch <= 0 || max_kv_len <= 0 || dims->num_kv_heads <= 0) return 1;
  DeviceState* ds;
  int sms = 148;
  if (current_state(&ds) == GROUT_OK) sms = ds->num_sms;
  return choose_splits(batch, max_kv_len, dims->num_kv_heads, sms);
}

// Split counts up to kDecodeMaxClusterSplits merge inside a thread-block
// cluster and need no workspace.
static size_t decode_ws_bytes(int32_t batch, int32_t hq, int32_t nks) {
  if (nks <= kDecodeMaxClusterSplits) return 0;
  return (size_t)batch * hq * nks * (128 + 1) * sizeof(float);
}

size_t grout_attn_decode_workspace_bytes(int32_t batch, int32_t max_kv_len,
                                         const grout_attn_dims* dims) {
  if (!dims) return 0;
  return decode_ws_bytes(batch, dims->num_q_heads, grout_attn_decode_splits(batch, max_kv_len, dims));
}

// Shared by the decode entry points: validation of the cache / workspace
// arguments, the tensor maps and the launch.  `fused` (may be null) carries
// the fused norm/RoPE/KV-write inputs; then q is unused.
static grout_status decode_common(const void* q, const void* k_cache, const void* v_cache,
                                  int64_t cache_batch_stride, int64_t cache_head_stride,
                                  const uint32_t* d_position, void* out, int32_t batch,
                                  int32_t max_kv_len, int32_t num_splits,
                                  const grout_attn_dims* dims, void* workspace,
                                  size_t workspace_bytes, DecodeArgs* fused,
                                  grout_stream_t stream) {
  grout_status st = check_dims(dims, 8);
  if (st != GROUT_OK) return st;
  if (batch < 0) return fail(GROUT_ERR_INVALID_ARG, "batch=%d", batch);
  if (batch == 0) return GROUT_OK;  // empty call: nothing to read or write
  const void* ptrs[] = {fused ? k_cache : q, k_cache, v_cache, out};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  if (!d_position) return fail(GROUT_ERR_INVALID_ARG, "d_position is null");
  if (max_kv_len <= 0 || max_kv_len > dims->max_seq)
    return fail(GROUT_ERR_INVALID_ARG, "max_kv_len=%d must be in [1, max_seq=%d]", max_kv_len,
                dims->max_seq);
  if (num_splits < 1 || num_splits > 1024)
    return fail(GROUT_ERR_INVALID_ARG, "num_splits=%d", num_splits);
  if (cache_head_stride < (int64_t)dims->max_seq * 128 || cache_head_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "cache_head_stride=%lld", (long long)cache_head_stride);
  if (batch > 1 &&
      (cache_batch_stride < cache_head_stride * dims->num_kv_heads || cache_batch_stride % 8))
    return fail(GROUT_ERR_INVALID_ARG, "cache_batch_stride=%lld", (long long)cache_batch_stride);
  const size_t need = decode_ws_bytes(batch, dims->num_q_heads, num_splits);
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned16(workspace)))
    return fail(GROUT_ERR_INVALID_ARG, "workspace of %zu bytes (16-byte aligned) required, got %zu",
                need, workspace ? workspace_bytes : (size_t)0);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  CUtensorMap tk, tv;
  const uint64_t dk[4] = {128, (uint64_t)dims->max_seq, (uint64_t)dims->num_kv_heads,
                          (uint64_t)batch};
  const uint64_t sk[3] = {128, (uint64_t)cache_head_stride,
                          (uint64_t)(batch > 1 ? cache_batch_stride : cache_head_stride * dims->num_kv_heads)};
  const uint32_t bk[4] = {64, 64, 1, 1};
  st = encode_map(&tk, k_cache, 4, dk, sk, bk, "k_cache");
  if (st != GROUT_OK) return st;
  st = encode_map(&tv, v_cache, 4, dk, sk, bk, "v_cache");
  if (st != GROUT_OK) return st;
  DecodeArgs a = fused ? *fused : DecodeArgs{};
  a.q = static_cast<const __half*>(q);
  a.out = static_cast<__half*>(out);
  a.part_o = need ? static_cast<float*>(workspace) : nullptr;
  a.part_lse = need ? static_cast<float*>(workspace) + (size_t)batch * dims->num_q_heads * num_splits * 128
                    : nullptr;
  a.d_position = d_position;
  a.batch = batch;
  a.hq = dims->num_q_heads;
  a.hkv = dims->num_kv_heads;
  a.nks = num_splits;
  a.cluster = num_splits > 1 && need == 0;
  a.max_seq = dims->max_seq;
  float scale = qk_scale(dims);
  if (dims->flags & GROUT_FLAG_DECODE_SCALE_F16) scale = __half2float(__float2half_rn(scale));
  a.scale_log2 = scale / logf(2.0f);
  a.err = ds->err;
  a.k_cache = static_cast<__half*>(const_cast<void*>(k_cache));
  a.v_cache = static_cast<__half*>(const_cast<void*>(v_cache));
  a.cache_batch_stride = batch > 1 ? cache_batch_stride : 0;
  a.cache_head_stride = cache_head_stride;
  CUDA_TRY(launch_decode(a, tk, tv, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

grout_status grout_attn_decode_ex(const void* q, const void* k_cache, const void* v_cache,
                                  int64_t cache_batch_stride, int64_t cache_head_stride,
                                  const uint32_t* d_position, void* out, int32_t batch,
                                  int32_t max_kv_len, int32_t num_splits,
                                  const grout_attn_dims* dims, void* workspace,
                                  size_t workspace_bytes, grout_stream_t stream) {
  return decode_common(q, k_cache, v_cache, cache_batch_stride, cache_head_stride, d_position,
                       out, batch, max_kv_len, num_splits, dims, workspace, workspace_bytes,
                       nullptr, stream);
}

grout_status grout_attn_decode_fused(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                     const float* rope_table, void* q_out, void* k_cache,
                                     void* v_cache, int64_t cache_batch_stride,
                                     int64_t cache_head_stride, const uint32_t* d_position,
                                     void* out, int32_t batch, int32_t max_kv_len,
                                     const grout_attn_dims* dims, void* workspace,
                                     size_t workspace_bytes, grout_stream_t stream) {
  grout_status st = check_dims(dims, 8);
  if (st != GROUT_OK) return st;
  if (batch <= 0) return batch == 0 ? GROUT_OK : fail(GROUT_ERR_INVALID_ARG, "batch=%d", batch);
  const void* ptrs[] = {qkv, q_norm_w, k_norm_w, rope_table};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  if (q_out && !aligned16(q_out))
    return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", q_out);
  DecodeArgs f{};
  f.qkv = static_cast<const __half*>(qkv);
  f.qkv_row_stride = (int64_t)(dims->num_q_heads + 2 * dims->num_kv_heads) * 128;
  f.q_w = static_cast<const __half*>(q_norm_w);
  f.k_w = static_cast<const __half*>(k_norm_w);
  f.table = rope_table;
  f.eps = dims->rms_eps;
  f.q_out = static_cast<__half*>(q_out);
  return decode_common(nullptr, k_cache, v_cache, cache_batch_stride, cache_head_stride,
                       d_position, out, batch, max_kv_len,
                       grout_attn_decode_splits(batch, max_kv_len, dims), dims, workspace,
                       workspace_bytes, &f, stream);
}

grout_status grout_attn_decode(const void* q, const void* k_cache, const void* v_cache,
                               int64_t cache_batch_stride, int64_t cache_head_stride,
                               const uint32_t* d_position, void* out, int32_t batch,
                               int32_t max_kv_len, const grout_attn_dims* dims, void* workspace,
                               size_t workspace_bytes, grout_stream_t stream) {
  grout_status st = check_dims(dims, 8);
  if (st != GROUT_OK) return st;
  if (batch <= 0) return batch == 0 ? GROUT_OK : fail(GROUT_ERR_INVALID_ARG, "batch=%d", batch);
  const int32_t nks = grout_attn_decode_splits(batch, max_kv_len, dims);
  return grout_attn_decode_ex(q, k_cache, v_cache, cache_batch_stride, cache_head_stride,
                              d_position, out, batch, max_kv_len, nks, dims, workspace,
                              workspace_bytes, stream);
}

/* ------------------------------------------------------- decode-graph glue */

grout_status grout_add_rms_norm(const void* x, const void* residual, const void* weight, void* out,
                                void* residual_out, int32_t rows, int32_t n, float eps,
                                grout_stream_t stream) {
  if (rows < 0 || n <= 0 || n % 8 || n > 16384)
    return fail(GROUT_ERR_INVALID_ARG, "add_rms_norm: rows=%d n=%d (n a multiple of 8, <= 16384)",
                rows, n);
  if (rows == 0) return GROUT_OK;
  const void* ptrs[] = {x, weight, out};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  if ((residual && !aligned16(residual)) || (residual_out && !aligned16(residual_out)))
    return fail(GROUT_ERR_INVALID_ARG, "residual pointers must be 16-byte aligned");
  DeviceState* ds;
  grout_status st = current_state(&ds);
  if (st != GROUT_OK) return st;
  CUDA_TRY(launch_add_rms_norm(static_cast<const __half*>(x), static_cast<const __half*>(residual),
                               static_cast<const __half*>(weight), static_cast<__half*>(out),
                               static_cast<__half*>(residual_out), rows, n, eps,
                               reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

grout_status grout_silu_mul(const void* gate_up, void* out, int32_t rows, int32_t n,
                            grout_stream_t stream) {
  if (rows < 0 || n <= 0 || n % 8)
    return fail(GROUT_ERR_INVALID_ARG, "silu_mul: rows=%d n=%d (n a multiple of 8)", rows, n);
  if (rows == 0) return GROUT_OK;
  if (!gate_up || !out) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned16(gate_up) || !aligned16(out))
    return fail(GROUT_ERR_INVALID_ARG, "gate_up and out must be 16-byte aligned");
  DeviceState* ds;
  grout_status st = current_state(&ds);
  if (st != GROUT_OK) return st;
  CUDA_TRY(launch_silu_mul(static_cast<const __half*>(gate_up), static_cast<__half*>(out), rows, n,
                           ds->num_sms, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

/* ----------------------------------------------------------- paged caches */

static grout_status check_pages(const void* k_pages, const void* v_pages, int32_t num_pages,
                                int32_t page_size, const int32_t* page_table,
                                int64_t table_stride, const grout_attn_dims* dims) {
  if (!k_pages || !v_pages || !page_table) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned16(k_pages) || !aligned16(v_pages))
    return fail(GROUT_ERR_INVALID_ARG, "page pools must be 16-byte aligned");
  if (page_size < 64 || page_size > 4096 || page_size % 64)
    return fail(GROUT_ERR_INVALID_ARG, "page_size=%d must be a multiple of 64 in [64, 4096]",
                page_size);
  if (num_pages < 1) return fail(GROUT_ERR_INVALID_ARG, "num_pages=%d", num_pages);
  const int64_t need = ((int64_t)dims->max_seq + page_size - 1) / page_size;
  if (table_stride < need)
    return fail(GROUT_ERR_INVALID_ARG, "table_stride=%lld < ceil(max_seq / page_size)=%lld",
                (long long)table_stride, (long long)need);
  return GROUT_OK;
}

grout_status grout_attn_prefill_paged(const grout_prefill_paged_args* p,
                                      const grout_attn_dims* dims, grout_stream_t stream) {
  if (!p) return fail(GROUT_ERR_INVALID_ARG, "args is null");
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (p->batch < 0 || p->max_q_len < 0)
    return fail(GROUT_ERR_INVALID_ARG, "batch=%d max_q_len=%d", p->batch, p->max_q_len);
  if (p->batch == 0 || p->max_q_len == 0) return GROUT_OK;
  if (!p->q || !p->out) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned16(p->q) || !aligned16(p->out))
    return fail(GROUT_ERR_INVALID_ARG, "q and out must be 16-byte aligned");
  if (!p->cu_seqlens_q && p->batch != 1)
    return fail(GROUT_ERR_INVALID_ARG, "cu_seqlens_q is null with batch=%d", p->batch);
  st = check_pages(p->k_pages, p->v_pages, p->num_pages, p->page_size, p->page_table,
                   p->table_stride, dims);
  if (st != GROUT_OK) return st;
  const int64_t hq = dims->num_q_heads, hkv = dims->num_kv_heads;
  if (p->q_row_stride < hq * 128 || p->q_row_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "q_row_stride=%lld", (long long)p->q_row_stride);
  if (p->q_rows <= 0 || (!p->cu_seqlens_q && p->q_rows < p->max_q_len))
    return fail(GROUT_ERR_INVALID_ARG, "q_rows=%lld", (long long)p->q_rows);
  if (!p->position_start && p->max_q_len > dims->max_seq)
    return fail(GROUT_ERR_INVALID_ARG, "max_q_len=%d exceeds max_seq %d", p->max_q_len,
                dims->max_seq);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  CUtensorMap tq, tk, tv;
  const uint64_t dq[3] = {128, (uint64_t)hq, (uint64_t)p->q_rows};
  const uint64_t sq[2] = {128, (uint64_t)p->q_row_stride};
  const uint32_t bq[3] = {64, 1, 128};
  st = encode_map(&tq, p->q, 3, dq, sq, bq, "q");
  if (st != GROUT_OK) return st;
  const uint64_t dk[4] = {128, (uint64_t)p->page_size, (uint64_t)hkv, (uint64_t)p->num_pages};
  const uint64_t sk[3] = {128, (uint64_t)p->page_size * 128, (uint64_t)p->page_size * 128 * hkv};
  const uint32_t bk[4] = {64, 64, 1, 1};
  st = encode_map(&tk, p->k_pages, 4, dk, sk, bk, "k_pages");
  if (st != GROUT_OK) return st;
  st = encode_map(&tv, p->v_pages, 4, dk, sk, bk, "v_pages");
  if (st != GROUT_OK) return st;
  PrefillArgs a{};
  a.out = static_cast<__half*>(p->out);
  a.q_row_stride = p->q_row_stride;
  a.cu_q = p->cu_seqlens_q;
  a.pos0 = p->position_start;
  a.kv_start = nullptr;
  a.batch = p->batch;
  a.max_q_len = p->max_q_len;
  a.hq = (int32_t)hq;
  a.hkv = (int32_t)hkv;
  a.kv_batched = 0;
  a.single_len = p->max_q_len;
  a.single_pos0 = 0;
  a.scale_log2 = qk_scale(dims) / logf(2.0f);
  a.err = ds->err;
  a.page_table = p->page_table;
  a.table_stride = p->table_stride;
  a.page_size = p->page_size;
  a.num_pages = p->num_pages;
  a.nsplit = 1;
  CUDA_TRY(launch_prefill(a, tq, tk, tv, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

grout_status grout_attn_decode_paged(const void* q, const void* k_pages, const void* v_pages,
                                     int32_t num_pages, int32_t page_size,
                                     const int32_t* page_table, int32_t table_stride,
                                     const uint32_t* d_position, void* out, int32_t batch,
                                     int32_t max_kv_len, int32_t num_splits,
                                     const grout_attn_dims* dims, void* workspace,
                                     size_t workspace_bytes, grout_stream_t stream) {
  grout_status st = check_dims(dims, 8);
  if (st != GROUT_OK) return st;
  if (batch < 0) return fail(GROUT_ERR_INVALID_ARG, "batch=%d", batch);
  if (batch == 0) return GROUT_OK;  // empty call: nothing to read or write
  if (!q || !out || !d_position) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned16(q) || !aligned16(out))
    return fail(GROUT_ERR_INVALID_ARG, "q and out must be 16-byte aligned");
  st = check_pages(k_pages, v_pages, num_pages, page_size, page_table, table_stride, dims);
  if (st != GROUT_OK) return st;
  if (max_kv_len <= 0 || max_kv_len > dims->max_seq)
    return fail(GROUT_ERR_INVALID_ARG, "max_kv_len=%d must be in [1, max_seq=%d]", max_kv_len,
                dims->max_seq);
  if (num_splits == 0) num_splits = grout_attn_decode_splits(batch, max_kv_len, dims);
  if (num_splits < 1 || num_splits > 1024)
    return fail(GROUT_ERR_INVALID_ARG, "num_splits=%d", num_splits);
  const size_t need = decode_ws_bytes(batch, dims->num_q_heads, num_splits);
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned16(workspace)))
    return fail(GROUT_ERR_INVALID_ARG, "workspace of %zu bytes (16-byte aligned) required, got %zu",
                need, workspace ? workspace_bytes : (size_t)0);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  CUtensorMap tk, tv;
  const uint64_t dk[4] = {128, (uint64_t)page_size, (uint64_t)dims->num_kv_heads,
                          (uint64_t)num_pages};
  const uint64_t sk[3] = {128, (uint64_t)page_size * 128,
                          (uint64_t)page_size * 128 * (uint64_t)dims->num_kv_heads};
  const uint32_t bk[4] = {64, 64, 1, 1};
  st = encode_map(&tk, k_pages, 4, dk, sk, bk, "k_pages");
  if (st != GROUT_OK) return st;
  st = encode_map(&tv, v_pages, 4, dk, sk, bk, "v_pages");
  if (st != GROUT_OK) return st;
  DecodeArgs a{};
  a.q = static_cast<const __half*>(q);
  a.out = static_cast<__half*>(out);
  a.part_o = need ? static_cast<float*>(workspace) : nullptr;
  a.part_lse = need ? static_cast<float*>(workspace) + (size_t)batch * dims->num_q_heads * num_splits * 128
                    : nullptr;
  a.d_position = d_position;
  a.batch = batch;
  a.hq = dims->num_q_heads;
  a.hkv = dims->num_kv_heads;
  a.nks = num_splits;
  a.cluster = num_splits > 1 && need == 0;
  a.max_seq = dims->max_seq;
  float scale = qk_scale(dims);
  if (dims->flags & GROUT_FLAG_DECODE_SCALE_F16) scale = __half2float(__float2half_rn(scale));
  a.scale_log2 = scale / logf(2.0f);
  a.err = ds->err;
  a.page_table = page_table;
  a.table_stride = table_stride;
  a.page_size = page_size;
  a.num_pages = num_pages;
  CUDA_TRY(launch_decode(a, tk, tv, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

grout_status grout_qk_norm_rope_kv_decode_paged(
    const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* rope_table,
    void* q_out, void* k_pages, void* v_pages, int32_t num_pages, int32_t page_size,
    const int32_t* page_table, int32_t table_stride, const uint32_t* d_position, int32_t batch,
    const grout_attn_dims* dims, grout_stream_t stream) {
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (batch < 0) return fail(GROUT_ERR_INVALID_ARG, "batch=%d", batch);
  if (batch == 0) return GROUT_OK;
  const void* ptrs[] = {qkv, q_norm_w, k_norm_w, rope_table, q_out};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  if (!d_position) return fail(GROUT_ERR_INVALID_ARG, "d_position is null");
  st = check_pages(k_pages, v_pages, num_pages, page_size, page_table, table_stride, dims);
  if (st != GROUT_OK) return st;
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  NormRopeArgs a{};
  a.q = static_cast<const __half*>(qkv);
  a.q_row_stride = (int64_t)(dims->num_q_heads + 2 * dims->num_kv_heads) * 128;
  a.q_w = static_cast<const __half*>(q_norm_w);
  a.k_w = static_cast<const __half*>(k_norm_w);
  a.table = rope_table;
  a.q_out = static_cast<__half*>(q_out);
  a.k_cache = static_cast<__half*>(k_pages);
  a.v_cache = static_cast<__half*>(v_pages);
  a.d_position = d_position;
  a.rows = batch;
  a.hq = dims->num_q_heads;
  a.hkv = dims->num_kv_heads;
  a.max_seq = dims->max_seq;
  a.eps = dims->rms_eps;
  a.decode = 1;
  a.err = ds->err;
  a.page_table = page_table;
  a.table_stride = table_stride;
  a.page_size = page_size;
  a.num_pages = num_pages;
  CUDA_TRY(launch_qk_norm_rope_kv(a, ds->num_sms, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

grout_status grout_qk_norm_rope_kv_prefill_paged(
    const void* q, const void* k, const void* v, int64_t q_row_stride, int64_t kv_row_stride,
    const void* q_norm_w, const void* k_norm_w, const float* rope_table, void* q_out,
    void* k_pages, void* v_pages, int32_t num_pages, int32_t page_size,
    const int32_t* page_table, int32_t position_start, int32_t seq_len,
    const grout_attn_dims* dims, grout_stream_t stream) {
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (seq_len == 0 && position_start >= 0 && position_start <= dims->max_seq) return GROUT_OK;
  const void* ptrs[] = {q, k, v, q_norm_w, k_norm_w, rope_table, q_out};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  const int64_t table_len = ((int64_t)dims->max_seq + page_size - 1) / (page_size > 0 ? page_size : 1);
  st = check_pages(k_pages, v_pages, num_pages, page_size, page_table, table_len, dims);
  if (st != GROUT_OK) return st;
  if (seq_len < 0 || position_start < 0)
    return fail(GROUT_ERR_INVALID_ARG, "seq_len=%d position_start=%d", seq_len, position_start);
  if ((int64_t)position_start + seq_len > dims->max_seq)
    return fail(GROUT_ERR_INVALID_ARG, "fused qk/rope/kv range [%d..%lld) exceeds max_seq %d",
                position_start, (long long)position_start + seq_len, dims->max_seq);
  if (q_row_stride < (int64_t)dims->num_q_heads * 128 || q_row_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "q_row_stride=%lld", (long long)q_row_stride);
  if (kv_row_stride < (int64_t)dims->num_kv_heads * 128 || kv_row_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "kv_row_stride=%lld", (long long)kv_row_stride);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  NormRopeArgs a{};
  a.q = static_cast<const __half*>(q);
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.q_row_stride = q_row_stride;
  a.kv_row_stride = kv_row_stride;
  a.q_w = static_cast<const __half*>(q_norm_w);
  a.k_w = static_cast<const __half*>(k_norm_w);
  a.table = rope_table;
  a.q_out = static_cast<__half*>(q_out);
  a.k_cache = static_cast<__half*>(k_pages);
  a.v_cache = static_cast<__half*>(v_pages);
  a.pos0 = position_start;
  a.rows = seq_len;
  a.hq = dims->num_q_heads;
  a.hkv = dims->num_kv_heads;
  a.max_seq = dims->max_seq;
  a.eps = dims->rms_eps;
  a.decode = 0;
  a.err = ds->err;
  a.page_table = page_table;
  a.table_stride = 0;
  a.page_size = page_size;
  a.num_pages = num_pages;
  CUDA_TRY(launch_qk_norm_rope_kv(a, ds->num_sms, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

grout_status grout_qkv_proj_norm_rope_kv_prefill(
    const void* x, int64_t x_row_stride, const void* w_qkv, int32_t hidden, const void* q_norm_w,
    const void* k_norm_w, const float* rope_table, void* q_out, void* k_cache, void* v_cache,
    int64_t cache_head_stride, void* qkv_out, int32_t position_start, int32_t seq_len,
    const grout_attn_dims* dims, grout_stream_t stream) {
  grout_status st = check_dims(dims, 0);
  if (st != GROUT_OK) return st;
  if (seq_len == 0 && position_start >= 0 && position_start <= dims->max_seq) return GROUT_OK;
  const void* ptrs[] = {x, w_qkv, q_norm_w, k_norm_w, rope_table, q_out, k_cache, v_cache};
  for (const void* p : ptrs) {
    if (!p) return fail(GROUT_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(p)) return fail(GROUT_ERR_INVALID_ARG, "pointer %p is not 16-byte aligned", p);
  }
  if (qkv_out && !aligned16(qkv_out))
    return fail(GROUT_ERR_INVALID_ARG, "qkv_out is not 16-byte aligned");
  if (seq_len < 0 || position_start < 0)
    return fail(GROUT_ERR_INVALID_ARG, "seq_len=%d position_start=%d", seq_len, position_start);
  if ((int64_t)position_start + seq_len > dims->max_seq)
    return fail(GROUT_ERR_INVALID_ARG, "fused qkv/rope/kv range [%d..%lld) exceeds max_seq %d",
                position_start, (long long)position_start + seq_len, dims->max_seq);
  if (hidden <= 0 || hidden % 64)
    return fail(GROUT_ERR_INVALID_ARG, "hidden=%d must be a positive multiple of 64", hidden);
  if (x_row_stride < hidden || x_row_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "x_row_stride=%lld", (long long)x_row_stride);
  if (cache_head_stride < (int64_t)dims->max_seq * 128 || cache_head_stride % 8)
    return fail(GROUT_ERR_INVALID_ARG, "cache_head_stride=%lld", (long long)cache_head_stride);
  DeviceState* ds;
  st = current_state(&ds);
  if (st != GROUT_OK) return st;
  const int64_t heads = (int64_t)dims->num_q_heads + 2 * dims->num_kv_heads;
  CUtensorMap tx, tw;
  {
    const uint64_t dx[3] = {(uint64_t)hidden, (uint64_t)seq_len, 1};
    const uint64_t sx[2] = {(uint64_t)x_row_stride, (uint64_t)x_row_stride * (uint64_t)seq_len};
    const uint32_t bx[3] = {64, 128, 1};
    st = encode_map(&tx, x, 3, dx, sx, bx, "x");
    if (st != GROUT_OK) return st;
    const uint64_t dw[3] = {(uint64_t)hidden, (uint64_t)(heads * 128), 1};
    const uint64_t sw[2] = {(uint64_t)hidden, (uint64_t)hidden * (uint64_t)(heads * 128)};
    const uint32_t bw[3] = {64, 256, 1};  // one tile's 256 output features
    st = encode_map(&tw, w_qkv, 3, dw, sw, bw, "w_qkv");
    if (st != GROUT_OK) return st;
  }
  QkvGemmArgs a{};
  a.rows = seq_len;
  a.hidden = hidden;
  a.hq = dims->num_q_heads;
  a.hkv = dims->num_kv_heads;
  a.pos0 = position_start;
  a.eps = dims->rms_eps;
  a.q_w = static_cast<const __half*>(q_norm_w);
  a.k_w = static_cast<const __half*>(k_norm_w);
  a.table = rope_table;
  a.q_out = static_cast<__half*>(q_out);
  a.q_out_row_stride = (int64_t)dims->num_q_heads * 128;
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.cache_head_stride = cache_head_stride;
  a.qkv_out = static_cast<__half*>(qkv_out);
  a.qkv_row_stride = heads * 128;
  a.err = ds->err;
  CUDA_TRY(launch_qkv_gemm(a, tx, tw, ds->num_sms, reinterpret_cast<cudaStream_t>(stream)));
  return GROUT_OK;
}

}  // extern "C"
