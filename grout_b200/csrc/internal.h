// Internal launch interface between the C ABI (abi.cu) and the kernels.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace grout {

constexpr int kHeadDim = 128;

// Sets the message grout_attn_last_error() returns on this thread.
void set_last_error(const char* msg);
// Device error word of the current device (initialising it if needed), or
// null if the device cannot be set up.
int* device_error_word();

struct NormRopeArgs {
  const __half* q;     // prefill: q rows; decode: qkv rows
  const __half* k;     // prefill only
  const __half* v;     // prefill only
  int64_t q_row_stride;   // prefill: q/q_out row stride; decode: qkv row length
  int64_t kv_row_stride;  // prefill only
  const __half* q_w;
  const __half* k_w;
  const float* table;
  __half* q_out;
  __half* k_cache;
  __half* v_cache;
  int64_t cache_batch_stride;  // decode only
  int64_t cache_head_stride;
  const uint32_t* d_position;  // decode only
  int32_t pos0;                // prefill only
  int32_t rows;                // prefill: seq_len; decode: batch
  int32_t hq;
  int32_t hkv;
  int32_t max_seq;
  float eps;
  int32_t decode;
  int* err;
  // Paged cache (page_table != null): k_cache / v_cache are page pools
  // [num_pages][hkv][page_size][128]; position p of sequence s is row
  // p % page_size of page page_table[s * table_stride + p / page_size]
  // (prefill: one sequence, table row page_table[0..]).
  const int32_t* page_table;
  int64_t table_stride;
  int32_t page_size;
  int32_t num_pages;
};

cudaError_t launch_qk_norm_rope_kv(const NormRopeArgs& a, int num_sms, cudaStream_t s);

// Splits of one (kv head, sequence) that decode merges inside a thread-block
// cluster (distributed shared memory) instead of a workspace + merge launch.
constexpr int kDecodeMaxClusterSplits = 16;

struct DecodeArgs {
  const __half* q;      // [B][hq][128] (unfused)
  __half* out;          // [B][hq][128]
  float* part_o;        // [B][hq][nks][128] (nks > 1, no cluster)
  float* part_lse;      // [B][hq][nks]      (nks > 1, no cluster)
  const uint32_t* d_position;
  int32_t batch;
  int32_t hq;
  int32_t hkv;
  int32_t nks;
  int32_t cluster;      // nks > 1: merge in a cluster of nks CTAs (nks <= 16)
  int32_t max_seq;      // positions >= max_seq are rejected on the device
  float scale_log2;
  int* err;
  // Fused norm/RoPE/KV write (qkv != null): qkv [B][(hq + 2 hkv) * 128] rows
  // (row stride qkv_row_stride), norm weights, RoPE table; q_out optional;
  // the new K/V rows go to the caches at position d_position[b]
  // (contiguous: b * cache_batch_stride + kh * cache_head_stride + pos * 128).
  const __half* qkv;
  int64_t qkv_row_stride;
  const __half* q_w;
  const __half* k_w;
  const float* table;
  float eps;
  __half* q_out;
  __half* k_cache;
  __half* v_cache;
  int64_t cache_batch_stride;
  int64_t cache_head_stride;
  // Paged cache (page_table != null): the maps are {128, page_size, hkv,
  // num_pages}; key row r of sequence b is row r % page_size of page
  // page_table[b * table_stride + r / page_size].
  const int32_t* page_table;
  int32_t table_stride;
  int32_t page_size;
  int32_t num_pages;
};

// tm_k / tm_v: 4-D maps {128, max_seq, hkv, batch} over the caches, box
// {64, 64, 1, 1}, 128B swizzle.
cudaError_t launch_decode(const DecodeArgs& a, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                          cudaStream_t s);
cudaError_t decode_set_attributes();

struct PrefillArgs {
  __half* out;
  int64_t q_row_stride;
  const int32_t* cu_q;       // device [B+1]
  const int32_t* pos0;       // device [B] or null
  const int32_t* kv_start;   // device [B] or null
  int32_t batch;
  int32_t max_q_len;
  int32_t hq;
  int32_t hkv;
  int32_t kv_batched;        // K/V maps carry a batch coordinate
  int32_t single_len;        // used when cu_q == null (batch 1)
  int32_t single_pos0;       // used when pos0 == null
  float scale_log2;
  int* err;
  // Paged K/V (page_table != null): the K/V maps are {128, page_size, hkv,
  // num_pages} with 64-row boxes; key n of sequence b is row n % page_size of
  // page page_table[b * table_stride + n / page_size].
  const int32_t* page_table;
  int32_t table_stride;
  int32_t page_size;
  int32_t num_pages;
  // Split-K (nsplit > 1): every (pair, head, sequence) item is cut into
  // nsplit KV ranges; each writes its unnormalised O and (m, l) per row to
  // part ([item][tile][128 rows][130] f32) and a merge kernel finishes.
  int32_t nsplit;
  float* part;
};

// tm_q: 3-D {128, hq, q_rows}, box {64, 1, 128}; tm_k / tm_v: 4-D
// {128, kv_rows, hkv, B} (or 3-D without the batch dim), box {64, 128, 1(,1)};
// all 128B swizzle.
// Number of f32 in one split partial of one query tile: O[128][128], m[128], l[128].
constexpr int kPrefillPartFloats = 128 * 130;
cudaError_t launch_prefill(const PrefillArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                           const CUtensorMap& tm_v, cudaStream_t s);
cudaError_t prefill_set_attributes();

// QKV projection + fused norm/RoPE/KV write (prefill): X [rows][hidden] f16
// (row stride x_row_stride) times W [(hq+2hkv)*128][hidden] f16; maps are
// 3-D {hidden, rows or features, 1} with 64x128 boxes, 128B swizzle.
struct QkvGemmArgs {
  int32_t rows;
  int32_t hidden;
  int32_t hq;
  int32_t hkv;
  int32_t pos0;
  float eps;
  const __half* q_w;
  const __half* k_w;
  const float* table;
  __half* q_out;
  int64_t q_out_row_stride;
  __half* k_cache;
  __half* v_cache;
  int64_t cache_head_stride;
  __half* qkv_out;           // optional f16 QKV activation
  int64_t qkv_row_stride;
  int* err;
};
cudaError_t launch_qkv_gemm(const QkvGemmArgs& a, const CUtensorMap& tm_x, const CUtensorMap& tm_w,
                            int num_sms, cudaStream_t s);
cudaError_t qkv_gemm_set_attributes();

// Decode-graph glue (glue.cu).
cudaError_t launch_add_rms_norm(const __half* x, const __half* residual, const __half* w,
                                __half* out, __half* residual_out, int rows, int n, float eps,
                                cudaStream_t s);
cudaError_t launch_silu_mul(const __half* gate_up, __half* out, int rows, int n, int num_sms,
                            cudaStream_t s);

}  // namespace grout
