/* grout_attn.h — C ABI of the B200 (sm_100a) attention hot path.
 *
 * Drop-in replacement for the device kernels behind three ops of the
 * reference engine (rtburger/grout):
 *   - fused Q/K RMSNorm + RoPE + KV-cache write (prefill and decode),
 *   - causal GQA prefill attention,
 *   - split-K GQA decode attention with its LSE merge.
 *
 * Conventions (all entry points):
 *   - plain pointers to DEVICE memory unless a name says _host; element type
 *     f16 (IEEE binary16) for activations, caches and norm weights, f32 for
 *     the RoPE table, u32/i32 for positions and offsets;
 *   - strides are in ELEMENTS; head_dim must be 128 (the reference requires
 *     head_dim == 128, src/model.rs:1446);
 *   - every pointer must be 16-byte aligned, every stride a multiple of 8;
 *   - calls are stream-ordered, never synchronise, never allocate, and take
 *     every position they need at run time from device memory where the
 *     reference does, so they can be recorded into a CUDA graph once
 *     grout_attn_init() has run for the device;
 *   - a call returns GROUT_OK or an error status; grout_attn_last_error()
 *     returns the message of the last failure on the calling thread.  All
 *     validation happens on the host before any launch.
 */
#ifndef GROUT_ATTN_H_
#define GROUT_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* grout_stream_t; /* a cudaStream_t; NULL = legacy default stream */

typedef enum {
  GROUT_OK = 0,
  GROUT_ERR_INVALID_ARG = 1,   /* bad shape, stride, alignment or null pointer */
  GROUT_ERR_UNSUPPORTED = 2,   /* e.g. head_dim != 128, GQA group > 8, not sm_100 */
  GROUT_ERR_CUDA = 3,          /* a CUDA runtime / driver call failed */
  GROUT_ERR_DEVICE = 4         /* a kernel recorded a device-side error (see check) */
} grout_status;

/* Decode only: round qk_scale to f16 before use, as the reference's decode
 * path does (qk_scale_f16, src/model.rs:3177). */
#define GROUT_FLAG_DECODE_SCALE_F16 0x1

/* Model-level attention shape (Qwen3Config fields, src/config.rs:6-21). */
typedef struct {
  int32_t num_q_heads;   /* num_attention_heads */
  int32_t num_kv_heads;  /* num_key_value_heads; num_q_heads % num_kv_heads == 0 */
  int32_t head_dim;      /* must be 128 */
  int32_t max_seq;       /* KV-cache capacity (positions) */
  float rms_eps;         /* rms_norm_eps */
  float qk_scale;        /* softmax scale; <= 0 selects 1/sqrt(head_dim) */
  int32_t flags;         /* GROUT_FLAG_* */
} grout_attn_dims;

/* ----------------------------------------------------------------- library */

/* Message of the last failed call on this thread ("" if none). */
const char* grout_attn_last_error(void);
const char* grout_attn_version(void);

/* Per-device setup (kernel attributes, device error word).  Idempotent; call
 * once per device, with that device current, before recording any call of
 * this library into a CUDA graph.  Replaces the JIT "prime" pass the
 * reference runs before capture (src/model.rs:2917-3245). */
grout_status grout_attn_init(int32_t device);

/* Reads and clears the device error word of the current device (0 = none;
 * 0x1xx = a bounded wait timed out at site xx; 0x200 = a decode position was
 * >= max_seq and the cache write was skipped).  Synchronises the device. */
grout_status grout_attn_check_device_error(int32_t* code);

/* ------------------------------------------------------------------- RoPE */

/* inv_freq[i] = 1 / theta^(2i / head_dim), i < head_dim/2, computed in f32
 * on the host.  Replaces build_inv_freq (src/model.rs:7295-7306). */
void grout_inv_freq_host(float theta, int32_t head_dim, float* inv_freq_host);

/* Bytes of the RoPE table for max_seq positions: max_seq * head_dim * 4. */
size_t grout_rope_table_bytes(int32_t max_seq, int32_t head_dim);

/* Fills d_table [max_seq][2][head_dim/2] (cos row, then sin row) with
 * cos/sin of the f32 angle f32(pos) * inv_freq[i] — the angle the reference
 * evaluates per call (src/kernels.rs:5076-5079) — each evaluated in double
 * precision and rounded once to f32.  Host work plus one blocking copy; an
 * init-time call (the reference uploads inv_freq once at load,
 * src/model.rs:7295-7306). */
grout_status grout_rope_table_init(float* d_table, const float* inv_freq_host, int32_t head_dim,
                                   int32_t max_seq, grout_stream_t stream);

/* ------------------------------------------- fused norm + RoPE + KV write */

/* Prefill: replaces qk_norm_rope_kv_prefill_raw_f16 (src/kernels.rs:4845-5168)
 * as launched by execute_qk_norm_rope_kv_prefill_op_ctx (src/model.rs:4753-4888).
 *   q [seq_len][num_q_heads][128] (row stride q_row_stride),
 *   k, v [seq_len][num_kv_heads][128] (row stride kv_row_stride),
 *   q_norm_w, k_norm_w [128], rope_table from grout_rope_table_init,
 *   q_out like q; k_cache, v_cache [num_kv_heads][max_seq][128] with head
 *   stride cache_head_stride.  Row s is written at cache position
 *   position_start + s; position_start + seq_len must be <= max_seq.
 * K and Q are RMS-normalised (eps = dims->rms_eps), rotated and rounded to
 * f16 once; V is copied bit for bit. */
grout_status grout_qk_norm_rope_kv_prefill(const void* q, const void* k, const void* v,
                                           int64_t q_row_stride, int64_t kv_row_stride,
                                           const void* q_norm_w, const void* k_norm_w,
                                           const float* rope_table, void* q_out, void* k_cache,
                                           void* v_cache, int64_t cache_head_stride,
                                           int32_t position_start, int32_t seq_len,
                                           const grout_attn_dims* dims, grout_stream_t stream);

/* Decode: replaces qk_norm_rope_kv_decode_raw_f16 (src/kernels.rs:5180-5452),
 * recorded at src/model.rs:2919-2943 and inside the decode graph; batched.
 *   qkv [batch][(num_q_heads + 2*num_kv_heads) * 128] = [Q | K | V] per row
 *   (the QKV GEMV output), d_position [batch] (u32, device memory: the
 *   position of the new token of each sequence), q_out [batch][num_q_heads][128],
 *   caches of sequence b at base + b * cache_batch_stride, layout
 *   [num_kv_heads][max_seq][128] (head stride cache_head_stride).
 * A position >= max_seq skips that sequence's cache write and records
 * device error 0x200. */
grout_status grout_qk_norm_rope_kv_decode(const void* qkv, const void* q_norm_w,
                                          const void* k_norm_w, const float* rope_table,
                                          void* q_out, void* k_cache, void* v_cache,
                                          int64_t cache_batch_stride, int64_t cache_head_stride,
                                          const uint32_t* d_position, int32_t batch,
                                          const grout_attn_dims* dims, grout_stream_t stream);

/* -------------------------------------------------------- prefill attention */

/* Engine layout, batch 1: replaces the Host-position arm of
 * attend_seq_arc_into_ctx_with_position (src/model.rs:6938-7134), i.e.
 * fmha_prefill_causal / fmha_prefill_gqa_lpt (src/kernels.rs:2570-2725,
 * 2943-3298).
 *   q, out [seq_len][num_q_heads][128] (contiguous),
 *   k_cache, v_cache [num_kv_heads][max_seq][128] (head stride cache_head_stride),
 *   query row m (position position_start + m) attends to cache keys
 *   0 .. position_start + m.  Scale dims->qk_scale (f32; default 1/sqrt(128)).
 * The kernel is persistent: min(work items, SM count) CTAs of 512 threads and
 * ~200 KB of shared memory each, so it occupies every SM until it finishes
 * (kernels on other streams do not overlap with it). */
grout_status grout_attn_prefill(const void* q, const void* k_cache, const void* v_cache,
                                void* out, int64_t cache_head_stride, int32_t position_start,
                                int32_t seq_len, const grout_attn_dims* dims,
                                grout_stream_t stream);

/* Varlen / batched causal prefill (no counterpart in the reference, which is
 * batch-1; same per-sequence math as grout_attn_prefill).
 *   q, out: packed [q_rows][num_q_heads][128], row stride q_row_stride;
 *     sequence b owns rows cu_seqlens_q[b] .. cu_seqlens_q[b+1].
 *   k, v: key n of sequence b, kv head h at
 *     b*kv_batch_stride + (kv_start[b] + n)*kv_row_stride + h*kv_head_stride;
 *     kv_rows = rows addressable from k/v (for the TMA bounds).
 *   position_start[b] (NULL = all 0): keys of sequence b are
 *     0 .. position_start[b] + len_b - 1 and row m sees keys <= position_start[b] + m.
 *   kv_start (NULL = all 0).  cu_seqlens_q, position_start, kv_start are
 *   DEVICE int32 arrays; max_q_len is a host upper bound on any len_b. */
typedef struct {
  const void* q;
  void* out;
  int64_t q_row_stride;
  int64_t q_rows;
  const void* k;
  const void* v;
  int64_t kv_batch_stride;
  int64_t kv_row_stride;
  int64_t kv_head_stride;
  int64_t kv_rows;
  const int32_t* cu_seqlens_q;
  const int32_t* position_start;
  const int32_t* kv_start;
  int32_t batch;
  int32_t max_q_len;
} grout_prefill_varlen_args;

grout_status grout_attn_prefill_varlen(const grout_prefill_varlen_args* args,
                                       const grout_attn_dims* dims, grout_stream_t stream);

/* Split-K varlen prefill: the reference's prefill split-K + merge
 * (fmha_prefill_gqa_lpt_split / prefill_splitk_reduce_merge,
 * src/kernels.rs:3302-3759, microbench only there).  For launches with fewer
 * (query-tile pair, head, sequence) items than SMs: every item's KV range is
 * cut into num_splits chunks, each writes its unnormalised rows and (max,
 * sum) to the workspace, and a merge rounds the combined rows to f16.
 * Same arguments as grout_attn_prefill_varlen (cu_seqlens_q may be NULL for
 * batch 1); results agree with it within the usual tolerance, not bitwise.
 * grout_attn_prefill_splits suggests a count (1 = no split needed). */
int32_t grout_attn_prefill_splits(int32_t batch, int32_t max_q_len, const grout_attn_dims* dims);
size_t grout_attn_prefill_splitk_workspace_bytes(int32_t batch, int32_t max_q_len,
                                                 int32_t num_q_heads, int32_t num_splits);
grout_status grout_attn_prefill_splitk(const grout_prefill_varlen_args* args, int32_t num_splits,
                                       const grout_attn_dims* dims, void* workspace,
                                       size_t workspace_bytes, grout_stream_t stream);

/* --------------------------------------------------------- decode attention */

/* Number of KV splits grout_attn_decode uses for this shape (a function of
 * batch, max_kv_len, num_kv_heads and the SM count of the current device). */
int32_t grout_attn_decode_splits(int32_t batch, int32_t max_kv_len, const grout_attn_dims* dims);

/* Workspace bytes grout_attn_decode needs: 0 when the split count is at most
 * 16 (the splits of one KV head and sequence then merge inside a thread-block
 * cluster through distributed shared memory), else
 * batch * num_q_heads * splits * (128 + 1) * 4. */
size_t grout_attn_decode_workspace_bytes(int32_t batch, int32_t max_kv_len,
                                         const grout_attn_dims* dims);

/* Split-K GQA decode + merge: replaces fmha_decode_gqa_split +
 * splitk_reduce_merge (src/kernels.rs:4016-4304) as recorded in the decode
 * graph (src/model.rs:3180-3225, 3728-3771); batched.
 *   q [batch][num_q_heads][128], out [batch][num_q_heads][128],
 *   caches of sequence b at base + b*cache_batch_stride, layout
 *   [num_kv_heads][max_seq][128] (head stride cache_head_stride),
 *   d_position [batch] u32 in device memory: sequence b attends to keys
 *   0 .. d_position[b] (kv_len = position + 1, src/kernels.rs:4045-4050).
 *   max_kv_len: host upper bound on position + 1 (fixes the split count, so
 *   a graph recorded once stays valid while positions grow below it).
 *   workspace: grout_attn_decode_workspace_bytes(batch, max_kv_len, dims)
 *   bytes of device memory owned by the caller (may be NULL if that is 0). */
grout_status grout_attn_decode(const void* q, const void* k_cache, const void* v_cache,
                               int64_t cache_batch_stride, int64_t cache_head_stride,
                               const uint32_t* d_position, void* out, int32_t batch,
                               int32_t max_kv_len, const grout_attn_dims* dims, void* workspace,
                               size_t workspace_bytes, grout_stream_t stream);

/* As grout_attn_decode with an explicit split count (1 .. 1024); workspace
 * size batch * num_q_heads * num_splits * 129 * 4 bytes when num_splits > 16
 * (none at or below 16, where the merge runs inside a cluster). */
grout_status grout_attn_decode_ex(const void* q, const void* k_cache, const void* v_cache,
                                  int64_t cache_batch_stride, int64_t cache_head_stride,
                                  const uint32_t* d_position, void* out, int32_t batch,
                                  int32_t max_kv_len, int32_t num_splits,
                                  const grout_attn_dims* dims, void* workspace,
                                  size_t workspace_bytes, grout_stream_t stream);

/* Decode step with the fused write folded in: replaces the pair the
 * reference launches back to back in its decode graph,
 * qk_norm_rope_kv_decode_raw_f16 then fmha_decode_gqa_split +
 * splitk_reduce_merge (src/model.rs:3494ff, 3728-3771), with one kernel.
 * Inputs as grout_qk_norm_rope_kv_decode (qkv [batch][(num_q_heads +
 * 2*num_kv_heads)*128], norm weights, RoPE table, caches, d_position);
 * q_out [batch][num_q_heads][128] may be NULL (the normalised, rotated query
 * is then only used inside the kernel).  Every CTA normalises and rotates its
 * own query heads; the one whose KV range holds the new position writes that
 * position's K and V rows into the cache before it reads them.  The cache rows,
 * q_out and out equal grout_qk_norm_rope_kv_decode followed by
 * grout_attn_decode bit for bit.  Split count and workspace as
 * grout_attn_decode (grout_attn_decode_workspace_bytes).  A position >=
 * max_seq writes nothing but a zero output row and records device error
 * 0x200. */
grout_status grout_attn_decode_fused(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                     const float* rope_table, void* q_out, void* k_cache,
                                     void* v_cache, int64_t cache_batch_stride,
                                     int64_t cache_head_stride, const uint32_t* d_position,
                                     void* out, int32_t batch, int32_t max_kv_len,
                                     const grout_attn_dims* dims, void* workspace,
                                     size_t workspace_bytes, grout_stream_t stream);

/* ------------------------------ tensor-parallel GEMV + all-reduce (NVLink) */

/* No counterpart in the reference (single-GPU); this is the row-parallel
 * o_proj / down_proj of a tensor-parallel decode step plus its all-reduce,
 * the next component after the attention path (config 5's layout).
 * Setup, once per rank (init-time; the exchange of IPC handles between the
 * processes is the caller's, e.g. an all-gather over torch.distributed):
 *   1. grout_tp_comm_create(world, hidden, &comm, handle): allocates and
 *      zeroes this rank's exchange buffer (cudaMalloc; 2*world*hidden*4 bytes
 *      plus flags) and returns its GROUT_IPC_HANDLE_BYTES-byte IPC handle;
 *   2. gather every rank's handle into [world][GROUT_IPC_HANDLE_BYTES];
 *   3. grout_tp_comm_connect(comm, rank, handles) opens the peers' buffers;
 *      all ranks must have connected before any rank calls
 *      grout_gemv_allreduce (e.g. a barrier).
 * Per call, on every rank in the same order:
 *   out[hidden] = residual[hidden] (may be NULL) + sum over ranks of W_r x_r,
 *   W_r [hidden][k] f16 row-major (this rank's column shard), x_r [k] f16,
 *   k a multiple of 8 in [256, 16384], hidden <= 8288.  Peers exchange f32 partials by direct
 *   stores over NVLink and per-block flags; every wait is bounded (2 s,
 *   then device error 0x13c, the output is left unwritten and the comm is
 *   marked out of step: later calls return at once with device error
 *   0x13d).  The result is bitwise identical on every rank.  Stream-ordered;
 *   a call recorded in a CUDA graph may be replayed (the sequence number
 *   lives on the device). */
#define GROUT_IPC_HANDLE_BYTES 64
typedef struct grout_tp_comm grout_tp_comm;
grout_status grout_tp_comm_create(int32_t world, int32_t hidden, grout_tp_comm** comm,
                                  void* handle_out);
grout_status grout_tp_comm_connect(grout_tp_comm* comm, int32_t rank, const void* all_handles);
void grout_tp_comm_destroy(grout_tp_comm* comm);
grout_status grout_gemv_allreduce(grout_tp_comm* comm, const void* w, int32_t k, const void* x,
                                  const void* residual, void* out, grout_stream_t stream);
/* The same exchange without the GEMV: out = residual (may be NULL) + sum over
 * ranks of partial_r, partial_r [hidden] f16 computed by the caller (e.g. a
 * cuBLAS GEMV).  Same ordering, bounds and errors as grout_gemv_allreduce;
 * the two may be interleaved on one comm. */
grout_status grout_allreduce_residual(grout_tp_comm* comm, const void* partial,
                                      const void* residual, void* out, grout_stream_t stream);

/* Allocation-free decode.  No counterpart in the reference.  For callers that
 * cannot provide a device workspace — an engine whose device memory is all
 * owned by a planner, an FFI host without a device allocator, code already
 * inside a stream capture.  Same arguments and result as grout_attn_decode
 * without the workspace: the split-K scratch lives in a fixed array in the
 * library's device memory (grout_attn_decode_noalloc_max_bytes() = 512 KiB,
 * held on every GPU that loads the library until the process exits).  Only
 * shapes with more than 16 splits per (sequence, KV head) use scratch: few
 * sequences and KV heads over long contexts, about SMs * G * 516 bytes at
 * most (G = num_q_heads / num_kv_heads).  A shape whose scratch
 * (grout_attn_decode_workspace_bytes) exceeds the array is rejected with
 * GROUT_ERR_INVALID_ARG.  The first call on a device resolves
 * the array's device address (the device must be current); make that first
 * call before any stream capture.  All calls on a device share the array:
 * calls that can overlap on the GPU (unordered streams) race; ordered calls
 * are safe.  Allocates nothing, ever. */
size_t grout_attn_decode_noalloc_max_bytes(void);
grout_status grout_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       int64_t cache_batch_stride, int64_t cache_head_stride,
                                       const uint32_t* d_position, void* out, int32_t batch,
                                       int32_t max_kv_len, const grout_attn_dims* dims,
                                       grout_stream_t stream);

/* QKV projection with the fused norm/RoPE/KV write as its epilogue
 * (prefill): replaces the QKV MatMulSlice (src/model.rs:4076-4098) plus
 * grout_qk_norm_rope_kv_prefill, without the f16 QKV activation round trip.
 *   x [seq_len][hidden] f16 (row stride x_row_stride), hidden % 64 == 0;
 *   w_qkv [(num_q_heads + 2*num_kv_heads)*128][hidden] f16 (torch Linear
 *     layout: Q heads, then K heads, then V heads);
 *   outputs as grout_qk_norm_rope_kv_prefill (q_out [seq_len][num_q_heads][128]);
 *   qkv_out (nullable): [seq_len][(num_q_heads + 2*num_kv_heads)*128] f16, the
 *     projection itself.
 * The accumulators are rounded to f16 before the norm, so q_out and the
 * caches equal grout_qk_norm_rope_kv_prefill applied to qkv_out bit for bit. */
grout_status grout_qkv_proj_norm_rope_kv_prefill(
    const void* x, int64_t x_row_stride, const void* w_qkv, int32_t hidden, const void* q_norm_w,
    const void* k_norm_w, const float* rope_table, void* q_out, void* k_cache, void* v_cache,
    int64_t cache_head_stride, void* qkv_out, int32_t position_start, int32_t seq_len,
    const grout_attn_dims* dims, grout_stream_t stream);

/* ------------------------------------------------------ decode-graph glue */

/* The neighbours of the attention ops in every layer of the reference's
 * decode graph (src/model.rs:3264-3354), one kernel each.
 *   grout_add_rms_norm: replaces add_rms_norm_f16 / add_rms_norm_decode_raw_f16
 *     / rms_norm_f16 (src/kernels.rs:4449-4600, 1530ff).  x, residual
 *     (NULL = none), out, residual_out (NULL = not written): [rows][n] f16;
 *     weight [n] f16; n a multiple of 8, <= 16384.  c = x + residual in f32,
 *     residual_out = f16(c), out = f16(c * rsqrt(sum(c^2) / n + eps) * w).
 *   grout_silu_mul: replaces silu_mul_2d_f16 (src/kernels.rs:1497-1526).
 *     gate_up [rows][2n] f16 (gate columns, then up columns), out [rows][n]:
 *     out = f16(sigmoid(g) * g * u), f32 math. */
grout_status grout_add_rms_norm(const void* x, const void* residual, const void* weight, void* out,
                                void* residual_out, int32_t rows, int32_t n, float eps,
                                grout_stream_t stream);
grout_status grout_silu_mul(const void* gate_up, void* out, int32_t rows, int32_t n,
                            grout_stream_t stream);

/* ------------------------------------------------------ paged KV caches */

/* Paged KV cache: no counterpart in the reference, whose caches are one
 * contiguous [num_kv_heads][max_seq][128] tensor per layer
 * (src/model.rs:1587-1599) and whose decode is batch-1 (src/kernels.rs:
 * 4003-4004); the batched / paged cache is the serving extension next to it.
 * Same math and rounding as the contiguous entry points.
 *   k_pages, v_pages: page pools [num_pages][num_kv_heads][page_size][128] f16;
 *   position p of sequence b lives in row p % page_size of page
 *   page_table[b * table_stride + p / page_size] (int32, device);
 *   page_size: a multiple of 64 in [64, 4096]; positions stay below
 *   dims->max_seq and table_stride >= ceil(max_seq / page_size).
 * A table entry outside [0, num_pages) is reported through
 * grout_attn_check_device_error (0x201): the fused writes skip that row,
 * decode reads zeros for that tile. */

/* Causal prefill attention over a paged cache (chunked prefill: the chunk's
 * K/V were written with grout_qk_norm_rope_kv_prefill_paged).  Same math as
 * grout_attn_prefill_varlen.
 *   q, out: packed [q_rows][num_q_heads][128], row stride q_row_stride;
 *     sequence b owns rows cu_seqlens_q[b] .. cu_seqlens_q[b+1] (DEVICE
 *     int32 [batch+1]; NULL with batch 1 = rows 0 .. max_q_len);
 *   position_start[b] (DEVICE int32 [batch], NULL = all 0): keys of
 *     sequence b are positions 0 .. position_start[b] + len_b - 1 of its
 *     pages, row m sees keys <= position_start[b] + m;
 *   max_q_len: host upper bound on any len_b. */
typedef struct {
  const void* q;
  void* out;
  int64_t q_row_stride;
  int64_t q_rows;
  const void* k_pages;
  const void* v_pages;
  int32_t num_pages;
  int32_t page_size;
  const int32_t* page_table;
  int32_t table_stride;
  const int32_t* cu_seqlens_q;
  const int32_t* position_start;
  int32_t batch;
  int32_t max_q_len;
} grout_prefill_paged_args;

grout_status grout_attn_prefill_paged(const grout_prefill_paged_args* args,
                                      const grout_attn_dims* dims, grout_stream_t stream);

/* Paged form of grout_attn_decode_ex (num_splits 0 = the automatic count). */
grout_status grout_attn_decode_paged(const void* q, const void* k_pages, const void* v_pages,
                                     int32_t num_pages, int32_t page_size,
                                     const int32_t* page_table, int32_t table_stride,
                                     const uint32_t* d_position, void* out, int32_t batch,
                                     int32_t max_kv_len, int32_t num_splits,
                                     const grout_attn_dims* dims, void* workspace,
                                     size_t workspace_bytes, grout_stream_t stream);

/* Paged form of grout_qk_norm_rope_kv_decode: sequence b's new K/V row goes
 * to position d_position[b]. */
grout_status grout_qk_norm_rope_kv_decode_paged(
    const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* rope_table,
    void* q_out, void* k_pages, void* v_pages, int32_t num_pages, int32_t page_size,
    const int32_t* page_table, int32_t table_stride, const uint32_t* d_position, int32_t batch,
    const grout_attn_dims* dims, grout_stream_t stream);

/* Paged form of grout_qk_norm_rope_kv_prefill for one sequence: page_table is
 * that sequence's row of the table (ceil(max_seq / page_size) entries). */
grout_status grout_qk_norm_rope_kv_prefill_paged(
    const void* q, const void* k, const void* v, int64_t q_row_stride, int64_t kv_row_stride,
    const void* q_norm_w, const void* k_norm_w, const float* rope_table, void* q_out,
    void* k_pages, void* v_pages, int32_t num_pages, int32_t page_size,
    const int32_t* page_table, int32_t position_start, int32_t seq_len,
    const grout_attn_dims* dims, grout_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* GROUT_ATTN_H_ */
