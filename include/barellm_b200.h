/*
 * barellm_b200 — C ABI of the B200 (sm_100a) paged-KV hot path.
 *
 * The reference (quanhua92/barellm, pure Python on PyTorch) has no native
 * code.  Each entry point below replaces a chain of ATen ops inside one of its
 * Python methods; the replaced method is cited beside each declaration.
 *
 * Conventions
 *   - Plain C: raw device pointers, int64 sizes/strides counted in ELEMENTS,
 *     a CUDA stream passed as `void*` (a cudaStream_t; NULL = legacy stream).
 *   - Every call validates its arguments on the host, enqueues kernels on the
 *     stream and returns without synchronising.  Return value 0 = BL_OK; any
 *     other value is one of BL_ERR_*, and bl_last_error() (thread-local)
 *     holds a one-line message.
 *   - Nothing here allocates device memory.  Scratch space for split-K decode
 *     is a caller-owned workspace sized by bl_paged_decode_workspace_bytes().
 *   - Device-side faults are never raised.  A block id outside [0, P) or a
 *     block-table column outside the table width makes the kernel skip that
 *     access and OR a BL_DEVERR_* bit into the caller's `err` word (a device
 *     int32, may be NULL).  Every wait inside a kernel is bounded; a wait that
 *     runs out sets BL_DEVERR_TIMEOUT and the kernel returns.
 *
 * Paged pool layout (identical to the reference's PagedKVCache tensors,
 * src/barellm/engine/paged_kv_cache.py:66-74):
 *   k_pool, v_pool : [num_layers, num_blocks, num_kv_heads, block_size, head_dim]
 *   contiguous, element type `dtype`.
 * Block tables (reference PagedBatchKVMetadata.block_tables,
 * src/barellm/engine/batched_kv_cache.py:124-132): int32, row r holds the
 * physical block of logical block j at block_tables[r * bt_stride + j] for
 * j < bt_width.  Request b uses row row_ids[b] (row_ids may be NULL: row b).
 */
#ifndef BARELLM_B200_H
#define BARELLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BL_ABI_VERSION 1

#if defined(__GNUC__)
#define BL_API __attribute__((visibility("default")))
#else
#define BL_API
#endif

/* return codes */
enum {
  BL_OK = 0,
  BL_ERR_ARG = 1,         /* bad shape, stride, pointer or size           */
  BL_ERR_DTYPE = 2,       /* unsupported element type                      */
  BL_ERR_CAPACITY = 3,    /* workspace or index range too small            */
  BL_ERR_LAUNCH = 4,      /* a CUDA launch or driver call failed           */
  BL_ERR_UNSUPPORTED = 5  /* valid request this build does not implement   */
};

/* element types */
enum { BL_F32 = 0, BL_F16 = 1, BL_BF16 = 2 };

/* bits OR-ed into the device error word */
enum {
  BL_DEVERR_BLOCK_ID = 1,   /* physical block id outside [0, num_blocks)        */
  BL_DEVERR_TABLE = 2,      /* logical block beyond the block-table width       */
  BL_DEVERR_TIMEOUT = 4,    /* a bounded wait inside a kernel ran out           */
  BL_DEVERR_WORKSPACE = 8   /* the decode plan needs more units than allocated  */
};

/* One layer of a paged K/V pool plus the block tables that index it. */
typedef struct bl_paged_layer {
  void* k_pool;
  void* v_pool;
  int64_t num_layers;
  int64_t num_blocks;
  int64_t num_kv_heads;
  int64_t block_size;
  int64_t head_dim;
  int32_t dtype;  /* BL_F32 / BL_F16 / BL_BF16 */
  int32_t layer;  /* which layer slice of the pool */
  const int32_t* block_tables;
  int64_t bt_stride;
  int64_t bt_width;
  const int32_t* row_ids; /* [batch] or NULL */
} bl_paged_layer;

/* ------------------------------------------------------------------------ */
/* Append: slot-mapped K/V scatter into the pool.                            */
/* Replaces PagedLayerKV.append_only (src/barellm/engine/paged_kv_cache.py:  */
/* 151-193) and its per-row loop BatchLayerKV.append_only                    */
/* (src/barellm/engine/batched_kv_cache.py:40-63).                           */
/*                                                                          */
/* Token t (0-based) of request b, head h, lives at                         */
/*   k_new + b*new_stride_b + (o_b + t)*new_stride_t + h*new_stride_h       */
/* (v_new likewise with the v_stride_* values), where o_b = new_offsets[b]  */
/* (ragged, packed along the token axis) or 0.                              */
/* Row b appends n_b tokens: new_offsets[b+1]-new_offsets[b], or            */
/* max_new_tokens when new_offsets is NULL.  They go to logical positions   */
/* start_pos[b] .. start_pos[b]+n_b-1.  The last axis (head_dim) must be    */
/* contiguous.  The copy is bit-exact.                                      */
typedef struct bl_append_args {
  bl_paged_layer kv;
  const void* k_new;
  const void* v_new;
  int64_t new_stride_b;
  int64_t new_stride_h;
  int64_t new_stride_t;
  int64_t v_stride_b;
  int64_t v_stride_h;
  int64_t v_stride_t;
  const int32_t* start_pos;   /* [batch], device */
  const int32_t* new_offsets; /* [batch+1], device, or NULL */
  int64_t batch;
  int64_t max_new_tokens;
  int32_t* err;               /* device int32 or NULL */
} bl_append_args;

BL_API int bl_paged_append(const bl_append_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Fused QK-RMSNorm + RoPE + append: the per-layer step before attention.    */
/* Replaces the reference's                                                  */
/*   q = apply_rope(q_norm(q), cos, sin); k = apply_rope(k_norm(k), cos, sin) */
/* (src/barellm/models/attention.py:161-169, models/norm.py:14-21,           */
/* models/rope.py:53-68) followed by PagedLayerKV.append_only of k and v     */
/* (src/barellm/engine/paged_kv_cache.py:151-193).  Writes the normalised,   */
/* rotated q to q_out (q_in's layout, own strides) and the rotated k         */
/* and the raw v into their pool slots (slot of token t of request b =       */
/* start_pos[b] + t, as bl_paged_append).  Inputs are [B, H, T, D] with any  */
/* strides and D contiguous, or packed [1, H, sum T, D] with new_offsets.    */
/* cos / sin: [B or 1, T, D] element rows at b * rope_stride_b +             */
/* token * rope_stride_t (token = packed index when new_offsets is given).   */
/* Weights: [D], element type.  head_dim 64, 128 or 256.                     */
typedef struct bl_qk_prep_args {
  bl_paged_layer kv;
  const void* q_in;
  int64_t q_in_stride_b;
  int64_t q_in_stride_h;
  int64_t q_in_stride_t;
  const void* k_in;
  int64_t k_in_stride_b;
  int64_t k_in_stride_h;
  int64_t k_in_stride_t;
  const void* v_in;
  int64_t v_in_stride_b;
  int64_t v_in_stride_h;
  int64_t v_in_stride_t;
  void* q_out;
  int64_t q_out_stride_b;
  int64_t q_out_stride_h;
  int64_t q_out_stride_t;
  const void* q_norm_weight;
  const void* k_norm_weight;
  const void* cos;
  const void* sin;
  int64_t rope_stride_b;
  int64_t rope_stride_t;
  float eps;
  int32_t pad0;
  int64_t num_q_heads;
  const int32_t* start_pos;   /* [batch], device */
  const int32_t* new_offsets; /* [batch+1], device, or NULL */
  int64_t batch;
  int64_t max_new_tokens;
  int32_t* err;               /* device int32 or NULL */
} bl_qk_prep_args;

BL_API int bl_qk_norm_rope_append(const bl_qk_prep_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Gather: dense read of pages, with optional zero padding.                  */
/* Replaces PagedLayerKV.read (src/barellm/engine/paged_kv_cache.py:215-240) */
/* and BatchLayerKV.read/_pad (src/barellm/engine/batched_kv_cache.py:65-95).*/
/* Writes out[b, h, t, :] for t < max_len: the cached token when             */
/* t < seq_lens[b], else zeros when zero_fill != 0 (left untouched if 0).    */
typedef struct bl_gather_args {
  bl_paged_layer kv;
  const int32_t* seq_lens; /* [batch], device */
  int64_t batch;
  void* k_out;
  void* v_out;
  int64_t out_stride_b;
  int64_t out_stride_h;
  int64_t out_stride_t;
  int64_t max_len;
  int32_t zero_fill;
  int32_t* err;
} bl_gather_args;

BL_API int bl_paged_gather(const bl_gather_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Decode attention: one query token per request, GQA, read in place.        */
/* Replaces gather + pad + repeat_interleave + padding mask + SDPA in        */
/* SDPAAttentionBackend.attend (src/barellm/attention/backend.py:34-61) for  */
/* the batched decode path (src/barellm/engine/engine.py:458-488).           */
/*                                                                          */
/* out[b, hq, :] = softmax(scale * q[b,hq,:] . K[b, hq/G, t, :]) V           */
/* over t < seq_lens[b] (post-append lengths, >= 1), G = Hq / Hkv.           */
/* Long rows are split into fixed 512-token chunks whose partial results    */
/* are merged by a separate reduce kernel; the split depends only on the    */
/* row's own length, so a row's result does not depend on the batch.       */
typedef struct bl_decode_args {
  bl_paged_layer kv;
  const void* q;
  int64_t q_stride_b;
  int64_t q_stride_h;
  void* out;
  int64_t out_stride_b;
  int64_t out_stride_h;
  const int32_t* seq_lens; /* [batch], device */
  int64_t batch;
  int64_t num_q_heads;
  float scale;
  void* workspace;          /* device scratch, >= bl_paged_decode_workspace_bytes */
  size_t workspace_bytes;
  int64_t max_seq_len;      /* host upper bound on seq_lens[] */
  int32_t plan_ready;       /* 1: workspace already holds the plan for these seq_lens */
  int32_t* err;
} bl_decode_args;

BL_API size_t bl_paged_decode_workspace_bytes(int64_t batch, int64_t num_q_heads,
                                       int64_t head_dim, int64_t block_size,
                                       int64_t max_seq_len);

/* Builds the split-K work plan for seq_lens into the workspace.  The plan
 * depends only on seq_lens, so one plan serves every layer of a step. */
BL_API int bl_paged_decode_plan(const bl_decode_args* args, void* stream);

/* The attention kernel alone (the plan must already be in the workspace
 * on the tensor-core path).  Rows that fit in one chunk get their output
 * here; longer rows leave (o, lse) partials in the workspace. */
BL_API int bl_paged_decode_attention(const bl_decode_args* args, void* stream);

/* The split-K reduce alone: merges the partials of multi-chunk rows into
 * `out`.  A no-op on the SIMT path, which never splits. */
BL_API int bl_paged_decode_reduce(const bl_decode_args* args, void* stream);

/* All of it: plan (unless plan_ready), attention, reduce. */
BL_API int bl_paged_decode(const bl_decode_args* args, void* stream);

/* Allocation-free variant of bl_paged_decode.  No counterpart in the
 * reference: it exists for callers that cannot provide device scratch -- a
 * host framework that owns all device memory and hands a plugin only its
 * input and output pointers, or a hot loop that must never call cudaMalloc.
 * The split-K scratch lives in a fixed 16 MiB array inside the library,
 * which every GPU that loads the
 * library keeps until the process exits; `workspace`, `workspace_bytes` and
 * `plan_ready` are ignored and no memory is allocated.  A batch whose split-K
 * scratch (bl_paged_decode_workspace_bytes) exceeds 16 MiB is rejected with
 * BL_ERR_CAPACITY.  The first call on a device looks up the array's device
 * address with that device current; make that first call before any stream
 * capture.  All calls share the one array: calls that overlap on the GPU (two
 * streams, or two host threads) race and corrupt each other's results, so
 * order them on one stream. */
BL_API int bl_paged_decode_noalloc(const bl_decode_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* KV-head-sharded decode: the heads of one decode batch split across the    */
/* GPUs of a node, the per-head outputs all-gathered over NVLink.            */
/* The reference runs on one device; its per-head math is the decode chain   */
/* of SDPAAttentionBackend.attend (src/barellm/attention/backend.py:34-61),  */
/* which this keeps head for head.  Rank r owns KV heads                     */
/* [r*Hkv/W, (r+1)*Hkv/W) of every request (its pool holds only those) and   */
/* the query heads that read them; every rank holds the same block tables.   */
/*                                                                          */
/* The all-gather is fused into the attention's epilogue: each output       */
/* element is stored straight into every rank's gathered buffer (peer       */
/* memory mapped with bl_ipc_import), then a one-warp barrier publishes     */
/* completion (st.release.sys into each rank's signal pad) and waits until  */
/* every rank has done the same (bounded by timeout_ns; BL_DEVERR_TIMEOUT). */
/* When the call's work has completed on this rank's stream, this rank's    */
/* gathered buffer holds all Hq heads.  No NCCL, no multicast.              */
#define BL_MAX_RANKS 8

typedef struct bl_head_gather {
  int32_t world;                        /* ranks, 1 .. BL_MAX_RANKS            */
  int32_t rank;                         /* this rank, 0 .. world-1             */
  void* peer_out[BL_MAX_RANKS];         /* rank r's gathered [batch, Hq, D]    */
                                        /* buffer as mapped in this process,   */
                                        /* element (0, 0, 0); strides are      */
                                        /* args->out_stride_b / _h, the same   */
                                        /* on every rank                       */
  int32_t* peer_signal[BL_MAX_RANKS];   /* rank r's signal pad: BL_MAX_RANKS   */
                                        /* int32 slots, slot s written only by */
                                        /* rank s; zero before the first call  */
  int32_t* epoch;                       /* this rank's call counter (device    */
                                        /* int32, zero before the first call)  */
  int64_t head_offset;                  /* this rank's first query head in the */
                                        /* gathered layout                     */
  int64_t timeout_ns;                   /* bound on the wait; <= 0: 2 s        */
} bl_head_gather;

/* args describes this rank's shard: q = its query heads [batch, Hq/W, D],
 * num_q_heads = Hq/W, kv = its pool shard (num_kv_heads = Hkv/W).
 * args->out is ignored (the outputs go to gather->peer_out).  Every rank
 * must make the same sequence of calls.  A rank reuses a gathered buffer only
 * after the next call's barrier, so callers alternate two buffers (or more)
 * when the output of one call is still being read during the next. */
BL_API int bl_paged_decode_allgather(const bl_decode_args* args, const bl_head_gather* gather,
                                     void* stream);

/* Peer mapping of device memory between the processes of one node (CUDA
 * IPC, no multicast).  export: handle of the allocation holding `ptr` plus
 * ptr's offset in it.  import: maps that allocation into this process for
 * the current device and returns the address matching the exporter's ptr.
 * close: unmaps an address returned by import. */
typedef struct bl_ipc_handle {
  unsigned char bytes[64];
  uint64_t offset;
} bl_ipc_handle;

BL_API int bl_ipc_export(const void* ptr, bl_ipc_handle* out);
BL_API int bl_ipc_import(const bl_ipc_handle* handle, void** ptr);
BL_API int bl_ipc_close(void* ptr);

/* ------------------------------------------------------------------------ */
/* Prefill attention: causal attention of new query tokens over a paged      */
/* prefix plus themselves, read in place.                                    */
/* Replaces the prefill SDPA(is_causal=True) of SDPAAttentionBackend.attend  */
/* (src/barellm/attention/backend.py:52-61) and generalises it to a          */
/* non-empty prefix (chunked prefill), where query i of a row whose total    */
/* length is L and query count is C attends keys 0 .. L-C+i (bottom-right    */
/* aligned causal mask).                                                     */
/*                                                                          */
/* Query i of row b, head hq: q + b*q_stride_b + (o_b + i)*q_stride_t        */
/*   + hq*q_stride_h, o_b = q_offsets[b] (packed) or 0; the row has C_b =    */
/* q_offsets[b+1]-q_offsets[b] queries, or max_q_len when q_offsets is NULL. */
/* `out` uses the same addressing with its own strides.                      */
typedef struct bl_prefill_args {
  bl_paged_layer kv;
  const void* q;
  int64_t q_stride_b;
  int64_t q_stride_t;
  int64_t q_stride_h;
  void* out;
  int64_t out_stride_b;
  int64_t out_stride_t;
  int64_t out_stride_h;
  const int32_t* q_offsets; /* [batch+1], device, or NULL */
  const int32_t* seq_lens;  /* [batch], device: prefix + C_b */
  int64_t batch;
  int64_t num_q_heads;
  int64_t max_q_len;
  float scale;
  int32_t* err;
} bl_prefill_args;

BL_API int bl_paged_prefill(const bl_prefill_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Decoder support: residual add + RMSNorm (not part of the paged-KV path)   */
/*
 * The norm around each attention call of the decoder that drives the path:
 *   h = rmsnorm(x) * weight                      (models/norm.py:14-21), or
 *   x_out = x + residual; h = rmsnorm(x_out) * weight   (models/block.py)
 * with the reference's roundings: the add rounded to the element type, the
 * mean square, rsqrt and the two products in fp32, one rounding at the end.
 * Rows of `hidden` elements; each row pointer advances by its own stride
 * (elements).  `residual` / `x_out` may both be NULL (plain norm).
 */
typedef struct bl_rms_norm_args {
  const void* x;
  const void* residual;
  void* x_out;
  void* out;
  const void* weight; /* [hidden] */
  int64_t rows;
  int64_t hidden;
  int64_t x_stride;
  int64_t residual_stride;
  int64_t x_out_stride;
  int64_t out_stride;
  float eps;
  int32_t dtype;
} bl_rms_norm_args;

BL_API int bl_rms_norm(const bl_rms_norm_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Misc.                                                                     */
BL_API const char* bl_last_error(void);
BL_API int bl_abi_version(void);

/* Which kernel variant a call with these shapes would use (for tests and the
 * bench):  0 = generic SIMT kernel, 1 = TMA + tensor-core kernel. */
BL_API int bl_decode_path(int32_t dtype, int64_t head_dim, int64_t block_size,
                   int64_t num_q_heads, int64_t num_kv_heads);
BL_API int bl_prefill_path(int32_t dtype, int64_t head_dim, int64_t block_size,
                    int64_t num_q_heads, int64_t num_kv_heads);

#ifdef __cplusplus
}
#endif

#endif /* BARELLM_B200_H */
