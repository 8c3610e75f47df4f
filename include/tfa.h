/*
 * tfa.h -- C ABI of the B200 (sm_100a) paged-KV attention forward.
 *
 * This library is the drop-in replacement for the reference's torch op
 *   flash_attn_varlen_with_block_v8_64(q, k, v, max_seqlen_q, cu_seqlens_q,
 *       max_seqlen_k, seqused_k, causal, window_left, window_right, block_table, out)
 * (solidcc2/cuda-learn, flash_attention_backend/toy_flash_attn/v8/flash_attn_func.cu:800-813,
 * bound at :911-913), which the Python wrapper flash_attn_varlen_with_block_cu_bf16
 * (flash_attention_backend/toy_flash_attn/flash_attention_func.py:518-600) calls.
 *
 * Differences in the contract, all additive:
 *   - every buffer, including the split-KV workspace, is owned by the caller; the library
 *     allocates nothing and keeps no state except per-device attribute caches;
 *   - an optional natural-log softmax LSE output;
 *   - an optional softmax scale (the reference hardcodes 1/sqrt(head_dim), which stays the
 *     default);
 *   - errors are returned as negative status codes instead of exceptions.
 *
 * All pointers are device pointers unless stated otherwise. Launches are asynchronous on
 * the given stream (a cudaStream_t passed as void*; NULL = legacy default stream).
 */
#ifndef TFA_H_
#define TFA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TFA_ABI_VERSION 1

#if defined(__GNUC__)
#define TFA_API __attribute__((visibility("default")))
#else
#define TFA_API
#endif

typedef enum tfa_status {
  TFA_OK = 0,
  TFA_ERR_NULL_POINTER = -1, /* a required pointer is NULL */
  TFA_ERR_HEAD_DIM = -2,     /* head_dim is not 64 or 128 */
  TFA_ERR_GQA = -3,          /* num_q_heads is not a multiple of num_kv_heads */
  TFA_ERR_BLOCK_SIZE = -4,   /* block_size is neither a divisor nor a multiple of 16 */
  TFA_ERR_LAYOUT = -5,       /* head_dim not contiguous, or pointer / stride not 16-byte aligned */
  TFA_ERR_SHAPE = -6,        /* negative sizes, window < -1, too many work items */
  TFA_ERR_WORKSPACE = -7,    /* workspace NULL or smaller than tfa_workspace_size() */
  TFA_ERR_TENSOR_MAP = -8,   /* the TMA descriptor for the KV cache could not be encoded */
  TFA_ERR_CUDA = -9,         /* a CUDA runtime call or launch failed */
  TFA_ERR_DEVICE = -10,      /* the current device is not an sm_100 GPU */
  TFA_ERR_KERNEL = -11,      /* a kernel reported an error (see tfa_read_device_error) */
  TFA_ERR_STATIC_WORKSPACE_LIMIT = -12 /* the call needs more workspace than TFA_STATIC_WORKSPACE_BYTES */
} tfa_status;

/* Size of the fixed device-resident workspace of tfa_fwd_static_workspace (32 MiB). */
#define TFA_STATIC_WORKSPACE_BYTES (32u * 1024u * 1024u)

/* Arguments of one forward call. Strides are in elements. */
typedef struct tfa_fwd_params {
  const void* q;          /* bf16 [total_q, num_q_heads, head_dim] */
  int64_t q_stride[3];
  const void* k;          /* bf16 [num_blocks, block_size, num_kv_heads, head_dim] (K cache) */
  int64_t k_stride[4];
  const void* v;          /* bf16, same shape as k (V cache) */
  int64_t v_stride[4];
  void* out;              /* bf16 [total_q, num_q_heads, head_dim], written */
  int64_t out_stride[3];
  float* softmax_lse;     /* optional fp32 [total_q, num_q_heads] contiguous, natural log; NULL = skip */
  const int32_t* cu_seqlens_q; /* [batch + 1], query offsets of each sequence in q */
  const int32_t* seqused_k;    /* [batch], kv length of each sequence */
  const int32_t* block_table;  /* [batch, >= ceil(max kv_len / block_size)], physical block ids */
  int64_t block_table_stride0;
  int64_t batch;
  int64_t total_q;
  int64_t num_q_heads;
  int64_t num_kv_heads;
  int64_t head_dim;
  int64_t block_size;
  int64_t num_blocks;
  int64_t max_seqlen_q;   /* upper bound of the per-sequence query length */
  int64_t max_seqlen_k;   /* upper bound of seqused_k */
  int32_t causal;         /* non-zero: right window forced to 0 */
  int32_t window_left;    /* -1 = unbounded */
  int32_t window_right;   /* -1 = unbounded */
  float softmax_scale;    /* <= 0: 1 / sqrt(head_dim) (the reference's fixed scale) */
  int32_t num_splits;     /* 0 = automatic split-KV; > 0 forces at most this many splits */
} tfa_fwd_params;

/* What tfa_fwd will launch for a given call (for tests, benches and tuning). */
typedef struct tfa_plan_info {
  int32_t kernel;         /* 0 = decode kernel (<= 16 packed q rows), 1 = prefill kernel, 2 = both: the
                             decode kernel on sequences with q_len * group <= 16, the prefill kernel
                             on the others (calls of >= 8 sequences that need the prefill kernel;
                             the other fields then describe the prefill kernel's part) */
  int32_t rows_per_tile;  /* packed (q token, q head) rows per work item */
  int32_t q_tiles;        /* q tiles per (sequence, kv head) */
  int32_t max_splits;     /* split-KV slots per q tile */
  int32_t split_cap;      /* kv tiles (128 tokens) per split, at most */
  int32_t num_items;      /* work-item slots (unused split slots are skipped on device) */
  int32_t grid;           /* persistent CTAs launched */
  int32_t combine;        /* how split partials are merged: 0 = no splits, 1 = by the LSE combine
                             kernel launched after the prefill kernel, 2 = inside the decode kernel
                             (the last split of each group to finish merges the group) */
  uint64_t workspace_bytes;
  int32_t item_list;      /* 1 if the decode kernel takes its items from a list built on the
                             device for the call (longest first; one extra small kernel) */
  int32_t pages;          /* 1 if the decode kernel works over whole pages (8 kv heads, 16-slot
                             pages, one q token per sequence): an item is one sequence's split
                             over all kv heads, so max_splits and num_items count per sequence */
} tfa_plan_info;

/* Fills *info for the call described by p on CUDA device `device` (device < 0: plan for
 * a 148-SM B200 without touching the CUDA runtime). */
TFA_API int tfa_plan(const tfa_fwd_params* p, int device, tfa_plan_info* info);

/* Bytes of workspace tfa_fwd needs for this call on `device` (0 on invalid arguments;
 * device < 0 as in tfa_plan).
 * The workspace must be zero-filled once when it is first allocated; the library leaves
 * its control words zeroed after every call. One workspace must not be shared by calls
 * that can run concurrently. */
TFA_API size_t tfa_workspace_size(const tfa_fwd_params* p, int device);

/* Paged attention forward. Replaces flash_attn_varlen_with_block_v8_64
 * (v8/flash_attn_func.cu:800-908): same tensors, same masking rule (q and kv tail
 * aligned, window -1 = unbounded, causal forces the right window to 0), writes `out`
 * in place. Runs on the current CUDA device. */
TFA_API int tfa_fwd(const tfa_fwd_params* p, void* workspace, size_t workspace_bytes, void* stream);

/* tfa_fwd plus two cudaEvent_t (passed as void*) recorded on `stream` immediately before
 * and after the attention kernel, so that kernel can be timed alone (the split-KV combine,
 * when there is one, runs after main_end). Profiling aid; no counterpart in the reference. */
TFA_API int tfa_fwd_timed(const tfa_fwd_params* p, void* workspace, size_t workspace_bytes, void* stream,
                          void* main_begin, void* main_end);

/* The forward for callers that cannot allocate device memory: a serving loop that must
 * not call cudaMalloc once it is running (cudaMalloc can synchronise the device and can
 * fail when memory is fragmented), or a host in another language that binds this C ABI
 * but has no device allocator to create the workspace tfa_fwd needs. Same arguments,
 * checks and results as tfa_fwd, but the split-KV workspace is a TFA_STATIC_WORKSPACE_BYTES
 * array in the library's own device memory (present on every GPU where the library is
 * loaded, until exit); nothing is allocated. Decode calls are planned for the per-head
 * decode kernel (the page decode kernel's split partials can exceed the array), so the
 * plan and the workspace it needs may differ from tfa_plan / tfa_workspace_size; calls
 * whose plan still needs more than the array return TFA_ERR_STATIC_WORKSPACE_LIMIT (a
 * call with num_splits forced, for example). All calls on a device share
 * the array, so calls that can overlap on the GPU race and must not be issued. The first
 * call on a device looks up the array's address with that device current and should come
 * before any stream capture. Kernel errors of these calls land in the array's error word,
 * which tfa_read_static_workspace_error reads.
 * No counterpart in the reference (its op allocates its split buffers on every call,
 * v8/flash_attn_func.cu:850-862). */
TFA_API int tfa_fwd_static_workspace(const tfa_fwd_params* p, void* stream);

/* tfa_read_device_error for the library-owned workspace of tfa_fwd_static_workspace on the
 * current device: synchronises `stream`, copies the error word into *err (0 = none) and
 * clears it (the next tfa_fwd_static_workspace call also starts from a cleared control
 * block). Returns TFA_ERR_CUDA if no tfa_fwd_static_workspace call has run on this device.
 * No counterpart in the reference. */
TFA_API int tfa_read_static_workspace_error(void* stream, int* err);

/* Synchronises `stream`, copies the device error word of `workspace` into *err (0 = none)
 * and clears it. A non-zero word means a kernel hit an internal time limit (codes
 * 101-103; the workspace must then be zero-filled again before reuse) or found a block id
 * outside [0, num_blocks) (code 110; those rows were read as zeros). */
TFA_API int tfa_read_device_error(void* workspace, void* stream, int* err);

/* Number of SMs of `device` (cached). */
TFA_API int tfa_device_sm_count(int device);

/* Human-readable name of a status code. */
TFA_API const char* tfa_status_string(int status);

/* Debug entry for the bit-exact gather check: stages the K and V tiles of every
 * (sequence, kv head) through the same TMA gather path the attention kernels use and
 * writes them densely as bf16 [sum(seqused_k), num_kv_heads, head_dim] into k_out / v_out
 * (sequence order, matching the reference's k[block_table[b][t // bs], t % bs] gather,
 * flash_attention_func.py:343-346). kv_offsets is the device int64 prefix sum of seqused_k
 * ([batch + 1]); workspace is a zero-filled buffer of at least 256 bytes whose error word
 * tfa_read_device_error reads. The q / out fields of p are ignored. No counterpart call in
 * the reference: its tests compare the gathered values only through the attention output. */
TFA_API int tfa_gather_kv(const tfa_fwd_params* p, const int64_t* kv_offsets, void* k_out, void* v_out, void* workspace,
                  void* stream);

/* Paged KV-cache write: for every token i with slot_mapping[i] >= 0, copies key[i] and
 * value[i] ([num_kv_heads, head_dim] bf16 each) into
 * k_cache[slot / block_size, slot % block_size] and v_cache[...]. Replaces the eager torch
 * scatter of ToyFlashAttentionImpl.do_kv_cache_update
 * (flash_attention_backend/toy_flash_attn/impl.py:121-144); negative slots are skipped
 * as there. slot_mapping is int64 [num_tokens]. Strides in elements, head_dim contiguous.
 * Slots at or beyond num_blocks * block_size are skipped and reported through the error
 * word of `workspace` (zero-filled, >= 256 bytes; may be NULL to skip the report). */
TFA_API int tfa_kv_cache_update(const void* key, const int64_t key_stride[2], const void* value,
                                const int64_t value_stride[2], void* k_cache, const int64_t k_cache_stride[3],
                                void* v_cache, const int64_t v_cache_stride[3], const int64_t* slot_mapping,
                                int64_t num_tokens, int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                                int64_t num_blocks, void* workspace, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TFA_H_ */
