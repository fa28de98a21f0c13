/*
 * stickykv_b200 — C ABI of the B200 windowed-eviction KV cache kernels.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns an
 * int status (skv_status).  No entry point allocates device memory,
 * synchronises, or keeps state between calls; scratch memory is supplied by
 * the caller through a workspace pointer sized by the matching *_size()
 * query.  Nothing here depends on PyTorch.
 *
 * Reference interfaces replaced (file:line in shaswata965-coder/StickyKV):
 *   skv_append               CacheState.append          modules/windowed_cache/state.py:68-119
 *   skv_decode_attention     eager attention + score hook
 *                            modules/windowed_eager_cache/hooks.py:145-180,
 *                            modules/windowed_cache/hooks.py:199-290,
 *                            scorer.compute_window_scores/accumulate
 *                            modules/windowed_cache/scorer.py:17-109,
 *                            WindowedCache.update score accumulation
 *                            modules/windowed_cache/cache.py:163-228
 *   skv_decode_attention_append  skv_append + skv_decode_attention of one
 *                            decode step (state.py:68-119 + the above)
 *   skv_evict                WindowedCache.update eviction block
 *                            modules/windowed_cache/cache.py:230-286 =
 *                            EvictionPolicy.compute_retain_window_indices +
 *                            expand_to_token_indices policy.py:81-209,
 *                            CacheState.slice_and_keep + rerotate_keys
 *                            state.py:125-232
 *   skv_evict_append         skv_append + skv_evict of an evicting decode
 *                            step (state.py:68-119 + the above)
 *   skv_evict_plan_compute   the integer bookkeeping of the same block
 *                            (policy.py:108-132, :197-207)
 *   skv_prefill_scores       the prefill branch of the flash score hook
 *                            modules/windowed_cache/hooks.py:245-290
 *   skv_pack_pages           int4 tier demotion (design.md:130-187; no code in
 *                            the reference)
 */
#ifndef STICKYKV_B200_H
#define STICKYKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SKV_ABI_VERSION 1

typedef enum skv_status {
  SKV_OK = 0,
  SKV_ERR_INVALID_ARG = 1,   /* null pointer, bad size, inconsistent counts */
  SKV_ERR_UNSUPPORTED = 2,   /* geometry/dtype this build has no kernel for */
  SKV_ERR_MISALIGNED = 3,    /* pointer or stride not aligned as required */
  SKV_ERR_CAPACITY = 4,      /* a buffer is too small for the request */
  SKV_ERR_CUDA = 5,          /* a CUDA launch failed (see skv_last_cuda_error) */
  SKV_ERR_WORKSPACE = 6      /* workspace smaller than the *_size() query */
} skv_status;

typedef enum skv_dtype { SKV_F32 = 0, SKV_F16 = 1, SKV_BF16 = 2 } skv_dtype;

/*
 * Static description of one layer's cache storage.  All rows of the batch
 * hold the same number of tokens (eviction keeps the same count per row).
 *
 * fp store   k_fp/v_fp [batch][num_kv_heads][fp_capacity][head_dim] (kv_dtype,
 *            post-RoPE keys).  Slots [0, num_sink) hold the attention sinks,
 *            slots [sink_pad, ...) the tokens after the int4 tier in logical
 *            order; sink_pad = num_sink rounded up to 8.
 * int4 tier  tier_pages [batch][num_kv_heads][tier_page_capacity][page_bytes]
 *            (page = 8 tokens of K and V, group-32 int4 codes + fp16
 *            scale/zero, see skv_page_bytes); tier_table
 *            [batch][tier_page_capacity] maps logical tier page -> physical
 *            page.  tier_page_capacity == 0 disables the tier (reference
 *            mode: every retained token stays in kv_dtype).
 * rope       rope_cos/rope_sin [rope_positions][head_dim/2] fp32: the model
 *            rotary module's cos/sin (first half; the second half repeats it)
 *            for positions 0..rope_positions-1; 16-byte aligned.
 */
typedef struct skv_layer_desc {
  int32_t batch;
  int32_t num_kv_heads;
  int32_t num_q_heads;
  int32_t head_dim;
  int32_t kv_dtype;
  int32_t window_size;
  int32_t num_sink;
  int32_t sink_pad;
  int32_t fp_capacity;
  int32_t tier_page_capacity;
  void* k_fp;
  void* v_fp;
  uint8_t* tier_pages;
  int32_t* tier_table;
  const float* rope_cos;
  const float* rope_sin;
  int32_t rope_positions;
  int32_t reserved[7];
} skv_layer_desc;

/* Integer bookkeeping of one eviction; identical for every row. */
typedef struct skv_evict_plan {
  int32_t local_windows;      /* min(local_windows, num_windows) */
  int32_t evictable_windows;  /* num_windows - local */
  int32_t kept_evictable;     /* min(top_k, evictable) */
  int32_t retained_windows;   /* kept_evictable + local */
  int32_t seq_len_new;        /* tokens after compaction */
  int32_t tier_pages_new;     /* logical int4 pages after (0 without tier) */
  int32_t fp_len_new;         /* occupied fp slots after */
  int32_t reserved;
} skv_evict_plan;

typedef struct skv_evict_args {
  int32_t seq_len;            /* tokens before eviction (after this step's append) */
  int32_t tier_pages;         /* logical int4 pages before */
  int32_t num_windows;        /* width of the accumulated window scores */
  int32_t top_k_windows;
  int32_t local_windows;      /* resolved local_tokens / window_size */
  int32_t scores_capacity;    /* allocated width of the score buffers */
  const float* scores_src;    /* [batch][num_q_heads][scores_capacity] */
  float* scores_dst;          /* same shape; receives the gathered scores */
  const int64_t* ids_src;     /* [batch][scores_capacity] original window ids */
  int64_t* ids_dst;
  int32_t* retained_out;      /* optional [batch][scores_capacity] window idx */
  int64_t next_window_id;     /* original id of the next window to appear; the
                                 slots after the retained windows are seeded
                                 with next_window_id, next_window_id+1, ...
                                 With num_windows > 0 the kernel takes it from
                                 the device instead (one past ids_src of the
                                 newest window, which equals it whenever ids
                                 grow by one per new window, as the cache
                                 keeps them), so a captured launch stays
                                 valid on replay; this value serves
                                 num_windows == 0. */
} skv_evict_args;

int skv_abi_version(void);
const char* skv_status_string(int status);
/* Message of the last CUDA error seen by this library on this thread. */
const char* skv_last_cuda_error(void);
/* Bytes of one 8-token int4 page of K and V for head_dim. */
int32_t skv_page_bytes(int32_t head_dim);
/* sizeof of the ABI structs (0 skv_layer_desc, 1 skv_evict_plan,
 * 2 skv_evict_args) so a binding can check its own struct layout. */
int32_t skv_struct_size(int32_t which);

/* Host-only: counts after an eviction (no GPU work). */
int skv_evict_plan_compute(int32_t seq_len, int32_t num_windows, int32_t num_sink,
                           int32_t window_size, int32_t top_k_windows, int32_t local_windows,
                           int32_t tier_enabled, skv_evict_plan* plan);

/*
 * Append n_new tokens at logical positions seq_len .. seq_len+n_new-1.
 * k_new/v_new are kv_dtype with element strides (stride_b, stride_h,
 * stride_t) and unit stride along head_dim.
 */
int skv_append(const skv_layer_desc* layer, int32_t seq_len, int32_t tier_pages,
               const void* k_new, const void* v_new, int64_t stride_b, int64_t stride_h,
               int64_t stride_t, int32_t n_new, void* stream);

/*
 * One decode step: out[b,h,:] = softmax(q·Kᵀ·scaling) V over the whole
 * retained cache (sinks, int4 tier, fp tokens), and, when window_scores is not
 * NULL, window_scores[b,h,w] += attention mass of post-sink window w
 * (w < ceil((seq_len-num_sink)/window_size)).  q/out are kv_dtype
 * [batch][num_q_heads][head_dim] with strides (q_stride_b, q_stride_h).
 */
size_t skv_decode_workspace_size(const skv_layer_desc* layer, int32_t seq_len);
int skv_decode_attention(const skv_layer_desc* layer, int32_t seq_len, int32_t tier_pages,
                         const void* q, int64_t q_stride_b, int64_t q_stride_h, void* out,
                         int64_t out_stride_b, int64_t out_stride_h, float scaling,
                         float* window_scores, int32_t scores_capacity, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * One decode step with its token append fused in: the effect of
 *   skv_append(layer, seq_len - 1, tier_pages, k_new, v_new, stride_b,
 *              stride_h, 0, 1, stream)
 * followed by skv_decode_attention(layer, seq_len, ...), in one launch on the
 * tensor-core path (the block that reads the last unit writes the new key and
 * value first).  seq_len counts the new token; k_new/v_new hold one token per
 * (row, kv head) with element strides (stride_b, stride_h).  Replaces the
 * reference's update() append (modules/windowed_cache/state.py:68-119, a
 * torch.cat) and the attention that follows it in the same layer call.
 */
int skv_decode_attention_append(const skv_layer_desc* layer, int32_t seq_len, int32_t tier_pages,
                                const void* k_new, const void* v_new, int64_t stride_b,
                                int64_t stride_h, const void* q, int64_t q_stride_b,
                                int64_t q_stride_h, void* out, int64_t out_stride_b,
                                int64_t out_stride_h, float scaling, float* window_scores,
                                int32_t scores_capacity, void* workspace, size_t workspace_bytes,
                                void* stream);

/*
 * skv_decode_attention without a workspace argument (no counterpart in the
 * reference).  For callers that cannot allocate device memory: a binding from
 * a language without a CUDA allocator, a service that forbids allocation on
 * its decode path, or a plugin that only receives tensors it did not create.
 * The scratch is a fixed array of SKV_NOALLOC_SCRATCH_BYTES (16 MiB) inside
 * this library, reserved on every GPU that loads it until the process exits;
 * a request whose scratch (skv_decode_workspace_size) is larger returns
 * SKV_ERR_CAPACITY.  The first call on a device looks up the array's device
 * address with that device current; make that first call before any stream
 * capture.  No cudaMalloc/cudaFree or other allocation happens.  All calls
 * share the one array: calls whose kernels overlap on the GPU (different
 * streams, or the same layer from two threads) race on it and must be
 * serialised by the caller.
 */
#define SKV_NOALLOC_SCRATCH_BYTES (16u << 20)
int skv_decode_attention_noalloc(const skv_layer_desc* layer, int32_t seq_len, int32_t tier_pages,
                                 const void* q, int64_t q_stride_b, int64_t q_stride_h, void* out,
                                 int64_t out_stride_b, int64_t out_stride_h, float scaling,
                                 float* window_scores, int32_t scores_capacity, void* stream);

/*
 * Eviction: select the kept windows per row from args->scores_src (head
 * mean, top-k over the evictable prefix, lowest index wins ties,
 * chronological order), compact src into dst (dst has its own fp buffers and
 * tier_table; both share tier_pages), re-rotate kept fp keys from their old
 * to their new positions with the reference's rounding, quantise kept fp
 * windows that enter the int4 tier, and gather scores / window ids.
 */
size_t skv_evict_workspace_size(const skv_layer_desc* layer, int32_t num_windows);
int skv_evict(const skv_layer_desc* src, const skv_layer_desc* dst, const skv_evict_args* args,
              void* workspace, size_t workspace_bytes, void* stream);

/*
 * skv_append of an evicting decode step's one token followed by skv_evict
 * (the same block of WindowedCache.update, cache.py:230-286 after the
 * CacheState.append of state.py:68-119), in the eviction's own launches: the
 * token, at logical position args->seq_len - 1 (args->seq_len counts it),
 * is kept by the local windows, so the eviction's move reads it straight
 * from k_new / v_new ([batch][kv_heads][1][head_dim], element strides
 * stride_b and stride_h, 16-byte aligned) into dst; it is never written to
 * src.  dst, the scores and the ids end as after the two calls.
 */
int skv_evict_append(const skv_layer_desc* src, const skv_layer_desc* dst, const skv_evict_args* args,
                     const void* k_new, const void* v_new, int64_t stride_b, int64_t stride_h,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Prefill: causal attention of q [batch][num_q_heads][T][head_dim] over
 * k/v [batch][num_kv_heads][T][head_dim] (all kv_dtype, contiguous, 16-byte
 * aligned like out; else SKV_ERR_MISALIGNED) ->
 * out [batch][T][num_q_heads][head_dim], and window_scores[b,h,w] += the
 * column mass of window w summed over all T query rows.
 */
size_t skv_prefill_workspace_size(const skv_layer_desc* layer, int32_t T);
int skv_prefill_attention(const skv_layer_desc* layer, int32_t T, const void* q, const void* k,
                          const void* v, void* out, float scaling, float* window_scores,
                          int32_t scores_capacity, void* workspace, size_t workspace_bytes,
                          void* stream);

/*
 * The retained cache as plain keys and values in logical order,
 * k_out/v_out [batch][num_kv_heads][seq_len][head_dim] (kv_dtype, contiguous):
 * the reference's CacheState.key_states / value_states
 * (modules/windowed_cache/state.py:20-35), which its flash score hook
 * (modules/windowed_cache/hooks.py:218) and parity runner read.  fp tokens
 * are copied; int4 tier tokens are dequantised (code * scale + zero in fp32)
 * and their keys rotated from the page frame to their current position.
 */
int skv_materialize(const skv_layer_desc* layer, int32_t seq_len, int32_t tier_pages, void* k_out,
                    void* v_out, void* stream);

/*
 * Quantise n_pages*8 kv_dtype tokens (k/v [n_pages*8][head_dim], keys
 * post-RoPE at positions first_pos..) into int4 pages (keys in their
 * page-relative frame), out [n_pages][page_bytes].
 */
int skv_pack_pages(const skv_layer_desc* layer, const void* k, const void* v, int32_t first_pos,
                   int32_t n_pages, uint8_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* STICKYKV_B200_H */
