/*
 * paged_attn.h — C ABI of the B200 (sm_100a) paged-attention backend.
 *
 * These entry points replace the FlashInfer 0.6.11 calls that
 * harsh-vsingh/LLM-Inference-Runtime makes from its monkey-patched LLaMA
 * attention (src/models/llama.py) and its step executor
 * (src/engine/runtime/step_executor.py). Each declaration names the
 * reference call it stands in for.
 *
 * Conventions shared by every function:
 *   - Plain pointers and sizes only. Device pointers are CUDA device
 *     addresses; `stream` is a cudaStream_t passed as void* (NULL = legacy
 *     default stream). Work is enqueued on `stream`; no call synchronises
 *     the device except pa_device_status().
 *   - The return value is a pa_status code (0 = success). Argument errors
 *     are detected on the host before anything is launched. Errors that only
 *     the device can see (page ids out of range, malformed indptr, bounded
 *     waits that expired) are recorded in a per-device status word that
 *     pa_device_status() reads and clears.
 *   - KV pool layout is FlashInfer's: a page holds `page_size` tokens; the
 *     key and value caches are addressed by base pointer plus element
 *     strides (page, head, token), the last dimension (head_dim) contiguous.
 *     For the engine's single 5-D pool [num_pages, 2, H_kv, P, D] ("HND")
 *     the value base is key base + H_kv*P*D and page stride 2*H_kv*P*D.
 *   - dtype codes: PA_DTYPE_F16 or PA_DTYPE_BF16 for q / k / v / pool / out.
 *   - LSE values (optional outputs, merge inputs) are base-2:
 *     log2(sum_j 2^(s_j)), s_j = sm_scale * log2(e) * <q, k_j>, which is
 *     FlashInfer's convention.
 */
#ifndef PAGED_ATTN_H_
#define PAGED_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum pa_status {
  PA_OK = 0,
  PA_ERR_INVALID_ARGUMENT = 1,   /* bad pointer, size, stride or alignment */
  PA_ERR_UNSUPPORTED = 2,        /* head_dim / page_size / group size / dtype not built */
  PA_ERR_WORKSPACE_TOO_SMALL = 3,
  PA_ERR_CUDA = 4,               /* a CUDA runtime call or launch failed */
  PA_ERR_DEVICE_CHECK = 5,       /* device-side validation failed (indptr, page id, last_page_len, position) */
  PA_ERR_TIMEOUT = 6,            /* a bounded device-side wait expired */
  PA_ERR_NOT_PLANNED = 7         /* run called on a workspace without a matching plan */
};

enum pa_dtype { PA_DTYPE_F16 = 0, PA_DTYPE_BF16 = 1 };

enum pa_kv_layout { PA_LAYOUT_NHD = 0, PA_LAYOUT_HND = 1 };

/* Describes one layer of the paged KV cache. */
typedef struct pa_kv_cache {
  const void* k_base;     /* device address of key page 0 */
  const void* v_base;     /* device address of value page 0 */
  int64_t page_stride;    /* elements between consecutive pages */
  int64_t head_stride;    /* elements between consecutive kv heads inside a page */
  int64_t token_stride;   /* elements between consecutive tokens inside a page */
  int64_t num_pages;      /* pages addressable from k_base / v_base */
  int32_t num_kv_heads;
  int32_t page_size;
  int32_t head_dim;
  int32_t dtype;          /* enum pa_dtype */
} pa_kv_cache;

/* Human-readable name of a status code (static string). */
const char* pa_status_string(int status);

/* ABI version this header describes (major * 100 + minor). 101: the append,
 * RoPE + append, fused QKV and cascade-plan calls take the number of page ids
 * (num_kv_indices) after kv_indptr. A caller built against another version
 * must refuse the library (the Python binding does). */
#define PA_ABI_VERSION 101

/* ABI version of this library (major * 100 + minor); equals PA_ABI_VERSION
 * of the header it was built from. */
int pa_abi_version(void);

/* Reads and clears the device-side status word of the current device.
 * Synchronises the device. Returns PA_OK, PA_ERR_DEVICE_CHECK or
 * PA_ERR_TIMEOUT (the first error recorded since the last read). */
int pa_device_status(void);

/* Replaces flashinfer.get_batch_indices_positions (called from
 * src/models/llama.py:70-83, which step_executor.py:155 drives):
 *   batch_indices[t] = b and positions[t] = seq_lens[b] - (append_indptr[b+1]
 *   - append_indptr[b]) + (t - append_indptr[b]) for append_indptr[b] <= t <
 *   append_indptr[b+1]. Entries t >= append_indptr[batch_size] (up to nnz)
 *   get batch index -1 and position 0. */
int pa_batch_indices_positions(const int32_t* append_indptr, const int32_t* seq_lens,
                               int32_t batch_size, int32_t nnz, int32_t* batch_indices,
                               int32_t* positions, void* stream);

/* Replaces flashinfer.append_paged_kv_cache(..., kv_layout) (called at
 * src/models/llama.py:188-210). Scatters append_key/append_value rows
 * [nnz, H_kv, D] (strides in elements, last dim contiguous) into the pool:
 *   page = kv_indices[kv_indptr[b] + pos / P], slot = pos % P,
 *   with b = batch_indices[t], pos = positions[t].
 * kv_indices holds num_kv_indices page ids; a kv_indptr range outside them,
 * or a page outside the request's pages or the pool, skips the row and
 * reports PA_ERR_DEVICE_CHECK. Bit-exact copy. */
int pa_append_paged_kv_cache(const void* append_key, int64_t key_stride_n, int64_t key_stride_h,
                             const void* append_value, int64_t value_stride_n,
                             int64_t value_stride_h, const int32_t* batch_indices,
                             const int32_t* positions, int32_t nnz, const pa_kv_cache* cache,
                             const int32_t* kv_indices, int64_t num_kv_indices,
                             const int32_t* kv_indptr, int32_t batch_size, void* stream);

/* Replaces flashinfer.apply_rope_pos_ids_inplace(q, k, pos_ids,
 * rotary_dim, interleave, rope_scale, rope_theta) (src/models/llama.py:175-182).
 * Rotates the first rotary_dim dims of every q row [nnz, H_q, D] and k row
 * [nnz, H_kv, D] in place, angle = pos / rope_scale * rope_theta^(-2i/rotary_dim). */
int pa_apply_rope_pos_ids_inplace(void* q, int64_t q_stride_n, int64_t q_stride_h, void* k,
                                  int64_t k_stride_n, int64_t k_stride_h, const int32_t* pos_ids,
                                  int32_t nnz, int32_t num_qo_heads, int32_t num_kv_heads,
                                  int32_t head_dim, int32_t rotary_dim, int32_t interleave,
                                  float rope_scale, float rope_theta, int32_t dtype, void* stream);

/* Replaces the reference's per-layer pair (src/models/llama.py:175-210)
 *   flashinfer.apply_rope_pos_ids_inplace(q, k, positions, ...)
 *   flashinfer.append_paged_kv_cache(k, v, batch_indices, positions, cache, ...)
 * with one launch: q and k are rotated in place exactly as
 * pa_apply_rope_pos_ids_inplace does (bit-identical rows), and the rotated k
 * and v rows are written into their page slots exactly as
 * pa_append_paged_kv_cache does (same slot rule, same device checks, padding
 * rows with batch index -1 rotated but not appended). The cache dtype is the
 * q / k / v dtype. Rows that are not 16-byte aligned or rotary_dim not a
 * multiple of 16 take the two separate kernels, with the same results. */
int pa_apply_rope_append(void* q, int64_t q_stride_n, int64_t q_stride_h, void* k,
                         int64_t k_stride_n, int64_t k_stride_h, const void* v,
                         int64_t v_stride_n, int64_t v_stride_h, const int32_t* batch_indices,
                         const int32_t* positions, int32_t nnz, int32_t num_qo_heads,
                         int32_t rotary_dim, int32_t interleave, float rope_scale,
                         float rope_theta, const pa_kv_cache* cache, const int32_t* kv_indices,
                         int64_t num_kv_indices, const int32_t* kv_indptr, int32_t batch_size,
                         void* stream);

/* Replaces the Python table build of StepExecutor._run_decode
 * (src/engine/runtime/step_executor.py:204-225) with a device build:
 *   kv_indices = concatenation of each sequence's whole block table (the
 *   first num_blocks[b] entries of row b of block_tables, rows
 *   block_table_stride elements apart), kv_indptr its offsets,
 *   kv_last_page_len[b] = seq_lens[b] % page_size or page_size,
 *   batch_indices[b] = b, positions[b] = seq_lens[b] - 1.
 * seq_lens is the sequence's get_len. counts (device int32[3]) receives
 * {batch_size, batch_size, 0}. A table that cannot cover its length, or more
 * pages than kv_indices_capacity, writes counts = {0, 0, 1} and records
 * PA_ERR_DEVICE_CHECK. All inputs and outputs are device memory; two
 * launches, no synchronisation (capturable in a CUDA graph). */
int pa_build_decode_tables(const int32_t* block_tables, int64_t block_table_stride,
                           const int32_t* num_blocks, const int32_t* seq_lens, int32_t batch_size,
                           int32_t page_size, int32_t* kv_indptr, int32_t* kv_indices,
                           int64_t kv_indices_capacity, int32_t* kv_last_page_len,
                           int32_t* batch_indices, int32_t* positions, int32_t* counts,
                           void* stream);

/* Replaces the Python table build of StepExecutor._run_prefill
 * (src/engine/runtime/step_executor.py:98-155) and the batch indices /
 * positions it then requests (step_executor.py:155) with a device build.
 * Per input sequence b: chunk = min(chunk_lens[b], prompt_lens[b] -
 * computed_lens[b]); sequences with chunk <= 0 are dropped, the others fill
 * output slots in input order (active[slot] = b) with
 *   qo_indptr = offsets of the chunks, seq_lens[slot] = computed + chunk,
 *   kv_indices = the first ceil(seq_lens / page_size) blocks of the table,
 *   kv_last_page_len = seq_lens % page_size or page_size,
 *   rows t of the chunk: batch_indices[t] = slot,
 *   positions[t] = computed + (t - qo_indptr[slot]).
 * counts (device int32[3]) receives {active sequences, rows, error flag}. */
int pa_build_prefill_tables(const int32_t* block_tables, int64_t block_table_stride,
                            const int32_t* num_blocks, const int32_t* prompt_lens,
                            const int32_t* computed_lens, const int32_t* chunk_lens,
                            int32_t batch_size, int32_t page_size, int32_t* qo_indptr,
                            int32_t* kv_indptr, int32_t* kv_indices, int64_t kv_indices_capacity,
                            int32_t* kv_last_page_len, int32_t* seq_lens, int32_t* active,
                            int32_t* batch_indices, int32_t* positions, int64_t rows_capacity,
                            int32_t* counts, void* stream);

/* Copy-on-write fork of pages (the reference plans it for shared partial
 * pages, todo.md "Incremental Radix Cache Insertion & Copy-on-Write"; its
 * allocator, src/engine/memory/allocator.py, has no fork yet): for every
 * pair i and layer l, the page_bytes bytes at
 *   pool + l * layer_stride_bytes + src_pages[i] * page_stride_bytes
 * are copied to the same place of page dst_pages[i]. For the engine's pool
 * [L, N, 2, H_kv, P, D] a page of a layer (K and V of every head) is one
 * contiguous block: page_bytes = page_stride_bytes = 2 * H_kv * P * D * elem.
 * dst pages must be distinct and not among the sources. Page ids outside
 * [0, num_pages) are skipped and recorded as PA_ERR_DEVICE_CHECK. */
int pa_fork_pages(void* pool, int64_t layer_stride_bytes, int32_t num_layers,
                  int64_t page_stride_bytes, int64_t page_bytes, int64_t num_pages,
                  const int32_t* src_pages, const int32_t* dst_pages, int32_t num_pairs,
                  void* stream);

/* Replaces the per-layer prologue of the reference's patched attention
 * (src/models/llama.py:163-210): qkv = x W^T with W the fused [q; k; v]
 * projection weight of _fuse_qkv_proj_plain (llama.py:256-280, no bias),
 * RoPE on the q and k heads (apply_rope_pos_ids_inplace), and the append of
 * k and v into the paged cache (append_paged_kv_cache) — one tcgen05 GEMM
 * whose epilogue rotates in fp32 straight from the accumulator.
 *   x       [num_tokens, hidden], row stride x_stride elements
 *   weight  [(H_q + 2 H_kv) * D, hidden], row stride w_stride elements
 *   q_out   [num_tokens, H_q, D] rotated q, token stride q_stride_n elements
 * k / v rows of token t go to the slot of (batch_indices[t], positions[t])
 * exactly as pa_append_paged_kv_cache places them (batch index -1: not
 * appended). RoPE uses positions[t]. Values match the unfused sequence up to
 * the one rounding of qkv to 16 bits that the fusion removes. Needs D = 64
 * or 128, hidden % 64 == 0 and H_q * D, H_kv * D multiples of 128. */
int pa_qkv_rope_append(const void* x, int64_t x_stride, const void* weight, int64_t w_stride,
                       int32_t num_tokens, int32_t hidden, int32_t num_qo_heads, void* q_out,
                       int64_t q_stride_n, const int32_t* batch_indices, const int32_t* positions,
                       int32_t rotary_dim, int32_t interleave, float rope_scale, float rope_theta,
                       const pa_kv_cache* cache, const int32_t* kv_indices,
                       int64_t num_kv_indices, const int32_t* kv_indptr, int32_t batch_size,
                       void* stream);

/* Diagnostic with no reference counterpart: launches one warp that waits on
 * a barrier nothing completes, with a limit of limit_cycles SM clocks (at
 * most the kernels' own limit). The wait gives up, PA_ERR_TIMEOUT lands in
 * the device status word, the kernel returns and the context stays usable —
 * the path every bounded wait in this library takes, exercised without a
 * fault. */
int pa_selftest_wait_timeout(int64_t limit_cycles, void* stream);

/* Workspace bytes pa_decode_plan needs for this batch geometry. */
size_t pa_decode_workspace_bytes(int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads,
                                 int32_t head_dim);

/* Replaces BatchDecodeWithPagedKVCacheWrapper.plan / begin_forward
 * (src/models/llama.py:119-147, called from step_executor.py:227-234).
 * Runs on the device: validates the CSR table, splits the (request,
 * kv-head, page) stream evenly over the persistent decode warps and writes
 * that partition into `workspace`. Reused by every layer until the next plan. */
int pa_decode_plan(const int32_t* kv_indptr, const int32_t* kv_last_page_len, int32_t batch_size,
                   int64_t num_kv_indices, int32_t num_qo_heads, int32_t num_kv_heads,
                   int32_t head_dim, int32_t page_size, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Replaces BatchDecodeWithPagedKVCacheWrapper.forward / run
 * (src/models/llama.py:230-245). q [B, H_q, D] with strides in elements;
 * out [B, H_q, D] contiguous; lse [B, H_q] float (may be NULL).
 * sm_scale <= 0 selects 1/sqrt(head_dim). Split requests are merged by
 * log-sum-exp inside the same launch. */
int pa_decode_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
                  const int32_t* kv_indices, const int32_t* kv_indptr,
                  const int32_t* kv_last_page_len, int32_t batch_size, int32_t num_qo_heads,
                  float sm_scale, void* workspace, size_t workspace_bytes, void* out, float* lse,
                  void* stream);

/* Replaces the reference's decode-step pair (src/models/llama.py:188-210 then
 * 230-245, with the batch indices / positions step_executor.py:204-225
 * builds for decode: one new token per request, batch_indices = arange(B))
 *   flashinfer.append_paged_kv_cache(k, v, arange(B), positions, cache, ...)
 *   BatchDecodeWithPagedKVCacheWrapper.forward(q, cache)
 * with one launch. Row b of append_key / append_value [B, H_kv, D] (strides
 * in elements, last dim contiguous) goes to position positions[b] of request
 * b's pages exactly as pa_append_paged_kv_cache places it (bit-identical pool,
 * same device checks), and the attention sees it as if the append had run
 * first: the output equals pa_append_paged_kv_cache followed by
 * pa_decode_run. The other arguments mean what they mean for pa_decode_run;
 * the same plan serves both. */
int pa_decode_append_run(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                         const void* append_key, int64_t key_stride_n, int64_t key_stride_h,
                         const void* append_value, int64_t value_stride_n,
                         int64_t value_stride_h, const int32_t* positions,
                         const pa_kv_cache* cache, const int32_t* kv_indices,
                         const int32_t* kv_indptr, const int32_t* kv_last_page_len,
                         int32_t batch_size, int32_t num_qo_heads, float sm_scale,
                         void* workspace, size_t workspace_bytes, void* out, float* lse,
                         void* stream);

/* Two-level (cascade) decode, FlashInfer's MultiLevelCascadeAttentionWrapper
 * with two levels, for a batch whose requests all begin with the same shared
 * prefix pages — what the reference's RadixCache produces when requests share
 * a system prompt (src/engine/memory/radix_cache.py:28-88). The reference
 * decodes such a batch with BatchDecodeWithPagedKVCacheWrapper over each
 * request's full table (src/models/llama.py:230-245), reading the prefix
 * once per request; here it is attended once for all requests.
 *   level 0: shared_kv_indptr = {0, n0}, shared_kv_indices[n0],
 *            shared_kv_last_page_len[1] — the prefix pages (the plan is
 *            given num_shared_indices, the page ids the array holds; n0
 *            beyond it is a device-check error);
 *   level 1: unique_kv_indptr[B+1], unique_kv_indices,
 *            unique_kv_last_page_len[B] — each request's pages after it
 *            (a request may have none).
 * Output equals decoding each request over prefix + unique pages, within the
 * bf16 tolerance. Plan once per step (device side, no host synchronisation);
 * run per layer. */
size_t pa_cascade_workspace_bytes(int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads,
                                  int32_t head_dim);
int pa_cascade_plan(const int32_t* shared_kv_indptr, const int32_t* shared_kv_last_page_len,
                    int64_t num_shared_indices, const int32_t* unique_kv_indptr,
                    const int32_t* unique_kv_last_page_len, int32_t batch_size,
                    int64_t num_unique_indices, int32_t num_qo_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t page_size, void* workspace, size_t workspace_bytes,
                    void* stream);
int pa_cascade_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
                   const int32_t* shared_kv_indices, const int32_t* unique_kv_indices,
                   const int32_t* unique_kv_indptr, const int32_t* unique_kv_last_page_len,
                   int32_t batch_size, int32_t num_qo_heads, float sm_scale, void* workspace,
                   size_t workspace_bytes, void* out, float* lse, void* stream);

/* pa_cascade_run with the decode step's KV append fused into level 1, as
 * pa_decode_append_run does for the plain decode: row b of append_key /
 * append_value goes to global position positions[b] of request b (the
 * reference's append_paged_kv_cache, src/models/llama.py:188-210), which must
 * fall inside the request's level-1 pages (position - prefix keys in
 * [0, keys of level 1)); otherwise the device status reports
 * PA_ERR_DEVICE_CHECK. Shared prefix pages are never written. */
int pa_cascade_append_run(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                          const void* append_key, int64_t key_stride_n, int64_t key_stride_h,
                          const void* append_value, int64_t value_stride_n,
                          int64_t value_stride_h, const int32_t* positions,
                          const pa_kv_cache* cache, const int32_t* shared_kv_indices,
                          const int32_t* unique_kv_indices, const int32_t* unique_kv_indptr,
                          const int32_t* unique_kv_last_page_len, int32_t batch_size,
                          int32_t num_qo_heads, float sm_scale, void* workspace,
                          size_t workspace_bytes, void* out, float* lse, void* stream);

/* Workspace bytes pa_prefill_plan needs. */
size_t pa_prefill_workspace_bytes(int32_t batch_size, int64_t max_total_qo, int32_t num_qo_heads,
                                  int32_t num_kv_heads, int32_t head_dim);

/* Replaces BatchPrefillWithPagedKVCacheWrapper.plan / begin_forward
 * (src/models/llama.py:86-116, called from step_executor.py:157-165).
 * Device-side: validates qo_indptr / kv_indptr / kv_last_page_len and writes
 * the list of (request, kv-head, 128-row query tile) work items. */
int pa_prefill_plan(const int32_t* qo_indptr, const int32_t* kv_indptr,
                    const int32_t* kv_last_page_len, int32_t batch_size, int64_t total_qo,
                    int64_t num_kv_indices, int32_t num_qo_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t page_size, void* workspace, size_t workspace_bytes,
                    void* stream);

/* Replaces BatchPrefillWithPagedKVCacheWrapper.forward(q, cache, causal)
 * (src/models/llama.py:212-228). q [total_qo, H_q, D] (strides in elements),
 * out [total_qo, H_q, D] contiguous, lse [total_qo, H_q] (may be NULL).
 * causal != 0 aligns the mask bottom-right: query i of a request with
 * qo_len rows and kv_len keys sees key j iff j <= i + kv_len - qo_len. */
int pa_prefill_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
                   const int32_t* qo_indptr, const int32_t* kv_indices, const int32_t* kv_indptr,
                   const int32_t* kv_last_page_len, int32_t batch_size, int64_t total_qo,
                   int32_t num_qo_heads, int32_t causal, float sm_scale, void* workspace,
                   size_t workspace_bytes, void* out, float* lse, void* stream);

/* Replaces flashinfer.merge_states (the split-KV log-sum-exp merge):
 * v [seq_len, num_states, num_heads, D] (dtype), s [seq_len, num_states,
 * num_heads] float base-2 LSE -> v_merged [seq_len, num_heads, D] (dtype),
 * s_merged [seq_len, num_heads] (may be NULL). */
int pa_merge_states(const void* v, const float* s, int32_t seq_len, int32_t num_states,
                    int32_t num_heads, int32_t head_dim, int32_t dtype, void* v_merged,
                    float* s_merged, void* stream);

/* Size of the static device scratch that pa_decode_noalloc uses (24 MiB). */
#define PA_NOALLOC_SCRATCH_BYTES (24u * 1024u * 1024u)

/* No counterpart in the reference (FlashInfer always takes a caller-owned
 * workspace). Decode attention — plan and run in one call — that allocates
 * nothing and needs no workspace: for callers that cannot allocate device
 * memory, such as C / FFI hosts that only hold buffers another runtime
 * allocated (the pool, q, out) and have no allocator of their own, or
 * serving loops that must not call cudaMalloc once the KV pool has claimed
 * most of HBM (it can fail then, and it synchronises the device).
 * Arguments mean what they mean for pa_decode_plan + pa_decode_run.
 * Scratch (plan, split-KV partials, merge counters) lives in one static
 * device array of PA_NOALLOC_SCRATCH_BYTES that every GPU loading this
 * library holds until exit. Batches whose scratch would exceed it return
 * PA_ERR_WORKSPACE_TOO_SMALL before anything is launched.
 * The first call on a device looks up that array's device address (with
 * that device current); make the first call before any stream capture.
 * All calls share the one array and the plan is rewritten (and the merge
 * counters cleared) by every call, so calls whose GPU work overlaps — two
 * streams, or two host threads on the same device — race; serialise them. */
int pa_decode_noalloc(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                      const pa_kv_cache* cache, const int32_t* kv_indices,
                      const int32_t* kv_indptr, const int32_t* kv_last_page_len,
                      int32_t batch_size, int64_t num_kv_indices, int32_t num_qo_heads,
                      float sm_scale, void* out, float* lse, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_ATTN_H_ */
