// Device-side page-table build for a step: the CSR tables, batch indices and
// positions that the reference's StepExecutor assembles in Python lists and
// copies to the device every step (src/engine/runtime/step_executor.py:
// 98-155 for prefill chunks, 204-225 for decode). Inputs are the sequences'
// block tables as a padded int32 matrix [batch, stride] plus their lengths,
// all on the device, so a step needs no host loop, no host-to-device copy
// and no synchronisation, and can be captured in a CUDA graph.
//
// Two launches per build: a one-CTA scan (lengths -> indptrs, last-page
// lengths, the compacted list of active sequences, totals checked against
// the output capacities) and a gather over the active sequences (block ids
// -> kv_indices; prefill rows -> batch indices / positions).
#pragma once

#include "pa_common.cuh"

namespace pa {

constexpr int kTablesScanThreads = 1024;

struct TablesParams {
  const int32_t* block_tables;
  int64_t stride;               // elements between two sequences' rows
  const int32_t* num_blocks;    // block_table length per sequence
  const int32_t* lens;          // decode: get_len; prefill: computed_len
  const int32_t* prompt_lens;   // prefill only
  const int32_t* chunk_lens;    // prefill only: chunk the scheduler authorised
  int batch, page_size, prefill;
  int32_t* qo_indptr;           // prefill only
  int32_t* kv_indptr;
  int32_t* kv_indices;
  int64_t kv_capacity;
  int32_t* last_page_len;
  int32_t* seq_lens_out;        // prefill only: computed_len + chunk
  int32_t* active;              // prefill only: input index of each output slot
  int32_t* batch_indices;
  int32_t* positions;
  int64_t rows_capacity;
  int32_t* counts;              // [0] active sequences, [1] rows, [2] error flag
};

// Per sequence: chunk (prefill) / 1 (decode), pages, and validity.
__device__ __forceinline__ void tables_entry(const TablesParams& p, int b, int* chunk, int* pages,
                                             bool* bad) {
  const int nb = p.num_blocks[b];
  const int len = p.lens[b];
  *bad = nb < 0 || nb > p.stride || len < 0;
  if (p.prefill) {
    // step_executor.py:102-118: chunk = min(authorised, prompt - computed);
    // a chunk <= 0 drops the sequence from the step; the chunk uses the
    // first ceil(new_len / P) blocks of the table.
    const int c = min(p.chunk_lens[b], p.prompt_lens[b] - len);
    *chunk = c > 0 ? c : 0;
    const int new_len = len + *chunk;
    *pages = *chunk > 0 ? (new_len + p.page_size - 1) / p.page_size : 0;
    if (*pages > nb) *bad = true;
  } else {
    // step_executor.py:208-214: the whole block table; get_len >= 1 must be
    // covered by it.
    *chunk = 1;
    *pages = nb;
    if (len < 1 || static_cast<int64_t>(nb) * p.page_size < len) *bad = true;
  }
}

__global__ void __launch_bounds__(kTablesScanThreads) tables_scan_kernel(const TablesParams p) {
  __shared__ int64_t s_rows[kTablesScanThreads], s_pages[kTablesScanThreads];
  __shared__ int s_act[kTablesScanThreads];
  __shared__ int s_bad;
  const int tid = threadIdx.x;
  if (tid == 0) s_bad = 0;
  // each thread scans a contiguous range of sequences
  const int per = (p.batch + kTablesScanThreads - 1) / kTablesScanThreads;
  const int b0 = min(tid * per, p.batch), b1 = min(b0 + per, p.batch);
  int64_t rows = 0, pages = 0;
  int act = 0;
  bool bad = false;
  for (int b = b0; b < b1; ++b) {
    int c, pg;
    bool e;
    tables_entry(p, b, &c, &pg, &e);
    bad |= e;
    if (c > 0) {
      rows += c;
      pages += pg;
      ++act;
    }
  }
  s_rows[tid] = rows;
  s_pages[tid] = pages;
  s_act[tid] = act;
  __syncthreads();
  if (bad) atomicOr(&s_bad, 1);
  // inclusive Hillis-Steele scan over the per-thread totals
  for (int off = 1; off < kTablesScanThreads; off <<= 1) {
    int64_t r = 0, g = 0;
    int a = 0;
    if (tid >= off) {
      r = s_rows[tid - off];
      g = s_pages[tid - off];
      a = s_act[tid - off];
    }
    __syncthreads();
    s_rows[tid] += r;
    s_pages[tid] += g;
    s_act[tid] += a;
    __syncthreads();
  }
  const int64_t total_rows = s_rows[kTablesScanThreads - 1];
  const int64_t total_pages = s_pages[kTablesScanThreads - 1];
  const int total_act = s_act[kTablesScanThreads - 1];
  const bool err = s_bad != 0 || total_pages > p.kv_capacity || total_rows > p.rows_capacity ||
                   total_pages > 0x7fffffffLL || total_rows > 0x7fffffffLL;
  if (err) {
    if (tid == 0) {
      p.counts[0] = 0;
      p.counts[1] = 0;
      p.counts[2] = 1;
      set_status(PA_ERR_DEVICE_CHECK);
    }
    return;
  }
  // exclusive offsets of this thread's range
  int64_t row = s_rows[tid] - rows, pg = s_pages[tid] - pages;
  int slot = s_act[tid] - act;
  if (tid == 0) {
    if (p.prefill) p.qo_indptr[0] = 0;
    p.kv_indptr[0] = 0;
    p.counts[0] = total_act;
    p.counts[1] = static_cast<int>(total_rows);
    p.counts[2] = 0;
  }
  for (int b = b0; b < b1; ++b) {
    int c, n;
    bool e;
    tables_entry(p, b, &c, &n, &e);
    if (c <= 0) continue;
    row += c;
    pg += n;
    const int len = p.lens[b];
    if (p.prefill) {
      const int new_len = len + c;
      const int ll = new_len % p.page_size;
      p.qo_indptr[slot + 1] = static_cast<int>(row);
      p.seq_lens_out[slot] = new_len;
      p.active[slot] = b;
      p.last_page_len[slot] = ll > 0 ? ll : p.page_size;
    } else {
      const int ll = len % p.page_size;
      p.last_page_len[slot] = ll > 0 ? ll : p.page_size;
      p.batch_indices[slot] = slot;
      p.positions[slot] = len - 1;
    }
    p.kv_indptr[slot + 1] = static_cast<int>(pg);
    ++slot;
  }
}

// One CTA per output slot (grid = batch; slots past the active count exit).
__global__ void tables_gather_kernel(const TablesParams p) {
  if (p.counts[2] != 0) return;
  const int s = blockIdx.x;
  if (s >= p.counts[0]) return;
  const int b = p.prefill ? p.active[s] : s;
  const int k0 = p.kv_indptr[s], k1 = p.kv_indptr[s + 1];
  const int32_t* row = p.block_tables + static_cast<int64_t>(b) * p.stride;
  for (int i = threadIdx.x; i < k1 - k0; i += blockDim.x) p.kv_indices[k0 + i] = __ldg(row + i);
  if (p.prefill) {
    // get_batch_indices_positions(qo_indptr, seq_lens) for this chunk's rows
    const int q0 = p.qo_indptr[s], q1 = p.qo_indptr[s + 1];
    const int first = p.lens[b];
    for (int t = q0 + threadIdx.x; t < q1; t += blockDim.x) {
      p.batch_indices[t] = s;
      p.positions[t] = first + (t - q0);
    }
  }
}

}  // namespace pa
