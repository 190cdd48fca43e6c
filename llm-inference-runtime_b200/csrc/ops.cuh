// The small HBM-bound kernels around the attention kernels: batch indices /
// positions, the KV append scatter, RoPE in place, and the standalone
// log-sum-exp merge of attention states.
#pragma once

#include "pa_common.cuh"

namespace pa {

// ------------------------------------------------ batch indices / positions
// Behaviour of flashinfer.get_batch_indices_positions (the reference calls it
// at src/models/llama.py:79-83): block b < batch writes the rows of request
// b; block `batch` writes the tail rows [append_indptr[batch], nnz) as
// (-1, 0), which is how FlashInfer pre-fills its outputs.
__global__ void batch_indices_positions_kernel(const int32_t* __restrict__ append_indptr,
                                               const int32_t* __restrict__ seq_lens, int batch,
                                               int nnz, int32_t* __restrict__ batch_indices,
                                               int32_t* __restrict__ positions) {
  const int b = blockIdx.x;
  if (b < batch) {
    const int start = append_indptr[b], end = min(append_indptr[b + 1], nnz);
    const int first_pos = seq_lens[b] - (append_indptr[b + 1] - start);
    for (int t = start + threadIdx.x; t < end; t += blockDim.x) {
      batch_indices[t] = b;
      positions[t] = first_pos + (t - start);
    }
  } else {
    for (int t = max(append_indptr[batch], 0) + threadIdx.x; t < nnz; t += blockDim.x) {
      batch_indices[t] = -1;
      positions[t] = 0;
    }
  }
}

// ------------------------------------------------------------ KV append
struct AppendParams {
  const uint8_t* key;
  const uint8_t* value;
  int64_t key_stride_n, key_stride_h, value_stride_n, value_stride_h;  // bytes
  const int32_t* batch_indices;
  const int32_t* positions;
  int nnz;
  uint8_t* k_base;
  uint8_t* v_base;
  int64_t page_stride, head_stride, token_stride;  // bytes
  int64_t num_pages;
  const int32_t* kv_indices;
  const int32_t* kv_indptr;
  int batch;
  int num_kv_heads, page_size, row_chunks;  // row_chunks = head_dim * elem / 16
};

// One thread moves one 16-byte chunk of one (token, kv head) row of K or of
// V: page = kv_indices[kv_indptr[b] + pos / P], slot = pos % P. The
// reference's call site is src/models/llama.py:188-210 (kv_layout "HND").
__global__ void append_kernel(const AppendParams p) {
  const int64_t per_token = static_cast<int64_t>(p.num_kv_heads) * p.row_chunks * 2;
  const int64_t total = per_token * p.nnz;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(idx / per_token);
    int rem = static_cast<int>(idx - t * per_token);
    const int c = rem % p.row_chunks;
    rem /= p.row_chunks;
    const int h = rem % p.num_kv_heads;
    const int kv = rem / p.num_kv_heads;
    const int b = __ldg(p.batch_indices + t);
    if (b < 0) continue;  // padding row (batch index -1)
    const int pos = __ldg(p.positions + t);
    if (b >= p.batch || pos < 0) {
      set_status(PA_ERR_DEVICE_CHECK);
      continue;
    }
    const int start = __ldg(p.kv_indptr + b), end = __ldg(p.kv_indptr + b + 1);
    const int pi = start + pos / p.page_size;
    if (pi >= end) {
      set_status(PA_ERR_DEVICE_CHECK);
      continue;
    }
    const int page = __ldg(p.kv_indices + pi);
    if (page < 0 || page >= p.num_pages) {
      set_status(PA_ERR_DEVICE_CHECK);
      continue;
    }
    const int slot = pos % p.page_size;
    const uint8_t* src = kv ? p.value + t * p.value_stride_n + h * p.value_stride_h
                            : p.key + t * p.key_stride_n + h * p.key_stride_h;
    uint8_t* dst = (kv ? p.v_base : p.k_base) + page * p.page_stride + h * p.head_stride +
                   slot * p.token_stride;
    reinterpret_cast<uint4*>(dst)[c] = __ldg(reinterpret_cast<const uint4*>(src) + c);
  }
}

// ------------------------------------------------------------------ RoPE
// flashinfer.apply_rope_pos_ids_inplace (src/models/llama.py:175-182):
// for i < rotary_dim / 2, angle = pos / rope_scale * rope_theta^(-2i/rotary_dim).
// Non-interleaved pairs (i, i + rotary_dim/2); interleaved pairs (2i, 2i+1).
// One thread rotates one pair of one row; fp32 math, result rounded to T.
template <typename T>
__global__ void rope_kernel(T* q, int64_t q_sn, int64_t q_sh, T* k, int64_t k_sn, int64_t k_sh,
                            const int32_t* __restrict__ pos_ids, int nnz, int hq, int hkv,
                            int rotary_dim, int interleave, float inv_scale, float log2_theta) {
  const int half = rotary_dim / 2;
  const int64_t per_token = static_cast<int64_t>(hq + hkv) * half;
  const int64_t total = per_token * nnz;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(idx / per_token);
    const int rem = static_cast<int>(idx - t * per_token);
    const int head = rem / half;
    const int i = rem - head * half;
    T* row = head < hq ? q + t * q_sn + head * q_sh : k + t * k_sn + (head - hq) * k_sh;
    const float freq = exp2f(-(2.0f * i / rotary_dim) * log2_theta) * inv_scale;
    const float ang = static_cast<float>(__ldg(pos_ids + t)) * freq;
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const int a = interleave ? 2 * i : i;
    const int bidx = interleave ? 2 * i + 1 : i + half;
    const float x0 = static_cast<float>(row[a]);
    const float x1 = static_cast<float>(row[bidx]);
    row[a] = static_cast<T>(x0 * cs - x1 * sn);
    row[bidx] = static_cast<T>(x1 * cs + x0 * sn);
  }
}

// -------------------------------------------------------------- merge
// flashinfer.merge_states: v [n, S, H, D], s [n, S, H] (base-2 LSE) ->
// v_merged [n, H, D], s_merged [n, H]. One warp per (row, head).
template <typename T>
__global__ void merge_states_kernel(const T* __restrict__ v, const float* __restrict__ s, int n,
                                    int num_states, int heads, int head_dim, T* __restrict__ vm,
                                    float* __restrict__ sm) {
  const int warps = blockDim.x >> 5;
  const int item = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= n * heads) return;
  const int r = item / heads, h = item - r * heads;
  float lmax = -INFINITY;
  for (int k = 0; k < num_states; ++k)
    lmax = fmaxf(lmax, s[(static_cast<int64_t>(r) * num_states + k) * heads + h]);
  float wsum = 0.f;
  for (int k = 0; k < num_states; ++k) {
    const float sk = s[(static_cast<int64_t>(r) * num_states + k) * heads + h];
    wsum += (lmax == -INFINITY) ? 0.f : ex2(sk - lmax);
  }
  const float winv = wsum > 0.f ? 1.f / wsum : 0.f;
  for (int d = lane; d < head_dim; d += 32) {
    float acc = 0.f;
    for (int k = 0; k < num_states; ++k) {
      const int64_t row = (static_cast<int64_t>(r) * num_states + k) * heads + h;
      const float w = (lmax == -INFINITY) ? 0.f : ex2(s[row] - lmax);
      acc += w * static_cast<float>(v[row * head_dim + d]);
    }
    vm[(static_cast<int64_t>(r) * heads + h) * head_dim + d] = static_cast<T>(acc * winv);
  }
  if (sm != nullptr && lane == 0)
    sm[static_cast<int64_t>(r) * heads + h] = wsum > 0.f ? lmax + lg2(wsum) : -INFINITY;
}

}  // namespace pa
