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
  griddep_wait();
  griddep_launch_dependents();
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
  int64_t num_kv_indices;  // entries kv_indptr may index
  const int32_t* kv_indptr;
  int batch;
  int num_kv_heads, page_size, row_chunks;  // row_chunks = head_dim * elem / 16
};

// One thread moves one 16-byte chunk of one (token, kv head) row of K or of
// V: page = kv_indices[kv_indptr[b] + pos / P], slot = pos % P. The
// reference's call site is src/models/llama.py:188-210 (kv_layout "HND").
__global__ void append_kernel(const AppendParams p) {
  griddep_wait();
  griddep_launch_dependents();
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
    const int64_t pi = static_cast<int64_t>(start) + pos / p.page_size;
    if (start < 0 || end > p.num_kv_indices || pi >= end) {
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
// fp32 math, result rounded to T. The standalone kernel and the fused
// RoPE + append kernel share these two functions (no FMA contraction), so
// both paths give bit-identical rows.
__device__ __forceinline__ float rope_freq(int i, int rotary_dim, float inv_scale,
                                          float log2_theta) {
  return exp2f(-(2.0f * i / rotary_dim) * log2_theta) * inv_scale;
}
__device__ __forceinline__ void rope_cos_sin(int pos, int i, int rotary_dim, float inv_scale,
                                             float log2_theta, float* cs, float* sn) {
  sincosf(static_cast<float>(pos) * rope_freq(i, rotary_dim, inv_scale, log2_theta), sn, cs);
}
__device__ __forceinline__ void rope_rotate(float x0, float x1, float cs, float sn, float* y0,
                                            float* y1) {
  *y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
  *y1 = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x0, sn));
}

// One thread rotates one pair of one row.
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
    float cs, sn;
    rope_cos_sin(__ldg(pos_ids + t), i, rotary_dim, inv_scale, log2_theta, &cs, &sn);
    const int a = interleave ? 2 * i : i;
    const int bidx = interleave ? 2 * i + 1 : i + half;
    float y0, y1;
    rope_rotate(static_cast<float>(row[a]), static_cast<float>(row[bidx]), cs, sn, &y0, &y1);
    row[a] = static_cast<T>(y0);
    row[bidx] = static_cast<T>(y1);
  }
}

// ------------------------------------------------------- RoPE + append
// The reference's per-layer pair apply_rope_pos_ids_inplace(q, k, positions)
// then append_paged_kv_cache(k, v, batch_indices, positions, ...)
// (src/models/llama.py:175-210) in one pass: q and k are rotated in place
// and the rotated k and v rows are written into their page slots, so k is
// read once instead of three times. Work units per token: 8 rotary pairs of
// a q head or a k head (two 16-byte chunks), a 16-byte chunk of k past
// rotary_dim, a 16-byte chunk of v. Needs rotary_dim % 16 == 0 and 16-byte
// aligned rows (the host entry point checks).
struct RopeAppendParams {
  uint8_t* q;
  uint8_t* k;
  const uint8_t* v;
  int64_t q_sn, q_sh, k_sn, k_sh, v_sn, v_sh;  // bytes
  const int32_t* batch_indices;
  const int32_t* positions;
  int nnz, hq, hkv, head_dim, rotary_dim, interleave;
  float inv_scale, log2_theta;
  uint8_t* k_base;
  uint8_t* v_base;
  int64_t page_stride, head_stride, token_stride;  // bytes
  int64_t num_pages;
  const int32_t* kv_indices;
  int64_t num_kv_indices;  // entries kv_indptr may index
  const int32_t* kv_indptr;
  int batch, page_size;
};

// Page slot of token t's row of kv head h (nullptr: padding row or an error,
// recorded in the status word).
__device__ __forceinline__ int64_t rope_append_slot(const RopeAppendParams& p, int t, int h) {
  const int b = __ldg(p.batch_indices + t);
  if (b < 0) return -1;  // padding row (batch index -1): rotated, not appended
  const int pos = __ldg(p.positions + t);
  if (b >= p.batch || pos < 0) {
    set_status(PA_ERR_DEVICE_CHECK);
    return -1;
  }
  const int start = __ldg(p.kv_indptr + b), end = __ldg(p.kv_indptr + b + 1);
  const int64_t pi = static_cast<int64_t>(start) + pos / p.page_size;
  if (start < 0 || end > p.num_kv_indices || pi >= end) {
    set_status(PA_ERR_DEVICE_CHECK);
    return -1;
  }
  const int page = __ldg(p.kv_indices + pi);
  if (page < 0 || page >= p.num_pages) {
    set_status(PA_ERR_DEVICE_CHECK);
    return -1;
  }
  return page * p.page_stride + h * p.head_stride + (pos % p.page_size) * p.token_stride;
}

template <typename T>
__device__ __forceinline__ void rope_chunk8(uint4* lo, uint4* hi, int pos, int i0, int interleave,
                                            const RopeAppendParams& p) {
  // lo / hi: two 16-byte chunks holding 8 pairs: non-interleaved lo[e] pairs
  // with hi[e]; interleaved the 16 elements lo|hi are 8 adjacent pairs.
  T* a = reinterpret_cast<T*>(lo);
  T* b = reinterpret_cast<T*>(hi);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float cs, sn, y0, y1;
    rope_cos_sin(pos, i0 + e, p.rotary_dim, p.inv_scale, p.log2_theta, &cs, &sn);
    T* x0 = interleave ? (e < 4 ? a + 2 * e : b + 2 * (e - 4)) : a + e;
    T* x1 = interleave ? x0 + 1 : b + e;
    rope_rotate(static_cast<float>(*x0), static_cast<float>(*x1), cs, sn, &y0, &y1);
    *x0 = static_cast<T>(y0);
    *x1 = static_cast<T>(y1);
  }
}

template <typename T>
__global__ void rope_append_kernel(const RopeAppendParams p) {
  griddep_wait();
  griddep_launch_dependents();
  const int nrot = p.rotary_dim / 16;              // 8-pair units per head
  const int npass = (p.head_dim - p.rotary_dim) / 8;  // k chunks past rotary_dim
  const int nv = p.head_dim / 8;                   // v chunks
  const int64_t per_token =
      static_cast<int64_t>(p.hq + p.hkv) * nrot + static_cast<int64_t>(p.hkv) * (npass + nv);
  const int64_t total = per_token * p.nnz;
  const int half = p.rotary_dim / 2;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(idx / per_token);
    int u = static_cast<int>(idx - t * per_token);
    if (u < (p.hq + p.hkv) * nrot) {
      // rotary unit: 8 pairs of a q or k head
      const int head = u / nrot, c = u - head * nrot;
      const bool is_k = head >= p.hq;
      const int h = is_k ? head - p.hq : head;
      uint8_t* row = is_k ? p.k + t * p.k_sn + h * p.k_sh : p.q + t * p.q_sn + h * p.q_sh;
      // element offsets of the two chunks
      const int e_lo = p.interleave ? 16 * c : 8 * c;
      const int e_hi = p.interleave ? 16 * c + 8 : half + 8 * c;
      uint4* lo_ptr = reinterpret_cast<uint4*>(row + e_lo * 2);
      uint4* hi_ptr = reinterpret_cast<uint4*>(row + e_hi * 2);
      uint4 lo = *lo_ptr, hi = *hi_ptr;
      rope_chunk8<T>(&lo, &hi, __ldg(p.positions + t), 8 * c, p.interleave, p);
      *lo_ptr = lo;
      *hi_ptr = hi;
      if (is_k) {
        const int64_t off = rope_append_slot(p, t, h);
        if (off >= 0) {
          *reinterpret_cast<uint4*>(p.k_base + off + e_lo * 2) = lo;
          *reinterpret_cast<uint4*>(p.k_base + off + e_hi * 2) = hi;
        }
      }
      continue;
    }
    u -= (p.hq + p.hkv) * nrot;
    if (u < p.hkv * npass) {
      // k chunk past rotary_dim: copied as is
      const int h = u / npass, c = u - h * npass;
      const int e = p.rotary_dim + 8 * c;
      const int64_t off = rope_append_slot(p, t, h);
      if (off >= 0)
        *reinterpret_cast<uint4*>(p.k_base + off + e * 2) =
            *reinterpret_cast<const uint4*>(p.k + t * p.k_sn + h * p.k_sh + e * 2);
      continue;
    }
    u -= p.hkv * npass;
    {
      const int h = u / nv, c = u - h * nv;
      const int64_t off = rope_append_slot(p, t, h);
      if (off >= 0)
        *reinterpret_cast<uint4*>(p.v_base + off + c * 16) =
            __ldg(reinterpret_cast<const uint4*>(p.v + t * p.v_sn + h * p.v_sh) + c);
    }
  }
}

// ------------------------------------------------------------ page fork
// Copy-on-write of shared partial pages (the reference's planned incremental
// radix insertion, todo.md "Copy-on-Write"): before a sequence appends into
// a page another sequence still references, the page is forked — its bytes
// in every layer copied to a fresh page id — and the sequence's block table
// then points at the copy. One thread per 16-byte chunk of (pair, layer).
struct ForkParams {
  uint8_t* pool;
  int64_t layer_stride, page_stride, page_bytes;  // bytes
  int num_layers;
  int64_t num_pages;
  const int32_t* src;
  const int32_t* dst;
  int n;
};

__global__ void fork_pages_kernel(const ForkParams p) {
  const int64_t chunks = p.page_bytes / 16;
  const int64_t per_pair = chunks * p.num_layers;
  const int64_t total = per_pair * p.n;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx / per_pair);
    const int64_t rem = idx - i * per_pair;
    const int layer = static_cast<int>(rem / chunks);
    const int64_t c = rem - layer * chunks;
    const int s = __ldg(p.src + i), d = __ldg(p.dst + i);
    if (s < 0 || s >= p.num_pages || d < 0 || d >= p.num_pages) {
      set_status(PA_ERR_DEVICE_CHECK);
      continue;
    }
    const uint8_t* from = p.pool + layer * p.layer_stride + s * p.page_stride;
    uint8_t* to = p.pool + layer * p.layer_stride + d * p.page_stride;
    reinterpret_cast<uint4*>(to)[c] = reinterpret_cast<const uint4*>(from)[c];
  }
}

// ------------------------------------------------------- wait self-test
// Exercises the bounded-wait path every kernel relies on, without a fault:
// one warp waits on an mbarrier that nothing arrives on, with a short limit;
// the wait gives up, the kernel records PA_ERR_TIMEOUT and returns, and the
// context stays usable.
__global__ void wait_selftest_kernel(long long limit_cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  const bool ok = mbar_wait_warp_limit(&bar, 0, limit_cycles);
  if (!ok && threadIdx.x == 0) set_status(PA_ERR_TIMEOUT);
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
