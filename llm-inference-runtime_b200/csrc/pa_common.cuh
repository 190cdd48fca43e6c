// Shared definitions of the paged-attention kernels: device status word,
// workspace layouts produced by the plan kernels, and small helpers.
#pragma once

#include "pa_ptx.cuh"
#include "paged_attn.h"

namespace pa {

// The engine's page size (EngineConfig.block_size = 16 in the reference,
// src/engine/config.py:13). One page is one 16-key MMA tile.
constexpr int kPage = 16;
// Largest GQA group (q heads per kv head) one decode warp tile holds: the
// 16 rows of an m16n8k16 A fragment.
constexpr int kMaxGroup = 16;
constexpr int32_t kDecodeMagic = 0x50414431;   // "PAD1"
constexpr int32_t kPrefillMagic = 0x50415031;  // "PAP1"

// First error recorded by any kernel since the host last read it
// (pa_device_status). One word per device context.
__device__ int g_status;

__device__ __forceinline__ void set_status(int code) { atomicCAS(&g_status, 0, code); }

__host__ __device__ __forceinline__ size_t align256(size_t x) {
  return (x + 255) & ~static_cast<size_t>(255);
}

template <typename T>
__device__ __forceinline__ T* align1024(T* p) {
  return reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ------------------------------------------------------------------ decode
struct DecodePlanHeader {
  int32_t magic;
  int32_t status;          // PA_OK, or PA_ERR_DEVICE_CHECK when the table is malformed
  int32_t total;           // pages in the stream = head blocks * kv_indptr[B]
  int32_t per_unit;        // Q: pages per group
  int32_t num_units;       // groups the partition was built for
  int32_t batch_size;
  int32_t num_kv_heads;
  int32_t num_qo_heads;
  int32_t head_dim;
  int32_t page_size;
  int32_t num_empty;       // requests with zero pages (their output is zero)
  int32_t heads_per_unit;  // kv heads a group covers (one warp each)
  int32_t reserved[4];
};

// Byte offsets inside the caller's workspace. The stream of work is every
// (request b, head block, page j); group u owns positions [u*Q, (u+1)*Q).
struct DecodeWsLayout {
  size_t hdr, unit_start, empty, counter, part_lse, part_o, total;
};

__host__ __device__ inline DecodeWsLayout decode_ws_layout(int num_units, int batch, int hkv,
                                                           int head_dim, int heads_per_unit) {
  DecodeWsLayout L;
  const size_t slots = static_cast<size_t>(num_units) * 2 * heads_per_unit;
  size_t o = 0;
  L.hdr = o;
  o = align256(o + sizeof(DecodePlanHeader));
  L.unit_start = o;  // int4 {b, head block, j, 0} of each group's first page
  o = align256(o + sizeof(int4) * static_cast<size_t>(num_units));
  L.empty = o;  // int32 list of requests without pages
  o = align256(o + 4 * static_cast<size_t>(batch));
  L.counter = o;  // int32 per (request, kv head): pieces finished this launch
  o = align256(o + 4 * static_cast<size_t>(batch) * hkv);
  L.part_lse = o;  // float [units][2][heads][kMaxGroup]: base-2 LSE of split pieces
  o = align256(o + 4 * slots * kMaxGroup);
  L.part_o = o;  // float [units][2][heads][kMaxGroup][D]: normalised split outputs
  o = align256(o + 4 * slots * kMaxGroup * head_dim);
  L.total = o;
  return L;
}

struct DecodeParams {
  const void* q;
  int64_t q_stride_n, q_stride_h;
  void* out;
  float* lse;
  const int32_t* kv_indices;
  const int32_t* kv_indptr;
  const int32_t* kv_last_page_len;
  int32_t batch_size, num_qo_heads, num_kv_heads, group;
  int64_t num_pages;
  int32_t heads_inner;  // tensor-map dim order (D, H, P, pages) instead of (D, P, H, pages)
  float scale_log2;     // sm_scale * log2(e)
  // launch geometry (DecodeGeom)
  int32_t hb, nhb, groups_per_cta, stages, stage_bytes;
  const DecodePlanHeader* hdr;
  const int4* unit_start;
  const int32_t* empty;
  int32_t* counter;
  float* part_lse;
  float* part_o;
  // Optional decode-step append (pa_decode_append_run): request b's new K / V
  // row (row b of new_k / new_v) goes to position append_pos[b] of its pages
  // before the attention reads that page. append_pos == nullptr: no append.
  const int32_t* append_pos;
  // Optional device word subtracted from every append_pos entry (the cascade
  // passes global positions; its level-1 pages start after the shared prefix).
  const int32_t* append_pos_base;
  const uint8_t* new_k;
  const uint8_t* new_v;
  int64_t new_k_stride_n, new_k_stride_h, new_v_stride_n, new_v_stride_h;  // bytes
  uint8_t* k_pool;
  uint8_t* v_pool;
  int64_t pool_page_stride, pool_head_stride, pool_token_stride;  // bytes
};

}  // namespace pa
