// Two-level (cascade) decode for a batch whose requests all begin with the
// same shared prefix pages, the situation the reference's RadixCache creates
// when many requests share a system prompt (src/engine/memory/radix_cache.py:
// 28-88; identical refcounted page ids at the head of every block table).
//
// Level 0 — the shared prefix — is attended once for all requests: the
// prefix pages are cut into key chunks, and each chunk is one non-causal
// "request" of the tcgen05 prefill kernel whose query rows are all B decode
// queries (every chunk reads the same q rows and writes its own output rows
// and base-2 LSEs). Level 1 — each request's unique pages — is the ordinary
// decode kernel with LSE output. A merge kernel combines, per (request,
// head), the level-0 chunk states and the level-1 state by log-sum-exp.
//
// Equivalent to decoding over the concatenated tables (prefix pages, then
// the request's unique pages): outputs agree within the bf16 tolerance (the
// partial outputs are rounded to the storage type before the merge, as in
// FlashInfer's cascade).
#pragma once

#include "decode.cuh"
#include "prefill.cuh"

namespace pa {

constexpr int32_t kCascadeMagic = 0x50414331;  // "PAC1"
constexpr int kCascadeMaxChunks = 64;

struct CascadeHeader {
  int32_t magic;
  int32_t status;
  int32_t num_chunks;       // non-empty level-0 chunks this plan produced
  int32_t pages_per_chunk;
  int32_t batch_size;
  int32_t max_chunks;
  int32_t prefix_tokens;    // keys of level 0; level-1 positions start here
  int32_t reserved[9];
};

// Byte offsets inside the caller's workspace (all 256-byte aligned).
struct CascadeWsLayout {
  size_t hdr, qo_indptr, kv_indptr, last, q_rows;  // level-0 chunk tables
  size_t prefill;                                   // prefill plan (header + items)
  size_t decode;                                    // level-1 decode plan / partials
  size_t o0, lse0, o1, lse1;                        // level states
  size_t total;
  int64_t prefill_items;
};

__host__ __device__ inline CascadeWsLayout cascade_ws_layout(int batch, int hq, int hkv,
                                                             int head_dim, int max_chunks,
                                                             int span, int decode_units,
                                                             int decode_hb) {
  CascadeWsLayout L;
  size_t o = 0;
  L.hdr = o;
  o = align256(o + sizeof(CascadeHeader));
  L.qo_indptr = o;
  o = align256(o + 4 * static_cast<size_t>(max_chunks + 1));
  L.kv_indptr = o;
  o = align256(o + 4 * static_cast<size_t>(max_chunks + 1));
  L.last = o;
  o = align256(o + 4 * static_cast<size_t>(max_chunks));
  L.q_rows = o;
  o = align256(o + 4 * static_cast<size_t>(max_chunks));
  L.prefill_items = static_cast<int64_t>(max_chunks) * hkv * ((batch + span - 1) / span);
  L.prefill = o;
  o = align256(o + prefill_ws_layout(L.prefill_items).total);
  L.decode = o;
  o = align256(o + decode_ws_layout(decode_units, batch, hkv, head_dim, decode_hb).total);
  const size_t rows0 = static_cast<size_t>(max_chunks) * batch * hq;
  const size_t rows1 = static_cast<size_t>(batch) * hq;
  L.o0 = o;
  o = align256(o + rows0 * head_dim * 2);
  L.lse0 = o;
  o = align256(o + rows0 * 4);
  L.o1 = o;
  o = align256(o + rows1 * head_dim * 2);
  L.lse1 = o;
  o = align256(o + rows1 * 4);
  L.total = o;
  return L;
}

// One CTA: validates the level-0 table ([0, n0] pages within the
// num_shared_indices page ids given, last page length),
// cuts the prefix into chunks of whole 128-key tiles and writes the chunk
// tables, the prefill kernel's header and its work items (chunk, kv head,
// query span); then plans level 1 (the decode plan over each request's own
// pages) in the same launch.
__global__ void cascade_plan_kernel(const int32_t* __restrict__ shared_indptr,
                                    const int32_t* __restrict__ shared_last,
                                    int64_t num_shared_indices,
                                    const int32_t* __restrict__ unique_indptr,
                                    const int32_t* __restrict__ unique_last,
                                    int64_t num_unique_indices, int batch, int hq, int hkv,
                                    int head_dim, int page_size, int qt, int max_chunks,
                                    int decode_groups, int decode_hb, uint8_t* __restrict__ ws,
                                    CascadeWsLayout L) {
  griddep_wait();
  griddep_launch_dependents();
  CascadeHeader* ch = reinterpret_cast<CascadeHeader*>(ws + L.hdr);
  int32_t* qo_indptr = reinterpret_cast<int32_t*>(ws + L.qo_indptr);
  int32_t* kv_indptr = reinterpret_cast<int32_t*>(ws + L.kv_indptr);
  int32_t* last = reinterpret_cast<int32_t*>(ws + L.last);
  int32_t* q_rows = reinterpret_cast<int32_t*>(ws + L.q_rows);
  const PrefillWsLayout PL = prefill_ws_layout(L.prefill_items);
  PrefillPlanHeader* ph = reinterpret_cast<PrefillPlanHeader*>(ws + L.prefill + PL.hdr);
  int4* items = reinterpret_cast<int4*>(ws + L.prefill + PL.items);

  const int n0 = shared_indptr[1] - shared_indptr[0];
  const int lp = n0 > 0 ? shared_last[0] : page_size;
  const bool bad = shared_indptr[0] != 0 || n0 < 0 || n0 > num_shared_indices || lp < 1 ||
                   lp > page_size;
  const int tile_pages = kPfKeys / page_size;
  int ppc = n0 > 0 ? (n0 + max_chunks - 1) / max_chunks : tile_pages;
  ppc = (ppc + tile_pages - 1) / tile_pages * tile_pages;  // whole key tiles per chunk
  const int nch = bad || n0 <= 0 ? 0 : (n0 + ppc - 1) / ppc;
  const int span = 2 * qt, nq = (batch + span - 1) / span;
  for (int c = threadIdx.x; c <= max_chunks; c += blockDim.x) {
    qo_indptr[c] = c * batch;
    kv_indptr[c] = min(c * ppc, max(n0, 0));
    if (c < max_chunks) {
      last[c] = c == nch - 1 ? lp : page_size;
      q_rows[c] = 0;
    }
  }
  const int n_items = nch * hkv * nq;
  for (int i = threadIdx.x; i < n_items; i += blockDim.x) {
    const int c = i / (hkv * nq), rem = i - c * hkv * nq;
    items[i] = make_int4(c, rem / nq, (rem % nq) * span, 0);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ph->status = bad ? PA_ERR_DEVICE_CHECK : PA_OK;
    ph->num_items = bad ? 0 : n_items;
    ph->batch_size = max_chunks;
    ph->num_kv_heads = hkv;
    ph->num_qo_heads = hq;
    ph->head_dim = head_dim;
    ph->queries_per_tile = span;
    ph->next_item = 0;
    ph->ctas_done = 0;
    ph->magic = kPrefillMagic;
    ch->status = bad ? PA_ERR_DEVICE_CHECK : PA_OK;
    ch->num_chunks = nch;
    ch->pages_per_chunk = ppc;
    ch->batch_size = batch;
    ch->max_chunks = max_chunks;
    ch->prefix_tokens = nch > 0 ? (n0 - 1) * page_size + lp : 0;
    ch->magic = kCascadeMagic;
    if (bad) set_status(PA_ERR_DEVICE_CHECK);
  }
  decode_plan_block(unique_indptr, unique_last, batch, hkv, hq, head_dim, page_size,
                    num_unique_indices, decode_groups, decode_hb, /*min_per_group=*/4,
                    ws + L.decode);
}

// One warp per (request, q head): log-sum-exp merge of the non-empty level-0
// chunk states (rows c * B + b) and the level-1 state (row b). Base-2 LSEs;
// a state with LSE -inf (no keys) contributes nothing. The chunk LSEs are
// read at once (chunk c in lane c & 31, slot c >> 5), and the state rows in
// batches of kRows independent loads, so the warp waits on memory a few times
// rather than once per chunk.
template <typename T, int D>
__global__ void cascade_merge_kernel(const T* __restrict__ o0, const float* __restrict__ lse0,
                                     const T* __restrict__ o1, const float* __restrict__ lse1,
                                     const CascadeHeader* __restrict__ ch, int batch, int hq,
                                     T* __restrict__ out, float* __restrict__ lse) {
  static_assert(kCascadeMaxChunks <= 64, "two LSE slots per lane");
  griddep_wait();
  griddep_launch_dependents();
  constexpr int PER = D / 32;  // elements per lane
  constexpr int kRows = 8;
  struct alignas(2 * PER) Row { T e[PER]; };
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= batch * hq) return;
  if (ch->magic != kCascadeMagic || ch->batch_size != batch) {
    if (warp == 0 && lane == 0) set_status(PA_ERR_NOT_PLANNED);
    return;
  }
  const int nch = ch->status == PA_OK ? min(ch->num_chunks, kCascadeMaxChunks) : 0;
  const size_t r1 = static_cast<size_t>(warp);          // row b * hq + h
  const size_t step = static_cast<size_t>(batch) * hq;  // rows from chunk c to c + 1
  const float la = lane < nch ? __ldg(lse0 + lane * step + r1) : -INFINITY;
  const float lb = lane + 32 < nch ? __ldg(lse0 + (lane + 32) * step + r1) : -INFINITY;
  const float l1 = __ldg(lse1 + r1);
  float m = fmaxf(la, lb);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  m = fmaxf(m, l1);
  T* orow = out + r1 * D + lane * PER;
  if (m == -INFINITY) {  // no keys at either level
#pragma unroll
    for (int e = 0; e < PER; e += 2) *reinterpret_cast<uint32_t*>(orow + e) = 0u;
    if (lse != nullptr && lane == 0) lse[r1] = -INFINITY;
    return;
  }
  const float wa = la == -INFINITY ? 0.f : ex2(la - m);
  const float wb = lb == -INFINITY ? 0.f : ex2(lb - m);
  const float w1 = l1 == -INFINITY ? 0.f : ex2(l1 - m);
  float w = wa + wb;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
  w += w1;
  float acc[PER];
  {
    const Row v = *reinterpret_cast<const Row*>(o1 + r1 * D + lane * PER);
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = w1 > 0.f ? w1 * static_cast<float>(v.e[e]) : 0.f;
  }
  for (int c0 = 0; c0 < nch; c0 += kRows) {
    Row v[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i)
      if (c0 + i < nch)
        v[i] = *reinterpret_cast<const Row*>(o0 + ((c0 + i) * step + r1) * D + lane * PER);
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int c = c0 + i;
      if (c < nch) {
        const float wt = __shfl_sync(0xffffffffu, c < 32 ? wa : wb, c & 31);
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] = fmaf(wt, static_cast<float>(v[i].e[e]), acc[e]);
      }
    }
  }
  const float inv = 1.f / w;
#pragma unroll
  for (int e = 0; e < PER; e += 2)
    *reinterpret_cast<uint32_t*>(orow + e) = pack2<T>(acc[e] * inv, acc[e + 1] * inv);
  if (lse != nullptr && lane == 0) lse[r1] = m + lg2(w);
}

}  // namespace pa
