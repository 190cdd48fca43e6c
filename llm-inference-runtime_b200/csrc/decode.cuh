// Batched paged decode attention for sm_100a.
//
// Reference behaviour: BatchDecodeWithPagedKVCacheWrapper.forward as called
// from src/models/llama.py:230-245 — one query row per request and q head,
// o[b, hq] = softmax(sm_scale * q[b, hq] . K_b,hkv^T) V_b,hkv over the
// request's kv_len = (pages - 1) * P + kv_last_page_len[b] keys, hkv = hq / g.
//
// Design (HBM-bound). A page of the engine's pool holds K then V of every kv
// head contiguously (16 KiB for 4 heads x 64 dims, 64 KiB for 8 x 128), and
// random whole-page reads stream ~15 % faster from HBM3e than the 2 KiB
// per-head pieces a head-at-a-time kernel would issue. So:
//   * A "group" is one warp per kv head of a head block (HB = min(H_kv, 8)
//     heads). The group walks a run of pages; each stage of its shared-memory
//     ring holds one page of the head block — K and V, every panel — fetched
//     by one tiled TMA load per (K|V, 64-column panel) that completes on the
//     stage's mbarrier. Warp h of the group reads head h's rows.
//   * The work stream is every (request b, head block, page j) in that order.
//     decode_plan_kernel cuts it into equal runs of Q pages, one per group, so
//     every group moves the same bytes however skewed the context lengths are
//     (split-KV with no host-side plan).
//   * A stage is refilled by whichever warp of the group releases it last
//     (shared-memory arrival counter). With one head block per page the run
//     is a contiguous slice of kv_indices, read 32 page ids per load a chunk
//     ahead; otherwise a cursor loads each page id one refill ahead. No warp
//     ever blocks on another warp's progress.
//   * The g query heads of a kv head are the rows of one m16n8k16 tile, so a
//     loaded page is shared by the whole GQA group: S = Q K^T (mma.sync, fp32
//     accumulate), online softmax on the S fragments in registers (quad
//     shuffles), O += P V with V read through ldmatrix.trans.
//   * A (request, kv head) segment that straddles runs is written as
//     normalised fp32 partials plus base-2 LSE; the last warp to finish that
//     segment (atomic counter per segment) merges the pieces in the same launch.
//   * Decode-step append (optional): the warp that loads the page holding a
//     request's new token writes that token's K / V row of its head into the
//     pool and over the stale row of the loaded stage, so the step's append
//     costs no launch and no extra read of the page.
#pragma once

#include "pa_common.cuh"

namespace pa {

// Shared memory the decode rings use per CTA (144 KiB at both head sizes:
// 176 / 192 / 208 KiB rings measured no faster on configuration 2 and
// slower on long contexts at head_dim 128), and the stage cap.
__host__ __device__ constexpr int decode_ring_budget(int) { return 144 * 1024; }
constexpr int kDecodeMaxStages = 8;
// Warps per CTA (one per kv head of each group). head_dim 128 pages are
// 4x larger per head, so that kernel keeps 8 warps to fit >= 2 stages
// (head_dim 64: 12 warps; 8 measured slower, 16 no faster).
constexpr int kDecodeWarpsD64 = 12;
constexpr int kDecodeWarpsD128 = 8;

__host__ __device__ constexpr int decode_cta_warps(int head_dim) {
  return head_dim == 64 ? kDecodeWarpsD64 : kDecodeWarpsD128;
}

// Host-side launch geometry of the decode kernel for one cache shape.
struct DecodeGeom {
  int hb;            // kv heads per group (warps per group)
  int nhb;           // head blocks per page
  int groups_per_cta;
  int stages;
  int stage_bytes;   // hb * P * D * 2 (K, V) * 2 B
  int smem_bytes;
  int threads;       // 32 * groups_per_cta * hb
};

__host__ __device__ inline bool decode_geom(int hkv, int head_dim, DecodeGeom* g) {
  if (hkv <= 0 || (head_dim != 64 && head_dim != 128)) return false;
  const int hb = hkv <= 8 ? hkv : 8;
  if (hkv % hb) return false;
  g->hb = hb;
  g->nhb = hkv / hb;
  g->groups_per_cta = decode_cta_warps(head_dim) / hb;
  if (g->groups_per_cta < 1) return false;
  g->stage_bytes = hb * kPage * head_dim * 2 * 2;
  int s = decode_ring_budget(head_dim) / (g->groups_per_cta * g->stage_bytes);
  if (s > kDecodeMaxStages) s = kDecodeMaxStages;
  if (s < 2) return false;
  g->stages = s;
  const int warps = g->groups_per_cta * hb;
  // rings | full mbarriers (8 B) | release counters (4 B) | per-warp walk (2 x (S+1) ints)
  const int aux = g->groups_per_cta * s * 8 + g->groups_per_cta * s * 4 + warps * 2 * (s + 1) * 4;
  g->smem_bytes = g->groups_per_cta * s * g->stage_bytes + ((aux + 15) / 16) * 16 + 1024;
  g->threads = 32 * warps;
  return true;
}

// --------------------------------------------------------------------- plan
// One CTA (every thread calls it). Validates the CSR table, cuts the
// (request, head block, page) stream into runs of Q pages for `num_groups`
// groups, clears the merge counters.
__device__ void decode_plan_block(const int32_t* __restrict__ kv_indptr,
                                  const int32_t* __restrict__ last_len, int batch, int hkv,
                                  int hq, int head_dim, int page_size, int64_t num_indices,
                                  int num_groups, int hb, int min_per_group,
                                  uint8_t* __restrict__ ws) {
  const DecodeWsLayout L = decode_ws_layout(num_groups, batch, hkv, head_dim, hb);
  DecodePlanHeader* hdr = reinterpret_cast<DecodePlanHeader*>(ws + L.hdr);
  int4* unit_start = reinterpret_cast<int4*>(ws + L.unit_start);
  int32_t* empty = reinterpret_cast<int32_t*>(ws + L.empty);
  int32_t* counter = reinterpret_cast<int32_t*>(ws + L.counter);
  const int nhb = hkv / hb;

  __shared__ int s_err;
  __shared__ int s_empty;
  if (threadIdx.x == 0) {
    s_err = 0;
    s_empty = 0;
  }
  __syncthreads();
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    const int s = kv_indptr[b], e = kv_indptr[b + 1];
    bool bad = e < s || s < 0;
    if (!bad && e > s) {
      const int lp = last_len[b];
      bad = lp < 1 || lp > page_size;
    }
    if (bad) atomicOr(&s_err, 1);
    if (e == s) empty[atomicAdd(&s_empty, 1)] = b;
  }
  for (int i = threadIdx.x; i < batch * hkv; i += blockDim.x) counter[i] = 0;
  const int first = kv_indptr[0];
  const long long last_ptr = kv_indptr[batch];
  const long long total_ll = static_cast<long long>(nhb) * last_ptr;
  if (first != 0 || last_ptr > num_indices || total_ll > 0x3fffffffLL) {
    if (threadIdx.x == 0) atomicOr(&s_err, 1);
  }
  __syncthreads();
  const bool err = s_err != 0;
  const int total = err ? 0 : static_cast<int>(total_ll);
  int q = (total + num_groups - 1) / num_groups;
  q = max(q, min_per_group);
  // At most ~8 pieces per (request, head block) segment on average: the
  // warp that merges a split segment reads its pieces two per L2 round
  // trip, so short runs over long segments (32 requests of 256-2048 tokens
  // over 444 groups: 6 pages per run, 12 pieces) cost more in merges than
  // the extra groups gain.
  const int segs = nhb * (batch - s_empty);
  if (!err && segs > 0) q = max(q, (total + 8 * segs - 1) / (8 * segs));
  for (int w = threadIdx.x; w < num_groups; w += blockDim.x) {
    const long long s0 = static_cast<long long>(w) * q;
    int4 st = make_int4(0, 0, 0, 0);
    if (s0 < total) {
      // Largest b with nhb * kv_indptr[b] <= s0; requests without pages are
      // skipped because their start equals the next request's start.
      int lo = 0, hi = batch;  // invariant: nhb*indptr[lo] <= s0 < nhb*indptr[hi]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (static_cast<long long>(nhb) * kv_indptr[mid] <= s0) lo = mid; else hi = mid;
      }
      const int base = kv_indptr[lo];
      const int n = kv_indptr[lo + 1] - base;
      const int off = static_cast<int>(s0 - static_cast<long long>(nhb) * base);
      st = make_int4(lo, off / n, off % n, 0);
    }
    unit_start[w] = st;
  }
  if (threadIdx.x == 0) {
    hdr->status = err ? PA_ERR_DEVICE_CHECK : PA_OK;
    hdr->total = total;
    hdr->per_unit = q;
    hdr->num_units = num_groups;
    hdr->batch_size = batch;
    hdr->num_kv_heads = hkv;
    hdr->num_qo_heads = hq;
    hdr->head_dim = head_dim;
    hdr->page_size = page_size;
    hdr->num_empty = err ? 0 : s_empty;
    hdr->heads_per_unit = hb;
    hdr->magic = kDecodeMagic;
    if (err) set_status(PA_ERR_DEVICE_CHECK);
  }
}

__global__ void decode_plan_kernel(const int32_t* __restrict__ kv_indptr,
                                   const int32_t* __restrict__ last_len, int batch, int hkv,
                                   int hq, int head_dim, int page_size, int64_t num_indices,
                                   int num_groups, int hb, int min_per_group,
                                   uint8_t* __restrict__ ws) {
  griddep_wait();
  griddep_launch_dependents();
  decode_plan_block(kv_indptr, last_len, batch, hkv, hq, head_dim, page_size, num_indices,
                    num_groups, hb, min_per_group, ws);
}

// ---------------------------------------------------------------------- run
// Position in the work stream: request b, head block hblk, page j of n.
struct StreamCursor {
  int b, hblk, j, n, base;
};

__device__ __forceinline__ void cursor_load(StreamCursor& c, const int32_t* indptr) {
  c.base = __ldg(indptr + c.b);
  c.n = __ldg(indptr + c.b + 1) - c.base;
}

// Moves to the next stream position; must only be called when one exists.
__device__ __forceinline__ void cursor_next(StreamCursor& c, const int32_t* indptr, int nhb) {
  if (++c.j < c.n) return;
  c.j = 0;
  if (++c.hblk < nhb) return;
  c.hblk = 0;
  do {
    ++c.b;
    cursor_load(c, indptr);
  } while (c.n == 0);
}

// A split segment (request b, kv head `head`) whose pieces one warp merges.
struct MergeSeg {
  int b, head, seg_start, seg_len;
};

// Log-sum-exp merge of every piece of up to two segments (the two a warp's
// run can end pieces of): o = sum_u 2^(lse_u - max) o_u / sum_u 2^(lse_u -
// max). The G x D outputs are spread over the lanes in float4 granules,
// kItems granules per lane at a time; the LSEs and partial rows of kBatch
// pieces of every granule of both segments are loaded together (online
// max), so merging both segments costs one L2 round trip per kBatch pieces
// rather than one per granule, piece or segment.
template <typename T, int D>
__device__ __noinline__ void merge_segments(const float* part_lse, const float* part_o, T* out,
                                            float* lse, int* counter, int G, int hq, int hkv,
                                            int Q, int HB, int hh, MergeSeg sa, MergeSeg sb,
                                            int nseg, int lane) {
  constexpr int C4 = D / 4;
  constexpr int kItems = 4;
  constexpr int kBatch = 2;
  const int n_items = G * C4;
  const MergeSeg seg[2] = {sa, sb};
  int u0[2], np[2];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    u0[s] = seg[s].seg_start / Q;
    np[s] = s < nseg ? (seg[s].seg_start + seg[s].seg_len - 1) / Q - u0[s] + 1 : 0;
  }
  const int np_max = max(np[0], np[1]);
  for (int it0 = 0; it0 < n_items; it0 += 32 * kItems) {
    float m[2][kItems], w[2][kItems];
    float4 acc[2][kItems];
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int j = 0; j < kItems; ++j) {
        m[s][j] = -INFINITY;
        w[s][j] = 0.f;
        acc[s][j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    for (int ub = 0; ub < np_max; ub += kBatch) {
      float lb[2][kItems][kBatch];
      float4 vb[2][kItems][kBatch];
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
          const int it = it0 + j * 32 + lane;
          const int r = it / C4, c = (it - r * C4) * 4;
#pragma unroll
          for (int k = 0; k < kBatch; ++k) {
            lb[s][j][k] = -INFINITY;
            vb[s][j][k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (it < n_items && ub + k < np[s]) {
              const int uk = u0[s] + ub + k;
              const size_t sl =
                  static_cast<size_t>((uk * 2 + (seg[s].seg_start <= uk * Q ? 0 : 1)) * HB + hh);
              lb[s][j][k] = __ldcg(part_lse + sl * kMaxGroup + r);
              vb[s][j][k] =
                  __ldcg(reinterpret_cast<const float4*>(part_o + (sl * kMaxGroup + r) * D + c));
            }
          }
        }
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int j = 0; j < kItems; ++j)
#pragma unroll
          for (int k = 0; k < kBatch; ++k) {
            if (ub + k >= np[s]) break;
            const float mn = fmaxf(m[s][j], lb[s][j][k]);
            const float sc = ex2(m[s][j] - mn), wt = ex2(lb[s][j][k] - mn);
            acc[s][j].x = acc[s][j].x * sc + wt * vb[s][j][k].x;
            acc[s][j].y = acc[s][j].y * sc + wt * vb[s][j][k].y;
            acc[s][j].z = acc[s][j].z * sc + wt * vb[s][j][k].z;
            acc[s][j].w = acc[s][j].w * sc + wt * vb[s][j][k].w;
            w[s][j] = w[s][j] * sc + wt;
            m[s][j] = mn;
          }
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (s >= nseg) break;
      T* ob = out + (static_cast<size_t>(seg[s].b) * hq + seg[s].head * G) * D;
#pragma unroll
      for (int j = 0; j < kItems; ++j) {
        const int it = it0 + j * 32 + lane;
        if (it >= n_items) continue;
        const int r = it / C4, c = (it - r * C4) * 4;
        const float inv = 1.f / w[s][j];
        uint2 packed;
        packed.x = pack2<T>(acc[s][j].x * inv, acc[s][j].y * inv);
        packed.y = pack2<T>(acc[s][j].z * inv, acc[s][j].w * inv);
        *reinterpret_cast<uint2*>(ob + r * D + c) = packed;
        if (lse != nullptr && c == 0)
          lse[static_cast<size_t>(seg[s].b) * hq + seg[s].head * G + r] = m[s][j] + lg2(w[s][j]);
      }
    }
  }
  __syncwarp();
  if (lane == 0)  // ready for the next launch
    for (int s = 0; s < nseg; ++s) counter[seg[s].b * hkv + seg[s].head] = 0;
}

template <typename T, int D>
__global__ void __launch_bounds__(decode_cta_warps(D) * 32, 1)
    decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const DecodeParams p) {
  constexpr int NT = D / 8;       // 8-wide column tiles of O
  constexpr int KS = D / 16;      // 16-deep k steps of Q K^T
  constexpr int PANELS = D / 64;  // 128-byte swizzle panels per row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);

  const int HB = p.hb, NHB = p.nhb, S = p.stages, SB = p.stage_bytes, GPC = p.groups_per_cta;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int nwarps = GPC * HB;
  const int g_local = warp / HB, hh = warp - g_local * HB;
  const int num_groups = gridDim.x * GPC;
  const int grp = blockIdx.x * GPC + g_local;
  const int gw = blockIdx.x * nwarps + warp;  // global warp id
  const int total_warps = gridDim.x * nwarps;
  const DecodePlanHeader* hdr = p.hdr;

  // Shared memory: rings, full barriers, release counters, per-warp walk.
  uint8_t* rings = smem;
  uint64_t* fullb = reinterpret_cast<uint64_t*>(rings + GPC * S * SB);
  int* relc = reinterpret_cast<int*>(fullb + GPC * S);
  int* walk_all = relc + GPC * S;
  if (threadIdx.x == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < GPC * S; ++s) {
      mbar_init(&fullb[s], 1);
      relc[s] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  // everything above is private to this CTA; from here on the plan and the
  // pool (which the previous kernel may have written) are read
  griddep_wait();
  // this group's start, loaded alongside the header (the workspace is sized
  // for this grid, so the load is in bounds whatever the header holds)
  const int4 st = p.unit_start[grp];

  if (hdr->magic != kDecodeMagic || hdr->num_units != num_groups ||
      hdr->batch_size != p.batch_size || hdr->num_kv_heads != p.num_kv_heads ||
      hdr->num_qo_heads != p.num_qo_heads || hdr->head_dim != D || hdr->heads_per_unit != HB) {
    if (gw == 0 && lane == 0) set_status(PA_ERR_NOT_PLANNED);
    return;
  }
  if (hdr->status != PA_OK) return;
  const int Q = hdr->per_unit, total = hdr->total, hkv = p.num_kv_heads, G = p.group;
  const int hq = p.num_qo_heads;
  T* out = reinterpret_cast<T*>(p.out);

  // Requests without pages produce zeros (and LSE = -inf); none can take an
  // appended token.
  for (int e = gw; e < hdr->num_empty; e += total_warps) {
    const int b = p.empty[e];
    if (p.append_pos != nullptr && lane == 0) set_status(PA_ERR_DEVICE_CHECK);
    for (int i = lane; i < hq * D / 8; i += 32)
      reinterpret_cast<uint4*>(out + static_cast<size_t>(b) * hq * D)[i] = make_uint4(0, 0, 0, 0);
    if (p.lse != nullptr)
      for (int i = lane; i < hq; i += 32) p.lse[static_cast<size_t>(b) * hq + i] = -INFINITY;
  }

  const int s0 = grp * Q;
  if (s0 >= total) return;
  const int cnt = min(Q, total - s0);

  uint8_t* ring = rings + g_local * S * SB;
  uint64_t* bars = fullb + g_local * S;
  int* rel = relc + g_local * S;
  int* walk = walk_all + warp * 2 * (S + 1);

  StreamCursor pc;
  pc.b = st.x;
  pc.hblk = st.y;
  pc.j = st.z;
  cursor_load(pc, p.kv_indptr);
  StreamCursor cc = pc;
  const int panel_bytes = HB * 2048;

  // K/V pages are read once per launch: first to leave L2.
  const uint64_t evict_first = l2_evict_first_policy();
  // Fills stage `stage` with page `page` of head block `hblk` (one thread).
  auto issue = [&](int stage, int page, int hblk) {
    if (static_cast<unsigned>(page) >= static_cast<unsigned long long>(p.num_pages)) {
      set_status(PA_ERR_DEVICE_CHECK);
      page = 0;
    }
    uint8_t* dst = ring + stage * SB;
    mbar_arrive_expect_tx(&bars[stage], SB);
    const int h0 = hblk * HB;
    const int c1 = p.heads_inner ? h0 : 0, c2 = p.heads_inner ? 0 : h0;
#pragma unroll
    for (int pn = 0; pn < PANELS; ++pn) {
      tma_load_4d_hint(dst + pn * panel_bytes, &kmap, &bars[stage], pn * 64, c1, c2, page,
                       evict_first);
      tma_load_4d_hint(dst + (PANELS + pn) * panel_bytes, &vmap, &bars[stage], pn * 64, c1, c2,
                       page, evict_first);
    }
  };

  // Prologue: every warp of the group walks the first min(S + 1, cnt)
  // positions (one page-id round trip, lane-parallel); warp 0 of the group
  // fills the ring. Position S, if any, is the first refill: its id is kept
  // in pf_page so each refill issues with an id loaded one iteration early.
  //
  // With one head block per page (H_kv <= 8) run position k is simply
  // kv_indices[s0 + k]: the page ids are then read lane-parallel, 32 per
  // load (chunk c of the run: position 32 c + lane), one chunk ahead of the
  // refills that use them, so no dependent global load sits between two
  // refills. pg_a holds chunk ca, pg_b chunk ca + 1.
  const bool flat = NHB == 1;
  auto chunk_ids = [&](int c) {
    const int k = 32 * c + lane;
    return k < cnt ? __ldg(p.kv_indices + s0 + k) : 0;
  };
  int pg_a = 0, pg_b = 0, ca = 0;
  const int npro = min(S, cnt);
  const int nwalk = min(S + 1, cnt);
  int my_page = 0, my_hb = 0;
  if (flat) {
    pg_a = chunk_ids(0);
    pg_b = chunk_ids(1);
    my_page = pg_a;  // positions 0 .. S < 32 are all in chunk 0
  } else {
    if (lane == 0) {
      for (int k = 0; k < nwalk; ++k) {
        if (k > 0) cursor_next(pc, p.kv_indptr, NHB);
        walk[k] = pc.base + pc.j;
        walk[S + 1 + k] = pc.hblk;
      }
    }
    __syncwarp();
    if (lane < nwalk) {
      my_page = __ldg(p.kv_indices + walk[lane]);
      my_hb = walk[S + 1 + lane];
    }
  }
  int pf_page = __shfl_sync(0xffffffffu, my_page, npro < cnt ? npro : 0);
  int pf_hb = __shfl_sync(0xffffffffu, my_hb, npro < cnt ? npro : 0);
  for (int k = 0; k < npro; ++k) {
    const int pg = __shfl_sync(0xffffffffu, my_page, k);
    const int hbk = __shfl_sync(0xffffffffu, my_hb, k);
    if (hh == 0 && lane == 0) issue(k, pg, hbk);
  }

  const T* qbase = reinterpret_cast<const T*>(p.q);
  uint32_t qf[KS][4];
  float o[NT][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  int seg_start = 0, last_len = kPage, head = 0, apos = -1;
  const bool row0 = gid < G, row1 = gid + 8 < G;
  // Row of token r of this warp's head inside a panel of the stage.
  const int row_mul = p.heads_inner ? HB : 1;
  const int row_add = p.heads_inner ? hh : hh * kPage;

  // Split segments whose piece this warp wrote (at most the first and the
  // last segment of its run); counted and merged after the loop.
  int n_pend = 0;
  int pend_b[2] = {0, 0}, pend_head[2] = {0, 0}, pend_seg[2] = {0, 0}, pend_len[2] = {0, 0};

  int stage = 0;
  uint32_t phase = 0;
  for (int i = 0; i < cnt; ++i) {
    if (i == 0 || cc.j == 0) {
      // New (request, kv head) segment: load the group's q rows as A fragments.
      head = cc.hblk * HB + hh;
      const T* qh = qbase + static_cast<int64_t>(cc.b) * p.q_stride_n +
                    static_cast<int64_t>(head * G) * p.q_stride_h;
      const T* q0 = qh + static_cast<int64_t>(gid) * p.q_stride_h;
      const T* q1 = qh + static_cast<int64_t>(gid + 8) * p.q_stride_h;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int c = kk * 16 + 2 * tig;
        qf[kk][0] = row0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + c)) : 0u;
        qf[kk][1] = row1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + c)) : 0u;
        qf[kk][2] = row0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + c + 8)) : 0u;
        qf[kk][3] = row1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + c + 8)) : 0u;
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
      seg_start = NHB * cc.base + cc.hblk * cc.n;
      last_len = __ldg(p.kv_last_page_len + cc.b);
      if (p.append_pos != nullptr) {
        // the same rule as pa_append_paged_kv_cache: the position must fall
        // inside the request's pages
        apos = __ldg(p.append_pos + cc.b);
        if (p.append_pos_base != nullptr) apos -= __ldg(p.append_pos_base);
        if (apos < 0 || apos / kPage >= cc.n) {
          if (lane == 0) set_status(PA_ERR_DEVICE_CHECK);
          apos = -1;
        }
      }
    }

    if (!mbar_wait(&bars[stage], phase)) {
      set_status(PA_ERR_TIMEOUT);
      return;
    }
    uint8_t* kst = ring + stage * SB;
    const uint32_t kb = smem_u32(kst);
    const uint32_t vb = kb + PANELS * panel_bytes;
    const int valid = (cc.j == cc.n - 1) ? last_len : kPage;

    // ---- decode-step append: this page holds the request's new token
    if (apos >= 0 && cc.j == apos / kPage) {
      constexpr int CH = D / 8;  // 16-byte chunks per row: lanes [0, CH) K, [CH, 2 CH) V
      const int slot = apos % kPage;
      const int page = __ldg(p.kv_indices + cc.base + cc.j);
      if (lane < 2 * CH) {
        const int kv = lane / CH, c = lane - kv * CH;
        const uint8_t* src = kv ? p.new_v + cc.b * p.new_v_stride_n + head * p.new_v_stride_h
                                : p.new_k + cc.b * p.new_k_stride_n + head * p.new_k_stride_h;
        const uint4 val = __ldg(reinterpret_cast<const uint4*>(src) + c);
        if (page >= 0 && page < p.num_pages) {
          uint8_t* dst = (kv ? p.v_pool : p.k_pool) + page * p.pool_page_stride +
                         head * p.pool_head_stride + slot * p.pool_token_stride;
          reinterpret_cast<uint4*>(dst)[c] = val;
        }
        // the loaded stage still holds the slot's old bytes
        *reinterpret_cast<uint4*>(kst + (kv * PANELS + (c >> 3)) * panel_bytes +
                                  sw128(slot * row_mul + row_add, c & 7)) = val;
        fence_proxy_async();  // before the stage is refilled by TMA
      }
      __syncwarp();
    }

    // ---- S = Q K^T over the 16 keys of this page
    float s[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
    {
      const int krow = ((lane & 7) + ((lane >> 4) & 1) * 8) * row_mul + row_add;
      const int khalf = (lane >> 3) & 1;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int panel = kk >> 2;
        const int chunk = ((kk & 3) << 1) + khalf;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + panel * panel_bytes + sw128(krow, chunk), b0, b1, b2, b3);
        Mma16816<T>::run(s[0], qf[kk], b0, b1);
        Mma16816<T>::run(s[1], qf[kk], b2, b3);
      }
    }

    // ---- online softmax (base 2), rows gid and gid + 8
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = t * 8 + 2 * tig + (e & 1);
        s[t][e] = key < valid ? s[t][e] * p.scale_log2 : -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[t][0], s[t][1]));
      mx1 = fmaxf(mx1, fmaxf(s[t][2], s[t][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = ex2(m0 - mn0), c1 = ex2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float pr[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      pr[t][0] = ex2(s[t][0] - mn0);
      pr[t][1] = ex2(s[t][1] - mn0);
      pr[t][2] = ex2(s[t][2] - mn1);
      pr[t][3] = ex2(s[t][3] - mn1);
    }
    l0 = l0 * c0 + (pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1]);
    l1 = l1 * c1 + (pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3]);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      o[nt][0] *= c0;
      o[nt][1] *= c0;
      o[nt][2] *= c1;
      o[nt][3] *= c1;
    }
    uint32_t pa[4];
    pa[0] = pack2<T>(pr[0][0], pr[0][1]);
    pa[1] = pack2<T>(pr[0][2], pr[0][3]);
    pa[2] = pack2<T>(pr[1][0], pr[1][1]);
    pa[3] = pack2<T>(pr[1][2], pr[1][3]);

    // Slots past the last key hold stale pool bytes; zero this head's V rows
    // there so a non-finite value cannot reach O through 0 * Inf.
    if (valid < kPage) {
      uint8_t* vst = kst + PANELS * panel_bytes;
      for (int idx = lane; idx < (kPage - valid) * PANELS * 8; idx += 32) {
        const int r = valid + idx / (PANELS * 8);
        const int rem = idx % (PANELS * 8);
        *reinterpret_cast<uint4*>(vst + (rem >> 3) * panel_bytes + (r * row_mul + row_add) * 128 +
                                  (rem & 7) * 16) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async();
      __syncwarp();
    }

    // ---- O += P V
    {
      const int vrow = ((lane & 7) + ((lane >> 3) & 1) * 8) * row_mul + row_add;
      const int vhalf = lane >> 4;
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        const int panel = np >> 2;
        const int chunk = ((np & 3) << 1) + vhalf;
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vb + panel * panel_bytes + sw128(vrow, chunk), v0, v1, v2, v3);
        Mma16816<T>::run(o[2 * np], pa, v0, v1);
        Mma16816<T>::run(o[2 * np + 1], pa, v2, v3);
      }
    }
    __syncwarp();

    // Release the stage. The last warp of the group to release it refills it
    // with the page S positions ahead. Flat runs take that page id from the
    // chunk registers (every warp keeps its own copy in step); otherwise
    // every warp moves its copy of the refill cursor and loads the next page
    // id (used next iteration).
    const int kr = i + S;
    int rpage = pf_page;
    if (flat) {
      if ((kr >> 5) > ca) {
        pg_a = pg_b;
        ++ca;
        pg_b = chunk_ids(ca + 1);
      }
      rpage = __shfl_sync(0xffffffffu, pg_a, kr & 31);
    }
    if (lane == 0) {
      __threadfence_block();
      const int old = atomicAdd(&rel[stage], 1);
      if ((old + 1) % HB == 0 && kr < cnt) {
        __threadfence_block();
        issue(stage, rpage, flat ? 0 : pf_hb);
      }
      if (!flat && kr + 1 < cnt) {
        cursor_next(pc, p.kv_indptr, NHB);
        pf_page = __ldg(p.kv_indices + pc.base + pc.j);
        pf_hb = pc.hblk;
      }
    }

    // ---- end of this warp's piece of the segment
    if (cc.j == cc.n - 1 || i == cnt - 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      const float inv0 = 1.f / l0, inv1 = 1.f / l1;
      const int seg_end = seg_start + cc.n;
      const bool split = seg_start < s0 || seg_end > s0 + cnt;
      const int head0 = head * G;
      if (!split) {
        T* ob = out + (static_cast<size_t>(cc.b) * hq + head0) * D;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int d = nt * 8 + 2 * tig;
          if (row0)
            *reinterpret_cast<uint32_t*>(ob + gid * D + d) =
                pack2<T>(o[nt][0] * inv0, o[nt][1] * inv0);
          if (row1)
            *reinterpret_cast<uint32_t*>(ob + (gid + 8) * D + d) =
                pack2<T>(o[nt][2] * inv1, o[nt][3] * inv1);
        }
        if (p.lse != nullptr && tig == 0) {
          float* lb = p.lse + static_cast<size_t>(cc.b) * hq + head0;
          if (row0) lb[gid] = m0 + lg2(l0);
          if (row1) lb[gid + 8] = m1 + lg2(l1);
        }
      } else {
        const int slot = ((grp * 2 + (seg_start <= s0 ? 0 : 1)) * HB) + hh;
        float* po = p.part_o + static_cast<size_t>(slot) * kMaxGroup * D;
        float* pl = p.part_lse + static_cast<size_t>(slot) * kMaxGroup;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int d = nt * 8 + 2 * tig;
          if (row0) __stcg(reinterpret_cast<float2*>(po + gid * D + d),
                           make_float2(o[nt][0] * inv0, o[nt][1] * inv0));
          if (row1) __stcg(reinterpret_cast<float2*>(po + (gid + 8) * D + d),
                           make_float2(o[nt][2] * inv1, o[nt][3] * inv1));
        }
        if (tig == 0) {
          if (row0) __stcg(pl + gid, m0 + lg2(l0));
          if (row1) __stcg(pl + gid + 8, m1 + lg2(l1));
        }
        // Counted (and merged, if this piece turns out to be the last one)
        // after the main loop, so no fence or atomic stalls this group's ring.
        if (n_pend < 2) {
          pend_b[n_pend] = cc.b;
          pend_head[n_pend] = head;
          pend_seg[n_pend] = seg_start;
          pend_len[n_pend] = cc.n;
          ++n_pend;
        }
      }
    }

    if (i + 1 < cnt) cursor_next(cc, p.kv_indptr, NHB);
    if (++stage == S) {
      stage = 0;
      phase ^= 1;
    }
  }

  // the next kernel in the stream may start its prologue (it waits for this
  // grid's completion before reading anything)
  griddep_launch_dependents();

  if (n_pend > 0) {
    // Publish this warp's partials, then count its pieces (both counts in
    // flight together); the warp that completes a segment's count merges it,
    // both segments in one pass when it completes both.
    __threadfence();
    __syncwarp();
    int old0 = 0, old1 = 0;
    if (lane == 0) {
      old0 = atomicAdd(p.counter + pend_b[0] * hkv + pend_head[0], 1);
      if (n_pend > 1) old1 = atomicAdd(p.counter + pend_b[1] * hkv + pend_head[1], 1);
    }
    old0 = __shfl_sync(0xffffffffu, old0, 0);
    old1 = __shfl_sync(0xffffffffu, old1, 0);
    const bool last0 = old0 == (pend_seg[0] + pend_len[0] - 1) / Q - pend_seg[0] / Q;
    const bool last1 = n_pend > 1 && old1 == (pend_seg[1] + pend_len[1] - 1) / Q - pend_seg[1] / Q;
    if (last0 || last1) {
      const MergeSeg s0{pend_b[0], pend_head[0], pend_seg[0], pend_len[0]};
      const MergeSeg s1{pend_b[1], pend_head[1], pend_seg[1], pend_len[1]};
      __threadfence();
      merge_segments<T, D>(p.part_lse, p.part_o, out, p.lse, p.counter, G, hq, hkv, Q, HB, hh,
                           last0 ? s0 : s1, s1, last0 && last1 ? 2 : 1, lane);
    }
  }
}

}  // namespace pa
