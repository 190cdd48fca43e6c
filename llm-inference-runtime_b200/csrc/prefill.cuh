// Ragged / chunked prefill attention over a paged KV cache, sm_100a tcgen05.
//
// Reference behaviour: BatchPrefillWithPagedKVCacheWrapper.forward(q, cache,
// causal=True) as called from src/models/llama.py:212-228 — request b owns q
// rows [qo_indptr[b], qo_indptr[b+1]) and kv_len keys in its pages; with
// causal masking (bottom-right aligned, FlashInfer's convention) query row i
// of a request with qo_len rows sees key j iff j <= i + kv_len - qo_len.
//
// Work item = (request, kv head, two query tiles). The g query heads that
// share a kv head are packed into the 128 rows of a tcgen05 tile (row =
// query * g + head), so every K/V tile loaded serves the whole GQA group, and
// each CTA carries two such tiles so the tensor core always has one tile's
// GEMMs to run while the other tile's softmax is in flight. Per CTA:
//   * warp 8  — TMA producer: both Q tiles once (3-D map over [tokens, heads,
//     dim], 128-byte swizzle), then K and V tiles of 8 pages (128 keys) into
//     separate rings, each page one box per 64-column panel.
//   * warp 9  — tcgen05 issuer (lane 0), per K/V tile j and Q tile t:
//     in order O_t += P_t V_j then S_t(j+1) = Q_t K_{j+1}^T, with
//     P_t read from TMEM (bf16 / fp16 written over S_t's columns) and V from
//     shared memory; completion reported through tcgen05.commit on mbarriers.
//     It never waits on shared memory between MMAs (the tensor pipe queues
//     only a couple of MMAs, so any such wait would idle it): its hand-offs
//     are named barriers.
//   * warps 10 / 11 — relays: wait for each K (warp 10) or V (warp 11) tile's
//     TMA completion and meet the issuer on that tile's named barrier.
//   * warps 0-3 / 4-7 — softmax + epilogue of Q tile 0 / 1, one thread per
//     row (= TMEM lane): causal / length mask, online softmax in base 2 with
//     lazy O rescaling (only when a row's max grows by more than 2^8), P back
//     into TMEM, then a named barrier with the issuer; finally O is
//     normalised and staged in shared memory for TMA stores (tile 0 in a
//     buffer of its own, tile 1 in the V stage of the item's last key tile,
//     which the producer stores before reusing it).
#pragma once

#include "pa_common.cuh"

namespace pa {

// Two non-negative fp32 values -> packed 16-bit pair (lo in the low half).
// Both types: the hardware round-to-nearest-even conversion, one instruction
// per pair.
template <typename T>
__device__ __forceinline__ uint32_t pack_p(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack_p<__nv_bfloat16>(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
template <>
__device__ __forceinline__ uint32_t pack_p<__half>(float lo, float hi) {
  return pack2<__half>(lo, hi);
}

constexpr int kPfRows = 128;  // query rows per tile (MMA M)
constexpr int kPfKeys = 128;  // keys per K/V tile (MMA N of S, K of PV): 8 pages
// Warpgroups 0 / 1 (warps 0-3 / 4-7): softmax + epilogue of Q tile 0 / 1.
// Warpgroup 2: warp 8 TMA producer, warp 9 tcgen05 issuer, warps 10 / 11
// relay K / V TMA completions to the issuer.
// Launched at 168 registers per thread (384 x 168 = 64512 of 65536); after
// setup warpgroup 2 rises to 88 and warpgroups 0-1 to 208:
// 2 x 128 x 208 + 128 x 88 = 64512, exactly the launch total (the producer
// and the issuer carry the persistent loop's item state; at 56 they spilled).
constexpr int kPfSoftmaxThreads = 256;
constexpr int kPfProducerWarp = 8;
constexpr int kPfMmaWarp = 9;
constexpr int kPfRelayWarp = 10;   // K tiles
constexpr int kPfRelayVWarp = 11;  // V tiles
// Named barriers (0 is __syncthreads): P_t written (softmax warpgroup t ->
// issuer warp), K / V tile landed (relay warp -> issuer warp).
constexpr int kPfBarP = 1;  // + t
constexpr int kPfBarK = 3;
constexpr int kPfBarV = 4;
constexpr int kPfBarO = 5;  // warpgroup 0's output rows staged / staging buffer free
constexpr int kPfBarPThreads = 128 + 32;
constexpr int kPfBarKVThreads = 32 + 32;
constexpr int kPfThreads = 384;
constexpr int kPfItemReaders = 11;  // warps reading each work-item slot: 8 softmax, issuer, 2 relays
constexpr uint32_t kPfRegsSoftmax = 208;
constexpr uint32_t kPfRegsOther = 88;
static_assert(2 * 128 * kPfRegsSoftmax + 128 * kPfRegsOther <= kPfThreads * 168,
              "register split must fit the launch allocation");
static_assert(kPfRegsSoftmax % 8 == 0 && kPfRegsOther % 8 == 0 && kPfRegsOther >= 24,
              "setmaxnreg counts are multiples of 8 in [24, 256]");
constexpr float kPfRescaleLog2 = 8.0f;

struct PrefillPlanHeader {
  int32_t magic;
  int32_t status;
  int32_t num_items;
  int32_t batch_size;
  int32_t num_kv_heads;
  int32_t num_qo_heads;
  int32_t head_dim;
  int32_t queries_per_tile;
  int32_t next_item;  // work-item counter of the persistent kernel (zero between launches)
  int32_t ctas_done;  // CTAs that have stopped taking items
  int32_t reserved[6];
};

struct PrefillWsLayout {
  size_t hdr, items, total;
};

__host__ __device__ inline PrefillWsLayout prefill_ws_layout(int64_t max_items) {
  PrefillWsLayout L;
  L.hdr = 0;
  L.items = align256(sizeof(PrefillPlanHeader));
  L.total = align256(L.items + sizeof(int4) * static_cast<size_t>(max_items));
  return L;
}

// Work items for a batch with `total_qo` query rows: one per (request, kv
// head, tile of qt queries); ceil per request adds at most one tile each.
__host__ __device__ inline int64_t prefill_max_items(int batch, int64_t total_qo, int hkv, int qt) {
  return static_cast<int64_t>(hkv) * ((total_qo + qt - 1) / qt + batch);
}

template <int D>
struct PfCfg {
  static constexpr int kPanels = D / 64;
  static constexpr int kStages = D == 128 ? 2 : 4;
  static constexpr int kQBytes = kPfRows * D * 2;      // one Q tile (two are kept)
  static constexpr int kTileBytes = kPfKeys * D * 2;   // one K or V tile
  static constexpr int kPanelBytes = kPfRows * 128;    // 128 rows of 128 bytes
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + 2 * kQBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  // tile 0's output rows, staged for their TMA store (D / 64 panels of 128
  // rows x 128 bytes, the layout of a Q or V tile; tile 1's go to the V
  // stage of the item's last key tile)
  static constexpr int kOffStage = kOffV + kStages * kTileBytes;
  static constexpr int kStageBytes = kPfRows * D * 2;
  static constexpr int kOffBar = kOffStage + kStageBytes;
  // barriers: q_full, s_full[2], o_done[2], mma_done, k_full/k_empty/v_full/v_empty[S],
  // item_full[3], item_empty[3], q_empty, q_full1, q_empty1, o1_staged[S]
  static constexpr int kNumBars = 6 + 4 * kStages + 9 + kStages;
  static constexpr int kOffSlots = kOffBar + kNumBars * 8 + 16;  // three work-item slots
  // per V stage: tile 1 rows to store (int4 entries, 16-byte aligned)
  static constexpr int kOffPend = (kOffSlots + 3 * 64 + 15) / 16 * 16;
  static constexpr int kSmemBytes = kOffPend + kStages * 16 + 1024;
  static_assert(kOffPend % 16 == 0, "int4 entries");
  static_assert(kOffSlots % 8 == 0, "shared-memory alignment");
  static_assert(kOffStage % 1024 == 0, "128-byte swizzled panels start on 1024 bytes");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
  // TMEM columns: S0 | S1 | O0 | O1 (P_t is written over the first half of S_t)
  static constexpr uint32_t kTmemCols = 512;
};

struct PrefillParams {
  void* out;
  float* lse;
  const int32_t* qo_indptr;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_last_page_len;
  int32_t batch_size, num_qo_heads, num_kv_heads, group, qt, causal;
  int64_t num_pages;
  int32_t heads_inner;
  float scale_log2;
  const PrefillPlanHeader* hdr;
  const int4* items;
  int32_t* sched;  // the header's next_item, ctas_done
  // Optional: first q row of request b (default qo_indptr[b]). Lets several
  // requests read the same queries while writing their own output rows —
  // the key chunks of a shared prefix (cascade decode).
  const int32_t* q_rows;
};

// --------------------------------------------------------------------- plan
// One CTA: validates the tables and lists the work items, longest first
// (counting sort on the number of K/V tiles a causal item visits), so the
// hardware's in-order CTA dispatch approximates longest-processing-time.
constexpr int kPfCostBuckets = 1024;
static_assert(kPfCostBuckets == 1024, "the plan runs one thread per bucket, 32 warps");

__global__ void prefill_plan_kernel(const int32_t* __restrict__ qo_indptr,
                                    const int32_t* __restrict__ kv_indptr,
                                    const int32_t* __restrict__ last_len, int batch,
                                    int64_t total_qo, int64_t num_indices, int hq, int hkv,
                                    int head_dim, int page_size, int qt, int64_t max_items,
                                    uint8_t* __restrict__ ws) {
  const PrefillWsLayout L = prefill_ws_layout(max_items);
  PrefillPlanHeader* hdr = reinterpret_cast<PrefillPlanHeader*>(ws + L.hdr);
  int4* items = reinterpret_cast<int4*>(ws + L.items);
  __shared__ int s_err;
  __shared__ int s_count[kPfCostBuckets];
  __shared__ int s_total;
  for (int i = threadIdx.x; i < kPfCostBuckets; i += blockDim.x) s_count[i] = 0;
  if (threadIdx.x == 0) {
    s_err = 0;
    s_total = 0;
  }
  __syncthreads();
  auto kv_len_of = [&](int b) {
    const int n = kv_indptr[b + 1] - kv_indptr[b];
    return n > 0 ? (n - 1) * page_size + last_len[b] : 0;
  };
  auto cost_of = [&](int qo_len, int kv_len, int t0) {
    const int end = min(kv_len, kv_len - qo_len + t0 + qt);
    const int tiles = end > 0 ? (end + kPfKeys - 1) / kPfKeys : 0;
    return min(tiles, kPfCostBuckets - 1);
  };
  // pass 1: validate, histogram of costs
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    const int q0 = qo_indptr[b], q1 = qo_indptr[b + 1];
    const int k0 = kv_indptr[b], k1 = kv_indptr[b + 1];
    bool bad = q1 < q0 || k1 < k0 || q0 < 0 || k0 < 0;
    if (!bad && k1 > k0) {
      const int lp = last_len[b];
      bad = lp < 1 || lp > page_size;
    }
    if (!bad) {
      const int qo_len = q1 - q0, kv_len = kv_len_of(b);
      bad = qo_len > kv_len && qo_len > 0;  // a chunk's own keys are in the cache
      if (!bad) {
        for (int t0 = 0; t0 < qo_len; t0 += qt)
          atomicAdd(&s_count[cost_of(qo_len, kv_len, t0)], hkv);
      }
    }
    if (bad) atomicOr(&s_err, 1);
  }
  if (threadIdx.x == 0) {
    if (qo_indptr[0] != 0 || kv_indptr[0] != 0 || qo_indptr[batch] > total_qo ||
        kv_indptr[batch] > num_indices)
      atomicOr(&s_err, 1);
  }
  __syncthreads();
  // exclusive scan, most expensive bucket first: thread i holds bucket
  // kPfCostBuckets - 1 - i (the launch has one thread per bucket); a
  // shuffle scan per warp, then one over the 32 warp totals
  {
    __shared__ int s_warp[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int c = kPfCostBuckets - 1 - static_cast<int>(threadIdx.x);
    const int n = s_count[c];
    int incl = n;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) s_warp[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      int w = s_warp[lane];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, w, off);
        if (lane >= off) w += v;
      }
      s_warp[lane] = w;  // inclusive prefix over warps 0 .. lane
    }
    __syncthreads();
    const int before = (wid > 0 ? s_warp[wid - 1] : 0) + incl - n;
    s_count[c] = before;
    if (threadIdx.x == kPfCostBuckets - 1) {
      s_total = before + n;
      if (before + n > max_items) s_err = 1;
    }
  }
  __syncthreads();
  const bool err = s_err != 0;
  // pass 2: scatter items into their bucket ranges
  if (!err) {
    for (int b = threadIdx.x; b < batch; b += blockDim.x) {
      const int qo_len = qo_indptr[b + 1] - qo_indptr[b], kv_len = kv_len_of(b);
      for (int t0 = 0; t0 < qo_len; t0 += qt) {
        const int c = cost_of(qo_len, kv_len, t0);
        const int pos = atomicAdd(&s_count[c], hkv);
        for (int h = 0; h < hkv; ++h) items[pos + h] = make_int4(b, h, t0, c);
      }
    }
  }
  if (threadIdx.x == 0) {
    hdr->status = err ? PA_ERR_DEVICE_CHECK : PA_OK;
    hdr->num_items = err ? 0 : s_total;
    hdr->batch_size = batch;
    hdr->num_kv_heads = hkv;
    hdr->num_qo_heads = hq;
    hdr->head_dim = head_dim;
    hdr->queries_per_tile = qt;
    hdr->next_item = 0;
    hdr->ctas_done = 0;
    hdr->magic = kPrefillMagic;
    if (err) set_status(PA_ERR_DEVICE_CHECK);
  }
}

// ---------------------------------------------------------------------- run
// Persistent: one CTA per SM takes work items from the plan's list (longest
// first) through the counter in the plan header. The producer claims one
// item ahead and publishes it (its geometry worked out) in a two-slot ring
// that every other warp reads, so the next item's Q tiles and first K / V
// tiles load while the current item's last steps run, the issuer starts the
// next item's S MMAs right after the current item's last PV (while the
// softmax warps store O), and no CTA launch sits between items. Barrier
// phases run on across items: K / V ring stages by the CTA's running tile
// count, S / O hand-offs by its running step count, Q by its item count.

// One item's geometry, as every warp of the CTA needs it.
struct PfItem {
  int b, h, t0, qo_start, qo_len, q_row0, page0, npages, kv_len, ntiles;  // ntiles < 0: stop
};

__device__ __forceinline__ PfItem pf_item(const PrefillParams& p, int idx) {
  PfItem w;
  if (idx < 0) {
    w = PfItem{0, 0, 0, 0, 0, 0, 0, 0, 0, -1};
    return w;
  }
  const int4 it = p.items[idx];
  w.b = it.x;
  w.h = it.y;
  w.t0 = it.z;
  w.qo_start = __ldg(p.qo_indptr + w.b);
  w.qo_len = __ldg(p.qo_indptr + w.b + 1) - w.qo_start;
  w.q_row0 = p.q_rows != nullptr ? __ldg(p.q_rows + w.b) : w.qo_start;
  w.page0 = __ldg(p.kv_indptr + w.b);
  w.npages = __ldg(p.kv_indptr + w.b + 1) - w.page0;
  w.kv_len = w.npages > 0 ? (w.npages - 1) * kPage + __ldg(p.kv_last_page_len + w.b) : 0;
  // keys this item can see: up to its last query's position (causal) or all
  const int q_hi = min(w.t0 + 2 * p.qt, w.qo_len);
  const int kv_end = p.causal ? min(w.kv_len, w.kv_len - w.qo_len + q_hi) : w.kv_len;
  w.ntiles = kv_end > 0 ? (kv_end + kPfKeys - 1) / kPfKeys : 0;
  return w;
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap,
                   const PrefillParams p) {
  using C = PfCfg<D>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint8_t* sO = smem + C::kOffStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars + 0;  // Q tile 0 landed
  uint64_t* s_full = bars + 1;  // [2] per Q tile
  uint64_t* o_done = bars + 3;    // [2]
  uint64_t* mma_done = bars + 5;  // every MMA of the CTA has completed
  uint64_t* k_full = bars + 6;
  uint64_t* k_empty = k_full + S;
  uint64_t* v_full = k_empty + S;
  uint64_t* v_empty = v_full + S;
  uint64_t* item_full = v_empty + S;   // [3] item slot published
  uint64_t* item_empty = item_full + 3;  // [3] every reader is done with it
  uint64_t* q_empty = item_empty + 3;    // the item's S_0 MMAs are done with Q tile 0
  uint64_t* q_full1 = q_empty + 1;       // Q tile 1 landed
  uint64_t* q_empty1 = q_full1 + 1;      // the item's S_1 MMAs are done with Q tile 1
  uint64_t* o1_staged = q_empty1 + 1;    // [S] tile 1's rows are in V stage s
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
  PfItem* slots = reinterpret_cast<PfItem*>(smem + C::kOffSlots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const PrefillPlanHeader* hdr = p.hdr;
  if (hdr->magic != kPrefillMagic || hdr->batch_size != p.batch_size ||
      hdr->num_kv_heads != p.num_kv_heads || hdr->num_qo_heads != p.num_qo_heads ||
      hdr->head_dim != D || hdr->queries_per_tile != 2 * p.qt) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(PA_ERR_NOT_PLANNED);
    return;
  }
  if (hdr->status != PA_OK) return;
  const int num_items = hdr->num_items;
  const int G = p.group, QT = p.qt, hq = p.num_qo_heads;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    prefetch_tensormap(&omap);
    mbar_init(q_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&o_done[t], 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], kPfItemReaders);
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(mma_done, 1);
    mbar_init(q_empty, 1);
    mbar_init(q_full1, 1);
    mbar_init(q_empty1, 1);
    for (int s = 0; s < S; ++s) mbar_init(&o1_staged[s], 4);
    fence_mbar_init();
  }
  if (warp == kPfMmaWarp) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool failed = false;

  // Work items travel in a three-slot ring: item i in slot i % 3. Readers
  // wait for their item's slot and release it when they are done with the
  // item (the softmax warps after storing O, so they can read the item's
  // fields again there); the producer writes item i + 3 over it.
  auto wait_item = [&](int it) {
    PfItem w;
    if (!mbar_wait_warp(&item_full[it % 3], (it / 3) & 1)) {
      failed = true;
      w = PfItem{0, 0, 0, 0, 0, 0, 0, 0, 0, -1};
    } else {
      w = slots[it % 3];
    }
    return w;
  };
  auto done_item = [&](int it) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&item_empty[it % 3]);
  };
  auto next_item = [&](int it) {
    const PfItem w = wait_item(it);
    done_item(it);
    return w;
  };

  if (warp == kPfProducerWarp) {
    regs_dec<kPfRegsOther>();
    // ------------------------------------------------------------ producer
    auto claim = [&]() {
      int i = -1;
      if (lane == 0 && !failed) {
        i = atomicAdd(&p.sched[0], 1);
        if (i >= num_items) i = -1;
      }
      return __shfl_sync(0xffffffffu, i, 0);
    };
    auto publish = [&](int slot, const PfItem& w) {
      if (lane == 0) {
        slots[slot] = w;
        mbar_arrive(&item_full[slot]);  // release: the slot's contents first
      }
      __syncwarp();
    };
    PfItem w = pf_item(p, claim());
    publish(0, w);
    uint32_t kt = 0;  // K / V tiles loaded so far: ring position
    int qc = 0;       // items whose Q tiles were loaded
    // Tile 1's output rows of an item wait in the V stage of the item's
    // last key tile, which nothing reads again; before this warp loads the
    // next V tile into that stage it stores the rows (once tile 1 has staged
    // them) and lets the store read the stage. pend (shared memory, one
    // entry per stage): staged or written directly, head, first row.
    const uint32_t pend = smem_u32(smem + C::kOffPend);
    uint32_t pend_mask = 0, pend_par = 0;  // stages with rows to store; o1_staged phases
    auto flush_stage = [&](int st) {
      if (!mbar_wait_warp(&o1_staged[st], (pend_par >> st) & 1)) failed = true;
      pend_par ^= 1u << st;
      pend_mask &= ~(1u << st);
      if (lane == 0) {
        const float4 e = ld_shared_f4(pend + st * 16);
        if (__float_as_int(e.x) && !failed) {
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
            tma_store_3d(&omap, sV + st * C::kTileBytes + pn * C::kPanelBytes, pn * 64,
                         __float_as_int(e.y) * G, __float_as_int(e.z));
          bulk_commit();
          bulk_wait_read_all();
        }
      }
      __syncwarp();
    };
    for (int it = 0; w.ntiles >= 0; ++it) {
      // claim and publish item it + 1; its slot was item it - 2's
      const int nxt = claim();
      if (it >= 2 && !mbar_wait_warp(&item_empty[(it + 1) % 3], ((it - 2) / 3) & 1))
        failed = true;
      const PfItem wn = pf_item(p, failed ? -1 : nxt);
      publish((it + 1) % 3, wn);
      const int c1 = p.heads_inner ? w.h : 0, c2 = p.heads_inner ? 0 : w.h;
      if (w.ntiles > 0) {
        // Q tile 0, once the previous item's S_0 MMAs are done with it
        if (qc > 0 && !mbar_wait_warp(q_empty, (qc - 1) & 1)) failed = true;
        ++qc;
        if (lane == 0) {
          mbar_arrive_expect_tx(q_full, C::kQBytes);
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
            tma_load_3d(sQ + pn * C::kPanelBytes, &qmap, q_full, pn * 64, w.h * G,
                        w.q_row0 + w.t0);
        }
      }
      auto load_tile = [&](int j) {
        const uint32_t g = kt + j;
        const int st = g % S, use = g / S;
        const int np = min(8, w.npages - 8 * j);
        int page = 0;
        if (lane < np) {
          page = __ldg(p.kv_indices + w.page0 + 8 * j + lane);
          if (static_cast<unsigned>(page) >= static_cast<unsigned long long>(p.num_pages)) {
            set_status(PA_ERR_DEVICE_CHECK);
            page = 0;
          }
        }
        const uint32_t bytes = static_cast<uint32_t>(np) * C::kPanels * 2048;
        // after a timeout the stages still complete (no bytes expected), so
        // the relays and the issuer keep their rounds without waiting long
        if (use > 0 && !failed && !mbar_wait_warp(&k_empty[st], (use - 1) & 1)) failed = true;
        if (lane == 0) mbar_arrive_expect_tx(&k_full[st], failed ? 0u : bytes);
        __syncwarp();
        if (lane < np && !failed) {
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
            tma_load_4d(sK + st * C::kTileBytes + pn * C::kPanelBytes + lane * 2048, &kmap,
                        &k_full[st], pn * 64, c1, c2, page);
        }
        if (use > 0 && !failed && !mbar_wait_warp(&v_empty[st], (use - 1) & 1)) failed = true;
        if ((pend_mask >> st) & 1) flush_stage(st);
        if (lane == 0) mbar_arrive_expect_tx(&v_full[st], failed ? 0u : bytes);
        __syncwarp();
        if (lane < np && !failed) {
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
            tma_load_4d(sV + st * C::kTileBytes + pn * C::kPanelBytes + lane * 2048, &vmap,
                        &v_full[st], pn * 64, c1, c2, page);
        }
        __syncwarp();
      };
      if (w.ntiles > 0) {
        load_tile(0);
        // Q tile 1, once the previous item's S_1 MMAs are done with it
        if (qc > 1 && !mbar_wait_warp(q_empty1, (qc - 2) & 1)) failed = true;
        if (lane == 0) {
          mbar_arrive_expect_tx(q_full1, C::kQBytes);
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
            tma_load_3d(sQ + C::kQBytes + pn * C::kPanelBytes, &qmap, q_full1, pn * 64, w.h * G,
                        w.q_row0 + w.t0 + QT);
        }
        for (int j = 1; j < w.ntiles; ++j) load_tile(j);
        kt += w.ntiles;
        // tile 1's rows will wait in the last tile's V stage (the rule the
        // softmax warps apply)
        const int st = (kt - 1) % S;
        if (lane == 0)
          st_shared_u4(pend + st * 16, make_uint4(w.t0 + 2 * QT <= w.qo_len ? 1u : 0u, w.h,
                                                  w.qo_start + w.t0 + QT, 0u));
        __syncwarp();
        pend_mask |= 1u << st;
      }
      w = wn;
    }
#pragma unroll 1
    for (int k = 0; k < S; ++k)
      if ((pend_mask >> ((kt + k) % S)) & 1) flush_stage((kt + k) % S);
    if (lane == 0) bulk_wait_all();  // the stores have landed before the grid ends
    if (lane == 0) {
      if (failed) set_status(PA_ERR_TIMEOUT);
      // the last CTA to stop claiming resets the counter for the next launch
      __threadfence();
      if (atomicAdd(&p.sched[1], 1) == static_cast<int>(gridDim.x) - 1) {
        atomicExch(&p.sched[0], 0);
        atomicExch(&p.sched[1], 0);
      }
    }
  } else if (warp == kPfMmaWarp) {
    regs_dec<kPfRegsOther>();
    // ------------------------------------------------------------ tcgen05 issuer
    // The whole warp runs this loop and takes part in the named barriers
    // (hand-offs: P_t from softmax warpgroup t, K / V tiles from the relay
    // warps); lane 0 issues the MMAs. The issuing thread touches no shared
    // memory between MMAs: with only a couple of MMAs queued, a
    // shared-memory wait on this thread would idle the tensor pipe.
    const int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
    const uint32_t idesc_s = umma_idesc_f16(ab, kPfRows, kPfKeys, 0);
    const uint32_t idesc_o = umma_idesc_f16(ab, kPfRows, D, 1);
    // Shared-memory descriptors are formed once: a descriptor's address
    // field is the byte address / 16 (all of shared memory fits its 14
    // bits), so stepping through an operand is one add of a constant.
    // Between hand-offs the issuing thread then runs little more than the
    // MMAs themselves: it shares its sub-partition's issue slots with two
    // softmax warps, and every slot it waits for leaves the tensor pipe's
    // short queue emptier.
    const uint64_t dq0 = umma_desc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t dk0 = umma_desc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = umma_desc_sw128(smem_u32(sV), C::kPanelBytes, 1024);
    constexpr uint64_t kQStep = C::kQBytes >> 4, kTileStep = C::kTileBytes >> 4;
    // S_t = Q_t K_g^T (g: the CTA's running tile count) into TMEM columns
    // [128 t, 128 t + 128); lane 0 only
    auto issue_s = [&](int t, uint32_t g) {
      const uint64_t dq = dq0 + t * kQStep, dk = dk0 + (g % S) * kTileStep;
      const uint32_t d = tmem + t * kPfKeys;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = ((kk >> 2) * C::kPanelBytes + (kk & 3) * 32) >> 4;
        umma_f16(d, dq + off, dk + off, idesc_s, kk > 0 ? 1u : 0u);
      }
      umma_commit(&s_full[t]);
      if (t == 1) umma_commit(&k_empty[g % S]);
    };
    uint32_t kt = 0;
    int qc = 0;
    for (int it = 0;; ++it) {
      const PfItem w = next_item(it);
      if (w.ntiles < 0) break;
      if (w.ntiles == 0) continue;
      const int ntiles = w.ntiles;
      // S_0 as soon as Q tile 0 and the first K tile are in, S_1 once Q tile
      // 1 is in too
      if (!mbar_wait_warp(q_full, qc & 1)) failed = true;
      named_bar_sync(kPfBarK, kPfBarKVThreads);
      if (lane == 0) {
        tc_fence_after();
        issue_s(0, kt);
        if (ntiles == 1) umma_commit(q_empty);
      }
      __syncwarp();
      if (!mbar_wait_warp(q_full1, qc & 1)) failed = true;
      ++qc;
      if (lane == 0) {
        tc_fence_after();
        issue_s(1, kt);
        if (ntiles == 1) umma_commit(q_empty1);
      }
      __syncwarp();
      for (int j = 0; j < ntiles; ++j) {
        const uint32_t g = kt + j;
        const uint64_t dv = dv0 + (g % S) * kTileStep;
        named_bar_sync(kPfBarV, kPfBarKVThreads);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          named_bar_sync(kPfBarP + t, kPfBarPThreads);
          if (t == 0 && j + 1 < ntiles) named_bar_sync(kPfBarK, kPfBarKVThreads);
          if (lane == 0) {
            tc_fence_after();
            // O_t += P_t V_j; P_t: TMEM columns [128 t, 128 t + 64), 16 keys per 8 columns
            const uint32_t d = tmem + 256 + t * D, pa = tmem + t * kPfKeys;
#pragma unroll
            for (int kk = 0; kk < kPfKeys / 16; ++kk) {
              asm volatile(
                  "{\n"
                  "  .reg .pred p;\n"
                  "  setp.ne.b32 p, %4, 0;\n"
                  "  tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
                  "}\n" ::"r"(d),
                  "r"(pa + kk * 8), "l"(dv + ((kk * 2048) >> 4)), "r"(idesc_o),
                  "r"((j > 0 || kk > 0) ? 1u : 0u)
                  : "memory");
            }
            umma_commit(&o_done[t]);
            if (t == 1) umma_commit(&v_empty[g % S]);
            // the next S_t overwrites P_t only after this PV (same thread, in order)
            if (j + 1 < ntiles) {
              issue_s(t, g + 1);
              if (j + 2 == ntiles) umma_commit(t == 0 ? q_empty : q_empty1);  // last S_t
            }
          }
          __syncwarp();
        }
      }
      kt += ntiles;
    }
    // every MMA done before the TMEM is released
    if (lane == 0) umma_commit(mma_done);
    __syncwarp();
    if (!mbar_wait_warp(mma_done, 0)) failed = true;
    if (failed && lane == 0) set_status(PA_ERR_TIMEOUT);
  } else if (warp == kPfRelayWarp || warp == kPfRelayVWarp) {
    regs_dec<kPfRegsOther>();
    // ------------------------------------------------------------ relays
    // Each waits for its tiles' TMA completions (warp 10: K, warp 11: V) and
    // meets the issuer on that tile's named barrier. Separate warps, so a V
    // tile landing late never holds back the hand-off of the next K tile.
    // After a timeout a relay keeps meeting the issuer so no barrier is left
    // short of arrivals.
    const bool is_k = warp == kPfRelayWarp;
    uint64_t* full = is_k ? k_full : v_full;
    const int bar = is_k ? kPfBarK : kPfBarV;
    bool rfail = false;
    uint32_t kt = 0;
    for (int it = 0;; ++it) {
      const PfItem w = next_item(it);
      if (w.ntiles < 0) break;
      for (int j = 0; j < w.ntiles; ++j) {
        const uint32_t g = kt + j;
        if (!rfail && !mbar_wait_warp(&full[g % S], (g / S) & 1)) rfail = true;
        named_bar_sync(bar, kPfBarKVThreads);
      }
      kt += w.ntiles;
    }
    if ((rfail || failed) && lane == 0) set_status(PA_ERR_TIMEOUT);
  } else {
    regs_inc<kPfRegsSoftmax>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;                 // Q tile
    const int r = (warp & 3) * 32 + lane;    // tile row == TMEM lane
    const int qi = t * QT + r / G, gi = r % G;
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_addr + t * kPfKeys;
    const uint32_t tO = tmem + lane_addr + 256 + t * D;
    uint32_t kt = 0;  // running tile count = running step count
    for (int it = 0;; ++it) {
    int ntiles, kv_len, lim;
    {
      const PfItem w = wait_item(it);
      ntiles = w.ntiles;
      kv_len = w.kv_len;
      const int qpos = kv_len - w.qo_len + w.t0 + qi;
      lim = p.causal ? min(qpos + 1, kv_len) : kv_len;
    }
    if (ntiles < 0) {
      done_item(it);
      break;
    }
    float m_used = -INFINITY, l = 0.f;
    float s[kPfKeys];
    // Every step ends with this warpgroup meeting the issuer on the P_t
    // barrier, also after a timeout (the work is skipped then), so every
    // named barrier of the item completes.
    for (int j = 0; j < ntiles; ++j) {
      const uint32_t g = kt + j;
      if (!failed) do {
      if (!mbar_wait_warp(&s_full[t], g & 1)) {
        failed = true;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < kPfKeys / 32; ++c) tmem_ld32(tS + c * 32, s + c * 32);
      tmem_wait_ld();
      const int key0 = j * kPfKeys;
      if (!__all_sync(0xffffffffu, key0 + kPfKeys <= lim)) {
#pragma unroll
        for (int c = 0; c < kPfKeys; ++c)
          if (key0 + c >= lim) s[c] = -INFINITY;
      }
      float mx4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) mx4[e] = s[e];
#pragma unroll
      for (int c = 4; c < kPfKeys; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      const float m_new = fmaxf(m_used, mx);
      const bool need = m_new > m_used + kPfRescaleLog2;
      const float m_old = m_used;
      if (need) m_used = m_new;
      const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
      // P_t as 16-bit pairs, packed in place over s[0..63] and stored over the
      // first 64 columns of S_t in 32-key chunks as they are produced
#pragma unroll
      for (int ch = 0; ch < kPfKeys / 32; ++ch) {
#pragma unroll
        for (int c = 32 * ch; c < 32 * ch + 32; ++c) {
          const float x = fmaf(s[c], p.scale_log2, neg_m);
          s[c] = ex2(x);
          l4[c & 3] += s[c];
        }
#pragma unroll
        for (int e = 16 * ch; e < 16 * ch + 16; ++e)
          s[e] = __uint_as_float(pack_p<T>(s[2 * e], s[2 * e + 1]));
        tmem_st16(tS + 16 * ch, s + 16 * ch);
      }
      // Rows whose max moved rescale O_t (after PV_t of the previous tile).
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        if (!mbar_wait_warp(&o_done[t], (g - 1) & 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const float f = need ? ex2(m_old - m_used) : 1.f;
        float o[32];
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= f;
          tmem_st32(tO + c * 32, o);
        }
        l *= f;
      }
      l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      tmem_wait_st();
      // The last tile may hold keys past kv_len (stale slots, pages never
      // loaded): tile 0's warpgroup zeroes those V rows before its PV, which
      // precedes tile 1's PV on the tensor pipe.
      if (t == 0 && j == ntiles - 1 && key0 + kPfKeys > kv_len) {
        const int st = g % S;
        if (!mbar_wait_warp(&v_full[st], (g / S) & 1)) {
          failed = true;
          break;
        }
        if (key0 + r >= kv_len) {
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(sV + st * C::kTileBytes + pn * C::kPanelBytes + r * 128 +
                                        c * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
      }
      } while (false);
      tc_fence_before();
      // bar.sync, not arrive: the warpgroup meets the issuer once per step
      // and can never run a step ahead of it (it would have nothing to do:
      // the next scores come after this PV).
      named_bar_sync(kPfBarP + t, kPfBarPThreads);
    }
    // ---- epilogue: O_t / l -> out, LSE (the issuer is already running the
    // next item's first S MMAs; its first PV waits for this warpgroup's next
    // P_t hand-off, so O_t is not overwritten before it is read here)
    if (!failed && ntiles > 0) {
      if (!mbar_wait_warp(&o_done[t], (kt + ntiles - 1) & 1)) failed = true;
    }
    // Output rows. Row r of a tile is query r / G, head r % G, and a row
    // per thread makes every warp store touch 32 lines: D / 8 such stores
    // per thread keep the SM's load / store path busy for microseconds at
    // every item end, and the mbarrier polls of the issuer (the next item's
    // Q) and of the softmax warps (its first scores) queue behind them. So
    // both tiles' rows leave through TMA stores (one per 64-column panel:
    // a tile is one 3-D box of the output, 64 dims x G heads x QT queries),
    // staged in shared memory in the Q / V tile layout: tile 0's in a buffer
    // of its own (its thread 0 stores them and checks at the next use that
    // the store has read the buffer), tile 1's in the V stage of the item's
    // last key tile, free once this item's PV_1 MMAs are done (the producer
    // stores them before it loads the next V tile there). A tile that runs
    // past its request's rows (the rows after it belong to the next
    // request) is written directly.
    const PfItem& w = slots[it % 3];  // still this item's: released below
    const bool staged = ntiles > 0 && w.t0 + (t + 1) * QT <= w.qo_len;
    const int vst = (kt + ntiles - 1) % S;  // V stage of the item's last tile
    uint8_t* const stage = t == 0 ? sO : sV + vst * C::kTileBytes;
    if (t == 0 && staged) {
      if (r == 0) bulk_wait_read_all();
      named_bar_sync(kPfBarO, 128);
    }
    if (failed) {
      set_status(PA_ERR_TIMEOUT);
    } else {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = r / G < QT && w.t0 + qi < w.qo_len;
      const size_t row = static_cast<size_t>(w.qo_start + w.t0 + qi) * hq + w.h * G + gi;
      T* orow = reinterpret_cast<T*>(p.out) + row * D;
      const uint32_t srow = smem_u32(stage) + r * 128;
      // 64 of the row's O columns per TMEM round trip (one panel)
#pragma unroll
      for (int pn = 0; pn < C::kPanels; ++pn) {
        float o[64];
        if (ntiles > 0) {
          tmem_ld32(tO + pn * 64, o);
          tmem_ld32(tO + pn * 64 + 32, o + 32);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e) o[e] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 v;
          v.x = pack2<T>(o[8 * c] * inv, o[8 * c + 1] * inv);
          v.y = pack2<T>(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          v.z = pack2<T>(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          v.w = pack2<T>(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          if (staged) {
            // chunk c of row r at chunk c ^ (r % 8): the map's 128-byte swizzle
            st_shared_u4(srow + pn * C::kPanelBytes + ((c ^ (r & 7)) * 16), v);
          } else if (row_ok) {
            *reinterpret_cast<uint4*>(orow + pn * 64 + 8 * c) = v;
          }
        }
      }
      if (staged) fence_proxy_async();
      if (row_ok && p.lse != nullptr) p.lse[row] = l > 0.f ? m_used + lg2(l) : -INFINITY;
    }
    if (t == 1) {
      // every warp reports, staged or not, also after a timeout (the
      // producer holds the stage's next V load until then)
      __syncwarp();
      if (lane == 0 && ntiles > 0) mbar_arrive(&o1_staged[vst]);
    } else if (staged) {
      named_bar_sync(kPfBarO, 128);
      if (r == 0 && !failed) {
#pragma unroll
        for (int pn = 0; pn < C::kPanels; ++pn)
          tma_store_3d(&omap, sO + pn * C::kPanelBytes, pn * 64, w.h * G, w.qo_start + w.t0);
        bulk_commit();
      }
    }
    tc_fence_before();
    done_item(it);
    kt += ntiles;
    }
    // the output stores this thread issued have landed before the grid ends
    if (t == 0 && r == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kPfMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
// Queries per 128-row tile for a GQA group size (rows = queries * group).
inline int prefill_qt(int group) {
  return (group == 1 || group == 2 || group == 4 || group == 8 || group == 16) ? kPfRows / group
                                                                                : 0;
}

// Queries per work item (two tiles).
inline int prefill_span(int group) { return 2 * prefill_qt(group); }

}  // namespace pa
