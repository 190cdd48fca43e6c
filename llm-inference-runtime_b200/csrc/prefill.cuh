// Ragged / chunked prefill attention over a paged KV cache, sm_100a tcgen05.
//
// Reference behaviour: BatchPrefillWithPagedKVCacheWrapper.forward(q, cache,
// causal=True) as called from src/models/llama.py:212-228 — request b owns q
// rows [qo_indptr[b], qo_indptr[b+1]) and kv_len keys in its pages; with
// causal masking (bottom-right aligned, FlashInfer's convention) query row i
// of a request with qo_len rows sees key j iff j <= i + kv_len - qo_len.
//
// Work item = (request, kv head, query tile). The g query heads that share a
// kv head are packed into the 128 rows of one tcgen05 tile (row = query * g +
// head), so every K/V tile loaded serves the whole GQA group. Per CTA:
//   * warp 4  — TMA producer: the Q tile once (3-D map over [tokens, heads,
//     dim], 128-byte swizzle), then K and V tiles of 8 pages (128 keys) into
//     separate rings, each page one box per 64-column panel.
//   * warp 5  — tcgen05 issuer (one thread): S_j = Q K_j^T into one of two
//     TMEM S buffers, O += P_j V_j into a TMEM accumulator (fp32), completion
//     reported through tcgen05.commit on mbarriers.
//   * warps 0-3 — softmax / epilogue warpgroup, thread = row = TMEM lane:
//     loads its S row, applies the causal / length mask and an online softmax
//     in base 2 with lazy O rescaling (only when the running max grows by more
//     than 2^8), writes P (bf16 / fp16) into a 128B-swizzled shared tile for
//     the PV MMA, and finally normalises O and stores it.
#pragma once

#include "pa_common.cuh"

namespace pa {

constexpr int kPfRows = 128;  // query rows per tile (MMA M)
constexpr int kPfKeys = 128;  // keys per K/V tile (MMA N of S, K of PV): 8 pages
constexpr int kPfThreads = 192;
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
  int32_t reserved[8];
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
  static constexpr int kQBytes = kPfRows * D * 2;
  static constexpr int kTileBytes = kPfKeys * D * 2;  // one K or V tile
  static constexpr int kPBytes = kPfRows * kPfKeys * 2;
  static constexpr int kPanelBytes = kPfRows * 128;    // 128 rows of 128 bytes
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffP = kOffV + kStages * kTileBytes;
  static constexpr int kOffBar = kOffP + kPBytes;
  // barriers: q_full, s_full[2], p_full, o_done, k_full/k_empty/v_full/v_empty[S]
  static constexpr int kNumBars = 5 + 4 * kStages;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;  // S0 | S1 | O
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
};

// --------------------------------------------------------------------- plan
// One CTA: validates the tables and lists the work items, longest first
// (counting sort on the number of K/V tiles a causal item visits), so the
// hardware's in-order CTA dispatch approximates longest-processing-time.
constexpr int kPfCostBuckets = 1024;

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
  // exclusive scan, most expensive bucket first (one thread; 1024 entries)
  if (threadIdx.x == 0) {
    int run = 0;
    for (int c = kPfCostBuckets - 1; c >= 0; --c) {
      const int n = s_count[c];
      s_count[c] = run;
      run += n;
    }
    s_total = run;
    if (run > max_items) s_err = 1;
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
    hdr->magic = kPrefillMagic;
    if (err) set_status(PA_ERR_DEVICE_CHECK);
  }
}

// ---------------------------------------------------------------------- run
template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  using C = PfCfg<D>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint8_t* sP = smem + C::kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* s_full = bars + 1;  // [2]
  uint64_t* p_full = bars + 3;
  uint64_t* o_done = bars + 4;
  uint64_t* k_full = bars + 5;
  uint64_t* k_empty = k_full + S;
  uint64_t* v_full = k_empty + S;
  uint64_t* v_empty = v_full + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const PrefillPlanHeader* hdr = p.hdr;
  if (hdr->magic != kPrefillMagic || hdr->batch_size != p.batch_size ||
      hdr->num_kv_heads != p.num_kv_heads || hdr->num_qo_heads != p.num_qo_heads ||
      hdr->head_dim != D || hdr->queries_per_tile != p.qt) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(PA_ERR_NOT_PLANNED);
    return;
  }
  if (hdr->status != PA_OK || static_cast<int>(blockIdx.x) >= hdr->num_items) return;

  const int4 item = p.items[blockIdx.x];
  const int b = item.x, h = item.y, t0 = item.z;
  const int G = p.group, QT = p.qt, hq = p.num_qo_heads;
  const int qo_start = __ldg(p.qo_indptr + b);
  const int qo_len = __ldg(p.qo_indptr + b + 1) - qo_start;
  const int page0 = __ldg(p.kv_indptr + b);
  const int npages = __ldg(p.kv_indptr + b + 1) - page0;
  const int kv_len = npages > 0 ? (npages - 1) * kPage + __ldg(p.kv_last_page_len + b) : 0;
  // keys this tile can see: up to the last query's position (causal) or all
  const int q_hi = min(t0 + QT, qo_len);
  const int kv_end = p.causal ? min(kv_len, kv_len - qo_len + q_hi) : kv_len;
  const int ntiles = kv_end > 0 ? (kv_end + kPfKeys - 1) / kPfKeys : 0;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    mbar_init(q_full, 1);
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS0 = tmem, tO = tmem + 256;
  bool failed = false;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    const int c1 = p.heads_inner ? h : 0, c2 = p.heads_inner ? 0 : h;
    if (lane == 0 && ntiles > 0) {
      mbar_arrive_expect_tx(q_full, C::kQBytes);
#pragma unroll
      for (int pn = 0; pn < C::kPanels; ++pn)
        tma_load_3d(sQ + pn * C::kPanelBytes, &qmap, q_full, pn * 64, h * G, qo_start + t0);
    }
    for (int j = 0; j < ntiles && !failed; ++j) {
      const int st = j % S, use = j / S;
      const int np = min(8, npages - 8 * j);
      int page = 0;
      if (lane < np) {
        page = __ldg(p.kv_indices + page0 + 8 * j + lane);
        if (static_cast<unsigned>(page) >= static_cast<unsigned long long>(p.num_pages)) {
          set_status(PA_ERR_DEVICE_CHECK);
          page = 0;
        }
      }
      const uint32_t bytes = static_cast<uint32_t>(np) * C::kPanels * 2048;
      // K tile j
      if (use > 0 && !mbar_wait(&k_empty[st], (use - 1) & 1)) failed = true;
      if (!failed) {
        if (lane == 0) mbar_arrive_expect_tx(&k_full[st], bytes);
        __syncwarp();
        if (lane < np) {
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
            tma_load_4d(sK + st * C::kTileBytes + pn * C::kPanelBytes + lane * 2048, &kmap,
                        &k_full[st], pn * 64, c1, c2, page);
        }
      }
      // V tile j
      if (!failed && use > 0 && !mbar_wait(&v_empty[st], (use - 1) & 1)) failed = true;
      if (!failed) {
        if (lane == 0) mbar_arrive_expect_tx(&v_full[st], bytes);
        __syncwarp();
        if (lane < np) {
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn)
            tma_load_4d(sV + st * C::kTileBytes + pn * C::kPanelBytes + lane * 2048, &vmap,
                        &v_full[st], pn * 64, c1, c2, page);
        }
      }
      __syncwarp();
    }
    if (failed && lane == 0) set_status(PA_ERR_TIMEOUT);
  } else if (warp == 5) {
    // ------------------------------------------------------------ tcgen05 issuer
    if (lane == 0 && ntiles > 0) {
      const int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t idesc_s = umma_idesc_f16(ab, kPfRows, kPfKeys, 0);
      const uint32_t idesc_o = umma_idesc_f16(ab, kPfRows, D, 1);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV),
                     p_base = smem_u32(sP);
      if (!mbar_wait(q_full, 0)) failed = true;
      auto issue_s = [&](int j) {
        const int st = j % S;
        if (!mbar_wait(&k_full[st], (j / S) & 1)) {
          failed = true;
          return;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::kPanelBytes + (kk & 3) * 32;
          umma_f16(tS0 + (j & 1) * kPfKeys, umma_desc_sw128(q_base + off, 16, 1024),
                   umma_desc_sw128(k_base + st * C::kTileBytes + off, 16, 1024), idesc_s,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[st]);
        umma_commit(&s_full[j & 1]);
      };
      if (!failed) issue_s(0);
      if (!failed && ntiles > 1) issue_s(1);
      for (int j = 0; j < ntiles && !failed; ++j) {
        const int st = j % S;
        if (!mbar_wait(p_full, j & 1) || !mbar_wait(&v_full[st], (j / S) & 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kPfKeys / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * C::kPanelBytes + (kk & 3) * 32;
          umma_f16(tO, umma_desc_sw128(p_base + poff, 16, 1024),
                   umma_desc_sw128(v_base + st * C::kTileBytes + kk * 2048, C::kPanelBytes, 1024),
                   idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[st]);
        umma_commit(o_done);
        if (j + 2 < ntiles) issue_s(j + 2);
      }
      if (failed) set_status(PA_ERR_TIMEOUT);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int r = threadIdx.x;  // tile row == TMEM lane
    const int qi = r / G, gi = r - qi * G;
    const bool row_ok = qi < QT && t0 + qi < qo_len;
    const int qpos = kv_len - qo_len + t0 + qi;
    const int lim = p.causal ? min(qpos + 1, kv_len) : kv_len;
    const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    float s[kPfKeys];
    for (int j = 0; j < ntiles; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1)) {
        failed = true;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < kPfKeys / 32; ++c)
        tmem_ld32(tS0 + lane_addr + (j & 1) * kPfKeys + c * 32, s + c * 32);
      tmem_wait_ld();
      const int key0 = j * kPfKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kPfKeys; ++c) {
        const float v = key0 + c < lim ? s[c] * p.scale_log2 : -INFINITY;
        s[c] = v;
        mx = fmaxf(mx, v);
      }
      const float m_new = fmaxf(m_used, mx);
      const bool need = m_new > m_used + kPfRescaleLog2;
      if (j > 0) {
        if (!mbar_wait(o_done, (j - 1) & 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
          // rescale the rows whose running max moved (O = O * 2^(m_old - m_new))
          const float f = need ? ex2(m_used - m_new) : 1.f;
          float o[32];
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tmem_ld32(tO + lane_addr + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= f;
            tmem_st32(tO + lane_addr + c * 32, o);
          }
          tmem_wait_st();
          l *= f;
        }
      }
      if (need) m_used = m_new;
      const float ms = m_used == -INFINITY ? 0.f : m_used;
      // P row -> swizzled K-major tile: 16-byte chunk q holds keys 8q..8q+7
#pragma unroll
      for (int q = 0; q < kPfKeys / 8; ++q) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = ex2(s[q * 8 + e] - ms);
          l += pv[e];
        }
        uint4 w;
        w.x = pack2<T>(pv[0], pv[1]);
        w.y = pack2<T>(pv[2], pv[3]);
        w.z = pack2<T>(pv[4], pv[5]);
        w.w = pack2<T>(pv[6], pv[7]);
        *reinterpret_cast<uint4*>(sP + (q >> 3) * C::kPanelBytes + sw128(r, q & 7)) = w;
      }
      // The last tile may hold keys past kv_len (stale slots, pages never
      // loaded): zero those V rows so 0 * Inf cannot reach O.
      if (j == ntiles - 1 && key0 + kPfKeys > kv_len) {
        const int st = j % S;
        if (!mbar_wait(&v_full[st], (j / S) & 1)) {
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
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ---- epilogue: O / l -> out, LSE
    if (!failed && ntiles > 0) {
      if (!mbar_wait(o_done, (ntiles - 1) & 1)) failed = true;
    }
    if (failed) {
      set_status(PA_ERR_TIMEOUT);
    } else {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = reinterpret_cast<T*>(p.out) +
                (static_cast<size_t>(qo_start + t0 + qi) * hq + h * G + gi) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        if (ntiles > 0) {
          tmem_ld32(tO + lane_addr + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0.f;
        }
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = pack2<T>(o[e] * inv, o[e + 1] * inv);
            w.y = pack2<T>(o[e + 2] * inv, o[e + 3] * inv);
            w.z = pack2<T>(o[e + 4] * inv, o[e + 5] * inv);
            w.w = pack2<T>(o[e + 6] * inv, o[e + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = w;
          }
        }
      }
      if (row_ok && p.lse != nullptr)
        p.lse[static_cast<size_t>(qo_start + t0 + qi) * hq + h * G + gi] =
            l > 0.f ? m_used + lg2(l) : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
inline int prefill_qt(int group) {
  return (group == 1 || group == 2 || group == 4 || group == 8 || group == 16) ? kPfRows / group
                                                                                : 0;
}

}  // namespace pa
