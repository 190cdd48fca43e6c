// Batched paged decode attention for sm_100a.
//
// Reference behaviour: BatchDecodeWithPagedKVCacheWrapper.forward as called
// from src/models/llama.py:230-245 — one query row per request and q head,
// o[b, hq] = softmax(sm_scale * q[b, hq] . K_b,hkv^T) V_b,hkv over the
// request's kv_len = (pages - 1) * P + kv_last_page_len[b] keys, hkv = hq / g.
//
// Design (HBM-bound; one page of one kv head = P x D contiguous elements):
//   * The work stream is every (request b, kv head h, page j) in that order.
//     decode_plan_kernel cuts it into equal runs of Q page-heads, one run per
//     persistent warp, so every warp moves the same number of bytes however
//     skewed the context lengths are (split-KV without a host-side plan).
//   * Each warp owns a ring of shared-memory stages. Lane 0 fills a stage with
//     two tiled TMA loads (K tile and V tile of one page-head, 128-byte
//     swizzle) completing on the stage's mbarrier, and keeps the ring full
//     ahead of the warp's own compute. Warps never wait on each other.
//   * The g query heads of a kv head are the rows of one m16n8k16 tile, so a
//     loaded page is shared by the whole GQA group: S = Q K^T (mma.sync, fp32
//     accumulate), online softmax on the S fragments in registers (quad
//     shuffles), O += P V with V read through ldmatrix.trans.
//   * A request/head segment that straddles warps is written as normalised
//     fp32 partials plus base-2 LSE; the last warp to finish that segment
//     (atomic counter per segment) merges the pieces in the same launch.
#pragma once

#include "pa_common.cuh"

namespace pa {

template <int D>
struct DecodeCfg {
  static constexpr int kPanels = D / 64;           // 128-byte swizzle panels per row
  static constexpr int kTileBytes = kPage * D * 2;  // one page-head of K (or V)
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = (D == 64) ? 6 : 3;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kSmemBytes =
      kDecodeWarps * kRingBytes + kDecodeWarps * kStages * 8 + 1024;
};

// --------------------------------------------------------------------- plan
// One CTA. Validates the CSR table, partitions the stream, clears the merge
// counters. W = number of persistent warps the run kernel launches.
__global__ void decode_plan_kernel(const int32_t* __restrict__ kv_indptr,
                                   const int32_t* __restrict__ last_len, int batch, int hkv,
                                   int hq, int head_dim, int page_size, int64_t num_indices,
                                   int num_warps, int min_per_warp, uint8_t* __restrict__ ws) {
  const DecodeWsLayout L = decode_ws_layout(num_warps, batch, hkv, head_dim);
  DecodePlanHeader* hdr = reinterpret_cast<DecodePlanHeader*>(ws + L.hdr);
  int4* warp_start = reinterpret_cast<int4*>(ws + L.warp_start);
  int32_t* empty = reinterpret_cast<int32_t*>(ws + L.empty);
  int32_t* counter = reinterpret_cast<int32_t*>(ws + L.counter);

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
  const long long total_ll = static_cast<long long>(hkv) * last_ptr;
  if (first != 0 || last_ptr > num_indices || total_ll > 0x7fffffffLL) {
    if (threadIdx.x == 0) atomicOr(&s_err, 1);
  }
  __syncthreads();
  const bool err = s_err != 0;
  const int total = err ? 0 : static_cast<int>(total_ll);
  int q = (total + num_warps - 1) / num_warps;
  q = max(q, min_per_warp);
  for (int w = threadIdx.x; w < num_warps; w += blockDim.x) {
    const long long s0 = static_cast<long long>(w) * q;
    int4 st = make_int4(0, 0, 0, 0);
    if (s0 < total) {
      // Largest b with hkv * kv_indptr[b] <= s0 (empty requests are skipped
      // because their start equals the next request's start).
      int lo = 0, hi = batch;  // invariant: hkv*indptr[lo] <= s0 < hkv*indptr[hi]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (static_cast<long long>(hkv) * kv_indptr[mid] <= s0) lo = mid; else hi = mid;
      }
      const int base = kv_indptr[lo];
      const int n = kv_indptr[lo + 1] - base;
      const int off = static_cast<int>(s0 - static_cast<long long>(hkv) * base);
      st = make_int4(lo, off / n, off % n, 0);
    }
    warp_start[w] = st;
  }
  if (threadIdx.x == 0) {
    hdr->status = err ? PA_ERR_DEVICE_CHECK : PA_OK;
    hdr->total = total;
    hdr->per_warp = q;
    hdr->num_warps = num_warps;
    hdr->batch_size = batch;
    hdr->num_kv_heads = hkv;
    hdr->num_qo_heads = hq;
    hdr->head_dim = head_dim;
    hdr->page_size = page_size;
    hdr->num_empty = err ? 0 : s_empty;
    hdr->magic = kDecodeMagic;
    if (err) set_status(PA_ERR_DEVICE_CHECK);
  }
}

// ---------------------------------------------------------------------- run
struct StreamCursor {
  int b, h, j, n, base;
};

__device__ __forceinline__ void cursor_load(StreamCursor& c, const int32_t* indptr) {
  c.base = __ldg(indptr + c.b);
  c.n = __ldg(indptr + c.b + 1) - c.base;
}

// Moves to the next stream position; must only be called when one exists.
__device__ __forceinline__ void cursor_next(StreamCursor& c, const int32_t* indptr, int hkv) {
  if (++c.j < c.n) return;
  c.j = 0;
  if (++c.h < hkv) return;
  c.h = 0;
  do {
    ++c.b;
    cursor_load(c, indptr);
  } while (c.n == 0);
}

template <typename T, int D>
__global__ void __launch_bounds__(kDecodeWarps * 32, 1)
    decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const DecodeParams p) {
  using C = DecodeCfg<D>;
  constexpr int NT = D / 8;   // 8-wide column tiles of O
  constexpr int KS = D / 16;  // 16-deep k steps of Q K^T
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int W = gridDim.x * kDecodeWarps;
  const int gw = blockIdx.x * kDecodeWarps + warp;
  const DecodePlanHeader* hdr = p.hdr;

  if (hdr->magic != kDecodeMagic || hdr->num_warps != W || hdr->batch_size != p.batch_size ||
      hdr->num_kv_heads != p.num_kv_heads || hdr->num_qo_heads != p.num_qo_heads ||
      hdr->head_dim != D) {
    if (gw == 0 && lane == 0) set_status(PA_ERR_NOT_PLANNED);
    return;
  }
  if (hdr->status != PA_OK) return;
  const int Q = hdr->per_warp, total = hdr->total, hkv = p.num_kv_heads, G = p.group;
  const int hq = p.num_qo_heads;
  T* out = reinterpret_cast<T*>(p.out);

  // Requests without pages produce zeros (and LSE = -inf).
  for (int e = gw; e < hdr->num_empty; e += W) {
    const int b = p.empty[e];
    for (int i = lane; i < hq * D / 8; i += 32)
      reinterpret_cast<uint4*>(out + static_cast<size_t>(b) * hq * D)[i] = make_uint4(0, 0, 0, 0);
    if (p.lse != nullptr)
      for (int i = lane; i < hq; i += 32) p.lse[static_cast<size_t>(b) * hq + i] = -INFINITY;
  }

  const int s0 = gw * Q;
  if (s0 >= total) return;
  const int cnt = min(Q, total - s0);

  uint8_t* ring = smem + warp * C::kRingBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDecodeWarps * C::kRingBytes) + warp * S;
  if (lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int4 st = p.warp_start[gw];
  StreamCursor pc;
  pc.b = st.x;
  pc.h = st.y;
  pc.j = st.z;
  cursor_load(pc, p.kv_indptr);
  StreamCursor cc = pc;

  // Lane 0 fills stage `stage` with the K and V tiles of cursor position c.
  auto issue = [&](int stage, const StreamCursor& c) {
    if (lane == 0) {
      int page = __ldg(p.kv_indices + c.base + c.j);
      if (static_cast<unsigned>(page) >= static_cast<unsigned long long>(p.num_pages)) {
        set_status(PA_ERR_DEVICE_CHECK);
        page = 0;
      }
      uint8_t* dst = ring + stage * C::kStageBytes;
      mbar_arrive_expect_tx(&bars[stage], C::kStageBytes);
      const int c1 = p.heads_inner ? c.h : 0, c2 = p.heads_inner ? 0 : c.h;
#pragma unroll
      for (int pn = 0; pn < C::kPanels; ++pn) {
        tma_load_4d(dst + pn * 2048, &kmap, &bars[stage], pn * 64, c1, c2, page);
        tma_load_4d(dst + C::kTileBytes + pn * 2048, &vmap, &bars[stage], pn * 64, c1, c2, page);
      }
    }
  };

  const int npro = min(S, cnt);
  for (int k = 0; k < npro; ++k) {
    if (k > 0) cursor_next(pc, p.kv_indptr, hkv);
    issue(k, pc);
  }

  const T* qbase = reinterpret_cast<const T*>(p.q);
  uint32_t qf[KS][4];
  float o[NT][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  int seg_start = 0, last_len = kPage;
  const bool row0 = gid < G, row1 = gid + 8 < G;

  for (int i = 0; i < cnt; ++i) {
    if (i == 0 || cc.j == 0) {
      // New (request, kv head) segment: load the group's q rows as A fragments.
      const T* qh = qbase + static_cast<int64_t>(cc.b) * p.q_stride_n +
                    static_cast<int64_t>(cc.h * G) * p.q_stride_h;
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
      seg_start = hkv * cc.base + cc.h * cc.n;
      last_len = __ldg(p.kv_last_page_len + cc.b);
    }

    const int stage = i % S;
    if (!mbar_wait(&bars[stage], (i / S) & 1)) {
      set_status(PA_ERR_TIMEOUT);
      // Give the copies still in flight a bounded chance to land, then leave.
      for (int k = i + 1; k < min(i + S, cnt); ++k) mbar_wait(&bars[k % S], (k / S) & 1);
      return;
    }
    uint8_t* kst = ring + stage * C::kStageBytes;
    const uint32_t kb = smem_u32(kst);
    const uint32_t vb = kb + C::kTileBytes;
    const int valid = (cc.j == cc.n - 1) ? last_len : kPage;

    // ---- S = Q K^T over the 16 keys of this page
    float s[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
    {
      const int krow = (lane & 7) + ((lane >> 4) & 1) * 8;
      const int khalf = (lane >> 3) & 1;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int panel = kk >> 2;
        const int chunk = ((kk & 3) << 1) + khalf;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + panel * 2048 + sw128(krow, chunk), b0, b1, b2, b3);
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

    // Slots past the last key hold stale pool bytes; zero those V rows so a
    // non-finite value there cannot reach O through 0 * Inf.
    if (valid < kPage) {
      uint8_t* vst = kst + C::kTileBytes;
      const int per_row = C::kPanels * 8;
      for (int idx = lane; idx < (kPage - valid) * per_row; idx += 32) {
        const int r = valid + idx / per_row;
        const int rem = idx % per_row;
        *reinterpret_cast<uint4*>(vst + (rem >> 3) * 2048 + r * 128 + (rem & 7) * 16) =
            make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async();
      __syncwarp();
    }

    // ---- O += P V
    {
      const int vrow = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int vhalf = lane >> 4;
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        const int panel = np >> 2;
        const int chunk = ((np & 3) << 1) + vhalf;
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vb + panel * 2048 + sw128(vrow, chunk), v0, v1, v2, v3);
        Mma16816<T>::run(o[2 * np], pa, v0, v1);
        Mma16816<T>::run(o[2 * np + 1], pa, v2, v3);
      }
    }
    __syncwarp();

    // Refill the stage just consumed with the page S positions ahead.
    if (i + S < cnt) {
      cursor_next(pc, p.kv_indptr, hkv);
      issue(stage, pc);
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
      const int head0 = cc.h * G;
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
        const int slot = gw * 2 + (seg_start <= s0 ? 0 : 1);
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
        __threadfence();
        __syncwarp();
        int* cnt_ptr = p.counter + cc.b * hkv + cc.h;
        int old = 0;
        if (lane == 0) old = atomicAdd(cnt_ptr, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        const int w0 = seg_start / Q, w1 = (seg_end - 1) / Q;
        if (old == w1 - w0) {
          // Last piece of this segment to finish: merge all pieces.
          __threadfence();
          constexpr int E = D / 32;
          T* ob = out + (static_cast<size_t>(cc.b) * hq + head0) * D;
          for (int r = 0; r < G; ++r) {
            float lmax = -INFINITY;
            for (int w = w0; w <= w1; ++w) {
              const int sl = w * 2 + (seg_start <= w * Q ? 0 : 1);
              lmax = fmaxf(lmax, __ldcg(p.part_lse + static_cast<size_t>(sl) * kMaxGroup + r));
            }
            float acc[E];
#pragma unroll
            for (int e = 0; e < E; ++e) acc[e] = 0.f;
            float wsum = 0.f;
            for (int w = w0; w <= w1; ++w) {
              const int sl = w * 2 + (seg_start <= w * Q ? 0 : 1);
              const float wt =
                  ex2(__ldcg(p.part_lse + static_cast<size_t>(sl) * kMaxGroup + r) - lmax);
              wsum += wt;
              const float* src = p.part_o + (static_cast<size_t>(sl) * kMaxGroup + r) * D + lane * E;
              if constexpr (E == 2) {
                const float2 v = __ldcg(reinterpret_cast<const float2*>(src));
                acc[0] += wt * v.x;
                acc[1] += wt * v.y;
              } else {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(src));
                acc[0] += wt * v.x;
                acc[1] += wt * v.y;
                acc[2] += wt * v.z;
                acc[3] += wt * v.w;
              }
            }
            const float winv = 1.f / wsum;
            T* dst = ob + r * D + lane * E;
#pragma unroll
            for (int e = 0; e < E; e += 2)
              *reinterpret_cast<uint32_t*>(dst + e) = pack2<T>(acc[e] * winv, acc[e + 1] * winv);
            if (p.lse != nullptr && lane == 0)
              p.lse[static_cast<size_t>(cc.b) * hq + head0 + r] = lmax + lg2(wsum);
          }
          if (lane == 0) *cnt_ptr = 0;  // ready for the next launch on this plan
        }
      }
    }

    if (i + 1 < cnt) cursor_next(cc, p.kv_indptr, hkv);
  }
}

}  // namespace pa
