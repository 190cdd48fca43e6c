// Fused QKV projection -> RoPE -> KV append, sm_100a tcgen05.
//
// The reference's per-layer prologue of the patched attention
// (src/models/llama.py:163-210): qkv = x W^T with W the fused
// [q_proj; k_proj; v_proj] weight (_fuse_qkv_proj_plain, llama.py:256-280,
// no bias), split into q, k, v; RoPE on q and k
// (apply_rope_pos_ids_inplace); k and v scattered into their page slots
// (append_paged_kv_cache). Here one GEMM kernel does all of it: each CTA
// computes a 128-token x BN-column tile of qkv in TMEM and its epilogue
// rotates the q / k heads of the tile in fp32 straight from the fp32
// accumulator and stores q rows to the q buffer and k / v rows to the pool,
// so qkv never goes to memory.
//
// Per CTA (192 threads):
//   * warp 4 — TMA producer: x tile [128 tokens x 64] and W tile
//     [BN columns x 64] per 64-deep k block into a ring (both K-major,
//     128-byte swizzle).
//   * warp 5 — tcgen05 issuer: 4 MMAs (M=128, N=BN, K=16) per k block into
//     BN TMEM columns; tcgen05.commit frees the stage.
//   * warps 0-3 — epilogue, one thread per token row (= TMEM lane).
#pragma once

#include "pa_common.cuh"
#include "ops.cuh"

namespace pa {

constexpr int kQkvBM = 128, kQkvBK = 64;
constexpr int kQkvThreads = 192;
// Tile shapes: N=128 columns with a deep 6-stage ring for few tokens (the
// GEMM then streams the weight: more CTAs, more bytes in flight per CTA);
// N=256 columns for many tokens (MMAs of 128 cycles keep the issuer's
// per-stage barrier wait hidden behind the queued MMAs) with a 2-stage
// ring, so that two CTAs share an SM (96 KB of shared memory and 256 TMEM
// columns each) and one CTA's epilogue runs under the other's main loop.
//
// RoPE cos / sin of each (token, pair): with N=128 tiles (one CTA per SM)
// the epilogue warps tabulate them in TMEM columns [128, 256) while the main
// loop runs (cos of pair i in column 128 + i, sin in 192 + i); with N=256
// tiles TMEM is full, so they go to the released stage memory after it.
// Either way the pair frequencies are computed once per CTA (smem).
template <int BN, int STAGES, bool SPLITK = false>
struct QkvCfg {
  static constexpr int kStageBytes = (kQkvBM + BN) * kQkvBK * 2;
  // split-K: slots for the other splits' partial rows of the (at most two)
  // row quarters this CTA finishes, 16 KB per quarter and source
  static constexpr int kQuarterBytes = 32 * BN * 4;
  static constexpr int kSlotBytes = SPLITK ? 4 * kQuarterBytes : 0;
  static constexpr int kSmemBytes = STAGES * kStageBytes + kSlotBytes + 512 + 1024;
  static constexpr bool kTabTmem = BN == 128;
  static constexpr int kTmemCols = 256;
  static_assert(!SPLITK || BN == 128, "split-K tiles are 128 columns");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct QkvParams {
  int M, K, hq, hkv, head_dim;
  uint8_t* q_out;
  int64_t q_sn;  // bytes between token rows of q_out (heads contiguous, head_dim apart)
  const int32_t* batch_indices;
  const int32_t* positions;
  int rotary_dim, interleave;
  float inv_scale, log2_theta;
  uint8_t* k_base;
  uint8_t* v_base;
  int64_t page_stride, head_stride, token_stride;  // bytes
  int64_t num_pages;
  const int32_t* kv_indices;
  int64_t num_kv_indices;  // entries kv_indptr may index
  const int32_t* kv_indptr;
  int batch, page_size;
  int splits;  // split-K: CTAs (one cluster) per output tile, 2..4; else 1
};

// Page slot of token m's row of kv head h, or -1 (padding row / error).
__device__ __forceinline__ int64_t qkv_slot(const QkvParams& p, int m, int h) {
  const int b = __ldg(p.batch_indices + m);
  if (b < 0) return -1;
  const int pos = __ldg(p.positions + m);
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

template <typename T, int D, int BN, int STAGES, bool SPLITK>
__global__ void __launch_bounds__(kQkvThreads, 2)
    qkv_rope_append_kernel(const __grid_constant__ CUtensorMap xmap,
                           const __grid_constant__ CUtensorMap wmap, const QkvParams p) {
  using C = QkvCfg<BN, STAGES, SPLITK>;
  constexpr int S = STAGES;
  constexpr int kStageBytes = C::kStageBytes;
  constexpr bool kTabTmem = C::kTabTmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* slots = smem + S * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(slots + C::kSlotBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* red_full = acc_full + 1;  // [2], split-K: the other splits' rows landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_full + 2);
  float* freq = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // [half]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kQkvBM, n0 = blockIdx.y * BN;
  const int nk = p.K / kQkvBK;
  // Split-K: the `splits` CTAs of one cluster (grid z) each multiply the
  // tile over a contiguous range of k blocks; row quarter q (TMEM lanes of
  // warp q) is finished by the CTA of rank q % splits, which receives the
  // other ranks' fp32 partial rows in its shared memory and adds all of
  // them in rank order (deterministic).
  const int nsplit = SPLITK ? p.splits : 1;
  const int rank = SPLITK ? static_cast<int>(cluster_rank()) : 0;
  const int kb0 = nk * rank / nsplit, kb1 = nk * (rank + 1) / nsplit;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&wmap);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    if (SPLITK)
      for (int j = 0; j < 2; ++j) mbar_init(&red_full[j], (nsplit - 1) * 32);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (SPLITK) cluster_arrive();  // this CTA's barriers are initialised
  const uint32_t tmem = *tmem_slot;
  bool failed = false;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int kb = kb0; kb < kb1; ++kb) {
        const int it = kb - kb0, st = it % S;
        if (it >= S && !mbar_wait(&empty[st], ((it / S) - 1) & 1)) {
          failed = true;
          break;
        }
        uint8_t* sa = smem + st * kStageBytes;
        mbar_arrive_expect_tx(&full[st], kStageBytes);
        tma_load_2d(sa, &xmap, &full[st], kb * kQkvBK, m0);
        tma_load_2d(sa + kQkvBM * kQkvBK * 2, &wmap, &full[st], kb * kQkvBK, n0);
      }
      if (failed) set_status(PA_ERR_TIMEOUT);
    }
    __syncwarp();
    if constexpr (SPLITK) cluster_wait();
  } else if (warp == 5) {
    // ------------------------------------------------------------ tcgen05 issuer
    if (lane == 0) {
      const int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t idesc = umma_idesc_f16(ab, kQkvBM, BN, 0);
      const uint32_t base = smem_u32(smem);
      for (int kb = kb0; kb < kb1; ++kb) {
        const int it = kb - kb0, st = it % S;
        if (!mbar_wait(&full[st], (it / S) & 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t sa = base + st * kStageBytes, sb = sa + kQkvBM * kQkvBK * 2;
#pragma unroll
        for (int kk = 0; kk < kQkvBK / 16; ++kk)
          umma_f16(tmem, umma_desc_sw128(sa + kk * 32, 16, 1024),
                   umma_desc_sw128(sb + kk * 32, 16, 1024), idesc, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[st]);
      }
      // on a timeout the accumulator is garbage; the epilogue still runs
      // (bounded) and the status word says so
      umma_commit(acc_full);
      if (failed) set_status(PA_ERR_TIMEOUT);
    }
    __syncwarp();
    if constexpr (SPLITK) cluster_wait();
  } else {
    // ------------------------------------------------------------ epilogue
    const int r = warp * 32 + lane;  // tile row == TMEM lane
    const int m = m0 + r;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    constexpr int HPT = BN / D;  // heads per tile
    const int qcols = p.hq * D, kcols = p.hkv * D;
    const int region = n0 < qcols ? 0 : (n0 < qcols + kcols ? 1 : 2);  // q / k / v
    const int head0 = region == 0 ? n0 / D : (region == 1 ? (n0 - qcols) / D
                                                           : (n0 - qcols - kcols) / D);
    const bool active = m < p.M;
    const int half = p.rotary_dim / 2;
    const int owner = warp % nsplit, jq = warp / nsplit;  // this quarter's finisher
    const bool mine = owner == rank;
    // Page slots of this row's k / v heads, looked up (three dependent
    // global loads) while the main loop runs.
    int64_t slot[HPT];
#pragma unroll
    for (int hh = 0; hh < HPT; ++hh)
      slot[hh] = (mine && active && region > 0) ? qkv_slot(p, m, head0 + hh) : -1;
    const int pos = active ? __ldg(p.positions + m) : 0;
    if (threadIdx.x < half) freq[threadIdx.x] = rope_freq(threadIdx.x, p.rotary_dim, p.inv_scale,
                                                          p.log2_theta);
    named_bar_sync(1, 128);  // the four epilogue warps
    __syncwarp();  // tcgen05.ld / st below are warp-collective
    // cos / sin of pairs [i0, i0 + 16) of this row: computed, and stored to
    // TMEM columns or to the row's column of the shared-memory table
    float* tab = reinterpret_cast<float*>(smem);
    auto tabulate = [&](int i0) {
      float cs[16], sn[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int i = min(i0 + u, half - 1);
        sincosf(static_cast<float>(pos) * freq[i], &sn[u], &cs[u]);
      }
      if constexpr (kTabTmem) {
        tmem_st16(taddr + BN + i0, cs);
        tmem_st16(taddr + BN + 64 + i0, sn);
      } else {
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          if (i0 + u < half) {
            tab[(i0 + u) * kQkvBM + r] = cs[u];
            tab[(half + i0 + u) * kQkvBM + r] = sn[u];
          }
        }
      }
    };
    auto table = [&](int i0, float* cs, float* sn) {
      if constexpr (kTabTmem) {
        tmem_ld16(taddr + BN + i0, cs);
        tmem_ld16(taddr + BN + 64 + i0, sn);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int i = min(i0 + u, half - 1);
          cs[u] = tab[i * kQkvBM + r];
          sn[u] = tab[(half + i) * kQkvBM + r];
        }
      }
    };
    // split-K slot of (this quarter, source rank z) in the finishing CTA:
    // row `lane` at 4 * BN bytes, 16-byte chunk c at (c & ~7) | ((c ^ lane) & 7)
    auto slot_row = [&](int z) {
      return smem_u32(slots) + (jq * (nsplit - 1) + (z < owner ? z : z - 1)) * C::kQuarterBytes +
             lane * (BN * 4);
    };
    auto chunk_off = [&](int c) { return ((c & ~7) | ((c ^ lane) & 7)) * 16; };
    if constexpr (kTabTmem) {
      if (mine && region < 2) {
#pragma unroll 1
        for (int i0 = 0; i0 < half; i0 += 16) tabulate(i0);
        tmem_wait_st();
      }
    }
    const bool ok = mbar_wait_warp(acc_full, 0);
    if (!ok && lane == 0) set_status(PA_ERR_TIMEOUT);
    tc_fence_after();
    bool go = ok;
    if constexpr (SPLITK) {
      cluster_wait();  // every CTA of the cluster has initialised its barriers
      if (!mine) {
        // push this quarter's partial rows to the finishing CTA (also after
        // a timeout, so that it does not wait for them in vain)
        const uint32_t dst = cluster_map(slot_row(rank), owner);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 8; ++e)
            st_cluster_f4(dst + chunk_off(c * 8 + e), v[4 * e], v[4 * e + 1], v[4 * e + 2],
                          v[4 * e + 3]);
        }
        mbar_arrive_remote(cluster_map(smem_u32(&red_full[jq]), owner));
        go = false;
      } else if (!mbar_wait_cluster_warp(&red_full[jq], 0)) {
        if (lane == 0) set_status(PA_ERR_TIMEOUT);
        go = false;
      }
    }
    if (go) {
      if constexpr (!kTabTmem) {
        // in the stage memory the main loop has released: column r of
        // [2 * half][128] floats, read back only by this thread
        if (region < 2) {
#pragma unroll 1
          for (int i0 = 0; i0 < half; i0 += 16) tabulate(i0);
        }
      }
#pragma unroll 1
      for (int hh = 0; hh < HPT; ++hh) {
        float a[D];
        __syncwarp();
        if constexpr (SPLITK) {
          // the splits' partial rows, added in rank order
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
#pragma unroll 1
            for (int z = 0; z < nsplit; ++z) {
              float v[32];
              if (z == rank) {
                tmem_ld32(taddr + hh * D + c * 32, v);
                tmem_wait_ld();
              } else {
                const uint32_t src = slot_row(z);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float4 f = ld_shared_f4(src + chunk_off((hh * D + c * 32) / 4 + e));
                  v[4 * e] = f.x;
                  v[4 * e + 1] = f.y;
                  v[4 * e + 2] = f.z;
                  v[4 * e + 3] = f.w;
                }
              }
#pragma unroll
              for (int e = 0; e < 32; ++e) a[c * 32 + e] = z == 0 ? v[e] : a[c * 32 + e] + v[e];
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) tmem_ld32(taddr + hh * D + c * 32, a + c * 32);
          tmem_wait_ld();
        }
        if (region < 2) {
          // fp32 rotation of the accumulator (rope_rotate, as rope_kernel),
          // 16 pairs per table read; padding rows too (nothing stores them),
          // since the TMEM table loads are warp-collective
          if (p.rotary_dim == D && !p.interleave) {
#pragma unroll
            for (int i0 = 0; i0 < D / 2; i0 += 16) {
              float cs[16], sn[16];
              table(i0, cs, sn);
#pragma unroll
              for (int u = 0; u < 16; ++u)
                rope_rotate(a[i0 + u], a[i0 + u + D / 2], cs[u], sn[u], &a[i0 + u],
                            &a[i0 + u + D / 2]);
            }
          } else if (p.rotary_dim == D) {
#pragma unroll
            for (int i0 = 0; i0 < D / 2; i0 += 16) {
              float cs[16], sn[16];
              table(i0, cs, sn);
#pragma unroll
              for (int u = 0; u < 16; ++u)
                rope_rotate(a[2 * (i0 + u)], a[2 * (i0 + u) + 1], cs[u], sn[u], &a[2 * (i0 + u)],
                            &a[2 * (i0 + u) + 1]);
            }
          } else {
            float tmp[D];
#pragma unroll
            for (int e = 0; e < D; ++e) tmp[e] = a[e];
#pragma unroll 1
            for (int i0 = 0; i0 < half; i0 += 16) {
              float cs[16], sn[16];
              table(i0, cs, sn);
#pragma unroll 1
              for (int u = 0; u < 16 && i0 + u < half; ++u) {
                const int i = i0 + u;
                const int ia = p.interleave ? 2 * i : i, ib = p.interleave ? 2 * i + 1 : i + half;
                float y0, y1;
                rope_rotate(tmp[ia], tmp[ib], cs[u], sn[u], &y0, &y1);
                tmp[ia] = y0;
                tmp[ib] = y1;
              }
            }
#pragma unroll
            for (int e = 0; e < D; ++e) a[e] = tmp[e];
          }
        }
        // pack pairs in place over a[0 .. D/2)
#pragma unroll
        for (int e = 0; e < D / 2; ++e) a[e] = __uint_as_float(pack2<T>(a[2 * e], a[2 * e + 1]));
        uint8_t* dst = nullptr;
        if (active && region == 0) {
          dst = p.q_out + m * p.q_sn + static_cast<int64_t>(head0 + hh) * D * 2;
        } else if (slot[hh] >= 0) {
          dst = (region == 1 ? p.k_base : p.v_base) + slot[hh];
        }
        if (dst != nullptr) {
#pragma unroll
          for (int e = 0; e < D / 8; ++e)
            reinterpret_cast<uint4*>(dst)[e] =
                make_uint4(__float_as_uint(a[4 * e]), __float_as_uint(a[4 * e + 1]),
                           __float_as_uint(a[4 * e + 2]), __float_as_uint(a[4 * e + 3]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace pa
