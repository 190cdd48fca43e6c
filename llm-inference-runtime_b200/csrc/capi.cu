// C ABI of the paged-attention backend (declarations: include/paged_attn.h).
// Host-side argument checks, TMA descriptor encoding, launch configuration.
// Single translation unit: every kernel header is included here so device
// globals (the status word) need no relocatable device code.
#include <atomic>
#include <type_traits>
#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <mutex>

#include "decode.cuh"
#include "ops.cuh"
#include "prefill.cuh"
#include "tables.cuh"
#include "qkv.cuh"
#include "cascade.cuh"

namespace {

using namespace pa;

constexpr int kMaxDevices = 64;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int sm_count(int dev) {
  static std::atomic<int> cache[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return 0;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// cudaFuncSetAttribute is per device; remember which (kernel, device) pairs
// already allow their dynamic shared memory size.
template <typename K>
cudaError_t allow_smem(K kernel, int bytes, std::atomic<uint64_t>* done_mask, int dev) {
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (done_mask->load(std::memory_order_relaxed) & bit) return cudaSuccess;
  cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done_mask->fetch_or(bit);
  return e;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// True when the cache keeps the heads of a token next to each other
// ("NHD": token stride > head stride). The tensor map then orders its dims
// (D, H_kv, P, pages) so strides increase; otherwise (D, P, H_kv, pages).
bool heads_inner(const pa_kv_cache& c) { return c.token_stride > c.head_stride; }

// 4-D map over one of the K / V caches, 128-byte swizzled boxes of 64
// columns x box_rows tokens x box_heads heads of one page. The box lands in
// shared memory as box_rows * box_heads rows of 128 bytes, head-major for
// HND pools and token-major for NHD pools.
int encode_kv_map(CUtensorMap* map, const void* base, const pa_kv_cache& c, int box_rows,
                  int box_heads) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return PA_ERR_CUDA;
  const bool hi = heads_inner(c);
  const cuuint64_t P = static_cast<cuuint64_t>(c.page_size);
  const cuuint64_t H = static_cast<cuuint64_t>(c.num_kv_heads);
  const cuuint64_t ts = static_cast<cuuint64_t>(c.token_stride) * 2;
  const cuuint64_t hs = static_cast<cuuint64_t>(c.head_stride) * 2;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(c.head_dim), hi ? H : P, hi ? P : H,
                              static_cast<cuuint64_t>(c.num_pages)};
  const cuuint64_t strides[3] = {hi ? hs : ts, hi ? ts : hs,
                                 static_cast<cuuint64_t>(c.page_stride) * 2};
  const cuuint32_t br = static_cast<cuuint32_t>(box_rows);
  const cuuint32_t bh = static_cast<cuuint32_t>(box_heads);
  const cuuint32_t box[4] = {64, hi ? bh : br, hi ? br : bh, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = c.dtype == PA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PA_OK : PA_ERR_INVALID_ARGUMENT;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// 2-D map over a row-major matrix [rows, cols] (row stride in elements), box
// (64 columns, box_rows rows), 128-byte swizzle: the K-major operand tile of
// a tcgen05 GEMM. Rows past the end read as zeros.
int encode_2d_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                  int64_t row_stride, int box_rows, int dtype) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return PA_ERR_CUDA;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == PA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PA_OK : PA_ERR_INVALID_ARGUMENT;
}

bool valid_dtype(int dt) { return dt == PA_DTYPE_F16 || dt == PA_DTYPE_BF16; }

// Checks a cache description for the attention kernels (TMA needs 16-byte
// aligned bases and strides).
int check_cache(const pa_kv_cache* c) {
  if (c == nullptr || c->k_base == nullptr || c->v_base == nullptr) return PA_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(c->dtype)) return PA_ERR_UNSUPPORTED;
  if (c->num_kv_heads <= 0 || c->num_pages <= 0 || c->page_size <= 0 || c->head_dim <= 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (!aligned16(c->k_base) || !aligned16(c->v_base)) return PA_ERR_INVALID_ARGUMENT;
  if (c->page_stride % 8 || c->head_stride % 8 || c->token_stride % 8)
    return PA_ERR_INVALID_ARGUMENT;
  return PA_OK;
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PA_OK : PA_ERR_CUDA;
}

// Kernels of the per-step chain (positions, plan, append, decode) launch with
// programmatic stream serialization: each may start while its predecessor in
// the stream drains and waits (griddepcontrol.wait) before reading its
// inputs, which hides the launch gap between dependent kernels. PA_PDL=0 in
// the environment turns it off (plain stream order).
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("PA_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
int launch_chain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                 cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) != cudaSuccess) {
    (void)cudaGetLastError();
    return PA_ERR_CUDA;
  }
  return launch_status();
}

// Decode partition for a cache shape on device `dev`: one CTA per SM, each
// holding DecodeGeom::groups_per_cta groups.
struct DecodePlanShape {
  DecodeGeom g;
  int ctas;
  int units;  // groups in the grid
};

bool decode_shape(int dev, int hkv, int head_dim, DecodePlanShape* s) {
  if (!decode_geom(hkv, head_dim, &s->g)) return false;
  s->ctas = sm_count(dev);
  s->units = s->ctas * s->g.groups_per_cta;
  return s->ctas > 0;
}

size_t decode_ws_bytes(const DecodePlanShape& s, int batch, int hkv, int head_dim) {
  return decode_ws_layout(s.units, batch, hkv, head_dim, s.g.hb).total;
}

template <typename T, int D>
int launch_decode(const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& prm,
                  const DecodePlanShape& sh, int dev, cudaStream_t stream) {
  // Largest dynamic shared memory already allowed for this kernel, per device.
  static std::atomic<int> allowed[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return PA_ERR_CUDA;
  if (allowed[dev].load(std::memory_order_relaxed) < sh.g.smem_bytes) {
    if (cudaFuncSetAttribute(decode_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             sh.g.smem_bytes) != cudaSuccess)
      return PA_ERR_CUDA;
    allowed[dev].store(sh.g.smem_bytes, std::memory_order_relaxed);
  }
  return launch_chain(decode_kernel<T, D>, dim3(sh.ctas), dim3(sh.g.threads), sh.g.smem_bytes,
                      stream, km, vm, prm);
}

// 3-D map over q [tokens, heads, dim] (strides in elements), box (64 dims,
// g heads, qt tokens): the box lands as 128 rows (token-major, head-minor)
// of 128 bytes, 128-byte swizzled — the K-major A tile of S = Q K^T.
int encode_q_map(CUtensorMap* map, const void* q, int64_t stride_n, int64_t stride_h,
                 int64_t total_qo, int hq, int head_dim, int g, int qt, int dtype) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return PA_ERR_CUDA;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(hq),
                              static_cast<cuuint64_t>(total_qo)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_h) * 2,
                                 static_cast<cuuint64_t>(stride_n) * 2};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(g), static_cast<cuuint32_t>(qt)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == PA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 3, const_cast<void*>(q), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PA_OK : PA_ERR_INVALID_ARGUMENT;
}

template <typename T, int D>
int launch_prefill(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                   const CUtensorMap& om, const PrefillParams& prm, int64_t grid, int dev,
                   cudaStream_t stream) {
  static std::atomic<uint64_t> done{0};
  constexpr int smem = PfCfg<D>::kSmemBytes;
  if (allow_smem(prefill_kernel<T, D>, smem, &done, dev) != cudaSuccess) return PA_ERR_CUDA;
  if (grid <= 0) return PA_OK;
  // persistent: one CTA per SM at most, each taking items until none is left
  const int sms = sm_count(dev) > 0 ? sm_count(dev) : 148;
  grid = std::min<int64_t>(grid, sms);
  prefill_kernel<T, D><<<static_cast<unsigned>(grid), kPfThreads, smem, stream>>>(qm, km, vm, om,
                                                                                  prm);
  return launch_status();
}

}  // namespace

extern "C" {

const char* pa_status_string(int status) {
  switch (status) {
    case PA_OK: return "ok";
    case PA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PA_ERR_UNSUPPORTED: return "unsupported configuration";
    case PA_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case PA_ERR_CUDA: return "CUDA error";
    case PA_ERR_DEVICE_CHECK: return "device-side validation failed";
    case PA_ERR_TIMEOUT: return "bounded device wait expired";
    case PA_ERR_NOT_PLANNED: return "run without a matching plan";
    default: return "unknown status";
  }
}

int pa_abi_version(void) { return PA_ABI_VERSION; }

int pa_device_status(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return PA_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_status, sizeof(int)) != cudaSuccess) return PA_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_status, &zero, sizeof(int)) != cudaSuccess) return PA_ERR_CUDA;
  return v;
}

int pa_batch_indices_positions(const int32_t* append_indptr, const int32_t* seq_lens,
                               int32_t batch_size, int32_t nnz, int32_t* batch_indices,
                               int32_t* positions, void* stream) {
  if (batch_size < 0 || nnz < 0) return PA_ERR_INVALID_ARGUMENT;
  if (append_indptr == nullptr || (batch_size > 0 && seq_lens == nullptr)) return PA_ERR_INVALID_ARGUMENT;
  if (nnz > 0 && (batch_indices == nullptr || positions == nullptr)) return PA_ERR_INVALID_ARGUMENT;
  if (nnz == 0) return PA_OK;
  return launch_chain(batch_indices_positions_kernel, dim3(batch_size + 1), dim3(256), 0,
                      static_cast<cudaStream_t>(stream), append_indptr, seq_lens, batch_size, nnz,
                      batch_indices, positions);
}

int pa_append_paged_kv_cache(const void* append_key, int64_t key_stride_n, int64_t key_stride_h,
                             const void* append_value, int64_t value_stride_n,
                             int64_t value_stride_h, const int32_t* batch_indices,
                             const int32_t* positions, int32_t nnz, const pa_kv_cache* cache,
                             const int32_t* kv_indices, int64_t num_kv_indices,
                             const int32_t* kv_indptr, int32_t batch_size, void* stream) {
  if (nnz < 0 || batch_size < 0 || num_kv_indices < 0) return PA_ERR_INVALID_ARGUMENT;
  if (nnz == 0) return PA_OK;
  if (cache == nullptr || append_key == nullptr || append_value == nullptr ||
      batch_indices == nullptr || positions == nullptr || kv_indices == nullptr ||
      kv_indptr == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(cache->dtype)) return PA_ERR_UNSUPPORTED;
  if (cache->k_base == nullptr || cache->v_base == nullptr || cache->page_size <= 0 ||
      cache->num_kv_heads <= 0 || cache->head_dim <= 0 || cache->head_dim % 8)
    return PA_ERR_INVALID_ARGUMENT;
  // 16-byte vector copies: rows and row starts must be 16-byte aligned.
  if (!aligned16(append_key) || !aligned16(append_value) || !aligned16(cache->k_base) ||
      !aligned16(cache->v_base))
    return PA_ERR_INVALID_ARGUMENT;
  if (key_stride_n % 8 || key_stride_h % 8 || value_stride_n % 8 || value_stride_h % 8 ||
      cache->page_stride % 8 || cache->head_stride % 8 || cache->token_stride % 8)
    return PA_ERR_INVALID_ARGUMENT;
  AppendParams p;
  p.key = static_cast<const uint8_t*>(append_key);
  p.value = static_cast<const uint8_t*>(append_value);
  p.key_stride_n = key_stride_n * 2;
  p.key_stride_h = key_stride_h * 2;
  p.value_stride_n = value_stride_n * 2;
  p.value_stride_h = value_stride_h * 2;
  p.batch_indices = batch_indices;
  p.positions = positions;
  p.nnz = nnz;
  p.k_base = static_cast<uint8_t*>(const_cast<void*>(cache->k_base));
  p.v_base = static_cast<uint8_t*>(const_cast<void*>(cache->v_base));
  p.page_stride = cache->page_stride * 2;
  p.head_stride = cache->head_stride * 2;
  p.token_stride = cache->token_stride * 2;
  p.num_pages = cache->num_pages;
  p.kv_indices = kv_indices;
  p.num_kv_indices = num_kv_indices;
  p.kv_indptr = kv_indptr;
  p.batch = batch_size;
  p.num_kv_heads = cache->num_kv_heads;
  p.page_size = cache->page_size;
  p.row_chunks = cache->head_dim * 2 / 16;
  const int64_t work = static_cast<int64_t>(nnz) * cache->num_kv_heads * p.row_chunks * 2;
  const int dev = current_device();
  const int64_t max_blocks = static_cast<int64_t>(sm_count(dev) > 0 ? sm_count(dev) : 148) * 8;
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, max_blocks));
  return launch_chain(append_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                      p);
}

int pa_apply_rope_pos_ids_inplace(void* q, int64_t q_stride_n, int64_t q_stride_h, void* k,
                                  int64_t k_stride_n, int64_t k_stride_h, const int32_t* pos_ids,
                                  int32_t nnz, int32_t num_qo_heads, int32_t num_kv_heads,
                                  int32_t head_dim, int32_t rotary_dim, int32_t interleave,
                                  float rope_scale, float rope_theta, int32_t dtype,
                                  void* stream) {
  if (nnz < 0 || num_qo_heads < 0 || num_kv_heads < 0) return PA_ERR_INVALID_ARGUMENT;
  if (nnz == 0 || num_qo_heads + num_kv_heads == 0) return PA_OK;
  if (pos_ids == nullptr || (num_qo_heads > 0 && q == nullptr) ||
      (num_kv_heads > 0 && k == nullptr))
    return PA_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(dtype)) return PA_ERR_UNSUPPORTED;
  if (rotary_dim <= 0 || rotary_dim % 2 || rotary_dim > head_dim) return PA_ERR_INVALID_ARGUMENT;
  if (!(rope_scale > 0.f) || !(rope_theta > 0.f)) return PA_ERR_INVALID_ARGUMENT;
  const int64_t work = static_cast<int64_t>(nnz) * (num_qo_heads + num_kv_heads) * (rotary_dim / 2);
  const int dev = current_device();
  const int64_t max_blocks = static_cast<int64_t>(sm_count(dev) > 0 ? sm_count(dev) : 148) * 8;
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, max_blocks));
  const float inv_scale = 1.0f / rope_scale;
  const float log2_theta = std::log2(rope_theta);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == PA_DTYPE_BF16)
    rope_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        static_cast<__nv_bfloat16*>(q), q_stride_n, q_stride_h, static_cast<__nv_bfloat16*>(k),
        k_stride_n, k_stride_h, pos_ids, nnz, num_qo_heads, num_kv_heads, rotary_dim, interleave,
        inv_scale, log2_theta);
  else
    rope_kernel<__half><<<blocks, 256, 0, st>>>(
        static_cast<__half*>(q), q_stride_n, q_stride_h, static_cast<__half*>(k), k_stride_n,
        k_stride_h, pos_ids, nnz, num_qo_heads, num_kv_heads, rotary_dim, interleave, inv_scale,
        log2_theta);
  return launch_status();
}

int pa_apply_rope_append(void* q, int64_t q_stride_n, int64_t q_stride_h, void* k,
                         int64_t k_stride_n, int64_t k_stride_h, const void* v,
                         int64_t v_stride_n, int64_t v_stride_h, const int32_t* batch_indices,
                         const int32_t* positions, int32_t nnz, int32_t num_qo_heads,
                         int32_t rotary_dim, int32_t interleave, float rope_scale,
                         float rope_theta, const pa_kv_cache* cache, const int32_t* kv_indices,
                         int64_t num_kv_indices, const int32_t* kv_indptr, int32_t batch_size,
                         void* stream) {
  if (nnz < 0 || batch_size < 0 || num_qo_heads < 0 || num_kv_indices < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (nnz == 0) return PA_OK;
  if (cache == nullptr || q == nullptr || k == nullptr || v == nullptr ||
      batch_indices == nullptr || positions == nullptr || kv_indices == nullptr ||
      kv_indptr == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(cache->dtype)) return PA_ERR_UNSUPPORTED;
  const int D = cache->head_dim, hkv = cache->num_kv_heads;
  if (cache->k_base == nullptr || cache->v_base == nullptr || cache->page_size <= 0 || hkv <= 0 ||
      D <= 0 || D % 8)
    return PA_ERR_INVALID_ARGUMENT;
  if (rotary_dim <= 0 || rotary_dim % 2 || rotary_dim > D) return PA_ERR_INVALID_ARGUMENT;
  if (!(rope_scale > 0.f) || !(rope_theta > 0.f)) return PA_ERR_INVALID_ARGUMENT;
  const bool fused = rotary_dim % 16 == 0 && aligned16(q) && aligned16(k) && aligned16(v) &&
                     aligned16(cache->k_base) && aligned16(cache->v_base) && q_stride_n % 8 == 0 &&
                     q_stride_h % 8 == 0 && k_stride_n % 8 == 0 && k_stride_h % 8 == 0 &&
                     v_stride_n % 8 == 0 && v_stride_h % 8 == 0 && cache->page_stride % 8 == 0 &&
                     cache->head_stride % 8 == 0 && cache->token_stride % 8 == 0;
  if (!fused) {
    const int rc = pa_apply_rope_pos_ids_inplace(q, q_stride_n, q_stride_h, k, k_stride_n,
                                                 k_stride_h, positions, nnz, num_qo_heads, hkv, D,
                                                 rotary_dim, interleave, rope_scale, rope_theta,
                                                 cache->dtype, stream);
    if (rc != PA_OK) return rc;
    return pa_append_paged_kv_cache(k, k_stride_n, k_stride_h, v, v_stride_n, v_stride_h,
                                    batch_indices, positions, nnz, cache, kv_indices,
                                    num_kv_indices, kv_indptr, batch_size, stream);
  }
  RopeAppendParams p;
  p.q = static_cast<uint8_t*>(q);
  p.k = static_cast<uint8_t*>(k);
  p.v = static_cast<const uint8_t*>(v);
  p.q_sn = q_stride_n * 2;
  p.q_sh = q_stride_h * 2;
  p.k_sn = k_stride_n * 2;
  p.k_sh = k_stride_h * 2;
  p.v_sn = v_stride_n * 2;
  p.v_sh = v_stride_h * 2;
  p.batch_indices = batch_indices;
  p.positions = positions;
  p.nnz = nnz;
  p.hq = num_qo_heads;
  p.hkv = hkv;
  p.head_dim = D;
  p.rotary_dim = rotary_dim;
  p.interleave = interleave ? 1 : 0;
  p.inv_scale = 1.0f / rope_scale;
  p.log2_theta = std::log2(rope_theta);
  p.k_base = static_cast<uint8_t*>(const_cast<void*>(cache->k_base));
  p.v_base = static_cast<uint8_t*>(const_cast<void*>(cache->v_base));
  p.page_stride = cache->page_stride * 2;
  p.head_stride = cache->head_stride * 2;
  p.token_stride = cache->token_stride * 2;
  p.num_pages = cache->num_pages;
  p.kv_indices = kv_indices;
  p.num_kv_indices = num_kv_indices;
  p.kv_indptr = kv_indptr;
  p.batch = batch_size;
  p.page_size = cache->page_size;
  const int64_t per_token = static_cast<int64_t>(num_qo_heads + hkv) * (rotary_dim / 16) +
                            static_cast<int64_t>(hkv) * ((D - rotary_dim) / 8 + D / 8);
  const int64_t work = per_token * nnz;
  const int dev = current_device();
  const int64_t max_blocks = static_cast<int64_t>(sm_count(dev) > 0 ? sm_count(dev) : 148) * 8;
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, max_blocks));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cache->dtype == PA_DTYPE_BF16)
    return launch_chain(rope_append_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, p);
  return launch_chain(rope_append_kernel<__half>, dim3(blocks), dim3(256), 0, st, p);
}

int pa_build_decode_tables(const int32_t* block_tables, int64_t block_table_stride,
                           const int32_t* num_blocks, const int32_t* seq_lens, int32_t batch_size,
                           int32_t page_size, int32_t* kv_indptr, int32_t* kv_indices,
                           int64_t kv_indices_capacity, int32_t* kv_last_page_len,
                           int32_t* batch_indices, int32_t* positions, int32_t* counts,
                           void* stream) {
  if (batch_size < 0 || page_size <= 0 || block_table_stride < 0 || kv_indices_capacity < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (kv_indptr == nullptr || counts == nullptr) return PA_ERR_INVALID_ARGUMENT;
  if (batch_size > 0 && (block_tables == nullptr || num_blocks == nullptr || seq_lens == nullptr ||
                         kv_last_page_len == nullptr || batch_indices == nullptr ||
                         positions == nullptr || (kv_indices_capacity > 0 && kv_indices == nullptr)))
    return PA_ERR_INVALID_ARGUMENT;
  TablesParams p{};
  p.block_tables = block_tables;
  p.stride = block_table_stride;
  p.num_blocks = num_blocks;
  p.lens = seq_lens;
  p.batch = batch_size;
  p.page_size = page_size;
  p.prefill = 0;
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.kv_capacity = kv_indices_capacity;
  p.last_page_len = kv_last_page_len;
  p.batch_indices = batch_indices;
  p.positions = positions;
  p.rows_capacity = batch_size;
  p.counts = counts;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tables_scan_kernel<<<1, kTablesScanThreads, 0, st>>>(p);
  if (batch_size > 0) tables_gather_kernel<<<batch_size, 128, 0, st>>>(p);
  return launch_status();
}

int pa_build_prefill_tables(const int32_t* block_tables, int64_t block_table_stride,
                            const int32_t* num_blocks, const int32_t* prompt_lens,
                            const int32_t* computed_lens, const int32_t* chunk_lens,
                            int32_t batch_size, int32_t page_size, int32_t* qo_indptr,
                            int32_t* kv_indptr, int32_t* kv_indices, int64_t kv_indices_capacity,
                            int32_t* kv_last_page_len, int32_t* seq_lens, int32_t* active,
                            int32_t* batch_indices, int32_t* positions, int64_t rows_capacity,
                            int32_t* counts, void* stream) {
  if (batch_size < 0 || page_size <= 0 || block_table_stride < 0 || kv_indices_capacity < 0 ||
      rows_capacity < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (qo_indptr == nullptr || kv_indptr == nullptr || counts == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (batch_size > 0 &&
      (block_tables == nullptr || num_blocks == nullptr || prompt_lens == nullptr ||
       computed_lens == nullptr || chunk_lens == nullptr || kv_last_page_len == nullptr ||
       seq_lens == nullptr || active == nullptr ||
       (kv_indices_capacity > 0 && kv_indices == nullptr) ||
       (rows_capacity > 0 && (batch_indices == nullptr || positions == nullptr))))
    return PA_ERR_INVALID_ARGUMENT;
  TablesParams p{};
  p.block_tables = block_tables;
  p.stride = block_table_stride;
  p.num_blocks = num_blocks;
  p.lens = computed_lens;
  p.prompt_lens = prompt_lens;
  p.chunk_lens = chunk_lens;
  p.batch = batch_size;
  p.page_size = page_size;
  p.prefill = 1;
  p.qo_indptr = qo_indptr;
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.kv_capacity = kv_indices_capacity;
  p.last_page_len = kv_last_page_len;
  p.seq_lens_out = seq_lens;
  p.active = active;
  p.batch_indices = batch_indices;
  p.positions = positions;
  p.rows_capacity = rows_capacity;
  p.counts = counts;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tables_scan_kernel<<<1, kTablesScanThreads, 0, st>>>(p);
  if (batch_size > 0) tables_gather_kernel<<<batch_size, 128, 0, st>>>(p);
  return launch_status();
}

int pa_fork_pages(void* pool, int64_t layer_stride_bytes, int32_t num_layers,
                  int64_t page_stride_bytes, int64_t page_bytes, int64_t num_pages,
                  const int32_t* src_pages, const int32_t* dst_pages, int32_t num_pairs,
                  void* stream) {
  if (num_pairs < 0 || num_layers < 0 || num_pages < 0) return PA_ERR_INVALID_ARGUMENT;
  if (num_pairs == 0 || num_layers == 0 || page_bytes == 0) return PA_OK;
  if (pool == nullptr || src_pages == nullptr || dst_pages == nullptr) return PA_ERR_INVALID_ARGUMENT;
  if (!aligned16(pool) || page_bytes % 16 || page_stride_bytes % 16 || layer_stride_bytes % 16 ||
      page_bytes < 0 || page_bytes > page_stride_bytes)
    return PA_ERR_INVALID_ARGUMENT;
  ForkParams p;
  p.pool = static_cast<uint8_t*>(pool);
  p.layer_stride = layer_stride_bytes;
  p.page_stride = page_stride_bytes;
  p.page_bytes = page_bytes;
  p.num_layers = num_layers;
  p.num_pages = num_pages;
  p.src = src_pages;
  p.dst = dst_pages;
  p.n = num_pairs;
  const int64_t work = (page_bytes / 16) * num_layers * static_cast<int64_t>(num_pairs);
  const int dev = current_device();
  const int64_t max_blocks = static_cast<int64_t>(sm_count(dev) > 0 ? sm_count(dev) : 148) * 8;
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, max_blocks));
  fork_pages_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return launch_status();
}

int pa_qkv_rope_append(const void* x, int64_t x_stride, const void* weight, int64_t w_stride,
                       int32_t num_tokens, int32_t hidden, int32_t num_qo_heads, void* q_out,
                       int64_t q_stride_n, const int32_t* batch_indices, const int32_t* positions,
                       int32_t rotary_dim, int32_t interleave, float rope_scale, float rope_theta,
                       const pa_kv_cache* cache, const int32_t* kv_indices,
                       int64_t num_kv_indices, const int32_t* kv_indptr, int32_t batch_size,
                       void* stream) {
  if (num_tokens < 0 || hidden <= 0 || num_qo_heads <= 0 || batch_size < 0 ||
      num_kv_indices < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return PA_OK;
  if (x == nullptr || weight == nullptr || q_out == nullptr || cache == nullptr ||
      batch_indices == nullptr || positions == nullptr || kv_indices == nullptr ||
      kv_indptr == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(cache->dtype)) return PA_ERR_UNSUPPORTED;
  const int D = cache->head_dim, hkv = cache->num_kv_heads;
  if (D != 64 && D != 128) return PA_ERR_UNSUPPORTED;
  if (cache->k_base == nullptr || cache->v_base == nullptr || cache->page_size <= 0 || hkv <= 0)
    return PA_ERR_INVALID_ARGUMENT;
  // tiles of 128 columns never straddle the q / k / v column ranges
  if ((num_qo_heads * D) % 128 || (hkv * D) % 128 || hidden % kQkvBK)
    return PA_ERR_UNSUPPORTED;
  if (rotary_dim <= 0 || rotary_dim % 2 || rotary_dim > D) return PA_ERR_INVALID_ARGUMENT;
  if (!(rope_scale > 0.f) || !(rope_theta > 0.f)) return PA_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(weight) || !aligned16(q_out) || !aligned16(cache->k_base) ||
      !aligned16(cache->v_base) || x_stride % 8 || w_stride % 8 || q_stride_n % 8 ||
      x_stride < hidden || w_stride < hidden || q_stride_n < static_cast<int64_t>(num_qo_heads) * D ||
      cache->page_stride % 8 || cache->head_stride % 8 || cache->token_stride % 8)
    return PA_ERR_INVALID_ARGUMENT;
  const int64_t N = static_cast<int64_t>(num_qo_heads + 2 * hkv) * D;
  CUtensorMap xm, wm;
  int rc = encode_2d_map(&xm, x, num_tokens, hidden, x_stride, kQkvBM, cache->dtype);
  if (rc != PA_OK) return rc;
  QkvParams p;
  p.M = num_tokens;
  p.K = hidden;
  p.hq = num_qo_heads;
  p.hkv = hkv;
  p.head_dim = D;
  p.q_out = static_cast<uint8_t*>(q_out);
  p.q_sn = q_stride_n * 2;
  p.batch_indices = batch_indices;
  p.positions = positions;
  p.rotary_dim = rotary_dim;
  p.interleave = interleave ? 1 : 0;
  p.inv_scale = 1.0f / rope_scale;
  p.log2_theta = std::log2(rope_theta);
  p.k_base = static_cast<uint8_t*>(const_cast<void*>(cache->k_base));
  p.v_base = static_cast<uint8_t*>(const_cast<void*>(cache->v_base));
  p.page_stride = cache->page_stride * 2;
  p.head_stride = cache->head_stride * 2;
  p.token_stride = cache->token_stride * 2;
  p.num_pages = cache->num_pages;
  p.kv_indices = kv_indices;
  p.num_kv_indices = num_kv_indices;
  p.kv_indptr = kv_indptr;
  p.batch = batch_size;
  p.page_size = cache->page_size;
  const int dev = current_device();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // few tokens: weight-streaming tiles (N=128, 6 stages); many: N=256
  const bool wide = num_tokens > 512 && N % 256 == 0 && (num_qo_heads * D) % 256 == 0 &&
                    (hkv * D) % 256 == 0;
  const int bn = wide ? 256 : 128;
  rc = encode_2d_map(&wm, weight, N, hidden, w_stride, bn, cache->dtype);
  if (rc != PA_OK) return rc;
  const int mt = (num_tokens + kQkvBM - 1) / kQkvBM, nt = static_cast<int>(N / bn);
  const dim3 grid(static_cast<unsigned>(mt), static_cast<unsigned>(nt));
  const bool bf = cache->dtype == PA_DTYPE_BF16;
  p.splits = 1;
  auto go = [&](auto kernel, int smem, std::atomic<uint64_t>* done) -> int {
    if (allow_smem(kernel, smem, done, dev) != cudaSuccess) return PA_ERR_CUDA;
    kernel<<<grid, kQkvThreads, smem, st>>>(xm, wm, p);
    return launch_status();
  };
  // Few tiles (decode-sized batches): split K over a cluster of 2-4 CTAs
  // per tile so that the weight streams through (nearly) every SM, as long
  // as every cluster fits on the GPU at once.
  auto go_split = [&](auto kernel, std::atomic<uint64_t>* done, int vi) -> int {
    using SK = QkvCfg<128, 5, true>;
    if (allow_smem(kernel, SK::kSmemBytes, done, dev) != cudaSuccess) return PA_ERR_CUDA;
    static std::atomic<int> fits[4][5];  // clusters resident at once, by variant and size; 0 = unknown
    const int sms = sm_count(dev) > 0 ? sm_count(dev) : 148;
    int splits = std::min(4, sms / (mt * nt));
    while (splits > 1 && hidden / kQkvBK < 4 * splits) --splits;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    cfg.blockDim = dim3(kQkvThreads);
    cfg.dynamicSmemBytes = SK::kSmemBytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    for (; splits > 1; --splits) {
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = static_cast<unsigned>(splits);
      cfg.gridDim = dim3(static_cast<unsigned>(mt), static_cast<unsigned>(nt),
                         static_cast<unsigned>(splits));
      int n = fits[vi][splits].load(std::memory_order_relaxed);
      if (n == 0) {
        if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
          (void)cudaGetLastError();
          n = -1;
        }
        fits[vi][splits].store(n == 0 ? -1 : n, std::memory_order_relaxed);
      }
      if (n >= mt * nt) break;
    }
    if (splits < 2) return -1;  // not worth it: the one-CTA-per-tile kernel
    p.splits = splits;
    if (cudaLaunchKernelEx(&cfg, kernel, xm, wm, p) != cudaSuccess) return PA_ERR_CUDA;
    return launch_status();
  };
  static std::atomic<uint64_t> done[12];
  using N6 = QkvCfg<128, 6>;
  using W2 = QkvCfg<256, 2>;
  if (!wide) {
    int rs = -1;
    if (bf && D == 64) rs = go_split(qkv_rope_append_kernel<__nv_bfloat16, 64, 128, 5, true>, &done[8], 0);
    else if (bf) rs = go_split(qkv_rope_append_kernel<__nv_bfloat16, 128, 128, 5, true>, &done[9], 1);
    else if (D == 64) rs = go_split(qkv_rope_append_kernel<__half, 64, 128, 5, true>, &done[10], 2);
    else rs = go_split(qkv_rope_append_kernel<__half, 128, 128, 5, true>, &done[11], 3);
    if (rs != -1) return rs;
  }
  if (bf && D == 64)
    return wide ? go(qkv_rope_append_kernel<__nv_bfloat16, 64, 256, 2, false>, W2::kSmemBytes, &done[0])
                : go(qkv_rope_append_kernel<__nv_bfloat16, 64, 128, 6, false>, N6::kSmemBytes, &done[1]);
  if (bf)
    return wide ? go(qkv_rope_append_kernel<__nv_bfloat16, 128, 256, 2, false>, W2::kSmemBytes, &done[2])
                : go(qkv_rope_append_kernel<__nv_bfloat16, 128, 128, 6, false>, N6::kSmemBytes, &done[3]);
  if (D == 64)
    return wide ? go(qkv_rope_append_kernel<__half, 64, 256, 2, false>, W2::kSmemBytes, &done[4])
                : go(qkv_rope_append_kernel<__half, 64, 128, 6, false>, N6::kSmemBytes, &done[5]);
  return wide ? go(qkv_rope_append_kernel<__half, 128, 256, 2, false>, W2::kSmemBytes, &done[6])
              : go(qkv_rope_append_kernel<__half, 128, 128, 6, false>, N6::kSmemBytes, &done[7]);
}

int pa_selftest_wait_timeout(int64_t limit_cycles, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > kWaitLimitCycles) return PA_ERR_INVALID_ARGUMENT;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_cycles);
  return launch_status();
}

size_t pa_decode_workspace_bytes(int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads,
                                 int32_t head_dim) {
  (void)num_qo_heads;
  const int dev = current_device();
  if (dev < 0 || batch_size < 0 || num_kv_heads <= 0 || head_dim <= 0) return 0;
  DecodePlanShape sh;
  if (!decode_shape(dev, num_kv_heads, head_dim, &sh)) return 0;
  return decode_ws_bytes(sh, batch_size, num_kv_heads, head_dim);
}

int pa_decode_plan(const int32_t* kv_indptr, const int32_t* kv_last_page_len, int32_t batch_size,
                   int64_t num_kv_indices, int32_t num_qo_heads, int32_t num_kv_heads,
                   int32_t head_dim, int32_t page_size, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (kv_indptr == nullptr || kv_last_page_len == nullptr || workspace == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (batch_size <= 0 || num_kv_indices < 0 || num_qo_heads <= 0 || num_kv_heads <= 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (num_qo_heads % num_kv_heads) return PA_ERR_INVALID_ARGUMENT;
  if (num_qo_heads / num_kv_heads > kMaxGroup) return PA_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return PA_ERR_UNSUPPORTED;
  if (page_size != kPage) return PA_ERR_UNSUPPORTED;
  if (!aligned16(workspace)) return PA_ERR_INVALID_ARGUMENT;
  const int dev = current_device();
  DecodePlanShape sh;
  if (!decode_shape(dev, num_kv_heads, head_dim, &sh))
    return dev < 0 ? PA_ERR_CUDA : PA_ERR_UNSUPPORTED;
  if (decode_ws_bytes(sh, batch_size, num_kv_heads, head_dim) > workspace_bytes)
    return PA_ERR_WORKSPACE_TOO_SMALL;
  return launch_chain(decode_plan_kernel, dim3(1), dim3(1024), 0,
                      static_cast<cudaStream_t>(stream), kv_indptr, kv_last_page_len, batch_size,
                      num_kv_heads, num_qo_heads, head_dim, page_size, num_kv_indices, sh.units,
                      sh.g.hb, /*min_per_group=*/4, static_cast<uint8_t*>(workspace));
}

}  // extern "C"

namespace {

// Decode-step append rows handed to decode_run (nullptr: plain decode).
struct DecodeAppend {
  const void* key;
  int64_t key_stride_n, key_stride_h;
  const void* value;
  int64_t value_stride_n, value_stride_h;
  const int32_t* positions;
  const int32_t* pos_base;  // device word subtracted from each position, or nullptr
};

int decode_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
               const int32_t* kv_indices, const int32_t* kv_indptr,
               const int32_t* kv_last_page_len, int32_t batch_size, int32_t num_qo_heads,
               float sm_scale, void* workspace, size_t workspace_bytes, void* out, float* lse,
               void* stream, const DecodeAppend* app) {
  int st = check_cache(cache);
  if (st != PA_OK) return st;
  if (q == nullptr || out == nullptr || kv_indices == nullptr || kv_indptr == nullptr ||
      kv_last_page_len == nullptr || workspace == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (batch_size <= 0 || num_qo_heads <= 0) return PA_ERR_INVALID_ARGUMENT;
  const int hkv = cache->num_kv_heads, D = cache->head_dim;
  if (num_qo_heads % hkv) return PA_ERR_INVALID_ARGUMENT;
  const int G = num_qo_heads / hkv;
  if (G > kMaxGroup) return PA_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return PA_ERR_UNSUPPORTED;
  if (cache->page_size != kPage) return PA_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(out) || q_stride_n % 8 || q_stride_h % 8)
    return PA_ERR_INVALID_ARGUMENT;
  const int dev = current_device();
  DecodePlanShape sh;
  if (!decode_shape(dev, hkv, D, &sh)) return dev < 0 ? PA_ERR_CUDA : PA_ERR_UNSUPPORTED;
  const DecodeWsLayout L = decode_ws_layout(sh.units, batch_size, hkv, D, sh.g.hb);
  if (L.total > workspace_bytes) return PA_ERR_WORKSPACE_TOO_SMALL;
  CUtensorMap km, vm;
  if ((st = encode_kv_map(&km, cache->k_base, *cache, kPage, sh.g.hb)) != PA_OK) return st;
  if ((st = encode_kv_map(&vm, cache->v_base, *cache, kPage, sh.g.hb)) != PA_OK) return st;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DecodeParams p;
  p.q = q;
  p.q_stride_n = q_stride_n;
  p.q_stride_h = q_stride_h;
  p.out = out;
  p.lse = lse;
  p.kv_indices = kv_indices;
  p.kv_indptr = kv_indptr;
  p.kv_last_page_len = kv_last_page_len;
  p.batch_size = batch_size;
  p.num_qo_heads = num_qo_heads;
  p.num_kv_heads = hkv;
  p.group = G;
  p.num_pages = cache->num_pages;
  p.heads_inner = heads_inner(*cache) ? 1 : 0;
  const float scale = sm_scale > 0.f ? sm_scale : 1.0f / std::sqrt(static_cast<float>(D));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.hdr = reinterpret_cast<const DecodePlanHeader*>(ws + L.hdr);
  p.unit_start = reinterpret_cast<const int4*>(ws + L.unit_start);
  p.hb = sh.g.hb;
  p.nhb = sh.g.nhb;
  p.groups_per_cta = sh.g.groups_per_cta;
  p.stages = sh.g.stages;
  p.stage_bytes = sh.g.stage_bytes;
  p.empty = reinterpret_cast<const int32_t*>(ws + L.empty);
  p.counter = reinterpret_cast<int32_t*>(ws + L.counter);
  p.part_lse = reinterpret_cast<float*>(ws + L.part_lse);
  p.part_o = reinterpret_cast<float*>(ws + L.part_o);
  p.append_pos = nullptr;
  p.append_pos_base = nullptr;
  p.new_k = p.new_v = nullptr;
  p.new_k_stride_n = p.new_k_stride_h = p.new_v_stride_n = p.new_v_stride_h = 0;
  p.k_pool = p.v_pool = nullptr;
  p.pool_page_stride = p.pool_head_stride = p.pool_token_stride = 0;
  if (app != nullptr) {
    const int esz = 2;  // bf16 / fp16
    p.append_pos = app->positions;
    p.append_pos_base = app->pos_base;
    p.new_k = static_cast<const uint8_t*>(app->key);
    p.new_v = static_cast<const uint8_t*>(app->value);
    p.new_k_stride_n = app->key_stride_n * esz;
    p.new_k_stride_h = app->key_stride_h * esz;
    p.new_v_stride_n = app->value_stride_n * esz;
    p.new_v_stride_h = app->value_stride_h * esz;
    // the descriptor's bases are const for the read-only entry points; the
    // append writes through them as pa_append_paged_kv_cache does
    p.k_pool = const_cast<uint8_t*>(static_cast<const uint8_t*>(cache->k_base));
    p.v_pool = const_cast<uint8_t*>(static_cast<const uint8_t*>(cache->v_base));
    p.pool_page_stride = cache->page_stride * esz;
    p.pool_head_stride = cache->head_stride * esz;
    p.pool_token_stride = cache->token_stride * esz;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cache->dtype == PA_DTYPE_BF16)
    return D == 64 ? launch_decode<__nv_bfloat16, 64>(km, vm, p, sh, dev, s)
                   : launch_decode<__nv_bfloat16, 128>(km, vm, p, sh, dev, s);
  return D == 64 ? launch_decode<__half, 64>(km, vm, p, sh, dev, s)
                 : launch_decode<__half, 128>(km, vm, p, sh, dev, s);
}

}  // namespace

extern "C" {

int pa_decode_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
                  const int32_t* kv_indices, const int32_t* kv_indptr,
                  const int32_t* kv_last_page_len, int32_t batch_size, int32_t num_qo_heads,
                  float sm_scale, void* workspace, size_t workspace_bytes, void* out, float* lse,
                  void* stream) {
  return decode_run(q, q_stride_n, q_stride_h, cache, kv_indices, kv_indptr, kv_last_page_len,
                    batch_size, num_qo_heads, sm_scale, workspace, workspace_bytes, out, lse,
                    stream, nullptr);
}

int pa_decode_append_run(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                         const void* append_key, int64_t key_stride_n, int64_t key_stride_h,
                         const void* append_value, int64_t value_stride_n,
                         int64_t value_stride_h, const int32_t* positions,
                         const pa_kv_cache* cache, const int32_t* kv_indices,
                         const int32_t* kv_indptr, const int32_t* kv_last_page_len,
                         int32_t batch_size, int32_t num_qo_heads, float sm_scale,
                         void* workspace, size_t workspace_bytes, void* out, float* lse,
                         void* stream) {
  if (append_key == nullptr || append_value == nullptr || positions == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (!aligned16(append_key) || !aligned16(append_value) || key_stride_n % 8 ||
      key_stride_h % 8 || value_stride_n % 8 || value_stride_h % 8)
    return PA_ERR_INVALID_ARGUMENT;
  const DecodeAppend app{append_key, key_stride_n, key_stride_h, append_value,
                         value_stride_n, value_stride_h, positions, nullptr};
  return decode_run(q, q_stride_n, q_stride_h, cache, kv_indices, kv_indptr, kv_last_page_len,
                    batch_size, num_qo_heads, sm_scale, workspace, workspace_bytes, out, lse,
                    stream, &app);
}

int pa_merge_states(const void* v, const float* s, int32_t seq_len, int32_t num_states,
                    int32_t num_heads, int32_t head_dim, int32_t dtype, void* v_merged,
                    float* s_merged, void* stream) {
  if (seq_len < 0 || num_states <= 0 || num_heads <= 0 || head_dim <= 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (seq_len == 0) return PA_OK;
  if (v == nullptr || s == nullptr || v_merged == nullptr) return PA_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(dtype)) return PA_ERR_UNSUPPORTED;
  const int64_t items = static_cast<int64_t>(seq_len) * num_heads;
  const int blocks = static_cast<int>((items + 7) / 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == PA_DTYPE_BF16)
    merge_states_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(v), s, seq_len, num_states, num_heads, head_dim,
        static_cast<__nv_bfloat16*>(v_merged), s_merged);
  else
    merge_states_kernel<__half><<<blocks, 256, 0, st>>>(
        static_cast<const __half*>(v), s, seq_len, num_states, num_heads, head_dim,
        static_cast<__half*>(v_merged), s_merged);
  return launch_status();
}

size_t pa_prefill_workspace_bytes(int32_t batch_size, int64_t max_total_qo, int32_t num_qo_heads,
                                  int32_t num_kv_heads, int32_t head_dim) {
  if (batch_size <= 0 || max_total_qo < 0 || num_kv_heads <= 0 || num_qo_heads <= 0 ||
      num_qo_heads % num_kv_heads || head_dim <= 0)
    return 0;
  const int span = prefill_span(num_qo_heads / num_kv_heads);
  if (span == 0) return 0;
  return prefill_ws_layout(prefill_max_items(batch_size, max_total_qo, num_kv_heads, span)).total;
}

int pa_prefill_plan(const int32_t* qo_indptr, const int32_t* kv_indptr,
                    const int32_t* kv_last_page_len, int32_t batch_size, int64_t total_qo,
                    int64_t num_kv_indices, int32_t num_qo_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t page_size, void* workspace, size_t workspace_bytes,
                    void* stream) {
  if (qo_indptr == nullptr || kv_indptr == nullptr || kv_last_page_len == nullptr ||
      workspace == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (batch_size <= 0 || total_qo < 0 || num_kv_indices < 0 || num_qo_heads <= 0 ||
      num_kv_heads <= 0 || num_qo_heads % num_kv_heads)
    return PA_ERR_INVALID_ARGUMENT;
  const int span = prefill_span(num_qo_heads / num_kv_heads);
  if (span == 0) return PA_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return PA_ERR_UNSUPPORTED;
  if (page_size != kPage) return PA_ERR_UNSUPPORTED;
  if (!aligned16(workspace)) return PA_ERR_INVALID_ARGUMENT;
  const int64_t max_items = prefill_max_items(batch_size, total_qo, num_kv_heads, span);
  if (prefill_ws_layout(max_items).total > workspace_bytes) return PA_ERR_WORKSPACE_TOO_SMALL;
  // one thread per cost bucket (the plan's scan relies on it)
  prefill_plan_kernel<<<1, kPfCostBuckets, 0, static_cast<cudaStream_t>(stream)>>>(
      qo_indptr, kv_indptr, kv_last_page_len, batch_size, total_qo, num_kv_indices, num_qo_heads,
      num_kv_heads, head_dim, page_size, span, max_items, static_cast<uint8_t*>(workspace));
  return launch_status();
}

int pa_prefill_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
                   const int32_t* qo_indptr, const int32_t* kv_indices, const int32_t* kv_indptr,
                   const int32_t* kv_last_page_len, int32_t batch_size, int64_t total_qo,
                   int32_t num_qo_heads, int32_t causal, float sm_scale, void* workspace,
                   size_t workspace_bytes, void* out, float* lse, void* stream) {
  int st = check_cache(cache);
  if (st != PA_OK) return st;
  if (q == nullptr || out == nullptr || qo_indptr == nullptr || kv_indices == nullptr ||
      kv_indptr == nullptr || kv_last_page_len == nullptr || workspace == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (batch_size <= 0 || total_qo < 0 || num_qo_heads <= 0) return PA_ERR_INVALID_ARGUMENT;
  const int hkv = cache->num_kv_heads, D = cache->head_dim;
  if (num_qo_heads % hkv) return PA_ERR_INVALID_ARGUMENT;
  const int G = num_qo_heads / hkv;
  const int qt = prefill_qt(G);
  if (qt == 0) return PA_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return PA_ERR_UNSUPPORTED;
  if (cache->page_size != kPage) return PA_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(out) || q_stride_n % 8 || q_stride_h % 8)
    return PA_ERR_INVALID_ARGUMENT;
  if (total_qo == 0) return PA_OK;
  const int64_t max_items = prefill_max_items(batch_size, total_qo, hkv, 2 * qt);
  const PrefillWsLayout L = prefill_ws_layout(max_items);
  if (L.total > workspace_bytes) return PA_ERR_WORKSPACE_TOO_SMALL;
  CUtensorMap qm, km, vm, om;
  if ((st = encode_q_map(&qm, q, q_stride_n, q_stride_h, total_qo, num_qo_heads, D, G, qt,
                         cache->dtype)) != PA_OK)
    return st;
  // out [total_qo, num_qo_heads, head_dim]: the q map's shape and boxes
  if ((st = encode_q_map(&om, out, static_cast<int64_t>(num_qo_heads) * D, D, total_qo,
                         num_qo_heads, D, G, qt, cache->dtype)) != PA_OK)
    return st;
  if ((st = encode_kv_map(&km, cache->k_base, *cache, kPage, 1)) != PA_OK) return st;
  if ((st = encode_kv_map(&vm, cache->v_base, *cache, kPage, 1)) != PA_OK) return st;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  PrefillParams p;
  p.out = out;
  p.lse = lse;
  p.qo_indptr = qo_indptr;
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.kv_last_page_len = kv_last_page_len;
  p.batch_size = batch_size;
  p.num_qo_heads = num_qo_heads;
  p.num_kv_heads = hkv;
  p.group = G;
  p.qt = qt;
  p.causal = causal ? 1 : 0;
  p.num_pages = cache->num_pages;
  p.heads_inner = heads_inner(*cache) ? 1 : 0;
  const float scale = sm_scale > 0.f ? sm_scale : 1.0f / std::sqrt(static_cast<float>(D));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.hdr = reinterpret_cast<const PrefillPlanHeader*>(ws + L.hdr);
  p.items = reinterpret_cast<const int4*>(ws + L.items);
  p.sched = reinterpret_cast<int32_t*>(ws + L.hdr + offsetof(PrefillPlanHeader, next_item));
  p.q_rows = nullptr;
  const int dev = current_device();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cache->dtype == PA_DTYPE_BF16)
    return D == 64 ? launch_prefill<__nv_bfloat16, 64>(qm, km, vm, om, p, max_items, dev, s)
                   : launch_prefill<__nv_bfloat16, 128>(qm, km, vm, om, p, max_items, dev, s);
  return D == 64 ? launch_prefill<__half, 64>(qm, km, vm, om, p, max_items, dev, s)
                 : launch_prefill<__half, 128>(qm, km, vm, om, p, max_items, dev, s);
}

}  // extern "C"

namespace {

// Cascade geometry for a batch: level-0 chunk count sized so the chunks'
// prefill items fill the SMs once, the decode partition of level 1, and the
// workspace layout of both.
struct CascadeShape {
  int qt, span, max_chunks;
  DecodePlanShape dec;
  CascadeWsLayout L;
};

bool cascade_shape(int dev, int batch, int hq, int hkv, int head_dim, CascadeShape* s) {
  if (batch <= 0 || hq <= 0 || hkv <= 0 || hq % hkv) return false;
  if (!decode_shape(dev, hkv, head_dim, &s->dec)) return false;
  s->qt = prefill_qt(hq / hkv);
  if (s->qt == 0) return false;
  s->span = 2 * s->qt;
  const int nq = (batch + s->span - 1) / s->span;
  const int per_chunk = hkv * nq;
  // level-0 items fill the SMs once (fewer, longer chunks lengthen each
  // CTA's chain more than they shorten the merge)
  const int target = std::max(1, s->dec.ctas);
  s->max_chunks = std::max(1, std::min((target + per_chunk - 1) / per_chunk, kCascadeMaxChunks));
  s->L = cascade_ws_layout(batch, hq, hkv, head_dim, s->max_chunks, s->span, s->dec.units,
                           s->dec.g.hb);
  return true;
}

template <typename T, int D>
int launch_cascade_merge(const CascadeWsLayout& L, uint8_t* ws, int batch, int hq, void* out,
                         float* lse, cudaStream_t s) {
  const int64_t threads = static_cast<int64_t>(batch) * hq * 32;
  const int blocks = static_cast<int>((threads + 255) / 256);
  return launch_chain(cascade_merge_kernel<T, D>, dim3(blocks), dim3(256), 0, s,
                      reinterpret_cast<const T*>(ws + L.o0),
                      reinterpret_cast<const float*>(ws + L.lse0),
                      reinterpret_cast<const T*>(ws + L.o1),
                      reinterpret_cast<const float*>(ws + L.lse1),
                      reinterpret_cast<const CascadeHeader*>(ws + L.hdr), batch, hq,
                      static_cast<T*>(out), lse);
}

}  // namespace

extern "C" {

size_t pa_cascade_workspace_bytes(int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads,
                                  int32_t head_dim) {
  CascadeShape sh;
  if (!cascade_shape(current_device(), batch_size, num_qo_heads, num_kv_heads, head_dim, &sh))
    return 0;
  return sh.L.total;
}

int pa_cascade_plan(const int32_t* shared_kv_indptr, const int32_t* shared_kv_last_page_len,
                    int64_t num_shared_indices, const int32_t* unique_kv_indptr,
                    const int32_t* unique_kv_last_page_len, int32_t batch_size,
                    int64_t num_unique_indices, int32_t num_qo_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t page_size, void* workspace, size_t workspace_bytes,
                    void* stream) {
  if (shared_kv_indptr == nullptr || shared_kv_last_page_len == nullptr ||
      unique_kv_indptr == nullptr || unique_kv_last_page_len == nullptr || workspace == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (batch_size <= 0 || num_unique_indices < 0 || num_shared_indices < 0 || num_qo_heads <= 0 ||
      num_kv_heads <= 0 || num_qo_heads % num_kv_heads)
    return PA_ERR_INVALID_ARGUMENT;
  if (num_qo_heads / num_kv_heads > kMaxGroup) return PA_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return PA_ERR_UNSUPPORTED;
  if (page_size != kPage) return PA_ERR_UNSUPPORTED;
  if (!aligned16(workspace)) return PA_ERR_INVALID_ARGUMENT;
  CascadeShape sh;
  if (!cascade_shape(current_device(), batch_size, num_qo_heads, num_kv_heads, head_dim, &sh))
    return PA_ERR_UNSUPPORTED;
  if (sh.L.total > workspace_bytes) return PA_ERR_WORKSPACE_TOO_SMALL;
  return launch_chain(cascade_plan_kernel, dim3(1), dim3(1024), 0,
                      static_cast<cudaStream_t>(stream), shared_kv_indptr,
                      shared_kv_last_page_len, num_shared_indices, unique_kv_indptr,
                      unique_kv_last_page_len,
                      num_unique_indices, batch_size, num_qo_heads, num_kv_heads, head_dim,
                      page_size, sh.qt, sh.max_chunks, sh.dec.units, sh.dec.g.hb,
                      static_cast<uint8_t*>(workspace), sh.L);
}

}  // extern "C"

namespace {

// Level 0 (prefill over the prefix chunks), level 1 (decode over the unique
// pages, with the step's append fused in when `app` is given), merge.
int cascade_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
                const int32_t* shared_kv_indices, const int32_t* unique_kv_indices,
                const int32_t* unique_kv_indptr, const int32_t* unique_kv_last_page_len,
                int32_t batch_size, int32_t num_qo_heads, float sm_scale, void* workspace,
                size_t workspace_bytes, void* out, float* lse, void* stream,
                const DecodeAppend* app) {
  int st = check_cache(cache);
  if (st != PA_OK) return st;
  if (q == nullptr || out == nullptr || shared_kv_indices == nullptr ||
      unique_kv_indices == nullptr || unique_kv_indptr == nullptr ||
      unique_kv_last_page_len == nullptr || workspace == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  const int hkv = cache->num_kv_heads, D = cache->head_dim;
  if (batch_size <= 0 || num_qo_heads <= 0 || num_qo_heads % hkv) return PA_ERR_INVALID_ARGUMENT;
  if (D != 64 && D != 128) return PA_ERR_UNSUPPORTED;
  if (cache->page_size != kPage) return PA_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(out) || q_stride_n % 8 || q_stride_h % 8)
    return PA_ERR_INVALID_ARGUMENT;
  const int dev = current_device();
  CascadeShape sh;
  if (!cascade_shape(dev, batch_size, num_qo_heads, hkv, D, &sh)) return PA_ERR_UNSUPPORTED;
  const CascadeWsLayout& L = sh.L;
  if (L.total > workspace_bytes) return PA_ERR_WORKSPACE_TOO_SMALL;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int G = num_qo_heads / hkv;
  // ---- level 0: the shared prefix, key chunks as non-causal prefill requests
  CUtensorMap qm, km, vm, om;
  if ((st = encode_q_map(&qm, q, q_stride_n, q_stride_h, batch_size, num_qo_heads, D, G, sh.qt,
                         cache->dtype)) != PA_OK)
    return st;
  // level-0 states: one [batch, num_qo_heads, head_dim] block per key chunk
  if ((st = encode_q_map(&om, ws + L.o0, static_cast<int64_t>(num_qo_heads) * D, D,
                         static_cast<int64_t>(sh.max_chunks) * batch_size, num_qo_heads, D, G,
                         sh.qt, cache->dtype)) != PA_OK)
    return st;
  if ((st = encode_kv_map(&km, cache->k_base, *cache, kPage, 1)) != PA_OK) return st;
  if ((st = encode_kv_map(&vm, cache->v_base, *cache, kPage, 1)) != PA_OK) return st;
  const PrefillWsLayout PL = prefill_ws_layout(L.prefill_items);
  PrefillParams p;
  p.out = ws + L.o0;
  p.lse = reinterpret_cast<float*>(ws + L.lse0);
  p.qo_indptr = reinterpret_cast<const int32_t*>(ws + L.qo_indptr);
  p.kv_indptr = reinterpret_cast<const int32_t*>(ws + L.kv_indptr);
  p.kv_indices = shared_kv_indices;
  p.kv_last_page_len = reinterpret_cast<const int32_t*>(ws + L.last);
  p.batch_size = sh.max_chunks;
  p.num_qo_heads = num_qo_heads;
  p.num_kv_heads = hkv;
  p.group = G;
  p.qt = sh.qt;
  p.causal = 0;
  p.num_pages = cache->num_pages;
  p.heads_inner = heads_inner(*cache) ? 1 : 0;
  const float scale = sm_scale > 0.f ? sm_scale : 1.0f / std::sqrt(static_cast<float>(D));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.hdr = reinterpret_cast<const PrefillPlanHeader*>(ws + L.prefill + PL.hdr);
  p.items = reinterpret_cast<const int4*>(ws + L.prefill + PL.items);
  p.sched = reinterpret_cast<int32_t*>(ws + L.prefill + PL.hdr +
                                       offsetof(PrefillPlanHeader, next_item));
  p.q_rows = reinterpret_cast<const int32_t*>(ws + L.q_rows);
  const bool bf16 = cache->dtype == PA_DTYPE_BF16;
  st = bf16 ? (D == 64 ? launch_prefill<__nv_bfloat16, 64>(qm, km, vm, om, p, L.prefill_items,
                                                            dev, s)
                       : launch_prefill<__nv_bfloat16, 128>(qm, km, vm, om, p, L.prefill_items,
                                                             dev, s))
            : (D == 64 ? launch_prefill<__half, 64>(qm, km, vm, om, p, L.prefill_items, dev, s)
                       : launch_prefill<__half, 128>(qm, km, vm, om, p, L.prefill_items, dev, s));
  if (st != PA_OK) return st;
  // ---- level 1: each request's unique pages (positions of an appended token
  // are global; the plan recorded the prefix length they are taken from)
  DecodeAppend app1;
  if (app != nullptr) {
    app1 = *app;
    app1.pos_base = reinterpret_cast<const int32_t*>(ws + L.hdr +
                                                     offsetof(CascadeHeader, prefix_tokens));
  }
  st = decode_run(q, q_stride_n, q_stride_h, cache, unique_kv_indices, unique_kv_indptr,
                  unique_kv_last_page_len, batch_size, num_qo_heads, sm_scale, ws + L.decode,
                  L.o0 - L.decode, ws + L.o1, reinterpret_cast<float*>(ws + L.lse1), stream,
                  app != nullptr ? &app1 : nullptr);
  if (st != PA_OK) return st;
  // ---- merge
  return bf16 ? (D == 64 ? launch_cascade_merge<__nv_bfloat16, 64>(L, ws, batch_size,
                                                                   num_qo_heads, out, lse, s)
                         : launch_cascade_merge<__nv_bfloat16, 128>(L, ws, batch_size,
                                                                    num_qo_heads, out, lse, s))
              : (D == 64 ? launch_cascade_merge<__half, 64>(L, ws, batch_size, num_qo_heads, out,
                                                            lse, s)
                         : launch_cascade_merge<__half, 128>(L, ws, batch_size, num_qo_heads,
                                                             out, lse, s));
}

}  // namespace

extern "C" {

int pa_cascade_run(const void* q, int64_t q_stride_n, int64_t q_stride_h, const pa_kv_cache* cache,
                   const int32_t* shared_kv_indices, const int32_t* unique_kv_indices,
                   const int32_t* unique_kv_indptr, const int32_t* unique_kv_last_page_len,
                   int32_t batch_size, int32_t num_qo_heads, float sm_scale, void* workspace,
                   size_t workspace_bytes, void* out, float* lse, void* stream) {
  return cascade_run(q, q_stride_n, q_stride_h, cache, shared_kv_indices, unique_kv_indices,
                     unique_kv_indptr, unique_kv_last_page_len, batch_size, num_qo_heads,
                     sm_scale, workspace, workspace_bytes, out, lse, stream, nullptr);
}

int pa_cascade_append_run(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                          const void* append_key, int64_t key_stride_n, int64_t key_stride_h,
                          const void* append_value, int64_t value_stride_n,
                          int64_t value_stride_h, const int32_t* positions,
                          const pa_kv_cache* cache, const int32_t* shared_kv_indices,
                          const int32_t* unique_kv_indices, const int32_t* unique_kv_indptr,
                          const int32_t* unique_kv_last_page_len, int32_t batch_size,
                          int32_t num_qo_heads, float sm_scale, void* workspace,
                          size_t workspace_bytes, void* out, float* lse, void* stream) {
  if (append_key == nullptr || append_value == nullptr || positions == nullptr)
    return PA_ERR_INVALID_ARGUMENT;
  if (!aligned16(append_key) || !aligned16(append_value) || key_stride_n % 8 ||
      key_stride_h % 8 || value_stride_n % 8 || value_stride_h % 8)
    return PA_ERR_INVALID_ARGUMENT;
  const DecodeAppend app{append_key, key_stride_n, key_stride_h, append_value,
                         value_stride_n, value_stride_h, positions, nullptr};
  return cascade_run(q, q_stride_n, q_stride_h, cache, shared_kv_indices, unique_kv_indices,
                     unique_kv_indptr, unique_kv_last_page_len, batch_size, num_qo_heads,
                     sm_scale, workspace, workspace_bytes, out, lse, stream, &app);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode: the same plan and run kernels with their scratch in
// a static device array instead of a caller workspace.
namespace {

__device__ __align__(256) uint8_t g_noalloc_scratch[PA_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch for device `dev`, looked up once per
// device with that device current. In host code the symbol itself is only a
// host-side stand-in, never a device address.
void* noalloc_scratch(int dev) {
  static std::atomic<void*> addr[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  void* p = addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return nullptr;
    addr[dev].store(p, std::memory_order_release);
  }
  return p;
}

}  // namespace

extern "C" int pa_decode_noalloc(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                                 const pa_kv_cache* cache, const int32_t* kv_indices,
                                 const int32_t* kv_indptr, const int32_t* kv_last_page_len,
                                 int32_t batch_size, int64_t num_kv_indices, int32_t num_qo_heads,
                                 float sm_scale, void* out, float* lse, void* stream) {
  int st = check_cache(cache);
  if (st != PA_OK) return st;
  if (batch_size <= 0 || num_qo_heads <= 0) return PA_ERR_INVALID_ARGUMENT;
  const int dev = current_device();
  DecodePlanShape sh;
  if (!decode_shape(dev, cache->num_kv_heads, cache->head_dim, &sh))
    return dev < 0 ? PA_ERR_CUDA : PA_ERR_UNSUPPORTED;
  const size_t need = decode_ws_bytes(sh, batch_size, cache->num_kv_heads, cache->head_dim);
  if (need > PA_NOALLOC_SCRATCH_BYTES) return PA_ERR_WORKSPACE_TOO_SMALL;
  void* scratch = noalloc_scratch(dev);
  if (scratch == nullptr) return PA_ERR_CUDA;
  st = pa_decode_plan(kv_indptr, kv_last_page_len, batch_size, num_kv_indices, num_qo_heads,
                      cache->num_kv_heads, cache->head_dim, cache->page_size, scratch,
                      PA_NOALLOC_SCRATCH_BYTES, stream);
  if (st != PA_OK) return st;
  return pa_decode_run(q, q_stride_n, q_stride_h, cache, kv_indices, kv_indptr, kv_last_page_len,
                       batch_size, num_qo_heads, sm_scale, scratch, PA_NOALLOC_SCRATCH_BYTES, out,
                       lse, stream);
}
