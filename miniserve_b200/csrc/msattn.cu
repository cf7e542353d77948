// C-ABI entry points of libmsattn.so (declared in include/msattn.h).
//
// This translation unit owns the kernels (included below), the per-thread error string, the
// tensor-map cache for KV pools and the launch logic.  Nothing here allocates device memory or
// synchronises a stream, except ms_device_status.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>

#include "../../include/msattn.h"
#include "ms_common.cuh"
#include "norm_rope_scatter.cuh"
#include "paged_attention.cuh"
#include "prefill_tc.cuh"
#include "qkv_proj_tc.cuh"

namespace ms_host {

thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

static int cuda_fail(const char* what, cudaError_t e) {
  set_error(std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
  return MS_ERR_CUDA;
}

// ---- TMA descriptors for KV pools -----------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct MapKey {
  int device;
  uintptr_t base;
  int num_blocks;
  int num_kv;
  int box;  // 0: whole (block, head) page pair; 1: one 2 KiB quarter; 2: two quarters (4 KiB)
  bool operator==(const MapKey& o) const {
    return device == o.device && base == o.base && num_blocks == o.num_blocks &&
           num_kv == o.num_kv && box == o.box;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.base) ^ (static_cast<size_t>(k.num_blocks) << 20) ^
           (static_cast<size_t>(k.device) << 56) ^ static_cast<size_t>(k.num_kv) ^
           (static_cast<size_t>(k.box) << 40);
  }
};

static std::mutex g_map_mutex;
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// One layer's pool region viewed as a 5-D tensor {64 dims, 16 tokens, 4 quarters (K lo, K hi,
// V lo, V hi), KV heads, blocks}.  Box kind 0 is a whole 8 KiB (block, head) page pair (decode
// kernel); box kind 1 is one 2 KiB quarter, so the tensor-core kernel can lay 8 pages' K out as a
// contiguous 128-key operand tile; box kind 2 is two quarters (a page's whole V, 4 KiB), which the
// tensor-core kernel reads as an MN-major operand one page per 16-key step.
static int kv_tensor_map(const void* k_cache, int num_blocks, int num_kv, int box_kind,
                         CUtensorMap* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  const MapKey key{dev, reinterpret_cast<uintptr_t>(k_cache), num_blocks, num_kv, box_kind};
  std::lock_guard<std::mutex> lock(g_map_mutex);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return MS_OK;
  }
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return MS_ERR_CUDA;
  }
  const cuuint64_t dims[5] = {64, 16, 4, static_cast<cuuint64_t>(num_kv),
                              static_cast<cuuint64_t>(num_blocks)};
  const cuuint64_t strides[4] = {128, 2048, ms::kPageKVBytes,
                                 static_cast<cuuint64_t>(num_kv) * ms::kPageKVBytes};
  const cuuint32_t box[5] = {64, 16, box_kind == 0 ? 4u : (box_kind == 1 ? 1u : 2u), 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUtensorMap map;
  const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(k_cache), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)));
    return MS_ERR_CUDA;
  }
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, map);
  *out = map;
  return MS_OK;
}

// A row-major bf16 matrix [rows, cols] (row stride in elements) as a 2-D tensor map with
// 128-byte-swizzled {64 columns, 128 rows} boxes: one K-major tcgen05 operand tile.  Rows past
// the end read as zeros.
static int matrix_tile_map(const void* base, int64_t rows, int64_t cols, int64_t row_stride,
                           CUtensorMap* out) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return MS_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (matrix) failed with CUresult " +
              std::to_string(static_cast<int>(r)));
    return MS_ERR_CUDA;
  }
  return MS_OK;
}

// Every kernel is launched with programmatic stream serialization (see pdl_wait in
// ms_common.cuh): its grid may start while the previous kernel in the stream finishes.
template <typename... KArgs, typename... Args>
static cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, unsigned block, size_t smem,
                          cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same, as clusters of two CTAs (consecutive blockIdx.x) that share distributed shared memory.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pairs(void (*kernel)(KArgs...), dim3 grid, unsigned block, size_t smem,
                                cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- attention launch configurations --------------------------------------------------------

constexpr int kDecodeWarps = 4, kDecodeStages = 8;
constexpr int kTileWarps = 8, kTileStages = 8;
using DecodeCfg = ms::AttnCfg<0, kDecodeWarps, kDecodeStages>;
using TileCfg = ms::AttnCfg<1, kTileWarps, kTileStages>;
using UnitsCfg = ms::UnitsCfg<kDecodeWarps, kDecodeStages>;
// Decode launches of more than one resident wave whose items read at most this many pages on
// average run persistent over work units (see paged_decode_units_kernel).
constexpr int kUnitsMaxAvgPages = 32;
static_assert(ms::TcCfg::kSmemBytes <= 232448, "tensor-core kernel exceeds 227 KiB of smem");

static int ensure_smem_attrs() {
  // Per device: the attribute is a property of the function on the current device.
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= 64) return MS_ERR_ARG;
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return MS_OK;
  e = cudaFuncSetAttribute(ms::paged_attn_kernel<0, kDecodeWarps, kDecodeStages>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, DecodeCfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(decode)", e);
  e = cudaFuncSetAttribute(ms::paged_attn_kernel<0, kDecodeWarps, kDecodeStages, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, DecodeCfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(decode, early)", e);
  e = cudaFuncSetAttribute(ms::paged_attn_kernel<1, kTileWarps, kTileStages>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, TileCfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(tile)", e);
  e = cudaFuncSetAttribute(ms::paged_decode_units_kernel<kDecodeWarps, kDecodeStages>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, UnitsCfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(decode units)", e);
  e = cudaFuncSetAttribute(ms::paged_decode_units_kernel<kDecodeWarps, kDecodeStages, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, UnitsCfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(decode units, cascade)", e);
  e = cudaFuncSetAttribute(ms::paged_attn_kernel<1, kTileWarps, kTileStages, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, TileCfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(tile, early)", e);
  e = cudaFuncSetAttribute(ms::prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           ms::TcCfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(tc)", e);
  {
    // The tensor-core kernel moves registers between its warpgroups (setmaxnreg); the increase
    // can only be met out of what the launch allocated, so a build that gave the kernel fewer
    // registers per thread than the split assumes must never be launched.
    cudaFuncAttributes fa{};
    e = cudaFuncGetAttributes(&fa, ms::prefill_tc_kernel);
    if (e != cudaSuccess) return cuda_fail("cudaFuncGetAttributes(tc)", e);
    if (fa.numRegs < ms::TcCfg::kLaunchRegs) {
      ms_host::set_error("prefill_tc_kernel was compiled with " + std::to_string(fa.numRegs) +
                         " registers per thread; its register split needs " +
                         std::to_string(ms::TcCfg::kLaunchRegs));
      return MS_ERR_CUDA;
    }
  }
  e = cudaFuncSetAttribute(ms::qkv_proj_norm_rope_kernel<1>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, ms::QkvCfg<1>::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(qkv 1)", e);
  e = cudaFuncSetAttribute(ms::qkv_proj_norm_rope_kernel<2>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, ms::QkvCfg<2>::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(qkv 2)", e);
  e = cudaFuncSetAttribute(ms::qkv_proj_norm_rope_kernel<1, 2>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           ms::QkvCfg<1, 2>::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(qkv split-K)", e);
  done[dev] = true;
  return MS_OK;
}

static int sm_count(int* out) {
  // Per device, cached.
  static std::mutex mu;
  static int counts[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= 64) return MS_ERR_ARG;
  std::lock_guard<std::mutex> lock(mu);
  if (counts[dev] == 0) {
    e = cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail("cudaDeviceGetAttribute(SM count)", e);
  }
  *out = counts[dev];
  return MS_OK;
}

// A second stream per (host thread, device), with its fork/join events: ms_paged_attention runs
// the bandwidth-bound decode launch on it beside the tensor-bound prefill launch when the two are
// independent.  Created on first use in relaxed capture mode, so that a first call made while a
// stream is being captured into a CUDA graph may create it; never destroyed.  If it cannot be
// created the launches simply stay on the caller's stream.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr;
  cudaEvent_t join = nullptr;
  bool tried = false;
};

static SideStream* side_stream() {
  thread_local SideStream per_dev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  SideStream& ss = per_dev[dev];
  if (!ss.tried) {
    ss.tried = true;
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    const bool ok = cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking) == cudaSuccess &&
                    cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) == cudaSuccess &&
                    cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) == cudaSuccess;
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (!ok) {
      cudaGetLastError();
      ss.stream = nullptr;
    }
  }
  return ss.stream != nullptr ? &ss : nullptr;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int check_pool(const void* k_cache, const void* v_cache, int num_blocks, int num_kv) {
  if (k_cache == nullptr || v_cache == nullptr || num_blocks <= 0 || num_kv <= 0) {
    set_error("KV pool: null pointer or empty pool");
    return MS_ERR_ARG;
  }
  if (static_cast<const char*>(v_cache) != static_cast<const char*>(k_cache) + ms::kPageBytes) {
    set_error("KV pool: v_cache must start 4096 bytes after k_cache (layout "
              "[blocks][kv_heads][K,V][d/64][16][64])");
    return MS_ERR_LAYOUT;
  }
  if (!aligned(k_cache, 16)) {
    set_error("KV pool: k_cache must be 16-byte aligned");
    return MS_ERR_LAYOUT;
  }
  return MS_OK;
}

}  // namespace ms_host

using namespace ms_host;

extern "C" int ms_version(void) { return MS_ABI_VERSION * 100 + 0; }

extern "C" const char* ms_last_error(void) { return g_last_error.c_str(); }

extern "C" int ms_device_status(void* stream, uint32_t* flags, int clear) {
  if (flags == nullptr) {
    set_error("ms_device_status: null flags");
    return MS_ERR_ARG;
  }
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("cudaStreamSynchronize", e);
  unsigned v = 0;
  e = cudaMemcpyFromSymbol(&v, ms::g_status_word, sizeof(v));
  if (e != cudaSuccess) return cuda_fail("cudaMemcpyFromSymbol", e);
  *flags = v;
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(ms::g_status_word, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail("cudaMemcpyToSymbol", e);
  }
  return MS_OK;
}

static unsigned* status_ptr(int* rc) {
  // Address of this device's status word (a __device__ symbol has one instance per device).
  static thread_local int cached_dev = -1;
  static thread_local unsigned* cached = nullptr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *rc = cuda_fail("cudaGetDevice", e);
    return nullptr;
  }
  if (dev != cached_dev) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, ms::g_status_word);
    if (e != cudaSuccess) {
      *rc = cuda_fail("cudaGetSymbolAddress(status)", e);
      return nullptr;
    }
    cached = static_cast<unsigned*>(p);
    cached_dev = dev;
  }
  *rc = MS_OK;
  return cached;
}

extern "C" int ms_qk_norm_rope_scatter(const void* qkv, int64_t qkv_row_stride, int32_t num_tokens,
                                       int32_t num_heads, int32_t num_kv_heads,
                                       const void* q_weight, const void* k_weight, float eps,
                                       const float* cos, const float* sin, int64_t cs_row_stride,
                                       const int64_t* positions, int64_t max_positions,
                                       const int64_t* slot_mapping, void* q_out,
                                       int64_t q_out_row_stride, void* k_cache, void* v_cache,
                                       int32_t num_blocks, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || num_heads != ms::kGroup * num_kv_heads) {
    set_error("ms_qk_norm_rope_scatter: need num_heads == 2 * num_kv_heads > 0, num_tokens >= 0");
    return MS_ERR_ARG;
  }
  if (num_tokens == 0) return MS_OK;
  int rc = check_pool(k_cache, v_cache, num_blocks, num_kv_heads);
  if (rc) return rc;
  if (!qkv || !q_weight || !k_weight || !cos || !sin || !slot_mapping || !q_out) {
    set_error("ms_qk_norm_rope_scatter: null pointer argument");
    return MS_ERR_ARG;
  }
  const int64_t width = static_cast<int64_t>(num_heads + 2 * num_kv_heads) * ms::kHeadDim;
  if (qkv_row_stride < width || q_out_row_stride < num_heads * ms::kHeadDim ||
      cs_row_stride < ms::kHeadDim || qkv_row_stride % 4 || q_out_row_stride % 4 ||
      cs_row_stride % 4 || !aligned(qkv, 8) || !aligned(q_out, 8) || !aligned(cos, 16) ||
      !aligned(sin, 16)) {
    set_error("ms_qk_norm_rope_scatter: strides/alignment (qkv, q_out rows 8-byte aligned; "
              "cos/sin rows 16-byte aligned)");
    return MS_ERR_ARG;
  }
  if (positions != nullptr && max_positions <= 0) {
    set_error("ms_qk_norm_rope_scatter: positions given with an empty table");
    return MS_ERR_ARG;
  }
  unsigned* st = status_ptr(&rc);
  if (rc) return rc;
  ms::NormRopeArgs a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.qkv_row_stride = qkv_row_stride;
  a.q_weight = static_cast<const __nv_bfloat16*>(q_weight);
  a.k_weight = static_cast<const __nv_bfloat16*>(k_weight);
  a.eps = eps;
  a.cos = cos;
  a.sin = sin;
  a.cs_row_stride = cs_row_stride;
  a.positions = reinterpret_cast<const long long*>(positions);
  a.max_positions = max_positions;
  a.slots = reinterpret_cast<const long long*>(slot_mapping);
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.q_out_row_stride = q_out_row_stride;
  a.k_pool = static_cast<__nv_bfloat16*>(k_cache);
  a.head_stride = ms::kPageKVBytes / 2;
  a.block_stride = static_cast<long long>(num_kv_heads) * a.head_stride;
  a.num_slots = static_cast<long long>(num_blocks) * ms::kBlockTokens;
  a.num_tokens = num_tokens;
  a.num_heads = num_heads;
  a.num_kv = num_kv_heads;
  if (num_kv_heads % ms::kRowsPerWarp != 0) {
    set_error("ms_qk_norm_rope_scatter: num_kv_heads must be a multiple of 8");
    return MS_ERR_ARG;
  }
  constexpr int kWarps = 8;
  const long long warps =
      static_cast<long long>(num_tokens) * (num_heads + 2 * num_kv_heads) / ms::kRowsPerWarp;
  const long long blocks = (warps + kWarps - 1) / kWarps;
  if (blocks > 0x7fffffffLL) {
    set_error("ms_qk_norm_rope_scatter: batch too large");
    return MS_ERR_ARG;
  }
  // The 16-byte form (two whole rows per warp instruction, half the instructions) whenever the
  // rows and the norm weights allow 16-byte accesses; both forms give the same bits.
  const bool v16 = aligned(qkv, 16) && aligned(q_out, 16) && qkv_row_stride % 8 == 0 &&
                   q_out_row_stride % 8 == 0 && aligned(q_weight, 16) && aligned(k_weight, 16);
  const cudaError_t e =
      v16 ? launch(ms::qk_norm_rope_scatter_v16_kernel<kWarps>, static_cast<unsigned>(blocks),
                   kWarps * 32, 0, static_cast<cudaStream_t>(stream), a, st)
          : launch(ms::qk_norm_rope_scatter_kernel<kWarps>, static_cast<unsigned>(blocks),
                   kWarps * 32, 0, static_cast<cudaStream_t>(stream), a, st);
  if (e != cudaSuccess) return cuda_fail("qk_norm_rope_scatter launch", e);
  return MS_OK;
}

extern "C" int ms_qkv_proj_norm_rope_scatter(
    const void* x, int64_t x_row_stride, int32_t num_tokens, int32_t hidden, const void* w_qkv,
    int64_t w_row_stride, int32_t num_heads, int32_t num_kv_heads, const void* q_weight,
    const void* k_weight, float eps, const float* cos, const float* sin, int64_t cs_row_stride,
    const int64_t* positions, int64_t max_positions, const int64_t* slot_mapping, void* q_out,
    int64_t q_out_row_stride, void* k_cache, void* v_cache, int32_t num_blocks, void* stream) {
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || hidden <= 0 || hidden % 64) {
    set_error("ms_qkv_proj_norm_rope_scatter: need num_tokens >= 0, heads > 0 and hidden a "
              "positive multiple of 64");
    return MS_ERR_ARG;
  }
  if (num_tokens == 0) return MS_OK;
  int rc = check_pool(k_cache, v_cache, num_blocks, num_kv_heads);
  if (rc) return rc;
  if (!x || !w_qkv || !q_weight || !k_weight || !cos || !sin || !slot_mapping || !q_out) {
    set_error("ms_qkv_proj_norm_rope_scatter: null pointer argument");
    return MS_ERR_ARG;
  }
  if (x_row_stride < hidden || w_row_stride < hidden || x_row_stride % 8 || w_row_stride % 8 ||
      q_out_row_stride < static_cast<int64_t>(num_heads) * ms::kHeadDim || q_out_row_stride % 8 ||
      cs_row_stride < ms::kHeadDim || cs_row_stride % 4 || !aligned(x, 16) || !aligned(w_qkv, 16) ||
      !aligned(q_weight, 16) || !aligned(k_weight, 16) || !aligned(q_out, 16) ||
      !aligned(cos, 16) || !aligned(sin, 16)) {
    set_error("ms_qkv_proj_norm_rope_scatter: strides/alignment (x, w_qkv, q_out rows and the "
              "norm weights 16-byte aligned; cos/sin rows 16-byte aligned)");
    return MS_ERR_ARG;
  }
  if (positions != nullptr && max_positions <= 0) {
    set_error("ms_qkv_proj_norm_rope_scatter: positions given with an empty table");
    return MS_ERR_ARG;
  }
  const int64_t m_tiles = (static_cast<int64_t>(num_tokens) + 127) / 128;
  if (m_tiles > 65535) {
    set_error("ms_qkv_proj_norm_rope_scatter: batch too large");
    return MS_ERR_ARG;
  }
  rc = ensure_smem_attrs();
  if (rc) return rc;
  unsigned* st = status_ptr(&rc);
  if (rc) return rc;
  const int rows = num_heads + 2 * num_kv_heads;
  CUtensorMap xmap, wmap;
  rc = matrix_tile_map(x, num_tokens, hidden, x_row_stride, &xmap);
  if (rc) return rc;
  rc = matrix_tile_map(w_qkv, static_cast<int64_t>(rows) * ms::kHeadDim, hidden, w_row_stride,
                       &wmap);
  if (rc) return rc;
  ms::QkvArgs qa;
  ms::NormRopeArgs& a = qa.e;
  a.qkv = nullptr;
  a.qkv_row_stride = 0;
  a.q_weight = static_cast<const __nv_bfloat16*>(q_weight);
  a.k_weight = static_cast<const __nv_bfloat16*>(k_weight);
  a.eps = eps;
  a.cos = cos;
  a.sin = sin;
  a.cs_row_stride = cs_row_stride;
  a.positions = reinterpret_cast<const long long*>(positions);
  a.max_positions = max_positions;
  a.slots = reinterpret_cast<const long long*>(slot_mapping);
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.q_out_row_stride = q_out_row_stride;
  a.k_pool = static_cast<__nv_bfloat16*>(k_cache);
  a.head_stride = ms::kPageKVBytes / 2;
  a.block_stride = static_cast<long long>(num_kv_heads) * a.head_stride;
  a.num_slots = static_cast<long long>(num_blocks) * ms::kBlockTokens;
  a.num_tokens = num_tokens;
  a.num_heads = num_heads;
  a.num_kv = num_kv_heads;
  qa.hidden = hidden;
  int sms = 0;
  rc = sm_count(&sms);
  if (rc) return rc;
  // Two heads per tile (less L2 traffic per flop) once the two-head tiles cover at least half the
  // SMs and the heads pair up by kind; one head per tile below that (twice the tiles, each SM
  // streaming half the bytes).  Measured crossover (16q/8kv heads, hidden 1024): 512 tokens
  // 12.3 us one-head vs 16.5 two-head; 768 tokens 18.9 vs 16.9; 2048 tokens 31.9 vs 24.6.
  const bool pairs = num_heads % 2 == 0 && num_kv_heads % 2 == 0 &&
                     2 * m_tiles * (rows / 2) >= static_cast<int64_t>(sms);
  qa.num_tiles = static_cast<int>(m_tiles * (pairs ? rows / 2 : rows));
  // Few one-head tiles (decode-sized steps: up to 2 x 128 tokens for 32 head rows on 148 SMs):
  // each tile runs on a pair of CTAs that split the hidden dimension, so every CTA streams half
  // the operands and stages half the rows.
  const bool split = !pairs && (hidden / 64) % 2 == 0 && 2 * qa.num_tiles <= sms;
  const int grid = split ? 2 * qa.num_tiles
                         : (qa.num_tiles < sms ? qa.num_tiles : sms);  // persistent: one CTA/SM
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      pairs   ? launch(ms::qkv_proj_norm_rope_kernel<2>, grid, ms::QkvCfg<2>::kThreads,
                       ms::QkvCfg<2>::kSmemBytes, s, xmap, wmap, qa, st)
      : split ? launch_pairs(ms::qkv_proj_norm_rope_kernel<1, 2>, grid, ms::QkvCfg<1, 2>::kThreads,
                             ms::QkvCfg<1, 2>::kSmemBytes, s, xmap, wmap, qa, st)
              : launch(ms::qkv_proj_norm_rope_kernel<1>, grid, ms::QkvCfg<1>::kThreads,
                       ms::QkvCfg<1>::kSmemBytes, s, xmap, wmap, qa, st);
  if (e != cudaSuccess) return cuda_fail("qkv_proj_norm_rope launch", e);
  return MS_OK;
}

extern "C" int ms_kv_scatter(const void* k, int64_t k_row_stride, const void* v,
                             int64_t v_row_stride, int32_t num_tokens, int32_t num_kv_heads,
                             const int64_t* slot_mapping, void* k_cache, void* v_cache,
                             int32_t num_blocks, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0) {
    set_error("ms_kv_scatter: bad sizes");
    return MS_ERR_ARG;
  }
  if (num_tokens == 0) return MS_OK;
  int rc = check_pool(k_cache, v_cache, num_blocks, num_kv_heads);
  if (rc) return rc;
  if (!k || !v || !slot_mapping || k_row_stride < num_kv_heads * ms::kHeadDim ||
      v_row_stride < num_kv_heads * ms::kHeadDim || k_row_stride % 4 || v_row_stride % 4 ||
      !aligned(k, 8) || !aligned(v, 8)) {
    set_error("ms_kv_scatter: null pointer, stride or alignment");
    return MS_ERR_ARG;
  }
  unsigned* st = status_ptr(&rc);
  if (rc) return rc;
  ms::ScatterArgs a;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.k_row_stride = k_row_stride;
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.v_row_stride = v_row_stride;
  a.slots = reinterpret_cast<const long long*>(slot_mapping);
  a.k_pool = static_cast<__nv_bfloat16*>(k_cache);
  a.head_stride = ms::kPageKVBytes / 2;
  a.block_stride = static_cast<long long>(num_kv_heads) * a.head_stride;
  a.num_slots = static_cast<long long>(num_blocks) * ms::kBlockTokens;
  a.num_tokens = num_tokens;
  a.num_kv = num_kv_heads;
  constexpr int kWarps = 8;
  const long long warps = static_cast<long long>(num_tokens) * 2 * num_kv_heads;
  const long long blocks = (warps + kWarps - 1) / kWarps;
  const cudaError_t e = launch(ms::kv_scatter_kernel<kWarps>, static_cast<unsigned>(blocks),
                               kWarps * 32, 0, static_cast<cudaStream_t>(stream), a, st);
  if (e != cudaSuccess) return cuda_fail("kv_scatter launch", e);
  return MS_OK;
}

extern "C" int ms_paged_attention(const void* q, int64_t q_row_stride, void* out,
                                  int64_t out_row_stride, int32_t num_heads, int32_t num_kv_heads,
                                  const void* k_cache, const void* v_cache, int32_t num_blocks,
                                  const int32_t* plan_dev, const MsPlanInfo* plan, void* workspace,
                                  int64_t workspace_bytes, float scale, void* stream) {
  if (plan == nullptr || num_kv_heads <= 0 || num_heads != ms::kGroup * num_kv_heads) {
    set_error("ms_paged_attention: need a plan and num_heads == 2 * num_kv_heads > 0");
    return MS_ERR_ARG;
  }
  const int64_t n_items = static_cast<int64_t>(plan->n_decode_items) + plan->n_tile_items +
                          plan->n_tc_items;
  if (n_items == 0) return MS_OK;
  int rc = check_pool(k_cache, v_cache, num_blocks, num_kv_heads);
  if (rc) return rc;
  if (!q || !out || !plan_dev || q_row_stride < num_heads * ms::kHeadDim ||
      out_row_stride < num_heads * ms::kHeadDim || q_row_stride % 8 || out_row_stride % 8 ||
      !aligned(q, 16) || !aligned(out, 16) || !aligned(plan_dev, 16)) {
    set_error("ms_paged_attention: null pointer, or q/out rows not 16-byte aligned");
    return MS_ERR_ARG;
  }
  const int64_t need = plan->workspace_bytes_per_kv_head * num_kv_heads;
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16))) {
    set_error("ms_paged_attention: workspace of " + std::to_string(need) +
              " bytes (16-byte aligned) required");
    return MS_ERR_ARG;
  }
  if (n_items * num_kv_heads > 0x7fffffffLL ||
      static_cast<int64_t>(plan->n_combine) * num_kv_heads > 0x7fffffffLL) {
    set_error("ms_paged_attention: plan too large for one launch");
    return MS_ERR_ARG;
  }
  rc = ensure_smem_attrs();
  if (rc) return rc;
  CUtensorMap map;
  rc = kv_tensor_map(k_cache, num_blocks, num_kv_heads, 0, &map);
  if (rc) return rc;
  CUtensorMap kmap, vmap;
  if (plan->n_tc_items > 0) {
    rc = kv_tensor_map(k_cache, num_blocks, num_kv_heads, 1, &kmap);
    if (rc) return rc;
    rc = kv_tensor_map(k_cache, num_blocks, num_kv_heads, 2, &vmap);
    if (rc) return rc;
  }

  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  ms::AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_row_stride = q_row_stride;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_row_stride = out_row_stride;
  a.seqs = plan_dev + plan->off_seqs;
  a.tables = plan_dev + plan->off_tables;
  a.num_kv = num_kv_heads;
  a.num_blocks = num_blocks;
  float* ws = static_cast<float*>(workspace);
  a.ws_o = ws;
  a.ws_lse = ws != nullptr ? ws + plan->part_rows * num_kv_heads * ms::kHeadDim : nullptr;
  a.scale_log2 = scale * 1.4426950408889634f;

  // The tensor-core kernel is launched first (it then takes its SMs first).  Without cascade
  // groups the decode launch is independent of it (disjoint output rows; the combine pass, which
  // reads both launches' partials, runs after the join), so it goes on a side stream and the two
  // run at once: the decode items stream KV from HBM on the SMs the tensor-core CTAs leave free
  // and on each SM they release (config 3: 73.5 -> 62.6 us).  With cascade groups the decode
  // items merge the shared-prefix partials the tensor-core kernel writes, so they follow it.
  SideStream* side = nullptr;
  if (plan->n_tc_items > 0 && plan->n_decode_items > 0 && plan->n_cascade == 0) side = side_stream();
  cudaStream_t ds = s;
  if (side != nullptr) {
    cudaError_t e = cudaEventRecord(side->fork, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side->stream, side->fork, 0);
    if (e != cudaSuccess) return cuda_fail("fork to the side stream", e);
    ds = side->stream;
  }
  // Joins the side stream back into the caller's (also on the error paths below, so that a
  // stream capture is never left with an open branch).
  auto join = [&]() -> cudaError_t {
    if (side == nullptr) return cudaSuccess;
    cudaError_t e = cudaEventRecord(side->join, ds);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, side->join, 0);
    side = nullptr;
    return e;
  };
  if (plan->n_tc_items > 0) {
    a.items = plan_dev + plan->off_tc;
    a.n_items = plan->n_tc_items;
    const cudaError_t e = launch(ms::prefill_tc_kernel, plan->n_tc_items * num_kv_heads,
                                 ms::TcCfg::kThreads, ms::TcCfg::kSmemBytes, s, kmap, vmap, a);
    if (e != cudaSuccess) {
      join();
      return cuda_fail("prefill_tc launch", e);
    }
  }
  int sms = 0;
  rc = sm_count(&sms);
  if (rc) {
    join();
    return rc;
  }
  if (plan->n_decode_items > 0) {
    a.items = plan_dev + plan->off_decode;
    a.n_items = plan->n_decode_items;
    // One resident wave (two decode CTAs per SM): latency-bound, so stream earlier steps' pages
    // while the previous kernel finishes.
    const int ctas = plan->n_decode_items * num_kv_heads;
    cudaError_t e;
    if (ctas <= 2 * sms) {
      e = launch(ms::paged_attn_kernel<0, kDecodeWarps, kDecodeStages, true>, ctas,
                 DecodeCfg::kThreads, DecodeCfg::kSmemBytes, ds, map, a);
    } else if (static_cast<int64_t>(plan->decode_pages) <=
               static_cast<int64_t>(kUnitsMaxAvgPages) * plan->n_decode_items) {
      // Many short items: two persistent CTAs per SM walk the work units.  Right after the
      // tensor-core kernel of a cascade plan they also overlap its last wave.
      const bool after_prefix = plan->n_cascade > 0 && plan->n_tc_items > 0 && ds == s;
      // When the tensor-core kernel ends in a small partial wave (e.g. 160 CTAs on 148 SMs), the
      // CTAs placed on the SMs that wave holds start one tensor-core CTA later than the rest but
      // get the same share of the units (a static stride), so they finish last (config 4: 24
      // CTAs ending at 83-88 us against 74 us for the rest).  Those SMs are left out of the grid.
      int grid = 2 * sms;
      if (after_prefix) {
        const int64_t tc_ctas = static_cast<int64_t>(plan->n_tc_items) * num_kv_heads;
        const int rem = static_cast<int>(tc_ctas % sms);
        if (tc_ctas > sms && rem > 0 && rem <= sms / 8) grid = 2 * (sms - rem);
      }
      e = after_prefix
              ? launch(ms::paged_decode_units_kernel<kDecodeWarps, kDecodeStages, true>, grid,
                       UnitsCfg::kThreads, UnitsCfg::kSmemBytes, ds, map, a)
              : launch(ms::paged_decode_units_kernel<kDecodeWarps, kDecodeStages>, grid,
                       UnitsCfg::kThreads, UnitsCfg::kSmemBytes, ds, map, a);
    } else {
      e = launch(ms::paged_attn_kernel<0, kDecodeWarps, kDecodeStages>, ctas,
                 DecodeCfg::kThreads, DecodeCfg::kSmemBytes, ds, map, a);
    }
    if (e != cudaSuccess) {
      join();
      return cuda_fail("paged_attn decode launch", e);
    }
  }
  if (plan->n_tile_items > 0) {
    a.items = plan_dev + plan->off_tile;
    a.n_items = plan->n_tile_items;
    const int ctas = plan->n_tile_items * num_kv_heads;
    const cudaError_t e =
        ctas <= sms ? launch(ms::paged_attn_kernel<1, kTileWarps, kTileStages, true>, ctas,
                             TileCfg::kThreads, TileCfg::kSmemBytes, s, map, a)
                    : launch(ms::paged_attn_kernel<1, kTileWarps, kTileStages>, ctas,
                             TileCfg::kThreads, TileCfg::kSmemBytes, s, map, a);
    if (e != cudaSuccess) {
      join();
      return cuda_fail("paged_attn tile launch", e);
    }
  }
  {
    const cudaError_t e = join();
    if (e != cudaSuccess) return cuda_fail("join of the side stream", e);
  }
  if (plan->n_combine > 0) {
    ms::CombineArgs c;
    c.out = a.out;
    c.out_row_stride = out_row_stride;
    c.seqs = a.seqs;
    c.combines = plan_dev + plan->off_combine;
    c.n_combine = plan->n_combine;
    c.num_kv = num_kv_heads;
    c.ws_o = a.ws_o;
    c.ws_lse = a.ws_lse;
    // One CTA per (record, KV head, kCombineRows rows): a tensor-core record has 256 rows, and
    // one CTA walking them all is latency-bound (each row is a few dependent loads).
    const int64_t rows_max = static_cast<int64_t>(std::max(plan->combine_tokens_max, 1)) * 2;
    const unsigned row_ctas = static_cast<unsigned>(
        std::min<int64_t>((rows_max + ms::kCombineRows - 1) / ms::kCombineRows, 65535));
    const cudaError_t e = launch(ms::combine_kernel, dim3(plan->n_combine * num_kv_heads, row_ctas),
                                 ms::kCombineThreads, 0, s, c);
    if (e != cudaSuccess) return cuda_fail("combine launch", e);
  }
  return MS_OK;
}
