// ms_paged_attention_noalloc: the attention entry point for callers that cannot allocate device
// memory themselves.
//
// Some hosts never let a plugin call cudaMalloc: an engine that hands every byte of the GPU to
// its own arena up front, a runtime whose custom-op interface has no allocator hook, or a loop
// that must not take cudaMalloc's implicit device synchronisation.  Such a caller still owns q,
// out, the pool and the plan, but it has nowhere to put the split-KV partial results.  This
// entry point keeps them in a fixed array compiled into the library instead.
//
// The array is MS_NOALLOC_SCRATCH_BYTES (16 MiB) in every GPU's memory once the library is
// loaded there, and it stays until the process exits.  All calls share it, so two calls that
// overlap on the GPU (different streams, or different host threads without ordering) race on
// it; calls on one stream are ordered and safe.  Nothing in it needs to start at zero: within
// one call every partial row is written by its split before the combine kernel reads it, and the
// previous call's leftovers are never read.
#include <cuda_runtime.h>

#include <string>

#include "../../include/msattn.h"

namespace ms_host {
void set_error(const std::string& msg);
}

namespace {

// Split-KV partials: [part_rows][kv_heads][128] fp32 followed by [part_rows][kv_heads] fp32.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MS_NOALLOC_SCRATCH_BYTES];

// Device address of the current context's copy of the array.  In host code the array's name
// only stands for it; the runtime gives the real address for the device that is current.  It is
// looked up on every call (cheap once the module is loaded), so a context that was destroyed and
// created again (cudaDeviceReset) never sees a stale address.
int scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    ms_host::set_error(std::string("ms_paged_attention_noalloc: cudaGetSymbolAddress: ") +
                       cudaGetErrorString(e));
    return MS_ERR_CUDA;
  }
  *out = p;
  return MS_OK;
}

}  // namespace

extern "C" int ms_paged_attention_noalloc(const void* q, int64_t q_row_stride, void* out,
                                          int64_t out_row_stride, int32_t num_heads,
                                          int32_t num_kv_heads, const void* k_cache,
                                          const void* v_cache, int32_t num_blocks,
                                          const int32_t* plan_dev, const MsPlanInfo* plan,
                                          float scale, void* stream) {
  if (plan == nullptr || num_kv_heads <= 0) {
    ms_host::set_error("ms_paged_attention_noalloc: need a plan and num_kv_heads > 0");
    return MS_ERR_ARG;
  }
  const int64_t need = plan->workspace_bytes_per_kv_head * num_kv_heads;
  if (need > static_cast<int64_t>(MS_NOALLOC_SCRATCH_BYTES)) {
    ms_host::set_error("ms_paged_attention_noalloc: this plan needs " + std::to_string(need) +
                       " bytes of split-KV scratch but the built-in scratch holds " +
                       std::to_string(MS_NOALLOC_SCRATCH_BYTES) +
                       "; plan with a larger pages_per_split or call ms_paged_attention with a "
                       "workspace");
    return MS_ERR_CAPACITY;
  }
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != MS_OK) return rc;
  return ms_paged_attention(q, q_row_stride, out, out_row_stride, num_heads, num_kv_heads,
                            k_cache, v_cache, num_blocks, plan_dev, plan, scratch,
                            static_cast<int64_t>(MS_NOALLOC_SCRATCH_BYTES), scale, stream);
}
