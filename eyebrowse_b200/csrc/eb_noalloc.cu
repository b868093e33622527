// eb_noalloc.cu -- eb_attention_decode_noalloc: the single-sequence decode
// step with its split-K scratch in library-owned device memory.
//
// Some callers cannot allocate device memory at all: a plugin loaded into a
// host framework that owns the whole device pool and passes the plugin only
// its input and output buffers, or a serving loop that must never call into
// an allocator between steps. eb_attention_decode needs a caller workspace
// for its combine step; this entry point takes none. Its scratch is the
// file-scope array below, which every GPU that loads this library holds
// (EB_NOALLOC_SCRATCH_BYTES each) until the process exits.
#include <mutex>

#include "../../include/eyebrowse_attn.h"
#include "eb_common.cuh"
#include "eb_kernels.cuh"

namespace eb {

// Split-K scratch of eb_attention_decode_noalloc: ticket counters, then the
// per-chunk partial (m, l) and accumulators, laid out as the caller workspace
// of eb_attention_decode is.
static __device__ __align__(256) unsigned char g_noalloc_scratch[EB_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device. In host code the
// array's name only stands in for the device object, so its address must come
// from cudaGetSymbolAddress, once per device, with that device current.
static unsigned char* noalloc_scratch_ptr() {
  static unsigned char* ptrs[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    ptrs[dev] = static_cast<unsigned char*>(p);
  }
  return ptrs[dev];
}

}  // namespace eb

using namespace eb;

extern "C" int eb_attention_decode_noalloc(const eb_attn_desc* d, const eb_attn_layer* L,
                                           int64_t pos, const void* q, const void* k,
                                           const void* v, void* kcache, void* vcache, void* o,
                                           eb_stream_t stream) {
  if (!d || d->n_heads <= 0 || d->n_kv_heads <= 0 || d->n_heads % d->n_kv_heads ||
      d->head_dim <= 0 || d->head_dim > 256 || (d->head_dim & 1) || d->max_seq <= 0 || pos < 0 ||
      pos >= d->max_seq || d->window < 0)
    return EB_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !kcache || !vcache || !o) return EB_ERR_INVALID_ARGUMENT;
  // The split-K plan for this shape must fit the fixed scratch; refuse, before
  // touching the device, a shape whose partials would not.
  const size_t need = decode_plan_bytes(d, 1, pos);
  if (need > (size_t)EB_NOALLOC_SCRATCH_BYTES) return EB_ERR_WORKSPACE;
  int major = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10) {
    cudaGetLastError();
    return EB_ERR_NO_DEVICE;
  }
  unsigned char* scratch = noalloc_scratch_ptr();
  if (!scratch) return EB_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (need > 0) {
    // The array keeps the previous call's contents. The ticket counters sit at
    // its start (one 32-bit word per query head, padded to 256 bytes) and must
    // start at zero; the partials are always written before they are read.
    const size_t counters = ((size_t)d->n_heads * sizeof(unsigned) + 255) / 256 * 256;
    if (cudaMemsetAsync(scratch, 0, counters, st) != cudaSuccess) {
      cudaGetLastError();
      return EB_ERR_CUDA;
    }
  }
  return decode_impl(d, L, 1, nullptr, pos, pos, q, k, v, kcache, vcache, 0, o, 0, 0, 0, scratch,
                     (size_t)EB_NOALLOC_SCRATCH_BYTES, st);
}
