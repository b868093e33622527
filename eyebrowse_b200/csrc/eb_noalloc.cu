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
static std::mutex g_scratch_mu;
static unsigned char* g_scratch_ptrs[64] = {};

static unsigned char* noalloc_scratch_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    g_scratch_ptrs[dev] = static_cast<unsigned char*>(p);
  }
  return g_scratch_ptrs[dev];
}

bool noalloc_clear_tickets() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return false;
  }
  unsigned char* p = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    p = g_scratch_ptrs[dev];
  }
  if (!p) return true;  // never used on this device: still all zero
  // The tickets sit at the start of the array; the rest is always written
  // before it is read, so clearing the whole array is simply the bound.
  if (cudaMemset(p, 0, EB_NOALLOC_SCRATCH_BYTES) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

}  // namespace eb

using namespace eb;

extern "C" int eb_attention_decode_noalloc(const eb_attn_desc* d, const eb_attn_layer* L,
                                           int64_t pos, const void* q, const void* k,
                                           const void* v, void* kcache, void* vcache, void* o,
                                           eb_stream_t stream) {
  // The same argument checks as eb_attention_decode (shape, dtype codes,
  // strides, window, position, pointers, device).
  if (!desc_ok(d) || pos < 0 || pos >= d->max_seq) return EB_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !kcache || !vcache || !o) return EB_ERR_INVALID_ARGUMENT;
  // The split-K plan for this shape must fit the fixed scratch; refuse, before
  // touching the device, a shape whose partials would not.
  const size_t need = decode_plan_bytes(d, 1, pos);
  if (need > (size_t)EB_NOALLOC_SCRATCH_BYTES) return EB_ERR_WORKSPACE;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  unsigned char* scratch = noalloc_scratch_ptr();
  if (!scratch) return EB_ERR_CUDA;
  // The array keeps the previous call's contents. Its split-K tickets must be
  // zero when a call starts: device memory of a __device__ array is zero when
  // the library loads, and every call that completes leaves its tickets at
  // zero again (the CTA that merges the partials resets them). A call whose
  // kernel gave up can leave them set; eb_get_device_error, which reports
  // that, also zeroes them. The partials are always written before they are
  // read, so nothing is cleared per call.
  return decode_impl(d, L, 1, nullptr, pos, pos, q, k, v, kcache, vcache, 0, o, 0, 0, 0, scratch,
                     (size_t)EB_NOALLOC_SCRATCH_BYTES, reinterpret_cast<cudaStream_t>(stream));
}
