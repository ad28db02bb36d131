// iak_decode_noalloc: the decode for callers that cannot allocate device
// memory.  Its split-KV scratch is a file-scope __device__ array; see the
// declaration in intent_attention_b200.h for the contract.
#include <mutex>

#include "iak_internal.cuh"

namespace iak {
namespace {

// Split-KV partials ((m, l) per row and split + the unnormalised row sums)
// of every call share this array.  Every GPU that loads the library holds it
// until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[IAK_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of the scratch array on the current device.  Looked up once
// per device, with that device current; host code cannot use the symbol itself
// (on the host it names a stand-in, not device memory).  The cached address
// belongs to the device's primary context (the one the CUDA runtime uses): it
// does not survive cudaDeviceReset of that device, and a call made while a
// different driver context is current would use the wrong address.
int scratch_address(void** out) {
  int dev = 0;
  int st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  if (dev < 0 || dev >= 64) return fail(IAK_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    st = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
    if (st) return st;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return IAK_OK;
}

}  // namespace
}  // namespace iak

using namespace iak;

extern "C" int iak_decode_noalloc(const iak_page_pools* pools, const iak_decode_args* args, void* stream) {
  size_t need = 0;
  int st = iak_decode_workspace_size(pools, args, &need);
  if (st) return st;
  if (need > static_cast<size_t>(IAK_NOALLOC_SCRATCH_BYTES))
    return fail(IAK_ERR_WORKSPACE,
                "this decode needs %zu bytes of split-KV scratch but the static scratch holds %d bytes; "
                "pass fewer splits (num_splits) or use iak_decode with a caller workspace",
                need, IAK_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need > 0) {
    st = scratch_address(&scratch);
    if (st) return st;
  }
  // Nothing in the scratch has to start at zero: every launch writes each
  // (row, split) entry before the merge reads it.
  return iak_decode(pools, args, scratch, need > 0 ? static_cast<size_t>(IAK_NOALLOC_SCRATCH_BYTES) : 0, stream);
}
