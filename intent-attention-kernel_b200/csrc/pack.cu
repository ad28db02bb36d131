// Device-side metadata packing: router page lists -> page tables.
//
// Replaces the per-element Python loops of metadata_to_kernel_tensors
// (fused_selected_quant_decode.py:372-398) and
// make_page_tables_from_selected_pages (triton_intent_quant_attention.py:152-201):
// one launch writes the [B, Ht, W] table (physical id = base(b, h) + logical
// id, padded), the per-(b, h) counts min(n, W) and, optionally, scatters the
// per-logical-page tags to the physical pages of every (b, h).
#include "iak_internal.cuh"

namespace iak {
namespace {

__global__ void pack_kernel(const iak_pack_args a) {
  const int64_t row = blockIdx.x;
  const int32_t base = a.bases ? a.bases[row] : 0;
  const int W = a.table_width;
  const int cnt = a.num_ids < W ? a.num_ids : W;
  int32_t* t = a.page_table + row * W;
  for (int j = threadIdx.x; j < W; j += blockDim.x) t[j] = j < cnt ? base + a.logical_ids[j] : a.pad_value;
  if (threadIdx.x == 0 && a.page_counts) a.page_counts[row] = cnt;
  if (a.logical_tags && a.page_tags)
    for (int i = threadIdx.x; i < a.num_logical_pages; i += blockDim.x) {
      const int64_t dst = static_cast<int64_t>(base) + i;
      if (dst >= 0 && dst < a.num_tag_pages) a.page_tags[dst] = a.logical_tags[i];
    }
}

}  // namespace
}  // namespace iak

using namespace iak;

extern "C" int iak_pack_metadata(const iak_pack_args* a, void* stream) {
  if (!a) return fail(IAK_ERR_INVALID_ARG, "null args");
  if (a->batch < 0 || a->num_table_heads < 0 || a->table_width < 0 || a->num_ids < 0 || a->num_logical_pages < 0)
    return fail(IAK_ERR_INVALID_ARG, "negative size in pack args");
  const int64_t rows = static_cast<int64_t>(a->batch) * a->num_table_heads;
  if (rows == 0) return IAK_OK;
  if (!a->page_table && a->table_width > 0) return fail(IAK_ERR_INVALID_ARG, "page_table is NULL");
  if (a->num_ids > 0 && a->table_width > 0 && !a->logical_ids) return fail(IAK_ERR_INVALID_ARG, "logical_ids is NULL");
  if (rows > 0x7FFFFFFFLL) return fail(IAK_ERR_UNSUPPORTED, "too many rows");
  pack_kernel<<<static_cast<unsigned>(rows), 128, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return check_cuda(cudaGetLastError(), "pack launch");
}
