// KV append with quantise-on-write (iak_append_tokens) and page format
// transitions (iak_convert_pages).  Both rebuild whole pages with the page
// quantiser of quant_page.cuh, so a page written here holds exactly the codes
// and scales iak_quantize_pages would give for the same dense rows.
//
// Append: one CTA per (sequence, table head, plane).  The rows of the
// (b, h)'s open page live in an fp32 stage in global memory; the CTA writes
// the new rows into the stage (zeroing the rest of a page that begins inside
// the appended range), then re-quantises the staged page into its pool
// format.  Rebuilding from fp32 rows, rather than from the page's previous
// codes, keeps repeated appends free of double rounding.
//
// Convert: one CTA per listed page.  Both planes are dequantised into shared
// memory (code x scale as the decode kernels read it), then quantised into the
// target format over the same pool page, and the tag is rewritten.
#include "quant_page.cuh"

namespace iak {
namespace {

using qpage::kThreads;

struct AppendParams {
  qpage::PlanePools k, v;
  const void* k_new; const void* v_new; int new_dtype;
  int B, Ht, n_new;
  const int32_t* positions; int32_t* new_lengths;
  const int32_t* bases;
  const void* tags; int tag_bytes; uint8_t tag_map[16]; uint8_t tag_default;
  float* k_stage; float* v_stage;
  int32_t* dropped;
};

struct ConvertParams {
  qpage::PlanePools k, v;
  const int32_t* ids; int n;
  const uint8_t* new_formats;
  void* tags; int tag_bytes; uint8_t tag_map[16]; uint8_t tag_default;
  uint8_t fmt_to_tag[8];
  int32_t* rejected;
};

__device__ __forceinline__ int tag_format(const void* tags, int tag_bytes, const uint8_t* tag_map, int tag_default,
                                          int64_t pid) {
  const int tag = tag_bytes == 1 ? static_cast<int>(static_cast<const uint8_t*>(tags)[pid])
                                 : static_cast<const int32_t*>(tags)[pid];
  return (tag >= 0 && tag < 16) ? tag_map[tag] : tag_default;
}

__global__ void __launch_bounds__(kThreads) append_kernel(const AppendParams p) {
  __shared__ qpage::Scratch scratch;
  const int u = blockIdx.x, plane = blockIdx.y;
  const int b = u / p.Ht;
  const qpage::PlanePools q = plane ? p.v : p.k;
  const void* src = plane ? p.v_new : p.k_new;
  const int PS = q.PS, D = q.D, n = p.n_new;
  float* stage = (plane ? p.v_stage : p.k_stage) + static_cast<int64_t>(u) * PS * D;
  const int pos0 = p.positions[b];
  if (threadIdx.x == 0 && plane == 0 && (u % p.Ht) == 0 && p.new_lengths) p.new_lengths[b] = pos0 + n;
  if (pos0 < 0) {
    if (threadIdx.x == 0 && plane == 0 && p.dropped) atomicAdd(p.dropped, 1);
    return;
  }
  const int64_t base = p.bases ? p.bases[u] : 0;
  const int64_t src_row0 = static_cast<int64_t>(u) * n;
  auto X = [&](int t, int d) { return stage[t * D + d]; };
  for (int pg = pos0 / PS; pg <= (pos0 + n - 1) / PS; ++pg) {
    const int r0 = max(pos0, pg * PS) - pg * PS;
    const int r1 = min(pos0 + n, (pg + 1) * PS) - pg * PS;
    for (int e = threadIdx.x; e < PS * D; e += kThreads) {
      const int t = e / D, d = e - t * D;
      if (t >= r0 && t < r1)
        stage[e] = load_as_float(src, p.new_dtype, (src_row0 + pg * PS + t - pos0) * D + d);
      else if (r0 == 0 && t >= r1)
        stage[e] = 0.f;
    }
    __syncthreads();
    const int64_t phys = base + pg;
    if (phys >= 0 && phys < q.num_pages) {
      const int fmt = tag_format(p.tags, p.tag_bytes, p.tag_map, p.tag_default, phys);
      if (qpage::writable(q, fmt)) qpage::quantize_page(q, X, fmt, phys, nullptr, nullptr, scratch);
    } else if (threadIdx.x == 0 && plane == 0 && p.dropped) {
      atomicAdd(p.dropped, 1);
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kThreads) convert_kernel(const ConvertParams p) {
  extern __shared__ float page[];   // [PS * D]
  __shared__ qpage::Scratch scratch;
  const int64_t pid = p.ids[blockIdx.x];
  if (pid < 0 || pid >= p.k.num_pages) return;
  const int nf = p.new_formats[blockIdx.x];
  if (nf > IAK_FMT_SPARSE) return;
  const int cur = tag_format(p.tags, p.tag_bytes, p.tag_map, p.tag_default, pid);
  if (cur == nf) return;
  const bool keeps_data = nf != IAK_FMT_SKIP && nf != IAK_FMT_SPARSE;
  if (keeps_data && !(qpage::writable(p.k, nf) && qpage::writable(p.v, nf))) {
    if (threadIdx.x == 0 && p.rejected) atomicAdd(p.rejected, 1);
    return;
  }
  if (keeps_data) {
    const int PS = p.k.PS, D = p.k.D;
    auto X = [&](int t, int d) { return page[t * D + d]; };
    for (int plane = 0; plane < 2; ++plane) {
      const qpage::PlanePools q = plane ? p.v : p.k;
      for (int e = threadIdx.x; e < PS * D; e += kThreads) {
        const int t = e / D;
        page[e] = qpage::dequant(q, cur, pid, t, e - t * D);
      }
      __syncthreads();
      qpage::quantize_page(q, X, nf, pid, nullptr, nullptr, scratch);
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    const uint8_t tag = p.fmt_to_tag[nf];
    if (p.tag_bytes == 1) static_cast<uint8_t*>(p.tags)[pid] = tag;
    else static_cast<int32_t*>(p.tags)[pid] = tag;
  }
}

// Plane pools of one page-pool descriptor (plane 0 = K, 1 = V).
qpage::PlanePools plane_pools(const iak_page_pools& s, int plane) {
  qpage::PlanePools o;
  o.f16 = static_cast<__half*>(plane ? s.v_f16 : s.k_f16);
  o.fp8 = static_cast<uint8_t*>(plane ? s.v_fp8 : s.k_fp8);
  o.i8 = static_cast<int8_t*>(plane ? s.v_i8 : s.k_i8);
  o.i4 = static_cast<uint8_t*>(plane ? s.v_i4 : s.k_i4);
  o.i4r = static_cast<uint8_t*>(plane ? s.v_i4r : s.k_i4r);
  o.scale = plane ? s.v_scale : s.k_scale;
  o.res_scale = plane ? s.v_res_scale : s.k_res_scale;
  o.num_pages = s.num_pages; o.PS = s.page_size; o.D = s.head_dim; o.mode = s.scale_mode;
  o.ns = n_scales_of(s.scale_mode, s.head_dim);
  return o;
}

int check_pools(const iak_page_pools* s) {
  if (!s) return fail(IAK_ERR_INVALID_ARG, "null pools");
  const int D = s->head_dim, PS = s->page_size;
  if (D <= 0 || D > qpage::kMaxD || D % 16) return fail(IAK_ERR_UNSUPPORTED, "head_dim %d unsupported", D);
  if (PS <= 0) return fail(IAK_ERR_INVALID_ARG, "page_size must be positive");
  if (s->num_pages < 0) return fail(IAK_ERR_INVALID_ARG, "num_pages < 0");
  if (s->scale_mode < 0 || s->scale_mode > 2) return fail(IAK_ERR_INVALID_ARG, "bad scale_mode");
  if (s->scale_mode == IAK_SCALE_GROUP32 && D % 32) return fail(IAK_ERR_INVALID_ARG, "group32 needs head_dim %% 32 == 0");
  return IAK_OK;
}

}  // namespace
}  // namespace iak

using namespace iak;

extern "C" int iak_append_tokens(const iak_page_pools* pools, const iak_append_args* a, void* stream) {
  if (int st = check_pools(pools)) return st;
  if (!a) return fail(IAK_ERR_INVALID_ARG, "null append args");
  if (a->batch < 0 || a->num_table_heads < 0 || a->num_new < 0) return fail(IAK_ERR_INVALID_ARG, "negative size");
  if (a->batch == 0 || a->num_table_heads == 0 || a->num_new == 0) return IAK_OK;
  if (!a->k_new || !a->v_new || !a->positions || !a->page_tags || !a->k_stage || !a->v_stage)
    return fail(IAK_ERR_INVALID_ARG, "null append input / stage");
  if (a->new_dtype < 0 || a->new_dtype > 2) return fail(IAK_ERR_INVALID_ARG, "bad new_dtype");
  if (a->tag_bytes != 1 && a->tag_bytes != 4) return fail(IAK_ERR_INVALID_ARG, "tag_bytes must be 1 or 4");
  const int64_t units = static_cast<int64_t>(a->batch) * a->num_table_heads;
  if (units > 0x7FFFFFFFLL) return fail(IAK_ERR_UNSUPPORTED, "too many (sequence, head) units");
  AppendParams p;
  p.k = plane_pools(*pools, 0); p.v = plane_pools(*pools, 1);
  p.k_new = a->k_new; p.v_new = a->v_new; p.new_dtype = a->new_dtype;
  p.B = a->batch; p.Ht = a->num_table_heads; p.n_new = a->num_new;
  p.positions = a->positions; p.new_lengths = a->new_lengths; p.bases = a->bases;
  p.tags = a->page_tags; p.tag_bytes = a->tag_bytes;
  for (int i = 0; i < 16; ++i) p.tag_map[i] = a->tag_map[i];
  p.tag_default = a->tag_default;
  p.k_stage = a->k_stage; p.v_stage = a->v_stage; p.dropped = a->dropped;
  append_kernel<<<dim3(static_cast<unsigned>(units), 2), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "append launch");
}

extern "C" int iak_convert_pages(const iak_page_pools* pools, const iak_convert_args* a, void* stream) {
  if (int st = check_pools(pools)) return st;
  if (!a) return fail(IAK_ERR_INVALID_ARG, "null convert args");
  if (a->num_ids < 0) return fail(IAK_ERR_INVALID_ARG, "num_ids < 0");
  if (a->num_ids == 0) return IAK_OK;
  if (!a->page_ids || !a->new_formats || !a->page_tags) return fail(IAK_ERR_INVALID_ARG, "null convert input");
  if (a->tag_bytes != 1 && a->tag_bytes != 4) return fail(IAK_ERR_INVALID_ARG, "tag_bytes must be 1 or 4");
  const int64_t elems = static_cast<int64_t>(pools->page_size) * pools->head_dim;
  if (elems > IAK_CONVERT_MAX_ELEMS)
    return fail(IAK_ERR_UNSUPPORTED, "page_size * head_dim = %lld exceeds %d", static_cast<long long>(elems),
                IAK_CONVERT_MAX_ELEMS);
  ConvertParams p;
  p.k = plane_pools(*pools, 0); p.v = plane_pools(*pools, 1);
  p.ids = a->page_ids; p.n = a->num_ids; p.new_formats = a->new_formats;
  p.tags = a->page_tags; p.tag_bytes = a->tag_bytes;
  for (int i = 0; i < 16; ++i) p.tag_map[i] = a->tag_map[i];
  p.tag_default = a->tag_default;
  for (int i = 0; i < 8; ++i) p.fmt_to_tag[i] = a->fmt_to_tag[i];
  p.rejected = a->rejected;
  const size_t smem = static_cast<size_t>(elems) * sizeof(float);
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(convert_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               IAK_CONVERT_MAX_ELEMS * static_cast<int>(sizeof(float)));
    if (e != cudaSuccess) return check_cuda(e, "convert smem attribute");
    attr = true;
  }
  convert_kernel<<<static_cast<unsigned>(a->num_ids), kThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "convert launch");
}
