// Quantise-on-write: dense K or V pages -> the page-pool formats (the page
// arithmetic lives in quant_page.cuh).
#include "quant_page.cuh"

namespace iak {

namespace {

using qpage::kThreads;
using qpage::kMaxD;

struct QuantParams {
  const void* x; int x_dtype; int64_t P;
  const int32_t* dst_ids; const uint8_t* formats;
  const float* given; const float* given_res;
  qpage::PlanePools pools;
};

__global__ void __launch_bounds__(kThreads) quantize_kernel(const QuantParams q) {
  __shared__ qpage::Scratch scratch;
  const int64_t i = blockIdx.x;
  const int fmt = q.formats[i];
  const int64_t dst = q.dst_ids ? static_cast<int64_t>(q.dst_ids[i]) : i;
  if (dst < 0 || dst >= q.pools.num_pages) return;
  // formats live in device memory, so a page whose pool (or scale array) was
  // not supplied is skipped rather than written through a null pointer
  if (!qpage::writable(q.pools, fmt)) return;
  const int PS = q.pools.PS, D = q.pools.D, ns = q.pools.ns;
  const int64_t src = i * PS * D;
  auto X = [&](int t, int d) { return load_as_float(q.x, q.x_dtype, src + static_cast<int64_t>(t) * D + d); };
  qpage::quantize_page(q.pools, X, fmt, dst, q.given ? q.given + i * ns : nullptr,
                       q.given_res ? q.given_res + i * ns : nullptr, scratch);
}

}  // namespace

}  // namespace iak

using namespace iak;

extern "C" int iak_quantize_pages(const iak_quant_args* a, void* stream) {
  if (!a) return fail(IAK_ERR_INVALID_ARG, "null args");
  if (a->num_src_pages < 0) return fail(IAK_ERR_INVALID_ARG, "num_src_pages < 0");
  if (a->num_src_pages == 0) return IAK_OK;
  const int D = a->head_dim, PS = a->page_size;
  if (D <= 0 || D > kMaxD || D % 16) return fail(IAK_ERR_UNSUPPORTED, "head_dim %d unsupported", D);
  if (PS <= 0) return fail(IAK_ERR_INVALID_ARG, "page_size must be positive");
  if (a->scale_mode < 0 || a->scale_mode > 2) return fail(IAK_ERR_INVALID_ARG, "bad scale_mode");
  if (a->scale_mode == IAK_SCALE_GROUP32 && D % 32) return fail(IAK_ERR_INVALID_ARG, "group32 needs head_dim %% 32 == 0");
  if (!a->x || !a->formats) return fail(IAK_ERR_INVALID_ARG, "x/formats is NULL");
  if (a->x_dtype < 0 || a->x_dtype > 2) return fail(IAK_ERR_INVALID_ARG, "bad x dtype");
  if (a->num_src_pages > 0x7FFFFFFFLL) return fail(IAK_ERR_UNSUPPORTED, "too many pages in one call");
  QuantParams q;
  q.x = a->x; q.x_dtype = a->x_dtype; q.P = a->num_src_pages;
  q.dst_ids = a->dst_ids; q.formats = a->formats; q.given = a->given_scale; q.given_res = a->given_res_scale;
  qpage::PlanePools& o = q.pools;
  o.f16 = static_cast<__half*>(a->f16); o.fp8 = static_cast<uint8_t*>(a->fp8); o.i8 = static_cast<int8_t*>(a->i8);
  o.i4 = static_cast<uint8_t*>(a->i4); o.i4r = static_cast<uint8_t*>(a->i4r);
  o.scale = a->scale; o.res_scale = a->res_scale;
  o.num_pages = a->num_pages; o.PS = PS; o.D = D; o.mode = a->scale_mode; o.ns = n_scales_of(a->scale_mode, D);
  quantize_kernel<<<static_cast<unsigned>(a->num_src_pages), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(q);
  return check_cuda(cudaGetLastError(), "quantize launch");
}
