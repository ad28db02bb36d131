// Multi-query (prefill / chunked prefill) attention over selected pages:
// host entry point, argument checks, and the CUDA-core kernel used for the
// shapes the tensor-core kernel (prefill_tc.cu) does not take and as its
// independent cross-check.
//
// Semantics: reference.py:82-130 semantic_block_attention with causal masks on
// original positions (reference.py:16-45), over page pools: the keys of unit
// (b, h) are the rows selected by each slot's row mask, at token position
// (page - base) * page_size + row; a query row that sees no key writes 0.
#include "prefill_internal.cuh"

namespace iak {
namespace {

constexpr int kGenericWarps = 8;
constexpr int kMaxPerLane = 8;   // head_dim <= 256

// One warp per query row (b, hq, m): each lane holds head_dim / 32 channels of
// q and of the accumulator; keys are visited one row at a time with a warp
// reduction per score and an online softmax in the exp2 domain.
__global__ void __launch_bounds__(kGenericWarps * 32) prefill_generic_kernel(const PrefillParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x * kGenericWarps + warp;
  const int hq = blockIdx.y, b = blockIdx.z;
  if (m >= p.M) return;
  const int h = hq / p.G, D = p.k.D, PS = p.k.PS;
  const float qs = p.sm_scale * 1.4426950408889634f;
  float qv[kMaxPerLane], acc[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < D ? load_as_float(p.q, p.q_dtype, b * p.q_sb + hq * p.q_sh + m * p.q_sm + d) * qs : 0.f;
    acc[i] = 0.f;
  }
  const int qpos = p.qpos ? p.qpos[static_cast<int64_t>(b) * p.qp_sb + m] : m;
  const int count = prefill_count(p, b, h);
  const int64_t base = p.bases ? p.bases[static_cast<int64_t>(b) * p.Ht + h] : 0;
  const int32_t* row = p.pt + static_cast<int64_t>(b) * p.pt_sb + static_cast<int64_t>(h) * p.pt_sh;
  float mx = -INFINITY, l = 0.f;
  for (int o = 0; o < count; ++o) {
    const int64_t pid = row[o];
    if (pid < 0 || pid >= p.k.num_pages) continue;
    const int fmt = prefill_fmt(p, pid);
    if (!qpage::writable(p.k, fmt) || !qpage::writable(p.v, fmt)) continue;
    const uint64_t mask = prefill_mask(p, b, o);
    const int64_t pos0 = prefill_pos0(p, b, h, o, pid, base);
    for (int r = 0; r < PS; ++r) {
      if (!((mask >> r) & 1ull)) continue;
      if (p.causal && pos0 + r > qpos) continue;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < D) s += qv[i] * qpage::dequant(p.k, fmt, pid, r, d);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      const float mn = fmaxf(mx, s);
      const float corr = exp2f(mx - mn);   // 0 on the first visible key (mx = -inf)
      const float e = exp2f(s - mn);
      l = l * corr + e;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] = acc[i] * corr + e * qpage::dequant(p.v, fmt, pid, r, d);
      }
      mx = mn;
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < D) store_from_float(p.out, p.out_dtype, b * p.o_sb + hq * p.o_sh + m * p.o_sm + d, acc[i] * inv);
  }
}

qpage::PlanePools plane_of(const iak_page_pools& s, int plane) {
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

}  // namespace
}  // namespace iak

using namespace iak;

extern "C" int iak_prefill(const iak_page_pools* pools, const iak_prefill_args* a, void* stream) {
  if (!pools || !a) return fail(IAK_ERR_INVALID_ARG, "null prefill args");
  const int D = pools->head_dim, PS = pools->page_size;
  if (D <= 0 || D > 256 || D % 16) return fail(IAK_ERR_UNSUPPORTED, "prefill head_dim %d unsupported (16..256)", D);
  if (PS <= 0) return fail(IAK_ERR_INVALID_ARG, "page_size must be positive");
  if (pools->scale_mode < 0 || pools->scale_mode > 2) return fail(IAK_ERR_INVALID_ARG, "bad scale_mode");
  if (pools->scale_mode == IAK_SCALE_GROUP32 && D % 32) return fail(IAK_ERR_INVALID_ARG, "group32 needs head_dim %% 32 == 0");
  if (a->batch < 0 || a->num_q_heads < 0 || a->num_table_heads < 0 || a->num_queries < 0 || a->table_width < 0)
    return fail(IAK_ERR_INVALID_ARG, "negative size in prefill args");
  if (a->batch == 0 || a->num_q_heads == 0 || a->num_queries == 0) return IAK_OK;
  if (a->num_table_heads == 0 || a->num_q_heads % a->num_table_heads)
    return fail(IAK_ERR_INVALID_ARG, "num_q_heads (%d) must be a multiple of num_table_heads (%d)", a->num_q_heads,
                a->num_table_heads);
  if (!a->q || !a->out || (a->table_width > 0 && !a->page_table) || !a->page_tags)
    return fail(IAK_ERR_INVALID_ARG, "null prefill input / output");
  if (a->q_dtype < 0 || a->q_dtype > 2 || a->out_dtype < 0 || a->out_dtype > 2)
    return fail(IAK_ERR_INVALID_ARG, "bad q / out dtype");
  if (a->tag_bytes != 1 && a->tag_bytes != 4) return fail(IAK_ERR_INVALID_ARG, "tag_bytes must be 1 or 4");
  if (a->row_masks && PS > 64) return fail(IAK_ERR_UNSUPPORTED, "row masks need page_size <= 64");
  if (a->batch > 65535 || a->num_q_heads > 65535) return fail(IAK_ERR_UNSUPPORTED, "batch / heads too large");
  PrefillParams p;
  p.k = plane_of(*pools, 0); p.v = plane_of(*pools, 1);
  p.q = a->q; p.q_dtype = a->q_dtype; p.q_sb = a->q_stride_b; p.q_sh = a->q_stride_h; p.q_sm = a->q_stride_m;
  p.out = a->out; p.out_dtype = a->out_dtype;
  p.o_sb = a->out_stride_b; p.o_sh = a->out_stride_h; p.o_sm = a->out_stride_m;
  p.B = a->batch; p.Hq = a->num_q_heads; p.Ht = a->num_table_heads; p.G = a->num_q_heads / a->num_table_heads;
  p.M = a->num_queries;
  p.qpos = a->q_positions; p.qp_sb = a->qp_stride_b; p.causal = a->causal ? 1 : 0;
  p.pt = a->page_table; p.pt_sb = a->pt_stride_b; p.pt_sh = a->pt_stride_h; p.W = a->table_width;
  p.pc = a->page_counts; p.pc_sb = a->pc_stride_b;
  p.bases = a->bases; p.masks = a->row_masks; p.rm_sb = a->rm_stride_b;
  p.ppos = a->page_positions; p.pp_sb = a->pp_stride_b; p.pp_sh = a->pp_stride_h;
  p.tags = a->page_tags; p.tag_bytes = a->tag_bytes;
  for (int i = 0; i < 16; ++i) p.tag_map[i] = a->tag_map[i];
  p.tag_default = a->tag_default;
  p.sm_scale = a->sm_scale;
  p.q_vec = (a->q_dtype != IAK_DT_F32 && reinterpret_cast<uintptr_t>(a->q) % 16 == 0 && a->q_stride_b % 8 == 0 &&
             a->q_stride_h % 8 == 0 && a->q_stride_m % 8 == 0) ? 1 : 0;
  {
    const int64_t esz = a->out_dtype == IAK_DT_F32 ? 4 : 2, per16 = 16 / esz;
    p.o_vec = (reinterpret_cast<uintptr_t>(a->out) % 16 == 0 && a->out_stride_b % per16 == 0 &&
               a->out_stride_h % per16 == 0 && a->out_stride_m % per16 == 0) ? 1 : 0;
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tc_ok = prefill_tc_eligible(p);
  if (a->kernel == IAK_KERNEL_TENSOR && !tc_ok)
    return fail(IAK_ERR_UNSUPPORTED, "the tensor-core prefill needs head_dim 128, page_size in {8,16,32,64}, "
                                     "table_width <= 1024, 16-byte aligned pools and a positive sm_scale");
  if (a->kernel != IAK_KERNEL_GENERIC && tc_ok) return launch_prefill_tc(p, s);
  const dim3 grid(static_cast<unsigned>((p.M + kGenericWarps - 1) / kGenericWarps), static_cast<unsigned>(p.Hq),
                  static_cast<unsigned>(p.B));
  prefill_generic_kernel<<<grid, kGenericWarps * 32, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "prefill launch");
}
