// MLA (absorbed latent) decode: argument validation, split planning, the
// CUDA-core kernel for any shape, and the C ABI entry points.
//
// Reference semantics (manishklach/intent-attention-kernel,
// src/intent_attention/triton_mla_decode.py:155-186 _mla_decode_cpu): per
// query row, an online softmax over the selected latent pages with the
// latent row as key (d_qk channels) and value (its first d_v channels),
// scale 1/sqrt(d_c) by default, rows without pages -> 0.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "iak_internal.cuh"
#include "mla_internal.cuh"

namespace iak {
namespace {

constexpr int kGenWarps = 4;  // query rows per CTA of the CUDA-core kernel

__device__ __forceinline__ int mla_page_format(const MlaParams& p, int64_t pid) {
  if (!p.tags) return IAK_MLA_DENSE;
  const int tag = p.tag_bytes == 1 ? static_cast<int>(static_cast<const uint8_t*>(p.tags)[pid])
                                   : static_cast<const int32_t*>(p.tags)[pid];
  return (tag >= 0 && tag < 16) ? p.tag_map[tag] : p.tag_default;
}

// One warp per query row (b, h); lane owns channels lane + 32 i.  Pages
// are read straight from global memory (rows of one CTA share them in L1/L2).
template <int QPL, int VPL>
__global__ void __launch_bounds__(kGenWarps * 32) mla_generic_kernel(const MlaParams p) {
  const int split = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.z * kGenWarps + warp;
  if (h >= p.H) return;
  const int64_t row = static_cast<int64_t>(b) * p.H + h;
  const int n_tab = p.pc ? min(max(p.pc[b], 0), p.W) : p.W;
  const int lo = split * p.pages_per_split, hi = min(n_tab, lo + p.pages_per_split);

  float q[QPL];
#pragma unroll
  for (int i = 0; i < QPL; ++i) {
    const int d = lane + 32 * i;
    q[i] = d < p.Dqk ? load_as_float(p.q, p.q_dtype, b * p.q_sb + h * p.q_sh + d) * p.sm_scale : 0.f;
  }
  float m = -INFINITY, l = 0.f, acc[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc[i] = 0.f;

  const int32_t* table = p.pt + static_cast<int64_t>(b) * p.pt_sb;
  for (int j = lo; j < hi; ++j) {
    const int64_t pid = table[j];
    if (pid < 0 || pid >= p.num_pages) continue;
    const int fmt = mla_page_format(p, pid);
    if (fmt != IAK_MLA_DENSE && fmt != IAK_MLA_FP8) continue;
    const float sc = fmt == IAK_MLA_FP8 ? p.fp8_scale[pid] : 1.f;
    const int64_t base = pid * p.PS * p.Dqk;
    for (int t = 0; t < p.PS; ++t) {
      const int64_t rb = base + static_cast<int64_t>(t) * p.Dqk;
      float c[QPL];
#pragma unroll
      for (int i = 0; i < QPL; ++i) {
        const int d = lane + 32 * i;
        float x = 0.f;
        if (d < p.Dqk)
          x = fmt == IAK_MLA_FP8 ? e4m3_to_float(p.fp8[rb + d]) * sc : load_as_float(p.dense, p.dense_dtype, rb + d);
        c[i] = x;
      }
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < QPL; ++i) s = fmaf(q[i], c[i], s);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      const float mn = fmaxf(m, s);
      const float alpha = expf(m - mn);
      const float e = expf(s - mn);
      l = l * alpha + e;
#pragma unroll
      for (int i = 0; i < VPL; ++i) acc[i] = acc[i] * alpha + e * c[i];
      m = mn;
    }
  }

  if (p.num_splits > 1) {
    const int64_t wi = row * p.num_splits + split;
    if (lane == 0) {
      p.ws_m[wi] = m;
      p.ws_l[wi] = l;
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int d = lane + 32 * i;
      if (d < p.Dv) p.ws_acc[wi * p.Dv + d] = acc[i];
    }
  } else if (p.ex_l) {
    if (lane == 0) {
      p.ex_m[row] = m;
      p.ex_l[row] = l;
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int d = lane + 32 * i;
      if (d < p.Dv) p.ex_acc[row * p.Dv + d] = acc[i];
    }
  } else {
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int d = lane + 32 * i;
      if (d < p.Dv) store_from_float(p.out, p.out_dtype, b * p.o_sb + h * p.o_sh + d, acc[i] * inv);
    }
  }
}

template <int QPL>
int launch_generic_q(const MlaParams& p, int vpl, cudaStream_t s) {
  dim3 grid(p.num_splits, p.B, (p.H + kGenWarps - 1) / kGenWarps);
  if (vpl <= 4) mla_generic_kernel<QPL, 4><<<grid, kGenWarps * 32, 0, s>>>(p);
  else if (vpl <= 8) mla_generic_kernel<QPL, 8><<<grid, kGenWarps * 32, 0, s>>>(p);
  else if (vpl <= 16) mla_generic_kernel<QPL, 16><<<grid, kGenWarps * 32, 0, s>>>(p);
  else mla_generic_kernel<QPL, 32><<<grid, kGenWarps * 32, 0, s>>>(p);
  return check_cuda(cudaGetLastError(), "mla_generic launch");
}

int launch_mla_generic(const MlaParams& p, cudaStream_t s) {
  const int qpl = (p.Dqk + 31) / 32, vpl = (p.Dv + 31) / 32;
  kernel_timer_begin(s);
  int st;
  if (qpl <= 4) st = launch_generic_q<4>(p, vpl, s);
  else if (qpl <= 8) st = launch_generic_q<8>(p, vpl, s);
  else if (qpl <= 16) st = launch_generic_q<16>(p, vpl, s);
  else if (qpl <= 24) st = launch_generic_q<24>(p, vpl, s);
  else st = launch_generic_q<32>(p, vpl, s);
  kernel_timer_end(s);
  return st;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

int prepare_mla(const iak_mla_args* a, MlaParams* p) {
  if (!a) return fail(IAK_ERR_INVALID_ARG, "null mla args");
  if (a->batch < 0 || a->num_heads <= 0) return fail(IAK_ERR_INVALID_ARG, "batch/heads must be positive");
  if (a->d_qk <= 0 || a->d_qk > 1024) return fail(IAK_ERR_UNSUPPORTED, "d_qk %d unsupported (1..1024)", a->d_qk);
  if (a->d_v <= 0 || a->d_v > a->d_qk) return fail(IAK_ERR_INVALID_ARG, "d_v %d must be in 1..d_qk", a->d_v);
  if (a->page_size <= 0 || a->page_size > 1024) return fail(IAK_ERR_INVALID_ARG, "page_size %d out of range", a->page_size);
  if (a->num_pages < 0 || a->table_width < 0) return fail(IAK_ERR_INVALID_ARG, "negative num_pages / table_width");
  if (a->q_dtype < 0 || a->q_dtype > 2 || a->out_dtype < 0 || a->out_dtype > 2 || a->dense_dtype < 0 ||
      a->dense_dtype > 2)
    return fail(IAK_ERR_INVALID_ARG, "bad dtype");
  if (a->page_tags && a->tag_bytes != 1 && a->tag_bytes != 4) return fail(IAK_ERR_INVALID_ARG, "tag_bytes must be 1 or 4");
  bool dense_used = !a->page_tags, fp8_used = false;
  if (a->page_tags) {
    for (int i = 0; i < 16; ++i) {
      if (a->tag_map[i] > IAK_MLA_FP8) return fail(IAK_ERR_INVALID_ARG, "tag_map[%d]=%d is not an MLA format", i, a->tag_map[i]);
      dense_used |= a->tag_map[i] == IAK_MLA_DENSE;
      fp8_used |= a->tag_map[i] == IAK_MLA_FP8;
    }
    if (a->tag_default > IAK_MLA_FP8) return fail(IAK_ERR_INVALID_ARG, "bad tag_default");
    dense_used |= a->tag_default == IAK_MLA_DENSE;
    fp8_used |= a->tag_default == IAK_MLA_FP8;
  }
  const bool work = a->batch > 0 && a->table_width > 0;
  if (work) {
    if (!a->q || !a->page_table) return fail(IAK_ERR_INVALID_ARG, "q / page_table is NULL");
    if (!a->out && !a->partial_l) return fail(IAK_ERR_INVALID_ARG, "out is NULL");
    if (dense_used && !a->dense_pages) return fail(IAK_ERR_INVALID_ARG, "a tag maps to dense pages but dense_pages is NULL");
    if (fp8_used && (!a->fp8_pages || !a->fp8_scale))
      return fail(IAK_ERR_INVALID_ARG, "a tag maps to FP8 pages but fp8_pages / fp8_scale is NULL");
  }
  if (a->partial_l && (!a->partial_m || !a->partial_acc)) return fail(IAK_ERR_INVALID_ARG, "partial export needs m, l and acc");
  std::memset(p, 0, sizeof(*p));
  p->q = a->q; p->q_dtype = a->q_dtype; p->q_sb = a->q_stride_b; p->q_sh = a->q_stride_h;
  p->out = a->out; p->out_dtype = a->out_dtype; p->o_sb = a->out_stride_b; p->o_sh = a->out_stride_h;
  p->B = a->batch; p->H = a->num_heads; p->Dqk = a->d_qk; p->Dv = a->d_v;
  p->dense = a->dense_pages; p->dense_dtype = a->dense_dtype;
  p->fp8 = a->fp8_pages; p->fp8_scale = a->fp8_scale;
  p->num_pages = a->num_pages; p->PS = a->page_size;
  p->pt = a->page_table; p->pt_sb = a->pt_stride_b; p->W = a->table_width; p->pc = a->page_counts;
  p->tags = a->page_tags; p->tag_bytes = a->tag_bytes;
  std::memcpy(p->tag_map, a->tag_map, 16); p->tag_default = a->tag_default;
  p->sm_scale = a->sm_scale;
  p->ex_m = a->partial_m; p->ex_l = a->partial_l; p->ex_acc = a->partial_acc;
  p->kernel = a->kernel;
  const bool tc_ok = mla_tc_eligible(*p);
  if (a->kernel == IAK_KERNEL_TENSOR && !tc_ok)
    return fail(IAK_ERR_UNSUPPORTED, "tensor-core MLA needs d_qk=576, d_v=512, heads<=128, page_size%%64==0, "
                "bf16/f16 q, dense pages bf16/f16, a positive sm_scale (got d_qk=%d d_v=%d H=%d PS=%d)", p->Dqk, p->Dv, p->H, p->PS);
  p->tensor = tc_ok && a->kernel != IAK_KERNEL_GENERIC && work;
  int splits = a->num_splits;
  const int W = a->table_width;
  if (p->tensor) {
    plan_mla_tc(p, splits);
  } else {
    if (splits <= 0) {
      const int64_t ctas = static_cast<int64_t>(a->batch) * ((a->num_heads + kGenWarps - 1) / kGenWarps);
      const int64_t target = 4LL * device_sm_count();
      const int64_t s = ctas > 0 ? (target + ctas - 1) / ctas : 1;
      splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(s, std::max(1, W / 2))));
    }
    splits = std::max(1, std::min(splits, std::max(1, W)));
    p->pages_per_split = W > 0 ? (W + splits - 1) / splits : 1;
    p->num_splits = W > 0 ? (W + p->pages_per_split - 1) / p->pages_per_split : 1;
  }
  if (p->num_splits > 65535) return fail(IAK_ERR_UNSUPPORTED, "too many splits");
  return IAK_OK;
}

size_t mla_workspace_bytes(const MlaParams& p) {
  if (p.num_splits <= 1) return 0;
  const size_t n = static_cast<size_t>(p.B) * p.H * p.num_splits;
  return align256(n * 4) * 2 + align256(n * p.Dv * 4);
}

}  // namespace
}  // namespace iak

using namespace iak;

extern "C" {

int iak_mla_workspace_size(const iak_mla_args* args, size_t* bytes) {
  if (!bytes) return fail(IAK_ERR_INVALID_ARG, "bytes is NULL");
  MlaParams p;
  const int st = prepare_mla(args, &p);
  if (st) return st;
  *bytes = mla_workspace_bytes(p);
  return IAK_OK;
}

int iak_mla_decode(const iak_mla_args* args, void* workspace, size_t ws_bytes, void* stream) {
  MlaParams p;
  int st = prepare_mla(args, &p);
  if (st) return st;
  if (p.B == 0) return IAK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t need = mla_workspace_bytes(p);
  if (need > 0) {
    if (!workspace || ws_bytes < need)
      return fail(IAK_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace ? ws_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(IAK_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    const size_t n = static_cast<size_t>(p.B) * p.H * p.num_splits;
    char* w = static_cast<char*>(workspace);
    p.ws_m = reinterpret_cast<float*>(w);
    p.ws_l = reinterpret_cast<float*>(w + align256(n * 4));
    p.ws_acc = reinterpret_cast<float*>(w + 2 * align256(n * 4));
  }
  if (p.W == 0) {
    MlaParams z = p;
    z.num_splits = 1; z.pages_per_split = 1; z.tensor = 0;
    return launch_mla_generic(z, s);
  }
  st = p.tensor ? launch_mla_tc(p, s) : launch_mla_generic(p, s);
  if (st) return st;
  if (p.num_splits > 1) {
    DecodeParams rowmap;
    std::memset(&rowmap, 0, sizeof(rowmap));
    rowmap.Hq = p.H; rowmap.o_sb = p.o_sb; rowmap.o_sh = p.o_sh;
    st = launch_merge(p.ws_m, p.ws_l, p.ws_acc, static_cast<int64_t>(p.B) * p.H, p.num_splits, p.Dv, p.out,
                      p.out_dtype, 0, &rowmap, p.ex_m, p.ex_l, p.ex_acc, s);
  }
  return st;
}

}  // extern "C"
