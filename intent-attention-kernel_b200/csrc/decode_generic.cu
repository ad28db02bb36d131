// Generic split-KV paged decode: any head_dim <= 256 (multiple of 16), any
// page size, G <= 8 query heads per page table, every page format and scale
// mode.  CUDA-core fp32 arithmetic, one warp per page, loads straight from
// global memory.  It serves shapes the tensor-core kernel does not cover and
// doubles as an independent cross-check of that kernel.
//
// Semantics follow fused_selected_quant_decode.py:290-334 (per (b, h) online
// softmax over the selected pages, SKIP pages contribute nothing, empty ->
// zeros) generalised to G query heads per page list.
#include <cfloat>

#include "iak_internal.cuh"

namespace iak {

namespace {

constexpr int kWarps = 4;
constexpr int kMaxG = 8;

__device__ __forceinline__ float scale_at(const float* s, int mode, int64_t pid, int n_scales, int d) {
  if (mode == IAK_SCALE_PAGE) return s[pid];
  if (mode == IAK_SCALE_GROUP32) return s[pid * n_scales + (d >> 5)];
  return s[pid * n_scales + d];
}

template <int DPL>
__device__ __forceinline__ void load_plane(const DecodeParams& p, int fmt, bool is_v, int64_t pid, int t, int lane,
                                           const float (&sc)[DPL], const float (&rsc)[DPL], float (&x)[DPL]) {
  const int D = p.D;
  const int64_t row = pid * p.PS + t;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int d = lane + 32 * i;
    float v = 0.f;
    if (d < D) {
      switch (fmt) {
        case IAK_FMT_F16:
          v = __half2float((is_v ? p.v_f16 : p.k_f16)[row * D + d]);
          break;
        case IAK_FMT_FP8:
          v = e4m3_to_float((is_v ? p.v_fp8 : p.k_fp8)[row * D + d]) * sc[i];
          break;
        case IAK_FMT_INT8:
          v = static_cast<float>((is_v ? p.v_i8 : p.k_i8)[row * D + d]) * sc[i];
          break;
        case IAK_FMT_INT4:
          v = static_cast<float>(int4_code((is_v ? p.v_i4 : p.k_i4) + row * (D / 2), d)) * sc[i];
          break;
        case IAK_FMT_INT4R: {
          const float base = static_cast<float>(int4_code((is_v ? p.v_i4 : p.k_i4) + row * (D / 2), d)) * sc[i];
          const float res = static_cast<float>(int4_code((is_v ? p.v_i4r : p.k_i4r) + row * (D / 2), d)) * rsc[i];
          v = base + res;
          break;
        }
        default:
          break;
      }
    }
    x[i] = v;
  }
}

template <int DPL>
__global__ void __launch_bounds__(kWarps * 32) decode_generic_kernel(const DecodeParams p) {
  __shared__ float q_s[kMaxG * 256];
  __shared__ float red_m[kWarps][kMaxG];
  __shared__ float red_l[kWarps][kMaxG];
  __shared__ float red_acc[kWarps][kMaxG][256];

  const int unit = blockIdx.y, split = blockIdx.x;
  const int b = unit / p.Ht, hk = unit % p.Ht;
  const int G = p.G, D = p.D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int count = p.W;
  if (p.pc) {
    const int c = p.pc[b * p.pc_sb + hk];
    count = c < 0 ? 0 : (c > p.W ? p.W : c);
  }
  const int lo = split * p.pages_per_split;
  const int hi = min(lo + p.pages_per_split, count);

  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    const int hq = hk * G + g;
    q_s[idx] = load_as_float(p.q, p.q_dtype, b * p.q_sb + hq * p.q_sh + d);
  }
  __syncthreads();

  float m[kMaxG], l[kMaxG], acc[kMaxG][DPL];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[g][i] = 0.f;
  }

  const int32_t* table = p.pt + b * p.pt_sb + hk * p.pt_sh;
  for (int j = lo + warp; j < hi; j += kWarps) {
    const int64_t pid = table[j];
    if (pid < 0 || pid >= p.num_pages) continue;
    const int fmt = page_format(p, pid);
    if (fmt == IAK_FMT_SKIP || fmt == IAK_FMT_SPARSE) continue;
    float ks[DPL], vs[DPL], krs[DPL], vrs[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = min(lane + 32 * i, D - 1);
      ks[i] = vs[i] = krs[i] = vrs[i] = 1.f;
      if (fmt != IAK_FMT_F16) {
        ks[i] = scale_at(p.k_scale, p.scale_mode, pid, p.n_scales, d);
        vs[i] = scale_at(p.v_scale, p.scale_mode, pid, p.n_scales, d);
      }
      if (fmt == IAK_FMT_INT4R) {
        krs[i] = scale_at(p.k_rscale, p.scale_mode, pid, p.n_scales, d);
        vrs[i] = scale_at(p.v_rscale, p.scale_mode, pid, p.n_scales, d);
      }
    }
    for (int t = 0; t < p.PS; ++t) {
      float kx[DPL], vx[DPL];
      load_plane<DPL>(p, fmt, false, pid, t, lane, ks, krs, kx);
      load_plane<DPL>(p, fmt, true, pid, t, lane, vs, vrs, vx);
      float s[kMaxG];
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        float a = 0.f;
        if (g < G) {
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            if (d < D) a = fmaf(q_s[g * D + d], kx[i], a);
          }
        }
        s[g] = a;
      }
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s[g] += __shfl_xor_sync(0xffffffffu, s[g], off);
      }
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        if (g < G) {
          const float sc = s[g] * p.sm_scale;
          const float mn = fmaxf(m[g], sc);
          const float alpha = expf(m[g] - mn);
          const float e = expf(sc - mn);
          l[g] = l[g] * alpha + e;
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[g][i] = acc[g][i] * alpha + e * vx[i];
          m[g] = mn;
        }
      }
    }
  }

  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      red_m[warp][g] = m[g];
      red_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g < G) {
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        if (d < D) red_acc[warp][g][d] = acc[g][i];
      }
    }
  }
  __syncthreads();

  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      if (red_l[w][g] > 0.f) M = fmaxf(M, red_m[w][g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (red_l[w][g] > 0.f) {
          const float e = expf(red_m[w][g] - M);
          L += red_l[w][g] * e;
          A += red_acc[w][g][d] * e;
        }
      }
    }
    const int hq = hk * G + g;
    const int64_t r = static_cast<int64_t>(b) * p.Hq + hq;
    if (p.num_splits > 1) {
      const int64_t wi = r * p.ws_slots + split;
      if (d == 0) {
        p.ws_m[wi] = M;
        p.ws_l[wi] = L;
      }
      p.ws_acc[wi * D + d] = A;
    } else if (p.ex_l) {
      if (d == 0) {
        p.ex_m[r] = M;
        p.ex_l[r] = L;
      }
      p.ex_acc[r * D + d] = A;
    } else {
      store_from_float(p.out, p.out_dtype, b * p.o_sb + hq * p.o_sh + d, L > 0.f ? A / L : 0.f);
    }
  }
}

// LSE merge over splits: rows x splits partials -> normalised rows (or a
// merged partial when ex_l != nullptr).
// Partial (s) of row r: m/l at [r * ms_r + s * ms_s], acc at [r * as_r + s * as_s + d].
__global__ void merge_kernel(const float* __restrict__ m, const float* __restrict__ l, const float* __restrict__ acc,
                             int64_t ms_r, int64_t ms_s, int64_t as_r, int64_t as_s,
                             int64_t rows, int S, int D, void* out, int out_dtype, int64_t out_row_stride, int Hq,
                             int64_t o_sb, int64_t o_sh, float* ex_m, float* ex_l, float* ex_acc) {
  extern __shared__ float w_s[];
  __shared__ float stat[2];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* mr = m + r * ms_r;
    const float* lr = l + r * ms_r;
    if (threadIdx.x < 32) {
      float M = -INFINITY;
      for (int s = threadIdx.x; s < S; s += 32)
        if (lr[s * ms_s] > 0.f) M = fmaxf(M, mr[s * ms_s]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.f;
      for (int s = threadIdx.x; s < S; s += 32) {
        const float ls = lr[s * ms_s];
        const float w = (ls > 0.f && M != -INFINITY) ? expf(mr[s * ms_s] - M) : 0.f;
        w_s[s] = w;
        L += ls * w;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      if (threadIdx.x == 0) {
        stat[0] = M;
        stat[1] = L;
      }
    }
    __syncthreads();
    const float M = stat[0], L = stat[1];
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float A = 0.f;
      for (int s = 0; s < S; ++s) {
        const float w = w_s[s];
        if (w != 0.f) A = fmaf(acc[r * as_r + s * as_s + d], w, A);
      }
      if (ex_l) {
        ex_acc[r * D + d] = A;
      } else {
        int64_t off;
        if (Hq > 0) {
          const int64_t bb = r / Hq, hq = r % Hq;
          off = bb * o_sb + hq * o_sh + d;
        } else {
          off = r * out_row_stride + d;
        }
        store_from_float(out, out_dtype, off, L > 0.f ? A / L : 0.f);
      }
    }
    if (ex_l && threadIdx.x == 0) {
      ex_m[r] = M;
      ex_l[r] = L;
    }
    __syncthreads();
  }
}

// Vectorised LSE merge (same contract as merge_kernel) for D % 4 == 0 and
// 16-byte aligned acc rows: the 8 warps of a CTA take every 8th split slot,
// lanes take float4 groups of channels, and the warps' sums meet in shared memory.
constexpr int kMergeWarps = 8;
template <int C>   // float4 groups per lane: D <= 128 * C
__global__ void __launch_bounds__(kMergeWarps * 32) merge_vec_kernel(
    const float* __restrict__ m, const float* __restrict__ l, const float* __restrict__ acc, int64_t ms_r,
    int64_t ms_s, int64_t as_r, int64_t as_s, int64_t rows, int S, int D, void* out, int out_dtype,
    int64_t out_row_stride, int Hq, int64_t o_sb, int64_t o_sh, float* ex_m, float* ex_l, float* ex_acc) {
  extern __shared__ float sm_f[];
  float* w_s = sm_f;                       // [S]
  float* red = sm_f + ((S + 3) & ~3);      // [kMergeWarps][D]
  __shared__ float stat[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* mr = m + r * ms_r;
    const float* lr = l + r * ms_r;
    if (warp == 0) {
      float M = -INFINITY;
      for (int s = lane; s < S; s += 32)
        if (lr[s * ms_s] > 0.f) M = fmaxf(M, mr[s * ms_s]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.f;
      for (int s = lane; s < S; s += 32) {
        const float ls = lr[s * ms_s];
        const float w = (ls > 0.f && M != -INFINITY) ? expf(mr[s * ms_s] - M) : 0.f;
        w_s[s] = w;
        L += ls * w;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      if (lane == 0) {
        stat[0] = M;
        stat[1] = L;
      }
    }
    __syncthreads();
    float4 a[C];
#pragma unroll
    for (int c = 0; c < C; ++c) a[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* ar = acc + r * as_r;
#pragma unroll 4
    for (int s = warp; s < S; s += kMergeWarps) {
      const float w = w_s[s];
      if (w == 0.f) continue;
      const float4* src = reinterpret_cast<const float4*>(ar + s * as_s);
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int g = lane + 32 * c;
        if (4 * g < D) {
          const float4 v = src[g];
          a[c].x = fmaf(v.x, w, a[c].x); a[c].y = fmaf(v.y, w, a[c].y);
          a[c].z = fmaf(v.z, w, a[c].z); a[c].w = fmaf(v.w, w, a[c].w);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int g = lane + 32 * c;
      if (4 * g < D) reinterpret_cast<float4*>(red + warp * D)[g] = a[c];
    }
    __syncthreads();
    const float M = stat[0], L = stat[1];
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float A = 0.f;
#pragma unroll
      for (int w = 0; w < kMergeWarps; ++w) A += red[w * D + d];
      if (ex_l) {
        ex_acc[r * D + d] = A;
      } else {
        int64_t off;
        if (Hq > 0) {
          const int64_t bb = r / Hq, hq = r % Hq;
          off = bb * o_sb + hq * o_sh + d;
        } else {
          off = r * out_row_stride + d;
        }
        store_from_float(out, out_dtype, off, L > 0.f ? A / L : 0.f);
      }
    }
    if (ex_l && threadIdx.x == 0) {
      ex_m[r] = M;
      ex_l[r] = L;
    }
    __syncthreads();
  }
}

}  // namespace

int launch_decode_generic(const DecodeParams& p, cudaStream_t s) {
  const int units = p.B * p.Ht;
  if (units == 0) return IAK_OK;
  dim3 grid(p.num_splits, units);
  const int dpl = (p.D + 31) / 32;
  kernel_timer_begin(s);
  if (dpl <= 1) decode_generic_kernel<1><<<grid, kWarps * 32, 0, s>>>(p);
  else if (dpl <= 2) decode_generic_kernel<2><<<grid, kWarps * 32, 0, s>>>(p);
  else if (dpl <= 4) decode_generic_kernel<4><<<grid, kWarps * 32, 0, s>>>(p);
  else decode_generic_kernel<8><<<grid, kWarps * 32, 0, s>>>(p);
  const cudaError_t err = cudaGetLastError();
  kernel_timer_end(s);
  return check_cuda(err, "decode_generic launch");
}

int launch_merge(const float* m, const float* l, const float* acc, int64_t rows, int splits, int D, void* out,
                 int out_dtype, int64_t out_row_stride, const DecodeParams* rowmap, float* ex_m, float* ex_l,
                 float* ex_acc, cudaStream_t s) {
  return launch_merge_strided(m, l, acc, splits, 1, static_cast<int64_t>(splits) * D, D, rows, splits, D, out,
                              out_dtype, out_row_stride, rowmap, ex_m, ex_l, ex_acc, s);
}

int launch_merge_strided(const float* m, const float* l, const float* acc, int64_t ms_r, int64_t ms_s, int64_t as_r,
                         int64_t as_s, int64_t rows, int splits, int D, void* out, int out_dtype,
                         int64_t out_row_stride, const DecodeParams* rowmap, float* ex_m, float* ex_l, float* ex_acc,
                         cudaStream_t s) {
  if (rows == 0) return IAK_OK;
  if (splits > 12288) return fail(IAK_ERR_UNSUPPORTED, "too many splits to merge (%d)", splits);
  const int64_t blocks = std::min<int64_t>(rows, 65535LL * 8);
  const bool vec = D % 4 == 0 && D <= 1024 && as_r % 4 == 0 && as_s % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(acc) % 16 == 0;
  if (vec) {
    const size_t vsmem = (static_cast<size_t>((splits + 3) & ~3) + static_cast<size_t>(kMergeWarps) * D) * sizeof(float);
    const int Hq = rowmap ? rowmap->Hq : 0;
    const int64_t o_sb = rowmap ? rowmap->o_sb : 0, o_sh = rowmap ? rowmap->o_sh : 0;
    auto go = [&](auto kern) -> int {
      if (vsmem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(vsmem));
        if (e != cudaSuccess) return check_cuda(e, "merge smem attribute");
      }
      kern<<<static_cast<unsigned>(blocks), kMergeWarps * 32, vsmem, s>>>(m, l, acc, ms_r, ms_s, as_r, as_s, rows,
                                                                          splits, D, out, out_dtype, out_row_stride,
                                                                          Hq, o_sb, o_sh, ex_m, ex_l, ex_acc);
      return check_cuda(cudaGetLastError(), "merge launch");
    };
    if (D <= 128) return go(merge_vec_kernel<1>);
    if (D <= 256) return go(merge_vec_kernel<2>);
    if (D <= 512) return go(merge_vec_kernel<4>);
    return go(merge_vec_kernel<8>);
  }
  const int threads = D >= 128 ? 128 : (D >= 64 ? 64 : 32);
  const size_t smem = static_cast<size_t>(splits) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return check_cuda(e, "merge smem attribute");
  }
  merge_kernel<<<static_cast<unsigned>(blocks), threads, smem, s>>>(
      m, l, acc, ms_r, ms_s, as_r, as_s, rows, splits, D, out, out_dtype, out_row_stride, rowmap ? rowmap->Hq : 0,
      rowmap ? rowmap->o_sb : 0,
      rowmap ? rowmap->o_sh : 0, ex_m, ex_l, ex_acc);
  return check_cuda(cudaGetLastError(), "merge launch");
}

}  // namespace iak
