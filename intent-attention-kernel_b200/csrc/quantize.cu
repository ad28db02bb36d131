// Quantise-on-write: dense K or V pages -> the page-pool formats.
//
// Arithmetic restates intent_quant.py:221-312 (absmax/127 scale clamped at
// 1e-8, clamp-then-round-half-even codes, e4m3 of x/scale, INT4 with the same
// /127 scale, two-stage INT4_RESIDUAL) over a per-page scale span.  Every
// step uses explicitly rounded IEEE operations (__fdiv_rn, __fmul_rn,
// __fsub_rn) so that the compiler cannot contract or approximate them and the
// codes are bit-identical to the reference's torch float32 arithmetic.
#include <cfloat>

#include "iak_internal.cuh"

namespace iak {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxD = 1024;  // dense K/V heads and MLA latent rows (576)

struct QuantParams {
  const void* x; int x_dtype; int64_t P;
  const int32_t* dst_ids; const uint8_t* formats;
  const float* given; const float* given_res;
  __half* f16; uint8_t* fp8; int8_t* i8; uint8_t* i4; uint8_t* i4r;
  float* scale; float* res_scale;
  int64_t num_pages; int PS, D, mode, ns;
};

__device__ __constant__ int kNibOff[8] = {0, 2, 16, 18, 1, 3, 17, 19};

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = -FLT_MAX;
  for (int w = 0; w < kThreads / 32; ++w) r = fmaxf(r, red[w]);
  return r;
}

__device__ __forceinline__ int scale_slot(int mode, int d) {
  return mode == IAK_SCALE_PAGE ? 0 : (mode == IAK_SCALE_GROUP32 ? (d >> 5) : d);
}

__device__ __forceinline__ float to_scale(float absmax) {
  return fmaxf(__fdiv_rn(absmax, 127.0f), 1e-8f);
}

__device__ __forceinline__ int int_code(float x, float s, float qmax) {
  float y = __fdiv_rn(x, s);
  y = fminf(fmaxf(y, -qmax), qmax);
  return static_cast<int>(rintf(y));
}

// absmax over the scale span of f(t, d) into out[ns]
template <class F>
__device__ void span_absmax(const QuantParams& q, F f, float* out, float* chmax, float* red) {
  const int PS = q.PS, D = q.D;
  if (q.mode == IAK_SCALE_PAGE) {
    float v = 0.f;
    for (int e = threadIdx.x; e < PS * D; e += kThreads) v = fmaxf(v, fabsf(f(e / D, e % D)));
    v = block_max(v, red);
    if (threadIdx.x == 0) out[0] = v;
  } else {
    for (int d = threadIdx.x; d < D; d += kThreads) {
      float v = 0.f;
      for (int t = 0; t < PS; ++t) v = fmaxf(v, fabsf(f(t, d)));
      chmax[d] = v;
    }
    __syncthreads();
    if (q.mode == IAK_SCALE_CHANNEL) {
      for (int d = threadIdx.x; d < D; d += kThreads) out[d] = chmax[d];
    } else {
      for (int gi = threadIdx.x; gi < D / 32; gi += kThreads) {
        float v = 0.f;
        for (int k = 0; k < 32; ++k) v = fmaxf(v, chmax[gi * 32 + k]);
        out[gi] = v;
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads) quantize_kernel(const QuantParams q) {
  __shared__ float sc[kMaxD], rsc[kMaxD], chmax[kMaxD], red[kThreads / 32];
  const int64_t i = blockIdx.x;
  const int fmt = q.formats[i];
  if (fmt == IAK_FMT_SKIP || fmt == IAK_FMT_SPARSE) return;
  const int64_t dst = q.dst_ids ? static_cast<int64_t>(q.dst_ids[i]) : i;
  if (dst < 0 || dst >= q.num_pages) return;
  // formats live in device memory, so a page whose pool (or scale array) was
  // not supplied is skipped rather than written through a null pointer
  const bool ok = (fmt == IAK_FMT_F16 && q.f16) || (fmt == IAK_FMT_FP8 && q.fp8 && q.scale) ||
                  (fmt == IAK_FMT_INT8 && q.i8 && q.scale) || (fmt == IAK_FMT_INT4 && q.i4 && q.scale) ||
                  (fmt == IAK_FMT_INT4R && q.i4 && q.i4r && q.scale && q.res_scale);
  const bool int4 = fmt == IAK_FMT_INT4 || fmt == IAK_FMT_INT4R;
  if (!ok || (int4 && (q.D % 32))) return;
  const int PS = q.PS, D = q.D, ns = q.ns;
  const int64_t src = i * PS * D;
  auto X = [&](int t, int d) { return load_as_float(q.x, q.x_dtype, src + static_cast<int64_t>(t) * D + d); };

  if (fmt == IAK_FMT_F16) {
    for (int e = threadIdx.x; e < PS * D; e += kThreads)
      q.f16[dst * PS * D + e] = __float2half_rn(X(e / D, e % D));
    return;
  }
  // ---- scale of the base codes
  if (q.given) {
    for (int j = threadIdx.x; j < ns; j += kThreads) sc[j] = q.given[i * ns + j];
    __syncthreads();
  } else {
    span_absmax(q, X, sc, chmax, red);
    for (int j = threadIdx.x; j < ns; j += kThreads) sc[j] = to_scale(sc[j]);
    __syncthreads();
  }
  for (int j = threadIdx.x; j < ns; j += kThreads) q.scale[dst * ns + j] = sc[j];

  const int mode = q.mode;
  if (fmt == IAK_FMT_INT8) {
    for (int e = threadIdx.x; e < PS * D; e += kThreads) {
      const int d = e % D;
      q.i8[dst * PS * D + e] = static_cast<int8_t>(int_code(X(e / D, d), sc[scale_slot(mode, d)], 127.f));
    }
    return;
  }
  if (fmt == IAK_FMT_FP8) {
    for (int e = threadIdx.x; e < PS * D; e += kThreads) {
      const int d = e % D;
      const float y = __fdiv_rn(X(e / D, d), sc[scale_slot(mode, d)]);
      q.fp8[dst * PS * D + e] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3));
    }
    return;
  }
  // ---- INT4 / INT4_RESIDUAL (packed, 8 codes per 32-bit word)
  const int words = D / 8;
  auto base_code = [&](int t, int d) { return int_code(X(t, d), sc[scale_slot(mode, d)], 7.f); };
  for (int e = threadIdx.x; e < PS * words; e += kThreads) {
    const int t = e / words, w = e % words;
    const int d0 = 32 * (w >> 2) + 4 * (w & 3);
    uint32_t word = 0;
#pragma unroll
    for (int n = 0; n < 8; ++n) word |= static_cast<uint32_t>(base_code(t, d0 + kNibOff[n]) + 8) << (4 * n);
    reinterpret_cast<uint32_t*>(q.i4 + (dst * PS + t) * (D / 2))[w] = word;
  }
  if (fmt != IAK_FMT_INT4R) return;
  auto residual = [&](int t, int d) {
    const float s = sc[scale_slot(mode, d)];
    const float x = X(t, d);
    return __fsub_rn(x, __fmul_rn(static_cast<float>(int_code(x, s, 7.f)), s));
  };
  if (q.given_res) {
    for (int j = threadIdx.x; j < ns; j += kThreads) rsc[j] = q.given_res[i * ns + j];
    __syncthreads();
  } else {
    span_absmax(q, residual, rsc, chmax, red);
    for (int j = threadIdx.x; j < ns; j += kThreads) rsc[j] = to_scale(rsc[j]);
    __syncthreads();
  }
  for (int j = threadIdx.x; j < ns; j += kThreads) q.res_scale[dst * ns + j] = rsc[j];
  for (int e = threadIdx.x; e < PS * words; e += kThreads) {
    const int t = e / words, w = e % words;
    const int d0 = 32 * (w >> 2) + 4 * (w & 3);
    uint32_t word = 0;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int d = d0 + kNibOff[n];
      const int c = int_code(residual(t, d), rsc[scale_slot(mode, d)], 7.f);
      word |= static_cast<uint32_t>(c + 8) << (4 * n);
    }
    reinterpret_cast<uint32_t*>(q.i4r + (dst * PS + t) * (D / 2))[w] = word;
  }
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
  q.f16 = static_cast<__half*>(a->f16); q.fp8 = static_cast<uint8_t*>(a->fp8); q.i8 = static_cast<int8_t*>(a->i8);
  q.i4 = static_cast<uint8_t*>(a->i4); q.i4r = static_cast<uint8_t*>(a->i4r);
  q.scale = a->scale; q.res_scale = a->res_scale;
  q.num_pages = a->num_pages; q.PS = PS; q.D = D; q.mode = a->scale_mode; q.ns = n_scales_of(a->scale_mode, D);
  quantize_kernel<<<static_cast<unsigned>(a->num_src_pages), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(q);
  return check_cuda(cudaGetLastError(), "quantize launch");
}
