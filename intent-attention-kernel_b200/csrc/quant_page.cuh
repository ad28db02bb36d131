// One page of quantise-on-write, shared by iak_quantize_pages (dense source
// pages), iak_append_tokens (open pages rebuilt from their staged rows) and
// iak_convert_pages (format transitions of pool pages).
//
// Arithmetic restates intent_quant.py:221-312 (absmax/127 scale clamped at
// 1e-8, clamp-then-round-half-even codes, e4m3 of x/scale, INT4 with the same
// /127 scale, two-stage INT4_RESIDUAL) over a per-page scale span.  Every
// step uses explicitly rounded IEEE operations (__fdiv_rn, __fmul_rn,
// __fsub_rn) so that the compiler cannot contract or approximate them and the
// codes are bit-identical to the reference's torch float32 arithmetic.
#pragma once

#include <cfloat>

#include "iak_internal.cuh"

namespace iak {
namespace qpage {

constexpr int kThreads = 256;   // every kernel that calls quantize_page runs 256 threads
constexpr int kMaxD = 1024;     // dense K/V heads and MLA latent rows (576)

// Destination pools of one plane (K or V).
struct PlanePools {
  __half* f16; uint8_t* fp8; int8_t* i8; uint8_t* i4; uint8_t* i4r;
  float* scale; float* res_scale;
  int64_t num_pages; int PS, D, mode, ns;
};

// Per-CTA scratch of quantize_page (static shared memory of the caller).
struct Scratch {
  float sc[kMaxD], rsc[kMaxD], chmax[kMaxD], red[kThreads / 32];
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
__device__ void span_absmax(const PlanePools& q, F f, float* out, float* chmax, float* red) {
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

// Whether page format fmt can be written to q (its pool and scales are
// present and the head dim suits it).  SKIP and SPARSE hold no pool data.
__device__ __forceinline__ bool writable(const PlanePools& q, int fmt) {
  const bool ok = (fmt == IAK_FMT_F16 && q.f16) || (fmt == IAK_FMT_FP8 && q.fp8 && q.scale) ||
                  (fmt == IAK_FMT_INT8 && q.i8 && q.scale) || (fmt == IAK_FMT_INT4 && q.i4 && q.scale) ||
                  (fmt == IAK_FMT_INT4R && q.i4 && q.i4r && q.scale && q.res_scale);
  const bool int4 = fmt == IAK_FMT_INT4 || fmt == IAK_FMT_INT4R;
  return ok && !(int4 && (q.D % 32));
}

// Quantise the page X(t, d) (t < PS, d < D) into pool page dst in format fmt.
// given / given_res: this page's n_scales scales to use instead of the
// computed ones (or NULL).  Called by all kThreads threads of the CTA, which
// must not diverge around it; fmt must pass writable().
template <class F>
__device__ void quantize_page(const PlanePools& q, F X, int fmt, int64_t dst, const float* given,
                              const float* given_res, Scratch& s) {
  const int PS = q.PS, D = q.D, ns = q.ns;
  if (fmt == IAK_FMT_F16) {
    for (int e = threadIdx.x; e < PS * D; e += kThreads)
      q.f16[dst * PS * D + e] = __float2half_rn(X(e / D, e % D));
    return;
  }
  float* sc = s.sc;
  float* rsc = s.rsc;
  // ---- scale of the base codes
  if (given) {
    for (int j = threadIdx.x; j < ns; j += kThreads) sc[j] = given[j];
    __syncthreads();
  } else {
    span_absmax(q, X, sc, s.chmax, s.red);
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
    const float sv = sc[scale_slot(mode, d)];
    const float x = X(t, d);
    return __fsub_rn(x, __fmul_rn(static_cast<float>(int_code(x, sv, 7.f)), sv));
  };
  if (given_res) {
    for (int j = threadIdx.x; j < ns; j += kThreads) rsc[j] = given_res[j];
    __syncthreads();
  } else {
    span_absmax(q, residual, rsc, s.chmax, s.red);
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

// Dequantised value of channel d of row t of pool page pid in format fmt,
// as every decode kernel reads it: code x scale (+ residual code x residual
// scale) in float32; SKIP / SPARSE / absent pools read as 0.
__device__ __forceinline__ float dequant(const PlanePools& q, int fmt, int64_t pid, int t, int d) {
  const int PS = q.PS, D = q.D;
  const int64_t e = (pid * PS + t) * D + d;
  if (!writable(q, fmt)) return 0.f;
  if (fmt == IAK_FMT_F16) return __half2float(q.f16[e]);
  const float s = q.scale[pid * q.ns + scale_slot(q.mode, d)];
  if (fmt == IAK_FMT_FP8) return __fmul_rn(e4m3_to_float(q.fp8[e]), s);
  if (fmt == IAK_FMT_INT8) return __fmul_rn(static_cast<float>(q.i8[e]), s);
  const uint8_t* row = q.i4 + (pid * PS + t) * (D / 2);
  const float base = __fmul_rn(static_cast<float>(int4_code(row, d)), s);
  if (fmt == IAK_FMT_INT4) return base;
  const uint8_t* rrow = q.i4r + (pid * PS + t) * (D / 2);
  const float rs = q.res_scale[pid * q.ns + scale_slot(q.mode, d)];
  return __fadd_rn(base, __fmul_rn(static_cast<float>(int4_code(rrow, d)), rs));
}

}  // namespace qpage
}  // namespace iak
