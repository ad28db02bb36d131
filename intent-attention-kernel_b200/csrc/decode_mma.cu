// Tensor-core split-KV paged decode for sm_100a.
//
// One CTA = one (sequence, page-table head) unit x one contiguous range of its
// page table (a KV split).  Warp 4 is the producer: one lane gathers every
// selected page with TMA tensor copies (128-byte swizzle, no multicast) into a
// ring of shared-memory stages guarded by mbarriers.  Warps 0-3 consume the
// stages round-robin; each warp owns one 16-token page at a time and runs
//
//   S^T[16 tok x 8 q] = K[16 x D] . Q^T        (mma.sync m16n8k16, fp16 -> fp32)
//   online softmax over tokens (exp2 domain, running max per query head)
//   O^T[D x 8 q]     += V^T[D x 16] . P^T       (mma.sync m16n8k16)
//
// with the page's codes dequantised in registers: int8 / int4 codes become
// exact fp16 integers by exponent-bias tricks, e4m3 codes by cvt.f16x2.e4m3x2,
// and the per-page (or per-32-channel) scale is applied in fp32 to S and folded
// into P for V.  The query group of a GQA head is the MMA's N dimension, so G
// <= 8 query heads share every K/V byte.  The four warps' (m, l, O) are merged
// in shared memory; with several splits the partials go to the workspace and
// the LSE merge kernel combines them.
//
// Register-fragment index maps (m16n8k16, lane = 4*r + c):
//   QK, 8-bit / 4-bit pages: k-step kk, thread c holds channels 16kk+4c..+3
//   QK, fp16 pages:          the ldmatrix layout (channels 16kk+2c, +1, +8, +9)
//   PV (all formats):        output row m of m-tile mt is channel
//                            d = 32*(w/4) + 4*(w%4) + {0,2,16,18,1,3,17,19}[n]
//                            with (w, n) = (m, mt) for D = 128 and
//                            (m % 8, mt + 4*(m/8)) for D = 64, i.e. the packed
//                            INT4 nibble order, so every format's V loads are
//                            whole 32-bit words.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "iak_internal.cuh"

namespace iak {

__device__ unsigned int g_decode_timeouts = 0;

namespace {

constexpr int kPS = 16;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kChunkMax = 512;
constexpr int kStages = 8;
constexpr int kStageBytes = 9216;   // K region 4 KB | V region 4 KB | scale rows 1 KB
constexpr int kVOff = 4096;
constexpr int kResOff = 1024;       // INT4 residual plane inside a K or V region
constexpr int kScaleOff = 8192;
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at boost clock, then give up

enum MapIdx { M_KF16 = 0, M_VF16, M_KFP8, M_VFP8, M_KI8, M_VI8, M_KI4, M_VI4, M_KI4R, M_VI4R, M_COUNT };
struct TmaMaps {
  CUtensorMap m[M_COUNT];
};

struct SmemLayout {
  static constexpr int stages = 0;
  static constexpr int bars = kStages * kStageBytes;                 // full[kStages], empty[kStages]
  static constexpr int pid = bars + 2 * kStages * 8;
  static constexpr int scal = pid + kChunkMax * 4;                   // ks, vs, krs, vrs
  static constexpr int fmt = scal + 4 * kChunkMax * 4;
  static constexpr int misc = fmt + kChunkMax;
  static constexpr int total = misc + 64;
};

// ----------------------------------------------------------------- PTX ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when the phase did not complete within kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > kWaitCycles) return false;
  return true;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
  return r;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t v16) {
  uint32_t r;
  const uint16_t h = static_cast<uint16_t>(v16);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(h));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t sw128(uint32_t lin) { return lin ^ (((lin >> 7) & 7u) << 4); }
__device__ __forceinline__ uint32_t lds32(const char* base, uint32_t off) {
  return *reinterpret_cast<const uint32_t*>(base + off);
}
__device__ __forceinline__ uint2 lds64(const char* base, uint32_t off) {
  return *reinterpret_cast<const uint2*>(base + off);
}

// exact int / fp8 -> fp16 pair conversions
constexpr uint32_t kH1152 = 0x64806480u;  // half2(1152, 1152): 1024 + 128 bias of offset-binary bytes
constexpr uint32_t kH1032 = 0x64086408u;  // half2(1032, 1032): 1024 + 8 bias of offset-binary nibbles
constexpr uint32_t kH16th = 0x2C002C00u;  // half2(1/16, 1/16)
constexpr uint32_t kHm72 = 0xD480D480u;   // half2(-72, -72)

// byte-pair register t = [x0, y0, x1, y1] of offset-binary int8 -> half2(x0, y0) / half2(x1, y1)
__device__ __forceinline__ uint32_t i8pair_lo(uint32_t t) { return hsub2(__byte_perm(t, 0x64646464u, 0x4140), kH1152); }
__device__ __forceinline__ uint32_t i8pair_hi(uint32_t t) { return hsub2(__byte_perm(t, 0x64646464u, 0x4342), kH1152); }
// register t = [a, ., b, .] of offset-binary nibble pairs -> low / high nibbles as half2
__device__ __forceinline__ uint32_t i4pair_lo(uint32_t t) { return hsub2(lop_and_or(t, 0x000F000Fu, 0x64006400u), kH1032); }
__device__ __forceinline__ uint32_t i4pair_hi(uint32_t t) {
  return hfma2(lop_and_or(t, 0x00F000F0u, 0x64006400u), kH16th, kHm72);
}

// ------------------------------------------------------------ layouts ---
// PV word of output row-set ws (0: rows r, 1: rows r+8) for lane row r
template <int D>
__device__ __forceinline__ int pv_word(int r, int ws) { return D == 128 ? r + 8 * ws : r; }
__device__ __forceinline__ int word_d0(int w) { return 32 * (w >> 2) + 4 * (w & 3); }
__device__ __constant__ int kNibOff[8] = {0, 2, 16, 18, 1, 3, 17, 19};

// Channel of PV output (m-tile mt, row m).
template <int D>
__device__ __forceinline__ int pv_channel(int mt, int m) {
  if constexpr (D == 128) return word_d0(m) + kNibOff[mt];
  return word_d0(m & 7) + kNibOff[mt + 4 * (m >> 3)];
}

// A fragment of PV m-tile mt from the per-lane half2 table vh[tp][ws][nibble]
template <int D>
__device__ __forceinline__ void pv_afrag(const uint32_t (&vh)[2][D / 64][8], int mt, uint32_t& a0, uint32_t& a1,
                                         uint32_t& a2, uint32_t& a3) {
  if constexpr (D == 128) {
    a0 = vh[0][0][mt]; a1 = vh[0][D / 64 - 1][mt]; a2 = vh[1][0][mt]; a3 = vh[1][D / 64 - 1][mt];
  } else {
    a0 = vh[0][0][mt]; a1 = vh[0][0][mt + 4]; a2 = vh[1][0][mt]; a3 = vh[1][0][mt + 4];
  }
}

// ------------------------------------------------ per-format V tables ---
// Fill vh[tp][ws][n] = half2(V[t0][d], V[t1][d]) for the lane's token pairs
// tp 0 = (2c, 2c+1), tp 1 = (2c+8, 2c+9) and PV words.
template <int D>
__device__ __forceinline__ void v_table_8bit(const char* tile, int r, int c, bool fp8, uint32_t (&vh)[2][D / 64][8]) {
#pragma unroll
  for (int tp = 0; tp < 2; ++tp) {
    const int t0 = 2 * c + 8 * tp, t1 = t0 + 1;
#pragma unroll
    for (int ws = 0; ws < D / 64; ++ws) {
      const int d0 = word_d0(pv_word<D>(r, ws));
      const uint32_t a0 = lds32(tile, sw128(t0 * D + d0)), a1 = lds32(tile, sw128(t1 * D + d0));
      const uint32_t b0 = lds32(tile, sw128(t0 * D + d0 + 16)), b1 = lds32(tile, sw128(t1 * D + d0 + 16));
      uint32_t tA01 = __byte_perm(a0, a1, 0x5140), tA23 = __byte_perm(a0, a1, 0x7362);
      uint32_t tB01 = __byte_perm(b0, b1, 0x5140), tB23 = __byte_perm(b0, b1, 0x7362);
      if (fp8) {
        vh[tp][ws][0] = e4m3x2_f16x2(tA01); vh[tp][ws][4] = e4m3x2_f16x2(tA01 >> 16);
        vh[tp][ws][1] = e4m3x2_f16x2(tA23); vh[tp][ws][5] = e4m3x2_f16x2(tA23 >> 16);
        vh[tp][ws][2] = e4m3x2_f16x2(tB01); vh[tp][ws][6] = e4m3x2_f16x2(tB01 >> 16);
        vh[tp][ws][3] = e4m3x2_f16x2(tB23); vh[tp][ws][7] = e4m3x2_f16x2(tB23 >> 16);
      } else {
        tA01 ^= 0x80808080u; tA23 ^= 0x80808080u; tB01 ^= 0x80808080u; tB23 ^= 0x80808080u;
        vh[tp][ws][0] = i8pair_lo(tA01); vh[tp][ws][4] = i8pair_hi(tA01);
        vh[tp][ws][1] = i8pair_lo(tA23); vh[tp][ws][5] = i8pair_hi(tA23);
        vh[tp][ws][2] = i8pair_lo(tB01); vh[tp][ws][6] = i8pair_hi(tB01);
        vh[tp][ws][3] = i8pair_lo(tB23); vh[tp][ws][7] = i8pair_hi(tB23);
      }
    }
  }
}

template <int D>
__device__ __forceinline__ void v_table_int4(const char* tile, int r, int c, uint32_t (&vh)[2][D / 64][8]) {
  constexpr int RB = D / 2;
#pragma unroll
  for (int tp = 0; tp < 2; ++tp) {
    const int t0 = 2 * c + 8 * tp, t1 = t0 + 1;
#pragma unroll
    for (int ws = 0; ws < D / 64; ++ws) {
      const int w = pv_word<D>(r, ws);
      const uint32_t x0 = lds32(tile, sw128(t0 * RB + 4 * w)), x1 = lds32(tile, sw128(t1 * RB + 4 * w));
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t t = __byte_perm(x0, x1, b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12));
        vh[tp][ws][2 * b] = i4pair_lo(t);
        vh[tp][ws][2 * b + 1] = i4pair_hi(t);
      }
    }
  }
}

template <int D>
__device__ __forceinline__ void v_table_f16(const char* tile, int r, int c, uint32_t (&vh)[2][D / 64][8]) {
#pragma unroll
  for (int tp = 0; tp < 2; ++tp) {
    const int t0 = 2 * c + 8 * tp, t1 = t0 + 1;
#pragma unroll
    for (int ws = 0; ws < D / 64; ++ws) {
      const int d0 = word_d0(pv_word<D>(r, ws));
#pragma unroll
      for (int part = 0; part < 2; ++part) {     // channels d0+{0..3}, d0+16+{0..3}
        const int d = d0 + 16 * part;
        const uint32_t o0 = sw128((d >> 6) * 2048 + t0 * 128 + ((2 * d) & 127));
        const uint32_t o1 = sw128((d >> 6) * 2048 + t1 * 128 + ((2 * d) & 127));
        const uint2 x0 = lds64(tile, o0), x1 = lds64(tile, o1);
        // nibble order: part 0 -> (0, 4, 1, 5), part 1 -> (2, 6, 3, 7)
        vh[tp][ws][0 + 2 * part] = __byte_perm(x0.x, x1.x, 0x5410);
        vh[tp][ws][4 + 2 * part] = __byte_perm(x0.x, x1.x, 0x7632);
        vh[tp][ws][1 + 2 * part] = __byte_perm(x0.y, x1.y, 0x5410);
        vh[tp][ws][5 + 2 * part] = __byte_perm(x0.y, x1.y, 0x7632);
      }
    }
  }
}

// ------------------------------------------------ per-format QK A frags ---
template <int D>
__device__ __forceinline__ void k_frag_8bit(const char* tile, int r, int c, int kk, bool fp8, uint32_t (&a)[4]) {
  const uint32_t x0 = lds32(tile, sw128(r * D + 16 * kk + 4 * c));
  const uint32_t x1 = lds32(tile, sw128((r + 8) * D + 16 * kk + 4 * c));
  if (fp8) {
    a[0] = e4m3x2_f16x2(x0); a[2] = e4m3x2_f16x2(x0 >> 16);
    a[1] = e4m3x2_f16x2(x1); a[3] = e4m3x2_f16x2(x1 >> 16);
  } else {
    const uint32_t y0 = x0 ^ 0x80808080u, y1 = x1 ^ 0x80808080u;
    a[0] = i8pair_lo(y0); a[2] = i8pair_hi(y0);
    a[1] = i8pair_lo(y1); a[3] = i8pair_hi(y1);
  }
}

// two k-steps (2p, 2p+1) of an INT4 plane
template <int D>
__device__ __forceinline__ void k_frag_int4(const char* tile, int r, int c, int p, uint32_t (&a)[2][4]) {
  constexpr int RB = D / 2;
  const uint32_t x0 = lds32(tile, sw128(r * RB + 16 * p + 4 * c));
  const uint32_t x1 = lds32(tile, sw128((r + 8) * RB + 16 * p + 4 * c));
  a[0][0] = i4pair_lo(x0); a[0][2] = i4pair_hi(x0);
  a[0][1] = i4pair_lo(x1); a[0][3] = i4pair_hi(x1);
  a[1][0] = i4pair_lo(x0 >> 8); a[1][2] = i4pair_hi(x0 >> 8);
  a[1][1] = i4pair_lo(x1 >> 8); a[1][3] = i4pair_hi(x1 >> 8);
}

template <int D>
__device__ __forceinline__ void k_frag_f16(uint32_t tile_u32, int lane, int kk, uint32_t (&a)[4]) {
  const int mi = lane >> 3, rr = lane & 7;
  const int tok = rr + 8 * (mi & 1);
  const int d = 16 * kk + 8 * (mi >> 1);
  const uint32_t off = sw128((d >> 6) * 2048 + tok * 128 + ((2 * d) & 127));
  ldsm_x4(tile_u32 + off, a[0], a[1], a[2], a[3]);
}

// ------------------------------------------------------------- kernel ---
template <int D, bool GROUP>
__global__ void __launch_bounds__(kThreads, 2)
    decode_mma_kernel(const DecodeParams p, const __grid_constant__ TmaMaps maps) {
  constexpr int KT = D / 16;   // k-steps of QK, m-tiles of PV
  constexpr int NG = GROUP ? D / 32 : 1;
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::bars);
  int32_t* pid_s = reinterpret_cast<int32_t*>(smem + SmemLayout::pid);
  float* scal_s = reinterpret_cast<float*>(smem + SmemLayout::scal);
  uint8_t* fmt_s = reinterpret_cast<uint8_t*>(smem + SmemLayout::fmt);
  int* misc = reinterpret_cast<int*>(smem + SmemLayout::misc);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int unit = blockIdx.y, split = blockIdx.x;
  const int b = unit / p.Ht, hk = unit % p.Ht;
  int count = p.W;
  if (p.pc) {
    const int cc = p.pc[b * p.pc_sb + hk];
    count = cc < 0 ? 0 : (cc > p.W ? p.W : cc);
  }
  const int lo = split * p.pages_per_split;
  const int hi = min(lo + p.pages_per_split, count);

  if (tid == 0) {
    for (int s = 0; s < 2 * kStages; ++s) mbar_init(smem_u32(&bars[s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    misc[0] = 0;
  }
  __syncthreads();

  // ---- compact the split's valid pages (order preserving) + page-scale scalars
  const int32_t* table = p.pt + b * p.pt_sb + hk * p.pt_sh;
  for (int base = lo; base < hi; base += kThreads) {
    const int j = base + tid;
    int pid = -1, fmt = IAK_FMT_SKIP;
    if (j < hi) {
      pid = table[j];
      if (pid >= 0 && pid < p.num_pages) fmt = page_format(p, pid);
    }
    const bool valid = fmt != IAK_FMT_SKIP && fmt != IAK_FMT_SPARSE;
    const unsigned bal = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) misc[8 + warp] = __popc(bal);
    __syncthreads();
    int off = misc[0];
    for (int w = 0; w < warp; ++w) off += misc[8 + w];
    if (valid) {
      const int idx = off + __popc(bal & ((1u << lane) - 1u));
      pid_s[idx] = pid;
      fmt_s[idx] = static_cast<uint8_t>(fmt);
      if (!GROUP) {
        const bool q = fmt != IAK_FMT_F16;
        scal_s[idx] = q ? p.k_scale[pid] : 1.f;
        scal_s[kChunkMax + idx] = q ? p.v_scale[pid] : 1.f;
        scal_s[2 * kChunkMax + idx] = fmt == IAK_FMT_INT4R ? p.k_rscale[pid] : 0.f;
        scal_s[3 * kChunkMax + idx] = fmt == IAK_FMT_INT4R ? p.v_rscale[pid] : 0.f;
      }
    }
    __syncthreads();
    if (tid == 0) {
      int tot = misc[0];
      for (int w = 0; w < kConsumerWarps + 1; ++w) tot += misc[8 + w];
      misc[0] = tot;
    }
    __syncthreads();
  }
  const int n_valid = misc[0];

  bool timed_out = false;
  const float qk_log2 = p.sm_scale * 1.4426950408889634f;
  // per-lane running state: query columns g = 2c, 2c+1
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float oacc[KT][4];
#pragma unroll
  for (int mt = 0; mt < KT; ++mt) oacc[mt][0] = oacc[mt][1] = oacc[mt][2] = oacc[mt][3] = 0.f;
  const int r = lane >> 2, c = lane & 3;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int i = 0; i < n_valid; ++i) {
        const int s = i & (kStages - 1), round = i / kStages;
        const uint32_t full = smem_u32(&bars[s]), empty = smem_u32(&bars[kStages + s]);
        if (round > 0 && !mbar_wait(empty, (round - 1) & 1)) {
          timed_out = true;
          break;
        }
        const int fmt = fmt_s[i];
        const int pid = pid_s[i];
        const uint32_t st = smem_u32(smem + s * kStageBytes);
        uint32_t bytes;
        if (fmt == IAK_FMT_F16) bytes = 2 * kPS * D * 2;
        else if (fmt == IAK_FMT_INT4) bytes = 2 * kPS * D / 2;
        else bytes = 2 * kPS * D;   // FP8, INT8, INT4R (two half-size planes)
        const bool gs = GROUP && fmt != IAK_FMT_F16;
        if (gs) bytes += (fmt == IAK_FMT_INT4R ? 4 : 2) * NG * 4;
        mbar_arrive_expect_tx(full, bytes);
        const int y16 = pid * kPS;  // first token row of the page
        if (fmt == IAK_FMT_F16) {
          tma_load_2d(st, &maps.m[M_KF16], 0, y16, full);
          tma_load_2d(st + kVOff, &maps.m[M_VF16], 0, y16, full);
          if constexpr (D == 128) {
            tma_load_2d(st + 2048, &maps.m[M_KF16], 64, y16, full);
            tma_load_2d(st + kVOff + 2048, &maps.m[M_VF16], 64, y16, full);
          }
        } else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) {
          const int y = pid * (kPS * D / 128);   // 128-byte lines of 8-bit token rows
          const int mk = fmt == IAK_FMT_FP8 ? M_KFP8 : M_KI8;
          tma_load_2d(st, &maps.m[mk], 0, y, full);
          tma_load_2d(st + kVOff, &maps.m[mk + 1], 0, y, full);
        } else {
          const int y = pid * (kPS * D / 256);   // 128-byte lines of packed int4 token rows
          tma_load_2d(st, &maps.m[M_KI4], 0, y, full);
          tma_load_2d(st + kVOff, &maps.m[M_VI4], 0, y, full);
          if (fmt == IAK_FMT_INT4R) {
            tma_load_2d(st + kResOff, &maps.m[M_KI4R], 0, y, full);
            tma_load_2d(st + kVOff + kResOff, &maps.m[M_VI4R], 0, y, full);
          }
        }
        if (gs) {
          bulk_load(st + kScaleOff, p.k_scale + static_cast<int64_t>(pid) * NG, NG * 4, full);
          bulk_load(st + kScaleOff + 16 * 4, p.v_scale + static_cast<int64_t>(pid) * NG, NG * 4, full);
          if (fmt == IAK_FMT_INT4R) {
            bulk_load(st + kScaleOff + 32 * 4, p.k_rscale + static_cast<int64_t>(pid) * NG, NG * 4, full);
            bulk_load(st + kScaleOff + 48 * 4, p.v_rscale + static_cast<int64_t>(pid) * NG, NG * 4, full);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    // Q^T B fragments (row n = r is query head g = r), both channel orders
    uint32_t qstd[KT][2], qperm[KT][2];
    {
      const bool live = r < p.G;
      const int64_t qoff = static_cast<int64_t>(b) * p.q_sb + static_cast<int64_t>(hk * p.G + (live ? r : 0)) * p.q_sh;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        float v[8];
        const int ds[8] = {16 * kk + 2 * c, 16 * kk + 2 * c + 1, 16 * kk + 2 * c + 8, 16 * kk + 2 * c + 9,
                           16 * kk + 4 * c, 16 * kk + 4 * c + 1, 16 * kk + 4 * c + 2, 16 * kk + 4 * c + 3};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = live ? load_as_float(p.q, p.q_dtype, qoff + ds[e]) : 0.f;
        qstd[kk][0] = pack_f16x2(v[0], v[1]); qstd[kk][1] = pack_f16x2(v[2], v[3]);
        qperm[kk][0] = pack_f16x2(v[4], v[5]); qperm[kk][1] = pack_f16x2(v[6], v[7]);
      }
    }
    for (int i = warp; i < n_valid; i += kConsumerWarps) {
      const int s = i & (kStages - 1), round = i / kStages;
      if (!mbar_wait(smem_u32(&bars[s]), round & 1)) {
        timed_out = true;
        break;
      }
      const char* st = smem + s * kStageBytes;
      const uint32_t st_u32 = smem_u32(st);
      const int fmt = fmt_s[i];
      const float* gsc = reinterpret_cast<const float*>(st + kScaleOff);
      // ---------------- S^T = K Q^T
      float sacc[NG][4], racc[NG][4];
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[g][e] = racc[g][e] = 0.f;
      if (fmt == IAK_FMT_F16) {
#pragma unroll
        for (int kk = 0; kk < KT; ++kk) {
          uint32_t a[4];
          k_frag_f16<D>(st_u32, lane, kk, a);
          mma16816(sacc[GROUP ? kk / 2 : 0], a[0], a[1], a[2], a[3], qstd[kk][0], qstd[kk][1]);
        }
      } else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) {
        const bool fp8 = fmt == IAK_FMT_FP8;
#pragma unroll
        for (int kk = 0; kk < KT; ++kk) {
          uint32_t a[4];
          k_frag_8bit<D>(st, r, c, kk, fp8, a);
          mma16816(sacc[GROUP ? kk / 2 : 0], a[0], a[1], a[2], a[3], qperm[kk][0], qperm[kk][1]);
        }
      } else {
#pragma unroll
        for (int pp = 0; pp < KT / 2; ++pp) {
          uint32_t a[2][4];
          k_frag_int4<D>(st, r, c, pp, a);
          mma16816(sacc[GROUP ? pp : 0], a[0][0], a[0][1], a[0][2], a[0][3], qperm[2 * pp][0], qperm[2 * pp][1]);
          mma16816(sacc[GROUP ? pp : 0], a[1][0], a[1][1], a[1][2], a[1][3], qperm[2 * pp + 1][0],
                   qperm[2 * pp + 1][1]);
          if (fmt == IAK_FMT_INT4R) {
            k_frag_int4<D>(st + kResOff, r, c, pp, a);
            mma16816(racc[GROUP ? pp : 0], a[0][0], a[0][1], a[0][2], a[0][3], qperm[2 * pp][0], qperm[2 * pp][1]);
            mma16816(racc[GROUP ? pp : 0], a[1][0], a[1][1], a[1][2], a[1][3], qperm[2 * pp + 1][0],
                     qperm[2 * pp + 1][1]);
          }
        }
      }
      // ---------------- scale + online softmax (log2 domain)
      float sc[4];
      if (!GROUP) {
        const float ks = scal_s[i], krs = scal_s[2 * kChunkMax + i];
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] = (sacc[0][e] * ks + racc[0][e] * krs) * qk_log2;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] = 0.f;
        const bool q = fmt != IAK_FMT_F16;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const float ks = q ? gsc[g] : 1.f, krs = fmt == IAK_FMT_INT4R ? gsc[32 + g] : 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[e] += sacc[g][e] * ks + racc[g][e] * krs;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] *= qk_log2;
      }
      float pm0 = fmaxf(sc[0], sc[2]), pm1 = fmaxf(sc[1], sc[3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        pm0 = fmaxf(pm0, __shfl_xor_sync(0xffffffffu, pm0, off));
        pm1 = fmaxf(pm1, __shfl_xor_sync(0xffffffffu, pm1, off));
      }
      const float mn0 = fmaxf(m_run[0], pm0), mn1 = fmaxf(m_run[1], pm1);
      const float al0 = exp2f(m_run[0] - mn0), al1 = exp2f(m_run[1] - mn1);
      m_run[0] = mn0; m_run[1] = mn1;
      const float p0 = exp2f(sc[0] - mn0), p1 = exp2f(sc[1] - mn1);
      const float p2 = exp2f(sc[2] - mn0), p3 = exp2f(sc[3] - mn1);
      l_run[0] = l_run[0] * al0 + p0 + p2;
      l_run[1] = l_run[1] * al1 + p1 + p3;
#pragma unroll
      for (int mt = 0; mt < KT; ++mt) {
        oacc[mt][0] *= al0; oacc[mt][1] *= al1; oacc[mt][2] *= al0; oacc[mt][3] *= al1;
      }
      // ---------------- O^T += V^T P^T
      uint32_t vh[2][D / 64][8];
      if (!GROUP) {
        // per-page V scale folded into P
        const float vs = scal_s[kChunkMax + i];
        const uint32_t pb0 = movm_t(pack_f16x2(p0 * vs, p1 * vs));
        const uint32_t pb1 = movm_t(pack_f16x2(p2 * vs, p3 * vs));
        if (fmt == IAK_FMT_F16) v_table_f16<D>(st + kVOff, r, c, vh);
        else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) v_table_8bit<D>(st + kVOff, r, c, fmt == IAK_FMT_FP8, vh);
        else v_table_int4<D>(st + kVOff, r, c, vh);
#pragma unroll
        for (int mt = 0; mt < KT; ++mt) {
          uint32_t a0, a1, a2, a3;
          pv_afrag<D>(vh, mt, a0, a1, a2, a3);
          mma16816(oacc[mt], a0, a1, a2, a3, pb0, pb1);
        }
        if (fmt == IAK_FMT_INT4R) {
          const float vrs = scal_s[3 * kChunkMax + i];
          const uint32_t rb0 = movm_t(pack_f16x2(p0 * vrs, p1 * vrs));
          const uint32_t rb1 = movm_t(pack_f16x2(p2 * vrs, p3 * vrs));
          v_table_int4<D>(st + kVOff + kResOff, r, c, vh);
#pragma unroll
          for (int mt = 0; mt < KT; ++mt) {
            uint32_t a0, a1, a2, a3;
            pv_afrag<D>(vh, mt, a0, a1, a2, a3);
            mma16816(oacc[mt], a0, a1, a2, a3, rb0, rb1);
          }
        }
      } else {
        // per-32-channel V scales: rows r use group gA, rows r+8 group gB
        const uint32_t pb0 = movm_t(pack_f16x2(p0, p1));
        const uint32_t pb1 = movm_t(pack_f16x2(p2, p3));
        const int gA = pv_word<D>(r, 0) >> 2, gB = pv_word<D>(r, D / 64 - 1) >> 2;
        const bool q = fmt != IAK_FMT_F16;
        const int nplanes = fmt == IAK_FMT_INT4R ? 2 : 1;
        for (int pl = 0; pl < nplanes; ++pl) {
          const float* vsc = gsc + (pl == 0 ? 16 : 48);
          const float sA = q ? vsc[gA] : 1.f, sB = q ? vsc[gB] : 1.f;
          const char* vt = st + kVOff + pl * kResOff;
          if (fmt == IAK_FMT_F16) v_table_f16<D>(vt, r, c, vh);
          else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) v_table_8bit<D>(vt, r, c, fmt == IAK_FMT_FP8, vh);
          else v_table_int4<D>(vt, r, c, vh);
#pragma unroll
          for (int mt = 0; mt < KT; ++mt) {
            uint32_t a0, a1, a2, a3;
            pv_afrag<D>(vh, mt, a0, a1, a2, a3);
            float t[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(t, a0, a1, a2, a3, pb0, pb1);
            oacc[mt][0] = fmaf(t[0], sA, oacc[mt][0]); oacc[mt][1] = fmaf(t[1], sA, oacc[mt][1]);
            oacc[mt][2] = fmaf(t[2], sB, oacc[mt][2]); oacc[mt][3] = fmaf(t[3], sB, oacc[mt][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[kStages + s]));
    }
    // full l per query column: sum the 8 lanes that share c
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], off);
      l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], off);
    }
  }
  if (timed_out) atomicAdd(&g_decode_timeouts, 1u);
  __syncthreads();  // every stage consumed: the ring is free for the epilogue

  // ---------------------------------------------------------------- epilogue
  float* red_m = reinterpret_cast<float*>(smem);          // [4][8]
  float* red_l = red_m + 32;                               // [4][8]
  float* red_o = red_m + 64;                               // [4][8][D]
  if (warp < kConsumerWarps) {
    if (r == 0) {
      red_m[warp * 8 + 2 * c] = m_run[0]; red_m[warp * 8 + 2 * c + 1] = m_run[1];
      red_l[warp * 8 + 2 * c] = l_run[0]; red_l[warp * 8 + 2 * c + 1] = l_run[1];
    }
#pragma unroll
    for (int mt = 0; mt < KT; ++mt) {
      const int d0 = pv_channel<D>(mt, r), d1 = pv_channel<D>(mt, r + 8);
      float* o0 = red_o + (warp * 8 + 2 * c) * D;
      float* o1 = o0 + D;
      o0[d0] = oacc[mt][0]; o1[d0] = oacc[mt][1];
      o0[d1] = oacc[mt][2]; o1[d1] = oacc[mt][3];
    }
  }
  __syncthreads();
  const int G = p.G;
  for (int idx = tid; idx < G * D; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w)
      if (red_l[w * 8 + g] > 0.f) M = fmaxf(M, red_m[w * 8 + g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float lw = red_l[w * 8 + g];
        if (lw > 0.f) {
          const float e = exp2f(red_m[w * 8 + g] - M);
          L += lw * e;
          A += red_o[(w * 8 + g) * D + d] * e;
        }
      }
    }
    const float Mn = M * 0.6931471805599453f;  // partials carry the natural-log max
    const int hq = hk * G + g;
    const int64_t row = static_cast<int64_t>(b) * p.Hq + hq;
    if (p.num_splits > 1) {
      const int64_t wi = row * p.num_splits + split;
      if (d == 0) {
        p.ws_m[wi] = Mn;
        p.ws_l[wi] = L;
      }
      p.ws_acc[wi * D + d] = A;
    } else if (p.ex_l) {
      if (d == 0) {
        p.ex_m[row] = Mn;
        p.ex_l[row] = L;
      }
      p.ex_acc[row * D + d] = A;
    } else {
      store_from_float(p.out, p.out_dtype, b * p.o_sb + hq * p.o_sh + d, L > 0.f ? A / L : 0.f);
    }
  }
}

// --------------------------------------------------------- tensor maps ---
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D view [rows, inner] of a pool with a [box_rows, box_inner] box, 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
             uint64_t rows, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(IAK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * elem_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(IAK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return IAK_OK;
}

struct MapKey {
  const void* base; uint64_t inner, rows; int kind;
  bool operator==(const MapKey& o) const { return base == o.base && inner == o.inner && rows == o.rows && kind == o.kind; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.base) ^ (k.inner * 1315423911u) ^ (k.rows * 2654435761u) ^ k.kind;
  }
};

int cached_map(CUtensorMap* out, const void* base, int kind, int D, int64_t num_pages) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  // kind 0: fp16 rows (box 64 halves x 16 tokens); 1: 8-bit; 2: packed int4
  uint64_t inner, rows;
  uint32_t box_rows;
  CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  int eb = 1;
  const uint64_t tokens = static_cast<uint64_t>(num_pages) * kPS;
  if (kind == 0) {
    dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; eb = 2; inner = D; rows = tokens; box_rows = kPS;
  } else {
    const uint64_t row_bytes = kind == 1 ? D : D / 2;      // bytes per token row
    const uint64_t per_line = 128 / row_bytes;             // token rows per 128-byte line
    inner = 128; rows = tokens / per_line; box_rows = static_cast<uint32_t>(kPS / per_line);
  }
  MapKey key{base, inner, rows, kind * 1000 + D};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return IAK_OK;
    }
  }
  const uint32_t box_inner = kind == 0 ? 64 : 128;
  int st = make_map(out, base, dt, eb, inner, rows, box_inner, box_rows);
  if (st) return st;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 256) cache.clear();
  cache.emplace(key, *out);
  return IAK_OK;
}

}  // namespace

bool mma_path_eligible(const DecodeParams& p) {
  if (p.PS != kPS || (p.D != 64 && p.D != 128)) return false;
  if (p.q_dtype != IAK_DT_F16 && p.q_dtype != IAK_DT_BF16) return false;
  if (p.scale_mode == IAK_SCALE_CHANNEL) return false;
  if (p.scale_mode == IAK_SCALE_GROUP32 && p.D != 128) return false;
  if (p.pages_per_split > kChunkMax) return false;
  return true;
}

int launch_decode_mma(const DecodeParams& p, const iak_page_pools& P, cudaStream_t s, bool* launched) {
  *launched = false;
  if (!mma_path_eligible(p)) return IAK_OK;
  TmaMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  struct { const void* ptr; int idx; int kind; } pools[] = {
      {P.k_f16, M_KF16, 0}, {P.v_f16, M_VF16, 0}, {P.k_fp8, M_KFP8, 1}, {P.v_fp8, M_VFP8, 1},
      {P.k_i8, M_KI8, 1},   {P.v_i8, M_VI8, 1},   {P.k_i4, M_KI4, 2},   {P.v_i4, M_VI4, 2},
      {P.k_i4r, M_KI4R, 2}, {P.v_i4r, M_VI4R, 2}};
  for (auto& e : pools) {
    if (!e.ptr) continue;
    if (reinterpret_cast<uintptr_t>(e.ptr) % 16) return fail(IAK_ERR_INVALID_ARG, "page pool not 16-byte aligned");
    int st = cached_map(&maps.m[e.idx], e.ptr, e.kind, p.D, P.num_pages);
    if (st) return st;
  }
  const size_t smem = SmemLayout::total + 1024;
  const int units = p.B * p.Ht;
  dim3 grid(p.num_splits, units);
  cudaError_t err;
  if (p.D == 128 && p.scale_mode == IAK_SCALE_GROUP32) {
    err = cudaFuncSetAttribute(decode_mma_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err == cudaSuccess) decode_mma_kernel<128, true><<<grid, kThreads, smem, s>>>(p, maps);
  } else if (p.D == 128) {
    err = cudaFuncSetAttribute(decode_mma_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err == cudaSuccess) decode_mma_kernel<128, false><<<grid, kThreads, smem, s>>>(p, maps);
  } else {
    err = cudaFuncSetAttribute(decode_mma_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err == cudaSuccess) decode_mma_kernel<64, false><<<grid, kThreads, smem, s>>>(p, maps);
  }
  if (err != cudaSuccess) return check_cuda(err, "decode_mma smem attribute");
  *launched = true;
  return check_cuda(cudaGetLastError(), "decode_mma launch");
}

}  // namespace iak
