// Tensor-core split-KV paged decode for sm_100a.
//
// A persistent kernel, two CTAs per SM, walks a list of work items; an item is
// one (sequence, page-table head) unit x one contiguous range of its page table
// (a KV split).  Per CTA: warp 0 (the preparer) compacts the next item's page
// list and bulk-copies its query table, warp 1 (the producer) gathers every
// selected page with TMA tensor copies (128-byte swizzle, no multicast) into a
// ring of shared-memory stages guarded by mbarriers, and warps 2-5 consume the
// stages round-robin; each consumer warp owns one 16-token page at a time and
// runs
//
//   S^T[16 tok x 8 q] = K[16 x D] . Q^T        (mma.sync m16n8k16, fp16 -> fp32)
//   online softmax over tokens (exp2 domain, running max per query head)
//   O^T[D x 8 q]     += V^T[D x 16] . P^T       (mma.sync m16n8k16)
//
// with the page's codes dequantised in registers: int8 / int4 codes become
// exact fp16 integers by exponent-bias tricks, e4m3 codes by cvt.f16x2.e4m3x2,
// and the per-page (or per-32-channel) scale is applied in fp32 to S and folded
// into P for V.  The query group of a GQA head is the MMA's N dimension, so G
// <= 8 query heads share every K/V byte.  At the end of an item each consumer
// warp leaves its (m, l, O) partial in a shared-memory merge area; the
// preparer merges the four into the item's partial in the workspace, and the
// last item of a unit to finish (a counter per unit) merges the unit's splits
// into the output row, the caller's partial export, or every peer's exchange
// slot, so no merge launch follows.
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

#include <algorithm>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "iak_internal.cuh"

namespace iak {

__device__ unsigned int g_decode_timeouts = 0;

namespace {

constexpr int kPS = 16;
// Warp roles of the persistent decode CTA (two CTAs per SM): warp 0 prepares the
// next work item, warp 1 issues the TMA page loads, warps 2-5 consume the pages.
// Measured alternatives, all correct and all slower at C2 / C3 / C5: one CTA per SM
// with 12 consumer warps (setmaxnreg 56 / 152) fed by one or three producer warps,
// by the consumers themselves (TMA, bulk or cp.async copies) through per-warp byte
// FIFOs, or from a 24-stage ring (C2 394-466 us against 275 us for this layout); and
// bulk L2 prefetches of the pages 16 or 32 slots ahead of the copies (C2 370 us against
// 283: the prefetches queue on the same TMA unit as the stage copies).
constexpr int kConsumerWarps = 4;
constexpr int kPrepWarp = 0;                      // prepares the next work item
constexpr int kProducerWarps = 1;                 // warp 1 issues the TMA page loads
constexpr int kFirstConsumerWarp = 2;
constexpr int kThreads = (kFirstConsumerWarp + kConsumerWarps) * 32;
constexpr int kCtasPerSm = 2;
constexpr int kChunkMax = 256;                    // table slots per work item
// Page slots: every consumer warp owns a sub-ring of slots, filled in its own order by
// the producer lane that feeds it; page i of an item goes to consumer warp
// i % kConsumerWarps.  With per-page scales a warp has two 8 KB slots, one page each
// (K 4 KB | V 4 KB).  With group-32 scales it has four 4 KB slots: a D = 128 FP16 page
// takes two and every other page one (K at 0, V at 2 KB, INT4 residual planes at +1 KB),
// so a warp has three to four low-bit pages in flight (C3 455 -> 434 us).  The same
// compact slots for page-scaled pools measured C2 280 -> 308 us and C5 529 -> 545 us:
// there the consumers, not the pages in flight, are the bound.
constexpr int kSlots = 16;                        // barrier pairs (four 4 KB slots per warp)
constexpr int kSlotRegion = 65536;                // shared memory of all slots
constexpr int kResOff = 1024;                     // INT4 residual plane inside a K or V region
constexpr int kStageScaleBytes = 64;              // group scales of a slot: k | v | k res | v res
constexpr long long kWaitCycles = kDefaultWaitCycles;  // budget of the drain waits
constexpr float kLazyLog2 = 8.f;                  // rescale O only when the max grows by > 2^8
// F16 pages at D = 128: one TMA box of 32 half-rows (token-major, 256-byte token rows)
constexpr bool kF16OneBox = true;
// Issuing lanes of the producer warp: one per consumer warp, each feeding that warp's slot
// sub-ring in its page order.  With two lanes feeding two sub-rings each, a lane waiting for
// one warp's slot holds back the other warp's pages; once page-scaled slots free their K and
// V halves separately that coupling costs C2 310 us against 260-264 with four lanes.
constexpr int kProducerLanes = 4;

enum MapIdx { M_KF16 = 0, M_VF16, M_KFP8, M_VFP8, M_KI8, M_VI8, M_KI4, M_VI4, M_KI4R, M_VI4R, M_COUNT };
struct TmaMaps {
  CUtensorMap m[M_COUNT];
};

// Per-unit query table (built by decode_prep_kernel, bulk-copied per work item):
// fp16 fragments [D/16][32] uint4 | int8 terms [D/32][32] uint4 | the same in
// INT4 order | 128 words: term scales s1[8], s2[8] = s1 / 256 (floats); at kQB1 / kQB2 the
// int32 offsets -8 * sum(i1) / -8 * sum(i2) of each 32-channel block and query
// head ([block][head]), at kQB1T / kQB2T the same over all channels, which start
// the INT4 integer-MMA accumulators so that the +8 of the offset-binary codes
// cancels exactly; at kQScF the power-of-two factor of each head's fp16 fragments.
constexpr int kQFrag = 0, kQI8 = 4096, kQI4 = 6144, kQSc = 8192, kQTab = 8704;
constexpr int kQB1 = 16, kQB2 = 48, kQScF = 80, kQB1T = 88, kQB2T = 96;

// One work-item buffer: query table | page ids | 4 scale scalars | formats | meta.
struct ItemLayout {
  static constexpr int qtab = 0;
  static constexpr int pid = kQTab;
  static constexpr int scal = pid + kChunkMax * 4;
  static constexpr int fmt = scal + 4 * kChunkMax * 4;
  static constexpr int meta = fmt + kChunkMax;                     // n_valid, unit, split
  static constexpr int bytes = (meta + 16 + 127) / 128 * 128;
};

// Merge area: each consumer warp's (acc[D], m, l) per query head of the item, read by
// the preparer when the item is finished.  Sized for head_dim 128 and 8 query heads.
constexpr int kMergeRow = 128 + 2;                // floats per (warp, head): acc | m | l
constexpr int kMergeFloats = kConsumerWarps * 8 * kMergeRow;

struct SmemLayout {
  static constexpr int stages = 0;                                      // the page slots
  static constexpr int scales = kSlotRegion;                            // [kSlots][64] group scales
  static constexpr int items = scales + kSlots * kStageScaleBytes;      // two ItemLayout buffers
  static constexpr int merge = items + 2 * ItemLayout::bytes;           // [warp][head][kMergeRow] floats
  static constexpr int bars = merge + kMergeFloats * 4;                 // full[16], empty[16], ilist[2], ifull[2], iempty[2], mfree
  static constexpr int total = bars + (2 * kSlots + 7) * 8;
  static_assert(total + 1024 <= 116736, "two persistent decode CTAs per SM");
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
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when the phase did not complete within `budget` SM cycles.  The
// budget is checked between a non-blocking test and each (suspending) try_wait, so a
// budget shorter than a global-memory round trip gives up on any phase that is not
// already complete.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long budget) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (clock64() - t0 > budget) return false;
    if (mbar_try_wait(bar, parity)) return true;
  }
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
// integer MMA m16n8k32: s32 += A(16x32, s8 or u8) * B(32x8, s8)
__device__ __forceinline__ void imma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
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
__device__ __forceinline__ void st_release_sys(uint32_t* ptr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
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
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

// INT4_RESIDUAL V with group scales, both planes in one table (D = 128): the base and residual
// codes of each pair, dequantised and combined as base * rb + residual * rr in f16, with rb / rr
// the groups' base / residual scales over the page's largest V scale (rows r: rbA / rrA, rows
// r + 8: rbB / rrB), so the page needs one P.V instead of one per plane.
__device__ __forceinline__ void v_table_int4r_group(const char* tb, const char* tr, int r, int c, uint32_t rbA,
                                                    uint32_t rbB, uint32_t rrA, uint32_t rrB,
                                                    uint32_t (&vh)[2][2][8]) {
  constexpr int RB = 64;
#pragma unroll
  for (int tp = 0; tp < 2; ++tp) {
    const int t0 = 2 * c + 8 * tp, t1 = t0 + 1;
#pragma unroll
    for (int ws = 0; ws < 2; ++ws) {
      const int w = pv_word<128>(r, ws);
      const uint32_t rb = ws == 0 ? rbA : rbB, rr = ws == 0 ? rrA : rrB;
      const uint32_t x0 = lds32(tb, sw128(t0 * RB + 4 * w)), x1 = lds32(tb, sw128(t1 * RB + 4 * w));
      const uint32_t y0 = lds32(tr, sw128(t0 * RB + 4 * w)), y1 = lds32(tr, sw128(t1 * RB + 4 * w));
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t sel = b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12);
        const uint32_t t = __byte_perm(x0, x1, sel), u = __byte_perm(y0, y1, sel);
        vh[tp][ws][2 * b] = hfma2(i4pair_lo(u), rr, hmul2(i4pair_lo(t), rb));
        vh[tp][ws][2 * b + 1] = hfma2(i4pair_hi(u), rr, hmul2(i4pair_hi(t), rb));
      }
    }
  }
}

// shared-memory offset of fp16 channel d (multiple of 4) of token t
template <int D>
__device__ __forceinline__ uint32_t f16_off(int t, int d) {
  if constexpr (D == 128 && kF16OneBox) return sw128(t * 256 + 2 * d);
  return sw128((d >> 6) * 2048 + t * 128 + ((2 * d) & 127));
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
        const uint32_t o0 = f16_off<D>(t0, d);
        const uint32_t o1 = f16_off<D>(t1, d);
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
// (fp16 and e4m3 pages use fp16 MMAs; INT8 / INT4 pages use the integer MMA
// on the raw codes, see the consumer loop)
// Raw code words of two consecutive 16-byte chunks (ch, ch+1) of the 16 token
// rows: x[0] = (row r, chunk ch), x[1] = (row r+8, ch), x[2] = (r, ch+1),
// x[3] = (r+8, ch+1), each the 4 bytes 4c..4c+3 of that chunk (ldmatrix of
// 8x16-byte matrices hands lane (r, c) exactly those bytes).
__device__ __forceinline__ void ldsm_rows(uint32_t tile_u32, int row_bytes, int lane, int ch, uint32_t (&x)[4]) {
  const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
  const int chunk = ch + (lane >> 4);
  ldsm_x4(tile_u32 + sw128(row * row_bytes + 16 * chunk), x[0], x[1], x[2], x[3]);
}

__device__ __forceinline__ void k_frag_8bit_from(uint32_t x0, uint32_t x1, bool fp8, uint32_t (&a)[4]) {
  if (fp8) {
    a[0] = e4m3x2_f16x2(x0); a[2] = e4m3x2_f16x2(x0 >> 16);
    a[1] = e4m3x2_f16x2(x1); a[3] = e4m3x2_f16x2(x1 >> 16);
  } else {
    const uint32_t y0 = x0 ^ 0x80808080u, y1 = x1 ^ 0x80808080u;
    a[0] = i8pair_lo(y0); a[2] = i8pair_hi(y0);
    a[1] = i8pair_lo(y1); a[3] = i8pair_hi(y1);
  }
}

template <int D>
__device__ __forceinline__ void k_frag_f16(uint32_t tile_u32, int lane, int kk, uint32_t (&a)[4]) {
  const int mi = lane >> 3, rr = lane & 7;
  const int tok = rr + 8 * (mi & 1);
  const int d = 16 * kk + 8 * (mi >> 1);
  ldsm_x4(tile_u32 + f16_off<D>(tok, d), a[0], a[1], a[2], a[3]);
}

// ------------------------------------------------------------- kernels ---
// Query table of one (sequence, page-table head) unit: fp16 fragments for the
// fp16 / e4m3 pages and the two int8 terms q = s1*i1 + s2*i2 (per query head;
// |error| <= s2/2 ~ absmax/32258) for the integer MMA of INT8 / INT4 pages,
// plus the per-32-channel sums of the terms that undo the INT4 +8 offset.
template <int D>
__global__ void __launch_bounds__(256) decode_prep_kernel(const DecodeParams p, char* __restrict__ qtab) {
  constexpr int KT = D / 16;
  constexpr int E = D / 32;            // channels per lane: d = E * lane + e
  constexpr int GL = 32 / E;           // lanes of one 32-channel block
  __shared__ float qs[8 * D];
  __shared__ int8_t i1s[8 * D], i2s[8 * D];
  __shared__ float qsc[128];
  __shared__ float qfi[8];
  const int unit = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = unit / p.Ht, hk = unit % p.Ht;
  // the decode kernel may start now (programmatic dependent launch); it waits for
  // this grid before it reads a query table or touches a merge counter
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid < 128) qsc[tid] = 0.f;
  // merge counters start at zero on every call
  if (tid == 0) p.ws_cnt[unit] = 0u;
  if (tid == 0 && unit == 0) *p.ws_done = 0u;
  {
    // warp g quantises query head g of the group (zeros past G): q = s1 * i1 + s2 * i2
    const int g = warp;
    const int64_t off = static_cast<int64_t>(b) * p.q_sb + static_cast<int64_t>(hk * p.G + g) * p.q_sh + E * lane;
    float q[E];
#pragma unroll
    for (int e = 0; e < E; ++e) q[e] = g < p.G ? load_as_float(p.q, p.q_dtype, off + e) : 0.f;
    float am = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) am = fmaxf(am, fabsf(q[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    // The fp16 fragments hold q / 2^fe with the head's absmax in [2^14, 2^15): bf16 queries
    // outside fp16's normal range (|q| > 65504, or below 2^-14) still convert exactly, and the
    // scores of fp16 / e4m3 pages are multiplied back by 2^fe.
    const int fe = min(max(((__float_as_int(am) >> 23) & 0xFF) - 127 - 14, -126), 126);
    if (lane == 0) qfi[g] = __int_as_float((127 - fe) << 23);
    const float s1 = am > 0.f ? am / 127.f : 1.f;
    // s2 = s1 / 256 exactly (the residual q - s1 * i1 is at most s1 / 2, i.e. 128 steps of s2):
    // the integer paths then combine the two terms' sums as 256 * I1 + I2 in int32 and apply
    // one scale, s2
    const float s2 = s1 * (1.f / 256.f);
    float t1[E];
#pragma unroll
    for (int e = 0; e < E; ++e) t1[e] = fminf(fmaxf(rintf(q[e] / s1), -127.f), 127.f);
    int sum1 = 0, sum2 = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float t2 = fminf(fmaxf(rintf((q[e] - t1[e] * s1) / s2), -127.f), 127.f);
      const int d = E * lane + e;
      qs[g * D + d] = q[e];
      i1s[g * D + d] = static_cast<int8_t>(t1[e]);
      i2s[g * D + d] = static_cast<int8_t>(t2);
      sum1 += static_cast<int>(t1[e]);
      sum2 += static_cast<int>(t2);
    }
    // sums of the terms over each 32-channel block and over all channels (they undo the
    // INT4 +8 offset)
    int tot1 = sum1, tot2 = sum2;
#pragma unroll
    for (int o = 1; o < GL; o <<= 1) {
      sum1 += __shfl_xor_sync(0xffffffffu, sum1, o);
      sum2 += __shfl_xor_sync(0xffffffffu, sum2, o);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      tot1 += __shfl_xor_sync(0xffffffffu, tot1, o);
      tot2 += __shfl_xor_sync(0xffffffffu, tot2, o);
    }
    __syncthreads();                   // qsc zeroed
    if (lane == 0) {
      qsc[g] = s1;
      qsc[8 + g] = s2;
      qsc[kQScF + g] = __int_as_float((fe + 127) << 23);
      qsc[kQB1T + g] = __int_as_float(-8 * tot1);
      qsc[kQB2T + g] = __int_as_float(-8 * tot2);
    }
    if (lane % GL == 0) {
      const int j = lane / GL;
      qsc[kQB1 + j * 8 + g] = __int_as_float(-8 * sum1);
      qsc[kQB2 + j * 8 + g] = __int_as_float(-8 * sum2);
    }
  }
  __syncthreads();
  char* out = qtab + static_cast<int64_t>(unit) * kQTab;
  const int r = lane >> 2, c = lane & 3;
  if (warp == 0) {
    const float* qr = qs + r * D;
    const float fi = qfi[r];
    uint4* qfrag = reinterpret_cast<uint4*>(out + kQFrag);
    auto h2 = [&](int d) { return pack_f16x2(qr[d] * fi, qr[d + 1] * fi); };
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
      const int b0 = 16 * kk + 2 * c, b1 = 16 * kk + 4 * c;
      qfrag[kk * 32 + lane] = make_uint4(h2(b0), h2(b0 + 8), h2(b1), h2(b1 + 2));
    }
  } else if (warp == 1) {
    uint4* qi8 = reinterpret_cast<uint4*>(out + kQI8);
    uint4* qi4 = reinterpret_cast<uint4*>(out + kQI4);
    auto pack4 = [&](const int8_t* t, int d0, int d1, int d2, int d3) {
      return static_cast<uint32_t>(static_cast<uint8_t>(t[d0])) |
             (static_cast<uint32_t>(static_cast<uint8_t>(t[d1])) << 8) |
             (static_cast<uint32_t>(static_cast<uint8_t>(t[d2])) << 16) |
             (static_cast<uint32_t>(static_cast<uint8_t>(t[d3])) << 24);
    };
    const int8_t* t1 = i1s + r * D;
    const int8_t* t2 = i2s + r * D;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      const int e = 32 * j + 4 * c;   // k = 4c..4c+3 and 16+4c..16+4c+3 of k-step j
      qi8[j * 32 + lane] = make_uint4(pack4(t1, e, e + 1, e + 2, e + 3), pack4(t1, e + 16, e + 17, e + 18, e + 19),
                                      pack4(t2, e, e + 1, e + 2, e + 3), pack4(t2, e + 16, e + 17, e + 18, e + 19));
      // INT4 word 4j+c expands to bytes of channels e+{0,16,1,17} (low nibbles) and e+{2,18,3,19}
      qi4[j * 32 + lane] = make_uint4(pack4(t1, e, e + 16, e + 1, e + 17), pack4(t1, e + 2, e + 18, e + 3, e + 19),
                                      pack4(t2, e, e + 16, e + 1, e + 17), pack4(t2, e + 2, e + 18, e + 3, e + 19));
    }
  }
  if (tid < 128) reinterpret_cast<float*>(out + kQSc)[tid] = qsc[tid];
}

// Work item -> (unit, split) and its table-slot range [lo, hi).
__device__ __forceinline__ void item_range(const DecodeParams& p, int item, int& unit, int& split, int& lo, int& hi) {
  unit = item / p.num_splits;
  split = item - unit * p.num_splits;
  const int b = unit / p.Ht, hk = unit - (unit / p.Ht) * p.Ht;
  int count = p.W;
  if (p.pc) {
    const int cc = p.pc[b * p.pc_sb + hk];
    count = cc < 0 ? 0 : (cc > p.W ? p.W : cc);
  }
  lo = split * p.pages_per_split;
  hi = min(lo + p.pages_per_split, count);
}

// One warp merges S partials (m natural-log max, l, acc[D]; m / l at stride 1, acc
// rows at stride D) into (M, L, A): the recurrence of the reference's decode loop
// (fused_selected_quant_decode.py:323-332) applied across partials.  Lane t owns
// channels t * D/32 .. t * D/32 + D/32 - 1.  Reads bypass L1 (other SMs wrote them)
// and are batched (all m / l, then the accumulator rows eight at a time) so that the
// merge costs a few L2 round trips, not one per partial.
template <int D>
__device__ __forceinline__ void warp_merge(const float* m, const float* l, const float* acc, int S, int lane,
                                           float& M, float& L, float (&A)[D / 32]) {
  constexpr int C = D / 32;
  float mx = -INFINITY, lsum = 0.f;
#pragma unroll
  for (int j = 0; j < C; ++j) A[j] = 0.f;
  for (int s0 = 0; s0 < S; s0 += 32) {
    const int s = s0 + lane;
    const float ls = s < S ? __ldcg(l + s) : 0.f;
    const float ms = s < S ? __ldcg(m + s) : -INFINITY;
    float cm = ls > 0.f ? ms : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    // rescale what earlier chunks accumulated to the new running max
    const float mnew = fmaxf(mx, cm);
    if (mnew != -INFINITY && mnew > mx && mx != -INFINITY) {
      const float a = expf(mx - mnew);
      lsum *= a;
#pragma unroll
      for (int j = 0; j < C; ++j) A[j] *= a;
    }
    mx = mnew;
    const float w = (ls > 0.f && mx != -INFINITY) ? expf(ms - mx) : 0.f;
    lsum = fmaf(ls, w, lsum);
    const int n = min(32, S - s0);
    for (int k0 = 0; k0 < n; k0 += 8) {
      float v[8][C];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (k0 + u < n) {
          const float* a = acc + static_cast<int64_t>(s0 + k0 + u) * D + lane * C;
          if constexpr (C == 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(a));
            v[u][0] = x.x; v[u][1] = x.y; v[u][2] = x.z; v[u][3] = x.w;
          } else {
            const float2 x = __ldcg(reinterpret_cast<const float2*>(a));
            v[u][0] = x.x; v[u][1] = x.y;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float wk = __shfl_sync(0xffffffffu, w, (k0 + u) & 31);
        if (k0 + u < n && wk != 0.f) {
#pragma unroll
          for (int j = 0; j < C; ++j) A[j] = fmaf(wk, v[u][j], A[j]);
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
  M = mx;
  L = lsum;
}

// Persistent split-KV decode, kCtasPerSm CTAs per SM.  CTA c processes one work item
// (unit, split) of <= kChunkMax table slots per wave of gridDim.x items (the full waves
// rotated by the CTA's turn, see item_of).  The
// preparer fills one of two item buffers ahead of use (compacted page list,
// scales, query table by bulk copy); the TMA warp streams every item's pages
// into the consumer warps' slot sub-rings (page i of an item goes to warp
// i % kConsumerWarps) without draining between items; each consumer warp writes
// its (m, l, acc) partial of an item into the shared-memory merge area.  The
// preparer merges the item's partials into the item's workspace slot, and the
// last item merged of a unit merges the unit's items into the output (or the
// exported partial block, or every peer's receive slot): no merge launch.
template <int D, bool GROUP>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    decode_mma_kernel(const DecodeParams p, const __grid_constant__ TmaMaps maps, const char* __restrict__ qtab,
                      int n_items) {
  constexpr int KT = D / 16;   // k-steps of QK, m-tiles of PV
  constexpr int NG = GROUP ? D / 32 : 1;
  constexpr int SPW = GROUP ? 4 : 2;             // slots per consumer warp
  // Page-scaled pools: each 8 KB slot holds one page, K at 0 and V at 4 KB, with a barrier
  // pair per half, so that the K half is released (and refilled with the page two ahead)
  // as soon as the page's scores are computed, and the V half after its P.V.
  constexpr bool SKV = !GROUP;
  constexpr int SB = GROUP ? 4096 : 8192;        // bytes per slot
  constexpr int LPW = kProducerLanes;
  static_assert(kConsumerWarps == 4 && kProducerWarps == 1 && kConsumerWarps % LPW == 0, "slot sub-ring mapping");
  using SL = SmemLayout;
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SL::bars);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, c = lane & 3;
  auto full_bar = [&](int st) { return smem_u32(&bars[st]); };
  auto empty_bar = [&](int st) { return smem_u32(&bars[kSlots + st]); };
  auto ilist_bar = [&](int buf) { return smem_u32(&bars[2 * kSlots + buf]); };
  auto ifull_bar = [&](int buf) { return smem_u32(&bars[2 * kSlots + 2 + buf]); };
  auto iempty_bar = [&](int buf) { return smem_u32(&bars[2 * kSlots + 4 + buf]); };
  const uint32_t mfree_bar = smem_u32(&bars[2 * kSlots + 6]);   // the preparer has read the merge area
  // slots a page of format fmt takes, and where its V plane starts
  auto page_slots = [&](int fmt) { return (GROUP && D == 128 && fmt == IAK_FMT_F16) ? 2 : 1; };
  auto v_off = [&](int fmt) { return (!GROUP || (D == 128 && fmt == IAK_FMT_F16)) ? 4096u : 2048u; };
  float* merge_area = reinterpret_cast<float*>(smem + SL::merge);
  auto item_buf = [&](int buf) { return smem + SL::items + buf * ItemLayout::bytes; };
  auto stage_scales = [&](int st) { return smem + SL::scales + st * kStageScaleBytes; };

  if (tid == 0) {
    for (int i = 0; i < 2 * kSlots; ++i) mbar_init(smem_u32(&bars[i]), 1);
    // list-ready: the preparer's arrive; item-ready: its arrive after the page list +
    // its arrive.expect_tx of the query-table bytes; item-free: one per consumer warp
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(ilist_bar(b2), 1);
      mbar_init(ifull_bar(b2), 2);
      mbar_init(iempty_bar(b2), kConsumerWarps);
    }
    mbar_init(mfree_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  // A role whose bounded wait gives up (p.wait_cycles) stops; every wait result is
  // made warp-uniform first, so the warp's collectives stay converged.  Before the
  // CTA exits, the lanes that issued bulk / TMA copies wait (with the default budget)
  // for the copies they issued, so no copy lands in a finished CTA's shared memory.
  bool timed_out = false;
  const long long budget = p.wait_cycles;
  auto wait_all = [&](uint32_t bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, budget));
  };

  if (warp == kPrepWarp) {
    // -------------------------------------------------------------- preparer
    constexpr int kPer = kChunkMax / 32;
    // Merge of a finished item (all its consumer warps have written their level-0
    // partials and arrived on its item-free barrier): the kConsumerWarps partials ->
    // the item's level-1 slot; the unit's last merged item merges the unit's splits into
    // the output (level 2).  Done here, off the consumers and the stage ring.
    auto merge_item = [&](int item_done) {
      const int unit = item_done / p.num_splits, split = item_done - unit * p.num_splits;
      const int bb = unit / p.Ht, hk = unit - bb * p.Ht;
      const int64_t row0 = static_cast<int64_t>(bb) * p.Hq + hk * p.G;
      for (int g = 0; g < p.G; ++g) {
        const int64_t row = row0 + g;
        float M = -INFINITY, L = 0.f, A[D / 32], wt[kConsumerWarps];
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float* mr = merge_area + (w * 8 + g) * kMergeRow;
          if (mr[129] > 0.f) M = fmaxf(M, mr[128]);
        }
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float* mr = merge_area + (w * 8 + g) * kMergeRow;
          wt[w] = (mr[129] > 0.f && M != -INFINITY) ? expf(mr[128] - M) : 0.f;
          L = fmaf(mr[129], wt[w], L);
        }
#pragma unroll
        for (int j = 0; j < D / 32; ++j) {
          float a = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w)
            if (wt[w] != 0.f) a = fmaf(wt[w], merge_area[(w * 8 + g) * kMergeRow + lane * (D / 32) + j], a);
          A[j] = a;
        }
        const int64_t w1 = row * p.num_splits + split;
        if (lane == 0) {
          p.ws_m1[w1] = M;
          p.ws_l1[w1] = L;
        }
#pragma unroll
        for (int j = 0; j < D / 32; ++j) p.ws_acc1[w1 * D + lane * (D / 32) + j] = A[j];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mfree_bar);          // the consumers may write the next item's partials
      __threadfence();
      __syncwarp();
      unsigned ulast = 0;
      if (lane == 0) ulast = atomicAdd(&p.ws_cnt[unit], 1u) == static_cast<unsigned>(p.num_splits) - 1;
      if (__shfl_sync(0xffffffffu, ulast, 0)) {
        __threadfence();
        // fused exchange: the epoch this launch publishes (the merge that follows on
        // every rank reads the receive array of its parity)
        uint32_t epoch = 0;
        if (p.x_world > 0)
          epoch = *reinterpret_cast<const volatile uint32_t*>(
                      reinterpret_cast<const char*>(p.x_areas[p.x_rank]) + p.x_flags_off +
                      (2 * p.x_world + 2) * sizeof(uint32_t)) + 1u;
        const int64_t xrows = static_cast<int64_t>(p.B) * p.Hq;
        for (int g = 0; g < p.G; ++g) {
          const int64_t row = row0 + g;
          const int64_t w1 = row * p.num_splits;
          float M, L, A[D / 32];
          warp_merge<D>(p.ws_m1 + w1, p.ws_l1 + w1, p.ws_acc1 + w1 * D, p.num_splits, lane, M, L, A);
          if (p.x_world > 0) {
            // the row's partial straight into slot x_rank of every rank's receive array
            for (int rk = 0; rk < p.x_world; ++rk) {
              float* blk = p.x_areas[rk] + static_cast<int64_t>((epoch & 1u) * p.x_world + p.x_rank) * p.x_bs;
              if (lane == 0) {
                blk[row] = M;
                blk[xrows + row] = L;
              }
#pragma unroll
              for (int j = 0; j < D / 32; ++j) blk[2 * xrows + row * D + lane * (D / 32) + j] = A[j];
            }
          } else if (p.ex_l) {
            if (lane == 0) {
              p.ex_m[row] = M;
              p.ex_l[row] = L;
            }
#pragma unroll
            for (int j = 0; j < D / 32; ++j) p.ex_acc[row * D + lane * (D / 32) + j] = A[j];
          } else {
            const int64_t off = static_cast<int64_t>(bb) * p.o_sb + static_cast<int64_t>(hk * p.G + g) * p.o_sh;
            const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
            for (int j = 0; j < D / 32; ++j) store_from_float(p.out, p.out_dtype, off + lane * (D / 32) + j, A[j] * inv);
          }
        }
        if (p.x_world > 0) {
          // once every unit of this launch has stored its rows, raise this rank's flag
          // (the epoch) in every area, then advance the epoch
          __threadfence_system();
          __syncwarp();
          unsigned dlast = 0;
          if (lane == 0) dlast = atomicAdd(p.ws_done, 1u) == static_cast<unsigned>(p.B * p.Ht) - 1;
          if (__shfl_sync(0xffffffffu, dlast, 0)) {
            __threadfence_system();
            if (lane < p.x_world)
              st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(p.x_areas[lane]) + p.x_flags_off) +
                                 (epoch & 1u) * p.x_world + p.x_rank,
                             epoch);
            __syncwarp();
            if (lane == 0)
              *reinterpret_cast<volatile uint32_t*>(reinterpret_cast<char*>(p.x_areas[p.x_rank]) + p.x_flags_off +
                                                    (2 * p.x_world + 2) * sizeof(uint32_t)) = epoch;
          }
        }
      }
    };
    int last_k[2] = {-1, -1};   // last item whose query table was copied into each buffer
    const int n_mine = blockIdx.x < n_items ? (n_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    // This CTA's k-th item: items go in waves of gridDim.x, each full wave rotated by k CTAs,
    // so that a CTA visits different splits of the units (unrotated, a grid that is a multiple
    // of the split count would hand every CTA the same split of each unit it visits, and the
    // splits differ in their page formats and so in cost); the partial last wave is not rotated.
    // The producer and consumers only count turns, which the rotation leaves unchanged.
    const int nb = static_cast<int>(gridDim.x);
    auto item_of = [&](int k) {
      const int base = k * nb;
      return base + nb <= n_items ? base + (static_cast<int>(blockIdx.x) + k) % nb : base + static_cast<int>(blockIdx.x);
    };
    for (int k = 0, turn = blockIdx.x; turn < n_items; ++k, turn += gridDim.x) {
      const int item = item_of(k);
      const int buf = k & 1;
      char* ib = item_buf(buf);
      if (k >= 2) {
        // item k - 2 is finished: merge it, then reuse its buffer
        if (!wait_all(iempty_bar(buf), ((k >> 1) - 1) & 1)) {
          timed_out = true;
          break;
        }
        merge_item(item_of(k - 2));
      }
      int unit, split, lo, hi;
      item_range(p, item, unit, split, lo, hi);
      const int bb = unit / p.Ht, hk = unit - bb * p.Ht;
      const int32_t* table = p.pt + bb * p.pt_sb + hk * p.pt_sh;
      int32_t* pid_s = reinterpret_cast<int32_t*>(ib + ItemLayout::pid);
      float* scal_s = reinterpret_cast<float*>(ib + ItemLayout::scal);
      uint8_t* fmt_s = reinterpret_cast<uint8_t*>(ib + ItemLayout::fmt);
      // All loads of the item first, in three dependent rounds (the table slice with the
      // page count, the formats, the page scales), then compaction.  The table loads are
      // bounded by the table row, not by the page count, so they do not wait for it.
      const int hw = min(lo + p.pages_per_split, p.W);
      int pids[kPer], fmts[kPer];
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const int j = lo + 32 * t + lane;
        pids[t] = j < hw ? table[j] : -1;
      }
#pragma unroll
      for (int t = 0; t < kPer; ++t)
        if (lo + 32 * t + lane >= hi) pids[t] = -1;
#pragma unroll
      for (int t = 0; t < kPer; ++t)
        fmts[t] = (pids[t] >= 0 && pids[t] < p.num_pages) ? page_format(p, pids[t]) : IAK_FMT_SKIP;
      // page scales into registers (issued before the compaction's shared-memory stores,
      // which loads placed after them would wait for)
      float ksc[GROUP ? 1 : kPer], vsc[GROUP ? 1 : kPer], krs[GROUP ? 1 : kPer], vrs[GROUP ? 1 : kPer];
      if constexpr (!GROUP) {
#pragma unroll
        for (int t = 0; t < kPer; ++t) {
          const int fmt = fmts[t], pid = pids[t];
          const bool q = fmt != IAK_FMT_F16 && fmt != IAK_FMT_SKIP && fmt != IAK_FMT_SPARSE;
          const bool r4 = fmt == IAK_FMT_INT4R;
          ksc[t] = q ? __ldg(p.k_scale + pid) : 1.f;
          vsc[t] = q ? __ldg(p.v_scale + pid) : 1.f;
          krs[t] = r4 ? __ldg(p.k_rscale + pid) : 0.f;
          vrs[t] = r4 ? __ldg(p.v_rscale + pid) : 0.f;
        }
      }
      int n = 0, idxs[kPer];
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const int fmt = fmts[t], pid = pids[t];
        const bool valid = fmt != IAK_FMT_SKIP && fmt != IAK_FMT_SPARSE;
        const unsigned bal = __ballot_sync(0xffffffffu, valid);
        idxs[t] = valid ? n + __popc(bal & ((1u << lane) - 1u)) : -1;
        if (valid) {
          pid_s[idxs[t]] = pid;
          fmt_s[idxs[t]] = static_cast<uint8_t>(fmt);
        }
        n += __popc(bal);
      }
      if (lane == 0) {
        int* meta = reinterpret_cast<int*>(ib + ItemLayout::meta);
        meta[0] = n;
        meta[1] = unit;
        meta[2] = split;
      }
      __syncwarp();
      // the page list is all the producer reads: it may start the item's copies while
      // the scales land
      if (lane == 0) mbar_arrive(ilist_bar(buf));
      if constexpr (!GROUP) {
#pragma unroll
        for (int t = 0; t < kPer; ++t)
          if (idxs[t] >= 0) {
            scal_s[idxs[t]] = ksc[t];
            scal_s[kChunkMax + idxs[t]] = vsc[t];
            scal_s[2 * kChunkMax + idxs[t]] = krs[t];
            scal_s[3 * kChunkMax + idxs[t]] = vrs[t];
          }
        __syncwarp();
      }
      if (lane == 0) mbar_arrive(ifull_bar(buf));
      // the query tables come from the preparation kernel, which may still be
      // running (programmatic dependent launch): wait for it before the first copy
      if (k == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
      last_k[buf] = k;
      if (lane == 0) {
        mbar_arrive_expect_tx(ifull_bar(buf), kQTab);
        bulk_load(smem_u32(ib + ItemLayout::qtab), qtab + static_cast<int64_t>(unit) * kQTab, kQTab, ifull_bar(buf));
      }
    }
    // the items whose merge the loop has not reached: this CTA's last two
    for (int j = max(0, n_mine - 2); j < n_mine && !timed_out; ++j) {
      if (!wait_all(iempty_bar(j & 1), (j >> 1) & 1)) {
        timed_out = true;
        break;
      }
      merge_item(item_of(j));
    }
    // drain: the query-table copies this warp issued
    for (int b2 = 0; b2 < 2; ++b2)
      if (lane == 0 && last_k[b2] >= 0 && !mbar_wait(ifull_bar(b2), (last_k[b2] >> 1) & 1, kWaitCycles))
        timed_out = true;
  } else if (warp < kFirstConsumerWarp) {
    // -------------------------------------------------------------- TMA producers
    // Lane l < LPW of the producer warp handles pages i = l (mod LPW) of every item; page i
    // goes to consumer warp i % 4, so lane l feeds the sub-rings of warps l, l + LPW, ...
    // and keeps one slot counter per fed warp (slot u of warp w is sub-ring slot u % 4 in
    // its round u / 4).  A two-slot page never wraps: if it would start at the last slot,
    // that slot is skipped (its phase completed without data), which the consumer mirrors.
    const int pl = (warp - 1) * LPW + lane;
    constexpr int kFed = kConsumerWarps / LPW;
    int cnt[kFed];
#pragma unroll
    for (int t = 0; t < kFed; ++t) cnt[t] = 0;
    // claim slot u of warp w: wait until its previous round was released
    auto claim = [&](int w, int u, int part = 0) -> bool {
      const int st = w * SPW + u % SPW, round = u / SPW;
      return round == 0 || mbar_wait(empty_bar(SKV ? 2 * st + part : st), (round - 1) & 1, budget);
    };
    for (int k = 0, item = blockIdx.x; item < n_items && !timed_out; ++k, item += gridDim.x) {
      const int buf = k & 1;
      const char* ib = item_buf(buf);
      if (!wait_all(ilist_bar(buf), (k >> 1) & 1)) {
        timed_out = true;
        break;
      }
      const int n = reinterpret_cast<const int*>(ib + ItemLayout::meta)[0];
      const int32_t* pid_s = reinterpret_cast<const int32_t*>(ib + ItemLayout::pid);
      const uint8_t* fmt_s = reinterpret_cast<const uint8_t*>(ib + ItemLayout::fmt);
      if (lane < LPW) {
        for (int i = pl; i < n; i += kProducerLanes) {
          const int w = i % kConsumerWarps, t = w / LPW;
          const int fmt = fmt_s[i], pid = pid_s[i];
          const int ns = page_slots(fmt);
          int u = cnt[t];
          if constexpr (SKV) {
            // K half, then V half, each armed with its own bytes
            if (!claim(w, u, 0)) { timed_out = true; break; }
            const int st = w * SPW + u % SPW;
            cnt[t] = u + 1;
            const uint32_t sa = smem_u32(smem + SL::stages + st * SB);
            const uint32_t kfull = full_bar(2 * st), vfull = full_bar(2 * st + 1);
            const uint32_t half = fmt == IAK_FMT_F16 ? kPS * D * 2 : (fmt == IAK_FMT_INT4 ? kPS * D / 2 : kPS * D);
            mbar_arrive_expect_tx(kfull, half);
            if (fmt == IAK_FMT_F16) {
              if constexpr (D == 128 && kF16OneBox) tma_load_2d(sa, &maps.m[M_KF16], 0, pid * kPS * 2, kfull);
              else tma_load_2d(sa, &maps.m[M_KF16], 0, pid * kPS, kfull);
            } else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) {
              tma_load_2d(sa, &maps.m[fmt == IAK_FMT_FP8 ? M_KFP8 : M_KI8], 0, pid * (kPS * D / 128), kfull);
            } else {
              const int y = pid * (kPS * D / 256);
              tma_load_2d(sa, &maps.m[M_KI4], 0, y, kfull);
              if (fmt == IAK_FMT_INT4R) tma_load_2d(sa + kResOff, &maps.m[M_KI4R], 0, y, kfull);
            }
            if (!claim(w, u, 1)) { timed_out = true; break; }
            const uint32_t va = sa + 4096u;
            mbar_arrive_expect_tx(vfull, half);
            if (fmt == IAK_FMT_F16) {
              if constexpr (D == 128 && kF16OneBox) tma_load_2d(va, &maps.m[M_VF16], 0, pid * kPS * 2, vfull);
              else tma_load_2d(va, &maps.m[M_VF16], 0, pid * kPS, vfull);
            } else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) {
              tma_load_2d(va, &maps.m[fmt == IAK_FMT_FP8 ? M_VFP8 : M_VI8], 0, pid * (kPS * D / 128), vfull);
            } else {
              const int y = pid * (kPS * D / 256);
              tma_load_2d(va, &maps.m[M_VI4], 0, y, vfull);
              if (fmt == IAK_FMT_INT4R) tma_load_2d(va + kResOff, &maps.m[M_VI4R], 0, y, vfull);
            }
            continue;
          }
          if (ns == 2 && u % SPW == SPW - 1) {
            if (!claim(w, u)) { timed_out = true; break; }
            mbar_arrive(full_bar(w * SPW + u % SPW));   // skipped slot
            ++u;
          }
          if (!claim(w, u) || (ns == 2 && !claim(w, u + 1))) { timed_out = true; break; }
          const int st = w * SPW + u % SPW;
          cnt[t] = u + ns;
          const uint32_t full = full_bar(st);
          if (ns == 2) mbar_arrive(full_bar(st + 1));     // the second slot carries no barrier bytes
          const uint32_t sa = smem_u32(smem + SL::stages + st * SB);
          const uint32_t vo = v_off(fmt);
          uint32_t bytes;
          if (fmt == IAK_FMT_F16) bytes = 2 * kPS * D * 2;
          else if (fmt == IAK_FMT_INT4) bytes = 2 * kPS * D / 2;
          else bytes = 2 * kPS * D;   // FP8, INT8, INT4R (two half-size planes)
          if (GROUP && fmt != IAK_FMT_F16) bytes += (fmt == IAK_FMT_INT4R ? 4 : 2) * NG * 4;
          mbar_arrive_expect_tx(full, bytes);
          if (fmt == IAK_FMT_F16) {
            if constexpr (D == 128 && kF16OneBox) {
              tma_load_2d(sa, &maps.m[M_KF16], 0, pid * kPS * 2, full);
              tma_load_2d(sa + vo, &maps.m[M_VF16], 0, pid * kPS * 2, full);
            } else {
              tma_load_2d(sa, &maps.m[M_KF16], 0, pid * kPS, full);
              tma_load_2d(sa + vo, &maps.m[M_VF16], 0, pid * kPS, full);
            }
          } else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) {
            const int y = pid * (kPS * D / 128);   // 128-byte lines of 8-bit token rows
            const int mk = fmt == IAK_FMT_FP8 ? M_KFP8 : M_KI8;
            tma_load_2d(sa, &maps.m[mk], 0, y, full);
            tma_load_2d(sa + vo, &maps.m[mk + 1], 0, y, full);
          } else {
            const int y = pid * (kPS * D / 256);   // 128-byte lines of packed int4 token rows
            tma_load_2d(sa, &maps.m[M_KI4], 0, y, full);
            tma_load_2d(sa + vo, &maps.m[M_VI4], 0, y, full);
            if (fmt == IAK_FMT_INT4R) {
              tma_load_2d(sa + kResOff, &maps.m[M_KI4R], 0, y, full);
              tma_load_2d(sa + vo + kResOff, &maps.m[M_VI4R], 0, y, full);
            }
          }
          if (GROUP && fmt != IAK_FMT_F16) {
            const uint32_t sc = smem_u32(stage_scales(st));
            bulk_load(sc, p.k_scale + static_cast<int64_t>(pid) * NG, NG * 4, full);
            bulk_load(sc + 16, p.v_scale + static_cast<int64_t>(pid) * NG, NG * 4, full);
            if (fmt == IAK_FMT_INT4R) {
              bulk_load(sc + 32, p.k_rscale + static_cast<int64_t>(pid) * NG, NG * 4, full);
              bulk_load(sc + 48, p.v_rscale + static_cast<int64_t>(pid) * NG, NG * 4, full);
            }
          }
        }
      }
      timed_out = __any_sync(0xffffffffu, timed_out);
    }
    // drain: the last round this lane armed on each slot of the sub-rings it feeds
    if (lane < LPW)
#pragma unroll
      for (int t = 0; t < kFed; ++t) {
        const int w = pl + t * LPW;
        for (int u = max(0, cnt[t] - SPW); u < cnt[t]; ++u)
          for (int part = 0; part < (SKV ? 2 : 1); ++part)
            if (!mbar_wait(full_bar(SKV ? 2 * (w * SPW + u % SPW) + part : w * SPW + u % SPW), (u / SPW) & 1,
                           kWaitCycles))
              timed_out = true;
      }
    timed_out = __any_sync(0xffffffffu, timed_out);
  } else {
    // -------------------------------------------------------------- consumers
    asm volatile("griddepcontrol.wait;" ::: "memory");   // the counters the preparation kernel zeroed
    const int cw = warp - kFirstConsumerWarp;
    const float qk_log2 = p.sm_scale * 1.4426950408889634f;
    int cnt = 0;        // slots of this warp's sub-ring used so far (mirrors the producer lane)
    for (int k = 0, item = blockIdx.x; item < n_items; ++k, item += gridDim.x) {
      const int buf = k & 1;
      const char* ib = item_buf(buf);
      if (!wait_all(ifull_bar(buf), (k >> 1) & 1)) {
        timed_out = true;
        break;
      }
      const int* meta = reinterpret_cast<const int*>(ib + ItemLayout::meta);
      const int n_valid = meta[0];
      const float* scal_s = reinterpret_cast<const float*>(ib + ItemLayout::scal);
      const uint8_t* fmt_s = reinterpret_cast<const uint8_t*>(ib + ItemLayout::fmt);
      const uint4* qfrag = reinterpret_cast<const uint4*>(ib + kQFrag);
      const uint4* qi8 = reinterpret_cast<const uint4*>(ib + kQI8);
      const uint4* qi4 = reinterpret_cast<const uint4*>(ib + kQI4);
      const float* qsc = reinterpret_cast<const float*>(ib + kQSc);
      float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
      float oacc[KT][4];
#pragma unroll
      for (int mt = 0; mt < KT; ++mt) oacc[mt][0] = oacc[mt][1] = oacc[mt][2] = oacc[mt][3] = 0.f;
      // Pages i = cw (mod 4) of the item, from this warp's sub-ring, in order; a skipped slot
      // (a two-slot page that would wrap) is waited for and released like a page.
      for (int i = cw; i < n_valid; i += kConsumerWarps) {
        const int fmt = fmt_s[i];
        const int ns = page_slots(fmt);
        int u = cnt;
        if (ns == 2 && u % SPW == SPW - 1) {
          const int sk = cw * SPW + SPW - 1;
          if (!wait_all(full_bar(sk), (u / SPW) & 1)) {
            timed_out = true;
            break;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(empty_bar(sk));
          ++u;
        }
        const int st = cw * SPW + u % SPW;
        cnt = u + ns;
        // the page's K (page-scaled pools: the slot's K half; its V half is waited for
        // before P.V), or the whole page
        if (!wait_all(full_bar(SKV ? 2 * st : st), (u / SPW) & 1) ||
            (ns == 2 && !wait_all(full_bar(st + 1), ((u + 1) / SPW) & 1))) {
          timed_out = true;
          break;
        }
        const uint32_t vo = v_off(fmt);
        const char* pg = smem + SL::stages + st * SB;
        const uint32_t pg_u32 = smem_u32(pg);
        const float* gsc = reinterpret_cast<const float*>(stage_scales(st));
        // ---------------- S^T = K Q^T
        // accumulator of k-step kk: its 32-channel group (group scales) or its
        // parity (two independent MMA chains per page)
        constexpr int NA = GROUP ? NG : 2;
        float sacc[NA][4];
  #pragma unroll
        for (int g = 0; g < NA; ++g)
  #pragma unroll
          for (int e = 0; e < 4; ++e) sacc[g][e] = 0.f;
        if (fmt == IAK_FMT_F16) {
  #pragma unroll
          for (int kk = 0; kk < KT; ++kk) {
            uint32_t a[4];
            k_frag_f16<D>(pg_u32, lane, kk, a);
            const uint4 qf = qfrag[kk * 32 + lane];
            mma16816(sacc[GROUP ? kk / 2 : (kk & 1)], a[0], a[1], a[2], a[3], qf.x, qf.y);
          }
        } else if (fmt == IAK_FMT_FP8) {
  #pragma unroll
          for (int kk = 0; kk < KT; kk += 2) {
            uint32_t x[4];
            ldsm_rows(pg_u32, D, lane, kk, x);
  #pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t a[4];
              k_frag_8bit_from(x[2 * h], x[2 * h + 1], true, a);
              const uint4 qf = qfrag[(kk + h) * 32 + lane];
              mma16816(sacc[GROUP ? (kk + h) / 2 : h], a[0], a[1], a[2], a[3], qf.z, qf.w);
            }
          }
        }
        // ---------------- scores (times the K scale; INT8 / INT4 on the integer tensor path)
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        const float s2a = qsc[8 + 2 * c], s2b = qsc[8 + 2 * c + 1];
        if (fmt == IAK_FMT_F16 || fmt == IAK_FMT_FP8) {
          // fp16 fragments carry q / 2^fe: the factor 2^fe of each query column comes back here
          const float qfa = qsc[kQScF + 2 * c], qfb = qsc[kQScF + 2 * c + 1];
          if (!GROUP) {
            const float ks = scal_s[i];
            const float ka = ks * qfa, kb = ks * qfb;
  #pragma unroll
            for (int e = 0; e < 4; ++e) sc[e] = (sacc[0][e] + sacc[1][e]) * ((e & 1) ? kb : ka);
          } else {
            const bool q = fmt != IAK_FMT_F16;
  #pragma unroll
            for (int g = 0; g < NA; ++g) {
              const float ks = q ? gsc[g] : 1.f;
  #pragma unroll
              for (int e = 0; e < 4; ++e) sc[e] = fmaf(sacc[g][e], ks, sc[e]);
            }
  #pragma unroll
            for (int e = 0; e < 4; ++e) sc[e] *= (e & 1) ? qfb : qfa;
          }
        } else if (fmt == IAK_FMT_INT8) {
          // q = s2 * (256 * i1 + i2): one int32 combine and one scale per score
          int i1[4] = {0, 0, 0, 0}, i2[4] = {0, 0, 0, 0};
  #pragma unroll
          for (int j = 0; j < D / 32; ++j) {
            uint32_t x[4];
            ldsm_rows(pg_u32, D, lane, 2 * j, x);
            const uint4 qi = qi8[j * 32 + lane];
            imma_s8(i1, x, qi.x, qi.y);
            imma_s8(i2, x, qi.z, qi.w);
            if (GROUP) {
              const float ks = gsc[j];
  #pragma unroll
              for (int e = 0; e < 4; ++e) {
                sc[e] = fmaf(ks, static_cast<float>(i1[e] * 256 + i2[e]), sc[e]);
                i1[e] = i2[e] = 0;
              }
            }
          }
          if (GROUP) {
  #pragma unroll
            for (int e = 0; e < 4; ++e) sc[e] *= (e & 1) ? s2b : s2a;
          } else {
            const float ks = scal_s[i];
            const float ka = ks * s2a, kb = ks * s2b;
  #pragma unroll
            for (int e = 0; e < 4; ++e) sc[e] = static_cast<float>(i1[e] * 256 + i2[e]) * ((e & 1) ? kb : ka);
          }
        } else {
          // INT4 / INT4R: nibbles -> bytes (code + 8) on the u8 x s8 path; the
          // accumulators start at -8 * sum(q term) of their channels, so the +8
          // offset cancels exactly in the integer sums
          const int nplanes = fmt == IAK_FMT_INT4R ? 2 : 1;
          const int2* qbi = reinterpret_cast<const int2*>(qsc);   // [word / 2]
          for (int pl = 0; pl < nplanes; ++pl) {
            int i1[4], i2[4];
            if (!GROUP) {
              const int2 b1 = qbi[(kQB1T >> 1) + c], b2 = qbi[(kQB2T >> 1) + c];
              i1[0] = i1[2] = b1.x; i1[1] = i1[3] = b1.y;
              i2[0] = i2[2] = b2.x; i2[1] = i2[3] = b2.y;
            }
  #pragma unroll
            for (int jj = 0; jj < D / 64; ++jj) {
              uint32_t x[4];
              ldsm_rows(pg_u32 + pl * kResOff, D / 2, lane, 2 * jj, x);
  #pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int j = 2 * jj + h;
                const uint32_t a[4] = {x[2 * h] & 0x0F0F0F0Fu, x[2 * h + 1] & 0x0F0F0F0Fu,
                                       (x[2 * h] >> 4) & 0x0F0F0F0Fu, (x[2 * h + 1] >> 4) & 0x0F0F0F0Fu};
                const uint4 qi = qi4[j * 32 + lane];
                if (GROUP) {
                  const int2 b1 = qbi[((kQB1 + 8 * j) >> 1) + c], b2 = qbi[((kQB2 + 8 * j) >> 1) + c];
                  i1[0] = i1[2] = b1.x; i1[1] = i1[3] = b1.y;
                  i2[0] = i2[2] = b2.x; i2[1] = i2[3] = b2.y;
                }
                imma_u8(i1, a, qi.x, qi.y);
                imma_u8(i2, a, qi.z, qi.w);
                if (GROUP) {
                  const float ks = gsc[8 * pl + j];
  #pragma unroll
                  for (int e = 0; e < 4; ++e) sc[e] = fmaf(ks, static_cast<float>(i1[e] * 256 + i2[e]), sc[e]);
                }
              }
            }
            if (!GROUP) {
              const float ks = scal_s[(pl == 0 ? 0 : 2) * kChunkMax + i];
  #pragma unroll
              for (int e = 0; e < 4; ++e) sc[e] = fmaf(ks, static_cast<float>(i1[e] * 256 + i2[e]), sc[e]);
            }
          }
  #pragma unroll
          for (int e = 0; e < 4; ++e) sc[e] *= (e & 1) ? s2b : s2a;
        }
  #pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] *= qk_log2;
        if constexpr (SKV) {
          // the page's K half is read: free it for the page two ahead
          __syncwarp();
          if (lane == 0) mbar_arrive(empty_bar(2 * st));
        }
        // ---------------- online softmax (log2 domain)
        float pm0 = fmaxf(sc[0], sc[2]), pm1 = fmaxf(sc[1], sc[3]);
        // Lazy rescaling: the running max only moves (and O, l are rescaled)
        // when some query's page max exceeds it by more than kLazyLog2; until
        // then p <= 2^kLazyLog2, far inside fp16 / fp32 range.  Warp-uniform.
        // A lane's own scores decide whether any column max crossed the bound,
        // so the column maxima are only reduced on the (rare) rescaling pages.
        if (__any_sync(0xffffffffu, pm0 > m_run[0] + kLazyLog2 || pm1 > m_run[1] + kLazyLog2)) {
  #pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            pm0 = fmaxf(pm0, __shfl_xor_sync(0xffffffffu, pm0, off));
            pm1 = fmaxf(pm1, __shfl_xor_sync(0xffffffffu, pm1, off));
          }
          const float mn0 = fmaxf(m_run[0], pm0), mn1 = fmaxf(m_run[1], pm1);
          const float al0 = exp2f(m_run[0] - mn0), al1 = exp2f(m_run[1] - mn1);
          m_run[0] = mn0; m_run[1] = mn1;
          l_run[0] *= al0; l_run[1] *= al1;
  #pragma unroll
          for (int mt = 0; mt < KT; ++mt) {
            oacc[mt][0] *= al0; oacc[mt][1] *= al1; oacc[mt][2] *= al0; oacc[mt][3] *= al1;
          }
        }
        // hardware exp2 (arguments <= kLazyLog2; results below 2^-126 flush to 0, far below fp16's range)
        const float p0 = ex2_approx(sc[0] - m_run[0]), p1 = ex2_approx(sc[1] - m_run[1]);
        const float p2 = ex2_approx(sc[2] - m_run[0]), p3 = ex2_approx(sc[3] - m_run[1]);
        l_run[0] += p0 + p2;
        l_run[1] += p1 + p3;
        // ---------------- O^T += V^T P^T
        if constexpr (SKV) {
          if (!wait_all(full_bar(2 * st + 1), (u / SPW) & 1)) {
            timed_out = true;
            break;
          }
        }
        uint32_t vh[2][D / 64][8];
        if (!GROUP) {
          // per-page V scale folded into P
          const float vs = scal_s[kChunkMax + i];
          const uint32_t pb0 = movm_t(pack_f16x2(p0 * vs, p1 * vs));
          const uint32_t pb1 = movm_t(pack_f16x2(p2 * vs, p3 * vs));
          if (fmt == IAK_FMT_F16) v_table_f16<D>(pg + vo, r, c, vh);
          else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) v_table_8bit<D>(pg + vo, r, c, fmt == IAK_FMT_FP8, vh);
          else v_table_int4<D>(pg + vo, r, c, vh);
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
            v_table_int4<D>(pg + vo + kResOff, r, c, vh);
  #pragma unroll
            for (int mt = 0; mt < KT; ++mt) {
              uint32_t a0, a1, a2, a3;
              pv_afrag<D>(vh, mt, a0, a1, a2, a3);
              mma16816(oacc[mt], a0, a1, a2, a3, rb0, rb1);
            }
          }
        } else {
          // per-32-channel V scales.  The page's largest V scale rides on P (as a page
          // scale does); each group's ratio to it (<= 1) multiplies the V fragments in
          // fp16.  Rows r of the lane's PV fragments are group gA, rows r + 8 group gB.
          const int gA = pv_word<D>(r, 0) >> 2, gB = pv_word<D>(r, D / 64 - 1) >> 2;
          const bool q = fmt != IAK_FMT_F16;
          if constexpr (D == 128) {
            if (fmt == IAK_FMT_INT4R) {
              // both planes in one table, one P.V (the scales over the largest of the page's
              // base and residual V scales, so every ratio is at most 1)
              const float* vb = gsc + 4;
              const float* vr = gsc + 12;
              float vmax = fmaxf(vb[0], vr[0]);
  #pragma unroll
              for (int g = 1; g < NG; ++g) vmax = fmaxf(vmax, fmaxf(vb[g], vr[g]));
              const float inv = __frcp_rn(vmax);
              v_table_int4r_group(pg + vo, pg + vo + kResOff, r, c, pack_f16x2(vb[gA] * inv, vb[gA] * inv),
                                  pack_f16x2(vb[gB] * inv, vb[gB] * inv), pack_f16x2(vr[gA] * inv, vr[gA] * inv),
                                  pack_f16x2(vr[gB] * inv, vr[gB] * inv), vh);
              const uint32_t pb0 = movm_t(pack_f16x2(p0 * vmax, p1 * vmax));
              const uint32_t pb1 = movm_t(pack_f16x2(p2 * vmax, p3 * vmax));
  #pragma unroll
              for (int mt = 0; mt < KT; ++mt) {
                uint32_t a0, a1, a2, a3;
                pv_afrag<D>(vh, mt, a0, a1, a2, a3);
                mma16816(oacc[mt], a0, a1, a2, a3, pb0, pb1);
              }
            }
          }
          const int nplanes = (D == 128 && fmt == IAK_FMT_INT4R) ? 0 : 1;
          for (int pl = 0; pl < nplanes; ++pl) {
            const char* vt = pg + vo + pl * kResOff;
            if (fmt == IAK_FMT_F16) v_table_f16<D>(vt, r, c, vh);
            else if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) v_table_8bit<D>(vt, r, c, fmt == IAK_FMT_FP8, vh);
            else v_table_int4<D>(vt, r, c, vh);
            float vmax = 1.f;
            if (q) {
              const float* vsc = gsc + (pl == 0 ? 4 : 12);
              vmax = vsc[0];
  #pragma unroll
              for (int g = 1; g < NG; ++g) vmax = fmaxf(vmax, vsc[g]);
              const float inv = __frcp_rn(vmax);
              const uint32_t rA = pack_f16x2(vsc[gA] * inv, vsc[gA] * inv);
              const uint32_t rB = pack_f16x2(vsc[gB] * inv, vsc[gB] * inv);
  #pragma unroll
              for (int tp = 0; tp < 2; ++tp)
  #pragma unroll
                for (int n = 0; n < 8; ++n) {
                  vh[tp][0][n] = hmul2(vh[tp][0][n], rA);
                  vh[tp][D / 64 - 1][n] = hmul2(vh[tp][D / 64 - 1][n], rB);
                }
            }
            const uint32_t pb0 = movm_t(pack_f16x2(p0 * vmax, p1 * vmax));
            const uint32_t pb1 = movm_t(pack_f16x2(p2 * vmax, p3 * vmax));
  #pragma unroll
            for (int mt = 0; mt < KT; ++mt) {
              uint32_t a0, a1, a2, a3;
              pv_afrag<D>(vh, mt, a0, a1, a2, a3);
              mma16816(oacc[mt], a0, a1, a2, a3, pb0, pb1);
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          if constexpr (SKV) {
            mbar_arrive(empty_bar(2 * st + 1));
          } else {
            mbar_arrive(empty_bar(st));
            if (ns == 2) mbar_arrive(empty_bar(st + 1));
          }
        }
      }
      if (timed_out) break;
      // ---- this warp's partial of the item, into the CTA's merge area once the preparer
      // has merged the previous item out of it
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], off);
        l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], off);
      }
      if (k >= 1 && !wait_all(mfree_bar, (k - 1) & 1)) {
        timed_out = true;
        break;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int g = 2 * c + h;
        if (g < p.G) {
          float* mr = merge_area + (cw * 8 + g) * kMergeRow;
          if (r == 0) {
            mr[128] = l_run[h] > 0.f ? m_run[h] * 0.6931471805599453f : -INFINITY;  // natural-log max
            mr[129] = l_run[h];
          }
#pragma unroll
          for (int mt = 0; mt < KT; ++mt) {
            mr[pv_channel<D>(mt, r)] = oacc[mt][h];
            mr[pv_channel<D>(mt, r + 8)] = oacc[mt][2 + h];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(iempty_bar(buf));
    }
  }
  if (timed_out && lane == 0) {
    atomicAdd(&g_decode_timeouts, 1u);
    if (p.status) atomicOr(p.status, static_cast<unsigned int>(IAK_STATUS_DECODE_TIMEOUT));
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
  if (kind == 0 && D == 128 && kF16OneBox) {
    // 256-byte token rows viewed as two 128-byte half-rows; one box = one page
    dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; eb = 2; inner = 64; rows = tokens * 2; box_rows = 2 * kPS;
  } else if (kind == 0) {
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

int read_decode_timeouts(unsigned int* value, bool reset) {
  unsigned int v = 0;
  int st = check_cuda(cudaMemcpyFromSymbol(&v, g_decode_timeouts, sizeof(v)), "read decode timeouts");
  if (st) return st;
  if (reset && v) {
    const unsigned int zero = 0;
    st = check_cuda(cudaMemcpyToSymbol(g_decode_timeouts, &zero, sizeof(zero)), "reset decode timeouts");
    if (st) return st;
  }
  *value = v;
  return IAK_OK;
}

bool mma_shape_eligible(const DecodeParams& p) {
  if (p.PS != kPS || (p.D != 64 && p.D != 128)) return false;
  if (p.q_dtype != IAK_DT_F16 && p.q_dtype != IAK_DT_BF16) return false;
  if (p.scale_mode == IAK_SCALE_CHANNEL) return false;
  if (p.scale_mode == IAK_SCALE_GROUP32 && p.D != 128) return false;
  return true;
}

template <int D, bool GROUP>
static int launch_persistent(const DecodeParams& p, const TmaMaps& maps, int n_items, cudaStream_t s) {
  const size_t smem = SmemLayout::total + 1024;
  auto kern = decode_mma_kernel<D, GROUP>;
  // the smem attribute and occupancy are per (device, instantiation): look them up once
  static std::mutex mu;
  static int per_sm_cache[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return check_cuda(err, "cudaGetDevice");
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    per_sm = (dev >= 0 && dev < 64) ? per_sm_cache[dev] : 0;
    if (per_sm == 0) {
      err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return check_cuda(err, "decode_mma smem attribute");
      err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
      if (err != cudaSuccess) return check_cuda(err, "decode_mma occupancy");
      if (per_sm <= 0) return fail(IAK_ERR_UNSUPPORTED, "decode_mma does not fit on an SM");
      if (dev >= 0 && dev < 64) per_sm_cache[dev] = per_sm;
    }
  }
  const int ctas = std::max(1, std::min(n_items, per_sm * device_sm_count()));
  decode_prep_kernel<D><<<p.B * p.Ht, 256, 0, s>>>(p, p.ws_qtab);
  err = cudaGetLastError();
  if (err != cudaSuccess) return check_cuda(err, "decode_prep launch");
  // Programmatic dependent launch: the decode CTAs start while the query tables are
  // still being built, stream their first pages, and wait (griddepcontrol.wait) only
  // before they read a query table or a merge counter.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  kernel_timer_begin(s);
  err = cudaLaunchKernelEx(&cfg, kern, p, maps, static_cast<const char*>(p.ws_qtab), n_items);
  kernel_timer_end(s);
  return check_cuda(err, "decode_mma launch");
}

int launch_decode_mma(const DecodeParams& p, const iak_page_pools& P, cudaStream_t s) {
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
  if (!p.ws_qtab) return fail(IAK_ERR_WORKSPACE, "tensor-core decode needs a workspace");
  const int n_items = p.B * p.Ht * p.num_splits;
  if (p.D == 128 && p.scale_mode == IAK_SCALE_GROUP32) return launch_persistent<128, true>(p, maps, n_items, s);
  if (p.D == 128) return launch_persistent<128, false>(p, maps, n_items, s);
  return launch_persistent<64, false>(p, maps, n_items, s);
}

}  // namespace iak
