// Tensor-core (tcgen05 / TMEM) MLA decode for the absorbed DeepSeek-V2 shape:
// d_qk = 576 (512 latent + 64 rope channels), d_v = 512, up to 128 query
// heads per sequence, latent pages of a multiple of 16 tokens, dense BF16 /
// F16 or FP8-e4m3 (per-page scale) pages.
//
// One CTA = one work item (sequence b, page range `split`, value half h):
//   * the 128 head rows are the M = 128 rows of every MMA; Q (f16, K-major,
//     128-byte swizzle) stays in shared memory for the whole item;
//   * 16-token page tiles stream through a 4-stage TMA ring; FP8 and BF16
//     tiles are converted to f16 in place by a converter warpgroup (FP8 via
//     cvt.e4m3x2, exact; BF16 via f32, exact inside the f16 range);
//   * S = Q . C^T (M=128, N=16, K=576: 36 tcgen05.mma, f32 in TMEM, three
//     S buffers); the softmax warpgroup owns one TMEM lane (= one head) per
//     thread, so the online softmax needs no cross-thread reduction;
//     P (f16) is written back into the S columns and is the TMEM A operand
//     of O_h += P . C[:, h*256 : h*256+256] (M=128, N=256, K=16, the tile
//     read MN-major from the same shared-memory bytes), O_h in TMEM;
//   * FP8 tiles stay codes: the page scale multiplies the scores and P
//     (so O accumulates code x scale x weight); l sums unscaled weights;
//   * the O accumulator is rescaled lazily (only when a row max grows by
//     more than 2^8), in TMEM.
// TMEM: O_h 256 columns + 3 x 16 S/P columns (512 allocated: one CTA per SM).
// The two value halves of a (b, split) recompute S: TMEM cannot hold
// 128 x 512 fp32 next to S.
//
// Reference: triton_mla_decode.py:155-186 (_mla_decode_cpu) per query row,
// restated per head; rows without pages give 0.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "mla_internal.cuh"

namespace iak {

__device__ unsigned int g_mla_timeouts = 0;

namespace {

constexpr int kDqk = 576, kDv = 512, kHalf = kDv / 2, kRows = 128, kTile = 16;
constexpr int kStages = 4, kSBuf = 3;
constexpr int kKBlocks = kDqk / 64;                 // 128-byte swizzle atoms along the channels
constexpr int kKbQ = kRows * 128;                   // bytes of one Q k-block (128 rows x 128 B)
constexpr int kKbTile = kTile * 128;                // bytes of one tile k-block (16 rows x 128 B)
constexpr int kQBytes = kKBlocks * kKbQ;            // 147456
constexpr int kTileBytes = kKBlocks * kKbTile;      // 18432
constexpr int kRawOff = kTileBytes / 2;             // an FP8 tile lands in the upper half
constexpr int kFp8Part = 192;                       // bytes per row of one FP8 TMA box (3 boxes per row)
constexpr int kMaxItemPages = 512;
constexpr int kThreads = 320;                       // softmax wg | converter wg | TMA warp | MMA warp
constexpr int kConvWarp0 = 4, kTmaWarp = 8, kMmaWarp = 9;
constexpr int kOCol = 0, kSCol = kHalf, kTmemCols = 512;
constexpr long long kWaitCycles = 4000000000LL;     // ~2 s at boost clock, then give up
constexpr float kLazyLog2 = 8.f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum {
  B_FULL = 0,                    // TMA -> converters (tx bytes)
  B_CONV = B_FULL + kStages,     // converters -> MMA (f16 tile ready)
  B_EMPTY = B_CONV + kStages,    // MMA commit -> TMA (tile no longer read)
  B_SFULL = B_EMPTY + kStages,   // MMA commit -> softmax (S ready)
  B_PFULL = B_SFULL + kSBuf,     // softmax -> MMA (P written, O rescaled)
  B_PVDONE = B_PFULL + kSBuf,    // MMA commit -> softmax / MMA (PV done: O current, S/P buffer free)
  B_DONE = B_PVDONE + kSBuf,     // MMA commit -> MMA (all MMAs retired)
  B_CREAD,                       // converters: every FP8 code of the tile read (in-place conversion)
  B_COUNT
};

struct Smem {
  static constexpr int q = 0;
  static constexpr int tiles = kQBytes;
  static constexpr int pid = tiles + kStages * kTileBytes;
  static constexpr int pfmt = pid + kMaxItemPages * 4;
  static constexpr int bars = pfmt + kMaxItemPages;
  static constexpr int tmem = bars + B_COUNT * 8;
  static constexpr int nvalid = tmem + 4;
  static constexpr int total = nvalid + 12;
};
static_assert(Smem::tiles % 1024 == 0 && kTileBytes % 1024 == 0, "swizzle atoms need 1024-byte alignment");
static_assert(Smem::bars % 8 == 0, "mbarriers need 8-byte alignment");

// ----------------------------------------------------------------- PTX ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
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
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 format: version 1 at bit 46).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: f16 A and B, f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (static_cast<uint32_t>(a_mn_major) << 15) | (static_cast<uint32_t>(b_mn_major) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t h) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(h));
  return r;
}
// two bf16 (low half = first element) -> two f16, exact inside the f16 range
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  const __half2 h = __floats2half2_rn(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ int mla_fmt(const MlaParams& p, int64_t pid) {
  if (!p.tags) return IAK_MLA_DENSE;
  const int tag = p.tag_bytes == 1 ? static_cast<int>(static_cast<const uint8_t*>(p.tags)[pid])
                                   : static_cast<const int32_t*>(p.tags)[pid];
  return (tag >= 0 && tag < 16) ? p.tag_map[tag] : p.tag_default;
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128-byte-swizzled atom column.
__device__ __forceinline__ uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }

// ---------------------------------------------------------------- kernel ---
__global__ void __launch_bounds__(kThreads, 1)
    mla_tc_kernel(const MlaParams p, const __grid_constant__ CUtensorMap dmap, const __grid_constant__ CUtensorMap fmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (sbase - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int S = p.num_splits;
  const int half = blockIdx.x & 1;
  const int split = (blockIdx.x >> 1) % S;
  const int b = (blockIdx.x >> 1) / S;

  int32_t* s_pid = reinterpret_cast<int32_t*>(sm + Smem::pid);
  uint8_t* s_fmt = sm + Smem::pfmt;
  volatile uint32_t* s_tmem = reinterpret_cast<volatile uint32_t*>(sm + Smem::tmem);
  volatile int* s_nvalid = reinterpret_cast<volatile int*>(sm + Smem::nvalid);
  const uint32_t q_s = sbase + Smem::q, tiles_s = sbase + Smem::tiles;
  auto bar = [&](int i) -> uint32_t { return sbase + Smem::bars + 8u * static_cast<uint32_t>(i); };

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_FULL + s), 1);
      mbar_init(bar(B_CONV + s), 128);
      mbar_init(bar(B_EMPTY + s), 1);
    }
    for (int k = 0; k < kSBuf; ++k) {
      mbar_init(bar(B_SFULL + k), 1);
      mbar_init(bar(B_PFULL + k), 128);
      mbar_init(bar(B_PVDONE + k), 1);
    }
    mbar_init(bar(B_DONE), 1);
    mbar_init(bar(B_CREAD), 128);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + Smem::tmem),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kTmaWarp) {
    // compact this item's slice of the page table: valid ids of dense / FP8 pages, in order
    const int n_tab = p.pc ? min(max(p.pc[b], 0), p.W) : p.W;
    const int lo = split * p.pages_per_split, hi = min(n_tab, lo + p.pages_per_split);
    const int32_t* table = p.pt + static_cast<int64_t>(b) * p.pt_sb;
    int cnt = 0;
    for (int j0 = lo; j0 < hi; j0 += 32) {
      const int j = j0 + lane;
      int pid = -1, fmt = IAK_MLA_SKIP;
      if (j < hi) {
        pid = table[j];
        if (pid >= 0 && pid < p.num_pages) fmt = mla_fmt(p, pid);
      }
      const bool ok = fmt == IAK_MLA_DENSE || fmt == IAK_MLA_FP8;
      const unsigned m = __ballot_sync(0xffffffffu, ok);
      if (ok) {
        const int r = cnt + __popc(m & ((1u << lane) - 1u));
        s_pid[r] = pid;
        s_fmt[r] = static_cast<uint8_t>(fmt);
      }
      cnt += __popc(m);
    }
    if (lane == 0) *s_nvalid = cnt;
  }
  if (warp < kTmaWarp) {
    // Q rows (heads) as f16 in the K-major 128-byte-swizzled layout; rows >= H are zero
    const bool bf = p.q_dtype == IAK_DT_BF16;
    for (int u = tid; u < kRows * (kDqk / 8); u += 256) {
      const int r = u / (kDqk / 8), c8 = u % (kDqk / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < p.H) {
        const uint4 x = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.q) + b * p.q_sb + r * p.q_sh +
                                                        c8 * 8);
        v = bf ? make_uint4(bf16x2_to_f16x2(x.x), bf16x2_to_f16x2(x.y), bf16x2_to_f16x2(x.z), bf16x2_to_f16x2(x.w)) : x;
      }
      *reinterpret_cast<uint4*>(sm + Smem::q + (c8 >> 3) * kKbQ + swz(r, c8 & 7)) = v;
    }
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_valid = *s_nvalid;
  const int tpp = p.PS / kTile;
  const int T = n_valid * tpp;
  bool timed_out = false;

  if (warp == kTmaWarp) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      for (int j = 0; j < T && !timed_out; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(bar(B_EMPTY + s), ((j / kStages) - 1) & 1)) { timed_out = true; break; }
        const int pg = j / tpp, sub = j % tpp;
        const int pid = s_pid[pg];
        const int y = pid * p.PS + sub * kTile;
        const uint32_t dst = tiles_s + s * kTileBytes;
        if (s_fmt[pg] == IAK_MLA_FP8) {
          mbar_arrive_expect_tx(bar(B_FULL + s), kTile * kDqk);
#pragma unroll
          for (int part = 0; part < kDqk / kFp8Part; ++part)
            tma_load_2d(dst + kRawOff + part * kTile * kFp8Part, &fmap, part * kFp8Part, y, bar(B_FULL + s));
        } else {
          mbar_arrive_expect_tx(bar(B_FULL + s), kTileBytes);
#pragma unroll
          for (int kb = 0; kb < kKBlocks; ++kb) tma_load_2d(dst + kb * kKbTile, &dmap, kb * 64, y, bar(B_FULL + s));
        }
      }
    }
  } else if (warp >= kConvWarp0 && warp < kTmaWarp) {
    // ---------------------------------------------------------------- converters
    const int ct = tid - kConvWarp0 * 32;
    const bool dense_bf16 = p.dense_dtype == IAK_DT_BF16;
    int n_fp8 = 0;   // FP8 tiles converted so far (phase of B_CREAD)
    for (int j = 0; j < T && !timed_out; ++j) {
      const int s = j % kStages;
      if (!mbar_wait(bar(B_FULL + s), (j / kStages) & 1)) { timed_out = true; break; }
      const int fmt = s_fmt[j / tpp];
      uint8_t* tile = sm + Smem::tiles + s * kTileBytes;
      if (fmt == IAK_MLA_FP8) {
        // 1152 units of 8 codes (one 16-byte f16 chunk each); read all, then write (in place)
        uint2 x[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) {
          const int u = ct + 128 * i, r = u / 72, c8 = u % 72;
          const int e = c8 * 8;
          x[i] = *reinterpret_cast<const uint2*>(tile + kRawOff + (e / kFp8Part) * (kTile * kFp8Part) +
                                                 r * kFp8Part + e % kFp8Part);
        }
        // every converter has its codes in registers before any f16 chunk overwrites them
        mbar_arrive(bar(B_CREAD));
        if (!mbar_wait(bar(B_CREAD), n_fp8 & 1)) { timed_out = true; break; }
        ++n_fp8;
#pragma unroll
        for (int i = 0; i < 9; ++i) {
          const int u = ct + 128 * i, r = u / 72, c8 = u % 72;
          uint4 v;
          v.x = e4m3x2_to_f16x2(static_cast<uint16_t>(x[i].x & 0xFFFFu));
          v.y = e4m3x2_to_f16x2(static_cast<uint16_t>(x[i].x >> 16));
          v.z = e4m3x2_to_f16x2(static_cast<uint16_t>(x[i].y & 0xFFFFu));
          v.w = e4m3x2_to_f16x2(static_cast<uint16_t>(x[i].y >> 16));
          *reinterpret_cast<uint4*>(tile + (c8 >> 3) * kKbTile + swz(r, c8 & 7)) = v;
        }
      } else if (dense_bf16) {
#pragma unroll
        for (int i = 0; i < 9; ++i) {
          uint4* c = reinterpret_cast<uint4*>(tile + 16 * (ct + 128 * i));
          uint4 v = *c;
          v = make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z), bf16x2_to_f16x2(v.w));
          *c = v;
        }
      }
      fence_proxy_async();
      mbar_arrive(bar(B_CONV + s));
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(kRows, kTile, 0, 0);   // S = Q . C^T
      constexpr uint32_t kIdPV = idesc_f16(kRows, kHalf, 0, 1);  // O += P . C (C read MN-major)
      auto issue_s = [&](int j) -> bool {
        const int s = j % kStages, k = j % kSBuf;
        if (!mbar_wait(bar(B_CONV + s), (j / kStages) & 1)) return false;
        if (j >= kSBuf && !mbar_wait(bar(B_PVDONE + k), ((j / kSBuf) - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t d = tmem + kSCol + k * kTile;
        const uint32_t tile = tiles_s + s * kTileBytes;
#pragma unroll 4
        for (int ks = 0; ks < kDqk / 16; ++ks) {
          const uint32_t off = static_cast<uint32_t>(ks & 3) << 5;   // 16 channels = 32 bytes inside the atom
          const uint64_t a = sw128_desc(q_s + (ks >> 2) * kKbQ + off, 16, 1024);
          const uint64_t bd = sw128_desc(tile + (ks >> 2) * kKbTile + off, 16, 1024);
          mma_ss(d, a, bd, kIdS, ks > 0 ? 1u : 0u);
        }
        mma_commit(bar(B_SFULL + k));
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int s = j % kStages, k = j % kSBuf;
        if (!mbar_wait(bar(B_PFULL + k), (j / kSBuf) & 1)) return false;
        tc_fence_after();
        const uint32_t tile = tiles_s + s * kTileBytes;
        const uint64_t bd = sw128_desc(tile + half * (kHalf / 64) * kKbTile, kKbTile, 1024);
        mma_ts(tmem + kOCol, tmem + kSCol + k * kTile, bd, kIdPV, j > 0 ? 1u : 0u);
        mma_commit(bar(B_PVDONE + k));
        mma_commit(bar(B_EMPTY + s));
        return true;
      };
      if (T > 0 && !issue_s(0)) timed_out = true;
      for (int j = 0; j < T && !timed_out; ++j) {
        if (j + 1 < T && !issue_s(j + 1)) { timed_out = true; break; }
        if (!issue_pv(j)) { timed_out = true; break; }
      }
      // every MMA issued above has retired once this commit lands
      mma_commit(bar(B_DONE));
      if (!mbar_wait(bar(B_DONE), 0)) timed_out = true;
    }
  } else {
    // ---------------------------------------------------------------- softmax (warps 0-3, one head row per thread)
    const int r = tid;                                   // TMEM lane = head row
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float base_scale = p.sm_scale * kLog2e;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < T && !timed_out; ++j) {
      const int k = j % kSBuf;
      // warp-uniform outcome: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + k), (j / kSBuf) & 1))) { timed_out = true; break; }
      tc_fence_after();
      uint32_t sr[16];
      tmem_ld16(lane_addr + kSCol + k * kTile, sr);
      tmem_wait_ld();
      const int pg = j / tpp;
      // FP8 tiles hold codes: the page scale multiplies the scores (key side)
      // and P (value side); l stays in unscaled softmax weights
      const float vs = s_fmt[pg] == IAK_MLA_FP8 ? p.fp8_scale[s_pid[pg]] : 1.f;
      const float sc = base_scale * vs;
      float x[16], tmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        x[i] = __uint_as_float(sr[i]) * sc;
        tmax = fmaxf(tmax, x[i]);
      }
      if (j == 0) {
        m_used = tmax;
      } else {
        const bool need = tmax > m_used + kLazyLog2;
        if (__any_sync(0xffffffffu, need)) {
          // rescale O_h in TMEM: every earlier PV must have landed
          if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + (j - 1) % kSBuf), ((j - 1) / kSBuf) & 1))) {
            timed_out = true;
            break;
          }
          tc_fence_after();
          const float f = need ? exp2f(m_used - tmax) : 1.f;
          if (need) {
            l *= f;
            m_used = tmax;
          }
#pragma unroll 1
          for (int c = 0; c < kHalf / 16; ++c) {
            uint32_t o[16];
            tmem_ld16(lane_addr + kOCol + c * 16, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st16(lane_addr + kOCol + c * 16, o);
          }
          tmem_wait_st();
        }
      }
      uint32_t pk[8];
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float p0 = exp2f(x[2 * i] - m_used), p1 = exp2f(x[2 * i + 1] - m_used);
        lsum += p0 + p1;
        const __half2 h = __floats2half2_rn(p0 * vs, p1 * vs);
        pk[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
      l += lsum;
      tmem_st8(lane_addr + kSCol + k * kTile, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(B_PFULL + k));
    }
    // ---------------------------------------------------------------- epilogue
    bool have = T > 0 && !timed_out;
    if (have) {
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + (T - 1) % kSBuf), ((T - 1) / kSBuf) & 1))) {
        timed_out = true;
        have = false;
      }
      tc_fence_after();
    }
    const bool row_ok = r < p.H;
    const int64_t row = static_cast<int64_t>(b) * p.H + r;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float m_nat = l > 0.f ? m_used * kLn2 : -INFINITY;
    float* acc_dst = nullptr;
    if (S > 1) {
      const int64_t wi = row * S + split;
      if (row_ok && half == 0) {
        p.ws_m[wi] = have ? m_nat : -INFINITY;
        p.ws_l[wi] = have ? l : 0.f;
      }
      acc_dst = p.ws_acc + wi * p.Dv;
    } else if (p.ex_l) {
      if (row_ok && half == 0) {
        p.ex_m[row] = have ? m_nat : -INFINITY;
        p.ex_l[row] = have ? l : 0.f;
      }
      acc_dst = p.ex_acc + row * p.Dv;
    }
#pragma unroll 1
    for (int c = 0; c < kHalf / 16; ++c) {
      uint32_t o[16];
      if (have) {
        tmem_ld16(lane_addr + kOCol + c * 16, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = 0u;
      }
      if (!row_ok) continue;
      const int d0 = half * kHalf + c * 16;
      if (acc_dst) {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(acc_dst + d0 + i) =
              make_float4(__uint_as_float(o[i]), __uint_as_float(o[i + 1]), __uint_as_float(o[i + 2]),
                          __uint_as_float(o[i + 3]));
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          store_from_float(p.out, p.out_dtype, b * p.o_sb + r * p.o_sh + d0 + i, __uint_as_float(o[i]) * inv);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  if (timed_out) atomicAdd(&g_mla_timeouts, 1u);
}

// --------------------------------------------------------- tensor maps ---
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult res;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &res) == cudaSuccess &&
        res == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(q);
  });
  return fn;
}

// [rows, 576] latent rows: dense 16-bit (box 64 x 16, 128-byte swizzle) or FP8 bytes (box 192 x 16, no swizzle).
int make_latent_map(CUtensorMap* m, const void* base, int kind, int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return fail(IAK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const bool fp8 = kind == 2;
  const CUtensorMapDataType dt =
      fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : (kind == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  const uint64_t eb = fp8 ? 1 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kDqk), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kDqk * eb)};
  cuuint32_t box[2] = {fp8 ? static_cast<cuuint32_t>(kFp8Part) : 64u, static_cast<cuuint32_t>(kTile)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  fp8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(IAK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return IAK_OK;
}

int cached_latent_map(CUtensorMap* out, const void* base, int kind, int64_t rows) {
  struct Key {
    const void* base; int kind; int64_t rows;
    bool operator==(const Key& o) const { return base == o.base && kind == o.kind && rows == o.rows; }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.base) ^ (static_cast<size_t>(k.rows) * 2654435761u) ^ k.kind;
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  const Key key{base, kind, rows};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return IAK_OK;
    }
  }
  const int st = make_latent_map(out, base, kind, rows);
  if (st) return st;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 64) cache.clear();
  cache.emplace(key, *out);
  return IAK_OK;
}

}  // namespace

bool mla_tc_eligible(const MlaParams& p) {
  if (p.Dqk != kDqk || p.Dv != kDv || p.H > kRows || p.PS % kTile) return false;
  if (p.q_dtype != IAK_DT_BF16 && p.q_dtype != IAK_DT_F16) return false;
  if (reinterpret_cast<uintptr_t>(p.q) % 16 || p.q_sb % 8 || p.q_sh % 8) return false;
  if (p.dense && ((p.dense_dtype != IAK_DT_BF16 && p.dense_dtype != IAK_DT_F16) ||
                  reinterpret_cast<uintptr_t>(p.dense) % 16))
    return false;
  if (p.fp8 && reinterpret_cast<uintptr_t>(p.fp8) % 16) return false;
  if (p.num_pages * static_cast<int64_t>(p.PS) >= (1LL << 31)) return false;
  if (p.ex_acc && reinterpret_cast<uintptr_t>(p.ex_acc) % 16) return false;
  return true;
}

// Items = batch x splits x 2 value halves, one CTA each, one CTA per SM:
// pick the split count minimising waves x (pages per item + a fixed cost
// of about four pages for the Q staging and pipeline fill).
void plan_mla_tc(MlaParams* p, int requested) {
  const int W = std::max(1, p->W);
  int splits = requested;
  if (splits <= 0) {
    const int64_t sms = device_sm_count();
    int64_t best = -1, best_cost = 0;
    for (int c = 1; c <= std::min(W, 64); ++c) {
      const int64_t pps = (W + c - 1) / c;
      if (pps > kMaxItemPages) continue;
      const int64_t items = static_cast<int64_t>(p->B) * c * 2;
      const int64_t waves = (items + sms - 1) / sms;
      const int64_t cost = waves * (pps + 4);
      if (best < 0 || cost < best_cost) { best = c; best_cost = cost; }
    }
    splits = best < 0 ? (W + kMaxItemPages - 1) / kMaxItemPages : static_cast<int>(best);
  }
  splits = std::max(1, std::min(splits, W));
  int pps = (W + splits - 1) / splits;
  if (pps > kMaxItemPages) pps = kMaxItemPages;
  p->pages_per_split = pps;
  p->num_splits = (W + pps - 1) / pps;
}

int launch_mla_tc(const MlaParams& p, cudaStream_t s) {
  CUtensorMap dmap, fmap;
  std::memset(&dmap, 0, sizeof(dmap));
  std::memset(&fmap, 0, sizeof(fmap));
  const int64_t rows = p.num_pages * p.PS;
  if (rows <= 0) return fail(IAK_ERR_INVALID_ARG, "empty latent pool");
  if (p.dense) {
    const int st = cached_latent_map(&dmap, p.dense, p.dense_dtype == IAK_DT_BF16 ? 1 : 0, rows);
    if (st) return st;
  }
  if (p.fp8) {
    const int st = cached_latent_map(&fmap, p.fp8, 2, rows);
    if (st) return st;
  }
  const int64_t items = static_cast<int64_t>(p.B) * p.num_splits * 2;
  if (items > 0x7FFFFFFF) return fail(IAK_ERR_UNSUPPORTED, "too many MLA work items");
  const size_t smem = Smem::total + 1024;
  static std::mutex mu;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return check_cuda(err, "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      err = cudaFuncSetAttribute(mla_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return check_cuda(err, "mla_tc smem attribute");
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
  }
  kernel_timer_begin(s);
  mla_tc_kernel<<<static_cast<unsigned>(items), kThreads, smem, s>>>(p, dmap, fmap);
  err = cudaGetLastError();
  kernel_timer_end(s);
  return check_cuda(err, "mla_tc launch");
}

}  // namespace iak
