// Tensor-core (tcgen05 / TMEM) MLA decode for the absorbed DeepSeek-V2 shape:
// d_qk = 576 (512 latent + 64 rope channels), d_v = 512, up to 128 query
// heads per sequence, latent pages of a multiple of 64 tokens, dense BF16 /
// F16 or FP8-e4m3 (per-page scale) pages.
//
// One work item (sequence b, page range `split`) runs on a cluster of two
// CTAs on two SMs, which split the latent channels between them:
//   * CTA 0 owns latent channels [0, 256) and rope channels [512, 544), CTA 1
//     channels [256, 512) and [544, 576).  Each CTA converts only its own channels of
//     every latent row, computes the partial scores S_c = Q_c . C_c^T over
//     them, and accumulates the value half O_c += P . C[:, 256c : 256c+256];
//   * the 128 head rows are the M = 128 rows of every MMA; Q_c's 256 latent
//     channels sit in TMEM (the A operand of the TS-form MMA), the rope
//     channels in shared memory (K-major, 128-byte swizzle);
//   * latents are consumed in 64-token chunks.  A converter warpgroup loads
//     the CTA's k-blocks (64 channels each) of a chunk from global memory,
//     one chunk ahead in registers (chunks are bulk-prefetched into L2 a few
//     chunks ahead), converts them to f16 x 2^-8 (FP8 by the hardware e4m3x2
//     conversion and a multiply, exact; dense by one multiply) and stores them
//     swizzled into one of three chunk sets;
//   * S_c: M=128, N=64 tokens, K=288 (18 MMAs), fp32 in TMEM, two S buffers.  The
//     softmax warpgroup owns one TMEM lane (= one head) per thread.  Each
//     thread reads its row of S_c and writes it into a local staging block;
//     each warp then sends its 32 rows (8 KB) into the other CTA's shared
//     memory with one bulk copy (distributed shared memory, no multicast) whose
//     bytes complete the receiving CTA's mbarrier, waits for the other CTA's
//     rows and adds the two; the otherwise idle page-list warp tells the other
//     CTA when the block has been read (a cluster-scope release that stays off
//     the softmax's path).  Both CTAs
//     add the same two fp32 numbers (a + b == b + a), so they hold identical
//     scores, maxima, P and l without further exchange.  P (f16) is written
//     back over S and is the TMEM A operand of O_c += P . C_c (M=128, N=256,
//     K=64 in 4 MMAs, the value k-blocks read MN-major), O_c fp32 in TMEM;
//   * FP8 latents stay codes: the page scale multiplies the scores and P (so
//     O accumulates code x scale x weight); l sums unscaled weights;
//   * the O accumulator is rescaled lazily (only when a row max grows by
//     more than 2^8), in TMEM.
// TMEM: O_c 256 | S/P 2 x 64 | Q_c 128 columns (512 allocated: one CTA per SM).
//
// Measured at the C4 shape (batch 64, 154 pages, per launch): this kernel 398 us.
// One CTA per value half computing the whole S (no exchange, twice the S MMAs and
// conversions): 519 us with its converters loading a chunk at once, 499 us with a
// two-chunk ring, 815-1060 us with loads pipelined one unit or eight jobs ahead
// in registers (each use then waits on loads issued after it).  Exchanging the
// partial scores with per-thread st.async stores instead of per-warp bulk copies:
// 504 us; with plain remote stores and cluster-scope release arrivals: 695 us.
//
// Reference: triton_mla_decode.py:155-186 (_mla_decode_cpu) per query row,
// restated per head; rows without pages give 0.
#include <cmath>
#include <algorithm>
#include <cstring>
#include <mutex>

#include "mla_internal.cuh"
#include "tc_ptx.cuh"

namespace iak {

__device__ unsigned int g_mla_timeouts = 0;

int read_mla_timeouts(unsigned int* value, bool reset) {
  unsigned int v = 0;
  int st = check_cuda(cudaMemcpyFromSymbol(&v, g_mla_timeouts, sizeof(v)), "read mla timeouts");
  if (st) return st;
  if (reset && v) {
    const unsigned int zero = 0;
    st = check_cuda(cudaMemcpyToSymbol(g_mla_timeouts, &zero, sizeof(zero)), "reset mla timeouts");
    if (st) return st;
  }
  *value = v;
  return IAK_OK;
}

namespace {

using namespace tc;

constexpr int kDqk = 576, kDv = 512, kHalf = kDv / 2, kRows = 128, kChunk = 64;
constexpr int kValBlocks = kHalf / 64;              // 64-channel k-blocks of one value half (and of Q_c in TMEM)
constexpr int kMaxBlocks = kValBlocks + 1;          // + the rope block (each CTA fills its 32 channels)
constexpr int kRopeHalf = 32;                       // rope channels per CTA
constexpr int kSets = 3;                            // chunk sets in flight
constexpr int kPrefetchAhead = 4;                   // chunks prefetched into L2 ahead of the converters
constexpr int kQTmemCols = kHalf / 2;               // Q_c: 256 f16 channels, two per 32-bit column
constexpr int kKbQ = kRows * 128;                   // bytes of one Q k-block (128 rows x 128 B)
constexpr int kKb = kChunk * 128;                   // bytes of one f16 latent k-block (64 rows x 128 B)
constexpr int kSetBytes = kMaxBlocks * kKb;
constexpr int kXRow = kChunk * 4;                   // one head's fp32 partial scores of a chunk
constexpr int kXBuf = kRows * kXRow;
constexpr int kMaxItemPages = 512;
constexpr int kThreads = 320;                       // softmax wg | converter wg | page-list warp | MMA warp
constexpr int kConvWarp0 = 4, kListWarp = 8, kMmaWarp = 9;
constexpr int kSBuf = 2;
constexpr int kOCol = 0, kSCol = kHalf, kQCol = kSCol + kSBuf * kChunk, kTmemCols = 512;
static_assert(kQCol + kQTmemCols <= kTmemCols, "TMEM budget");
constexpr float kLazyLog2 = 8.f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum {
  B_SETFULL = 0,                  // chunk set: converters -> MMA (f16 k-blocks stored)
  B_SETEMPTY = B_SETFULL + kSets, // chunk set: MMA commit after P.V -> converters
  B_SFULL = B_SETEMPTY + kSets,   // MMA commit -> softmax (S_c ready)
  B_PFULL = B_SFULL + kSBuf,      // softmax -> MMA (P written, O rescaled)
  B_PVDONE = B_PFULL + kSBuf,     // MMA commit -> softmax / MMA (P.V done: O current, S/P buffer free)
  B_XFULL = B_PVDONE + kSBuf,     // the other CTA's bulk copies (32 KB per chunk) -> this CTA's softmax
  B_XEMPTY,                       // the other CTA's page-list warp -> this CTA: it has read what this CTA sent
  B_XREAD,                        // this CTA's softmax -> its page-list warp: received block read
  B_DONE,                         // MMA commit -> MMA (all MMAs retired)
  B_QREADY,                       // softmax warps -> MMA: Q_c stored in TMEM
  B_COUNT
};

struct Smem {
  static constexpr int q = 0;                                       // Q rope k-block
  static constexpr int sets = q + kKbQ;                             // [kSets][kMaxBlocks] latent k-blocks
  static constexpr int xstage = sets + kSets * kSetBytes;           // [kRows][kXRow]: this CTA's S rows, sent
  static constexpr int xbuf = xstage + kXBuf;                       // [kRows][kXRow]: the other CTA's S rows
  static constexpr int pid = xbuf + kXBuf;
  static constexpr int pscale = pid + kMaxItemPages * 4;
  static constexpr int pfmt = pscale + kMaxItemPages * 4;
  static constexpr int bars = pfmt + kMaxItemPages;
  static constexpr int tmem = bars + B_COUNT * 8;
  static constexpr int nvalid = tmem + 4;
  static constexpr int total = nvalid + 12;
};
static_assert(Smem::sets % 1024 == 0 && kSetBytes % 1024 == 0, "1024-byte alignment");
static_assert(Smem::bars % 8 == 0, "mbarriers need 8-byte alignment");
static_assert(Smem::total + 1024 <= 232448, "shared memory budget");

// Latent tiles are stored in shared memory as f16 holding value * 2^-8 (kTileScale):
// * FP8 codes: hardware e4m3x2 -> f16x2 conversion, then times 2^-8 (both exact);
// * dense rows are multiplied by 2^-8 on the way (exact above the f16 subnormal
//   range, 2^-24 absolute resolution below it).
// The 2^8 is restored in the score scale and in the final normalisation.
constexpr float kTileScale = 1.f / 256.f;
// two bf16 (low half = first element) -> two f16, exact inside the f16 range
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w, float mul = 1.f) {
  const __half2 h = __floats2half2_rn(__uint_as_float(w << 16) * mul, __uint_as_float(w & 0xFFFF0000u) * mul);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// two f16 times 2^-8
__device__ __forceinline__ uint32_t f16x2_tile_scale(uint32_t w) {
  const __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&w), __float2half2_rn(kTileScale));
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ int mla_fmt(const MlaParams& p, int64_t pid) {
  if (!p.tags) return IAK_MLA_DENSE;
  const int tag = p.tag_bytes == 1 ? static_cast<int>(static_cast<const uint8_t*>(p.tags)[pid])
                                   : static_cast<const int32_t*>(p.tags)[pid];
  return (tag >= 0 && tag < 16) ? p.tag_map[tag] : p.tag_default;
}

__device__ __forceinline__ uint4 to_f16x8(uint4 x, bool bf) {
  return bf ? make_uint4(bf16x2_to_f16x2(x.x), bf16x2_to_f16x2(x.y), bf16x2_to_f16x2(x.z), bf16x2_to_f16x2(x.w)) : x;
}

// Byte offset of 16-byte chunk q (0..15) of head row r in an exchange buffer (XOR swizzle: the 32
// rows of a warp spread over all banks).
__device__ __forceinline__ uint32_t xoff(int r, int q) {
  return static_cast<uint32_t>(r * kXRow + ((q ^ (r & 15)) << 4));
}

// The converters' work comes in loads of two 16-byte words per k-block per thread: one whole
// chunk of an FP8 page (64 rows x 64 codes per k-block), or half of a chunk of a dense page
// (32 rows x 64 channels per k-block).
struct LoadUnit {
  int chunk;     // chunk index, -1 when past the end
  int half;      // dense pages: which 32 rows
};

// ---------------------------------------------------------------- kernel ---
__global__ void __launch_bounds__(kThreads, 1) mla_tc_kernel(const MlaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (sbase - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int S = p.num_splits;
  const int cta = static_cast<int>(cluster_ctarank());   // which channels this CTA owns
  const int peer = cta ^ 1;
  const int split = (blockIdx.x >> 1) % S;
  const int b = (blockIdx.x >> 1) / S;
  const int kb0 = cta * kValBlocks;                        // its first latent k-block
  const int rope0 = 2 * kHalf + cta * kRopeHalf;           // its first rope channel

  int32_t* s_pid = reinterpret_cast<int32_t*>(sm + Smem::pid);
  float* s_scale = reinterpret_cast<float*>(sm + Smem::pscale);
  uint8_t* s_fmt = sm + Smem::pfmt;
  volatile uint32_t* s_tmem = reinterpret_cast<volatile uint32_t*>(sm + Smem::tmem);
  volatile int* s_nvalid = reinterpret_cast<volatile int*>(sm + Smem::nvalid);
  auto bar = [&](int i) -> uint32_t { return sbase + Smem::bars + 8u * static_cast<uint32_t>(i); };
  // byte offset (from sbase) of k-block i of chunk set s
  auto blk = [&](int s, int i) -> uint32_t { return Smem::sets + s * kSetBytes + i * kKb; };
  const bool q_bf16 = p.q_dtype == IAK_DT_BF16;
  const uint16_t* qrow0 = static_cast<const uint16_t*>(p.q) + b * p.q_sb;

  if (tid == 0) {
    for (int i = 0; i < kSets; ++i) {
      mbar_init(bar(B_SETFULL + i), 128);
      mbar_init(bar(B_SETEMPTY + i), 1);
    }
    for (int k = 0; k < kSBuf; ++k) {
      mbar_init(bar(B_SFULL + k), 1);
      mbar_init(bar(B_PFULL + k), 128);
      mbar_init(bar(B_PVDONE + k), 1);
    }
    mbar_init(bar(B_XFULL), 1);
    mbar_init(bar(B_XEMPTY), 1);
    mbar_init(bar(B_XREAD), 128);
    mbar_init(bar(B_DONE), 1);
    mbar_init(bar(B_QREADY), 128);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // the receive block expects the other CTA's rows of chunk 0
    mbar_arrive_expect_tx(bar(B_XFULL), kXBuf);
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + Smem::tmem),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kListWarp) {
    // compact this item's slice of the page table (valid ids of dense / FP8 pages, in order) with
    // page scales; both CTAs of the pair derive the same list from the same table
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
        s_scale[r] = fmt == IAK_MLA_FP8 ? p.fp8_scale[pid] : 1.f;
      }
      cnt += __popc(m);
    }
    if (lane == 0) *s_nvalid = cnt;
  }
  if (warp >= kConvWarp0 && warp < kListWarp) {
    // Q rope channels [512, 576) as f16 in the K-major 128-byte-swizzled layout; rows >= H are zero
    const int ct = tid - kConvWarp0 * 32;
#pragma unroll
    for (int i = 0; i < kRows * 8 / 128; ++i) {
      const int u = ct + 128 * i, r = u >> 3, c = u & 7;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < p.H) v = to_f16x8(*reinterpret_cast<const uint4*>(qrow0 + r * p.q_sh + 2 * kHalf + c * 8), q_bf16);
      *reinterpret_cast<uint4*>(sm + Smem::q + swz(r, c)) = v;
    }
    fence_proxy_async();
  }
  tc_fence_before();
  // every barrier of both CTAs is initialised before either CTA arrives on the other's
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_valid = *s_nvalid;
  const int cpp = p.PS / kChunk;     // chunks per page
  const int T = n_valid * cpp;
  bool timed_out = false;
  // first latent row of chunk j in its pool
  auto chunk_row0 = [&](int j) -> int64_t {
    return static_cast<int64_t>(s_pid[j / cpp]) * p.PS + (j % cpp) * kChunk;
  };

  if (warp == kListWarp) {
    // ---------------------------------------------------------------- exchange-buffer release
    // once this CTA's softmax has read the row block the other CTA sent for chunk j, tell the other
    // CTA (it sends chunk j + 1 into the same block, and reuses its staging block)
    const uint32_t xempty_remote = mapa_shared(bar(B_XEMPTY), static_cast<uint32_t>(peer));
    for (int j = 0; j + 1 < T; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait_sleep(bar(B_XREAD), j & 1))) {
        timed_out = true;
        break;
      }
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_cluster(xempty_remote);
      }
      __syncwarp();
    }
    if (lane != 0) timed_out = false;           // counted once
  } else if (warp >= kConvWarp0 && warp < kListWarp) {
    // ---------------------------------------------------------------- converters: global -> f16 -> shared
    const int ct = tid - kConvWarp0 * 32;
    const bool dense_bf16 = p.dense_dtype == IAK_DT_BF16;
    auto prefetch_chunk = [&](int j) {
      const int64_t row0 = chunk_row0(j);
      if (s_fmt[j / cpp] == IAK_MLA_FP8)
        prefetch_l2(p.fp8 + row0 * kDqk, kChunk * kDqk);
      else
        prefetch_l2(static_cast<const uint16_t*>(p.dense) + row0 * kDqk, kChunk * kDqk * 2);
    };
    // the two CTAs of the pair prefetch alternate chunks (each prefetch covers whole rows)
    if (ct == 0)
      for (int j = cta; j < kPrefetchAhead && j < T; j += 2) prefetch_chunk(j);
    auto next_unit = [&](LoadUnit u) -> LoadUnit {
      if (u.chunk < 0) return u;
      if (s_fmt[u.chunk / cpp] != IAK_MLA_FP8 && u.half == 0) return LoadUnit{u.chunk, 1};
      return u.chunk + 1 < T ? LoadUnit{u.chunk + 1, 0} : LoadUnit{-1, 0};
    };
    // FP8 unit: thread words t = 0, 1 of value k-block i are row (ct + 128t) / 4, 16-code segment
    // (ct + 128t) % 4; of the rope block (word 0 only) row ct / 2, 16-code segment ct % 2 of this
    // CTA's 32 rope channels.  Dense half h: value words row 32h + (ct + 128t) / 8, 8-channel segment
    // (ct + 128t) % 8; rope word row 32h + ct / 4, 8-channel segment ct % 4.
    auto load_unit = [&](LoadUnit u, uint4 (&x)[kMaxBlocks][2]) {
      if (u.chunk < 0) return;
      const int64_t row0 = chunk_row0(u.chunk);
      if (s_fmt[u.chunk / cpp] == IAK_MLA_FP8) {
        const uint8_t* rows = p.fp8 + row0 * kDqk;
#pragma unroll
        for (int i = 0; i < kValBlocks; ++i)
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int w = ct + 128 * t;
            x[i][t] = *reinterpret_cast<const uint4*>(rows + (w >> 2) * kDqk + (kb0 + i) * 64 + (w & 3) * 16);
          }
        x[kValBlocks][0] = *reinterpret_cast<const uint4*>(rows + (ct >> 1) * kDqk + rope0 + (ct & 1) * 16);
      } else {
        const uint16_t* rows = static_cast<const uint16_t*>(p.dense) + (row0 + 32 * u.half) * kDqk;
#pragma unroll
        for (int i = 0; i < kValBlocks; ++i)
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int w = ct + 128 * t;
            x[i][t] = *reinterpret_cast<const uint4*>(rows + (w >> 3) * kDqk + (kb0 + i) * 64 + (w & 7) * 8);
          }
        x[kValBlocks][0] = *reinterpret_cast<const uint4*>(rows + (ct >> 2) * kDqk + rope0 + (ct & 3) * 8);
      }
    };
    auto store_fp8 = [&](uint32_t off, int r, int c, const uint4& x) {   // 16 codes -> f16 chunks c, c + 1
      const uint32_t wd[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint4 v;
        e4m3x4_to_f16_scaled(wd[2 * h], v.x, v.y);
        e4m3x4_to_f16_scaled(wd[2 * h + 1], v.z, v.w);
        *reinterpret_cast<uint4*>(sm + off + swz(r, c + h)) = v;
      }
    };
    auto store_dense = [&](uint32_t off, int r, int c, const uint4& y) {   // 8 channels -> f16 chunk c
      *reinterpret_cast<uint4*>(sm + off + swz(r, c)) =
          dense_bf16 ? make_uint4(bf16x2_to_f16x2(y.x, kTileScale), bf16x2_to_f16x2(y.y, kTileScale),
                                  bf16x2_to_f16x2(y.z, kTileScale), bf16x2_to_f16x2(y.w, kTileScale))
                     : make_uint4(f16x2_tile_scale(y.x), f16x2_tile_scale(y.y), f16x2_tile_scale(y.z),
                                  f16x2_tile_scale(y.w));
    };
    // store one unit into chunk set s (the rope block holds this CTA's 32 channels at their place:
    // 16-byte chunks 4 * cta .. 4 * cta + 3 of each row)
    auto store_unit = [&](LoadUnit u, int s, const uint4 (&x)[kMaxBlocks][2]) {
      if (s_fmt[u.chunk / cpp] == IAK_MLA_FP8) {
#pragma unroll
        for (int i = 0; i < kValBlocks; ++i)
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int w = ct + 128 * t;
            store_fp8(blk(s, i), w >> 2, 2 * (w & 3), x[i][t]);
          }
        store_fp8(blk(s, kValBlocks), ct >> 1, 4 * cta + 2 * (ct & 1), x[kValBlocks][0]);
      } else {
#pragma unroll
        for (int i = 0; i < kValBlocks; ++i)
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int w = ct + 128 * t;
            store_dense(blk(s, i), 32 * u.half + (w >> 3), w & 7, x[i][t]);
          }
        store_dense(blk(s, kValBlocks), 32 * u.half + (ct >> 2), 4 * cta + (ct & 3), x[kValBlocks][0]);
      }
    };
    // Process one unit whose words are in x: wait for its set at the chunk's first unit, store,
    // and publish the set at the chunk's last unit.
    auto process = [&](LoadUnit u, LoadUnit nxt, const uint4 (&x)[kMaxBlocks][2]) -> bool {
      const int j = u.chunk, s = j % kSets;
      if (u.half == 0) {
        if (ct == 0 && j + kPrefetchAhead < T && ((j + kPrefetchAhead) & 1) == cta) prefetch_chunk(j + kPrefetchAhead);
        if (j >= kSets && !mbar_wait_sleep(bar(B_SETEMPTY + s), ((j / kSets) - 1) & 1)) return false;
      }
      store_unit(u, s, x);
      if (nxt.chunk != j) {
        fence_proxy_async();
        mbar_arrive(bar(B_SETFULL + s));
      }
      return true;
    };
    // Two register sets in turn: the loads of the next unit are in flight while this one is stored.
    uint4 xa[kMaxBlocks][2], xb[kMaxBlocks][2];
    LoadUnit cur = T > 0 ? LoadUnit{0, 0} : LoadUnit{-1, 0};
    load_unit(cur, xa);
    while (cur.chunk >= 0) {
      LoadUnit nxt = next_unit(cur);
      load_unit(nxt, xb);
      if (!process(cur, nxt, xa)) { timed_out = true; break; }
      cur = nxt;
      if (cur.chunk < 0) break;
      nxt = next_unit(cur);
      load_unit(nxt, xa);
      if (!process(cur, nxt, xb)) { timed_out = true; break; }
      cur = nxt;
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop and polls every barrier; one elected lane issues the MMAs and
    // their commits, so the operands stay warp-uniform.
    {
      constexpr uint32_t kIdS = idesc_f16(kRows, kChunk, 0, 0);  // S_c = Q_c . C_c^T
      constexpr uint32_t kIdPV = idesc_f16(kRows, kHalf, 0, 1);  // O_c += P . C_c (value blocks read MN-major)
      const uint64_t q_rope_desc = sw128_desc(sbase + Smem::q, 16, 1024);
      auto wait = [&](int b, uint32_t parity) -> bool { return __all_sync(0xffffffffu, mbar_wait(bar(b), parity)); };
      if (!wait(B_QREADY, 0)) timed_out = true;
      auto issue_s = [&](int j) -> bool {
        const int k = j & 1, s = j % kSets;
        if (j >= kSBuf && !wait(B_PVDONE + k, ((j >> 1) - 1) & 1)) return false;
        if (!wait(B_SETFULL + s, (j / kSets) & 1)) return false;
        tc_fence_after();
        const uint32_t d = tmem + kSCol + k * kChunk;
        if (elect_one()) {
          for (int i = 0; i < kValBlocks; ++i) {
            const uint64_t bd = sw128_desc(sbase + blk(s, i), 16, 1024);
#pragma unroll
            for (int t = 0; t < 4; ++t)
              mma_ts(d, tmem + kQCol + i * 32 + t * 8, bd + (t * 2), kIdS, (i == 0 && t == 0) ? 0u : 1u);
          }
          {
            // this CTA's 32 rope channels: k-steps 2 * cta and 2 * cta + 1 of the rope block
            const uint64_t bd = sw128_desc(sbase + blk(s, kValBlocks), 16, 1024);
#pragma unroll
            for (int t = 2 * cta; t < 2 * cta + 2; ++t)
              mma_ss(d, q_rope_desc + ((t * 32) >> 4), bd + (t * 2), kIdS, 1u);
          }
          mma_commit(bar(B_SFULL + k));
        }
        __syncwarp();
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int k = j & 1, s = j % kSets;
        if (!wait(B_PFULL + k, (j >> 1) & 1)) return false;
        tc_fence_after();
        const uint64_t bd = sw128_desc(sbase + blk(s, 0), kKb, 1024);
        if (elect_one()) {
#pragma unroll
          for (int t = 0; t < kChunk / 16; ++t)
            mma_ts(tmem + kOCol, tmem + kSCol + k * kChunk + t * 8, bd + ((t * 2048) >> 4), kIdPV,
                   (j > 0 || t > 0) ? 1u : 0u);
          mma_commit(bar(B_PVDONE + k));
          mma_commit(bar(B_SETEMPTY + s));
        }
        __syncwarp();
        return true;
      };
      if (!timed_out && T > 0 && !issue_s(0)) timed_out = true;
      for (int j = 0; j < T && !timed_out; ++j) {
        if (j + 1 < T && !issue_s(j + 1)) { timed_out = true; break; }
        if (!issue_pv(j)) { timed_out = true; break; }
      }
      // every MMA issued above has retired once this commit lands
      if (elect_one()) mma_commit(bar(B_DONE));
      __syncwarp();
      if (!wait(B_DONE, 0)) timed_out = true;
      if (lane != 0) timed_out = false;           // counted once
    }
  } else if (warp < kConvWarp0) {
    // ---------------------------------------------------------------- softmax (warps 0-3, one head row per thread)
    const int r = tid;                                   // TMEM lane = head row
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    {
      // Q_c (latent channels [256c, 256c + 256)) of this row into TMEM columns kQCol.. (f16 pairs)
      const uint16_t* qr = qrow0 + r * p.q_sh + cta * kHalf;
#pragma unroll 1
      for (int c = 0; c < kQTmemCols / 32; ++c) {
        uint32_t v[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint4 x = make_uint4(0u, 0u, 0u, 0u);
          if (r < p.H) x = to_f16x8(*reinterpret_cast<const uint4*>(qr + c * 64 + i * 8), q_bf16);
          v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
        }
        tmem_st32(lane_addr + kQCol + c * 32, v);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(B_QREADY));
    }
    // the other CTA's receive block and its barrier; this warp's 32 rows of the blocks
    const uint32_t x_remote = mapa_shared(sbase + Smem::xbuf, static_cast<uint32_t>(peer)) + warp * 32 * kXRow;
    const uint32_t xfull_remote = mapa_shared(bar(B_XFULL), static_cast<uint32_t>(peer));
    const uint32_t x_stage = sbase + Smem::xstage + warp * 32 * kXRow;
    const float base_scale = p.sm_scale * kLog2e / kTileScale;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < T && !timed_out; ++j) {
      const int k = j & 1;
      // one lane polls; the outcome is broadcast (warp-uniform: the TMEM loads below are warp-collective)
      bool ok = true;
      if (lane == 0) ok = mbar_wait(bar(B_SFULL + k), (j >> 1) & 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) { timed_out = true; break; }
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(lane_addr + kSCol + k * kChunk, sr[0]);
      tmem_ld32(lane_addr + kSCol + k * kChunk + 32, sr[1]);
      tmem_wait_ld();
      // ---- exchange the partial rows with the other CTA.  Its receive block (and this CTA's staging
      // block, which the last bulk copy read) are free once its page-list warp has reported the
      // read of chunk j - 1.
      if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait_cluster(bar(B_XEMPTY), (j - 1) & 1))) {
        timed_out = true;
        break;
      }
#pragma unroll
      for (int q = 0; q < kChunk / 4; ++q) {
        const int h = q >> 3, c = (q & 7) * 4;
        *reinterpret_cast<uint4*>(sm + Smem::xstage + xoff(r, q)) = make_uint4(sr[h][c], sr[h][c + 1], sr[h][c + 2], sr[h][c + 3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) bulk_copy_to_cluster(x_remote, x_stage, 32 * kXRow, xfull_remote);
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(bar(B_XFULL), j & 1))) {
        timed_out = true;
        break;
      }
      // the receive block expects the other CTA's rows of chunk j + 1 (sent only after this CTA's
      // read of chunk j is reported, so they land in the next phase)
      if (r == 0 && j + 1 < T) mbar_arrive_expect_tx(bar(B_XFULL), kXBuf);
      // FP8 latents hold codes: the page scale multiplies the scores (key side)
      // and P (value side); l stays in unscaled softmax weights
      const float vs = s_scale[j / cpp];
      const float sc = base_scale * vs;
      float x[kChunk], tmax;
      {
        const uint8_t* xl = sm + Smem::xbuf;
        float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
        for (int q = 0; q < kChunk / 4; ++q) {
          const uint4 o = *reinterpret_cast<const uint4*>(xl + xoff(r, q));
          const int h = q >> 3, c = (q & 7) * 4;
          // own + other: the other CTA adds the same two numbers in the other order (identical sums)
          x[4 * q] = __uint_as_float(sr[h][c]) + __uint_as_float(o.x);
          x[4 * q + 1] = __uint_as_float(sr[h][c + 1]) + __uint_as_float(o.y);
          x[4 * q + 2] = __uint_as_float(sr[h][c + 2]) + __uint_as_float(o.z);
          x[4 * q + 3] = __uint_as_float(sr[h][c + 3]) + __uint_as_float(o.w);
          ma = fmaxf(ma, fmaxf(x[4 * q], x[4 * q + 2]));
          mb = fmaxf(mb, fmaxf(x[4 * q + 1], x[4 * q + 3]));
        }
        // sc > 0: the max of the scaled scores is the scaled max
        tmax = fmaxf(ma, mb) * sc;
      }
      // the received block has been read (the page-list warp forwards this to the other CTA)
      mbar_arrive(bar(B_XREAD));
      if (j == 0) {
        m_used = tmax;
      } else {
        const bool need = tmax > m_used + kLazyLog2;
        if (__any_sync(0xffffffffu, need)) {
          // rescale O_c in TMEM: every earlier P.V must have landed
          if (!__all_sync(0xffffffffu, mbar_wait_sleep(bar(B_PVDONE + ((j - 1) & 1)), ((j - 1) >> 1) & 1))) {
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
          for (int c = 0; c < kHalf / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(lane_addr + kOCol + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st32(lane_addr + kOCol + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      uint32_t pk[kChunk / 2];
      float ls[2] = {0.f, 0.f};
      const float neg_m = -m_used;
#pragma unroll
      for (int i = 0; i < kChunk / 2; ++i) {
        const float p0 = ex2(fmaf(x[2 * i], sc, neg_m)), p1 = ex2(fmaf(x[2 * i + 1], sc, neg_m));
        ls[i & 1] += p0 + p1;
        const __half2 h = __floats2half2_rn(p0 * vs, p1 * vs);
        pk[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
      l += ls[0] + ls[1];
      tmem_st32(lane_addr + kSCol + k * kChunk, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(B_PFULL + k));
    }
    // ---------------------------------------------------------------- epilogue
    bool have = T > 0 && !timed_out;
    if (have) {
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + ((T - 1) & 1)), ((T - 1) >> 1) & 1))) {
        timed_out = true;
        have = false;
      }
      tc_fence_after();
    }
    const bool row_ok = r < p.H;
    const int64_t row = static_cast<int64_t>(b) * p.H + r;
    const float inv = l > 0.f ? 1.f / (l * kTileScale) : 0.f;   // O holds values * 2^-8
    const float m_nat = l > 0.f ? m_used * kLn2 : -INFINITY;
    float* acc_dst = nullptr;
    if (S > 1) {
      const int64_t wi = row * S + split;
      if (row_ok && cta == 0) {
        p.ws_m[wi] = have ? m_nat : -INFINITY;
        p.ws_l[wi] = have ? l : 0.f;
      }
      acc_dst = p.ws_acc + wi * p.Dv;
    } else if (p.ex_l) {
      if (row_ok && cta == 0) {
        p.ex_m[row] = have ? m_nat : -INFINITY;
        p.ex_l[row] = have ? l : 0.f;
      }
      acc_dst = p.ex_acc + row * p.Dv;
    }
#pragma unroll 1
    for (int c = 0; c < kHalf / 32; ++c) {
      uint32_t o[32];
      if (have) {
        tmem_ld32(lane_addr + kOCol + c * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (!row_ok) continue;
      const int d0 = cta * kHalf + c * 32;
      if (acc_dst) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(acc_dst + d0 + i) =
              make_float4(__uint_as_float(o[i]) / kTileScale, __uint_as_float(o[i + 1]) / kTileScale,
                          __uint_as_float(o[i + 2]) / kTileScale, __uint_as_float(o[i + 3]) / kTileScale);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
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
  __syncwarp();
  // neither CTA leaves while the other may still store into its shared memory or arrive on its barriers
  cluster_sync();
}

}  // namespace

bool mla_tc_eligible(const MlaParams& p) {
  if (p.Dqk != kDqk || p.Dv != kDv || p.H > kRows || p.PS % kChunk) return false;
  if (p.q_dtype != IAK_DT_BF16 && p.q_dtype != IAK_DT_F16) return false;
  if (reinterpret_cast<uintptr_t>(p.q) % 16 || p.q_sb % 8 || p.q_sh % 8) return false;
  if (p.dense && ((p.dense_dtype != IAK_DT_BF16 && p.dense_dtype != IAK_DT_F16) ||
                  reinterpret_cast<uintptr_t>(p.dense) % 16))
    return false;
  if (p.fp8 && reinterpret_cast<uintptr_t>(p.fp8) % 16) return false;
  if (p.num_pages * static_cast<int64_t>(p.PS) >= (1LL << 31)) return false;
  if (p.ex_acc && reinterpret_cast<uintptr_t>(p.ex_acc) % 16) return false;
  // the softmax takes the max of the raw scores times a positive scale
  if (!(p.sm_scale > 0.f) || !std::isfinite(p.sm_scale)) return false;
  return true;
}

// Items = batch x splits, each a cluster of two CTAs (one per SM):
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
  // one cluster of two CTAs (on two SMs) per work item
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(items));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  kernel_timer_begin(s);
  err = cudaLaunchKernelEx(&cfg, mla_tc_kernel, p);
  if (err == cudaSuccess) err = cudaGetLastError();
  kernel_timer_end(s);
  return check_cuda(err, "mla_tc launch");
}

}  // namespace iak
