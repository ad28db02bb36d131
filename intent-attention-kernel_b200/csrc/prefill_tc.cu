// Tensor-core (tcgen05 / TMEM) multi-query attention over selected pages, for
// head_dim 128 and page sizes 8..64 (any page format of the pools).
//
// One CTA = one work item (sequence b, page-table head h, two tiles of 128
// query rows that share every converted K / V chunk).  Rows are (query m,
// head g of the group) pairs, m-major, so a tile holds 128 / G consecutive
// queries of the G query heads sharing the table.
//   * the producer warp first compacts the unit's table into shared memory
//     (slots with a page in a supported format, a non-empty row mask and,
//     causal, a first selected row not after the CTA's last query position;
//     64-token chunks of 64 / PS slots) and flags the chunks every row sees
//     whole; then, per chunk, it stages the pages' scales in shared memory and
//     bulk-copies their raw K and V bytes (cp.async.bulk, mbarrier transaction
//     counts; one lane per slot and plane) into a 3-stage ring, running ahead
//     of the converters;
//   * two converter warpgroups (one 32-channel row segment per thread and
//     plane) widen the staged rows to f16 tiles, 128-byte swizzled, rows the
//     slot mask does not select written as zero, over a 3-stage ring: F16 rows
//     are copied, page-scaled FP8 / INT8 / INT4 codes are widened exactly (the
//     page scale goes to the softmax), group / channel scales and
//     INT4_RESIDUAL are applied in fp32;
//   * per chunk and query tile, S = Q . K^T (M = 128, N = 64, K = 128: 8
//     tcgen05.mma, Q f16 in TMEM as the A operand) lands in TMEM; each tile's
//     softmax warpgroup owns one TMEM lane (= one query row) per thread: it
//     applies the row masks and the causal comparison of each key's token
//     position with the row's query position (skipped for chunks seen whole),
//     multiplies in the slots' score factors, runs the online softmax in the
//     exp2 domain (S read once per chunk; lazy O rescaling) and writes P (f16,
//     times the slots' value factors) back over S;
//   * O += P . V (M = 128, N = 128, K = 64: 4 tcgen05.mma per tile, P the
//     TMEM A operand, V read MN-major) accumulates in TMEM (fp32).  The MMA
//     warp issues, per chunk, P.V of tile 0 and tile 0's next S, then the
//     same for tile 1, so one tile's softmax overlaps the other's MMAs.
// TMEM: O 2 x 128 | S/P 2 x 64 | Q 2 x 64 columns (512 allocated, one CTA per SM).
// Rows that see no key are written as 0.
//
// Reference semantics: reference.py:82-130 semantic_block_attention with the
// causal mask on original token positions of reference.py:16-45.
#include <cmath>
#include <mutex>

#include "prefill_internal.cuh"
#include "tc_ptx.cuh"

namespace iak {

__device__ unsigned int g_prefill_timeouts = 0;

int read_prefill_timeouts(unsigned int* value, bool reset) {
  unsigned int v = 0;
  int st = check_cuda(cudaMemcpyFromSymbol(&v, g_prefill_timeouts, sizeof(v)), "read prefill timeouts");
  if (st) return st;
  if (reset && v) {
    const unsigned int zero = 0;
    st = check_cuda(cudaMemcpyToSymbol(g_prefill_timeouts, &zero, sizeof(zero)), "reset prefill timeouts");
    if (st) return st;
  }
  *value = v;
  return IAK_OK;
}

namespace {

using namespace tc;

constexpr int kD = 128, kRows = 128, kChunk = 64;
constexpr int kQTiles = 2;                    // 128-row query tiles per CTA, sharing every converted K/V chunk
constexpr int kTileStages = 3, kRawStages = 3;
constexpr int kMaxSlots = 1024;
constexpr int kThreads = 576;                 // 2 softmax wgs | 2 converter wgs | producer warp | MMA warp
constexpr int kSoftWarps = 4 * kQTiles, kConvWarp0 = 8, kConvThreads = 256, kProdWarp = 16, kMmaWarp = 17;
constexpr int kKb = kChunk * 128;             // 64 token rows x 64 channels of f16 (one swizzle-atom column)
constexpr int kTile = 2 * kKb;                // 64 tokens x 128 channels
constexpr int kRawPlane = kChunk * kD * 2;    // staged bytes of one plane of a chunk (room for f16 rows)
constexpr int kRawStage = 2 * kRawPlane;      // K plane, then V plane
// TMEM columns: O of each tile | S / P of each tile | Q of each tile (f16 pairs)
constexpr int kOCol = 0, kSCol = kQTiles * kD, kQCol = kSCol + kQTiles * kChunk, kTmemCols = 512;
static_assert(kQCol + kQTiles * kD / 2 <= kTmemCols, "TMEM budget");
constexpr float kLazyLog2 = 8.f;
constexpr float kLog2e = 1.4426950408889634f;

enum {
  B_KFULL = 0,                         // converters -> MMA: K tile of a stage stored
  B_VFULL = B_KFULL + kTileStages,     // converters -> MMA: V tile of a stage stored
  B_EMPTY = B_VFULL + kTileStages,     // MMA commit after P.V -> converters: tile stage free
  B_RFULL = B_EMPTY + kTileStages,     // producer expect_tx + bulk copies -> converters: raw stage staged
  B_REMPTY = B_RFULL + kRawStages,     // converters -> producer: raw stage read
  B_SFULL = B_REMPTY + kRawStages,     // MMA commit -> softmax of a tile: S ready
  B_PFULL = B_SFULL + kQTiles,         // softmax of a tile -> MMA: P written
  B_PVDONE = B_PFULL + kQTiles,        // MMA commit -> softmax / MMA: a tile's P.V retired
  B_DONE = B_PVDONE + kQTiles,         // MMA commit: every MMA retired
  B_QREADY,                            // softmax warps -> MMA: Q rows stored in TMEM
  B_COUNT
};

struct Smem {
  static constexpr int tiles = 0;                                // tile stages x (K tile, V tile)
  static constexpr int raw = tiles + kTileStages * 2 * kTile;    // raw staging ring
  static constexpr int pid = raw + kRawStages * kRawStage;       // compacted slots: page id
  static constexpr int mask = pid + kMaxSlots * 4;               //   row mask
  static constexpr int pos0 = mask + kMaxSlots * 8;              //   token position of row 0
  static constexpr int fmt = pos0 + kMaxSlots * 4;               //   format
  static constexpr int cfull = fmt + kMaxSlots;                  // per chunk: every key visible to every row
  static constexpr int scales = cfull + kMaxSlots;               // raw stages x slots x {k, v, k res, v res} x 4
  static constexpr int fac = scales + kRawStages * 8 * 4 * 4 * 4; // tile stages x slots x {score, value} factor
  static constexpr int bars = fac + kTileStages * 8 * 2 * 4;
  static constexpr int tmem = bars + B_COUNT * 8;
  static constexpr int nvalid = tmem + 4;
  static constexpr int qmax = nvalid + 4;
  static constexpr int qmin = qmax + 4;
  static constexpr int total = qmin + 4;
};
static_assert(Smem::raw % 1024 == 0 && Smem::pid % 1024 == 0, "1024-byte alignment");
static_assert(Smem::mask % 8 == 0 && Smem::bars % 8 == 0, "8-byte alignment");
static_assert(Smem::total + 1024 <= 232448, "shared memory budget");

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// max of three (one instruction)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// packed pairs of fp32 (one instruction each, round to nearest)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n add.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mul.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Bytes of one plane of one page of format fmt as staged (row r of a slot's
// region at r * row_bytes; INT4_RESIDUAL's residual rows follow the base rows).
__device__ __forceinline__ uint32_t staged_plane_bytes(int fmt, int PS) {
  return fmt == IAK_FMT_F16 ? PS * 256u : (fmt == IAK_FMT_INT4 ? PS * 64u : PS * 128u);
}

// Page-scaled FP8 / INT8 / INT4 rows are widened to f16 without their scale, exactly:
// FP8 by bit placement (code * 2^-8), INT8 and the INT4 nibbles through the
// f16 magic number 1024 (0x6400) + the offset-binary code, then one half2
// subtraction.  The page scale (x 256 for FP8) is applied to the scores and to
// P by the softmax.
__device__ __forceinline__ uint32_t hsub_bits(uint32_t a, uint32_t b) {
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}
// 16 consecutive channels [ch0, ch0 + 16) of an FP8 / INT8 row from one 16-byte chunk w, as 8 f16
// pairs: widened exactly (fold: the page scale goes to the softmax) or times their scales in fp32.
__device__ __forceinline__ void cvt8(uint4 w4, int fmt, bool fold, int ch0, float s_all, const float* chs,
                                     uint32_t (&h)[8]) {
  const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
  if (fold) {
    if (fmt == IAK_FMT_FP8) {
#pragma unroll
      for (int i = 0; i < 4; ++i) e4m3x4_to_f16(w[i], h[2 * i], h[2 * i + 1]);
    } else {
      constexpr uint32_t kBias = 0x64806480u;    // half2(1152, 1152) = 1024 + 128
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t x = w[i] ^ 0x80808080u;  // offset binary
        h[2 * i] = hsub_bits(__byte_perm(x, 0x64646464u, 0x4140), kBias);
        h[2 * i + 1] = hsub_bits(__byte_perm(x, 0x64646464u, 0x4342), kBias);
      }
    }
    return;
  }
  auto sc = [&](int c) { return chs ? chs[ch0 + c] : s_all; };
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = 4 * i + 2 * k;
      const uint32_t pair = (w[i] >> (16 * k)) & 0xFFFFu;
      float x0, x1;
      if (fmt == IAK_FMT_FP8) {
        const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(pair), __NV_E4M3);
        const float2 f = __half22float2(__half2(hr));
        x0 = f.x; x1 = f.y;
      } else {
        x0 = static_cast<float>(static_cast<int8_t>(pair & 0xFFu));
        x1 = static_cast<float>(static_cast<int8_t>(pair >> 8));
      }
      h[c / 2] = pack_h2(x0 * sc(c), x1 * sc(c + 1));
    }
  }
}

// The 32 channels [32g, 32g + 32) of a packed INT4 row from one 16-byte chunk (4 words), plus the
// residual chunk for INT4_RESIDUAL, as 16 f16 pairs in channel order.  Word j holds channels
// 4j + {0, 2, 16, 18, 1, 3, 17, 19} in nibbles 0..7; nibbles (n, n + 4) are a channel pair.
__device__ __forceinline__ void cvt4(uint4 b4, uint4 r4, bool resid, bool fold, int g, float s_all, float rs_all,
                                     const float* chs, const float* rchs, uint32_t (&h)[16]) {
  const uint32_t base[4] = {b4.x, b4.y, b4.z, b4.w};
  if (fold) {
    constexpr uint32_t kBias4 = 0x64086408u;     // half2(1032, 1032) = 1024 + 8
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int c = 4 * j + (n & 1) * 2 + (n >> 1) * 16;
        h[c / 2] = hsub_bits(((base[j] >> (4 * n)) & 0x000F000Fu) | 0x64006400u, kBias4);
      }
    return;
  }
  const uint32_t res[4] = {r4.x, r4.y, r4.z, r4.w};
  auto sc = [&](int c) { return chs ? chs[g * 32 + c] : s_all; };
  auto rsc = [&](int c) { return rchs ? rchs[g * 32 + c] : rs_all; };
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int c = 4 * j + (n & 1) * 2 + (n >> 1) * 16;
      const int c0 = static_cast<int>((base[j] >> (4 * n)) & 0xFu) - 8;
      const int c1 = static_cast<int>((base[j] >> (4 * n + 16)) & 0xFu) - 8;
      float x0 = static_cast<float>(c0) * sc(c), x1 = static_cast<float>(c1) * sc(c + 1);
      if (resid) {
        const int r0 = static_cast<int>((res[j] >> (4 * n)) & 0xFu) - 8;
        const int r1 = static_cast<int>((res[j] >> (4 * n + 16)) & 0xFu) - 8;
        x0 += static_cast<float>(r0) * rsc(c);
        x1 += static_cast<float>(r1) * rsc(c + 1);
      }
      h[c / 2] = pack_h2(x0, x1);
    }
  }
}

template <int PS>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const PrefillParams p, int tiles) {
  constexpr int kSlotsPerChunk = kChunk / PS;
  constexpr int kSlotRaw = PS * 256;            // staged bytes reserved per slot and plane
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (sbase - raw_addr);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int tile = blockIdx.x % tiles;
  const int unit = blockIdx.x / tiles;
  const int h = unit % p.Ht, b = unit / p.Ht;
  const int64_t base = p.bases ? p.bases[static_cast<int64_t>(b) * p.Ht + h] : 0;

  int32_t* s_pid = reinterpret_cast<int32_t*>(sm + Smem::pid);
  uint64_t* s_mask = reinterpret_cast<uint64_t*>(sm + Smem::mask);
  int32_t* s_pos0 = reinterpret_cast<int32_t*>(sm + Smem::pos0);
  uint8_t* s_fmt = sm + Smem::fmt;
  volatile uint32_t* s_tmem = reinterpret_cast<volatile uint32_t*>(sm + Smem::tmem);
  volatile int* s_nvalid = reinterpret_cast<volatile int*>(sm + Smem::nvalid);
  int* s_qmax = reinterpret_cast<int*>(sm + Smem::qmax);
  int* s_qmin = reinterpret_cast<int*>(sm + Smem::qmin);
  uint8_t* s_cfull = sm + Smem::cfull;
  float* s_scales = reinterpret_cast<float*>(sm + Smem::scales);
  float* s_fac = reinterpret_cast<float*>(sm + Smem::fac);     // [tile stage][slot][score, value]
  // staged page / group scales: [raw stage][slot in chunk][k, v, k residual, v residual][group]
  auto scale_at = [&](int rs, int sl, int kind, int g) -> float* {
    return s_scales + (((rs * 8 + sl) * 4 + kind) * 4 + g);
  };
  auto bar = [&](int i) -> uint32_t { return sbase + Smem::bars + 8u * static_cast<uint32_t>(i); };
  auto tile_off = [&](int st, int plane) -> uint32_t { return Smem::tiles + (st * 2 + plane) * kTile; };
  auto raw_off = [&](int rs, int plane, int slot) -> uint32_t {
    return Smem::raw + rs * kRawStage + plane * kRawPlane + slot * kSlotRaw;
  };

  if (tid == 0) {
    for (int i = 0; i < kTileStages; ++i) {
      mbar_init(bar(B_KFULL + i), kConvThreads);
      mbar_init(bar(B_VFULL + i), kConvThreads);
      mbar_init(bar(B_EMPTY + i), 1);
    }
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(bar(B_RFULL + i), 1);
      mbar_init(bar(B_REMPTY + i), kConvThreads);
    }
    for (int k = 0; k < kQTiles; ++k) {
      mbar_init(bar(B_SFULL + k), 1);
      mbar_init(bar(B_PFULL + k), 128);
      mbar_init(bar(B_PVDONE + k), 1);
    }
    mbar_init(bar(B_DONE), 1);
    mbar_init(bar(B_QREADY), 32 * kSoftWarps);
    *s_qmax = -1;
    *s_qmin = 0x7FFFFFFF;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + Smem::tmem),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  // ---- this thread's query row (softmax warps): position, and Q into TMEM.  Query tile qt = warp / 4
  // of the CTA owns TMEM lane (warp % 4) * 32 + lane of its own O, S and Q columns.
  const int R = tile * (kQTiles * kRows) + tid;
  const int qm = R / p.G, qg = R % p.G;
  const bool row_ok = warp < kSoftWarps && qm < p.M;
  const int hq = h * p.G + qg;
  const int qt = warp >> 2;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  int qpos = -1;
  if (warp < kSoftWarps) {
    if (row_ok) {
      qpos = p.qpos ? p.qpos[static_cast<int64_t>(b) * p.qp_sb + qm] : qm;
      if (p.causal) {
        atomicMax(s_qmax, qpos);
        atomicMin(s_qmin, qpos);
      }
    }
    const int64_t qoff = b * p.q_sb + static_cast<int64_t>(hq) * p.q_sh + static_cast<int64_t>(qm) * p.q_sm;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      uint32_t v[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 x = make_uint4(0u, 0u, 0u, 0u);
        const int ch = half * 64 + c * 8;
        if (row_ok) {
          if (p.q_vec && p.q_dtype == IAK_DT_F16) {
            x = *reinterpret_cast<const uint4*>(static_cast<const __half*>(p.q) + qoff + ch);
          } else {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = load_as_float(p.q, p.q_dtype, qoff + ch + i);
            x = make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]), pack_h2(f[6], f[7]));
          }
        }
        v[4 * c] = x.x; v[4 * c + 1] = x.y; v[4 * c + 2] = x.z; v[4 * c + 3] = x.w;
      }
      tmem_st32(lane_addr + kQCol + qt * (kD / 2) + half * 32, v);
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(bar(B_QREADY));
  }
  __syncthreads();

  // ---- producer warp: compact the unit's table
  if (warp == kProdWarp) {
    const int count = prefill_count(p, b, h);
    const int32_t* row = p.pt + static_cast<int64_t>(b) * p.pt_sb + static_cast<int64_t>(h) * p.pt_sh;
    const int qmax = *s_qmax;
    int cnt = 0;
    for (int o0 = 0; o0 < count; o0 += 32) {
      const int o = o0 + lane;
      bool ok = false;
      int64_t pid = -1;
      int fmt = IAK_FMT_SKIP;
      uint64_t mask = 0;
      int64_t pos0 = 0;
      if (o < count) {
        pid = row[o];
        if (pid >= 0 && pid < p.k.num_pages) {
          fmt = prefill_fmt(p, pid);
          if (qpage::writable(p.k, fmt) && qpage::writable(p.v, fmt)) {
            mask = prefill_mask(p, b, o);
            pos0 = prefill_pos0(p, b, h, o, pid, base);
            // positions outside int32 cannot be compared with a query position: such slots are dropped
            ok = mask != 0 && pos0 >= -(1LL << 30) && pos0 < (1LL << 30);
            if (ok && p.causal) ok = pos0 + (__ffsll(static_cast<long long>(mask)) - 1) <= qmax;
          }
        }
      }
      const unsigned bal = __ballot_sync(0xffffffffu, ok);
      if (ok) {
        const int r = cnt + __popc(bal & ((1u << lane) - 1u));
        if (r < kMaxSlots) {
          s_pid[r] = static_cast<int32_t>(pid);
          s_mask[r] = mask;
          s_pos0[r] = static_cast<int32_t>(pos0);
          s_fmt[r] = static_cast<uint8_t>(fmt);
        }
      }
      cnt += __popc(bal);
    }
    const int nv = min(cnt, kMaxSlots);
    if (lane == 0) *s_nvalid = nv;
    __syncwarp();
    // chunks whose every key every row sees: all slots present, full row masks, and
    // (causal) the chunk's last key position not after the tile's first query position
    const uint64_t all = PS >= 64 ? ~0ull : ((1ull << PS) - 1ull);
    const int qmin = *s_qmin;
    for (int c = lane; c * kSlotsPerChunk < nv; c += 32) {
      bool full = true;
      for (int sl = 0; sl < kSlotsPerChunk; ++sl) {
        const int si = c * kSlotsPerChunk + sl;
        full = full && si < nv && s_mask[si] == all && (!p.causal || s_pos0[si] + PS - 1 <= qmin);
      }
      s_cfull[c] = full ? 1 : 0;
    }
  }
  __syncthreads();
  const int n_valid = *s_nvalid;
  const int T = (n_valid + kSlotsPerChunk - 1) / kSlotsPerChunk;
  bool timed_out = false;

  if (warp == kProdWarp) {
    // ---------------------------------------------------------------- producer: scales + bulk copies
    const int mode = p.k.mode, ns = p.k.ns;
    const int lg = mode == IAK_SCALE_GROUP32 ? 2 : 0;     // log2 of the groups per row (channel-mode scales
    const int ngrp = 1 << lg;                              // are read by the converters)
    // (slot, kind, group) items of a chunk's page / group scales: at most 8 x 4 x 4 = 128, 4 per lane
    constexpr int kScaleItemsPerLane = 4;
    const int n_items = mode == IAK_SCALE_CHANNEL ? 0 : kSlotsPerChunk * 4 * ngrp;
    for (int j = 0; j < T; ++j) {
      const int rs = j % kRawStages;
      // the chunk's scales are loaded before the wait for a free stage, so their latency
      // overlaps it; they are stored once the stage is free
      float sv[kScaleItemsPerLane];
#pragma unroll
      for (int q = 0; q < kScaleItemsPerLane; ++q) {
        const int it = lane + 32 * q;
        sv[q] = 0.f;
        if (it < n_items) {
          const int sl = it >> (2 + lg), kind = (it >> lg) & 3, g = it & (ngrp - 1);
          const int si = j * kSlotsPerChunk + sl;
          if (si < n_valid) {
            const int fmt = s_fmt[si];
            const float* arr = kind == 0 ? p.k.scale : (kind == 1 ? p.v.scale : (kind == 2 ? p.k.res_scale : p.v.res_scale));
            const bool need = fmt != IAK_FMT_F16 && (kind < 2 || fmt == IAK_FMT_INT4R);
            if (need && arr) sv[q] = arr[static_cast<int64_t>(s_pid[si]) * ns + g];
          }
        }
      }
      bool ok = true;
      if (lane == 0 && j >= kRawStages) ok = mbar_wait_sleep(bar(B_REMPTY + rs), ((j / kRawStages) - 1) & 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) { timed_out = true; break; }
#pragma unroll
      for (int q = 0; q < kScaleItemsPerLane; ++q) {
        const int it = lane + 32 * q;
        if (it < n_items) {
          const int sl = it >> (2 + lg), kind = (it >> lg) & 3, g = it & (ngrp - 1);
          *scale_at(rs, sl, kind, g) = sv[q];
        }
      }
      __syncwarp();
      // one lane per (slot, plane) of the chunk: lane 0 posts the byte count, then every lane
      // issues its page's bulk copy (and the residual rows of an INT4_RESIDUAL page); issued
      // from one lane, the copies of a chunk took most of the producer's time
      {
        const int sl = lane >> 1, plane = lane & 1;
        const int si = j * kSlotsPerChunk + sl;
        const bool mine = sl < kSlotsPerChunk && si < n_valid;
        int fmt = 0;
        int64_t pid = 0;
        uint32_t bytes = 0;
        const uint8_t* src = nullptr;
        if (mine) {
          fmt = s_fmt[si];
          pid = s_pid[si];
          // pool base of this page's format and plane (selected pointer by pointer: a reference
          // to one of the two by-value parameter structs would be copied to local memory)
          if (fmt == IAK_FMT_F16) {
            src = reinterpret_cast<const uint8_t*>(plane ? p.v.f16 : p.k.f16) + pid * PS * kD * 2;
            bytes = PS * 256;
          } else if (fmt == IAK_FMT_FP8) {
            src = (plane ? p.v.fp8 : p.k.fp8) + pid * PS * kD;
            bytes = PS * 128;
          } else if (fmt == IAK_FMT_INT8) {
            src = reinterpret_cast<const uint8_t*>(plane ? p.v.i8 : p.k.i8) + pid * PS * kD;
            bytes = PS * 128;
          } else {
            src = (plane ? p.v.i4 : p.k.i4) + pid * PS * (kD / 2);
            bytes = PS * 64;
          }
        }
        const uint32_t total = __reduce_add_sync(0xffffffffu, mine ? staged_plane_bytes(fmt, PS) : 0u);
        if (lane == 0) mbar_arrive_expect_tx(bar(B_RFULL + rs), total);
        __syncwarp();
        if (mine) {
          const uint32_t dst = sbase + raw_off(rs, plane, sl);
          bulk_load(dst, src, bytes, bar(B_RFULL + rs));
          if (fmt == IAK_FMT_INT4R)
            bulk_load(dst + PS * 64, (plane ? p.v.i4r : p.k.i4r) + pid * PS * (kD / 2), PS * 64, bar(B_RFULL + rs));
        }
      }
      __syncwarp();
    }
  } else if (warp >= kConvWarp0 && warp < kProdWarp) {
    // ---------------------------------------------------------------- converters: staged pages -> f16 tiles
    const int ct = tid - kConvWarp0 * 32;
    const int mode = p.k.mode, ns = p.k.ns;
    for (int j = 0; j < T && !timed_out; ++j) {
      const int st = j % kTileStages, rs = j % kRawStages;
      if (!mbar_wait_sleep(bar(B_RFULL + rs), (j / kRawStages) & 1)) { timed_out = true; break; }
      if (j >= kTileStages && !mbar_wait_sleep(bar(B_EMPTY + st), ((j / kTileStages) - 1) & 1)) {
        timed_out = true;
        break;
      }
      // per-slot score / probability factors of this chunk: pages whose codes are widened
      // without their scale (page scale mode) hand the scale to the softmax
      if (ct < 2 * kSlotsPerChunk) {
        const int sl = ct >> 1, pl = ct & 1, s2 = j * kSlotsPerChunk + sl;
        float f = 1.f;
        if (s2 < n_valid && mode == IAK_SCALE_PAGE) {
          const int f2 = s_fmt[s2];
          if (f2 == IAK_FMT_FP8 || f2 == IAK_FMT_INT8 || f2 == IAK_FMT_INT4)
            f = *scale_at(rs, sl, pl, 0) * (f2 == IAK_FMT_FP8 ? 256.f : 1.f);
        }
        s_fac[(st * 8 + sl) * 2 + pl] = f;
      }
#pragma unroll 1
      for (int plane = 0; plane < 2; ++plane) {
        const uint32_t toff = tile_off(st, plane);
        const float* scale_rows = plane ? p.v.scale : p.k.scale;
        const float* rscale_rows = plane ? p.v.res_scale : p.k.res_scale;
        {
          // this thread's unit: (token row, 32-channel group); a warp covers 8 rows of one slot,
          // so the format is warp-uniform
          const int u = ct;
          const int trow = u >> 2, g = u & 3, slot = trow / PS, r = trow % PS;
          const int si = j * kSlotsPerChunk + slot;
          const bool live = si < n_valid && ((s_mask[si] >> r) & 1ull);
          const int f = live ? s_fmt[si] : IAK_FMT_SKIP;
          const uint8_t* rawp = sm + raw_off(rs, plane, slot);
          auto put = [&](int c, uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3) {
            // 16-byte chunk c (0..15) of the tile row, 128-byte swizzled
            *reinterpret_cast<uint4*>(sm + toff + (c >> 3) * kKb + swz(trow, c & 7)) = make_uint4(x0, x1, x2, x3);
          };
          // Staged rows are 256 (F16) or 128 (8-bit) bytes apart, so a warp's eight rows share banks.
          // A 16-byte access of the warp runs in phases of 8 lanes (two rows x four groups): each
          // thread visits its chunks in an order (chunk k ^ (g >> 1) ^ 2 (r & 1) for F16, pair
          // (r & 1) ^ (g >> 1) first for 8-bit rows) under which the 8 lanes of a phase hit 8
          // distinct bank groups both in the staged rows and in the 128-byte-swizzled tile.  All
          // loads precede the stores.
          if (f == IAK_FMT_F16 || f == IAK_FMT_SKIP) {
            uint4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int kk = k ^ (g >> 1) ^ ((r & 1) << 1);
              v[k] = f == IAK_FMT_F16 ? *reinterpret_cast<const uint4*>(rawp + r * 256 + g * 64 + kk * 16)
                                      : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) put(g * 4 + (k ^ (g >> 1) ^ ((r & 1) << 1)), v[k].x, v[k].y, v[k].z, v[k].w);
          } else {
            const int64_t pid = s_pid[si];
            const bool ch = mode == IAK_SCALE_CHANNEL;
            const int grp = mode == IAK_SCALE_GROUP32 ? g : 0;
            if (f == IAK_FMT_FP8 || f == IAK_FMT_INT8) {
              const bool fold = mode == IAK_SCALE_PAGE;
              const float s_all = (fold || ch) ? 0.f : *scale_at(rs, slot, plane, grp);
              const float* chs = ch ? scale_rows + pid * ns : nullptr;
              const int k0 = (r & 1) ^ (g >> 1);
              const uint4 w0 = *reinterpret_cast<const uint4*>(rawp + r * 128 + g * 32 + k0 * 16);
              const uint4 w1 = *reinterpret_cast<const uint4*>(rawp + r * 128 + g * 32 + (k0 ^ 1) * 16);
              uint32_t h0[8], h1[8];
              cvt8(w0, f, fold, g * 32 + k0 * 16, s_all, chs, h0);
              cvt8(w1, f, fold, g * 32 + (k0 ^ 1) * 16, s_all, chs, h1);
              put(g * 4 + 2 * k0, h0[0], h0[1], h0[2], h0[3]);
              put(g * 4 + 2 * k0 + 1, h0[4], h0[5], h0[6], h0[7]);
              put(g * 4 + 2 * (k0 ^ 1), h1[0], h1[1], h1[2], h1[3]);
              put(g * 4 + 2 * (k0 ^ 1) + 1, h1[4], h1[5], h1[6], h1[7]);
            } else {
              const bool resid = f == IAK_FMT_INT4R;
              const bool fold = mode == IAK_SCALE_PAGE && !resid;
              const float s_all = (fold || ch) ? 0.f : *scale_at(rs, slot, plane, grp);
              const float rs_all = (resid && !ch) ? *scale_at(rs, slot, 2 + plane, grp) : 0.f;
              const uint4 b4 = *reinterpret_cast<const uint4*>(rawp + r * 64 + g * 16);
              const uint4 r4 = resid ? *reinterpret_cast<const uint4*>(rawp + PS * 64 + r * 64 + g * 16)
                                     : make_uint4(0u, 0u, 0u, 0u);
              uint32_t hv[16];
              cvt4(b4, r4, resid, fold, g, s_all, rs_all, ch ? scale_rows + pid * ns : nullptr,
                   (ch && resid) ? rscale_rows + pid * ns : nullptr, hv);
#pragma unroll
              for (int qd = 0; qd < 4; ++qd) put(g * 4 + qd, hv[4 * qd], hv[4 * qd + 1], hv[4 * qd + 2], hv[4 * qd + 3]);
            }
          }
        }
        fence_proxy_async();
        mbar_arrive(bar((plane ? B_VFULL : B_KFULL) + st));
      }
      mbar_arrive(bar(B_REMPTY + rs));
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop and polls every barrier; one elected lane issues the MMAs and
    // their commits, so the operands stay warp-uniform (a lane issuing alone was ~1.5x slower per
    // MMA).  The tcgen05 fence follows only the hand-offs of TMEM contents.
    {
      auto wait = [&](int b, uint32_t parity) -> bool { return __all_sync(0xffffffffu, mbar_wait(bar(b), parity)); };
      constexpr uint32_t kIdS = idesc_f16(kRows, kChunk, 0, 0);  // S = Q . K^T
      constexpr uint32_t kIdPV = idesc_f16(kRows, kD, 0, 1);     // O += P . V (V read MN-major)
      // per chunk: P.V of tile 0 and its next S, then the same for tile 1 (a tile's S columns are
      // reused once its P.V, which reads P over them, has retired), so one tile's softmax overlaps
      // the other tile's MMAs
      auto issue_s = [&](int j, int t2) -> bool {
        const int st = j % kTileStages;
        if (j >= 1 && !wait(B_PVDONE + t2, (j - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t d = tmem + kSCol + t2 * kChunk;
        if (elect_one()) {
#pragma unroll
          for (int kb = 0; kb < 2; ++kb) {
            const uint64_t bd = sw128_desc(sbase + tile_off(st, 0) + kb * kKb, 16, 1024);
#pragma unroll
            for (int t = 0; t < 4; ++t)
              mma_ts(d, tmem + kQCol + t2 * (kD / 2) + kb * 32 + t * 8, bd + (t * 2), kIdS, (kb | t) ? 1u : 0u);
          }
          mma_commit(bar(B_SFULL + t2));
        }
        __syncwarp();
        return true;
      };
      auto issue_pv = [&](int j, int t2) -> bool {
        const int st = j % kTileStages;
        if (!wait(B_PFULL + t2, j & 1)) return false;
        tc_fence_after();
        const uint64_t bd = sw128_desc(sbase + tile_off(st, 1), kKb, 1024);
        if (elect_one()) {
#pragma unroll
          for (int t = 0; t < kChunk / 16; ++t)
            mma_ts(tmem + kOCol + t2 * kD, tmem + kSCol + t2 * kChunk + t * 8, bd + ((t * 2048) >> 4), kIdPV,
                   (j > 0 || t > 0) ? 1u : 0u);
          mma_commit(bar(B_PVDONE + t2));
        }
        __syncwarp();
        return true;
      };
      if (!wait(B_QREADY, 0)) timed_out = true;
      tc_fence_after();
      if (!timed_out && T > 0) {
        if (!wait(B_KFULL + 0, 0) || !issue_s(0, 0) || !issue_s(0, 1)) timed_out = true;
      }
      for (int j = 0; j < T && !timed_out; ++j) {
        const int st = j % kTileStages, st1 = (j + 1) % kTileStages;
        if (!wait(B_VFULL + st, (j / kTileStages) & 1)) { timed_out = true; break; }
        const bool more = j + 1 < T;
        if (more && !wait(B_KFULL + st1, ((j + 1) / kTileStages) & 1)) { timed_out = true; break; }
        bool ok = true;
#pragma unroll 1
        for (int t2 = 0; t2 < kQTiles && ok; ++t2) ok = issue_pv(j, t2) && (!more || issue_s(j + 1, t2));
        if (!ok) { timed_out = true; break; }
        if (elect_one()) mma_commit(bar(B_EMPTY + st));
        __syncwarp();
      }
      if (elect_one()) mma_commit(bar(B_DONE));
      __syncwarp();
      if (!wait(B_DONE, 0)) timed_out = true;
      if (lane != 0) timed_out = false;           // counted once
    }
  } else if (warp < kSoftWarps) {
    // ---------------------------------------------------------------- softmax (one query row per thread)
    const float scale = p.sm_scale * kLog2e;
    float m_used = -INFINITY, l = 0.f;
    const uint32_t s_col = kSCol + qt * kChunk, o_col = kOCol + qt * kD;
    for (int j = 0; j < T && !timed_out; ++j) {
      bool ok = true;
      const int st = j % kTileStages;
      // S ready; the K tile barrier (already complete) orders the converters' factor writes
      if (lane == 0)
        ok = mbar_wait(bar(B_SFULL + qt), j & 1) && mbar_wait(bar(B_KFULL + st), (j / kTileStages) & 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) { timed_out = true; break; }
      tc_fence_after();
      // the chunk's S in one read; masked columns become -inf
      uint32_t r0[32], r1[32];
      tmem_ld32(lane_addr + s_col, r0);
      tmem_ld32(lane_addr + s_col + 32, r1);
      tmem_wait_ld();
      // score factor of a slot (clamped above 0 so that -inf scores stay -inf) and value factor
      auto factors = [&](int sl) -> float2 {
        const float2 f = *reinterpret_cast<const float2*>(s_fac + (st * 8 + sl) * 2);
        return make_float2(fmaxf(f.x, 1e-30f), f.y);
      };
      if (s_cfull[j] == 0) {
        // columns this row does not see (row masks, causal positions, padding slots)
        uint64_t vis = 0;
#pragma unroll
        for (int q = 0; q < kSlotsPerChunk; ++q) {
          const int si = j * kSlotsPerChunk + q;
          if (si < n_valid) {
            const int64_t lim = p.causal ? static_cast<int64_t>(qpos) - s_pos0[si] : PS - 1;   // last visible row
            const uint64_t upto = lim < 0 ? 0ull : (lim >= PS - 1 ? ~0ull : ((2ull << lim) - 1ull));
            uint64_t v = s_mask[si] & upto;
            if (PS < 64) v = (v & ((1ull << (PS & 63)) - 1ull)) << (q * PS);
            vis |= v;
          }
        }
        const uint32_t vlo = static_cast<uint32_t>(vis), vhi = static_cast<uint32_t>(vis >> 32);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (!((vlo >> c) & 1u)) r0[c] = 0xFF800000u;
          if (!((vhi >> c) & 1u)) r1[c] = 0xFF800000u;
        }
      }
      auto X = [&](int c) -> float { return __uint_as_float(c < 32 ? r0[c & 31] : r1[c & 31]); };
      float tmax_raw = -INFINITY;               // max over visible columns of score x factor (factors > 0)
#pragma unroll
      for (int q = 0; q < kSlotsPerChunk; ++q) {
        float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
        for (int r = 0; r < PS; r += 4) {
          ma = fmax3(ma, X(q * PS + r), X(q * PS + r + 1));
          mb = fmax3(mb, X(q * PS + r + 2), X(q * PS + r + 3));
        }
        tmax_raw = fmaxf(tmax_raw, fmaxf(ma, mb) * factors(q).x);
      }
      const float tmax = tmax_raw == -INFINITY ? -INFINITY : tmax_raw * scale;
      // lazy rescaling: the running max moves only when it grows by more than 2^kLazyLog2; O is
      // rescaled after P is written (the scores are no longer live then)
      float f = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_used = tmax;
      } else {
        const bool need = tmax > m_used + kLazyLog2;
        rescale = __any_sync(0xffffffffu, need);
        if (need) {
          f = exp2f(m_used - tmax);
          l *= f;
          m_used = tmax;
        }
      }
      // l sums the softmax weights; P (f16, packed over the first 32 columns of the S buffer)
      // carries them times the value factor of their slot.  A row with no visible column so far
      // (m_used = -inf) has only -inf scores here: its weights are 0.
      const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
      float2 ls = make_float2(0.f, 0.f);
#pragma unroll
      for (int g2 = 0; g2 < kChunk / 16; ++g2) {
        uint32_t pk[8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int g = 2 * g2 + h;             // 8 columns of one slot
          const float2 fv = factors((8 * g) / PS);
          const float a = scale * fv.x;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 t = ffma2(make_float2(X(8 * g + 2 * e), X(8 * g + 2 * e + 1)), make_float2(a, a),
                                   make_float2(neg_m, neg_m));
            const float2 pr = make_float2(ex2(t.x), ex2(t.y));
            ls = fadd2(ls, pr);
            const float2 pv = fmul2(pr, make_float2(fv.y, fv.y));
            pk[4 * h + e] = pack_h2(pv.x, pv.y);
          }
        }
        tmem_st8(lane_addr + s_col + g2 * 8, pk);
      }
      l += ls.x + ls.y;
      if (rescale) {
        // rescale O in TMEM: every earlier P.V must have landed
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(bar(B_PVDONE + qt), (j - 1) & 1))) {
          timed_out = true;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_addr + o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st32(lane_addr + o_col + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(B_PFULL + qt));
    }
    // ---------------------------------------------------------------- epilogue
    bool have = T > 0 && !timed_out;
    if (have) {
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + qt), (T - 1) & 1))) {
        timed_out = true;
        have = false;
      }
      tc_fence_after();
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t obase = b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh + static_cast<int64_t>(qm) * p.o_sm;
    const bool ovec = p.o_vec;
#pragma unroll 1
    for (int c = 0; c < kD / 32; ++c) {
      uint32_t o[32];
      if (have) {
        tmem_ld32(lane_addr + o_col + c * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (!row_ok) continue;
      const int64_t e0 = obase + c * 32;
      if (ovec && p.out_dtype == IAK_DT_F32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + e0);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                               __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
      } else if (ovec) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + e0);
        const bool bf = p.out_dtype == IAK_DT_BF16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float a0 = __uint_as_float(o[8 * i + 2 * k]) * inv, a1 = __uint_as_float(o[8 * i + 2 * k + 1]) * inv;
            if (bf) {
              const __nv_bfloat162 hb = __floats2bfloat162_rn(a0, a1);
              w[k] = *reinterpret_cast<const uint32_t*>(&hb);
            } else {
              w[k] = pack_h2(a0, a1);
            }
          }
          dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) store_from_float(p.out, p.out_dtype, e0 + i, __uint_as_float(o[i]) * inv);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  if (timed_out) atomicAdd(&g_prefill_timeouts, 1u);
}

template <int PS>
int launch_ps(const PrefillParams& p, cudaStream_t s) {
  const int64_t tiles = (static_cast<int64_t>(p.G) * p.M + kQTiles * kRows - 1) / (kQTiles * kRows);
  const int64_t items = static_cast<int64_t>(p.B) * p.Ht * tiles;
  if (items > 0x7FFFFFFF) return fail(IAK_ERR_UNSUPPORTED, "too many prefill work items");
  const size_t smem = Smem::total + 1024;
  static std::mutex mu;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return check_cuda(err, "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      err = cudaFuncSetAttribute(prefill_tc_kernel<PS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
      if (err != cudaSuccess) return check_cuda(err, "prefill_tc smem attribute");
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
  }
  kernel_timer_begin(s);
  prefill_tc_kernel<PS><<<static_cast<unsigned>(items), kThreads, smem, s>>>(p, static_cast<int>(tiles));
  err = cudaGetLastError();
  kernel_timer_end(s);
  return check_cuda(err, "prefill_tc launch");
}

bool aligned16(const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; }

}  // namespace

bool prefill_tc_eligible(const PrefillParams& p) {
  if (p.k.D != kD) return false;
  const int PS = p.k.PS;
  if (PS != 8 && PS != 16 && PS != 32 && PS != 64) return false;
  if (p.W > kMaxSlots) return false;
  // the softmax takes each slot's max score times a positive factor and scale
  if (!(p.sm_scale > 0.f) || !std::isfinite(p.sm_scale)) return false;
  for (const qpage::PlanePools* pl : {&p.k, &p.v})
    if (!aligned16(pl->f16) || !aligned16(pl->fp8) || !aligned16(pl->i8) || !aligned16(pl->i4) || !aligned16(pl->i4r))
      return false;
  return true;
}

int launch_prefill_tc(const PrefillParams& p, cudaStream_t s) {
  switch (p.k.PS) {
    case 8: return launch_ps<8>(p, s);
    case 16: return launch_ps<16>(p, s);
    case 32: return launch_ps<32>(p, s);
    default: return launch_ps<64>(p, s);
  }
}

}  // namespace iak
