// Tensor-core (tcgen05 / TMEM) MLA decode for the absorbed DeepSeek-V2 shape:
// d_qk = 576 (512 latent + 64 rope channels), d_v = 512, up to 128 query
// heads per sequence, latent pages of a multiple of 64 tokens, dense BF16 /
// F16 or FP8-e4m3 (per-page scale) pages.
//
// One CTA = one work item (sequence b, page range `split`, value half h):
//   * the 128 head rows are the M = 128 rows of every MMA.  Q is f16: its
//     channels [0, 256) sit in TMEM (A operand of the TS-form MMA), channels
//     [256, 576) in shared memory (K-major, 128-byte swizzle);
//   * latents are consumed in 64-token chunks of nine 64-channel k-blocks.
//     A converter warpgroup loads each k-block from global memory (the
//     producer warp bulk-prefetches chunks into L2 a few chunks ahead),
//     converts it to f16 x 2^-8 in registers (FP8 by integer bit placement,
//     exact; dense by one multiply, exact above the f16 subnormal range) and
//     stores it once, swizzled, into
//     shared memory: the 5 k-blocks outside this CTA's value half go to a
//     9-slot ring released as soon as S has read them, the 4 value k-blocks
//     to a double-buffered set held until P.V has read them;
//   * S = Q . C^T: M=128, N=64 tokens, K=576 (36 tcgen05.mma; N = 64 keeps
//     the MMA above the per-instruction floor that makes N <= 32 slow),
//     fp32 in TMEM, two S buffers.  The softmax warpgroup owns one TMEM lane
//     (= one head) per thread, so the online softmax needs no cross-thread
//     reduction; P (f16) is written back over S and is the TMEM A operand of
//     O_h += P . C[:, h*256 : h*256+256] (M=128, N=256, K=64 in 4 MMAs, the
//     value k-blocks read MN-major), O_h fp32 in TMEM;
//   * FP8 latents stay codes: the page scale multiplies the scores and P (so
//     O accumulates code x scale x weight); l sums unscaled weights;
//   * the O accumulator is rescaled lazily (only when a row max grows by
//     more than 2^8), in TMEM.
// TMEM: O_h 256 | S/P 2 x 64 | Q 128 columns (512 allocated: one CTA per SM).
// The two value halves of a (b, split) each compute S: TMEM cannot hold a
// 128 x 512 fp32 accumulator next to S.
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
constexpr int kKBlocks = kDqk / 64;                 // 64-channel k-blocks (128-byte swizzle atoms)
constexpr int kVBlocks = kHalf / 64;                // k-blocks of one value half
constexpr int kKOnly = kKBlocks - kVBlocks;         // k-blocks only S reads
constexpr int kKSlots = 9;                          // ring slots for them (more than one chunk)
constexpr int kPrefetchAhead = 4;                   // chunks prefetched into L2 ahead of the converters
constexpr int kQTmemDims = 256;                     // Q channels [0, 256) live in TMEM (A operand)
constexpr int kQTmemCols = kQTmemDims / 2;          // two f16 per 32-bit column
constexpr int kQSmemKb0 = kQTmemDims / 64;          // first Q k-block kept in shared memory
constexpr int kQSmemKbs = kKBlocks - kQSmemKb0;     // 5 blocks: channels [256, 576)
constexpr int kKbQ = kRows * 128;                   // bytes of one Q k-block (128 rows x 128 B)
constexpr int kKb = kChunk * 128;                   // bytes of one f16 latent k-block (64 rows x 128 B)
constexpr int kMaxItemPages = 512;
constexpr int kThreads = 320;                       // softmax wg | converter wg | prefetch warp | MMA warp
constexpr int kConvWarp0 = 4, kPrefWarp = 8, kMmaWarp = 9;
constexpr int kSBuf = 2;
constexpr int kOCol = 0, kSCol = kHalf, kQCol = kSCol + kSBuf * kChunk, kTmemCols = 512;
static_assert(kQCol + kQTmemCols <= kTmemCols, "TMEM budget");
constexpr float kLazyLog2 = 8.f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum {
  B_VCONV = 0,                    // value set: converters -> MMA (f16 k-blocks stored)
  B_VEMPTY = B_VCONV + 2,         // value set: MMA commit after P.V -> converters
  B_KCONV = B_VEMPTY + 2,         // ring slot: converters -> MMA
  B_KEMPTY = B_KCONV + kKSlots,   // ring slot: MMA commit after S -> converters
  B_SFULL = B_KEMPTY + kKSlots,   // MMA commit -> softmax (S ready)
  B_PFULL = B_SFULL + kSBuf,      // softmax -> MMA (P written, O rescaled)
  B_PVDONE = B_PFULL + kSBuf,     // MMA commit -> softmax / MMA (P.V done: O current, S/P buffer free)
  B_DONE = B_PVDONE + kSBuf,      // MMA commit -> MMA (all MMAs retired)
  B_QREADY,                       // softmax warps -> MMA: Q channels stored in TMEM
  B_COUNT
};

struct Smem {
  static constexpr int q = 0;                                       // Q k-blocks 4..8
  static constexpr int vset = q + kQSmemKbs * kKbQ;                 // 2 x 4 value k-blocks
  static constexpr int kring = vset + 2 * kVBlocks * kKb;           // 9 ring k-blocks
  static constexpr int pid = kring + kKSlots * kKb;
  static constexpr int pscale = pid + kMaxItemPages * 4;
  static constexpr int pfmt = pscale + kMaxItemPages * 4;
  static constexpr int bars = pfmt + kMaxItemPages;
  static constexpr int tmem = bars + B_COUNT * 8;
  static constexpr int nvalid = tmem + 4;
  static constexpr int total = nvalid + 12;
};
static_assert(Smem::vset % 1024 == 0 && Smem::kring % 1024 == 0, "1024-byte alignment");
static_assert(Smem::bars % 8 == 0, "mbarriers need 8-byte alignment");
static_assert(Smem::total + 1024 <= 232448, "shared memory budget");

// Latent tiles are stored in shared memory as f16 holding value * 2^-8 (kTileScale):
// * an e4m3 code s.eeee.mmm placed as the f16 bit pattern s.0eeee.mmm0000000 is
//   exactly code * 2^-8 for every finite code, normals and subnormals alike (e4m3
//   bias 7, f16 bias 15, both keep an implicit 1 above 0 and the same subnormal
//   scaling), so FP8 k-blocks need only integer ops, no conversion instructions;
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

// ---------------------------------------------------------------- kernel ---
// k-block order of a chunk: the blocks outside this CTA's value half ascending (ring), then the value half.
__device__ __forceinline__ int chunk_kb(int half, int i) {
  if (i >= kKOnly) return half * kVBlocks + (i - kKOnly);
  return i < half * kVBlocks ? i : i + kVBlocks;
}

__global__ void __launch_bounds__(kThreads, 1) mla_tc_kernel(const MlaParams p) {
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
  float* s_scale = reinterpret_cast<float*>(sm + Smem::pscale);
  uint8_t* s_fmt = sm + Smem::pfmt;
  volatile uint32_t* s_tmem = reinterpret_cast<volatile uint32_t*>(sm + Smem::tmem);
  volatile int* s_nvalid = reinterpret_cast<volatile int*>(sm + Smem::nvalid);
  auto bar = [&](int i) -> uint32_t { return sbase + Smem::bars + 8u * static_cast<uint32_t>(i); };
  // byte offsets (from sbase) of the f16 k-block slots
  auto vslot = [&](int set, int i) -> uint32_t { return Smem::vset + (set * kVBlocks + i) * kKb; };
  auto kslot = [&](int slot) -> uint32_t { return Smem::kring + slot * kKb; };
  const bool q_bf16 = p.q_dtype == IAK_DT_BF16;
  const uint16_t* qrow0 = static_cast<const uint16_t*>(p.q) + b * p.q_sb;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_VCONV + i), 128);
      mbar_init(bar(B_VEMPTY + i), 1);
    }
    for (int i = 0; i < kKSlots; ++i) {
      mbar_init(bar(B_KCONV + i), 128);
      mbar_init(bar(B_KEMPTY + i), 1);
    }
    for (int k = 0; k < kSBuf; ++k) {
      mbar_init(bar(B_SFULL + k), 1);
      mbar_init(bar(B_PFULL + k), 128);
      mbar_init(bar(B_PVDONE + k), 1);
    }
    mbar_init(bar(B_DONE), 1);
    mbar_init(bar(B_QREADY), 128);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + Smem::tmem),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kPrefWarp) {
    // compact this item's slice of the page table (valid ids of dense / FP8 pages, in order) with page scales
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
  if (warp >= kConvWarp0 && warp < kPrefWarp) {
    // Q channels [256, 576) as f16 in the K-major 128-byte-swizzled layout; rows >= H are zero
    const int ct = tid - kConvWarp0 * 32;
    constexpr int kChunks = kQSmemKbs * 8;   // 16-byte chunks per row kept in shared memory
#pragma unroll 8
    for (int i = 0; i < kRows * kChunks / 128; ++i) {
      const int u = ct + 128 * i, r = u / kChunks, c = u % kChunks;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < p.H)
        v = to_f16x8(*reinterpret_cast<const uint4*>(qrow0 + r * p.q_sh + kQTmemDims + c * 8), q_bf16);
      *reinterpret_cast<uint4*>(sm + Smem::q + (c >> 3) * kKbQ + swz(r, c & 7)) = v;
    }
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
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

  if (warp == kPrefWarp) {
    // ---------------------------------------------------------------- L2 prefetch, paced by the converters
    if (lane == 0) {
      auto prefetch_chunk = [&](int j) {
        const int64_t row0 = chunk_row0(j);
        if (s_fmt[j / cpp] == IAK_MLA_FP8)
          prefetch_l2(p.fp8 + row0 * kDqk, kChunk * kDqk);
        else
          prefetch_l2(static_cast<const uint16_t*>(p.dense) + row0 * kDqk, kChunk * kDqk * 2);
      };
      for (int j = 0; j < kPrefetchAhead && j < T; ++j) prefetch_chunk(j);
      for (int j = 0; j + kPrefetchAhead < T; ++j) {
        // chunk j's value set is stored: the converters have moved past it
        if (!mbar_wait_sleep(bar(B_VCONV + (j & 1)), (j >> 1) & 1)) { timed_out = true; break; }
        prefetch_chunk(j + kPrefetchAhead);
      }
    }
  } else if (warp >= kConvWarp0 && warp < kPrefWarp) {
    // ---------------------------------------------------------------- converters: global -> f16 -> shared
    const int ct = tid - kConvWarp0 * 32;
    const bool dense_bf16 = p.dense_dtype == IAK_DT_BF16;
    // FP8: one 16-byte load = 16 codes of a row = two f16 chunks; 256 loads per k-block (2 per thread)
    // dense: one 16-byte load = one f16 chunk; 512 loads per k-block (4 per thread)
    auto load_fp8 = [&](const uint8_t* rows, int kb, uint4 (&x)[2]) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int u = ct + 128 * i, r = u >> 2, q = u & 3;
        x[i] = *reinterpret_cast<const uint4*>(rows + r * kDqk + kb * 64 + q * 16);
      }
    };
    auto store_fp8 = [&](uint32_t off, const uint4 (&x)[2]) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int u = ct + 128 * i, r = u >> 2, q = u & 3;
        const uint32_t w[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 v;
          e4m3x4_to_f16(w[2 * h], v.x, v.y);
          e4m3x4_to_f16(w[2 * h + 1], v.z, v.w);
          *reinterpret_cast<uint4*>(sm + off + swz(r, 2 * q + h)) = v;
        }
      }
    };
    auto load_dense = [&](const uint16_t* rows, int kb, uint4 (&x)[4]) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int u = ct + 128 * i, r = u >> 3, c = u & 7;
        x[i] = *reinterpret_cast<const uint4*>(rows + r * kDqk + kb * 64 + c * 8);
      }
    };
    auto store_dense = [&](uint32_t off, const uint4 (&x)[4]) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int u = ct + 128 * i, r = u >> 3, c = u & 7;
        const uint4 y = x[i];
        *reinterpret_cast<uint4*>(sm + off + swz(r, c)) =
            dense_bf16 ? make_uint4(bf16x2_to_f16x2(y.x, kTileScale), bf16x2_to_f16x2(y.y, kTileScale),
                                    bf16x2_to_f16x2(y.z, kTileScale), bf16x2_to_f16x2(y.w, kTileScale))
                       : make_uint4(f16x2_tile_scale(y.x), f16x2_tile_scale(y.y), f16x2_tile_scale(y.z),
                                    f16x2_tile_scale(y.w));
      }
    };
    // Per chunk: issue the global loads of every k-block first (FP8: all nine; dense: the five ring
    // blocks, then the four value blocks), then wait for each destination slot and store.
    int ring_c = 0;     // ring slot uses so far (5 per chunk)
    for (int j = 0; j < T && !timed_out; ++j) {
      const int vs = j & 1;
      const int pg = j / cpp;
      const bool fp8 = s_fmt[pg] == IAK_MLA_FP8;
      const int64_t row0 = static_cast<int64_t>(s_pid[pg]) * p.PS + (j - pg * cpp) * kChunk;
      auto ring_store = [&](int i, auto&& store) -> bool {
        const int c = ring_c + i, ks = c % kKSlots;
        if (c >= kKSlots && !mbar_wait_sleep(bar(B_KEMPTY + ks), ((c / kKSlots) - 1) & 1)) return false;
        store(kslot(ks));
        fence_proxy_async();
        mbar_arrive(bar(B_KCONV + ks));
        return true;
      };
      bool ok = true;
      if (fp8) {
        const uint8_t* rows = p.fp8 + row0 * kDqk;
        uint4 x[kKBlocks][2];
#pragma unroll
        for (int i = 0; i < kKBlocks; ++i) load_fp8(rows, chunk_kb(half, i), x[i]);
#pragma unroll
        for (int i = 0; i < kKOnly; ++i)
          if (ok) ok = ring_store(i, [&](uint32_t off) { store_fp8(off, x[i]); });
        if (ok && j >= 2) ok = mbar_wait_sleep(bar(B_VEMPTY + vs), ((j >> 1) - 1) & 1);
        if (ok) {
#pragma unroll
          for (int i = 0; i < kVBlocks; ++i) store_fp8(vslot(vs, i), x[kKOnly + i]);
        }
      } else {
        const uint16_t* rows = static_cast<const uint16_t*>(p.dense) + row0 * kDqk;
        {
          uint4 x[kKOnly][4];
#pragma unroll
          for (int i = 0; i < kKOnly; ++i) load_dense(rows, chunk_kb(half, i), x[i]);
#pragma unroll
          for (int i = 0; i < kKOnly; ++i)
            if (ok) ok = ring_store(i, [&](uint32_t off) { store_dense(off, x[i]); });
        }
        if (ok) {
          uint4 x[kVBlocks][4];
#pragma unroll
          for (int i = 0; i < kVBlocks; ++i) load_dense(rows, chunk_kb(half, kKOnly + i), x[i]);
          if (j >= 2) ok = mbar_wait_sleep(bar(B_VEMPTY + vs), ((j >> 1) - 1) & 1);
          if (ok) {
#pragma unroll
            for (int i = 0; i < kVBlocks; ++i) store_dense(vslot(vs, i), x[i]);
          }
        }
      }
      if (!ok) { timed_out = true; break; }
      fence_proxy_async();
      mbar_arrive(bar(B_VCONV + vs));
      ring_c += kKOnly;
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop and polls every barrier; one elected lane issues the MMAs and
    // their commits, so the operands stay warp-uniform.
    {
      constexpr uint32_t kIdS = idesc_f16(kRows, kChunk, 0, 0);  // S = Q . C^T
      constexpr uint32_t kIdPV = idesc_f16(kRows, kHalf, 0, 1);  // O += P . C (value blocks read MN-major)
      const uint64_t q_desc0 = sw128_desc(sbase + Smem::q, 16, 1024);
      auto wait = [&](int b, uint32_t parity) -> bool { return __all_sync(0xffffffffu, mbar_wait(bar(b), parity)); };
      // S MMAs over one k-block: A = Q block kb (TMEM for kb < 4, else shared), B = the latent block
      auto s_block = [&](uint32_t d, int kb, uint32_t blk_off, bool first) {
        const uint64_t bd = sw128_desc(sbase + blk_off, 16, 1024);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t acc = (first && t == 0) ? 0u : 1u;
          if (kb < kQSmemKb0)
            mma_ts(d, tmem + kQCol + kb * 32 + t * 8, bd + (t * 2), kIdS, acc);
          else
            mma_ss(d, q_desc0 + (((kb - kQSmemKb0) * kKbQ + t * 32) >> 4), bd + (t * 2), kIdS, acc);
        }
      };
      if (!wait(B_QREADY, 0)) timed_out = true;
      auto issue_s = [&](int j) -> bool {
        const int k = j & 1, vs = j & 1;
        if (j >= kSBuf && !wait(B_PVDONE + k, ((j >> 1) - 1) & 1)) return false;
        const uint32_t d = tmem + kSCol + k * kChunk;
        for (int i = 0; i < kKOnly; ++i) {
          const int c = kKOnly * j + i, ks = c % kKSlots;
          if (!wait(B_KCONV + ks, (c / kKSlots) & 1)) return false;
          tc_fence_after();
          if (elect_one()) {
            s_block(d, chunk_kb(half, i), kslot(ks), i == 0);
            mma_commit(bar(B_KEMPTY + ks));
          }
          __syncwarp();
        }
        if (!wait(B_VCONV + vs, (j >> 1) & 1)) return false;
        tc_fence_after();
        if (elect_one()) {
          for (int i = 0; i < kVBlocks; ++i) s_block(d, chunk_kb(half, kKOnly + i), vslot(vs, i), false);
          mma_commit(bar(B_SFULL + k));
        }
        __syncwarp();
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int k = j & 1, vs = j & 1;
        if (!wait(B_PFULL + k, (j >> 1) & 1)) return false;
        tc_fence_after();
        const uint64_t bd = sw128_desc(sbase + vslot(vs, 0), kKb, 1024);
        if (elect_one()) {
#pragma unroll
          for (int t = 0; t < kChunk / 16; ++t)
            mma_ts(tmem + kOCol, tmem + kSCol + k * kChunk + t * 8, bd + ((t * 2048) >> 4), kIdPV,
                   (j > 0 || t > 0) ? 1u : 0u);
          mma_commit(bar(B_PVDONE + k));
          mma_commit(bar(B_VEMPTY + vs));
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
  } else {
    // ---------------------------------------------------------------- softmax (warps 0-3, one head row per thread)
    const int r = tid;                                   // TMEM lane = head row
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    {
      // Q channels [0, 256) of this row into TMEM columns kQCol.. (f16 pairs), the A operand of S
      const uint16_t* qr = qrow0 + r * p.q_sh;
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
    const float base_scale = p.sm_scale * kLog2e / kTileScale;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < T && !timed_out; ++j) {
      const int k = j & 1;
      // warp-uniform outcome: the TMEM loads below are warp-collective
      // one lane polls; the outcome is broadcast (warp-uniform: the TMEM loads below are warp-collective)
      bool ok = true;
      if (lane == 0) ok = mbar_wait(bar(B_SFULL + k), (j >> 1) & 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) { timed_out = true; break; }
      tc_fence_after();
      // FP8 latents hold codes: the page scale multiplies the scores (key side)
      // and P (value side); l stays in unscaled softmax weights
      const float vs = s_scale[j / cpp];
      const float sc = base_scale * vs;
      float x[kChunk], tmax = -INFINITY;
      {
        uint32_t sr[2][32];
        tmem_ld32(lane_addr + kSCol + k * kChunk, sr[0]);
        tmem_ld32(lane_addr + kSCol + k * kChunk + 32, sr[1]);
        tmem_wait_ld();
        float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          x[i] = __uint_as_float(sr[i >> 5][i & 31]);
          if (i & 1) mb = fmaxf(mb, x[i]);
          else ma = fmaxf(ma, x[i]);
        }
        // sc > 0: the max of the scaled scores is the scaled max
        tmax = fmaxf(ma, mb) * sc;
      }
      if (j == 0) {
        m_used = tmax;
      } else {
        const bool need = tmax > m_used + kLazyLog2;
        if (__any_sync(0xffffffffu, need)) {
          // rescale O_h in TMEM: every earlier P.V must have landed
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
      const int d0 = half * kHalf + c * 32;
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
  mla_tc_kernel<<<static_cast<unsigned>(items), kThreads, smem, s>>>(p);
  err = cudaGetLastError();
  kernel_timer_end(s);
  return check_cuda(err, "mla_tc launch");
}

}  // namespace iak
