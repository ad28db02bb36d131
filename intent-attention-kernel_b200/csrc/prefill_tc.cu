// Tensor-core (tcgen05 / TMEM) multi-query attention over selected pages, for
// head_dim 128 and page sizes 8..64 (any page format of the pools).
//
// One CTA = one work item (sequence b, page-table head h, tile of 128 query
// rows).  Rows are (query m, head g of the group) pairs, m-major, so a tile
// holds 128 / G consecutive queries of the G query heads sharing the table.
//   * the planner warp compacts the unit's table into shared memory: slots
//     with a page in a supported format, a non-empty row mask and (causal) a
//     first selected row not after the tile's last query position; the
//     compacted slots form 64-token chunks (64 / PS slots each);
//   * a converter warpgroup dequantises each chunk's K and V rows (code x
//     scale, fp32) to f16 into shared memory, 128-byte swizzled, rows the slot
//     mask does not select written as zero, over a 3-stage ring;
//   * S = Q . K^T (M = 128, N = 64, K = 128: 8 tcgen05.mma, Q f16 in shared
//     memory) lands in TMEM; the softmax warpgroup owns one TMEM lane (= one
//     query row) per thread: it applies the row masks and the causal
//     comparison of each key's token position with the row's query position,
//     runs the online softmax in the exp2 domain with lazy O rescaling, and
//     writes P (f16) back over S;
//   * O += P . V (M = 128, N = 128, K = 64: 4 tcgen05.mma, P the TMEM A
//     operand, V read MN-major) accumulates in TMEM (fp32).
// TMEM: O 128 | S/P 2 x 64 columns.  Rows that see no key are written as 0.
//
// Reference semantics: reference.py:82-130 semantic_block_attention with the
// causal mask on original token positions of reference.py:16-45.
#include <mutex>

#include "prefill_internal.cuh"
#include "tc_ptx.cuh"

namespace iak {

__device__ unsigned int g_prefill_timeouts = 0;

namespace {

using namespace tc;

constexpr int kD = 128, kRows = 128, kChunk = 64;
constexpr int kStages = 3;
constexpr int kMaxSlots = 4096;
constexpr int kThreads = 320;                 // softmax wg | converter wg | planner warp | MMA warp
constexpr int kConvWarp0 = 4, kPlanWarp = 8, kMmaWarp = 9;
constexpr int kKb = kChunk * 128;             // 64 token rows x 64 channels of f16 (one swizzle-atom column)
constexpr int kKbQ = kRows * 128;             // 128 query rows x 64 channels
constexpr int kTile = 2 * kKb;                // 64 tokens x 128 channels
constexpr int kSBuf = 2;
constexpr int kOCol = 0, kSCol = kD, kTmemCols = 256;
constexpr float kLazyLog2 = 8.f;
constexpr float kLog2e = 1.4426950408889634f;

enum {
  B_KFULL = 0,                     // converters -> MMA: K tile of a stage stored
  B_VFULL = B_KFULL + kStages,     // converters -> MMA: V tile of a stage stored
  B_EMPTY = B_VFULL + kStages,     // MMA commit after P.V -> converters: stage free
  B_SFULL = B_EMPTY + kStages,     // MMA commit -> softmax: S ready
  B_PFULL = B_SFULL + kSBuf,       // softmax -> MMA: P written
  B_PVDONE = B_PFULL + kSBuf,      // MMA commit -> softmax / MMA: P.V retired
  B_DONE = B_PVDONE + kSBuf,       // MMA commit: every MMA retired
  B_COUNT
};

struct Smem {
  static constexpr int q = 0;                                   // 2 Q k-blocks
  static constexpr int kv = q + 2 * kKbQ;                       // stages x (K tile, V tile)
  static constexpr int pid = kv + kStages * 2 * kTile;          // compacted slots: page id
  static constexpr int mask = pid + kMaxSlots * 4;              //   row mask
  static constexpr int pos0 = mask + kMaxSlots * 8;             //   token position of row 0
  static constexpr int fmt = pos0 + kMaxSlots * 4;              //   format
  static constexpr int bars = fmt + kMaxSlots;
  static constexpr int tmem = bars + B_COUNT * 8;
  static constexpr int nvalid = tmem + 4;
  static constexpr int qmax = nvalid + 4;
  static constexpr int total = qmax + 8;
};
static_assert(Smem::kv % 1024 == 0 && Smem::pid % 1024 == 0, "1024-byte alignment");
static_assert(Smem::mask % 8 == 0 && Smem::bars % 8 == 0, "8-byte alignment");
static_assert(Smem::total + 1024 <= 232448, "shared memory budget");

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Channels [32g, 32g + 32) of row r of pool page pid, dequantised (code x
// scale in fp32) and packed as 16 f16 pairs in channel order.
__device__ __forceinline__ void load_group(const qpage::PlanePools& q, int fmt, int64_t pid, int r, int g,
                                           uint32_t (&h)[16]) {
  const int64_t row = pid * q.PS + r;
  if (fmt == IAK_FMT_F16) {
    const uint4* src = reinterpret_cast<const uint4*>(q.f16 + row * kD + g * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 x = src[i];
      h[4 * i] = x.x; h[4 * i + 1] = x.y; h[4 * i + 2] = x.z; h[4 * i + 3] = x.w;
    }
    return;
  }
  const float* sp = q.scale + pid * q.ns;
  const float* rsp = q.res_scale ? q.res_scale + pid * q.ns : nullptr;
  const bool per_ch = q.mode == IAK_SCALE_CHANNEL;
  const float s_all = per_ch ? 0.f : sp[q.mode == IAK_SCALE_GROUP32 ? g : 0];
  auto sc = [&](int c) { return per_ch ? sp[g * 32 + c] : s_all; };
  if (fmt == IAK_FMT_FP8 || fmt == IAK_FMT_INT8) {
    const uint4* src = reinterpret_cast<const uint4*>((fmt == IAK_FMT_FP8 ? q.fp8 : reinterpret_cast<const uint8_t*>(q.i8)) +
                                                      row * kD + g * 32);
    const uint4 a = src[0], b = src[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
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
    return;
  }
  // packed INT4 (+ residual): word j of the group holds channels 4j + {0, 2, 16, 18, 1, 3, 17, 19}
  // in nibbles 0..7, offset-binary; nibbles (n, n + 4) are the channel pair (d, d + 1)
  const uint4 bw = *reinterpret_cast<const uint4*>(q.i4 + row * (kD / 2) + g * 16);
  const uint32_t base[4] = {bw.x, bw.y, bw.z, bw.w};
  uint32_t res[4] = {0u, 0u, 0u, 0u};
  const bool resid = fmt == IAK_FMT_INT4R;
  if (resid) {
    const uint4 rw = *reinterpret_cast<const uint4*>(q.i4r + row * (kD / 2) + g * 16);
    res[0] = rw.x; res[1] = rw.y; res[2] = rw.z; res[3] = rw.w;
  }
  const float rs_all = (resid && !per_ch) ? rsp[q.mode == IAK_SCALE_GROUP32 ? g : 0] : 0.f;
  auto rsc = [&](int c) { return per_ch ? rsp[g * 32 + c] : rs_all; };
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int c = 4 * j + (n & 1) * 2 + (n >> 1) * 16;      // first channel of the pair
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
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (sbase - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int tile = blockIdx.x % tiles;
  const int unit = blockIdx.x / tiles;
  const int h = unit % p.Ht, b = unit / p.Ht;
  const int64_t base = p.bases ? p.bases[static_cast<int64_t>(b) * p.Ht + h] : 0;

  int32_t* s_pid = reinterpret_cast<int32_t*>(sm + Smem::pid);
  uint64_t* s_mask = reinterpret_cast<uint64_t*>(sm + Smem::mask);
  uint8_t* s_fmt = sm + Smem::fmt;
  int32_t* s_pos0 = reinterpret_cast<int32_t*>(sm + Smem::pos0);
  volatile uint32_t* s_tmem = reinterpret_cast<volatile uint32_t*>(sm + Smem::tmem);
  volatile int* s_nvalid = reinterpret_cast<volatile int*>(sm + Smem::nvalid);
  int* s_qmax = reinterpret_cast<int*>(sm + Smem::qmax);
  auto bar = [&](int i) -> uint32_t { return sbase + Smem::bars + 8u * static_cast<uint32_t>(i); };
  auto tile_off = [&](int st, int plane) -> uint32_t { return Smem::kv + (st * 2 + plane) * kTile; };

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar(B_KFULL + i), 128);
      mbar_init(bar(B_VFULL + i), 128);
      mbar_init(bar(B_EMPTY + i), 1);
    }
    for (int k = 0; k < kSBuf; ++k) {
      mbar_init(bar(B_SFULL + k), 1);
      mbar_init(bar(B_PFULL + k), 128);
      mbar_init(bar(B_PVDONE + k), 1);
    }
    mbar_init(bar(B_DONE), 1);
    *s_qmax = -1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + Smem::tmem),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();

  // ---- this thread's query row (softmax warps): position, and Q into shared memory
  const int R = tile * kRows + tid;
  const int qm = R / p.G, qg = R % p.G;
  const bool row_ok = warp < 4 && qm < p.M;
  const int hq = h * p.G + qg;
  int qpos = -1;
  if (warp < 4) {
    if (row_ok) {
      qpos = p.qpos ? p.qpos[static_cast<int64_t>(b) * p.qp_sb + qm] : qm;
      if (p.causal) atomicMax(s_qmax, qpos);
    }
    const int64_t qoff = b * p.q_sb + static_cast<int64_t>(hq) * p.q_sh + static_cast<int64_t>(qm) * p.q_sm;
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row_ok) {
        if (p.q_vec && p.q_dtype == IAK_DT_F16) {
          v = *reinterpret_cast<const uint4*>(static_cast<const __half*>(p.q) + qoff + c * 8);
        } else {
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = load_as_float(p.q, p.q_dtype, qoff + c * 8 + i);
          v = make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]), pack_h2(f[6], f[7]));
        }
      }
      *reinterpret_cast<uint4*>(sm + Smem::q + (c >> 3) * kKbQ + swz(tid, c & 7)) = v;
    }
    fence_proxy_async();
  }
  __syncthreads();

  // ---- planner: compact the unit's table
  if (warp == kPlanWarp) {
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
    if (lane == 0) *s_nvalid = min(cnt, kMaxSlots);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_valid = *s_nvalid;
  const int T = (n_valid + kSlotsPerChunk - 1) / kSlotsPerChunk;
  bool timed_out = false;

  if (warp >= kConvWarp0 && warp < kPlanWarp) {
    // ---------------------------------------------------------------- converters: pools -> f16 tiles
    const int ct = tid - kConvWarp0 * 32;
    for (int j = 0; j < T && !timed_out; ++j) {
      const int st = j % kStages, use = j / kStages;
      if (j >= kStages && !mbar_wait_sleep(bar(B_EMPTY + st), (use - 1) & 1)) { timed_out = true; break; }
#pragma unroll 1
      for (int plane = 0; plane < 2; ++plane) {
        const qpage::PlanePools pl = plane ? p.v : p.k;
        const uint32_t toff = tile_off(st, plane);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int u = ct + 128 * i;              // 256 units: 64 token rows x 4 groups of 32 channels
          const int trow = u >> 2, g = u & 3;
          const int si = j * kSlotsPerChunk + trow / PS, r = trow % PS;
          uint32_t hv[16];
          if (si < n_valid && ((s_mask[si] >> r) & 1ull)) {
            load_group(pl, s_fmt[si], s_pid[si], r, g, hv);
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) hv[k] = 0u;
          }
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) {
            const int c = g * 4 + qd;               // 16-byte chunk index of the row (0..15)
            *reinterpret_cast<uint4*>(sm + toff + (c >> 3) * kKb + swz(trow, c & 7)) =
                make_uint4(hv[4 * qd], hv[4 * qd + 1], hv[4 * qd + 2], hv[4 * qd + 3]);
          }
        }
        fence_proxy_async();
        mbar_arrive(bar((plane ? B_VFULL : B_KFULL) + st));
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(kRows, kChunk, 0, 0);  // S = Q . K^T
      constexpr uint32_t kIdPV = idesc_f16(kRows, kD, 0, 1);     // O += P . V (V read MN-major)
      const uint64_t q_desc = sw128_desc(sbase + Smem::q, 16, 1024);
      auto issue_s = [&](int j) -> bool {
        const int k = j & 1, st = j % kStages;
        if (j >= kSBuf && !mbar_wait(bar(B_PVDONE + k), ((j >> 1) - 1) & 1)) return false;
        if (!mbar_wait(bar(B_KFULL + st), (j / kStages) & 1)) return false;
        tc_fence_after();
        const uint32_t d = tmem + kSCol + k * kChunk;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t bd = sw128_desc(sbase + tile_off(st, 0) + kb * kKb, 16, 1024);
#pragma unroll
          for (int t = 0; t < 4; ++t)
            mma_ss(d, q_desc + ((kb * kKbQ + t * 32) >> 4), bd + (t * 2), kIdS, (kb | t) ? 1u : 0u);
        }
        mma_commit(bar(B_SFULL + k));
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int k = j & 1, st = j % kStages;
        if (!mbar_wait(bar(B_PFULL + k), (j >> 1) & 1)) return false;
        if (!mbar_wait(bar(B_VFULL + st), (j / kStages) & 1)) return false;
        tc_fence_after();
        const uint64_t bd = sw128_desc(sbase + tile_off(st, 1), kKb, 1024);
#pragma unroll
        for (int t = 0; t < kChunk / 16; ++t)
          mma_ts(tmem + kOCol, tmem + kSCol + k * kChunk + t * 8, bd + ((t * 2048) >> 4), kIdPV,
                 (j > 0 || t > 0) ? 1u : 0u);
        mma_commit(bar(B_PVDONE + k));
        mma_commit(bar(B_EMPTY + st));
        return true;
      };
      if (T > 0 && !issue_s(0)) timed_out = true;
      for (int j = 0; j < T && !timed_out; ++j) {
        if (j + 1 < T && !issue_s(j + 1)) { timed_out = true; break; }
        if (!issue_pv(j)) { timed_out = true; break; }
      }
      mma_commit(bar(B_DONE));
      if (!mbar_wait(bar(B_DONE), 0)) timed_out = true;
    }
  } else if (warp < 4) {
    // ---------------------------------------------------------------- softmax (one query row per thread)
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float scale = p.sm_scale * kLog2e;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < T && !timed_out; ++j) {
      const int k = j & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait_sleep(bar(B_SFULL + k), (j >> 1) & 1);
      if (!__shfl_sync(0xffffffffu, ok, 0)) { timed_out = true; break; }
      tc_fence_after();
      float x[kChunk];
      float tmax = -INFINITY;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t sr[32];
        tmem_ld32(lane_addr + kSCol + k * kChunk + h2 * 32, sr);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) x[h2 * 32 + i] = __uint_as_float(sr[i]) * scale;
      }
#pragma unroll
      for (int sl = 0; sl < kSlotsPerChunk; ++sl) {
        const int si = j * kSlotsPerChunk + sl;
        uint64_t mask = 0;
        int64_t lim = -1;                       // last visible row offset within the page
        if (si < n_valid) {
          mask = s_mask[si];
          lim = p.causal ? static_cast<int64_t>(qpos) - s_pos0[si] : static_cast<int64_t>(PS);
        }
#pragma unroll
        for (int r = 0; r < PS; ++r) {
          const bool vis = ((mask >> r) & 1ull) && r <= lim;
          const int c = sl * PS + r;
          x[c] = vis ? x[c] : -INFINITY;
          tmax = fmaxf(tmax, x[c]);
        }
      }
      if (j == 0) {
        m_used = tmax;
      } else {
        const bool need = tmax > m_used + kLazyLog2;
        if (__any_sync(0xffffffffu, need)) {
          // rescale O in TMEM: every earlier P.V must have landed
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
          for (int c = 0; c < kD / 32; ++c) {
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
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < kChunk / 2; ++i) {
        const float p0 = x[2 * i] != -INFINITY ? exp2f(x[2 * i] - m_used) : 0.f;
        const float p1 = x[2 * i + 1] != -INFINITY ? exp2f(x[2 * i + 1] - m_used) : 0.f;
        lsum += p0 + p1;
        pk[i] = pack_h2(p0, p1);
      }
      l += lsum;
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
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t obase = b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh + static_cast<int64_t>(qm) * p.o_sm;
#pragma unroll 1
    for (int c = 0; c < kD / 32; ++c) {
      uint32_t o[32];
      if (have) {
        tmem_ld32(lane_addr + kOCol + c * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (!row_ok) continue;
#pragma unroll
      for (int i = 0; i < 32; ++i) store_from_float(p.out, p.out_dtype, obase + c * 32 + i, __uint_as_float(o[i]) * inv);
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
  const int64_t tiles = (static_cast<int64_t>(p.G) * p.M + kRows - 1) / kRows;
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
