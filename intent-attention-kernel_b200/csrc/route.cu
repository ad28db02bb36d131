// Device router.  Per sequence: the block routing of block_router.py:101-266
// (route_layout) with the precision policy of intent_quant.py:77-131
// (assign_block_precision), the page list of block_router.py:283-296
// (selected_page_ids) and the page precision map of :383-421
// (routing_to_kernel_metadata), written straight into packed page-table rows.
//
// One CTA per sequence.  The per-block state lives in shared memory sized for
// the longest layout of the launch: sort keys (ordered score bits; rank r is
// the r-th scored ATTEND block in descending score, ties in layout order, found
// by counting for layouts of up to 1024 blocks and by a bitonic sort of
// (key, index) pairs above that), routed positions, precisions and a scan
// scratch array.  Routed positions come from three CTA-wide exclusive
// scans (pinned blocks in layout order, the selected top-k in rank order,
// selected SKIP-policy blocks in layout order); a fourth scan over the
// per-block counts of first-occurrence pages gives every block its output
// offset.  Pages strictly inside a block belong to it alone (blocks do not
// overlap), so only a block's first and last page need the first-occurrence
// test against its neighbours that share that page.
#include <cmath>
#include <cstring>

#include "iak_internal.cuh"

namespace iak {
namespace {

constexpr int kRouteThreads = 1024;
constexpr int kMaxBlocks = IAK_ROUTE_MAX_BLOCKS;
constexpr uint64_t kNoKey = ~0ull;

// Shared-memory bytes per block slot: sort key (8) + sort index (4) + position
// (4) + scan scratch (4) + precision (1).
constexpr size_t kSlotBytes = 21;

// IntentQuantizer.assign_block_precision (intent_quant.py:77-131); the
// comparisons are made in double precision as Python makes them.
__device__ int block_precision(const iak_route_args& p, int policy, double score) {
  const double mp = p.memory_pressure;
  if (policy == IAK_POLICY_ALWAYS || policy == IAK_POLICY_GLOBAL) {
    if (policy == IAK_POLICY_GLOBAL && p.preserve_global) return mp > 0.8 ? IAK_PREC_INT8 : IAK_PREC_FP16;
    if (mp > 0.9) return IAK_PREC_INT8;
    if (mp > 0.7) return IAK_PREC_FP8;
    return IAK_PREC_FP16;
  }
  if (policy == IAK_POLICY_RECENT) {
    if (p.preserve_recent) return mp > 0.8 ? IAK_PREC_INT8 : IAK_PREC_FP8;
    return mp > 0.6 ? IAK_PREC_INT4_RESIDUAL : IAK_PREC_INT8;
  }
  if (policy == IAK_POLICY_ATTEND) {
    if (isnan(score)) return mp > 0.5 ? IAK_PREC_INT8 : IAK_PREC_FP16;
    if (score >= p.high_score_threshold) {
      if (mp > 0.8) return IAK_PREC_INT8;
      if (mp > 0.5) return IAK_PREC_FP8;
      return IAK_PREC_INT8;
    }
    if (score >= p.medium_score_threshold) return mp > 0.6 ? IAK_PREC_INT4 : IAK_PREC_INT4_RESIDUAL;
    return mp > 0.3 ? IAK_PREC_SKIP : IAK_PREC_INT4;
  }
  if (policy == IAK_POLICY_SKIP) return IAK_PREC_SKIP;
  return IAK_PREC_FP16;
}

// Key that sorts ascending in descending score order.  -0.0 and +0.0 compare
// equal in Python, so both map to the key of +0.0.  Never equals kNoKey for a
// non-NaN score.
__device__ __forceinline__ uint64_t descending_key(double s) {
  if (s == 0.0) s = 0.0;
  const uint64_t u = static_cast<uint64_t>(__double_as_longlong(s));
  const uint64_t ordered = (u >> 63) ? ~u : (u | (1ull << 63));
  return ~ordered;
}

// Exclusive prefix sum of data[0, n) (n <= kMaxBlocks) by the whole CTA, in
// place; returns the total.  Thread t owns the 8 consecutive elements from 8t.
__device__ int cta_exclusive_scan(int* data, int n, int* warp_sums) {
  constexpr int kPer = kMaxBlocks / kRouteThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int base = tid * kPer;
  int v[kPer];
  int local = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    v[k] = base + k < n ? data[base + k] : 0;
    local += v[k];
  }
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += t;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_sums[lane];
    int wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += t;
    }
    warp_sums[lane] = wi - w;
    if (lane == 31) warp_sums[32] = wi;
  }
  __syncthreads();
  int run = warp_sums[warp] + incl - local;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    if (base + k < n) data[base + k] = run;
    run += v[k];
  }
  const int total = warp_sums[32];
  __syncthreads();
  return total;
}

__device__ __forceinline__ bool is_pinned(int policy) {
  return policy == IAK_POLICY_ALWAYS || policy == IAK_POLICY_GLOBAL || policy == IAK_POLICY_RECENT;
}

__global__ void __launch_bounds__(kRouteThreads) route_kernel(const iak_route_args p, int slots) {
  extern __shared__ __align__(16) unsigned char rsm[];
  uint64_t* key = reinterpret_cast<uint64_t*>(rsm);          // [slots]
  int* kidx = reinterpret_cast<int*>(key + slots);            // [slots]
  int* pos = kidx + slots;                                    // [slots] routed position or -1
  int* work = pos + slots;                                    // [slots]
  uint8_t* prec = reinterpret_cast<uint8_t*>(work + slots);   // [slots]
  __shared__ int warp_sums[33];
  __shared__ int n_scored;

  const int b = blockIdx.x, tid = threadIdx.x;
  const int Ht = p.num_table_heads, W = p.table_width, PS = p.page_size;
  const int64_t lo = static_cast<int64_t>(b) * p.layout_stride;
  const int32_t* bstart = p.block_start + lo;
  const int32_t* bend = p.block_end + lo;
  const uint8_t* bpol = p.block_policy + lo;
  const double* sc = p.scores + static_cast<int64_t>(b) * p.score_stride;
  const int n = p.block_counts ? p.block_counts[b] : p.num_blocks;
  const int32_t seq_len = p.seq_lens ? p.seq_lens[b] : 0x7FFFFFFF;
  if (tid == 0) n_scored = 0;

  // ---- BlockLayout.validate, on the device --------------------------------
  bool bad = n < 0 || n > p.num_blocks;
  if (!bad) {
    for (int i = tid; i < n; i += kRouteThreads) {
      const int s = bstart[i], e = bend[i], pol = bpol[i];
      bool ok = s >= 0 && e > s && e <= seq_len && pol <= IAK_POLICY_GLOBAL;
      if (pol == IAK_POLICY_ATTEND && isnan(sc[i])) ok = false;
      if (i > 0 && s < bend[i - 1]) ok = false;   // also catches unsorted starts, as end > start
      bad |= !ok;
    }
  }
  bad = __syncthreads_or(bad);
  int32_t* table = p.page_table + static_cast<int64_t>(b) * Ht * W;
  int32_t* counts = p.page_counts + static_cast<int64_t>(b) * Ht;
  uint8_t* prow = p.page_prec ? p.page_prec + static_cast<int64_t>(b) * W : nullptr;
  uint64_t* mrow = p.row_masks ? p.row_masks + static_cast<int64_t>(b) * W : nullptr;
  if (bad) {
    if (mrow)
      for (int o = tid; o < W; o += kRouteThreads) mrow[o] = 0ull;
    for (int o = tid; o < Ht * W; o += kRouteThreads) table[o] = p.pad_value;
    if (prow)
      for (int o = tid; o < W; o += kRouteThreads) prow[o] = IAK_PREC_SKIP;
    for (int h = tid; h < Ht; h += kRouteThreads) counts[h] = 0;
    if (tid == 0 && p.num_selected) p.num_selected[b] = -1;
    return;
  }

  // ---- precisions and ATTEND ranking ----------------------------------------
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  int scored = 0;
  for (int i = tid; i < n2; i += kRouteThreads) {
    uint64_t k = kNoKey;
    if (i < n) {
      const int pol = bpol[i];
      const double s = sc[i];
      prec[i] = static_cast<uint8_t>(block_precision(p, pol, s));
      if (pol == IAK_POLICY_ATTEND && !isnan(s)) {
        k = descending_key(s);
        ++scored;
      }
    }
    key[i] = k;
    kidx[i] = i;
  }
  if (scored) atomicAdd(&n_scored, scored);
  __syncthreads();
  const int nA = n_scored;
  if (n <= kRouteThreads) {
    // rank by counting: every scored block counts the keys before it (the
    // reads are shared-memory broadcasts, no barrier per step); ranks are a
    // permutation of [0, nA) because ties are broken by block index
    if (tid < n) {
      const uint64_t ki = key[tid];
      if (ki != kNoKey) {
        int r = 0;
        for (int j = 0; j < n; ++j) {
          const uint64_t kj = key[j];
          r += (kj < ki) || (kj == ki && j < tid);
        }
        kidx[r] = tid;
      }
    }
    __syncthreads();
  } else {
    // bitonic sort of (key, index) pairs
    for (int size = 2; size <= n2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < n2; i += kRouteThreads) {
          const int j = i ^ stride;
          if (j > i) {
            const bool up = (i & size) == 0;
            const uint64_t ka = key[i], kb = key[j];
            const int ia = kidx[i], ib = kidx[j];
            const bool greater = ka > kb || (ka == kb && ia > ib);
            if (greater == up) {
              key[i] = kb; key[j] = ka;
              kidx[i] = ib; kidx[j] = ia;
            }
          }
        }
        __syncthreads();
      }
    }
  }
  // top_k = scored_attends[:k] with Python slice bounds
  const int k_cfg = p.top_k_blocks;
  const int K = k_cfg >= 0 ? min(k_cfg, nA) : max(0, nA + k_cfg);

  // ---- routed positions -------------------------------------------------------
  for (int i = tid; i < n; i += kRouteThreads) {
    work[i] = is_pinned(bpol[i]) ? 1 : 0;
    pos[i] = -1;
  }
  __syncthreads();
  const int H = cta_exclusive_scan(work, n, warp_sums);
  for (int i = tid; i < n; i += kRouteThreads)
    if (is_pinned(bpol[i])) pos[i] = work[i];
  __syncthreads();
  for (int r = tid; r < K; r += kRouteThreads) work[r] = prec[kidx[r]] != IAK_PREC_SKIP ? 1 : 0;
  __syncthreads();
  const int K1 = cta_exclusive_scan(work, K, warp_sums);
  for (int r = tid; r < K; r += kRouteThreads)
    if (prec[kidx[r]] != IAK_PREC_SKIP) pos[kidx[r]] = H + work[r];
  __syncthreads();
  auto skip_selected = [&](int i) {
    const double s = sc[i];
    return bpol[i] == IAK_POLICY_SKIP && !isnan(s) && s >= p.score_threshold;
  };
  for (int i = tid; i < n; i += kRouteThreads) work[i] = skip_selected(i) ? 1 : 0;
  __syncthreads();
  const int S2 = cta_exclusive_scan(work, n, warp_sums);
  for (int i = tid; i < n; i += kRouteThreads)
    if (skip_selected(i)) pos[i] = H + K1 + work[i];
  __syncthreads();
  const int nsel = H + K1 + S2;

  // ---- first-occurrence page counts and output offsets ------------------------
  // Page pg of selected block i is listed by i when no selected block that
  // also covers pg comes earlier in routed order.  Interior pages always are,
  // so the pages a block lists form one run [first, first + cnt).
  auto owns = [&](int i, int pg) -> bool {
    const int me = pos[i];
    for (int j = i - 1; j >= 0 && (bend[j] - 1) / PS >= pg; --j)
      if (pos[j] >= 0 && pos[j] < me) return false;
    for (int j = i + 1; j < n && bstart[j] / PS <= pg; ++j)
      if (pos[j] >= 0 && pos[j] < me) return false;
    return true;
  };
  int2* run = reinterpret_cast<int2*>(key);   // [nsel] (first listed page, block) by routed position
  for (int i = tid; i < n; i += kRouteThreads) {
    const int me = pos[i];
    if (me < 0) continue;
    const int ps = bstart[i] / PS, pe = (bend[i] - 1) / PS;
    const bool skip_first = !owns(i, ps);
    int cnt = pe - ps + 1 - (skip_first ? 1 : 0);
    if (pe != ps && !owns(i, pe)) --cnt;
    work[me] = cnt;   // positions are a permutation of [0, nsel)
    run[me] = make_int2(ps + (skip_first ? 1 : 0), i);
  }
  __syncthreads();
  const int total = cta_exclusive_scan(work, nsel, warp_sums);
  const int listed = min(total, W);

  // ---- emit: every slot in parallel, all heads per slot --------------------------
  // slot o belongs to the last routed position r with work[r] <= o (positions
  // that list no page share their successor's offset)
  const int32_t* hbase = p.bases ? p.bases + static_cast<int64_t>(b) * Ht : nullptr;
  for (int o = tid; o < W; o += kRouteThreads) {
    if (o >= listed) {
      for (int h = 0; h < Ht; ++h) table[static_cast<int64_t>(h) * W + o] = p.pad_value;
      if (prow) prow[o] = IAK_PREC_SKIP;
      if (mrow) mrow[o] = 0ull;
      continue;
    }
    int lo = 0, hi = nsel - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (work[mid] <= o) lo = mid; else hi = mid - 1;
    }
    const int2 r = run[lo];
    const int pg = r.x + (o - work[lo]);
    const int pr = prec[r.y];
    if (prow) prow[o] = static_cast<uint8_t>(pr);
    if (mrow) {
      // rows of the page covered by any selected block: the owner and its neighbours sharing the page
      const int i = r.y;
      const int64_t lo = static_cast<int64_t>(pg) * PS, hi = lo + PS;
      auto cover = [&](int blk) -> uint64_t {
        const int64_t s0 = max(static_cast<int64_t>(bstart[blk]), lo), e0 = min(static_cast<int64_t>(bend[blk]), hi);
        if (e0 <= s0) return 0ull;
        const int rows = static_cast<int>(e0 - s0);
        return (rows >= 64 ? ~0ull : ((1ull << rows) - 1ull)) << (s0 - lo);
      };
      uint64_t m = cover(i);
      for (int jb = i - 1; jb >= 0 && (bend[jb] - 1) / PS >= pg; --jb)
        if (pos[jb] >= 0) m |= cover(jb);
      for (int jb = i + 1; jb < n && bstart[jb] / PS <= pg; ++jb)
        if (pos[jb] >= 0) m |= cover(jb);
      mrow[o] = m;
    }
    for (int h = 0; h < Ht; ++h) {
      const int32_t phys = (hbase ? hbase[h] : 0) + pg;
      table[static_cast<int64_t>(h) * W + o] = phys;
      if (p.page_tags && phys >= 0 && phys < p.num_tag_pages) p.page_tags[phys] = p.prec_to_tag[pr];
    }
  }
  for (int h = tid; h < Ht; h += kRouteThreads) counts[h] = listed;
  if (tid == 0 && p.num_selected) p.num_selected[b] = total;
}

}  // namespace
}  // namespace iak

using namespace iak;

extern "C" int iak_route_pages(const iak_route_args* a, void* stream) {
  if (!a) return fail(IAK_ERR_INVALID_ARG, "null route args");
  if (a->batch < 0 || a->num_blocks < 0 || a->num_table_heads < 0 || a->table_width < 0)
    return fail(IAK_ERR_INVALID_ARG, "negative size in route args");
  if (a->num_blocks > IAK_ROUTE_MAX_BLOCKS)
    return fail(IAK_ERR_UNSUPPORTED, "%d blocks exceed the device router's %d", a->num_blocks, IAK_ROUTE_MAX_BLOCKS);
  if (a->page_size <= 0) return fail(IAK_ERR_INVALID_ARG, "page_size must be positive");
  if (!(a->memory_pressure >= 0.0 && a->memory_pressure <= 1.0))
    return fail(IAK_ERR_INVALID_ARG, "memory_pressure must be in [0, 1], got %g", a->memory_pressure);
  if (a->layout_stride < 0 || a->score_stride < 0) return fail(IAK_ERR_INVALID_ARG, "negative stride");
  if (a->layout_stride > 0 && a->layout_stride < a->num_blocks)
    return fail(IAK_ERR_INVALID_ARG, "layout_stride < num_blocks");
  if (a->score_stride > 0 && a->score_stride < a->num_blocks)
    return fail(IAK_ERR_INVALID_ARG, "score_stride < num_blocks");
  if (a->page_tags)
    for (int i = 0; i < 6; ++i)
      if (a->prec_to_tag[i] > 15) return fail(IAK_ERR_INVALID_ARG, "prec_to_tag[%d] > 15", i);
  if (a->batch == 0 || a->num_table_heads == 0) return IAK_OK;
  if (!a->page_counts || (a->table_width > 0 && !a->page_table))
    return fail(IAK_ERR_INVALID_ARG, "null route output");
  if (a->num_blocks > 0 && (!a->block_start || !a->block_end || !a->block_policy || !a->scores))
    return fail(IAK_ERR_INVALID_ARG, "null route input");
  if (a->row_masks && a->page_size > 64) return fail(IAK_ERR_UNSUPPORTED, "row masks need page_size <= 64");
  if (static_cast<int64_t>(a->num_table_heads) * a->table_width > 0x7FFFFFFFLL)
    return fail(IAK_ERR_UNSUPPORTED, "page table row too large");
  int slots = 1;
  while (slots < a->num_blocks) slots <<= 1;
  const size_t smem = static_cast<size_t>(slots) * kSlotBytes;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kMaxBlocks * kSlotBytes));
    if (e != cudaSuccess) return check_cuda(e, "route smem attribute");
    attr = true;
  }
  route_kernel<<<a->batch, kRouteThreads, smem, static_cast<cudaStream_t>(stream)>>>(*a, slots);
  return check_cuda(cudaGetLastError(), "route launch");
}
