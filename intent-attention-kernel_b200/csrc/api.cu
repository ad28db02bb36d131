// C ABI entry points: argument validation, split planning, dispatch.
#include <algorithm>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "iak_internal.cuh"

namespace iak {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int fail(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return IAK_OK;
  return fail(IAK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int device_sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int device_clock_khz() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1965000;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int k = 0;
    if (cudaDeviceGetAttribute(&k, cudaDevAttrClockRate, dev) != cudaSuccess || k <= 0) k = 1965000;
    cache[dev] = k;
  }
  return cache[dev];
}

// Process-wide kernel timer: event pairs recorded around the main decode launch.
struct KernelTimer {
  std::mutex mu;
  std::vector<cudaEvent_t> start, stop;
  int used = 0;
  bool on = false;
  bool open = false;  // a begin without its end yet
};
static KernelTimer g_timer;

// During stream capture the records become event-record nodes of the graph
// (cudaEventRecordExternal), so every replay of the graph times the kernel.
static cudaError_t timer_record(cudaEvent_t e, cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive)
    return cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
  return cudaEventRecord(e, s);
}

void kernel_timer_begin(cudaStream_t s) {
  std::lock_guard<std::mutex> lock(g_timer.mu);
  if (!g_timer.on || g_timer.used >= static_cast<int>(g_timer.start.size())) return;
  if (timer_record(g_timer.start[g_timer.used], s) == cudaSuccess) g_timer.open = true;
}

void kernel_timer_end(cudaStream_t s) {
  std::lock_guard<std::mutex> lock(g_timer.mu);
  if (!g_timer.open) return;
  g_timer.open = false;
  if (timer_record(g_timer.stop[g_timer.used], s) == cudaSuccess) ++g_timer.used;
}

static void timer_release_locked() {
  for (auto e : g_timer.start) cudaEventDestroy(e);
  for (auto e : g_timer.stop) cudaEventDestroy(e);
  g_timer.start.clear(); g_timer.stop.clear();
  g_timer.used = 0; g_timer.on = false; g_timer.open = false;
}

static bool fmt_reachable(const iak_decode_args* a, int fmt) {
  for (int i = 0; i < 16; ++i)
    if (a->tag_map[i] == fmt) return true;
  return a->tag_default == fmt;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Validate pools + args and fill the flattened kernel parameters (without
// workspace pointers).  Returns IAK_OK or an error status.
static int prepare(const iak_page_pools* P, const iak_decode_args* a, DecodeParams* p) {
  if (!P || !a) return fail(IAK_ERR_INVALID_ARG, "null pools/args");
  if (a->batch < 0 || a->num_q_heads <= 0 || a->num_table_heads <= 0)
    return fail(IAK_ERR_INVALID_ARG, "batch/heads must be positive (batch=%d, Hq=%d, Ht=%d)", a->batch,
                a->num_q_heads, a->num_table_heads);
  if (a->num_q_heads % a->num_table_heads)
    return fail(IAK_ERR_INVALID_ARG, "num_q_heads %d is not a multiple of num_table_heads %d", a->num_q_heads,
                a->num_table_heads);
  const int D = P->head_dim, PS = P->page_size;
  if (D <= 0 || D > 256 || D % 16) return fail(IAK_ERR_UNSUPPORTED, "head_dim %d unsupported (16..256, multiple of 16)", D);
  if (PS <= 0 || PS > 1024) return fail(IAK_ERR_INVALID_ARG, "page_size %d out of range", PS);
  if (P->num_pages < 0) return fail(IAK_ERR_INVALID_ARG, "num_pages < 0");
  if (P->scale_mode < 0 || P->scale_mode > 2) return fail(IAK_ERR_INVALID_ARG, "bad scale_mode %d", P->scale_mode);
  if (P->scale_mode == IAK_SCALE_GROUP32 && D % 32)
    return fail(IAK_ERR_INVALID_ARG, "group32 scales need head_dim %% 32 == 0");
  if (a->table_width < 0) return fail(IAK_ERR_INVALID_ARG, "table_width < 0");
  if (a->tag_bytes != 1 && a->tag_bytes != 4) return fail(IAK_ERR_INVALID_ARG, "tag_bytes must be 1 or 4");
  if (a->q_dtype < 0 || a->q_dtype > 2 || a->out_dtype < 0 || a->out_dtype > 2)
    return fail(IAK_ERR_INVALID_ARG, "bad q/out dtype");
  const int G = a->num_q_heads / a->num_table_heads;
  if (G > 8) return fail(IAK_ERR_UNSUPPORTED, "more than 8 query heads per page table (%d)", G);
  for (int i = 0; i < 16; ++i)
    if (a->tag_map[i] > IAK_FMT_SPARSE) return fail(IAK_ERR_INVALID_ARG, "tag_map[%d]=%d is not a format", i, a->tag_map[i]);
  if (a->tag_default > IAK_FMT_SPARSE) return fail(IAK_ERR_INVALID_ARG, "bad tag_default");
  const bool any_work = a->batch > 0 && a->table_width > 0;
  if (any_work) {
    if (!a->q || !a->page_table || !a->page_tags) return fail(IAK_ERR_INVALID_ARG, "q/page_table/page_tags is NULL");
    struct { int fmt; const void* k; const void* v; const char* name; } need[] = {
        {IAK_FMT_F16, P->k_f16, P->v_f16, "f16"},   {IAK_FMT_FP8, P->k_fp8, P->v_fp8, "fp8"},
        {IAK_FMT_INT8, P->k_i8, P->v_i8, "int8"},    {IAK_FMT_INT4, P->k_i4, P->v_i4, "int4"},
        {IAK_FMT_INT4R, P->k_i4, P->v_i4, "int4"},   {IAK_FMT_INT4R, P->k_i4r, P->v_i4r, "int4 residual"}};
    for (auto& n : need)
      if (fmt_reachable(a, n.fmt) && (!n.k || !n.v))
        return fail(IAK_ERR_INVALID_ARG, "a tag maps to format %d but the %s K/V pool is NULL", n.fmt, n.name);
    const bool quant = fmt_reachable(a, IAK_FMT_FP8) || fmt_reachable(a, IAK_FMT_INT8) ||
                       fmt_reachable(a, IAK_FMT_INT4) || fmt_reachable(a, IAK_FMT_INT4R);
    if (quant && (!P->k_scale || !P->v_scale)) return fail(IAK_ERR_INVALID_ARG, "quantised formats need k_scale/v_scale");
    if (fmt_reachable(a, IAK_FMT_INT4R) && (!P->k_res_scale || !P->v_res_scale))
      return fail(IAK_ERR_INVALID_ARG, "INT4_RESIDUAL needs k_res_scale/v_res_scale");
    if ((fmt_reachable(a, IAK_FMT_INT4) || fmt_reachable(a, IAK_FMT_INT4R)) && D % 32)
      return fail(IAK_ERR_UNSUPPORTED, "INT4 pages need head_dim %% 32 == 0");
  }
  std::memset(p, 0, sizeof(*p));
  p->k_f16 = static_cast<const __half*>(P->k_f16); p->v_f16 = static_cast<const __half*>(P->v_f16);
  p->k_fp8 = static_cast<const uint8_t*>(P->k_fp8); p->v_fp8 = static_cast<const uint8_t*>(P->v_fp8);
  p->k_i8 = static_cast<const int8_t*>(P->k_i8); p->v_i8 = static_cast<const int8_t*>(P->v_i8);
  p->k_i4 = static_cast<const uint8_t*>(P->k_i4); p->v_i4 = static_cast<const uint8_t*>(P->v_i4);
  p->k_i4r = static_cast<const uint8_t*>(P->k_i4r); p->v_i4r = static_cast<const uint8_t*>(P->v_i4r);
  p->k_scale = P->k_scale; p->v_scale = P->v_scale; p->k_rscale = P->k_res_scale; p->v_rscale = P->v_res_scale;
  p->num_pages = P->num_pages; p->PS = PS; p->D = D; p->scale_mode = P->scale_mode;
  p->n_scales = n_scales_of(P->scale_mode, D);
  p->q = a->q; p->q_dtype = a->q_dtype; p->q_sb = a->q_stride_b; p->q_sh = a->q_stride_h;
  p->out = a->out; p->out_dtype = a->out_dtype; p->o_sb = a->out_stride_b; p->o_sh = a->out_stride_h;
  p->B = a->batch; p->Hq = a->num_q_heads; p->Ht = a->num_table_heads; p->G = G;
  p->pt = a->page_table; p->pt_sb = a->pt_stride_b; p->pt_sh = a->pt_stride_h; p->W = a->table_width;
  p->pc = a->page_counts; p->pc_sb = a->pc_stride_b;
  p->tags = a->page_tags; p->tag_bytes = a->tag_bytes;
  std::memcpy(p->tag_map, a->tag_map, 16); p->tag_default = a->tag_default;
  p->sm_scale = a->sm_scale;
  p->ex_m = a->partial_m; p->ex_l = a->partial_l; p->ex_acc = a->partial_acc;
  p->status = a->status;
  p->wait_cycles = a->wait_budget_ns == 0
                       ? kDefaultWaitCycles
                       : std::max<long long>(1, static_cast<long long>(a->wait_budget_ns) * device_clock_khz() / 1000000);
  if (p->ex_l && (!p->ex_m || !p->ex_acc)) return fail(IAK_ERR_INVALID_ARG, "partial export needs m, l and acc");
  const int64_t units = static_cast<int64_t>(a->batch) * a->num_table_heads;
  if (a->kernel < 0 || a->kernel > 2) return fail(IAK_ERR_INVALID_ARG, "bad kernel selector %d", a->kernel);
  p->kernel = a->kernel;
  const bool shape_ok = mma_shape_eligible(*p);
  if (a->kernel == IAK_KERNEL_TENSOR && !shape_ok)
    return fail(IAK_ERR_UNSUPPORTED, "the tensor-core decode needs page_size 16, head_dim 64/128, fp16/bf16 q and "
                "page (or, at head_dim 128, group32) scales");
  p->tensor = shape_ok && a->kernel != IAK_KERNEL_GENERIC;
  const int W = a->table_width;
  int splits = a->num_splits, pps;
  if (p->tensor) {
    // persistent kernel (two CTAs per SM) over (unit, split) items of <= kTensorItemSlots slots
    if (splits <= 0) {
      // Static item striding over the resident CTAs: minimise
      // waves * (slots per item + a fixed per-item cost of ~16 slots).
      const int64_t ctas = 2LL * device_sm_count();
      int64_t best = -1, best_cost = 0;
      const int max_s = std::max(1, std::min(W, 256));
      for (int cand = 1; cand <= max_s; ++cand) {
        const int64_t slots = (W + cand - 1) / cand;
        if (slots > kTensorItemSlots) continue;
        const int64_t items = units * cand;
        const int64_t waves = (items + ctas - 1) / ctas;
        const int64_t cost = waves * (slots + 16);
        if (best < 0 || cost < best_cost) { best = cand; best_cost = cost; }
      }
      splits = static_cast<int>(best < 0 ? 1 : best);
    }
    splits = std::max(1, std::min(splits, std::max(1, W)));
    pps = W > 0 ? (W + splits - 1) / splits : 1;
    if (pps > kTensorItemSlots) pps = kTensorItemSlots;
  } else {
    // one CTA per (unit, split): aim for ~4 CTAs per SM, at least 8 slots per split
    if (splits <= 0) {
      const int64_t target = 4LL * device_sm_count();
      const int64_t s = units > 0 ? (target + units - 1) / units : 1;
      const int64_t max_s = std::max<int64_t>(1, (W + 7) / 8);
      splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(s, max_s)));
    }
    splits = std::max(1, std::min(splits, std::max(1, W)));
    pps = W > 0 ? (W + splits - 1) / splits : 1;
  }
  splits = W > 0 ? (W + pps - 1) / pps : 1;
  if (units * splits > 0x7FFFFFFFLL) return fail(IAK_ERR_UNSUPPORTED, "too many work units");
  p->num_splits = splits; p->pages_per_split = pps;
  p->ws_slots = p->tensor ? splits * kTensorConsumerWarps : splits;
  return IAK_OK;
}

// Tensor-path workspace head: [query tables][unit counters + the launch's done counter]
static size_t qtab_bytes_for(const DecodeParams& p) {
  if (!p.tensor) return 0;
  const size_t units = static_cast<size_t>(p.B) * p.Ht;
  return align_up(units * kQueryTableBytes, 256) + align_up((units + 1) * 4, 256);
}

// per-row partial arrays of `slots` slots: [m: rows x slots] [l] [acc: rows x slots x D]
static size_t partial_bytes(const DecodeParams& p, int slots) {
  const size_t n = static_cast<size_t>(p.B) * p.Hq * slots;
  return align_up(n * 4, 256) * 2 + align_up(n * p.D * 4, 256);
}

// Workspace: tensor path [head] [per-split partials: num_splits per row] (the partials of
// the consumer warps of a work item are merged in shared memory); CUDA-core path
// [per-split partials: ws_slots per row] when it splits the page lists
static size_t workspace_bytes_for(const DecodeParams& p) {
  if (p.tensor) return qtab_bytes_for(p) + partial_bytes(p, p.num_splits);
  return p.num_splits <= 1 ? 0 : partial_bytes(p, p.ws_slots);
}

static void carve_partials(char* w, const DecodeParams& p, int slots, float** m, float** l, float** acc) {
  const size_t n = static_cast<size_t>(p.B) * p.Hq * slots;
  *m = reinterpret_cast<float*>(w);
  *l = reinterpret_cast<float*>(w + align_up(n * 4, 256));
  *acc = reinterpret_cast<float*>(w + 2 * align_up(n * 4, 256));
}

}  // namespace iak

using namespace iak;

extern "C" {

int iak_version(void) { return IAK_ABI_VERSION; }

int iak_device_status(uint32_t* decode_timeouts, uint32_t* mla_timeouts, uint32_t* prefill_timeouts,
                      int32_t reset) {
  unsigned int v[3] = {0, 0, 0};
  int st = read_decode_timeouts(&v[0], reset != 0);
  if (!st) st = read_mla_timeouts(&v[1], reset != 0);
  if (!st) st = read_prefill_timeouts(&v[2], reset != 0);
  if (st) return st;
  if (decode_timeouts) *decode_timeouts = v[0];
  if (mla_timeouts) *mla_timeouts = v[1];
  if (prefill_timeouts) *prefill_timeouts = v[2];
  if (v[0] || v[1] || v[2])
    return fail(IAK_ERR_TIMEOUT, "device-side waits gave up: decode %u, mla %u, prefill %u warps", v[0], v[1], v[2]);
  return IAK_OK;
}

const char* iak_last_error(void) { return g_last_error.c_str(); }

int iak_decode_workspace_size(const iak_page_pools* pools, const iak_decode_args* args, size_t* bytes) {
  if (!bytes) return fail(IAK_ERR_INVALID_ARG, "bytes is NULL");
  DecodeParams p;
  int st = prepare(pools, args, &p);
  if (st) return st;
  *bytes = workspace_bytes_for(p);
  return IAK_OK;
}

}  // extern "C"

// iak_decode, or with x != NULL iak_decode_exchange (fused peer stores of the rows)
static int decode_impl(const iak_page_pools* pools, const iak_decode_args* args, void* workspace, size_t ws_bytes,
                       void* stream, const iak_peer_exchange* x) {
  DecodeParams p;
  int st = prepare(pools, args, &p);
  if (st) return st;
  if (!x && p.B > 0 && p.W > 0 && !args->out && !args->partial_l) return fail(IAK_ERR_INVALID_ARG, "out is NULL");
  if (x) {
    if (!p.tensor)
      return fail(IAK_ERR_UNSUPPORTED, "the fused exchange runs on the tensor-core decode (page_size 16, head_dim "
                  "64/128, fp16/bf16 q, page or group32 scales)");
    if (args->partial_l) return fail(IAK_ERR_INVALID_ARG, "the fused exchange writes the partials itself (partial_* must be NULL)");
    if (x->world < 1 || x->world > IAK_MAX_PEERS || x->rank < 0 || x->rank >= x->world)
      return fail(IAK_ERR_INVALID_ARG, "bad exchange rank %d / world %d", x->rank, x->world);
    if (x->rows != static_cast<int64_t>(p.B) * p.Hq || x->head_dim != p.D)
      return fail(IAK_ERR_INVALID_ARG, "exchange blocks are %lld rows x %d, the decode has %lld x %d",
                  static_cast<long long>(x->rows), x->head_dim, static_cast<long long>(p.B) * p.Hq, p.D);
    for (int r = 0; r < x->world; ++r) {
      if (!x->areas[r] || reinterpret_cast<uintptr_t>(x->areas[r]) % 256)
        return fail(IAK_ERR_INVALID_ARG, "exchange area of rank %d is NULL or not 256-byte aligned", r);
      p.x_areas[r] = static_cast<float*>(x->areas[r]);
    }
    p.x_world = x->world;
    p.x_rank = x->rank;
    p.x_bs = exchange_block_stride(x->rows, x->head_dim);
    p.x_flags_off = static_cast<int64_t>(exchange_flags_offset(x->world, x->rows, x->head_dim));
  }
  if (p.B == 0) return IAK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t need = workspace_bytes_for(p);
  if (need > 0) {
    if (!workspace || ws_bytes < need)
      return fail(IAK_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace ? ws_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(IAK_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    char* w = static_cast<char*>(workspace);
    if (p.tensor) {
      const size_t units = static_cast<size_t>(p.B) * p.Ht;
      p.ws_qtab = w;
      p.ws_cnt = reinterpret_cast<unsigned int*>(w + align_up(units * kQueryTableBytes, 256));
      p.ws_done = p.ws_cnt + units;
    }
    w += qtab_bytes_for(p);
    if (p.tensor) carve_partials(w, p, p.num_splits, &p.ws_m1, &p.ws_l1, &p.ws_acc1);
    else carve_partials(w, p, p.ws_slots, &p.ws_m, &p.ws_l, &p.ws_acc);
  }
  if (p.W == 0 && !x) {
    // nothing selected anywhere: every output row is zero (or an empty partial)
    DecodeParams z = p;
    z.num_splits = 1; z.pages_per_split = 1; z.tensor = 0; z.ws_slots = 1;
    return launch_decode_generic(z, s);
  }
  st = p.tensor ? launch_decode_mma(p, *pools, s) : launch_decode_generic(p, s);
  if (st) return st;
  // the tensor-core decode merges each unit's partials itself (its last consumer warp)
  if (p.ws_slots > 1 && !p.tensor) {
    st = launch_merge(p.ws_m, p.ws_l, p.ws_acc, static_cast<int64_t>(p.B) * p.Hq, p.ws_slots, p.D, p.out,
                      p.out_dtype, 0, &p, p.ex_m, p.ex_l, p.ex_acc, s);
    if (st) return st;
  }
  return IAK_OK;
}

extern "C" {

int iak_decode(const iak_page_pools* pools, const iak_decode_args* args, void* workspace, size_t ws_bytes,
               void* stream) {
  return decode_impl(pools, args, workspace, ws_bytes, stream, nullptr);
}

int iak_decode_exchange(const iak_page_pools* pools, const iak_decode_args* args, const iak_peer_exchange* x,
                        void* workspace, size_t ws_bytes, void* stream) {
  if (!x) return fail(IAK_ERR_INVALID_ARG, "null exchange descriptor");
  return decode_impl(pools, args, workspace, ws_bytes, stream, x);
}

int iak_kernel_timer_enable(int32_t max_launches) {
  if (max_launches <= 0 || max_launches > (1 << 20)) return fail(IAK_ERR_INVALID_ARG, "max_launches out of range");
  std::lock_guard<std::mutex> lock(g_timer.mu);
  timer_release_locked();
  g_timer.start.resize(max_launches); g_timer.stop.resize(max_launches);
  for (int i = 0; i < max_launches; ++i) {
    cudaError_t e0 = cudaEventCreate(&g_timer.start[i]);
    cudaError_t e1 = cudaEventCreate(&g_timer.stop[i]);
    if (e0 != cudaSuccess || e1 != cudaSuccess) {
      g_timer.start.resize(e0 == cudaSuccess ? i + 1 : i);
      g_timer.stop.resize(e1 == cudaSuccess ? i + 1 : i);
      timer_release_locked();
      return check_cuda(e0 != cudaSuccess ? e0 : e1, "kernel timer events");
    }
  }
  g_timer.on = true;
  return IAK_OK;
}

int iak_kernel_timer_read(double* total_ms, int32_t* launches) {
  if (!total_ms || !launches) return fail(IAK_ERR_INVALID_ARG, "null output pointer");
  std::lock_guard<std::mutex> lock(g_timer.mu);
  double t = 0.0;
  for (int i = 0; i < g_timer.used; ++i) {
    cudaError_t e = cudaEventSynchronize(g_timer.stop[i]);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, g_timer.start[i], g_timer.stop[i]);
    if (e != cudaSuccess) return check_cuda(e, "kernel timer read");
    t += ms;
  }
  *total_ms = t;
  *launches = g_timer.used;
  return IAK_OK;
}

int iak_kernel_timer_disable(void) {
  std::lock_guard<std::mutex> lock(g_timer.mu);
  timer_release_locked();
  return IAK_OK;
}

int iak_merge_partials(const float* m, const float* l, const float* acc, int64_t rows, int32_t splits,
                       int32_t head_dim, void* out, int32_t out_dtype, int64_t out_row_stride, void* stream) {
  if (rows < 0 || splits <= 0 || head_dim <= 0) return fail(IAK_ERR_INVALID_ARG, "bad merge sizes");
  if (rows == 0) return IAK_OK;
  if (!m || !l || !acc || !out) return fail(IAK_ERR_INVALID_ARG, "null merge pointer");
  if (out_dtype < 0 || out_dtype > 2) return fail(IAK_ERR_INVALID_ARG, "bad out dtype");
  if (out_row_stride < head_dim) return fail(IAK_ERR_INVALID_ARG, "out_row_stride < head_dim");
  return launch_merge(m, l, acc, rows, splits, head_dim, out, out_dtype, out_row_stride, nullptr, nullptr, nullptr,
                      nullptr, static_cast<cudaStream_t>(stream));
}

int iak_merge_partial_blocks(const float* blocks, int32_t num_parts, int64_t rows, int32_t head_dim, void* out,
                             int32_t out_dtype, int64_t out_row_stride, void* stream) {
  if (rows < 0 || num_parts <= 0 || head_dim <= 0) return fail(IAK_ERR_INVALID_ARG, "bad merge sizes");
  if (rows == 0) return IAK_OK;
  if (!blocks || !out) return fail(IAK_ERR_INVALID_ARG, "null merge pointer");
  if (out_dtype < 0 || out_dtype > 2) return fail(IAK_ERR_INVALID_ARG, "bad out dtype");
  if (out_row_stride < head_dim) return fail(IAK_ERR_INVALID_ARG, "out_row_stride < head_dim");
  const int64_t blk = rows * (static_cast<int64_t>(head_dim) + 2);
  return launch_merge_strided(blocks, blocks + rows, blocks + 2 * rows, 1, blk, head_dim, blk, rows, num_parts,
                              head_dim, out, out_dtype, out_row_stride, nullptr, nullptr, nullptr, nullptr,
                              static_cast<cudaStream_t>(stream));
}

}  // extern "C"
