// Internal declarations shared by the libiak_b200 translation units.
#pragma once

#include <cstdint>
#include <cstdio>
#include <string>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "intent_attention_b200.h"

namespace iak {

// ---------------------------------------------------------------- errors ---
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int device_sm_count();
// SM clock of the current device in kHz (cached per device)
int device_clock_khz();
// timeout counters of each kernel family (defined beside the kernels)
int read_decode_timeouts(unsigned int* value, bool reset);
int read_mla_timeouts(unsigned int* value, bool reset);
int read_prefill_timeouts(unsigned int* value, bool reset);
// default budget of a bounded device-side wait: about 2 s at the boost clock
constexpr long long kDefaultWaitCycles = 4000000000LL;

// Exchange area of one rank (device memory of its GPU), for world W and block size
// rows * (head_dim + 2) floats padded to BS (a multiple of 64 floats):
//   float  blocks[2][W][BS]      receive arrays, one per parity
//   float  staging[BS]           this rank's partial block
//   uint32 flags[2][W]           arrival epoch of each sender, per parity
//   uint32 push_count[2]         CTAs of this rank's push kernel that finished
//   uint32 epoch                 last epoch this rank published
__host__ __device__ inline int64_t exchange_block_stride(int64_t rows, int D) {
  const int64_t bf = rows * (static_cast<int64_t>(D) + 2);
  return (bf + 63) / 64 * 64;
}
__host__ __device__ inline size_t exchange_staging_offset(int world, int64_t rows, int D) {
  return static_cast<size_t>(2) * world * exchange_block_stride(rows, D) * sizeof(float);
}
__host__ __device__ inline size_t exchange_flags_offset(int world, int64_t rows, int D) {
  return exchange_staging_offset(world, rows, D) + exchange_block_stride(rows, D) * sizeof(float);
}
// kernel timer hooks around the main decode launch (no-ops unless enabled)
void kernel_timer_begin(cudaStream_t s);
void kernel_timer_end(cudaStream_t s);

// --------------------------------------------------------- device params ---
// Flattened, by-value kernel parameters of one decode launch.
struct DecodeParams {
  const __half* k_f16; const __half* v_f16;
  const uint8_t* k_fp8; const uint8_t* v_fp8;
  const int8_t* k_i8; const int8_t* v_i8;
  const uint8_t* k_i4; const uint8_t* v_i4;
  const uint8_t* k_i4r; const uint8_t* v_i4r;
  const float* k_scale; const float* v_scale;
  const float* k_rscale; const float* v_rscale;
  int64_t num_pages;
  int PS, D, scale_mode, n_scales;
  const void* q; int q_dtype; int64_t q_sb, q_sh;
  void* out; int out_dtype; int64_t o_sb, o_sh;
  int B, Hq, Ht, G;
  const int32_t* pt; int64_t pt_sb, pt_sh; int W;
  const int32_t* pc; int64_t pc_sb;
  const void* tags; int tag_bytes;
  uint8_t tag_map[16]; uint8_t tag_default;
  float sm_scale;
  int num_splits, pages_per_split;
  int kernel;    // IAK_KERNEL_*
  int tensor;    // 1: the tensor-core path runs (per-warp partial slots, query tables)
  int ws_slots;  // partial slots per query row in the workspace
  char* ws_qtab; // per-unit query tables (tensor path)
  // tensor path, zeroed by the prep kernel on every call: per-unit count of merged items
  unsigned int* ws_cnt;
  // tensor path: per-item merged partials [row][split] (level 1 of the in-kernel merge)
  float* ws_m1; float* ws_l1; float* ws_acc1;
  // fused peer exchange (iak_decode_exchange; x_world = 0 otherwise): each row's merged
  // partial goes straight into slot x_rank of every rank's receive array, and the
  // last unit to finish raises this rank's flag in every area
  float* x_areas[IAK_MAX_PEERS];
  int x_world, x_rank;
  int64_t x_bs;                 // partial-block stride in floats
  int64_t x_flags_off;          // byte offset of the flags inside an area
  unsigned int* ws_done;        // units merged by this launch (tensor path, zeroed by the prep kernel)
  // split partials, [unit][split][g] and [unit][split][g][D]
  float* ws_m; float* ws_l; float* ws_acc;
  // optional export of final per-row partials (rows = B*Hq)
  float* ex_m; float* ex_l; float* ex_acc;
  unsigned int* status;   // IAK_STATUS_* bits ORed on a timeout (or NULL)
  long long wait_cycles;  // budget of each bounded device-side wait, in SM cycles
};

// Launchers (return IAK_OK or a status; errors recorded with set_error).
int launch_decode_generic(const DecodeParams& p, cudaStream_t s);
int launch_decode_mma(const DecodeParams& p, const iak_page_pools& pools, cudaStream_t s);
bool mma_shape_eligible(const DecodeParams& p);
constexpr int kQueryTableBytes = 8704;   // per-unit query table of the tensor path
constexpr int kTensorItemSlots = 256;    // max table slots per tensor-path work item
constexpr int kTensorConsumerWarps = 4;  // partial slots per work item
int launch_merge(const float* m, const float* l, const float* acc, int64_t rows, int splits, int D,
                 void* out, int out_dtype, int64_t out_row_stride,
                 const DecodeParams* rowmap, float* ex_m, float* ex_l, float* ex_acc, cudaStream_t s);
// partial (s) of row r: m/l at [r * ms_r + s * ms_s], acc at [r * as_r + s * as_s + d]
int launch_merge_strided(const float* m, const float* l, const float* acc, int64_t ms_r, int64_t ms_s, int64_t as_r,
                         int64_t as_s, int64_t rows, int splits, int D, void* out, int out_dtype,
                         int64_t out_row_stride, const DecodeParams* rowmap, float* ex_m, float* ex_l, float* ex_acc,
                         cudaStream_t s);

// ------------------------------------------------------- device helpers ---
__host__ __device__ inline int n_scales_of(int mode, int D) {
  return mode == IAK_SCALE_PAGE ? 1 : (mode == IAK_SCALE_GROUP32 ? D / 32 : D);
}

__device__ __forceinline__ float load_as_float(const void* base, int dtype, int64_t idx) {
  if (dtype == IAK_DT_F32) return static_cast<const float*>(base)[idx];
  if (dtype == IAK_DT_F16) return __half2float(static_cast<const __half*>(base)[idx]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
}

__device__ __forceinline__ void store_from_float(void* base, int dtype, int64_t idx, float v) {
  if (dtype == IAK_DT_F32) static_cast<float*>(base)[idx] = v;
  else if (dtype == IAK_DT_F16) static_cast<__half*>(base)[idx] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float e4m3_to_float(uint8_t c) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(c), __NV_E4M3);
  return __half2float(__half(h));
}

// Packed INT4 layout: channel d lives in word 4*(d/32) + (d%16)/4 at nibble
// NIB[(d%4)] + 2*((d%32) >= 16), stored as code + 8.
__device__ __forceinline__ int int4_code(const uint8_t* row, int d) {
  const int r = d & 31;
  const int o = r & 3;
  const int n = ((o & 1) << 2) + (o >> 1) + ((r >> 4) << 1);  // {0,4,1,5}[o] + 2*hi
  const int w = ((d >> 5) << 2) + ((r & 15) >> 2);
  const uint8_t byte = row[w * 4 + (n >> 1)];
  return static_cast<int>((n & 1) ? (byte >> 4) : (byte & 0xF)) - 8;
}

__device__ __forceinline__ int page_format(const DecodeParams& p, int64_t pid) {
  int tag = p.tag_bytes == 1 ? static_cast<int>(static_cast<const uint8_t*>(p.tags)[pid])
                             : static_cast<const int32_t*>(p.tags)[pid];
  return (tag >= 0 && tag < 16) ? p.tag_map[tag] : p.tag_default;
}

}  // namespace iak
