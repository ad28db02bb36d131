// Shared declarations of the multi-query (prefill) attention kernels.
#pragma once

#include "quant_page.cuh"

namespace iak {

// Flattened, by-value parameters of one iak_prefill launch.
struct PrefillParams {
  qpage::PlanePools k, v;
  const void* q; int q_dtype; int64_t q_sb, q_sh, q_sm;
  void* out; int out_dtype; int64_t o_sb, o_sh, o_sm;
  int B, Hq, Ht, G, M;
  const int32_t* qpos; int64_t qp_sb;
  int causal;
  const int32_t* pt; int64_t pt_sb, pt_sh; int W;
  const int32_t* pc; int64_t pc_sb;
  const int32_t* bases;
  const int32_t* ppos; int64_t pp_sb, pp_sh;
  const uint64_t* masks; int64_t rm_sb;
  const void* tags; int tag_bytes; uint8_t tag_map[16]; uint8_t tag_default;
  float sm_scale;
  int q_vec;     // q rows are 16-byte aligned f16 / bf16 (vector loads)
  int o_vec;     // output rows are 16-byte aligned (vector stores)
};

__device__ __forceinline__ int prefill_fmt(const PrefillParams& p, int64_t pid) {
  const int tag = p.tag_bytes == 1 ? static_cast<int>(static_cast<const uint8_t*>(p.tags)[pid])
                                   : static_cast<const int32_t*>(p.tags)[pid];
  return (tag >= 0 && tag < 16) ? p.tag_map[tag] : p.tag_default;
}

// Number of table slots of unit (b, h).
__device__ __forceinline__ int prefill_count(const PrefillParams& p, int b, int h) {
  return p.pc ? min(max(p.pc[static_cast<int64_t>(b) * p.pc_sb + h], 0), p.W) : p.W;
}

// Rows of a page that the slot selects (bits [0, PS)).
__device__ __forceinline__ uint64_t prefill_mask(const PrefillParams& p, int b, int o) {
  const uint64_t all = p.k.PS >= 64 ? ~0ull : ((1ull << p.k.PS) - 1ull);
  return p.masks ? (p.masks[static_cast<int64_t>(b) * p.rm_sb + o] & all) : all;
}

// Token position of row 0 of slot o's page pid in unit (b, h).
__device__ __forceinline__ int64_t prefill_pos0(const PrefillParams& p, int b, int h, int o, int64_t pid,
                                                int64_t base) {
  return p.ppos ? static_cast<int64_t>(p.ppos[static_cast<int64_t>(b) * p.pp_sb + static_cast<int64_t>(h) * p.pp_sh + o])
                : (pid - base) * p.k.PS;
}

bool prefill_tc_eligible(const PrefillParams& p);
int launch_prefill_tc(const PrefillParams& p, cudaStream_t s);

}  // namespace iak
