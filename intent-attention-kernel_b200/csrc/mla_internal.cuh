// Internal declarations of the MLA decode (mla.cu: validation, planning,
// CUDA-core kernel, C ABI; mla_tc.cu: tcgen05 / TMEM kernel).
#pragma once

#include "iak_internal.cuh"

namespace iak {

// Flattened, by-value parameters of one MLA decode launch.
struct MlaParams {
  const void* q; int q_dtype; int64_t q_sb, q_sh;
  void* out; int out_dtype; int64_t o_sb, o_sh;
  int B, H, Dqk, Dv;
  const void* dense; int dense_dtype;
  const uint8_t* fp8; const float* fp8_scale;
  int64_t num_pages; int PS;
  const int32_t* pt; int64_t pt_sb; int W;
  const int32_t* pc;
  const void* tags; int tag_bytes;
  uint8_t tag_map[16]; uint8_t tag_default;
  float sm_scale;
  float* ex_m; float* ex_l; float* ex_acc;   // optional per-row partial export
  int kernel;                                // IAK_KERNEL_*
  int tensor;                                // 1: the tcgen05 kernel runs
  int num_splits, pages_per_split;
  float* ws_m; float* ws_l; float* ws_acc;   // split partials [row][split] (acc x Dv)
};

// tcgen05 kernel (mla_tc.cu)
bool mla_tc_eligible(const MlaParams& p);
void plan_mla_tc(MlaParams* p, int requested_splits);
int launch_mla_tc(const MlaParams& p, cudaStream_t s);

}  // namespace iak
