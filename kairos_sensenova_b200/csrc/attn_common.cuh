// attn_common.cuh -- parameters and conversions shared by the FP8 attention kernels.
#pragma once
#include "common.cuh"

namespace kb {
namespace attn {

constexpr float E4M3_MAX = 448.f;

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  uint8_t* q8;   // [B, H, S_pad, D]  e4m3
  uint8_t* k8;   // [B, H, S_pad, D]  e4m3
  __nv_bfloat16* vt;  // [B, H, D, S_pad]  V^T, bf16
  float* amax;   // [2, B, H]           max |q|, max |k| per (batch, head)
  float* qn;     // [B, H, S_pad]      |q/s_q| per row (before e4m3 rounding)
  float* kn;     // [B, H, S_pad/64]   max |k/s_k| over each 64-key tile
  int B, S, H, S_pad;
  int64_t ld;    // elements between consecutive tokens of q/k/v (H*D when contiguous)
  float softmax_scale;
  int win_left, win_right;   // sliding window (query i sees keys i - left .. i + right); -1: unbounded
  long long* trace;  // optional event timestamps of CTA (0,0) (builds with KB_ATTN_TRACE only)
};

KB_DEVI uint32_t f2_to_e4m3x2(float lo, float hi) {
  __nv_fp8x2_storage_t r = __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
  return (uint32_t)r;
}

KB_DEVI float e4m3_to_float(uint8_t b) {
  __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(hr));
}

KB_DEVI float scale_of(float amax) { return amax > 0.f ? amax / E4M3_MAX : 1.f; }

// tcgen05 attention launcher (attn_fp8_tc.cu).
int launch_attn_tc(const Params& p, int* err, cudaStream_t st);

}  // namespace attn
}  // namespace kb
