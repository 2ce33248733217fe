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
  uint8_t* q8;   // [B, H, S_pad, D]
  uint8_t* k8;   // [B, H, S_pad, D]
  uint8_t* vt8;  // [B, H, D, S_pad]
  uint8_t* q8r;  // [B, H, S_pad, D]  e4m3 residual q/s - e4m3(q/s)   (two_term only)
  uint8_t* vt8r; // [B, H, D, S_pad]  e4m3 residual of v             (two_term only)
  float* amax;   // [3, B, H]
  int B, S, H, S_pad;
  int64_t ld;    // elements between consecutive tokens of q/k/v (H*D when contiguous)
  float softmax_scale;
  int vperm;     // 1: permute tokens inside 16-groups of vt8 for the mma.sync fragment order
  int two_term;  // 1: q and v carry a second e4m3 term (residual, same scale)
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

// tcgen05 attention launcher (attn_fp8_tc.cu); V^T must be unpermuted (vperm = 0).
int launch_attn_tc(const Params& p, int* err, cudaStream_t st);

}  // namespace attn
}  // namespace kb
