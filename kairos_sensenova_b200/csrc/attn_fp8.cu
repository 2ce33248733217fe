// attn_fp8.cu -- non-causal softmax attention with FP8-e4m3 Q/K (per-head
// amax scaling) and a bf16 P.V product, bf16 output (sm_100a).
//
// Replaces the attention core behind AttentionModule.forward
// (kairos/modules/dits/kairos_dit.py:367-373 -> flash_attention :232-277),
// i.e. softmax(q k^T / sqrt(d)) v per head, q/k/v given as [B, S, H*D] bf16.
//
// Launch sequence of kb200_attn_fp8_fwd:
//   1. attn_amax_kernel     per-(tensor, batch, head) max |x| over the sequence, q and k
//   2. attn_quant_kernel    x / (amax/448) -> e4m3 for Q and K as [B,H,S_pad,D],
//                           their row norms (|q| per row, max |k| per 64-key
//                           tile), and V transposed to bf16 [B,H,D,S_pad] so the
//                           P.V contraction reads it K-major (keys contiguous)
//   3. attn_fp8_tc_kernel   flash-attention forward on tcgen05 (attn_fp8_tc.cu)
#include "common.cuh"
#include "kb200_internal.h"
#include "attn_common.cuh"

namespace kb {
namespace attn {

// ---------------------------------------------------------------------------
// 1. amax.  Grid (ceil(S/32), B); 256 threads; D = 128 (one 16-byte vector per
// lane covers 8 channels, 16 lanes cover one head).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) attn_amax_kernel(Params p) {
  extern __shared__ float red[];  // [2 * H]
  const int b = blockIdx.y, H = p.H, HD = H * D;
  for (int i = threadIdx.x; i < 2 * H; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  const int t0 = blockIdx.x * 32, t1 = min(p.S, t0 + 32);
  const int vecs_per_tok = HD / 8;
  for (int tsr = 0; tsr < 2; ++tsr) {
    const __nv_bfloat16* x = tsr == 0 ? p.q : p.k;
    const int total = (t1 - t0) * vecs_per_tok;
    for (int base = 0; base < total; base += blockDim.x) {
      const int idx = base + threadIdx.x;
      const bool valid = idx < total;
      const int t = t0 + (valid ? idx / vecs_per_tok : 0), c = valid ? (idx % vecs_per_tok) * 8 : 0;
      float m = 0.f;
      if (valid) {
        uint4 raw = *reinterpret_cast<const uint4*>(x + ((size_t)b * p.S + t) * p.ld + c);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(__bfloat162float(e[j])));
      }
      // the 16 lanes of a half-warp cover one head (D = 128 channels): reduce there first
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
      if (valid && (threadIdx.x & 15) == 0)
        atomicMax(reinterpret_cast<int*>(&red[tsr * H + c / D]), __float_as_int(m));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * H; i += blockDim.x) {
    const int tsr = i / H, h = i % H;
    atomicMax(reinterpret_cast<int*>(&p.amax[(tsr * p.B + b) * H + h]), __float_as_int(red[i]));
  }
}

// ---------------------------------------------------------------------------
// 2. quantise.  Grid (S_pad / 64, B * H); 256 threads; one 64-token x D tile
// of one head.  Pad tokens (>= S) are written as zeros.
// ---------------------------------------------------------------------------
KB_DEVI uint32_t quant8(const __nv_bfloat16* e, float r, int j0) {
  return f2_to_e4m3x2(__bfloat162float(e[j0]) * r, __bfloat162float(e[j0 + 1]) * r) |
         (f2_to_e4m3x2(__bfloat162float(e[j0 + 2]) * r, __bfloat162float(e[j0 + 3]) * r) << 16);
}

template <int D>
__global__ void __launch_bounds__(256) attn_quant_kernel(Params p) {
  // bf16 elements per V^T row in shared memory: padded by 2, so the 16 lanes that hold
  // 8-channel groups of one token (channels 8 apart) store into 4 banks, not one
  constexpr int LDT = 64 + 2;
  __shared__ __align__(16) __nv_bfloat16 vts[D * LDT];
  __shared__ int kmax;          // max key norm of this 64-token tile (float bits, >= 0)
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H, H = p.H;
  const int t0 = blockIdx.x * 64;
  const float rq = 1.f / scale_of(p.amax[(0 * p.B + b) * H + h]);
  const float rk = 1.f / scale_of(p.amax[(1 * p.B + b) * H + h]);
  if (threadIdx.x == 0) kmax = 0;
  __syncthreads();
  constexpr int VPT = D / 8;  // 16-byte bf16 vectors per token row
  for (int idx = threadIdx.x; idx < 64 * VPT; idx += blockDim.x) {
    const int r = idx / VPT, c = (idx % VPT) * 8, t = t0 + r;
    uint4 rq4 = make_uint4(0, 0, 0, 0), rk4 = rq4, rv4 = rq4;
    if (t < p.S) {
      const size_t off = ((size_t)b * p.S + t) * p.ld + h * D + c;
      rq4 = *reinterpret_cast<const uint4*>(p.q + off);
      rk4 = *reinterpret_cast<const uint4*>(p.k + off);
      rv4 = *reinterpret_cast<const uint4*>(p.v + off);
    }
    const __nv_bfloat16* eq = reinterpret_cast<const __nv_bfloat16*>(&rq4);
    const __nv_bfloat16* ek = reinterpret_cast<const __nv_bfloat16*>(&rk4);
    const __nv_bfloat16* ev = reinterpret_cast<const __nv_bfloat16*>(&rv4);
    const size_t qoff = ((size_t)bh * p.S_pad + t) * D + c;
    *reinterpret_cast<uint2*>(p.q8 + qoff) = make_uint2(quant8(eq, rq, 0), quant8(eq, rq, 4));
    *reinterpret_cast<uint2*>(p.k8 + qoff) = make_uint2(quant8(ek, rk, 0), quant8(ek, rk, 4));
    // row norms of the scaled (pre-rounding) q and k: the 16 lanes of one token
    float nq = 0.f, nk = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = __bfloat162float(eq[j]) * rq, bk = __bfloat162float(ek[j]) * rk;
      nq = fmaf(a, a, nq);
      nk = fmaf(bk, bk, nk);
    }
#pragma unroll
    for (int o = VPT / 2; o > 0; o >>= 1) {
      nq += __shfl_xor_sync(0xffffffffu, nq, o);
      nk += __shfl_xor_sync(0xffffffffu, nk, o);
    }
    if (c == 0) {
      p.qn[(size_t)bh * p.S_pad + t] = sqrtf(nq);
      atomicMax(&kmax, __float_as_int(sqrtf(nk)));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) vts[(c + j) * LDT + r] = ev[j];
  }
  __syncthreads();
  if (threadIdx.x == 0) p.kn[(size_t)bh * (p.S_pad / 64) + blockIdx.x] = __int_as_float(kmax);
  // write the V^T tile: D rows x 64 tokens (128 bytes per row)
  for (int idx = threadIdx.x; idx < D * 8; idx += blockDim.x) {
    const int d = idx >> 3, seg = (idx & 7) * 8;
    // (rows are 4-byte aligned: four 32-bit reads)
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&vts[d * LDT + seg]);
    *reinterpret_cast<uint4*>(p.vt + ((size_t)bh * D + d) * p.S_pad + t0 + seg) =
        make_uint4(src[0], src[1], src[2], src[3]);
  }
}

}  // namespace attn
}  // namespace kb

// ===========================================================================
// Host side: C ABI
// ===========================================================================
namespace {
using namespace kb;
constexpr int AD = 128;

struct AttnWs { size_t q8, k8, vt, qn, kn, amax, err, total; int S_pad; };

AttnWs attn_ws(int64_t B, int64_t S, int64_t H) {
  AttnWs w{};
  w.S_pad = (int)((S + 255) / 256 * 256);
  const size_t n = (size_t)B * H * w.S_pad * AD;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes); return o; };
  w.q8 = take(n);
  w.k8 = take(n);
  w.vt = take(2 * n);
  w.qn = take((size_t)B * H * w.S_pad * 4);
  w.kn = take((size_t)B * H * (w.S_pad / 64) * 4);
  w.amax = take((size_t)2 * B * H * 4 + 16);   // amax, then the device error word
  w.err = w.amax + (size_t)2 * B * H * 4;
  w.total = off;
  return w;
}

int attn_validate(const void* q, const void* k, const void* v, const void* o, int64_t B, int64_t S,
                  int64_t H, int64_t D) {
  if (D != AD) return set_error(KB200_ERR_INVALID, "attn_fp8: head dim %lld unsupported (128)", (long long)D);
  if (B <= 0 || S <= 0 || H <= 0) return set_error(KB200_ERR_INVALID, "attn_fp8: bad shape");
  if (B * S * H * D >= ((int64_t)1 << 31))
    return set_error(KB200_ERR_INVALID, "attn_fp8: tensor too large for 32-bit indexing");
  const void* ptrs[] = {q, k, v, o};
  for (const void* p : ptrs) {
    if (!p) return set_error(KB200_ERR_INVALID, "attn_fp8: null tensor pointer");
    if (!aligned16(p)) return set_error(KB200_ERR_ALIGN, "attn_fp8: q/k/v/o must be 16-byte aligned");
  }
  return KB200_OK;
}
}  // namespace

extern "C" size_t kb200_attn_fp8_workspace_size(int64_t B, int64_t S, int64_t H, int64_t D) {
  if (D != AD || B <= 0 || S <= 0 || H <= 0) return 0;
  return attn_ws(B, S, H).total;
}

namespace {
int attn_setup(attn::Params& p, AttnWs& w, const void* q, const void* k, const void* v, void* o,
               int64_t B, int64_t S, int64_t H, int64_t D, int64_t row_stride, float softmax_scale,
               void* workspace, size_t workspace_bytes) {
  if (int e = attn_validate(q, k, v, o, B, S, H, D)) return e;
  if (row_stride == 0) row_stride = H * D;
  if (row_stride < H * D || row_stride % 8)
    return set_error(KB200_ERR_ALIGN, "attn_fp8: row_stride must be >= H*D and a multiple of 8");
  w = attn_ws(B, S, H);
  if (!workspace || workspace_bytes < w.total)
    return set_error(KB200_ERR_WORKSPACE, "attn_fp8: workspace needs %zu bytes, got %zu", w.total,
                     workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error(KB200_ERR_ALIGN, "attn_fp8: workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  p = attn::Params{};
  p.q = (const __nv_bfloat16*)q;
  p.k = (const __nv_bfloat16*)k;
  p.v = (const __nv_bfloat16*)v;
  p.o = (__nv_bfloat16*)o;
  p.q8 = (uint8_t*)(ws + w.q8);
  p.k8 = (uint8_t*)(ws + w.k8);
  p.vt = (__nv_bfloat16*)(ws + w.vt);
  p.qn = (float*)(ws + w.qn);
  p.kn = (float*)(ws + w.kn);
  p.amax = (float*)(ws + w.amax);
  p.B = (int)B;
  p.S = (int)S;
  p.H = (int)H;
  p.S_pad = w.S_pad;
  p.ld = row_stride;
  p.softmax_scale = softmax_scale;
  p.win_left = p.win_right = -1;   // no window
  return KB200_OK;
}

int attn_quantize(const attn::Params& p, const AttnWs& w, cudaStream_t st) {
  if (cudaMemsetAsync(p.amax, 0, (size_t)2 * p.B * p.H * 4 + 16, st) != cudaSuccess)
    return check_launch("attn_fp8 amax memset");
  attn::attn_amax_kernel<AD><<<dim3((unsigned)((p.S + 31) / 32), (unsigned)p.B), 256, 2 * p.H * 4, st>>>(p);
  if (int e = check_launch("attn_amax_kernel")) return e;
  attn::attn_quant_kernel<AD><<<dim3(w.S_pad / 64, (unsigned)(p.B * p.H)), 256, 0, st>>>(p);
  return check_launch("attn_quant_kernel");
}

int attn_attend(const attn::Params& p, const AttnWs& w, cudaStream_t st) {
  return attn::launch_attn_tc(p, reinterpret_cast<int*>(reinterpret_cast<char*>(p.amax) + (w.err - w.amax)), st);
}
}  // namespace

#define KB_ATTN_ARGS                                                                         \
  const void *q, const void *k, const void *v, void *o, int64_t B, int64_t S, int64_t H,    \
      int64_t D, int64_t row_stride, float softmax_scale, void *workspace,                        \
      size_t workspace_bytes, void *stream
#define KB_ATTN_SETUP                                                                          \
  attn::Params p;                                                                              \
  AttnWs w;                                                                                    \
  if (int e = attn_setup(p, w, q, k, v, o, B, S, H, D, row_stride, softmax_scale, workspace,          \
                         workspace_bytes))                                                     \
    return e;                                                                                  \
  cudaStream_t st = static_cast<cudaStream_t>(stream);

extern "C" int kb200_attn_fp8_fwd(KB_ATTN_ARGS) {
  KB_ATTN_SETUP
  if (int e = attn_quantize(p, w, st)) return e;
  return attn_attend(p, w, st);
}

extern "C" int kb200_attn_fp8_quantize(KB_ATTN_ARGS) {
  KB_ATTN_SETUP
  return attn_quantize(p, w, st);
}

extern "C" int kb200_attn_fp8_attend(KB_ATTN_ARGS) {
  KB_ATTN_SETUP
  return attn_attend(p, w, st);
}

// Sliding-window variants: query i attends keys i - window_left .. i + window_right
// (a negative bound is unbounded), flash-attention's window_size semantics.
namespace {
int set_window(attn::Params& p, int64_t window_left, int64_t window_right) {
  if (window_left > INT32_MAX || window_right > INT32_MAX)
    return set_error(KB200_ERR_INVALID, "attn_fp8: window bound too large");
  p.win_left = window_left < 0 ? -1 : (int)window_left;
  p.win_right = window_right < 0 ? -1 : (int)window_right;
  return KB200_OK;
}
}  // namespace

extern "C" int kb200_attn_fp8_fwd_window(KB_ATTN_ARGS, int64_t window_left, int64_t window_right) {
  KB_ATTN_SETUP
  if (int e = set_window(p, window_left, window_right)) return e;
  if (int e = attn_quantize(p, w, st)) return e;
  return attn_attend(p, w, st);
}

extern "C" int kb200_attn_fp8_attend_window(KB_ATTN_ARGS, int64_t window_left, int64_t window_right) {
  KB_ATTN_SETUP
  if (int e = set_window(p, window_left, window_right)) return e;
  return attn_attend(p, w, st);
}

extern "C" int kb200_attn_fp8_status(const void* workspace, int64_t B, int64_t S, int64_t H, void* stream) {
  if (!workspace || B <= 0 || S <= 0 || H <= 0) return set_error(KB200_ERR_INVALID, "attn_fp8_status: bad args");
  const AttnWs w = attn_ws(B, S, H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int code = 0;
  if (cudaMemcpyAsync(&code, static_cast<const char*>(workspace) + w.err, sizeof(int), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return check_launch("attn_fp8_status");
  if (code != 0) return set_error(KB200_ERR_TIMEOUT, "attn_fp8: a device-side wait gave up (site %d)", code);
  return KB200_OK;
}
