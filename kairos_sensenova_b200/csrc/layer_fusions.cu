// layer_fusions.cu -- the GatedDeltaNet prologue and output-norm epilogue
// as single memory-bound passes (sm_100a).
//
// Prologue (kairos/third_party/fla/layers/gated_deltanet.py:238-271):
//   q, k, v = SiLU(causal depthwise conv_W(x) + bias)       (fla/modules/convolution.py:53-140)
//   beta    = sigmoid(b)            (x2 when allow_neg_eigval)
//   g       = -exp(A_log) * softplus(a + dt_bias)           in fp32
// One launch covers the three convolutions and the gates (grid.z selects).
//
// Epilogue (gated_deltanet.py:309-311, FusedRMSNormGated,
// fla/modules/fused_norm_gate.py:60-110 with activation 'swish'):
//   y = o * rsqrt(mean(o^2) + eps) * w * gate * sigmoid(gate)   per (token, head) row
#include "common.cuh"
#include "kb200_internal.h"

namespace kb {
namespace fuse {

struct ConvSet {
  const __nv_bfloat16* x;
  const float* w;     // [C, W]
  const float* bias;  // [C] or null
  __nv_bfloat16* y;
  int C;
  int64_t ldx, ldy;   // row strides in elements
  const __nv_bfloat16* cache;  // [B, C, W] conv state (the last W inputs before token 0) or null
};

struct PrologueParams {
  ConvSet set[3];
  const __nv_bfloat16* a;
  const __nv_bfloat16* b;
  int64_t lda, ldb;
  const float* A_log;
  const float* dt_bias;
  float* g;
  __nv_bfloat16* beta;
  int B, T, H, W;
  int allow_neg_eigval;
};

constexpr int PT = 64, PC = 256, PTHREADS = 128;   // tokens and channels per CTA tile
constexpr int PRUN = PT / (PTHREADS / (PC / 8));   // tokens per thread (16)

// Two consecutive bf16 channels of a packed word as an fp32 pair.
KB_DEVI float2 bf16x2_to_float2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
KB_DEVI float2 silu2(float2 a) {
  const float2 e = fmul2(a, make_float2(-1.4426950408889634f, -1.4426950408889634f));   // -a log2(e)
  float2 d;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(d.x) : "f"(e.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(d.y) : "f"(e.y));
  d = fadd2(d, make_float2(1.f, 1.f));
  float2 r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
  return fmul2(a, r);
}

// Grid (ceil(maxC / PC), ceil(T / PT), B * 4): z = 4*b + {0,1,2: conv q,k,v; 3: gates}.
// Conv: the CTA stages its (PT + 3 halo) x PC input tile with cp.async in one
// shot (every load in flight at once).  Each thread then owns 8 channels
// (weights in registers as fp32 channel pairs) and slides a 4-row window down
// PRUN consecutive tokens: one shared-memory row load and 16 packed FMAs per token.
__global__ void __launch_bounds__(PTHREADS, 5) gdn_prologue_kernel(PrologueParams p) {
  const int which = blockIdx.z & 3, bb = blockIdx.z >> 2;
  const int tok0 = blockIdx.y * PT;
  const int tid = threadIdx.x;
  if (which < 3) {
    __shared__ __align__(16) __nv_bfloat16 tile[PT + 3][PC];
    // channel c = 8 * grp + j lives at wsm[j][grp]: lanes (consecutive grp) read 16 B apart
    __shared__ __align__(16) float wsm[8][PC / 8][4];
    __shared__ float bsm[8][PC / 8];
    const ConvSet cs = p.set[which];
    const int c0 = blockIdx.x * PC;
    if (c0 >= cs.C) return;
    const __nv_bfloat16* xb = cs.x + (size_t)bb * p.T * cs.ldx;
    for (int idx = tid; idx < (PT + 3) * (PC / 8); idx += PTHREADS) {
      const int r = idx / (PC / 8), cv = (idx % (PC / 8)) * 8;
      const int t = tok0 - 3 + r;
      if (t < 0 && cs.cache) {
        // history rows from the conv state: input t (< 0) sits at state column W + t
        alignas(16) __nv_bfloat16 hv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = c0 + cv + j;
          hv[j] = (c < cs.C && p.W + t >= 0) ? cs.cache[((size_t)bb * cs.C + c) * p.W + p.W + t]
                                              : __float2bfloat16(0.f);
        }
        *reinterpret_cast<uint4*>(&tile[r][cv]) = *reinterpret_cast<const uint4*>(hv);
        continue;
      }
      const bool ok = t >= 0 && t < p.T && c0 + cv < cs.C;
      cp_async16(&tile[r][cv], xb + (size_t)(ok ? t : 0) * cs.ldx + (ok ? c0 + cv : 0), ok);
    }
    cp_async_commit();
    // weights right-aligned into 4 taps: tap i multiplies x[t - 3 + i] (leading taps zero when W < 4)
    for (int idx = tid; idx < PC * 4; idx += PTHREADS) {
      const int c = idx >> 2, wi = (idx & 3) - (4 - p.W);
      wsm[c & 7][c >> 3][idx & 3] = (wi >= 0 && c0 + c < cs.C) ? cs.w[(size_t)(c0 + c) * p.W + wi] : 0.f;
    }
    for (int c = tid; c < PC; c += PTHREADS)
      bsm[c & 7][c >> 3] = (cs.bias && c0 + c < cs.C) ? cs.bias[c0 + c] : 0.f;
    const int grp = tid % (PC / 8), cv = grp * 8, tg = tid / (PC / 8);
    const int c8 = c0 + cv;
    cp_async_wait<0>();
    __syncthreads();
    if (c8 >= cs.C) return;
    float2 wp[4][4], bp[4];   // [tap][channel pair]
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 w0 = *reinterpret_cast<const float4*>(wsm[2 * q][grp]);
      const float4 w1 = *reinterpret_cast<const float4*>(wsm[2 * q + 1][grp]);
      wp[0][q] = make_float2(w0.x, w1.x); wp[1][q] = make_float2(w0.y, w1.y);
      wp[2][q] = make_float2(w0.z, w1.z); wp[3][q] = make_float2(w0.w, w1.w);
      bp[q] = make_float2(bsm[2 * q][grp], bsm[2 * q + 1][grp]);
    }
    const int tl0 = tg * PRUN;
    float2 win[4][4];   // ring of rows: row tl0 + r sits in slot r & 3
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const uint4 raw = *reinterpret_cast<const uint4*>(&tile[tl0 + r][cv]);
      win[r][0] = bf16x2_to_float2(raw.x); win[r][1] = bf16x2_to_float2(raw.y);
      win[r][2] = bf16x2_to_float2(raw.z); win[r][3] = bf16x2_to_float2(raw.w);
    }
    __nv_bfloat16* yrow = cs.y + ((size_t)bb * p.T + tok0 + tl0) * cs.ldy + c8;
    const int nt = min(PRUN, p.T - tok0 - tl0);
#pragma unroll
    for (int k = 0; k < PRUN; ++k) {
      if (k >= nt) break;
      {
        const uint4 raw = *reinterpret_cast<const uint4*>(&tile[tl0 + k + 3][cv]);
        float2* w = win[(k + 3) & 3];
        w[0] = bf16x2_to_float2(raw.x); w[1] = bf16x2_to_float2(raw.y);
        w[2] = bf16x2_to_float2(raw.z); w[3] = bf16x2_to_float2(raw.w);
      }
      uint4 outv;
      uint32_t* ov = reinterpret_cast<uint32_t*>(&outv);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 a = bp[q];
#pragma unroll
        for (int i = 0; i < 4; ++i) a = ffma2(win[(k + i) & 3][q], wp[i][q], a);
        a = silu2(a);
        ov[q] = pack_bf16(a.x, a.y);
      }
      *reinterpret_cast<uint4*>(yrow + (size_t)k * cs.ldy) = outv;
    }
  } else {
    if (blockIdx.x != 0) return;
    for (int idx = tid; idx < PT * p.H; idx += blockDim.x) {
      const int t = tok0 + idx / p.H, h = idx % p.H;
      if (t >= p.T) break;
      const size_t row = (size_t)bb * p.T + t;
      const float bv = __bfloat162float(p.b[row * p.ldb + h]);
      float beta = 1.f / (1.f + expf(-bv));
      beta = __bfloat162float(__float2bfloat16_rn(beta));   // sigmoid output in activation dtype
      if (p.allow_neg_eigval) beta *= 2.f;
      p.beta[row * p.H + h] = __float2bfloat16_rn(beta);
      const float av = __bfloat162float(p.a[row * p.lda + h]) + p.dt_bias[h];
      const float sp = av > 20.f ? av : log1pf(expf(av));   // F.softplus(beta=1, threshold=20)
      p.g[row * p.H + h] = -expf(p.A_log[h]) * sp;
    }
  }
}

// One warp per (token, head) row of D channels (D = 32 * EPL).
template <int EPL>
__global__ void __launch_bounds__(256) rmsnorm_gated_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ gate,
                                                            const float* __restrict__ w,
                                                            __nv_bfloat16* __restrict__ y,
                                                            int64_t rows, int heads, int64_t ldg,
                                                            float eps) {
  constexpr int D = 32 * EPL;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t tok = row / heads, h = row % heads;
  const __nv_bfloat16* xr = x + row * D + lane * EPL;
  const __nv_bfloat16* gr = gate + tok * ldg + h * D + lane * EPL;
  float xv[EPL], gv[EPL];
#pragma unroll
  for (int e = 0; e < EPL; e += 4) {
    uint2 rx = *reinterpret_cast<const uint2*>(xr + e);
    uint2 rg = *reinterpret_cast<const uint2*>(gr + e);
    const __nv_bfloat16* ex = reinterpret_cast<const __nv_bfloat16*>(&rx);
    const __nv_bfloat16* eg = reinterpret_cast<const __nv_bfloat16*>(&rg);
#pragma unroll
    for (int j = 0; j < 4; ++j) { xv[e + j] = __bfloat162float(ex[j]); gv[e + j] = __bfloat162float(eg[j]); }
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) ss += xv[e] * xv[e];
  ss = warp_sum(ss);
  const float rstd = 1.f / sqrtf(ss / D + eps);
#pragma unroll
  for (int e = 0; e < EPL; e += 4) {
    uint2 out;
    uint32_t* o32 = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      float r[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int ee = e + j + q;
        const float gg = gv[ee];
        r[q] = xv[ee] * rstd * w[lane * EPL + ee] * gg / (1.f + __expf(-gg));
      }
      o32[j / 2] = pack_bf16(r[0], r[1]);
    }
    *reinterpret_cast<uint2*>(y + row * D + lane * EPL + e) = out;
  }
}

// Attention prologue: y = RoPE(bf16(RMSNorm_dim(x) * w)) per token row, in place allowed.
// RMSNorm over the full `dim` channels (apex FusedRMSNorm as used at
// kairos_dit.py:437-438,453-454); RoPE per head on channel pairs (2j, 2j+1) as
// the complex product with (cos, sin) of the token (rope_apply, kairos_dit.py:324-329).
// Channel c of row t lives at base + (h / hpb) * bstride + t * ld + (h % hpb) * hd + c % hd,
// h = c / hd, so q/k can be read straight out of a destination-grouped projection.
// One CTA per RR rows (all loads issued up front), one 8-channel vector per
// thread and row (blockDim = dim / 8).
#ifndef KB_NORM_RR
#define KB_NORM_RR 4
#endif
constexpr int RR = KB_NORM_RR;
__global__ void rmsnorm_rope_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, int rows, int dim, int hd, int64_t ld,
                                    int hpb, int64_t bstride, const float* __restrict__ w,
                                    const float* __restrict__ cs, float eps) {
  __shared__ float red[RR][32];
  const int c = threadIdx.x * 8;
  const int h = c / hd, cc = c % hd;
  const int64_t coff = (int64_t)(h / hpb) * bstride + (int64_t)(h % hpb) * hd + cc;
  const int nw = (blockDim.x + 31) / 32;
  uint4 raw[RR];
#pragma unroll
  for (int q = 0; q < RR; ++q) {
    const int t = blockIdx.x * RR + q;
    raw[q] = t < rows ? *reinterpret_cast<const uint4*>(x + coff + (int64_t)t * ld) : make_uint4(0, 0, 0, 0);
  }
  float ss[RR];
#pragma unroll
  for (int q = 0; q < RR; ++q) {
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw[q]);
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) { const float v = __bfloat162float(e[j]); a += v * v; }
    ss[q] = warp_sum(a);
    if ((threadIdx.x & 31) == 0) red[q][threadIdx.x >> 5] = ss[q];
  }
  __syncthreads();
  float wv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) wv[j] = w ? w[c + j] : 1.f;
#pragma unroll
  for (int q = 0; q < RR; ++q) {
    const int t = blockIdx.x * RR + q;
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot += red[q][i];
    if (t >= rows) continue;
    const float rstd = 1.f / sqrtf(tot / dim + eps);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw[q]);
    // no table: plain RMSNorm (identity rotation)
    float4 cs0 = make_float4(1.f, 0.f, 1.f, 0.f), cs1 = cs0;
    if (cs) {
      const float* csr = cs + ((int64_t)t * (hd / 2) + cc / 2) * 2;
      cs0 = *reinterpret_cast<const float4*>(csr);
      cs1 = *reinterpret_cast<const float4*>(csr + 4);
    }
    const float co[4] = {cs0.x, cs0.z, cs1.x, cs1.z}, si[4] = {cs0.y, cs0.w, cs1.y, cs1.w};
    uint4 outv;
    uint32_t* ov = reinterpret_cast<uint32_t*>(&outv);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float a = bf16_round(__bfloat162float(e[j]) * rstd * wv[j]);
      const float bb = bf16_round(__bfloat162float(e[j + 1]) * rstd * wv[j + 1]);
      ov[j / 2] = pack_bf16(a * co[j / 2] - bb * si[j / 2], a * si[j / 2] + bb * co[j / 2]);
    }
    *reinterpret_cast<uint4*>(y + coff + (int64_t)t * ld) = outv;
  }
}

// ---------------------------------------------------------------------------
// Residual add + LayerNorm + modulation (the DiT block's norm sites,
// kairos_dit.py:873-874, 929-933, 955-957 and Head.forward :1047-1052):
//   x <- bf16(x + gate * r)                 (when r is given; gate NULL = 1)
//   y  = bf16(LN(x) * m + a),  m = (mul_plus_one ? 1 + mul : mul)  (mul NULL: m = 1; add NULL: a = 0)
// One CTA of dim/8 threads per LR rows; each thread holds 8 channels of a row in
// registers; mean and variance by two block reductions (two-pass, fp32).
// ---------------------------------------------------------------------------
// Rows per CTA of residual_ln_mod_kernel.  Each thread keeps its loads of all LR
// rows in flight before the first store; with LR = 2 and at most 56 registers
// three CTAs of 384 threads (3072 channels) fit on an SM.
#ifndef KB_LN_ROWS
#define KB_LN_ROWS 2
#endif
constexpr int LR = KB_LN_ROWS;
#ifndef KB_LN_REGS
#define KB_LN_REGS __maxnreg__(56)
#endif
__global__ void KB_LN_REGS residual_ln_mod_kernel(__nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r, int rows,
                                       int dim, int64_t ldr, const float* __restrict__ gate,
                                       const float* __restrict__ mul, const float* __restrict__ add, int plus_one,
                                       float eps, __nv_bfloat16* __restrict__ y) {
  __shared__ float red[2][LR][32];
  const int c = threadIdx.x * 8, nw = (blockDim.x + 31) / 32, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  // every load of the CTA's rows is issued before the first store (the residual
  // is written back in place)
  uint4 raw[LR], rr[LR];
#pragma unroll
  for (int q = 0; q < LR; ++q) {
    const int t = blockIdx.x * LR + q;
    raw[q] = rr[q] = make_uint4(0, 0, 0, 0);
    if (t < rows) {
      raw[q] = *reinterpret_cast<const uint4*>(x + (int64_t)t * dim + c);
      if (r) rr[q] = *reinterpret_cast<const uint4*>(r + (int64_t)t * ldr + c);
    }
  }
  float gv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) gv[j] = gate ? gate[c + j] : 1.f;
  float xv[LR][8];
#pragma unroll
  for (int q = 0; q < LR; ++q) {
    const int t = blockIdx.x * LR + q;
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw[q]);
    const __nv_bfloat16* er = reinterpret_cast<const __nv_bfloat16*>(&rr[q]);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = __bfloat162float(e[j]);
      if (r) v = bf16_round(fmaf(gv[j], __bfloat162float(er[j]), v));
      xv[q][j] = v;
      s += v;
    }
    if (r && t < rows) {
      uint4 o;
      uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 8; j += 2) ov[j / 2] = pack_bf16(xv[q][j], xv[q][j + 1]);
      *reinterpret_cast<uint4*>(x + (int64_t)t * dim + c) = o;
    }
    s = warp_sum(s);
    if (lane == 0) red[0][q][wid] = s;
  }
  __syncthreads();
  float mean[LR];
#pragma unroll
  for (int q = 0; q < LR; ++q) {
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot += red[0][q][i];
    mean[q] = tot / dim;
    float s2 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) { const float d = xv[q][j] - mean[q]; s2 = fmaf(d, d, s2); }
    s2 = warp_sum(s2);
    if (lane == 0) red[1][q][wid] = s2;
  }
  __syncthreads();
  float mv[8], av[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    mv[j] = mul ? (plus_one ? 1.f + mul[c + j] : mul[c + j]) : 1.f;
    av[j] = add ? add[c + j] : 0.f;
  }
#pragma unroll
  for (int q = 0; q < LR; ++q) {
    const int t = blockIdx.x * LR + q;
    if (t >= rows) continue;
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot += red[1][q][i];
    const float rstd = rsqrtf(tot / dim + eps);
    uint4 o;
    uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 8; j += 2)
      ov[j / 2] = pack_bf16(fmaf((xv[q][j] - mean[q]) * rstd, mv[j], av[j]),
                            fmaf((xv[q][j + 1] - mean[q]) * rstd, mv[j + 1], av[j + 1]));
    *reinterpret_cast<uint4*>(y + (int64_t)t * dim + c) = o;
  }
}

// ---------------------------------------------------------------------------
// Warp-per-row forms of the two row norms for dim = 256 NV (NV vectors of 8
// channels per lane; 3072 channels: NV = 12).  A warp owns a whole row, so no
// block barrier separates a row's loads from its stores: every lane issues all
// of its row's 16-byte loads up front and the warps of an SM stream
// independently (the CTA-per-rows forms above stall all their warps at the
// reduction barrier; they remain for other widths).
// ---------------------------------------------------------------------------
constexpr int WROWS = 8;   // rows (warps) per CTA

template <int NV>
__global__ void __launch_bounds__(WROWS * 32, 2) residual_ln_mod_warp_kernel(
    __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r, int rows, int64_t ldr,
    const float* __restrict__ gate, const float* __restrict__ mul, const float* __restrict__ add, int plus_one,
    float eps, __nv_bfloat16* __restrict__ y) {
  constexpr int dim = 256 * NV;
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * WROWS + (threadIdx.x >> 5);
  if (t >= rows) return;
  __nv_bfloat16* xr = x + (int64_t)t * dim;
  uint4 xv[NV], rv[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) xv[i] = *reinterpret_cast<const uint4*>(xr + (lane + 32 * i) * 8);
  if (r) {
#pragma unroll
    for (int i = 0; i < NV; ++i) rv[i] = *reinterpret_cast<const uint4*>(r + (int64_t)t * ldr + (lane + 32 * i) * 8);
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + 32 * i) * 8;
    uint32_t* xw = reinterpret_cast<uint32_t*>(&xv[i]);
    if (r) {
      const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rv[i]);
      float4 g0 = make_float4(1.f, 1.f, 1.f, 1.f), g1 = g0;
      if (gate) {
        g0 = *reinterpret_cast<const float4*>(gate + c);
        g1 = *reinterpret_cast<const float4*>(gate + c + 4);
      }
      const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack_bf16(xw[j]), b = unpack_bf16(rw[j]);
        xw[j] = pack_bf16(fmaf(gg[2 * j], b.x, a.x), fmaf(gg[2 * j + 1], b.y, a.y));
      }
      *reinterpret_cast<uint4*>(xr + c) = xv[i];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = unpack_bf16(xw[j]);
      s += a.x + a.y;
    }
  }
  const float mean = warp_sum(s) * (1.f / dim);
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = unpack_bf16(xw[j]);
      s2 = fmaf(a.x - mean, a.x - mean, s2);
      s2 = fmaf(a.y - mean, a.y - mean, s2);
    }
  }
  const float rstd = rsqrtf(warp_sum(s2) * (1.f / dim) + eps);
  __nv_bfloat16* yr = y + (int64_t)t * dim;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + 32 * i) * 8;
    float mm[8], aa[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { mm[j] = 1.f; aa[j] = 0.f; }
    if (mul) {
      const float4 m0 = *reinterpret_cast<const float4*>(mul + c), m1 = *reinterpret_cast<const float4*>(mul + c + 4);
      mm[0] = m0.x; mm[1] = m0.y; mm[2] = m0.z; mm[3] = m0.w; mm[4] = m1.x; mm[5] = m1.y; mm[6] = m1.z; mm[7] = m1.w;
      if (plus_one) {
#pragma unroll
        for (int j = 0; j < 8; ++j) mm[j] += 1.f;
      }
    }
    if (add) {
      const float4 a0 = *reinterpret_cast<const float4*>(add + c), a1 = *reinterpret_cast<const float4*>(add + c + 4);
      aa[0] = a0.x; aa[1] = a0.y; aa[2] = a0.z; aa[3] = a0.w; aa[4] = a1.x; aa[5] = a1.y; aa[6] = a1.z; aa[7] = a1.w;
    }
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[i]);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = unpack_bf16(xw[j]);
      ow[j] = pack_bf16(fmaf((a.x - mean) * rstd, mm[2 * j], aa[2 * j]),
                        fmaf((a.y - mean) * rstd, mm[2 * j + 1], aa[2 * j + 1]));
    }
    *reinterpret_cast<uint4*>(yr + c) = o;
    // keep the per-channel vector loads of the next vector below this store: hoisting
    // all of them would not fit the register budget
    asm volatile("" ::: "memory");
  }
}

template <int NV>
__global__ void __launch_bounds__(WROWS * 32, 2) rmsnorm_rope_warp_kernel(
    const __nv_bfloat16* x, __nv_bfloat16* y, int rows, int hd, int64_t ld, int hpb, int64_t bstride,
    const float* __restrict__ w, const float* __restrict__ cs, float eps) {
  constexpr int dim = 256 * NV;
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * WROWS + (threadIdx.x >> 5);
  if (t >= rows) return;
  uint4 xv[NV];
  auto offset = [&](int c) {
    const int h = c / hd;
    return (int64_t)(h / hpb) * bstride + (int64_t)(h % hpb) * hd + c % hd + (int64_t)t * ld;
  };
#pragma unroll
  for (int i = 0; i < NV; ++i) xv[i] = *reinterpret_cast<const uint4*>(x + offset((lane + 32 * i) * 8));
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = unpack_bf16(xw[j]);
      ss = fmaf(a.x, a.x, fmaf(a.y, a.y, ss));
    }
  }
  const float rstd = 1.f / sqrtf(warp_sum(ss) / dim + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + 32 * i) * 8, cc = c % hd;
    float wv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) wv[j] = 1.f;
    if (w) {
      const float4 w0 = *reinterpret_cast<const float4*>(w + c), w1 = *reinterpret_cast<const float4*>(w + c + 4);
      wv[0] = w0.x; wv[1] = w0.y; wv[2] = w0.z; wv[3] = w0.w; wv[4] = w1.x; wv[5] = w1.y; wv[6] = w1.z; wv[7] = w1.w;
    }
    float4 cs0 = make_float4(1.f, 0.f, 1.f, 0.f), cs1 = cs0;   // no table: identity rotation
    if (cs) {
      const float* csr = cs + ((int64_t)t * (hd / 2) + cc / 2) * 2;
      cs0 = *reinterpret_cast<const float4*>(csr);
      cs1 = *reinterpret_cast<const float4*>(csr + 4);
    }
    const float co[4] = {cs0.x, cs0.z, cs1.x, cs1.z}, si[4] = {cs0.y, cs0.w, cs1.y, cs1.w};
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[i]);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 e = unpack_bf16(xw[j]);
      const float a = bf16_round(e.x * rstd * wv[2 * j]);
      const float b = bf16_round(e.y * rstd * wv[2 * j + 1]);
      ow[j] = pack_bf16(a * co[j] - b * si[j], a * si[j] + b * co[j]);
    }
    *reinterpret_cast<uint4*>(y + offset(c)) = o;
    asm volatile("" ::: "memory");   // as in residual_ln_mod_warp_kernel
  }
}

}  // namespace fuse
}  // namespace kb

// ===========================================================================
// Host side: C ABI
// ===========================================================================
using namespace kb;

extern "C" int kb200_gdn_prologue(const KB200GdnPrologueArgs* a, void* stream) {
  if (!a) return set_error(KB200_ERR_INVALID, "gdn_prologue: null args");
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->W < 1 || a->W > 4)
    return set_error(KB200_ERR_INVALID, "gdn_prologue: bad shape (B,T,H > 0, 1 <= W <= 4)");
  fuse::PrologueParams p{};
  const void* xs[3] = {a->xq, a->xk, a->xv};
  const float* ws[3] = {a->wq, a->wk, a->wv};
  const float* bs[3] = {a->bq, a->bk, a->bv};
  void* ys[3] = {a->q, a->k, a->v};
  const int64_t cs[3] = {a->Cqk, a->Cqk, a->Cv};
  const int64_t lx[3] = {a->ldq, a->ldk, a->ldv};
  const void* cc[3] = {a->cache_q, a->cache_k, a->cache_v};
  int maxc = 0;
  for (int i = 0; i < 3; ++i) {
    if (!xs[i] || !ws[i] || !ys[i]) return set_error(KB200_ERR_INVALID, "gdn_prologue: null tensor");
    if (cs[i] <= 0 || cs[i] % 8 || lx[i] % 8 || !aligned16(xs[i]) || !aligned16(ys[i]))
      return set_error(KB200_ERR_ALIGN, "gdn_prologue: channels/strides must be multiples of 8, rows 16-byte aligned");
    p.set[i] = fuse::ConvSet{(const __nv_bfloat16*)xs[i], ws[i], bs[i], (__nv_bfloat16*)ys[i], (int)cs[i],
                             lx[i], cs[i], (const __nv_bfloat16*)cc[i]};
    maxc = maxc > (int)cs[i] ? maxc : (int)cs[i];
  }
  if (!a->a || !a->b || !a->A_log || !a->dt_bias || !a->g || !a->beta)
    return set_error(KB200_ERR_INVALID, "gdn_prologue: null gate tensor");
  p.a = (const __nv_bfloat16*)a->a;
  p.b = (const __nv_bfloat16*)a->b;
  p.lda = a->lda;
  p.ldb = a->ldb;
  p.A_log = a->A_log;
  p.dt_bias = a->dt_bias;
  p.g = a->g;
  p.beta = (__nv_bfloat16*)a->beta;
  p.B = (int)a->B;
  p.T = (int)a->T;
  p.H = (int)a->H;
  p.W = a->W;
  p.allow_neg_eigval = a->allow_neg_eigval;
  dim3 grid((unsigned)((maxc + fuse::PC - 1) / fuse::PC), (unsigned)((a->T + fuse::PT - 1) / fuse::PT),
            (unsigned)(a->B * 4));
  fuse::gdn_prologue_kernel<<<grid, fuse::PTHREADS, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("gdn_prologue_kernel");
}

extern "C" int kb200_rmsnorm_gated(const void* x, const void* gate, const float* weight, void* y,
                                   int64_t rows, int64_t heads, int64_t D, int64_t ld_gate,
                                   float eps, void* stream) {
  if (!x || !gate || !weight || !y) return set_error(KB200_ERR_INVALID, "rmsnorm_gated: null pointer");
  if (rows < 0 || heads <= 0 || rows % heads)
    return set_error(KB200_ERR_INVALID, "rmsnorm_gated: rows must be a multiple of heads");
  if (D != 128 && D != 256 && D != 512)
    return set_error(KB200_ERR_INVALID, "rmsnorm_gated: D must be 128, 256 or 512");
  if (ld_gate % 4 || !aligned16(x) || !aligned16(y) || (reinterpret_cast<uintptr_t>(gate) & 7))
    return set_error(KB200_ERR_ALIGN, "rmsnorm_gated: misaligned tensor or gate stride");
  if (rows == 0) return KB200_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((rows + 7) / 8);
  const int hh = (int)heads;
  const __nv_bfloat16* xb = (const __nv_bfloat16*)x;
  const __nv_bfloat16* gb = (const __nv_bfloat16*)gate;
  __nv_bfloat16* yb = (__nv_bfloat16*)y;
  if (D == 128) fuse::rmsnorm_gated_kernel<4><<<grid, 256, 0, st>>>(xb, gb, weight, yb, rows, hh, ld_gate, eps);
  else if (D == 256) fuse::rmsnorm_gated_kernel<8><<<grid, 256, 0, st>>>(xb, gb, weight, yb, rows, hh, ld_gate, eps);
  else fuse::rmsnorm_gated_kernel<16><<<grid, 256, 0, st>>>(xb, gb, weight, yb, rows, hh, ld_gate, eps);
  return check_launch("rmsnorm_gated_kernel");
}

extern "C" int kb200_rmsnorm_rope(const void* x, void* y, int64_t rows, int64_t dim, int64_t head_dim,
                                  int64_t ld, int64_t heads_per_block, int64_t block_stride,
                                  const float* weight, const float* cos_sin, float eps, void* stream) {
  if (!x || !y) return set_error(KB200_ERR_INVALID, "rmsnorm_rope: null pointer");
  if (rows < 0 || dim <= 0 || dim % 8 || dim / 8 > 1024 || head_dim <= 0 || head_dim % 8 ||
      dim % head_dim || heads_per_block <= 0)
    return set_error(KB200_ERR_INVALID, "rmsnorm_rope: need dim %% 8 == 0, dim <= 8192, head_dim | dim");
  if (ld % 8 || block_stride % 8 || !aligned16(x) || !aligned16(y))
    return set_error(KB200_ERR_ALIGN, "rmsnorm_rope: rows must be 16-byte aligned");
  if (rows == 0) return KB200_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned wgrid = (unsigned)((rows + fuse::WROWS - 1) / fuse::WROWS);
#define KB_RMS_WARP(NV)                                                                                       if (dim == 256 * NV) {                                                                                        fuse::rmsnorm_rope_warp_kernel<NV><<<wgrid, fuse::WROWS * 32, 0, st>>>(                                         (const __nv_bfloat16*)x, (__nv_bfloat16*)y, (int)rows, (int)head_dim, ld, (int)heads_per_block,             block_stride, weight, cos_sin, eps);                                                                    return check_launch("rmsnorm_rope_warp_kernel");                                                           }
  KB_RMS_WARP(1) KB_RMS_WARP(2) KB_RMS_WARP(4) KB_RMS_WARP(8) KB_RMS_WARP(12)
#undef KB_RMS_WARP
  fuse::rmsnorm_rope_kernel<<<(unsigned)((rows + fuse::RR - 1) / fuse::RR), (unsigned)(dim / 8), 0,
                               static_cast<cudaStream_t>(stream)>>>(
      (const __nv_bfloat16*)x, (__nv_bfloat16*)y, (int)rows, (int)dim, (int)head_dim, ld, (int)heads_per_block,
      block_stride, weight, cos_sin, eps);
  return check_launch("rmsnorm_rope_kernel");
}

extern "C" int kb200_residual_ln_mod(void* x, const void* r, int64_t rows, int64_t dim, int64_t ld_r,
                                     const float* gate, const float* mul, const float* add, int mul_plus_one,
                                     float eps, void* y, void* stream) {
  if (!x || !y) return set_error(KB200_ERR_INVALID, "residual_ln_mod: null pointer");
  if (rows < 0 || dim <= 0 || dim % 8 || dim / 8 > 1024)
    return set_error(KB200_ERR_INVALID, "residual_ln_mod: need dim %% 8 == 0 and dim <= 8192");
  if (!aligned16(x) || !aligned16(y) || (r && (!aligned16(r) || ld_r % 8 || ld_r < dim)))
    return set_error(KB200_ERR_ALIGN, "residual_ln_mod: rows must be 16-byte aligned");
  if (x == y) return set_error(KB200_ERR_INVALID, "residual_ln_mod: y must not alias x");
  if (rows == 0) return KB200_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned wgrid = (unsigned)((rows + fuse::WROWS - 1) / fuse::WROWS);
#define KB_LN_WARP(NV)                                                                                        if (dim == 256 * NV) {                                                                                        fuse::residual_ln_mod_warp_kernel<NV><<<wgrid, fuse::WROWS * 32, 0, st>>>(                                      (__nv_bfloat16*)x, (const __nv_bfloat16*)r, (int)rows, r ? ld_r : dim, gate, mul, add, mul_plus_one,         eps, (__nv_bfloat16*)y);                                                                                return check_launch("residual_ln_mod_warp_kernel");                                                        }
  KB_LN_WARP(1) KB_LN_WARP(2) KB_LN_WARP(4) KB_LN_WARP(8) KB_LN_WARP(12)
#undef KB_LN_WARP
  fuse::residual_ln_mod_kernel<<<(unsigned)((rows + fuse::LR - 1) / fuse::LR), (unsigned)(dim / 8), 0,
                                 static_cast<cudaStream_t>(stream)>>>(
      (__nv_bfloat16*)x, (const __nv_bfloat16*)r, (int)rows, (int)dim, r ? ld_r : dim, gate, mul, add,
      mul_plus_one, eps, (__nv_bfloat16*)y);
  return check_launch("residual_ln_mod_kernel");
}
