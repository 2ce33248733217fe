// attn_fp8.cu -- non-causal softmax attention with FP8-e4m3 Q/K/V and
// per-head amax scaling, bf16 output (sm_100a).
//
// Replaces the attention core behind AttentionModule.forward
// (kairos/modules/dits/kairos_dit.py:367-373 -> flash_attention :232-277),
// i.e. softmax(q k^T / sqrt(d)) v per head, q/k/v given as [B, S, H*D] bf16.
//
// Launch sequence of kb200_attn_fp8_fwd:
//   1. attn_amax_kernel     per-(tensor, batch, head) max |x| over the sequence
//   2. attn_quant_kernel    x / (amax/448) -> e4m3; Q,K as [B,H,S_pad,D];
//                           V transposed to [B,H,D,S_pad] so the P.V contraction
//                           reads V with the token dimension contiguous.  With
//                           two_term, q and v also get the e4m3 rounding
//                           residual (same scale) as a second term.
//   3. attention kernel     flash-attention forward: S = Q K^T (e4m3 tensor
//                           cores, fp32 accumulate), online softmax in fp32 on
//                           exp2, P quantised to e4m3, O += P V, O / l -> bf16
#include "common.cuh"
#include "kb200_internal.h"
#include "attn_common.cuh"
#include <cstdlib>

namespace kb {
namespace attn {

// ---------------------------------------------------------------------------
// 1. amax.  Grid (ceil(S/32), B); 256 threads; D = 128 (one 16-byte vector per
// lane covers 8 channels, 16 lanes cover one head).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) attn_amax_kernel(Params p) {
  extern __shared__ float red[];  // [3 * H]
  const int b = blockIdx.y, H = p.H, HD = H * D;
  for (int i = threadIdx.x; i < 3 * H; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  const int t0 = blockIdx.x * 32, t1 = min(p.S, t0 + 32);
  const int vecs_per_tok = HD / 8;
  for (int tsr = 0; tsr < 3; ++tsr) {
    const __nv_bfloat16* x = tsr == 0 ? p.q : (tsr == 1 ? p.k : p.v);
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
  for (int i = threadIdx.x; i < 3 * H; i += blockDim.x) {
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
  __shared__ __align__(16) uint8_t vt[D][64 + 16];
  __shared__ __align__(16) uint8_t vtr[D][64 + 16];
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H, H = p.H;
  const int t0 = blockIdx.x * 64;
  const float rq = 1.f / scale_of(p.amax[(0 * p.B + b) * H + h]);
  const float rk = 1.f / scale_of(p.amax[(1 * p.B + b) * H + h]);
  const float rv = 1.f / scale_of(p.amax[(2 * p.B + b) * H + h]);
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
    uint2 oq, ok;
    oq.x = quant8(eq, rq, 0);
    oq.y = quant8(eq, rq, 4);
    ok.x = quant8(ek, rk, 0);
    ok.y = quant8(ek, rk, 4);
    const size_t qoff = ((size_t)bh * p.S_pad + t) * D + c;
    *reinterpret_cast<uint2*>(p.q8 + qoff) = oq;
    *reinterpret_cast<uint2*>(p.k8 + qoff) = ok;
    if (p.two_term) {
      uint2 res;
      uint8_t* rq8 = reinterpret_cast<uint8_t*>(&res);
      const uint8_t* hq = reinterpret_cast<const uint8_t*>(&oq);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float x = __bfloat162float(eq[j]) * rq;
        rq8[j] = (uint8_t)__nv_cvt_float_to_fp8(x - e4m3_to_float(hq[j]), __NV_SATFINITE, __NV_E4M3);
      }
      *reinterpret_cast<uint2*>(p.q8r + qoff) = res;
    }
    // V: position of token r inside its 16-group (fragment order when vperm)
    int pos = r;
    if (p.vperm) {
      const int kk = r & 15, base = r & ~15;
      pos = base + (kk < 8 ? 4 * (kk >> 1) + (kk & 1) : 4 * ((kk - 8) >> 1) + 2 + (kk & 1));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = __bfloat162float(ev[j]) * rv;
      __nv_fp8_storage_t e = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
      vt[c + j][pos] = (uint8_t)e;
      vtr[c + j][pos] = (uint8_t)__nv_cvt_float_to_fp8(x - e4m3_to_float(e), __NV_SATFINITE, __NV_E4M3);
    }
  }
  __syncthreads();
  // write the V^T tile: D rows x 64 tokens
  for (int idx = threadIdx.x; idx < D * 4; idx += blockDim.x) {
    const int d = idx >> 2, seg = (idx & 3) * 16;
    *reinterpret_cast<uint4*>(p.vt8 + ((size_t)bh * D + d) * p.S_pad + t0 + seg) =
        *reinterpret_cast<const uint4*>(&vt[d][seg]);
    if (p.two_term)
      *reinterpret_cast<uint4*>(p.vt8r + ((size_t)bh * D + d) * p.S_pad + t0 + seg) =
          *reinterpret_cast<const uint4*>(&vtr[d][seg]);
  }
}

// ---------------------------------------------------------------------------
// 3a. attention on mma.sync (m16n8k32 e4m3).  Grid (S_pad / BM, B * H); 8 warps,
// warp w owns query rows 16w..16w+15 of the BM = 128 tile.  K and V^T tiles of
// BN = 64 tokens stream through a STAGES-deep cp.async ring.  Row strides are
// padded by 16 bytes so ldmatrix row reads are bank-conflict free.
// ---------------------------------------------------------------------------
KB_DEVI void mma_e4m3(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <int D, int BM, int BN, int STAGES>
struct MmaSmem {
  static constexpr int LDQ = D + 16, LDK = D + 16, LDV = BN + 16;  // bytes
  uint8_t qs[2][BM * LDQ];        // e4m3 q and its residual term
  uint8_t ks[STAGES][BN * LDK];
  uint8_t vs[STAGES][2][D * LDV];  // e4m3 v^T and its residual term
};

template <int D, int BM, int BN, int STAGES, int TT>
__global__ void __launch_bounds__(256) attn_fp8_mma_kernel(Params p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  using S = MmaSmem<D, BM, BN, STAGES>;
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int q0 = blockIdx.x * BM;
  const uint8_t* qg = p.q8 + ((size_t)bh * p.S_pad + q0) * D;
  const uint8_t* qgr = p.q8r + ((size_t)bh * p.S_pad + q0) * D;
  const uint8_t* kg = p.k8 + (size_t)bh * p.S_pad * D;
  const uint8_t* vg = p.vt8 + (size_t)bh * D * p.S_pad;
  const uint8_t* vgr = p.vt8r + (size_t)bh * D * p.S_pad;
  const int ntiles = (p.S + BN - 1) / BN;

  auto load_kv = [&](int j, int st) {
    const int k0 = j * BN;
    for (int idx = tid; idx < BN * (D / 16); idx += 256) {
      const int r = idx / (D / 16), c = (idx % (D / 16)) * 16;
      cp_async16(&sm.ks[st][r * S::LDK + c], kg + (size_t)(k0 + r) * D + c, true);
    }
    for (int idx = tid; idx < D * (BN / 16); idx += 256) {
      const int r = idx / (BN / 16), c = (idx % (BN / 16)) * 16;
      cp_async16(&sm.vs[st][0][r * S::LDV + c], vg + (size_t)r * p.S_pad + k0 + c, true);
      if (TT == 2) cp_async16(&sm.vs[st][1][r * S::LDV + c], vgr + (size_t)r * p.S_pad + k0 + c, true);
    }
  };
  for (int idx = tid; idx < BM * (D / 16); idx += 256) {
    const int r = idx / (D / 16), c = (idx % (D / 16)) * 16;
    cp_async16(&sm.qs[0][r * S::LDQ + c], qg + (size_t)r * D + c, true);
    if (TT == 2) cp_async16(&sm.qs[1][r * S::LDQ + c], qgr + (size_t)r * D + c, true);
  }
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < ntiles) load_kv(s, s);
    cp_async_commit();
  }
  const float sq = scale_of(p.amax[(0 * p.B + b) * p.H + h]);
  const float sk = scale_of(p.amax[(1 * p.B + b) * p.H + h]);
  const float sv = scale_of(p.amax[(2 * p.B + b) * p.H + h]);
  const float sl2 = sq * sk * p.softmax_scale * 1.4426950408889634f;

  uint32_t qf[TT][D / 32][4];
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int tt = 0; tt < TT; ++tt)
#pragma unroll
        for (int ks = 0; ks < D / 32; ++ks)
          load_a_rowmajor(qf[tt][ks], reinterpret_cast<const __nv_bfloat16*>(sm.qs[tt]), S::LDQ / 2,
                          warp * 16, ks * 16, lane);
    }
    {
      const int jn = j + STAGES - 1;
      if (jn < ntiles) load_kv(jn, jn % STAGES);
      cp_async_commit();
    }
    const int st = j % STAGES;
    const __nv_bfloat16* ksb = reinterpret_cast<const __nv_bfloat16*>(sm.ks[st]);
    float s[BN / 8][4];
#pragma unroll
    for (int i = 0; i < BN / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 32; ++ks)
#pragma unroll
      for (int n0 = 0; n0 < BN; n0 += 16) {
        uint32_t bb[4];
        load_b_nmajor_rows_x2n(bb, ksb, S::LDK / 2, ks * 16, n0, lane);
#pragma unroll
        for (int tt = 0; tt < TT; ++tt) {
          mma_e4m3(s[n0 / 8], qf[tt][ks], bb);
          mma_e4m3(s[n0 / 8 + 1], qf[tt][ks], bb + 2);
        }
      }
    // scale to the log2 domain, mask the ragged tail
    const int kbase = j * BN;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int i = 0; i < BN / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + i * 8 + 2 * t4 + (e & 1);
        float x = s[i][e] * sl2;
        if (key >= p.S) x = -INFINITY;
        s[i][e] = x;
        if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // P is formed as 2^(x - m + 8) in (0, 256] so that e4m3 keeps its precision
    const float a0 = exp2f(m0 - mx0), a1 = exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    const float b0 = mx0 - 8.f, b1 = mx1 - 8.f;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int i = 0; i < BN / 8; ++i) {
      s[i][0] = exp2f(s[i][0] - b0);
      s[i][1] = exp2f(s[i][1] - b0);
      s[i][2] = exp2f(s[i][2] - b1);
      s[i][3] = exp2f(s[i][3] - b1);
      rs0 += s[i][0] + s[i][1];
      rs1 += s[i][2] + s[i][3];
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= a0; o[i][1] *= a0;
      o[i][2] *= a1; o[i][3] *= a1;
    }
    // P (e4m3) fragments: a k-step of 32 keys = n-tiles 4ks..4ks+3 (the token
    // order inside 16-groups matches the permuted V^T layout of the quantiser)
#pragma unroll
    for (int ks = 0; ks < BN / 32; ++ks) {
      uint32_t pa[4];
      const int n = ks * 4;
      pa[0] = f2_to_e4m3x2(s[n][0], s[n][1]) | (f2_to_e4m3x2(s[n + 1][0], s[n + 1][1]) << 16);
      pa[1] = f2_to_e4m3x2(s[n][2], s[n][3]) | (f2_to_e4m3x2(s[n + 1][2], s[n + 1][3]) << 16);
      pa[2] = f2_to_e4m3x2(s[n + 2][0], s[n + 2][1]) | (f2_to_e4m3x2(s[n + 3][0], s[n + 3][1]) << 16);
      pa[3] = f2_to_e4m3x2(s[n + 2][2], s[n + 2][3]) | (f2_to_e4m3x2(s[n + 3][2], s[n + 3][3]) << 16);
#pragma unroll
      for (int tt = 0; tt < TT; ++tt) {
        const __nv_bfloat16* vsb = reinterpret_cast<const __nv_bfloat16*>(sm.vs[st][tt]);
#pragma unroll
        for (int d0 = 0; d0 < D; d0 += 16) {
          uint32_t bb[4];
          load_b_nmajor_rows_x2n(bb, vsb, S::LDV / 2, ks * 16, d0, lane);
          mma_e4m3(o[d0 / 8], pa, bb);
          mma_e4m3(o[d0 / 8 + 1], pa, bb + 2);
        }
      }
    }
  }
  cp_async_wait<0>();
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float f0 = sv / l0, f1 = sv / l1;
  const int r0 = q0 + warp * 16 + g8, r1 = r0 + 8;
  const size_t HD = (size_t)p.H * D;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int c = h * D + i * 8 + 2 * t4;
    if (r0 < p.S)
      *reinterpret_cast<uint32_t*>(p.o + ((size_t)b * p.S + r0) * HD + c) = pack_bf16(o[i][0] * f0, o[i][1] * f0);
    if (r1 < p.S)
      *reinterpret_cast<uint32_t*>(p.o + ((size_t)b * p.S + r1) * HD + c) = pack_bf16(o[i][2] * f1, o[i][3] * f1);
  }
}

}  // namespace attn
}  // namespace kb

// ===========================================================================
// Host side: C ABI
// ===========================================================================
namespace {
using namespace kb;
constexpr int AD = 128, ABM = 128, ABN = 64, ASTAGES = 3;

struct AttnWs { size_t q8, k8, vt8, q8r, vt8r, amax, err, total; int S_pad; };

AttnWs attn_ws(int64_t B, int64_t S, int64_t H, int two_term) {
  AttnWs w{};
  w.S_pad = (int)((S + 255) / 256 * 256);
  const size_t n = (size_t)B * H * w.S_pad * AD;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes); return o; };
  w.q8 = take(n);
  w.k8 = take(n);
  w.vt8 = take(n);
  w.q8r = take(two_term ? n : 0);
  w.vt8r = take(two_term ? n : 0);
  w.amax = take((size_t)3 * B * H * 4 + 16);   // amax, then the device error word
  w.err = w.amax + (size_t)3 * B * H * 4;
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

extern "C" size_t kb200_attn_fp8_workspace_size(int64_t B, int64_t S, int64_t H, int64_t D,
                                                int two_term) {
  if (D != AD || B <= 0 || S <= 0 || H <= 0) return 0;
  return attn_ws(B, S, H, two_term).total;
}

namespace {
// KB200_ATTN_MMA_SYNC=1 selects the mma.sync kernel (kept only for A/B timing while the
// tcgen05 kernel is brought up).
bool use_tc() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("KB200_ATTN_MMA_SYNC");
    v = (e && e[0] == '1') ? 0 : 1;
  }
  return v == 1;
}

int attn_setup(attn::Params& p, AttnWs& w, const void* q, const void* k, const void* v, void* o,
               int64_t B, int64_t S, int64_t H, int64_t D, int64_t row_stride, float softmax_scale,
               int two_term, void* workspace, size_t workspace_bytes) {
  if (int e = attn_validate(q, k, v, o, B, S, H, D)) return e;
  if (row_stride == 0) row_stride = H * D;
  if (row_stride < H * D || row_stride % 8)
    return set_error(KB200_ERR_ALIGN, "attn_fp8: row_stride must be >= H*D and a multiple of 8");
  w = attn_ws(B, S, H, two_term);
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
  p.vt8 = (uint8_t*)(ws + w.vt8);
  p.q8r = (uint8_t*)(ws + w.q8r);
  p.vt8r = (uint8_t*)(ws + w.vt8r);
  p.amax = (float*)(ws + w.amax);
  p.B = (int)B;
  p.S = (int)S;
  p.H = (int)H;
  p.S_pad = w.S_pad;
  p.ld = row_stride;
  p.softmax_scale = softmax_scale;
  p.vperm = use_tc() ? 0 : 1;
  p.two_term = two_term ? 1 : 0;
  return KB200_OK;
}

int attn_quantize(const attn::Params& p, const AttnWs& w, cudaStream_t st) {
  if (cudaMemsetAsync(p.amax, 0, (size_t)3 * p.B * p.H * 4 + 16, st) != cudaSuccess)
    return check_launch("attn_fp8 amax memset");
  attn::attn_amax_kernel<AD><<<dim3((unsigned)((p.S + 31) / 32), (unsigned)p.B), 256, 3 * p.H * 4, st>>>(p);
  if (int e = check_launch("attn_amax_kernel")) return e;
  attn::attn_quant_kernel<AD><<<dim3(w.S_pad / 64, (unsigned)(p.B * p.H)), 256, 0, st>>>(p);
  return check_launch("attn_quant_kernel");
}

int attn_attend(const attn::Params& p, const AttnWs& w, cudaStream_t st) {
  if (!p.vperm) return attn::launch_attn_tc(p, reinterpret_cast<int*>(reinterpret_cast<char*>(p.amax) + (w.err - w.amax)), st);
  const size_t smem = sizeof(attn::MmaSmem<AD, ABM, ABN, ASTAGES>);
  auto kern = p.two_term ? attn::attn_fp8_mma_kernel<AD, ABM, ABN, ASTAGES, 2>
                         : attn::attn_fp8_mma_kernel<AD, ABM, ABN, ASTAGES, 1>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<dim3(w.S_pad / ABM, (unsigned)(p.B * p.H)), 256, smem, st>>>(p);
  return check_launch("attn_fp8_mma_kernel");
}
}  // namespace

#define KB_ATTN_ARGS                                                                         \
  const void *q, const void *k, const void *v, void *o, int64_t B, int64_t S, int64_t H,    \
      int64_t D, int64_t row_stride, float softmax_scale, int two_term, void *workspace,           \
      size_t workspace_bytes, void *stream
#define KB_ATTN_SETUP                                                                          \
  attn::Params p;                                                                              \
  AttnWs w;                                                                                    \
  if (int e = attn_setup(p, w, q, k, v, o, B, S, H, D, row_stride, softmax_scale, two_term, workspace, \
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

extern "C" int kb200_attn_fp8_status(const void* workspace, int64_t B, int64_t S, int64_t H, int two_term,
                                     void* stream) {
  if (!workspace || B <= 0 || S <= 0 || H <= 0) return set_error(KB200_ERR_INVALID, "attn_fp8_status: bad args");
  const AttnWs w = attn_ws(B, S, H, two_term);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int code = 0;
  if (cudaMemcpyAsync(&code, static_cast<const char*>(workspace) + w.err, sizeof(int), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return check_launch("attn_fp8_status");
  if (code != 0) return set_error(KB200_ERR_TIMEOUT, "attn_fp8: a device-side wait gave up (site %d)", code);
  return KB200_OK;
}
