// attn_fp8_tc.cu -- FP8 (e4m3) flash-attention forward on 5th-generation
// tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// One CTA per (two 128-query tiles, batch*head); keys in tiles of BN = 128.
//   warp 8      : TMA producer (Q once; K, V^T (+ residual terms) per key tile
//                 into a STAGES-deep ring)
//   warp 9      : MMA issuer (one elected thread) and TMEM owner
//                 S_t = Q_t K_j^T  -> TMEM S[t]   (kind::f8f6f4, f32 accumulate)
//                 O_t += P_t V_j   -> TMEM O[t]   (P_t from shared memory)
//   warps 0..7  : softmax, warpgroup t for query tile t, one thread per row / TMEM lane:
//                 S row from TMEM -> running max (lazy rescale of O when the
//                 max grows by more than TAU) -> P = 2^(s - m + SHIFT) as e4m3
//                 into a 128B-swizzled smem tile -> final O / l -> bf16.
// The two query tiles ping-pong: while one warpgroup exponentiates its scores
// the tensor pipe computes the other tile's scores or products, and the MMA
// warp issues QK(j+1) before PV(j).
//
// Every mbarrier wait is bounded; a wait that gives up records an error code in
// the workspace and the CTA skips the rest of its work, frees TMEM and exits.
#include "attn_common.cuh"
#include "kb200_internal.h"
#include "tc_common.cuh"

namespace kb {
namespace attn {

constexpr int TC_BM = 128, TC_BN = 128, TC_D = 128;
constexpr int TC_QT = 2;          // query tiles per CTA (ping-pong between two softmax warpgroups)
constexpr float TC_SHIFT = 6.f;   // P = 2^(s - m + SHIFT): keeps small probabilities out of e4m3 subnormals
constexpr float TC_TAU = 2.5f;    // lazy-rescale threshold (log2 units); P <= 2^(SHIFT+TAU) < 448

template <int TT>
struct TcSmem {
  // K and V^T have separate rings: a K tile is free once both QK products that
  // read it are done, a V tile only after both PV products.
  static constexpr int KS = 3, VS = TT == 2 ? 2 : 3;
  uint8_t q[TC_QT][TT][TC_BM * TC_D];           // e4m3 q (+ residual term)        SW128 K-major
  uint8_t p[TC_QT][TC_BM * TC_BN];              // e4m3 probabilities               SW128 K-major (keys)
  uint8_t k[KS][TC_BN * TC_D];                  // e4m3 k tiles                     SW128 K-major
  uint8_t v[VS][TT][TC_D * TC_BN];              // e4m3 v^T tiles (+ residual)      SW128 K-major (keys)
  uint64_t q_full;
  uint64_t k_full[KS], k_empty[KS], v_full[VS], v_empty[VS];
  uint64_t s_full[TC_QT], s_free[TC_QT], p_full[TC_QT], pv_done[TC_QT];
  uint64_t o_done[TC_QT];
  uint32_t tmem_base;
  int abort_flag;
};

struct TcMaps {
  CUtensorMap q, qr, k, vt, vtr;
};

#ifdef KB_ATTN_TRACE
#define TRACE(slot, j) do { if (p.trace && blockIdx.x == 0 && blockIdx.y == 0) p.trace[(j) * 16 + (slot)] = clock64(); } while (0)
#else
#define TRACE(slot, j) do { } while (0)
#endif

template <class S>
KB_DEVI void fail(S& sm, int* err, int code) {
  sm.abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
}

KB_DEVI float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


KB_DEVI float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair on the FMA pipe, to share the exponential load with the MUFU
// unit.  Round-to-nearest split x = j + f (f in [-1/2, 1/2]) with the
// 1.5 * 2^23 addition trick; 2^f by a degree-3 polynomial whose coefficients
// were fitted here (iteratively reweighted least squares on relative error,
// max relative error 1.0e-4 -- far below the e4m3 step of the probabilities it
// feeds); 2^j is added into the exponent field.  x < -127 flushes to 0.
KB_DEVI float2 exp2_poly2(float2 x) {
  constexpr float C = 12582912.f;   // 1.5 * 2^23
  x.x = fmaxf(x.x, -127.f);
  x.y = fmaxf(x.y, -127.f);
  const float2 t = fadd2(x, make_float2(C, C));
  const float2 jf = fadd2(t, make_float2(-C, -C));
  const float2 f = ffma2(jf, make_float2(-1.f, -1.f), x);
  float2 q = ffma2(make_float2(0.055008627f, 0.055008627f), f, make_float2(0.24221043f, 0.24221043f));
  q = ffma2(q, f, make_float2(0.69328302f, 0.69328302f));
  q = ffma2(q, f, make_float2(1.f, 1.f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// Block: warps 0-3 softmax for query tile 0, warps 4-7 for query tile 1,
// warp 8 TMA producer of Q and K, warp 9 MMA issuer of tile 0 + TMEM owner,
// warp 10 TMA producer of V^T, warp 11 MMA issuer of tile 1.
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
template <int TT>
__global__ void __launch_bounds__(384, 1) attn_fp8_tc_kernel(const __grid_constant__ TcMaps maps, Params p,
                                                             int* err) {
  using SM = TcSmem<TT>;
  constexpr int KS = SM::KS, VS = SM::VS;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  SM& sm = *reinterpret_cast<SM*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int q0 = blockIdx.x * (TC_QT * TC_BM);
  const int ntiles = (p.S + TC_BN - 1) / TC_BN;

  if (tid == 0) {
    tc::mbar_init(&sm.q_full, 1);
    for (int s = 0; s < KS; ++s) {
      tc::mbar_init(&sm.k_full[s], 1);
      tc::mbar_init(&sm.k_empty[s], TC_QT);
    }
    for (int s = 0; s < VS; ++s) {
      tc::mbar_init(&sm.v_full[s], 1);
      tc::mbar_init(&sm.v_empty[s], TC_QT);
    }
    for (int i = 0; i < TC_QT; ++i) {
      tc::mbar_init(&sm.s_full[i], 1);
      tc::mbar_init(&sm.s_free[i], 128);
      tc::mbar_init(&sm.p_full[i], 128);
      tc::mbar_init(&sm.pv_done[i], 1);
    }
    for (int i = 0; i < TC_QT; ++i) tc::mbar_init(&sm.o_done[i], 1);
    sm.abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 9) {
    tc::tmem_alloc(&sm.tmem_base, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tc::prefetch_tmap(&maps.q);
      tc::prefetch_tmap(&maps.k);
      tc::mbar_expect_tx(&sm.q_full, TC_QT * TT * TC_BM * TC_D);
      for (int qt = 0; qt < TC_QT; ++qt) {
        const int qrow = bh * p.S_pad + q0 + qt * TC_BM;
        tc::tma_load_2d(sm.q[qt][0], &maps.q, &sm.q_full, 0, qrow);
        if (TT == 2) tc::tma_load_2d(sm.q[qt][TT - 1], &maps.qr, &sm.q_full, 0, qrow);
      }
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % KS, use = j / KS;
        if (j >= KS && !tc::mbar_wait(&sm.k_empty[st], (use - 1) & 1)) { fail(sm, err, 11); break; }
        if (sm.abort_flag) break;
        tc::mbar_expect_tx(&sm.k_full[st], TC_BN * TC_D);
        tc::tma_load_2d(sm.k[st], &maps.k, &sm.k_full[st], 0, bh * p.S_pad + j * TC_BN);
      }
    }
  } else if (warp == 10) {
    // ------------------------------------------------------------ TMA producer of V^T
    if (lane == 0) {
      tc::prefetch_tmap(&maps.vt);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % VS, use = j / VS;
        if (j >= VS && !tc::mbar_wait(&sm.v_empty[st], (use - 1) & 1)) { fail(sm, err, 16); break; }
        if (sm.abort_flag) break;
        tc::mbar_expect_tx(&sm.v_full[st], TT * TC_BN * TC_D);
        tc::tma_load_2d(sm.v[st][0], &maps.vt, &sm.v_full[st], j * TC_BN, bh * TC_D);
        if (TT == 2) tc::tma_load_2d(sm.v[st][TT - 1], &maps.vtr, &sm.v_full[st], j * TC_BN, bh * TC_D);
      }
    }
  } else if (warp == 9 || warp == 11) {
    // ------------------------------------------------------------ MMA issuers
    // One thread per query tile, so each tile's QK -> softmax -> PV chain runs
    // independently; both feed the same tensor pipe.  A K (V) slot is free
    // once both issuers committed their QK (PV) products on it (count 2).
    if (lane == 0) {
      const int qt = warp == 9 ? 0 : 1;
      constexpr uint32_t IDESC = tc::idesc_e4m3_f32(TC_BM, TC_BN);
      const uint32_t tS = tmem + qt * 128, tO = tmem + 256 + qt * 128;
      bool ok = tc::mbar_wait(&sm.q_full, 0);
      if (!ok) fail(sm, err, 12);
      for (int j = 0; ok && j <= ntiles; ++j) {
        if (j < ntiles) {
          // S_t(j) = Q_t K_j^T once K_j landed and the softmax has read S_t(j-1)
          const int st = j % KS;
          if (!tc::mbar_wait(&sm.k_full[st], (j / KS) & 1)) { fail(sm, err, 14); ok = false; break; }
          if (j >= 1 && !tc::mbar_wait(&sm.s_free[qt], (j - 1) & 1)) { fail(sm, err, 15); ok = false; break; }
          if (sm.abort_flag) { ok = false; break; }
          tc::tc_fence_after();
          const uint64_t dk = tc::sdesc_sw128_kmajor(sm.k[st]);
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            const uint64_t dq = tc::sdesc_sw128_kmajor(sm.q[qt][t]);
#pragma unroll
            for (int ks = 0; ks < TC_D / 32; ++ks)
              tc::mma_f8f6f4(tS, dq + 2 * ks, dk + 2 * ks, IDESC, (t > 0 || ks > 0) ? 1u : 0u);
          }
          tc::tc_commit(&sm.s_full[qt]);
          tc::tc_commit(&sm.k_empty[st]);
          TRACE(qt, j);
        }
        if (j >= 1) {
          // O_t += P_t(j-1) V_{j-1}
          const int jj = j - 1, sv = jj % VS;
          if (!tc::mbar_wait(&sm.v_full[sv], (jj / VS) & 1)) { fail(sm, err, 17); ok = false; break; }
          if (!tc::mbar_wait(&sm.p_full[qt], jj & 1)) { fail(sm, err, 13); ok = false; break; }
          tc::tc_fence_after();
          const uint64_t dp = tc::sdesc_sw128_kmajor(sm.p[qt]);
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            const uint64_t dv = tc::sdesc_sw128_kmajor(sm.v[sv][t]);
#pragma unroll
            for (int ks = 0; ks < TC_BN / 32; ++ks)
              tc::mma_f8f6f4(tO, dp + 2 * ks, dv + 2 * ks, IDESC, (jj > 0 || t > 0 || ks > 0) ? 1u : 0u);
          }
          tc::tc_commit(&sm.pv_done[qt]);
          tc::tc_commit(&sm.v_empty[sv]);
          TRACE(2 + qt, jj);
        }
      }
      tc::tc_commit(&sm.o_done[qt]);
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 0..7)
    const int qt = warp >> 2;                        // query tile of this warpgroup
    const int r = tid & 127;                         // row in the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + qt * 128 + lane_off, tO = tmem + 256 + qt * 128 + lane_off;
    const float sq = scale_of(p.amax[(0 * p.B + b) * p.H + h]);
    const float sk = scale_of(p.amax[(1 * p.B + b) * p.H + h]);
    const float sv = scale_of(p.amax[(2 * p.B + b) * p.H + h]);
    const float sl2 = sq * sk * p.softmax_scale * 1.4426950408889634f;   // raw score -> log2 units
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    uint8_t* prow = sm.p[qt] + (r >> 3) * 1024 + (r & 7) * 128;
    for (int j = 0; j < ntiles; ++j) {
      if (r == 0) TRACE(4 + qt * 5, j);
      if (!tc::mbar_wait(&sm.s_full[qt], j & 1)) { fail(sm, err, 21); ok = false; }
      if (r == 0) TRACE(5 + qt * 5, j);
      if (__any_sync(0xffffffffu, !ok || sm.abort_flag)) { ok = false; break; }
      tc::tc_fence_after();
      uint32_t s[TC_BN];
#pragma unroll
      for (int c = 0; c < TC_BN / 32; ++c) tc::tmem_ld32(tS + c * 32, s + c * 32);
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      tc::mbar_arrive(&sm.s_free[qt]);
      const int kvalid = p.S - j * TC_BN;
      if (kvalid < TC_BN) {
#pragma unroll
        for (int c = 0; c < TC_BN; ++c)
          if (c >= kvalid) s[c] = __float_as_uint(-INFINITY);
      }
      float mx[8];
#pragma unroll
      for (int z = 0; z < 8; ++z) mx[z] = __uint_as_float(s[z]);
#pragma unroll
      for (int c = 8; c < TC_BN; c += 16)
#pragma unroll
        for (int z = 0; z < 8; ++z)
          mx[z] = fmax3(mx[z], __uint_as_float(s[c + z]), c + 8 + z < TC_BN ? __uint_as_float(s[c + 8 + z]) : mx[z]);
      const float mraw = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7]));
      const float m_new = fmaxf(m_ref, mraw * sl2);
      const bool rescale = __any_sync(0xffffffffu, m_new > m_ref + TC_TAU);
      float alpha = 1.f;
      if (rescale) {
        alpha = ex2(m_ref - m_new);                  // 0 on the first tile
        m_ref = m_new;
      }
      // exponentials: per 8 scores, 4 on the MUFU unit and 4 as a polynomial on
      // the FMA pipe (the e4m3 conversions also occupy the MUFU-side pipe, so
      // an even split balances the two); scaling and row sums as f32x2
      const float bias = TC_SHIFT - m_ref;
      const float2 sl2v = make_float2(sl2, sl2), biasv = make_float2(bias, bias);
      float2 ls0 = make_float2(0.f, 0.f), ls1 = make_float2(0.f, 0.f);
      uint32_t pk[TC_BN / 4];
#pragma unroll
      for (int c = 0; c < TC_BN; c += 8) {
        float2 x[4];
#pragma unroll
        for (int z = 0; z < 4; ++z)
          x[z] = ffma2(make_float2(__uint_as_float(s[c + 2 * z]), __uint_as_float(s[c + 2 * z + 1])), sl2v, biasv);
        float2 e[4];
        e[0] = make_float2(ex2(x[0].x), ex2(x[0].y));
        e[1] = exp2_poly2(x[1]);
        e[2] = make_float2(ex2(x[2].x), ex2(x[2].y));
        e[3] = exp2_poly2(x[3]);
        ls0 = fadd2(ls0, fadd2(e[0], e[1]));
        ls1 = fadd2(ls1, fadd2(e[2], e[3]));
        pk[c / 4] = f2_to_e4m3x2(e[0].x, e[0].y) | (f2_to_e4m3x2(e[1].x, e[1].y) << 16);
        pk[c / 4 + 1] = f2_to_e4m3x2(e[2].x, e[2].y) | (f2_to_e4m3x2(e[3].x, e[3].y) << 16);
      }
      if (r == 0) TRACE(6 + qt * 5, j);
      const float2 lsum = fadd2(ls0, ls1);
      l = l * alpha + (lsum.x + lsum.y);
      // PV(j-1) has finished reading the P buffer and adding into O
      if (j >= 1) {
        if (!tc::mbar_wait(&sm.pv_done[qt], (j - 1) & 1)) { fail(sm, err, 22); ok = false; }
        if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
        tc::tc_fence_after();
        if (rescale) {
#pragma unroll
          for (int c = 0; c < TC_D / 32; ++c) {
            uint32_t o[32];
            tc::tmem_ld32(tO + c * 32, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tc::tmem_st32(tO + c * 32, o);
          }
          tc::tmem_wait_st();
        }
      }
#pragma unroll
      for (int c16 = 0; c16 < TC_BN / 16; ++c16)
        *reinterpret_cast<uint4*>(prow + ((c16 ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c16], pk[4 * c16 + 1], pk[4 * c16 + 2], pk[4 * c16 + 3]);
      if (r == 0) TRACE(7 + qt * 5, j);
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(&sm.p_full[qt]);
      if (r == 0) TRACE(8 + qt * 5, j);
    }
    // epilogue: O / l -> bf16 row
    if (ok && __all_sync(0xffffffffu, tc::mbar_wait(&sm.o_done[qt], 0))) {
      tc::tc_fence_after();
      const float f = sv / l;
      const int row = q0 + qt * TC_BM + r;
      __nv_bfloat16* orow = p.o + ((size_t)b * p.S + row) * ((size_t)p.H * TC_D) + (size_t)h * TC_D;
#pragma unroll
      for (int c = 0; c < TC_D / 32; ++c) {
        uint32_t o[32];
        tc::tmem_ld32(tO + c * 32, o);
        tc::tmem_wait_ld();
        if (row < p.S) {
#pragma unroll
          for (int z = 0; z < 32; z += 8) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(o[z + 0]) * f, __uint_as_float(o[z + 1]) * f);
            v.y = pack_bf16(__uint_as_float(o[z + 2]) * f, __uint_as_float(o[z + 3]) * f);
            v.z = pack_bf16(__uint_as_float(o[z + 4]) * f, __uint_as_float(o[z + 5]) * f);
            v.w = pack_bf16(__uint_as_float(o[z + 6]) * f, __uint_as_float(o[z + 7]) * f);
            *reinterpret_cast<uint4*>(orow + c * 32 + z) = v;
          }
        }
      }
    } else if (ok) {
      fail(sm, err, 24);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// 2-D uint8 map over [rows, cols] (row stride `ld` bytes), 128 x 128 boxes, 128-byte swizzle.
static int make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(KB200_ERR_LAUNCH, "attn_fp8_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KB200_ERR_LAUNCH, "attn_fp8_tc: tensor map encode failed (%d)", (int)r);
  return KB200_OK;
}

int launch_attn_tc(const Params& p, int* err, cudaStream_t st) {
  TcMaps maps;
  const uint64_t rows_q = (uint64_t)p.B * p.H * p.S_pad, rows_v = (uint64_t)p.B * p.H * TC_D;
  if (int e = make_map(&maps.q, p.q8, TC_D, rows_q, TC_D)) return e;
  if (int e = make_map(&maps.k, p.k8, TC_D, rows_q, TC_D)) return e;
  if (int e = make_map(&maps.vt, p.vt8, p.S_pad, rows_v, p.S_pad)) return e;
  if (p.two_term) {
    if (int e = make_map(&maps.qr, p.q8r, TC_D, rows_q, TC_D)) return e;
    if (int e = make_map(&maps.vtr, p.vt8r, p.S_pad, rows_v, p.S_pad)) return e;
  } else {
    maps.qr = maps.q;
    maps.vtr = maps.vt;
  }
  if (p.S_pad % (TC_QT * TC_BM)) return set_error(KB200_ERR_INVALID, "attn_fp8_tc: S_pad must be a multiple of 256");
  const size_t smem = (p.two_term ? sizeof(TcSmem<2>) : sizeof(TcSmem<1>)) + 1024;
  auto kern = p.two_term ? attn_fp8_tc_kernel<2> : attn_fp8_tc_kernel<1>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<dim3(p.S_pad / (TC_QT * TC_BM), (unsigned)(p.B * p.H)), 384, smem, st>>>(maps, p, err);
  return check_launch("attn_fp8_tc_kernel");
}

}  // namespace attn
}  // namespace kb
