// attn_fp8_tc.cu -- softmax attention forward on 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a: e4m3 Q K^T, bf16 P V, fp32 accumulation.
//
// One CTA per (two 128-query tiles, batch*head); keys in tiles of BN = 128.
//   warp 16    : TMA producer (Q once; K and V^T per key tile, each into its own ring)
//   warp 17    : MMA issuer (one elected thread, both query tiles) + TMEM owner
//                S   = Q_t K_j^T  -> TMEM S    (kind::f8f6f4, e4m3, M128 N128 K32)
//                O_t += P_t V_j   -> TMEM O[t] (kind::f16, bf16; A = P_t read from
//                                               TMEM, B = V^T from shared memory)
//   warps 0..15: softmax, four warpgroups (query tile t, key half): each thread
//                owns the 64 scores of one row in its key half (TMEM lane).
//
// TMEM (512 columns): O_0 | O_1 | S | P_0 P_1.  The two query tiles share ONE score
// buffer S: the softmax of tile t loads its 64 scores per row into registers and
// releases S at once, so the product of the other tile (or of the next key tile)
// is computed while the exponentials of this one run; the probabilities go to the
// tile's own P columns (bf16 pairs).  The issuer's order per key tile j is
//   QK_1(j) [S released by tile 0]  PV_1(j-1) [P_1 published]
//   QK_0(j+1) [S released by tile 1]  PV_0(j) [P_0 published]
// (tcgen05.mma operations of one thread execute in issue order), so the score
// buffer alternates between the tiles and each tile's exponentials overlap the
// other tile's products on the tensor pipe.  The softmax of tile t writes P_t(j)
// only after PV_t(j-1) has completed (it has read P_t(j-1) and added into O_t).
//
// Every mbarrier wait is bounded; a wait that gives up records an error code in
// the workspace and the CTA skips the rest of its work.  Before it exits, the
// producer waits (bounded) for the last TMA load of every ring slot and the MMA
// issuer for all of its MMAs (one final commit); only then is TMEM freed.  If
// one of those drain waits gives up too, TMEM is left allocated rather than
// freed under a running MMA.
#include "attn_common.cuh"
#include "kb200_internal.h"
#include "tc_common.cuh"

namespace kb {
namespace attn {

constexpr int TC_BM = 128, TC_BN = 128, TC_D = 128;
constexpr int TC_QT = 2;          // query tiles per CTA
constexpr float TC_SHIFT = 6.f;   // P = 2^(s - m + SHIFT)
// Lazy-rescale threshold (log2 units): O and l are rescaled only when the
// running max grows by more than TAU, so P <= 2^(SHIFT+TAU) = 2^46 and a row sum
// over 2^15 keys stays below 2^61 -- far inside bf16's (fp32's) exponent range.  A
// wide threshold keeps the norm bound below it for ordinary data (N(0,1) q and k
// give bounds ~15 log2 units above the first tile's max), so the exact row max is
// rarely needed.
constexpr float TC_TAU = 40.f;
// Whether the two query tiles' softmax groups take turns with their exponentials.
#ifndef KB_ATTN_TURNS
#define KB_ATTN_TURNS 0
#endif
// Which score pairs of every 8 take the FMA-pipe polynomial instead of MUFU ex2 (none
// by default: with the shared score buffer the MUFU-only exponentials measured fastest,
// 7.6 ms against 7.8 ms with one pair in four on the polynomial).
#ifndef KB_ATTN_POLY_MASK
#define KB_ATTN_POLY_MASK 0x0
#endif
constexpr int TC_POLY_MASK = KB_ATTN_POLY_MASK;
// TMEM columns: O_t [128 t, 128 t + 128), S [256, 384), P_t [384 + 64 t, 384 + 64 t + 64).
constexpr uint32_t TM_O = 0, TM_S = 256, TM_P = 384;

struct TcSmem {
  static constexpr int KS = 4, VS = 3;
  uint8_t q[TC_QT][TC_BM * TC_D];               // e4m3 q               SW128 K-major, 128 rows
  uint8_t k[KS][TC_BN * TC_D];                  // e4m3 k tiles         SW128 K-major, 128 rows
  __nv_bfloat16 v[VS][2][TC_D * 64];            // bf16 v^T tiles: 2 atoms of 64 keys x 128 rows
  uint64_t q_full;
  uint64_t k_full[KS], k_empty[KS], v_full[VS], v_empty[VS];
  uint64_t s_full[TC_QT];    // S holds tile t's scores of the next key tile (MMA commit)
  uint64_t s_free[TC_QT];    // tile t's softmax has loaded S (one arrival per warp)
  uint64_t p_full[TC_QT];    // tile t's P (and any O rescale) is in TMEM (one arrival per warp)
  uint64_t pv_done[TC_QT];   // PV_t of a key tile has completed (MMA commit)
  uint64_t turn[TC_QT];      // optional: the other tile finished its exponentials
  uint64_t o_done[TC_QT];
  uint64_t xbar[TC_QT][4];                      // per (tile, lane quarter): the two key halves of a row exchange a value
  float xch[TC_QT][2][2][TC_BM];                // [tile][use parity][half][row]
  uint64_t drain[TC_QT];
  uint32_t tmem_base;
  int abort_flag;
  int keep_tmem;
};

struct TcMaps {
  CUtensorMap q, k, vt;
};

#ifdef KB_ATTN_TRACE
__device__ long long* g_attn_trace;
// the trace pointer is read once per thread (trp); a probe is one clock read and one store
#define ATRACE(j, slot) do { if (trp && (threadIdx.x & 31) == 0 && (j) < 128) trp[(j) * 32 + (slot)] = clock64(); } while (0)
#else
#define ATRACE(j, slot) do { } while (0)
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

// One arrival per warp: every lane's earlier tcgen05 loads/stores are ordered before
// the arrival (fence, then warp barrier, then lane 0 arrives).
KB_DEVI void warp_arrive_tc(uint64_t* bar, int lane) {
  tc::tc_fence_before();
  __syncwarp();
  if (lane == 0) tc::mbar_arrive(bar);
}

// Block: warps 0-15 softmax (warp w: TMEM lane quarter w & 3, query tile (w >> 2) & 1,
// key half w >> 3), warp 16 TMA producer, warp 17 MMA issuer + TMEM owner.
constexpr int TC_THREADS = 576;
__global__ void __launch_bounds__(TC_THREADS, 1) attn_fp8_tc_kernel(const __grid_constant__ TcMaps maps, Params p,
                                                             int* err) {
  using SM = TcSmem;
  constexpr int KS = SM::KS, VS = SM::VS;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-align by pointer arithmetic on the shared array (keeps shared addressing)
  SM& sm = *reinterpret_cast<SM*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int q0 = blockIdx.x * (TC_QT * TC_BM);
  // key tiles this CTA visits: all of them, or those a sliding window (flash-attention's
  // window_size = (left, right): query i sees keys i - left .. i + right) reaches from
  // its 256 queries.  Loop indices below count from j_lo.
  int j_lo = 0, j_hi = (p.S + TC_BN - 1) / TC_BN;
  if (p.win_left >= 0) j_lo = max(0, q0 - p.win_left) / TC_BN;
  if (p.win_right >= 0) j_hi = min(j_hi, (q0 + TC_QT * TC_BM - 1 + p.win_right) / TC_BN + 1);
  const int ntiles = j_hi - j_lo;

  if (tid == 0) {
    tc::mbar_init(&sm.q_full, 1);
    for (int s = 0; s < KS; ++s) {
      tc::mbar_init(&sm.k_full[s], 1);
      tc::mbar_init(&sm.k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      tc::mbar_init(&sm.v_full[s], 1);
      tc::mbar_init(&sm.v_empty[s], 1);
    }
    for (int i = 0; i < TC_QT; ++i) {
      tc::mbar_init(&sm.s_full[i], 1);
      tc::mbar_init(&sm.s_free[i], 8);
      tc::mbar_init(&sm.p_full[i], 8);
      tc::mbar_init(&sm.pv_done[i], 1);
      tc::mbar_init(&sm.turn[i], 8);
      for (int w = 0; w < 4; ++w) tc::mbar_init(&sm.xbar[i][w], 64);
    }
    for (int i = 0; i < TC_QT; ++i) {
      tc::mbar_init(&sm.o_done[i], 1);
      tc::mbar_init(&sm.drain[i], 1);
    }
    sm.abort_flag = 0;
    sm.keep_tmem = 0;
    tc::fence_barrier_init();
  }
  if (warp == 17) {
    tc::tmem_alloc(&sm.tmem_base, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  auto aborted = [&]() { return *((volatile int*)&sm.abort_flag) != 0; };
#ifdef KB_ATTN_TRACE
  long long* const trp = (blockIdx.x == 3 && blockIdx.y == 5) ? g_attn_trace : nullptr;
#endif

  if (warp == 16) {
    // ------------------------------------------------------------ TMA producer
    // K(j) and V^T(j) in key-tile order; each ring slot is reused once the issuer's
    // commit says every MMA reading it has completed.
    if (lane == 0) {
      tc::prefetch_tmap(&maps.q);
      tc::prefetch_tmap(&maps.k);
      tc::prefetch_tmap(&maps.vt);
      tc::mbar_expect_tx(&sm.q_full, TC_QT * TC_BM * TC_D);
      for (int qt = 0; qt < TC_QT; ++qt)
        tc::tma_load_2d(sm.q[qt], &maps.q, &sm.q_full, 0, bh * p.S_pad + q0 + qt * TC_BM);
      int kiss = 0, viss = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % KS, sv = j % VS;
        if (j >= KS && !tc::mbar_wait(&sm.k_empty[st], (j / KS - 1) & 1)) { fail(sm, err, 11); break; }
        if (aborted()) break;
        tc::mbar_expect_tx(&sm.k_full[st], TC_BN * TC_D);
        tc::tma_load_2d(sm.k[st], &maps.k, &sm.k_full[st], 0, bh * p.S_pad + (j_lo + j) * TC_BN);
        ++kiss;
        if (j >= VS && !tc::mbar_wait(&sm.v_empty[sv], (j / VS - 1) & 1)) { fail(sm, err, 16); break; }
        if (aborted()) break;
        tc::mbar_expect_tx(&sm.v_full[sv], 2 * TC_BN * TC_D);
        tc::tma_load_2d(sm.v[sv][0], &maps.vt, &sm.v_full[sv], (j_lo + j) * TC_BN, bh * TC_D);
        tc::tma_load_2d(sm.v[sv][1], &maps.vt, &sm.v_full[sv], (j_lo + j) * TC_BN + 64, bh * TC_D);
        ++viss;
      }
      // before the CTA may exit, every load it issued must have landed
      bool drained = tc::mbar_wait(&sm.q_full, 0);
      for (int j = kiss > KS ? kiss - KS : 0; j < kiss; ++j)
        drained &= tc::mbar_wait(&sm.k_full[j % KS], (j / KS) & 1);
      for (int j = viss > VS ? viss - VS : 0; j < viss; ++j)
        drained &= tc::mbar_wait(&sm.v_full[j % VS], (j / VS) & 1);
      if (!drained) { fail(sm, err, 18); sm.keep_tmem = 1; }
    }
  } else if (warp == 17) {
    // ------------------------------------------------------------ MMA issuer
    // One issuer for both tiles, in the order QK_1(j), PV_1(j-1), QK_0(j+1), PV_0(j).
    // The whole warp runs the schedule (waits, operand arithmetic) so every MMA operand
    // is warp-uniform and stays in uniform registers; one elected lane issues each
    // group of MMAs and its commits.
    const bool leader = tc::elect_one();
    constexpr uint32_t IDESC_QK = tc::idesc_e4m3_f32(TC_BM, TC_BN);
    constexpr uint32_t IDESC_PV = tc::idesc_bf16_f32(TC_BM, TC_D);
    const uint32_t tmem_u = __shfl_sync(0xffffffffu, tmem, 0);
    const uint32_t tS = tmem_u + TM_S;
    // descriptors of ring slot 0; slot s adds its byte offset >> 4
    const uint64_t dq0 = tc::sdesc_sw128_kmajor(sm.q[0]);
    const uint64_t dk0 = tc::sdesc_sw128_kmajor(sm.k[0]);
    const uint64_t dv0 = tc::sdesc_sw128_kmajor(sm.v[0][0]);
    auto commit = [&](uint64_t* bar) {
      if (leader) tc::tc_commit(bar);
      __syncwarp();
    };
    auto qk = [&](int t, int j) {   // S = Q_t K_j^T
      const uint64_t dq = dq0 + (uint64_t)(t * (TC_BM * TC_D / 16));
      const uint64_t dk = dk0 + (uint64_t)((j % KS) * (TC_BN * TC_D / 16));
      if (leader) {
#pragma unroll
        for (int ks = 0; ks < TC_D / 32; ++ks)
          tc::mma_f8f6f4(tS, dq + 2 * ks, dk + 2 * ks, IDESC_QK, ks > 0 ? 1u : 0u);
        tc::tc_commit(&sm.s_full[t]);
      }
      __syncwarp();
    };
    auto pv = [&](int t, int j) {   // O_t += P_t V_j: K = 16 keys per instruction (8 P columns)
      const uint32_t tO = tmem_u + TM_O + t * TC_D, tP = tmem_u + TM_P + t * 64;
      const uint64_t dv = dv0 + (uint64_t)((j % VS) * (2 * TC_D * 64 * 2 / 16));
      if (leader) {
#pragma unroll
        for (int ks = 0; ks < TC_BN / 16; ++ks)
          tc::mma_bf16_ts(tO, tP + ks * 8, dv + (ks >> 2) * (TC_D * 64 * 2 / 16) + 2 * (ks & 3), IDESC_PV,
                          (j > 0 || ks > 0) ? 1u : 0u);
        tc::tc_commit(&sm.pv_done[t]);
      }
      __syncwarp();
    };
    // A probe of an mbarrier phase is issued before the current group of MMAs (its
    // latency overlaps the issue); finish() only polls if that probe said no.
    auto probe = [&](uint64_t* bar, uint32_t parity) { return tc::mbar_test_wait(bar, parity); };
    auto finish = [&](uint64_t* bar, uint32_t parity, bool pre, int code) {
      const bool w = __all_sync(0xffffffffu, pre || tc::mbar_test_wait_loop(bar, parity));
      if (!w) fail(sm, err, code);
      return w;
    };
    bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&sm.q_full, 0) && tc::mbar_wait(&sm.k_full[0], 0));
    if (!ok) fail(sm, err, 12);
    if (ok) {
      tc::tc_fence_after();
      qk(0, 0);
      ATRACE(0, 0);
    }
    bool pre_s0 = probe(&sm.s_free[0], 0);
    for (int j = 0; ok && j < ntiles; ++j) {
      const bool last = j + 1 == ntiles;
      const int kn = (j + 1) % KS, vn = j % VS;
      // QK_1(j): S is free once tile 0 has loaded its scores of key tile j
      if (!finish(&sm.s_free[0], j & 1, pre_s0, 13) || aborted()) { ok = false; break; }
      tc::tc_fence_after();
      const bool pre_p1 = j >= 1 ? probe(&sm.p_full[1], (j - 1) & 1) : true;
      qk(1, j);
      commit(&sm.k_empty[j % KS]);   // both tiles' products with K_j issued
      ATRACE(j, 1);
      // PV_1(j-1)
      bool pre_s1 = false, pre_k = true;
      if (j >= 1) {
        if (!finish(&sm.p_full[1], (j - 1) & 1, pre_p1, 14)) { ok = false; break; }
        tc::tc_fence_after();
        pre_s1 = probe(&sm.s_free[1], j & 1);
        if (!last) pre_k = probe(&sm.k_full[kn], ((j + 1) / KS) & 1);
        pv(1, j - 1);
        commit(&sm.v_empty[(j - 1) % VS]);   // both tiles' products with V_{j-1} issued
        ATRACE(j - 1, 3);
      } else if (!last) {
        pre_s1 = probe(&sm.s_free[1], j & 1);
        pre_k = probe(&sm.k_full[kn], ((j + 1) / KS) & 1);
      }
      // QK_0(j+1): S is free once tile 1 has loaded its scores of key tile j
      bool pre_p0, pre_v;
      if (!last) {
        if (!finish(&sm.k_full[kn], ((j + 1) / KS) & 1, pre_k, 15)) { ok = false; break; }
        if (!finish(&sm.s_free[1], j & 1, pre_s1, 13)) { ok = false; break; }
        tc::tc_fence_after();
        pre_p0 = probe(&sm.p_full[0], j & 1);
        pre_v = probe(&sm.v_full[vn], (j / VS) & 1);
        qk(0, j + 1);
        ATRACE(j + 1, 0);
      } else {
        pre_p0 = probe(&sm.p_full[0], j & 1);
        pre_v = probe(&sm.v_full[vn], (j / VS) & 1);
      }
      // PV_0(j)
      if (!finish(&sm.v_full[vn], (j / VS) & 1, pre_v, 17)) { ok = false; break; }
      if (!finish(&sm.p_full[0], j & 1, pre_p0, 14)) { ok = false; break; }
      tc::tc_fence_after();
      pre_s0 = last ? true : probe(&sm.s_free[0], (j + 1) & 1);
      pv(0, j);
      ATRACE(j, 2);
    }
    if (ok) {   // PV_1 of the last key tile
      const int j = ntiles - 1;
      if (finish(&sm.p_full[1], j & 1, false, 14)) {
        tc::tc_fence_after();
        pv(1, j);
        commit(&sm.v_empty[j % VS]);
        ATRACE(j, 3);
        commit(&sm.o_done[0]);
        commit(&sm.o_done[1]);
      }
    }
    // every MMA this warp issued must complete before TMEM is freed
    commit(&sm.drain[0]);
    if (!__all_sync(0xffffffffu, tc::mbar_wait(&sm.drain[0], 0))) {
      fail(sm, err, 20);
      sm.keep_tmem = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 0..15)
    const int qt = (warp >> 2) & 1;                  // query tile
    const int half = warp >> 3;                      // key half: columns [64 half, 64 half + 64) of S
    const int r = (warp & 3) * 32 + lane;            // row in the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + TM_S + half * 64 + lane_off, tO = tmem + TM_O + qt * TC_D + lane_off,
                   tP = tmem + TM_P + qt * 64 + half * 32 + lane_off;
    const float sq = scale_of(p.amax[(0 * p.B + b) * p.H + h]);
    const float sk = scale_of(p.amax[(1 * p.B + b) * p.H + h]);
    const float sl2 = sq * sk * p.softmax_scale * 1.4426950408889634f;   // raw score -> log2 units
    const float qb = 1.0625f * p.qn[(size_t)bh * p.S_pad + q0 + qt * TC_BM + r] + 0.012f;
    const float* knp = p.kn + (size_t)bh * (p.S_pad / 64);
    const int nk64 = p.S_pad / 64;
    const bool tr = r == 0 && half == 0;
    float m_ref = -INFINITY, l = 0.f;
    // key-norm bound of the coming 128-key tile
    float kn_next = fmaxf(knp[min(2 * j_lo, nk64 - 1)], knp[min(2 * j_lo + 1, nk64 - 1)]);
    const int row_i = q0 + qt * TC_BM + r;   // this row's query index
    int xuse = 0;
    bool ok = true;
    uint64_t* xb = &sm.xbar[qt][warp & 3];
    auto exchange = [&](float v) -> float {
      float* slot = sm.xch[qt][xuse & 1][0];
      slot[half * TC_BM + r] = v;
      tc::mbar_arrive(xb);
      if (!tc::mbar_wait(xb, xuse & 1)) { fail(sm, err, 26); ok = false; }
      const float o = slot[(half ^ 1) * TC_BM + r];
      ++xuse;
      return o;
    };
    for (int j = 0; j < ntiles; ++j) {
      const float kn_j = kn_next;
      const int jn = j_lo + min(j + 1, ntiles - 1);
      kn_next = fmaxf(knp[min(2 * jn, nk64 - 1)], knp[min(2 * jn + 1, nk64 - 1)]);
      if (!tc::mbar_wait(&sm.s_full[qt], j & 1)) { fail(sm, err, 21); ok = false; }
      if (tr) ATRACE(j, 8 + 4 * qt);
      if (__any_sync(0xffffffffu, !ok || aborted())) { ok = false; break; }
      tc::tc_fence_after();
      // the row's 64 scores of this key half into registers; then S is released
      uint32_t s[64];
      tc::tmem_ld32(tS, s);
      tc::tmem_ld32(tS + 32, s + 32);
      tc::tmem_wait_ld();
      warp_arrive_tc(&sm.s_free[qt], lane);
      if (tr) ATRACE(j, 9 + 4 * qt);
      // keys outside the sequence, or outside this row's window, score -inf
      const int kb = (j_lo + j) * TC_BN + half * 64;
      int c_lo = 0, c_hi = min(64, p.S - kb);
      if (p.win_left >= 0) c_lo = max(c_lo, row_i - p.win_left - kb);
      if (p.win_right >= 0) c_hi = min(c_hi, row_i + p.win_right - kb + 1);
      if (c_lo > 0 || c_hi < 64) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c < c_lo || c >= c_hi) s[c] = __float_as_uint(-INFINITY);
      }
      // Every score of this tile is at most |sl2| |q8_row| max|k8| (Cauchy-Schwarz on the
      // e4m3 vectors the MMA multiplies; the factors cover e4m3 rounding of the stored
      // unrounded norms and the fp32 accumulation).  While that bound stays within TAU
      // of the running max no rescale can be due and the row max is not needed.  Both
      // halves of a row evaluate the same bound, so they take the same branch.
      bool need_max = j == 0;
      if (!need_max) {
        const float kbd = 1.0625f * kn_j + 0.012f;
        need_max = __any_sync(0xffffffffu, fabsf(sl2) * qb * kbd * 1.001f > m_ref + TC_TAU);
      }
      float alpha = 1.f;
      if (need_max) {
        float mpart = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) mpart = fmaxf(mpart, __uint_as_float(s[c]));
        const float mraw = fmaxf(mpart, exchange(mpart));
        if (__any_sync(0xffffffffu, !ok)) break;
        const float m_new = fmaxf(m_ref, mraw * sl2);
        // the warp rescales together; a row that has seen no key yet (all of its scores
        // so far masked by a window) keeps m = -inf
        if (__any_sync(0xffffffffu, m_new > m_ref + TC_TAU) && m_new != -INFINITY) {
          alpha = ex2(m_ref - m_new);                // 0 on the row's first seen key tile
          m_ref = m_new;
          l *= alpha;
        }
      }
#if KB_ATTN_TURNS
      if (qt == 0 ? j >= 1 : true)
        if (!tc::mbar_wait(&sm.turn[qt], (qt == 0 ? j - 1 : j) & 1)) { fail(sm, err, 27); ok = false; }
#endif
      // exponentials: P packed as bf16 pairs (8 TMEM columns per 16 scores); scaling and
      // row sums as f32x2
      // (no score of this row seen yet: every score here is -inf, and so is x)
      const float bias = m_ref == -INFINITY ? 0.f : TC_SHIFT - m_ref;
      const float2 sl2v = make_float2(sl2, sl2), biasv = make_float2(bias, bias);
      float2 ls0 = make_float2(0.f, 0.f), ls1 = make_float2(0.f, 0.f);
      uint32_t pk[32];
#pragma unroll
      for (int z = 0; z < 32; ++z) {
        const float2 x = ffma2(make_float2(__uint_as_float(s[2 * z]), __uint_as_float(s[2 * z + 1])), sl2v, biasv);
        const float2 e = ((TC_POLY_MASK >> (z & 7)) & 1) ? exp2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
        if (z & 1) ls1 = fadd2(ls1, e); else ls0 = fadd2(ls0, e);
        pk[z] = pack_bf16(e.x, e.y);
      }
#if KB_ATTN_TURNS
      warp_arrive_tc(&sm.turn[qt ^ 1], lane);
#endif
      if (tr) ATRACE(j, 10 + 4 * qt);
      const float2 lsum = fadd2(ls0, ls1);
      l += lsum.x + lsum.y;
      // P_t(j) overwrites P_t(j-1) and O_t may be rescaled: PV_t(j-1) must have completed
      if (j >= 1 && !tc::mbar_wait(&sm.pv_done[qt], (j - 1) & 1)) { fail(sm, err, 22); ok = false; }
      if (__any_sync(0xffffffffu, !ok)) break;
      tc::tc_fence_after();
      tc::tmem_st16(tP, pk);
      tc::tmem_st16(tP + 16, pk + 16);
      // O_t *= alpha before PV_t(j) adds into it; each key half rescales 64 of its columns
      if (__any_sync(0xffffffffu, alpha != 1.f) && j >= 1) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tc::tmem_ld32(tO + half * 64 + c * 32, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tc::tmem_st32(tO + half * 64 + c * 32, o);
        }
      }
      tc::tmem_wait_st();
      warp_arrive_tc(&sm.p_full[qt], lane);
      if (tr) ATRACE(j, 11 + 4 * qt);
    }
    // epilogue: the row sum of both halves; each half writes 64 of the 128 output
    // columns once the last PV has completed
    if (ok) l += exchange(l);
    if (ok && __all_sync(0xffffffffu, tc::mbar_wait(&sm.o_done[qt], 0))) {
      tc::tc_fence_after();
      const float f = 1.f / l;
      const int row = q0 + qt * TC_BM + r;
      __nv_bfloat16* orow = p.o + ((size_t)b * p.S + row) * ((size_t)p.H * TC_D) + (size_t)h * TC_D;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;
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
  if (warp == 17 && !sm.keep_tmem) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// 2-D map over [rows, cols] elements of `esize` bytes (uint8 or bf16), row pitch `ld`
// bytes, boxes of 128 bytes x `box_rows` rows, 128-byte swizzle.
static int make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, int esize,
                    int box_rows) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn) return set_error(KB200_ERR_LAUNCH, "attn_fp8_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esize), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KB200_ERR_LAUNCH, "attn_fp8_tc: tensor map encode failed (%d)", (int)r);
  return KB200_OK;
}

#ifdef KB_ATTN_TRACE
extern "C" int kb200_attn_set_trace(long long* t) {
  return cudaMemcpyToSymbol(g_attn_trace, &t, sizeof(t)) == cudaSuccess ? 0 : 4;
}
#endif

int launch_attn_tc(const Params& p, int* err, cudaStream_t st) {
  TcMaps maps;
  const uint64_t rows_q = (uint64_t)p.B * p.H * p.S_pad, rows_v = (uint64_t)p.B * p.H * TC_D;
  if (p.S_pad % (TC_QT * TC_BM)) return set_error(KB200_ERR_INVALID, "attn_fp8_tc: S_pad must be a multiple of 256");
  if (int e = make_map(&maps.q, p.q8, TC_D, rows_q, TC_D, 1, TC_BM)) return e;
  if (int e = make_map(&maps.k, p.k8, TC_D, rows_q, TC_D, 1, TC_BN)) return e;
  if (int e = make_map(&maps.vt, p.vt, p.S_pad, rows_v, (uint64_t)p.S_pad * 2, 2, TC_D)) return e;   // boxes: 64 keys x 128 rows
  const size_t smem = sizeof(TcSmem) + 1024;
  cudaFuncSetAttribute(attn_fp8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  attn_fp8_tc_kernel<<<dim3(p.S_pad / (TC_QT * TC_BM), (unsigned)(p.B * p.H)), TC_THREADS, smem, st>>>(maps, p,
                                                                                                         err);
  return check_launch("attn_fp8_tc_kernel");
}

}  // namespace attn
}  // namespace kb
