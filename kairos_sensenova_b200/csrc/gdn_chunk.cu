// gdn_chunk.cu -- chunked gated delta rule forward for sm_100a.
//
// Three launches per call (chunk size BT = 64):
//   1. gdn_prepare_kernel  (parallel over chunks x heads)
//        optional L2-norm of q,k  (fla/modules/l2norm.py:98-130)
//        in-chunk gate cumsum      (fla/ops/utils/cumsum.py:27-65)
//        A = beta e^{g_i-g_j} K K^T, strictly lower  (fla/ops/common/chunk_scaled_dot_kkt.py:28-73)
//        Ai = (I + A)^-1           (fla/ops/utils/solve_tril.py:184-331)
//        u = Ai (beta v), w = Ai (beta e^g k)   (fla/ops/gated_delta_rule/wy_fast.py:27-81)
//   2. gdn_state_kernel    (sequential over chunks; parallel over heads x V-slices)
//        h snapshot, v_new = u - w h, gate, h <- e^{g_last} h + k^T v_new
//        (fla/ops/common/chunk_delta_h.py:52-224)
//   3. gdn_output_kernel   (parallel over chunks x heads x V-slices)
//        o = scale (e^g (q h) + tril(q k^T e^{g_i-g_j}) v_new)   (fla/ops/common/chunk_o.py:41-128)
//
// Numerics follow the reference's bf16 rounding points: normalised q/k, Ai,
// w, u, h snapshots and v_new are bf16; A, the cumsum, the state and all
// accumulations are fp32.  Tensor-core work uses mma.sync m16n8k16 bf16.
#include "common.cuh"
#include "kb200_internal.h"
#include "tc_common.cuh"
#include "gdn_tc.cuh"
#include <type_traits>
#include <cstring>
#include <algorithm>

namespace kb {
namespace gdn {

constexpr int BT = 64;
constexpr int NTHREADS = 128;

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* g;
  const __nv_bfloat16* beta;
  const float* h0;
  __nv_bfloat16* o;
  float* ht;
  const int32_t* cu_seqlens;
  const int32_t* chunk_indices;
  const int32_t* chunk_offsets;
  // workspace
  __nv_bfloat16* qn;  // normalised q (or == q)
  __nv_bfloat16* kn;  // normalised k (or == k)
  float* gc;          // in-chunk cumsum of g
  __nv_bfloat16* w;
  __nv_bfloat16* u;
  __nv_bfloat16* vnew;
  __nv_bfloat16* hs;  // [num_chunks, H, K, V] state snapshots
  int T, H, NT;       // NT = chunks per sequence when cu_seqlens == nullptr
  float scale;
  int l2norm;
  // Segmented state pass (fixed-length sequences only): each sequence's chunks are
  // split into nseg segments of seg_chunks.  seg_mode 1 runs every segment but the
  // last from a zero state (seg_b: its end state) and, in the extra CTAs of grid.x,
  // from identity columns with u = 0 (seg_m: the segment's transition, stored
  // transposed); seg_mode 2 runs every segment from its start state (seg_h, written
  // by the combine kernel) and writes the snapshots, v_new and the final state.
  int seg_mode, nseg, seg_chunks;
  int* err;           // device error word: the site code of the first wait that gave up (0 = none)
  float* seg_b;       // [N*H, nseg, K, V]
  float* seg_m;       // [N*H, nseg, K(col), K(row)]
  float* seg_h;       // [N*H, nseg, K, V]
};

// Warp-level 16x16 fp32 product: C = +-(A B [+ C]), row-major operands with
// leading dimensions; lane l computes row l/2, columns 8*(l&1)..+8.  C must not
// alias A or B.
KB_DEVI void warp_mm16(float* C, int ldc, const float* A, int lda, const float* B, int ldb, bool acc,
                       bool neg, int lane) {
  const int r = lane >> 1, c0 = (lane & 1) * 8;
  float o[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) o[q] = acc ? C[r * ldc + c0 + q] : 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float a = A[r * lda + k];
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = fmaf(a, B[k * ldb + c0 + q], o[q]);
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) C[r * ldc + c0 + q] = neg ? -o[q] : o[q];
}

// Locate chunk `c` (global index): sequence n, first token bos, in-sequence chunk it, length L.
struct ChunkLoc { int n, it, bos, len; };
KB_DEVI ChunkLoc locate_chunk(const Params& p, int c) {
  ChunkLoc r;
  if (p.cu_seqlens) {
    r.n = p.chunk_indices[2 * c];
    r.it = p.chunk_indices[2 * c + 1];
    if (r.n < 0) {   // unused row of a table sized for the chunk-count upper bound
      r.n = r.it = r.bos = r.len = 0;
      return r;
    }
    int s = p.cu_seqlens[r.n], e = p.cu_seqlens[r.n + 1];
    r.bos = s;
    r.len = min(BT, e - s - r.it * BT);
  } else {
    r.n = c / p.NT;
    r.it = c % p.NT;
    r.bos = r.n * p.T;
    r.len = min(BT, p.T - r.it * BT);
  }
  return r;
}

// ---------------------------------------------------------------------------
// Kernel 1: per-chunk preparation.
// ---------------------------------------------------------------------------
template <int K, int V>
struct PrepSmem {
  static constexpr int LDK = K + 8, LDV = V + 8, LDA = BT + 1, LDI = BT + 8;
  // The fp32 solve area (A, its inverse, merge temporaries) is first used to
  // stage the q rows, and after the solve holds the bf16 inverse.
  static constexpr int SOLVE_BYTES = (2 * BT * LDA + 4 * 256) * 4;
  static constexpr int SCRATCH = SOLVE_BYTES > BT * LDK * 2 ? SOLVE_BYTES : BT * LDK * 2;
  __nv_bfloat16 ks[BT * LDK];   // k (normalised) then reused for beta e^g k
  __nv_bfloat16 vb[BT * LDV];   // v, then beta v
  alignas(16) unsigned char scratch[SCRATCH];
  float gcs[BT];
  float bs[BT];
  __device__ float* af() { return reinterpret_cast<float*>(scratch); }                 // A, strictly lower
  __device__ float* xf() { return reinterpret_cast<float*>(scratch) + BT * LDA; }      // (I+A)^-1
  __device__ float* yf() { return reinterpret_cast<float*>(scratch) + 2 * BT * LDA; }  // merge temporaries
  __device__ __nv_bfloat16* qs() { return reinterpret_cast<__nv_bfloat16*>(scratch); } // staged q rows
  __device__ __nv_bfloat16* ai() { return reinterpret_cast<__nv_bfloat16*>(scratch); } // bf16 inverse
};

template <int K, int V>
__global__ void __launch_bounds__(NTHREADS) gdn_prepare_kernel(Params p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  using S = PrepSmem<K, V>;
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x, h = blockIdx.y, H = p.H;
  const ChunkLoc loc = locate_chunk(p, c);
  const int t0 = loc.bos + loc.it * BT, L = loc.len;
  if (L <= 0) return;

  // ---- stage the chunk: every k, q, v row with cp.async at once (one memory round trip) ----
  {
    constexpr int KV = K / 8, VV = V / 8;
    for (int idx = tid; idx < BT * KV; idx += NTHREADS) {
      const int r = idx / KV, cv = (idx % KV) * 8;
      const bool ok = r < L;
      const size_t off = ((size_t)(t0 + (ok ? r : 0)) * H + h) * K + cv;
      cp_async16(sm.ks + r * S::LDK + cv, p.k + off, ok);
      if (p.l2norm) cp_async16(sm.qs() + r * S::LDK + cv, p.q + off, ok);
    }
    for (int idx = tid; idx < BT * VV; idx += NTHREADS) {
      const int r = idx / VV, cv = (idx % VV) * 8;
      const bool ok = r < L;
      cp_async16(sm.vb + r * S::LDV + cv, p.v + ((size_t)(t0 + (ok ? r : 0)) * H + h) * V + cv, ok);
    }
    cp_async_commit();
  }
  // ---- gate cumsum (warp 0) and beta (warp 1) while the copies fly ----
  if (warp == 0) {
    const int i0 = 2 * lane, i1 = 2 * lane + 1;
    float g0 = (i0 < L) ? p.g[(size_t)(t0 + i0) * H + h] : 0.f;
    float g1 = (i1 < L) ? p.g[(size_t)(t0 + i1) * H + h] : 0.f;
    float pair = g0 + g1, incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float excl = incl - pair;
    const float c0 = excl + g0, c1 = excl + g0 + g1;
    sm.gcs[i0] = c0;
    sm.gcs[i1] = c1;
    if (i0 < L) p.gc[(size_t)(t0 + i0) * H + h] = c0;
    if (i1 < L) p.gc[(size_t)(t0 + i1) * H + h] = c1;
  } else if (warp == 1) {
    for (int i = lane; i < BT; i += 32)
      sm.bs[i] = (i < L) ? __bfloat162float(p.beta[(size_t)(t0 + i) * H + h]) : 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();
  // ---- optional L2 norm of q/k rows (l2norm.py:118-121: y = x / sqrt(sum x^2 + 1e-6),
  // stored in bf16); one warp per row, one 8/16-byte vector per lane ----
  if (p.l2norm) {
    constexpr int EPL = K / 32;  // elements per lane (4 or 8)
    using Vec = typename std::conditional<EPL == 4, uint2, uint4>::type;
    for (int r = warp; r < L; r += NTHREADS / 32) {
      Vec* kp = reinterpret_cast<Vec*>(sm.ks + r * S::LDK + lane * EPL);
      const Vec kr = *kp;
      const Vec qr = *reinterpret_cast<const Vec*>(sm.qs() + r * S::LDK + lane * EPL);
      const __nv_bfloat16* ke = reinterpret_cast<const __nv_bfloat16*>(&kr);
      const __nv_bfloat16* qe = reinterpret_cast<const __nv_bfloat16*>(&qr);
      float sk = 0.f, sq = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const float xk = __bfloat162float(ke[e]), xq = __bfloat162float(qe[e]);
        sk += xk * xk;
        sq += xq * xq;
      }
      sk = warp_sum(sk);
      sq = warp_sum(sq);
      const float rk = 1.0f / sqrtf(sk + 1e-6f), rq = 1.0f / sqrtf(sq + 1e-6f);
      Vec ko, qo;
      uint32_t* ko32 = reinterpret_cast<uint32_t*>(&ko);
      uint32_t* qo32 = reinterpret_cast<uint32_t*>(&qo);
#pragma unroll
      for (int e = 0; e < EPL; e += 2) {
        ko32[e / 2] = pack_bf16(__bfloat162float(ke[e]) * rk, __bfloat162float(ke[e + 1]) * rk);
        qo32[e / 2] = pack_bf16(__bfloat162float(qe[e]) * rq, __bfloat162float(qe[e + 1]) * rq);
      }
      *kp = ko;
      const size_t off = ((size_t)(t0 + r) * H + h) * K + lane * EPL;
      *reinterpret_cast<Vec*>(p.kn + off) = ko;
      *reinterpret_cast<Vec*>(p.qn + off) = qo;
    }
  }
  // ---- beta v in place (bf16(v * beta), wy_fast.py:67) ----
  {
    constexpr int VPR = V / 8;
    for (int idx = tid; idx < BT * VPR; idx += NTHREADS) {
      const int r = idx / VPR, cv = (idx % VPR) * 8;
      uint4* ptr = reinterpret_cast<uint4*>(sm.vb + r * S::LDV + cv);
      const uint4 raw = *ptr;
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
      const float b = sm.bs[r];
      uint4 outv;
      uint32_t* ov = reinterpret_cast<uint32_t*>(&outv);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        ov[j] = pack_bf16(__bfloat162float(e[2 * j]) * b, __bfloat162float(e[2 * j + 1]) * b);
      *ptr = outv;
    }
  }
  __syncthreads();
  // ---- A = beta_i e^{g_i - g_j} <k_i, k_j>, strictly lower (warp w: rows 16w..16w+15) ----
  {
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < K; kk += 16) {
      uint32_t a[4];
      load_a_rowmajor(a, sm.ks, S::LDK, warp * 16, kk, lane);
#pragma unroll
      for (int n0 = 0; n0 < BT; n0 += 16) {
        uint32_t b[4];
        load_b_nmajor_rows_x2n(b, sm.ks, S::LDK, kk, n0, lane);
        mma_bf16(acc[n0 / 8], a, b);
        mma_bf16(acc[n0 / 8 + 1], a, b + 2);
      }
    }
    const int g8 = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = warp * 16 + g8 + ((e >> 1) << 3);
        const int j = n * 8 + 2 * t4 + (e & 1);
        float val = 0.f;
        if (i > j && i < L) val = acc[n][e] * __expf(sm.gcs[i] - sm.gcs[j]) * sm.bs[i];
        sm.af()[i * S::LDA + j] = val;
      }
  }
  __syncthreads();
  // ---- k rows -> bf16(bf16(k * beta) * e^{g}) in place (wy_fast.py:77-79) ----
  {
    constexpr int VPR = K / 8;
    for (int idx = tid; idx < BT * VPR; idx += NTHREADS) {
      const int r = idx / VPR, cv = (idx % VPR) * 8;
      __nv_bfloat16* row = sm.ks + r * S::LDK + cv;
      uint4 raw = *reinterpret_cast<uint4*>(row);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
      const float b = sm.bs[r], eg = __expf(sm.gcs[r]);
      uint4 outv;
      uint32_t* ov = reinterpret_cast<uint32_t*>(&outv);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        ov[j] = pack_bf16(bf16_round(__bfloat162float(e[2 * j]) * b) * eg,
                          bf16_round(__bfloat162float(e[2 * j + 1]) * b) * eg);
      *reinterpret_cast<uint4*>(row) = outv;
    }
  }
  // ---- (I + A)^-1: 16x16 diagonal blocks by forward substitution ----
  if (tid < 64) {
    const int blk = tid >> 4, col = tid & 15, base = blk * 16;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) x[r] = (r == col) ? 1.f : 0.f;
#pragma unroll
    for (int r = 1; r < 16; ++r) {
      float s = 0.f;
#pragma unroll
      for (int m = 0; m < r; ++m) s += sm.af()[(base + r) * S::LDA + base + m] * x[m];
      if (r > col) x[r] = -s;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sm.xf()[(base + r) * S::LDA + base + col] = x[r];
  }
  // zero the strictly-upper blocks
  for (int idx = tid; idx < BT * BT; idx += NTHREADS) {
    const int r = idx >> 6, cc = idx & 63;
    if ((cc >> 4) > (r >> 4)) sm.xf()[r * S::LDA + cc] = 0.f;
  }
  __syncthreads();
  // ---- block merge (solve_tril.py:265-290, fp32 like its 'ieee' dots):
  //   X21 = -D2 A21 D1, X32 = -D3 A32 D2, X43 = -D4 A43 D3,
  //   X31 = -D3 (A31 D1 + A32 X21), X42 = -D4 (A42 D2 + A43 X32),
  //   X41 = -D4 (A41 D1 + A42 X21 + A43 X31)      (block indices 1-based)
  // as warp-level 16x16 fp32 products, three warps in parallel per level ----
  {
    auto Ab = [&](int i, int j) { return sm.af() + (16 * i) * S::LDA + 16 * j; };
    auto Xb = [&](int i, int j) { return sm.xf() + (16 * i) * S::LDA + 16 * j; };
    float* T = sm.yf() + warp * 256;
    if (warp < 3) {
      const int i = warp + 1;
      warp_mm16(T, 16, Ab(i, i - 1), S::LDA, Xb(i - 1, i - 1), S::LDA, false, false, lane);
      __syncwarp();
      warp_mm16(Xb(i, i - 1), S::LDA, Xb(i, i), S::LDA, T, 16, false, true, lane);
    }
    __syncthreads();
    if (warp == 0) {
      warp_mm16(T, 16, Ab(2, 0), S::LDA, Xb(0, 0), S::LDA, false, false, lane);
      __syncwarp();
      warp_mm16(T, 16, Ab(2, 1), S::LDA, Xb(1, 0), S::LDA, true, false, lane);
      __syncwarp();
      warp_mm16(Xb(2, 0), S::LDA, Xb(2, 2), S::LDA, T, 16, false, true, lane);
    } else if (warp == 1) {
      warp_mm16(T, 16, Ab(3, 1), S::LDA, Xb(1, 1), S::LDA, false, false, lane);
      __syncwarp();
      warp_mm16(T, 16, Ab(3, 2), S::LDA, Xb(2, 1), S::LDA, true, false, lane);
      __syncwarp();
      warp_mm16(Xb(3, 1), S::LDA, Xb(3, 3), S::LDA, T, 16, false, true, lane);
    } else if (warp == 2) {
      warp_mm16(T, 16, Ab(3, 0), S::LDA, Xb(0, 0), S::LDA, false, false, lane);
      __syncwarp();
      warp_mm16(T, 16, Ab(3, 1), S::LDA, Xb(1, 0), S::LDA, true, false, lane);
    }
    __syncthreads();
    if (warp == 0) {
      float* T2 = sm.yf() + 2 * 256;
      warp_mm16(T2, 16, Ab(3, 2), S::LDA, Xb(2, 0), S::LDA, true, false, lane);
      __syncwarp();
      warp_mm16(Xb(3, 0), S::LDA, Xb(3, 3), S::LDA, T2, 16, false, true, lane);
    }
    __syncthreads();
  }
  for (int idx = tid; idx < BT * BT; idx += NTHREADS) {
    const int r = idx >> 6, cc = idx & 63;
    sm.ai()[r * S::LDI + cc] = __float2bfloat16_rn(sm.xf()[r * S::LDA + cc]);
  }
  __syncthreads();
  // ---- u = Ai (beta v), w = Ai (beta e^g k), 64-column slabs ----
  {
    const int g8 = lane >> 2, t4 = lane & 3;
    uint32_t afr[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) load_a_rowmajor(afr[ks], sm.ai(), S::LDI, warp * 16, ks * 16, lane);
    const int r0 = warp * 16 + g8, r1 = r0 + 8;
    for (int slab = 0; slab < (V + K) / 64; ++slab) {
      const bool isu = slab < V / 64;
      const __nv_bfloat16* src = isu ? sm.vb : sm.ks;
      const int ld = isu ? S::LDV : S::LDK;
      const int c0 = (isu ? slab : slab - V / 64) * 64;
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int n0 = 0; n0 < 64; n0 += 16) {
          uint32_t b[4];
          load_b_kmajor_rows_x2n(b, src, ld, ks * 16, c0 + n0, lane);
          mma_bf16(acc[n0 / 8], afr[ks], b);
          mma_bf16(acc[n0 / 8 + 1], afr[ks], b + 2);
        }
      __nv_bfloat16* dst = isu ? p.u : p.w;
      const int D = isu ? V : K;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int col = c0 + n * 8 + 2 * t4;
        if (r0 < L)
          *reinterpret_cast<uint32_t*>(dst + ((size_t)(t0 + r0) * H + h) * D + col) =
              pack_bf16(acc[n][0], acc[n][1]);
        if (r1 < L)
          *reinterpret_cast<uint32_t*>(dst + ((size_t)(t0 + r1) * H + h) * D + col) =
              pack_bf16(acc[n][2], acc[n][3]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Kernel 2: sequential state pass.  Grid (V / BV, N * H); 8 warps.
//   v_new = u - w h   : warp w computes rows 16 (w & 3).., columns BV/2 (w >> 2)..
//   h <- e^{g_last} h + k^T vg : warp w owns state rows [w K/8, (w+1) K/8)
// The next chunk's w, k, u and g tiles stream in with cp.async while the
// current one is processed; the bf16 state snapshot and the gated v_new are
// double-buffered, so each step needs two block barriers.
// ---------------------------------------------------------------------------
constexpr int STATE_THREADS = 256;

#ifdef KB_GDN_TRACE
__device__ long long g_state_trace[1024 * 8];
#define STRACE(slot, it) do { if (blockIdx.x == 0 && blockIdx.y == 0 && tid == 0 && (it) < 1024) g_state_trace[(it) * 8 + (slot)] = clock64(); } while (0)
#else
#define STRACE(slot, it) do { } while (0)
#endif

template <int K, int BV>
struct StateSmem {
  static constexpr int LDV = BV + 8;
  // w and k tiles (BT tokens x K) as TMA writes them: K/64 atoms of BT rows x 128 B,
  // 128-byte swizzle; the struct is placed 1024-byte aligned
  __nv_bfloat16 ws[2][BT * K];
  __nv_bfloat16 ks[2][BT * K];
  __nv_bfloat16 us[2][BT * LDV];
  __nv_bfloat16 hb[2][K * LDV];   // bf16 snapshot of the state (B operand of w h)
  __nv_bfloat16 vg[2][BT * LDV];  // gated v_new (B operand of k^T v)
  __nv_bfloat16 vn[BT * LDV];     // v_new staged for coalesced 16-byte stores
  float gcs[2][BT];
  uint64_t full[2];               // the w and k tiles of buffer b landed (TMA)
};

// Element (r, c) (c a multiple of 8) of a BT-row tile stored as 64-column SW128 atoms.
KB_DEVI const __nv_bfloat16* sw128_at(const __nv_bfloat16* base, int r, int c) {
  return base + (c >> 6) * (BT * 64) + r * 64 + ((((c >> 3) & 7) ^ (r & 7)) << 3);
}
// load_a_rowmajor / load_a_transposed for such swizzled tiles
KB_DEVI void load_a_rowmajor_sw(uint32_t* a, const __nv_bfloat16* base, int r0, int c0, int lane) {
  ldsm_x4(a[0], a[1], a[2], a[3], sw128_at(base, r0 + (lane & 15), c0 + ((lane >> 4) << 3)));
}
KB_DEVI void load_a_transposed_sw(uint32_t* a, const __nv_bfloat16* base, int m0, int k0, int lane) {
  const int mat = lane >> 3, r = lane & 7;
  ldsm_x4_t(a[0], a[1], a[2], a[3], sw128_at(base, k0 + ((mat >> 1) << 3) + r, m0 + ((mat & 1) << 3)));
}

// TMA maps of the w and k tensors ([tokens, H, K] bf16) as 3-D (K, H, tokens),
// boxes of 64 channels x 1 head x BT tokens.
struct StateMaps {
  CUtensorMap w, k;
};

KB_DEVI void cp_async4(void* smem, const void* gmem, bool pred) {
  int n = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n));
}

// Per-thread copy plan, fixed for the whole pass: thread tid copies 16-byte
// vectors (row kr0 + i * KRS, column kc) of the w / k tiles, one vector (ur, uc)
// of the u tile and, for tid < 64, the gate value of row tid.
template <int K, int BV>
struct StateCopyPlan {
  static constexpr int VPR = K / 8, KRS = STATE_THREADS / VPR, KIT = BT / KRS;
  int kr0, kc, ur, uc;
  KB_DEVI StateCopyPlan(int tid) {
    kr0 = tid / VPR;
    kc = (tid % VPR) * 8;
    ur = tid / (BV / 8);
    uc = (tid % (BV / 8)) * 8;
  }
};

// Loads of one chunk into buffer `buf`: thread 0 issues the TMA boxes of the w
// and k tiles (counted on sm.full[buf]; rows past the chunk end carry the next
// sequence's rows or zero fill -- finite values that only ever meet zero gates);
// u rows and the strided gate values go through cp.async with zero fill.
template <int K, int BV>
KB_DEVI void state_issue_loads(StateSmem<K, BV>& sm, const StateMaps& maps, int buf, const Params& p,
                               const StateCopyPlan<K, BV>& cp, int t0, int L, int h, int v0, int V, int tid,
                               bool load_u) {
  using S = StateSmem<K, BV>;
  if (tid == 0) {
    // every ldmatrix read of this buffer completed before the block barrier that precedes this call
    tc::mbar_expect_tx(&sm.full[buf], 2 * BT * K * 2);
#pragma unroll
    for (int a = 0; a < K / 64; ++a) {
      tc::tma_load_3d(sm.ws[buf] + a * BT * 64, &maps.w, &sm.full[buf], a * 64, h, t0);
      tc::tma_load_3d(sm.ks[buf] + a * BT * 64, &maps.k, &sm.full[buf], a * 64, h, t0);
    }
  }
  if (load_u && cp.ur < BT) {
    const bool ok = cp.ur < L;
    cp_async16(&sm.us[buf][cp.ur * S::LDV + cp.uc],
               p.u + ((size_t)(t0 + (ok ? cp.ur : 0)) * p.H + h) * V + v0 + cp.uc, ok);
  }
  if (tid < BT) cp_async4(&sm.gcs[buf][tid], p.gc + (size_t)(t0 + (tid < L ? tid : 0)) * p.H + h, tid < L);
  cp_async_commit();
}

template <int K, int V, int BV>
__global__ void __launch_bounds__(STATE_THREADS) gdn_state_kernel(Params p, const __grid_constant__ StateMaps maps) {
  static_assert(BV == 16 || BV == 32, "state kernel tiles assume BV = 16 or 32");
  static_assert(K % 64 == 0, "w/k tiles are 64-column swizzled atoms");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  using S = StateSmem<K, BV>;
  S& sm = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int nseg = p.seg_mode ? p.nseg : 1;
  const int nh = blockIdx.y / nseg, seg = blockIdx.y % nseg, n = nh / p.H, h = nh % p.H, H = p.H;
  // transition CTA of the segmented local pass: columns mcol0.. of the K x K transition
  const bool trans = p.seg_mode == 1 && (int)blockIdx.x >= V / BV;
  const int v0 = trans ? 0 : blockIdx.x * BV;
  const int mcol0 = trans ? ((int)blockIdx.x - V / BV) * BV : 0;
  // the local pass needs no end state of the last segment and no transition of the first
  if (p.seg_mode == 1 && (seg == nseg - 1 || (trans && seg == 0))) return;
  int bos, Tn, cbase;
  if (p.cu_seqlens) {
    bos = p.cu_seqlens[n];
    Tn = p.cu_seqlens[n + 1] - bos;
    cbase = p.chunk_offsets[n];
  } else {
    bos = n * p.T;
    Tn = p.T;
    cbase = n * p.NT;
  }
  const int NTn = (Tn + BT - 1) / BT;
  const int it0 = p.seg_mode ? seg * p.seg_chunks : 0;
  const int it1 = p.seg_mode ? min(NTn, it0 + p.seg_chunks) : NTn;
  const bool seg_start0 = p.seg_mode != 0 && seg > 0;   // this run does not start at the sequence start
  constexpr int RW = K / 8;        // state rows per warp
  constexpr int MT = RW / 16;      // m-tiles per warp
  constexpr int NB = BV / 8;       // n-tiles of the state
  const int m0 = warp * RW;
  float hacc[MT][NB][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int nn = 0; nn < NB; ++nn)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = m0 + m * 16 + g8 + ((e >> 1) << 3);
        const int cc = v0 + nn * 8 + 2 * t4 + (e & 1);
        float init;
        if (trans)
          init = (r == mcol0 + nn * 8 + 2 * t4 + (e & 1)) ? 1.f : 0.f;
        else if (seg_start0)
          init = p.seg_mode == 2 ? p.seg_h[(((size_t)nh * nseg + seg) * K + r) * V + cc] : 0.f;
        else
          init = p.h0 ? p.h0[((size_t)nh * K + r) * V + cc] : 0.f;
        hacc[m][nn][e] = init;
      }
  const StateCopyPlan<K, BV> cplan(tid);
  if (tid == 0) {
    tc::mbar_init(&sm.full[0], 1);
    tc::mbar_init(&sm.full[1], 1);
    tc::fence_barrier_init();
  }
  if (trans)   // u = 0 for the transition: its tiles are never loaded
    for (int i = tid; i < 2 * BT * S::LDV; i += STATE_THREADS) (&sm.us[0][0])[i] = __float2bfloat16(0.f);
  __syncthreads();
  if (it1 > it0)
    state_issue_loads<K, BV>(sm, maps, 0, p, cplan, bos + it0 * BT, min(BT, Tn - it0 * BT), h, v0, V, tid,
                             !trans);
  const int rg = warp & 3, c0 = (warp >> 2) * (BV / 2);

  const bool write_seq = p.seg_mode != 1;   // snapshots and v_new are written by the final pass only
  for (int it = it0; it < it1; ++it) {
    const int li = it - it0, buf = li & 1;
    const int t0 = bos + it * BT, L = min(BT, Tn - it * BT);
    STRACE(0, it);
    // (a) snapshot: bf16 state -> smem operand and -> global h[chunk]
    __nv_bfloat16* hg = p.hs + ((size_t)(cbase + it) * H + h) * K * V;
    __nv_bfloat16* hb = sm.hb[buf];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int nn = 0; nn < NB; ++nn) {
        const int r = m0 + m * 16 + g8;
        const int cc = nn * 8 + 2 * t4;
        const uint32_t lo = pack_bf16(hacc[m][nn][0], hacc[m][nn][1]);
        const uint32_t hi = pack_bf16(hacc[m][nn][2], hacc[m][nn][3]);
        *reinterpret_cast<uint32_t*>(&hb[r * S::LDV + cc]) = lo;
        *reinterpret_cast<uint32_t*>(&hb[(r + 8) * S::LDV + cc]) = hi;
      }
    STRACE(1, it);
    cp_async_wait<0>();
    // bounded: on a timeout the pass records the error and stops here (outputs of
    // later chunks are left unwritten) instead of hanging the GPU.  The load it
    // waited for is the only one in flight (the next is issued after this wait):
    // wait for it once more, bounded, before the CTA may exit.
    if (!__syncthreads_and(tc::mbar_wait(&sm.full[buf], (li >> 1) & 1))) {
      if (tid == 0) {
        atomicCAS(p.err, 0, 31);
        tc::mbar_wait(&sm.full[buf], (li >> 1) & 1);
      }
      __syncthreads();
      return;
    }
    STRACE(2, it);
    STRACE(3, it);
    // snapshot -> global h[chunk] as coalesced 16-byte vectors
#pragma unroll
    for (int i = 0; i < (write_seq ? K * (BV / 8) / STATE_THREADS : 0); ++i) {
      const int idx = tid + i * STATE_THREADS, r = idx / (BV / 8), cv = (idx % (BV / 8)) * 8;
      *reinterpret_cast<uint4*>(hg + (size_t)r * V + v0 + cv) = *reinterpret_cast<const uint4*>(&hb[r * S::LDV + cv]);
    }
    STRACE(7, it);
    if (it + 1 < it1)
      state_issue_loads<K, BV>(sm, maps, buf ^ 1, p, cplan, t0 + BT, min(BT, Tn - (it + 1) * BT), h, v0, V, tid,
                               !trans);
    STRACE(4, it);
    // (b) v_new = u - w h   (rows 16 rg.., columns c0..c0+BV/2); two accumulator sets halve the chain
    const float glast = sm.gcs[buf][L - 1];
    __nv_bfloat16* vg = sm.vg[buf];
    {
      constexpr int NBW = BV / 16;   // n-tiles of 8 per warp
      float acc0[NBW][4], acc1[NBW][4];
#pragma unroll
      for (int nn = 0; nn < NBW; ++nn)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc0[nn][e] = acc1[nn][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < K; kk += 32) {
        uint32_t a0[4], a1[4], b0[2 * NBW], b1[2 * NBW];
        load_a_rowmajor_sw(a0, sm.ws[buf], rg * 16, kk, lane);
        load_a_rowmajor_sw(a1, sm.ws[buf], rg * 16, kk + 16, lane);
        if constexpr (NBW == 2) {
          load_b_kmajor_rows_x2n(b0, hb, S::LDV, kk, c0, lane);
          load_b_kmajor_rows_x2n(b1, hb, S::LDV, kk + 16, c0, lane);
        } else {
          load_b_kmajor_rows_x1n(b0, hb, S::LDV, kk, c0, lane);
          load_b_kmajor_rows_x1n(b1, hb, S::LDV, kk + 16, c0, lane);
        }
#pragma unroll
        for (int nn = 0; nn < NBW; ++nn) {
          mma_bf16(acc0[nn], a0, b0 + 2 * nn);
          mma_bf16(acc1[nn], a1, b1 + 2 * nn);
        }
      }
      const int r0 = rg * 16 + g8, r1 = r0 + 8;
      const float e0 = (r0 < L) ? __expf(glast - sm.gcs[buf][r0]) : 0.f;
      const float e1 = (r1 < L) ? __expf(glast - sm.gcs[buf][r1]) : 0.f;
#pragma unroll
      for (int nn = 0; nn < NBW; ++nn) {
        const int cc = c0 + nn * 8 + 2 * t4;
        const __nv_bfloat162 u0 = *reinterpret_cast<const __nv_bfloat162*>(&sm.us[buf][r0 * S::LDV + cc]);
        const __nv_bfloat162 u1 = *reinterpret_cast<const __nv_bfloat162*>(&sm.us[buf][r1 * S::LDV + cc]);
        const float a0 = __low2float(u0) - (acc0[nn][0] + acc1[nn][0]);
        const float a1 = __high2float(u0) - (acc0[nn][1] + acc1[nn][1]);
        const float a2 = __low2float(u1) - (acc0[nn][2] + acc1[nn][2]);
        const float a3 = __high2float(u1) - (acc0[nn][3] + acc1[nn][3]);
        *reinterpret_cast<uint32_t*>(&sm.vn[r0 * S::LDV + cc]) = pack_bf16(a0, a1);
        *reinterpret_cast<uint32_t*>(&sm.vn[r1 * S::LDV + cc]) = pack_bf16(a2, a3);
        *reinterpret_cast<uint32_t*>(&vg[r0 * S::LDV + cc]) = pack_bf16(a0 * e0, a1 * e0);
        *reinterpret_cast<uint32_t*>(&vg[r1 * S::LDV + cc]) = pack_bf16(a2 * e1, a3 * e1);
      }
    }
    STRACE(5, it);
    __syncthreads();
    STRACE(6, it);
    // v_new -> global as 16-byte vectors (rows < L)
    if (write_seq && cplan.ur < L)
      *reinterpret_cast<uint4*>(p.vnew + ((size_t)(t0 + cplan.ur) * H + h) * V + v0 + cplan.uc) =
          *reinterpret_cast<const uint4*>(&sm.vn[cplan.ur * S::LDV + cplan.uc]);
    // (c) h <- e^{g_last} h + k^T vg
    {
      const float dec = __expf(glast);
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int nn = 0; nn < NB; ++nn)
#pragma unroll
          for (int e = 0; e < 4; ++e) hacc[m][nn][e] *= dec;
#pragma unroll
      for (int kk = 0; kk < BT; kk += 16) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          uint32_t a[4];
          load_a_transposed_sw(a, sm.ks[buf], m0 + m * 16, kk, lane);
#pragma unroll
          for (int n0 = 0; n0 < BV; n0 += 16) {
            uint32_t b[4];
            load_b_kmajor_rows_x2n(b, vg, S::LDV, kk, n0, lane);
            mma_bf16(hacc[m][n0 / 8], a, b);
            mma_bf16(hacc[m][n0 / 8 + 1], a, b + 2);
          }
        }
      }
    }
  }
  float* dst = nullptr;
  if (p.seg_mode == 1)
    dst = trans ? p.seg_m + ((size_t)nh * nseg + seg) * K * K : p.seg_b + ((size_t)nh * nseg + seg) * K * V;
  else if (p.ht && (p.seg_mode == 0 || seg == nseg - 1))
    dst = p.ht + (size_t)nh * K * V;
  if (dst) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int nn = 0; nn < NB; ++nn)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = m0 + m * 16 + g8 + ((e >> 1) << 3);
          const int c = nn * 8 + 2 * t4 + (e & 1);
          if (trans)
            dst[(size_t)(mcol0 + c) * K + r] = hacc[m][nn][e];
          else
            dst[(size_t)r * V + v0 + c] = hacc[m][nn][e];
        }
  }
}

// ---------------------------------------------------------------------------
// Kernel 2b: segment combine.  Grid (V / 8, N * H); 256 threads.  Start states
// of the segments of one sequence, a short sequential scan in fp32:
//   h_1 = B_0,  h_s = M_{s-1} h_{s-1} + B_{s-1}   (s = 2 .. nseg-1)
// (B_0 already starts from the initial state).  Thread t owns rows t/2 (+128 i)
// and columns 4 (t % 2) .. + 4 of the CTA's 8-column slice.  The transposed
// transitions stream through shared memory in 64-row chunks by bulk copies,
// double-buffered: every chunk is issued two chunks ahead of its use, across
// the step boundary.  Waits are bounded; on a timeout the scan stops and the
// later start states are left unwritten.
// ---------------------------------------------------------------------------
constexpr int COMB_THREADS = 256, COMB_COLS = 8, COMB_KCH = 64;

template <int K>
struct CombSmem {
  float mt[2][COMB_KCH * K];     // rows k of M^T (k = the input index of the transition)
  float hs[K * COMB_COLS];       // current start state slice
  uint64_t full[2];
};

template <int K, int V>
__global__ void __launch_bounds__(COMB_THREADS) gdn_seg_combine_kernel(Params p) {
  constexpr int RPT = K / 128, NKC = K / COMB_KCH;
  constexpr uint32_t CH_BYTES = COMB_KCH * K * 4;
  extern __shared__ __align__(16) unsigned char csm_raw[];
  CombSmem<K>& sm = *reinterpret_cast<CombSmem<K>*>(csm_raw);
  const int nh = blockIdx.y, v0 = blockIdx.x * COMB_COLS, tid = threadIdx.x;
  const int nseg = p.nseg, rr = tid >> 1, c0 = (tid & 1) * 4;
  const size_t sKV = (size_t)K * V;
  const float* B = p.seg_b + (size_t)nh * nseg * sKV;
  const float* M = p.seg_m + (size_t)nh * nseg * K * K;
  float* Hs = p.seg_h + (size_t)nh * nseg * sKV;
  const int nch = (nseg - 2) * NKC;                 // chunks of M_1 .. M_{nseg-2}
  auto issue = [&](int f) {                         // thread 0: chunk f into buffer f & 1
    const int s = 1 + f / NKC, kc = f % NKC;
    tc::mbar_expect_tx(&sm.full[f & 1], CH_BYTES);
    tc::bulk_load(sm.mt[f & 1], M + (size_t)s * K * K + (size_t)kc * COMB_KCH * K, CH_BYTES, &sm.full[f & 1]);
  };
  if (tid == 0) {
    tc::mbar_init(&sm.full[0], 1);
    tc::mbar_init(&sm.full[1], 1);
    tc::fence_barrier_init();
    for (int f = 0; f < 2 && f < nch; ++f) issue(f);
  }
  __syncthreads();
  int f = 0;
  for (int s = 1; s < nseg; ++s) {
    float acc[RPT][4];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const float4 b = *reinterpret_cast<const float4*>(B + (size_t)(s - 1) * sKV + (size_t)(rr + 128 * i) * V + v0 + c0);
      acc[i][0] = b.x; acc[i][1] = b.y; acc[i][2] = b.z; acc[i][3] = b.w;
    }
    if (s > 1) {
      for (int kc = 0; kc < NKC; ++kc, ++f) {
        if (!__syncthreads_and(tc::mbar_wait(&sm.full[f & 1], (f >> 1) & 1))) {
          // record, then let the (at most two) bulk copies in flight land before exiting
          if (tid == 0) {
            atomicCAS(p.err, 0, 32);
            for (int g = f; g < f + 2 && g < nch; ++g) tc::mbar_wait(&sm.full[g & 1], (g >> 1) & 1);
          }
          __syncthreads();
          return;
        }
        const float* mt = sm.mt[f & 1];
        const float* hk = sm.hs + kc * COMB_KCH * COMB_COLS + c0;
#pragma unroll 8
        for (int k = 0; k < COMB_KCH; ++k) {
          const float4 hv = *reinterpret_cast<const float4*>(hk + k * COMB_COLS);
#pragma unroll
          for (int i = 0; i < RPT; ++i) {
            const float a = mt[k * K + rr + 128 * i];
            acc[i][0] = fmaf(a, hv.x, acc[i][0]);
            acc[i][1] = fmaf(a, hv.y, acc[i][1]);
            acc[i][2] = fmaf(a, hv.z, acc[i][2]);
            acc[i][3] = fmaf(a, hv.w, acc[i][3]);
          }
        }
        __syncthreads();                            // buffer f & 1 fully read
        if (tid == 0 && f + 2 < nch) issue(f + 2);
      }
    }
    __syncthreads();                                // every read of hs of this step is done
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const float4 o = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      *reinterpret_cast<float4*>(sm.hs + (rr + 128 * i) * COMB_COLS + c0) = o;
      *reinterpret_cast<float4*>(Hs + (size_t)s * sKV + (size_t)(rr + 128 * i) * V + v0 + c0) = o;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Kernel 3: output.  Grid (V / BVO, num_chunks, H); 4 warps, warp w: rows 16w..16w+15.
// ---------------------------------------------------------------------------
template <int K, int BVO>
struct OutSmem {
  static constexpr int LDK = K + 8, LDV = BVO + 8;
  __nv_bfloat16 qs[BT * LDK];
  __nv_bfloat16 ks[BT * LDK];
  __nv_bfloat16 hs[K * LDV];
  __nv_bfloat16 vs[BT * LDV];
  float gcs[BT];
};

template <int K, int V, int BVO>
__global__ void __launch_bounds__(NTHREADS) gdn_output_kernel(Params p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  using S = OutSmem<K, BVO>;
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int v0 = blockIdx.x * BVO, c = blockIdx.y, h = blockIdx.z, H = p.H;
  const ChunkLoc loc = locate_chunk(p, c);
  const int t0 = loc.bos + loc.it * BT, L = loc.len;
  if (L <= 0) return;
  {
    constexpr int KV = K / 8, VV = BVO / 8;
    for (int idx = tid; idx < BT * KV; idx += NTHREADS) {
      const int r = idx / KV, cv = (idx % KV) * 8;
      const bool ok = r < L;
      const size_t off = ((size_t)(t0 + (ok ? r : 0)) * H + h) * K + cv;
      cp_async16(&sm.qs[r * S::LDK + cv], p.qn + off, ok);
      cp_async16(&sm.ks[r * S::LDK + cv], p.kn + off, ok);
    }
    const __nv_bfloat16* hg = p.hs + ((size_t)c * H + h) * K * V + v0;
    for (int idx = tid; idx < K * VV; idx += NTHREADS) {
      const int r = idx / VV, cv = (idx % VV) * 8;
      cp_async16(&sm.hs[r * S::LDV + cv], hg + (size_t)r * V + cv, true);
    }
    for (int idx = tid; idx < BT * VV; idx += NTHREADS) {
      const int r = idx / VV, cv = (idx % VV) * 8;
      const bool ok = r < L;
      cp_async16(&sm.vs[r * S::LDV + cv], p.vnew + ((size_t)(t0 + (ok ? r : 0)) * H + h) * V + v0 + cv, ok);
    }
    cp_async_commit();
    if (tid < BT) sm.gcs[tid] = (tid < L) ? p.gc[(size_t)(t0 + tid) * H + h] : 0.f;
    cp_async_wait<0>();
    __syncthreads();
  }
  constexpr int NB = BVO / 8;
  float acc[NB][4];
  float sa[8][4];
#pragma unroll
  for (int nn = 0; nn < NB; ++nn)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nn][e] = 0.f;
#pragma unroll
  for (int nn = 0; nn < 8; ++nn)
#pragma unroll
    for (int e = 0; e < 4; ++e) sa[nn][e] = 0.f;
#pragma unroll 2
  for (int kk = 0; kk < K; kk += 16) {
    uint32_t a[4];
    load_a_rowmajor(a, sm.qs, S::LDK, warp * 16, kk, lane);
#pragma unroll
    for (int n0 = 0; n0 < BVO; n0 += 16) {
      uint32_t b[4];
      load_b_kmajor_rows_x2n(b, sm.hs, S::LDV, kk, n0, lane);
      mma_bf16(acc[n0 / 8], a, b);
      mma_bf16(acc[n0 / 8 + 1], a, b + 2);
    }
#pragma unroll
    for (int n0 = 0; n0 < BT; n0 += 16) {
      uint32_t b[4];
      load_b_nmajor_rows_x2n(b, sm.ks, S::LDK, kk, n0, lane);
      mma_bf16(sa[n0 / 8], a, b);
      mma_bf16(sa[n0 / 8 + 1], a, b + 2);
    }
  }
  const int r0 = warp * 16 + g8, r1 = r0 + 8;
  const float gr0 = sm.gcs[r0], gr1 = sm.gcs[r1];
  const float eg0 = __expf(gr0), eg1 = __expf(gr1);
#pragma unroll
  for (int nn = 0; nn < NB; ++nn) {
    acc[nn][0] *= eg0; acc[nn][1] *= eg0;
    acc[nn][2] *= eg1; acc[nn][3] *= eg1;
  }
  // gated causal scores -> bf16 A fragments (C-fragment layout equals A-fragment layout pairwise)
  uint32_t af[4][4];
#pragma unroll
  for (int nn = 0; nn < 8; ++nn) {
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = (e < 2) ? r0 : r1;
      const int j = nn * 8 + 2 * t4 + (e & 1);
      x[e] = (j <= i && i < L) ? sa[nn][e] * __expf(sm.gcs[i] - sm.gcs[j]) : 0.f;
    }
    const int kstep = nn >> 1, hi = nn & 1;
    af[kstep][hi ? 2 : 0] = pack_bf16(x[0], x[1]);
    af[kstep][hi ? 3 : 1] = pack_bf16(x[2], x[3]);
  }
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
#pragma unroll
    for (int n0 = 0; n0 < BVO; n0 += 16) {
      uint32_t b[4];
      load_b_kmajor_rows_x2n(b, sm.vs, S::LDV, ks * 16, n0, lane);
      mma_bf16(acc[n0 / 8], af[ks], b);
      mma_bf16(acc[n0 / 8 + 1], af[ks], b + 2);
    }
  const float sc = p.scale;
#pragma unroll
  for (int nn = 0; nn < NB; ++nn) {
    const int cc = v0 + nn * 8 + 2 * t4;
    if (r0 < L)
      *reinterpret_cast<uint32_t*>(p.o + ((size_t)(t0 + r0) * H + h) * V + cc) =
          pack_bf16(acc[nn][0] * sc, acc[nn][1] * sc);
    if (r1 < L)
      *reinterpret_cast<uint32_t*>(p.o + ((size_t)(t0 + r1) * H + h) * V + cc) =
          pack_bf16(acc[nn][2] * sc, acc[nn][3] * sc);
  }
}

}  // namespace gdn

int gdn_seg_combine(float* seg_b, float* seg_m, float* seg_h, int nseg, int nh, int K, int V, int* err,
                    cudaStream_t st) {
  gdn::Params p{};
  p.seg_b = seg_b;
  p.seg_m = seg_m;
  p.seg_h = seg_h;
  p.nseg = nseg;
  p.err = err;
  auto go = [&](auto kern, int KK) {
    const size_t sc = sizeof(gdn::CombSmem<128>) + (KK == 256 ? sizeof(gdn::CombSmem<256>) - sizeof(gdn::CombSmem<128>) : 0);
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sc);
    kern<<<dim3(V / gdn::COMB_COLS, nh), gdn::COMB_THREADS, sc, st>>>(p);
    return check_launch("gdn_seg_combine_kernel");
  };
  if (K == 128 && V == 128) return go(gdn::gdn_seg_combine_kernel<128, 128>, 128);
  if (K == 128 && V == 256) return go(gdn::gdn_seg_combine_kernel<128, 256>, 128);
  if (K == 128 && V == 512) return go(gdn::gdn_seg_combine_kernel<128, 512>, 128);
  return set_error(KB200_ERR_INVALID, "gdn_seg_combine: unsupported dims");
}
}  // namespace kb

// ===========================================================================
// Host side: C ABI
// ===========================================================================
namespace {
using namespace kb;

// State-pass V-slice width: 0 = chosen from the grid size, 16 or 32 forced by the
// KB200_GDN_STATE_BV environment variable (a tuning knob, read once).
int state_bv() {
  static const int bv = [] {
    const char* s = getenv("KB200_GDN_STATE_BV");
    const int v = s ? atoi(s) : 0;
    return (v == 16 || v == 32) ? v : 0;
  }();
  return bv;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}


// How the state pass runs: V-slice width and segment count.
//
// The pass is a chain of dependent chunk steps; its time is the latency of one
// step times the chunk count.  Narrower V slices shorten each step and put more
// CTAs on the SMs, so they are used when the 16-wide grid still fits one CTA per
// SM (few heads, e.g. one Ulysses rank's share).  Measured on B200 at T 32760:
// H 24 1.69 ms (32) vs 1.81 (16); H 12 1.18 vs 1.10; H 3 0.78 vs 0.67.
//
// When even that leaves SMs idle, the chunks of each (fixed-length) sequence
// are split into segments that run concurrently: a local pass per segment from
// a zero state plus its K x K transition (K/BV more CTAs per segment), a short
// fp32 scan over the segments, then the final pass from each segment's start
// state.  Segments are sized so the local pass holds at most two CTAs per SM
// and each segment has at least 16 chunks.  KB200_GDN_SEGMENTS forces a count.
struct StatePlan { int bv, nseg, seg_chunks; };

StatePlan state_plan(const KB200GdnArgs* a) {
  StatePlan s{32, 1, 0};
  const long nh = (long)a->N * a->H;
  const int sms = sm_count();
  if (state_bv() == 16 || (state_bv() == 0 && 2 * (a->V / 32) * nh <= sms)) s.bv = 16;
  if (a->cu_seqlens) return s;
  const long nt = (a->T + gdn::BT - 1) / gdn::BT;
  long cap = std::max(1L, 2L * sms / (nh * ((a->V + a->K) / s.bv)));
  if (const char* e = getenv("KB200_GDN_SEGMENTS")) cap = std::max(1, atoi(e));
  long nseg = std::min(std::min(cap, nt / 16), 32L);
  if (nseg > 1) {
    s.seg_chunks = (int)((nt + nseg - 1) / nseg);
    s.nseg = (int)((nt + s.seg_chunks - 1) / s.seg_chunks);
  }
  if (s.nseg < 2) { s.nseg = 1; s.seg_chunks = 0; }
  return s;
}

struct WsLayout { size_t err, qn, kn, gc, w, u, vnew, hs, seg_b, seg_m, seg_h, total; StatePlan sp; };

WsLayout ws_layout(const KB200GdnArgs* a) {
  const size_t TT = (size_t)a->B * a->T, H = a->H, K = a->K, V = a->V;
  WsLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes); return o; };
  const size_t nqk = a->use_qk_l2norm ? TT * H * K * 2 : 0;
  L.err = take(16);
  L.qn = take(nqk);
  L.kn = take(nqk);
  L.gc = take(TT * H * 4);
  L.w = take(TT * H * K * 2);
  L.u = take(TT * H * V * 2);
  L.vnew = take(TT * H * V * 2);
  L.hs = take((size_t)a->num_chunks * H * K * V * 2);
  L.sp = state_plan(a);
  const size_t segs = L.sp.nseg > 1 ? (size_t)a->N * H * L.sp.nseg : 0;
  L.seg_b = take(segs * K * V * 4);
  L.seg_m = take(segs * K * K * 4);
  L.seg_h = take(segs * K * V * 4);
  L.total = off;
  return L;
}

int validate(const KB200GdnArgs* a) {
  if (!a) return set_error(KB200_ERR_INVALID, "gdn: null args");
  if (a->B <= 0 || a->T < 0 || a->H <= 0)
    return set_error(KB200_ERR_INVALID, "gdn: bad shape B=%lld T=%lld H=%lld", (long long)a->B,
                     (long long)a->T, (long long)a->H);
  if (!((a->K == 128 || a->K == 256) && (a->V == 128 || a->V == 256 || a->V == 512)))
    return set_error(KB200_ERR_INVALID, "gdn: unsupported head dims K=%lld V=%lld (K in {128,256}, V in {128,256,512})",
                     (long long)a->K, (long long)a->V);
  if (a->cu_seqlens && (a->B != 1 || !a->chunk_indices || !a->chunk_offsets))
    return set_error(KB200_ERR_INVALID, "gdn: varlen needs B == 1 and chunk_indices/chunk_offsets");
  if (!a->cu_seqlens) {
    const int64_t nt = (a->T + 63) / 64;
    if (a->N != a->B || a->num_chunks != a->B * nt)
      return set_error(KB200_ERR_INVALID, "gdn: N must be B and num_chunks B*ceil(T/64)");
  }
  if ((a->B * a->T) * a->H * (a->K > a->V ? a->K : a->V) >= (int64_t)1 << 31)
    return set_error(KB200_ERR_INVALID, "gdn: tensor too large for 32-bit token indexing");
  const void* ptrs[] = {a->q, a->k, a->v, a->o};
  for (const void* p : ptrs) {
    if (!p) return set_error(KB200_ERR_INVALID, "gdn: null tensor pointer");
    if (!aligned16(p)) return set_error(KB200_ERR_ALIGN, "gdn: q/k/v/o must be 16-byte aligned");
  }
  if (!a->g || !a->beta) return set_error(KB200_ERR_INVALID, "gdn: null g/beta");
  return KB200_OK;
}

// 3-D map (K, H, tokens) of a [tokens, H, K] bf16 tensor: boxes of 64 channels x
// 1 head x 64 tokens, 128-byte swizzle, zero fill past the last token.
int state_map(CUtensorMap* m, const void* base, int64_t tokens, int64_t H, int K) {
  kb::tc::EncodeTiledFn fn = kb::tc::encode_tiled_fn();
  if (!fn) return kb::set_error(KB200_ERR_LAUNCH, "gdn: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)H, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)H * K * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)gdn::BT};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return kb::set_error(KB200_ERR_LAUNCH, "gdn: tensor map encode failed (%d)", (int)r);
  return KB200_OK;
}

template <int K, int V, int BV>
int launch_state(gdn::Params p, const gdn::StateMaps& maps, const StatePlan& sp, unsigned nh, cudaStream_t st) {
  const size_t s2 = sizeof(gdn::StateSmem<K, BV>) + 1024;
  cudaFuncSetAttribute(gdn::gdn_state_kernel<K, V, BV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2);
  if (sp.nseg < 2) {
    p.seg_mode = 0;
    gdn::gdn_state_kernel<K, V, BV><<<dim3(V / BV, nh), gdn::STATE_THREADS, s2, st>>>(p, maps);
    return check_launch("gdn_state_kernel");
  }
  p.nseg = sp.nseg;
  p.seg_chunks = sp.seg_chunks;
  p.seg_mode = 1;
  gdn::gdn_state_kernel<K, V, BV><<<dim3((V + K) / BV, nh * sp.nseg), gdn::STATE_THREADS, s2, st>>>(p, maps);
  if (int e = check_launch("gdn_state_kernel (segment-local)")) return e;
  const size_t sc = sizeof(gdn::CombSmem<K>);
  cudaFuncSetAttribute(gdn::gdn_seg_combine_kernel<K, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sc);
  gdn::gdn_seg_combine_kernel<K, V><<<dim3(V / gdn::COMB_COLS, nh), gdn::COMB_THREADS, sc, st>>>(p);
  if (int e = check_launch("gdn_seg_combine_kernel")) return e;
  p.seg_mode = 2;
  gdn::gdn_state_kernel<K, V, BV><<<dim3(V / BV, nh * sp.nseg), gdn::STATE_THREADS, s2, st>>>(p, maps);
  return check_launch("gdn_state_kernel");
}

template <int K, int V>
int launch(const KB200GdnArgs* a, const WsLayout& L, char* ws, cudaStream_t st) {
  gdn::Params p{};
  p.q = (const __nv_bfloat16*)a->q;
  p.k = (const __nv_bfloat16*)a->k;
  p.v = (const __nv_bfloat16*)a->v;
  p.g = a->g;
  p.beta = (const __nv_bfloat16*)a->beta;
  p.h0 = a->initial_state;
  p.o = (__nv_bfloat16*)a->o;
  p.ht = a->final_state;
  p.cu_seqlens = a->cu_seqlens;
  p.chunk_indices = a->chunk_indices;
  p.chunk_offsets = a->chunk_offsets;
  p.qn = a->use_qk_l2norm ? (__nv_bfloat16*)(ws + L.qn) : (__nv_bfloat16*)a->q;
  p.kn = a->use_qk_l2norm ? (__nv_bfloat16*)(ws + L.kn) : (__nv_bfloat16*)a->k;
  p.gc = (float*)(ws + L.gc);
  p.w = (__nv_bfloat16*)(ws + L.w);
  p.u = (__nv_bfloat16*)(ws + L.u);
  p.vnew = (__nv_bfloat16*)(ws + L.vnew);
  p.hs = (__nv_bfloat16*)(ws + L.hs);
  p.T = (int)a->T;
  p.H = (int)a->H;
  p.NT = (int)((a->T + 63) / 64);
  p.scale = a->scale;
  p.l2norm = a->use_qk_l2norm;
  p.err = (int*)(ws + L.err);
  p.seg_b = (float*)(ws + L.seg_b);
  p.seg_m = (float*)(ws + L.seg_m);
  p.seg_h = (float*)(ws + L.seg_h);
  const int H = (int)a->H;
  const int nchunks = (int)a->num_chunks;
  constexpr int BV = 32, BVO = 64;
  if (cudaMemsetAsync(p.err, 0, sizeof(int), st) != cudaSuccess) return check_launch("gdn error word reset");
  if (nchunks > 0) {
    const size_t s1 = sizeof(gdn::PrepSmem<K, V>);
    cudaFuncSetAttribute(gdn::gdn_prepare_kernel<K, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s1);
    gdn::gdn_prepare_kernel<K, V><<<dim3(nchunks, H), gdn::NTHREADS, s1, st>>>(p);
    if (int e = check_launch("gdn_prepare_kernel")) return e;
  }
  gdn::StateMaps maps;
  if (int e = state_map(&maps.w, p.w, a->B * a->T, H, K)) return e;
  if (int e = state_map(&maps.k, p.kn, a->B * a->T, H, K)) return e;
  if (L.sp.bv == 16) {
    if (int e = launch_state<K, V, 16>(p, maps, L.sp, (unsigned)(a->N * H), st)) return e;
  } else {
    if (int e = launch_state<K, V, BV>(p, maps, L.sp, (unsigned)(a->N * H), st)) return e;
  }
  if (nchunks > 0) {
    const size_t s3 = sizeof(gdn::OutSmem<K, BVO>);
    cudaFuncSetAttribute(gdn::gdn_output_kernel<K, V, BVO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s3);
    gdn::gdn_output_kernel<K, V, BVO><<<dim3(V / BVO, nchunks, H), gdn::NTHREADS, s3, st>>>(p);
    if (int e = check_launch("gdn_output_kernel")) return e;
  }
  return KB200_OK;
}

// Head dim K = 128 (every configuration of the benchmarked path) runs the tcgen05
// kernels of gdn_tc.cu; K = 256 runs the mma.sync kernels above.
size_t gdn_ws_total(const KB200GdnArgs* a) {
  return gdntc::supported(a) ? gdntc::layout(a).total : ws_layout(a).total;
}

int gdn_launch_any(const KB200GdnArgs* a, char* ws, cudaStream_t st) {
  if (gdntc::supported(a)) return gdntc::launch(a, gdntc::layout(a), ws, st);
  const WsLayout L = ws_layout(a);
#define KB_GDN_CASE(KK, VV) \
  if (a->K == KK && a->V == VV) return launch<KK, VV>(a, L, ws, st);
  KB_GDN_CASE(256, 128)
  KB_GDN_CASE(256, 256)
  KB_GDN_CASE(256, 512)
#undef KB_GDN_CASE
  return kb::set_error(KB200_ERR_INVALID, "gdn: unsupported dims");
}
}  // namespace

extern "C" size_t kb200_gdn_workspace_size(const KB200GdnArgs* a) {
  if (validate(a) != KB200_OK) return 0;
  return gdn_ws_total(a);
}

extern "C" int kb200_gdn_status(const void* workspace, void* stream) {
  if (!workspace) return kb::set_error(KB200_ERR_INVALID, "gdn_status: null workspace");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int code = 0;
  if (cudaMemcpyAsync(&code, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return check_launch("gdn_status");
  if (code != 0) return kb::set_error(KB200_ERR_TIMEOUT, "gdn: a device-side wait gave up (site %d)", code);
  return KB200_OK;
}

extern "C" int kb200_gdn_launch_count(const KB200GdnArgs* a) {
  if (validate(a) != KB200_OK) return -1;
  if (gdntc::supported(a)) return gdntc::launch_count(a);
  const StatePlan sp = state_plan(a);
  return (a->num_chunks > 0 ? 2 : 0) + (sp.nseg > 1 ? 3 : 1);
}

extern "C" int kb200_gdn_chunk_fwd(const KB200GdnArgs* a, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  if (int e = validate(a)) return e;
  const size_t total = gdn_ws_total(a);
  if (!workspace || workspace_bytes < total)
    return kb::set_error(KB200_ERR_WORKSPACE, "gdn: workspace needs %zu bytes, got %zu", total, workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return kb::set_error(KB200_ERR_ALIGN, "gdn: workspace must be 256-byte aligned");
  return gdn_launch_any(a, static_cast<char*>(workspace), static_cast<cudaStream_t>(stream));
}

// ===========================================================================
// Allocation-free variant of kb200_gdn_chunk_fwd.
//
// Some callers cannot call cudaMalloc (or ask an allocator) at the point where
// they run the operator -- for example code running inside a host callback or
// a plugin host that owns all device memory and hands out only inputs and
// outputs.  For them this entry point takes its scratch from a fixed,
// file-scope device array instead of a caller-provided workspace.  The array
// lives in every GPU that loads this library until the process exits.
// ===========================================================================

namespace {
constexpr size_t kGdnNoAllocScratchBytes = size_t(64) << 20;   // 64 MiB per device
static __device__ __align__(256) unsigned char g_gdn_noalloc_scratch[kGdnNoAllocScratchBytes];

// Device address of the scratch array on the current device.  Looked up on every
// call (cheap, allocates nothing), so it stays right after a device reset or a
// re-created primary context.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_gdn_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return set_error(KB200_ERR_LAUNCH, "gdn_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
  *out = p;
  return KB200_OK;
}
}  // namespace

extern "C" size_t kb200_gdn_noalloc_scratch_bytes(void) { return kGdnNoAllocScratchBytes; }

extern "C" int kb200_gdn_chunk_fwd_noalloc(const KB200GdnArgs* a, void* stream) {
  if (int e = validate(a)) return e;
  const size_t total = gdn_ws_total(a);
  if (total > kGdnNoAllocScratchBytes)
    return kb::set_error(KB200_ERR_WORKSPACE,
                         "gdn_noalloc: problem needs %zu bytes of scratch, the built-in array "
                         "holds %zu; use kb200_gdn_chunk_fwd with a caller workspace",
                         total, kGdnNoAllocScratchBytes);
  void* ws = nullptr;
  if (int e = noalloc_scratch(&ws)) return e;
  return gdn_launch_any(a, static_cast<char*>(ws), static_cast<cudaStream_t>(stream));
}
