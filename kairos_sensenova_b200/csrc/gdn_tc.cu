// gdn_tc.cu -- chunked gated delta rule forward on 5th-generation tensor cores
// (tcgen05 + TMEM, TMA / bulk copies), sm_100a, head dim K = 128.
//
// Two kernels (plus the segment combine of gdn_chunk.cu when the state pass is
// split into concurrent segments):
//
// 1. gdn_prep_tc_kernel -- one CTA per (64-token chunk, head), parallel:
//      q, k, v tiles by TMA; optional L2 norm of q, k     (fla/modules/l2norm.py:98-130)
//      in-chunk gate cumsum (warp scan)                    (fla/ops/utils/cumsum.py:27-65)
//      S = K K^T and Q K^T on tcgen05 (M64 N64, bf16)      (fla/ops/common/chunk_scaled_dot_kkt.py:28-73)
//      A = beta_i e^{g_i-g_j} S_ij (i > j); Aqk = S^qk_ij e^{g_i-g_j} (j <= i)
//      (I + A)^-1 by blocks (fla/ops/utils/solve_tril.py:184-331): the four
//        16x16 diagonal inverses by forward substitution in fp32, then the merge
//        on tcgen05 in tf32 (K-major operands) with the transposed factors
//          M = Lo^T D^T,  E = D^T (I - M),  X^T = E (I + M^2)
//        (D: the diagonal-block inverses, Lo: the off-diagonal blocks of A;
//        (I + A) = (I + Ld)(I + D Lo) and (I + M)^-1 = (I - M)(I + M^2), M^4 = 0)
//      w = Ai (beta e^g k) and u^T = (beta v)^T Ai^T on tcgen05  (fla/ops/gated_delta_rule/wy_fast.py:27-81)
//    and writes per (chunk, head) blobs that are already the shared-memory images
//    the state pass multiplies from: W, U^T, Aqk (bf16, 128-byte swizzled) and the
//    gate factors e^{g_t}, e^{g_last - g_t}, e^{g_last}.
// 2. gdn_state_tc_kernel -- one CTA per (sequence x head, 128-wide V slice[, segment]),
//    sequential over chunks, in the transposed frame (rows of h^T = V columns of
//    the state live in the 128 TMEM lanes and in the registers of 128 threads):
//      P    = h^T W^T           (tcgen05, M128 N64 K128)
//      v_new = u - P; vg = v_new e^{g_last - g_t}   (threads, fp32)
//      X    = vg^T K            (tcgen05, M128 N128 K64); h <- e^{g_last} h + X
//                                                  (fla/ops/common/chunk_delta_h.py:52-224)
//      O    = scale (e^{g_i} h^T Q^T + v_new^T Aqk^T)   (tcgen05, two M128 N64 products)
//                                                  (fla/ops/common/chunk_o.py:41-128)
//    The output is formed in the same pass from the state at the chunk start, so
//    no per-chunk state snapshot is written or read back.  Warps 0-3 run the
//    dependent chain, warps 4-7 drain the output products, warp 8 issues the
//    MMAs and warp 9 streams the next chunks' blobs and q/k tiles.
//
// Numerics follow the reference's rounding points: normalised q/k, Ai, w, u,
// v_new, the gated v_new and the state operand are bf16; S, A, the solve (tf32
// operands), gates, the state and every accumulation are fp32.
//
// Every mbarrier wait is bounded.  A wait that gives up records its site in the
// workspace error word; the CTA stops issuing work, waits (bounded) for the
// copies and MMAs it already issued, and frees TMEM only if those completed.
#include "common.cuh"
#include "kb200_internal.h"
#include "tc_common.cuh"
#include "gdn_tc.cuh"
#include <algorithm>
#include <cstdlib>

namespace kb {
namespace gdntc {

using bf16 = __nv_bfloat16;
constexpr int BT = 64;

// Byte offset of 16-byte chunk `ch` (0..7) of row `row` inside a 128-byte-swizzled
// atom (the atom base is 1024-aligned; rows are 128 bytes).
KB_DEVI uint32_t swz(int row, int ch) { return (uint32_t)(row * 128 + ((ch ^ (row & 7)) << 4)); }

// Round a dynamic shared-memory pointer up to 1024 bytes by pointer arithmetic on
// the shared array itself, so the compiler keeps knowing it is shared memory (and
// emits shared, not generic, loads and stores).
KB_DEVI unsigned char* align1024(unsigned char* p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// Bounded wait of this file: about 0.2 s at B200 clocks, far above any normal wait
// (microseconds), so a lost arrival ends the CTA quickly instead of holding the GPU.
constexpr long long WAIT_BUDGET = 400000000LL;
KB_DEVI bool wait_(uint64_t* bar, uint32_t parity) { return tc::mbar_wait(bar, parity, WAIT_BUDGET); }

KB_DEVI void fail(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

struct ChunkLoc { int n, it, bos, len; };
KB_DEVI ChunkLoc locate(const TcParams& p, int c) {
  ChunkLoc r;
  if (p.cu_seqlens) {
    r.n = p.chunk_indices[2 * c];
    r.it = p.chunk_indices[2 * c + 1];
    if (r.n < 0) { r.n = r.it = r.bos = r.len = 0; return r; }
    const int s = p.cu_seqlens[r.n], e = p.cu_seqlens[r.n + 1];
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

// Timing probes of the debug build (-DKB_GDN_TRACE): clock64() at phase boundaries
// of one CTA of each kernel, written to a buffer set by kb200_gdn_set_trace.
#ifdef KB_GDN_TRACE
__device__ long long* g_gdn_trace;
// the buffer pointer is read once per thread (gtr, set at kernel entry); a probe is one
// clock read and one store
#define PTRACE(slot) do { if (gtr && blockIdx.x == 200 && blockIdx.y == 0 && threadIdx.x == 0) \
  gtr[(slot)] = clock64(); } while (0)
#define STRACE(li, slot) do { if (gtr && blockIdx.x == 0 && blockIdx.y == 0 && (li) < 256) \
  gtr[64 + (li) * 8 + (slot)] = clock64(); } while (0)
#define GTR_INIT long long* const gtr = g_gdn_trace
#else
#define PTRACE(slot) do { } while (0)
#define STRACE(li, slot) do { } while (0)
#define GTR_INIT do { } while (0)
#endif

KB_DEVI float bf(uint32_t u, int hi) { return hi ? __uint_as_float(u & 0xffff0000u) : __uint_as_float(u << 16); }

// ===========================================================================
// 1. Prep.  Grid (chunk slots, H); 128 threads.  An M = 64 tcgen05 product puts
// row r in TMEM lane 32 (r / 16) + r % 16; each warp reads its 16 rows with the
// two-half load, so thread (warp w, lane l) owns row r = 16 w + l % 16 and the
// 32-column half l / 16 of it: all 128 threads work on every phase.
// ===========================================================================
template <int V>
struct PrepLayout {
  static constexpr uint32_t KT = 0;            // k tile                       [2 atoms][64][128 B]
  static constexpr uint32_t QT = 16384;        // q tile; then T1: Lo^T, E (fp32); then the bf16 Ai^T tile
  static constexpr uint32_t T2 = 32768;        // D^T rows (fp32), then the beta-scaled bf16 Ai^T tile
  static constexpr uint32_t T3 = 49152;        // A (fp32 [64][64], column-swizzled), then M rows
  static constexpr uint32_t T4 = 65536;        // D rows, then M^T rows, then (M^2)^T rows (fp32)
  static constexpr uint32_t VT = 81920;        // v tile                        [V/64 atoms][64][128 B]
  static constexpr uint32_t AQS = VT + V * 128;  // staging of the Aqk blob for its bulk store
  static constexpr uint32_t MISC = AQS + 8192;
  static constexpr uint32_t BYTES = MISC + 640 + 1024;
  static constexpr uint32_t TMEM_COLS = (128 + V / 2) <= 256 ? 256 : 512;
};

struct PrepMisc {
  float gcs[64];
  float bs[64];
  uint64_t tma_bar, mma_bar;
  uint32_t tmem_base;
  int abort;
};

// A scratch: element (r, j) of a [64][64] fp32 array at r * 64 + (j ^ (r & 31)), so
// that both a row and a column are read without bank conflicts.
KB_DEVI int as_idx(int r, int j) { return r * 64 + (j ^ (r & 31)); }

// 8 consecutive fp32 of row `row`, columns 8c..8c+7 (c in 0..7), of a fp32 K-major
// tile [2 atoms of 32 columns][64 rows][128 B] -> two 16-byte chunks.
KB_DEVI void st_f32x8(unsigned char* tile, int row, int c, const float* x) {
  unsigned char* base = tile + (c >> 2) * 8192;
  const int ch = (c & 3) * 2;
  *reinterpret_cast<float4*>(base + swz(row, ch)) = make_float4(x[0], x[1], x[2], x[3]);
  *reinterpret_cast<float4*>(base + swz(row, ch + 1)) = make_float4(x[4], x[5], x[6], x[7]);
}
KB_DEVI void ld_f32x8(const unsigned char* tile, int row, int c, float* x) {
  const unsigned char* base = tile + (c >> 2) * 8192;
  const int ch = (c & 3) * 2;
  const float4 a = *reinterpret_cast<const float4*>(base + swz(row, ch));
  const float4 b = *reinterpret_cast<const float4*>(base + swz(row, ch + 1));
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <int V>
__global__ void __launch_bounds__(128, 2) gdn_prep_tc_kernel(const __grid_constant__ PrepMaps maps, TcParams p) {
  using LY = PrepLayout<V>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = align1024(smem_raw);
  PrepMisc& ms = *reinterpret_cast<PrepMisc*>(sm + LY::MISC);
  float* As = reinterpret_cast<float*>(sm + LY::T3);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, h = blockIdx.y, H = p.H;
  GTR_INIT;
  const ChunkLoc loc = locate(p, c);
  const int t0 = loc.bos + loc.it * BT, L = loc.len;
  if (L <= 0) return;
  if (*reinterpret_cast<volatile int*>(p.err)) return;   // an earlier CTA already gave up
  if (tid == 0) {
    tc::mbar_init(&ms.tma_bar, 1);
    tc::mbar_init(&ms.mma_bar, 1);
    ms.abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&ms.tmem_base, LY::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  PTRACE(0);
  tc::tc_fence_after();
  // warp-uniform TMEM base (broadcast from lane 0): MMA operands stay in uniform registers
  const uint32_t tmem = __shfl_sync(0xffffffffu, ms.tmem_base, 0);
  // shared-memory descriptors of every MMA operand tile, computed by every thread (warp-uniform)
  const uint64_t d_kt = tc::sdesc_sw128_kmajor(sm + LY::KT), d_qt = tc::sdesc_sw128_kmajor(sm + LY::QT);
  const uint64_t d_t2 = tc::sdesc_sw128_kmajor(sm + LY::T2), d_t3 = tc::sdesc_sw128_kmajor(sm + LY::T3);
  const uint64_t d_t4 = tc::sdesc_sw128_kmajor(sm + LY::T4);
  const uint64_t d_ai_mn = tc::sdesc_sw128_mnmajor(sm + LY::QT, 8192), d_kt_mn = tc::sdesc_sw128_mnmajor(sm + LY::KT, 8192);
  const uint64_t d_vt_mn = tc::sdesc_sw128_mnmajor(sm + LY::VT, 8192);
  const uint64_t d_t2_mn = tc::sdesc_sw128_mnmajor(sm + LY::T2, 8192);   // the beta-scaled Ai^T (u product)
  const uint32_t tq = tmem + ((uint32_t)(warp * 32) << 16);     // this warp's TMEM lane quarter
  const int r = warp * 16 + (lane & 15);                          // row of M = 64 products
  const int hc = lane >> 4;                                       // column half
  const int blk = warp;                                           // r / 16
  int mma_uses = 0;
  bool ok = true;

  if (tid == 0) {
    tc::mbar_expect_tx(&ms.tma_bar, (uint32_t)(4 + V / 64) * 8192u);
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      tc::tma_load_3d(sm + LY::KT + a * 8192, &maps.k, &ms.tma_bar, a * 64, h, t0);
      tc::tma_load_3d(sm + LY::QT + a * 8192, &maps.q, &ms.tma_bar, a * 64, h, t0);
    }
#pragma unroll
    for (int a = 0; a < V / 64; ++a) tc::tma_load_3d(sm + LY::VT + a * 8192, &maps.v, &ms.tma_bar, a * 64, h, t0);
  }
  // gate cumsum (warp 0) and beta (warp 1) while the tiles land
  if (warp == 0) {
    const int i0 = 2 * lane, i1 = i0 + 1;
    const float g0 = (i0 < L) ? p.g[(size_t)(t0 + i0) * H + h] : 0.f;
    const float g1 = (i1 < L) ? p.g[(size_t)(t0 + i1) * H + h] : 0.f;
    const float pair = g0 + g1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float excl = incl - pair;
    ms.gcs[i0] = excl + g0;
    ms.gcs[i1] = excl + g0 + g1;
  } else if (warp == 1) {
    for (int i = lane; i < BT; i += 32) ms.bs[i] = (i < L) ? __bfloat162float(p.beta[(size_t)(t0 + i) * H + h]) : 0.f;
  }
  ok = wait_(&ms.tma_bar, 0);
  if (!__syncthreads_and(ok)) {
    if (tid == 0) {
      fail(p.err, 41);
      wait_(&ms.tma_bar, 0);   // let the copies land before the CTA exits
    }
    ok = false;
  }
  PTRACE(1);
  // gate factors of the chunk for the state pass: e^{g_t}, e^{g_last - g_t} (0 past the
  // chunk end, so those rows drop out of the state update) and e^{g_last}
  if (ok && tid < 64) {
    float* gb = p.gb + ((size_t)c * H + h) * G_FLOATS;
    const float gl = ms.gcs[L - 1], gt = ms.gcs[tid];
    gb[tid] = tid < L ? __expf(gt) : 0.f;
    gb[64 + tid] = tid < L ? __expf(gl - gt) : 0.f;
    if (tid == 0) {
      gb[128] = __expf(gl);
      gb[129] = gb[130] = gb[131] = 0.f;
    }
  }
  // optional L2 norm of the q and k rows (y = x / sqrt(sum x^2 + 1e-6), bf16), in
  // place in shared memory and to the normalised global copies the state pass reads
  if (ok && p.l2norm) {
    const int rr = tid & 63;
    unsigned char* tile = sm + (tid < 64 ? LY::KT : LY::QT);
    bf16* dst = tid < 64 ? p.kn : p.qn;
    uint4 x[16];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      x[j] = *reinterpret_cast<const uint4*>(tile + (j >> 3) * 8192 + swz(rr, j & 7));
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&x[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = bf(w[e], 0), b = bf(w[e], 1);
        ss = fmaf(a, a, fmaf(b, b, ss));
      }
    }
    const float rs = 1.0f / sqrtf(ss + 1e-6f);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&x[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = pack_bf16(bf(w[e], 0) * rs, bf(w[e], 1) * rs);
      *reinterpret_cast<uint4*>(tile + (j >> 3) * 8192 + swz(rr, j & 7)) = x[j];
      // a partial chunk's tail rows belong to the next sequence: row stores there
      if (L < BT && rr < L) *reinterpret_cast<uint4*>(dst + ((size_t)(t0 + rr) * H + h) * 128 + j * 8) = x[j];
    }
  }
  tc::fence_proxy_async_smem();
  __syncthreads();
  if (ok && p.l2norm && L == BT && tid == 0) {
    // a full chunk's normalised q and k tiles -> global by TMA (read back by the state pass)
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      tc::tma_store_3d(&maps.kn, sm + LY::KT + a * 8192, a * 64, h, t0);
      tc::tma_store_3d(&maps.qn, sm + LY::QT + a * 8192, a * 64, h, t0);
    }
    tc::bulk_commit_group();
  }
  // ---- S_kk = K K^T (TMEM cols 0..63), S_qk = Q K^T (cols 64..127) ----
  if (ok && warp == 0 && tc::elect_one()) {
    tc::tc_fence_after();
    constexpr uint32_t ID = tc::idesc_f32acc(1, 64, 64, 0, 0);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t off = ((ks >> 2) * 8192 + (ks & 3) * 32) >> 4;
      tc::mma_bf16(tmem + 0, d_kt + off, d_kt + off, ID, ks > 0);
      tc::mma_bf16(tmem + 64, d_qt + off, d_kt + off, ID, ks > 0);
    }
    tc::tc_commit(&ms.mma_bar);
  }
  auto mma_wait = [&]() {
    ++mma_uses;
    bool w = wait_(&ms.mma_bar, (mma_uses - 1) & 1);
    tc::tc_fence_after();
    if (!__syncthreads_and(w)) {
      if (tid == 0) fail(p.err, 42);
      ok = false;
    }
  };
  if (ok) mma_wait();
  PTRACE(2);
  const float gr = ms.gcs[r], br = ms.bs[r];
  const bool rv = r < L;
  // ---- elementwise: Aqk half-row -> global blob; A half-row -> A scratch ----
  if (ok) {
    uint32_t sk[32], sq[32];
    tc::tmem_ld16x32bx2_x32<32>(tq + 0, sk);
    tc::tmem_ld16x32bx2_x32<32>(tq + 64, sq);
    // the gate cumsums of this thread's 32 columns, loaded up front (the A scratch stores
    // below would otherwise hold every later load behind them)
    float gj[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 g4 = reinterpret_cast<const float4*>(ms.gcs)[8 * hc + i];
      gj[4 * i] = g4.x; gj[4 * i + 1] = g4.y; gj[4 * i + 2] = g4.z; gj[4 * i + 3] = g4.w;
    }
    tc::tmem_wait_ld();
    PTRACE(23);
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float f[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int jj = c8 * 8 + e + q, j = 32 * hc + jj;
          // e^{g_r - g_j} where the causal masks keep the entry (j <= r)
          const float fac = (rv && j <= r) ? __expf(gr - gj[jj]) : 0.f;
          f[q] = __uint_as_float(sq[jj]) * fac;
          As[as_idx(r, j)] = (j < r) ? br * fac * __uint_as_float(sk[jj]) : 0.f;   // A = beta_r e^{..} S_kk
        }
        w[e >> 1] = pack_bf16(f[0], f[1]);
      }
      *reinterpret_cast<uint4*>(sm + LY::AQS + swz(r, 4 * hc + c8)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  PTRACE(24);
  tc::fence_proxy_async_smem();
  // the q tile is overwritten next: the TMA store of the normalised q / k must have read it
  if (tid == 0) tc::bulk_wait_group_read0();
  PTRACE(25);
  __syncthreads();
  if (ok && tid == 0) {
    tc::bulk_store(reinterpret_cast<unsigned char*>(p.ab) + ((size_t)c * H + h) * AQK_BYTES, sm + LY::AQS, AQK_BYTES);
    tc::bulk_commit_group();
  }
  PTRACE(3);
  // ---- Lo^T half-row r (column r of A below the diagonal blocks) -> T1; D^T row /
  // D row of the diagonal-block inverse (forward / back substitution, fp32) ----
  float x[16];
  if (ok) {
    unsigned char* t1 = sm + LY::QT;
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) {
      float v8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = 32 * hc + 8 * c8 + e;
        v8[e] = ((k >> 4) > blk) ? As[as_idx(k, r)] : 0.f;
      }
      st_f32x8(t1, r, 4 * hc + c8, v8);
    }
    PTRACE(20);
    // thread t < 64: column t % 16 of block t / 16's inverse (row t of D^T);
    // thread t >= 64: row (t - 64) % 16 of it (row t - 64 of D)
    const int rr = tid & 63, b = rr >> 4, cc = rr & 15;
    const float* Ab = As;   // A rows 16 b + i, columns 16 b + j
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = (i == cc) ? 1.f : 0.f;
    if (tid < 64) {
#pragma unroll
      for (int i = 1; i < 16; ++i) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < i; ++j) acc = fmaf(Ab[as_idx(16 * b + i, 16 * b + j)], x[j], acc);
        if (i > cc) x[i] = -acc;
      }
    } else {
#pragma unroll
      for (int j = 14; j >= 0; --j) {
        float acc = 0.f;
#pragma unroll
        for (int i = j + 1; i < 16; ++i) acc = fmaf(Ab[as_idx(16 * b + i, 16 * b + j)], x[i], acc);
        if (j < cc) x[j] = -acc;
      }
    }
    PTRACE(21);
    unsigned char* dst = sm + (tid < 64 ? LY::T2 : LY::T4);
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      float v8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v8[e] = ((c8 >> 1) == b) ? x[(c8 & 1) * 8 + e] : 0.f;
      st_f32x8(dst, rr, c8, v8);
    }
    PTRACE(22);
  }
  tc::fence_proxy_async_smem();
  __syncthreads();
  PTRACE(4);
  constexpr uint32_t ID_TF = tc::idesc_f32acc(2, 64, 64, 0, 0);   // tf32, both K-major
  // C[cols] = A B^T (M64 N64 K64, tf32): A rows [m][k], B rows [n][k], fp32, K-major
  auto tf32_product = [&](uint32_t col, uint64_t da, uint64_t db) {
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t off = ((ks >> 2) * 8192 + (ks & 3) * 32) >> 4;
      tc::mma_tf32(tmem + col, da + off, db + off, ID_TF, ks > 0);
    }
  };
  // half-row r of an M = 64 product (TMEM cols col..col+63) -> registers
  auto ld_half = [&](uint32_t col, float* dst) {
    uint32_t u[32];
    tc::tmem_ld16x32bx2_x32<32>(tq + col, u);
    tc::tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) dst[i] = __uint_as_float(u[i]);
  };
  auto st_half = [&](uint32_t off, const float* v) {
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) st_f32x8(sm + off, r, 4 * hc + c8, v + 8 * c8);
  };
  // ---- round 1: M = Lo^T D^T -> cols 128..191, M^T = D Lo -> cols 192..255 ----
  if (ok && warp == 0 && tc::elect_one()) {
    tc::tc_fence_after();
    tf32_product(128, d_qt, d_t4);
    tf32_product(192, d_t4, d_qt);
    tc::tc_commit(&ms.mma_bar);
  }
  if (ok) mma_wait();
  PTRACE(5);
  float e[32];
  if (ok) {
    ld_half(128, e);
    st_half(LY::T3, e);      // M rows
    ld_half(192, e);
    st_half(LY::T4, e);      // M^T rows
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  // ---- round 2: Q = D^T M -> cols 128..191, (M^2)^T = M^T M^T -> cols 192..255 ----
  if (ok && warp == 0 && tc::elect_one()) {
    tc::tc_fence_after();
    tf32_product(128, d_t2, d_t4);
    tf32_product(192, d_t4, d_t3);
    tc::tc_commit(&ms.mma_bar);
  }
  if (ok) mma_wait();
  PTRACE(6);
  if (ok) {
    // E = D^T - Q (half-row r), kept in registers and as the A rows of round 3
    float dt[32];
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) ld_f32x8(sm + LY::T2, r, 4 * hc + c8, dt + 8 * c8);
    ld_half(128, e);
#pragma unroll
    for (int i = 0; i < 32; ++i) e[i] = dt[i] - e[i];
    st_half(LY::QT, e);
    float m2[32];
    ld_half(192, m2);
    st_half(LY::T4, m2);     // (M^2)^T rows
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  // ---- round 3: F = E M^2 -> cols 128..191 ----
  if (ok && warp == 0 && tc::elect_one()) {
    tc::tc_fence_after();
    tf32_product(128, d_qt, d_t4);
    tc::tc_commit(&ms.mma_bar);
  }
  if (ok) mma_wait();
  PTRACE(7);
  if (ok) {
    // (I + A)^-1 transposed, half-row r = E + F.  The gates of the w / u products scale
    // the rows of the key / value operands (w = Ai diag(beta e^g) K, u = Ai diag(beta) V,
    // wy_fast.py:67,77-79); they are applied to the columns of Ai instead, i.e. to the
    // rows of Ai^T held here: two bf16 tiles, Ai^T diag-scaled by beta e^g (QT, the w
    // product) and by beta (T2, the u product), and the K and V tiles stay as loaded.
    float f[32];
    ld_half(128, f);
    const float sw = ms.bs[r] * __expf(ms.gcs[r]), su = ms.bs[r];
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) {
      uint32_t ww[4], wu[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a0 = e[8 * c8 + 2 * q] + f[8 * c8 + 2 * q], a1 = e[8 * c8 + 2 * q + 1] + f[8 * c8 + 2 * q + 1];
        ww[q] = pack_bf16(a0 * sw, a1 * sw);
        wu[q] = pack_bf16(a0 * su, a1 * su);
      }
      *reinterpret_cast<uint4*>(sm + LY::QT + swz(r, 4 * hc + c8)) = make_uint4(ww[0], ww[1], ww[2], ww[3]);
      *reinterpret_cast<uint4*>(sm + LY::T2 + swz(r, 4 * hc + c8)) = make_uint4(wu[0], wu[1], wu[2], wu[3]);
    }
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  // ---- w = Ai (beta e^g k) -> cols 0..127 (M64 N128); u^T = (beta v)^T Ai^T -> cols
  // 128 + 64 s (M128 N64 per 128-wide V slice s).  Ai^T rows are Ai's MN-major image. ----
  if (ok && warp == 0 && tc::elect_one()) {
    tc::tc_fence_after();
    constexpr uint32_t ID_W = tc::idesc_f32acc(1, 64, 128, 1, 1);
    constexpr uint32_t ID_U = tc::idesc_f32acc(1, 128, 64, 1, 1);
    const uint64_t dai = d_ai_mn, dkt = d_kt_mn;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) tc::mma_bf16(tmem + 0, dai + ks * 128, dkt + ks * 128, ID_W, ks > 0);
#pragma unroll
    for (int vs = 0; vs < V / 128; ++vs) {
      const uint64_t dv = d_vt_mn + (uint64_t)(vs * 16384 / 16);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) tc::mma_bf16(tmem + 128 + 64 * vs, dv + ks * 128, d_t2_mn + ks * 128, ID_U, ks > 0);
    }
    tc::tc_commit(&ms.mma_bar);
  }
  if (ok) mma_wait();
  PTRACE(8);
  if (ok) {
    // w row r, columns 64 hc .. 64 hc + 63 -> W blob atom hc (bf16, 128-byte swizzle)
    // W and U^T are staged in shared memory in their blob layout (T2, and T3 onwards: all
    // free once the products completed) and leave by two bulk stores
    unsigned char* wb = sm + LY::T2 + hc * 8192;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t u[32];
      tc::tmem_ld16x32bx2_x32<64>(tq + 32 * q, u);
      tc::tmem_wait_ld();
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint4 o;
        o.x = pack_bf16(__uint_as_float(u[8 * c8]), __uint_as_float(u[8 * c8 + 1]));
        o.y = pack_bf16(__uint_as_float(u[8 * c8 + 2]), __uint_as_float(u[8 * c8 + 3]));
        o.z = pack_bf16(__uint_as_float(u[8 * c8 + 4]), __uint_as_float(u[8 * c8 + 5]));
        o.w = pack_bf16(__uint_as_float(u[8 * c8 + 6]), __uint_as_float(u[8 * c8 + 7]));
        *reinterpret_cast<uint4*>(wb + swz(r, 4 * q + c8)) = o;
      }
    }
    // u^T row v = tid (M = 128: all lanes) -> U^T blob ([V rows][64 tokens] bf16 swizzled)
    const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
    unsigned char* ub = sm + LY::T3;
#pragma unroll
    for (int vs = 0; vs < V / 128; ++vs) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t u[32];
        tc::tmem_ld32(tl + 128 + 64 * vs + 32 * q, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint4 o;
          o.x = pack_bf16(__uint_as_float(u[8 * c8]), __uint_as_float(u[8 * c8 + 1]));
          o.y = pack_bf16(__uint_as_float(u[8 * c8 + 2]), __uint_as_float(u[8 * c8 + 3]));
          o.z = pack_bf16(__uint_as_float(u[8 * c8 + 4]), __uint_as_float(u[8 * c8 + 5]));
          o.w = pack_bf16(__uint_as_float(u[8 * c8 + 6]), __uint_as_float(u[8 * c8 + 7]));
          *reinterpret_cast<uint4*>(ub + vs * 16384 + swz(tid, 4 * q + c8)) = o;
        }
      }
    }
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  if (ok && tid == 0) {
    tc::bulk_store(reinterpret_cast<unsigned char*>(p.wb) + ((size_t)c * H + h) * W_BYTES, sm + LY::T2, W_BYTES);
    tc::bulk_store(reinterpret_cast<unsigned char*>(p.ub) + ((size_t)c * H + h) * (size_t)(V * 128), sm + LY::T3,
                   V * 128);
    tc::bulk_commit_group();
  }
  // shared memory stays allocated until every bulk store has read its source
  if (tid == 0) tc::bulk_wait_group_read0();
  PTRACE(9);
  if (!ok && mma_uses > 0 && tid == 0) {
    // a wait gave up with MMAs issued: one more (bounded) wait for their completion
    // before TMEM may be freed
    ms.abort = !wait_(&ms.mma_bar, (mma_uses - 1) & 1);
  }
  __syncthreads();
  if (warp == 0 && !ms.abort) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, LY::TMEM_COLS);
  }
}

// ===========================================================================
// 2. State pass with the output fused.  Grid (V/128 [+ 1 transition CTA in the
// segment-local pass], N*H*nseg); three warpgroups: state (thread v owns row v of
// h^T: its V column of the state, 128 fp32 registers), output, and control (one
// thread issues every MMA, one streams the loads).  The state threads hand each
// operand to the issuer through an mbarrier (h_ready, vg_ready) and wait for the
// products on the commits (p_full, x_full), so the chain never waits on MMA issue.
// ===========================================================================
struct StLayout {
  static constexpr uint32_t W = 0, Q = 16384, K = 32768, U = 49152, A = 65536;
  static constexpr uint32_t STAGE = 73728;                     // 72 KB, 1024-aligned
  static constexpr uint32_t H = 2 * STAGE;                     // bf16 h^T  [2 atoms][128 rows][128 B]
  static constexpr uint32_t VG = H + 32768;                    // bf16 gated v_new^T [128 rows][64 tokens]
  static constexpr uint32_t VN = VG + 16384;                   // bf16 v_new^T
  static constexpr uint32_t OST = VN + 16384;                  // bf16 output tile [2 atoms][64 tokens][128 B] (TMA store)
  static constexpr uint32_t MISC = OST + 16384;
  static constexpr uint32_t BYTES = MISC + 2048 + 1024;        // = the 227 KB a CTA may use
};
static_assert(StLayout::STAGE % 1024 == 0 && StLayout::H % 1024 == 0 && StLayout::OST % 1024 == 0,
              "tiles must be 1024-aligned");
static_assert(StLayout::BYTES <= 232448, "shared memory of one CTA");

struct StMisc {
  float g[2][G_FLOATS];            // gate factors of the chunk in each stage (bulk-copied with the stage)
  float eg[4][64];                 // e^{g_i} of chunk li in slot li & 3, for the output warps
  uint64_t in_full[2], in_empty[2], p_full, x_full, o_full[2], o_free[2], h_ready, vg_ready, drain;
  uint32_t tmem_base;
  int abort;
  int keep_tmem;
  int err_seen;                    // the error word as thread 0 read it at entry
};

// The output tile of one chunk into the staging tile: thread v (TMEM lane v) writes
// o[t][v] = scale (e^{g_t} O_inter[v][t] + O_intra[v][t]) for the 64 tokens t
// (bf16, [2 atoms][64 tokens][128 B], 128-byte swizzle) and releases the O buffer
// once both halves are in registers.  One copy of the code (not inlined), so the
// state loop stays small in the instruction cache.
__device__ __noinline__ void emit_stage(unsigned char* __restrict__ ost_base, uint32_t t_oi, uint32_t t_oa,
                                        const float* __restrict__ eg_s, float scale, int v, uint64_t* o_free) {
  // e^{g_t} for the 64 tokens, into registers before any store
  float eg[64];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float4 t = reinterpret_cast<const float4*>(eg_s)[i];
    eg[4 * i] = t.x; eg[4 * i + 1] = t.y; eg[4 * i + 2] = t.z; eg[4 * i + 3] = t.w;
  }
  // lanes v (even) and v + 1 pair up: per token pair (2u, 2u + 1) the even lane
  // writes token 2u and the odd lane token 2u + 1, each as one 32-bit word holding
  // columns (v & ~1, v | 1)
  const bool odd = v & 1;
  const uint32_t row0 = smem_u32(ost_base) + (v >> 6) * 8192 + (v & 6) * 2;
  const int vc = (v & 63) >> 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t oi[32], oa[32];
    tc::tmem_ld32(t_oi + 32 * half, oi);
    tc::tmem_ld32(t_oa + 32 * half, oa);
    tc::tmem_wait_ld();
    if (half == 1) {
      tc::tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) tc::mbar_arrive(o_free);   // one arrival per output warp
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int ta = 32 * half + 2 * u, tb = ta + 1;
      const float ya = scale * fmaf(eg[ta], __uint_as_float(oi[2 * u]), __uint_as_float(oa[2 * u]));
      const float yb = scale * fmaf(eg[tb], __uint_as_float(oi[2 * u + 1]), __uint_as_float(oa[2 * u + 1]));
      // even lane keeps token ta and receives the odd lane's ta; odd lane the reverse
      const float mine = odd ? ya : yb;
      const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
      const int tt = odd ? tb : ta;
      const uint32_t w = odd ? pack_bf16(other, yb) : pack_bf16(ya, other);
      asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(row0 + tt * 128 + ((vc ^ (tt & 7)) << 4)), "r"(w) : "memory");
    }
  }
}

// TMEM columns of the state pass
constexpr uint32_t XCOL = 0, PCOL = 128, OICOL = 192, OACOL = 256;   // O buffers at +128 b

// Warps 0-7: the state chain (warp w: TMEM lane quarter w & 3, rows k of the state
// in half w >> 2); warps 8-11: the output of each chunk; warp 12: MMA issuer; warp
// 13: loads.  Splitting each state column over two threads halves the TMEM reads
// (and their latency) on the chain: a thread holds 64 state values.
constexpr int ST_THREADS = 448;

template <int V>
__global__ void __launch_bounds__(ST_THREADS, 1) gdn_state_tc_kernel(const __grid_constant__ StMaps maps, TcParams p) {
  using LY = StLayout;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = align1024(smem_raw);
  StMisc& ms = *reinterpret_cast<StMisc*>(sm + LY::MISC);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, H = p.H;
  // the 1024-byte alignment of the dynamic shared memory must leave room for the
  // control block (it runs into the alignment slack); otherwise report and stop
  if ((uint32_t)(sm - smem_raw) + LY::MISC + (uint32_t)sizeof(StMisc) > LY::BYTES) {
    if (tid == 0) fail(p.err, 73);
    return;
  }
  const int nseg = p.seg_mode ? p.nseg : 1;
  GTR_INIT;
  const int nh = blockIdx.y / nseg, seg = blockIdx.y % nseg, n = nh / H, h = nh % H;
  const bool trans = p.seg_mode == 1 && (int)blockIdx.x >= V / 128;
  const int v0 = trans ? 0 : blockIdx.x * 128;
  if (p.seg_mode == 1 && (seg == nseg - 1 || (trans && seg == 0))) return;
  // an earlier kernel or CTA already gave up: the whole CTA leaves together (one read,
  // shared), since the state and output warps later meet at named barriers
  if (tid == 0) ms.err_seen = *reinterpret_cast<volatile int*>(p.err);
  __syncthreads();
  if (ms.err_seen) return;
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
  const int nl = max(0, it1 - it0);
  const bool out = p.seg_mode != 1;           // this pass writes o
  const bool load_u = !trans;                 // the transition runs with u = 0
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&ms.in_full[s], 1);
      tc::mbar_init(&ms.in_empty[s], 1);
      tc::mbar_init(&ms.o_full[s], 1);
      tc::mbar_init(&ms.o_free[s], 4);
    }
    tc::mbar_init(&ms.p_full, 1);
    tc::mbar_init(&ms.x_full, 1);
    tc::mbar_init(&ms.h_ready, 8);    // one arrival per state warp
    tc::mbar_init(&ms.vg_ready, 8);
    tc::mbar_init(&ms.drain, 1);
    ms.abort = 0;
    ms.keep_tmem = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&ms.tmem_base, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  // warp-uniform TMEM base (broadcast from lane 0): MMA operands stay in uniform registers
  const uint32_t tmem = __shfl_sync(0xffffffffu, ms.tmem_base, 0);
  auto aborted = [&]() { return *((volatile int*)&ms.abort) != 0; };

  if (warp >= 12) {
    if (warp == 12) {
      // ---------------------------------------------------------------- MMA issuer
      // The whole warp runs the schedule (bounded waits, operand arithmetic) so every MMA
      // operand is warp-uniform and stays in uniform registers; one elected lane issues.
      const bool leader = tc::elect_one();
      constexpr uint32_t ID_P = tc::idesc_f32acc(1, 128, 64, 0, 0);
      constexpr uint32_t ID_X = tc::idesc_f32acc(1, 128, 128, 0, 1);
      const uint64_t dh = tc::sdesc_sw128_kmajor(sm + LY::H);
      const uint64_t dvg = tc::sdesc_sw128_kmajor(sm + LY::VG), dvn = tc::sdesc_sw128_kmajor(sm + LY::VN);
      const uint64_t dw0 = tc::sdesc_sw128_kmajor(sm + LY::W), dq0 = tc::sdesc_sw128_kmajor(sm + LY::Q);
      const uint64_t dk0 = tc::sdesc_sw128_mnmajor(sm + LY::K, 8192), da0 = tc::sdesc_sw128_kmajor(sm + LY::A);
      auto wait_all = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, wait_(bar, parity));
      };
      bool ok = true;
      for (int li = 0; li < nl && ok; ++li) {
        const int s = li & 1, b = li & 1;
        const uint64_t so = (uint64_t)(s * (LY::STAGE / 16));   // stage offset in descriptor units
        // P = h^T W^T and O_inter = h^T Q^T once the state threads wrote h^T
        ok = wait_all(&ms.in_full[s], (li >> 1) & 1) && wait_all(&ms.h_ready, li & 1) &&
             (!out || li < 2 || wait_all(&ms.o_free[b], ((li >> 1) - 1) & 1)) && !aborted();
        if (!ok) { if (leader) fail(p.err, 81); break; }
        tc::tc_fence_after();
        if (lane == 0) STRACE(li, 6);
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc::mma_bf16(tmem + PCOL, dh + (((ks >> 2) * 16384 + (ks & 3) * 32) >> 4),
                         dw0 + so + (((ks >> 2) * 8192 + (ks & 3) * 32) >> 4), ID_P, ks > 0);
          tc::tc_commit(&ms.p_full);
          if (out) {
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              tc::mma_bf16(tmem + OICOL + 128 * b, dh + (((ks >> 2) * 16384 + (ks & 3) * 32) >> 4),
                           dq0 + so + (((ks >> 2) * 8192 + (ks & 3) * 32) >> 4), ID_P, ks > 0);
          }
        }
        __syncwarp();
        // X = vg^T K (the state update) and O_intra = v_new^T Aqk^T once vg, v_new are written
        ok = wait_all(&ms.vg_ready, li & 1) && !aborted();
        if (!ok) { if (leader) fail(p.err, 82); break; }
        tc::tc_fence_after();
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) tc::mma_bf16(tmem + XCOL, dvg + ks * 2, dk0 + so + ks * 128, ID_X, ks > 0);
          tc::tc_commit(&ms.x_full);
          if (out) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              tc::mma_bf16(tmem + OACOL + 128 * b, dvn + ks * 2, da0 + so + ks * 2, ID_P, ks > 0);
            tc::tc_commit(&ms.o_full[b]);
          }
          tc::tc_commit(&ms.in_empty[s]);
        }
        __syncwarp();
        if (lane == 0) STRACE(li, 5);
      }
      if (!ok) ms.abort = 1;
      // every MMA issued here completes before TMEM is freed
      if (leader) tc::tc_commit(&ms.drain);
      __syncwarp();
      if (!wait_all(&ms.drain, 0)) {
        if (leader) fail(p.err, 72);
        ms.keep_tmem = 1;
      }
    } else if (warp == 13 && lane == 0) {
      // ---------------------------------------------------------------- loads
      const uint32_t bytes = W_BYTES + 16384u + G_BYTES + (load_u ? 16384u : 0u) + (out ? 16384u + AQK_BYTES : 0u);
      int issued = 0;
      for (int li = 0; li < nl; ++li) {
        const int s = li & 1;
        if (li >= 2 && !wait_(&ms.in_empty[s], ((li >> 1) - 1) & 1)) {
          if (!aborted()) fail(p.err, 51);
          ms.abort = 1;
          break;
        }
        if (aborted()) break;
        const int it = it0 + li;
        const size_t ch = (size_t)(cbase + it) * H + h;
        const int t0 = bos + it * BT;
        unsigned char* st = sm + s * LY::STAGE;
        tc::mbar_expect_tx(&ms.in_full[s], bytes);
        tc::bulk_load(st + LY::W, reinterpret_cast<const unsigned char*>(p.wb) + ch * W_BYTES, W_BYTES, &ms.in_full[s]);
        tc::bulk_load(ms.g[s], p.gb + ch * G_FLOATS, G_BYTES, &ms.in_full[s]);
        tc::tma_load_3d(st + LY::K, &maps.k, &ms.in_full[s], 0, h, t0);
        tc::tma_load_3d(st + LY::K + 8192, &maps.k, &ms.in_full[s], 64, h, t0);
        if (load_u)
          tc::bulk_load(st + LY::U, reinterpret_cast<const unsigned char*>(p.ub) + ch * (size_t)(V * 128) + v0 * 128,
                        16384, &ms.in_full[s]);
        if (out) {
          tc::tma_load_3d(st + LY::Q, &maps.q, &ms.in_full[s], 0, h, t0);
          tc::tma_load_3d(st + LY::Q + 8192, &maps.q, &ms.in_full[s], 64, h, t0);
          tc::bulk_load(st + LY::A, reinterpret_cast<const unsigned char*>(p.ab) + ch * AQK_BYTES, AQK_BYTES,
                        &ms.in_full[s]);
        }
        ++issued;
      }
      // every load issued here lands before the CTA may exit
      bool drained = true;
      for (int li = max(0, issued - 2); li < issued; ++li) drained &= wait_(&ms.in_full[li & 1], (li >> 1) & 1);
      if (!drained) { fail(p.err, 52); ms.keep_tmem = 1; }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ output
    if (out) {
      const int v = tid - 256;
      const uint32_t tl = tmem + ((uint32_t)((warp - 8) * 32) << 16);
      // output of chunk lo: o = scale (e^{g_i} O_inter + O_intra), bf16, token rows of
      // this V slice
    const float scale = p.scale;
    const size_t ostride = (size_t)H * V;
    auto emit = [&](int lo) {
      const int b = lo & 1;
      const int it = it0 + lo, L = min(BT, Tn - it * BT);
      const int t0 = bos + it * BT;
      // the previous chunk's TMA store must have finished reading the staging tile
      if (tid == 256) tc::bulk_wait_group_read0();
      tc::bar_sync_named(2, 128);
      if (tid == 256) STRACE(lo, 1);
      emit_stage(sm + LY::OST, tl + OICOL + 128 * b, tl + OACOL + 128 * b, ms.eg[lo & 3], scale, v, &ms.o_free[b]);
      if (tid == 256) STRACE(lo, 7);
      tc::fence_proxy_async_smem();
      tc::bar_sync_named(2, 128);
      if (L == BT) {
        if (tid == 256) {
          tc::tma_store_3d(&maps.o, sm + LY::OST, v0, h, t0);
          tc::tma_store_3d(&maps.o, sm + LY::OST + 8192, v0 + 64, h, t0);
          tc::bulk_commit_group();
        }
      } else {
        // the last, partial chunk of a sequence: only its L rows, as 16-byte vectors
        for (int j = v; j < L * 16; j += 128) {
          const int t = j >> 4, c = j & 15;
          *reinterpret_cast<uint4*>(p.o + (size_t)(t0 + t) * ostride + (size_t)h * V + v0 + c * 8) =
              *reinterpret_cast<const uint4*>(sm + LY::OST + (c >> 3) * 8192 + swz(t, c & 7));
        }
      }
    };
      for (int lo = 0; lo < nl; ++lo) {
        const bool w = wait_(&ms.o_full[lo & 1], (lo >> 1) & 1);
        // the four output warps decide together (they meet at named barrier 2 in emit)
        if (!tc::bar_red_and(2, 128, w)) {
          if (tid == 256) fail(p.err, 61);
          ms.abort = 1;
          break;
        }
        tc::tc_fence_after();
        emit(lo);
      }
      if (tid == 256) tc::bulk_wait_group0();   // the output stores complete before the CTA exits
    }
  } else {
    // ------------------------------------------------------------------ state chain
    // thread: state column v (TMEM lane v) and its rows k = 64 kh .. 64 kh + 63
    const int v = tid & 127, kh = tid >> 7, k0 = 64 * kh;
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    float hr[64];
    const bool seg_start0 = p.seg_mode != 0 && seg > 0;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int k = k0 + i;
      float init;
      if (trans)
        init = (k == v) ? 1.f : 0.f;
      else if (seg_start0)
        init = p.seg_mode == 2 ? p.seg_h[(((size_t)nh * nseg + seg) * 128 + k) * V + v0 + v] : 0.f;
      else
        init = p.h0 ? p.h0[((size_t)nh * 128 + k) * V + v0 + v] : 0.f;
      hr[i] = init;
    }
    float dec = 1.f;
    bool ok = true;
    // h <- e^{g_last} h + X (the last chunk's state update): this thread's 64 columns
    // of X in one TMEM wait
    auto update_h = [&]() {
      uint32_t xr[64];
      tc::tmem_ld32(tl + XCOL + k0, xr);
      tc::tmem_ld32(tl + XCOL + k0 + 32, xr + 32);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 64; ++i) hr[i] = fmaf(dec, hr[i], __uint_as_float(xr[i]));
    };
    for (int li = 0; li < nl; ++li) {
      const int s = li & 1;
      unsigned char* st = sm + s * LY::STAGE;
      if (tid == 0) STRACE(li, 0);
      // (a) the previous chunk's update, then this thread's half of the bf16 h^T operand
      if (li > 0) {
        ok = wait_(&ms.x_full, (li - 1) & 1);
        if (!__all_sync(0xffffffffu, ok) || aborted()) { ok = false; break; }
        tc::tc_fence_after();
        update_h();
      }
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        uint4 o;
        o.x = pack_bf16(hr[8 * c8], hr[8 * c8 + 1]);
        o.y = pack_bf16(hr[8 * c8 + 2], hr[8 * c8 + 3]);
        o.z = pack_bf16(hr[8 * c8 + 4], hr[8 * c8 + 5]);
        o.w = pack_bf16(hr[8 * c8 + 6], hr[8 * c8 + 7]);
        *reinterpret_cast<uint4*>(sm + LY::H + kh * 16384 + swz(v, c8)) = o;
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ms.h_ready);
      if (tid == 0) STRACE(li, 2);
      // (b) v_new = u - h^T w^T (chunk_delta_h.py:142-163), gated by e^{g_last - g_t};
      // this thread: tokens 32 kh .. 32 kh + 31 of column v
      ok = wait_(&ms.p_full, li & 1) && wait_(&ms.in_full[s], (li >> 1) & 1);
      if (!__all_sync(0xffffffffu, ok) || aborted()) { ok = false; break; }
      tc::tc_fence_after();
      if (tid == 0) STRACE(li, 3);
      const float* G = ms.g[s];
      {
        uint32_t pr[32];
        tc::tmem_ld32(tl + PCOL + 32 * kh, pr);
        tc::tmem_wait_ld();
#pragma unroll
        for (int ch = 4 * kh; ch < 4 * kh + 4; ++ch) {
          uint4 u4 = make_uint4(0, 0, 0, 0);
          if (load_u) u4 = *reinterpret_cast<const uint4*>(st + LY::U + swz(v, ch));
          const float4 f0 = reinterpret_cast<const float4*>(G + 64)[2 * ch];
          const float4 f1 = reinterpret_cast<const float4*>(G + 64)[2 * ch + 1];
          const float fg[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
          const uint32_t uw[4] = {u4.x, u4.y, u4.z, u4.w};
          uint32_t vnw[4], vgw[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float a0 = bf(uw[q], 0) - __uint_as_float(pr[8 * (ch & 3) + 2 * q]);
            const float a1 = bf(uw[q], 1) - __uint_as_float(pr[8 * (ch & 3) + 2 * q + 1]);
            vnw[q] = pack_bf16(a0, a1);
            vgw[q] = pack_bf16(a0 * fg[2 * q], a1 * fg[2 * q + 1]);
          }
          *reinterpret_cast<uint4*>(sm + LY::VN + swz(v, ch)) = make_uint4(vnw[0], vnw[1], vnw[2], vnw[3]);
          *reinterpret_cast<uint4*>(sm + LY::VG + swz(v, ch)) = make_uint4(vgw[0], vgw[1], vgw[2], vgw[3]);
        }
      }
      dec = G[128];
      if (out && tid < 64) ms.eg[li & 3][tid] = G[tid];
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ms.vg_ready);
      if (tid == 0) STRACE(li, 4);
    }
    if (ok && nl > 0) {
      ok = wait_(&ms.x_full, (nl - 1) & 1);
      tc::tc_fence_after();
      update_h();
    }
    ok = tc::bar_red_and(1, 256, ok && !aborted());
    if (!ok) {
      if (tid == 0) fail(p.err, 71);
      ms.abort = 1;
    } else {
      float* dst = nullptr;
      if (p.seg_mode == 1)
        dst = trans ? p.seg_m + ((size_t)nh * nseg + seg) * 128 * 128 : p.seg_b + ((size_t)nh * nseg + seg) * 128 * V;
      else if (p.ht && (p.seg_mode == 0 || seg == nseg - 1))
        dst = p.ht + (size_t)nh * 128 * V;
      if (dst) {
        if (trans) {
          // row v of the transposed transition (column v of M), this thread's 64 entries
#pragma unroll
          for (int i = 0; i < 64; i += 4)
            *reinterpret_cast<float4*>(dst + (size_t)v * 128 + k0 + i) =
                make_float4(hr[i], hr[i + 1], hr[i + 2], hr[i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) dst[(size_t)(k0 + i) * V + v0 + v] = hr[i];
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0 && !ms.keep_tmem) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace gdntc
}  // namespace kb

#ifdef KB_GDN_TRACE
extern "C" int kb200_gdn_set_trace(long long* p) {
  return cudaMemcpyToSymbol(kb::gdntc::g_gdn_trace, &p, sizeof(p)) == cudaSuccess ? 0 : 4;
}
#endif

// ===========================================================================
// Host side
// ===========================================================================
namespace {
using namespace kb::gdntc;

int map3d(CUtensorMap* m, const void* base, int64_t tokens, int64_t H, int D) {
  kb::tc::EncodeTiledFn fn = kb::tc::encode_tiled_fn();
  if (!fn) return kb::set_error(KB200_ERR_LAUNCH, "gdn_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)(tokens > 0 ? tokens : 1)};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)BT};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return kb::set_error(KB200_ERR_LAUNCH, "gdn_tc: tensor map encode failed (%d)", (int)r);
  return KB200_OK;
}

int sm_count_tc() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int V>
int launch_v(const KB200GdnArgs* a, const kb::gdntc::TcWs& L, char* ws, cudaStream_t st) {
  TcParams p{};
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
  p.qn = a->use_qk_l2norm ? (__nv_bfloat16*)(ws + L.qn) : nullptr;
  p.kn = a->use_qk_l2norm ? (__nv_bfloat16*)(ws + L.kn) : nullptr;
  p.wb = ws + L.wb;
  p.ab = ws + L.ab;
  p.ub = ws + L.ub;
  p.gb = (float*)(ws + L.gb);
  p.T = (int)a->T;
  p.H = (int)a->H;
  p.V = V;
  p.NT = (int)((a->T + BT - 1) / BT);
  p.scale = a->scale;
  p.l2norm = a->use_qk_l2norm;
  p.err = (int*)(ws + L.err);
  p.seg_b = (float*)(ws + L.seg_b);
  p.seg_m = (float*)(ws + L.seg_m);
  p.seg_h = (float*)(ws + L.seg_h);
  const int H = (int)a->H;
  const int64_t tokens = a->B * a->T;
  if (cudaMemsetAsync(p.err, 0, sizeof(int), st) != cudaSuccess) return kb::check_launch("gdn error word reset");
  const int nchunks = (int)a->num_chunks;
  if (nchunks > 0) {
    PrepMaps pm;
    if (int e = map3d(&pm.q, a->q, tokens, H, 128)) return e;
    if (int e = map3d(&pm.k, a->k, tokens, H, 128)) return e;
    if (int e = map3d(&pm.v, a->v, tokens, H, V)) return e;
    pm.qn = pm.q;
    pm.kn = pm.k;
    if (a->use_qk_l2norm) {
      if (int e = map3d(&pm.qn, p.qn, tokens, H, 128)) return e;
      if (int e = map3d(&pm.kn, p.kn, tokens, H, 128)) return e;
    }
    const size_t s1 = PrepLayout<V>::BYTES;
    cudaFuncSetAttribute(gdn_prep_tc_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s1);
    gdn_prep_tc_kernel<V><<<dim3(nchunks, H), 128, s1, st>>>(pm, p);
    if (int e = kb::check_launch("gdn_prep_tc_kernel")) return e;
  }
  StMaps sm;
  const void* qsrc = a->use_qk_l2norm ? (const void*)p.qn : a->q;
  const void* ksrc = a->use_qk_l2norm ? (const void*)p.kn : a->k;
  if (int e = map3d(&sm.q, qsrc, tokens, H, 128)) return e;
  if (int e = map3d(&sm.k, ksrc, tokens, H, 128)) return e;
  if (int e = map3d(&sm.o, a->o, tokens, H, V)) return e;
  const size_t s2 = StLayout::BYTES;
  cudaFuncSetAttribute(gdn_state_tc_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2);
  const unsigned nh = (unsigned)(a->N * H);
  if (L.nseg < 2) {
    p.seg_mode = 0;
    gdn_state_tc_kernel<V><<<dim3(V / 128, nh), ST_THREADS, s2, st>>>(sm, p);
    return kb::check_launch("gdn_state_tc_kernel");
  }
  p.nseg = L.nseg;
  p.seg_chunks = L.seg_chunks;
  p.seg_mode = 1;
  gdn_state_tc_kernel<V><<<dim3(V / 128 + 1, nh * L.nseg), ST_THREADS, s2, st>>>(sm, p);
  if (int e = kb::check_launch("gdn_state_tc_kernel (segment-local)")) return e;
  if (int e = kb::gdn_seg_combine(p.seg_b, p.seg_m, p.seg_h, L.nseg, (int)nh, 128, V, p.err, st)) return e;
  p.seg_mode = 2;
  gdn_state_tc_kernel<V><<<dim3(V / 128, nh * L.nseg), ST_THREADS, s2, st>>>(sm, p);
  return kb::check_launch("gdn_state_tc_kernel");
}
}  // namespace

namespace kb {
namespace gdntc {

bool supported(const KB200GdnArgs* a) { return a->K == 128 && (a->V == 128 || a->V == 256 || a->V == 512); }

// Segments of the state pass: the final pass holds one CTA per (sequence x head,
// V slice, segment) and should fill the SMs; every segment keeps >= 16 chunks.
void plan(const KB200GdnArgs* a, int* nseg, int* seg_chunks) {
  *nseg = 1;
  *seg_chunks = 0;
  if (a->cu_seqlens) return;
  const long nt = (a->T + BT - 1) / BT;
  // the segment-local pass runs N*H*(V/128 + 1) CTAs per segment after the first (the
  // B slices and the transition); as many segments as keep it within one wave (H 24:
  // 4 segments, 1.08 ms against 1.10 with 6; H 3: 25, 0.285 ms against 0.317 with 32)
  const long per_seg = (long)a->N * a->H * (a->V / 128 + 1);
  long cap = 1 + (long)sm_count_tc() / per_seg;
  if (const char* e = getenv("KB200_GDN_SEGMENTS")) cap = std::max(1, atoi(e));
  long ns = std::min(std::min(cap, nt / 16), 32L);
  if (ns > 1) {
    *seg_chunks = (int)((nt + ns - 1) / ns);
    *nseg = (int)((nt + *seg_chunks - 1) / *seg_chunks);
  }
  if (*nseg < 2) { *nseg = 1; *seg_chunks = 0; }
}

TcWs layout(const KB200GdnArgs* a) {
  const size_t TT = (size_t)a->B * a->T, H = a->H, V = a->V, C = (size_t)a->num_chunks;
  TcWs L{};
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes); return o; };
  L.err = take(16);
  const size_t nqk = a->use_qk_l2norm ? TT * H * 128 * 2 : 0;
  L.qn = take(nqk);
  L.kn = take(nqk);
  L.wb = take(C * H * W_BYTES);
  L.ab = take(C * H * AQK_BYTES);
  L.ub = take(C * H * V * 128);
  L.gb = take(C * H * G_BYTES);
  plan(a, &L.nseg, &L.seg_chunks);
  const size_t segs = L.nseg > 1 ? (size_t)a->N * H * L.nseg : 0;
  L.seg_b = take(segs * 128 * V * 4);
  L.seg_m = take(segs * 128 * 128 * 4);
  L.seg_h = take(segs * 128 * V * 4);
  L.total = off;
  return L;
}

int launch_count(const KB200GdnArgs* a) {
  int ns, sc;
  plan(a, &ns, &sc);
  return (a->num_chunks > 0 ? 1 : 0) + (ns > 1 ? 3 : 1);
}

int launch(const KB200GdnArgs* a, const TcWs& L, char* ws, cudaStream_t st) {
  if (a->V == 128) return launch_v<128>(a, L, ws, st);
  if (a->V == 256) return launch_v<256>(a, L, ws, st);
  if (a->V == 512) return launch_v<512>(a, L, ws, st);
  return set_error(KB200_ERR_INVALID, "gdn_tc: unsupported V");
}

}  // namespace gdntc
}  // namespace kb
