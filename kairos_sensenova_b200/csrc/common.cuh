// common.cuh -- small device helpers shared by the kb200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#define KB_DEVI __device__ __forceinline__

namespace kb {

// ---------------------------------------------------------------- conversions
KB_DEVI uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}
KB_DEVI float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// The two bf16 of a pack_bf16 word as floats (low half first).
KB_DEVI float2 unpack_bf16(uint32_t v) { return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u)); }

KB_DEVI uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- cp.async
KB_DEVI void cp_async16(void* smem, const void* gmem, bool pred) {
  int n = pred ? 16 : 0;   // zero-fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(n));
}
KB_DEVI void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
KB_DEVI void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---------------------------------------------------------------- ldmatrix
KB_DEVI void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
KB_DEVI void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
KB_DEVI void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
KB_DEVI void ldsm_x2_t(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}

// ---------------------------------------------------------------- mma.sync
// D(16x8 f32) += A(16x16 bf16, row) * B(16x8 bf16, col)
KB_DEVI void mma_bf16(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Fragment loaders for a 16x16 A tile stored row-major in shared memory
// (element (r, c) at base[r*ld + c], bf16) and for B tiles.
// A (row-major, M x K): rows r0..r0+15, cols c0..c0+15.
KB_DEVI void load_a_rowmajor(uint32_t* a, const __nv_bfloat16* base, int ld, int r0, int c0,
                             int lane) {
  const __nv_bfloat16* p = base + (r0 + (lane & 15)) * ld + c0 + ((lane >> 4) << 3);
  ldsm_x4(a[0], a[1], a[2], a[3], p);
}
// A given as its transpose stored row-major: A(m, k) = S[k*ld + m]   (K x M storage)
KB_DEVI void load_a_transposed(uint32_t* a, const __nv_bfloat16* base, int ld, int m0, int k0,
                               int lane) {
  // matrices: 0:(m0..7,k0..7) 1:(m0+8..,k0..7) 2:(m0..7,k0+8..) 3:(m0+8..,k0+8..)
  int mat = lane >> 3, r = lane & 7;
  int kk = k0 + ((mat >> 1) << 3) + r;
  int mm = m0 + ((mat & 1) << 3);
  ldsm_x4_t(a[0], a[1], a[2], a[3], base + kk * ld + mm);
}
// B (K x N) stored row-major (element (k, n) at base[k*ld + n]); two n-tiles of 8.
// b[0..1] -> n-tile n0, b[2..3] -> n-tile n0+8.
KB_DEVI void load_b_kmajor_rows_x2n(uint32_t* b, const __nv_bfloat16* base, int ld, int k0, int n0,
                                    int lane) {
  int mat = lane >> 3, r = lane & 7;
  int kk = k0 + ((mat & 1) << 3) + r;
  int nn = n0 + ((mat >> 1) << 3);
  ldsm_x4_t(b[0], b[1], b[2], b[3], base + kk * ld + nn);
}
// One n-tile of 8 of such a B: b[0..1] -> n-tile n0 (lanes 16-31 repeat 0-15's addresses).
KB_DEVI void load_b_kmajor_rows_x1n(uint32_t* b, const __nv_bfloat16* base, int ld, int k0, int n0, int lane) {
  const int kk = k0 + (((lane >> 3) & 1) << 3) + (lane & 7);
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(b[0]), "=r"(b[1]) : "r"(smem_u32(base + kk * ld + n0)));
}
// B given as N x K row-major storage (element (k, n) at base[n*ld + k]); two n-tiles.
KB_DEVI void load_b_nmajor_rows_x2n(uint32_t* b, const __nv_bfloat16* base, int ld, int k0, int n0,
                                    int lane) {
  int mat = lane >> 3, r = lane & 7;
  int nn = n0 + ((mat >> 1) << 3) + r;
  int kk = k0 + ((mat & 1) << 3);
  ldsm_x4(b[0], b[1], b[2], b[3], base + nn * ld + kk);
}

KB_DEVI float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
KB_DEVI float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Packed fp32 pair arithmetic (Blackwell f32x2 instructions): one issue slot for two lanes.
KB_DEVI float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{.reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;}\n"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
KB_DEVI float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;}\n"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
KB_DEVI float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;}\n"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

}  // namespace kb
