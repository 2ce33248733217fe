// gdn_tc.cuh -- shared declarations of the tcgen05 GDN chunk forward (gdn_tc.cu)
// and its dispatch from the C ABI (gdn_chunk.cu).
#pragma once
#include <cuda.h>
#include "common.cuh"
#include "kb200_internal.h"

namespace kb {
namespace gdntc {

// Per (chunk, head) blobs written by the prep kernel, laid out as the
// shared-memory tiles the state pass multiplies from.
constexpr uint32_t W_BYTES = 64 * 128 * 2;     // w rows, bf16 [2 atoms][64 tokens][128 B], 128-byte swizzle
constexpr uint32_t AQK_BYTES = 64 * 64 * 2;    // gated causal q.k, bf16 [64 i][64 j], 128-byte swizzle
constexpr int G_FLOATS = 132;                  // e^{g_t} [64], e^{g_last - g_t} [64], e^{g_last}, 3 pad
constexpr uint32_t G_BYTES = G_FLOATS * 4;     // 528 (16-byte multiple)
// U^T: per 128-wide V slice, bf16 [128 v][64 tokens], 128-byte swizzle (16 KB)

struct TcParams {
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
  __nv_bfloat16* qn;   // L2-normalised q / k ([tokens, H, 128]) when l2norm, else null
  __nv_bfloat16* kn;
  void* wb;
  void* ab;
  void* ub;
  float* gb;
  int T, H, V, NT;
  float scale;
  int l2norm;
  int* err;
  int seg_mode, nseg, seg_chunks;
  float* seg_b;        // [N*H, nseg, 128, V]  segment end states from zero
  float* seg_m;        // [N*H, nseg, 128, 128] segment transitions, transposed
  float* seg_h;        // [N*H, nseg, 128, V]  segment start states
};

struct PrepMaps { CUtensorMap q, k, v, qn, kn; };   // qn / kn: the l2-normalised copies (stores)
struct StMaps { CUtensorMap q, k, o; };

struct TcWs { size_t err, qn, kn, wb, ab, ub, gb, seg_b, seg_m, seg_h, total; int nseg, seg_chunks; };

bool supported(const KB200GdnArgs* a);
TcWs layout(const KB200GdnArgs* a);
int launch_count(const KB200GdnArgs* a);
int launch(const KB200GdnArgs* a, const TcWs& L, char* ws, cudaStream_t st);

}  // namespace gdntc

// Segment combine of the state pass (gdn_chunk.cu): start states
// h_1 = B_0, h_s = M_{s-1} h_{s-1} + B_{s-1} in fp32.
int gdn_seg_combine(float* seg_b, float* seg_m, float* seg_h, int nseg, int nh, int K, int V, int* err,
                    cudaStream_t st);
}  // namespace kb
