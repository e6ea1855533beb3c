// Host-side launch interface of the sm_100a kernels (internal to librustane_cuda).
// All pointers are device pointers; every launch is asynchronous on `stream`.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rt {

// Fused epilogues of the tcgen05 GEMM C[M,N] = sum_k A[m,k] * B[n,k].
enum GemmEpilogue : int {
  kEpiBf16 = 0,        // out(bf16)[m,n] = C
  kEpiF32 = 1,         // out(f32)[m,n] = C
  kEpiF32Acc = 2,      // out(f32)[m,n] = (beta ? out[m,n] : 0) + C          (weight gradients)
  kEpiResidual = 3,    // out(f32)[m,n] = aux(f32)[m,n] + alpha * C          (x + a*o residual)
  kEpiRope = 4,        // out(bf16) = C, interleaved-pair RoPE on columns < rope_cols
  kEpiSwiglu = 5,      // tile holds h1|h3 for BN/2 hidden units: out=h13(bf16), out2=gate(bf16)
  kEpiSwigluBwd = 6,   // C = dgate; aux = h13(bf16): out = dh13(bf16) (dh1 | dh3 halves)
  // out(bf16) = C (= dO of attention); aux = O(bf16) [M][ld_aux]; out2(f32) =
  // D[b][h][pos] = sum over head h's 128 columns of bf16(C) * O, m = b * seq + pos
  // (the attention backward's rowsum).  256-wide tiles only, N % 128 == 0.
  kEpiBf16RowDot = 7,
};

struct GemmArgs {
  // Operand A: a_mn == false -> A stored [M][K] (row stride lda); true -> [K][M].
  const void* a = nullptr;
  int64_t lda = 0;
  bool a_mn = false;
  // Operand B: b_mn == false -> B stored [N][K] (row stride ldb); true -> [K][N].
  const void* b = nullptr;
  int64_t ldb = 0;
  bool b_mn = false;
  int M = 0, N = 0, K = 0;  // kEpiSwiglu: N = number of hidden units (output h1/h3 columns)
  int epi = kEpiBf16;
  void* out = nullptr;
  int64_t ldo = 0;
  void* out2 = nullptr;
  int64_t ldo2 = 0;
  const void* aux = nullptr;
  int64_t ld_aux = 0;
  float alpha = 1.f;
  int beta = 0;
  const float* rope_cos = nullptr;  // [seq][64]
  const float* rope_sin = nullptr;
  int seq = 0;
  int rope_cols = 0;
  int n_half = 0;  // kEpiSwiglu / kEpiSwigluBwd: column offset of the h3 / dh3 half
  int* err = nullptr;
  int force_bn = 0;  // 0: choose from the wave count; 128/192/256 force a 1-CTA tile width, -256/-192/-128 the CTA-pair kernel
  // Restrict the choice to the single-CTA kernels.  The LM step does not set it:
  // with the fitted tile cost model, CTA-pair grids also win in the overlapped
  // backward, where another stream's GEMMs share the SMs (600M step 196.5k ->
  // 201k tok/s, same-box A/B).
  bool shared_sms = false;
  // kEpiF32Acc only: sum of squares of the written (final) values, one float per
  // epilogue warp of every CTA (slot = CTA * 8 + warp; CTA pairs: pair * 16 + rank * 8
  // + warp), the slots of CTAs the grid does not have set to zero, so the
  // sumsq_slots floats always add up to the output's squared norm in a fixed order.
  float* sumsq = nullptr;
  int sumsq_slots = 0;  // at least gemm_sumsq_slots()
};

// Returns a cudaError_t-compatible code (0 = launched) or -1 on bad arguments.
int gemm_launch(const GemmArgs& g, cudaStream_t stream);
// 2-D bf16 tensor map [outer][inner] (row stride ld elements), 128-byte swizzled
// boxes of box_inner x box_outer; false if the driver entry point is missing.
bool make_tmap_bf16(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                    uint32_t box_inner, uint32_t box_outer);
int num_sms();
// Floats a GemmArgs::sumsq buffer needs (8 per SM).
int gemm_sumsq_slots();

}  // namespace rt
