// Launch interface of the causal attention kernels (internal).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rt {

struct AttnArgs {
  int batch = 0, S = 0, heads = 0, hd = 128, D = 0;
  const __nv_bfloat16* qkv = nullptr;  // [M, ldq]: Q | K | V, roped Q and K
  int64_t ldq = 0;
  __nv_bfloat16* out = nullptr;  // forward: O [M, ldo]; backward: O (input)
  int64_t ldo = 0;
  float* lse2 = nullptr;  // [batch, heads, S] log2-domain softmax statistic
  // backward only
  const __nv_bfloat16* dout = nullptr;  // dO [M, lddo]
  int64_t lddo = 0;
  float* dvec = nullptr;  // [batch, heads, S] scratch: rowsum(dO * O)
  // tcgen05 backward: dvec already holds rowsum(dO * O) (written by the epilogue of
  // the GEMM that produced dO), so the rowsum pass is skipped.
  bool dvec_ready = false;
  __nv_bfloat16* dqkv = nullptr;  // [M, lddq]: dQ | dK | dV (RoPE backward applied)
  int64_t lddq = 0;
  const float* rope_cos_b = nullptr;  // [hd/2][S]
  const float* rope_sin_b = nullptr;
  int* err = nullptr;  // device error word (bounded-wait timeouts of the tcgen05 kernels)
  // tcgen05 backward: dS^T tiles, attn_bwd_scratch_bytes(batch, S, heads) bytes, 16-B aligned
  __nv_bfloat16* ds_scratch = nullptr;
};

// Forward on tcgen05 / TMEM (attention_tc.cu).
int attn_forward(const AttnArgs& a, cudaStream_t s);
// Backward with mma.sync (attention.cu): needs only the dvec scratch.
int attn_backward(const AttnArgs& a, cudaStream_t s);
// Backward on tcgen05 / TMEM (attention_bwd_tc.cu): needs dvec and ds_scratch.
int attn_backward_tc(const AttnArgs& a, cudaStream_t s);
size_t attn_bwd_scratch_bytes(int batch, int S, int heads);
// rowsum(dO * O) per (sequence, head, query) into a.dvec (attention.cu).
int attn_bwd_rowsum(const AttnArgs& a, cudaStream_t s);

}  // namespace rt
