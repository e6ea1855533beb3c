// Memory-bound kernels of the LM step: 128-bit vector loads/stores, warp-shuffle
// reductions, fixed-order (deterministic) cross-block reductions.
#include "common.cuh"
#include "elementwise.h"

namespace rt {
namespace {

constexpr float kRmsEps = 1e-5f;  // crates/engine/src/cpu/rmsnorm.rs:10

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block-wide sum in fixed order; result broadcast to all threads. `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < nw ? red[lane] : 0.f;
  r = warp_sum(r);
  return r;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < nw ? red[lane] : -INFINITY;
  return warp_max(r);
}

// ------------------------------------------------------------- embedding
__global__ void embed_gather_kernel(const float* __restrict__ E, const uint32_t* __restrict__ tok,
                                    float* __restrict__ x, int M, int D, int V, int* err) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint32_t t = tok[row];
  float4* dst = reinterpret_cast<float4*>(x + static_cast<int64_t>(row) * D);
  const int D4 = D >> 2;
  if (t >= static_cast<uint32_t>(V)) {
    if (lane == 0) set_error(err, kDevBadToken);
    for (int c = lane; c < D4; c += 32) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(E + static_cast<int64_t>(t) * D);
  for (int c = lane; c < D4; c += 32) dst[c] = src[c];
}

__global__ void embed_scatter_kernel(const float* __restrict__ dx, const int32_t* __restrict__ perm,
                                     const int32_t* __restrict__ seg_start, const uint32_t* __restrict__ seg_tok,
                                     float* __restrict__ dE, int D) {
  const int j = blockIdx.x;
  const int b = seg_start[j], e = seg_start[j + 1];
  float4* row = reinterpret_cast<float4*>(dE + static_cast<int64_t>(seg_tok[j]) * D);
  const int D4 = D >> 2;
  for (int c = threadIdx.x; c < D4; c += blockDim.x) {
    float4 acc = row[c];
    for (int i = b; i < e; ++i) {  // positions in ascending order (embedding.rs:34-44)
      const float4 v = reinterpret_cast<const float4*>(dx + static_cast<int64_t>(perm[i]) * D)[c];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    row[c] = acc;
  }
}

// --------------------------------------------------------------- RMSNorm
// One warp per token row (cpu/rmsnorm.rs:149-183): the row's NV float4 per lane
// are loaded once into registers (all loads in flight together), reduced, then
// scaled and written; NV = D / 128.  Generic widths re-read the row.
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_fwd_reg_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ gamma,
                                                              __nv_bfloat16* __restrict__ out,
                                                              float* __restrict__ rms_inv, int M, int D) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<int64_t>(row) * D);
  float4 v[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = xr[lane + 32 * k];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(D)) + kRmsEps);
  if (lane == 0) rms_inv[row] = r;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<int64_t>(row) * D);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = lane + 32 * k;
    const float4 g = __ldg(g4 + c);
    o[c] = make_uint2(pack_bf16x2(v[k].x * r * g.x, v[k].y * r * g.y), pack_bf16x2(v[k].z * r * g.z, v[k].w * r * g.w));
  }
}

__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                   __nv_bfloat16* __restrict__ out, float* __restrict__ rms_inv, int M, int D) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<int64_t>(row) * D);
  const int D4 = D >> 2;
  float ss = 0.f;
  for (int c = lane; c < D4; c += 32) {
    const float4 v = xr[c];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(D)) + kRmsEps);
  if (lane == 0) rms_inv[row] = r;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<int64_t>(row) * D);
  for (int c = lane; c < D4; c += 32) {
    const float4 v = xr[c], g = g4[c];
    o[c] = make_uint2(pack_bf16x2(v.x * r * g.x, v.y * r * g.y), pack_bf16x2(v.z * r * g.z, v.w * r * g.w));
  }
}

// RMSNorm backward, row part: one warp per token row, two passes over the row
// (the second pass re-reads dy and x from L1/L2).  dgamma is computed by the
// column kernels below, so this kernel is a pure stream.
__global__ void __launch_bounds__(256)
    rmsnorm_bwd_rows_kernel(const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ gamma,
                            const float* __restrict__ rms_inv, const float* __restrict__ resid, float* __restrict__ dx,
                            __nv_bfloat16* __restrict__ dx_bf16, float bf16_scale, int M, int D) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int D4 = D >> 2;
  const int64_t off = static_cast<int64_t>(row) * D;
  const float4* dyr = reinterpret_cast<const float4*>(dy + off);
  const float4* xr = reinterpret_cast<const float4*>(x + off);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float r = rms_inv[row];
  float dot = 0.f;
  for (int c = lane; c < D4; c += 32) {
    const float4 a = dyr[c], b = xr[c], g = g4[c];
    dot += a.x * g.x * (b.x * r) + a.y * g.y * (b.y * r) + a.z * g.z * (b.z * r) + a.w * g.w * (b.w * r);
  }
  dot = warp_sum(dot) * (1.0f / static_cast<float>(D));
  float4* o = reinterpret_cast<float4*>(dx + off);
  const float4* rr = resid ? reinterpret_cast<const float4*>(resid + off) : nullptr;
  uint2* ob = dx_bf16 ? reinterpret_cast<uint2*>(dx_bf16 + off) : nullptr;
  for (int c = lane; c < D4; c += 32) {
    const float4 a = dyr[c], b = xr[c], g = g4[c];
    float4 v;  // dx = rms_inv * (dy*gamma - xhat * dot)   (cpu/rmsnorm.rs:229-236)
    v.x = r * (a.x * g.x - (b.x * r) * dot);
    v.y = r * (a.y * g.y - (b.y * r) * dot);
    v.z = r * (a.z * g.z - (b.z * r) * dot);
    v.w = r * (a.w * g.w - (b.w * r) * dot);
    if (rr) {
      const float4 q = rr[c];
      v.x += q.x;
      v.y += q.y;
      v.z += q.z;
      v.w += q.w;
    }
    o[c] = v;
    if (ob)
      ob[c] = make_uint2(pack_bf16x2(v.x * bf16_scale, v.y * bf16_scale), pack_bf16x2(v.z * bf16_scale, v.w * bf16_scale));
  }
}

// RMSNorm backward writes one dgamma partial row per CTA of a fixed grid of
// G = min(ceil(M / 4), kNormCtas) CTAs; dgamma_reduce adds the G rows in order.
constexpr int kNormCtas = 148;
constexpr int kGroupRows = 4;
__host__ __device__ inline int norm_ctas(int M) {
  const int g = (M + kGroupRows - 1) / kGroupRows;
  return g < kNormCtas ? g : kNormCtas;
}

// Fallback dgamma column partials (widths the pipelined kernel does not take):
// part[b][d] = sum over rows [b * rpb, (b + 1) * rpb) ascending of dy * x * rms_inv.
__global__ void __launch_bounds__(256)
    rmsnorm_dgamma_part_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                               const float* __restrict__ rms_inv, float* __restrict__ part, int M, int D, int rpb) {
  const int d = blockIdx.x * 256 + threadIdx.x;
  if (d >= D) return;
  const int m0 = blockIdx.y * rpb;
  const int m1 = min(M, m0 + rpb);
  float acc = 0.f;
#pragma unroll 4
  for (int m = m0; m < m1; ++m) {
    const int64_t i = static_cast<int64_t>(m) * D + d;
    acc += dy[i] * (x[i] * rms_inv[m]);
  }
  part[static_cast<int64_t>(blockIdx.y) * D + d] = acc;
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// RMSNorm backward, pipelined, for D = 256 * NV2: persistent CTAs take groups
// of 4 rows (g = blockIdx.x, + gridDim.x, ...); the dy and x rows of the next
// STAGES - 1 groups stream into shared memory with cp.async while the current
// group is computed, so HBM stays busy without holding rows in registers (the
// residual-gradient row is loaded into registers one group ahead).  Warps 2r and 2r+1 own the two halves of row r of a group.  Each
// thread sums dgamma for its columns over the rows it handles (its CTA's groups
// in order); the CTA adds its four row slots in order into partial row
// blockIdx.x: deterministic.
template <int NV2, int STAGES>
__global__ void __launch_bounds__(256, 1)
    rmsnorm_bwd_pipe_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                            const float* __restrict__ gamma, const float* __restrict__ rms_inv,
                            const float* __restrict__ resid, float* __restrict__ dx,
                            __nv_bfloat16* __restrict__ dx_bf16, float bf16_scale, float* __restrict__ part, int M,
                            int D) {
  extern __shared__ float4 sm[];  // [STAGES][2 arrays][kGroupRows][D / 4]
  __shared__ float dots[8];
  constexpr int D4 = 64 * NV2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp >> 1, h = warp & 1;
  const int ngroups = (M + kGroupRows - 1) / kGroupRows;
  const uint32_t sbase = smem_u32(sm);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);

  auto issue = [&](int grp, int stage) {
    if (grp < ngroups) {
      for (int a = 0; a < 2; ++a) {
        const float* src = a == 0 ? dy : x;
        for (int i = threadIdx.x; i < kGroupRows * D4; i += 256) {
          const int row = grp * kGroupRows + i / D4;
          if (row < M)
            cp_async16(sbase + static_cast<uint32_t>(((stage * 2 + a) * kGroupRows * D4 + i) * 16),
                       src + static_cast<int64_t>(row) * D + (i % D4) * 4);
        }
      }
    }
    cp_async_commit();  // empty groups too: keeps the wait_group count uniform
  };

  float4 dg[NV2];
#pragma unroll
  for (int k = 0; k < NV2; ++k) dg[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) issue(blockIdx.x + st * gridDim.x, st);
  const float inv_d = 1.0f / static_cast<float>(D);
  // residual gradient of this thread's columns: loaded one group ahead, in registers
  float4 q[NV2], qn[NV2];
  auto load_resid = [&](int grp, float4 (&dst)[NV2]) {
    const int rw = grp * kGroupRows + r;
    if (resid && grp < ngroups && rw < M) {
      const float4* rs = reinterpret_cast<const float4*>(resid + static_cast<int64_t>(rw) * D);
#pragma unroll
      for (int k = 0; k < NV2; ++k) dst[k] = __ldcs(rs + h * (D4 / 2) + lane + 32 * k);
    }
  };
  load_resid(blockIdx.x, qn);
  int it = 0;
  for (int g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
#pragma unroll
    for (int k = 0; k < NV2; ++k) q[k] = qn[k];
    load_resid(g + gridDim.x, qn);
    issue(g + (STAGES - 1) * gridDim.x, (it + STAGES - 1) % STAGES);
    cp_async_wait<STAGES - 1>();
    __syncthreads();  // every thread's copies of group g have landed
    const int stage = it % STAGES;
    const int row = g * kGroupRows + r;
    const float4* sdy = sm + (stage * 2 + 0) * kGroupRows * D4 + r * D4;
    const float4* sx = sm + (stage * 2 + 1) * kGroupRows * D4 + r * D4;
    const float rinv = row < M ? rms_inv[row] : 0.f;
    if (row < M) {
      float dot = 0.f;
#pragma unroll
      for (int k = 0; k < NV2; ++k) {
        const int c = h * (D4 / 2) + lane + 32 * k;
        const float4 a = sdy[c], b = sx[c], gm = __ldg(g4 + c);
        const float hx = b.x * rinv, hy = b.y * rinv, hz = b.z * rinv, hw = b.w * rinv;
        dot += a.x * gm.x * hx + a.y * gm.y * hy + a.z * gm.z * hz + a.w * gm.w * hw;
        dg[k].x += a.x * hx;  // dgamma = sum_m dy * xhat   (cpu/rmsnorm.rs:218-227)
        dg[k].y += a.y * hy;
        dg[k].z += a.z * hz;
        dg[k].w += a.w * hw;
      }
      dot = warp_sum(dot);
      if (lane == 0) dots[warp] = dot;
    }
    __syncthreads();
    if (row < M) {
      const float dot = (dots[2 * r] + dots[2 * r + 1]) * inv_d;
      const int64_t off = static_cast<int64_t>(row) * D;
      float4* o = reinterpret_cast<float4*>(dx + off);
      uint2* ob = dx_bf16 ? reinterpret_cast<uint2*>(dx_bf16 + off) : nullptr;
#pragma unroll
      for (int k = 0; k < NV2; ++k) {
        const int c = h * (D4 / 2) + lane + 32 * k;
        const float4 a = sdy[c], b = sx[c], gm = __ldg(g4 + c);
        float4 v;  // dx = rms_inv * (dy*gamma - xhat * dot)   (cpu/rmsnorm.rs:229-236)
        v.x = rinv * (a.x * gm.x - (b.x * rinv) * dot);
        v.y = rinv * (a.y * gm.y - (b.y * rinv) * dot);
        v.z = rinv * (a.z * gm.z - (b.z * rinv) * dot);
        v.w = rinv * (a.w * gm.w - (b.w * rinv) * dot);
        if (resid) {
          v.x += q[k].x;
          v.y += q[k].y;
          v.z += q[k].z;
          v.w += q[k].w;
        }
        o[c] = v;
        if (ob)
          ob[c] = make_uint2(pack_bf16x2(v.x * bf16_scale, v.y * bf16_scale),
                             pack_bf16x2(v.z * bf16_scale, v.w * bf16_scale));
      }
    }
    __syncthreads();  // stage and dots free for reuse
  }
  cp_async_wait<0>();
  __syncthreads();
  float4* red = sm;  // [kGroupRows][D4]: this CTA's dgamma per row slot
#pragma unroll
  for (int k = 0; k < NV2; ++k) red[r * D4 + h * (D4 / 2) + lane + 32 * k] = dg[k];
  __syncthreads();
  float4* prow = reinterpret_cast<float4*>(part + static_cast<int64_t>(blockIdx.x) * D);
  for (int c = threadIdx.x; c < D4; c += 256) {
    float4 t = red[c];
#pragma unroll
    for (int q = 1; q < kGroupRows; ++q) {
      const float4 u = red[q * D4 + c];
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    prow[c] = t;
  }
}

// dgamma[d] = (accumulate ? dgamma[d] : 0) + sum_b part[b][d]: 32 columns per block of
// 32 warps; warp w sums partials w, w+32, ... in order (at most five rows at the 148-row
// grid of the backward, all loads in flight), then the 32 warp sums in order.  Latency-
// bound: with 8 warps per block the loop ran five dependent rounds of loads (7.5 us).
// blockIdx.y selects one of several gammas: partials at part + y * part_stride, result
// at dgamma + y * D (the gammas sit next to each other in the parameter arena).
constexpr int kDgWarps = 32;
__global__ void __launch_bounds__(32 * kDgWarps) dgamma_reduce_kernel(const float* __restrict__ part, int nblk,
                                                                     float* __restrict__ dgamma, int D,
                                                                     int accumulate, int64_t part_stride) {
  __shared__ float red[kDgWarps][33];
  part += blockIdx.y * part_stride;
  dgamma += static_cast<int64_t>(blockIdx.y) * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int d = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (d < D) {
    int b = warp;
    for (; b + 3 * kDgWarps < nblk; b += 4 * kDgWarps) {
      const float a0 = part[static_cast<int64_t>(b) * D + d];
      const float a1 = part[static_cast<int64_t>(b + kDgWarps) * D + d];
      const float a2 = part[static_cast<int64_t>(b + 2 * kDgWarps) * D + d];
      const float a3 = part[static_cast<int64_t>(b + 3 * kDgWarps) * D + d];
      s += a0;
      s += a1;
      s += a2;
      s += a3;
    }
    for (; b < nblk; b += kDgWarps) s += part[static_cast<int64_t>(b) * D + d];
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && d < D) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kDgWarps; ++w) t += red[w][lane];
    dgamma[d] = accumulate ? dgamma[d] + t : t;
  }
}

// --------------------------------------------------------- cross-entropy
constexpr int kCeThreads = 256;
constexpr int kCeVec = 8;  // float4 per thread -> V <= 8192

__device__ __forceinline__ float capz(float l, float softcap) {
  return softcap > 0.f ? softcap * tanhf(l * (1.0f / softcap)) : l;
}

__global__ void __launch_bounds__(kCeThreads)
    ce_forward_kernel(const float* __restrict__ logits, const uint32_t* __restrict__ tgt, float* __restrict__ row_loss,
                      float* __restrict__ row_lse, int V, float softcap) {
  __shared__ float red[32];
  const int m = blockIdx.x;
  const float4* lr = reinterpret_cast<const float4*>(logits + static_cast<int64_t>(m) * V);
  const int V4 = V >> 2;
  float4 z[kCeVec];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kCeVec; ++j) {
    const int c = threadIdx.x + j * kCeThreads;
    if (c < V4) {
      float4 v = lr[c];
      v.x = capz(v.x, softcap);
      v.y = capz(v.y, softcap);
      v.z = capz(v.z, softcap);
      v.w = capz(v.w, softcap);
      z[j] = v;
      mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
  }
  mx = block_max(mx, red);
  float se = 0.f;
#pragma unroll
  for (int j = 0; j < kCeVec; ++j) {
    const int c = threadIdx.x + j * kCeThreads;
    if (c < V4) se += __expf(z[j].x - mx) + __expf(z[j].y - mx) + __expf(z[j].z - mx) + __expf(z[j].w - mx);
  }
  se = block_sum(se, red);
  if (threadIdx.x == 0) {
    const float lse = mx + logf(se);
    const uint32_t t = tgt[m];
    row_lse[m] = lse;
    row_loss[m] = lse - capz(logits[static_cast<int64_t>(m) * V + t], softcap);
  }
}

__global__ void __launch_bounds__(kCeThreads)
    ce_backward_kernel(const float* __restrict__ logits, const float* __restrict__ row_lse,
                       const uint32_t* __restrict__ tgt, __nv_bfloat16* __restrict__ dl, int V, float softcap,
                       float scale) {
  const int m = blockIdx.x;
  const float4* lr = reinterpret_cast<const float4*>(logits + static_cast<int64_t>(m) * V);
  uint2* o = reinterpret_cast<uint2*>(dl + static_cast<int64_t>(m) * V);
  const int V4 = V >> 2;
  const float lse = row_lse[m];
  const int t = static_cast<int>(tgt[m]);
  for (int c = threadIdx.x; c < V4; c += kCeThreads) {
    const float4 v = lr[c];
    float l[4] = {v.x, v.y, v.z, v.w};
    float d[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float z = l[e], dz = 1.f;
      if (softcap > 0.f) {
        const float th = tanhf(l[e] * (1.0f / softcap));
        z = softcap * th;
        dz = 1.f - th * th;  // full_model.rs:267-273
      }
      float p = __expf(z - lse);
      if (4 * c + e == t) p -= 1.f;
      d[e] = p * scale * dz;
    }
    o[c] = make_uint2(pack_bf16x2(d[0], d[1]), pack_bf16x2(d[2], d[3]));
  }
}

// Forward and backward of the train step in one read of the logits: the row is
// held in registers (kCeVec float4 per thread), so loss, lse and the bf16 dlogits
// come out of the same pass (cross_entropy.rs:58-96 forward and backward).
__global__ void __launch_bounds__(kCeThreads)
    ce_fused_kernel(const float* __restrict__ logits, const uint32_t* __restrict__ tgt, float* __restrict__ row_loss,
                    float* __restrict__ row_lse, __nv_bfloat16* __restrict__ dl, int V, float softcap, float scale) {
  __shared__ float red[32];
  const int m = blockIdx.x;
  const float4* lr = reinterpret_cast<const float4*>(logits + static_cast<int64_t>(m) * V);
  uint2* o = reinterpret_cast<uint2*>(dl + static_cast<int64_t>(m) * V);
  const int V4 = V >> 2;
  const int t = static_cast<int>(tgt[m]);
  float4 z[kCeVec];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kCeVec; ++j) {
    const int c = threadIdx.x + j * kCeThreads;
    if (c < V4) {
      float4 v = __ldcs(lr + c);  // read once: keep it out of L2's way
      v.x = capz(v.x, softcap);
      v.y = capz(v.y, softcap);
      v.z = capz(v.z, softcap);
      v.w = capz(v.w, softcap);
      z[j] = v;
      mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
  }
  mx = block_max(mx, red);
  if (softcap <= 0.f) {
    // uncapped: exp(z - max) once, kept in registers; p = e / sum (the row's target
    // score is read from the logits before the registers are overwritten)
    float zt = 0.f;
    float se = 0.f;
#pragma unroll
    for (int j = 0; j < kCeVec; ++j) {
      const int c = threadIdx.x + j * kCeThreads;
      if (c < V4) {
        if ((t >> 2) == c) {
          const int e = t & 3;
          zt = e == 0 ? z[j].x : (e == 1 ? z[j].y : (e == 2 ? z[j].z : z[j].w));
        }
        z[j].x = __expf(z[j].x - mx);
        z[j].y = __expf(z[j].y - mx);
        z[j].z = __expf(z[j].z - mx);
        z[j].w = __expf(z[j].w - mx);
        se += (z[j].x + z[j].y) + (z[j].z + z[j].w);
      }
    }
    se = block_sum(se, red);
    const float lse = mx + logf(se);
    const float inv = 1.0f / se;
#pragma unroll
    for (int j = 0; j < kCeVec; ++j) {
      const int c = threadIdx.x + j * kCeThreads;
      if (c < V4) {
        float d0 = z[j].x * inv, d1 = z[j].y * inv, d2 = z[j].z * inv, d3 = z[j].w * inv;
        if ((t >> 2) == c) {  // the target column: one thread of the row
          const int e = t & 3;
          d0 -= e == 0 ? 1.f : 0.f;
          d1 -= e == 1 ? 1.f : 0.f;
          d2 -= e == 2 ? 1.f : 0.f;
          d3 -= e == 3 ? 1.f : 0.f;
          row_loss[m] = lse - zt;
        }
        o[c] = make_uint2(pack_bf16x2(d0 * scale, d1 * scale), pack_bf16x2(d2 * scale, d3 * scale));
      }
    }
    if (threadIdx.x == 0) row_lse[m] = lse;
    return;
  }
  float se = 0.f;
#pragma unroll
  for (int j = 0; j < kCeVec; ++j) {
    const int c = threadIdx.x + j * kCeThreads;
    if (c < V4) se += __expf(z[j].x - mx) + __expf(z[j].y - mx) + __expf(z[j].z - mx) + __expf(z[j].w - mx);
  }
  se = block_sum(se, red);
  const float lse = mx + logf(se);
  const float inv_sc = 1.0f / softcap;
#pragma unroll
  for (int j = 0; j < kCeVec; ++j) {
    const int c = threadIdx.x + j * kCeThreads;
    if (c < V4) {
      const float zz[4] = {z[j].x, z[j].y, z[j].z, z[j].w};
      float d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float p = __expf(zz[e] - lse);
        if (4 * c + e == t) {  // the target column: one thread of the row
          p -= 1.f;
          row_loss[m] = lse - zz[e];
        }
        const float th = zz[e] * inv_sc;  // tanh(l / softcap)
        const float dz = 1.f - th * th;   // full_model.rs:267-273
        d[e] = p * scale * dz;
      }
      o[c] = make_uint2(pack_bf16x2(d[0], d[1]), pack_bf16x2(d[2], d[3]));
    }
  }
  if (threadIdx.x == 0) row_lse[m] = lse;
}

__global__ void mean_reduce_kernel(const float* __restrict__ x, int n, float* __restrict__ out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (warp == 0) {
    double r = lane < (blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (lane == 0) out[0] = static_cast<float>(r / n);
  }
}

// ---------------------------------------------------------- grad norm
constexpr int kNormBlocks = 1024;
constexpr int kNormThreads = 256;
constexpr int kSegNormBlocks = 148;  // partials per gradient segment of the train step (one per SM)

__global__ void __launch_bounds__(kNormThreads) sumsq_partial_kernel(const float* __restrict__ x, int64_t n,
                                                                      float* __restrict__ partials) {
  __shared__ double red[32];
  const int64_t n4 = n >> 2;
  const int64_t per = (n4 + gridDim.x - 1) / gridDim.x;
  const int64_t b = per * blockIdx.x, e = min(n4, b + per);
  // eight independent 16-byte loads in flight per thread; fixed order, so the result is deterministic
  constexpr int U = 8;
  float acc[U] = {};
  const int64_t step = static_cast<int64_t>(blockDim.x) * U;
  int64_t i0 = b + threadIdx.x;
  for (; i0 + (U - 1) * blockDim.x < e; i0 += step) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = __ldcs(reinterpret_cast<const float4*>(x) + i0 + u * blockDim.x);
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
  }
  for (int64_t i = i0; i < e; i += blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    acc[0] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u) s += acc[u];
  if (blockIdx.x == gridDim.x - 1)  // tail elements not covered by float4s
    for (int64_t i = (n4 << 2) + threadIdx.x; i < n; i += blockDim.x) s += x[i] * x[i];
  double d = s;
#pragma unroll
  for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = d;
  __syncthreads();
  if (warp == 0) {
    double r = lane < (blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (lane == 0) partials[blockIdx.x] = static_cast<float>(r);
  }
}

// Sum of the partials in a fixed order (double): out_norm = sqrt(sum) as float, or
// out_sq = sum when out_norm is null.
__global__ void sumsq_final_kernel(const float* __restrict__ partials, int n, float* __restrict__ out,
                                   double* __restrict__ out_sq) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += partials[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (warp == 0) {
    double r = lane < (blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (lane == 0) {
      if (out) out[0] = static_cast<float>(sqrt(r));
      if (out_sq) out_sq[0] = r;
    }
  }
}

// out[0] = sum of n floats (fixed order: strided per thread in double, then a fixed
// tree), out[1 .. nout) = 0: folds the per-warp sums of squares the weight-gradient
// GEMMs wrote into a gradient segment's grad-norm partial slots.
__global__ void __launch_bounds__(256) sumsq_fold_kernel(const float* __restrict__ in, int n,
                                                         float* __restrict__ out, int nout) {
  __shared__ double red[8];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += in[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    out[0] = static_cast<float>(t);
  }
  for (int i = 1 + threadIdx.x; i < nout; i += blockDim.x) out[i] = 0.f;
}

__global__ void sqrt_to_float_kernel(const double* __restrict__ sq, float* __restrict__ out) {
  out[0] = static_cast<float>(sqrt(sq[0]));
}

// ----------------------------------------------------------------- AdamW
struct AdamKParams {
  AdamSegment seg[kMaxAdamSegments];
  int nseg;
  float beta1, beta2, eps, bc1, bc2, grad_scale, gsc, clip;
};

__global__ void __launch_bounds__(256) adam_kernel(float* __restrict__ param, const float* __restrict__ grad,
                                                   float* __restrict__ m, float* __restrict__ v,
                                                   __nv_bfloat16* __restrict__ pb, const float* __restrict__ norm,
                                                   const AdamKParams k) {
  float scale = k.grad_scale;
  if (norm) {  // full_model.rs:696-704
    const float raw = *norm;
    scale = (k.clip > 0.f && raw * k.gsc > k.clip) ? k.clip / raw : k.gsc;
  }
  const float omb1 = 1.0f - k.beta1, omb2 = 1.0f - k.beta2;
  for (int s = 0; s < k.nseg; ++s) {
    const AdamSegment sg = k.seg[s];
    const int64_t b4 = sg.begin >> 2, e4 = sg.end >> 2;
    for (int64_t i = b4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < e4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const float4 g4 = reinterpret_cast<const float4*>(grad)[i];
      float4 p4 = reinterpret_cast<float4*>(param)[i];
      float4 m4 = reinterpret_cast<float4*>(m)[i];
      float4 v4 = reinterpret_cast<float4*>(v)[i];
      float gg[4] = {g4.x, g4.y, g4.z, g4.w}, pp[4] = {p4.x, p4.y, p4.z, p4.w}, mm[4] = {m4.x, m4.y, m4.z, m4.w},
            vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // crates/engine/src/cpu/adam.rs:119-131
        const float g = gg[e] * scale;
        const float mi = k.beta1 * mm[e] + omb1 * g;
        const float vi = k.beta2 * vv[e] + omb2 * g * g;
        mm[e] = mi;
        vv[e] = vi;
        const float mh = mi * k.bc1, vh = vi * k.bc2;
        const float upd = mh / (sqrtf(vh) + k.eps);
        pp[e] -= sg.lr * (upd + sg.wd * pp[e]);
      }
      reinterpret_cast<float4*>(param)[i] = make_float4(pp[0], pp[1], pp[2], pp[3]);
      reinterpret_cast<float4*>(m)[i] = make_float4(mm[0], mm[1], mm[2], mm[3]);
      reinterpret_cast<float4*>(v)[i] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      if (sg.write_bf16)
        reinterpret_cast<uint2*>(pb)[i] = make_uint2(pack_bf16x2(pp[0], pp[1]), pack_bf16x2(pp[2], pp[3]));
    }
  }
}

// ---------------------------------------------------------------- misc
__global__ void cast_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n4,
                                 float scale) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    reinterpret_cast<uint2*>(dst)[i] =
        make_uint2(pack_bf16x2(v.x * scale, v.y * scale), pack_bf16x2(v.z * scale, v.w * scale));
  }
}
__global__ void fill_kernel(float* __restrict__ dst, int64_t n, float value) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = value;
}
__global__ void scale_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n, float a) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = a * x[i];
}
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Box-Muller on two 24-bit uniforms per pair of elements.
__global__ void init_normal_kernel(float* __restrict__ dst, int64_t n, uint64_t seed, float std) {
  const int64_t npair = (n + 1) >> 1;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < npair;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = splitmix64(seed ^ splitmix64(static_cast<uint64_t>(i)));
    const float u1 = (static_cast<float>(h >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = static_cast<float>((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1)) * std;
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    dst[2 * i] = r * cs;
    if (2 * i + 1 < n) dst[2 * i + 1] = r * sn;
  }
}
// x_out = x + alpha * p; optional RMSNorm of x_out (one warp per row)
__global__ void residual_rmsnorm_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ p, float alpha,
                                        const float* __restrict__ gamma, float* __restrict__ x_out,
                                        __nv_bfloat16* __restrict__ xn, float* __restrict__ rms_inv, int M, int D) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int64_t off = static_cast<int64_t>(row) * D;
  const float4* xr = reinterpret_cast<const float4*>(x + off);
  const uint2* pr = reinterpret_cast<const uint2*>(p + off);
  float4* outr = reinterpret_cast<float4*>(x_out + off);
  const int D4 = D >> 2;
  float ss = 0.f;
  for (int c = lane; c < D4; c += 32) {
    const float4 a = xr[c];
    const uint2 q = pr[c];
    float4 v;
    v.x = a.x + alpha * bf16lo(q.x);
    v.y = a.y + alpha * bf16hi(q.x);
    v.z = a.z + alpha * bf16lo(q.y);
    v.w = a.w + alpha * bf16hi(q.y);
    outr[c] = v;
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  if (!gamma) return;
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(D)) + kRmsEps);
  if (lane == 0) rms_inv[row] = r;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  uint2* o = reinterpret_cast<uint2*>(xn + off);
  for (int c = lane; c < D4; c += 32) {
    const float4 v = outr[c], g = g4[c];
    o[c] = make_uint2(pack_bf16x2(v.x * r * g.x, v.y * r * g.y), pack_bf16x2(v.z * r * g.z, v.w * r * g.w));
  }
}

__device__ __forceinline__ float normal_at(uint64_t seed, int64_t g, float std) {
  const uint64_t h = splitmix64(seed ^ splitmix64(static_cast<uint64_t>(g >> 1)));
  const float u1 = (static_cast<float>(h >> 40) + 1.0f) * (1.0f / 16777217.0f);
  const float u2 = static_cast<float>((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
  const float r = sqrtf(-2.0f * logf(u1)) * std;
  float sn, cs;
  sincospif(2.0f * u2, &sn, &cs);
  return (g & 1) ? r * sn : r * cs;
}

__global__ void init_normal_block_kernel(float* __restrict__ dst, int64_t rows, int64_t cols, int64_t dst_ld,
                                         int64_t gbase, int64_t gld, int64_t gcol0, uint64_t seed, float std) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    dst[r * dst_ld + c] = normal_at(seed, gbase + r * gld + gcol0 + c, std);
  }
}

__global__ void nonfinite_kernel(const float* __restrict__ x, int64_t n, int* flag) {
  bool bad = false;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    bad |= !isfinite(x[i]);
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicExch(flag, 1);
}

int grid_for(int64_t work, int threads) {
  const int64_t b = (work + threads - 1) / threads;
  const int64_t cap = 148 * 16;
  return static_cast<int>(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

int embed_gather(const float* E, const uint32_t* tok, float* x, int M, int D, int V, int* err, cudaStream_t s) {
  if (D % 4) return -1;
  embed_gather_kernel<<<(M * 32 + 255) / 256, 256, 0, s>>>(E, tok, x, M, D, V, err);
  return cudaGetLastError();
}
int embed_scatter(const float* dx, const int32_t* perm, const int32_t* seg_start, const uint32_t* seg_tok, int nseg,
                  float* dE, int D, cudaStream_t s) {
  if (D % 4) return -1;
  if (nseg == 0) return 0;
  embed_scatter_kernel<<<nseg, 256, 0, s>>>(dx, perm, seg_start, seg_tok, dE, D);
  return cudaGetLastError();
}
int rmsnorm_fwd(const float* x, const float* gamma, __nv_bfloat16* out, float* rms_inv, int M, int D, cudaStream_t s) {
  if (D % 4) return -1;
  // 128-thread blocks (4 rows): at 600M widths seven fit on an SM by registers, so 4096 rows
  // are one wave of 1024 blocks; 256-thread blocks fit three per SM and left a second, mostly
  // empty wave (1.15 waves: 10.4 us cold, DRAM 30% busy)
  constexpr int T = 128;
  const int grid = (M * 32 + T - 1) / T;
  switch (D % 128 == 0 ? D / 128 : 0) {
    case 6: rmsnorm_fwd_reg_kernel<6><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    case 8: rmsnorm_fwd_reg_kernel<8><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    case 10: rmsnorm_fwd_reg_kernel<10><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    case 12: rmsnorm_fwd_reg_kernel<12><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    case 14: rmsnorm_fwd_reg_kernel<14><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    case 16: rmsnorm_fwd_reg_kernel<16><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    case 18: rmsnorm_fwd_reg_kernel<18><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    case 20: rmsnorm_fwd_reg_kernel<20><<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
    default: rmsnorm_fwd_kernel<<<grid, T, 0, s>>>(x, gamma, out, rms_inv, M, D); break;
  }
  return cudaGetLastError();
}
int rmsnorm_bwd_blocks(int M) { return norm_ctas(M); }

template <int NV2, int STAGES>
int launch_norm_pipe(const float* dy, const float* x, const float* gamma, const float* rms_inv, const float* resid,
                     float* dx, __nv_bfloat16* dx_bf16, float bf16_scale, float* part, int M, int D, cudaStream_t s) {
  constexpr int smem = STAGES * 2 * kGroupRows * 64 * NV2 * 16;
  const cudaError_t attr = smem_limit_once(reinterpret_cast<const void*>(rmsnorm_bwd_pipe_kernel<NV2, STAGES>), smem);
  if (attr != cudaSuccess) return attr;
  rmsnorm_bwd_pipe_kernel<NV2, STAGES><<<norm_ctas(M), 256, smem, s>>>(dy, x, gamma, rms_inv, resid, dx, dx_bf16,
                                                                       bf16_scale, part, M, D);
  return cudaGetLastError();
}

int rmsnorm_bwd(const float* dy, const float* x, const float* gamma, const float* rms_inv, const float* resid,
                float* dx, __nv_bfloat16* dx_bf16, float bf16_scale, float* dgamma_part, int M, int D,
                cudaStream_t s) {
  if (D % 4) return -1;
  switch (D % 256 == 0 ? D / 256 : 0) {  // shared-memory stages of 32 D bytes: 4 up to D = 1536, then 3
    case 1: return launch_norm_pipe<1, 4>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    case 2: return launch_norm_pipe<2, 4>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    case 3: return launch_norm_pipe<3, 4>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    case 4: return launch_norm_pipe<4, 4>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    case 5: return launch_norm_pipe<5, 4>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    case 6: return launch_norm_pipe<6, 4>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    case 7: return launch_norm_pipe<7, 3>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    case 8: return launch_norm_pipe<8, 3>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale, dgamma_part, M, D, s);
    default: break;
  }
  // other widths: dgamma partials first (they read dy and x, which dx may alias), then the rows
  const int nb = norm_ctas(M);
  const int rpb = (M + nb - 1) / nb;
  dim3 g2((D + 255) / 256, nb);
  rmsnorm_dgamma_part_kernel<<<g2, 256, 0, s>>>(dy, x, rms_inv, dgamma_part, M, D, rpb);
  rmsnorm_bwd_rows_kernel<<<(M * 32 + 255) / 256, 256, 0, s>>>(dy, x, gamma, rms_inv, resid, dx, dx_bf16, bf16_scale,
                                                               M, D);
  return cudaGetLastError();
}
int dgamma_reduce(const float* part, int nblk, float* dgamma, int D, int accumulate, cudaStream_t s) {
  dgamma_reduce_kernel<<<(D + 31) / 32, 32 * kDgWarps, 0, s>>>(part, nblk, dgamma, D, accumulate, 0);
  return cudaGetLastError();
}
int dgamma_reduce_many(const float* part, int64_t part_stride, int nblk, float* dgamma, int D, int ngamma,
                       int accumulate, cudaStream_t s) {
  if (ngamma <= 0) return 0;
  dgamma_reduce_kernel<<<dim3((D + 31) / 32, ngamma), 32 * kDgWarps, 0, s>>>(part, nblk, dgamma, D, accumulate,
                                                                            part_stride);
  return cudaGetLastError();
}
int ce_forward(const float* logits, const uint32_t* tgt, float* row_loss, float* row_lse, int M, int V,
               float softcap, cudaStream_t s) {
  if (V % 4 || V > 4 * kCeThreads * kCeVec) return -1;
  ce_forward_kernel<<<M, kCeThreads, 0, s>>>(logits, tgt, row_loss, row_lse, V, softcap);
  return cudaGetLastError();
}
int ce_backward(const float* logits, const float* row_lse, const uint32_t* tgt, __nv_bfloat16* dl, int M, int V,
                float softcap, float scale, cudaStream_t s) {
  if (V % 4) return -1;
  ce_backward_kernel<<<M, kCeThreads, 0, s>>>(logits, row_lse, tgt, dl, V, softcap, scale);
  return cudaGetLastError();
}
int ce_fused(const float* logits, const uint32_t* tgt, float* row_loss, float* row_lse, __nv_bfloat16* dl, int M,
             int V, float softcap, float scale, cudaStream_t s) {
  if (V % 4 != 0 || V > 4 * kCeVec * kCeThreads) return -1;
  ce_fused_kernel<<<M, kCeThreads, 0, s>>>(logits, tgt, row_loss, row_lse, dl, V, softcap, scale);
  return cudaGetLastError();
}
int mean_reduce(const float* row_loss, int M, float* out, cudaStream_t s) {
  mean_reduce_kernel<<<1, 1024, 0, s>>>(row_loss, M, out);
  return cudaGetLastError();
}
int sumsq_partials_count() { return kNormBlocks; }
int sumsq_seg_blocks() { return kSegNormBlocks; }
int sumsq_partials(const float* x, int64_t n, float* partials, cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(x) & 15) return -1;
  sumsq_partial_kernel<<<kSegNormBlocks, kNormThreads, 0, s>>>(x, n, partials);
  return cudaGetLastError();
}
int sumsq_fold(const float* in, int n, float* out, int nout, cudaStream_t s) {
  sumsq_fold_kernel<<<1, 256, 0, s>>>(in, n, out, nout);
  return cudaGetLastError();
}
int sumsq_finish(const float* partials, int n, float* out_norm, cudaStream_t s) {
  sumsq_final_kernel<<<1, 1024, 0, s>>>(partials, n, out_norm, nullptr);
  return cudaGetLastError();
}
int sumsq_finish_sq(const float* partials, int n, double* out_sq, cudaStream_t s) {
  sumsq_final_kernel<<<1, 1024, 0, s>>>(partials, n, nullptr, out_sq);
  return cudaGetLastError();
}
int sqrt_to_float(const double* sq, float* out, cudaStream_t s) {
  sqrt_to_float_kernel<<<1, 1, 0, s>>>(sq, out);
  return cudaGetLastError();
}
int sumsq_norm(const float* x, int64_t n, float* partials, float* out_norm, cudaStream_t s) {
  sumsq_partial_kernel<<<kNormBlocks, kNormThreads, 0, s>>>(x, n, partials);
  sumsq_final_kernel<<<1, 1024, 0, s>>>(partials, kNormBlocks, out_norm, nullptr);
  return cudaGetLastError();
}
int adam_step(const AdamArgs& a, cudaStream_t s) {
  AdamKParams k;
  if (a.nseg < 0 || a.nseg > kMaxAdamSegments) return -1;
  for (int i = 0; i < a.nseg; ++i) k.seg[i] = a.seg[i];
  k.nseg = a.nseg;
  int64_t total = 0;
  for (int i = 0; i < a.nseg; ++i) {
    if (a.seg[i].begin % 4 || a.seg[i].end % 4) return -1;
    total += a.seg[i].end - a.seg[i].begin;
  }
  k.beta1 = a.beta1;
  k.beta2 = a.beta2;
  k.eps = a.eps;
  k.bc1 = a.bc1;
  k.bc2 = a.bc2;
  k.grad_scale = a.grad_scale;
  k.gsc = a.gsc;
  k.clip = a.clip;
  adam_kernel<<<grid_for(total / 4, 256), 256, 0, s>>>(a.param, a.grad, a.m, a.v, a.param_bf16, a.norm, k);
  return cudaGetLastError();
}
int cast_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t s) {
  return cast_bf16_scaled(src, dst, n, 1.0f, s);
}
int cast_bf16_scaled(const float* src, __nv_bfloat16* dst, int64_t n, float scale, cudaStream_t s) {
  if (n % 4) return -1;
  cast_bf16_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(src, dst, n / 4, scale);
  return cudaGetLastError();
}
int fill_f32(float* dst, int64_t n, float value, cudaStream_t s) {
  fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, n, value);
  return cudaGetLastError();
}
int init_normal(float* dst, int64_t n, uint64_t seed, float std, cudaStream_t s) {
  init_normal_kernel<<<grid_for((n + 1) / 2, 256), 256, 0, s>>>(dst, n, seed, std);
  return cudaGetLastError();
}
int scale_f32(const float* x, float* y, int64_t n, float a, cudaStream_t s) {
  scale_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, y, n, a);
  return cudaGetLastError();
}
int residual_rmsnorm_fwd(const float* x, const __nv_bfloat16* p, float alpha, const float* gamma, float* x_out,
                         __nv_bfloat16* xn, float* rms_inv, int M, int D, cudaStream_t s) {
  if (D % 4) return -1;
  residual_rmsnorm_kernel<<<(M * 32 + 255) / 256, 256, 0, s>>>(x, p, alpha, gamma, x_out, xn, rms_inv, M, D);
  return cudaGetLastError();
}
int init_normal_block(float* dst, int64_t rows, int64_t cols, int64_t dst_ld, int64_t gbase, int64_t gld,
                      int64_t gcol0, uint64_t seed, float std, cudaStream_t s) {
  init_normal_block_kernel<<<grid_for(rows * cols, 256), 256, 0, s>>>(dst, rows, cols, dst_ld, gbase, gld, gcol0,
                                                                      seed, std);
  return cudaGetLastError();
}
int nonfinite_check(const float* x, int64_t n, int* flag, cudaStream_t s) {
  nonfinite_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, flag);
  return cudaGetLastError();
}

}  // namespace rt
