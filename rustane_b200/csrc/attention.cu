// Causal scaled-dot-product attention, head_dim 128, flash-style (S x S never
// materialised), bf16 operands with fp32 accumulation and fp32 softmax.
//
// Semantics follow the reference sdpaFwd / sdpaBwd1 / sdpaBwd2 graphs
// (crates/engine/src/kernels/sdpa_fwd.rs:130-150, sdpa_bwd.rs:44-162):
//   S = Q K^T / sqrt(hd) + causal mask, P = softmax(S), O = P V
//   dV = P^T dO, dP = dO V^T, dS = P * (dP - rowsum(P * dP)) / sqrt(hd),
//   dQ = dS K, dK = dS^T Q,
// followed by the RoPE backward rotation of dQ and dK (layer.rs:1880-1897),
// which is fused into the dQ / dK epilogues here.  rowsum(P * dP) is computed
// as rowsum(dO * O), which is the same quantity.
//
// Data layout (token-major): qkv [M, 3D] bf16 with head h of Q, K, V at columns
// h*128, D + h*128, 2D + h*128; O [M, D]; dqkv [M, 3D] (same column layout).
// The softmax statistic is kept in the log2 domain: lse2 = max + log2(sum).
//
// The backward's matrix products use mma.sync m16n8k16 (bf16 -> fp32) fed by
// ldmatrix from 128-byte-swizzled shared-memory tiles filled with cp.async; the
// forward runs on tcgen05 / TMEM (attention_tc.cu).
#include "attention.h"
#include "common.cuh"

namespace rt {
namespace {

constexpr int HD = 128;
constexpr int ROW_BYTES = HD * 2;  // 256 B per tile row, 16 chunks of 16 B

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// byte offset of 16-B chunk c of row r in a swizzled [rows][128] bf16 tile
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * ROW_BYTES + ((c ^ (r & 7)) << 4));
}

// Copy rows [0, ROWS) x 128 bf16 (row stride ld elements) into a swizzled tile.
template <int ROWS, int NT>
__device__ __forceinline__ void load_tile(uint8_t* tile, const __nv_bfloat16* src, int64_t ld, int tid) {
#pragma unroll
  for (int i = 0; i < ROWS * 16 / NT; ++i) {
    const int idx = tid + i * NT;
    const int r = idx >> 4, c = idx & 15;
    cp_async16(tile + swz(r, c), src + static_cast<int64_t>(r) * ld + c * 8);
  }
}
// Store a swizzled tile to global memory rows (16-B stores).
template <int ROWS, int NT>
__device__ __forceinline__ void store_tile(const uint8_t* tile, __nv_bfloat16* dst, int64_t ld, int tid) {
#pragma unroll
  for (int i = 0; i < ROWS * 16 / NT; ++i) {
    const int idx = tid + i * NT;
    const int r = idx >> 4, c = idx & 15;
    *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(r) * ld + c * 8) =
        *reinterpret_cast<const uint4*>(tile + swz(r, c));
  }
}

// A fragment (16 rows x 16 k) from a row-major swizzled tile: rows r0.., k chunk pair kc.
__device__ __forceinline__ void lds_a(uint32_t (&a)[4], uint32_t tile, int r0, int kk, int lane) {
  const int r = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = 2 * kk + (lane >> 4);
  ldsm_x4(a, tile + swz(r, c));
}
// B fragments for two n8 tiles (rows n0..n0+15 of the stored tile are the n index,
// the 128 columns are k): b[0],b[1] -> tile n0, b[2],b[3] -> tile n0+8.
__device__ __forceinline__ void lds_b_nk(uint32_t (&b)[4], uint32_t tile, int n0, int kk, int lane) {
  const int r = n0 + (lane & 7) + (lane >> 4) * 8;
  const int c = 2 * kk + ((lane >> 3) & 1);
  ldsm_x4(b, tile + swz(r, c));
}
// B fragments for two n8 tiles where the stored tile rows are the k index and the
// 128 columns are n: k rows k0..k0+15, n columns 16*np .. 16*np+15.
__device__ __forceinline__ void lds_b_kn(uint32_t (&b)[4], uint32_t tile, int k0, int np, int lane) {
  const int r = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = 2 * np + (lane >> 4);
  ldsm_x4_t(b, tile + swz(r, c));
}

// Write one warp's 16 x 128 fp32 accumulator (fragment layout) into a swizzled bf16 tile.
__device__ __forceinline__ void frag_to_tile(uint8_t* tile, int r0, const float (&acc)[16][4], int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int ra = r0 + g, rb = r0 + g + 8;
    *reinterpret_cast<uint32_t*>(tile + swz(ra, nt) + 4 * t) = pack_bf16x2(acc[nt][0], acc[nt][1]);
    *reinterpret_cast<uint32_t*>(tile + swz(rb, nt) + 4 * t) = pack_bf16x2(acc[nt][2], acc[nt][3]);
  }
}

// RoPE backward on an accumulator row pair: cols (2i, 2i+1) of head_dim with
// cos/sin table laid out [hd/2][seq] (layer.rs:197-217, 1880-1897).
__device__ __forceinline__ void rope_bwd_frag(float (&acc)[16][4], int pos_a, int pos_b, const float* cosb,
                                              const float* sinb, int S, int lane) {
  const int t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int i = nt * 4 + t;  // pair index (cols nt*8 + 2t, +1)
    const float ca = cosb[i * S + pos_a], sa = sinb[i * S + pos_a];
    const float cb = cosb[i * S + pos_b], sb = sinb[i * S + pos_b];
    const float d0 = acc[nt][0], d1 = acc[nt][1];
    acc[nt][0] = ca * d0 + sa * d1;
    acc[nt][1] = -sa * d0 + ca * d1;
    const float e0 = acc[nt][2], e1 = acc[nt][3];
    acc[nt][2] = cb * e0 + sb * e1;
    acc[nt][3] = -sb * e0 + cb * e1;
  }
}

// ------------------------------------------------------ backward: prepare
// Dv[b, h, s] = sum_e dO[s, h*128 + e] * O[s, h*128 + e]: 16 lanes per (token,
// head), 8 elements (16 B) each, two (token, head) pairs per warp.
__global__ void attn_bwd_dot_kernel(const __nv_bfloat16* __restrict__ O, int64_t ldo,
                                    const __nv_bfloat16* __restrict__ dO, int64_t lddo, float* __restrict__ Dv,
                                    int M, int S, int nh) {
  const int gid = (blockIdx.x * blockDim.x + threadIdx.x) >> 4;  // (token, head) index
  const int l16 = threadIdx.x & 15;
  const bool live = gid < M * nh;
  const int m = live ? gid / nh : 0, h = live ? gid % nh : 0;
  float s = 0.f;
  if (live) {
    const uint4 o = __ldg(reinterpret_cast<const uint4*>(O + static_cast<int64_t>(m) * ldo + h * HD) + l16);
    const uint4 d = __ldg(reinterpret_cast<const uint4*>(dO + static_cast<int64_t>(m) * lddo + h * HD) + l16);
    s = bf16lo(o.x) * bf16lo(d.x) + bf16hi(o.x) * bf16hi(d.x) + bf16lo(o.y) * bf16lo(d.y) +
        bf16hi(o.y) * bf16hi(d.y) + bf16lo(o.z) * bf16lo(d.z) + bf16hi(o.z) * bf16hi(d.z) +
        bf16lo(o.w) * bf16lo(d.w) + bf16hi(o.w) * bf16hi(d.w);
  }
#pragma unroll
  for (int off = 8; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (live && l16 == 0) {
    const int b = m / S, pos = m % S;
    Dv[(static_cast<int64_t>(b) * nh + h) * S + pos] = s;
  }
}

// ------------------------------------------------------ backward: dK, dV
// grid (S/64, heads, batch), 128 threads: warp w owns keys kv0 + 16w .. +15.
constexpr int BWD_B = 64, BWD_NT = 128;
constexpr int BWD_SMEM = 6 * BWD_B * ROW_BYTES + 4 * BWD_B * 4;  // K, V, 2x(Q, dO), 2x(lse, Dv)

__global__ void __launch_bounds__(BWD_NT, 2)
    attn_bwd_dkdv_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ldq, int D,
                         const __nv_bfloat16* __restrict__ dO, int64_t lddo, const float* __restrict__ lse2,
                         const float* __restrict__ Dv, __nv_bfloat16* __restrict__ dqkv, int64_t lddq, int S, int nh,
                         float scale, float scale_log2, const float* __restrict__ rope_cos_b,
                         const float* __restrict__ rope_sin_b) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sK = smem;
  uint8_t* sV = sK + BWD_B * ROW_BYTES;
  uint8_t* sQ = sV + BWD_B * ROW_BYTES;    // [2]
  uint8_t* sdO = sQ + 2 * BWD_B * ROW_BYTES;  // [2]
  float* sL = reinterpret_cast<float*>(sdO + 2 * BWD_B * ROW_BYTES);  // [2][64]
  float* sD = sL + 2 * BWD_B;                                          // [2][64]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int kb = blockIdx.z, h = blockIdx.x, b = blockIdx.y;  // key block 0 has the most work: dispatched first
  const int kv0 = kb * BWD_B;
  const int64_t tok0 = static_cast<int64_t>(b) * S;
  const int64_t stat0 = (static_cast<int64_t>(b) * nh + h) * S;
  const __nv_bfloat16* gQ = qkv + tok0 * ldq + h * HD;
  const __nv_bfloat16* gK = qkv + (tok0 + kv0) * ldq + D + h * HD;
  const __nv_bfloat16* gV = qkv + (tok0 + kv0) * ldq + 2 * D + h * HD;
  const __nv_bfloat16* gdO = dO + tok0 * lddo + h * HD;

  const int nqb = S / BWD_B;
  const int i0 = kb;  // first query block touching these keys
  load_tile<BWD_B, BWD_NT>(sK, gK, ldq, tid);
  load_tile<BWD_B, BWD_NT>(sV, gV, ldq, tid);
  auto load_q = [&](int i, int buf) {
    load_tile<BWD_B, BWD_NT>(sQ + buf * BWD_B * ROW_BYTES, gQ + static_cast<int64_t>(i) * BWD_B * ldq, ldq, tid);
    load_tile<BWD_B, BWD_NT>(sdO + buf * BWD_B * ROW_BYTES, gdO + static_cast<int64_t>(i) * BWD_B * lddo, lddo, tid);
    if (tid < BWD_B / 4) {
      cp_async16(sL + buf * BWD_B + tid * 4, lse2 + stat0 + i * BWD_B + tid * 4);
    } else if (tid < BWD_B / 2) {
      const int u = tid - BWD_B / 4;
      cp_async16(sD + buf * BWD_B + u * 4, Dv + stat0 + i * BWD_B + u * 4);
    }
  };
  load_q(i0, 0);
  cp_async_commit();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  const int r0 = warp * 16;
  const int ka = kv0 + r0 + g, kbr = ka + 8;  // key positions of this thread's rows
  const uint32_t kt = smem_u32(sK), vt = smem_u32(sV);

  for (int i = i0; i < nqb; ++i) {
    const int buf = (i - i0) & 1;
    if (i + 1 < nqb) {
      load_q(i + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int q0 = i * BWD_B;
    const uint32_t qt = smem_u32(sQ + buf * BWD_B * ROW_BYTES);
    const uint32_t dot = smem_u32(sdO + buf * BWD_B * ROW_BYTES);
    const float* L = sL + buf * BWD_B;
    const float* Dd = sD + buf * BWD_B;
    // S^T = K Q^T and dP^T = V dO^T (rows = keys, cols = queries)
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int x = 0; x < 8; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) st[x][y] = dpt[x][y] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t ak[4], av[4];
      lds_a(ak, kt, r0, kk, lane);
      lds_a(av, vt, r0, kk, lane);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bq[4], bo[4];
        lds_b_nk(bq, qt, np * 16, kk, lane);
        lds_b_nk(bo, dot, np * 16, kk, lane);
        mma16816(st[2 * np], ak, bq[0], bq[1]);
        mma16816(st[2 * np + 1], ak, bq[2], bq[3]);
        mma16816(dpt[2 * np], av, bo[0], bo[1]);
        mma16816(dpt[2 * np + 1], av, bo[2], bo[3]);
      }
    }
    // P^T and dS^T
    uint32_t pa[8][2], sa[8][2];
    const bool diag = q0 < kv0 + r0 + 16;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float p[4], d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = nt * 8 + 2 * t + (e & 1);
        const int key = (e < 2) ? ka : kbr;
        float pe = exp2f(st[nt][e] * scale_log2 - L[ql]);
        if (diag && q0 + ql < key) pe = 0.f;
        p[e] = pe;
        d[e] = pe * (dpt[nt][e] - Dd[ql]);
      }
      pa[nt][0] = pack_bf16x2(p[0], p[1]);
      pa[nt][1] = pack_bf16x2(p[2], p[3]);
      sa[nt][0] = pack_bf16x2(d[0], d[1]);
      sa[nt][1] = pack_bf16x2(d[2], d[3]);
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t ap[4] = {pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1]};
      const uint32_t as[4] = {sa[2 * kk][0], sa[2 * kk][1], sa[2 * kk + 1][0], sa[2 * kk + 1][1]};
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t bo[4], bq[4];
        lds_b_kn(bo, dot, kk * 16, np, lane);
        lds_b_kn(bq, qt, kk * 16, np, lane);
        mma16816(dv[2 * np], ap, bo[0], bo[1]);
        mma16816(dv[2 * np + 1], ap, bo[2], bo[3]);
        mma16816(dk[2 * np], as, bq[0], bq[1]);
        mma16816(dk[2 * np + 1], as, bq[2], bq[3]);
      }
    }
    __syncthreads();
  }
  // epilogue: dK = scale * dS^T Q, RoPE backward; dV as is.
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[nt][e] *= scale;
  rope_bwd_frag(dk, ka, kbr, rope_cos_b, rope_sin_b, S, lane);
  frag_to_tile(sQ, r0, dk, lane);
  frag_to_tile(sdO, r0, dv, lane);
  __syncthreads();
  store_tile<BWD_B, BWD_NT>(sQ, dqkv + (tok0 + kv0) * lddq + D + h * HD, lddq, tid);
  store_tile<BWD_B, BWD_NT>(sdO, dqkv + (tok0 + kv0) * lddq + 2 * D + h * HD, lddq, tid);
}

// ---------------------------------------------------------- backward: dQ
// grid (S/64, heads, batch), 128 threads: warp w owns queries q0 + 16w .. +15.
__global__ void __launch_bounds__(BWD_NT, 2)
    attn_bwd_dq_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ldq, int D,
                       const __nv_bfloat16* __restrict__ dO, int64_t lddo, const float* __restrict__ lse2,
                       const float* __restrict__ Dv, __nv_bfloat16* __restrict__ dqkv, int64_t lddq, int S, int nh,
                       float scale, float scale_log2, const float* __restrict__ rope_cos_b,
                       const float* __restrict__ rope_sin_b) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + BWD_B * ROW_BYTES;
  uint8_t* sK = sdO + BWD_B * ROW_BYTES;  // [2]
  uint8_t* sV = sK + 2 * BWD_B * ROW_BYTES;  // [2]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int qb = gridDim.z - 1 - blockIdx.z;  // heaviest first, over all heads and sequences
  const int h = blockIdx.x, b = blockIdx.y;
  const int q0 = qb * BWD_B;
  const int64_t tok0 = static_cast<int64_t>(b) * S;
  const int64_t stat0 = (static_cast<int64_t>(b) * nh + h) * S;
  const __nv_bfloat16* gK = qkv + tok0 * ldq + D + h * HD;
  const __nv_bfloat16* gV = qkv + tok0 * ldq + 2 * D + h * HD;
  load_tile<BWD_B, BWD_NT>(sQ, qkv + (tok0 + q0) * ldq + h * HD, ldq, tid);
  load_tile<BWD_B, BWD_NT>(sdO, dO + (tok0 + q0) * lddo + h * HD, lddo, tid);
  load_tile<BWD_B, BWD_NT>(sK, gK, ldq, tid);
  load_tile<BWD_B, BWD_NT>(sV, gV, ldq, tid);
  cp_async_commit();

  const int r0 = warp * 16;
  const int qa = q0 + r0 + g, qbr = qa + 8;
  const float la = lse2[stat0 + qa], lb = lse2[stat0 + qbr];
  const float da = Dv[stat0 + qa], db = Dv[stat0 + qbr];
  float dq[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  const uint32_t qt = smem_u32(sQ), dot = smem_u32(sdO);
  const int nkb = qb + 1;
  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile<BWD_B, BWD_NT>(sK + (buf ^ 1) * BWD_B * ROW_BYTES, gK + static_cast<int64_t>(j + 1) * BWD_B * ldq,
                               ldq, tid);
      load_tile<BWD_B, BWD_NT>(sV + (buf ^ 1) * BWD_B * ROW_BYTES, gV + static_cast<int64_t>(j + 1) * BWD_B * ldq,
                               ldq, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int key0 = j * BWD_B;
    const uint32_t kt = smem_u32(sK + buf * BWD_B * ROW_BYTES);
    const uint32_t vt = smem_u32(sV + buf * BWD_B * ROW_BYTES);
    float s[8][4], dp[8][4];
#pragma unroll
    for (int x = 0; x < 8; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) s[x][y] = dp[x][y] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t aq[4], ao[4];
      lds_a(aq, qt, r0, kk, lane);
      lds_a(ao, dot, r0, kk, lane);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bk[4], bv[4];
        lds_b_nk(bk, kt, np * 16, kk, lane);
        lds_b_nk(bv, vt, np * 16, kk, lane);
        mma16816(s[2 * np], aq, bk[0], bk[1]);
        mma16816(s[2 * np + 1], aq, bk[2], bk[3]);
        mma16816(dp[2 * np], ao, bv[0], bv[1]);
        mma16816(dp[2 * np + 1], ao, bv[2], bv[3]);
      }
    }
    uint32_t sa[8][2];
    const bool diag = key0 + BWD_B - 1 > q0 + r0;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + nt * 8 + 2 * t + (e & 1);
        const bool hi = e >= 2;
        float p = exp2f(s[nt][e] * scale_log2 - (hi ? lb : la));
        if (diag && key > (hi ? qbr : qa)) p = 0.f;
        d[e] = p * (dp[nt][e] - (hi ? db : da));
      }
      sa[nt][0] = pack_bf16x2(d[0], d[1]);
      sa[nt][1] = pack_bf16x2(d[2], d[3]);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t as[4] = {sa[2 * kk][0], sa[2 * kk][1], sa[2 * kk + 1][0], sa[2 * kk + 1][1]};
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t bk[4];
        lds_b_kn(bk, kt, kk * 16, np, lane);
        mma16816(dq[2 * np], as, bk[0], bk[1]);
        mma16816(dq[2 * np + 1], as, bk[2], bk[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) dq[nt][e] *= scale;
  rope_bwd_frag(dq, qa, qbr, rope_cos_b, rope_sin_b, S, lane);
  frag_to_tile(sQ, r0, dq, lane);
  __syncthreads();
  store_tile<BWD_B, BWD_NT>(sQ, dqkv + (tok0 + q0) * lddq + h * HD, lddq, tid);
}

}  // namespace

int attn_bwd_rowsum(const AttnArgs& a, cudaStream_t s) {
  if (a.ldo % 8 != 0 || a.lddo % 8 != 0) return -1;
  const int M = a.batch * a.S;
  const int64_t threads = static_cast<int64_t>(M) * a.heads * 16;
  attn_bwd_dot_kernel<<<static_cast<int>((threads + 255) / 256), 256, 0, s>>>(a.out, a.ldo, a.dout, a.lddo, a.dvec, M,
                                                                              a.S, a.heads);
  return cudaGetLastError();
}

int attn_backward(const AttnArgs& a, cudaStream_t s) {
  if (a.S % 128 != 0 || a.hd != HD || a.D != a.heads * HD) return -1;
  cudaError_t attr = smem_limit_once(reinterpret_cast<const void*>(attn_bwd_dkdv_kernel), BWD_SMEM);
  if (attr == cudaSuccess) attr = smem_limit_once(reinterpret_cast<const void*>(attn_bwd_dq_kernel), BWD_SMEM);
  if (attr != cudaSuccess) return attr;
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  const float scale_log2 = scale * 1.4426950408889634f;
  const int rc = attn_bwd_rowsum(a, s);
  if (rc) return rc;
  dim3 grid(a.heads, a.batch, a.S / BWD_B);
  attn_bwd_dkdv_kernel<<<grid, BWD_NT, BWD_SMEM, s>>>(a.qkv, a.ldq, a.D, a.dout, a.lddo, a.lse2, a.dvec, a.dqkv,
                                                      a.lddq, a.S, a.heads, scale, scale_log2, a.rope_cos_b,
                                                      a.rope_sin_b);
  attn_bwd_dq_kernel<<<grid, BWD_NT, BWD_SMEM, s>>>(a.qkv, a.ldq, a.D, a.dout, a.lddo, a.lse2, a.dvec, a.dqkv, a.lddq,
                                                    a.S, a.heads, scale, scale_log2, a.rope_cos_b, a.rope_sin_b);
  return cudaGetLastError();
}

}  // namespace rt
