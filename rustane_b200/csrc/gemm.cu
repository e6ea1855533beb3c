// tcgen05 / TMEM / TMA GEMM for sm_100a with the LM step's fused epilogues.
//
// C[M,N] = sum_k A[m,k] * B[n,k], bf16 operands, fp32 accumulation in TMEM.
// Either operand may be K-major ([rows][K]) or MN-major ([K][rows]); the
// major-ness is a bit of the tcgen05 instruction descriptor plus a different
// shared-memory descriptor, so the weights are kept once, in the reference's
// [D_in, D_out] layout (crates/engine/src/layer.rs:16-26), and used as
//   forward      y  = x  * W    : B MN-major
//   backward     dx = dy * W^T  : B K-major
//   weight grad  dW = x^T * dy  : A and B MN-major (contract over tokens)
// without any transposed copy.
//
// Kernel organisation (one CTA per SM, persistent over output tiles):
//   warp 0      : TMA producer (one lane) -> STAGES-deep smem ring
//   warp 1      : MMA issuer  (one lane)  -> tcgen05.mma, 128 x BN x 16 per instruction
//   warp 2      : TMEM allocator (2 accumulator buffers of BN fp32 columns)
//   warps 4..11 : epilogue; warp w reads TMEM lanes 32*(w%4).. (accumulator rows)
//                 and one half of the tile's 32-column chunks, prefetching the
//                 next chunk's auxiliary input (residual, h1|h3, old gradient)
// The epilogue of tile i overlaps the MMAs of tile i+1.  Tile widths BN = 128,
// 192 or 256 are chosen per shape from a wave-count cost model.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace rt {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 B = one swizzle row

constexpr int kEpiWarps = 8;                    // warps 4..11: two per TMEM lane quadrant
constexpr int kRasterGroup = 16;                // M-tiles (of 128 rows) per raster band
constexpr int kThreads = 128 + 32 * kEpiWarps;  // + producer, MMA, allocator, spare

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  // One 64-deep k-block per stage: with 48 KB per k-block at BN = 256, stages
  // of two k-blocks leave only two stages, which measured 10-12% slower here
  // (the CTA-pair kernel, at 32 KB per k-block and SM, does use two).
  static constexpr int KPS = 1;  // k-blocks per stage
  static constexpr int SUB_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = KPS * SUB_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 192 ? 4 : 6);
  static constexpr int ACC_STRIDE = (BN == 192) ? 256 : BN;  // TMEM columns per accumulator buffer
  static constexpr int TMEM_COLS = 2 * ACC_STRIDE;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;       // epilogue transpose buffers
  static constexpr int BAR_OFF = EPI_OFF + kEpiWarps * 32 * 128;
  static constexpr int SMEM_BYTES = BAR_OFF + 1024 + 256;
};

struct KParams {
  int M, N, num_kb;
  int num_m, num_n, num_tiles;
  int n_half;
  int beta;
  float alpha;
  int seq, rope_cols;
  void* out;
  int64_t ldo;
  void* out2;
  int64_t ldo2;
  const void* aux;
  int64_t ld_aux;
  const float* rope_cos;
  const float* rope_sin;
  int* err;
  float* sumsq;  // kEpiF32Acc: per-warp sums of squares of the output (nullptr: none)
  int sumsq_slots;
};

// Tile order: groups of `group` M-tiles; inside a group M runs fastest, then N.
// The CTAs resident at one time then share a band of A rows and a few B column
// tiles, so operands larger than L2 are read from HBM about once instead of
// once per N tile (with M running fastest over all of M, every wave would
// stream all of A).  With num_m <= group this is plain M-fastest order.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group, int& tm, int& tn) {
  const int band = tile / (group * num_n);
  const int m_first = band * group;
  const int gm = min(num_m - m_first, group);
  const int r = tile - band * group * num_n;
  tm = m_first + r % gm;
  tn = r / gm;
}

// sigmoid by the SFU exponential and the fast (approximate, ~2 ulp) division: the
// epilogue's results are rounded to bf16, so the IEEE division's extra work buys nothing
__device__ __forceinline__ float silu_sigmoid(float x, float& sig) {
  sig = __fdividef(1.f, 1.f + __expf(-x));
  return x * sig;
}

// ------------------------------------------------------------------ epilogue
// TMEM gives each epilogue lane one accumulator row.  Writing rows straight to
// global memory makes every warp access touch 32 different lines with 16 bytes
// each; instead each 32 x 32 chunk is transposed through a 4 KB per-warp
// shared-memory buffer (16-byte units XOR-swizzled by row, conflict-free both
// ways) into the coalesced layout: lane l holds rows 4i + (l >> 3), i = 0..7,
// columns 4 (l & 7) .. 4 (l & 7) + 3 of the chunk, so one warp access covers
// four whole rows of the chunk.  Auxiliary inputs are loaded in the same layout.
constexpr int kEpiBufBytes = 32 * 128;  // per epilogue warp

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ float4 lds128(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Row of the chunk held in slot i by this lane, and the lane's first column.
__device__ __forceinline__ int crow(int i, int lane) { return 4 * i + (lane >> 3); }
__device__ __forceinline__ int ccol(int lane) { return 4 * (lane & 7); }

// TMEM chunk (32 lanes x 32 columns at taddr) -> coalesced layout w[8].
__device__ __forceinline__ void tmem_chunk_coalesced(uint32_t taddr, uint32_t wbuf, int lane, float4 (&w)[8]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_ld_wait();
  const uint32_t row = wbuf + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) sts128(row + ((j ^ (lane & 7)) << 4), r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = crow(i, lane);
    w[i] = lds128(wbuf + rr * 128 + (((lane & 7) ^ (rr & 7)) << 4));
  }
  __syncwarp();  // the buffer is rewritten by the next chunk
}

__device__ __forceinline__ uint2 pack_bf16x4(float4 v) { return make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w)); }
__device__ __forceinline__ float4 unpack_bf16x4(uint32_t lo, uint32_t hi) {
  return make_float4(bf16lo(lo), bf16hi(lo), bf16lo(hi), bf16hi(hi));
}

// Per-chunk auxiliary inputs in the coalesced layout (loaded one chunk ahead
// so their latency overlaps the previous chunk's work).  fp32 aux: u[i] is a
// float4; SwiGLU backward: u[i].xy = 4 bf16 of h1, u[i].zw = 4 bf16 of h3;
// RoPE: u[i].xy = cos, u[i].zw = sin of the lane's two column pairs.
struct AuxRegs {
  uint4 u[8];
};

template <int EPI>
__device__ __forceinline__ void load_aux(const KParams& p, int mbase, int n, int lane, AuxRegs& a) {
  if (n >= p.N) return;
  const int col = n + ccol(lane);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = mbase + crow(i, lane);
    if (m >= p.M) continue;
    const int64_t mr = m;
    if constexpr (EPI == kEpiResidual) {
      a.u[i] = *reinterpret_cast<const uint4*>(static_cast<const float*>(p.aux) + mr * p.ld_aux + col);
    } else if constexpr (EPI == kEpiSwigluBwd) {
      const __nv_bfloat16* h13 = static_cast<const __nv_bfloat16*>(p.aux) + mr * p.ld_aux;
      const uint2 h1 = *reinterpret_cast<const uint2*>(h13 + col);
      const uint2 h3 = *reinterpret_cast<const uint2*>(h13 + p.n_half + col);
      a.u[i] = make_uint4(h1.x, h1.y, h3.x, h3.y);
    } else if constexpr (EPI == kEpiBf16RowDot) {
      const uint2 o = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.aux) + mr * p.ld_aux + col);
      a.u[i] = make_uint4(o.x, o.y, 0u, 0u);
    } else if constexpr (EPI == kEpiF32Acc) {
      if (p.beta) a.u[i] = *reinterpret_cast<const uint4*>(static_cast<const float*>(p.out) + mr * p.ldo + col);
    } else if constexpr (EPI == kEpiRope) {
      if (col < p.rope_cols) {
        const int pos = static_cast<int>(mr % p.seq);
        const int ip = (col & 127) >> 1;
        const uint2 c2 = *reinterpret_cast<const uint2*>(p.rope_cos + pos * 64 + ip);
        const uint2 s2 = *reinterpret_cast<const uint2*>(p.rope_sin + pos * 64 + ip);
        a.u[i] = make_uint4(c2.x, c2.y, s2.x, s2.y);
      }
    }
  }
}

// One 32 x 32 chunk of the epilogue in the coalesced layout: w[i] holds the fp32
// accumulators of row mbase + crow(i), columns n + ccol .. n + ccol + 3.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const KParams& p, int mbase, int n, int lane, float4 (&w)[8],
                                               const AuxRegs& a, float& ss) {
  const int col = n + ccol(lane);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = mbase + crow(i, lane);
    if (m >= p.M) continue;
    const int64_t mr = m;
    float4 v = w[i];
    if constexpr (EPI == kEpiBf16) {
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + mr * p.ldo + col) = pack_bf16x4(v);
    } else if constexpr (EPI == kEpiF32 || EPI == kEpiF32Acc || EPI == kEpiResidual) {
      if constexpr (EPI == kEpiF32Acc) {
        if (p.beta) {
          const float4 o = *reinterpret_cast<const float4*>(&a.u[i]);
          v.x += o.x;
          v.y += o.y;
          v.z += o.z;
          v.w += o.w;
        }
      }
      if constexpr (EPI == kEpiResidual) {
        const float4 o = *reinterpret_cast<const float4*>(&a.u[i]);
        v.x = o.x + p.alpha * v.x;
        v.y = o.y + p.alpha * v.y;
        v.z = o.z + p.alpha * v.z;
        v.w = o.w + p.alpha * v.w;
      }
      if constexpr (EPI == kEpiF32Acc) ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
      *reinterpret_cast<float4*>(static_cast<float*>(p.out) + mr * p.ldo + col) = v;
    } else if constexpr (EPI == kEpiRope) {
      // Interleaved-pair rotation per head of 128 (kernels/sdpa_fwd.rs:18-33, 100-128):
      //   y[2i] = x[2i] cos - x[2i+1] sin,  y[2i+1] = x[2i+1] cos + x[2i] sin
      if (col < p.rope_cols) {
        const float c0 = __uint_as_float(a.u[i].x), c1 = __uint_as_float(a.u[i].y);
        const float s0 = __uint_as_float(a.u[i].z), s1 = __uint_as_float(a.u[i].w);
        const float x0 = v.x, x1 = v.y, x2 = v.z, x3 = v.w;
        v.x = x0 * c0 - x1 * s0;
        v.y = x1 * c0 + x0 * s0;
        v.z = x2 * c1 - x3 * s1;
        v.w = x3 * c1 + x2 * s1;
      }
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + mr * p.ldo + col) = pack_bf16x4(v);
    } else if constexpr (EPI == kEpiSwigluBwd) {
      // C = dgate = dffn * W2 (layer.rs:1627-1641); SiLU-gate backward
      // (layer.rs:1660-1666): dh3 = dg * silu(h1); dh1 = dg * h3 * sig * (1 + h1 (1 - sig)),
      // sig = 1 / (1 + 2^(-h1 log2 e)) on the SFU, the rest in fp32 pairs (one instruction
      // per two elements): the epilogue, not the MMAs, bounds this GEMM.
      const float4 h1 = unpack_bf16x4(a.u[i].x, a.u[i].y);
      const float4 h3 = unpack_bf16x4(a.u[i].z, a.u[i].w);
      const uint64_t one2 = f2_pack(1.f, 1.f);
      const uint64_t nl2 = f2_pack(-1.4426950408889634f, -1.4426950408889634f);
      uint32_t o1[2], o3[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint64_t x2 = e ? f2_pack(h1.z, h1.w) : f2_pack(h1.x, h1.y);
        const uint64_t g2 = e ? f2_pack(v.z, v.w) : f2_pack(v.x, v.y);
        const uint64_t y2 = e ? f2_pack(h3.z, h3.w) : f2_pack(h3.x, h3.y);
        float ta, tb;
        f2_unpack(f2_mul(x2, nl2), ta, tb);
        f2_unpack(f2_add(f2_pack(ex2_approx(ta), ex2_approx(tb)), one2), ta, tb);
        const uint64_t sig = f2_pack(rcp_approx(ta), rcp_approx(tb));
        const uint64_t d3 = f2_mul(g2, f2_mul(x2, sig));                  // dg * silu(h1)
        const uint64_t q = f2_fma(x2, f2_sub(one2, sig), one2);            // 1 + h1 (1 - sig)
        const uint64_t d1 = f2_mul(f2_mul(g2, y2), f2_mul(sig, q));        // dg h3 sig (1 + h1 (1 - sig))
        f2_unpack(d1, ta, tb);
        o1[e] = pack_bf16x2(ta, tb);
        f2_unpack(d3, ta, tb);
        o3[e] = pack_bf16x2(ta, tb);
      }
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + mr * p.ldo;
      *reinterpret_cast<uint2*>(o + col) = make_uint2(o1[0], o1[1]);
      *reinterpret_cast<uint2*>(o + p.n_half + col) = make_uint2(o3[0], o3[1]);
    }
  }
}

// Epilogue of this warp's share of one accumulator tile: TMEM lanes of rows
// mbase .. mbase + 31 (tbase addresses them), 32-column chunks [c0, c1) of
// output tile column tn.  `pre` holds chunk c0's auxiliary inputs; wbuf is the
// warp's shared-memory transpose buffer.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const KParams& p, uint32_t tbase, uint32_t wbuf, int lane, int mbase,
                                              int tn, int c0, int c1, AuxRegs& pre, float& ss) {
  if constexpr (EPI == kEpiSwiglu) {
    // Columns [0, BN/2) hold h1 = x W1, [BN/2, BN) hold h3 = x W3 for the
    // same BN/2 hidden units (kernels/ffn_fused.rs:46-63 semantics).
    constexpr int HALF = BN / 2;
#pragma unroll 1
    for (int c = c0; c < c1; ++c) {
      float4 g[8], u[8];
      tmem_chunk_coalesced(tbase + c * 32, wbuf, lane, g);
      tmem_chunk_coalesced(tbase + HALF + c * 32, wbuf, lane, u);
      const int j = tn * HALF + c * 32;
      if (j >= p.N) continue;
      const int col = j + ccol(lane);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int m = mbase + crow(i, lane);
        if (m >= p.M) continue;
        const int64_t mr = m;
        const float a1[4] = {g[i].x, g[i].y, g[i].z, g[i].w}, a3[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
        float gt[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float sig;
          gt[e] = silu_sigmoid(a1[e], sig) * a3[e];
        }
        __nv_bfloat16* h13 = static_cast<__nv_bfloat16*>(p.out) + mr * p.ldo;
        *reinterpret_cast<uint2*>(h13 + col) = pack_bf16x4(g[i]);
        *reinterpret_cast<uint2*>(h13 + p.n_half + col) = pack_bf16x4(u[i]);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out2) + mr * p.ldo2 + col) =
            pack_bf16x4(make_float4(gt[0], gt[1], gt[2], gt[3]));
      }
    }
  } else if constexpr (EPI == kEpiBf16RowDot) {
    // The warp's chunks [c0, c1) are the 128 columns of one attention head
    // (BN = 256: two heads per tile, one per epilogue half).  Each lane sums
    // bf16(C) * O over its 4 columns of the 4 chunks for its 8 rows; the 8 lanes
    // holding one row then combine in a fixed xor order.
    static_assert(BN == 256, "row dot needs one whole head per epilogue warp");
    float rd[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) rd[i] = 0.f;
    AuxRegs cur = pre;
#pragma unroll 1
    for (int c = c0; c < c1; ++c) {
      const int n = tn * BN + c * 32;
      AuxRegs nxt;
      if (c + 1 < c1) load_aux<EPI>(p, mbase, n + 32, lane, nxt);
      float4 w[8];
      tmem_chunk_coalesced(tbase + c * 32, wbuf, lane, w);
      if (n < p.N) {
        const int col = n + ccol(lane);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = mbase + crow(i, lane);
          if (m >= p.M) continue;
          const uint2 d2 = pack_bf16x4(w[i]);
          *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + int64_t(m) * p.ldo + col) = d2;
          const float4 d = unpack_bf16x4(d2.x, d2.y);
          const float4 o = unpack_bf16x4(cur.u[i].x, cur.u[i].y);
          rd[i] += (d.x * o.x + d.y * o.y) + (d.z * o.z + d.w * o.w);
        }
      }
      cur = nxt;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      rd[i] += __shfl_xor_sync(0xffffffffu, rd[i], 1);
      rd[i] += __shfl_xor_sync(0xffffffffu, rd[i], 2);
      rd[i] += __shfl_xor_sync(0xffffffffu, rd[i], 4);
    }
    const int n0 = tn * BN + c0 * 32;
    if (n0 < p.N && (lane & 7) == 0) {
      const int head = n0 >> 7, heads = p.N >> 7;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int m = mbase + crow(i, lane);
        if (m >= p.M) continue;
        const int b = m / p.seq, pos = m - b * p.seq;
        static_cast<float*>(p.out2)[(int64_t(b) * heads + head) * p.seq + pos] = rd[i];
      }
    }
  } else {
    AuxRegs cur = pre;
#pragma unroll 1
    for (int c = c0; c < c1; ++c) {
      const int n = tn * BN + c * 32;
      AuxRegs nxt;
      if (c + 1 < c1) load_aux<EPI>(p, mbase, n + 32, lane, nxt);
      float4 w[8];
      tmem_chunk_coalesced(tbase + c * 32, wbuf, lane, w);
      if (n < p.N) epilogue_chunk<EPI>(p, mbase, n, lane, w, cur, ss);
      cur = nxt;
    }
  }
}

// The warp's sum of squares into its slot; the first warp also zeroes the slots of
// CTAs the grid does not have, so all sumsq_slots floats add up to the squared norm.
__device__ __forceinline__ void write_sumsq_slots(const KParams& p, float ss, int slot, int used, bool zero_rest,
                                                  int lane) {
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) p.sumsq[slot] = ss;
  if (zero_rest)
    for (int i = used + lane; i < p.sumsq_slots; i += 32) p.sumsq[i] = 0.f;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const KParams p) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tfull_bar = empty_bar + C::STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int it = 0;  // stages armed so far
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, p.num_m, p.num_n, kRasterGroup, tm, tn);
        const int m0 = tm * BM;
        for (int kb = 0; kb < p.num_kb; kb += C::KPS, ++it) {  // one stage: k-blocks kb .. kb + KPS - 1
          const int stage = it % C::STAGES;
          const uint32_t phase = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) {
            set_error(p.err, kDevTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          if (*abort_flag) {
            ok = false;
            break;
          }
          const int nsub = min(C::KPS, p.num_kb - kb);
          mbar_arrive_expect_tx(&full_bar[stage], nsub * C::SUB_BYTES);
          for (int sub = 0; sub < nsub; ++sub) {
            uint8_t* sA = smem + stage * C::STAGE_BYTES + sub * C::SUB_BYTES;
            uint8_t* sB = sA + C::A_BYTES;
            const int k0 = (kb + sub) * BK;
            if constexpr (A_MN) {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) tma_load_2d(sA + j * 8192, &tmA, &full_bar[stage], m0 + 64 * j, k0);
            } else {
              tma_load_2d(sA, &tmA, &full_bar[stage], k0, m0);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) {
                int nphys;
                if constexpr (EPI == kEpiSwiglu) {
                  constexpr int HALF = BN / 2;
                  nphys = (j < HALF / 64) ? tn * HALF + 64 * j : p.n_half + tn * HALF + 64 * (j - HALF / 64);
                } else {
                  nphys = tn * BN + 64 * j;
                }
                tma_load_2d(sB + j * 8192, &tmB, &full_bar[stage], nphys, k0);
              }
            } else {
              tma_load_2d(sB, &tmB, &full_bar[stage], k0, tn * BN);
            }
          }
        }
      }
      if (!ok) {
        // Drain copies that may still be in flight before the CTA exits.
        for (int i = (it > C::STAGES ? it - C::STAGES : 0); i < it; ++i)
          mbar_wait(&full_bar[i % C::STAGES], (i / C::STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_par = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_par ^ 1) || *abort_flag) {
          set_error(p.err, kDevTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::ACC_STRIDE);
        for (int kb = 0; kb < p.num_kb; kb += C::KPS, ++it) {
          const int stage = it % C::STAGES;
          const uint32_t phase = (it / C::STAGES) & 1;
          if (!mbar_wait(&full_bar[stage], phase) || *abort_flag) {
            set_error(p.err, kDevTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const int nsub = min(C::KPS, p.num_kb - kb);
          for (int sub = 0; sub < nsub; ++sub) {
            const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES + sub * C::SUB_BYTES);
            const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
              const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
              umma_bf16(d_tmem, ad, bd, idesc, (kb | sub | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit(&empty_bar[stage]);  // frees the smem slot once these MMAs finish
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
      // All MMAs issued by this thread must finish before TMEM is released.
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;               // TMEM lane quadrant = accumulator rows 32q..32q+31
    const int half = (warp - 4) >> 2;     // which half of the tile's 32-column chunks
    constexpr int NCH = (EPI == kEpiSwiglu) ? (BN / 2) / 32 : BN / 32;
    const int c0 = half * NCH / 2, c1 = (half + 1) * NCH / 2;
    const uint32_t wbuf = smem_u32(smem + C::EPI_OFF + (warp - 4) * kEpiBufBytes);
    int local = 0;
    float ss = 0.f;  // kEpiF32Acc: this warp's sum of squares over its tiles
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_par = (local >> 1) & 1;
      int tm, tn;
      tile_coords(tile, p.num_m, p.num_n, kRasterGroup, tm, tn);
      const int mbase = tm * BM + q * 32;
      AuxRegs pre;  // first chunk's auxiliary inputs do not depend on the MMA: fetch before waiting
      if constexpr (EPI != kEpiSwiglu) {
        if (c0 < c1) load_aux<EPI>(p, mbase, tn * BN + c0 * 32, lane, pre);
      }
      bool ok = mbar_wait(&tfull_bar[acc], acc_par);
      ok = __all_sync(0xffffffffu, ok);
      const int aborted = __shfl_sync(0xffffffffu, *abort_flag, 0);
      if (!ok || aborted) {
        if (!ok && lane == 0) {
          set_error(p.err, kDevTimeoutEpilogue);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + static_cast<uint32_t>(acc * C::ACC_STRIDE) + (static_cast<uint32_t>(q * 32) << 16);
      epilogue_tile<BN, EPI>(p, tbase, wbuf, lane, mbase, tn, c0, c1, pre, ss);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
    if constexpr (EPI == kEpiF32Acc) {
      if (p.sumsq) write_sumsq_slots(p, ss, static_cast<int>(blockIdx.x) * kEpiWarps + (warp - 4),
                                     static_cast<int>(gridDim.x) * kEpiWarps, blockIdx.x == 0 && warp == 4, lane);
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// --------------------------------------------------------- CTA-pair kernel
// Same pipeline as above, but a cluster of two CTAs computes a 256 x BN tile
// with tcgen05.mma.cta_group::2: each CTA loads its own 128 rows of A and its
// own half of the B columns into its own shared memory (completion bytes
// counted on the leader's barrier), the leader (cluster rank 0) issues the
// MMAs, which read both CTAs' shared memory and write each CTA's 128 rows of
// the accumulator into that CTA's TMEM; both CTAs run the epilogue on their rows.
// Per SM this halves the B tile traffic for the same math.
template <int BN>
struct Gemm2Cfg {
  static constexpr int BNH = BN / 2;  // B columns held by each CTA
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = BNH * BK * 2;
  // A stage holds up to two 64-deep k-blocks (one mbarrier round trip and one
  // pair of commits per eight MMAs instead of four: measured 10-15% faster).
  static constexpr int SUB_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = 2 * SUB_BYTES;
  static constexpr int STAGES = (BN == 128) ? 4 : 3;
  static constexpr int ACC_STRIDE = (BN == 192) ? 256 : BN;  // TMEM columns per accumulator buffer
  static constexpr int TMEM_COLS = 2 * ACC_STRIDE;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + kEpiWarps * 32 * 128;
  static constexpr int SMEM_BYTES = BAR_OFF + 1024 + 256;
};

// BN = 192 puts 96 B columns in each CTA: fine for K-major B (96 rows), not
// for MN-major B, whose 128-byte swizzle atoms are 64 columns wide.
template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const KParams p) {
  using C = Gemm2Cfg<BN>;
  static_assert(!(B_MN && BN == 192), "MN-major B needs 64-column halves");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tfull_bar = empty_bar + C::STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);  // epilogue warps of both CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {  // same warp in both CTAs, same slot offset
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m2 = (p.M + 255) / 256;
  const int num_tiles = num_m2 * p.num_n;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer (both CTAs)
      int it = 0;
      bool ok = true;
      const uint32_t full0 = mapa_shared(smem_u32(&full_bar[0]), 0);  // the leader's barriers
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int tm, tn;
        tile_coords(tile, num_m2, p.num_n, kRasterGroup / 2, tm, tn);
        const int m0 = tm * 256 + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < p.num_kb; kb += 2, ++it) {  // one stage: k-blocks kb and kb + 1
          const int stage = it % C::STAGES;
          const uint32_t phase = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty_bar[stage], phase ^ 1) || *abort_flag) {
            set_error(p.err, kDevTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const int nsub = p.num_kb - kb > 1 ? 2 : 1;
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * nsub * C::SUB_BYTES);  // both CTAs' copies
          const uint32_t fbar = full0 + 8 * stage;
          for (int sub = 0; sub < nsub; ++sub) {
            uint8_t* sA = smem + stage * C::STAGE_BYTES + sub * C::SUB_BYTES;
            uint8_t* sB = sA + C::A_BYTES;
            const int k0 = (kb + sub) * BK;
            if constexpr (A_MN) {
#pragma unroll
              for (int j = 0; j < 2; ++j) tma_load_2d_pair(sA + j * 8192, &tmA, fbar, m0 + 64 * j, k0);
            } else {
              tma_load_2d_pair(sA, &tmA, fbar, k0, m0);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < C::BNH / 64; ++j) {
                const int lc = static_cast<int>(rank) * C::BNH + 64 * j;  // column within the tile
                int nphys;
                if constexpr (EPI == kEpiSwiglu) {
                  constexpr int HALF = BN / 2;  // rank 0 holds the W1 columns, rank 1 the W3 columns
                  nphys = (lc < HALF) ? tn * HALF + lc : p.n_half + tn * HALF + (lc - HALF);
                } else {
                  nphys = tn * BN + lc;
                }
                tma_load_2d_pair(sB + j * 8192, &tmB, fbar, nphys, k0);
              }
            } else {
              tma_load_2d_pair(sB, &tmB, fbar, k0, tn * BN + static_cast<int>(rank) * C::BNH);
            }
          }
        }
      }
      if (!ok && leader) {  // the leader's full barriers also count the peer's copies
        for (int i = (it > C::STAGES ? it - C::STAGES : 0); i < it; ++i)
          mbar_wait(&full_bar[i % C::STAGES], (i / C::STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------------------------------------------------- MMA issuer (leader)
      constexpr uint32_t idesc = idesc_bf16_f32(256, BN, A_MN, B_MN);
      // the same barrier offsets in the peer CTA (cluster rank 1)
      const uint32_t empty0 = smem_u32(&empty_bar[0]), empty1 = mapa_shared(empty0, 1);
      const uint32_t tfull0 = smem_u32(&tfull_bar[0]), tfull1 = mapa_shared(tfull0, 1);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_par = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_par ^ 1) || *abort_flag) {
          set_error(p.err, kDevTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::ACC_STRIDE);
        for (int kb = 0; kb < p.num_kb; kb += 2, ++it) {
          const int stage = it % C::STAGES;
          const uint32_t phase = (it / C::STAGES) & 1;
          if (!mbar_wait(&full_bar[stage], phase) || *abort_flag) {
            set_error(p.err, kDevTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const int nsub = p.num_kb - kb > 1 ? 2 : 1;
          for (int sub = 0; sub < nsub; ++sub) {
            const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES + sub * C::SUB_BYTES);
            const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
              const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
              umma_bf16_pair(d_tmem, ad, bd, idesc, (kb | kk | sub) != 0 ? 1u : 0u);
            }
          }
          umma_commit_pair(empty0 + 8 * stage);  // both CTAs' slots are free once these finish
          umma_commit_pair(empty1 + 8 * stage);
        }
        if (ok) {
          umma_commit_pair(tfull0 + 8 * acc);
          umma_commit_pair(tfull1 + 8 * acc);
        }
      }
      umma_commit_pair(smem_u32(drain_bar));
      mbar_wait(drain_bar, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    constexpr int NCH = (EPI == kEpiSwiglu) ? (BN / 2) / 32 : BN / 32;
    const int c0 = half * NCH / 2, c1 = (half + 1) * NCH / 2;
    const uint32_t wbuf = smem_u32(smem + C::EPI_OFF + (warp - 4) * kEpiBufBytes);
    const uint32_t tempty0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);  // the leader's barriers
    int local = 0;
    float ss = 0.f;  // kEpiF32Acc: this warp's sum of squares over its tiles
    for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_par = (local >> 1) & 1;
      int tm, tn;
      tile_coords(tile, num_m2, p.num_n, kRasterGroup / 2, tm, tn);
      const int mbase = tm * 256 + static_cast<int>(rank) * 128 + q * 32;
      AuxRegs pre;
      if constexpr (EPI != kEpiSwiglu) {
        if (c0 < c1) load_aux<EPI>(p, mbase, tn * BN + c0 * 32, lane, pre);
      }
      bool ok = mbar_wait(&tfull_bar[acc], acc_par);
      ok = __all_sync(0xffffffffu, ok);
      const int aborted = __shfl_sync(0xffffffffu, *abort_flag, 0);
      if (!ok || aborted) {
        if (!ok && lane == 0) {
          set_error(p.err, kDevTimeoutEpilogue);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + static_cast<uint32_t>(acc * C::ACC_STRIDE) + (static_cast<uint32_t>(q * 32) << 16);
      epilogue_tile<BN, EPI>(p, tbase, wbuf, lane, mbase, tn, c0, c1, pre, ss);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + 8 * acc);
    }
    if constexpr (EPI == kEpiF32Acc) {
      if (p.sumsq)
        write_sumsq_slots(p, ss, pair * 2 * kEpiWarps + static_cast<int>(rank) * kEpiWarps + (warp - 4),
                          npairs * 2 * kEpiWarps, pair == 0 && rank == 0 && warp == 4, lane);
    }
  }

  __syncthreads();
  cluster_sync();  // the leader's MMAs into this CTA's TMEM and both epilogues are done
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool encoder_ready() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

// 2-D bf16 tensor [outer][inner] with row stride `ld` elements, 128-B swizzled boxes.
bool make_tmap(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
               uint32_t box_outer) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
int launch_inst(const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, int grid, cudaStream_t s) {
  using C = GemmCfg<BN>;
  const cudaError_t attr =
      smem_limit_once(reinterpret_cast<const void*>(gemm_tc_kernel<BN, A_MN, B_MN, EPI>), C::SMEM_BYTES);
  if (attr != cudaSuccess) return attr;
  gemm_tc_kernel<BN, A_MN, B_MN, EPI><<<grid, kThreads, C::SMEM_BYTES, s>>>(ta, tb, kp);
  return cudaGetLastError();
}

template <int BN, bool A_MN, bool B_MN, int EPI>
int launch_inst2(const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, int grid, cudaStream_t s) {
  using C = Gemm2Cfg<BN>;
  const cudaError_t attr =
      smem_limit_once(reinterpret_cast<const void*>(gemm_tc2_kernel<BN, A_MN, B_MN, EPI>), C::SMEM_BYTES);
  if (attr != cudaSuccess) return attr;
  gemm_tc2_kernel<BN, A_MN, B_MN, EPI><<<grid, kThreads, C::SMEM_BYTES, s>>>(ta, tb, kp);
  return cudaGetLastError();
}

// Every (A major, B major, epilogue) combination the LM step launches.
#define RT_GEMM_COMBOS(X)                                                                    \
  /* forward projections (B = weight, MN-major) */                                          \
  X(false, true, kEpiRope) X(false, true, kEpiResidual) X(false, true, kEpiSwiglu)           \
  X(false, true, kEpiSwigluBwd) X(false, true, kEpiF32) X(false, true, kEpiBf16)             \
  X(false, true, kEpiF32Acc)                                                                 \
  /* K-major weights (W2 forward, logits, data gradients) */                                \
  X(false, false, kEpiBf16) X(false, false, kEpiF32) X(false, false, kEpiF32Acc)             \
  X(false, false, kEpiResidual) X(false, false, kEpiRope) X(false, false, kEpiSwigluBwd)     \
  /* weight gradients: both operands contract over tokens */                                \
  X(true, true, kEpiF32Acc) X(true, true, kEpiF32) X(true, true, kEpiBf16)                   \
  X(true, false, kEpiF32) X(true, false, kEpiF32Acc)

// Combinations with K-major B (the only ones the 192-wide CTA pair supports).
#define RT_GEMM_COMBOS_BK(X)                                                                 \
  X(false, false, kEpiBf16) X(false, false, kEpiF32) X(false, false, kEpiF32Acc)             \
  X(false, false, kEpiResidual) X(false, false, kEpiRope) X(false, false, kEpiSwigluBwd)     \
  X(true, false, kEpiF32) X(true, false, kEpiF32Acc)

int dispatch2_192(const GemmArgs& g, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, int grid,
                  cudaStream_t s) {
#define RT_GEMM_CASE(AMN, BMN, EPI) \
  if (g.a_mn == AMN && g.b_mn == BMN && g.epi == EPI) return launch_inst2<192, AMN, BMN, EPI>(ta, tb, kp, grid, s);
  RT_GEMM_COMBOS_BK(RT_GEMM_CASE)
#undef RT_GEMM_CASE
  return -1;
}

template <int BN>
int dispatch2(const GemmArgs& g, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, int grid,
              cudaStream_t s) {
#define RT_GEMM_CASE(AMN, BMN, EPI) \
  if (g.a_mn == AMN && g.b_mn == BMN && g.epi == EPI) return launch_inst2<BN, AMN, BMN, EPI>(ta, tb, kp, grid, s);
  RT_GEMM_COMBOS(RT_GEMM_CASE)
#undef RT_GEMM_CASE
  if constexpr (BN == 256) {
    if (!g.a_mn && !g.b_mn && g.epi == kEpiBf16RowDot)
      return launch_inst2<256, false, false, kEpiBf16RowDot>(ta, tb, kp, grid, s);
  }
  return -1;
}

template <int BN>
int dispatch(const GemmArgs& g, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, int grid,
             cudaStream_t s) {
#define RT_GEMM_CASE(AMN, BMN, EPI) \
  if (g.a_mn == AMN && g.b_mn == BMN && g.epi == EPI) return launch_inst<BN, AMN, BMN, EPI>(ta, tb, kp, grid, s);
  RT_GEMM_COMBOS(RT_GEMM_CASE)
#undef RT_GEMM_CASE
  if constexpr (BN == 256) {
    if (!g.a_mn && !g.b_mn && g.epi == kEpiBf16RowDot)
      return launch_inst<256, false, false, kEpiBf16RowDot>(ta, tb, kp, grid, s);
  }
  return -1;
}

int g_num_sms = 0;

}  // namespace

int gemm_sumsq_slots() { return kEpiWarps * num_sms(); }

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

namespace {

// CTA-pair path: the cluster of two CTAs owns a 256 x bn output tile.
int gemm_launch_pair(const GemmArgs& g, int bn, cudaStream_t stream) {
  const bool swiglu = g.epi == kEpiSwiglu;
  if (swiglu && g.N % (bn / 2) != 0) return -1;
  if (bn == 192 && (g.b_mn || swiglu)) return -1;
  if (g.epi == kEpiBf16RowDot && bn != 256) return -1;
  KParams kp{};
  kp.M = g.M;
  kp.N = g.N;
  kp.num_kb = g.K / BK;
  kp.num_m = (g.M + 255) / 256;
  kp.num_n = swiglu ? g.N / (bn / 2) : (g.N + bn - 1) / bn;
  kp.num_tiles = kp.num_m * kp.num_n;
  kp.n_half = g.n_half;
  kp.beta = g.beta;
  kp.alpha = g.alpha;
  kp.seq = g.seq;
  kp.rope_cols = g.rope_cols;
  kp.out = g.out;
  kp.ldo = g.ldo;
  kp.out2 = g.out2;
  kp.ldo2 = g.ldo2;
  kp.aux = g.aux;
  kp.ld_aux = g.ld_aux;
  kp.rope_cos = g.rope_cos;
  kp.rope_sin = g.rope_sin;
  kp.err = g.err;
  kp.sumsq = g.sumsq;
  kp.sumsq_slots = g.sumsq_slots;

  CUtensorMap ta, tb;
  bool ok;
  if (g.a_mn)
    ok = make_tmap(&ta, g.a, g.M, g.K, g.lda, 64, 64);
  else
    ok = make_tmap(&ta, g.a, g.K, g.M, g.lda, 64, BM);
  if (!ok) return -3;
  const uint64_t b_inner_mn = swiglu ? uint64_t(g.n_half) + g.N : uint64_t(g.N);
  if (g.b_mn)
    ok = make_tmap(&tb, g.b, b_inner_mn, g.K, g.ldb, 64, 64);
  else
    ok = make_tmap(&tb, g.b, g.K, g.N, g.ldb, 64, bn / 2);
  if (!ok) return -3;

  const int max_pairs = num_sms() / 2;
  const int grid = 2 * (kp.num_tiles < max_pairs ? kp.num_tiles : max_pairs);
  if (bn == 256) return dispatch2<256>(g, ta, tb, kp, grid, stream);
  if (bn == 192) return dispatch2_192(g, ta, tb, kp, grid, stream);
  return dispatch2<128>(g, ta, tb, kp, grid, stream);
}

}  // namespace

bool make_tmap_bf16(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                    uint32_t box_inner, uint32_t box_outer) {
  return encoder_ready() && make_tmap(tm, ptr, inner, outer, ld, box_inner, box_outer);
}

int gemm_launch(const GemmArgs& g, cudaStream_t stream) {
  if (!encoder_ready()) return -2;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || g.K % BK != 0 || g.N % 32 != 0) return -1;
  if (g.lda % 8 != 0 || g.ldb % 8 != 0) return -1;
  if ((reinterpret_cast<uintptr_t>(g.a) | reinterpret_cast<uintptr_t>(g.b) | reinterpret_cast<uintptr_t>(g.out)) & 15)
    return -1;
  if (g.a_mn && g.M % 64 != 0) return -1;
  const bool swiglu = g.epi == kEpiSwiglu;
  if (swiglu && (!g.b_mn || g.n_half % 64 != 0 || g.N % 64 != 0)) return -1;
  if (g.epi == kEpiRope && (g.seq <= 0 || g.rope_cols % 128 != 0)) return -1;
  if (g.sumsq && (g.epi != kEpiF32Acc || g.sumsq_slots < gemm_sumsq_slots())) return -1;
  const bool rowdot = g.epi == kEpiBf16RowDot;
  if (rowdot) {
    // One head of 128 columns per epilogue warp: 256-wide tiles, K-major operands.
    if (g.a_mn || g.b_mn || g.N % 128 != 0 || g.seq <= 0 || g.M % g.seq != 0 || !g.aux || !g.out2 ||
        g.ld_aux % 4 != 0 || (reinterpret_cast<uintptr_t>(g.aux) & 7) || (reinterpret_cast<uintptr_t>(g.out2) & 3))
      return -1;
    if (g.force_bn != 0 && g.force_bn != 256 && g.force_bn != -256) return -1;
  }

  const int sms = num_sms();
  auto tiles_for = [&](int bn) {
    const int per_tile_n = swiglu ? bn / 2 : bn;
    return ((g.M + BM - 1) / BM) * ((g.N + per_tile_n - 1) / per_tile_n);
  };
  // force_bn: 128/192/256 pick the single-CTA kernel with that tile width,
  // -256/-128 the CTA-pair kernel (256-row tiles); anything else chooses.
  if (g.force_bn == -256 || g.force_bn == -192 || g.force_bn == -128)
    return gemm_launch_pair(g, -g.force_bn, stream);
  int bn = g.force_bn;
  if (bn != 128 && bn != 192 && bn != 256) {
    // time ~ waves x tile width / efficiency, where a partial last wave costs
    // 0.6 + 0.4 x its fill of a full one (its tiles run faster: fewer SMs share HBM,
    // L2 and the power budget).  The 0.6 and the efficiencies are a least-squares fit
    // (4% rms) to every variant timed on every 600M GEMM shape (K = 1536 .. 8192):
    // relative to the single-CTA 256-wide tile, single-CTA 192 0.885 and 128 0.669
    // (narrow tiles re-read A per tile and sit at the shared-memory read limit), CTA
    // pair 256 x 256 1.137, 256 x 192 1.007, 256 x 128 0.777 (each SM of a pair reads
    // only half of B).  The fit picks the fastest measured variant on 10 of the 11
    // shapes (the 11th within 1.5%) and keeps pair 256 x 256 on the 7B / 30B shapes.
    auto waves = [](int t, int units) {
      if (t <= units) return 1.0;
      const int full = t / units;
      const double frac = double(t) / units - full;
      return full + (frac > 0 ? 0.6 + 0.4 * frac : 0.0);
    };
    double best = 1e30;
    for (int cand : {256, 192, 128}) {
      if (swiglu && (cand == 192 || g.N % (cand / 2) != 0)) continue;
      if (rowdot && cand != 256) continue;
      const double eff = cand == 256 ? 1.0 : (cand == 192 ? 0.885 : 0.669);
      const double cost = waves(tiles_for(cand), sms) * cand / eff;
      if (cost < best * 0.999) {
        best = cost;
        bn = cand;
      }
    }
    if (!g.shared_sms && (!swiglu || g.N % 128 == 0)) {
      const int pairs = sms / 2;
      int pbn = 0;
      for (int cand : {192, 256, 128}) {
        if (cand == 192 && (g.b_mn || swiglu)) continue;
        if (swiglu && g.N % (cand / 2) != 0) continue;
        if (rowdot && cand != 256) continue;
        const int t2 = ((g.M + 255) / 256) * (swiglu ? g.N / (cand / 2) : (g.N + cand - 1) / cand);
        const double eff2 = cand == 192 ? 1.007 : (cand == 256 ? 1.137 : 0.777);
        const double cost2 = waves(t2, pairs) * cand / eff2;
        if (cost2 < best * 0.999) {
          best = cost2;
          pbn = cand;
        }
      }
      if (pbn) return gemm_launch_pair(g, pbn, stream);
    }
  }
  if (swiglu && (bn == 192 || g.N % (bn / 2) != 0)) bn = 128;

  KParams kp{};
  kp.M = g.M;
  kp.N = g.N;
  kp.num_kb = g.K / BK;
  kp.num_m = (g.M + BM - 1) / BM;
  kp.num_n = swiglu ? (g.N + bn / 2 - 1) / (bn / 2) : (g.N + bn - 1) / bn;
  kp.num_tiles = kp.num_m * kp.num_n;
  kp.n_half = g.n_half;
  kp.beta = g.beta;
  kp.alpha = g.alpha;
  kp.seq = g.seq;
  kp.rope_cols = g.rope_cols;
  kp.out = g.out;
  kp.ldo = g.ldo;
  kp.out2 = g.out2;
  kp.ldo2 = g.ldo2;
  kp.aux = g.aux;
  kp.ld_aux = g.ld_aux;
  kp.rope_cos = g.rope_cos;
  kp.rope_sin = g.rope_sin;
  kp.err = g.err;
  kp.sumsq = g.sumsq;
  kp.sumsq_slots = g.sumsq_slots;

  CUtensorMap ta, tb;
  bool ok;
  if (g.a_mn)
    ok = make_tmap(&ta, g.a, g.M, g.K, g.lda, 64, 64);
  else
    ok = make_tmap(&ta, g.a, g.K, g.M, g.lda, 64, BM);
  if (!ok) return -3;
  const uint64_t b_inner_mn = swiglu ? uint64_t(g.n_half) + g.N : uint64_t(g.N);
  if (g.b_mn)
    ok = make_tmap(&tb, g.b, b_inner_mn, g.K, g.ldb, 64, 64);
  else
    ok = make_tmap(&tb, g.b, g.K, g.N, g.ldb, 64, bn);
  if (!ok) return -3;

  const int grid = kp.num_tiles < sms ? kp.num_tiles : sms;
  if (bn == 256) return dispatch<256>(g, ta, tb, kp, grid, stream);
  if (bn == 192) return dispatch<192>(g, ta, tb, kp, grid, stream);
  return dispatch<128>(g, ta, tb, kp, grid, stream);
}

}  // namespace rt
