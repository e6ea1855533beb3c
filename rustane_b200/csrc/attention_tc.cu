// Causal attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same semantics and layout as the mma.sync kernels in attention.cu
// (crates/engine/src/kernels/sdpa_fwd.rs:130-150): per (sequence, head, block
// of 128 queries), S = Q K^T / sqrt(128) with the causal mask, P = softmax(S),
// O = P V; O [M, D] bf16 and the log2-domain statistic lse2 = max + log2(sum)
// that the backward kernels use to rebuild P.
//
// One CTA per query block, 256 threads:
//   warp 0      TMA producer: Q once, then K_j and V_j (128 keys x 128) into
//               two-deep rings;
//   warp 1      one lane issues the MMAs: S_j = Q K_j^T into one of two TMEM
//               S buffers (128 columns each), O += P_j V_j into the TMEM O
//               buffer; S_{j+1} is issued before O += P_j V_j so the softmax of
//               block j+1 overlaps the P V product of block j;
//   warp 2      owns the TMEM allocation (512 columns);
//   warps 4-11  softmax, two threads per query row (TMEM lane = row, each
//               thread 64 of the 128 key columns; row max and sum exchanged
//               through shared memory): P_j = exp2(S_j * scale - m) in bf16
//               pairs written back over the thread's own S_j columns in TMEM,
//               where the P V MMA reads it as its TMEM operand (the MMA's
//               commit frees the S buffer), running sum l; O rescaled in TMEM only
//               when the row max grew by more than 2^8 (otherwise the stale
//               max is kept: P <= 256); O / l goes through a swizzled shared-
//               memory tile to one TMA store per 64 columns.
// All waits are bounded; a timeout sets the device error word.
#include "attention.h"
#include "common.cuh"
#include "kernels.h"

namespace rt {
namespace {

constexpr int kHd = 128;
constexpr int kBlk = 128;                    // queries per CTA and keys per KV block
constexpr int kTileBytes = kBlk * kHd * 2;   // 32 KB: two 64-column swizzle atoms of 128 rows
constexpr int kAtomBytes = kTileBytes / 2;   // 16 KB
constexpr int kFwdThreads = 384;   // 8 softmax warps, two threads per query row
constexpr float kRescaleLog2 = 8.0f;         // keep a stale row max while P stays <= 2^8

struct FwdSmem {
  static constexpr int Q = 0;
  static constexpr int K = Q + kTileBytes;          // [2]
  static constexpr int V = K + 2 * kTileBytes;      // [2]
  static constexpr int P = V + 2 * kTileBytes;
  static constexpr int RED = P + kTileBytes;        // float [2 parities][2 halves][128 rows]: row max
  static constexpr int SUM = RED + 2 * 2 * kBlk * 4; // float [2 halves][128 rows]: row sum
  static constexpr int BAR = SUM + 2 * kBlk * 4;
  static constexpr int BYTES = BAR + 256 + 1024;    // barriers, TMEM slot, alignment slack
};

enum Bar : int {
  kQFull = 0,
  kKFull = 1,   // [2]
  kKEmpty = 3,  // [2]
  kVFull = 5,   // [2]
  kVEmpty = 7,  // [2]
  kSFull = 9,   // [2]
  kSFree = 11,  // [2]
  kPFull = 13,
  kPvDone = 14,
  kDrain = 15,
  kNumBars = 16
};

__device__ __forceinline__ void softmax_bar() {  // the 8 softmax warps only
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_out,
                       float* __restrict__ lse2, int S, int nh, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + FwdSmem::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (heads, batch, query blocks): the heaviest (last) query blocks go out first
  const int qb = gridDim.z - 1 - blockIdx.z;
  const int h = blockIdx.x, b = blockIdx.y;
  const int nb = qb + 1;  // causal: key blocks 0 .. qb
  const int tok0 = b * S;
  const int q0 = qb * kBlk;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kQFull], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[kKFull + i], 1);
      mbar_init(&bar[kKEmpty + i], 1);
      mbar_init(&bar[kVFull + i], 1);
      mbar_init(&bar[kVEmpty + i], 1);
      mbar_init(&bar[kSFull + i], 1);
      mbar_init(&bar[kSFree + i], 1);
    }
    mbar_init(&bar[kPFull], 8);
    mbar_init(&bar[kPvDone], 1);
    mbar_init(&bar[kDrain], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // columns [0,128) S0, [128,256) S1, [256,384) O

  if (warp == 0) {
    if (lane == 0) {
      // --------------------------------------------------------------- producer
      const int D = nh * kHd;
      const int qc = h * kHd, kc = D + h * kHd, vc = 2 * D + h * kHd;
      int issued = 0;  // key blocks whose K and V loads were issued
      mbar_arrive_expect_tx(&bar[kQFull], kTileBytes);
      tma_load_2d(smem + FwdSmem::Q, &tm_qkv, &bar[kQFull], qc, tok0 + q0);
      tma_load_2d(smem + FwdSmem::Q + kAtomBytes, &tm_qkv, &bar[kQFull], qc + 64, tok0 + q0);
      for (int j = 0; j < nb; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int row = tok0 + j * kBlk;
        if (!mbar_wait(&bar[kKEmpty + st], ph ^ 1) || *abort_flag) {
          set_error(err, kDevTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        uint8_t* sk = smem + FwdSmem::K + st * kTileBytes;
        mbar_arrive_expect_tx(&bar[kKFull + st], kTileBytes);
        tma_load_2d(sk, &tm_qkv, &bar[kKFull + st], kc, row);
        tma_load_2d(sk + kAtomBytes, &tm_qkv, &bar[kKFull + st], kc + 64, row);
        if (!mbar_wait(&bar[kVEmpty + st], ph ^ 1) || *abort_flag) {
          set_error(err, kDevTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        uint8_t* sv = smem + FwdSmem::V + st * kTileBytes;
        mbar_arrive_expect_tx(&bar[kVFull + st], kTileBytes);
        tma_load_2d(sv, &tm_qkv, &bar[kVFull + st], vc, row);
        tma_load_2d(sv + kAtomBytes, &tm_qkv, &bar[kVFull + st], vc + 64, row);
        issued = j + 1;
      }
      if (*abort_flag) {  // let copies still in flight land before the CTA exits
        mbar_wait(&bar[kQFull], 0);
        for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j) {
          mbar_wait(&bar[kKFull + (j & 1)], (j >> 1) & 1);
          mbar_wait(&bar[kVFull + (j & 1)], (j >> 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = idesc_bf16_f32(kBlk, kBlk, false, false);  // Q, K: both hd-contiguous
      constexpr uint32_t idesc_o = idesc_bf16_f32(kBlk, kHd, false, true);    // P key-contiguous, V hd-contiguous
      const uint32_t sq = smem_u32(smem + FwdSmem::Q);
      bool ok = mbar_wait(&bar[kQFull], 0);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&bar[kKFull + st], ph) || !mbar_wait(&bar[kSFree + st], ph ^ 1) || *abort_flag) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + FwdSmem::K + st * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtomBytes + (kk & 3) * 32;
          umma_bf16(tmem + st * kBlk, smem_desc_sw128(sq + off, 16, 1024), smem_desc_sw128(sk + off, 16, 1024),
                    idesc_s, kk != 0 ? 1u : 0u);
        }
        umma_commit(&bar[kKEmpty + st]);
        umma_commit(&bar[kSFull + st]);
        return true;
      };
      ok = ok && issue_s(0);
      for (int j = 0; ok && j < nb; ++j) {
        if (j + 1 < nb && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        const int st = j & 1;
        if (!mbar_wait(&bar[kPFull], j & 1) || !mbar_wait(&bar[kVFull + st], (j >> 1) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + FwdSmem::V + st * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk) {
          // P from TMEM (bf16 pairs over the S_j columns: keys 16 kk.. at column 8 kk, or 64 + 8 (kk - 4)
          // for the second half); V: hd-contiguous rows, 16 keys = 2 KB
          const uint32_t acol = st * kBlk + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8);
          umma_bf16_ts(tmem + 2 * kBlk, tmem + acol, smem_desc_sw128(sv + kk * 2048, kAtomBytes, 1024), idesc_o,
                       (j | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&bar[kVEmpty + st]);
        umma_commit(&bar[kPvDone]);
        umma_commit(&bar[kSFree + st]);  // P_j (over S_j) consumed: the buffer can take S_{j+2}
      }
      if (!ok) {
        set_error(err, kDevTimeoutMma);
        *abort_flag = 1;
      }
      umma_commit(&bar[kDrain]);
      mbar_wait(&bar[kDrain], 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax
    const int qw = warp & 3;               // TMEM lane quadrant
    const int hh = (warp - 4) >> 2;        // key columns [64 hh, 64 hh + 64) of the block
    const int r = qw * 32 + lane;          // query row within the block
    const uint32_t lane_off = static_cast<uint32_t>(qw * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + FwdSmem::RED);
    float* sum = reinterpret_cast<float*>(smem + FwdSmem::SUM);
    float m_used = -INFINITY, l = 0.f;
    // A failed (timed-out) wait does not leave the loop: every softmax warp must
    // reach the same sequence of named barriers.  After the first failure the
    // abort flag makes every later wait return at once.
    bool ok = true;
    auto wait = [&](uint64_t* bb, uint32_t parity) {
      bool w = !*abort_flag && mbar_wait(bb, parity);
      w = __all_sync(0xffffffffu, w);
      if (!w) {
        ok = false;
        *abort_flag = 1;
      }
    };
    for (int j = 0; j < nb; ++j) {
      const int st = j & 1;
      wait(&bar[kSFull + st], (j >> 1) & 1);
      tc_fence_after();
      const uint32_t ts = tmem + st * kBlk + lane_off + hh * 64;
      uint32_t v[64];
      tmem_ld32(ts, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(ts + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld_wait();
      // keys past the query are masked in the diagonal block: key column 64 hh + e vs row r
      const int lim = j == qb ? r - hh * 64 : 64;  // valid columns e < lim + 1
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < 64; ++e)
        if (e <= lim) mx = fmaxf(mx, __uint_as_float(v[e]));
      red[(st * 2 + hh) * kBlk + r] = mx;
      softmax_bar();
      mx = fmaxf(red[(st * 2) * kBlk + r], red[(st * 2 + 1) * kBlk + r]);
      const float m_new = fmaxf(m_used, mx * scale_log2);
      if (j > 0) {  // P V of block j - 1 must be done before P or O is touched
        wait(&bar[kPvDone], (j - 1) & 1);
        tc_fence_after();
      }
      if (j == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, m_new > m_used + kRescaleLog2)) {
        // rescale this warp's half of the O rows (warp-wide TMEM access; factor 1 where the max held)
        const bool grow = m_new > m_used + kRescaleLog2;
        const float f = grow ? exp2f(m_used - m_new) : 1.f;
        if (grow) {
          l *= f;
          m_used = m_new;
        }
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          const uint32_t to = tmem + 2 * kBlk + lane_off + hh * 64 + c * 32;
          tmem_ld32(to, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(to, o);
        }
        tmem_st_wait();
      }
      // P = exp2(S * scale - m) in bf16 pairs, written back over this thread's own (already
      // read) S_j columns: keys 64 hh + 2 i, + 1 at column 64 hh + i; the P V MMA reads it there
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int e = c * 32 + 2 * t;
          const float p0 = e <= lim ? exp2f(__uint_as_float(v[e]) * scale_log2 - m_used) : 0.f;
          const float p1 = e + 1 <= lim ? exp2f(__uint_as_float(v[e + 1]) * scale_log2 - m_used) : 0.f;
          l += p0 + p1;
          pk[t] = pack_bf16x2(p0, p1);
        }
        tmem_st16(ts + c * 16, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kPFull]);
    }
    wait(&bar[kPvDone], (nb - 1) & 1);
    sum[hh * kBlk + r] = l;
    softmax_bar();
    l = sum[r] + sum[kBlk + r];
    if (!ok) {
      if (lane == 0) set_error(err, kDevTimeoutEpilogue);
    } else {
      // O / l in bf16 into the (now idle) P tile, 128-byte swizzled, head-dim columns
      // [64 hh, 64 hh + 64) = atom hh; one TMA store per atom below
      tc_fence_after();
      const float inv_l = 1.f / l;
      uint8_t* orow = smem + FwdSmem::P + hh * kAtomBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        float f[32];
        tmem_ld32(tmem + 2 * kBlk + lane_off + hh * 64 + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(o[e]) * inv_l;
        store_chunk32(orow, c, r, f);
      }
      fence_proxy_async_smem();
      if (hh == 0) lse2[(static_cast<int64_t>(b) * nh + h) * S + q0 + r] = m_used + log2f(l);
    }
    softmax_bar();  // every softmax warp has written its rows (failed warps skip only their work)
    if (threadIdx.x == 128 && !*abort_flag) {
      tma_store_2d(&tm_out, smem + FwdSmem::P, h * kHd, tok0 + q0);
      tma_store_2d(&tm_out, smem + FwdSmem::P + kAtomBytes, h * kHd + 64, tok0 + q0);
      bulk_commit();
      bulk_wait_read_all();
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int attn_forward(const AttnArgs& a, cudaStream_t s) {
  if (a.S % kBlk != 0 || a.hd != kHd || a.D != a.heads * kHd || a.ldq % 8 != 0 || a.ldo % 8 != 0) return -1;
  if (reinterpret_cast<uintptr_t>(a.out) & 15) return -1;
  CUtensorMap tm, tm_out;
  const uint64_t M = static_cast<uint64_t>(a.batch) * a.S;
  if (!make_tmap_bf16(&tm, a.qkv, static_cast<uint64_t>(3) * a.D, M, a.ldq, 64, kBlk) ||
      !make_tmap_bf16(&tm_out, a.out, static_cast<uint64_t>(a.D), M, a.ldo, 64, kBlk))
    return -3;
  const cudaError_t attr = smem_limit_once(reinterpret_cast<const void*>(attn_fwd_tc_kernel), FwdSmem::BYTES);
  if (attr != cudaSuccess) return attr;
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kHd));
  dim3 grid(a.heads, a.batch, a.S / kBlk);
  attn_fwd_tc_kernel<<<grid, kFwdThreads, FwdSmem::BYTES, s>>>(tm, tm_out, a.lse2, a.S, a.heads, scale_log2, a.err);
  return cudaGetLastError();
}


}  // namespace rt
