// Causal attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same semantics and layout as the mma.sync kernels in attention.cu
// (crates/engine/src/kernels/sdpa_fwd.rs:130-150): per (sequence, head, block
// of 128 queries), S = Q K^T / sqrt(128) with the causal mask, P = softmax(S),
// O = P V; O [M, D] bf16 and the log2-domain statistic lse2 = max + log2(sum)
// that the backward kernels use to rebuild P.
//
// Persistent: one CTA per SM walks a fixed list of work items (sequence, head,
// 128-query block), heaviest first (the causal block with the most key blocks),
// CTA c taking items c, 2P-1-c, 2P+c, 4P-1-c, ... (P CTAs) so the per-CTA key
// block counts even out.  TMEM is allocated and the barriers initialised once;
// the K/V ring, the S buffers and their barrier phases run on across items, so
// the next item's Q load and first S MMA overlap this item's last P V product
// and its epilogue.  384 threads:
//   warp 0      TMA producer: Q of each item, then K_j and V_j (128 keys x
//               128) into two-deep rings;
//   warp 1      one lane issues the MMAs: S_j = Q K_j^T into one of two TMEM
//               S buffers (128 columns each), O += P_j V_j into the item's TMEM
//               O buffer (two, alternating by item, so one item's epilogue reads
//               its O while the next accumulates); S_{j+1} is issued before
//               O += P_j V_j so the softmax of block j+1 overlaps the P V product
//               of block j;
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
// All waits are bounded; a timeout sets the device error word and every role
// runs out its item list without waiting, then the CTA drains and exits.
#include "attention.h"
#include "common.cuh"
#include "kernels.h"

namespace rt {
namespace {

constexpr int kHd = 128;
constexpr int kBlk = 128;                    // queries per work item and keys per KV block
constexpr int kTileBytes = kBlk * kHd * 2;   // 32 KB: two 64-column swizzle atoms of 128 rows
constexpr int kAtomBytes = kTileBytes / 2;   // 16 KB
constexpr int kFwdThreads = 384;   // 8 softmax warps, two threads per query row
constexpr float kRescaleLog2 = 8.0f;         // keep a stale row max while P stays <= 2^8

struct FwdSmem {
  static constexpr int Q = 0;
  static constexpr int K = Q + kTileBytes;          // [2]
  static constexpr int V = K + 2 * kTileBytes;      // [2]
  static constexpr int O = V + 2 * kTileBytes;      // O / l staging for the TMA store
  static constexpr int RED = O + kTileBytes;        // float [2 parities][2 halves][128 rows]: row max
  static constexpr int SUM = RED + 2 * 2 * kBlk * 4; // float [2 halves][128 rows]: row sum
  static constexpr int BAR = SUM + 2 * kBlk * 4;
  static constexpr int BYTES = BAR + 256 + 1024;    // barriers, TMEM slot, alignment slack
};

enum Bar : int {
  kQFull = 0,
  kQEmpty = 1,  // every S MMA of the item done: Q can take the next item
  kKFull = 2,   // [2]
  kKEmpty = 4,  // [2]
  kVFull = 6,   // [2]
  kVEmpty = 8,  // [2]
  kSFull = 10,  // [2]
  kSFree = 12,  // [2]
  kPFull = 14,
  kPvDone = 15, // [2] by S buffer: the P V product of a block read its P
  kOFree = 17,  // [2] the epilogue has read O buffer 0 / 1
  kDrain = 19,
  kNumBars = 20
};
static_assert(kNumBars * 8 + 8 <= 256, "barrier area");

// Work item t of CTA c (P CTAs, n items, heaviest first): c, 2P-1-c, 2P+c, 4P-1-c, ...
// The sequence grows with t, so the first index >= n ends the CTA's list.
__device__ __forceinline__ int fwd_item(int c, int P, int t) {
  return (t >> 1) * 2 * P + ((t & 1) ? 2 * P - 1 - c : c);
}

__device__ __forceinline__ void softmax_bar() {  // the 8 softmax warps only
  asm volatile("bar.sync 1, 256;" ::: "memory");
}
// The two softmax warps that share TMEM lane quadrant qw (warps 4 + qw and 8 + qw hold the
// two column halves of the same 32 query rows) meet here to exchange their row maxima.
__device__ __forceinline__ void row_pair_bar(int qw) {
  asm volatile("bar.sync %0, 64;" ::"r"(2 + qw) : "memory");
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_out,
                       float* __restrict__ lse2, int S, int nh, int batch, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + FwdSmem::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = S / kBlk;           // query blocks per (sequence, head)
  const int per_qb = batch * nh;     // work items per query-block level
  const int n_items = nq * per_qb;   // items [0, per_qb) are the last query block: the most key blocks
  const int P = gridDim.x, c = blockIdx.x;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kQFull], 1);
    mbar_init(&bar[kQEmpty], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[kKFull + i], 1);
      mbar_init(&bar[kKEmpty + i], 1);
      mbar_init(&bar[kVFull + i], 1);
      mbar_init(&bar[kVEmpty + i], 1);
      mbar_init(&bar[kSFull + i], 1);
      mbar_init(&bar[kSFree + i], 1);
      mbar_init(&bar[kOFree + i], 8);
    }
    mbar_init(&bar[kPFull], 8);
    mbar_init(&bar[kPvDone], 1);
    mbar_init(&bar[kPvDone + 1], 1);
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
  const uint32_t tmem = *tmem_slot;  // columns [0,128) S0, [128,256) S1, [256,384) O0, [384,512) O1

  if (warp == 0) {
    if (lane == 0) {
      // --------------------------------------------------------------- producer
      const int D = nh * kHd;
      int g = 0;                            // K/V blocks of the items so far
      int q_issued = 0, k_issued = 0, v_issued = 0;
      bool ok = true;
      for (int t = 0, it = 0; ok; ++t, ++it) {
        const int item = fwd_item(c, P, t);
        if (item >= n_items) break;
        const int qb = nq - 1 - item / per_qb, rem = item % per_qb;
        const int b = rem / nh, h = rem % nh;
        const int tok0 = b * S;
        const int qc = h * kHd, kc = D + h * kHd, vc = 2 * D + h * kHd;
        if (it > 0 && (!mbar_wait(&bar[kQEmpty], (it - 1) & 1) || *abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bar[kQFull], kTileBytes);
        tma_load_2d(smem + FwdSmem::Q, &tm_qkv, &bar[kQFull], qc, tok0 + qb * kBlk);
        tma_load_2d(smem + FwdSmem::Q + kAtomBytes, &tm_qkv, &bar[kQFull], qc + 64, tok0 + qb * kBlk);
        q_issued = it + 1;
        for (int j = 0; j <= qb; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          const int row = tok0 + j * kBlk;
          if (!mbar_wait(&bar[kKEmpty + st], ph ^ 1) || *abort_flag) {
            ok = false;
            break;
          }
          uint8_t* sk = smem + FwdSmem::K + st * kTileBytes;
          mbar_arrive_expect_tx(&bar[kKFull + st], kTileBytes);
          tma_load_2d(sk, &tm_qkv, &bar[kKFull + st], kc, row);
          tma_load_2d(sk + kAtomBytes, &tm_qkv, &bar[kKFull + st], kc + 64, row);
          k_issued = g + 1;
          if (!mbar_wait(&bar[kVEmpty + st], ph ^ 1) || *abort_flag) {
            ok = false;
            break;
          }
          uint8_t* sv = smem + FwdSmem::V + st * kTileBytes;
          mbar_arrive_expect_tx(&bar[kVFull + st], kTileBytes);
          tma_load_2d(sv, &tm_qkv, &bar[kVFull + st], vc, row);
          tma_load_2d(sv + kAtomBytes, &tm_qkv, &bar[kVFull + st], vc + 64, row);
          v_issued = g + 1;
        }
      }
      if (!ok) {  // let copies still in flight land before the CTA exits
        set_error(err, kDevTimeoutProducer);
        *abort_flag = 1;
        if (q_issued > 0) mbar_wait(&bar[kQFull], (q_issued - 1) & 1);
        for (int x = (k_issued > 2 ? k_issued - 2 : 0); x < k_issued; ++x)
          mbar_wait(&bar[kKFull + (x & 1)], (x >> 1) & 1);
        for (int x = (v_issued > 2 ? v_issued - 2 : 0); x < v_issued; ++x)
          mbar_wait(&bar[kVFull + (x & 1)], (x >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = idesc_bf16_f32(kBlk, kBlk, false, false);  // Q, K: both hd-contiguous
      constexpr uint32_t idesc_o = idesc_bf16_f32(kBlk, kHd, false, true);    // P key-contiguous, V hd-contiguous
      const uint32_t sq = smem_u32(smem + FwdSmem::Q);
      auto issue_s = [&](int gg) -> bool {
        const int st = gg & 1;
        const uint32_t ph = (gg >> 1) & 1;
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
      bool ok = true;
      int g = 0;
      for (int t = 0, it = 0; ok; ++t, ++it) {
        const int item = fwd_item(c, P, t);
        if (item >= n_items) break;
        const int nb = nq - item / per_qb;  // causal: key blocks 0 .. qb
        const int ob = it & 1;
        if (!mbar_wait(&bar[kQFull], it & 1) || *abort_flag || !issue_s(g)) {
          ok = false;
          break;
        }
        for (int j = 0; j < nb; ++j, ++g) {
          if (j + 1 < nb) {
            if (!issue_s(g + 1)) {
              ok = false;
              break;
            }
          } else {
            umma_commit(&bar[kQEmpty]);  // every S MMA of the item issued: Q is free once they complete
          }
          const int st = g & 1;
          if (!mbar_wait(&bar[kPFull], g & 1) || !mbar_wait(&bar[kVFull + st], (g >> 1) & 1) || *abort_flag ||
              (j == 0 && it >= 2 && !mbar_wait(&bar[kOFree + ob], ((it >> 1) - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sv = smem_u32(smem + FwdSmem::V + st * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kBlk / 16; ++kk) {
            // P from TMEM (bf16 pairs over the S columns: keys 16 kk.. at column 8 kk, or 64 + 8 (kk - 4)
            // for the second half); V: hd-contiguous rows, 16 keys = 2 KB
            const uint32_t acol = st * kBlk + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8);
            umma_bf16_ts(tmem + (2 + ob) * kBlk, tmem + acol, smem_desc_sw128(sv + kk * 2048, kAtomBytes, 1024),
                         idesc_o, (j | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&bar[kVEmpty + st]);
          umma_commit(&bar[kPvDone + st]);
          umma_commit(&bar[kSFree + st]);  // P (over S) consumed: the buffer can take the block after next
        }
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
    // A failed (timed-out) wait does not leave the loops: every softmax warp must
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
    int g = 0;
    for (int t = 0, it = 0;; ++t, ++it) {
      const int item = fwd_item(c, P, t);
      if (item >= n_items) break;
      const int qb = nq - 1 - item / per_qb, rem = item % per_qb;
      const int b = rem / nh, h = rem % nh;
      const int nb = qb + 1, tok0 = b * S, q0 = qb * kBlk;
      const int ob = it & 1;
      const uint32_t to = tmem + (2 + ob) * kBlk + lane_off + hh * 64;  // this thread's O columns
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nb; ++j, ++g) {
        const int st = g & 1;
        wait(&bar[kSFull + st], (g >> 1) & 1);
        tc_fence_after();
        const uint32_t ts = tmem + st * kBlk + lane_off + hh * 64;
        uint32_t v[64];
        tmem_ld32(ts, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(ts + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_ld_wait();
        // keys past the query are masked in the diagonal block (key column 64 hh + e vs row r):
        // their scores become -inf, so the max and P below need no per-element test
        if (j == qb) {
          const int lim = r - hh * 64;  // valid columns e <= lim
#pragma unroll
          for (int e = 0; e < 64; ++e)
            if (e > lim) v[e] = __float_as_uint(-INFINITY);
        }
        // row max of the 64 columns: four independent chains of three-input max
        float mc[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t* w = v + 16 * q;
          mc[q] = fmax3(__uint_as_float(w[0]), __uint_as_float(w[1]), __uint_as_float(w[2]));
#pragma unroll
          for (int e = 3; e < 15; e += 2) mc[q] = fmax3(mc[q], __uint_as_float(w[e]), __uint_as_float(w[e + 1]));
          mc[q] = fmaxf(mc[q], __uint_as_float(w[15]));
        }
        float mx = fmax3(mc[0], mc[1], fmaxf(mc[2], mc[3]));
        red[(st * 2 + hh) * kBlk + r] = mx;
        row_pair_bar(qw);
        mx = fmaxf(red[(st * 2) * kBlk + r], red[(st * 2 + 1) * kBlk + r]);
        const float m_new = fmaxf(m_used, mx * scale_log2);
        if (j == 0) {
          m_used = m_new;
        } else if (__any_sync(0xffffffffu, m_new > m_used + kRescaleLog2)) {
          // rescale this warp's half of the O rows (warp-wide TMEM access; factor 1 where the max held)
          // once the P V product of the block before is done; without a rescale, P of this block (over
          // the other S buffer) is written while that product still runs
          wait(&bar[kPvDone + ((g - 1) & 1)], ((g - 1) >> 1) & 1);
          tc_fence_after();
          const bool grow = m_new > m_used + kRescaleLog2;
          const float f = grow ? exp2f(m_used - m_new) : 1.f;
          if (grow) {
            l *= f;
            m_used = m_new;
          }
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            uint32_t o[32];
            tmem_ld32(to + cc * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st32(to + cc * 32, o);
          }
          tmem_st_wait();
        }
        // P = exp2(S * scale - m) in bf16 pairs, written back over this thread's own (already
        // read) S columns: keys 64 hh + 2 i, + 1 at column 64 hh + i; the P V MMA reads it there.
        // Pairs of columns go through the packed fp32x2 multiply-add and add (masked: 2^-inf = 0).
        const uint64_t sc2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(-m_used, -m_used);
        uint64_t ls2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t pk[16];
#pragma unroll
          for (int tt = 0; tt < 16; ++tt) {
            const int e = cc * 32 + 2 * tt;
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), sc2, nm2), x0, x1);
            const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            ls2[cc] = f2_add(ls2[cc], f2_pack(p0, p1));
            pk[tt] = pack_bf16x2(p0, p1);
          }
          tmem_st16(ts + cc * 16, pk);
        }
        {
          float a0, a1, b0, b1;
          f2_unpack(ls2[0], a0, a1);
          f2_unpack(ls2[1], b0, b1);
          l += (a0 + a1) + (b0 + b1);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[kPFull]);
      }
      wait(&bar[kPvDone + ((g - 1) & 1)], ((g - 1) >> 1) & 1);  // the item's last P V product
      sum[hh * kBlk + r] = l;
      if (threadIdx.x == 128) bulk_wait_read_all();  // the previous item's O store has left the staging tile
      softmax_bar();
      l = sum[r] + sum[kBlk + r];
      if (ok) {
        // O / l in bf16 into the staging tile, 128-byte swizzled, head-dim columns
        // [64 hh, 64 hh + 64) = atom hh; one TMA store per atom below
        tc_fence_after();
        const float inv_l = 1.f / l;
        uint8_t* orow = smem + FwdSmem::O + hh * kAtomBytes + r * 128;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t o[32];
          float f[32];
          tmem_ld32(to + cc * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(o[e]) * inv_l;
          store_chunk32(orow, cc, r, f);
        }
        fence_proxy_async_smem();
        if (hh == 0) lse2[(static_cast<int64_t>(b) * nh + h) * S + q0 + r] = m_used + log2f(l);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kOFree + ob]);  // this O buffer can take the item after next
      softmax_bar();  // every softmax warp has written its rows (failed warps skip only their work)
      if (threadIdx.x == 128 && !*abort_flag) {
        tma_store_2d(&tm_out, smem + FwdSmem::O, h * kHd, tok0 + q0);
        tma_store_2d(&tm_out, smem + FwdSmem::O + kAtomBytes, h * kHd + 64, tok0 + q0);
        bulk_commit();
      }
    }
    if (threadIdx.x == 128) bulk_wait_read_all();
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
  const int n_items = (a.S / kBlk) * a.batch * a.heads;
  const int grid = n_items < num_sms() ? n_items : num_sms();
  attn_fwd_tc_kernel<<<grid, kFwdThreads, FwdSmem::BYTES, s>>>(tm, tm_out, a.lse2, a.S, a.heads, a.batch, scale_log2,
                                                               a.err);
  return cudaGetLastError();
}


}  // namespace rt
