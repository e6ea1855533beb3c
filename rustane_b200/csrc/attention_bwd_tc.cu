// Causal attention backward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same semantics as the mma.sync kernels of attention.cu (sdpaBwd1 / sdpaBwd2,
// crates/engine/src/kernels/sdpa_bwd.rs:44-162, RoPE backward layer.rs:1880-1897):
//   P = exp2(S * scale_log2 - lse2),  dP = dO V^T,  dS = P * (dP - rowsum(dO * O)),
//   dV = P^T dO,  dK = scale * dS^T Q,  dQ = scale * dS K,
// then the RoPE backward rotation of dK and dQ.  Two kernels:
//
// attn_bwd_kv_tc_kernel — one CTA per (head, sequence, block of 128 keys),
// looping over the 128-query blocks at or after the keys (causal):
//   warp 0      TMA producer: K and V once, then Q_t, dO_t (128 x 128) into a
//               two-deep ring;
//   warp 1      one lane issues the MMAs, all 128 x 128 x 16 (the full tensor
//               rate): S^T_t = K Q_t^T and dP^T_t = V dO_t^T into TMEM, then
//               dV += P^T_t dO_t with P^T read from TMEM (the elementwise warps
//               write it in bf16 over their own S^T columns) and dK += dS^T_t Q_t;
//               issue order dV(t), S^T(t+1), dK(t), dP^T(t+1);
//   warp 2      owns the TMEM allocation (512 columns: S^T / P^T, dP^T, dV, dK);
//   warp 3      stores each dS^T tile (bf16, two 64-query halves) to the scratch
//               with TMA, for the dQ kernel;
//   warps 4-11  elementwise: two threads per key row (TMEM lane = key), 64
//               queries each: P^T = exp2(S^T * scale_log2 - lse2) (causal mask)
//               back into TMEM, dS^T = P^T * (dP^T - rowsum) in bf16 into shared
//               memory in the 128-byte-swizzled K-major layout the MMA reads;
//               lse2 / rowsum come from L2, two per lane, passed around by
//               shuffles; at the end dV and dK (scale, RoPE backward) go from
//               TMEM through swizzled shared-memory tiles to dqkv by TMA stores.
//
// attn_bwd_dq_tc_kernel — one CTA per (head, sequence, block of 128 queries):
//   dQ = sum over key blocks j of dS_j K_j (both operands MN-major in shared
//   memory: dS^T tiles as stored, K as laid out in qkv), accumulated in TMEM;
//   epilogue scale + RoPE backward -> shared memory -> TMA store into dqkv (the
//   RoPE tables are read while the MMAs run).  The dS scratch replaces atomics:
//   every dQ element is summed in a fixed order, so the result is deterministic.
//
// All waits are bounded; a timeout sets the device error word and the CTA drains.
#include "attention.h"
#include "common.cuh"
#include "kernels.h"

namespace rt {
namespace {

constexpr int kHd = 128;
constexpr int kKeys = 128;                     // keys per kv CTA (and per dQ step)
constexpr int kSub = 64;                       // queries per sub-block
constexpr int kKvTile = kKeys * kHd * 2;       // 32 KB: two 64-column atoms of 128 rows
constexpr int kKvAtom = kKvTile / 2;           // 16 KB
constexpr int kKvThreads = 384;
constexpr int kDqThreads = 256;
constexpr int kDqStages = 3;

struct KvSmem {
  static constexpr int K = 0;
  static constexpr int V = K + kKvTile;
  static constexpr int Q = V + kKvTile;        // [2] 128-query tiles
  static constexpr int DO = Q + 2 * kKvTile;   // [2]
  static constexpr int DS = DO + 2 * kKvTile;  // dS^T: 128 keys x 128 queries, two 64-query atoms
  static constexpr int BAR = DS + kKvTile;
  static constexpr int BYTES = BAR + 256 + 1024;
};
static_assert(KvSmem::BYTES <= 232448, "kv kernel shared memory");

enum KvBar : int {
  kKvFull = 0,
  kQFull = 1,    // [2] Q and dO of a 128-query block
  kQEmpty = 3,   // [2]
  kSFull = 5,    // S^T in TMEM
  kSFree = 6,    // dV of the block done: its P^T (over the S^T columns) consumed
  kDpFull = 7,   // dP^T in TMEM
  kDpFree = 8,
  kPFull = 9,    // P^T in TMEM
  kDsFull = 10,  // dS^T in shared memory
  kDsFree = 11,  // dK MMA done and the tile stored
  kAccFull = 12,
  kKvDrain = 13,
  kKvNumBars = 14
};

struct DqSmem {
  static constexpr int STAGE = 2 * kKvTile;  // dS (two 64-query tiles of 128 keys) + K_j
  static constexpr int OUT = kDqStages * STAGE;  // dQ staging for the TMA store
  static constexpr int BAR = OUT + kKvTile;
  static constexpr int BYTES = BAR + 128 + 1024;
};
static_assert(DqSmem::BYTES <= 232448, "dq kernel shared memory");

// ------------------------------------------------------------------ dK, dV
__global__ void __launch_bounds__(kKvThreads, 1)
    attn_bwd_kv_tc_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_ds, const __grid_constant__ CUtensorMap tm_out,
                          const float* __restrict__ lse2, const float* __restrict__ rowsum, int D, int S, int nh,
                          float scale, float scale_log2, const float* __restrict__ cosb,
                          const float* __restrict__ sinb, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + KvSmem::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kKvNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y, j = blockIdx.z;  // key block 0 has the most work: dispatched first
  const int nsub = S / kSub, nkb = S / kKeys;
  const int n = nkb - j;  // 128-query blocks at or after the keys
  const int tok0 = b * S;
  const int k0 = j * kKeys;
  const int bh = b * nh + h;
  const int64_t stat0 = static_cast<int64_t>(bh) * S;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kKvFull], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[kQFull + i], 1);
      mbar_init(&bar[kQEmpty + i], 1);
    }
    mbar_init(&bar[kSFull], 1);
    mbar_init(&bar[kSFree], 1);
    mbar_init(&bar[kDpFull], 1);
    mbar_init(&bar[kDpFree], 8);
    mbar_init(&bar[kPFull], 8);
    mbar_init(&bar[kDsFull], 8);
    mbar_init(&bar[kDsFree], 2);
    mbar_init(&bar[kAccFull], 1);
    mbar_init(&bar[kKvDrain], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_kv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_ds);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // TMEM columns: S^T (then P^T in bf16 pairs) [0,128), dP^T [128,256), dV [256,384), dK [384,512)
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t kColS = 0, kColDp = 128, kColDv = 256, kColDk = 384;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      const int qc = h * kHd, kc = D + h * kHd, vc = 2 * D + h * kHd;
      int issued = 0;
      mbar_arrive_expect_tx(&bar[kKvFull], 2 * kKvTile);
      tma_load_2d(smem + KvSmem::K, &tm_kv, &bar[kKvFull], kc, tok0 + k0);
      tma_load_2d(smem + KvSmem::K + kKvAtom, &tm_kv, &bar[kKvFull], kc + 64, tok0 + k0);
      tma_load_2d(smem + KvSmem::V, &tm_kv, &bar[kKvFull], vc, tok0 + k0);
      tma_load_2d(smem + KvSmem::V + kKvAtom, &tm_kv, &bar[kKvFull], vc + 64, tok0 + k0);
      for (int t = 0; t < n; ++t) {
        const int st = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&bar[kQEmpty + st], ph ^ 1) || *abort_flag) {
          set_error(err, kDevTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        const int q0 = (j + t) * kKeys;
        uint64_t* fb = &bar[kQFull + st];
        mbar_arrive_expect_tx(fb, 2 * kKvTile);
        uint8_t* sq = smem + KvSmem::Q + st * kKvTile;
        uint8_t* sd = smem + KvSmem::DO + st * kKvTile;
        tma_load_2d(sq, &tm_kv, fb, qc, tok0 + q0);
        tma_load_2d(sq + kKvAtom, &tm_kv, fb, qc + 64, tok0 + q0);
        tma_load_2d(sd, &tm_do, fb, h * kHd, tok0 + q0);
        tma_load_2d(sd + kKvAtom, &tm_do, fb, h * kHd + 64, tok0 + q0);
        issued = t + 1;
      }
      if (*abort_flag) {  // let copies still in flight land before the CTA exits
        mbar_wait(&bar[kKvFull], 0);
        for (int t = (issued > 2 ? issued - 2 : 0); t < issued; ++t) mbar_wait(&bar[kQFull + (t & 1)], (t >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      // per 128-query block t: S^T = K Q^T, dP^T = V dO^T (all 128 x 128 x 128, full rate);
      // dV += P^T dO with P^T read from TMEM; dK += dS^T Q.  Issue order dV(t), S^T(t+1),
      // dK(t), dP^T(t+1): the next block's S^T is ready while the elementwise warps finish dS^T(t).
      constexpr uint32_t idesc_kk = idesc_bf16_f32(kKeys, kKeys, false, false);
      constexpr uint32_t idesc_kn = idesc_bf16_f32(kKeys, kHd, false, true);
      const uint32_t sk = smem_u32(smem + KvSmem::K), sv = smem_u32(smem + KvSmem::V);
      const uint32_t sds = smem_u32(smem + KvSmem::DS);
      auto qaddr = [&](int t) { return smem_u32(smem + KvSmem::Q + (t & 1) * kKvTile); };
      auto daddr = [&](int t) { return smem_u32(smem + KvSmem::DO + (t & 1) * kKvTile); };
      auto issue_st = [&](int t) {
        const uint32_t sq = qaddr(t);
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kKvAtom + (kk & 3) * 32;
          umma_bf16(tmem + kColS, smem_desc_sw128(sk + off, 16, 1024), smem_desc_sw128(sq + off, 16, 1024), idesc_kk,
                    kk != 0 ? 1u : 0u);
        }
        umma_commit(&bar[kSFull]);
      };
      auto issue_dp = [&](int t) {
        const uint32_t sd = daddr(t);
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kKvAtom + (kk & 3) * 32;
          umma_bf16(tmem + kColDp, smem_desc_sw128(sv + off, 16, 1024), smem_desc_sw128(sd + off, 16, 1024), idesc_kk,
                    kk != 0 ? 1u : 0u);
        }
        umma_commit(&bar[kDpFull]);
      };
      bool ok = mbar_wait(&bar[kKvFull], 0) && mbar_wait(&bar[kQFull], 0) && !*abort_flag;
      if (ok) {
        tc_fence_after();
        issue_st(0);
        issue_dp(0);
      }
      for (int t = 0; ok && t < n; ++t) {
        const int ph = t & 1;
        // dV += P^T dO: P^T of query k-chunk kk sits in TMEM columns 8 kk (queries < 64) or 64 + 8 (kk - 4)
        if (!mbar_wait(&bar[kPFull], ph) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sd = daddr(t), sq = qaddr(t);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint32_t acol = kColS + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8);
          umma_bf16_ts(tmem + kColDv, tmem + acol, smem_desc_sw128(sd + kk * 2048, kKvAtom, 1024), idesc_kn,
                       (t | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&bar[kSFree]);
        if (t + 1 < n) {  // S^T(t+1) overwrites P^T(t): after dV(t)
          if (!mbar_wait(&bar[kQFull + ((t + 1) & 1)], ((t + 1) >> 1) & 1) || !mbar_wait(&bar[kSFree], ph) ||
              *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_st(t + 1);
        }
        // dK += dS^T Q
        if (!mbar_wait(&bar[kDsFull], ph) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)
          umma_bf16(tmem + kColDk, smem_desc_sw128(sds + (kk >> 2) * kKvAtom + (kk & 3) * 32, 16, 1024),
                    smem_desc_sw128(sq + kk * 2048, kKvAtom, 1024), idesc_kn, (t | kk) != 0 ? 1u : 0u);
        umma_commit(&bar[kDsFree]);
        umma_commit(&bar[kQEmpty + (t & 1)]);
        if (t + 1 < n) {  // dP^T(t+1) overwrites dP^T(t): after the elementwise warps have read it
          if (!mbar_wait(&bar[kDpFree], ph) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_dp(t + 1);
        }
      }
      if (!ok) {
        set_error(err, kDevTimeoutMma);
        *abort_flag = 1;
      } else {
        umma_commit(&bar[kAccFull]);
      }
      umma_commit(&bar[kKvDrain]);
      mbar_wait(&bar[kKvDrain], 0);
    }
  } else if (warp == 3) {
    if (lane == 0) {
      // ------------------------------------------------- dS^T tiles -> scratch
      // scratch row of (sequence-head bh, key block j, 64-query sub-block i): ((bh * nkb + j) * nsub + i) * 128;
      // the two 64-query halves of block t are sub-blocks 2 (j + t) and 2 (j + t) + 1
      int t = 0;
      for (; t < n; ++t) {
        if (!mbar_wait(&bar[kDsFull], t & 1) || *abort_flag) break;
        const int row = ((bh * nkb + j) * nsub + 2 * (j + t)) * kKeys;
        tma_store_2d(&tm_ds, smem + KvSmem::DS, 0, row);
        tma_store_2d(&tm_ds, smem + KvSmem::DS + kKvAtom, 0, row + kKeys);
        bulk_commit();
        bulk_wait_read_all();
        mbar_arrive(&bar[kDsFree]);
      }
      if (t < n) {
        set_error(err, kDevTimeoutEpilogue);
        *abort_flag = 1;
      }
      bulk_wait_all();
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- elementwise
    const int qw = warp & 3;            // TMEM lane quadrant: key rows 32 qw ..
    const int hh = (warp - 4) >> 2;     // query columns [64 hh, 64 hh + 64) of a block
    const int r = qw * 32 + lane;       // key row within the block
    const int kpos = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(qw * 32) << 16;
    bool ok = true;
    auto wait = [&](uint64_t* bb, uint32_t parity) {
      bool w = ok && !*abort_flag && mbar_wait(bb, parity);
      w = __all_sync(0xffffffffu, w);
      if (!w) {
        ok = false;
        *abort_flag = 1;
      }
      return w;
    };
    for (int t = 0; ok && t < n; ++t) {
      const uint32_t ph = t & 1;
      const int q0 = (j + t) * kKeys + hh * 64;  // first query of this thread's 64 columns
      // lse2 and rowsum of this warp's 64 queries: lane e holds queries q0 + e and q0 + 32 + e (from L2,
      // loaded while the MMAs run); every lane needs all 64, passed around by shuffles
      const float l0 = __ldg(lse2 + stat0 + q0 + lane), l1 = __ldg(lse2 + stat0 + q0 + 32 + lane);
      const float d0 = __ldg(rowsum + stat0 + q0 + lane), d1 = __ldg(rowsum + stat0 + q0 + 32 + lane);
      if (!wait(&bar[kSFull], ph)) break;
      tc_fence_after();
      // P^T = exp2(S^T * scale - lse) on column pairs (packed fp32x2); kept as pairs for dS^T
      uint64_t p2[32];
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + kColS + lane_off + hh * 64 + c * 32, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int e = 4 * u + 2 * h2;
            const float la = __shfl_sync(0xffffffffu, c ? l1 : l0, e);
            const float lb = __shfl_sync(0xffffffffu, c ? l1 : l0, e + 1);
            float x0, x1;
            f2_unpack(f2_sub(f2_mul(f2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), sc2), f2_pack(la, lb)),
                      x0, x1);
            float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            if (t == 0) {  // the diagonal block: a query before the key -> 0 (causal)
              const int qa = q0 + c * 32 + e;
              p0 = qa >= kpos ? p0 : 0.f;
              p1 = qa + 1 >= kpos ? p1 : 0.f;
            }
            p2[c * 16 + e / 2] = f2_pack(p0, p1);
            pk[e / 2] = pack_bf16x2(p0, p1);
          }
        }
        // P^T in bf16 pairs over this thread's own S^T columns (chunk 0, already read)
        tmem_st16(tmem + kColS + lane_off + hh * 64 + c * 16, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kPFull]);
      if (!wait(&bar[kDpFull], ph)) break;
      tc_fence_after();
      uint32_t dk[32];  // dS^T = P^T * (dP^T - rowsum) of the 64 columns, bf16 pairs
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + kColDp + lane_off + hh * 64 + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int u = 0; u < 8; ++u) {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int e = 4 * u + 2 * h2;
            const float da = __shfl_sync(0xffffffffu, c ? d1 : d0, e);
            const float db = __shfl_sync(0xffffffffu, c ? d1 : d0, e + 1);
            const uint64_t ds = f2_mul(p2[c * 16 + e / 2],
                                       f2_sub(f2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), f2_pack(da, db)));
            float x0, x1;
            f2_unpack(ds, x0, x1);
            dk[c * 16 + e / 2] = pack_bf16x2(x0, x1);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kDpFree]);
      // dS^T row r, query atom hh (64 columns = 128 B): chunk u at (u ^ r % 8) * 16
      if (!wait(&bar[kDsFree], ph ^ 1)) break;
      uint8_t* drow = smem + KvSmem::DS + hh * kKvAtom + r * 128;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<uint4*>(drow + ((u ^ (r & 7)) << 4)) =
            make_uint4(dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kDsFull]);
    }
    // RoPE tables of this key position for head-dim pairs [32 hh, 32 hh + 32), loaded
    // while the last MMAs run
    float rc[32], rs[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      rc[i] = __ldg(cosb + static_cast<int64_t>(hh * 32 + i) * S + kpos);
      rs[i] = __ldg(sinb + static_cast<int64_t>(hh * 32 + i) * S + kpos);
    }
    if (ok) wait(&bar[kAccFull], 0);
    if (!ok && lane == 0) set_error(err, kDevTimeoutEpilogue);
    if (ok) {
      tc_fence_after();
      // dK (scale, RoPE backward) and dV rows -> bf16 tiles in the (now idle) Q ring, 128-byte
      // swizzled, head-dim columns [64 hh, 64 hh + 64) = atom hh; then TMA stores into dqkv
      uint8_t* tk = smem + KvSmem::Q + hh * kKvAtom + r * 128;
      uint8_t* tv = smem + KvSmem::Q + kKvTile + hh * kKvAtom + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        float f[32];
        tmem_ld32(tmem + kColDv + lane_off + hh * 64 + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(v[e]);
        store_chunk32(tv, c, r, f);
        tmem_ld32(tmem + kColDk + lane_off + hh * 64 + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float e0 = __uint_as_float(v[e]) * scale, e1 = __uint_as_float(v[e + 1]) * scale;
          const float cc = rc[c * 16 + e / 2], ss = rs[c * 16 + e / 2];
          f[e] = cc * e0 + ss * e1;
          f[e + 1] = -ss * e0 + cc * e1;
        }
        store_chunk32(tk, c, r, f);
      }
      fence_proxy_async_smem();
    }
    // every elementwise warp reaches the named barrier (a failed warp skips only its work)
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (threadIdx.x == 128 && !*abort_flag) {
      const int y = tok0 + k0;
      tma_store_2d(&tm_out, smem + KvSmem::Q, D + h * kHd, y);
      tma_store_2d(&tm_out, smem + KvSmem::Q + kKvAtom, D + h * kHd + 64, y);
      tma_store_2d(&tm_out, smem + KvSmem::Q + kKvTile, 2 * D + h * kHd, y);
      tma_store_2d(&tm_out, smem + KvSmem::Q + kKvTile + kKvAtom, 2 * D + h * kHd + 64, y);
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

// ---------------------------------------------------------------------- dQ
// Persistent: one CTA per SM walks the (sequence, head, 128-query block) items,
// heaviest first, CTA c taking items c, 2P-1-c, 2P+c, ...; the dS / K ring runs on
// across items and the TMEM accumulator is double-buffered, so one item's
// epilogue overlaps the next item's MMAs.
__device__ __forceinline__ int dq_item(int c, int P, int t) {
  return (t >> 1) * 2 * P + ((t & 1) ? 2 * P - 1 - c : c);
}

__global__ void __launch_bounds__(kDqThreads, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_ds2,
                          const __grid_constant__ CUtensorMap tm_out, int D, int S, int nh, int batch, float scale,
                          const float* __restrict__ cosb, const float* __restrict__ sinb, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + DqSmem::BAR);
  uint64_t* full = bar;                    // [kDqStages]
  uint64_t* empty = bar + kDqStages;       // [kDqStages]
  uint64_t* acc_full = bar + 2 * kDqStages;  // [2] accumulator buffer complete
  uint64_t* acc_free = acc_full + 2;         // [2] the epilogue has read it
  uint64_t* drain = acc_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsub = S / kSub, nkb = S / kKeys;
  const int per_qb = batch * nh;
  const int n_items = nkb * per_qb;  // items [0, per_qb) are the last query block: the most key blocks
  const int P = gridDim.x, c = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kDqStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_free[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_kv);
    tma_prefetch_desc(&tm_ds2);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // accumulators: columns [0,128) and [128,256)

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, issued = 0;  // ring slots used so far / whose loads were issued
      bool ok = true;
      for (int t = 0; ok; ++t) {
        const int item = dq_item(c, P, t);
        if (item >= n_items) break;
        const int qb = nkb - 1 - item / per_qb, rem = item % per_qb;
        const int b = rem / nh, h = rem % nh, bh = b * nh + h;
        const int kc = D + h * kHd, tok0 = b * S;
        for (int jj = 0; jj <= qb; ++jj, ++g) {
          const int st = g % kDqStages;
          const uint32_t ph = (g / kDqStages) & 1;
          if (!mbar_wait(&empty[st], ph ^ 1) || *abort_flag) {
            ok = false;
            break;
          }
          uint8_t* s = smem + st * DqSmem::STAGE;
          mbar_arrive_expect_tx(&full[st], DqSmem::STAGE);
          // dS^T of sub-blocks 2 qb and 2 qb + 1 (consecutive 128-row tiles of the scratch)
          tma_load_2d(s, &tm_ds2, &full[st], 0, ((bh * nkb + jj) * nsub + 2 * qb) * kKeys);
          tma_load_2d(s + kKvTile, &tm_kv, &full[st], kc, tok0 + jj * kKeys);
          tma_load_2d(s + kKvTile + kKvAtom, &tm_kv, &full[st], kc + 64, tok0 + jj * kKeys);
          issued = g + 1;
        }
      }
      if (!ok) {  // let copies still in flight land before the CTA exits
        set_error(err, kDevTimeoutProducer);
        *abort_flag = 1;
        for (int x = (issued > kDqStages ? issued - kDqStages : 0); x < issued; ++x)
          mbar_wait(&full[x % kDqStages], (x / kDqStages) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // dQ (128 queries x 128) += dS_j (queries contiguous) K_j (head dim contiguous); K = 128 keys
      constexpr uint32_t idesc = idesc_bf16_f32(kKeys, kHd, true, true);
      bool ok = true;
      int g = 0;
      for (int t = 0; ok; ++t) {
        const int item = dq_item(c, P, t);
        if (item >= n_items) break;
        const int nb = nkb - item / per_qb;  // key blocks 0 .. qb
        const int ab = t & 1;
        if (t >= 2 && (!mbar_wait(&acc_free[ab], ((t >> 1) - 1) & 1) || *abort_flag)) {
          ok = false;
          break;
        }
        for (int jj = 0; jj < nb; ++jj, ++g) {
          const int st = g % kDqStages;
          if (!mbar_wait(&full[st], (g / kDqStages) & 1) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + st * DqSmem::STAGE), sb = sa + kKvTile;
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk)
            umma_bf16(tmem + ab * kHd, smem_desc_sw128(sa + kk * 2048, kKvAtom, 1024),
                      smem_desc_sw128(sb + kk * 2048, kKvAtom, 1024), idesc, (jj | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      if (!ok) {
        set_error(err, kDevTimeoutMma);
        *abort_flag = 1;
      }
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp >= 4) {
    const int qw = warp & 3;
    const int r = qw * 32 + lane;  // query row within the block
    const uint32_t lane_off = static_cast<uint32_t>(qw * 32) << 16;
    uint8_t* stage_out = smem + DqSmem::OUT;
    for (int t = 0;; ++t) {
      const int item = dq_item(c, P, t);
      if (item >= n_items) break;
      const int qb = nkb - 1 - item / per_qb, rem = item % per_qb;
      const int b = rem / nh, h = rem % nh;
      const int qpos = qb * kKeys + r;
      const int ab = t & 1;
      float rc[64], rs[64];  // RoPE tables of this query position, loaded while the MMAs run
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        rc[i] = __ldg(cosb + static_cast<int64_t>(i) * S + qpos);
        rs[i] = __ldg(sinb + static_cast<int64_t>(i) * S + qpos);
      }
      bool w = !*abort_flag && mbar_wait(&acc_full[ab], (t >> 1) & 1);
      w = __all_sync(0xffffffffu, w);
      if (!w) {
        if (lane == 0) set_error(err, kDevTimeoutEpilogue);
        *abort_flag = 1;
      }
      if (threadIdx.x == 128) bulk_wait_read_all();  // the previous item's dQ has left the staging tile
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
      if (w) {
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t v[32];
          float f[32];
          tmem_ld32(tmem + ab * kHd + lane_off + cc * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float d0 = __uint_as_float(v[e]) * scale, d1 = __uint_as_float(v[e + 1]) * scale;
            const float co = rc[cc * 16 + e / 2], si = rs[cc * 16 + e / 2];
            f[e] = co * d0 + si * d1;
            f[e + 1] = -si * d0 + co * d1;
          }
          store_chunk32(stage_out + (cc >> 1) * kKvAtom + r * 128, cc & 1, r, f);
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[ab]);  // this accumulator can take the item after next
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 128 && !*abort_flag) {
        const int y = b * S + qb * kKeys;
        tma_store_2d(&tm_out, stage_out, h * kHd, y);
        tma_store_2d(&tm_out, stage_out + kKvAtom, h * kHd + 64, y);
        bulk_commit();
      }
    }
    if (threadIdx.x == 128) bulk_wait_read_all();
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

size_t attn_bwd_scratch_bytes(int batch, int S, int heads) {
  return static_cast<size_t>(batch) * heads * S * S * 2;
}

int attn_backward_tc(const AttnArgs& a, cudaStream_t s) {
  if (a.S % kKeys != 0 || a.hd != kHd || a.D != a.heads * kHd || a.ldq % 8 != 0 || a.lddo % 8 != 0 ||
      a.lddq % 8 != 0 || !a.ds_scratch)
    return -1;
  if ((reinterpret_cast<uintptr_t>(a.lse2) | reinterpret_cast<uintptr_t>(a.dvec) |
       reinterpret_cast<uintptr_t>(a.ds_scratch) | reinterpret_cast<uintptr_t>(a.dqkv)) & 15)
    return -1;
  const uint64_t M = static_cast<uint64_t>(a.batch) * a.S;
  const uint64_t ds_rows = static_cast<uint64_t>(a.batch) * a.heads * a.S * a.S / kSub;
  CUtensorMap tm_kv, tm_do, tm_ds, tm_ds2, tm_out;
  if (!make_tmap_bf16(&tm_kv, a.qkv, 3 * static_cast<uint64_t>(a.D), M, a.ldq, 64, kKeys) ||
      !make_tmap_bf16(&tm_do, a.dout, static_cast<uint64_t>(a.D), M, a.lddo, 64, kKeys) ||
      !make_tmap_bf16(&tm_ds, a.ds_scratch, kSub, ds_rows, kSub, 64, kKeys) ||
      !make_tmap_bf16(&tm_ds2, a.ds_scratch, kSub, ds_rows, kSub, 64, 2 * kKeys) ||
      !make_tmap_bf16(&tm_out, a.dqkv, 3 * static_cast<uint64_t>(a.D), M, a.lddq, 64, kKeys))
    return -3;
  const cudaError_t attr1 = smem_limit_once(reinterpret_cast<const void*>(attn_bwd_kv_tc_kernel), KvSmem::BYTES);
  const cudaError_t attr2 = smem_limit_once(reinterpret_cast<const void*>(attn_bwd_dq_tc_kernel), DqSmem::BYTES);
  if (attr1 != cudaSuccess) return attr1;
  if (attr2 != cudaSuccess) return attr2;
  if (!a.dvec_ready) {
    const int rc = attn_bwd_rowsum(a, s);
    if (rc) return rc;
  }
  const float scale = 1.0f / sqrtf(static_cast<float>(kHd));
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(a.heads, a.batch, a.S / kKeys);
  attn_bwd_kv_tc_kernel<<<grid, kKvThreads, KvSmem::BYTES, s>>>(tm_kv, tm_do, tm_ds, tm_out, a.lse2, a.dvec, a.D,
                                                               a.S, a.heads, scale, scale_log2, a.rope_cos_b,
                                                               a.rope_sin_b, a.err);
  const int dq_items = (a.S / kKeys) * a.batch * a.heads;
  const int dq_grid = dq_items < num_sms() ? dq_items : num_sms();
  attn_bwd_dq_tc_kernel<<<dq_grid, kDqThreads, DqSmem::BYTES, s>>>(tm_kv, tm_ds2, tm_out, a.D, a.S, a.heads, a.batch,
                                                                   scale, a.rope_cos_b, a.rope_sin_b, a.err);
  return cudaGetLastError();
}

}  // namespace rt
