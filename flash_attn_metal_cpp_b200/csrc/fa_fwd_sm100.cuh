// fa_fwd_sm100.cuh - FlashAttention-2 forward kernel for B200 (sm_100a).
//
// Computes, per (batch, query head, 256-row query block), the online-softmax
// attention of the reference kernel (kernels/flash_attention_fwd_optimized.metal:79-221:
// running max m, running sum l, O rescale by exp(m_old - m_new), final O / l),
// with the score scale applied before the mask (.metal:138-143) and the
// top-left causal mask (key k masked for query q iff k > q, common.metal:90-92).
// GQA reads KV head h / group (common.metal:215-217).
//
// Blackwell mapping: one CTA = two 128-row query tiles (t = 0, 1) of one
// (batch, query head), 12 warps:
//   warps 0-3   softmax of tile 0, warps 4-7 softmax of tile 1: thread r of a
//               warpgroup owns query row r = TMEM lane r of its tile. These two
//               warpgroups take the registers the third gives up (setmaxnreg).
//   warps 8,10  TMA producers: warp 8 loads Q_0, Q_1 once and K_j into an
//               NS-stage ring, warp 10 loads V_j into its own NS-stage ring
//               (128B-swizzled boxes of 64 columns).
//   warp 9      MMA issuer (one thread); warp 11 idle. Per KV tile j, in this order:
//               O_0 += P_0 V_{j-1}; S_0 = Q_0 K_j^T; O_1 += P_1 V_{j-1}; S_1 = Q_1 K_j^T
//               (tcgen05.mma kind::f16, fp32 accumulate in TMEM). While the
//               tensor cores run one tile's MMAs, the other tile's softmax runs.
// Softmax of tile t at step j: load the S_t row (tcgen05.ld), mask only
// diagonal / tail tiles, update the running max lazily (O_t is rescaled in
// TMEM only when the max grows by more than 2^8), and write
// P = exp2(S*scale*log2e - m) as fp16 into the first 64 columns of S_t's own
// TMEM region; the PV MMA reads it from there as its A operand and the next
// S_t MMA, issued after that PV by the same thread, overwrites it. The S_t
// commit also covers the previous PV_t, so O_t is stable when the softmax
// sees S_t. At the end each softmax warpgroup normalises O_t, stores it with
// 16-byte stores and writes LSE.
// Causal tiles beyond the diagonal are never loaded or computed.
//
// TMEM columns: S_0/P_0 [0,128) S_1/P_1 [128,256) O_0 [256,256+D) O_1 [384,384+D).
#pragma once
#include "fa_internal.h"
#include "fa_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

namespace fa {
namespace sm100 {

constexpr int BM = 128;          // query rows per tile (= TMEM lanes)
constexpr int NT = 2;            // query tiles per CTA
constexpr int BN = 128;          // keys per KV tile
constexpr int kThreads = 384;    // 2 softmax warpgroups + 1 warpgroup with the producer and MMA warps
constexpr int kProducerWarp = 8, kMmaWarp = 9, kProducerVWarp = 10;
// Register split: launched at 168 per thread (384 x 168 = 64512); the
// producer/MMA warpgroup drops to 72 and the softmax warpgroups rise to 216:
// 2 * 128 * 216 + 128 * 72 = 64512, exactly the launch allocation.
constexpr uint32_t kRegsLaunch = 168, kRegsSoftmax = 216, kRegsOther = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsOther <= kThreads * kRegsLaunch, "register split exceeds launch");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;  // + t * 128
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale when max grows by > 2^8
// Of every 16 exp2 pairs, this many run as a polynomial on the FMA pipe
// (exp2_poly2) instead of MUFU ex2, per head dim. Measured at D = 128
// (cfg4 / cfg5a kernel TFLOP/s): 0 -> 1078 / 1075, 2 -> 1063 / 1055,
// 4 -> 1051 / 1036, 6 -> 1032 / 1010; the extra FMA-pipe instructions cost
// more issue slots (and power, under the power cap) than the MUFU time they
// save. At D = 64 a step has half the MMA work for the same exponentials,
// and 2 of 16 pays (cfg2 / D=64 causal S8192 kernel TFLOP/s: 0 -> 376 / 635,
// 2 -> 385 / 649, 4 -> 376 / 641, 6 -> 359 / 630).
template <int D>
constexpr int poly_pairs() { return D == 64 ? 2 : 0; }

template <int D>
struct Cfg {
  static constexpr int NBOX = D / 64;                  // 64-col (128 B) boxes per row
  static constexpr int BOX_BYTES = 128 * 128;          // 128 rows x 128 B
  static constexpr int TILE_BYTES = NBOX * BOX_BYTES;  // one Q / K / V tile
  static constexpr int NS = (D == 128) ? 2 : 4;        // stages of the K ring and of the V ring
  static constexpr int OFF_Q = 0;                      // NT query tiles
  static constexpr int OFF_K = NT * TILE_BYTES;
  static constexpr int OFF_V = OFF_K + NS * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_V + NS * TILE_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;  // + barriers + alignment slack
};

struct Bars {
  uint64_t q_full[NT];
  uint64_t s_full[NT];
  uint64_t p_full[NT][2];    // P of keys [0, 64) and [64, 128) written to TMEM
  uint64_t o_full[NT];
  uint64_t mma_final;
  uint64_t k_full[4];
  uint64_t v_full[4];
  uint64_t k_empty[4];
  uint64_t v_empty[4];
  uint32_t tmem_base;
  int abort_flag;
};

template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const float* v);

template <>
__device__ __forceinline__ void store_row32<__half>(__half* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 w;
    w.x = pack_half2(v[8 * i + 0], v[8 * i + 1]);
    w.y = pack_half2(v[8 * i + 2], v[8 * i + 3]);
    w.z = pack_half2(v[8 * i + 4], v[8 * i + 5]);
    w.w = pack_half2(v[8 * i + 6], v[8 * i + 7]);
    d[i] = w;
  }
}

template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 w;
    w.x = pack_bf162(v[8 * i + 0], v[8 * i + 1]);
    w.y = pack_bf162(v[8 * i + 2], v[8 * i + 3]);
    w.z = pack_bf162(v[8 * i + 4], v[8 * i + 5]);
    w.w = pack_bf162(v[8 * i + 6], v[8 * i + 7]);
    d[i] = w;
  }
}

template <>
__device__ __forceinline__ void store_row32<float>(float* dst, const float* v) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// EXT: the sliding-window and ALiBi variant (common.metal:95-128). Without
// it those code paths are compiled out, so the plain kernel keeps its
// critical path (the per-step softmax) free of their checks.
template <int D, bool CAUSAL, bool QK_BF16, typename OutT, bool EXT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::OFF_BAR);
  const uint32_t sQ = smem_addr(smem + C::OFF_Q);
  const uint32_t sK = smem_addr(smem + C::OFF_K);
  const uint32_t sV = smem_addr(smem + C::OFF_V);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const unsigned long long wlim = a.wait_limit_ns ? a.wait_limit_ns : kWaitLimitNs;

  // Work item. (batch, KV head) units are taken in groups whose K/V fit in
  // L2 (units_per_group, chosen on the host), one group after another, so
  // the CTAs in flight re-read K/V tiles from L2 (with every unit in flight
  // at once a cfg4 launch moved 2.06 GB of DRAM traffic instead of 0.63 GB).
  // Inside a group the heaviest causal blocks come first across the group's
  // units (longest rows first keeps the launch's tail short), then the unit,
  // then the group's query heads, adjacent.
  const int n_blocks = (a.q_end - a.q_begin + NT * BM - 1) / (NT * BM);
  const int n_units = a.B * a.Hk;
  const int gu = a.units_per_group;
  const int per_group = gu * n_blocks * a.group;
  const int grp = blockIdx.x / per_group;
  const int rem = blockIdx.x - grp * per_group;
  const int per_rank = min(gu, n_units - grp * gu) * a.group;  // the last group may be smaller
  const int blk_rank = rem / per_rank;
  const int r2 = rem - blk_rank * per_rank;
  const int unit = grp * gu + r2 / a.group;
  const int bz = unit / a.Hk;
  const int hk = unit - bz * a.Hk;
  const int hq = hk * a.group + (r2 - (r2 / a.group) * a.group);
  const int blk = CAUSAL ? (n_blocks - 1 - blk_rank) : blk_rank;
  const int q0 = a.q_begin + blk * NT * BM;

  // KV tiles of each query tile: absolute tiles [jlo, jhi) counted from
  // kv_begin in steps of BN. The causal mask and the right side of a sliding
  // window cap the last tile; the left side of the window skips whole tiles
  // before the first visible key. The CTA streams tiles [j_min, j_min + n_kv)
  // through its K/V rings (ring index j); tile t takes part in ring indices
  // [s_lo[t], s_lo[t] + n_kv_t[t]).
  int s_lo[NT], n_kv_t[NT];
  int j_min = 0x7fffffff, j_max = 0;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int r0 = q0 + t * BM;
    int lo = 0, hi = 0;
    if (r0 < a.q_end) {
      const int r_last = min(r0 + BM, a.q_end) - 1;
      long long kv_hi = a.kv_end;
      if (CAUSAL) kv_hi = min(kv_hi, (long long)r_last + 1);
      int kv_lo = a.kv_begin;
      if constexpr (EXT) {
        if (a.win_right >= 0) kv_hi = min(kv_hi, (long long)r_last + a.win_right + 1);
        if (a.win_left >= 0) kv_lo = max(kv_lo, r0 - a.win_left);
      }
      if (kv_hi > kv_lo) {
        lo = EXT ? (kv_lo - a.kv_begin) / BN : 0;
        hi = (int)((kv_hi - a.kv_begin + BN - 1) / BN);
      }
    }
    s_lo[t] = lo;
    n_kv_t[t] = hi - lo;
    if (hi > lo) {
      j_min = min(j_min, lo);
      j_max = max(j_max, hi);
    }
  }
  if constexpr (!EXT) j_min = 0;  // every tile starts at the first key
  const int n_kv = (j_max > 0) ? j_max - j_min : 0;
  if constexpr (EXT) {
#pragma unroll
    for (int t = 0; t < NT; ++t) s_lo[t] -= (n_kv > 0) ? j_min : 0;  // ring-relative
  }

  if (threadIdx.x == kProducerWarp * 32) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      mbar_init(smem_addr(&bars->q_full[t]), 1);
      mbar_init(smem_addr(&bars->s_full[t]), 1);
      mbar_init(smem_addr(&bars->p_full[t][0]), 4);  // one arrival per softmax warp
      mbar_init(smem_addr(&bars->p_full[t][1]), 4);
      mbar_init(smem_addr(&bars->o_full[t]), 1);
    }
    mbar_init(smem_addr(&bars->mma_final), 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(smem_addr(&bars->k_full[s]), 1);
      mbar_init(smem_addr(&bars->v_full[s]), 1);
      mbar_init(smem_addr(&bars->k_empty[s]), 1);
      mbar_init(smem_addr(&bars->v_empty[s]), 1);
    }
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_addr(&bars->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  // Launched as a programmatic dependent of the staging pass (or whatever
  // kernel ran before it on the stream): the set-up above overlaps that
  // kernel's end; no global memory is touched before this wait.
  grid_dep_wait();
  grid_dep_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;
  if (warp >= 8) {
    reg_alloc_dec<kRegsOther>();
    if ((warp == kProducerWarp || warp == kProducerVWarp) && lane == 0 && n_kv > 0) {
      // -------------------------------------------------------- producers
      // warp 8 streams Q_0, Q_1 and the K ring, warp 10 the V ring. K_j is
      // released right after the S MMAs of step j, V_j after the PV MMAs of
      // step j+1, so each ring refills as early as its consumer allows.
      const bool is_k = (warp == kProducerWarp);
      const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
      const uint32_t ring = is_k ? sK : sV;
      uint64_t* full = is_k ? bars->k_full : bars->v_full;
      uint64_t* empty = is_k ? bars->k_empty : bars->v_empty;
      prefetch_tmap(tm);
      if (is_k) {
        prefetch_tmap(&tm_q);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (n_kv_t[t] == 0) continue;
          const uint32_t bq = smem_addr(&bars->q_full[t]);
          mbar_arrive_expect_tx(bq, C::TILE_BYTES);
#pragma unroll
          for (int bx = 0; bx < C::NBOX; ++bx)
            tma_load_4d(sQ + t * C::TILE_BYTES + bx * C::BOX_BYTES, &tm_q, bq, bx * 64, hq, q0 + t * BM, bz);
        }
      }
      // Test hook (AttnArgs::skip_k_tile): CTA 0 never loads one K tile, so
      // the MMA thread's wait for it runs out and the kernel takes its abort
      // path. Off (0) in every production launch.
      const int skip_j = (is_k && blockIdx.x == 0) ? a.skip_k_tile - 1 : -1;
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        if (*abort_flag) break;
        const int st = j % C::NS;
        if (!fa_wait(smem_addr(&empty[st]), ((j / C::NS) + 1) & 1, a.status, wlim)) {
          *abort_flag = 1;
          break;
        }
        if (j == skip_j) continue;
        const uint32_t bfull = smem_addr(&full[st]);
        mbar_arrive_expect_tx(bfull, C::TILE_BYTES);
#pragma unroll
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_4d(ring + st * C::TILE_BYTES + bx * C::BOX_BYTES, tm, bfull, bx * 64, hk,
                      a.kv_begin + (j_min + j) * BN, bz);
        issued = j + 1;
      }
      // Never leave the CTA with bulk copies still writing shared memory.
      if (is_k) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (n_kv_t[t] > 0) fa_wait(smem_addr(&bars->q_full[t]), 0, a.status, wlim);
      }
      for (int j = max(0, issued - C::NS); j < issued; ++j)
        if (j != skip_j) fa_wait(smem_addr(&full[j % C::NS]), (j / C::NS) & 1, a.status, wlim);
    } else if (warp == kMmaWarp && lane == 0 && n_kv > 0) {
      // -------------------------------------------------------- MMA issuer
      constexpr uint32_t fmt_qk = QK_BF16 ? 1u : 0u;
      constexpr uint32_t idesc_s = make_idesc(BM, BN, fmt_qk, 0, 0);
      constexpr uint32_t idesc_o = make_idesc(BM, D, 0 /*f16*/, 0, 1 /*V is MN-major*/);
      // Descriptor words: the high words are fixed per operand kind; the low
      // words hold the start address (>> 4), advanced by constant offsets.
      const uint64_t qk_desc0 = smem_desc(smem_addr(smem), 16, 1024);        // K-major Q / K tiles
      const uint64_t v_desc0 = smem_desc(sV, C::BOX_BYTES, 1024);             // MN-major V tiles
      const uint32_t qk_lo0 = (uint32_t)qk_desc0, qk_hi = (uint32_t)(qk_desc0 >> 32);
      const uint32_t v_lo0 = (uint32_t)v_desc0, v_hi = (uint32_t)(v_desc0 >> 32);
      bool ok = true;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (ok && n_kv_t[t] > 0) ok = fa_wait(smem_addr(&bars->q_full[t]), 0, a.status, wlim);
      // j runs one past the last KV tile to issue the final PV of each tile.
      for (int j = 0; ok && j <= n_kv; ++j) {
        if (*abort_flag) { ok = false; break; }
        bool k_ready = false, v_ready = false;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint32_t tS = tmem + kColS + t * 128;
          const uint32_t tO = tmem + kColO + t * 128;
          if (j >= 1 && j - 1 >= s_lo[t] && j - 1 < s_lo[t] + n_kv_t[t]) {
            // O_t += P_t V_{j-1}: P from TMEM (first 64 columns of S_t), V MN-major from smem.
            const int i = j - 1;
            const int it = i - s_lo[t];  // this tile's step
            if (!v_ready) {
              if (!fa_wait(smem_addr(&bars->v_full[i % C::NS]), (i / C::NS) & 1, a.status, wlim)) { ok = false; break; }
              v_ready = true;
            }
            // 16 keys x D cols per MMA: D-halves C::BOX_BYTES apart (LBO), 8-key groups 1024 B (SBO).
            // The first 64 keys go as soon as their P is written, while the
            // softmax still computes the second half.
            const uint32_t v_lo = v_lo0 + (uint32_t)((i % C::NS) * C::TILE_BYTES >> 4);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              if (!fa_wait(smem_addr(&bars->p_full[t][half]), it & 1, a.status, wlim)) { ok = false; break; }
              tc_fence_after();
#pragma unroll
              for (int kk = half * 4; kk < half * 4 + 4; ++kk)
                mma_ts_lohi(tO, tS + kk * 8, v_lo + kk * (16 * 128 >> 4), v_hi, idesc_o, (it > 0 || kk > 0) ? 1u : 0u);
            }
            if (!ok) break;
            if (it == n_kv_t[t] - 1) mma_commit(smem_addr(&bars->o_full[t]));
          }
          if (j >= s_lo[t] && j < s_lo[t] + n_kv_t[t]) {
            // S_t = Q_t K_j^T.
            if (!k_ready) {
              if (!fa_wait(smem_addr(&bars->k_full[j % C::NS]), (j / C::NS) & 1, a.status, wlim)) { ok = false; break; }
              k_ready = true;
            }
            tc_fence_after();
            const uint32_t q_lo = qk_lo0 + (uint32_t)((C::OFF_Q + t * C::TILE_BYTES) >> 4);
            const uint32_t k_lo = qk_lo0 + (uint32_t)((C::OFF_K + (j % C::NS) * C::TILE_BYTES) >> 4);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = ((kk >> 2) * C::BOX_BYTES + (kk & 3) * 32) >> 4;
              mma_ss_lohi(tS, q_lo + off, qk_hi, k_lo + off, qk_hi, idesc_s, kk > 0 ? 1u : 0u);
            }
            mma_commit(smem_addr(&bars->s_full[t]));
          }
        }
        if (!ok) break;
        if (k_ready) mma_commit(smem_addr(&bars->k_empty[j % C::NS]));
        if (v_ready) mma_commit(smem_addr(&bars->v_empty[(j - 1) % C::NS]));
      }
      if (!ok) *abort_flag = 1;
      // All MMAs of this CTA must be complete before TMEM is released.
      mma_commit(smem_addr(&bars->mma_final));
      fa_wait(smem_addr(&bars->mma_final), 0, a.status, wlim);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    reg_alloc_inc<kRegsSoftmax>();
    const int t = warp >> 2;               // query tile of this warpgroup
    const int row = threadIdx.x & 127;     // TMEM lane
    const int row_g = q0 + t * BM + row;
    const int my_kv = (t == 0) ? n_kv_t[0] : n_kv_t[1];  // t is not a constant here
    const int my_lo = EXT ? j_min + ((t == 0) ? s_lo[0] : s_lo[1]) : 0;  // absolute first KV tile
    const int r_tile = q0 + t * BM;
    // The staging pass may have stored Q, K, V as x * 2^-e (e >= 0) to keep
    // them inside the fp16 range: the raw scores are then S * 2^-(e_q + e_k)
    // and O comes out 2^-e_v too small. Fold both back (exact powers of two).
    float sl2 = a.scale_log2, scale_raw = a.scale, o_mul = 1.f;
    if (a.range_exp != nullptr) {
      const int eq = a.range_exp[0], ek = a.range_exp[1], ev = a.range_exp[2];
      const float fq = __int_as_float((127 + eq) << 23), fk = __int_as_float((127 + ek) << 23);
      sl2 = sl2 * fq * fk;
      scale_raw = scale_raw * fq * fk;
      o_mul = __int_as_float((127 + ev) << 23);
    }
    // ALiBi (common.metal:123-128): slope * (k - q) on the scaled score, folded
    // into the raw score as (slope / scale) * (k - q) (scale != 0 on this path).
    const float slope_raw = (EXT && a.alibi != nullptr) ? a.alibi[hq] / scale_raw : 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t tS = lane_base + kColS + t * 128;
    const uint32_t tO = lane_base + kColO + t * 128;
    const uint32_t b_s_full = smem_addr(&bars->s_full[t]);
    const uint32_t b_p_full = smem_addr(&bars->p_full[t][0]);  // [t][1] is 8 bytes further
    float m_run = -INFINITY;  // running max in log2 units (value actually subtracted)
    float l_run = 0.f;
    bool ok = true;

    for (int j = 0; j < my_kv; ++j) {
      if (*abort_flag) { ok = false; break; }
      const bool got = fa_wait(b_s_full, j & 1, a.status, wlim);
      if (!__all_sync(0xffffffffu, got)) { ok = false; *abort_flag = 1; break; }
      tc_fence_after();
      float s[BN];
      tmem_ld128(tS, s);

      const int kv0 = a.kv_begin + (my_lo + j) * BN;
      bool need_mask = (kv0 + BN > a.kv_end) || (CAUSAL && kv0 + BN - 1 > r_tile);
      int key_lim = a.kv_end - kv0;                       // keys [kv0 + key_beg, kv0 + key_lim) visible
      if (CAUSAL) key_lim = min(key_lim, row_g - kv0 + 1);
      int key_beg = -1;
      if constexpr (EXT) {
        need_mask = need_mask || (a.win_right >= 0 && kv0 + BN - 1 > r_tile + a.win_right) ||
                    (a.win_left >= 0 && kv0 < r_tile + BM - 1 - a.win_left);
        if (a.win_right >= 0) key_lim = (int)min((long long)key_lim, (long long)row_g + a.win_right - kv0 + 1);
        if (a.win_left >= 0) key_beg = row_g - a.win_left - kv0;
        if (a.alibi != nullptr) {
          const float base = (float)(kv0 - row_g);
#pragma unroll
          for (int c = 0; c < BN; ++c) s[c] = fmaf(slope_raw, base + (float)c, s[c]);
        }
      }
      float ext;
      if (!need_mask && sl2 > 0.f) {
        ext = row_max128(s);  // hot path: full tile, positive scale
      } else if (sl2 >= 0.f) {
        ext = -INFINITY;
#pragma unroll
        for (int c = 0; c < BN; ++c) ext = fmaxf(ext, (!need_mask || (c < key_lim && c >= key_beg)) ? s[c] : -INFINITY);
      } else {
        ext = INFINITY;
#pragma unroll
        for (int c = 0; c < BN; ++c) ext = fminf(ext, (!need_mask || (c < key_lim && c >= key_beg)) ? s[c] : INFINITY);
      }
      const float m_cand = (sl2 == 0.f) ? 0.f : ext * sl2;
      const float m_new = fmaxf(m_run, m_cand);
      const bool grow = (m_new > m_run + kRescaleThreshold);
      const bool any_grow = __any_sync(0xffffffffu, grow);
      const float m_use = any_grow ? m_new : m_run;
      const float m_sub = (m_use == -INFINITY) ? 0.f : m_use;
      const float alpha = (m_use == m_run || m_use == -INFINITY) ? 1.f : ex2_approx(m_run - m_use);

      // O_t is stable here: the S_t commit also covered the previous PV_t.
      if (any_grow && j > 0) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tO + c * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(tO + c * 32, r);
        }
      }
      float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
      const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-m_sub, -m_sub);
#pragma unroll
      // Two halves of 64 keys with one 32-column P store each: 1-1.5 % faster
      // than four 16-column stores (fewer asynchronous stores whose source
      // registers the next chunk's results would have to wait for).
      for (int h = 0; h < 2; ++h) {
        uint32_t p[32];
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int c = h * 64 + 2 * i;
            const float p0 = (c < key_lim && c >= key_beg) ? ex2_approx(fmaf(s[c], sl2, -m_sub)) : 0.f;
            const float p1 = (c + 1 < key_lim && c + 1 >= key_beg) ? ex2_approx(fmaf(s[c + 1], sl2, -m_sub)) : 0.f;
            acc0 = __fadd2_rn(acc0, make_float2(p0, p1));
            p[i] = pack_half2(p0, p1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int c = h * 64 + 2 * i;
            const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), sc2, nm2);
            const float2 e = ((i & 15) < poly_pairs<D>()) ? exp2_poly2(x) : make_float2(ex2_approx(x.x), ex2_approx(x.y));
            if (i & 1) acc1 = __fadd2_rn(acc1, e);
            else acc0 = __fadd2_rn(acc0, e);
            p[i] = pack_half2(e.x, e.y);
          }
        }
        tmem_st32(tS + h * 32, p);  // P columns [32h, 32h+32) of S_t's region
        if (h == 0) {  // keys [0, 64) done: let the first half of PV start
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(b_p_full);
        }
      }
      const float rsum = (acc0.x + acc0.y) + (acc1.x + acc1.y);
      l_run = l_run * alpha + rsum;
      m_run = m_use;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_p_full + 8);  // p_full[t][1]
    }

    // ---------------------------------------------------------- epilogue
    const bool row_ok = (row_g < a.q_end) && (q0 + t * BM < a.q_end);
    if (ok && my_kv > 0) {
      const bool got = fa_wait(smem_addr(&bars->o_full[t]), 0, a.status, wlim);
      if (!__all_sync(0xffffffffu, got)) { ok = false; *abort_flag = 1; }
      tc_fence_after();
    }
    if (ok && q0 + t * BM < a.q_end) {
      const float inv_l = (l_run > 0.f) ? o_mul / l_run : 0.f;
      // Routed slots are a multiple of BM rows, so the tile's first row
      // names the owner of all its rows.
      RowDst dst = row_dst(a, q0 + t * BM);
      dst.row += row;
      if (row_ok && dst.lse != nullptr) {
        const float lse = (l_run > 0.f) ? (m_run + log2f(l_run)) * 0.69314718055994531f : -INFINITY;
        dst.lse[((int64_t)bz * a.Hq + hq) * dst.lse_rows + dst.row] = lse;
      }
      OutT* orow = reinterpret_cast<OutT*>(dst.o) + (int64_t)bz * dst.o_sb + (int64_t)dst.row * dst.o_ss +
                   (int64_t)hq * dst.o_sh;
      // The whole O row in one go: all TMEM loads in flight, one wait.
      float ov[D];
      if (my_kv > 0) {
        if constexpr (D == 128) tmem_ld128(tO, ov);
        else tmem_ld64(tO, ov);
#pragma unroll
        for (int i = 0; i < D; ++i) ov[i] *= inv_l;
      } else {
#pragma unroll
        for (int i = 0; i < D; ++i) ov[i] = 0.f;
      }
      bool routed = false;
      if constexpr (std::is_same<OutT, float>::value) routed = a.route_rows > 0;
      if (routed) {
        // Partial rows bound for their owner's staging slot, usually in a
        // peer GPU's memory. One 16-byte store per thread-row would reach
        // NVLink as 32 scattered 16-byte writes per warp instruction; instead
        // each warp stages its 32 rows in this tile's Q buffer (free: o_full
        // completed after the tile's last S MMA) and writes every row as a
        // contiguous run across the warp's lanes. Two passes of D/2 columns
        // (128 rows x D/2 fp32 = one Q tile); 16-byte chunks XOR-swizzled by
        // row so the staging writes and reads spread over the banks.
        constexpr int CW = D / 2;            // fp32 columns per pass
        constexpr int CH = CW / 4;           // 16-byte chunks per staged row (16 or 8)
        constexpr int RPI = 32 / CH;         // rows per warp store instruction
        float* stg = reinterpret_cast<float*>(smem + C::OFF_Q + t * C::TILE_BYTES);
        const int wrow = (warp & 3) * 32;
        const int rows_valid = min(BM, a.q_end - (q0 + t * BM));
        float* o_tile = reinterpret_cast<float*>(orow) - (int64_t)row * dst.o_ss;  // the tile's row 0
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
#pragma unroll
          for (int c = 0; c < CH; ++c)
            *reinterpret_cast<float4*>(stg + row * CW + ((c ^ (row & (CH - 1))) * 4)) =
                make_float4(ov[hp * CW + 4 * c], ov[hp * CW + 4 * c + 1], ov[hp * CW + 4 * c + 2],
                            ov[hp * CW + 4 * c + 3]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 32 / RPI; ++i) {
            const int r = wrow + i * RPI + lane / CH;
            const int c = lane % CH;
            if (r < rows_valid)
              *reinterpret_cast<float4*>(o_tile + (int64_t)r * dst.o_ss + hp * CW + 4 * c) =
                  *reinterpret_cast<const float4*>(stg + r * CW + ((c ^ (r & (CH - 1))) * 4));
          }
          __syncwarp();
        }
      } else if (row_ok) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) store_row32<OutT>(orow + c * 32, ov + c * 32);
      }
    }
  }

  __syncwarp();  // role branches ran on one lane; reconverge before the CTA barrier
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool CAUSAL, bool QK_BF16, typename OutT>
cudaError_t launch_t(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                     const CUtensorMap& tv, cudaStream_t stream) {
  const bool ext = a.win_left >= 0 || a.win_right >= 0 || a.alibi != nullptr;
  auto kern = ext ? attn_fwd_sm100<D, CAUSAL, QK_BF16, OutT, true> : attn_fwd_sm100<D, CAUSAL, QK_BF16, OutT, false>;
  constexpr int smem = Cfg<D>::SMEM_BYTES;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const long long blocks = (long long)((a.q_end - a.q_begin + NT * BM - 1) / (NT * BM)) * a.Hq * a.B;
  if (blocks <= 0) return cudaSuccess;
  // Units per group of the CTA order: as many (batch, KV-head) units as have
  // 32 MB of fp16 K/V together (a quarter of L2), at least one.
  AttnArgs ag = a;
  const long long unit_bytes = (long long)(a.kv_end - a.kv_begin) * D * 2 * 2;
  const long long n_units = (long long)a.B * a.Hk;
  ag.units_per_group = (int)std::max<long long>(1, std::min<long long>(n_units, (32ll << 20) / std::max(1ll, unit_bytes)));
  e = launch_pdl(kern, dim3((unsigned)blocks), dim3(kThreads), smem, stream, tq, tk, tv, ag);
  note_launch();
  return e;
}

template <int D, bool CAUSAL, bool QK_BF16>
cudaError_t launch_out(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                       const CUtensorMap& tv, int out_dtype, cudaStream_t stream) {
  switch (out_dtype) {
    case kF16: return launch_t<D, CAUSAL, QK_BF16, __half>(a, tq, tk, tv, stream);
    case kBF16: return launch_t<D, CAUSAL, QK_BF16, __nv_bfloat16>(a, tq, tk, tv, stream);
    default: return launch_t<D, CAUSAL, QK_BF16, float>(a, tq, tk, tv, stream);
  }
}

// One translation unit per (D, causal) pair keeps build times short.
cudaError_t launch_d64_causal(const AttnArgs&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, bool, int, cudaStream_t);
cudaError_t launch_d64_full(const AttnArgs&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, bool, int, cudaStream_t);
cudaError_t launch_d128_causal(const AttnArgs&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, bool, int, cudaStream_t);
cudaError_t launch_d128_full(const AttnArgs&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, bool, int, cudaStream_t);

}  // namespace sm100
}  // namespace fa
