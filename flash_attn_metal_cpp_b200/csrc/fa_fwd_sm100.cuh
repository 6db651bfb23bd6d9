// fa_fwd_sm100.cuh - FlashAttention-2 forward kernel for B200 (sm_100a).
//
// Computes, per (batch, query head, 128-row query tile), the online-softmax
// attention of the reference kernel (kernels/flash_attention_fwd_optimized.metal:79-221:
// running max m, running sum l, O rescale by exp(m_old - m_new), final O / l),
// with the score scale applied before the mask (.metal:138-143) and the
// top-left causal mask (key k masked for query q iff k > q, common.metal:90-92).
// GQA reads KV head h / group (common.metal:215-217).
//
// Blackwell mapping (one CTA = one 128-row query tile, 6 warps):
//   warp 4      TMA producer: Q tile once, then K_j / V_j tiles into a
//               NS-stage shared-memory ring (128B-swizzled boxes of 64 cols).
//   warp 5      MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM
//               S buffers (tcgen05.mma kind::f16, fp32 accumulate), then
//               O += P_{j-1} V_{j-1} with P read from TMEM (A operand) and V
//               from shared memory (MN-major B operand).
//   warps 0-3   softmax: thread t owns query row t = TMEM lane t. Reads S_j
//               (tcgen05.ld), masks only diagonal / tail tiles, updates the
//               running max lazily (O is rescaled in TMEM only when the max
//               grows by more than 2^8), writes P_j = exp2(S*scale*log2e - m)
//               as fp16 into TMEM (tcgen05.st), and finally normalises O,
//               writes it with 16-byte stores and writes LSE.
// Causal tiles beyond the diagonal are never loaded or computed.
//
// TMEM columns: S0 [0,128) S1 [128,256) O [256,256+D) P [384,448).
#pragma once
#include "fa_internal.h"
#include "fa_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace fa {
namespace sm100 {

constexpr int BM = 128;          // query rows per tile (= TMEM lanes)
constexpr int BN = 128;          // keys per KV tile
constexpr int kThreads = 192;    // 4 softmax warps + producer + MMA
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColO = 256, kColP = 384;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale when max grows by > 2^8

template <int D>
struct Cfg {
  static constexpr int NBOX = D / 64;                  // 64-col (128 B) boxes per row
  static constexpr int BOX_BYTES = 128 * 128;          // 128 rows x 128 B
  static constexpr int TILE_BYTES = NBOX * BOX_BYTES;  // one Q / K / V tile
  static constexpr int NS = (D == 128) ? 2 : 4;        // K/V pipeline stages
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = TILE_BYTES;
  static constexpr int OFF_V = OFF_K + NS * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_V + NS * TILE_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;  // + barriers + alignment slack
};

struct Bars {
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t o_done;
  uint64_t mma_final;
  uint64_t k_full[4];
  uint64_t v_full[4];
  uint64_t kv_empty[4];
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

template <int D, bool CAUSAL, bool QK_BF16, typename OutT>
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

  // Work item: heaviest causal tiles first, heads of one KV group adjacent.
  const int hb_count = a.Hq * a.B;
  const int tile_rank = blockIdx.x / hb_count;
  const int hb = blockIdx.x - tile_rank * hb_count;
  const int hq = hb % a.Hq;
  const int bz = hb / a.Hq;
  const int tile = CAUSAL ? (a.n_q_tiles - 1 - tile_rank) : tile_rank;
  const int hk = hq / a.group;
  const int q0 = a.q_begin + tile * BM;
  const int q_last = min(q0 + BM, a.q_end) - 1;
  int kv_hi = a.kv_end;
  if (CAUSAL) kv_hi = min(kv_hi, q_last + 1);
  const int n_kv = (kv_hi > a.kv_begin) ? (kv_hi - a.kv_begin + BN - 1) / BN : 0;

  const uint32_t b_q_full = smem_addr(&bars->q_full);
  const uint32_t b_p_full = smem_addr(&bars->p_full);
  const uint32_t b_o_done = smem_addr(&bars->o_done);
  const uint32_t b_final = smem_addr(&bars->mma_final);

  if (threadIdx.x == 128) {
    mbar_init(b_q_full, 1);
    mbar_init(smem_addr(&bars->s_full[0]), 1);
    mbar_init(smem_addr(&bars->s_full[1]), 1);
    mbar_init(smem_addr(&bars->s_free[0]), 128);
    mbar_init(smem_addr(&bars->s_free[1]), 128);
    mbar_init(b_p_full, 128);
    mbar_init(b_o_done, 1);
    mbar_init(b_final, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(smem_addr(&bars->k_full[s]), 1);
      mbar_init(smem_addr(&bars->v_full[s]), 1);
      mbar_init(smem_addr(&bars->kv_empty[s]), 1);
    }
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_addr(&bars->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_kv > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(b_q_full, C::TILE_BYTES);
#pragma unroll
      for (int bx = 0; bx < C::NBOX; ++bx)
        tma_load_4d(sQ + bx * C::BOX_BYTES, &tm_q, b_q_full, bx * 64, hq, q0, bz);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        if (*abort_flag) break;
        const int st = j % C::NS;
        const uint32_t use = j / C::NS;
        if (!fa_wait(smem_addr(&bars->kv_empty[st]), (use + 1) & 1, a.status)) {
          *abort_flag = 1;
          break;
        }
        const int kv0 = a.kv_begin + j * BN;
        const uint32_t bk = smem_addr(&bars->k_full[st]);
        const uint32_t bv = smem_addr(&bars->v_full[st]);
        mbar_arrive_expect_tx(bk, C::TILE_BYTES);
#pragma unroll
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_4d(sK + st * C::TILE_BYTES + bx * C::BOX_BYTES, &tm_k, bk, bx * 64, hk, kv0, bz);
        mbar_arrive_expect_tx(bv, C::TILE_BYTES);
#pragma unroll
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_4d(sV + st * C::TILE_BYTES + bx * C::BOX_BYTES, &tm_v, bv, bx * 64, hk, kv0, bz);
        issued = j + 1;
      }
      // Never leave the CTA with bulk copies still writing shared memory.
      fa_wait(b_q_full, 0, a.status);
      for (int j = max(0, issued - C::NS); j < issued; ++j) {
        const int st = j % C::NS;
        const uint32_t par = (j / C::NS) & 1;
        fa_wait(smem_addr(&bars->k_full[st]), par, a.status);
        fa_wait(smem_addr(&bars->v_full[st]), par, a.status);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t fmt_qk = QK_BF16 ? 1u : 0u;
      constexpr uint32_t idesc_s = make_idesc(BM, BN, fmt_qk, 0, 0);
      constexpr uint32_t idesc_o = make_idesc(BM, D, 0 /*f16*/, 0, 1 /*V is MN-major*/);
      const uint32_t tS = tmem + kColS0;
      const uint32_t tO = tmem + kColO;
      const uint32_t tP = tmem + kColP;
      bool ok = fa_wait(b_q_full, 0, a.status);
      tc_fence_after();

      auto issue_pv = [&](int i) -> bool {
        const int st = i % C::NS;
        if (!fa_wait(b_p_full, i & 1, a.status)) return false;
        if (!fa_wait(smem_addr(&bars->v_full[st]), (i / C::NS) & 1, a.status)) return false;
        tc_fence_after();
        const uint32_t vbase = sV + st * C::TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // 16 keys x D cols; D-halves are C::BOX_BYTES apart (LBO), 8-key groups 1024 B (SBO).
          const uint64_t bdesc = smem_desc(vbase + kk * 16 * 128, C::BOX_BYTES, 1024);
          mma_ts(tO, tP + kk * 8, bdesc, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(smem_addr(&bars->kv_empty[st]));
        mma_commit(b_o_done);
        return true;
      };

      for (int j = 0; ok && j < n_kv; ++j) {
        if (*abort_flag) { ok = false; break; }
        const int st = j % C::NS;
        const int sb = j & 1;
        if (!fa_wait(smem_addr(&bars->k_full[st]), (j / C::NS) & 1, a.status)) { ok = false; break; }
        if (j >= 2 && !fa_wait(smem_addr(&bars->s_free[sb]), ((j - 2) >> 1) & 1, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kbase = sK + st * C::TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::BOX_BYTES + (kk & 3) * 32;
          const uint64_t adesc = smem_desc(sQ + off, 16, 1024);
          const uint64_t bdesc = smem_desc(kbase + off, 16, 1024);
          mma_ss(tS + sb * BN, adesc, bdesc, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(smem_addr(&bars->s_full[sb]));
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && !issue_pv(n_kv - 1)) ok = false;
      if (!ok) *abort_flag = 1;
      // All MMAs of this CTA must be complete before TMEM is released.
      mma_commit(b_final);
      fa_wait(b_final, 0, a.status);
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int row = threadIdx.x;  // 0..127 == TMEM lane
    const int row_g = q0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const float sl2 = a.scale_log2;
    float m_run = -INFINITY;  // running max in log2 units (value actually subtracted)
    float l_run = 0.f;
    bool ok = true;

    for (int j = 0; j < n_kv; ++j) {
      if (*abort_flag) { ok = false; break; }
      const int sb = j & 1;
      bool got = fa_wait(smem_addr(&bars->s_full[sb]), (j >> 1) & 1, a.status);
      if (!__all_sync(0xffffffffu, got)) { ok = false; *abort_flag = 1; break; }
      tc_fence_after();
      float s[BN];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(lane_base + kColS0 + sb * BN + c * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(smem_addr(&bars->s_free[sb]));

      const int kv0 = a.kv_begin + j * BN;
      const bool need_mask = (kv0 + BN > a.kv_end) || (CAUSAL && kv0 + BN - 1 > q0);
      int key_lim = a.kv_end - kv0;                       // keys [kv0, kv0+key_lim) visible
      if (CAUSAL) key_lim = min(key_lim, row_g - kv0 + 1);
      float ext;
      if (sl2 >= 0.f) {
        ext = -INFINITY;
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN; ++c) ext = fmaxf(ext, c < key_lim ? s[c] : -INFINITY);
        } else {
#pragma unroll
          for (int c = 0; c < BN; ++c) ext = fmaxf(ext, s[c]);
        }
      } else {
        ext = INFINITY;
#pragma unroll
        for (int c = 0; c < BN; ++c) ext = fminf(ext, (!need_mask || c < key_lim) ? s[c] : INFINITY);
      }
      float m_cand = (sl2 == 0.f) ? 0.f : ext * sl2;
      const float m_new = fmaxf(m_run, m_cand);
      const bool grow = (m_new > m_run + kRescaleThreshold);
      const bool any_grow = __any_sync(0xffffffffu, grow);
      const float m_use = any_grow ? m_new : m_run;
      const float m_sub = (m_use == -INFINITY) ? 0.f : m_use;
      const float alpha = (m_use == m_run || m_use == -INFINITY) ? 1.f : ex2_approx(m_run - m_use);

      // PV_{j-1} must be complete before O is rescaled and P is overwritten.
      if (j > 0) {
        got = fa_wait(b_o_done, (j - 1) & 1, a.status);
        if (!__all_sync(0xffffffffu, got)) { ok = false; *abort_flag = 1; break; }
        tc_fence_after();
        if (any_grow) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(lane_base + kColO + c * 32, r);
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(lane_base + kColO + c * 32, r);
          }
        }
      }
      float rsum = 0.f;
      uint32_t p[BN / 2];
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < BN; c += 2) {
          float p0 = (c < key_lim) ? ex2_approx(fmaf(s[c], sl2, -m_sub)) : 0.f;
          float p1 = (c + 1 < key_lim) ? ex2_approx(fmaf(s[c + 1], sl2, -m_sub)) : 0.f;
          rsum += p0 + p1;
          p[c / 2] = pack_half2(p0, p1);
        }
      } else {
#pragma unroll
        for (int c = 0; c < BN; c += 2) {
          float p0 = ex2_approx(fmaf(s[c], sl2, -m_sub));
          float p1 = ex2_approx(fmaf(s[c + 1], sl2, -m_sub));
          rsum += p0 + p1;
          p[c / 2] = pack_half2(p0, p1);
        }
      }
      l_run = l_run * alpha + rsum;
      m_run = m_use;
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_st16(lane_base + kColP + c, &p[c]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(b_p_full);
    }

    // ---------------------------------------------------------- epilogue
    const bool row_ok = (row_g < a.q_end);
    if (ok && n_kv > 0) {
      bool got = fa_wait(b_o_done, (n_kv - 1) & 1, a.status);
      if (!__all_sync(0xffffffffu, got)) { ok = false; *abort_flag = 1; }
      tc_fence_after();
    }
    if (ok) {
      const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
      if (row_ok && a.lse != nullptr) {
        const float lse = (l_run > 0.f) ? (m_run + log2f(l_run)) * 0.69314718055994531f : -INFINITY;
        a.lse[((int64_t)bz * a.Hq + hq) * a.Sq + row_g] = lse;
      }
      OutT* orow = reinterpret_cast<OutT*>(a.o) + (int64_t)bz * a.o_sb + (int64_t)row_g * a.o_ss +
                   (int64_t)hq * a.o_sh;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        if (n_kv > 0) {
          uint32_t r[32];
          tmem_ld32(lane_base + kColO + c * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * inv_l;
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
        if (row_ok) store_row32<OutT>(orow + c * 32, v);
      }
    }
  }

  __syncwarp();  // role branches ran on one lane; reconverge before the CTA barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool CAUSAL, bool QK_BF16, typename OutT>
cudaError_t launch_t(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                     const CUtensorMap& tv, cudaStream_t stream) {
  auto kern = attn_fwd_sm100<D, CAUSAL, QK_BF16, OutT>;
  constexpr int smem = Cfg<D>::SMEM_BYTES;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const long long blocks = (long long)a.n_q_tiles * a.Hq * a.B;
  if (blocks <= 0) return cudaSuccess;
  kern<<<dim3((unsigned)blocks), dim3(kThreads), smem, stream>>>(tq, tk, tv, a);
  note_launch();
  return cudaGetLastError();
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
