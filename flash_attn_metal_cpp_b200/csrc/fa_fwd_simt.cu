// fa_fwd_simt.cu - CUDA-core FlashAttention forward for the cases the
// tensor-core kernel does not take: fp32 inputs (kept in fp32 end to end,
// so results stay within 1e-5 relative of an fp32 reference) and head dims
// other than 64 / 128 (any D <= 256, e.g. 32, 40, 59, 80, 96, 111).
//
// Same math as the reference kernel (kernels/flash_attention_fwd_optimized.metal:
// 79-221): scale, top-left causal mask, online softmax, O / l; plus the GQA
// head map (common.metal:215-217) and rotate-half RoPE on load
// (common.metal:150-167: x_i' = x_i cos - x_{i+D/2} sin,
// x_{i+D/2}' = x_i sin + x_{i+D/2} cos, table index pos * (D/2) + i).
//
// Layout: one CTA = 32 query rows of one (batch, head); 16 threads per row,
// thread c of a row owns columns c, c+16, c+32, ...; a score is reduced over
// the row's threads with xor shuffles. Keys stream through shared memory in
// tiles of 32, converted to fp32 once per CTA. The kernel is latency-bound
// (a CTA walks its keys in order): on B1 S512 H8 D64 causal fp32, 16 threads
// per row took 0.159 ms, 8 took 0.178 ms and 4 took 0.276 ms; 16-row CTAs
// were slower than 32-row ones.
#include "fa_internal.h"
#include "fa_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace fa {
namespace {

constexpr int ROWS = 32;
constexpr int TPR = 16;  // threads per row
constexpr int KT = 32;  // keys per tile
constexpr int THREADS = ROWS * TPR;

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// Element `col` of a row after optional rotate-half RoPE at position `pos`.
template <typename T>
__device__ __forceinline__ float load_rot(const T* row, int col, int D, int pos, const float* cs,
                                          const float* sn) {
  const float x = to_f<T>(row[col]);
  if (cs == nullptr) return x;
  const int h = D / 2;
  if (col < h) {
    const float y = to_f<T>(row[col + h]);
    const float c = cs[(int64_t)pos * h + col], s = sn[(int64_t)pos * h + col];
    return x * c - y * s;
  }
  if (col < 2 * h) {
    const float y = to_f<T>(row[col - h]);
    const float c = cs[(int64_t)pos * h + col - h], s = sn[(int64_t)pos * h + col - h];
    return y * s + x * c;
  }
  return x;  // odd D: last column has no partner
}

__device__ __forceinline__ void store_out(void* base, int64_t idx, int out_dtype, float x) {
  if (out_dtype == kF32) reinterpret_cast<float*>(base)[idx] = x;
  else if (out_dtype == kF16) reinterpret_cast<__half*>(base)[idx] = __float2half_rn(x);
  else reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(x);
}

template <typename InT, int DMAX>
__global__ void __launch_bounds__(THREADS)
    attn_fwd_simt(const AttnArgs a, const int out_dtype) {
  const bool CAUSAL = a.causal != 0;
  constexpr int DPT = DMAX / TPR;  // columns per thread
  extern __shared__ float sm[];
  float* Ks = sm;                  // [KT][DMAX]
  float* Vs = sm + KT * DMAX;      // [KT][DMAX]

  const int tid = threadIdx.x;
  const int r = tid / TPR;
  const int c = tid % TPR;
  const int hq = blockIdx.y;
  const int bz = blockIdx.z;
  const int hk = hq / a.group;
  const int q0 = a.q_begin + blockIdx.x * ROWS;
  const int row_g = q0 + r;
  const bool row_ok = row_g < a.q_end;
  const int D = a.D;

  const InT* Q = reinterpret_cast<const InT*>(a.q);
  const InT* K = reinterpret_cast<const InT*>(a.k);
  const InT* V = reinterpret_cast<const InT*>(a.v);

  float q[DPT], o[DPT];
  {
    const InT* qrow = Q + (int64_t)bz * a.q_sb + (int64_t)(row_ok ? row_g : q0) * a.q_ss +
                      (int64_t)hq * a.q_sh;
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      const int col = i * TPR + c;
      q[i] = (row_ok && col < D) ? load_rot(qrow, col, D, row_g, a.rope_cos, a.rope_sin) : 0.f;
      o[i] = 0.f;
    }
  }

  const int q_last = min(q0 + ROWS, a.q_end) - 1;
  int kv_hi = a.kv_end;
  if (CAUSAL) kv_hi = min(kv_hi, q_last + 1);
  if (a.win_right >= 0) kv_hi = min(kv_hi, q_last + a.win_right + 1);
  // Tiles wholly left of every row's window are skipped (tile starts stay
  // aligned to kv_begin).
  int kv_lo = a.kv_begin;
  if (a.win_left >= 0 && q0 - a.win_left > kv_lo) kv_lo += (q0 - a.win_left - kv_lo) / KT * KT;
  const float slope = a.alibi ? a.alibi[hq] : 0.f;

  float m_run = -INFINITY, l_run = 0.f;
  for (int kv0 = kv_lo; kv0 < kv_hi; kv0 += KT) {
    __syncthreads();
    for (int e = tid; e < KT * DMAX; e += THREADS) {
      const int kr = e / DMAX, col = e % DMAX;
      const int key = kv0 + kr;
      float kx = 0.f, vx = 0.f;
      if (key < a.kv_end && col < D) {
        const InT* krow = K + (int64_t)bz * a.k_sb + (int64_t)key * a.k_ss + (int64_t)hk * a.k_sh;
        const InT* vrow = V + (int64_t)bz * a.v_sb + (int64_t)key * a.v_ss + (int64_t)hk * a.v_sh;
        kx = load_rot(krow, col, D, key, a.rope_cos, a.rope_sin);
        vx = to_f<InT>(vrow[col]);
      }
      Ks[kr * DMAX + col] = kx;
      Vs[kr * DMAX + col] = vx;
    }
    __syncthreads();

    float s[KT];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      float acc = 0.f;
#pragma unroll 8
      for (int i = 0; i < DPT; ++i) acc = fmaf(q[i], Ks[j * DMAX + i * TPR + c], acc);
#pragma unroll
      for (int off = 1; off < TPR; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      const int key = kv0 + j;
      const int rel = key - row_g;  // k - q
      const bool vis = key < a.kv_end && (!CAUSAL || rel <= 0) && (a.win_left < 0 || rel >= -a.win_left) &&
                       (a.win_right < 0 || rel <= a.win_right);
      // scale before the mask (.metal:138-143); ALiBi slope * (k - q) on the scaled score
      s[j] = vis ? fmaf(slope, (float)rel, acc * a.scale) : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    const float m_new = fmaxf(m_run, mx);
    const float m_sub = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_sub);
    float rs = 0.f;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      s[j] = (s[j] == -INFINITY) ? 0.f : expf(s[j] - m_sub);
      rs += s[j];
    }
    l_run = l_run * alpha + rs;
    m_run = m_new;
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      float acc = o[i] * alpha;
#pragma unroll
      for (int j = 0; j < KT; ++j) acc = fmaf(s[j], Vs[j * DMAX + i * TPR + c], acc);
      o[i] = acc;
    }
  }

  if (!row_ok) return;
  const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
  const RowDst dst = row_dst(a, row_g);
  const int64_t orow = (int64_t)bz * dst.o_sb + (int64_t)dst.row * dst.o_ss + (int64_t)hq * dst.o_sh;
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    const int col = i * TPR + c;
    if (col < D) store_out(dst.o, orow + col, out_dtype, o[i] * inv_l);
  }
  if (c == 0 && dst.lse != nullptr)
    dst.lse[((int64_t)bz * a.Hq + hq) * dst.lse_rows + dst.row] =
        (l_run > 0.f) ? m_run + logf(l_run) : -INFINITY;
}

template <typename InT, int DMAX>
cudaError_t launch3(const AttnArgs& a, int out_dtype, cudaStream_t st) {
  const int smem = 2 * KT * DMAX * (int)sizeof(float);
  dim3 grid((unsigned)((a.q_end - a.q_begin + ROWS - 1) / ROWS), (unsigned)a.Hq, (unsigned)a.B);
  if (grid.x == 0) return cudaSuccess;
  auto k = attn_fwd_simt<InT, DMAX>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  k<<<grid, THREADS, smem, st>>>(a, out_dtype);
  note_launch();
  return cudaGetLastError();
}

template <typename InT>
cudaError_t launch1(const AttnArgs& a, int out_dtype, cudaStream_t st) {
  if (a.D <= 64) return launch3<InT, 64>(a, out_dtype, st);
  if (a.D <= 128) return launch3<InT, 128>(a, out_dtype, st);
  return launch3<InT, 256>(a, out_dtype, st);
}

}  // namespace

cudaError_t launch_attn_simt(const AttnArgs& a, int in_dtype, int out_dtype, cudaStream_t st) {
  if (a.D > 256) return cudaErrorInvalidValue;
  switch (in_dtype) {
    case kF16: return launch1<__half>(a, out_dtype, st);
    case kBF16: return launch1<__nv_bfloat16>(a, out_dtype, st);
    default: return launch1<float>(a, out_dtype, st);
  }
}

}  // namespace fa
