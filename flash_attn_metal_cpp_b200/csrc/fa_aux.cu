// fa_aux.cu - memory-bound helper kernels around the attention kernels:
//   * stage / stage_fixup: rotate-half RoPE (common.metal:150-167) and/or
//                  conversion to fp16 of Q, K and V in one launch, producing
//                  the contiguous fp16 operands the tensor-core kernel loads
//                  with TMA (zero-padded to 64 or 128 columns for other head
//                  dims); a tensor whose values would overflow fp16 is
//                  rescaled by a power of two, recorded for the kernel;
//   * rope_table:  cos/sin tables [rows, D/2] (layout of the reference's
//                  host tables, src/flash_attn_core.cpp:343-349), computed
//                  in double and rounded to float;
//   * combine:     merge of split-KV partials (O_j, LSE_j);
//   * fill_empty:  O = 0, LSE = -inf when there is no key at all;
//   * unpad:       first D columns of a padded output.
#include "fa_internal.h"
#include "fa_ptx.cuh"

#include <algorithm>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace fa {

namespace {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&x)[8]);

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&x)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&x)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&x)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }

// Largest finite value of fp16.
constexpr float kHalfMax = 65504.f;

// Stores 8 values as fp16; returns their largest magnitude (fmaxf drops NaN).
__device__ __forceinline__ float store8_half(__half* p, const float (&x)[8]) {
  uint4 w;
  w.x = pack_half2(x[0], x[1]);
  w.y = pack_half2(x[2], x[3]);
  w.z = pack_half2(x[4], x[5]);
  w.w = pack_half2(x[6], x[7]);
  *reinterpret_cast<uint4*>(p) = w;
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(x[i]));
  return m;
}

// Value of output column `col` of row (b, s, h) of a staging job, before any
// rescale: x (rotated over the pairs (i, i + D/2) of the original D when the
// job has tables; an odd D's last column has no partner and is kept), zero
// for the padding columns. Same rounding steps as rope_rotate8.
template <typename T>
__device__ __forceinline__ float stage_value(const StageJob& jb, int b, int s, int h, int col) {
  if (col >= jb.D) return 0.f;
  const T* src = reinterpret_cast<const T*>(jb.x) + (int64_t)b * jb.sb + (int64_t)s * jb.ss + (int64_t)h * jb.sh;
  const int half = jb.D / 2;
  if (jb.cs != nullptr && col < 2 * half) {
    const int i = col < half ? col : col - half;  // pair index
    const float c = jb.cs[(int64_t)s * half + i], sv = jb.sn[(int64_t)s * half + i];
    const float a0 = ld_f<T>(src + i), a1 = ld_f<T>(src + i + half);
    return (col < half) ? __fmaf_rn(a0, c, -__fmul_rn(a1, sv)) : __fmaf_rn(a0, sv, __fmul_rn(a1, c));
  }
  return ld_f<T>(src + col);
}

// Block-wide maximum of `v` (non-negative); the result is valid in thread 0.
__device__ __forceinline__ float block_max(float v) {
  __shared__ float part[32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) part[w] = v;
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) v = fmaxf(v, part[i]);
  return v;
}

// Records a block's largest magnitude of job `slot` when it is beyond the
// fp16 range (only those matter to the fixup; in-range blocks skip the atomic).
__device__ __forceinline__ void record_amax(RangeRec* rec, int slot, float amax) {
  const float m = block_max(amax > kHalfMax ? amax : 0.f);
  if (threadIdx.x == 0 && m > kHalfMax) atomicMax(&rec->amax_bits[slot], __float_as_uint(m));
}

// The job of this block: blocks [blk_end[j-1], blk_end[j]) stage job j.
__device__ __forceinline__ int block_job(const StageBatch& bt, int& first_block, int& n_blocks) {
  const int b = blockIdx.x;
  const int j = b < bt.blk_end[0] ? 0 : (b < bt.blk_end[1] ? 1 : 2);
  first_block = j == 0 ? 0 : bt.blk_end[j - 1];
  n_blocks = bt.blk_end[j] - first_block;
  return j;
}

// Items of the vectorised staging pass: one item is one 8-column chunk
// (and, with RoPE, its partner chunk D/2 further) of G heads at one (b, s).
// The G rows share table row s, loaded once, and their 2G 16-byte loads are
// in flight together.
template <typename T, int G, bool ROPE>
__device__ __forceinline__ float stage_vec_items(const StageJob& jb, unsigned first, unsigned stride) {
  const int half = jb.D / 2;
  const unsigned chunks = ROPE ? (unsigned)jb.D / 16 : (unsigned)jb.D / 8;  // 4, 8 or 16
  const unsigned shift = __ffs(chunks) - 1;
  const unsigned hg = (unsigned)jb.H / G;
  const unsigned items = ((unsigned)jb.B * jb.S * hg) << shift;
  float amax = 0.f;
  for (unsigned li = first; li < items; li += stride) {
    const unsigned rowi = li >> shift;
    const int c0 = (int)(li & (chunks - 1)) * 8;
    const unsigned bs = rowi / hg;
    const int h0 = (int)(rowi - bs * hg) * G;
    const unsigned b = bs / (unsigned)jb.S;
    const int s = (int)(bs - b * (unsigned)jb.S);
    const T* src = reinterpret_cast<const T*>(jb.x) + (int64_t)b * jb.sb + (int64_t)s * jb.ss + (int64_t)h0 * jb.sh + c0;
    __half* dst = jb.y + (((int64_t)b * jb.y_rows + s) * jb.H + h0) * jb.D + c0;
    if constexpr (ROPE) {
      float a[G][8], bb[G][8];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        load8<T>(src + g * jb.sh, a[g]);
        load8<T>(src + g * jb.sh + half, bb[g]);
      }
      const float4* cp = reinterpret_cast<const float4*>(jb.cs + (int64_t)s * half + c0);
      const float4* sp = reinterpret_cast<const float4*>(jb.sn + (int64_t)s * half + c0);
      const float4 c_lo = cp[0], c_hi = cp[1], s_lo = sp[0], s_hi = sp[1];
      const float cv[8] = {c_lo.x, c_lo.y, c_lo.z, c_lo.w, c_hi.x, c_hi.y, c_hi.z, c_hi.w};
      const float sv[8] = {s_lo.x, s_lo.y, s_lo.z, s_lo.w, s_hi.x, s_hi.y, s_hi.z, s_hi.w};
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float ra[8], rb[8];
        rope_rotate8(a[g], bb[g], cv, sv, ra, rb);
        amax = fmaxf(amax, fmaxf(store8_half(dst + g * jb.D, ra), store8_half(dst + g * jb.D + half, rb)));
      }
    } else {
      float a[G][8];
#pragma unroll
      for (int g = 0; g < G; ++g) load8<T>(src + g * jb.sh, a[g]);
#pragma unroll
      for (int g = 0; g < G; ++g) amax = fmaxf(amax, store8_half(dst + g * jb.D, a[g]));
    }
  }
  return amax;
}

// Staging pass, vectorised: 16-byte loads and stores, rows of up to four
// heads at one position per item (stage_vec_items). Requires Dp == D,
// D % 16 == 0 with tables (D % 8 == 0 without), 16-byte aligned rows and
// fewer than 2^31 chunks per job (checked on the host). Each block works on
// one job, so the job's fields sit in registers and the branches are
// uniform. Values are written unscaled; a block whose largest magnitude
// exceeds the fp16 range records it in rec->amax_bits (the fixup kernel
// then rewrites that tensor).
template <typename T>
__global__ void __launch_bounds__(256) stage_vec_kernel(const StageBatch bt) {
  grid_dep_wait();  // launched as a programmatic dependent of the previous kernel
  grid_dep_launch_dependents();
  int first_block, n_blocks;
  const int j = block_job(bt, first_block, n_blocks);
  const StageJob jb = bt.job[j];
  const unsigned first = (blockIdx.x - first_block) * blockDim.x + threadIdx.x;
  const unsigned stride = (unsigned)n_blocks * blockDim.x;
  const int G = jb.H % 4 == 0 ? 4 : (jb.H % 2 == 0 ? 2 : 1);
  float amax;
  if (jb.cs != nullptr)
    amax = G == 4 ? stage_vec_items<T, 4, true>(jb, first, stride)
                  : (G == 2 ? stage_vec_items<T, 2, true>(jb, first, stride) : stage_vec_items<T, 1, true>(jb, first, stride));
  else
    amax = G == 4 ? stage_vec_items<T, 4, false>(jb, first, stride)
                  : (G == 2 ? stage_vec_items<T, 2, false>(jb, first, stride) : stage_vec_items<T, 1, false>(jb, first, stride));
  record_amax(bt.rec, jb.slot, amax);
}

// Staging pass, one thread per output element of the Dp-wide rows (other
// head dims, padded with zeros; unaligned rows). Same per-block job split.
template <typename T>
__global__ void __launch_bounds__(256) stage_elem_kernel(const StageBatch bt) {
  grid_dep_wait();
  grid_dep_launch_dependents();
  int first_block, n_blocks;
  const int j = block_job(bt, first_block, n_blocks);
  const StageJob jb = bt.job[j];
  const long long total = (long long)jb.B * jb.S * jb.H * jb.Dp;
  float amax = 0.f;
  for (long long li = (long long)(blockIdx.x - first_block) * blockDim.x + threadIdx.x; li < total;
       li += (long long)n_blocks * blockDim.x) {
    const int col = (int)(li % jb.Dp);
    const long long rowi = li / jb.Dp;
    const int h = (int)(rowi % jb.H);
    const long long bs = rowi / jb.H;
    const int s = (int)(bs % jb.S);
    const int b = (int)(bs / jb.S);
    const float val = stage_value<T>(jb, b, s, h, col);
    amax = fmaxf(amax, fabsf(val));
    jb.y[(((int64_t)b * jb.y_rows + s) * jb.H + h) * jb.Dp + col] = __float2half_rn(val);
  }
  record_amax(bt.rec, jb.slot, amax);
}

// Exponent e >= 0 with amax * 2^-e <= 65504 (0 when amax is in range, or is
// inf / NaN: such inputs propagate as they would in fp32 arithmetic).
__device__ __forceinline__ int range_exponent(float amax) {
  if (!(amax > kHalfMax) || !isfinite(amax)) return 0;
  int e = 0;
  frexpf(amax / kHalfMax, &e);  // amax / 65504 = m * 2^e, m in [0.5, 1)
  return min(e, 126);
}

// Second half of the staging pass. Every block reads the recorded maxima;
// if none was recorded (the usual case) block 0 publishes zero exponents and
// every block exits. Otherwise each tensor with a finite maximum beyond the
// fp16 range is rewritten as round_fp16(value * 2^-e) from its source, and
// the last block to finish clears the maxima for the next call.
template <typename T>
__global__ void __launch_bounds__(256) stage_fixup_kernel(const StageBatch bt) {
  __shared__ int s_exp[3];
  __shared__ int s_recorded;
  grid_dep_wait();  // the staging launch before it has finished (and its record is visible)
  grid_dep_launch_dependents();
  RangeRec* rec = bt.rec;
  if (threadIdx.x == 0) {
    unsigned recorded = 0;
    for (int slot = 0; slot < 3; ++slot) {
      const unsigned bits = __ldcg(&rec->amax_bits[slot]);
      recorded |= bits;
      s_exp[slot] = range_exponent(__uint_as_float(bits));
    }
    s_recorded = recorded != 0u;
    if (blockIdx.x == 0)
      for (int slot = 0; slot < 4; ++slot) rec->exp[slot] = slot < 3 ? s_exp[slot] : 0;
  }
  __syncthreads();
  if (!s_recorded) return;
  for (int j = 0; j < bt.n; ++j) {
    const StageJob& jb = bt.job[j];
    const int e = s_exp[jb.slot];
    if (e == 0) continue;
    const float mul = __int_as_float((127 - e) << 23);  // 2^-e, exact
    const long long total = (long long)jb.B * jb.S * jb.H * jb.Dp;
    for (long long li = blockIdx.x * (long long)blockDim.x + threadIdx.x; li < total;
         li += (long long)gridDim.x * blockDim.x) {
      const int col = (int)(li % jb.Dp);
      const long long rowi = li / jb.Dp;
      const int h = (int)(rowi % jb.H);
      const long long bs = rowi / jb.H;
      const int s = (int)(bs % jb.S);
      const int b = (int)(bs / jb.S);
      const float val = stage_value<T>(jb, b, s, h, col);
      jb.y[(((int64_t)b * jb.y_rows + s) * jb.H + h) * jb.Dp + col] = __float2half_rn(__fmul_rn(val, mul));
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&rec->done, 1u) == gridDim.x - 1) {
      // Every block has read the maxima: clear them for the next call.
      for (int slot = 0; slot < 4; ++slot) rec->amax_bits[slot] = 0u;
      rec->done = 0u;
      __threadfence();
    }
  }
}

__global__ void rope_table_kernel(float* cs, float* sn, int rows, int D, double theta) {
  const int half = D / 2;
  const long long total = (long long)rows * half;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    const long long pos = idx / half;
    const double inv_freq = pow(theta, -2.0 * (double)i / (double)D);
    const double ang = (double)pos * inv_freq;
    double s, c;
    sincos(ang, &s, &c);
    cs[idx] = (float)c;
    sn[idx] = (float)s;
  }
}

template <typename OutT>
__device__ __forceinline__ OutT cvt_out(float x);
template <>
__device__ __forceinline__ float cvt_out<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half cvt_out<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// One warp per (b, q, h) row of the query range.
template <typename OutT>
__global__ void combine_kernel(const AttnArgs a, const float* __restrict__ o_parts,
                               const float* __restrict__ lse_parts, int n_splits,
                               const int* __restrict__ part_row_begin) {
  const int nq = a.q_end - a.q_begin;
  const long long rows = (long long)a.B * nq * a.Hq;
  const long long warp_id = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= rows) return;
  const int h = (int)(warp_id % a.Hq);
  const long long bq = warp_id / a.Hq;
  const int q = a.q_begin + (int)(bq % nq);
  const int b = (int)(bq / nq);
  const long long lse_stride = (long long)a.B * a.Hq * a.Sq;
  const long long o_stride = (long long)a.B * a.Sq * a.Hq * a.D;
  const long long lse_idx = ((long long)b * a.Hq + h) * a.Sq + q;
  const long long o_row = (((long long)b * a.Sq + q) * a.Hq + h) * a.D;
  // Lane j (< 32) holds LSE_j; larger split counts fold in 32 at a time.
  float mx = -INFINITY;
  // Partial j holds rows [part_row_begin[j], ...) only (when given): rows
  // before it skip it.
  for (int j = lane; j < n_splits; j += 32)
    if (part_row_begin == nullptr || q >= part_row_begin[j]) mx = fmaxf(mx, lse_parts[j * lse_stride + lse_idx]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  float w_sum = 0.f;
  for (int j = lane; j < n_splits; j += 32) {
    if (part_row_begin != nullptr && q < part_row_begin[j]) continue;
    const float l = lse_parts[j * lse_stride + lse_idx];
    w_sum += (l == -INFINITY) ? 0.f : expf(l - mx);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) w_sum += __shfl_xor_sync(0xffffffffu, w_sum, off);
  const float lse = (w_sum > 0.f) ? mx + logf(w_sum) : -INFINITY;
  OutT* orow = reinterpret_cast<OutT*>(a.o) + (int64_t)b * a.o_sb + (int64_t)q * a.o_ss +
               (int64_t)h * a.o_sh;
  // Each lane owns columns lane, lane+32, ... (head_dim <= 256: at most 8).
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int j = 0; j < n_splits; ++j) {
    if (part_row_begin != nullptr && q < part_row_begin[j]) continue;
    const float l = lse_parts[j * lse_stride + lse_idx];
    if (l == -INFINITY) continue;  // split saw no key of this row
    const float w = expf(l - lse);
    const float* src = o_parts + j * o_stride + o_row;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < a.D) acc[i] = fmaf(w, src[d], acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < a.D) orow[d] = cvt_out<OutT>(acc[i]);
  }
  if (lane == 0 && a.lse != nullptr) a.lse[lse_idx] = lse;
}

template <typename OutT>
__global__ void fill_empty_kernel(const AttnArgs a) {
  const int nq = a.q_end - a.q_begin;
  const long long total = (long long)a.B * nq * a.Hq * a.D;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(idx % a.D);
    const long long r = idx / a.D;
    const int h = (int)(r % a.Hq);
    const long long bq = r / a.Hq;
    const int q = a.q_begin + (int)(bq % nq);
    const int b = (int)(bq / nq);
    const RowDst dst = row_dst(a, q);
    OutT* orow = reinterpret_cast<OutT*>(dst.o) + (int64_t)b * dst.o_sb + (int64_t)dst.row * dst.o_ss +
                 (int64_t)h * dst.o_sh;
    orow[d] = cvt_out<OutT>(0.f);
    if (d == 0 && dst.lse != nullptr) dst.lse[((long long)b * a.Hq + h) * dst.lse_rows + dst.row] = -INFINITY;
  }
}

// O[b, q, h, 0:D] = O_pad[b, q, h, 0:D] for rows [q_begin, q_end); O_pad is
// contiguous [B, Sq, H, Dp], O has element strides (sb, ss, sh). Element size
// 2 or 4 bytes (the output dtype).
template <typename E>
__global__ void unpad_kernel(const E* __restrict__ src, E* __restrict__ dst, int64_t sb, int64_t ss, int64_t sh,
                             int B, int Sq, int H, int D, int Dp, int q_begin, int q_end) {
  const int nq = q_end - q_begin;
  const long long total = (long long)B * nq * H * D;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(idx % D);
    const long long r = idx / D;
    const int h = (int)(r % H);
    const long long bq = r / H;
    const int q = q_begin + (int)(bq % nq);
    const int b = (int)(bq / nq);
    dst[(int64_t)b * sb + (int64_t)q * ss + (int64_t)h * sh + d] = src[(((int64_t)b * Sq + q) * H + h) * Dp + d];
  }
}

template <typename T>
cudaError_t stage_t(const StageBatch& in, cudaStream_t st) {
  StageBatch bt = in;
  bool vec = true;
  long long items[3] = {0, 0, 0}, total = 0;
  for (int j = 0; j < bt.n; ++j) {
    const StageJob& jb = bt.job[j];
    const int need = jb.cs ? 16 : 8;
    const long long rows = (long long)jb.B * jb.S * jb.H;
    // The vector path reads table rows with 16-byte loads.
    const bool tables16 =
        jb.cs == nullptr || ((reinterpret_cast<uintptr_t>(jb.cs) | reinterpret_cast<uintptr_t>(jb.sn)) & 15) == 0;
    vec &= (jb.Dp == jb.D) && (jb.D % need == 0) && (jb.D / need == 4 || jb.D / need == 8 || jb.D / need == 16) &&
           rows * (jb.D / need) < (1ll << 31) && tables16;
    items[j] = rows * jb.Dp;
    total += items[j];
  }
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  // Up to 16 blocks of 256 threads per SM, split among the jobs by size
  // (every job with work gets at least one block).
  long long blocks = (total / (vec ? 8 : 1) + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  int end = 0;
  for (int j = 0; j < 3; ++j) {
    int nb = 0;
    if (j < bt.n && items[j] > 0) nb = (int)std::max<long long>(1, blocks * items[j] / total);
    end += nb;
    bt.blk_end[j] = end;
  }
  cudaError_t e = launch_pdl(vec ? stage_vec_kernel<T> : stage_elem_kernel<T>, dim3((unsigned)end), dim3(threads),
                             0, st, bt);
  note_launch();
  if (e != cudaSuccess) return e;
  // One block per SM: when nothing overflowed every block reads 16 bytes and exits.
  e = launch_pdl(stage_fixup_kernel<T>, dim3(148), dim3(threads), 0, st, bt);
  note_launch();
  return e;
}

}  // namespace

cudaError_t launch_stage(const StageBatch& bt, cudaStream_t st) {
  if (bt.n <= 0) return cudaSuccess;
  switch (bt.in_dtype) {
    case kF16: return stage_t<__half>(bt, st);
    case kBF16: return stage_t<__nv_bfloat16>(bt, st);
    default: return stage_t<float>(bt, st);
  }
}

cudaError_t launch_unpad(const void* src, void* dst, int elem_bytes, int64_t sb, int64_t ss, int64_t sh, int B,
                         int Sq, int H, int D, int Dp, int q_begin, int q_end, cudaStream_t st) {
  const long long total = (long long)B * (q_end - q_begin) * H * D;
  if (total <= 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (elem_bytes == 4)
    unpad_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const float*>(src), static_cast<float*>(dst),
                                                           sb, ss, sh, B, Sq, H, D, Dp, q_begin, q_end);
  else
    unpad_kernel<uint16_t><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint16_t*>(src),
                                                              static_cast<uint16_t*>(dst), sb, ss, sh, B, Sq, H, D,
                                                              Dp, q_begin, q_end);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_rope_table(float* cs, float* sn, int rows, int D, double theta, cudaStream_t st) {
  const long long total = (long long)rows * (D / 2);
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  rope_table_kernel<<<(unsigned)blocks, 256, 0, st>>>(cs, sn, rows, D, theta);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_combine(const AttnArgs& a, const float* o_parts, const float* lse_parts,
                           int n_splits, const int* part_row_begin, int out_dtype, cudaStream_t st) {
  const long long rows = (long long)a.B * (a.q_end - a.q_begin) * a.Hq;
  if (rows <= 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = (rows * 32 + threads - 1) / threads;
  switch (out_dtype) {
    case kF16:
      combine_kernel<__half><<<(unsigned)blocks, threads, 0, st>>>(a, o_parts, lse_parts, n_splits, part_row_begin);
      break;
    case kBF16:
      combine_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(a, o_parts, lse_parts, n_splits,
                                                                          part_row_begin);
      break;
    default:
      combine_kernel<float><<<(unsigned)blocks, threads, 0, st>>>(a, o_parts, lse_parts, n_splits, part_row_begin);
      break;
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_fill_empty(const AttnArgs& a, int out_dtype, cudaStream_t st) {
  const long long total = (long long)a.B * (a.q_end - a.q_begin) * a.Hq * a.D;
  if (total <= 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  switch (out_dtype) {
    case kF16: fill_empty_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(a); break;
    case kBF16: fill_empty_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(a); break;
    default: fill_empty_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(a); break;
  }
  note_launch();
  return cudaGetLastError();
}

}  // namespace fa
