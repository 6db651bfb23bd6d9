// fa_aux.cu - memory-bound helper kernels around the attention kernels:
//   * prep_fp16:   rotate-half RoPE (common.metal:150-167) and/or conversion
//                  to fp16, producing the contiguous fp16 operands the
//                  tensor-core kernel loads with TMA;
//   * rope_table:  cos/sin tables [rows, D/2] (layout of the reference's
//                  host tables, src/flash_attn_core.cpp:343-349), computed
//                  in double and rounded to float;
//   * combine:     merge of split-KV partials (O_j, LSE_j);
//   * fill_empty:  O = 0, LSE = -inf when there is no key at all.
#include "fa_internal.h"
#include "fa_ptx.cuh"

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

__device__ __forceinline__ bool store8_half(__half* p, const float (&x)[8]) {
  uint4 w;
  w.x = pack_half2(x[0], x[1]);
  w.y = pack_half2(x[2], x[3]);
  w.z = pack_half2(x[4], x[5]);
  w.w = pack_half2(x[6], x[7]);
  *reinterpret_cast<uint4*>(p) = w;
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 8; ++i) ok &= fabsf(x[i]) <= 65504.f;
  return ok;
}

// One thread = 8 columns of the first half and (with RoPE) the matching 8
// columns of the second half of one (b, s, h) row. Requires D % 16 == 0.
template <typename T, bool ROPE>
__global__ void prep_fp16_kernel(const T* __restrict__ x, int64_t sb, int64_t ss, int64_t sh, int S,
                                 int H, int D, long long n_rows, const float* __restrict__ cs,
                                 const float* __restrict__ sn, __half* __restrict__ y, int y_rows,
                                 unsigned* status) {
  const int chunks = ROPE ? D / 16 : D / 8;
  const long long total = n_rows * chunks;
  bool ok = true;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long rowi = idx / chunks;
    const int ch = (int)(idx - rowi * chunks);
    const int h = (int)(rowi % H);
    const long long bs = rowi / H;
    const int s = (int)(bs % S);
    const int b = (int)(bs / S);
    const T* src = x + (int64_t)b * sb + (int64_t)s * ss + (int64_t)h * sh;
    __half* dst = y + (((int64_t)b * y_rows + s) * H + h) * D;  // y: [B, y_rows, H, D]
    if (ROPE) {
      const int half = D / 2;
      const int c0 = ch * 8;
      float a[8], bb[8];
      load8<T>(src + c0, a);
      load8<T>(src + c0 + half, bb);
      const float4* cp = reinterpret_cast<const float4*>(cs + (int64_t)s * half + c0);
      const float4* sp = reinterpret_cast<const float4*>(sn + (int64_t)s * half + c0);
      const float4 c_lo = cp[0], c_hi = cp[1], s_lo = sp[0], s_hi = sp[1];
      const float cv[8] = {c_lo.x, c_lo.y, c_lo.z, c_lo.w, c_hi.x, c_hi.y, c_hi.z, c_hi.w};
      const float sv[8] = {s_lo.x, s_lo.y, s_lo.z, s_lo.w, s_hi.x, s_hi.y, s_hi.z, s_hi.w};
      float ra[8], rb[8];
      rope_rotate8(a, bb, cv, sv, ra, rb);
      ok &= store8_half(dst + c0, ra);
      ok &= store8_half(dst + c0 + half, rb);
    } else {
      float a[8];
      load8<T>(src + ch * 8, a);
      ok &= store8_half(dst + ch * 8, a);
    }
  }
  if (!ok) atomicOr(status, FA_DEV_RANGE);
}

template <typename T>
cudaError_t prep_t(const void* x, int64_t sb, int64_t ss, int64_t sh, int B, int S, int H, int D,
                   const float* cs, const float* sn, __half* y, int y_rows, unsigned* status,
                   cudaStream_t st) {
  const long long n_rows = (long long)B * S * H;
  const long long total = n_rows * (cs ? D / 16 : D / 8);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (cs)
    prep_fp16_kernel<T, true><<<(unsigned)blocks, threads, 0, st>>>(
        reinterpret_cast<const T*>(x), sb, ss, sh, S, H, D, n_rows, cs, sn, y, y_rows, status);
  else
    prep_fp16_kernel<T, false><<<(unsigned)blocks, threads, 0, st>>>(
        reinterpret_cast<const T*>(x), sb, ss, sh, S, H, D, n_rows, cs, sn, y, y_rows, status);
  note_launch();
  return cudaGetLastError();
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

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }

// Zero-padded fp16 staging for head dims the tensor-core kernel does not take
// natively: y[.., 0:D] = rope(x) with the pairs (i, i + D/2) of the ORIGINAL
// D (an odd D's last column has no partner and is kept, as in the oracle),
// y[.., D:Dp] = 0, so every dot product is unchanged. One thread per output
// element of rows [0, S); y is contiguous [B, y_rows, H, Dp].
template <typename T>
__global__ void prep_pad_kernel(const T* __restrict__ x, int64_t sb, int64_t ss, int64_t sh, int S, int H, int D,
                                int Dp, long long n_rows, const float* __restrict__ cs,
                                const float* __restrict__ sn, __half* __restrict__ y, int y_rows,
                                unsigned* status) {
  const long long total = n_rows * Dp;
  const int half = D / 2;
  bool ok = true;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int col = (int)(idx % Dp);
    const long long rowi = idx / Dp;
    const int h = (int)(rowi % H);
    const long long bs = rowi / H;
    const int s = (int)(bs % S);
    const int b = (int)(bs / S);
    const T* src = x + (int64_t)b * sb + (int64_t)s * ss + (int64_t)h * sh;
    float val = 0.f;
    if (col < D) {
      val = ld_f<T>(src + col);
      if (cs != nullptr && col < 2 * half) {
        const int i = col < half ? col : col - half;  // pair index
        const float c = cs[(int64_t)s * half + i], sv = sn[(int64_t)s * half + i];
        const float a0 = ld_f<T>(src + i), a1 = ld_f<T>(src + i + half);
        // same rounding steps as rope_rotate8
        val = (col < half) ? __fmaf_rn(a0, c, -__fmul_rn(a1, sv)) : __fmaf_rn(a0, sv, __fmul_rn(a1, c));
      }
      ok &= fabsf(val) <= 65504.f;
    }
    y[(((int64_t)b * y_rows + s) * H + h) * Dp + col] = __float2half_rn(val);
  }
  if (!ok) atomicOr(status, FA_DEV_RANGE);
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

}  // namespace

cudaError_t launch_prep_pad(const void* x, int in_dtype, int64_t sb, int64_t ss, int64_t sh, int B, int S, int H,
                            int D, int Dp, const float* cs, const float* sn, __half* y, int y_rows, unsigned* status,
                            cudaStream_t st) {
  const long long n_rows = (long long)B * S * H;
  const long long total = n_rows * Dp;
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  switch (in_dtype) {
    case kF16:
      prep_pad_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const __half*>(x), sb, ss, sh, S,
                                                                H, D, Dp, n_rows, cs, sn, y, y_rows, status);
      break;
    case kBF16:
      prep_pad_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(x), sb, ss, sh, S, H, D, Dp, n_rows, cs, sn, y, y_rows, status);
      break;
    default:
      prep_pad_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const float*>(x), sb, ss, sh, S,
                                                               H, D, Dp, n_rows, cs, sn, y, y_rows, status);
      break;
  }
  note_launch();
  return cudaGetLastError();
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

cudaError_t launch_prep_fp16(const void* x, int in_dtype, int64_t sb, int64_t ss, int64_t sh, int B,
                             int S, int H, int D, const float* cs, const float* sn, __half* y,
                             int y_rows, unsigned* status, cudaStream_t st) {
  switch (in_dtype) {
    case kF16: return prep_t<__half>(x, sb, ss, sh, B, S, H, D, cs, sn, y, y_rows, status, st);
    case kBF16: return prep_t<__nv_bfloat16>(x, sb, ss, sh, B, S, H, D, cs, sn, y, y_rows, status, st);
    default: return prep_t<float>(x, sb, ss, sh, B, S, H, D, cs, sn, y, y_rows, status, st);
  }
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
