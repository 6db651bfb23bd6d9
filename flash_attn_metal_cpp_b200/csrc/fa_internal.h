// fa_internal.h - declarations shared by the host dispatcher and the kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda.h>
#include <cuda_fp16.h>

namespace fa {

// Problem description handed to every attention kernel. Sizes are
// validated on the host; strides are in elements.
struct AttnArgs {
  int B, Sq, Sk, Hq, Hk, D;
  int group;               // Hq / Hk
  float scale;             // softmax_scale as given
  float scale_log2;        // softmax_scale * log2(e)
  int causal;              // top-left causal mask: key k masked for query q iff k > q
  int win_left, win_right; // sliding window: key k masked iff k - q < -win_left (win_left >= 0)
                           // or k - q > win_right (win_right >= 0); negative = unbounded
  const float* alibi;      // [Hq] slopes: slope[h] * (k - q) added to the scaled score (NULL = none)
  int q_begin, q_end;      // query rows computed (partial API); [0, Sq) otherwise
  int kv_begin, kv_end;    // keys visited (split-KV); [0, Sk) otherwise
  int n_q_tiles;           // tiles of the query range for the launch
  int units_per_group;     // CTA order: (batch, KV-head) units taken this many at a time (>= 1)
  // Direct pointers (SIMT kernel and epilogues).
  const void* q;
  const void* k;
  const void* v;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  void* o;
  int64_t o_sb, o_ss, o_sh;
  float* lse;              // [B, Hq, Sq] (NULL = not written)
  const float* rope_cos;   // [rows, D/2] (SIMT kernel applies RoPE on load when non-NULL)
  const float* rope_sin;
  unsigned* status;        // device status word (timeouts)
  // Power-of-two exponents (Q, K, V) by which the staging pass scaled the
  // fp16 operands down to keep them finite (RangeRec::exp; NULL = none):
  // scores are multiplied by 2^(e_q + e_k) and O by 2^e_v.
  const int* range_exp;
  // Limit of every in-kernel wait in nanoseconds (0 = the default limit).
  unsigned long long wait_limit_ns;
  // Test hook: when > 0, the K producer of the CTA working on blockIdx.x 0
  // never loads K tile (skip_k_tile - 1), so the waits for it run out.
  int skip_k_tile;
  // Routed output (split-KV across devices): when route_rows > 0, query row r
  // is owned by owner r / route_rows and its O / LSE go to that owner's
  // staging slot instead of o / lse: route[owner] is the slot's O base
  // (contiguous [B, route_rows, Hq, D]), route[route_n + owner] its LSE base
  // ([B, Hq, route_rows]). Slots may live in peer-device memory.
  const unsigned long long* route;
  int route_n;
  int route_rows;
};

// Where the O row / LSE entry of absolute query row `row` go.
struct RowDst {
  void* o;
  float* lse;
  int row;                 // row index inside that destination
  int lse_rows;            // LSE row stride of that destination
  int64_t o_sb, o_ss, o_sh;
};

#ifdef __CUDACC__
__device__ __forceinline__ RowDst row_dst(const AttnArgs& a, int row) {
  if (a.route_rows > 0) {
    const int owner = row / a.route_rows;
    RowDst d;
    d.o = reinterpret_cast<void*>(a.route[owner]);
    d.lse = reinterpret_cast<float*>(a.route[a.route_n + owner]);
    d.row = row - owner * a.route_rows;
    d.lse_rows = a.route_rows;
    d.o_ss = (int64_t)a.Hq * a.D;
    d.o_sh = a.D;
    d.o_sb = (int64_t)a.route_rows * d.o_ss;
    return d;
  }
  return RowDst{a.o, a.lse, row, a.Sq, a.o_sb, a.o_ss, a.o_sh};
}
#endif

// Element type codes shared with fa_b200.h.
enum DType : int { kF16 = 0, kBF16 = 1, kF32 = 2 };

// Tensor-core path: Q/K/V described by TMA maps over 16-bit tensors.
// qk_bf16: Q and K are bf16 (else fp16); V is always fp16.
cudaError_t launch_attn_sm100(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tv, bool qk_bf16, int out_dtype,
                              cudaStream_t stream);

// Generic CUDA-core path: any head_dim <= 256, fp32/fp16/bf16 inputs.
cudaError_t launch_attn_simt(const AttnArgs& a, int in_dtype, int out_dtype, cudaStream_t stream);

// Per-call record of the fp16 staging pass, at the start of the workspace.
// It must be zero before the first call that uses it; the staging kernels
// leave it zero again (amax and done) when they finish.
struct RangeRec {
  unsigned amax_bits[4];   // max |value| staged per tensor (Q, K, V), as float bits
  int exp[4];              // exponent e: the staged tensor holds value * 2^-e
  unsigned done;           // fixup blocks finished; the last one resets amax and done
};
constexpr size_t kRangeRecBytes = 256;
static_assert(sizeof(RangeRec) <= kRangeRecBytes, "range record");

// One tensor staged as fp16 for the tensor-core kernel: y = rope(x) (when
// cs != NULL; rotate-half over the pairs (i, i + D/2) of the original D)
// converted to fp16 with Dp - D zero columns appended. x has element
// strides (sb, ss, sh) and S rows starting at its row 0; y is contiguous
// [B, y_rows, H, Dp] at the same row offset, so a row range of a larger
// tensor can be staged in place. Row s uses table row s of cs / sn.
struct StageJob {
  const void* x;
  int64_t sb, ss, sh;
  int B, S, H, D, Dp;
  const float* cs;
  const float* sn;
  __half* y;
  int y_rows;
  int slot;                // 0 = Q, 1 = K, 2 = V (index into RangeRec)
};

struct StageBatch {
  StageJob job[3];
  int n;
  int in_dtype;
  RangeRec* rec;           // device record (zeroed before its first use)
  int blk_end[3];          // set by launch_stage: blocks [blk_end[j-1], blk_end[j]) stage job j
};

// Stage every job of `b` (one kernel) and, in a second kernel, rescale a
// tensor whose largest value would overflow fp16 (|x| > 65504) by the
// smallest power of two that keeps it finite; the exponents land in
// b.rec->exp for the attention kernel (AttnArgs::range_exp).
cudaError_t launch_stage(const StageBatch& b, cudaStream_t stream);

// Copy the first D of Dp columns of a contiguous padded O into O (strides in
// elements), rows [q_begin, q_end); elem_bytes 2 or 4.
cudaError_t launch_unpad(const void* src, void* dst, int elem_bytes, int64_t sb, int64_t ss, int64_t sh, int B,
                         int Sq, int H, int D, int Dp, int q_begin, int q_end, cudaStream_t stream);

// cos/sin tables [rows, D/2] in float32 from theta, computed in double.
cudaError_t launch_rope_table(float* cos, float* sin, int rows, int D, double theta,
                              cudaStream_t stream);

// (O, LSE) merge of n split-KV partials.
// part_row_begin (device, n_splits ints, may be NULL): partial j holds rows
// [part_row_begin[j], ...) only; rows before it do not read it.
cudaError_t launch_combine(const AttnArgs& a, const float* o_parts, const float* lse_parts,
                           int n_splits, const int* part_row_begin, int out_dtype, cudaStream_t stream);

// Zero-fill O rows and set LSE to -inf (used when there is no key at all).
cudaError_t launch_fill_empty(const AttnArgs& a, int out_dtype, cudaStream_t stream);

// Per-thread launch counter (incremented by every launch_* above).
void note_launch();

// Launch with programmatic stream serialization: the kernel may begin while
// the previous kernel of the stream finishes; it must call grid_dep_wait()
// (fa_ptx.cuh) in every thread before touching global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace fa
