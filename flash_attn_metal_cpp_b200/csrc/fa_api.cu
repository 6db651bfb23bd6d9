// fa_api.cu - host side of the library: the C ABI declared in fa_b200.h.
//
// Replaces the reference's host runtime (src/flash_attn_core.cpp): device
// set-up (MetalDevice::initialize, :50-64), the power-of-two buffer pool
// (BufferPool, :193-246), and FlashAttentionForward::execute (:276-407),
// whose steps are kept in the same order for the host-pointer entry point:
// size buffers, take them from the pool, copy Q/K/V in, bind tables,
// dispatch, wait, copy O (and LSE) out, return buffers to the pool.
//
// Dispatch: fp16/bf16 with head_dim 64 or 128 and 16-byte aligned rows run
// on the tcgen05 kernel (fa_fwd_sm100.cu); everything else (fp32 inputs,
// other head dims) runs on the CUDA-core kernel (fa_fwd_simt.cu). There is
// no CPU path: without a CUDA device every entry point returns an error.
#include "../../include/fa_b200.h"
#include "fa_host.h"
#include "fa_internal.h"
#include "fa_ptx.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace fa {

namespace {

thread_local std::string g_last_error;
thread_local uint64_t g_launches = 0;
// Limit of every in-kernel wait (fa_set_wait_limit; 0 = the kernels' default).
std::atomic<unsigned long long> g_wait_limit_ns{0};
// Test hook (fa_test_stall_next_launch): K tile to withhold in the next
// tensor-core launch of this thread (0 = none).
thread_local int g_stall_k_tile = 0;
// Attention-kernel timing (fa_kernel_timing_enable / _read).
thread_local bool g_timing = false;
thread_local std::vector<std::pair<cudaEvent_t, cudaEvent_t>> g_events;

fa_status fail(fa_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

fa_status cuda_fail(cudaError_t e, const char* what) {
  return fail(FA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define FA_CUDA(call)                                        \
  do {                                                       \
    cudaError_t e_ = (call);                                 \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);      \
  } while (0)

size_t dtype_size(int dt) { return dt == kF32 ? 4 : 2; }

// Power-of-two size-bucketed cache of device buffers (the reference's
// BufferPool, src/flash_attn_core.cpp:199-234), one per device.
class DevicePool {
 public:
  void* get(size_t bytes) {
    size_t rounded = 256;
    while (rounded < bytes) rounded <<= 1;
    std::lock_guard<std::mutex> g(mu_);
    auto it = free_.find(rounded);
    if (it != free_.end() && !it->second.empty()) {
      void* p = it->second.back();
      it->second.pop_back();
      ++hits_;
      return p;
    }
    void* p = nullptr;
    if (cudaMalloc(&p, rounded) != cudaSuccess) {
      cudaGetLastError();
      // Free everything cached and retry once before giving up.
      release_locked();
      if (cudaMalloc(&p, rounded) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
      }
    }
    size_of_[p] = rounded;
    reserved_ += rounded;
    ++misses_;
    return p;
  }
  void put(void* p) {
    if (!p) return;
    std::lock_guard<std::mutex> g(mu_);
    free_[size_of_[p]].push_back(p);
  }
  void clear() {
    std::lock_guard<std::mutex> g(mu_);
    release_locked();
    hits_ = misses_ = 0;
  }
  void stats(uint64_t* h, uint64_t* m, uint64_t* b) {
    std::lock_guard<std::mutex> g(mu_);
    if (h) *h = hits_;
    if (m) *m = misses_;
    if (b) *b = reserved_;
  }

 private:
  void release_locked() {
    for (auto& kv : free_)
      for (void* p : kv.second) {
        cudaFree(p);
        reserved_ -= size_of_[p];
        size_of_.erase(p);
      }
    free_.clear();
  }
  std::mutex mu_;
  std::map<size_t, std::vector<void*>> free_;
  std::map<void*, size_t> size_of_;
  uint64_t hits_ = 0, misses_ = 0, reserved_ = 0;
};

// RAII lease of a pool buffer.
struct Lease {
  DevicePool* pool = nullptr;
  void* p = nullptr;
  Lease() = default;
  Lease(DevicePool* pl, size_t bytes) : pool(pl), p(bytes ? pl->get(bytes) : nullptr) {}
  Lease(const Lease&) = delete;
  Lease& operator=(const Lease&) = delete;
  ~Lease() {
    if (pool && p) pool->put(p);
  }
};

struct DeviceState {
  int device = -1;
  bool ready = false;
  unsigned* status = nullptr;       // in-kernel status word
  void* status_host = nullptr;      // pinned copy of it, read back by the host-pointer path
  cudaStream_t host_stream = nullptr;   // host-pointer path: compute
  cudaStream_t h2d_stream = nullptr;    // host-pointer path: copies in
  cudaStream_t d2h_stream = nullptr;    // host-pointer path: copies out
  DevicePool pool;
  std::mutex mu;                    // serialises the host-pointer path and the caches
  // RoPE table cache: (theta, D) -> tables with `rows` rows (grown on demand).
  struct Rope {
    int rows = 0;
    float* cs = nullptr;
    float* sn = nullptr;
  };
  std::map<std::pair<float, int>, Rope> rope;
  // Stream-ordered workspaces for fa_forward calls without a workspace.
  std::map<cudaStream_t, std::pair<void*, size_t>> ws;
  // Buffers replaced by larger ones. Another host thread may still hold (and
  // be about to enqueue work on) a replaced pointer, so none is freed before
  // fa_pool_clear, which synchronises the device first.
  std::vector<void*> retired;
};

std::mutex g_devices_mu;
std::map<int, std::unique_ptr<DeviceState>> g_devices;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

fa_status get_encode() {
  if (g_encode) return FA_OK;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                   cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled entry point not available");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return FA_OK;
}

fa_status device_state(DeviceState** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(FA_ERR_NO_DEVICE, std::string("no CUDA device: ") + cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> g(g_devices_mu);
  auto& slot = g_devices[dev];
  if (!slot) slot.reset(new DeviceState());
  DeviceState* ds = slot.get();
  if (!ds->ready) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
      cudaGetLastError();
      return fail(FA_ERR_NO_DEVICE, "no CUDA device visible");
    }
    cudaDeviceProp prop;
    FA_CUDA(cudaGetDeviceProperties(&prop, dev));
    if (prop.major != 10)
      return fail(FA_ERR_UNSUPPORTED, std::string("device '") + prop.name +
                                          "' is not sm_100 (B200); this library is built for sm_100a only");
    FA_CUDA(cudaMalloc(&ds->status, sizeof(unsigned)));
    FA_CUDA(cudaMemset(ds->status, 0, sizeof(unsigned)));
    ds->status_host = pinned_get(sizeof(unsigned));  // NULL: the host path reads the word synchronously
    FA_CUDA(cudaStreamCreateWithFlags(&ds->host_stream, cudaStreamNonBlocking));
    FA_CUDA(cudaStreamCreateWithFlags(&ds->h2d_stream, cudaStreamNonBlocking));
    FA_CUDA(cudaStreamCreateWithFlags(&ds->d2h_stream, cudaStreamNonBlocking));
    ds->device = dev;
    ds->ready = true;
  }
  *out = ds;
  return FA_OK;
}

// ---------------------------------------------------------------- validation
struct Plan {
  AttnArgs a;
  int dtype, out_dtype;
  bool tc;          // tensor-core path
  bool rope;
  bool need_q16, need_k16, need_v16;   // operands staged as fp16 in the workspace
  bool pad;         // head dim padded with zeros to d_pad for the tensor-core kernel
  int d_pad;
  float rope_theta;
  size_t ws_bytes;
};

void default_strides(const int64_t in[3], int64_t out[3], int64_t S, int64_t H, int64_t D) {
  if (in[0] == 0 && in[1] == 0 && in[2] == 0) {
    out[0] = S * H * D;
    out[1] = H * D;
    out[2] = D;
  } else {
    out[0] = in[0];
    out[1] = in[1];
    out[2] = in[2];
  }
}

fa_status make_plan(const fa_params* p, Plan* pl) {
  if (!p) return fail(FA_ERR_INVALID_ARG, "params is NULL");
  if (p->dtype < 0 || p->dtype > 2) return fail(FA_ERR_INVALID_ARG, "dtype must be 0 (f16), 1 (bf16) or 2 (f32)");
  const int out_dt = p->out_dtype < 0 ? p->dtype : p->out_dtype;
  if (out_dt > 2) return fail(FA_ERR_INVALID_ARG, "out_dtype must be -1, 0, 1 or 2");
  if (p->dropout_p != 0.f)
    return fail(FA_ERR_UNSUPPORTED, "dropout_p != 0 is not supported (the reference kernel ignores it)");
  if (p->has_alibi && p->alibi_slopes == nullptr)
    return fail(FA_ERR_INVALID_ARG, "has_alibi needs alibi_slopes (float32, one slope per query head)");
  if (p->head_dim == 0 || p->head_dim > 256)
    return fail(FA_ERR_UNSUPPORTED, "head_dim must be in [1, 256]");
  if (p->num_heads_k == 0 || p->num_heads_q % p->num_heads_k != 0)
    return fail(FA_ERR_INVALID_ARG, "num_heads_q must be a positive multiple of num_heads_k");
  const uint32_t group = p->num_heads_q / p->num_heads_k;
  if (p->gqa_group_size != 0 && p->gqa_group_size != group)
    return fail(FA_ERR_INVALID_ARG, "gqa_group_size must equal num_heads_q / num_heads_k");
  const uint64_t lim = (1ull << 31) - 1;
  if (p->batch_size > 65535 || p->seqlen_q > lim || p->seqlen_k > lim || p->num_heads_q > 65535)
    return fail(FA_ERR_INVALID_ARG, "tensor dimensions out of range");
  if (!std::isfinite(p->softmax_scale)) return fail(FA_ERR_INVALID_ARG, "softmax_scale must be finite");

  AttnArgs& a = pl->a;
  std::memset(&a, 0, sizeof(a));
  a.B = (int)p->batch_size;
  a.Sq = (int)p->seqlen_q;
  a.Sk = (int)p->seqlen_k;
  a.Hq = (int)p->num_heads_q;
  a.Hk = (int)p->num_heads_k;
  a.D = (int)p->head_dim;
  a.group = (int)group;
  a.scale = p->softmax_scale;
  a.scale_log2 = (float)((double)p->softmax_scale * 1.4426950408889634);
  a.causal = p->is_causal ? 1 : 0;
  a.win_left = p->window_left < 0 ? -1 : p->window_left;
  a.win_right = p->window_right < 0 ? -1 : p->window_right;
  a.alibi = p->has_alibi ? p->alibi_slopes : nullptr;
  a.q_begin = 0;
  a.q_end = a.Sq;
  a.kv_begin = 0;
  a.kv_end = a.Sk;
  int64_t qs[3], ks[3], vs[3], os[3];
  default_strides(p->q_stride, qs, a.Sq, a.Hq, a.D);
  default_strides(p->k_stride, ks, a.Sk, a.Hk, a.D);
  default_strides(p->v_stride, vs, a.Sk, a.Hk, a.D);
  default_strides(p->o_stride, os, a.Sq, a.Hq, a.D);
  a.q_sb = qs[0]; a.q_ss = qs[1]; a.q_sh = qs[2];
  a.k_sb = ks[0]; a.k_ss = ks[1]; a.k_sh = ks[2];
  a.v_sb = vs[0]; a.v_ss = vs[1]; a.v_sh = vs[2];
  a.o_sb = os[0]; a.o_ss = os[1]; a.o_sh = os[2];
  for (int i = 0; i < 3; ++i)
    if (qs[i] < 0 || ks[i] < 0 || vs[i] < 0 || os[i] < 0)
      return fail(FA_ERR_INVALID_ARG, "strides must be non-negative");

  pl->dtype = p->dtype;
  pl->out_dtype = out_dt;
  pl->rope = p->has_rotary != 0;
  pl->rope_theta = p->rope_theta;
  const int D = a.D;
  auto al = [](int64_t s, int64_t mult) { return s % mult == 0; };
  const int64_t in_mult = 16 / (int64_t)dtype_size(p->dtype);
  const int64_t out_mult = 16 / (int64_t)dtype_size(out_dt);
  bool strides_ok = true;
  for (int i = 0; i < 3; ++i)
    strides_ok &= al(qs[i], in_mult) && al(ks[i], in_mult) && al(vs[i], in_mult) && al(os[i], out_mult);
  // The tensor-core kernel folds the ALiBi bias into the raw score as
  // (slope / scale) * (k - q), so a zero scale with ALiBi takes the CUDA-core kernel.
  const bool tc_ok = (p->dtype == kF16 || p->dtype == kBF16) && !(p->has_alibi && p->softmax_scale == 0.f);
  // Head dims 64 and 128 run natively (operands zero-copy when 16-byte
  // aligned); any other head dim <= 128 is zero-padded to 64 or 128 by the
  // staging pass (padding adds zero terms to every dot product) and the first
  // D columns of the padded output are copied out.
  pl->tc = tc_ok && (D == 64 || D == 128) && strides_ok;
  pl->pad = tc_ok && !pl->tc && D < 128 && D != 64;
  pl->d_pad = D <= 64 ? 64 : 128;
  pl->need_q16 = pl->tc && pl->rope;
  pl->need_k16 = pl->tc && pl->rope;
  pl->need_v16 = pl->tc && p->dtype == kBF16;
  // Workspace: the staging pass's range record (kRangeRecBytes), then the
  // staged fp16 operands (and, for padded head dims, the padded output).
  size_t ws = 0;
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  if (pl->need_q16) ws += up((size_t)a.B * a.Sq * a.Hq * D * 2);
  if (pl->need_k16) ws += up((size_t)a.B * a.Sk * a.Hk * D * 2);
  if (pl->need_v16) ws += up((size_t)a.B * a.Sk * a.Hk * D * 2);
  if (pl->pad) {
    const size_t dp = (size_t)pl->d_pad;
    ws = up((size_t)a.B * a.Sq * a.Hq * dp * 2) + 2 * up((size_t)a.B * a.Sk * a.Hk * dp * 2) +
         up((size_t)a.B * a.Sq * a.Hq * dp * dtype_size(out_dt));
  }
  pl->ws_bytes = ws ? ws + kRangeRecBytes : 0;
  return FA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

fa_status encode_map(CUtensorMap* m, const void* base, bool bf16, int D, int H, int S, int B,
                     int64_t sb, int64_t ss, int64_t sh) {
  fa_status st = get_encode();
  if (st != FA_OK) return st;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)ss * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, 1, 128, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ERR_INVALID_ARG, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return FA_OK;
}

// Cached RoPE tables from theta with at least `rows` rows, one entry per
// (theta, D). A table that grows is replaced by a new allocation; the old
// one is retired (freed only by fa_pool_clear), since a call on another
// stream or thread may still read it. The new tables are built on `stream`;
// a call on another stream that then finds them waits for that build
// through `ready`.
fa_status rope_from_theta(DeviceState* ds, float theta, int D, int rows, cudaStream_t stream,
                          const float** cs, const float** sn) {
  std::lock_guard<std::mutex> g(ds->mu);
  auto& r = ds->rope[std::make_pair(theta, D)];
  if (!(r.cs && r.rows >= rows)) {
    if (r.cs) {
      ds->retired.push_back(r.cs);
      ds->retired.push_back(r.sn);
      r.cs = r.sn = nullptr;
      r.rows = 0;
    }
    const size_t bytes = (size_t)rows * (D / 2) * sizeof(float) + 16;
    float *c = nullptr, *s = nullptr;
    FA_CUDA(cudaMalloc(&c, bytes));
    cudaError_t e = cudaMalloc(&s, bytes);
    if (e != cudaSuccess) {
      cudaFree(c);
      return cuda_fail(e, "cudaMalloc (RoPE tables)");
    }
    e = launch_rope_table(c, s, rows, D, (double)theta, stream);
    // Other streams must not read the tables before they are built: finish
    // the build here (once per (theta, D) and size, outside any hot loop).
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
      cudaFree(c);
      cudaFree(s);
      return cuda_fail(e, "RoPE tables");
    }
    r.cs = c;
    r.sn = s;
    r.rows = rows;
  }
  *cs = r.cs;
  *sn = r.sn;
  return FA_OK;
}

// Per-stream workspace, grown on demand. A replaced buffer is retired, not
// freed: another host thread may hold it for a call it is still enqueuing
// on the same stream.
fa_status stream_workspace(DeviceState* ds, cudaStream_t stream, size_t bytes, void** out) {
  std::lock_guard<std::mutex> g(ds->mu);
  auto& w = ds->ws[stream];
  if (w.second < bytes) {
    if (w.first) ds->retired.push_back(w.first);
    w.first = nullptr;
    w.second = 0;
    FA_CUDA(cudaMalloc(&w.first, bytes));
    w.second = bytes;
    // The staging record must start at zero; the staging kernels keep it so.
    FA_CUDA(cudaMemsetAsync(w.first, 0, kRangeRecBytes, stream));
  }
  *out = w.first;
  return FA_OK;
}

// Job staging rows [lo, hi) of one (B, S, H, D) tensor into the fp16
// buffer y ([B, S, H, Dp] contiguous) at the same rows.
StageJob stage_job(const void* x, int dtype, int64_t sb, int64_t ss, int64_t sh, int B, int S, int H, int D,
                   int Dp, int lo, int hi, const float* cs, const float* sn, __half* y, int slot) {
  StageJob j;
  const int hd = D / 2;
  j.x = static_cast<const uint8_t*>(x) + (size_t)lo * ss * dtype_size(dtype);
  j.sb = sb;
  j.ss = ss;
  j.sh = sh;
  j.B = B;
  j.S = hi - lo;
  j.H = H;
  j.D = D;
  j.Dp = Dp;
  j.cs = cs ? cs + (size_t)lo * hd : nullptr;
  j.sn = sn ? sn + (size_t)lo * hd : nullptr;
  j.y = y + (size_t)lo * H * Dp;
  j.y_rows = S;
  j.slot = slot;
  return j;
}

// Core of fa_forward / fa_forward_partial once the plan is fixed.
// Core of every forward entry point once the plan is fixed. `ds` supplies
// the cached RoPE tables and per-stream workspace; it may be NULL when the
// caller passes both (cos/sin when RoPE is on, and a workspace when
// pl.ws_bytes > 0), which is how the allocation-free entry point calls it.
fa_status run(Plan& pl, const void* q, const void* k, const void* v, const float* cos,
              const float* sin, void* workspace, size_t ws_bytes, cudaStream_t stream,
              DeviceState* ds, unsigned* status) {
  AttnArgs& a = pl.a;
  a.status = status;
  a.wait_limit_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  a.skip_k_tile = 0;
  a.range_exp = nullptr;
  // A workspace from the caller (or the host path's pool) may hold anything:
  // clear its staging record. The per-stream workspace is cleared once when
  // allocated and kept clear by the staging kernels.
  const bool clear_record = workspace != nullptr && pl.ws_bytes > 0;
  if (a.q_end <= a.q_begin || a.B == 0 || a.Hq == 0) return FA_OK;
  if (!a.o && a.route_rows == 0) return fail(FA_ERR_INVALID_ARG, "NULL output pointer");
  // No key at all (Sk == 0 or an empty split): O = 0, LSE = -inf.
  if (a.kv_end <= a.kv_begin) {
    cudaError_t e = launch_fill_empty(a, pl.out_dtype, stream);
    return e == cudaSuccess ? FA_OK : cuda_fail(e, "fill_empty");
  }
  if (!q || !k || !v) return fail(FA_ERR_INVALID_ARG, "NULL tensor pointer");
  const float* cs = cos;
  const float* sn = sin;
  if (pl.rope && (cs == nullptr || sn == nullptr)) {
    if (!(pl.rope_theta > 0.f) || !std::isfinite(pl.rope_theta))
      return fail(FA_ERR_INVALID_ARG, "has_rotary needs cos/sin tables or rope_theta > 0");
    if (a.D % 2 != 0) return fail(FA_ERR_UNSUPPORTED, "RoPE from rope_theta needs an even head_dim");
    if (ds == nullptr) return fail(FA_ERR_INVALID_ARG, "RoPE tables missing");
    fa_status st = rope_from_theta(ds, pl.rope_theta, a.D, a.Sq > a.Sk ? a.Sq : a.Sk, stream, &cs, &sn);
    if (st != FA_OK) return st;
  }
  if (!pl.rope) cs = sn = nullptr;

  if (pl.pad) {
    // Head dim D -> d_pad: Q, K, V staged zero-padded (RoPE applied on the
    // original D's pairs), the tensor-core kernel writes a padded O into the
    // workspace, and its first D columns are copied to the caller's O.
    if (a.route_rows > 0) return fail(FA_ERR_UNSUPPORTED, "routed output needs head_dim 64 or 128");
    if (workspace == nullptr) {
      if (ds == nullptr) return fail(FA_ERR_INVALID_ARG, "workspace missing");
      fa_status st = stream_workspace(ds, stream, pl.ws_bytes, &workspace);
      if (st != FA_OK) return st;
    } else if (ws_bytes < pl.ws_bytes) {
      return fail(FA_ERR_INVALID_ARG, "workspace smaller than fa_workspace_size()");
    }
    const int Dp = pl.d_pad;
    RangeRec* rec = static_cast<RangeRec*>(workspace);
    if (clear_record) FA_CUDA(cudaMemsetAsync(rec, 0, kRangeRecBytes, stream));
    uint8_t* wp = static_cast<uint8_t*>(workspace) + kRangeRecBytes;
    auto take = [&](size_t bytes) {
      uint8_t* r = wp;
      wp += (bytes + 255) & ~size_t(255);
      return r;
    };
    __half* q16 = reinterpret_cast<__half*>(take((size_t)a.B * a.Sq * a.Hq * Dp * 2));
    __half* k16 = reinterpret_cast<__half*>(take((size_t)a.B * a.Sk * a.Hk * Dp * 2));
    __half* v16 = reinterpret_cast<__half*>(take((size_t)a.B * a.Sk * a.Hk * Dp * 2));
    void* opad = take((size_t)a.B * a.Sq * a.Hq * Dp * dtype_size(pl.out_dtype));
    const int q_lo = a.q_begin, q_hi = std::min(a.Sq, a.q_begin + (a.q_end - a.q_begin + 127) / 128 * 128);
    const int k_lo = a.kv_begin, k_hi = std::min(a.Sk, a.kv_begin + (a.kv_end - a.kv_begin + 127) / 128 * 128);
    StageBatch sb{};
    sb.in_dtype = pl.dtype;
    sb.rec = rec;
    sb.job[0] = stage_job(q, pl.dtype, a.q_sb, a.q_ss, a.q_sh, a.B, a.Sq, a.Hq, a.D, Dp, q_lo, q_hi, cs, sn, q16, 0);
    sb.job[1] = stage_job(k, pl.dtype, a.k_sb, a.k_ss, a.k_sh, a.B, a.Sk, a.Hk, a.D, Dp, k_lo, k_hi, cs, sn, k16, 1);
    sb.job[2] = stage_job(v, pl.dtype, a.v_sb, a.v_ss, a.v_sh, a.B, a.Sk, a.Hk, a.D, Dp, k_lo, k_hi, nullptr,
                          nullptr, v16, 2);
    sb.n = 3;
    cudaError_t e = launch_stage(sb, stream);
    if (e != cudaSuccess) return cuda_fail(e, "padded staging");
    a.range_exp = rec->exp;
    AttnArgs ap = a;
    ap.D = Dp;
    ap.o = opad;
    ap.o_ss = (int64_t)a.Hq * Dp;
    ap.o_sh = Dp;
    ap.o_sb = (int64_t)a.Sq * ap.o_ss;
    ap.n_q_tiles = (a.q_end - a.q_begin + 127) / 128;
    CUtensorMap tq, tk, tv;
    const int64_t qsb = (int64_t)a.Sq * a.Hq * Dp, qss = (int64_t)a.Hq * Dp;
    const int64_t ksb = (int64_t)a.Sk * a.Hk * Dp, kss = (int64_t)a.Hk * Dp;
    fa_status st = encode_map(&tq, q16, false, Dp, a.Hq, a.Sq, a.B, qsb, qss, Dp);
    if (st == FA_OK) st = encode_map(&tk, k16, false, Dp, a.Hk, a.Sk, a.B, ksb, kss, Dp);
    if (st == FA_OK) st = encode_map(&tv, v16, false, Dp, a.Hk, a.Sk, a.B, ksb, kss, Dp);
    if (st != FA_OK) return st;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    if (g_timing) {
      FA_CUDA(cudaEventCreate(&ev0));
      FA_CUDA(cudaEventCreate(&ev1));
      FA_CUDA(cudaEventRecord(ev0, stream));
    }
    ap.skip_k_tile = g_stall_k_tile;
    g_stall_k_tile = 0;
    e = launch_attn_sm100(ap, tq, tk, tv, false, pl.out_dtype, stream);
    if (g_timing) {
      FA_CUDA(cudaEventRecord(ev1, stream));
      g_events.emplace_back(ev0, ev1);
    }
    if (e != cudaSuccess) return cuda_fail(e, "attention (tensor-core kernel, padded head dim)");
    e = launch_unpad(opad, a.o, (int)dtype_size(pl.out_dtype), a.o_sb, a.o_ss, a.o_sh, a.B, a.Sq, a.Hq, a.D, Dp,
                     a.q_begin, a.q_end, stream);
    return e == cudaSuccess ? FA_OK : cuda_fail(e, "unpad output");
  }

  if (!pl.tc) {
    a.q = q;
    a.k = k;
    a.v = v;
    a.rope_cos = cs;
    a.rope_sin = sn;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    if (g_timing) {
      FA_CUDA(cudaEventCreate(&ev0));
      FA_CUDA(cudaEventCreate(&ev1));
      FA_CUDA(cudaEventRecord(ev0, stream));
    }
    cudaError_t e = launch_attn_simt(a, pl.dtype, pl.out_dtype, stream);
    if (g_timing) {
      FA_CUDA(cudaEventRecord(ev1, stream));
      g_events.emplace_back(ev0, ev1);
    }
    return e == cudaSuccess ? FA_OK : cuda_fail(e, "attention (CUDA-core kernel)");
  }

  // Tensor-core path.
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (a.route_rows == 0 && !aligned16(a.o)))
    return fail(FA_ERR_INVALID_ARG, "tensor base addresses must be 16-byte aligned");
  if (pl.ws_bytes > 0) {
    if (workspace == nullptr) {
      if (ds == nullptr) return fail(FA_ERR_INVALID_ARG, "workspace missing");
      fa_status st = stream_workspace(ds, stream, pl.ws_bytes, &workspace);
      if (st != FA_OK) return st;
    } else if (ws_bytes < pl.ws_bytes) {
      return fail(FA_ERR_INVALID_ARG, "workspace smaller than fa_workspace_size()");
    } else if (!aligned16(workspace)) {
      return fail(FA_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
    }
  }
  cudaError_t e;
  const void* qs = q;
  const void* ks = k;
  const void* vs = v;
  int64_t q_sb = a.q_sb, q_ss = a.q_ss, q_sh = a.q_sh;
  int64_t k_sb = a.k_sb, k_ss = a.k_ss, k_sh = a.k_sh;
  int64_t v_sb = a.v_sb, v_ss = a.v_ss, v_sh = a.v_sh;
  bool qk_bf16 = (pl.dtype == kBF16);
  if (pl.ws_bytes > 0) {
    // One staging launch for every operand that needs it (RoPE and / or
    // fp16), then the range fixup. Only the rows the kernel's tiles can load
    // are staged: the query range and the key range, each rounded up to
    // whole 128-row tiles.
    RangeRec* rec = static_cast<RangeRec*>(workspace);
    if (clear_record) FA_CUDA(cudaMemsetAsync(rec, 0, kRangeRecBytes, stream));
    uint8_t* wp = static_cast<uint8_t*>(workspace) + kRangeRecBytes;
    auto take = [&](size_t bytes) {
      uint8_t* r = wp;
      wp += (bytes + 255) & ~size_t(255);
      return reinterpret_cast<__half*>(r);
    };
    const int q_lo = a.q_begin, q_hi = std::min(a.Sq, a.q_begin + (a.q_end - a.q_begin + 127) / 128 * 128);
    const int k_lo = a.kv_begin, k_hi = std::min(a.Sk, a.kv_begin + (a.kv_end - a.kv_begin + 127) / 128 * 128);
    StageBatch sb{};
    sb.in_dtype = pl.dtype;
    sb.rec = rec;
    if (pl.need_q16) {
      __half* y = take((size_t)a.B * a.Sq * a.Hq * a.D * 2);
      sb.job[sb.n++] = stage_job(q, pl.dtype, a.q_sb, a.q_ss, a.q_sh, a.B, a.Sq, a.Hq, a.D, a.D, q_lo, q_hi, cs, sn,
                                 y, 0);
      qs = y;
      q_sb = (int64_t)a.Sq * a.Hq * a.D; q_ss = (int64_t)a.Hq * a.D; q_sh = a.D;
    }
    if (pl.need_k16) {
      __half* y = take((size_t)a.B * a.Sk * a.Hk * a.D * 2);
      sb.job[sb.n++] = stage_job(k, pl.dtype, a.k_sb, a.k_ss, a.k_sh, a.B, a.Sk, a.Hk, a.D, a.D, k_lo, k_hi, cs, sn,
                                 y, 1);
      ks = y;
      k_sb = (int64_t)a.Sk * a.Hk * a.D; k_ss = (int64_t)a.Hk * a.D; k_sh = a.D;
    }
    if (pl.need_q16 || pl.need_k16) qk_bf16 = false;
    if (pl.need_v16) {
      __half* y = take((size_t)a.B * a.Sk * a.Hk * a.D * 2);
      sb.job[sb.n++] = stage_job(v, pl.dtype, a.v_sb, a.v_ss, a.v_sh, a.B, a.Sk, a.Hk, a.D, a.D, k_lo, k_hi,
                                 nullptr, nullptr, y, 2);
      vs = y;
      v_sb = (int64_t)a.Sk * a.Hk * a.D; v_ss = (int64_t)a.Hk * a.D; v_sh = a.D;
    }
    e = launch_stage(sb, stream);
    if (e != cudaSuccess) return cuda_fail(e, "fp16 staging");
    a.range_exp = rec->exp;
  }
  CUtensorMap tq, tk, tv;
  fa_status st = encode_map(&tq, qs, qk_bf16, a.D, a.Hq, a.Sq, a.B, q_sb, q_ss, q_sh);
  if (st != FA_OK) return st;
  st = encode_map(&tk, ks, qk_bf16, a.D, a.Hk, a.Sk, a.B, k_sb, k_ss, k_sh);
  if (st != FA_OK) return st;
  st = encode_map(&tv, vs, false, a.D, a.Hk, a.Sk, a.B, v_sb, v_ss, v_sh);
  if (st != FA_OK) return st;
  a.n_q_tiles = (a.q_end - a.q_begin + 127) / 128;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  if (g_timing) {
    FA_CUDA(cudaEventCreate(&ev0));
    FA_CUDA(cudaEventCreate(&ev1));
    FA_CUDA(cudaEventRecord(ev0, stream));
  }
  a.skip_k_tile = g_stall_k_tile;
  g_stall_k_tile = 0;
  e = launch_attn_sm100(a, tq, tk, tv, qk_bf16, pl.out_dtype, stream);
  if (g_timing) {
    FA_CUDA(cudaEventRecord(ev1, stream));
    g_events.emplace_back(ev0, ev1);
  }
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "attention (tensor-core kernel)");
}

}  // namespace

void note_launch() { ++g_launches; }

}  // namespace fa

using namespace fa;

extern "C" {

void fa_params_init(fa_params* p) {
  if (!p) return;
  std::memset(p, 0, sizeof(*p));
  p->window_left = -1;
  p->window_right = -1;
  p->dtype = FA_F16;
  p->out_dtype = -1;
}

fa_status fa_init(int device) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(FA_ERR_NO_DEVICE, "no CUDA device visible");
  }
  if (device == -1) FA_CUDA(cudaGetDevice(&device));  // the calling thread's current device
  if (device < 0 || device >= n) return fail(FA_ERR_INVALID_ARG, "device index out of range");
  FA_CUDA(cudaSetDevice(device));
  DeviceState* ds = nullptr;
  return device_state(&ds);
}

fa_status fa_device_info(int device, char* name, size_t name_len, uint64_t* total_mem, int* initialized) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    if (name && name_len) std::snprintf(name, name_len, "%s", "No device");
    if (total_mem) *total_mem = 0;
    if (initialized) *initialized = 0;
    return fail(FA_ERR_NO_DEVICE, "no CUDA device visible");
  }
  if (device == -1) FA_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= n) return fail(FA_ERR_INVALID_ARG, "device index out of range");
  cudaDeviceProp prop;
  FA_CUDA(cudaGetDeviceProperties(&prop, device));
  if (name && name_len) std::snprintf(name, name_len, "%s", prop.name);
  if (total_mem) *total_mem = (uint64_t)prop.totalGlobalMem;
  if (initialized) {
    std::lock_guard<std::mutex> g(g_devices_mu);
    auto it = g_devices.find(device);
    *initialized = (it != g_devices.end() && it->second && it->second->ready) ? 1 : 0;
  }
  return FA_OK;
}

size_t fa_workspace_size(const fa_params* p) {
  Plan pl;
  if (make_plan(p, &pl) != FA_OK) return 0;
  return pl.ws_bytes;
}

size_t fa_tensor_bytes(uint32_t batch, uint32_t seq, uint32_t heads, uint32_t dim, int32_t dtype) {
  return (size_t)batch * seq * heads * dim * dtype_size(dtype);
}

fa_status fa_forward(const fa_params* p, const void* q, const void* k, const void* v, void* o,
                     float* lse, const float* cos, const float* sin, void* workspace,
                     size_t workspace_bytes, void* stream) {
  Plan pl;
  fa_status st = make_plan(p, &pl);
  if (st != FA_OK) return st;
  DeviceState* ds = nullptr;
  st = device_state(&ds);
  if (st != FA_OK) return st;
  pl.a.o = o;
  pl.a.lse = lse;
  return run(pl, q, k, v, cos, sin, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), ds, ds->status);
}

fa_status fa_forward_partial(const fa_params* p, const void* q, const void* k, const void* v,
                             float* o_partial, float* lse_partial, const float* cos, const float* sin,
                             uint32_t q_begin, uint32_t q_end, uint32_t kv_begin, uint32_t kv_end,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (!p) return fail(FA_ERR_INVALID_ARG, "params is NULL");
  fa_params pp = *p;
  pp.out_dtype = FA_F32;
  pp.o_stride[0] = pp.o_stride[1] = pp.o_stride[2] = 0;
  Plan pl;
  fa_status st = make_plan(&pp, &pl);
  if (st != FA_OK) return st;
  if (q_begin > q_end || q_end > p->seqlen_q || kv_begin > kv_end || kv_end > p->seqlen_k)
    return fail(FA_ERR_INVALID_ARG, "partial ranges out of bounds");
  if (!lse_partial) return fail(FA_ERR_INVALID_ARG, "lse_partial is required");
  DeviceState* ds = nullptr;
  st = device_state(&ds);
  if (st != FA_OK) return st;
  pl.a.q_begin = (int)q_begin;
  pl.a.q_end = (int)q_end;
  pl.a.kv_begin = (int)kv_begin;
  pl.a.kv_end = (int)kv_end;
  pl.a.o = o_partial;
  pl.a.lse = lse_partial;
  return run(pl, q, k, v, cos, sin, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), ds, ds->status);
}

fa_status fa_combine(const fa_params* p, const float* o_parts, const float* lse_parts, int32_t n_splits,
                     void* o, float* lse, uint32_t q_begin, uint32_t q_end, void* stream) {
  return fa_combine_ranges(p, o_parts, lse_parts, n_splits, nullptr, o, lse, q_begin, q_end, stream);
}

fa_status fa_combine_ranges(const fa_params* p, const float* o_parts, const float* lse_parts, int32_t n_splits,
                            const int32_t* part_row_begin, void* o, float* lse, uint32_t q_begin, uint32_t q_end,
                            void* stream) {
  Plan pl;
  fa_status st = make_plan(p, &pl);
  if (st != FA_OK) return st;
  if (n_splits <= 0 || !o_parts || !lse_parts || !o) return fail(FA_ERR_INVALID_ARG, "bad combine arguments");
  if (q_begin > q_end || q_end > p->seqlen_q) return fail(FA_ERR_INVALID_ARG, "row range out of bounds");
  DeviceState* ds = nullptr;
  st = device_state(&ds);
  if (st != FA_OK) return st;
  pl.a.q_begin = (int)q_begin;
  pl.a.q_end = (int)q_end;
  pl.a.o = o;
  pl.a.lse = lse;
  cudaError_t e = launch_combine(pl.a, o_parts, lse_parts, n_splits, part_row_begin, pl.out_dtype,
                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "combine");
}

fa_status fa_forward_range(const fa_params* p, const void* q, const void* k, const void* v, void* o,
                           float* lse, const float* cos, const float* sin, uint32_t q_begin,
                           uint32_t q_end, uint32_t kv_begin, uint32_t kv_end, const fa_route* route,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (!p) return fail(FA_ERR_INVALID_ARG, "params is NULL");
  fa_params pp = *p;
  if (route) pp.o_stride[0] = pp.o_stride[1] = pp.o_stride[2] = 0;  // slots are contiguous
  Plan pl;
  fa_status st = make_plan(&pp, &pl);
  if (st != FA_OK) return st;
  if (q_begin > q_end || q_end > p->seqlen_q || kv_begin > kv_end || kv_end > p->seqlen_k)
    return fail(FA_ERR_INVALID_ARG, "row ranges out of bounds");
  AttnArgs& a = pl.a;
  if (route) {
    if (!route->table || route->n_owners <= 0 || route->owner_rows == 0 || route->owner_rows % 128 != 0)
      return fail(FA_ERR_INVALID_ARG, "route needs a table, n_owners > 0 and owner_rows a multiple of 128");
    if ((uint64_t)route->n_owners * route->owner_rows < q_end)
      return fail(FA_ERR_INVALID_ARG, "route does not cover the query range");
    // Every 128-row tile must fall inside one owner's block.
    if (q_begin % 128 != 0) return fail(FA_ERR_INVALID_ARG, "routed q_begin must be a multiple of 128");
    a.route = reinterpret_cast<const unsigned long long*>(route->table);
    a.route_n = route->n_owners;
    a.route_rows = (int)route->owner_rows;
    o = nullptr;  // rows go to the owners' slots
    lse = nullptr;
  }
  DeviceState* ds = nullptr;
  st = device_state(&ds);
  if (st != FA_OK) return st;
  a.q_begin = (int)q_begin;
  a.q_end = (int)q_end;
  a.kv_begin = (int)kv_begin;
  a.kv_end = (int)kv_end;
  a.o = o;
  a.lse = lse;
  return run(pl, q, k, v, cos, sin, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), ds, ds->status);
}

// ------------------------------------------------------------ CUDA IPC
// Staging buffers that peers write split-KV partials into. Plain cudaMalloc
// memory (the only kind cudaIpcGetMemHandle accepts), opened by peers with
// lazy peer access; plain device memory, nothing else is mapped.
static_assert(sizeof(fa_ipc_handle) == sizeof(cudaIpcMemHandle_t), "IPC handle size");

fa_status fa_ipc_alloc(size_t bytes, void** dev_ptr, fa_ipc_handle* handle) {
  if (!dev_ptr || !handle || bytes == 0) return fail(FA_ERR_INVALID_ARG, "bad fa_ipc_alloc arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (IPC staging)");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaIpcGetMemHandle");
  }
  std::memcpy(handle->bytes, &h, sizeof(h));
  *dev_ptr = p;
  return FA_OK;
}

fa_status fa_ipc_free(void* dev_ptr) {
  cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "cudaFree (IPC staging)");
}

fa_status fa_ipc_open(const fa_ipc_handle* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return fail(FA_ERR_INVALID_ARG, "bad fa_ipc_open arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

fa_status fa_ipc_close(void* dev_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

fa_status fa_forward_host(const fa_params* p, const void* q, const void* k, const void* v, void* o,
                          float* lse, const float* cos, const float* sin) {
  Plan pl;
  fa_status st = make_plan(p, &pl);
  if (st != FA_OK) return st;
  if (!q || !k || !v || !o) return fail(FA_ERR_INVALID_ARG, "NULL host pointer");
  DeviceState* ds = nullptr;
  st = device_state(&ds);
  if (st != FA_OK) return st;
  const AttnArgs& a = pl.a;
  // Host buffers are taken as contiguous BSHD (the reference assumes C order too).
  if (p->q_stride[0] || p->k_stride[0] || p->v_stride[0] || p->o_stride[0] || p->q_stride[1] ||
      p->k_stride[1] || p->v_stride[1] || p->o_stride[1])
    return fail(FA_ERR_INVALID_ARG, "host-pointer path takes contiguous tensors only");
  const size_t in_sz = dtype_size(pl.dtype), out_sz = dtype_size(pl.out_dtype);
  const size_t q_bytes = (size_t)a.B * a.Sq * a.Hq * a.D * in_sz;
  const size_t k_bytes = (size_t)a.B * a.Sk * a.Hk * a.D * in_sz;
  const size_t o_bytes = (size_t)a.B * a.Sq * a.Hq * a.D * out_sz;
  const size_t lse_bytes = (size_t)a.B * a.Hq * a.Sq * sizeof(float);
  const size_t tab_bytes = (size_t)(a.Sq > a.Sk ? a.Sq : a.Sk) * (a.D / 2) * sizeof(float);
  const bool tables = p->has_rotary && cos && sin && tab_bytes > 0;
  cudaStream_t s = ds->host_stream;
  Lease dq(&ds->pool, q_bytes), dk(&ds->pool, k_bytes), dv(&ds->pool, k_bytes), dout(&ds->pool, o_bytes),
      dl(&ds->pool, lse ? lse_bytes : 0), dc(&ds->pool, tables ? tab_bytes : 0),
      dsn(&ds->pool, tables ? tab_bytes : 0), dws(&ds->pool, pl.ws_bytes);
  if ((q_bytes && !dq.p) || (k_bytes && (!dk.p || !dv.p)) || (o_bytes && !dout.p) || (lse && lse_bytes && !dl.p) ||
      (tables && (!dc.p || !dsn.p)) || (pl.ws_bytes && !dws.p))
    return fail(FA_ERR_CUDA, "device allocation failed");
  const float* tc = tables ? static_cast<const float*>(dc.p) : nullptr;
  const float* tsn = tables ? static_cast<const float*>(dsn.p) : nullptr;
  // ALiBi slopes arrive in host memory here: stage them next to the tensors.
  Lease dal(&ds->pool, p->has_alibi ? (size_t)a.Hq * sizeof(float) : 0);
  if (p->has_alibi) {
    if (!dal.p) return fail(FA_ERR_CUDA, "device allocation failed");
    FA_CUDA(cudaMemcpyAsync(dal.p, p->alibi_slopes, (size_t)a.Hq * sizeof(float), cudaMemcpyHostToDevice, s));
    pl.a.alibi = static_cast<const float*>(dal.p);
  }

  // Pipeline over query-row blocks: for each batch, K and V are copied in
  // first, then Q in blocks of rows, the block with the LAST rows first (under
  // the causal mask it is the heaviest, and the final block -- whose compute
  // and copy-out form the tail after the last input byte -- is the lightest).
  // A block is computed as soon as it has landed, against the keys its rows
  // can see, and its O rows (contiguous in BSHD) are copied out while later
  // blocks stream in. Copy in, compute and copy out run on three streams
  // ordered by events.
  struct Chunk { int b, r0, r1; bool kv_first; };
  std::vector<Chunk> chunks;
  const bool small = q_bytes + 2 * k_bytes < (size_t(16) << 20);
  if (!small && a.Sq > 0) {
    // About 16 blocks in all, each still filling the GPU (>= 2 CTAs of 256
    // rows per SM). (Measured on cfg4: finer blocks lengthen the input
    // stream -- smaller copies and more copy-out interleaving -- and make the
    // kernels of the last batch trail the copies; 12 blocks end 0.8 ms after
    // the last input byte and are the fastest of the splits tried.)
    const long long max_blocks = std::max<long long>(1, (long long)a.Sq * a.Hq / (256LL * 296));
    const int per_batch = (int)std::min<long long>(std::max(1, (16 + a.B - 1) / a.B), max_blocks);
    // Block starts are multiples of 256 rows, so every CTA (and every warp's
    // rows) is the same as in a one-piece launch and the results are
    // bit-identical to fa_forward's.
    const int rows = ((a.Sq + per_batch - 1) / per_batch + 255) / 256 * 256;
    const int n_blk = (a.Sq + rows - 1) / rows;
    for (int b = 0; b < a.B; ++b)
      for (int i = n_blk - 1; i >= 0; --i)
        chunks.push_back({b, i * rows, std::min(a.Sq, (i + 1) * rows), i == n_blk - 1});
    // The last block's compute and copy-out come after the last input byte:
    // cut it into halving pieces down to 256 rows, so the tail is one small
    // block (measured on cfg4: 0.68 ms from the last input byte to the last
    // output byte with a 2816-row final block).
    if (chunks.size() > 1) {
      Chunk last = chunks.back();
      chunks.pop_back();
      int hi = last.r1;
      while (hi - last.r0 > 256) {
        const int lo = std::max(last.r0, (last.r0 + (hi - last.r0) / 2) / 256 * 256);
        if (lo == last.r0) break;
        chunks.push_back({last.b, lo, hi, last.kv_first && hi == last.r1});
        hi = lo;
      }
      chunks.push_back({last.b, last.r0, hi, last.kv_first && hi == last.r1});
    }
  }
  const bool one_piece = chunks.size() <= 1 || q_bytes == 0 || k_bytes == 0;
  if (one_piece) chunks.assign(1, Chunk{0, 0, a.Sq, true});

  // Host memory. Pinned (page-locked) buffers are DMA'd directly. Pageable
  // inputs are first copied into pinned staging by the copy workers, in the
  // order the copies below are issued, each DMA waiting only for its own
  // bytes; pageable outputs are DMA'd into pinned staging and copied out at
  // the end. (The driver's own route for pageable memory is several times
  // slower than the link.)
  struct Src { const void* user; size_t bytes; bool pageable; size_t stage_off; };
  Src srcs[5] = {{q, q_bytes, false, 0}, {k, k_bytes, false, 0}, {v, k_bytes, false, 0},
                 {cos, tables ? tab_bytes : 0, false, 0}, {sin, tables ? tab_bytes : 0, false, 0}};
  size_t stage_in = 0;
  for (Src& x : srcs)
    if (x.bytes && !host_is_pinned(x.user)) {
      x.pageable = true;
      x.stage_off = stage_in;
      stage_in += (x.bytes + 255) & ~size_t(255);
    }
  const bool o_pg = o_bytes && !host_is_pinned(o);
  const bool l_pg = lse && lse_bytes && !host_is_pinned(lse);
  const size_t o_stage = o_pg ? ((o_bytes + 255) & ~size_t(255)) : 0;
  const size_t stage_out = o_stage + (l_pg ? lse_bytes : 0);
  struct PinnedLease {
    void* p = nullptr;
    explicit PinnedLease(size_t n) : p(n ? pinned_get(n) : nullptr) {}
    ~PinnedLease() { pinned_put(p); }
  } pin_in(stage_in), pin_out(stage_out);
  if (stage_in && !pin_in.p)  // no pinned memory to spare: the driver's pageable route
    for (Src& x : srcs) x.pageable = false;
  char* st_in = static_cast<char*>(pin_in.p);
  char* st_out = static_cast<char*>(pin_out.p);
  void* o_dst = (o_pg && st_out) ? st_out : o;
  float* l_dst = (l_pg && st_out) ? reinterpret_cast<float*>(st_out + o_stage) : lse;

  // Every host->device copy in issue order: tables first, then per chunk the
  // batch's K and V (with its first block) and the block's Q rows.
  struct H2D { int chunk; void* dst; int src; size_t off, bytes; int region; };
  std::vector<H2D> h2d;
  if (tables) {
    h2d.push_back({-1, dc.p, 3, 0, tab_bytes, -1});
    h2d.push_back({-1, dsn.p, 4, 0, tab_bytes, -1});
  }
  const size_t q_row = (size_t)a.Hq * a.D, k_row = (size_t)a.Hk * a.D;  // elements per sequence row
  for (size_t c = 0; c < chunks.size(); ++c) {
    const Chunk& ch = chunks[c];
    if (one_piece) {
      if (k_bytes) {
        h2d.push_back({0, dk.p, 1, 0, k_bytes, -1});
        h2d.push_back({0, dv.p, 2, 0, k_bytes, -1});
      }
      if (q_bytes) h2d.push_back({0, dq.p, 0, 0, q_bytes, -1});
      continue;
    }
    const size_t k_off = (size_t)ch.b * a.Sk * k_row * in_sz;
    const size_t q_off = ((size_t)ch.b * a.Sq + ch.r0) * q_row * in_sz;
    if (ch.kv_first) {
      h2d.push_back({(int)c, static_cast<char*>(dk.p) + k_off, 1, k_off, (size_t)a.Sk * k_row * in_sz, -1});
      h2d.push_back({(int)c, static_cast<char*>(dv.p) + k_off, 2, k_off, (size_t)a.Sk * k_row * in_sz, -1});
    }
    h2d.push_back({(int)c, static_cast<char*>(dq.p) + q_off, 0, q_off, (size_t)(ch.r1 - ch.r0) * q_row * in_sz, -1});
  }
  std::vector<CopyRegion> regions;
  for (H2D& h : h2d) {
    const Src& x = srcs[h.src];
    if (!x.pageable) continue;
    h.region = (int)regions.size();
    regions.push_back({st_in + x.stage_off + h.off, static_cast<const char*>(x.user) + h.off, h.bytes});
  }
  Stager stager;
  if (!regions.empty()) stager.start(std::move(regions));
  auto issue_h2d = [&](const H2D& h, cudaStream_t stream) -> cudaError_t {
    const Src& x = srcs[h.src];
    const char* from = static_cast<const char*>(x.user) + h.off;
    if (h.region >= 0) {
      stager.wait((size_t)h.region);
      from = st_in + x.stage_off + h.off;
    }
    return cudaMemcpyAsync(h.dst, from, h.bytes, cudaMemcpyHostToDevice, stream);
  };
  // The in-kernel status word is read back with the results (no extra sync).
  unsigned* status_host = static_cast<unsigned*>(ds->status_host);
  auto finish_status = [&]() -> fa_status {
    if (status_host == nullptr || *status_host != 0) return fa_check_device_status();
    return FA_OK;
  };
  // Pageable outputs: copy the staged results out with the workers (the
  // same stager: start() ends the input job first, one job at a time).
  auto copy_out = [&]() {
    std::vector<CopyRegion> outs;
    if (o_pg && st_out) outs.push_back({o, st_out, o_bytes});
    if (l_pg && st_out) outs.push_back({lse, st_out + o_stage, lse_bytes});
    stager.finish();
    if (outs.empty()) return;
    stager.start(std::move(outs));
    stager.finish();
  };

  if (one_piece) {
    // One piece: copy in, run, copy out on one stream.
    for (const H2D& h : h2d) FA_CUDA(issue_h2d(h, s));
    pl.a.o = dout.p;
    pl.a.lse = static_cast<float*>(dl.p);
    st = run(pl, dq.p ? dq.p : (const void*)1, dk.p ? dk.p : (const void*)1, dv.p ? dv.p : (const void*)1, tc,
             tsn, dws.p, pl.ws_bytes, s, ds, ds->status);
    if (st != FA_OK) {
      stager.finish();
      cudaStreamSynchronize(s);
      return st;
    }
    if (o_bytes) FA_CUDA(cudaMemcpyAsync(o_dst, dout.p, o_bytes, cudaMemcpyDeviceToHost, s));
    if (lse && lse_bytes) FA_CUDA(cudaMemcpyAsync(l_dst, dl.p, lse_bytes, cudaMemcpyDeviceToHost, s));
    if (status_host) FA_CUDA(cudaMemcpyAsync(status_host, ds->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
    FA_CUDA(cudaStreamSynchronize(s));
    copy_out();
    return finish_status();
  }

  cudaStream_t s_in = ds->h2d_stream, s_out = ds->d2h_stream;
  auto sync_all = [&]() {
    cudaStreamSynchronize(s_in);
    cudaStreamSynchronize(s);
    cudaStreamSynchronize(s_out);
  };
  // The ALiBi copy above was queued on `s`; the copy stream waits for it too.
  cudaEvent_t ev_tab;
  FA_CUDA(cudaEventCreateWithFlags(&ev_tab, cudaEventDisableTiming));
  FA_CUDA(cudaEventRecord(ev_tab, s));
  FA_CUDA(cudaStreamWaitEvent(s_in, ev_tab, 0));
  cudaEventDestroy(ev_tab);
  std::vector<cudaEvent_t> ev_in(chunks.size()), ev_done(chunks.size());
  for (size_t c = 0; c < chunks.size(); ++c) {
    FA_CUDA(cudaEventCreateWithFlags(&ev_in[c], cudaEventDisableTiming));
    FA_CUDA(cudaEventCreateWithFlags(&ev_done[c], cudaEventDisableTiming));
  }
  auto destroy_events = [&]() {
    for (size_t c = 0; c < chunks.size(); ++c) {
      cudaEventDestroy(ev_in[c]);
      cudaEventDestroy(ev_done[c]);
    }
  };
  st = FA_OK;
  size_t hi = 0;  // next entry of h2d
  for (size_t c = 0; c < chunks.size() && st == FA_OK; ++c) {
    const Chunk& ch = chunks[c];
    const size_t k_off = (size_t)ch.b * a.Sk * k_row;                  // elements
    const size_t q_off = ((size_t)ch.b * a.Sq + ch.r0) * q_row;
    const size_t nrows = (size_t)(ch.r1 - ch.r0);
    // copy in: the tables (before the first chunk), the batch's K and V with
    // its first block, then the block's Q rows
    cudaError_t e = cudaSuccess;
    for (; hi < h2d.size() && h2d[hi].chunk <= (int)c && e == cudaSuccess; ++hi) e = issue_h2d(h2d[hi], s_in);
    if (e == cudaSuccess) e = cudaEventRecord(ev_in[c], s_in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ev_in[c], 0);
    if (e != cudaSuccess) {
      st = cuda_fail(e, "chunk copy in");
      break;
    }
    // compute: rows [r0, r1) of batch b against the keys they can see
    Plan sub = pl;
    sub.a.B = 1;
    sub.a.q_begin = ch.r0;
    sub.a.q_end = ch.r1;
    sub.a.kv_begin = 0;
    sub.a.kv_end = a.causal ? std::min(a.Sk, ch.r1) : a.Sk;
    sub.a.o = static_cast<char*>(dout.p) + (size_t)ch.b * a.Sq * q_row * out_sz;
    sub.a.lse = dl.p ? static_cast<float*>(dl.p) + (size_t)ch.b * a.Hq * a.Sq : nullptr;
    st = run(sub, static_cast<const char*>(dq.p) + (size_t)ch.b * a.Sq * q_row * in_sz,
             static_cast<const char*>(dk.p) + k_off * in_sz, static_cast<const char*>(dv.p) + k_off * in_sz, tc, tsn,
             dws.p, pl.ws_bytes, s, ds, ds->status);
    if (st != FA_OK) break;
    e = cudaEventRecord(ev_done[c], s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s_out, ev_done[c], 0);
    // copy out: the block's O rows, and its LSE columns [r0, r1) of every head
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<char*>(o_dst) + q_off * out_sz, static_cast<const char*>(dout.p) + q_off * out_sz,
                          nrows * q_row * out_sz, cudaMemcpyDeviceToHost, s_out);
    if (e == cudaSuccess && lse) {
      const size_t l_off = (size_t)ch.b * a.Hq * a.Sq + ch.r0;
      e = cudaMemcpy2DAsync(l_dst + l_off, (size_t)a.Sq * sizeof(float), static_cast<const float*>(dl.p) + l_off,
                            (size_t)a.Sq * sizeof(float), nrows * sizeof(float), (size_t)a.Hq,
                            cudaMemcpyDeviceToHost, s_out);
    }
    if (e != cudaSuccess) st = cuda_fail(e, "chunk copy out");
  }
  if (st == FA_OK && status_host) {
    cudaError_t e = cudaMemcpyAsync(status_host, ds->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) st = cuda_fail(e, "status read-back");
  }
  stager.finish();
  sync_all();
  destroy_events();
  if (st != FA_OK) return st;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "pipelined host path");
  copy_out();
  return finish_status();
}

fa_status fa_host_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(FA_ERR_INVALID_ARG, "bad fa_host_alloc arguments");
  *ptr = pinned_get(bytes);
  return *ptr ? FA_OK : fail(FA_ERR_CUDA, "pinned host allocation failed");
}

void fa_host_free(void* ptr) { pinned_put(ptr); }

fa_status fa_rope_tables(float* cos_out, float* sin_out, uint32_t rows, uint32_t head_dim, float theta) {
  if (!cos_out || !sin_out || head_dim == 0 || head_dim % 2 || !(theta > 0.f))
    return fail(FA_ERR_INVALID_ARG, "bad rope table arguments");
  const uint32_t half = head_dim / 2;
  for (uint32_t i = 0; i < half; ++i) {
    const double inv_freq = std::pow((double)theta, -2.0 * (double)i / (double)head_dim);
    for (uint32_t pos = 0; pos < rows; ++pos) {
      const double ang = (double)pos * inv_freq;
      cos_out[(size_t)pos * half + i] = (float)std::cos(ang);
      sin_out[(size_t)pos * half + i] = (float)std::sin(ang);
    }
  }
  return FA_OK;
}

fa_status fa_pool_stats(uint64_t* hits, uint64_t* misses, uint64_t* bytes_reserved) {
  DeviceState* ds = nullptr;
  fa_status st = device_state(&ds);
  if (st != FA_OK) return st;
  ds->pool.stats(hits, misses, bytes_reserved);
  return FA_OK;
}

fa_status fa_pool_clear(void) {
  DeviceState* ds = nullptr;
  fa_status st = device_state(&ds);
  if (st != FA_OK) return st;
  FA_CUDA(cudaDeviceSynchronize());
  ds->pool.clear();
  // With the device idle no call holds a cached table or workspace.
  std::lock_guard<std::mutex> g(ds->mu);
  for (void* p : ds->retired) cudaFree(p);
  ds->retired.clear();
  for (auto& kv : ds->rope) {
    cudaFree(kv.second.cs);
    cudaFree(kv.second.sn);
  }
  ds->rope.clear();
  for (auto& kv : ds->ws) cudaFree(kv.second.first);
  ds->ws.clear();
  pinned_release_cached();
  return FA_OK;
}

fa_status fa_check_device_status(void) {
  DeviceState* ds = nullptr;
  fa_status st = device_state(&ds);
  if (st != FA_OK) return st;
  unsigned v = 0;
  FA_CUDA(cudaMemcpy(&v, ds->status, sizeof(v), cudaMemcpyDeviceToHost));
  if (v == 0) return FA_OK;
  FA_CUDA(cudaMemset(ds->status, 0, sizeof(unsigned)));
  return fail(FA_ERR_TIMEOUT, "a kernel wait exceeded its time limit; the kernel returned early and its output is invalid");
}

fa_status fa_set_wait_limit(double seconds) {
  if (!(seconds > 0.0) || !(seconds <= 3600.0)) return fail(FA_ERR_INVALID_ARG, "wait limit must be in (0, 3600] s");
  g_wait_limit_ns.store((unsigned long long)(seconds * 1e9), std::memory_order_relaxed);
  return FA_OK;
}

double fa_get_wait_limit(void) {
  const unsigned long long ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  return (ns ? (double)ns : (double)fa::kWaitLimitNs) * 1e-9;
}

fa_status fa_test_stall_next_launch(int32_t k_tile) {
  if (k_tile < 0) return fail(FA_ERR_INVALID_ARG, "k_tile must be >= 0");
  g_stall_k_tile = k_tile + 1;
  return FA_OK;
}

uint64_t fa_launch_count(void) { return g_launches; }

fa_status fa_kernel_timing_enable(void) {
  for (auto& ev : g_events) {
    cudaEventDestroy(ev.first);
    cudaEventDestroy(ev.second);
  }
  g_events.clear();
  g_timing = true;
  return FA_OK;
}

fa_status fa_kernel_timing_read(double* total_ms, uint64_t* launches) {
  double tot = 0.0;
  fa_status st = FA_OK;
  for (auto& ev : g_events) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(ev.second);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, ev.first, ev.second);
    if (e != cudaSuccess && st == FA_OK) st = cuda_fail(e, "kernel timing");
    tot += ms;
    cudaEventDestroy(ev.first);
    cudaEventDestroy(ev.second);
  }
  if (total_ms) *total_ms = tot;
  if (launches) *launches = g_events.size();
  g_events.clear();
  g_timing = false;
  return st;
}

const char* fa_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free forward (no counterpart in the reference).
//
// For callers that must not allocate device memory themselves or through
// this library: code running inside a host application that owns every
// device allocation (a plugin whose host forbids cudaMalloc, or a runtime
// that budgets GPU memory up front). fa_forward_noalloc runs the same
// dispatch and kernels as fa_forward, but its scratch (the staging record,
// the fp16 staging of Q/K/V, padded operands for other head dims, and the
// RoPE tables built from rope_theta) lives in the fixed array below instead
// of a pool buffer, and its kernels report timeouts in a status word of
// their own (fa_noalloc_check_status).
//
// The array is a file-scope __device__ variable of kNoAllocScratchBytes: every
// GPU on which this module is loaded keeps it until the process exits. In
// host code its name is only a host-side stand-in, so the device address is
// taken with cudaGetSymbolAddress once per device (on the first call made
// with that device current; make that first call before any stream
// capture). All calls share the array and its contents persist between
// calls: each call clears the staging record it needs at zero, and every
// other byte it reads is written earlier in the same call. Calls that may
// overlap on the GPU (different streams, or several host threads) race on
// the array and must be serialised by the caller. Only the primary context
// of each device is supported (the addresses are cached per device).
namespace fa {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ unsigned g_noalloc_status;  // kernel status bits of this entry point

struct NoAllocDevice {
  bool ready = false;
  unsigned char* scratch = nullptr;
  unsigned* status = nullptr;
};
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_devices[kNoAllocMaxDevices];

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// Device addresses of the array and the status word on the current device,
// looked up once per device. A failed lookup is not cached, so a later call
// (for example one made outside stream capture) tries again.
fa_status noalloc_device(NoAllocDevice** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(FA_ERR_NO_DEVICE, std::string("no CUDA device: ") + cudaGetErrorString(e));
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(FA_ERR_INVALID_ARG, "device index out of range");
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  NoAllocDevice& nd = g_noalloc_devices[dev];
  if (!nd.ready) {
    unsigned char* scratch = nullptr;
    unsigned* status = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&scratch), g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_noalloc_status);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return cuda_fail(e, "cudaGetSymbolAddress (allocation-free scratch)");
    }
    nd.scratch = scratch;
    nd.status = status;
    nd.ready = true;
  }
  *out = &nd;
  return FA_OK;
}

}  // namespace
}  // namespace fa

extern "C" fa_status fa_forward_noalloc(const fa_params* p, const void* q, const void* k, const void* v,
                                        void* o, float* lse, const float* cos, const float* sin,
                                        void* stream_handle) {
  using namespace fa;
  Plan pl;
  fa_status st = make_plan(p, &pl);
  if (st != FA_OK) return st;
  AttnArgs& a = pl.a;
  const bool tables_from_theta = pl.rope && (cos == nullptr || sin == nullptr);
  const int rows = a.Sq > a.Sk ? a.Sq : a.Sk;
  const size_t table_bytes = tables_from_theta ? up256((size_t)rows * (a.D / 2) * sizeof(float)) : 0;
  const size_t need = 2 * table_bytes + pl.ws_bytes;
  if (need > kNoAllocScratchBytes)
    return fail(FA_ERR_INVALID_ARG, "fa_forward_noalloc: this problem needs " + std::to_string(need) +
                                        " bytes of scratch; the allocation-free entry point has a fixed " +
                                        std::to_string(kNoAllocScratchBytes) + "-byte array (use fa_forward)");
  if (a.q_end <= a.q_begin || a.B == 0 || a.Hq == 0) return FA_OK;
  if (!o) return fail(FA_ERR_INVALID_ARG, "NULL output pointer");
  NoAllocDevice* nd = nullptr;
  st = noalloc_device(&nd);
  if (st != FA_OK) return st;

  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  a.o = o;
  a.lse = lse;
  unsigned char* wp = nd->scratch;
  const float* cs = cos;
  const float* sn = sin;
  if (tables_from_theta && a.kv_end > a.kv_begin) {
    if (!(pl.rope_theta > 0.f) || !std::isfinite(pl.rope_theta))
      return fail(FA_ERR_INVALID_ARG, "has_rotary needs cos/sin tables or rope_theta > 0");
    if (a.D % 2 != 0) return fail(FA_ERR_UNSUPPORTED, "RoPE from rope_theta needs an even head_dim");
    float* tc = reinterpret_cast<float*>(wp);
    float* ts = reinterpret_cast<float*>(wp + table_bytes);
    wp += 2 * table_bytes;
    cudaError_t e = launch_rope_table(tc, ts, rows, a.D, (double)pl.rope_theta, stream);
    if (e != cudaSuccess) return cuda_fail(e, "rope tables");
    cs = tc;
    sn = ts;
  }
  // The rest of the array is the workspace (run() clears its staging record).
  return run(pl, q, k, v, cs, sn, pl.ws_bytes ? wp : nullptr, pl.ws_bytes, stream, nullptr, nd->status);
}

extern "C" fa_status fa_noalloc_check_status(void) {
  using namespace fa;
  NoAllocDevice* nd = nullptr;
  fa_status st = noalloc_device(&nd);
  if (st != FA_OK) return st;
  unsigned v = 0;
  FA_CUDA(cudaMemcpy(&v, nd->status, sizeof(v), cudaMemcpyDeviceToHost));
  if (v == 0) return FA_OK;
  FA_CUDA(cudaMemset(nd->status, 0, sizeof(unsigned)));
  return fail(FA_ERR_TIMEOUT,
              "a kernel wait of fa_forward_noalloc exceeded its time limit; the kernel returned early and its "
              "output is invalid");
}
