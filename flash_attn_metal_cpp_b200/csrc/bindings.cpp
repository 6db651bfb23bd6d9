// bindings.cpp - the `_flash_attn_metal` Python module over the C ABI in
// fa_b200.h. Keeps the reference module's surface (python/bindings.cpp:239-269):
//   initialize() -> bool
//   load_shaders(metallib_path) -> bool      accepted no-op (kernels are built ahead of time)
//   compile_shaders(shader_source) -> bool   accepted no-op
//   get_device_info() -> {device_name, max_buffer_length, initialized}
//   forward(Q, K, V, softmax_scale=0.0, is_causal=False, dropout_p=0.0,
//           alibi_slopes=None, window_size=None, cos=None, sin=None)
// with the reference's error behaviour: initialize/load/compile print to
// stderr and return False; forward raises RuntimeError("Forward pass error: ...").
//
// forward takes NumPy arrays (float16, float32, ml_dtypes.bfloat16; the host
// path copies to and from the device like FlashAttentionForward::execute) or
// torch tensors (CUDA tensors run zero-copy on the current stream; CPU
// tensors take the host path). Keyword-only extras: out_dtype, rope_theta,
// return_lse.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>
#include <iostream>
#include <stdexcept>
#include <string>

#include "../../include/fa_b200.h"

namespace py = pybind11;

namespace {

// initialize / get_device_info act on the calling thread's current CUDA
// device (device 0 unless the caller selected another, e.g. one per rank).
constexpr int g_device = -1;

std::string err_text(fa_status st) {
  std::string s = fa_last_error();
  if (s.empty()) s = "status " + std::to_string((int)st);
  return s;
}

[[noreturn]] void forward_error(const std::string& what) {
  throw std::runtime_error("Forward pass error: " + what);
}

bool is_torch_tensor(const py::object& o) {
  return py::hasattr(o, "data_ptr") && py::hasattr(o, "is_cuda") && py::hasattr(o, "stride");
}

int dtype_code_from_name(const std::string& n) {
  if (n == "float16" || n == "torch.float16" || n == "torch.half") return FA_F16;
  if (n == "bfloat16" || n == "torch.bfloat16") return FA_BF16;
  if (n == "float32" || n == "torch.float32" || n == "torch.float") return FA_F32;
  return -1;
}

int parse_out_dtype(const py::object& od) {
  if (od.is_none()) return -1;
  const std::string n = py::str(od);
  const int c = dtype_code_from_name(n);
  if (c < 0) forward_error("out_dtype must be float16, bfloat16 or float32");
  return c;
}

void fill_params(fa_params& p, const std::vector<int64_t>& qs, const std::vector<int64_t>& ks,
                 float scale, bool causal, float dropout_p, const py::object& alibi,
                 const py::object& window, bool rotary, float rope_theta) {
  fa_params_init(&p);
  p.batch_size = (uint32_t)qs[0];
  p.seqlen_q = (uint32_t)qs[1];
  p.num_heads_q = (uint32_t)qs[2];
  p.head_dim = (uint32_t)qs[3];
  p.seqlen_k = (uint32_t)ks[1];
  p.num_heads_k = (uint32_t)ks[2];
  p.softmax_scale = scale;
  p.is_causal = causal ? 1 : 0;
  p.dropout_p = dropout_p;
  if (!window.is_none()) {
    py::tuple ws = window.cast<py::tuple>();
    if (py::len(ws) == 2) {
      p.window_left = ws[0].cast<int>();
      p.window_right = ws[1].cast<int>();
    }
  }
  p.has_alibi = alibi.is_none() ? 0 : 1;
  p.has_rotary = rotary ? 1 : 0;
  p.rope_theta = rope_theta;
}

void check_slopes(int64_t n, int64_t heads_q) {
  if (n != heads_q) forward_error("alibi_slopes must hold one float32 slope per query head");
}

void check_shapes(const std::vector<int64_t>& qs, const std::vector<int64_t>& ks,
                  const std::vector<int64_t>& vs) {
  if (qs.size() != 4 || ks.size() != 4 || vs.size() != 4)
    forward_error("Input arrays must be 4D [batch, seqlen, num_heads, head_dim]");
  if (ks[0] != qs[0] || vs[0] != qs[0] || vs[1] != ks[1] || vs[2] != ks[2] || ks[3] != qs[3] ||
      vs[3] != qs[3])
    forward_error("K and V shapes must match");
}

// ------------------------------------------------------------------ numpy
py::object bf16_numpy_dtype() { return py::module_::import("ml_dtypes").attr("bfloat16"); }

int numpy_code(const py::array& a) {
  const std::string n = py::str(a.dtype());
  return dtype_code_from_name(n);
}

py::dtype numpy_dtype_of(int code) {
  if (code == FA_F16) return py::dtype("float16");
  if (code == FA_F32) return py::dtype("float32");
  return py::dtype::from_args(bf16_numpy_dtype());
}

// A C-ordered NumPy array in pinned host memory from the library's pool (the
// device-to-host copy of the result then runs by DMA at full link speed);
// the array owns the buffer and returns it to the pool when it dies. Falls
// back to ordinary memory when no pinned memory is left.
py::array pinned_array(const py::dtype& dt, std::vector<int64_t> shape) {
  size_t n = 1;
  for (int64_t d : shape) n *= (size_t)d;
  const size_t bytes = n * (size_t)dt.itemsize();
  std::vector<py::ssize_t> sh(shape.begin(), shape.end());
  void* buf = nullptr;
  if (bytes == 0 || fa_host_alloc(bytes, &buf) != FA_OK) return py::array(dt, sh);
  py::capsule owner(buf, [](void* p) { fa_host_free(p); });
  std::vector<py::ssize_t> strides(sh.size());
  py::ssize_t st = dt.itemsize();
  for (size_t i = sh.size(); i-- > 0;) {
    strides[i] = st;
    st *= sh[i];
  }
  return py::array(dt, sh, strides, buf, owner);
}

py::object forward_numpy(py::object Q, py::object K, py::object V, float scale, bool causal,
                         float dropout_p, py::object alibi, py::object window, py::object cos,
                         py::object sin, int out_code, float rope_theta, bool return_lse) {
  py::module_ np = py::module_::import("numpy");
  py::array q = np.attr("ascontiguousarray")(Q);
  py::array k = np.attr("ascontiguousarray")(K);
  py::array v = np.attr("ascontiguousarray")(V);
  const int code = numpy_code(q);
  if (code < 0 || numpy_code(k) != code || numpy_code(v) != code)
    forward_error("Input arrays must be float16, bfloat16 or float32, all of one dtype");
  std::vector<int64_t> qs(q.shape(), q.shape() + q.ndim()), ks(k.shape(), k.shape() + k.ndim()),
      vs(v.shape(), v.shape() + v.ndim());
  check_shapes(qs, ks, vs);
  const bool rotary_tables = !cos.is_none() && !sin.is_none();
  const bool rotary = rotary_tables || rope_theta > 0.f;
  fa_params p;
  fill_params(p, qs, ks, scale, causal, dropout_p, alibi, window, rotary, rope_theta);
  p.dtype = code;
  p.out_dtype = out_code;
  const int oc = out_code < 0 ? code : out_code;
  py::array slopes;
  if (!alibi.is_none()) {
    slopes = np.attr("ascontiguousarray")(alibi, "float32");
    check_slopes(slopes.size(), qs[2]);
    p.alibi_slopes = static_cast<const float*>(slopes.data());
  }
  py::array c_arr, s_arr;
  const float* cp = nullptr;
  const float* sp = nullptr;
  if (rotary_tables) {
    c_arr = np.attr("ascontiguousarray")(cos, "float32");
    s_arr = np.attr("ascontiguousarray")(sin, "float32");
    const int64_t need = std::max(qs[1], ks[1]) * (qs[3] / 2);
    if (c_arr.size() < need || s_arr.size() < need)
      forward_error("cos/sin tables must hold [max(seqlen_q, seqlen_k), head_dim/2] float32 values");
    cp = static_cast<const float*>(c_arr.data());
    sp = static_cast<const float*>(s_arr.data());
  }
  py::array out = pinned_array(numpy_dtype_of(oc), {qs[0], qs[1], qs[2], qs[3]});
  py::array lse;
  float* lp = nullptr;
  if (return_lse) {
    lse = pinned_array(py::dtype("float32"), {qs[0], qs[2], qs[1]});
    lp = static_cast<float*>(lse.mutable_data());
  }
  fa_status st;
  {
    py::gil_scoped_release nogil;
    st = fa_forward_host(&p, q.data(), k.data(), v.data(), out.mutable_data(), lp, cp, sp);
  }
  if (st != FA_OK) forward_error(err_text(st));
  if (return_lse) return py::make_tuple(out, lse);
  return out;
}

// ------------------------------------------------------------------ torch
std::vector<int64_t> tsize(const py::object& t) { return t.attr("shape").cast<std::vector<int64_t>>(); }
std::vector<int64_t> tstride(const py::object& t) { return t.attr("stride")().cast<std::vector<int64_t>>(); }

py::object torch_dtype_of(int code) {
  py::module_ torch = py::module_::import("torch");
  if (code == FA_F16) return torch.attr("float16");
  if (code == FA_BF16) return torch.attr("bfloat16");
  return torch.attr("float32");
}

// Innermost stride 1 (else a contiguous copy); returns the possibly-new tensor.
py::object inner_contig(py::object t) {
  auto st = tstride(t);
  if (st.size() == 4 && st[3] == 1) return t;
  return t.attr("contiguous")();
}

// A caller-provided output tensor must match shape, dtype and device and be contiguous.
py::object check_out(py::object out, const py::tuple& shape, int oc, bool cuda) {
  py::module_ torch = py::module_::import("torch");
  if (tsize(out) != shape.cast<std::vector<int64_t>>()) forward_error("out has the wrong shape");
  if (dtype_code_from_name(py::str(out.attr("dtype"))) != oc) forward_error("out has the wrong dtype");
  if (out.attr("is_cuda").cast<bool>() != cuda) forward_error("out is on the wrong device");
  if (!out.attr("is_contiguous")().cast<bool>()) forward_error("out must be contiguous");
  return out;
}

// A CPU torch tensor over pinned_array memory (bf16 through a 16-bit view,
// since NumPy has no bfloat16 that torch.from_numpy accepts).
py::object pinned_tensor(std::vector<int64_t> shape, int code) {
  py::module_ torch = py::module_::import("torch");
  const py::dtype nd = code == FA_F32 ? py::dtype("float32") : (code == FA_F16 ? py::dtype("float16")
                                                                                : py::dtype("int16"));
  py::object t = torch.attr("from_numpy")(pinned_array(nd, std::move(shape)));
  if (code == FA_BF16) t = t.attr("view")(torch.attr("bfloat16"));
  return t;
}

// cos/sin table as a contiguous float32 tensor on `dev`. The staging pass
// reads 16-byte aligned tables with vector loads and others element by
// element, so a view that starts off a 16-byte boundary is copied.
py::object device_table(py::module_& torch, py::object t, py::object dev) {
  py::object x = torch.attr("as_tensor")(t, py::arg("dtype") = torch.attr("float32"), py::arg("device") = dev)
                     .attr("contiguous")();
  if (x.attr("data_ptr")().cast<uintptr_t>() % 16 != 0) x = x.attr("clone")();
  return x;
}

py::object forward_torch(py::object Q, py::object K, py::object V, float scale, bool causal,
                         float dropout_p, py::object alibi, py::object window, py::object cos,
                         py::object sin, int out_code, float rope_theta, bool return_lse,
                         py::object out_arg) {
  py::module_ torch = py::module_::import("torch");
  const bool cuda = Q.attr("is_cuda").cast<bool>();
  if (K.attr("is_cuda").cast<bool>() != cuda || V.attr("is_cuda").cast<bool>() != cuda)
    forward_error("Q, K and V must all be CUDA tensors or all CPU tensors");
  const int code = dtype_code_from_name(py::str(Q.attr("dtype")));
  if (code < 0 || dtype_code_from_name(py::str(K.attr("dtype"))) != code ||
      dtype_code_from_name(py::str(V.attr("dtype"))) != code)
    forward_error("Input tensors must be float16, bfloat16 or float32, all of one dtype");
  std::vector<int64_t> qs = tsize(Q), ks = tsize(K), vs = tsize(V);
  check_shapes(qs, ks, vs);
  const bool rotary_tables = !cos.is_none() && !sin.is_none();
  const bool rotary = rotary_tables || rope_theta > 0.f;
  fa_params p;
  fill_params(p, qs, ks, scale, causal, dropout_p, alibi, window, rotary, rope_theta);
  p.dtype = code;
  p.out_dtype = out_code;
  const int oc = out_code < 0 ? code : out_code;
  py::tuple shape = py::make_tuple(qs[0], qs[1], qs[2], qs[3]);
  // ALiBi slopes as float32 next to the tensors (host memory for CPU tensors).
  py::object slopes = py::none();
  if (!alibi.is_none()) {
    slopes = torch.attr("as_tensor")(alibi, py::arg("dtype") = torch.attr("float32"),
                                     py::arg("device") = Q.attr("device")).attr("contiguous")();
    check_slopes(slopes.attr("numel")().cast<int64_t>(), qs[2]);
    p.alibi_slopes = reinterpret_cast<const float*>(slopes.attr("data_ptr")().cast<uintptr_t>());
  }

  if (!cuda) {
    // CPU tensors: host path (contiguous), like the NumPy route.
    py::object q = Q.attr("contiguous")(), k = K.attr("contiguous")(), v = V.attr("contiguous")();
    // Results in the library's pinned memory: copied back by DMA.
    py::object out = out_arg.is_none() ? pinned_tensor({qs[0], qs[1], qs[2], qs[3]}, oc)
                                       : check_out(out_arg, shape, oc, false);
    py::object lse = py::none();
    float* lp = nullptr;
    if (return_lse) {
      lse = pinned_tensor({qs[0], qs[2], qs[1]}, FA_F32);
      lp = reinterpret_cast<float*>(lse.attr("data_ptr")().cast<uintptr_t>());
    }
    py::object ct = py::none(), stt = py::none();
    const float* cp = nullptr;
    const float* sp = nullptr;
    if (rotary_tables) {
      ct = torch.attr("as_tensor")(cos, py::arg("dtype") = torch.attr("float32")).attr("contiguous")();
      stt = torch.attr("as_tensor")(sin, py::arg("dtype") = torch.attr("float32")).attr("contiguous")();
      cp = reinterpret_cast<const float*>(ct.attr("data_ptr")().cast<uintptr_t>());
      sp = reinterpret_cast<const float*>(stt.attr("data_ptr")().cast<uintptr_t>());
    }
    const void* qp = reinterpret_cast<const void*>(q.attr("data_ptr")().cast<uintptr_t>());
    const void* kp = reinterpret_cast<const void*>(k.attr("data_ptr")().cast<uintptr_t>());
    const void* vp = reinterpret_cast<const void*>(v.attr("data_ptr")().cast<uintptr_t>());
    void* op = reinterpret_cast<void*>(out.attr("data_ptr")().cast<uintptr_t>());
    fa_status st;
    {
      py::gil_scoped_release nogil;
      st = fa_forward_host(&p, qp, kp, vp, op, lp, cp, sp);
    }
    if (st != FA_OK) forward_error(err_text(st));
    if (return_lse) return py::make_tuple(out, lse);
    return out;
  }

  py::object dev = Q.attr("device");
  const int dev_index = dev.attr("index").is_none() ? 0 : dev.attr("index").cast<int>();
  fa_status st = fa_init(dev_index);
  if (st != FA_OK) forward_error(err_text(st));
  py::object q = inner_contig(Q), k = inner_contig(K), v = inner_contig(V);
  auto qst = tstride(q), kst = tstride(k), vst = tstride(v);
  for (int i = 0; i < 3; ++i) {
    p.q_stride[i] = qst[i];
    p.k_stride[i] = kst[i];
    p.v_stride[i] = vst[i];
  }
  py::object out = out_arg.is_none()
                       ? torch.attr("empty")(shape, py::arg("dtype") = torch_dtype_of(oc), py::arg("device") = dev)
                       : check_out(out_arg, shape, oc, true);
  py::object lse = py::none();
  float* lp = nullptr;
  if (return_lse) {
    lse = torch.attr("empty")(py::make_tuple(qs[0], qs[2], qs[1]), py::arg("dtype") = torch.attr("float32"),
                              py::arg("device") = dev);
    lp = reinterpret_cast<float*>(lse.attr("data_ptr")().cast<uintptr_t>());
  }
  py::object ct = py::none(), stt = py::none();
  const float* cp = nullptr;
  const float* sp = nullptr;
  if (rotary_tables) {
    ct = device_table(torch, cos, dev);
    stt = device_table(torch, sin, dev);
    const int64_t need = std::max(qs[1], ks[1]) * (qs[3] / 2);
    if (ct.attr("numel")().cast<int64_t>() < need || stt.attr("numel")().cast<int64_t>() < need)
      forward_error("cos/sin tables must hold [max(seqlen_q, seqlen_k), head_dim/2] float32 values");
    cp = reinterpret_cast<const float*>(ct.attr("data_ptr")().cast<uintptr_t>());
    sp = reinterpret_cast<const float*>(stt.attr("data_ptr")().cast<uintptr_t>());
  }
  void* stream = reinterpret_cast<void*>(
      torch.attr("cuda").attr("current_stream")(dev).attr("cuda_stream").cast<uintptr_t>());
  const void* qp = reinterpret_cast<const void*>(q.attr("data_ptr")().cast<uintptr_t>());
  const void* kp = reinterpret_cast<const void*>(k.attr("data_ptr")().cast<uintptr_t>());
  const void* vp = reinterpret_cast<const void*>(v.attr("data_ptr")().cast<uintptr_t>());
  void* op = reinterpret_cast<void*>(out.attr("data_ptr")().cast<uintptr_t>());
  st = fa_forward(&p, qp, kp, vp, op, lp, cp, sp, nullptr, 0, stream);
  if (st != FA_OK) forward_error(err_text(st));
  if (return_lse) return py::make_tuple(out, lse);
  return out;
}

// ------------------------------------------ range / combine / IPC (torch CUDA)
template <typename T>
T* tptr(const py::object& t) {
  return reinterpret_cast<T*>(t.attr("data_ptr")().cast<uintptr_t>());
}

void* current_stream_of(const py::object& t) {
  py::module_ torch = py::module_::import("torch");
  return reinterpret_cast<void*>(
      torch.attr("cuda").attr("current_stream")(t.attr("device")).attr("cuda_stream").cast<uintptr_t>());
}

void require_cuda(const py::object& t, const char* name) {
  if (!is_torch_tensor(t) || !t.attr("is_cuda").cast<bool>())
    forward_error(std::string(name) + " must be a CUDA torch tensor");
}

// Rows [q_begin, q_end) against keys [kv_begin, kv_end): writes out / lse,
// or the owners' slots listed in `route` (int64 CUDA tensor of 2*n_owners
// addresses) when given.
void py_forward_range(py::object Q, py::object K, py::object V, std::pair<int64_t, int64_t> q_range,
                      std::pair<int64_t, int64_t> kv_range, py::object out, py::object lse,
                      float softmax_scale, bool is_causal, py::object cos, py::object sin,
                      py::object rope_theta, py::object out_dtype, py::object route, int n_owners,
                      int64_t owner_rows, py::object window_size, py::object alibi_slopes) {
  require_cuda(Q, "Q");
  require_cuda(K, "K");
  require_cuda(V, "V");
  const int code = dtype_code_from_name(py::str(Q.attr("dtype")));
  if (code < 0 || dtype_code_from_name(py::str(K.attr("dtype"))) != code ||
      dtype_code_from_name(py::str(V.attr("dtype"))) != code)
    forward_error("Input tensors must be float16, bfloat16 or float32, all of one dtype");
  std::vector<int64_t> qs = tsize(Q), ks = tsize(K), vs = tsize(V);
  check_shapes(qs, ks, vs);
  const bool rotary_tables = !cos.is_none() && !sin.is_none();
  const float theta = rope_theta.is_none() ? 0.f : rope_theta.cast<float>();
  fa_params p;
  fill_params(p, qs, ks, softmax_scale, is_causal, 0.f, alibi_slopes, window_size, rotary_tables || theta > 0.f,
              theta);
  py::object slopes = py::none();
  if (!alibi_slopes.is_none()) {
    py::module_ torch = py::module_::import("torch");
    slopes = torch.attr("as_tensor")(alibi_slopes, py::arg("dtype") = torch.attr("float32"),
                                     py::arg("device") = Q.attr("device")).attr("contiguous")();
    check_slopes(slopes.attr("numel")().cast<int64_t>(), qs[2]);
    p.alibi_slopes = tptr<const float>(slopes);
  }
  p.dtype = code;
  p.out_dtype = parse_out_dtype(out_dtype);
  const int oc = p.out_dtype < 0 ? code : p.out_dtype;
  py::object q = inner_contig(Q), k = inner_contig(K), v = inner_contig(V);
  auto qst = tstride(q), kst = tstride(k), vst = tstride(v);
  for (int i = 0; i < 3; ++i) {
    p.q_stride[i] = qst[i];
    p.k_stride[i] = kst[i];
    p.v_stride[i] = vst[i];
  }
  const py::object dev = Q.attr("device");
  const int dev_index = dev.attr("index").is_none() ? 0 : dev.attr("index").cast<int>();
  fa_status st = fa_init(dev_index);
  if (st != FA_OK) forward_error(err_text(st));
  void* op = nullptr;
  float* lp = nullptr;
  fa_route rt{};
  if (!route.is_none()) {
    require_cuda(route, "route");
    if (route.attr("numel")().cast<int64_t>() != 2 * (int64_t)n_owners)
      forward_error("route must hold 2 * n_owners addresses");
    rt.table = tptr<const uint64_t>(route);
    rt.n_owners = n_owners;
    rt.owner_rows = (uint32_t)owner_rows;
  } else {
    require_cuda(out, "out");
    if (tsize(out) != qs) forward_error("out has the wrong shape");
    if (dtype_code_from_name(py::str(out.attr("dtype"))) != oc) forward_error("out has the wrong dtype");
    auto ost = tstride(out);
    if (ost[3] != 1) forward_error("out needs a unit innermost stride");
    for (int i = 0; i < 3; ++i) p.o_stride[i] = ost[i];
    op = tptr<void>(out);
    if (!lse.is_none()) {
      require_cuda(lse, "lse");
      if (tsize(lse) != std::vector<int64_t>{qs[0], qs[2], qs[1]} ||
          !lse.attr("is_contiguous")().cast<bool>() ||
          dtype_code_from_name(py::str(lse.attr("dtype"))) != FA_F32)
        forward_error("lse must be a contiguous float32 [batch, num_heads_q, seqlen_q] tensor");
      lp = tptr<float>(lse);
    }
  }
  py::object ct = py::none(), stt = py::none();
  const float* cp = nullptr;
  const float* sp = nullptr;
  if (rotary_tables) {
    py::module_ torch = py::module_::import("torch");
    ct = device_table(torch, cos, dev);
    stt = device_table(torch, sin, dev);
    const int64_t need = std::max(qs[1], ks[1]) * (qs[3] / 2);
    if (ct.attr("numel")().cast<int64_t>() < need || stt.attr("numel")().cast<int64_t>() < need)
      forward_error("cos/sin tables must hold [max(seqlen_q, seqlen_k), head_dim/2] float32 values");
    cp = tptr<const float>(ct);
    sp = tptr<const float>(stt);
  }
  if (q_range.first < 0 || kv_range.first < 0) forward_error("ranges must be non-negative");
  st = fa_forward_range(&p, tptr<const void>(q), tptr<const void>(k), tptr<const void>(v), op, lp, cp, sp,
                        (uint32_t)q_range.first, (uint32_t)q_range.second, (uint32_t)kv_range.first,
                        (uint32_t)kv_range.second, route.is_none() ? nullptr : &rt, nullptr, 0,
                        current_stream_of(Q));
  if (st != FA_OK) forward_error(err_text(st));
}

// Merge n split partials: o_parts [n, B, Sq, Hq, D] and lse_parts
// [n, B, Hq, Sq] (float32, contiguous) into rows q_range of out
// [B, >= q_range end, Hq, D] (any of the three dtypes, unit innermost
// stride) and optionally lse [B, Hq, Sq].
void py_combine(py::object o_parts, py::object lse_parts, py::object out, py::object lse,
                py::object q_range, py::object row_begin) {
  require_cuda(o_parts, "o_parts");
  require_cuda(lse_parts, "lse_parts");
  require_cuda(out, "out");
  std::vector<int64_t> os = tsize(o_parts), ls = tsize(lse_parts), outs = tsize(out);
  if (os.size() != 5 || ls.size() != 4 || outs.size() != 4)
    forward_error("o_parts must be [n, B, Sq, Hq, D], lse_parts [n, B, Hq, Sq], out [B, Sq, Hq, D]");
  int64_t q0 = 0, q1 = os[2];
  if (!q_range.is_none()) {
    auto r = q_range.cast<std::pair<int64_t, int64_t>>();
    q0 = r.first;
    q1 = r.second;
  }
  if (q0 < 0 || q1 < q0 || q1 > os[2]) forward_error("bad q_range");
  // out may have fewer rows than the staging (a ragged last block) as long
  // as it holds the merged range.
  if (ls != std::vector<int64_t>{os[0], os[1], os[3], os[2]} || outs[0] != os[1] || outs[1] < q1 ||
      outs[2] != os[3] || outs[3] != os[4])
    forward_error("o_parts, lse_parts and out disagree in shape");
  if (!o_parts.attr("is_contiguous")().cast<bool>() || !lse_parts.attr("is_contiguous")().cast<bool>() ||
      dtype_code_from_name(py::str(o_parts.attr("dtype"))) != FA_F32 ||
      dtype_code_from_name(py::str(lse_parts.attr("dtype"))) != FA_F32)
    forward_error("o_parts and lse_parts must be contiguous float32");
  const int oc = dtype_code_from_name(py::str(out.attr("dtype")));
  if (oc < 0) forward_error("out must be float16, bfloat16 or float32");
  auto ost = tstride(out);
  if (ost[3] != 1) forward_error("out needs a unit innermost stride");
  fa_params p;
  fa_params_init(&p);
  p.batch_size = (uint32_t)os[1];
  p.seqlen_q = (uint32_t)os[2];
  p.seqlen_k = 1;
  p.num_heads_q = p.num_heads_k = (uint32_t)os[3];
  p.head_dim = (uint32_t)os[4];
  p.dtype = FA_F32;
  p.out_dtype = oc;
  for (int i = 0; i < 3; ++i) p.o_stride[i] = ost[i];
  float* lp = nullptr;
  if (!lse.is_none()) {
    require_cuda(lse, "lse");
    if (tsize(lse) != std::vector<int64_t>{os[1], os[3], os[2]} || !lse.attr("is_contiguous")().cast<bool>())
      forward_error("lse must be a contiguous float32 [B, Hq, Sq] tensor");
    lp = tptr<float>(lse);
  }
  const py::object dev = out.attr("device");
  fa_status st = fa_init(dev.attr("index").is_none() ? 0 : dev.attr("index").cast<int>());
  if (st != FA_OK) forward_error(err_text(st));
  const int32_t* rb = nullptr;
  if (!row_begin.is_none()) {
    require_cuda(row_begin, "row_begin");
    if (row_begin.attr("numel")().cast<int64_t>() != os[0] ||
        py::str(row_begin.attr("dtype")).cast<std::string>() != "torch.int32")
      forward_error("row_begin must be an int32 CUDA tensor with one entry per partial");
    rb = tptr<const int32_t>(row_begin);
  }
  st = fa_combine_ranges(&p, tptr<const float>(o_parts), tptr<const float>(lse_parts), (int32_t)os[0], rb,
                         tptr<void>(out), lp, (uint32_t)q0, (uint32_t)q1, current_stream_of(out));
  if (st != FA_OK) forward_error(err_text(st));
}

py::tuple py_ipc_alloc(size_t bytes) {
  void* p = nullptr;
  fa_ipc_handle h;
  fa_status st = fa_ipc_alloc(bytes, &p, &h);
  if (st != FA_OK) throw std::runtime_error(err_text(st));
  return py::make_tuple(reinterpret_cast<uintptr_t>(p),
                        py::bytes(reinterpret_cast<const char*>(h.bytes), sizeof(h.bytes)));
}

uintptr_t py_ipc_open(py::bytes handle) {
  const std::string s = handle;
  if (s.size() != sizeof(fa_ipc_handle)) throw std::runtime_error("IPC handle must be 64 bytes");
  fa_ipc_handle h;
  std::memcpy(h.bytes, s.data(), sizeof(h.bytes));
  void* p = nullptr;
  fa_status st = fa_ipc_open(&h, &p);
  if (st != FA_OK) throw std::runtime_error(err_text(st));
  return reinterpret_cast<uintptr_t>(p);
}

// ------------------------------------------------------------ module API
bool py_initialize() {
  fa_status st = fa_init(g_device);
  if (st != FA_OK) {
    std::cerr << "Initialization error: " << err_text(st) << "\n";
    return false;
  }
  return true;
}

bool py_load_shaders(const std::string& /*metallib_path*/) {
  // Kernels are compiled ahead of time for sm_100a; there is nothing to load.
  return py_initialize();
}

bool py_compile_shaders(const std::string& /*shader_source*/) {
  // Accepted no-op: the CUDA kernels are compiled when the library is built.
  return py_initialize();
}

py::dict py_get_device_info() {
  py::dict info;
  char name[256] = {0};
  uint64_t mem = 0;
  int init = 0;
  fa_status st = fa_device_info(g_device, name, sizeof(name), &mem, &init);
  if (st != FA_OK && st != FA_ERR_NO_DEVICE) {
    std::cerr << "Device info error: " << err_text(st) << "\n";
    return py::dict();
  }
  info["device_name"] = std::string(name);
  info["max_buffer_length"] = mem;
  info["initialized"] = init != 0;
  return info;
}

py::object py_forward(py::object Q, py::object K, py::object V, float softmax_scale, bool is_causal,
                      float dropout_p, py::object alibi_slopes, py::object window_size, py::object cos,
                      py::object sin, py::object out_dtype, py::object rope_theta, bool return_lse,
                      py::object out) {
  const int oc = parse_out_dtype(out_dtype);
  const float theta = rope_theta.is_none() ? 0.f : rope_theta.cast<float>();
  if (is_torch_tensor(Q))
    return forward_torch(Q, K, V, softmax_scale, is_causal, dropout_p, alibi_slopes, window_size, cos,
                         sin, oc, theta, return_lse, out);
  if (!out.is_none()) forward_error("out= is supported for torch tensors only");
  return forward_numpy(Q, K, V, softmax_scale, is_causal, dropout_p, alibi_slopes, window_size, cos, sin,
                       oc, theta, return_lse);
}

void py_check_status() {
  fa_status st = fa_check_device_status();
  if (st != FA_OK) throw std::runtime_error("Device status error: " + err_text(st));
}

py::tuple py_pool_stats() {
  uint64_t h = 0, m = 0, b = 0;
  fa_status st = fa_pool_stats(&h, &m, &b);
  if (st != FA_OK) throw std::runtime_error(err_text(st));
  return py::make_tuple(h, m, b);
}

}  // namespace

PYBIND11_MODULE(_flash_attn_metal, m) {
  m.doc() = "FlashAttention-2 forward for NVIDIA B200 (sm_100a), drop-in for the Metal module";
  m.def("initialize", &py_initialize, "Initialize the CUDA device");
  m.def("load_shaders", &py_load_shaders, py::arg("metallib_path"),
        "Accepted for compatibility; kernels are compiled ahead of time");
  m.def("compile_shaders", &py_compile_shaders, py::arg("shader_source"),
        "Accepted for compatibility; kernels are compiled ahead of time");
  m.def("get_device_info", &py_get_device_info, "Get CUDA device information");
  m.def("forward", &py_forward, py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("softmax_scale") = 0.0f,
        py::arg("is_causal") = false, py::arg("dropout_p") = 0.0f, py::arg("alibi_slopes") = py::none(),
        py::arg("window_size") = py::none(), py::arg("cos") = py::none(), py::arg("sin") = py::none(),
        py::kw_only(), py::arg("out_dtype") = py::none(), py::arg("rope_theta") = py::none(),
        py::arg("return_lse") = false, py::arg("out") = py::none(), "Flash Attention forward pass");
  m.def("check_status", &py_check_status,
        "Raise if a kernel recorded a timeout or range error since the last check");
  m.def("launch_count", []() { return fa_launch_count(); },
        "Number of kernels this library launched on the calling thread");
  m.def("kernel_timing_enable", []() { fa_kernel_timing_enable(); },
        "Time every attention-kernel launch of this thread with CUDA events");
  m.def("kernel_timing_read", []() {
    double ms = 0;
    uint64_t n = 0;
    fa_status st = fa_kernel_timing_read(&ms, &n);
    if (st != FA_OK) throw std::runtime_error(err_text(st));
    return py::make_tuple(ms, n);
  }, "(summed ms, launches) of the attention kernel since kernel_timing_enable; disables timing");
  m.def("set_wait_limit", [](double seconds) {
    fa_status st = fa_set_wait_limit(seconds);
    if (st != FA_OK) throw std::runtime_error(err_text(st));
  }, py::arg("seconds"), "Wall-clock limit of every in-kernel wait of later launches (default 2 s)");
  m.def("get_wait_limit", []() { return fa_get_wait_limit(); }, "Current in-kernel wait limit in seconds");
  m.def("pool_stats", &py_pool_stats, "(hits, misses, bytes reserved) of the device buffer pool");
  m.def("pool_clear", []() {
    fa_status st = fa_pool_clear();
    if (st != FA_OK) throw std::runtime_error(err_text(st));
  });
  m.def("forward_range", &py_forward_range, py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("q_range"),
        py::arg("kv_range"), py::arg("out") = py::none(), py::arg("lse") = py::none(), py::kw_only(),
        py::arg("softmax_scale") = 0.0f, py::arg("is_causal") = false, py::arg("cos") = py::none(),
        py::arg("sin") = py::none(), py::arg("rope_theta") = py::none(), py::arg("out_dtype") = py::none(),
        py::arg("route") = py::none(), py::arg("n_owners") = 0, py::arg("owner_rows") = 0,
        py::arg("window_size") = py::none(), py::arg("alibi_slopes") = py::none(),
        "Rows q_range of the attention over keys kv_range (CUDA tensors, current stream)");
  m.def("combine", &py_combine, py::arg("o_parts"), py::arg("lse_parts"), py::arg("out"),
        py::arg("lse") = py::none(), py::arg("q_range") = py::none(), py::arg("row_begin") = py::none(),
        "Merge split-KV partials (O_j, LSE_j) into out (CUDA tensors, current stream); row_begin (int32 "
        "CUDA tensor, one per partial): rows before it ignore that partial");
  m.def("ipc_alloc", &py_ipc_alloc, py::arg("bytes"),
        "Allocate device memory shareable with other processes: (address, 64-byte handle)");
  m.def("ipc_open", &py_ipc_open, py::arg("handle"), "Map a peer process's allocation; returns its address");
  m.def("ipc_close", [](uintptr_t p) {
    fa_status st = fa_ipc_close(reinterpret_cast<void*>(p));
    if (st != FA_OK) throw std::runtime_error(err_text(st));
  }, py::arg("address"));
  m.def("ipc_free", [](uintptr_t p) {
    fa_status st = fa_ipc_free(reinterpret_cast<void*>(p));
    if (st != FA_OK) throw std::runtime_error(err_text(st));
  }, py::arg("address"));
}
