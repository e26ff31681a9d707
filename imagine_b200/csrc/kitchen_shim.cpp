// imagine_kitchen_call-compatible front end over libw8a8.
//
// The reference's Rust crate reaches its INT8 kernels through one C entry
// point, imagine_kitchen_call(name, KitchenArg*, n, int64_t* result)
// (inference/native/bridge.hpp:5-6, 29; inference/native/bridge.cpp:421-441),
// whose arguments are borrowed at::Tensor* handles, integers, doubles and
// bools, and its FP8 linear through imagine_fp8_scaled_mm
// (inference/native/bridge.cpp:401-413).  This file implements those two, and
// imagine_last_error / imagine_last_accelerator_code, on libw8a8's plain C
// entry points; kitchen_forward.cpp passes every other function of the
// bridge, and every kernel name imagine_kitchen_call does not map, through to
// the reference's own bridge library (IMAGINE_KITCHEN_FALLBACK_LIBRARY), so
// the crate can load this library through IMAGINE_KITCHEN_LIBRARY with every
// symbol it resolves present.  Error classes follow the bridge: 0 ok, -1
// runtime, -20 ValueError, -21 IndexError (and libw8a8's -9 / -10 pass
// through).
//
// Names and argument lists (call sites in inference/src/cuda_linear.rs and
// inference/src/convrot.rs):
//   quantize_int8_rowwise(x, q, scale, stochastic, seed, stream)        :605-616
//   int8_gemv_dequant(q, w, xs, ws, bias, out, code, stream, [r], [rs]) :657-677
//   cutlass_int8_dequant(q, w, xs, ws, bias, out, code, stream)        :746-764
//   cutlass_int8_dequant_residual(q, w, xs, ws, bias, rs, r, out, code, stream)
//                                                                        :724-743
//   cublas_gemm_int8(q, w, acc, workspace, stream)                      :769-780
//   dequantize_int8_linear(acc, xs, ws, bias, out, code, stream)        :782-795
//   int8_linear_m1(x, q, xs, w, ws, bias, out, code, convrot, group, act,
//                  act_w, eps, stream, [r], [rs])                       :557-583
//   quantize_int8_rowwise_convrot64(x, q, s, group, stochastic, act, seed,
//                                   act_w, eps, stream)        convrot.rs:189-204
// The route's numerics are the reference CUDA route's: Kitchen row scales and
// the chained dequant order.  A zero-element tensor stands for an absent
// bias / activation weight (cuda_linear.rs:16-24).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../../include/w8a8.h"
#include "kitchen_forward.h"

extern "C" {
struct KitchenArg {
  int64_t kind;  // 0 None, 1 borrowed at::Tensor*, 2 int64, 3 double, 4 bool
  void* tensor;
  int64_t integer;
  double real;
};
}

namespace {

thread_local std::string g_error;
thread_local int g_accel = 0;

struct ValueError : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};

// A kernel name (or an fp8_scaled_mm form) this library does not run itself:
// forwarded to the reference bridge library.
struct NotNative {};

class Args {
 public:
  Args(const KitchenArg* a, size_t n, const char* name) : a_(a), n_(n), name_(name) {}
  size_t size() const { return n_; }
  const at::Tensor& tensor(size_t i) const {
    check(i);
    if (a_[i].kind != 1 || !a_[i].tensor) {
      throw ValueError(std::string(name_) + ": argument " + std::to_string(i) + " must be a tensor");
    }
    return *static_cast<const at::Tensor*>(a_[i].tensor);
  }
  // optional tensor: None, or an empty tensor, reads as absent
  const at::Tensor* opt_tensor(size_t i) const {
    if (i >= n_ || a_[i].kind == 0) return nullptr;
    const at::Tensor& t = tensor(i);
    return t.numel() == 0 ? nullptr : &t;
  }
  int64_t integer(size_t i) const {
    check(i);
    if (a_[i].kind != 2 && a_[i].kind != 4) {
      throw ValueError(std::string(name_) + ": argument " + std::to_string(i) + " must be an integer");
    }
    return a_[i].integer;
  }
  double real(size_t i) const {
    check(i);
    if (a_[i].kind == 3) return a_[i].real;
    if (a_[i].kind == 2) return static_cast<double>(a_[i].integer);
    throw ValueError(std::string(name_) + ": argument " + std::to_string(i) + " must be a number");
  }

 private:
  void check(size_t i) const {
    if (i >= n_) {
      throw std::out_of_range(std::string(name_) + ": missing argument " + std::to_string(i));
    }
  }
  const KitchenArg* a_;
  size_t n_;
  const char* name_;
};

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return W8A8_F32;
    case at::kHalf: return W8A8_F16;
    case at::kBFloat16: return W8A8_BF16;
    default: break;
  }
  throw ValueError("unsupported floating dtype " + std::string(c10::toString(t.scalar_type())));
}

void* stream_of(int64_t s) { return reinterpret_cast<void*>(static_cast<uintptr_t>(s)); }

// rows x K view of the last dimension; K-contiguous rows required.
void rows_cols(const at::Tensor& t, int64_t& rows, int64_t& cols, int64_t& ld) {
  if (t.dim() == 0) throw ValueError("expected a tensor with at least one dimension");
  cols = t.size(-1);
  rows = cols ? t.numel() / cols : 0;
  if (t.numel() > 0 && t.stride(-1) != 1) throw ValueError("rows must be contiguous in the last dimension");
  ld = t.dim() >= 2 ? t.stride(-2) : cols;
  if (t.dim() > 2 && !t.is_contiguous()) throw ValueError("inputs of more than two dimensions must be contiguous");
  if (rows <= 1) ld = cols;
}

void rc_or_throw(int rc) {
  if (rc == 0) return;
  const char* msg = w8a8_last_error();
  std::string m = msg ? msg : "libw8a8 error";
  if (rc == W8A8_ERR_VALUE) throw ValueError(m);
  if (rc == W8A8_ERR_INDEX) throw std::out_of_range(m);
  if (rc == W8A8_ERR_ACCELERATOR) g_accel = w8a8_last_accelerator_code();
  throw std::runtime_error(m);
}

// Dequant order of the Kitchen kernel each entry stands for
// (native/comfy-port/kitchen/int8_linear.cu as built, fmad on):
//   one-row GEMV (586-667) and the stand-alone dequant with a bias (518-543):
//     (acc*xs)*ws, then + bias in a statement of its own -> SEPARATE;
//   two-row GEMV (669-708): acc*xs*ws + b in one expression -> CHAINED (FMA);
//   stand-alone dequant without a bias (545-583): acc*(xs*ws) for a scalar
//     weight scale and N % 4 == 0 (its vec4 kernel) -> SCALE_PRODUCT, else
//     (acc*xs)*ws -> CHAINED (no bias: the same two products).
w8a8_epilogue_t epilogue(const at::Tensor& ws, const at::Tensor* bias, const at::Tensor* resid,
                         const at::Tensor* rscale, int64_t n, int order = W8A8_DQ_CHAINED) {
  w8a8_epilogue_t e{};
  e.ws = ws.data_ptr<float>();
  e.ws_numel = ws.numel();
  e.bias = bias ? bias->data_ptr() : nullptr;
  e.residual = resid ? resid->data_ptr() : nullptr;
  e.ldr = n;
  e.residual_scale = rscale ? rscale->data_ptr() : nullptr;
  e.dequant_order = order;
  e.activation = W8A8_ACT_NONE;
  return e;
}

void check_ws(const at::Tensor& ws) {
  if (ws.scalar_type() != at::kFloat || !ws.is_contiguous()) {
    throw ValueError("weight scale must be a contiguous float32 tensor");
  }
}

int64_t dispatch(const char* name, const Args& a) {
  const std::string op(name);
  if (op == "quantize_int8_rowwise") {
    const at::Tensor& x = a.tensor(0);
    int64_t rows, k, ldx;
    rows_cols(x, rows, k, ldx);
    rc_or_throw(w8a8_quantize_rowwise(x.data_ptr(), dtype_code(x), rows, k, ldx,
                                      a.tensor(1).data_ptr<int8_t>(), k,
                                      a.tensor(2).data_ptr<float>(), W8A8_SCALE_KITCHEN_CUDA,
                                      a.integer(3) ? 1 : 0, static_cast<uint64_t>(a.integer(4)),
                                      stream_of(a.integer(5))));
    return 0;
  }
  if (op == "int8_gemv_dequant") {
    const at::Tensor& q = a.tensor(0);
    const at::Tensor& w = a.tensor(1);
    const at::Tensor& ws = a.tensor(3);
    const at::Tensor& out = a.tensor(5);
    check_ws(ws);
    const int64_t m = q.size(0), k = q.size(1), n = w.size(0);
    const w8a8_epilogue_t e = epilogue(ws, a.opt_tensor(4), a.opt_tensor(8), a.opt_tensor(9), n,
                                       m == 2 ? W8A8_DQ_CHAINED : W8A8_DQ_SEPARATE);
    rc_or_throw(w8a8_gemv_dequant(q.data_ptr<int8_t>(), w.data_ptr<int8_t>(),
                                  a.tensor(2).data_ptr<float>(), &e, out.data_ptr(),
                                  static_cast<int>(a.integer(6)), m, n, k,
                                  stream_of(a.integer(7))));
    return 0;
  }
  if (op == "cutlass_int8_dequant" || op == "cutlass_int8_dequant_residual") {
    const bool resid = op == "cutlass_int8_dequant_residual";
    const at::Tensor& q = a.tensor(0);
    const at::Tensor& w = a.tensor(1);
    const at::Tensor& ws = a.tensor(3);
    check_ws(ws);
    const at::Tensor& out = a.tensor(resid ? 7 : 5);
    const int64_t m = q.size(0), k = q.size(1), n = w.size(0);
    const w8a8_epilogue_t e = epilogue(ws, a.opt_tensor(4), resid ? &a.tensor(6) : nullptr,
                                       resid ? &a.tensor(5) : nullptr, n);
    rc_or_throw(w8a8_gemm_dequant(q.data_ptr<int8_t>(), k, w.data_ptr<int8_t>(), k,
                                  a.tensor(2).data_ptr<float>(), &e, out.data_ptr(),
                                  static_cast<int>(a.integer(resid ? 8 : 6)), n, m, n, k, nullptr,
                                  stream_of(a.integer(resid ? 9 : 7))));
    return 1;  // the reference reads a nonzero result as "the fused GEMM ran"
  }
  if (op == "cublas_gemm_int8") {
    const at::Tensor& q = a.tensor(0);
    const at::Tensor& w = a.tensor(1);
    const at::Tensor& acc = a.tensor(2);
    rc_or_throw(w8a8_gemm_s32(q.data_ptr<int8_t>(), w.data_ptr<int8_t>(), acc.data_ptr<int32_t>(),
                              q.size(0), w.size(0), q.size(1), nullptr, stream_of(a.integer(4))));
    return 0;
  }
  if (op == "dequantize_int8_linear") {
    const at::Tensor& acc = a.tensor(0);
    const at::Tensor& ws = a.tensor(2);
    check_ws(ws);
    const at::Tensor& out = a.tensor(4);
    const int64_t m = acc.size(0), n = acc.size(1);
    const at::Tensor* bias = a.opt_tensor(3);
    const int order = bias ? W8A8_DQ_SEPARATE
                    : (ws.numel() == 1 && n % 4 == 0) ? W8A8_DQ_SCALE_PRODUCT
                    : W8A8_DQ_CHAINED;
    const w8a8_epilogue_t e = epilogue(ws, bias, nullptr, nullptr, n, order);
    rc_or_throw(w8a8_dequantize_linear(acc.data_ptr<int32_t>(), a.tensor(1).data_ptr<float>(), &e,
                                       out.data_ptr(), static_cast<int>(a.integer(5)), m, n,
                                       stream_of(a.integer(6))));
    return 0;
  }
  if (op == "int8_linear_m1") {
    const at::Tensor& x = a.tensor(0);
    const at::Tensor& q = a.tensor(1);
    const at::Tensor& xs = a.tensor(2);
    const at::Tensor& w = a.tensor(3);
    const at::Tensor& ws = a.tensor(4);
    check_ws(ws);
    const at::Tensor& out = a.tensor(6);
    const int code = static_cast<int>(a.integer(7));
    const bool convrot = a.integer(8) != 0;
    const int group = static_cast<int>(a.integer(9));
    const int act = static_cast<int>(a.integer(10));
    const at::Tensor* act_w = a.opt_tensor(11);
    const float eps = static_cast<float>(a.real(12));
    void* stream = stream_of(a.integer(13));
    int64_t m, k, ldx;
    rows_cols(x, m, k, ldx);
    const int64_t n = w.size(0);
    const w8a8_epilogue_t e = epilogue(ws, a.opt_tensor(5), a.opt_tensor(14), a.opt_tensor(15), n,
                                       m == 2 ? W8A8_DQ_CHAINED : W8A8_DQ_SEPARATE);
    if (!convrot && act == 0) {
      rc_or_throw(w8a8_linear_small(x.data_ptr(), dtype_code(x), w.data_ptr<int8_t>(), &e,
                                    W8A8_SCALE_KITCHEN_CUDA, q.data_ptr<int8_t>(), xs.data_ptr<float>(),
                                    out.data_ptr(), code, m, n, k, stream));
    } else {
      rc_or_throw(w8a8_quantize_rowwise_convrot(
          x.data_ptr(), dtype_code(x), m, (act == W8A8_INPUT_ACT_SWIGLU || act == W8A8_INPUT_ACT_SITU) ? k / 2 : k, ldx,
          convrot ? group : 0, act, act_w ? act_w->data_ptr() : nullptr, eps,
          q.data_ptr<int8_t>(), q.size(-1), xs.data_ptr<float>(), W8A8_SCALE_KITCHEN_CUDA, stream));
      rc_or_throw(w8a8_gemv_dequant(q.data_ptr<int8_t>(), w.data_ptr<int8_t>(), xs.data_ptr<float>(),
                                    &e, out.data_ptr(), code, m, n, q.size(-1), stream));
    }
    return 0;
  }
  if (op == "quantize_int8_rowwise_convrot64") {
    const at::Tensor& x = a.tensor(0);
    const at::Tensor& q = a.tensor(1);
    if (a.integer(4)) throw ValueError("stochastic rounding is not offered by the fused ConvRot quantiser");
    const int act = static_cast<int>(a.integer(5));
    const at::Tensor* act_w = a.opt_tensor(7);
    int64_t rows, width, ldx;
    rows_cols(x, rows, width, ldx);
    rc_or_throw(w8a8_quantize_rowwise_convrot(
        x.data_ptr(), dtype_code(x), rows, q.size(-1), ldx, static_cast<int>(a.integer(3)), act,
        act_w ? act_w->data_ptr() : nullptr, static_cast<float>(a.real(8)), q.data_ptr<int8_t>(),
        q.size(-1), a.tensor(2).data_ptr<float>(), W8A8_SCALE_KITCHEN_CUDA, stream_of(a.integer(9))));
    return 0;
  }
  throw NotNative{};
}

// at::_scaled_mm_v2 TensorWise on e4m3 operands (bridge.cpp:401-413): a
// [M, K] e4m3 (made contiguous, as there), b [K, N] e4m3 column-major (the
// transposed view of a row-major [N, K] weight), fp32 scalar scales, optional
// bias [N], output dtype `kind` (an at::ScalarType code).  Forms the tcgen05
// kernel does not take -- other scalings, an fp8 or default (kind < 0)
// output, a row-major b -- are not native.
at::Tensor fp8_scaled_mm(const at::Tensor& a_in, const at::Tensor& b, const at::Tensor& sa,
                         const at::Tensor& sb, const at::Tensor* bias, int64_t kind) {
  if (kind < 0) throw NotNative{};
  const auto out_type = static_cast<at::ScalarType>(kind);
  if (out_type != at::kBFloat16 && out_type != at::kHalf && out_type != at::kFloat) throw NotNative{};
  if (a_in.scalar_type() != at::kFloat8_e4m3fn || b.scalar_type() != at::kFloat8_e4m3fn ||
      a_in.dim() != 2 || b.dim() != 2 || sa.numel() != 1 || sb.numel() != 1 ||
      sa.scalar_type() != at::kFloat || sb.scalar_type() != at::kFloat || !a_in.is_cuda()) {
    throw NotNative{};
  }
  const int64_t m = a_in.size(0), k = a_in.size(1), n = b.size(1);
  if (b.size(0) != k) throw ValueError("mat1 and mat2 shapes cannot be multiplied");
  // b column-major: b.t() is a row-major [N, K] weight
  if (!(b.stride(0) == 1 && (b.stride(1) == k || n == 1))) throw NotNative{};
  if (bias && (bias->numel() != n || bias->scalar_type() != out_type || !bias->is_contiguous())) {
    throw NotNative{};
  }
  const at::Tensor a = a_in.contiguous();
  at::Tensor out = at::empty({m, n}, a.options().dtype(out_type));
  const int code = out_type == at::kBFloat16 ? W8A8_BF16 : out_type == at::kHalf ? W8A8_F16 : W8A8_F32;
  void* stream = reinterpret_cast<void*>(c10::cuda::getCurrentCUDAStream(a.device().index()).stream());
  rc_or_throw(w8a8_fp8_gemm(static_cast<const uint8_t*>(a.data_ptr()),
                            static_cast<const uint8_t*>(b.data_ptr()), sa.data_ptr<float>(),
                            sb.data_ptr<float>(), bias ? bias->data_ptr() : nullptr, out.data_ptr(),
                            code, m, n, k, nullptr, stream));
  return out;
}

}  // namespace

namespace kitchen_forward {
void set_error(const std::string& message, int accelerator_code) {
  g_error = message;
  g_accel = accelerator_code;
}
}  // namespace kitchen_forward

extern "C" {

__attribute__((visibility("default"))) const char* imagine_last_error() { return g_error.c_str(); }

__attribute__((visibility("default"))) int imagine_last_accelerator_code() { return g_accel; }

__attribute__((visibility("default"))) int imagine_kitchen_call(const char* name,
                                                               const KitchenArg* args, size_t n,
                                                               int64_t* result) {
  try {
    if (!name || !result || (!args && n)) throw std::runtime_error("Null bridge argument");
    // the caller's device: the first tensor argument's (bridge.cpp:421-428)
    c10::optional<c10::cuda::CUDAGuard> guard;
    for (size_t i = 0; i < n; ++i) {
      if (args[i].kind == 1 && args[i].tensor) {
        const auto& t = *static_cast<const at::Tensor*>(args[i].tensor);
        if (t.is_cuda()) guard.emplace(t.device());
        break;
      }
    }
    try {
      *result = dispatch(name, Args(args, n, name));
    } catch (const NotNative&) {
      using Fn = int (*)(const char*, const KitchenArg*, size_t, int64_t*);
      auto f = reinterpret_cast<Fn>(kitchen_forward::symbol("imagine_kitchen_call"));
      if (!f) {
        kitchen_forward::missing((std::string("imagine_kitchen_call(\"") + name + "\")").c_str());
        g_error = "Unknown Kitchen kernel " + std::string(name) + " (" + g_error + ")";
        return W8A8_ERR_RUNTIME;
      }
      const int rc = f(name, args, n, result);
      if (rc != 0) kitchen_forward::copy_fallback_error();
      else g_error.clear();
      return rc;
    }
    g_error.clear();
    return 0;
  } catch (const std::invalid_argument& e) {
    g_error = e.what();
    return W8A8_ERR_VALUE;
  } catch (const std::out_of_range& e) {
    g_error = e.what();
    return W8A8_ERR_INDEX;
  } catch (const std::exception& e) {
    g_error = e.what();
    return W8A8_ERR_RUNTIME;
  } catch (...) {
    g_error = "Unknown native exception";
    return W8A8_ERR_RUNTIME;
  }
}

__attribute__((visibility("default"))) int imagine_fp8_scaled_mm(const void* a, const void* b,
                                                                const void* sa, const void* sb,
                                                                const void* bias, int64_t kind,
                                                                void** output) {
  try {
    if (!a || !b || !sa || !sb || !output) throw std::runtime_error("Null bridge argument");
    const auto& at_a = *static_cast<const at::Tensor*>(a);
    c10::optional<c10::cuda::CUDAGuard> guard;
    if (at_a.is_cuda()) guard.emplace(at_a.device());
    try {
      *output = new at::Tensor(fp8_scaled_mm(at_a, *static_cast<const at::Tensor*>(b),
                                             *static_cast<const at::Tensor*>(sa),
                                             *static_cast<const at::Tensor*>(sb),
                                             static_cast<const at::Tensor*>(bias), kind));
    } catch (const NotNative&) {
      using Fn = int (*)(const void*, const void*, const void*, const void*, const void*, int64_t,
                         void**);
      auto f = reinterpret_cast<Fn>(kitchen_forward::symbol("imagine_fp8_scaled_mm"));
      if (!f) return kitchen_forward::missing("imagine_fp8_scaled_mm (this scaling / output form)");
      const int rc = f(a, b, sa, sb, bias, kind, output);
      if (rc != 0) kitchen_forward::copy_fallback_error();
      else g_error.clear();
      return rc;
    }
    g_error.clear();
    return 0;
  } catch (const std::invalid_argument& e) {
    g_error = e.what();
    return W8A8_ERR_VALUE;
  } catch (const std::out_of_range& e) {
    g_error = e.what();
    return W8A8_ERR_INDEX;
  } catch (const std::exception& e) {
    g_error = e.what();
    return W8A8_ERR_RUNTIME;
  } catch (...) {
    g_error = "Unknown native exception";
    return W8A8_ERR_RUNTIME;
  }
}

// dtype code of imagine_w8a8_tensor_view for float8_e4m3fn (libw8a8 itself
// takes e4m3 data as bytes and has no code for it)
constexpr int64_t kViewE4M3 = 5;

// Test and host convenience: a borrowed at::Tensor handle over existing
// device memory (the reference bridge's imagine_tensor_* family plays this
// role for the crate), and its release.
__attribute__((visibility("default"))) int imagine_w8a8_tensor_view(
    void* data, const int64_t* sizes, const int64_t* strides, int64_t ndim, int64_t dtype,
    int64_t device, void** out) {
  try {
    at::ScalarType st;
    switch (dtype) {
      case W8A8_F32: st = at::kFloat; break;
      case W8A8_F16: st = at::kHalf; break;
      case W8A8_BF16: st = at::kBFloat16; break;
      case W8A8_S32: st = at::kInt; break;
      case W8A8_S8: st = at::kChar; break;
      case kViewE4M3: st = at::kFloat8_e4m3fn; break;
      default: throw ValueError("unsupported dtype code " + std::to_string(dtype));
    }
    auto opts = at::TensorOptions().dtype(st).device(at::Device(at::kCUDA, static_cast<int>(device)));
    int64_t numel = 1;
    for (int64_t i = 0; i < ndim; ++i) numel *= sizes[i];
    // a zero-element tensor (the bridge's "no bias") has no storage to wrap
    auto t = numel == 0 ? at::empty(at::IntArrayRef(sizes, ndim), opts)
                        : at::from_blob(data, at::IntArrayRef(sizes, ndim),
                                        at::IntArrayRef(strides, ndim), opts);
    *out = new at::Tensor(std::move(t));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return W8A8_ERR_VALUE;
  }
}

__attribute__((visibility("default"))) void imagine_w8a8_tensor_free(void* t) {
  delete static_cast<at::Tensor*>(t);
}

// Test and host convenience: data pointer, element count and libw8a8 dtype
// code (-1 for others) of an at::Tensor handle (e.g. one a bridge call
// returned).
__attribute__((visibility("default"))) int imagine_w8a8_tensor_info(const void* t, void** data,
                                                                   int64_t* numel,
                                                                   int64_t* dtype) {
  if (!t || !data || !numel || !dtype) return W8A8_ERR_VALUE;
  const auto& x = *static_cast<const at::Tensor*>(t);
  *data = x.data_ptr();
  *numel = x.numel();
  switch (x.scalar_type()) {
    case at::kFloat: *dtype = W8A8_F32; break;
    case at::kHalf: *dtype = W8A8_F16; break;
    case at::kBFloat16: *dtype = W8A8_BF16; break;
    case at::kInt: *dtype = W8A8_S32; break;
    case at::kChar: *dtype = W8A8_S8; break;
    default: *dtype = -1; break;
  }
  return 0;
}

}  // extern "C"
