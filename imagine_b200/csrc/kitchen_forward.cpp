// Pass-through half of libimagine_kitchen_w8a8.so: every function of the
// reference's native bridge (inference/native/bridge.hpp:11-84) that this
// library does not implement itself.
//
// The crate resolves 52 of these names eagerly when it loads its bridge
// library (Kitchen::load, inference/src/native.rs:1299-1354) and fails on the
// first one missing, so a drop-in for its W8A8 kernels must export them all.
// This library implements imagine_kitchen_call (the W8A8 kernels),
// imagine_fp8_scaled_mm, imagine_last_error and imagine_last_accelerator_code
// (kitchen_shim.cpp); everything else -- tensor, stream, event, generator and
// allocator helpers, SDPA, ATen boxed calls -- is LibTorch plumbing the
// reference's own bridge provides.  Each such function here forwards to the
// same-named function of the reference bridge library, opened on first use
// (dlopen, RTLD_LOCAL) from the path in IMAGINE_KITCHEN_FALLBACK_LIBRARY.
// Without that variable, or when the library lacks the name, an int-returning
// function fails with -1 (the bridge's RuntimeError family) and a message in
// imagine_last_error(); void functions do nothing, imagine_last_metadata()
// returns "" and imagine_tensor_identity() returns 0.  After a forwarded call
// fails, the fallback's error message and accelerator code are copied so that
// this library's imagine_last_error / imagine_last_accelerator_code report
// them.
#include <dlfcn.h>

#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <string>

#include "kitchen_forward.h"

namespace kitchen_forward {

namespace {
std::once_flag g_open_once;
void* g_handle = nullptr;
std::string g_open_error;

void open_fallback() {
  const char* path = std::getenv("IMAGINE_KITCHEN_FALLBACK_LIBRARY");
  if (!path || !*path) {
    g_open_error = "IMAGINE_KITCHEN_FALLBACK_LIBRARY is not set";
    return;
  }
  g_handle = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!g_handle) {
    const char* e = dlerror();
    g_open_error = std::string("cannot open IMAGINE_KITCHEN_FALLBACK_LIBRARY ") + path + ": " +
                   (e ? e : "unknown error");
  }
}
}  // namespace

void* symbol(const char* name) {
  std::call_once(g_open_once, open_fallback);
  if (!g_handle) return nullptr;
  return dlsym(g_handle, name);
}

int missing(const char* name) {
  std::call_once(g_open_once, open_fallback);
  std::string msg = std::string(name) +
                    " is not implemented by libimagine_kitchen_w8a8 (it provides the W8A8 kernels) "
                    "and has no reference bridge library to forward to: ";
  msg += g_handle ? "the library does not export it" : g_open_error;
  set_error(msg, 0);
  return -1;
}

void copy_fallback_error() {
  using ErrFn = const char* (*)();
  using AccFn = int (*)();
  auto err = reinterpret_cast<ErrFn>(symbol("imagine_last_error"));
  auto acc = reinterpret_cast<AccFn>(symbol("imagine_last_accelerator_code"));
  const char* e = err ? err() : nullptr;
  set_error(e ? e : "error in the reference bridge library", acc ? acc() : 0);
}

}  // namespace kitchen_forward

struct KitchenArg;
struct TensorTypeInfo;
struct TensorStorageInfo;
struct CudaDeviceProperties;
struct RmsTemporaryMetadata;

#define KF_VIS __attribute__((visibility("default")))

// An int-returning pass-through: PARAMS is the parameter list with names,
// ARGS the names alone.
#define KF_INT(NAME, PARAMS, ARGS)                                             \
  extern "C" KF_VIS int NAME PARAMS {                                          \
    using Fn = int(*) PARAMS;                                                  \
    auto kf_fn_ = reinterpret_cast<Fn>(kitchen_forward::symbol(#NAME));        \
    if (!kf_fn_) return kitchen_forward::missing(#NAME);                       \
    const int rc = kf_fn_ ARGS;                                                \
    if (rc != 0) kitchen_forward::copy_fallback_error();                       \
    return rc;                                                                 \
  }

#define KF_VOID(NAME, PARAMS, ARGS)                                            \
  extern "C" KF_VIS void NAME PARAMS {                                         \
    using Fn = void(*) PARAMS;                                                 \
    auto kf_fn_ = reinterpret_cast<Fn>(kitchen_forward::symbol(#NAME));        \
    if (kf_fn_) kf_fn_ ARGS;                                                   \
  }

KF_INT(imagine_beta_ppf, (double a, double b, double c, double* d, const char** e, const char** f),
       (a, b, c, d, e, f))
KF_INT(imagine_tensor_owned_buffer,
       (void* a, const int64_t* b, size_t c, int64_t d, void* e, void (*f)(void*), void** g),
       (a, b, c, d, e, f, g))
KF_INT(imagine_tensor_empty_scalar, (const int64_t* a, size_t b, int64_t c, void** d), (a, b, c, d))
KF_INT(imagine_tensor_buffer_context, (const void* a, void (*b)(void*), void** c), (a, b, c))
KF_INT(imagine_comfy_sdpa,
       (const void* a, const void* b, const void* c, const void* d, int64_t e, double f, int64_t g,
        int64_t h, void** i),
       (a, b, c, d, e, f, g, h, i))
KF_INT(imagine_sdpa_state, (int64_t* a, int64_t b), (a, b))
KF_INT(imagine_cuda_memory, (int64_t a, uint64_t* b), (a, b))
KF_INT(imagine_cuda_allocator_stats, (int64_t a, uint64_t* b), (a, b))
KF_INT(imagine_host_registration, (const void* a, int64_t b, int64_t* c), (a, b, c))
KF_INT(imagine_host_registration_raw, (uint64_t a, uint64_t b, int64_t c, int64_t* d), (a, b, c, d))
KF_INT(imagine_tensor_video_slice_assign, (void* a, int64_t b, int64_t c, const void* d),
       (a, b, c, d))
KF_INT(imagine_cuda_soft_empty_cache, (int64_t a), (a))
KF_INT(imagine_comfy_math_state, (int64_t* a, int64_t b), (a, b))
KF_INT(imagine_aten_boxed,
       (const char* a, const char* b, const void* const* c, size_t d, const char* const* e,
        const void* const* f, size_t g, void** h),
       (a, b, c, d, e, f, g, h))
KF_INT(imagine_cublaslt_available, (int64_t* a), (a))
KF_INT(imagine_cuda_current_device, (int64_t* a), (a))
KF_INT(imagine_cuda_device_count, (int64_t* a), (a))
KF_INT(imagine_cuda_current_capability, (int64_t* a, int64_t* b), (a, b))
KF_INT(imagine_cuda_device_properties, (int64_t a, CudaDeviceProperties* b), (a, b))
KF_INT(imagine_rms_metadata_begin, (), ())
KF_INT(imagine_rms_metadata_end, (RmsTemporaryMetadata* a), (a))
KF_INT(imagine_cat, (const void* const* a, size_t b, int64_t c, void** d), (a, b, c, d))
KF_INT(imagine_amax_last, (const void* a, void** b), (a, b))
KF_INT(imagine_embedding, (const void* a, const void* b, void** c), (a, b, c))
KF_INT(imagine_parse_device, (const char* a, int64_t* b, int64_t* c), (a, b, c))
KF_INT(imagine_tensor_empty_like_device_spec, (const void* a, int64_t b, int64_t c, void** d),
       (a, b, c, d))
KF_INT(imagine_tensor_to_device_spec, (const void* a, int64_t b, int64_t c, void** d), (a, b, c, d))
KF_INT(imagine_default_dtype, (int64_t* a), (a))
KF_INT(imagine_set_default_dtype, (int64_t a), (a))
KF_INT(imagine_current_stream, (int64_t a, uint64_t* b), (a, b))
KF_INT(imagine_stream_guard_new, (int64_t a, void** b), (a, b))
KF_VOID(imagine_stream_guard_free, (void* a), (a))
KF_INT(imagine_event_record, (int64_t a, void** b), (a, b))
KF_VOID(imagine_event_free, (void* a), (a))
KF_INT(imagine_event_wait, (void* a, int64_t b), (a, b))
KF_INT(imagine_event_synchronize, (void* a), (a))
KF_INT(imagine_timing_event_new, (void** a), (a))
KF_INT(imagine_event_record_existing, (void* a, int64_t b), (a, b))
KF_INT(imagine_event_elapsed, (void* a, void* b, double* c), (a, b, c))
KF_INT(imagine_device_synchronize, (int64_t a), (a))
KF_INT(imagine_tensor_clone, (const void* a, void** b), (a, b))
KF_INT(imagine_tensor_empty_like, (const void* a, int64_t b, void** c), (a, b, c))
KF_INT(imagine_tensor_empty_like_dtype, (const void* a, int64_t b, void** c), (a, b, c))
KF_INT(imagine_tensor_copy, (void* a, const void* b, int64_t c), (a, b, c))
KF_INT(imagine_tensor_type, (const void* a, TensorTypeInfo* b), (a, b))
KF_INT(imagine_tensor_storage, (const void* a, TensorStorageInfo* b), (a, b))
KF_INT(imagine_tensor_shell_view, (const void* a, int64_t b, void** c), (a, b, c))
KF_INT(imagine_generator_new, (int64_t a, uint64_t b, void** c), (a, b, c))
KF_VOID(imagine_generator_free, (void* a), (a))
KF_INT(imagine_generator_state, (void* a, void** b), (a, b))
KF_INT(imagine_generator_set_state, (void* a, const void* b), (a, b))
KF_INT(imagine_generator_randn, (void* a, const int64_t* b, size_t c, int64_t d, void** e),
       (a, b, c, d, e))
KF_INT(imagine_generator_rand, (void* a, const int64_t* b, size_t c, int64_t d, void** e),
       (a, b, c, d, e))
KF_INT(imagine_generator_randbytes, (void* a, const int64_t* b, size_t c, void** d), (a, b, c, d))
KF_INT(imagine_generator_randint, (void* a, int64_t b, const int64_t* c, size_t d, void** e),
       (a, b, c, d, e))
KF_INT(imagine_tensor_item_double, (const void* a, double* b), (a, b))
KF_INT(imagine_tensor_grad_name, (const void* a, const char** b), (a, b))
KF_INT(imagine_ivalue_uint, (uint64_t a, void** b), (a, b))
KF_INT(imagine_ivalue_get_uint, (const void* a, uint64_t* b), (a, b))

extern "C" KF_VIS const char* imagine_last_metadata() {
  using Fn = const char* (*)();
  auto f = reinterpret_cast<Fn>(kitchen_forward::symbol("imagine_last_metadata"));
  return f ? f() : "";
}

extern "C" KF_VIS uint64_t imagine_tensor_identity(const void* t) {
  using Fn = uint64_t (*)(const void*);
  auto f = reinterpret_cast<Fn>(kitchen_forward::symbol("imagine_tensor_identity"));
  return f ? f(t) : 0;
}
