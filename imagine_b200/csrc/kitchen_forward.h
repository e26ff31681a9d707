// Shared between the two halves of libimagine_kitchen_w8a8.so: the native
// W8A8 entry points (kitchen_shim.cpp) and the pass-throughs to the
// reference's bridge library (kitchen_forward.cpp).
#pragma once

#include <string>

namespace kitchen_forward {

// The same-named function of the library in IMAGINE_KITCHEN_FALLBACK_LIBRARY
// (opened once, on first use), or nullptr.
void* symbol(const char* name);
// Records "no fallback for NAME" as the last error; returns -1.
int missing(const char* name);
// After a failed forwarded call: the fallback's last error and accelerator
// code become this library's.
void copy_fallback_error();
// This library's thread-local last error and accelerator code
// (kitchen_shim.cpp).
void set_error(const std::string& message, int accelerator_code);

}  // namespace kitchen_forward
