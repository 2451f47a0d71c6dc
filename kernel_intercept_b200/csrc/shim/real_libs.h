// real_libs.h — lookup of the real CUDA runtime / driver / cuBLAS / cuBLASLt /
// cuDNN entry points behind the interposer.
//
// The interposer exports functions with the libraries' own names, so every
// call it makes to those libraries must go through pointers obtained here
// (never through the exported names, which would re-enter the wrappers).
// Lookup order per library: a copy already loaded in the process
// (dlopen(RTLD_NOLOAD) of the usual sonames), then the next definition after
// this library in the global scope (RTLD_NEXT), then loading the soname.
// The real cuBLAS / cuDNN are only used for descriptor getters, handle
// bookkeeping and for calls outside the captured dense-op contract.
#pragma once

namespace orion {
namespace real {

void* cudart(const char* name);
void* cudadrv(const char* name);
void* cublas(const char* name);
void* cublaslt(const char* name);
void* cudnn(const char* name);

}  // namespace real
}  // namespace orion

// Cached real pointer for a function whose prototype is visible (CUDA runtime /
// driver declarations from the CUDA headers).
#define ORION_REAL(lib, name)                                                               \
  ([]() {                                                                                   \
    static auto fp_ = reinterpret_cast<decltype(&::name)>(orion::real::lib(#name));        \
    return fp_;                                                                             \
  }())

// Cached real pointer with an explicit function-pointer type.
#define ORION_REAL_T(lib, type, name)                                                       \
  ([]() {                                                                                   \
    static auto fp_ = reinterpret_cast<type>(orion::real::lib(name));                       \
    return fp_;                                                                             \
  }())
