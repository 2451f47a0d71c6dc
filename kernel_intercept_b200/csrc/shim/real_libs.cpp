// real_libs.cpp — see real_libs.h.
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "real_libs.h"

#include <dlfcn.h>

#include <mutex>

namespace orion {
namespace real {
namespace {

struct Lib {
  const char* const* sonames;
  void* handle = nullptr;
  bool tried = false;
  std::mutex mu;
};

const char* const kCudart[] = {"libcudart.so.12", "libcudart.so.13", "libcudart.so", nullptr};
const char* const kCuda[] = {"libcuda.so.1", "libcuda.so", nullptr};
const char* const kCublas[] = {"libcublas.so.12", "libcublas.so.13", "libcublas.so", nullptr};
const char* const kCublasLt[] = {"libcublasLt.so.12", "libcublasLt.so.13", "libcublasLt.so",
                                 nullptr};
const char* const kCudnn[] = {"libcudnn.so.9", "libcudnn.so.8", "libcudnn.so", nullptr};

Lib g_cudart{kCudart}, g_cuda{kCuda}, g_cublas{kCublas}, g_cublaslt{kCublasLt}, g_cudnn{kCudnn};

void* self_handle() {
  static void* self = [] {
    Dl_info info;
    if (dladdr(reinterpret_cast<void*>(&self_handle), &info) && info.dli_fname)
      return dlopen(info.dli_fname, RTLD_NOW | RTLD_NOLOAD);
    return static_cast<void*>(nullptr);
  }();
  return self;
}

void* lookup(Lib& lib, const char* name) {
  {
    std::lock_guard<std::mutex> lk(lib.mu);
    if (!lib.tried) {
      lib.tried = true;
      for (int i = 0; lib.sonames[i] && !lib.handle; ++i)
        lib.handle = dlopen(lib.sonames[i], RTLD_NOW | RTLD_NOLOAD);
    }
  }
  void* fn = nullptr;
  if (lib.handle) fn = dlsym(lib.handle, name);
  if (!fn) {
    fn = dlsym(RTLD_NEXT, name);
    // RTLD_NEXT may hand back our own export when nothing follows us
    Dl_info a, b;
    if (fn && dladdr(fn, &a) && dladdr(reinterpret_cast<void*>(&self_handle), &b) &&
        a.dli_fbase == b.dli_fbase)
      fn = nullptr;
  }
  if (!fn) {
    std::lock_guard<std::mutex> lk(lib.mu);
    if (!lib.handle) {
      for (int i = 0; lib.sonames[i] && !lib.handle; ++i)
        lib.handle = dlopen(lib.sonames[i], RTLD_NOW | RTLD_GLOBAL);
    }
    if (lib.handle) fn = dlsym(lib.handle, name);
  }
  (void)self_handle;
  return fn;
}

}  // namespace

void* cudart(const char* name) { return lookup(g_cudart, name); }
void* cudadrv(const char* name) { return lookup(g_cuda, name); }
void* cublas(const char* name) { return lookup(g_cublas, name); }
void* cublaslt(const char* name) { return lookup(g_cublaslt, name); }
void* cudnn(const char* name) { return lookup(g_cudnn, name); }

}  // namespace real
}  // namespace orion
