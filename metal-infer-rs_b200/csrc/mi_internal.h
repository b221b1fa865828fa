// Internal types of the B200 engine: context, tensors, batches, errors.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdint>
#include <string>
#include <vector>

#include "mi.h"

namespace mi {

// ---- errors ---------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

struct Error {
  mi_status status;
  std::string message;
};

// Raised inside the engine, converted to mi_status at the C boundary.
[[noreturn]] void fail(mi_status status, const char* fmt, ...);

#define MI_CUDA(call)                                                         \
  do {                                                                        \
    cudaError_t err_ = (call);                                                \
    if (err_ != cudaSuccess)                                                  \
      ::mi::fail(MI_ERR_COMMAND, "%s failed: %s (%s:%d)", #call,              \
                 cudaGetErrorString(err_), __FILE__, __LINE__);               \
  } while (0)

#define MI_REQUIRE(cond, status, ...)                                         \
  do {                                                                        \
    if (!(cond)) ::mi::fail(status, __VA_ARGS__);                             \
  } while (0)

// Runs `body` and converts an Error into a status + thread-local message.
template <class F>
mi_status guard(F&& body) {
  try {
    clear_error();
    body();
    return MI_OK;
  } catch (const Error& e) {
    set_error("%s", e.message.c_str());
    return e.status;
  } catch (const std::bad_alloc&) {
    set_error("host allocation failed");
    return MI_ERR_RESOURCE;
  } catch (...) {
    set_error("unexpected internal error");
    return MI_ERR_COMMAND;
  }
}

inline size_t dtype_size(mi_dtype d) { return d == MI_F16 ? 2 : 4; }
inline const char* dtype_name(mi_dtype d) {
  return d == MI_F16 ? "f16" : d == MI_F32 ? "f32" : "u32";
}

// ---- device buffers ---------------------------------------------------------
// A device allocation shared by tensor views. Freed stream-ordered on the
// owning context's stream when the last reference goes away.
struct Buffer {
  mi_context* ctx = nullptr;
  void* ptr = nullptr;
  size_t bytes = 0;
  bool owned = true;
  std::atomic<int> refs{1};
};

void buffer_release(Buffer* b);

}  // namespace mi

// Opaque handles of the C ABI.
struct mi_tensor {
  mi::Buffer* buf = nullptr;
  size_t offset = 0;  // bytes
  std::vector<size_t> shape;
  mi_dtype dtype = MI_F16;

  size_t len() const {
    size_t n = 1;
    for (size_t d : shape) n *= d;
    return n;
  }
  size_t bytes() const { return len() * mi::dtype_size(dtype); }
  char* base() const { return static_cast<char*>(buf->ptr) + offset; }
  __half* f16() const { return reinterpret_cast<__half*>(base()); }
  float* f32() const { return reinterpret_cast<float*>(base()); }
  uint32_t* u32() const { return reinterpret_cast<uint32_t*>(base()); }
};

struct mi_context {
  // Released by mi_context_destroy and by every buffer, batch and model that
  // refers to the context; torn down when the count reaches zero, so handles
  // may be destroyed in any order.
  std::atomic<int> refs{1};
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string name;
  int sm_count = 0;
  size_t allocated = 0;  // live bytes of engine-owned buffers
  mi_matmul_backend backend = MI_MATMUL_AUTO;
  bool profiling = false;
  struct Profile {
    std::string kernel;
    cudaEvent_t start, stop;
  };
  std::vector<Profile> pending_profiles;
  std::vector<mi_kernel_profile> profiles;
  // Reusable zero-initialised scratch for split reductions (grown on demand).
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
};

struct mi_batch {
  mi_context* ctx = nullptr;
  cudaEvent_t start = nullptr;
  std::chrono::steady_clock::time_point wall_start;
};

struct mi_pending {
  mi_context* ctx = nullptr;
  cudaEvent_t start = nullptr;
  cudaEvent_t stop = nullptr;
  std::chrono::steady_clock::time_point wall_start;
};

namespace mi {

// Allocates a tensor on the context stream (stream-ordered, zero-filled when
// `zero`).
mi_tensor* new_tensor(mi_context* ctx, const std::vector<size_t>& shape, mi_dtype dtype,
                      bool zero = false);
mi_tensor* view(const mi_tensor* t, const std::vector<size_t>& shape, size_t extra_offset);
void context_retain(mi_context* ctx);
void context_release(mi_context* ctx);
void* context_scratch(mi_context* ctx, size_t bytes);
void sync_context(mi_context* ctx);
// First code recorded by any kernel's bounded device wait since the last
// read (0: none), cleared when read. Call after a synchronization.
unsigned take_device_wait_status();
// Fails with MI_ERR_TIMEOUT when a bounded device wait expired (after a
// synchronization): a launch that gave up returns early, so its outputs are
// not valid and must not be reported as a result.
void check_device_waits(const char* what);

// Per-launch profiling hooks (CUDA events around a launch when enabled).
struct ProfileScope {
  mi_context* ctx;
  const char* name;
  cudaEvent_t a = nullptr, b = nullptr;
  ProfileScope(mi_context* c, const char* n);
  ~ProfileScope();
};

}  // namespace mi
