// Runtime of the C ABI: errors, context (one CUDA stream per context),
// reference-counted tensor views over stream-ordered device memory, batches
// with CUDA-event completion, and per-launch profiling.
//
// Replaces MetalContext / CommandBatch / PendingBatch / Tensor
// (crates/metal-infer-core/src/context.rs:155-1128, tensor.rs:1-261).

#include <cstdio>
#include <cstring>
#include <mutex>

#include "kernels.h"
#include "mi_internal.h"

namespace mi {

namespace {
thread_local std::string g_error;
}

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
}

void clear_error() { g_error.clear(); }

void fail(mi_status status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw Error{status, buf};
}

void buffer_release(Buffer* b) {
  if (!b) return;
  if (b->refs.fetch_sub(1) != 1) return;
  mi_context* ctx = b->ctx;
  if (b->owned && b->ptr) {
    cudaSetDevice(ctx->device);
    cudaFreeAsync(b->ptr, ctx->stream);
    ctx->allocated -= b->bytes;
  }
  delete b;
  context_release(ctx);
}

void context_retain(mi_context* ctx) { ctx->refs.fetch_add(1); }

void context_release(mi_context* ctx) {
  if (!ctx || ctx->refs.fetch_sub(1) != 1) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (auto& p : ctx->pending_profiles) {
    cudaEventDestroy(p.start);
    cudaEventDestroy(p.stop);
  }
  if (ctx->scratch) cudaFreeAsync(ctx->scratch, ctx->stream);
  cudaStreamSynchronize(ctx->stream);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
}

mi_tensor* new_tensor(mi_context* ctx, const std::vector<size_t>& shape, mi_dtype dtype,
                      bool zero) {
  size_t n = 1;
  for (size_t d : shape) {
    MI_REQUIRE(d == 0 || n <= SIZE_MAX / d, MI_ERR_SHAPE, "tensor size overflow");
    n *= d;
  }
  size_t bytes = n * dtype_size(dtype);
  auto* b = new Buffer();
  b->ctx = ctx;
  b->bytes = bytes;
  size_t alloc = bytes ? ((bytes + 255) & ~size_t(255)) : 256;
  cudaError_t err = cudaMallocAsync(&b->ptr, alloc, ctx->stream);
  if (err != cudaSuccess) {
    delete b;
    fail(MI_ERR_RESOURCE, "device allocation of %zu bytes failed: %s", alloc,
         cudaGetErrorString(err));
  }
  b->bytes = alloc;
  ctx->allocated += alloc;
  context_retain(ctx);
  if (zero) {
    err = cudaMemsetAsync(b->ptr, 0, alloc, ctx->stream);
    if (err != cudaSuccess) {
      buffer_release(b);
      fail(MI_ERR_COMMAND, "cudaMemsetAsync failed: %s", cudaGetErrorString(err));
    }
  }
  auto* t = new mi_tensor();
  t->buf = b;
  t->shape = shape;
  t->dtype = dtype;
  return t;
}

mi_tensor* view(const mi_tensor* t, const std::vector<size_t>& shape, size_t extra_offset) {
  auto* v = new mi_tensor();
  v->buf = t->buf;
  t->buf->refs.fetch_add(1);
  v->offset = t->offset + extra_offset;
  v->shape = shape;
  v->dtype = t->dtype;
  return v;
}

void* context_scratch(mi_context* ctx, size_t bytes) {
  if (bytes > ctx->scratch_bytes) {
    if (ctx->scratch) MI_CUDA(cudaFreeAsync(ctx->scratch, ctx->stream));
    size_t alloc = std::max<size_t>(bytes, 1 << 20);
    MI_CUDA(cudaMallocAsync(&ctx->scratch, alloc, ctx->stream));
    ctx->scratch_bytes = alloc;
  }
  return ctx->scratch;
}

void sync_context(mi_context* ctx) { MI_CUDA(cudaStreamSynchronize(ctx->stream)); }

unsigned take_device_wait_status() {
  unsigned code = k::gemm_tc_status(true);
  if (unsigned g = k::gemv_status(true)) code = code ? code : g;
  if (unsigned a = k::attention_status(true)) code = code ? code : a;
  if (unsigned d = k::decode_loop_status(true)) code = code ? code : d;
  return code;
}

void check_device_waits(const char* what) {
  if (unsigned code = take_device_wait_status())
    fail(MI_ERR_TIMEOUT, "%s: a bounded device wait expired (code 0x%x); the results are not valid",
         what, code);
}

ProfileScope::ProfileScope(mi_context* c, const char* n) : ctx(c), name(n) {
  if (!ctx || !ctx->profiling) return;
  cudaStreamCaptureStatus cs;
  if (cudaStreamIsCapturing(ctx->stream, &cs) != cudaSuccess ||
      cs != cudaStreamCaptureStatusNone)
    return;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, ctx->stream);
}

ProfileScope::~ProfileScope() {
  if (!a) return;
  cudaEventRecord(b, ctx->stream);
  ctx->pending_profiles.push_back({name, a, b});
}

namespace {

void resolve_profiles(mi_context* ctx) {
  for (auto& p : ctx->pending_profiles) {
    float ms = 0.f;
    cudaEventSynchronize(p.stop);
    cudaEventElapsedTime(&ms, p.start, p.stop);
    mi_kernel_profile kp{};
    snprintf(kp.kernel, sizeof kp.kernel, "%s", p.kernel.c_str());
    kp.gpu_time = ms * 1e-3;
    ctx->profiles.push_back(kp);
    cudaEventDestroy(p.start);
    cudaEventDestroy(p.stop);
  }
  ctx->pending_profiles.clear();
}

std::vector<size_t> shape_of(const size_t* shape, size_t rank) {
  MI_REQUIRE(rank == 0 || shape, MI_ERR_INVALID_ARGUMENT, "shape is NULL");
  return std::vector<size_t>(shape, shape + rank);
}

size_t count_of(const std::vector<size_t>& s) {
  size_t n = 1;
  for (size_t d : s) n *= d;
  return n;
}

mi_tensor* upload(mi_context* ctx, const void* host, size_t bytes, const std::vector<size_t>& s,
                  mi_dtype dtype) {
  mi_tensor* t = new_tensor(ctx, s, dtype);
  if (bytes) {
    cudaError_t err = cudaMemcpyAsync(t->base(), host, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(ctx->stream);
    if (err != cudaSuccess) {
      mi_tensor_release(t);
      fail(MI_ERR_COMMAND, "upload failed: %s", cudaGetErrorString(err));
    }
  }
  return t;
}

void require_ctx(const void* p, const char* what) {
  MI_REQUIRE(p != nullptr, MI_ERR_INVALID_ARGUMENT, "%s is NULL", what);
}

// Round-to-nearest-even FP32 -> FP16 on the host.
uint16_t host_f16(float v) {
  __half h = __float2half_rn(v);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

}  // namespace
}  // namespace mi

using namespace mi;

extern "C" {

const char* mi_last_error_message(void) { return mi::g_error.c_str(); }

const char* mi_version(void) { return "metal-infer-b200 0.1.0 (sm_100a)"; }

mi_status mi_context_create(int device, mi_context** out) {
  return guard([&] {
    require_ctx(out, "out");
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
      fail(MI_ERR_NO_DEVICE, "no CUDA device is available");
    MI_REQUIRE(device >= 0 && device < count, MI_ERR_NO_DEVICE, "device %d out of range (%d)",
               device, count);
    MI_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    MI_CUDA(cudaGetDeviceProperties(&prop, device));
    MI_REQUIRE(prop.major == 10, MI_ERR_NO_DEVICE,
               "device %s is sm_%d%d; this build targets sm_100a", prop.name, prop.major,
               prop.minor);
    auto* ctx = new mi_context();
    ctx->device = device;
    ctx->name = prop.name;
    ctx->sm_count = prop.multiProcessorCount;
    cudaError_t err = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) {
      delete ctx;
      fail(MI_ERR_RESOURCE, "stream creation failed: %s", cudaGetErrorString(err));
    }
    // Keep freed stream-ordered memory in the pool (no release to the OS
    // between steps).
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      uint64_t threshold = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    *out = ctx;
  });
}

void mi_context_destroy(mi_context* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  resolve_profiles(ctx);
  context_release(ctx);
}

mi_status mi_context_device_name(const mi_context* ctx, char* buf, size_t len) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(buf, "buf");
    MI_REQUIRE(len > 0, MI_ERR_INVALID_ARGUMENT, "buffer length is 0");
    snprintf(buf, len, "%s", ctx->name.c_str());
  });
}

size_t mi_context_allocated_bytes(const mi_context* ctx) { return ctx ? ctx->allocated : 0; }

mi_status mi_context_set_matmul_backend(mi_context* ctx, mi_matmul_backend b) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    MI_REQUIRE(b != MI_MATMUL_MPS, MI_ERR_UNSUPPORTED,
               "the MPS matmul backend has no CUDA counterpart");
    MI_REQUIRE(b >= MI_MATMUL_AUTO && b <= MI_MATMUL_NATIVE, MI_ERR_INVALID_ARGUMENT,
               "unknown matmul backend %d", (int)b);
    ctx->backend = b;
  });
}

mi_matmul_backend mi_context_matmul_backend(const mi_context* ctx) {
  return ctx ? ctx->backend : MI_MATMUL_AUTO;
}

mi_status mi_context_set_kernel_profiling(mi_context* ctx, int enabled) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    ctx->profiling = enabled != 0;
  });
}

mi_status mi_context_take_kernel_profiles(mi_context* ctx, mi_kernel_profile* out,
                                          size_t capacity, size_t* count) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(count, "count");
    resolve_profiles(ctx);
    size_t n = std::min(capacity, ctx->profiles.size());
    if (out)
      for (size_t i = 0; i < n; ++i) out[i] = ctx->profiles[i];
    *count = out ? n : ctx->profiles.size();
    if (out) ctx->profiles.erase(ctx->profiles.begin(), ctx->profiles.begin() + n);
  });
}

mi_status mi_context_synchronize(mi_context* ctx) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    sync_context(ctx);
  });
}

void* mi_context_stream(mi_context* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

mi_status mi_context_kernel_status(mi_context* ctx, uint32_t* code) {
  mi_status st = guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(code, "code");
    sync_context(ctx);
    *code = take_device_wait_status();
  });
  if (st == MI_OK && *code != 0) {
    set_error("a bounded device wait expired (code %u)", *code);
    return MI_ERR_TIMEOUT;
  }
  return st;
}

// ---- tensors -----------------------------------------------------------------

mi_status mi_context_empty(mi_context* ctx, const size_t* shape, size_t rank, mi_dtype dtype,
                           mi_tensor** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    MI_REQUIRE(dtype >= MI_F16 && dtype <= MI_U32, MI_ERR_INVALID_ARGUMENT, "unknown dtype");
    *out = new_tensor(ctx, shape_of(shape, rank), dtype, true);
  });
}

mi_status mi_context_tensor_f16(mi_context* ctx, const float* values, size_t count,
                                const size_t* shape, size_t rank, mi_tensor** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    auto s = shape_of(shape, rank);
    size_t n = count_of(s);
    if (n != count) fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu", count, n);
    MI_REQUIRE(n == 0 || values, MI_ERR_INVALID_ARGUMENT, "values is NULL");
    std::vector<uint16_t> bits(n);
    for (size_t i = 0; i < n; ++i) bits[i] = host_f16(values[i]);
    *out = upload(ctx, bits.data(), n * 2, s, MI_F16);
  });
}

mi_status mi_context_tensor_f16_bits(mi_context* ctx, const uint16_t* bits, size_t count,
                                     const size_t* shape, size_t rank, mi_tensor** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    auto s = shape_of(shape, rank);
    size_t n = count_of(s);
    if (n != count) fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu", count, n);
    MI_REQUIRE(n == 0 || bits, MI_ERR_INVALID_ARGUMENT, "bits is NULL");
    *out = upload(ctx, bits, n * 2, s, MI_F16);
  });
}

mi_status mi_context_tensor_f16_bytes(mi_context* ctx, const uint8_t* bytes, size_t nbytes,
                                      const size_t* shape, size_t rank, mi_tensor** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    auto s = shape_of(shape, rank);
    size_t n = count_of(s);
    if (nbytes != n * 2)
      fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu", nbytes / 2, n);
    *out = upload(ctx, bytes, nbytes, s, MI_F16);
  });
}

mi_status mi_context_tensor_bf16_as_f16_bytes(mi_context* ctx, const uint8_t* bytes,
                                              size_t nbytes, const size_t* shape, size_t rank,
                                              mi_tensor** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    auto s = shape_of(shape, rank);
    size_t n = count_of(s);
    if (nbytes != n * 2)
      fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu", nbytes / 2, n);
    std::vector<uint16_t> bits(n);
    for (size_t i = 0; i < n; ++i) {
      uint32_t w = (uint32_t(bytes[2 * i]) | (uint32_t(bytes[2 * i + 1]) << 8)) << 16;
      float v;
      std::memcpy(&v, &w, 4);
      bits[i] = host_f16(v);
    }
    *out = upload(ctx, bits.data(), n * 2, s, MI_F16);
  });
}

mi_status mi_context_tensor_u32(mi_context* ctx, const uint32_t* values, size_t count,
                                const size_t* shape, size_t rank, mi_tensor** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    auto s = shape_of(shape, rank);
    size_t n = count_of(s);
    if (n != count) fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu", count, n);
    *out = upload(ctx, values, n * 4, s, MI_U32);
  });
}

mi_status mi_context_tensor_from_device(mi_context* ctx, void* device_ptr, const size_t* shape,
                                        size_t rank, mi_dtype dtype, mi_tensor** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    require_ctx(device_ptr, "device_ptr");
    auto* b = new Buffer();
    b->ctx = ctx;
    b->ptr = device_ptr;
    b->owned = false;
    context_retain(ctx);
    auto* t = new mi_tensor();
    t->buf = b;
    t->shape = shape_of(shape, rank);
    t->dtype = dtype;
    b->bytes = t->bytes();
    *out = t;
  });
}

mi_status mi_tensor_clone(const mi_tensor* t, mi_tensor** out) {
  return guard([&] {
    require_ctx(t, "tensor");
    require_ctx(out, "out");
    *out = view(t, t->shape, 0);
  });
}

void mi_tensor_release(mi_tensor* t) {
  if (!t) return;
  buffer_release(t->buf);
  delete t;
}

size_t mi_tensor_rank(const mi_tensor* t) { return t ? t->shape.size() : 0; }

size_t mi_tensor_shape(const mi_tensor* t, size_t* shape, size_t capacity) {
  if (!t) return 0;
  for (size_t i = 0; i < t->shape.size() && i < capacity; ++i) shape[i] = t->shape[i];
  return t->shape.size();
}

mi_dtype mi_tensor_dtype(const mi_tensor* t) { return t ? t->dtype : MI_F16; }
size_t mi_tensor_len(const mi_tensor* t) { return t ? t->len() : 0; }
size_t mi_tensor_byte_len(const mi_tensor* t) { return t ? t->bytes() : 0; }
void* mi_tensor_device_ptr(const mi_tensor* t) { return t ? t->base() : nullptr; }

// Tensor::reshape (tensor.rs:108-131)
mi_status mi_tensor_reshape(const mi_tensor* t, const size_t* shape, size_t rank,
                            mi_tensor** out) {
  return guard([&] {
    require_ctx(t, "tensor");
    require_ctx(out, "out");
    auto s = shape_of(shape, rank);
    size_t n = 1;
    bool zero = false;
    for (size_t d : s) {
      if (d == 0) zero = true;
      MI_REQUIRE(d == 0 || n <= SIZE_MAX / d, MI_ERR_SHAPE, "reshape element count overflow");
      n *= d;
    }
    if (s.empty() || zero || n != t->len()) fail(MI_ERR_SHAPE, "cannot reshape tensor");
    *out = view(t, s, 0);
  });
}

// Tensor::prefix (tensor.rs:133-157)
mi_status mi_tensor_prefix(const mi_tensor* t, size_t first, mi_tensor** out) {
  return guard([&] {
    require_ctx(t, "tensor");
    require_ctx(out, "out");
    MI_REQUIRE(!t->shape.empty(), MI_ERR_SHAPE, "prefix requires rank >= 1");
    MI_REQUIRE(first != 0 && first <= t->shape[0], MI_ERR_SHAPE,
               "prefix %zu is outside capacity %zu", first, t->shape[0]);
    auto s = t->shape;
    s[0] = first;
    *out = view(t, s, 0);
  });
}

// Tensor::row (tensor.rs:159-182)
mi_status mi_tensor_row(const mi_tensor* t, size_t row, mi_tensor** out) {
  return guard([&] {
    require_ctx(t, "tensor");
    require_ctx(out, "out");
    MI_REQUIRE(t->shape.size() == 2 && row < t->shape[0], MI_ERR_SHAPE,
               "row %zu is outside the matrix", row);
    *out = view(t, {1, t->shape[1]}, row * t->shape[1] * dtype_size(t->dtype));
  });
}

// Tensor::slice_1d (tensor.rs:184-207)
mi_status mi_tensor_slice_1d(const mi_tensor* t, size_t start, size_t len, mi_tensor** out) {
  return guard([&] {
    require_ctx(t, "tensor");
    require_ctx(out, "out");
    MI_REQUIRE(t->shape.size() == 1, MI_ERR_SHAPE, "slice_1d requires a rank-1 tensor");
    MI_REQUIRE(start <= SIZE_MAX - len, MI_ERR_SHAPE, "slice_1d range overflow");
    MI_REQUIRE(len != 0 && start + len <= t->shape[0], MI_ERR_SHAPE,
               "slice_1d range %zu..%zu is outside [%zu]", start, start + len, t->shape[0]);
    *out = view(t, {len}, start * dtype_size(t->dtype));
  });
}

namespace {
void download(const mi_tensor* t, void* out, size_t bytes) {
  mi_context* ctx = t->buf->ctx;
  MI_CUDA(cudaMemcpyAsync(out, t->base(), bytes, cudaMemcpyDeviceToHost, ctx->stream));
  MI_CUDA(cudaStreamSynchronize(ctx->stream));
}
}  // namespace

mi_status mi_tensor_f16_bits(const mi_tensor* t, uint16_t* out, size_t count) {
  return guard([&] {
    require_ctx(t, "tensor");
    if (t->dtype != MI_F16) fail(MI_ERR_DTYPE, "unsupported dtype: expected f16, got %s",
                                 dtype_name(t->dtype));
    if (count != t->len()) fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu",
                                count, t->len());
    download(t, out, t->bytes());
  });
}

mi_status mi_tensor_to_f32(const mi_tensor* t, float* out, size_t count) {
  return guard([&] {
    require_ctx(t, "tensor");
    if (count != t->len()) fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu",
                                count, t->len());
    if (t->dtype == MI_F32) {
      download(t, out, t->bytes());
    } else if (t->dtype == MI_F16) {
      std::vector<__half> tmp(count);
      download(t, tmp.data(), t->bytes());
      for (size_t i = 0; i < count; ++i) out[i] = __half2float(tmp[i]);
    } else {
      fail(MI_ERR_DTYPE, "unsupported dtype: expected f16 or f32, got u32");
    }
  });
}

mi_status mi_tensor_to_u32(const mi_tensor* t, uint32_t* out, size_t count) {
  return guard([&] {
    require_ctx(t, "tensor");
    if (t->dtype != MI_U32) fail(MI_ERR_DTYPE, "unsupported dtype: expected u32, got %s",
                                 dtype_name(t->dtype));
    if (count != t->len()) fail(MI_ERR_DATA_LENGTH, "host data has %zu elements, expected %zu",
                                count, t->len());
    download(t, out, t->bytes());
  });
}

mi_status mi_tensor_write(mi_tensor* t, const void* host, size_t nbytes) {
  return guard([&] {
    require_ctx(t, "tensor");
    if (nbytes != t->bytes()) fail(MI_ERR_DATA_LENGTH, "host data has %zu bytes, expected %zu",
                                   nbytes, t->bytes());
    mi_context* ctx = t->buf->ctx;
    MI_CUDA(cudaMemcpyAsync(t->base(), host, nbytes, cudaMemcpyHostToDevice, ctx->stream));
    MI_CUDA(cudaStreamSynchronize(ctx->stream));
  });
}

// ---- batches -------------------------------------------------------------------

mi_status mi_context_begin_batch(mi_context* ctx, mi_batch** out) {
  return guard([&] {
    require_ctx(ctx, "ctx");
    require_ctx(out, "out");
    auto* b = new mi_batch();
    b->ctx = ctx;
    context_retain(ctx);
    cudaError_t err = cudaEventCreate(&b->start);
    if (err == cudaSuccess) err = cudaEventRecord(b->start, ctx->stream);
    if (err != cudaSuccess) {
      mi_batch_abandon(b);
      fail(MI_ERR_COMMAND, "batch creation failed: %s", cudaGetErrorString(err));
    }
    b->wall_start = std::chrono::steady_clock::now();
    *out = b;
  });
}

mi_status mi_batch_commit(mi_batch* b, mi_pending** out) {
  return guard([&] {
    require_ctx(b, "batch");
    require_ctx(out, "out");
    auto* p = new mi_pending();
    p->ctx = b->ctx;
    p->start = b->start;
    p->wall_start = b->wall_start;
    b->start = nullptr;
    delete b;
    cudaError_t err = cudaEventCreate(&p->stop);
    if (err == cudaSuccess) err = cudaEventRecord(p->stop, p->ctx->stream);
    if (err != cudaSuccess) {
      cudaEventDestroy(p->start);
      context_release(p->ctx);
      delete p;
      fail(MI_ERR_COMMAND, "commit failed: %s", cudaGetErrorString(err));
    }
    *out = p;
  });
}

mi_status mi_pending_wait(mi_pending* p, mi_dispatch_stats* stats) {
  return guard([&] {
    require_ctx(p, "pending");
    cudaError_t err = cudaEventSynchronize(p->stop);
    float ms = 0.f;
    if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, p->start, p->stop);
    auto wall = std::chrono::steady_clock::now() - p->wall_start;
    cudaEventDestroy(p->start);
    cudaEventDestroy(p->stop);
    context_release(p->ctx);
    delete p;
    if (err != cudaSuccess) fail(MI_ERR_COMMAND, "command failed: %s", cudaGetErrorString(err));
    check_device_waits("batch");
    if (stats) {
      stats->gpu_time = ms * 1e-3;
      stats->wall_time = std::chrono::duration<double>(wall).count();
    }
  });
}

int mi_pending_is_complete(const mi_pending* p) {
  return p && cudaEventQuery(p->stop) == cudaSuccess ? 1 : 0;
}

mi_status mi_batch_finish(mi_batch* b, mi_dispatch_stats* stats) {
  mi_pending* p = nullptr;
  mi_status s = mi_batch_commit(b, &p);
  if (s != MI_OK) return s;
  return mi_pending_wait(p, stats);
}

void mi_batch_abandon(mi_batch* b) {
  if (!b) return;
  if (b->start) cudaEventDestroy(b->start);
  mi_context* ctx = b->ctx;
  delete b;
  context_release(ctx);
}

}  // extern "C"
