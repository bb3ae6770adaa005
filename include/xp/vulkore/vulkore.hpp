// vulkore::{Context, Buffer, Program, Kernel, launch, Batch, Fence,
// DescriptorCache} implemented over the C ABI of libxp_cuda.so.
//
// The C++ side of the drop-in: code written against the reference runtime's
// public headers (include/vulkore/{context,buffer,program,launch,sync}.hpp) --
// in particular examples/llm/decode.cpp's DecodeSession -- compiles unchanged
// with `-I <this repo>/include/xp` in place of the reference's include path and
// links against libxp_cuda.so. Kernels resolve by (module path, name) in the
// library's registry; a Batch is one CUDA graph; a Fence is a CUDA event.
// Errors throw vulkore::Error carrying the library's message.
//
// Covers the API surface the reference's LLM engine uses. Not thread-safe per
// Context (the reference's Context is single-threaded too).
#pragma once
#include <array>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <optional>
#include <span>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "../../xp_cuda.h"

#ifndef VK_VERSION_1_0
// Vulkan's byte-size type, used by callers of the reference's buffer API
// (include/vulkore/buffer.hpp) for offsets and sizes.
typedef uint64_t VkDeviceSize;
#endif

namespace vulkore {

class Error : public std::runtime_error {
 public:
  explicit Error(const std::string& m) : std::runtime_error(m) {}
};

namespace detail {
inline void check(xp_status s) {
  if (s != XP_OK && s != XP_TIMEOUT) throw Error(std::string(xp_status_name(s)) + ": " + xp_last_error());
}
}  // namespace detail

enum class Usage { DeviceLocal, HostVisible };

struct Grid {
  uint32_t x = 1, y = 1, z = 1;
};

class Context;

class Buffer {
 public:
  Buffer() = default;
  size_t size_bytes() const { return st_ ? st_->bytes : 0; }
  bool valid() const { return st_ && st_->dptr; }
  bool host_visible() const { return st_ && st_->host; }
  void* device_ptr() const { return st_ ? st_->dptr : nullptr; }

  template <typename T> void upload(std::span<const T> d, size_t off = 0) { upload_bytes(d.data(), d.size_bytes(), off); }
  template <typename T> void upload(std::span<T> d, size_t off = 0) { upload_bytes(d.data(), d.size_bytes(), off); }
  template <typename T> void download(std::span<T> out, size_t off = 0) const {
    download_bytes(out.data(), out.size_bytes(), off);
  }
  void upload_bytes(const void* src, size_t n, size_t off = 0) {
    if (!valid() || off + n > st_->bytes) throw Error("vulkore::Buffer::upload: out of range");
    detail::check(xp_upload(st_->ctx, st_->dptr, off, src, n));
  }
  void download_bytes(void* dst, size_t n, size_t off = 0) const {
    if (!valid() || off + n > st_->bytes) throw Error("vulkore::Buffer::download: out of range");
    detail::check(xp_download(st_->ctx, dst, st_->dptr, off, n));
  }

 private:
  friend class Context;
  struct State {
    xp_context* ctx = nullptr;
    void* dptr = nullptr;
    void* host = nullptr;
    size_t bytes = 0;
    ~State() {
      if (ctx && dptr) xp_free(ctx, dptr);
    }
  };
  std::shared_ptr<State> st_;
};

class Context {
 public:
  explicit Context(std::optional<uint32_t> device_index = std::nullopt) {
    detail::check(xp_context_create(device_index ? (int)*device_index : 0, &ctx_));
    char buf[256];
    if (xp_context_device_name(ctx_, buf, sizeof buf) == XP_OK) name_ = buf;
  }
  ~Context() { xp_context_destroy(ctx_); }
  Context(const Context&) = delete;
  Context& operator=(const Context&) = delete;

  const std::string& device_name() const { return name_; }
  xp_context* handle() const { return ctx_; }

  template <typename T> Buffer alloc(size_t count, Usage usage) {
    static_assert(sizeof(T) % 4 == 0, "storage buffer element types should be 4-byte aligned");
    return alloc_bytes(count * sizeof(T), usage);
  }
  template <typename T> Buffer alloc(size_t count) { return alloc<T>(count, Usage::DeviceLocal); }
  Buffer alloc_bytes(size_t n, Usage usage) {
    Buffer b;
    b.st_ = std::make_shared<Buffer::State>();
    b.st_->ctx = ctx_;
    b.st_->bytes = n;
    detail::check(xp_alloc(ctx_, n ? n : 4, usage == Usage::HostVisible ? XP_HOST_VISIBLE : XP_DEVICE_LOCAL,
                           &b.st_->dptr, &b.st_->host));
    return b;
  }
  void wait_idle() { detail::check(xp_context_wait_idle(ctx_)); }

 private:
  xp_context* ctx_ = nullptr;
  std::string name_;
};

class Kernel {
 public:
  Kernel() = default;
  bool valid() const { return id_ >= 0; }
  const std::string& name() const { return name_; }
  xp_kernel id() const { return id_; }
  // The reference's workgroup size query (include/vulkore/program.hpp:76):
  // a Grid counts global threads, rounded up to groups of 64; the kernels
  // here choose their own CTA shapes, so 64 is the grouping callers see.
  std::array<uint32_t, 3> local_size() const { return {64u, 1u, 1u}; }
  Context& context() const { return *ctx_; }

 private:
  friend class Program;
  xp_kernel id_ = -1;
  std::string name_;
  Context* ctx_ = nullptr;
};

class Program {
 public:
  static Program from_file(Context& ctx, const std::string& path) {
    Program p;
    p.ctx_ = &ctx;
    p.module_ = path;
    return p;
  }
  // Unknown name: throws, and the message lists the module's kernels.
  Kernel kernel(const std::string& name) {
    Kernel k;
    detail::check(xp_kernel_lookup(module_.c_str(), name.c_str(), &k.id_));
    k.name_ = name;
    k.ctx_ = ctx_;
    return k;
  }
  std::vector<std::string> kernel_names() const {
    std::vector<std::string> out;
    const std::string base = module_.substr(module_.find_last_of('/') + 1);
    for (int i = 0; i < xp_kernel_count(); ++i) {
      const char* m;
      const char* n;
      uint32_t na;
      if (xp_kernel_info(i, &m, &n, &na) != XP_OK) continue;
      const std::string mm(m);
      if (mm.substr(mm.find_last_of('/') + 1) == base) out.emplace_back(n);
    }
    return out;
  }

 private:
  Context* ctx_ = nullptr;
  std::string module_;
};

class Fence {
 public:
  Fence() = default;  // empty fence: wait() returns true
  explicit Fence(xp_fence* f) : f_(f, &xp_fence_destroy) {}
  // true when signaled, false on timeout; throws on a device error
  bool wait(uint64_t timeout_ns = UINT64_MAX) const {
    if (!f_) return true;
    const xp_status s = xp_fence_wait(f_.get(), timeout_ns);
    if (s == XP_TIMEOUT) return false;
    detail::check(s);
    return true;
  }
  bool is_signaled() const { return wait(0); }

 private:
  std::shared_ptr<xp_fence> f_;
};

// Descriptor sets do not exist here; kept so callers that cache them compile.
class DescriptorCache {
 public:
  explicit DescriptorCache(Context&) {}
  void clear() noexcept {}
  size_t size() const noexcept { return 0; }
};

namespace detail {
struct Packed {
  xp_arg a{};
  unsigned char pod[16];
};
template <typename T> Packed pack(const T& v) {
  Packed p;
  using U = std::remove_cvref_t<T>;
  if constexpr (std::is_same_v<U, Buffer>) {
    p.a = xp_arg{v.device_ptr(), 0, 1};
  } else {
    static_assert(!std::is_pointer_v<U>, "vulkore::launch: pass a vulkore::Buffer for global memory");
    static_assert(std::is_trivially_copyable_v<U> && sizeof(U) <= 16, "vulkore::launch: POD argument");
    std::memcpy(p.pod, &v, sizeof(U));
    p.a = xp_arg{nullptr, (uint32_t)sizeof(U), 0};
  }
  return p;
}
template <typename... Args> std::vector<xp_arg> args(std::vector<Packed>& store, const Args&... a) {
  store = {pack(a)...};
  std::vector<xp_arg> out(store.size());
  for (size_t i = 0; i < store.size(); ++i) {
    out[i] = store[i].a;
    if (!out[i].kind) out[i].ptr = store[i].pod;
  }
  return out;
}
}  // namespace detail

// Validates the arguments against the kernel's signature, enqueues it on the
// context's stream and returns a Fence for it.
template <typename... Args> Fence launch(Kernel& k, Grid g, const Args&... a) {
  std::vector<detail::Packed> store;
  auto v = detail::args(store, a...);
  xp_context* c = k.context().handle();
  detail::check(xp_launch(k.id(), xp_grid{g.x, g.y, g.z}, v.data(), (uint32_t)v.size(), xp_context_stream(c)));
  xp_fence* f = nullptr;
  detail::check(xp_context_fence(c, &f));
  return Fence(f);
}

// Many launches, one submission: recorded, then captured into one CUDA graph.
class Batch {
 public:
  explicit Batch(Context& ctx) { detail::check(xp_batch_create(ctx.handle(), &b_)); }
  Batch(Context& ctx, DescriptorCache&) : Batch(ctx) {}
  ~Batch() { xp_batch_destroy(b_); }
  Batch(const Batch&) = delete;
  Batch& operator=(const Batch&) = delete;
  template <typename... Args> Batch& add(Kernel& k, Grid g, const Args&... a) {
    std::vector<detail::Packed> store;
    auto v = detail::args(store, a...);
    detail::check(xp_batch_add(b_, k.id(), xp_grid{g.x, g.y, g.z}, v.data(), (uint32_t)v.size()));
    ++n_;
    return *this;
  }
  Fence submit() {
    xp_fence* f = nullptr;
    detail::check(xp_batch_submit(b_, &f));
    return Fence(f);
  }
  size_t size() const noexcept { return n_; }

 private:
  xp_batch* b_ = nullptr;
  size_t n_ = 0;
};

}  // namespace vulkore
