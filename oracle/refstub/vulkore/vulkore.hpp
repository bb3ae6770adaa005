// CPU stand-in for the reference runtime's public headers (include/vulkore/*),
// written for the checker only. The reference's Vulkan runtime cannot build
// here (its third_party submodules are empty and there is no graphics stack),
// so its host engine (examples/llm/decode.cpp) is compiled against THIS header
// instead: Buffer is host memory, Program::kernel resolves names in the
// checker's kernel table (ref_kernels.cpp), and Batch::add runs the kernel
// over its global grid immediately, which is the same ordering a Batch's
// COMPUTE->COMPUTE barriers guarantee (include/vulkore/launch.hpp:165-213).
// Mirrors only the API surface decode.cpp uses. Test infrastructure only.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "../../ref_kernels.h"

namespace vulkore {

class Error : public std::runtime_error {
 public:
  explicit Error(const std::string& m) : std::runtime_error(m) {}
};

enum class Usage { DeviceLocal, HostVisible };

struct Grid { uint32_t x = 1, y = 1, z = 1; };

class Context;

class Buffer {
 public:
  Buffer() = default;
  size_t size_bytes() const { return mem_ ? mem_->size() * 16 : 0; }
  bool valid() const { return (bool)mem_; }
  bool host_visible() const { return true; }
  void* data() const { return mem_ ? (void*)mem_->data() : nullptr; }
  template <typename T> void upload(std::span<const T> d, size_t off = 0) {
    upload_bytes(d.data(), d.size_bytes(), off);
  }
  template <typename T> void upload(std::span<T> d, size_t off = 0) {
    upload_bytes(d.data(), d.size_bytes(), off);
  }
  template <typename T> void download(std::span<T> out, size_t off = 0) const {
    download_bytes(out.data(), out.size_bytes(), off);
  }
  void upload_bytes(const void* src, size_t n, size_t off = 0) {
    if (off + n > bytes_) throw Error("refstub: upload out of range");
    std::memcpy((char*)data() + off, src, n);
  }
  void download_bytes(void* dst, size_t n, size_t off = 0) const {
    if (off + n > bytes_) throw Error("refstub: download out of range");
    std::memcpy(dst, (const char*)data() + off, n);
  }

 private:
  friend class Context;
  struct alignas(16) Chunk { unsigned char b[16]; };
  std::shared_ptr<std::vector<Chunk>> mem_;
  size_t bytes_ = 0;
};

class Context {
 public:
  Context() = default;
  const std::string& device_name() const { static std::string n = "refstub-cpu"; return n; }
  template <typename T> Buffer alloc(size_t count, Usage = Usage::DeviceLocal) {
    static_assert(sizeof(T) % 4 == 0, "storage buffer element types should be 4-byte aligned");
    return alloc_bytes(count * sizeof(T), Usage::DeviceLocal);
  }
  Buffer alloc_bytes(size_t n, Usage) {
    Buffer b;
    b.mem_ = std::make_shared<std::vector<Buffer::Chunk>>((n + 15) / 16 + 1);
    std::memset(b.mem_->data(), 0, b.mem_->size() * 16);
    b.bytes_ = n;
    return b;
  }
  void wait_idle() {}
};

class Kernel {
 public:
  Kernel() = default;
  bool valid() const { return id_ >= 0; }
  const std::string& name() const { return name_; }
  int id() const { return id_; }
 private:
  friend class Program;
  int id_ = -1;
  std::string module_, name_;
  friend class Batch;
};

class Program {
 public:
  static Program from_file(Context&, const std::string& path) {
    Program p;
    p.module_ = path;
    return p;
  }
  Kernel kernel(const std::string& name) {
    int id = xpref_find(module_.c_str(), name.c_str());
    if (id < 0) {
      std::string avail;
      for (const auto& n : kernel_names()) avail += (avail.empty() ? "" : ", ") + n;
      throw Error("vulkore::Program: no kernel named '" + name + "' (module has: " + avail + ")");
    }
    Kernel k;
    k.id_ = id;
    k.module_ = module_;
    k.name_ = name;
    return k;
  }
  std::vector<std::string> kernel_names() const {
    std::vector<std::string> out;
    for (int i = 0; i < xpref_count(); ++i) {
      const char* m; const char* n;
      xpref_kernel_info(i, &m, &n, nullptr, nullptr, nullptr);
      if (xpref_find(module_.c_str(), n) == i) out.emplace_back(n);
    }
    return out;
  }
 private:
  std::string module_;
};

class Fence {
 public:
  bool wait(uint64_t = UINT64_MAX) const { return true; }
  bool is_signaled() const { return true; }
};

class DescriptorCache {
 public:
  explicit DescriptorCache(Context&) {}
  void clear() noexcept {}
};

namespace detail {
struct Arg {
  xpref_arg a{};
  unsigned char pod[16];
};
template <typename T> Arg make(const T& v) {
  Arg r;
  using U = std::remove_cvref_t<T>;
  if constexpr (std::is_same_v<U, Buffer>) {
    r.a = xpref_arg{v.data(), 0, 1};
  } else {
    static_assert(std::is_trivially_copyable_v<U> && sizeof(U) <= 16, "POD arg");
    std::memcpy(r.pod, &v, sizeof(U));
    r.a = xpref_arg{nullptr, (uint32_t)sizeof(U), 0};
  }
  return r;
}
inline void run(const Kernel& k, Grid g, Arg* args, size_t n) {
  if (!k.valid()) throw Error("vulkore::launch: empty Kernel handle");
  if (g.x == 0 || g.y == 0 || g.z == 0) throw Error("vulkore::launch: grid must be nonzero");
  std::vector<xpref_arg> a(n);
  for (size_t i = 0; i < n; ++i) {
    a[i] = args[i].a;
    if (!a[i].is_buffer) a[i].ptr = args[i].pod;
  }
  const char* m; const char* name;
  xpref_kernel_info(k.id(), &m, &name, nullptr, nullptr, nullptr);
  int rc = xpref_launch(m, name, g.x * g.y * g.z, a.data(), (uint32_t)n, 0);
  if (rc != 0) throw Error(std::string("vulkore::launch('") + name + "'): " + xpref_last_error());
}
}  // namespace detail

class Batch {
 public:
  explicit Batch(Context&) {}
  Batch(Context&, DescriptorCache&) {}
  template <typename... Args> Batch& add(const Kernel& k, Grid g, const Args&... args) {
    detail::Arg a[] = {detail::make(args)..., detail::Arg{}};
    detail::run(k, g, a, sizeof...(Args));
    ++n_;
    return *this;
  }
  Fence submit() { return Fence{}; }
  size_t size() const noexcept { return n_; }
 private:
  size_t n_ = 0;
};

template <typename... Args> Fence launch(const Kernel& k, Grid g, const Args&... args) {
  detail::Arg a[] = {detail::make(args)..., detail::Arg{}};
  detail::run(k, g, a, sizeof...(Args));
  return Fence{};
}

}  // namespace vulkore
