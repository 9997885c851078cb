// Minimal eager stand-in for the slice of the MLX C++ API that the reference
// operators' CPU code paths (`eval_cpu`, the op front-ends and the intersect
// staging helpers) touch.  TEST INFRASTRUCTURE ONLY: it exists so that the
// reference's own `gsplat_core/*.cpp` can be compiled unmodified, in place,
// into `oracle/_ref/libgsplat_ref.so`, which pins the C restatement in
// `oracle/gsplat_oracle.c` and generates the golden fixtures.
//
// Semantics kept from MLX where the reference depends on them:
//   * arrays are ref-counted handles; copies alias the same buffer;
//   * `array::make_arrays` / the primitive-taking constructor build the
//     outputs of one primitive -- here they are evaluated immediately with
//     `Primitive::eval_cpu` (eager), so `mx::eval` is a no-op;
//   * `cumsum(a, reverse=false, inclusive=false)` is an exclusive scan;
//   * `argsort` is stable (std::stable_sort) and returns uint32 indices;
//     MLX's CPU argsort is also a stable sort, but it is not this code.
// Everything the reference does not use is absent.
//
// Device mode (compiled with -DGSPLAT_SHIM_CUDA, for the GPU test of the
// CUDA eval_gpu adapter only): buffers are CUDA managed memory, a primitive
// on a gpu stream is evaluated with eval_gpu instead of eval_cpu, and the
// host-side ops (reshape, cumsum, argsort, take) and `eval` first wait for
// the device, as MLX's eval does before the host reads a result.
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <numeric>
#include <stdexcept>
#include <string>
#include <utility>
#include <variant>
#include <vector>

#ifdef GSPLAT_SHIM_CUDA
#include <cuda_runtime_api.h>
#endif

namespace mlx {
namespace core {

using Shape = std::vector<int32_t>;

struct Dtype {
  enum class Val : uint8_t { bool_, int32, int64, uint32, float32 };
  Val v;
  uint8_t bytes;
  constexpr Val val() const { return v; }
  constexpr size_t size() const { return bytes; }
  constexpr bool operator==(const Dtype& o) const { return v == o.v; }
  constexpr bool operator!=(const Dtype& o) const { return v != o.v; }
};

inline constexpr Dtype bool_{Dtype::Val::bool_, 1};
inline constexpr Dtype int32{Dtype::Val::int32, 4};
inline constexpr Dtype int64{Dtype::Val::int64, 8};
inline constexpr Dtype uint32{Dtype::Val::uint32, 4};
inline constexpr Dtype float32{Dtype::Val::float32, 4};

struct Device {
  enum class DeviceType { cpu, gpu };
  static constexpr DeviceType cpu = DeviceType::cpu;
  static constexpr DeviceType gpu = DeviceType::gpu;
  DeviceType type;
  int index = 0;
  constexpr Device(DeviceType t, int i = 0) : type(t), index(i) {}
};

struct Stream {
  int index;
  Device device;
  Stream(int i, Device d) : index(i), device(d) {}
};

using StreamOrDevice = std::variant<std::monostate, Stream, Device>;

inline Stream to_stream(StreamOrDevice s) {
  if (std::holds_alternative<Stream>(s)) {
    return std::get<Stream>(s);
  }
  if (std::holds_alternative<Device>(s)) {
    return Stream(0, std::get<Device>(s));
  }
  return Stream(0, Device(Device::cpu));
}

namespace detail {
// Waits for the device before a host read (device mode only).
inline void sync() {
#ifdef GSPLAT_SHIM_CUDA
  if (cudaDeviceSynchronize() != cudaSuccess) {
    throw std::runtime_error("shim: device synchronisation failed");
  }
#endif
}
}  // namespace detail

namespace allocator {
struct Buffer {
  void* ptr;
};
inline Buffer malloc(size_t nbytes) {
  // Always hand out a real allocation so that zero-sized arrays still have a
  // valid data pointer, as MLX does.
  const size_t bytes = nbytes == 0 ? 16 : nbytes;
#ifdef GSPLAT_SHIM_CUDA
  void* p = nullptr;
  if (cudaMallocManaged(&p, bytes) != cudaSuccess) {
    p = nullptr;
  }
#else
  void* p = std::malloc(bytes);
#endif
  if (p == nullptr) {
    throw std::runtime_error("shim allocator: out of memory");
  }
  return Buffer{p};
}
inline void free(void* p) {
#ifdef GSPLAT_SHIM_CUDA
  cudaFree(p);
#else
  std::free(p);
#endif
}
}  // namespace allocator

class Primitive;

class array {
 public:
  array() : desc_(std::make_shared<Desc>()) {}

  // Eager construction of the single output of a primitive.
  array(Shape shape,
        Dtype dtype,
        std::shared_ptr<Primitive> prim,
        std::vector<array> inputs);

  static std::vector<array> make_arrays(std::vector<Shape> shapes,
                                        const std::vector<Dtype>& dtypes,
                                        const std::shared_ptr<Primitive>& prim,
                                        const std::vector<array>& inputs);

  // Owning copy of host data (used by the bridge, not by the reference).
  static array from_host(const void* data, Shape shape, Dtype dtype) {
    array a;
    a.desc_->shape = std::move(shape);
    a.desc_->dtype = dtype;
    a.set_data(allocator::malloc(a.nbytes()));
    if (data != nullptr && a.nbytes() != 0) {
      std::memcpy(a.data<void>(), data, a.nbytes());
    }
    return a;
  }

  size_t ndim() const { return desc_->shape.size(); }
  const Shape& shape() const { return desc_->shape; }
  int32_t shape(int dim) const {
    const int n = static_cast<int>(ndim());
    return desc_->shape.at(static_cast<size_t>(dim < 0 ? dim + n : dim));
  }
  size_t size() const {
    size_t n = 1;
    for (auto d : desc_->shape) {
      n *= static_cast<size_t>(d);
    }
    return n;
  }
  size_t nbytes() const { return size() * desc_->dtype.size(); }
  Dtype dtype() const { return desc_->dtype; }
  size_t itemsize() const { return desc_->dtype.size(); }

  template <typename T>
  T* data() {
    return static_cast<T*>(desc_->data.get());
  }
  template <typename T>
  const T* data() const {
    return static_cast<const T*>(desc_->data.get());
  }

  void set_data(allocator::Buffer buf) {
    desc_->data = std::shared_ptr<void>(buf.ptr, [](void* p) { allocator::free(p); });
  }
  void eval() {}

 private:
  struct Desc {
    Shape shape;
    Dtype dtype = float32;
    std::shared_ptr<void> data;
  };
  std::shared_ptr<Desc> desc_;

  void init(Shape shape, Dtype dtype) {
    desc_->shape = std::move(shape);
    desc_->dtype = dtype;
  }
  friend class Primitive;
};

class Primitive {
 public:
  explicit Primitive(Stream stream) : stream_(stream) {}
  virtual ~Primitive() = default;

  virtual void eval_cpu(const std::vector<array>& inputs,
                        std::vector<array>& outputs) = 0;
  virtual void eval_gpu(const std::vector<array>& inputs,
                        std::vector<array>& outputs) = 0;
  virtual std::vector<array> jvp(const std::vector<array>& primals,
                                 const std::vector<array>& tangents,
                                 const std::vector<int>& argnums) = 0;
  virtual std::vector<array> vjp(const std::vector<array>& primals,
                                 const std::vector<array>& cotangents,
                                 const std::vector<int>& argnums,
                                 const std::vector<array>& outputs) = 0;
  virtual std::pair<std::vector<array>, std::vector<int>> vmap(
      const std::vector<array>& inputs,
      const std::vector<int>& axes) = 0;
  virtual const char* name() const = 0;
  virtual bool is_equivalent(const Primitive&) const { return false; }

  Stream& stream() { return stream_; }

  // Eager evaluation: every node runs on the host, whichever stream the
  // front-end asked for.
  static std::vector<array> run(const std::shared_ptr<Primitive>& prim,
                                std::vector<Shape> shapes,
                                const std::vector<Dtype>& dtypes,
                                const std::vector<array>& inputs) {
    std::vector<array> outputs(shapes.size());
    for (size_t i = 0; i < shapes.size(); ++i) {
      outputs[i].init(std::move(shapes[i]), dtypes[i]);
    }
#ifdef GSPLAT_SHIM_CUDA
    if (prim->stream().device.type == Device::gpu) {
      prim->eval_gpu(inputs, outputs);
      return outputs;
    }
    detail::sync();
#endif
    prim->eval_cpu(inputs, outputs);
    return outputs;
  }

 private:
  Stream stream_;
};

inline array::array(Shape shape,
                    Dtype dtype,
                    std::shared_ptr<Primitive> prim,
                    std::vector<array> inputs)
    : array() {
  auto outs = Primitive::run(prim, {std::move(shape)}, {dtype}, inputs);
  desc_ = outs[0].desc_;
}

inline std::vector<array> array::make_arrays(
    std::vector<Shape> shapes,
    const std::vector<Dtype>& dtypes,
    const std::shared_ptr<Primitive>& prim,
    const std::vector<array>& inputs) {
  return Primitive::run(prim, std::move(shapes), dtypes, inputs);
}

template <typename... Arrays>
inline void eval(Arrays&&...) {
  detail::sync();
}

inline array contiguous(const array& a, bool = false, StreamOrDevice = {}) {
  return a;
}

inline array zeros(const Shape& shape, Dtype dtype, StreamOrDevice = {}) {
  array a = array::from_host(nullptr, shape, dtype);
  if (a.nbytes() != 0) {
    std::memset(a.data<void>(), 0, a.nbytes());
  }
  return a;
}

inline array zeros_like(const array& a, StreamOrDevice s = {}) {
  return zeros(a.shape(), a.dtype(), s);
}

inline array reshape(const array& a, Shape shape, StreamOrDevice = {}) {
  detail::sync();
  array out = array::from_host(a.data<void>(), std::move(shape), a.dtype());
  if (out.size() != a.size()) {
    throw std::runtime_error("shim reshape: size mismatch");
  }
  return out;
}

// Flattened scan over an int32 vector; only the forms the reference uses.
inline array cumsum(const array& a, bool reverse, bool inclusive,
                    StreamOrDevice = {}) {
  if (a.dtype() != int32 || reverse) {
    throw std::runtime_error("shim cumsum: only forward int32 scans");
  }
  detail::sync();
  array out = zeros(a.shape(), int32);
  const int32_t* in = a.data<int32_t>();
  int32_t* o = out.data<int32_t>();
  int64_t run = 0;
  for (size_t i = 0; i < a.size(); ++i) {
    if (inclusive) {
      run += in[i];
      o[i] = static_cast<int32_t>(run);
    } else {
      o[i] = static_cast<int32_t>(run);
      run += in[i];
    }
  }
  return out;
}

inline array argsort(const array& a, StreamOrDevice = {}) {
  if (a.dtype() != int64 || a.ndim() != 1) {
    throw std::runtime_error("shim argsort: only 1-D int64 keys");
  }
  detail::sync();
  const int64_t* k = a.data<int64_t>();
  std::vector<uint32_t> idx(a.size());
  std::iota(idx.begin(), idx.end(), 0u);
  std::stable_sort(idx.begin(), idx.end(),
                   [k](uint32_t x, uint32_t y) { return k[x] < k[y]; });
  return array::from_host(idx.data(), a.shape(), uint32);
}

inline array take(const array& a, const array& indices, StreamOrDevice = {}) {
  if (indices.dtype() != uint32 || a.ndim() != 1) {
    throw std::runtime_error("shim take: only 1-D gathers by uint32");
  }
  detail::sync();
  array out = zeros(indices.shape(), a.dtype());
  const uint32_t* idx = indices.data<uint32_t>();
  const size_t item = a.itemsize();
  const char* src = a.data<char>();
  char* dst = out.data<char>();
  for (size_t i = 0; i < indices.size(); ++i) {
    std::memcpy(dst + i * item, src + static_cast<size_t>(idx[i]) * item, item);
  }
  return out;
}

}  // namespace core
}  // namespace mlx
