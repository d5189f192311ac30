// Element types, buffers and tensors of the rg engine (restates src/tensor.rs:3-153).
//
// A buffer is a typed, contiguous, row-major array. The same three dtypes exist on the host and
// on the device; a plan slot is a (dtype, capacity) pair and may hold a shorter value than its
// capacity (plan.rs:190-217).
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace rg {

enum class DType : uint8_t { F32 = 0, F64 = 1, I32 = 2 };

// tensor.rs:10-24
inline const char* dtype_name(DType d) {
  switch (d) {
    case DType::F32: return "float32";
    case DType::F64: return "float64";
    default: return "int32";
  }
}
inline size_t dtype_size(DType d) { return d == DType::F64 ? 8 : 4; }

inline bool parse_dtype(const std::string& s, DType* out) {
  if (s == "float32" || s == "f32") { *out = DType::F32; return true; }
  if (s == "float64" || s == "f64") { *out = DType::F64; return true; }
  if (s == "int32" || s == "i32") { *out = DType::I32; return true; }
  return false;
}

inline size_t product(const std::vector<size_t>& s) {
  size_t n = 1;
  for (size_t d : s) n *= d;
  return n;
}

// A typed byte buffer (tensor.rs:27-98 `Buf`). Storage is 8-byte aligned for f64.
struct Buf {
  DType dtype = DType::F32;
  size_t n = 0;
  std::vector<uint64_t> store;  // 8-byte words, so every dtype is aligned

  Buf() = default;
  Buf(DType d, size_t len) : dtype(d), n(len), store((len * dtype_size(d) + 7) / 8, 0) {}

  size_t bytes() const { return n * dtype_size(dtype); }
  void* data() { return store.data(); }
  const void* data() const { return store.data(); }
  float* f32() { return reinterpret_cast<float*>(store.data()); }
  const float* f32() const { return reinterpret_cast<const float*>(store.data()); }
  double* f64() { return reinterpret_cast<double*>(store.data()); }
  const double* f64() const { return reinterpret_cast<const double*>(store.data()); }
  int32_t* i32() { return reinterpret_cast<int32_t*>(store.data()); }
  const int32_t* i32() const { return reinterpret_cast<const int32_t*>(store.data()); }

  double get(size_t i) const {
    switch (dtype) {
      case DType::F32: return (double)f32()[i];
      case DType::F64: return f64()[i];
      default: return (double)i32()[i];
    }
  }
  std::vector<double> to_f64() const {
    std::vector<double> v(n);
    for (size_t i = 0; i < n; ++i) v[i] = get(i);
    return v;
  }
  // Rust `as` conversions from f64 (tensor.rs:87-93): f32 rounds, i32 saturates with NaN -> 0.
  static Buf from_f64(DType d, const std::vector<double>& v);
  Buf prefix(size_t k) const {
    Buf b(dtype, k);
    std::memcpy(b.data(), data(), k * dtype_size(dtype));
    return b;
  }
  bool operator==(const Buf& o) const {
    return dtype == o.dtype && n == o.n && std::memcmp(data(), o.data(), bytes()) == 0;
  }
};

// Rust `f64 as i32`: saturating, NaN -> 0.
inline int32_t sat_i32(double x) {
  if (std::isnan(x)) return 0;
  if (x >= 2147483647.0) return 2147483647;
  if (x <= -2147483648.0) return (int32_t)-2147483648LL;
  return (int32_t)x;  // truncation toward zero, as Rust does
}
inline int32_t sat_i32f(float x) { return sat_i32((double)x); }

inline Buf Buf::from_f64(DType d, const std::vector<double>& v) {
  Buf b(d, v.size());
  for (size_t i = 0; i < v.size(); ++i) {
    switch (d) {
      case DType::F32: b.f32()[i] = (float)v[i]; break;
      case DType::F64: b.f64()[i] = v[i]; break;
      default: b.i32()[i] = sat_i32(v[i]); break;
    }
  }
  return b;
}

struct Tensor {
  std::vector<size_t> shape;
  Buf data;

  Tensor() = default;
  Tensor(std::vector<size_t> s, Buf b) : shape(std::move(s)), data(std::move(b)) {}
  static Tensor from_f64(DType d, const std::vector<size_t>& shape, const std::vector<double>& v) {
    if (product(shape) != v.size()) throw std::runtime_error("Tensor::from_f64 size mismatch");
    return Tensor(shape, Buf::from_f64(d, v));
  }
  static Tensor full(DType d, const std::vector<size_t>& shape, double x) {
    return from_f64(d, shape, std::vector<double>(product(shape), x));
  }
  DType dtype() const { return data.dtype; }
  size_t n() const { return data.n; }
  bool is_finite() const {
    if (data.dtype == DType::F32) {
      for (size_t i = 0; i < data.n; ++i)
        if (!std::isfinite(data.f32()[i])) return false;
    } else if (data.dtype == DType::F64) {
      for (size_t i = 0; i < data.n; ++i)
        if (!std::isfinite(data.f64()[i])) return false;
    }
    return true;
  }
  bool operator==(const Tensor& o) const { return shape == o.shape && data == o.data; }
};

using TensorP = std::shared_ptr<const Tensor>;

}  // namespace rg
