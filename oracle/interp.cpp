// TEST INFRASTRUCTURE — CPU restatement of rg's plan interpreter, used only as the parity
// checker and the timed CPU baseline. Each kernel cites the arm of src/plan.rs it follows.
// Built with -ffp-contract=off: rg (Rust) never fuses a multiply and an add, so neither may we.
#include "interp.h"
#include "../rustautograd_b200/csrc/host/rowchain.h"

#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <cmath>
#include <limits>
#include <map>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <thread>

namespace rg::oracle {

namespace {

// plan.rs:6-10, 1391-1401
constexpr size_t BLOCK = 256;
constexpr size_t TASK = 16 * BLOCK;
constexpr uint64_t GAMMA = 0x9E3779B97F4A7C15ull;
constexpr uint64_t GAMMA_SPLIT = 0xD1B54A32D192ED03ull;
constexpr size_t PARALLEL_RANDOM = size_t(1) << 15;
constexpr size_t PARALLEL_COPY = size_t(1) << 19;
constexpr size_t PARALLEL_SUM = size_t(1) << 20;
constexpr size_t PARALLEL_MINMAX = size_t(1) << 16;
constexpr size_t REDUCE_ROWS = 64;
constexpr size_t PARALLEL_FLOPS = 2000000;

// ---- a small fixed pool standing in for rayon ----
class Pool {
 public:
  explicit Pool(int n) { resize(n); }
  ~Pool() { shutdown(); }
  void resize(int n) {
    shutdown();
    stop_ = false;
    nthreads_ = std::max(1, n);
    for (int i = 1; i < nthreads_; ++i) workers_.emplace_back([this] { loop(); });
  }
  int size() const { return nthreads_; }
  void run(size_t n, const std::function<void(size_t)>& f) {
    if (n == 0) return;
    if (n == 1 || workers_.empty()) {
      for (size_t i = 0; i < n; ++i) f(i);
      return;
    }
    std::unique_lock<std::mutex> lk(m_);
    job_ = &f;
    n_ = n;
    next_.store(0);
    finished_ = 0;
    ++gen_;
    cv_.notify_all();
    lk.unlock();
    work();
    lk.lock();
    done_cv_.wait(lk, [&] { return finished_ == n_; });
    job_ = nullptr;
  }

 private:
  void work() {
    size_t did = 0;
    for (;;) {
      size_t i = next_.fetch_add(1);
      if (i >= n_) break;
      (*job_)(i);
      ++did;
    }
    std::lock_guard<std::mutex> lk(m_);
    finished_ += did;
    if (finished_ == n_) done_cv_.notify_all();
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(m_);
      cv_.wait(lk, [&] { return stop_ || (gen_ != seen && job_ != nullptr); });
      if (stop_) return;
      seen = gen_;
      lk.unlock();
      work();
    }
  }
  void shutdown() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
      cv_.notify_all();
    }
    for (auto& t : workers_) t.join();
    workers_.clear();
  }
  std::vector<std::thread> workers_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t)>* job_ = nullptr;
  size_t n_ = 0, finished_ = 0;
  std::atomic<size_t> next_{0};
  uint64_t gen_ = 0;
  bool stop_ = false;
  int nthreads_ = 1;
};

Pool& pool() {
  static Pool p((int)std::max(1u, std::thread::hardware_concurrency()));
  return p;
}

template <typename T> T* S(Buf& b) { return reinterpret_cast<T*>(b.data()); }
template <typename T> const T* S(const Buf& b) { return reinterpret_cast<const T*>(b.data()); }

void check_dtype(const Buf& b, DType d) {
  if (b.dtype != d) throw std::logic_error("dtype mismatch in plan");
}

// ---- element semantics (plan.rs:1190-1210, 1063-1071; tensor.rs:215-227 via libm) ----
template <typename T> T nan_max(T a, T b) { return a > b ? a : (b >= a ? b : (T)NAN); }
template <typename T> T nan_min(T a, T b) { return a < b ? a : (b <= a ? b : (T)NAN); }
template <typename T> T sign(T x) { return x > 0 ? (T)1 : (x < 0 ? (T)-1 : x); }

inline float m_exp(float x) { return expf(x); }
inline double m_exp(double x) { return exp(x); }
inline float m_log(float x) { return logf(x); }
inline double m_log(double x) { return log(x); }
inline float m_sin(float x) { return sinf(x); }
inline double m_sin(double x) { return sin(x); }
inline float m_cos(float x) { return cosf(x); }
inline double m_cos(double x) { return cos(x); }
inline float m_tanh(float x) { return tanhf(x); }
inline double m_tanh(double x) { return tanh(x); }
inline float m_sqrt(float x) { return sqrtf(x); }
inline double m_sqrt(double x) { return sqrt(x); }
inline float m_pow(float x, float y) { return powf(x, y); }
inline double m_pow(double x, double y) { return pow(x, y); }
inline float m_floor(float x) { return floorf(x); }
inline double m_floor(double x) { return floor(x); }

template <typename T> T unary_op(OpKind k, T x) {
  switch (k) {
    case OpKind::Neg: return -x;
    case OpKind::Exp: return m_exp(x);
    case OpKind::Log: return m_log(x);
    case OpKind::Sqrt: return m_sqrt(x);
    case OpKind::Sin: return m_sin(x);
    case OpKind::Cos: return m_cos(x);
    case OpKind::Tanh: return m_tanh(x);
    case OpKind::Abs: return std::fabs(x);
    case OpKind::Sign: return sign(x);
    case OpKind::Floor: return m_floor(x);
    default: throw std::logic_error("not unary");
  }
}

template <typename T> T binary_op(OpKind k, T a, T b) {
  switch (k) {
    case OpKind::Add: return a + b;
    case OpKind::Sub: return a - b;
    case OpKind::Mul: return a * b;
    case OpKind::Div: return a / b;
    case OpKind::Pow: return m_pow(a, b);
    case OpKind::Max: return nan_max(a, b);
    case OpKind::Min: return nan_min(a, b);
    case OpKind::Gt: return a > b ? (T)1 : (T)0;
    case OpKind::Ge: return a >= b ? (T)1 : (T)0;
    default: throw std::logic_error("not binary");
  }
}

// plan.rs:1272-1287: int arithmetic wraps.
int32_t binary_int(OpKind k, int32_t a, int32_t b) {
  switch (k) {
    case OpKind::Add: return (int32_t)((uint32_t)a + (uint32_t)b);
    case OpKind::Sub: return (int32_t)((uint32_t)a - (uint32_t)b);
    case OpKind::Mul: return (int32_t)((uint32_t)a * (uint32_t)b);
    case OpKind::Gt: return a > b;
    case OpKind::Ge: return a >= b;
    default: throw std::logic_error("integer op not supported");
  }
}

std::pair<std::vector<size_t>, size_t> split_rows(const std::vector<size_t>& shape) {
  if (shape.empty()) return {{}, 1};
  return {std::vector<size_t>(shape.begin(), shape.end() - 1), shape.back()};
}

// Odometer over `shape` tracking N flat offsets (plan.rs:1166-1188).
template <size_t N, typename F>
void walk(const std::vector<size_t>& shape, const std::array<const std::vector<size_t>*, N>& st, F f) {
  size_t total = product(shape);
  std::vector<size_t> idx(shape.size(), 0);
  std::array<size_t, N> off{};
  for (size_t t = 0; t < total; ++t) {
    f(off);
    for (size_t d = shape.size(); d-- > 0;) {
      idx[d] += 1;
      for (size_t k = 0; k < N; ++k) off[k] += (*st[k])[d];
      if (idx[d] < shape[d]) break;
      for (size_t k = 0; k < N; ++k) off[k] -= (*st[k])[d] * shape[d];
      idx[d] = 0;
    }
  }
}

// plan.rs:1213-1230: eight-lane accumulation, then the lanes, then the tail.
template <typename T> T fast_sum(const T* a, size_t n) {
  T acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t full = n / 8 * 8;
  for (size_t c = 0; c < full; c += 8)
    for (int k = 0; k < 8; ++k) acc[k] = acc[k] + a[c + k];
  T out = 0;
  for (int k = 0; k < 8; ++k) out = out + acc[k];
  for (size_t i = full; i < n; ++i) out = out + a[i];
  return out;
}

size_t clamp_index(int32_t ix, size_t dim) { return std::min<size_t>((size_t)std::max(ix, 0), dim - 1); }

uint64_t mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t read_key(const Buf& b) {
  const int32_t* k = S<int32_t>(b);
  return ((uint64_t)(uint32_t)k[0] << 32) | (uint64_t)(uint32_t)k[1];
}

// tensor.rs:238-251: out[m*n] = A @ B, k ascending, start from zero, no fused multiply-add.
template <typename T>
void gemm(size_t m, size_t k, size_t n, const T* a, bool ta, const T* b, bool tb, T* out) {
  std::fill(out, out + m * n, (T)0);
  for (size_t i = 0; i < m; ++i) {
    T* row = out + i * n;
    for (size_t p = 0; p < k; ++p) {
      T x = ta ? a[p * m + i] : a[i * k + p];
      if (tb) {
        for (size_t j = 0; j < n; ++j) row[j] = row[j] + x * b[j * k + p];
      } else {
        const T* br = b + p * n;
        for (size_t j = 0; j < n; ++j) row[j] = row[j] + x * br[j];
      }
    }
  }
}

// ---- fused groups (plan.rs:892-970) ----
template <typename T>
void run_block(const Fused& f, const std::vector<const T*>& inputs, std::vector<T>& temp, size_t start, size_t len,
               const std::vector<std::vector<size_t>>& bst) {
  for (size_t k = 0; k < f.inputs.size(); ++k) {
    const FusedInput& in = f.inputs[k];
    if (in.kind == ArgKind::Full) continue;
    T* r = temp.data() + in.reg * BLOCK;
    if (in.kind == ArgKind::Splat) {
      std::fill(r, r + len, inputs[k][0]);
    } else if (in.kind == ArgKind::Row) {
      for (size_t j = 0; j < len; ++j) r[j] = inputs[k][(start + j) % in.row];
    } else {
      // Any other broadcast: the element the materialised broadcast would hold (rg's Metal
      // kernels compute this index; its CPU groups never contain such inputs).
      const auto& st = bst[k];
      const auto& shape = f.shape;
      for (size_t j = 0; j < len; ++j) {
        size_t flat = start + j, off = 0;
        for (size_t d = shape.size(); d-- > 0;) {
          size_t c = flat % shape[d];
          flat /= shape[d];
          off += c * st[d];
        }
        r[j] = inputs[k][off];
      }
    }
  }
  for (const MicroOp& m : f.ops) {
    T* d = temp.data() + m.reg * BLOCK;
    auto arg = [&](size_t i) -> const T* {
      const Operand& o = m.args[i];
      return o.reg ? temp.data() + o.idx * BLOCK : inputs[o.idx] + start;
    };
    OpKind k = m.op.kind;
    if (m.op.is_unary_elementwise()) {
      const T* a = arg(0);
      for (size_t j = 0; j < len; ++j) d[j] = unary_op<T>(k, a[j]);
    } else if (k == OpKind::Where) {
      const T *c = arg(0), *x = arg(1), *y = arg(2);
      for (size_t j = 0; j < len; ++j) d[j] = c[j] != (T)0 ? x[j] : y[j];
    } else {
      const T *a = arg(0), *b = arg(1);
      for (size_t j = 0; j < len; ++j) d[j] = binary_op<T>(k, a[j], b[j]);
    }
  }
}

template <typename T> void run_fused(const Fused& f, std::vector<Buf>& s) {
  std::vector<const T*> inputs;
  std::vector<std::vector<size_t>> bst;
  for (size_t k = 0; k < f.inputs.size(); ++k) {
    inputs.push_back(S<T>(s[f.inputs[k].slot]));
    bst.push_back(f.inputs[k].kind == ArgKind::Broadcast ? bstrides(f.input_shapes[k], f.shape.size()) : std::vector<size_t>{});
  }
  std::vector<T*> outs;
  for (auto& o : f.outputs) outs.push_back(S<T>(s[o.second]));
  size_t tasks = (f.n + TASK - 1) / TASK;
  pool().run(tasks, [&](size_t c) {
    std::vector<T> temp(f.regs * BLOCK);
    size_t start = c * TASK, end = std::min(start + TASK, f.n);
    for (size_t b = start; b < end; b += BLOCK) {
      size_t len = std::min(BLOCK, end - b);
      run_block<T>(f, inputs, temp, b, len, bst);
      for (size_t k = 0; k < f.outputs.size(); ++k)
        std::memcpy(outs[k] + b, temp.data() + f.outputs[k].first * BLOCK, len * sizeof(T));
    }
  });
}

// ---- single instructions ----
template <typename T> void unary(const Instr& i, std::vector<Buf>& s) {
  // In place or not, each element is computed once from its own input (plan.rs:1053-1086).
  const T* a = S<T>(s[i.args[0]]);
  T* d = S<T>(s[i.dst]);
  for (size_t j = 0; j < i.n; ++j) d[j] = unary_op<T>(i.op.kind, a[j]);
}

template <typename T, typename F> void binary(const Instr& i, std::vector<Buf>& s, F f) {
  const T* av = S<T>(s[i.args[0]]);
  const T* bv = S<T>(s[i.args[1]]);
  T* dst = S<T>(s[i.dst]);
  size_t n = i.n;
  switch (i.mode) {
    case Mode::Same:
      for (size_t j = 0; j < n; ++j) dst[j] = f(av[j], bv[j]);
      break;
    case Mode::AScalar: {
      T c = av[0];
      for (size_t j = 0; j < n; ++j) dst[j] = f(c, bv[j]);
      break;
    }
    case Mode::BScalar: {
      T c = bv[0];
      for (size_t j = 0; j < n; ++j) dst[j] = f(av[j], c);
      break;
    }
    case Mode::General: {
      auto ds = strides(i.shape);
      auto sa = bstrides(i.arg_shapes[0], i.shape.size());
      auto sb = bstrides(i.arg_shapes[1], i.shape.size());
      auto [outer, len] = split_rows(i.shape);
      size_t ra = i.shape.empty() ? 0 : sa.back();
      size_t rb = i.shape.empty() ? 0 : sb.back();
      walk<3>(outer, {&ds, &sa, &sb}, [&](const std::array<size_t, 3>& o) {
        T* row = dst + o[0];
        if (ra == 0 && rb == 0) {
          T v = f(av[o[1]], bv[o[2]]);
          for (size_t j = 0; j < len; ++j) row[j] = v;
        } else if (ra == 0) {
          T c = av[o[1]];
          for (size_t j = 0; j < len; ++j) row[j] = f(c, bv[o[2] + j]);
        } else if (rb == 0) {
          T c = bv[o[2]];
          for (size_t j = 0; j < len; ++j) row[j] = f(av[o[1] + j], c);
        } else {
          for (size_t j = 0; j < len; ++j) row[j] = f(av[o[1] + j], bv[o[2] + j]);
        }
      });
      break;
    }
  }
}

// plan.rs:1290-1383
template <typename T> void structural(const Instr& i, std::vector<Buf>& s) {
  const T* a = S<T>(s[i.args[0]]);
  T* dst = S<T>(s[i.dst]);
  auto ds = strides(i.shape);
  switch (i.op.kind) {
    case OpKind::Where: {
      const T* x = S<T>(s[i.args[1]]);
      const T* y = S<T>(s[i.args[2]]);
      for (size_t j = 0; j < i.n; ++j) dst[j] = a[j] != (T)0 ? x[j] : y[j];
      break;
    }
    case OpKind::Transpose: {
      auto src = strides(i.arg_shapes[0]);
      std::vector<size_t> mapped;
      for (size_t p : i.op.shape) mapped.push_back(src[p]);
      auto [outer, len] = split_rows(i.shape);
      size_t last = mapped.empty() ? 1 : mapped.back();
      auto copy_row = [&](T* row, size_t p) {
        if (last == 1) std::memcpy(row, a + p, len * sizeof(T));
        else
          for (size_t j = 0; j < len; ++j) row[j] = a[p + j * last];
      };
      if (i.n >= PARALLEL_COPY && len > 0) {
        std::vector<size_t> offsets;
        offsets.reserve(i.n / len);
        walk<1>(outer, {&mapped}, [&](const std::array<size_t, 1>& o) { offsets.push_back(o[0]); });
        size_t rows = offsets.size();
        size_t chunk = std::max<size_t>(1, rows / (4 * pool().size()));
        pool().run((rows + chunk - 1) / chunk, [&](size_t c) {
          for (size_t r = c * chunk; r < std::min(rows, (c + 1) * chunk); ++r) copy_row(dst + r * len, offsets[r]);
        });
      } else {
        walk<2>(outer, {&ds, &mapped}, [&](const std::array<size_t, 2>& o) { copy_row(dst + o[0], o[1]); });
      }
      break;
    }
    case OpKind::BroadcastTo: {
      auto src = bstrides(i.arg_shapes[0], i.shape.size());
      auto [outer, len] = split_rows(i.shape);
      size_t last = src.empty() ? 0 : src.back();
      walk<2>(outer, {&ds, &src}, [&](const std::array<size_t, 2>& o) {
        if (last == 0) std::fill(dst + o[0], dst + o[0] + len, a[o[1]]);
        else std::memcpy(dst + o[0], a + o[1], len * sizeof(T));
      });
      break;
    }
    case OpKind::Slice: {
      auto src = strides(i.arg_shapes[0]);
      size_t base = 0;
      for (size_t k = 0; k < src.size(); ++k) base += i.op.starts[k] * src[k];
      auto [outer, len] = split_rows(i.shape);
      walk<2>(outer, {&ds, &src}, [&](const std::array<size_t, 2>& o) { std::memcpy(dst + o[0], a + base + o[1], len * sizeof(T)); });
      break;
    }
    case OpKind::Pad: {
      std::fill(dst, dst + i.n, (T)0);
      auto src = strides(i.arg_shapes[0]);
      size_t base = 0;
      for (size_t k = 0; k < ds.size(); ++k) base += i.op.starts[k] * ds[k];
      auto [outer, len] = split_rows(i.arg_shapes[0]);
      walk<2>(outer, {&ds, &src}, [&](const std::array<size_t, 2>& o) { std::memcpy(dst + base + o[0], a + o[1], len * sizeof(T)); });
      break;
    }
    case OpKind::Concat: {
      size_t axis = i.op.index;
      size_t tail = 1, outer = 1;
      for (size_t k = axis + 1; k < i.shape.size(); ++k) tail *= i.shape[k];
      for (size_t k = 0; k < axis; ++k) outer *= i.shape[k];
      size_t at = 0;
      for (size_t o = 0; o < outer; ++o) {
        for (size_t k = 0; k < i.args.size(); ++k) {
          size_t len = i.arg_shapes[k][axis] * tail;
          std::memcpy(dst + at, S<T>(s[i.args[k]]) + o * len, len * sizeof(T));
          at += len;
        }
      }
      break;
    }
    case OpKind::Take: {
      const auto& xs = i.arg_shapes[0];
      size_t axis = i.op.index, block = 1, outer = 1;
      for (size_t k = axis + 1; k < xs.size(); ++k) block *= xs[k];
      for (size_t k = 0; k < axis; ++k) outer *= xs[k];
      size_t dim = xs[axis];
      size_t n_idx = product(i.arg_shapes[1]);
      const int32_t* idx = S<int32_t>(s[i.args[1]]);
      for (size_t o = 0; o < outer; ++o)
        for (size_t j = 0; j < n_idx; ++j)
          std::memcpy(dst + (o * n_idx + j) * block, a + (o * dim + clamp_index(idx[j], dim)) * block, block * sizeof(T));
      break;
    }
    case OpKind::TakeAlong: {
      size_t v = i.arg_shapes[0].back(), k = i.arg_shapes[1].back();
      const int32_t* idx = S<int32_t>(s[i.args[1]]);
      for (size_t j = 0; j < i.n; ++j) dst[j] = a[(j / k) * v + clamp_index(idx[j], v)];
      break;
    }
    default: throw std::logic_error(std::string(i.op.name()) + " has no structural kernel");
  }
}

// plan.rs:1453-1493
template <typename T> void matmul(const Instr& i, std::vector<Buf>& s, bool ta, bool tb) {
  const auto &sa = i.arg_shapes[0], &sb = i.arg_shapes[1];
  const T* a = S<T>(s[i.args[0]]);
  const T* b = S<T>(s[i.args[1]]);
  T* dst = S<T>(s[i.dst]);
  size_t ar = sa.size(), br = sb.size();
  size_t m, k, n;
  if (ar >= 2) {
    m = ta ? sa[ar - 1] : sa[ar - 2];
    k = ta ? sa[ar - 2] : sa[ar - 1];
  } else {
    m = 1;
    k = sa[0];
  }
  n = br >= 2 ? (tb ? sb[br - 2] : sb[br - 1]) : 1;
  std::vector<size_t> ba(sa.begin(), sa.end() - std::min<size_t>(2, ar));
  std::vector<size_t> bb(sb.begin(), sb.end() - std::min<size_t>(2, br));
  if (i.n == 0) return;
  if (bb.empty() && !ta) {
    // Row-major batches of the left operand are one big matrix: a single call.
    gemm<T>(product(ba) * m, k, n, a, false, b, tb, dst);
    return;
  }
  std::vector<size_t> batch;
  broadcast_shapes(ba, bb, &batch);
  size_t sz_a = m * k, sz_b = k * n, sz_o = m * n;
  auto scale = [](std::vector<size_t> v, size_t by) {
    for (auto& x : v) x *= by;
    return v;
  };
  auto st_o = scale(strides(batch), sz_o), st_a = scale(bstrides(ba, batch.size()), sz_a), st_b = scale(bstrides(bb, batch.size()), sz_b);
  size_t count = product(batch);
  if (m * k * n * count >= PARALLEL_FLOPS) {
    std::vector<std::pair<size_t, size_t>> offsets;
    offsets.reserve(count);
    walk<2>(batch, {&st_a, &st_b}, [&](const std::array<size_t, 2>& o) { offsets.emplace_back(o[0], o[1]); });
    pool().run(count, [&](size_t c) { gemm<T>(m, k, n, a + offsets[c].first, ta, b + offsets[c].second, tb, dst + c * sz_o); });
  } else {
    walk<3>(batch, {&st_o, &st_a, &st_b}, [&](const std::array<size_t, 3>& o) { gemm<T>(m, k, n, a + o[1], ta, b + o[2], tb, dst + o[0]); });
  }
}

// plan.rs:1549-1622
template <typename T> void reduce(const Instr& i, std::vector<Buf>& s) {
  const T* a = S<T>(s[i.args[0]]);
  T* dst = S<T>(s[i.dst]);
  const auto& in_shape = i.arg_shapes[0];
  const auto& axes = i.op.shape;
  ReduceKind kind = i.op.reduce;
  size_t in_n = product(in_shape);
  if (kind == ReduceKind::Sum && axes.size() == in_shape.size()) {
    dst[0] = fast_sum(a, in_n);
    return;
  }
  auto keep = in_shape;
  for (size_t ax : axes) keep[ax] = 1;
  auto out_st = strides(keep);
  for (size_t ax : axes) out_st[ax] = 0;
  auto in_st = strides(in_shape);
  auto [outer, len] = split_rows(in_shape);
  bool last_reduced = !in_shape.empty() && out_st.back() == 0;
  auto combine = [kind](T acc, T x) {
    return kind == ReduceKind::Sum ? acc + x : kind == ReduceKind::Max ? nan_max(acc, x) : nan_min(acc, x);
  };
  T init = kind == ReduceKind::Sum ? (T)0 : kind == ReduceKind::Max ? -(T)INFINITY : (T)INFINITY;
  size_t rank = in_shape.size();
  if (in_n >= (kind == ReduceKind::Sum ? PARALLEL_SUM : PARALLEL_MINMAX) && len > 0) {
    if (axes.size() == 1 && axes[0] == rank - 1) {
      size_t rows = in_n / len;
      size_t chunk = std::max<size_t>(1, rows / (4 * pool().size()));
      pool().run((rows + chunk - 1) / chunk, [&](size_t c) {
        for (size_t r = c * chunk; r < std::min(rows, (c + 1) * chunk); ++r) {
          const T* row = a + r * len;
          if (kind == ReduceKind::Sum) {
            dst[r] = fast_sum(row, len);
          } else {
            T acc = init;
            for (size_t j = 0; j < len; ++j) acc = combine(acc, row[j]);
            dst[r] = acc;
          }
        }
      });
      return;
    }
    if (axes.size() + 1 == rank && std::find(axes.begin(), axes.end(), rank - 1) == axes.end()) {
      // Only the last axis survives: partial results combined in a fixed order.
      size_t chunk = REDUCE_ROWS * len;
      size_t nparts = (in_n + chunk - 1) / chunk;
      std::vector<std::vector<T>> parts(nparts);
      pool().run(nparts, [&](size_t c) {
        std::vector<T> part(len, init);
        size_t end = std::min(in_n, (c + 1) * chunk);
        for (size_t r = c * chunk; r + len <= end; r += len)
          for (size_t o = 0; o < len; ++o) part[o] = combine(part[o], a[r + o]);
        parts[c] = std::move(part);
      });
      std::fill(dst, dst + len, init);
      for (auto& part : parts)
        for (size_t o = 0; o < len; ++o) dst[o] = combine(dst[o], part[o]);
      return;
    }
  }
  std::fill(dst, dst + i.n, init);
  walk<2>(outer, {&in_st, &out_st}, [&](const std::array<size_t, 2>& o) {
    const T* row = a + o[0];
    size_t q = o[1];
    if (last_reduced && kind == ReduceKind::Sum) {
      dst[q] = dst[q] + fast_sum(row, len);
    } else if (last_reduced) {
      T acc = dst[q];
      for (size_t j = 0; j < len; ++j) acc = combine(acc, row[j]);
      dst[q] = acc;
    } else {
      for (size_t j = 0; j < len; ++j) dst[q + j] = combine(dst[q + j], row[j]);
    }
  });
}

// plan.rs:1496-1547
template <typename T> void numeric(const Instr& i, std::vector<Buf>& s) {
  T* dst = S<T>(s[i.dst]);
  switch (i.op.kind) {
    case OpKind::MatMul: matmul<T>(i, s, false, false); break;
    case OpKind::MatMulT: matmul<T>(i, s, i.op.flag_a, i.op.flag_b); break;
    case OpKind::Reduce: reduce<T>(i, s); break;
    case OpKind::TakeGrad: {
      const T* ct = S<T>(s[i.args[0]]);
      const auto& shape = i.op.shape;
      size_t axis = i.op.index, block = 1, outer = 1;
      for (size_t k = axis + 1; k < shape.size(); ++k) block *= shape[k];
      for (size_t k = 0; k < axis; ++k) outer *= shape[k];
      size_t dim = shape[axis];
      size_t n_idx = product(i.arg_shapes[1]);
      const int32_t* idx = S<int32_t>(s[i.args[1]]);
      std::fill(dst, dst + i.n, (T)0);
      for (size_t o = 0; o < outer; ++o)
        for (size_t j = 0; j < n_idx; ++j) {
          T* to = dst + (o * dim + clamp_index(idx[j], dim)) * block;
          const T* from = ct + (o * n_idx + j) * block;
          for (size_t e = 0; e < block; ++e) to[e] = to[e] + from[e];
        }
      break;
    }
    case OpKind::TakeAlongGrad: {
      const T* ct = S<T>(s[i.args[0]]);
      size_t v = i.op.shape.back(), k = i.arg_shapes[1].back();
      size_t n_ct = product(i.arg_shapes[1]);
      const int32_t* idx = S<int32_t>(s[i.args[1]]);
      std::fill(dst, dst + i.n, (T)0);
      for (size_t j = 0; j < n_ct; ++j) {
        size_t to = (j / k) * v + clamp_index(idx[j], v);
        dst[to] = dst[to] + ct[j];
      }
      break;
    }
    case OpKind::RandUniform: {
      uint64_t key = read_key(s[i.args[0]]);
      int mant = sizeof(T) == 4 ? 24 : 53;
      double scale = std::ldexp(1.0, -mant);
      auto f = [&](size_t j) { return (T)((double)(mix(key + (uint64_t)(j + 1) * GAMMA) >> (64 - mant)) * scale); };
      if (i.n >= PARALLEL_RANDOM) {
        size_t chunk = 1 << 14;
        pool().run((i.n + chunk - 1) / chunk, [&](size_t c) {
          for (size_t j = c * chunk; j < std::min(i.n, (c + 1) * chunk); ++j) dst[j] = f(j);
        });
      } else {
        for (size_t j = 0; j < i.n; ++j) dst[j] = f(j);
      }
      break;
    }
    case OpKind::RandNormal: {
      uint64_t key = read_key(s[i.args[0]]);
      const double two53 = std::ldexp(1.0, -53);
      auto unit = [&](uint64_t c) { return (double)(mix(key + c * GAMMA) >> 11) * two53; };
      const double TAU = 6.283185307179586;
      auto f = [&](size_t j) {
        double u1 = 1.0 - unit(2 * (uint64_t)j + 1), u2 = unit(2 * (uint64_t)j + 2);
        return (T)(sqrt(-2.0 * log(u1)) * cos(TAU * u2));
      };
      if (i.n >= PARALLEL_RANDOM) {
        size_t chunk = 1 << 14;
        pool().run((i.n + chunk - 1) / chunk, [&](size_t c) {
          for (size_t j = c * chunk; j < std::min(i.n, (c + 1) * chunk); ++j) dst[j] = f(j);
        });
      } else {
        for (size_t j = 0; j < i.n; ++j) dst[j] = f(j);
      }
      break;
    }
    default: throw std::logic_error(std::string(i.op.name()) + " has no numeric kernel");
  }
}

template <typename T> void cumsum(const Instr& i, std::vector<Buf>& s) {
  size_t v = i.shape.back();
  if (v == 0) return;
  const T* a = S<T>(s[i.args[0]]);
  T* d = S<T>(s[i.dst]);
  for (size_t r = 0; r < i.n / v; ++r) {
    T acc = 0;
    if (i.op.flag_a) {
      for (size_t j = v; j-- > 0;) {
        acc = acc + a[r * v + j];
        d[r * v + j] = acc;
      }
    } else {
      for (size_t j = 0; j < v; ++j) {
        acc = acc + a[r * v + j];
        d[r * v + j] = acc;
      }
    }
  }
}

int32_t wrap_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }

void cumsum_int(const Instr& i, std::vector<Buf>& s) {
  size_t v = i.shape.back();
  if (v == 0) return;
  const int32_t* a = S<int32_t>(s[i.args[0]]);
  int32_t* d = S<int32_t>(s[i.dst]);
  for (size_t r = 0; r < i.n / v; ++r) {
    int32_t acc = 0;
    if (i.op.flag_a) {
      for (size_t j = v; j-- > 0;) d[r * v + j] = acc = wrap_add(acc, a[r * v + j]);
    } else {
      for (size_t j = 0; j < v; ++j) d[r * v + j] = acc = wrap_add(acc, a[r * v + j]);
    }
  }
}

template <typename T> void argmax(const Instr& i, std::vector<Buf>& s) {
  size_t v = i.arg_shapes[0].back();
  const T* a = S<T>(s[i.args[0]]);
  int32_t* d = S<int32_t>(s[i.dst]);
  for (size_t r = 0; r < i.n; ++r) {
    const T* row = a + r * v;
    size_t best = 0;
    for (size_t j = 0; j < v; ++j)
      if (row[j] > row[best]) best = j;
    d[r] = (int32_t)best;
  }
}

// plan.rs:833-866: larger first, ties by index, NaN last; a total order.
template <typename T> void arg_top_k(const Instr& i, std::vector<Buf>& s) {
  size_t v = i.arg_shapes[0].back(), k = i.op.index;
  const T* a = S<T>(s[i.args[0]]);
  int32_t* d = S<int32_t>(s[i.dst]);
  size_t rows = i.n / k;
  auto select = [&](size_t r) {
    const T* row = a + r * v;
    std::vector<int32_t> idx(v);
    std::iota(idx.begin(), idx.end(), 0);
    auto less = [&](int32_t x, int32_t y) {
      T p = row[x], q = row[y];
      bool pn = std::isnan(p), qn = std::isnan(q);
      if (pn || qn) {
        if (pn != qn) return !pn;  // NaN ranks last
        return x < y;
      }
      if (p != q) return p > q;
      return x < y;
    };
    std::sort(idx.begin(), idx.end(), less);
    std::memcpy(d + r * k, idx.data(), k * sizeof(int32_t));
  };
  if (product(i.arg_shapes[0]) >= PARALLEL_MINMAX) pool().run(rows, select);
  else
    for (size_t r = 0; r < rows; ++r) select(r);
}

// plan.rs:1624-1642: Rust `as` casts.
void cast(const Instr& i, std::vector<Buf>& s) {
  const Buf& a = s[i.args[0]];
  Buf& d = s[i.dst];
  size_t n = i.n;
  if (d.dtype == DType::F32 && a.dtype == DType::F64) for (size_t j = 0; j < n; ++j) S<float>(d)[j] = (float)S<double>(a)[j];
  else if (d.dtype == DType::F64 && a.dtype == DType::F32) for (size_t j = 0; j < n; ++j) S<double>(d)[j] = (double)S<float>(a)[j];
  else if (d.dtype == DType::F32 && a.dtype == DType::I32) for (size_t j = 0; j < n; ++j) S<float>(d)[j] = (float)S<int32_t>(a)[j];
  else if (d.dtype == DType::F64 && a.dtype == DType::I32) for (size_t j = 0; j < n; ++j) S<double>(d)[j] = (double)S<int32_t>(a)[j];
  else if (d.dtype == DType::I32 && a.dtype == DType::F32) for (size_t j = 0; j < n; ++j) S<int32_t>(d)[j] = sat_i32f(S<float>(a)[j]);
  else if (d.dtype == DType::I32 && a.dtype == DType::F64) for (size_t j = 0; j < n; ++j) S<int32_t>(d)[j] = sat_i32(S<double>(a)[j]);
  else throw std::logic_error("same-dtype casts are aliases");
}

std::function<void(void*, size_t, DType)> g_all_reduce;

void all_reduce(const Instr& i, std::vector<Buf>& s) {
  std::memcpy(s[i.dst].data(), s[i.args[0]].data(), i.n * dtype_size(i.dtype));
  if (g_all_reduce) g_all_reduce(s[i.dst].data(), i.n, i.dtype);
}

void key_split(const Instr& i, std::vector<Buf>& s) {
  uint64_t key = read_key(s[i.args[0]]);
  int32_t* d = S<int32_t>(s[i.dst]);
  for (size_t j = 0; j < i.n / 2; ++j) {
    uint64_t bits = mix(key + (uint64_t)(j + 1) * GAMMA_SPLIT);
    d[2 * j] = (int32_t)(uint32_t)(bits >> 32);
    d[2 * j + 1] = (int32_t)(uint32_t)bits;
  }
}

// Fused attention (the device's own ops, no counterpart in rg): the CPU definition the device's
// kernels are checked against. Per batch entry and query row i: Z_j = mask_ij ? (q_i . k_j) / c :
// fill; m = max_j Z_j; E_j = exp(Z_j - m); s = sum_j E_j; P_j = E_j / s; O_i = sum_j P_j v_j.
// Sums run in index order. The backward recomputes P from the saved (m, s) and gives
// dS_j = mask_ij ? P_j (dP_j - sum_l P_l dP_l) / c : 0 with dP_j = dO_i . v_j, then
// dq = dS k, dk = dS^T q, dv = P^T dO.
// With a third attribute H (value = [c, fill, H]) q, k and v come packed as one (B, T, 3, H, d)
// tensor (the projection's output before the head split), batch entry b * H + h; dO comes as
// (B, T, H, d) and the backward's result is the gradient of that packed (B, T, 3, H, d) tensor.
struct AttnDims {
  size_t batch, t, d, dv;
  size_t heads = 0;  // > 0: the packed (B, T, 3, H, d) layout
};
AttnDims attn_dims(const Instr& i) {
  const auto& q = i.arg_shapes[0];
  size_t r = q.size();
  AttnDims a;
  if (i.op.value->n() == 3) {
    a.heads = (size_t)i.op.value->data.get(2);
    a.t = q[1];
    a.d = a.dv = q[4];
    a.batch = q[0] * a.heads;
    return a;
  }
  a.t = q[r - 2];
  a.d = q[r - 1];
  a.dv = i.arg_shapes[2][r - 1];
  a.batch = product(q) / (a.t * a.d);
  return a;
}

// Element (batch entry z, row t, column e) of part `which` (0 q, 1 k, 2 v) of the packed layout.
inline size_t packed_at(const AttnDims& a, size_t which, size_t z, size_t t, size_t e) {
  const size_t b = z / a.heads, h = z - b * a.heads;
  return ((b * a.t + t) * 3 + which) * a.heads * a.d + h * a.d + e;
}

// Z_ij for query row i, key j; `mask_row` is row i of the (T, T) mask.
template <typename T> T attn_score(const T* q, const T* k, const T* mask_row, size_t i, size_t j, size_t d, T c, T fill) {
  T acc = (T)0;
  for (size_t e = 0; e < d; ++e) acc = acc + q[i * d + e] * k[j * d + e];
  return mask_row[j] != (T)0 ? acc / c : fill;
}

// Batch entry z's q, k, v (and dO), contiguous (T, d) rows, from either layout.
template <typename T> struct AttnEntry {
  std::vector<T> q, k, v, dout;
  void load(const AttnDims& a, const Instr& i, std::vector<Buf>& s, size_t z, bool with_dout) {
    const T *Q = S<T>(s[i.args[0]]), *K = a.heads ? Q : S<T>(s[i.args[1]]), *V = a.heads ? Q : S<T>(s[i.args[2]]);
    q.resize(a.t * a.d);
    k.resize(a.t * a.d);
    v.resize(a.t * a.dv);
    for (size_t t = 0; t < a.t; ++t) {
      for (size_t e = 0; e < a.d; ++e) {
        q[t * a.d + e] = a.heads ? Q[packed_at(a, 0, z, t, e)] : Q[(z * a.t + t) * a.d + e];
        k[t * a.d + e] = a.heads ? K[packed_at(a, 1, z, t, e)] : K[(z * a.t + t) * a.d + e];
      }
      for (size_t e = 0; e < a.dv; ++e) v[t * a.dv + e] = a.heads ? V[packed_at(a, 2, z, t, e)] : V[(z * a.t + t) * a.dv + e];
    }
    if (!with_dout) return;
    const T* DO = S<T>(s[i.args[a.heads ? 3 : 5]]);
    dout.resize(a.t * a.dv);
    for (size_t t = 0; t < a.t; ++t)
      for (size_t e = 0; e < a.dv; ++e) {
        const size_t b = a.heads ? z / a.heads : 0, h = a.heads ? z - b * a.heads : 0;
        dout[t * a.dv + e] = a.heads ? DO[((b * a.t + t) * a.heads + h) * a.dv + e] : DO[(z * a.t + t) * a.dv + e];
      }
  }
};

template <typename T> void attn_fwd(const Instr& i, std::vector<Buf>& s) {
  const AttnDims a = attn_dims(i);
  const T c = (T)i.op.value->data.get(0), fill = (T)i.op.value->data.get(1);
  const T* M = S<T>(s[i.args[a.heads ? 1 : 3]]);
  T* out = S<T>(s[i.dst]);
  const size_t w = a.dv + 2;
  std::vector<T> z(a.t);
  AttnEntry<T> en;
  for (size_t b = 0; b < a.batch; ++b) {
    en.load(a, i, s, b, false);
    const T *q = en.q.data(), *k = en.k.data(), *v = en.v.data();
    for (size_t r = 0; r < a.t; ++r) {
      T m = -std::numeric_limits<T>::infinity();
      for (size_t j = 0; j < a.t; ++j) {
        z[j] = attn_score(q, k, M + r * a.t, r, j, a.d, c, fill);
        m = z[j] > m || std::isnan(z[j]) ? z[j] : m;
      }
      T sum = (T)0;
      for (size_t j = 0; j < a.t; ++j) {
        z[j] = std::exp(z[j] - m);
        sum = sum + z[j];
      }
      T* o = out + (b * a.t + r) * w;
      for (size_t e = 0; e < a.dv; ++e) o[e] = (T)0;
      for (size_t j = 0; j < a.t; ++j) {
        const T p = z[j] / sum;
        for (size_t e = 0; e < a.dv; ++e) o[e] = o[e] + p * v[j * a.dv + e];
      }
      o[a.dv] = m;
      o[a.dv + 1] = sum;
    }
  }
}

template <typename T> void attn_bwd(const Instr& i, std::vector<Buf>& s) {
  const AttnDims a = attn_dims(i);
  const T c = (T)i.op.value->data.get(0), fill = (T)i.op.value->data.get(1);
  const T* M = S<T>(s[i.args[a.heads ? 1 : 3]]);
  // The forward's packed output, (..., T, dv + 2) = O, row max, row exp-sum.
  const T* FW = S<T>(s[i.args[a.heads ? 2 : 4]]);
  T* out = S<T>(s[i.dst]);
  const size_t w = 2 * a.d + a.dv, fw = a.dv + 2;
  std::vector<T> p(a.t), dp(a.t), g(a.t * w);
  AttnEntry<T> en;
  if (!a.heads) std::fill(out, out + a.batch * a.t * w, (T)0);
  for (size_t b = 0; b < a.batch; ++b) {
    en.load(a, i, s, b, true);
    const T *q = en.q.data(), *k = en.k.data(), *v = en.v.data(), *dout = en.dout.data();
    std::fill(g.begin(), g.end(), (T)0);
    for (size_t r = 0; r < a.t; ++r) {
      const T* o = FW + (b * a.t + r) * fw;
      const T m = o[a.dv], sum = o[a.dv + 1];
      // D = sum_j P_rj dP_rj = dO_r . O_r (O_r = sum_j P_rj v_j).
      T dsum = (T)0;
      for (size_t e = 0; e < a.dv; ++e) dsum = dsum + dout[r * a.dv + e] * o[e];
      for (size_t j = 0; j < a.t; ++j) {
        p[j] = std::exp(attn_score(q, k, M + r * a.t, r, j, a.d, c, fill) - m) / sum;
        T acc = (T)0;
        for (size_t e = 0; e < a.dv; ++e) acc = acc + dout[r * a.dv + e] * v[j * a.dv + e];
        dp[j] = acc;
      }
      for (size_t j = 0; j < a.t; ++j) {
        const T ds = M[r * a.t + j] != (T)0 ? p[j] * (dp[j] - dsum) / c : (T)0;
        for (size_t e = 0; e < a.d; ++e) {
          g[r * w + e] = g[r * w + e] + ds * k[j * a.d + e];                 // dq
          g[j * w + a.d + e] = g[j * w + a.d + e] + ds * q[r * a.d + e];     // dk
        }
        for (size_t e = 0; e < a.dv; ++e) g[j * w + 2 * a.d + e] = g[j * w + 2 * a.d + e] + p[j] * dout[r * a.dv + e];  // dv
      }
    }
    for (size_t t = 0; t < a.t; ++t) {
      if (!a.heads) {
        std::copy(g.begin() + t * w, g.begin() + (t + 1) * w, out + (b * a.t + t) * w);
        continue;
      }
      for (size_t e = 0; e < a.d; ++e) {
        out[packed_at(a, 0, b, t, e)] = g[t * w + e];
        out[packed_at(a, 1, b, t, e)] = g[t * w + a.d + e];
        out[packed_at(a, 2, b, t, e)] = g[t * w + 2 * a.d + e];
      }
    }
  }
}

void copy_prefix(Buf& d, const Buf& s, size_t n) { std::memcpy(d.data(), s.data(), n * dtype_size(s.dtype)); }
void copy_range(Buf& d, size_t at, const Buf& s, size_t from, size_t n) {
  size_t es = dtype_size(s.dtype);
  std::memcpy((char*)d.data() + at * es, (const char*)s.data() + from * es, n * es);
}

void run_control(const Instr& i, std::vector<Buf>& s);

template <typename T> void step(const Instr& i, std::vector<Buf>& s) {
  OpKind k = i.op.kind;
  if (i.op.is_unary_elementwise()) return unary<T>(i, s);
  if (i.op.is_binary_elementwise()) return binary<T>(i, s, [k](T a, T b) { return binary_op<T>(k, a, b); });
  switch (k) {
    case OpKind::Cumsum: return cumsum<T>(i, s);
    case OpKind::Where: case OpKind::Transpose: case OpKind::BroadcastTo: case OpKind::Slice: case OpKind::Pad:
    case OpKind::Concat: case OpKind::Take: case OpKind::TakeAlong:
      return structural<T>(i, s);
    default: return numeric<T>(i, s);
  }
}

void step_int(const Instr& i, std::vector<Buf>& s) {
  OpKind k = i.op.kind;
  switch (k) {
    case OpKind::Add: case OpKind::Sub: case OpKind::Mul: case OpKind::Gt: case OpKind::Ge:
      return binary<int32_t>(i, s, [k](int32_t a, int32_t b) { return binary_int(k, a, b); });
    case OpKind::Cumsum: return cumsum_int(i, s);
    default: return structural<int32_t>(i, s);
  }
}

// plan.rs:692-712
void exec_instr(const Instr& i, std::vector<Buf>& s) {
  if (i.op.is_control_flow()) return run_control(i, s);
  switch (i.op.kind) {
    case OpKind::Cast: return cast(i, s);
    case OpKind::ArgTopK:
      if (s[i.args[0]].dtype == DType::F32) return arg_top_k<float>(i, s);
      return arg_top_k<double>(i, s);
    case OpKind::KeySplit: return key_split(i, s);
    case OpKind::AllReduce: return all_reduce(i, s);
    case OpKind::AttnFwd:
      if (i.dtype == DType::F32) return attn_fwd<float>(i, s);
      return attn_fwd<double>(i, s);
    case OpKind::AttnBwd:
      if (i.dtype == DType::F32) return attn_bwd<float>(i, s);
      return attn_bwd<double>(i, s);
    case OpKind::Argmax:
      if (s[i.args[0]].dtype == DType::F32) return argmax<float>(i, s);
      return argmax<double>(i, s);
    default: break;
  }
  switch (i.dtype) {
    case DType::F32: return step<float>(i, s);
    case DType::F64: return step<double>(i, s);
    default: return step_int(i, s);
  }
}

void load_inputs(const Plan& plan, std::vector<Buf>& f, const std::vector<Buf>& s, const std::vector<size_t>& args, size_t from) {
  for (size_t k = 0; k + from < args.size(); ++k) copy_prefix(f[plan.input_slots[k]], s[args[k + from]], plan.input_ns[k]);
}

// Body outputs go to the carry inputs through copies: an output may be another carry's input.
void feed_carry(const Plan& plan, std::vector<Buf>& f, size_t n_carry) {
  std::vector<Buf> next;
  for (size_t k = 0; k < n_carry; ++k) next.push_back(f[plan.outputs[k].slot].prefix(plan.outputs[k].n));
  for (size_t k = 0; k < n_carry; ++k) copy_prefix(f[plan.input_slots[k]], next[k], next[k].n);
}

// plan.rs:737-831
void run_control(const Instr& i, std::vector<Buf>& s) {
  if (i.op.kind == OpKind::Scan) {
    const Plan& plan = *i.body_plan;
    size_t c = i.op.n_carry, x = i.op.n_x, length = i.op.length;
    size_t n_y = plan.outputs.size() - c;
    auto f = frame(plan);
    for (size_t k = 0; k < i.args.size(); ++k)
      if (k < c || k >= c + x) copy_prefix(f[plan.input_slots[k]], s[i.args[k]], plan.input_ns[k]);
    for (size_t st = 0; st < length; ++st) {
      size_t at = i.op.flag_a ? length - 1 - st : st;
      for (size_t k = c; k < c + x; ++k) {
        size_t m = plan.input_ns[k];
        copy_range(f[plan.input_slots[k]], 0, s[i.args[k]], at * m, m);
      }
      for (auto& [index, slot] : i.outs) {
        if (index >= c + n_y) {
          size_t k = index - c - n_y;
          size_t m = plan.input_ns[k];
          copy_range(s[slot], at * m, f[plan.input_slots[k]], 0, m);
        }
      }
      exec_plan(plan, f);
      for (auto& [index, slot] : i.outs) {
        if (index >= c && index < c + n_y) {
          const auto& o = plan.outputs[index];
          copy_range(s[slot], at * o.n, f[o.slot], 0, o.n);
        }
      }
      feed_carry(plan, f, c);
    }
    for (auto& [index, slot] : i.outs)
      if (index < c) copy_prefix(s[slot], f[plan.input_slots[index]], plan.input_ns[index]);
    return;
  }
  if (i.op.kind == OpKind::While) {
    const Plan& cp = *i.body_plan;
    const Plan& bp = *i.body2_plan;
    auto cf = frame(cp), bf = frame(bp);
    load_inputs(cp, cf, s, i.args, 0);
    load_inputs(bp, bf, s, i.args, 0);
    size_t count = 0;
    for (;;) {
      exec_plan(cp, cf);
      const auto& o = cp.outputs[0];
      if (cf[o.slot].get(0) == 0.0) break;
      if (count == i.op.max_iterations) break;
      exec_plan(bp, bf);
      feed_carry(bp, bf, i.op.n_carry);
      for (size_t k = 0; k < i.op.n_carry; ++k) copy_prefix(cf[cp.input_slots[k]], bf[bp.input_slots[k]], bp.input_ns[k]);
      count += 1;
    }
    for (auto& [index, slot] : i.outs) {
      if (index < i.op.n_carry) copy_prefix(s[slot], bf[bp.input_slots[index]], bp.input_ns[index]);
      else S<int32_t>(s[slot])[0] = (int32_t)count;
    }
    return;
  }
  // Cond
  bool taken = s[i.args[0]].get(0) != 0.0;
  const Plan& plan = taken ? *i.body_plan : *i.body2_plan;
  auto f = frame(plan);
  load_inputs(plan, f, s, i.args, 1);
  exec_plan(plan, f);
  for (auto& [index, slot] : i.outs) {
    const auto& o = plan.outputs[index];
    copy_prefix(s[slot], f[o.slot], o.n);
  }
}

class CpuExec : public Exec {
 public:
  explicit CpuExec(const Plan& p) : plan_(p), slots_(frame(p)) {}
  void load(size_t k, const Tensor& t) override { copy_prefix(slots_[plan_.input_slots[k]], t.data, plan_.input_ns[k]); }
  void step() override { exec_plan(plan_, slots_); }
  void step_at(size_t k) override {
    const Step& st = plan_.steps[k];
    if (st.fused) {
      if (st.group.dtype == DType::F32) run_fused<float>(st.group, slots_);
      else run_fused<double>(st.group, slots_);
    } else {
      exec_instr(st.instr, slots_);
    }
  }
  void swap(size_t a, size_t b) override { std::swap(slots_[a], slots_[b]); }
  Buf prefix(size_t slot, size_t n) override { return slots_[slot].prefix(n); }
  void write_prefix(size_t slot, const Buf& b) override { copy_prefix(slots_[slot], b, b.n); }
  double scalar(size_t slot) override { return slots_[slot].get(0); }
  std::vector<Buf>& slots() { return slots_; }

 private:
  const Plan& plan_;
  std::vector<Buf> slots_;
};

class CpuProgram : public Program {
 public:
  explicit CpuProgram(const Plan& p) : plan_(p) {}
  std::unique_ptr<Exec> exec() override { return std::make_unique<CpuExec>(plan_); }
  bool step_timed(Exec& e, std::vector<double>& seconds) override {
    for (size_t k = 0; k < plan_.steps.size(); ++k) {
      auto t0 = std::chrono::steady_clock::now();
      e.step_at(k);
      seconds[k] += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    }
    return true;
  }

 private:
  Plan plan_;
};

class CpuDevice : public Device {
 public:
  std::string name() const override { return "cpu"; }
  bool available() const override { return true; }
  Fuse fuse() const override { return Fuse::DEFAULT(); }
  std::shared_ptr<Program> compile(const Plan& plan) override { return std::make_shared<CpuProgram>(plan); }
};

// Plans built as for the CUDA device (its fusion configuration and graph rewrites), executed by
// this interpreter: lets CPU tests check the plans the device runs.
class CudaPlanDevice : public CpuDevice {
 public:
  std::string name() const override { return "cuda-plan"; }
  Fuse fuse() const override { return Fuse::CUDA(); }
};

}  // namespace

void set_threads(int n) { pool().resize(n); }
void set_all_reduce(std::function<void(void*, size_t, DType)> hook) { g_all_reduce = std::move(hook); }
int threads() { return pool().size(); }

std::vector<Buf> frame(const Plan& plan) {
  std::vector<Buf> slots;
  slots.reserve(plan.slots.size());
  for (auto& [d, n] : plan.slots) slots.emplace_back(d, n);
  for (auto& [slot, t] : plan.consts) copy_prefix(slots[slot], t->data, t->n());
  return slots;
}

namespace {

void exec_step(const Step& st, std::vector<Buf>& slots) {
  if (st.fused) {
    if (st.group.dtype == DType::F32) run_fused<float>(st.group, slots);
    else if (st.group.dtype == DType::F64) run_fused<double>(st.group, slots);
    else throw std::logic_error("integer ops are never fused");
  } else {
    exec_instr(st.instr, slots);
  }
}

// A row chain as the CUDA device runs it (rowchain.h): the steps moved before it, then its
// members with the broadcasts moved after it in plan order, which computes what the chain
// computes. The device writes only the values the chain stores; every other slot the chain
// writes keeps whatever it held, which no later step may read. This interpreter fills those
// slots with NaN instead, so that a chain whose stored values were chosen wrongly changes the
// results of the tests that run its plans here.
void exec_chain(const Plan& plan, const RowChain& c, std::vector<Buf>& slots) {
  for (size_t p : c.before) exec_step(plan.steps[p], slots);
  std::vector<size_t> order = c.members;
  order.insert(order.end(), c.after.begin(), c.after.end());
  std::sort(order.begin(), order.end());
  for (size_t p : order) exec_step(plan.steps[p], slots);
  std::map<size_t, bool> keep;  // slot -> its final write in the range is kept
  for (size_t p : order) {
    auto m = std::find(c.members.begin(), c.members.end(), p);
    auto writes = step_writes(plan.steps[p]);
    for (size_t q = 0; q < writes.size(); ++q)
      keep[writes[q]] = m == c.members.end() || c.store[(size_t)(m - c.members.begin())][q];
  }
  for (auto& [slot, kept] : keep) {
    if (kept) continue;
    Buf& b = slots[slot];
    if (b.dtype == DType::F32) std::fill(b.f32(), b.f32() + b.n, std::numeric_limits<float>::quiet_NaN());
    else if (b.dtype == DType::F64) std::fill(b.f64(), b.f64() + b.n, std::numeric_limits<double>::quiet_NaN());
  }
}

}  // namespace

void exec_steps(const Plan& plan, const std::vector<size_t>& steps, std::vector<Buf>& slots) {
  for (size_t k : steps) exec_step(plan.steps.at(k), slots);
}

void exec_plan(const Plan& plan, std::vector<Buf>& slots) {
  // Plans built with the CUDA device's fusion configuration run their row chains as the device
  // does.
  std::vector<RowChain> chains = find_row_chains(plan);
  size_t next = 0;
  for (size_t k = 0; k < plan.steps.size();) {
    if (next < chains.size() && chains[next].first == k) {
      exec_chain(plan, chains[next], slots);
      k = chains[next].last + 1;
      ++next;
      continue;
    }
    exec_step(plan.steps[k], slots);
    ++k;
  }
}

std::shared_ptr<Device> cpu_device() {
  static auto d = std::make_shared<CpuDevice>();
  return d;
}

std::shared_ptr<Device> cuda_plan_device() {
  static auto d = std::make_shared<CudaPlanDevice>();
  return d;
}

}  // namespace rg::oracle
