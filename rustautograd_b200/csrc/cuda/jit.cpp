// NVRTC code generation for fused elementwise groups.
#include "jit.h"

#include <nvrtc.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <sstream>
#include <stdexcept>
#include <sys/stat.h>
#include <unistd.h>

namespace rgc {

using rg::ArgKind;
using rg::DType;
using rg::OpKind;

const Driver& Driver::get() {
  static Driver d = [] {
    Driver x;
    auto load = [](const char* name, void** fn) {
      cudaDriverEntryPointQueryResult q;
#pragma GCC diagnostic push
#pragma GCC diagnostic ignored "-Wdeprecated-declarations"
      cudaError_t e = cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q);
#pragma GCC diagnostic pop
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !*fn) throw std::runtime_error(std::string("CUDA driver entry point missing: ") + name);
    };
    load("cuModuleLoadData", (void**)&x.ModuleLoadData);
    load("cuModuleGetFunction", (void**)&x.ModuleGetFunction);
    load("cuModuleUnload", (void**)&x.ModuleUnload);
    load("cuLaunchKernel", (void**)&x.LaunchKernel);
    load("cuOccupancyMaxActiveBlocksPerMultiprocessor", (void**)&x.OccupancyMaxActiveBlocksPerMultiprocessor);
    load("cuLaunchKernelEx", (void**)&x.LaunchKernelEx);
    load("cuFuncSetAttribute", (void**)&x.FuncSetAttribute);
    return x;
  }();
  return d;
}

namespace {

const char* PRELUDE = R"(
struct Dims { int rank; long long d[8]; long long st[8]; };
struct FDiv { unsigned d, m, s; };
struct FDims { int rank; FDiv d[8]; long long st[8]; };
struct ElemArgs { long long n; int vec; int small; void* out[64]; const void* in[64]; FDiv row[64]; const FDims* bc; const Dims* bc64; };
__device__ __forceinline__ unsigned rg_fdiv(unsigned n, const FDiv& f) { return (__umulhi(n, f.m) + n) >> f.s; }
__device__ __forceinline__ long long bc_off(const Dims& b, long long e) {
  long long off = 0;
  for (int d = b.rank - 1; d >= 0; --d) { long long c = e % b.d[d]; e /= b.d[d]; off += c * b.st[d]; }
  return off;
}
// Offset of element e under a merged broadcast descriptor; *inner receives e's innermost coordinate.
__device__ __forceinline__ long long rg_bc_off(const FDims& b, unsigned e, unsigned* inner) {
  long long off = 0;
  *inner = 0;
  for (int d = b.rank - 1; d >= 0; --d) {
    unsigned q = rg_fdiv(e, b.d[d]);
    unsigned c = e - q * b.d[d].d;
    if (d == b.rank - 1) *inner = c;
    off += (long long)c * b.st[d];
    e = q;
  }
  return off;
}
// V consecutive elements of a broadcast input: one offset computation when they share the
// innermost run, else one per element.
template <typename T, int V> __device__ __forceinline__ void rg_bc_fill(T* r, const T* p, const FDims& b, unsigned e) {
  unsigned c;
  long long off = rg_bc_off(b, e, &c);
  if (b.rank == 0) {
    #pragma unroll
    for (int j = 0; j < V; ++j) r[j] = p[0];
    return;
  }
  const unsigned inner = b.d[b.rank - 1].d;
  const long long st = b.st[b.rank - 1];
  if (c + V <= inner) {
    #pragma unroll
    for (int j = 0; j < V; ++j) r[j] = p[off + j * st];
  } else {
    #pragma unroll
    for (int j = 0; j < V; ++j) { unsigned cj; r[j] = p[rg_bc_off(b, e + j, &cj)]; }
  }
}
// V consecutive elements of a row input (the input repeats every f.d elements).
template <typename T, int V> __device__ __forceinline__ void rg_row_fill(T* r, const T* p, unsigned e, const FDiv& f) {
  if (f.d >= V) {
    unsigned c = e - rg_fdiv(e, f) * f.d;
    #pragma unroll
    for (int j = 0; j < V; ++j) { unsigned i = c + j; i = i >= f.d ? i - f.d : i; r[j] = p[i]; }
  } else {
    #pragma unroll
    for (int j = 0; j < V; ++j) { unsigned ej = e + j; r[j] = p[ej - rg_fdiv(ej, f) * f.d]; }
  }
}
// V consecutive elements of a column input (value e / f.d for element e).
template <typename T, int V> __device__ __forceinline__ void rg_col_fill(T* r, const T* p, unsigned e, const FDiv& f) {
  const unsigned q = rg_fdiv(e, f);
  if (e - q * f.d + V <= f.d) {
    const T v = p[q];
    #pragma unroll
    for (int j = 0; j < V; ++j) r[j] = v;
  } else {
    #pragma unroll
    for (int j = 0; j < V; ++j) r[j] = p[rg_fdiv(e + j, f)];
  }
}
// IEEE x / y. A zero numerator would send the division down its slow path (taken when the
// quotient may underflow), which costs several times the fast one; causal masks make half of a
// softmax's numerators zero. For y neither zero nor NaN the quotient is a zero with the sign of
// x * y, so zero numerators are answered directly and never enter the division.
__device__ __forceinline__ float rg_div(float x, float y) {
  const bool z = x == 0.0f && y == y && y != 0.0f;
  const float q = (z ? 1.0f : x) / y;
  return z ? __int_as_float((__float_as_int(x) ^ __float_as_int(y)) & (int)0x80000000u) : q;
}
__device__ __forceinline__ double rg_div(double x, double y) {
  const bool z = x == 0.0 && y == y && y != 0.0;
  const double q = (z ? 1.0 : x) / y;
  return z ? __longlong_as_double((__double_as_longlong(x) ^ __double_as_longlong(y)) & (long long)0x8000000000000000ull) : q;
}
__device__ __forceinline__ float rg_nan(float) { return __int_as_float(0x7fc00000); }
__device__ __forceinline__ double rg_nan(double) { return __longlong_as_double(0x7ff8000000000000LL); }
template <typename T> __device__ __forceinline__ T rg_max(T a, T b) { return a > b ? a : (b >= a ? b : rg_nan(a)); }
template <typename T> __device__ __forceinline__ T rg_min(T a, T b) { return a < b ? a : (b <= a ? b : rg_nan(a)); }
template <typename T> __device__ __forceinline__ T rg_sign(T x) { return x > (T)0 ? (T)1 : (x < (T)0 ? (T)-1 : x); }
__device__ __forceinline__ int rg_iadd(int a, int b) { return (int)((unsigned)a + (unsigned)b); }
__device__ __forceinline__ int rg_isub(int a, int b) { return (int)((unsigned)a - (unsigned)b); }
__device__ __forceinline__ int rg_imul(int a, int b) { return (int)((unsigned)a * (unsigned)b); }
)";

std::string ctype(DType d) { return d == DType::F32 ? "float" : d == DType::F64 ? "double" : "int"; }
std::string vtype(DType d) { return d == DType::F32 ? "float4" : d == DType::F64 ? "double2" : "int4"; }
int vwidth(DType d) { return d == DType::F64 ? 2 : 4; }
const char* lane(int j) {
  static const char* n[] = {"x", "y", "z", "w"};
  return n[j];
}

std::string fn1(DType d, const char* f32, const char* f64, const std::string& x) {
  return std::string(d == DType::F64 ? f64 : f32) + "(" + x + ")";
}

// One micro-op as a C expression over operand expressions (plan.rs:935-963 semantics).
std::string expr(DType d, const rg::Op& op, const std::vector<std::string>& a) {
  bool I = d == DType::I32;
  std::string T = ctype(d);
  switch (op.kind) {
    case OpKind::Neg: return "(-" + a[0] + ")";
    case OpKind::Exp: return fn1(d, "expf", "exp", a[0]);
    case OpKind::Log: return fn1(d, "logf", "log", a[0]);
    case OpKind::Sqrt: return fn1(d, "sqrtf", "sqrt", a[0]);
    case OpKind::Sin: return fn1(d, "sinf", "sin", a[0]);
    case OpKind::Cos: return fn1(d, "cosf", "cos", a[0]);
    case OpKind::Tanh: return fn1(d, "tanhf", "tanh", a[0]);
    case OpKind::Abs: return fn1(d, "fabsf", "fabs", a[0]);
    case OpKind::Sign: return "rg_sign<" + T + ">(" + a[0] + ")";
    case OpKind::Floor: return fn1(d, "floorf", "floor", a[0]);
    case OpKind::Add: return I ? "rg_iadd(" + a[0] + "," + a[1] + ")" : "(" + a[0] + " + " + a[1] + ")";
    case OpKind::Sub: return I ? "rg_isub(" + a[0] + "," + a[1] + ")" : "(" + a[0] + " - " + a[1] + ")";
    case OpKind::Mul: return I ? "rg_imul(" + a[0] + "," + a[1] + ")" : "(" + a[0] + " * " + a[1] + ")";
    case OpKind::Div: return I ? "(" + a[0] + " / " + a[1] + ")" : "rg_div(" + a[0] + "," + a[1] + ")";
    case OpKind::Pow: return (d == DType::F64 ? "pow(" : "powf(") + a[0] + "," + a[1] + ")";
    case OpKind::Max: return "rg_max<" + T + ">(" + a[0] + "," + a[1] + ")";
    case OpKind::Min: return "rg_min<" + T + ">(" + a[0] + "," + a[1] + ")";
    case OpKind::Gt: return "((" + a[0] + " > " + a[1] + ") ? (" + T + ")1 : (" + T + ")0)";
    case OpKind::Ge: return "((" + a[0] + " >= " + a[1] + ") ? (" + T + ")1 : (" + T + ")0)";
    case OpKind::Where: return "((" + a[0] + " != (" + T + ")0) ? " + a[1] + " : " + a[2] + ")";
    default: throw std::runtime_error(std::string("op is not elementwise: ") + op.name());
  }
}

}  // namespace

std::string elem_expr(DType d, const rg::Op& op, const std::vector<std::string>& args) { return expr(d, op, args); }
std::string elem_ctype(DType d) { return ctype(d); }

std::string ElemSpec::source_key() const {
  std::string k = "d" + std::to_string((int)dtype) + "|";
  for (auto& in : inputs) k += std::to_string((int)in.kind) + (in.via ? "v" : "") + (in.col ? "c," : ",");
  k += "|";
  for (auto& m : ops) {
    k += std::to_string((int)m.op.kind) + ":" + std::to_string(m.reg) + "(";
    for (auto& a : m.args) k += (a.reg ? "r" : "i") + std::to_string(a.idx) + ",";
    k += ")";
  }
  k += "|";
  for (auto r : out_regs) k += std::to_string(r) + ",";
  return k;
}

// The column length when a broadcast input has the output's shape with a last extent of 1.
size_t column_of(const std::vector<size_t>& in, const std::vector<size_t>& out) {
  if (in.size() != out.size() || out.empty() || in.back() != 1 || out.back() <= 1) return 0;
  for (size_t d = 0; d + 1 < out.size(); ++d)
    if (in[d] != out[d]) return 0;
  return out.back();
}

ElemSpec spec_from_group(const rg::Fused& f) {
  ElemSpec s;
  s.dtype = f.dtype;
  s.shape = f.shape;
  s.n = f.n;
  int nbc = 0;
  for (size_t k = 0; k < f.inputs.size(); ++k) {
    ElemSpec::In in;
    in.kind = f.inputs[k].kind;
    in.row = f.inputs[k].row;
    in.shape = f.input_shapes[k];
    if (in.kind == ArgKind::Broadcast) {
      in.bc = nbc++;
      in.col = column_of(in.shape, f.shape);
    }
    s.inputs.push_back(in);
  }
  s.ops = f.ops;
  for (auto& o : f.outputs) s.out_regs.push_back(o.first);
  return s;
}

ElemSpec spec_from_instr(const rg::Instr& i) {
  ElemSpec s;
  s.dtype = i.dtype;
  s.shape = i.shape;
  s.n = i.n;
  size_t reg = 0;
  rg::MicroOp m;
  m.op = i.op;
  int nbc = 0;
  for (size_t k = 0; k < i.args.size(); ++k) {
    const auto& as = i.arg_shapes[k];
    ElemSpec::In in;
    in.shape = as;
    size_t n = rg::product(as);
    if (as == i.shape) in.kind = ArgKind::Full;
    else if (n == 1) in.kind = ArgKind::Splat;
    else if (!as.empty() && !i.shape.empty() && as.back() == i.shape.back() && n == as.back()) {
      in.kind = ArgKind::Row;
      in.row = n;
    } else {
      in.kind = ArgKind::Broadcast;
      in.bc = nbc++;
      in.col = column_of(as, i.shape);
    }
    if (in.kind == ArgKind::Full) {
      m.args.push_back(rg::Operand{false, k});
    } else {
      m.args.push_back(rg::Operand{true, reg});
      ++reg;
    }
    s.inputs.push_back(in);
  }
  // Registers of non-full inputs come first, in input order, as in compile_group.
  m.reg = reg;
  s.ops.push_back(m);
  s.out_regs.push_back(reg);
  return s;
}

static std::string kernel_source(const ElemSpec& s, const std::string& name) {
  std::ostringstream o;
  std::string T = ctype(s.dtype), VT = vtype(s.dtype);
  const int VW = vwidth(s.dtype);
  // Map: non-full input k -> register; compile_group assigns registers in input order.
  std::vector<long> in_reg(s.inputs.size(), -1);
  {
    size_t r = 0;
    for (size_t k = 0; k < s.inputs.size(); ++k)
      if (s.inputs[k].kind != ArgKind::Full) in_reg[k] = (long)r++;
  }
  auto in_ptr = [&](size_t k) { return "((const " + T + "*)a.in[" + std::to_string(k) + "])"; };
  // The micro-ops over G lanes, then the outputs.
  auto ops = [&](int G) {
    for (auto& m : s.ops) {
      o << "      " << T << " r" << m.reg << "[" << G << "];\n";
      o << "      #pragma unroll\n      for (int j = 0; j < " << G << "; ++j) r" << m.reg << "[j] = ";
      std::vector<std::string> args;
      for (auto& x : m.args) args.push_back((x.reg ? "r" : "i") + std::to_string(x.idx) + "[j]");
      o << expr(s.dtype, m.op, args) << ";\n";
    }
  };
  // Two kernels: `name` for n < 2^31 with 32-bit index math, `name_w` with 64-bit index math.
  // Separate kernels keep the 64-bit path's registers out of the common one's occupancy.
  // Each kernel first waits for the grids it depends on (programmatic dependent launch: it may be
  // scheduled while the previous kernel drains) and lets its own dependents launch, then reads its
  // operands.
  auto header = [&](const std::string& fn) {
    o << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const ElemArgs a) {\n";
    o << "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
    o << "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n";
    for (size_t k = 0; k < s.inputs.size(); ++k)
      if (s.inputs[k].kind == ArgKind::Splat) o << "  const " << T << " sp" << k << " = " << in_ptr(k) << "[0];\n";
  };
  header(name);
  o << "  {\n";
  o << "    const unsigned n = (unsigned)a.n, tid = blockIdx.x * blockDim.x + threadIdx.x, stride = gridDim.x * blockDim.x;\n";
  // Vector path: two 16-byte vectors per thread per iteration (all loads before any store).
  o << "    if (a.vec) {\n";
  o << "     const unsigned nv = n / " << VW << ";\n";
  o << "     for (unsigned q = tid; q < nv; q += 2u * stride) {\n";
  o << "      const unsigned q1 = q + stride;\n      const bool h1 = q1 < nv;\n";
  o << "      const unsigned ea = q * " << VW << ", eb = (h1 ? q1 : q) * " << VW << ";\n";
  const int G = 2 * VW;
  for (size_t k = 0; k < s.inputs.size(); ++k) {
    const auto& in = s.inputs[k];
    if (in.kind == ArgKind::Full && in.via) {
      o << "      " << T << " i" << k << "[" << G << "];\n";
      if (in.col) {
        o << "      rg_col_fill<" << T << ", " << VW << ">(i" << k << ", " << in_ptr(k) << ", ea, a.row[" << k << "]);\n";
        o << "      rg_col_fill<" << T << ", " << VW << ">(i" << k << " + " << VW << ", " << in_ptr(k) << ", eb, a.row[" << k << "]);\n";
      } else {
        o << "      rg_bc_fill<" << T << ", " << VW << ">(i" << k << ", " << in_ptr(k) << ", a.bc[" << in.bc << "], ea);\n";
        o << "      rg_bc_fill<" << T << ", " << VW << ">(i" << k << " + " << VW << ", " << in_ptr(k) << ", a.bc[" << in.bc << "], eb);\n";
      }
    } else if (in.kind == ArgKind::Full) {
      o << "      " << T << " i" << k << "[" << G << "];\n";
      o << "      { const " << VT << " va = ((const " << VT << "*)a.in[" << k << "])[q], vb = ((const " << VT << "*)a.in[" << k
        << "])[h1 ? q1 : q];";
      for (int j = 0; j < VW; ++j) o << " i" << k << "[" << j << "] = va." << lane(j) << ";";
      for (int j = 0; j < VW; ++j) o << " i" << k << "[" << VW + j << "] = vb." << lane(j) << ";";
      o << " }\n";
    } else {
      long r = in_reg[k];
      o << "      " << T << " r" << r << "[" << G << "];\n";
      if (in.kind == ArgKind::Splat) {
        o << "      #pragma unroll\n      for (int j = 0; j < " << G << "; ++j) r" << r << "[j] = sp" << k << ";\n";
      } else if (in.kind == ArgKind::Row) {
        o << "      rg_row_fill<" << T << ", " << VW << ">(r" << r << ", " << in_ptr(k) << ", ea, a.row[" << k << "]);\n";
        o << "      rg_row_fill<" << T << ", " << VW << ">(r" << r << " + " << VW << ", " << in_ptr(k) << ", eb, a.row[" << k << "]);\n";
      } else if (in.col) {
        o << "      rg_col_fill<" << T << ", " << VW << ">(r" << r << ", " << in_ptr(k) << ", ea, a.row[" << k << "]);\n";
        o << "      rg_col_fill<" << T << ", " << VW << ">(r" << r << " + " << VW << ", " << in_ptr(k) << ", eb, a.row[" << k << "]);\n";
      } else {
        o << "      rg_bc_fill<" << T << ", " << VW << ">(r" << r << ", " << in_ptr(k) << ", a.bc[" << in.bc << "], ea);\n";
        o << "      rg_bc_fill<" << T << ", " << VW << ">(r" << r << " + " << VW << ", " << in_ptr(k) << ", a.bc[" << in.bc << "], eb);\n";
      }
    }
  }
  ops(G);
  for (size_t q = 0; q < s.out_regs.size(); ++q) {
    size_t r = s.out_regs[q];
    o << "      { " << VT << " va, vb;";
    for (int j = 0; j < VW; ++j) o << " va." << lane(j) << " = r" << r << "[" << j << "];";
    for (int j = 0; j < VW; ++j) o << " vb." << lane(j) << " = r" << r << "[" << VW + j << "];";
    o << " ((" << VT << "*)a.out[" << q << "])[q] = va; if (h1) ((" << VT << "*)a.out[" << q << "])[q1] = vb; }\n";
  }
  o << "     }\n";
  o << "    } else {\n";
  // Scalar path with 32-bit index math.
  o << "     for (unsigned e = tid; e < n; e += stride) {\n";
  for (size_t k = 0; k < s.inputs.size(); ++k) {
    const auto& in = s.inputs[k];
    if (in.kind == ArgKind::Full && in.via) {
      if (in.col) o << "      " << T << " i" << k << "[1] = {" << in_ptr(k) << "[rg_fdiv(e, a.row[" << k << "])]};\n";
      else o << "      unsigned c" << k << "; " << T << " i" << k << "[1] = {" << in_ptr(k) << "[rg_bc_off(a.bc[" << in.bc << "], e, &c" << k << ")]};\n";
    } else if (in.kind == ArgKind::Full) {
      o << "      " << T << " i" << k << "[1] = {" << in_ptr(k) << "[e]};\n";
    } else {
      long r = in_reg[k];
      o << "      " << T << " r" << r << "[1];\n";
      if (in.kind == ArgKind::Splat) o << "      r" << r << "[0] = sp" << k << ";\n";
      else if (in.kind == ArgKind::Row) o << "      r" << r << "[0] = " << in_ptr(k) << "[e - rg_fdiv(e, a.row[" << k << "]) * a.row[" << k << "].d];\n";
      else if (in.col) o << "      r" << r << "[0] = " << in_ptr(k) << "[rg_fdiv(e, a.row[" << k << "])];\n";
      else o << "      { unsigned c; r" << r << "[0] = " << in_ptr(k) << "[rg_bc_off(a.bc[" << in.bc << "], e, &c)]; }\n";
    }
  }
  ops(1);
  for (size_t q = 0; q < s.out_regs.size(); ++q) o << "      ((" << T << "*)a.out[" << q << "])[e] = r" << s.out_regs[q] << "[0];\n";
  o << "     }\n    }\n";
  // 64-bit path for 2^31 elements or more.
  o << "  }\n}\n";
  header(name + "_w");
  o << "  {\n";
  o << "    const long long n = a.n, tid = (long long)blockIdx.x * blockDim.x + threadIdx.x, stride = (long long)gridDim.x * blockDim.x;\n";
  o << "    for (long long e = tid; e < n; e += stride) {\n";
  for (size_t k = 0; k < s.inputs.size(); ++k) {
    const auto& in = s.inputs[k];
    if (in.kind == ArgKind::Full && in.via) {
      o << "      " << T << " i" << k << "[1] = {" << in_ptr(k) << "[bc_off(a.bc64[" << in.bc << "], e)]};\n";
    } else if (in.kind == ArgKind::Full) {
      o << "      " << T << " i" << k << "[1] = {" << in_ptr(k) << "[e]};\n";
    } else {
      long r = in_reg[k];
      o << "      " << T << " r" << r << "[1];\n";
      if (in.kind == ArgKind::Splat) o << "      r" << r << "[0] = sp" << k << ";\n";
      else if (in.kind == ArgKind::Row) o << "      r" << r << "[0] = " << in_ptr(k) << "[e % (long long)a.row[" << k << "].d];\n";
      else o << "      r" << r << "[0] = " << in_ptr(k) << "[bc_off(a.bc64[" << in.bc << "], e)];\n";
    }
  }
  ops(1);
  for (size_t q = 0; q < s.out_regs.size(); ++q) o << "      ((" << T << "*)a.out[" << q << "])[e] = r" << s.out_regs[q] << "[0];\n";
  o << "    }\n  }\n}\n";
  return o.str();
}

static uint64_t fnv1a(const std::string& s) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

std::string Jit::add(const ElemSpec& s) {
  std::string key = s.source_key();
  char name[64];
  snprintf(name, sizeof name, "rg_elem_%016llx", (unsigned long long)fnv1a(key));
  if (!built_.count(name) && !pending_.count(name)) {
    pending_[name] = kernel_source(s, name);
    functions_[name] = {name, std::string(name) + "_w"};
  }
  return name;
}

void Jit::add_source(const std::string& name, const std::string& source) {
  if (built_.count(name) || pending_.count(name)) return;
  pending_[name] = source;
  functions_[name] = {name};
}

static const char* const NVRTC_OPTS[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--prec-div=true", "--prec-sqrt=true", "--ftz=false",
                                         "-default-device", "--std=c++17"};

std::string Jit::prelude() { return PRELUDE; }

std::string Jit::compile_check(const std::vector<std::string>& sources) {
  std::string src = PRELUDE;
  for (auto& s : sources) src += s;
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, src.c_str(), "rg_check.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) return "nvrtcCreateProgram failed";
  nvrtcResult r = nvrtcCompileProgram(prog, (int)(sizeof NVRTC_OPTS / sizeof NVRTC_OPTS[0]), NVRTC_OPTS);
  std::string log;
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    log.assign(n, '\0');
    nvrtcGetProgramLog(prog, log.data());
    if (log.empty()) log = "NVRTC compilation failed";
  }
  nvrtcDestroyProgram(&prog);
  return log;
}

static std::string cache_dir() {
  const char* env = getenv("RGC_JIT_CACHE");
  std::string d = env ? env : ("/tmp/rgc-jit-" + std::to_string(getuid()));
  mkdir(d.c_str(), 0700);
  return d;
}

void Jit::build() {
  if (pending_.empty()) return;
  std::string src = PRELUDE;
  std::vector<std::string> names;
  for (auto& [name, s] : pending_) {
    src += s;
    names.push_back(name);
  }
  const char* const* opts = NVRTC_OPTS;
  std::string path = cache_dir() + "/" + std::to_string(fnv1a(src + "v6")) + ".cubin";
  std::vector<char> cubin;
  {
    std::ifstream f(path, std::ios::binary);
    if (f) cubin.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  }
  if (cubin.empty()) {
    nvrtcProgram prog;
    if (nvrtcCreateProgram(&prog, src.c_str(), "rg_fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) throw std::runtime_error("nvrtcCreateProgram failed");
    nvrtcResult r = nvrtcCompileProgram(prog, (int)(sizeof NVRTC_OPTS / sizeof NVRTC_OPTS[0]), opts);
    if (r != NVRTC_SUCCESS) {
      size_t n = 0;
      nvrtcGetProgramLogSize(prog, &n);
      std::string log(n, '\0');
      nvrtcGetProgramLog(prog, log.data());
      nvrtcDestroyProgram(&prog);
      throw std::runtime_error("NVRTC compilation of fused kernels failed: " + log.substr(0, 4000));
    }
    size_t n = 0;
    nvrtcGetCUBINSize(prog, &n);
    cubin.resize(n);
    nvrtcGetCUBIN(prog, cubin.data());
    nvrtcDestroyProgram(&prog);
    std::string tmp = path + ".tmp" + std::to_string(getpid());
    std::ofstream f(tmp, std::ios::binary);
    f.write(cubin.data(), (std::streamsize)cubin.size());
    f.close();
    rename(tmp.c_str(), path.c_str());
  }
  const Driver& d = Driver::get();
  CUmodule mod;
  CUresult lr = d.ModuleLoadData(&mod, cubin.data());
  if (lr != CUDA_SUCCESS) throw std::runtime_error("loading the fused-kernel module failed (CUresult " + std::to_string((int)lr) + ")");
  modules_.push_back(mod);
  for (auto& name : names)
    for (const std::string& fname : functions_[name]) {
      CUfunction fn;
      if (d.ModuleGetFunction(&fn, mod, fname.c_str()) != CUDA_SUCCESS) throw std::runtime_error("missing fused kernel " + fname);
      built_[fname] = fn;
    }
  pending_.clear();
}

void Jit::launch_rows(CUfunction f, const ElemArgs& a, long long blocks, size_t smem, cudaStream_t s) {
  static int sms = [] {
    int dev = 0, v = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  static std::mutex mu;
  static std::unordered_map<CUfunction, int> resident;
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = resident.find(f);
    if (it != resident.end()) {
      per_sm = it->second;
    } else {
      const Driver& d = Driver::get();
      if (d.FuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem) != CUDA_SUCCESS)
        throw std::runtime_error("row-chain kernel: shared memory request refused");
      if (d.OccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, 256, smem) != CUDA_SUCCESS || per_sm <= 0) per_sm = 1;
      resident[f] = per_sm;
    }
  }
  long long cap = (long long)sms * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  void* params[] = {(void*)&a};
  CUlaunchConfig cfg = {};
  cfg.gridDimX = (unsigned)blocks;
  cfg.gridDimY = cfg.gridDimZ = 1;
  cfg.blockDimX = 256;
  cfg.blockDimY = cfg.blockDimZ = 1;
  cfg.sharedMemBytes = (unsigned)smem;
  cfg.hStream = (CUstream)s;
  CUlaunchAttribute attr[1];
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  CUresult r = Driver::get().LaunchKernelEx(&cfg, f, params, nullptr);
  if (r != CUDA_SUCCESS) throw std::runtime_error("row-chain kernel launch failed (CUresult " + std::to_string((int)r) + ")");
}

CUfunction Jit::function(const std::string& name) const {
  auto it = built_.find(name);
  if (it == built_.end()) throw std::runtime_error("fused kernel not built: " + name);
  return it->second;
}

void Jit::launch(CUfunction f, const ElemArgs& a, long long n, int vec_width, cudaStream_t s) {
  static int sms = [] {
    int dev = 0, v = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  // One wave of resident blocks: how many fit per SM depends on the generated kernel's
  // registers (a fixed 8 per SM would leave a partial second wave above 32 registers).
  static std::mutex mu;
  static std::unordered_map<CUfunction, int> resident;
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = resident.find(f);
    if (it != resident.end()) {
      per_sm = it->second;
    } else {
      if (Driver::get().OccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, 256, 0) != CUDA_SUCCESS || per_sm <= 0) per_sm = 1;
      resident[f] = per_sm;
    }
  }
  long long work = a.vec ? (n / vec_width + 1) / 2 : n;
  long long blocks = (work + 255) / 256;
  long long cap = (long long)sms * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  void* params[] = {(void*)&a};
  CUlaunchConfig cfg = {};
  cfg.gridDimX = (unsigned)blocks;
  cfg.gridDimY = cfg.gridDimZ = 1;
  cfg.blockDimX = 256;
  cfg.blockDimY = cfg.blockDimZ = 1;
  cfg.sharedMemBytes = 0;
  cfg.hStream = (CUstream)s;
  CUlaunchAttribute attr[1];
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  CUresult r = Driver::get().LaunchKernelEx(&cfg, f, params, nullptr);
  if (r != CUDA_SUCCESS) throw std::runtime_error("fused kernel launch failed (CUresult " + std::to_string((int)r) + ")");
}

}  // namespace rgc
