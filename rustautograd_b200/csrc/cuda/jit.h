// NVRTC code generation for fused elementwise groups (plan.rs:86-111 `Fused`).
//
// A group's kernel is generated from its structure alone: dtype, the kind of each input
// (full, splat, row, broadcast), the micro-op list and the outputs. Sizes, row lengths and
// broadcast strides are runtime parameters, so the layers of a model share kernels and a
// whole plan's kernels compile in one NVRTC call for sm_100a.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "kernels.cuh"
#include "plan.h"

namespace rgc {

constexpr int JIT_MAX_IN = 64;
constexpr int JIT_MAX_OUT = 64;

// Must match the struct emitted into every generated kernel.
struct ElemArgs {
  long long n;
  int vec;    // 1: full operands are 16-byte aligned and n is a multiple of the vector width
  int small;  // 1: n < 2^31 and every merged broadcast extent fits, so index math is 32-bit
  void* out[JIT_MAX_OUT];
  const void* in[JIT_MAX_IN];
  FDiv row[JIT_MAX_IN];  // row length of each row input, output last extent of each column input
  const FDims* bc;       // device array: one merged descriptor per broadcast input
  const Dims* bc64;      // device array: the same descriptors unmerged, for the 64-bit path
};

// A generated elementwise kernel: the structure (which decides the source) plus which argument
// slot each group input and output binds to at launch.
struct ElemSpec {
  rg::DType dtype = rg::DType::F32;
  struct In {
    rg::ArgKind kind;
    size_t row = 0;
    int bc = -1;  // broadcast descriptor index
    // A broadcast input of the output's shape with a last extent of 1 (a softmax or LayerNorm
    // statistic): element e reads value e / col, with col the output's last extent.
    size_t col = 0;
    // A full input whose slot holds a materialised broadcast of a constant or input: the kernel
    // reads the broadcast's source (`shape`) through broadcast indexing instead (same values).
    bool via = false;
    std::vector<size_t> shape;
  };
  std::vector<In> inputs;
  std::vector<rg::MicroOp> ops;
  std::vector<size_t> out_regs;
  std::vector<size_t> shape;  // output shape
  size_t n = 0;
  std::string source_key() const;
};

// The output's last extent when `in` is the output's shape with a last extent of 1, else 0.
size_t column_of(const std::vector<size_t>& in, const std::vector<size_t>& out);

// One micro-op as a C expression over operand expressions, and the C type of a dtype: what every
// generated kernel evaluates per element.
std::string elem_expr(rg::DType d, const rg::Op& op, const std::vector<std::string>& args);
std::string elem_ctype(rg::DType d);

// Builds an ElemSpec from a fused group or from a single elementwise instruction.
ElemSpec spec_from_group(const rg::Fused& f);
ElemSpec spec_from_instr(const rg::Instr& i);

class Jit {
 public:
  // Registers a kernel; returns its name. Nothing compiles until `build`.
  std::string add(const ElemSpec& s);
  // Registers a generated kernel given as source (one function `name`, ElemArgs parameter).
  void add_source(const std::string& name, const std::string& source);
  // Compiles `sources` with the prelude for sm_100a without loading them (no GPU needed): an
  // empty string, or the compiler's log.
  static std::string compile_check(const std::vector<std::string>& sources);
  // The definitions every generated kernel is compiled with (types, index helpers, rg_div...).
  static std::string prelude();
  // Compiles every registered kernel not yet built (one NVRTC program) and loads it.
  void build();
  CUfunction function(const std::string& name) const;
  static void launch(CUfunction f, const ElemArgs& a, long long n, int vec_width, cudaStream_t s);
  // A row-chain kernel: `blocks` blocks of 256 threads at most (capped at one wave), `smem` bytes
  // of dynamic shared memory each.
  static void launch_rows(CUfunction f, const ElemArgs& a, long long blocks, size_t smem, cudaStream_t s);

 private:
  std::unordered_map<std::string, std::string> pending_;  // name -> source
  std::unordered_map<std::string, std::vector<std::string>> functions_;  // name -> functions it defines
  std::unordered_map<std::string, CUfunction> built_;
  std::vector<CUmodule> modules_;
};

// Driver entry points, resolved through the runtime so that nothing links libcuda directly.
struct Driver {
  CUresult (*ModuleLoadData)(CUmodule*, const void*) = nullptr;
  CUresult (*ModuleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*ModuleUnload)(CUmodule) = nullptr;
  CUresult (*LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream, void**, void**) = nullptr;
  CUresult (*OccupancyMaxActiveBlocksPerMultiprocessor)(int*, CUfunction, int, size_t) = nullptr;
  CUresult (*LaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**) = nullptr;
  CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  static const Driver& get();
};

}  // namespace rgc
