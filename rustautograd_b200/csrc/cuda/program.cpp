// The rg CUDA device: plan lowering, device frames, the Exec contract, the device-resident run
// loop, and the C ABI of include/rgc.h.
//
// Lowering turns each plan step into a launch closure over slot indices; a frame maps slot
// indices to device pointers (one arena allocation per frame, 256-byte aligned slots), so a
// buffer swap between steps is a pointer swap. The run loop captures one CUDA graph per buffer
// layout (the state swaps are involutions, so two layouts alternate) and launches them back to
// back with no host synchronisation inside a chunk of steps.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unistd.h>
#include <unordered_map>
#include <vector>

#include "attention.cuh"
#include "blob.h"
#include "dist.h"
#include "gemm_tc.cuh"
#include "jit.h"
#include "kernels.cuh"
#include "rgc.h"
#include "rowkernel.h"

using rg::DType;
using rg::Instr;
using rg::OpKind;
using rg::Plan;

namespace rgc {

namespace {

thread_local std::string g_last_error;

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

EType et(DType d) { return d == DType::F32 ? EType::F32 : d == DType::F64 ? EType::F64 : EType::I32; }

constexpr size_t ALIGN = 256;
size_t align_up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

// GEMMs up to this many multiply-adds keep rg's exact loop arithmetic (bit-identical results);
// larger ones use fused multiply-add, within the 1e-4 parity tolerance.
long long exact_gemm_limit() {
  static long long v = [] {
    const char* e = getenv("RGC_EXACT_GEMM");
    if (e && std::string(e) == "1") return (long long)1 << 62;
    return (long long)1 << 24;
  }();
  return v;
}

bool tc_disabled() {
  static bool off = [] {
    const char* e = getenv("RGC_NO_TC");
    return e && std::string(e) == "1";
  }();
  return off;
}

Jit& jit() {
  static Jit j;
  return j;
}
std::mutex& jit_mu() {
  static std::mutex m;
  return m;
}

struct Frame;
struct Program;

struct Ctx {
  cudaStream_t s;
  Frame* f;
};

using StepFn = std::function<void(Ctx&)>;

struct Lowered {
  StepFn run;
  // Allocates what the step needs in a frame (nested body frames, staging) before any launch,
  // so that launches can be captured into CUDA graphs.
  std::function<void(Frame*, cudaStream_t)> prepare;
  int kernels = 1;
  bool capturable = true;
  // An NCCL collective: under data parallelism it is launched directly rather than from a CUDA
  // graph, because aborting a communicator whose kernels run inside a graph launch does not
  // return while they wait for a partner that has gone.
  bool collective = false;
};

struct Frame {
  Program* prog = nullptr;
  char* arena = nullptr;
  char* scratch = nullptr;
  std::vector<char*> ptr;
  cudaStream_t stream = nullptr;
  bool failed = false;
  std::string error;
  // Control-flow bodies: one nested frame per body program, created on first use.
  std::unordered_map<const Program*, std::unique_ptr<Frame>> bodies;
  char* staging = nullptr;  // carry copies of a scan body
  size_t staging_bytes = 0;
  // Control-flow bodies captured into conditional graph nodes: the stream their body graph is
  // captured on and a device iteration counter.
  cudaStream_t side = nullptr;
  long long* counter = nullptr;
  cudaGraphConditionalHandle ctl_handle = 0;
  // Pinned host memory for reads that the host polls (step counters, check flags, slot reads
  // under data parallelism): a device-to-host copy into pageable memory blocks the calling thread
  // until the stream reaches it, which behind a stalled collective is never.
  void* pinned = nullptr;
  size_t pinned_bytes = 0;
  void* host_buffer(size_t bytes);
  // What rgc_exec_run sets up, kept between runs on this frame: grow-only device buffers and
  // the step graphs captured for the last run, with the key they were captured for (run spec,
  // buffer addresses) and the two pointer layouts they replay. A run with the same key and
  // layouts (in either order) launches the cached graphs instead of capturing again.
  struct RunPiece {
    cudaGraphExec_t g[2] = {nullptr, nullptr};
    size_t first = 0, last = 0;  // plan steps; a direct piece has last == first + 1
    bool direct = false;
  };
  struct RunCache {
    double* hist = nullptr;
    size_t hist_cap = 0;  // doubles
    long long* ctr = nullptr;
    char* staging = nullptr;
    size_t staging_cap = 0;
    int* types = nullptr;
    void** hptr = nullptr;
    size_t nh_cap = 0;
    char* snap = nullptr;
    size_t snap_cap = 0;
    std::vector<char*> batch;
    std::vector<size_t> batch_cap;
    std::vector<RunPiece> pieces;
    bool alternating = false;
    bool captured = false;
    std::vector<uintptr_t> key;
    std::vector<char*> layout[2];
    void drop_graphs() {
      for (auto& pc : pieces) {
        if (pc.g[0]) cudaGraphExecDestroy(pc.g[0]);
        if (pc.g[1] && pc.g[1] != pc.g[0]) cudaGraphExecDestroy(pc.g[1]);
      }
      pieces.clear();
      captured = false;
      key.clear();
    }
    ~RunCache() {
      drop_graphs();
      for (void* q : {(void*)hist, (void*)ctr, (void*)staging, (void*)types, (void*)hptr, (void*)snap})
        if (q) cudaFree(q);
      for (char* q : batch)
        if (q) cudaFree(q);
    }
  } run;
  ~Frame();
};

struct Program {
  int device = 0;
  Plan plan;
  std::vector<Lowered> steps;
  std::vector<size_t> offsets;
  size_t arena_bytes = 0;
  size_t scratch_bytes = 0;
  bool capturable = true;
  std::vector<std::unique_ptr<Program>> subs;
  FDims* bc_dev = nullptr;  // broadcast descriptors of the fused kernels
  Dims* bc64_dev = nullptr;
  int* tc_error = nullptr;  // set by a tensor-core GEMM whose pipeline wait gave up
  std::mutex mu;
  std::vector<std::unique_ptr<Frame>> pool;
  std::atomic<bool> inject{false};
  std::atomic<uint64_t> launches{0};
  std::atomic<size_t> frames_allocated{0};
  int kernels_per_step = 0;
  ~Program() {
    pool.clear();
    if (bc_dev) cudaFree(bc_dev);
    if (bc64_dev) cudaFree(bc64_dev);
    if (tc_error) cudaFree(tc_error);
  }
};

Frame::~Frame() {
  bodies.clear();
  if (side) cudaStreamDestroy(side);
  if (counter) cudaFree(counter);
  if (stream) cudaStreamDestroy(stream);
  if (arena) cudaFree(arena);
  if (scratch) cudaFree(scratch);
  if (staging) cudaFree(staging);
  if (pinned) cudaFreeHost(pinned);
}

void* Frame::host_buffer(size_t bytes) {
  if (bytes > pinned_bytes) {
    if (pinned) cudaFreeHost(pinned);
    pinned = nullptr;
    pinned_bytes = 0;
    size_t want = std::max<size_t>(bytes, 4096);
    ck(cudaMallocHost(&pinned, want), "cudaMallocHost(frame host buffer)");
    pinned_bytes = want;
  }
  return pinned;
}

// A scalar read by the host between launches (host-driven while / cond), waited for with the
// polled wait that gives up on a stalled collective.
double read_scalar(Frame* f, const void* dev, DType d, cudaStream_t s, const char* what) {
  char* buf = (char*)f->host_buffer(8);
  ck(cudaMemcpyAsync(buf, dev, rg::dtype_size(d), cudaMemcpyDeviceToHost, s), what);
  std::string why;
  cudaError_t err = dist_sync(s, &why);
  if (err != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + (why.empty() ? cudaGetErrorString(err) : why));
  return d == DType::F32 ? (double)*(float*)buf : d == DType::F64 ? *(double*)buf : (double)*(int32_t*)buf;
}

std::unique_ptr<Program> make_program(const Plan& plan, int device);

std::unique_ptr<Frame> make_frame(Program* p, cudaStream_t stream) {
  auto f = std::make_unique<Frame>();
  f->prog = p;
  if (stream) {
    f->stream = nullptr;  // borrowed
  } else {
    ck(cudaStreamCreateWithFlags(&f->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  }
  if (p->arena_bytes) ck(cudaMalloc(&f->arena, p->arena_bytes), "cudaMalloc(frame)");
  if (p->scratch_bytes) ck(cudaMalloc(&f->scratch, p->scratch_bytes), "cudaMalloc(scratch)");
  f->ptr.resize(p->plan.slots.size());
  for (size_t s = 0; s < f->ptr.size(); ++s) f->ptr[s] = f->arena + p->offsets[s];
  cudaStream_t s = stream ? stream : f->stream;
  // Constants stay resident for the frame's life: they are never overwritten.
  for (auto& [slot, t] : p->plan.consts)
    if (t->data.bytes()) ck(cudaMemcpyAsync(f->ptr[slot], t->data.data(), t->data.bytes(), cudaMemcpyHostToDevice, s), "upload constants");
  ck(cudaStreamSynchronize(s), "upload constants");
  p->frames_allocated += 1;
  return f;
}

void prepare_frame(Program* p, Frame* f, cudaStream_t s) {
  for (auto& st : p->steps)
    if (st.prepare) st.prepare(f, s);
}

// The nested frame of a control-flow body, with `staging` bytes for carry copies and, for
// bodies that may be captured into conditional graph nodes, a side stream and a counter.
Frame* body_frame(Frame* parent, Program* body, cudaStream_t s, size_t staging = 0, bool control = false) {
  auto& slot = parent->bodies[body];
  if (!slot) {
    slot = make_frame(body, s);
    prepare_frame(body, slot.get(), s);
  }
  if (control && !slot->side) {
    ck(cudaStreamCreateWithFlags(&slot->side, cudaStreamNonBlocking), "cudaStreamCreate(control flow)");
    ck(cudaMalloc((void**)&slot->counter, sizeof(long long)), "cudaMalloc(iteration counter)");
  }
  if (slot->staging_bytes < staging) {
    if (slot->staging) cudaFree(slot->staging);
    ck(cudaMalloc(&slot->staging, staging), "cudaMalloc(carry staging)");
    slot->staging_bytes = staging;
  }
  return slot.get();
}

void run_steps(Program* p, Ctx& c) {
  for (auto& st : p->steps) st.run(c);
}

Dims dims_of(const std::vector<size_t>& shape, const std::vector<size_t>& st) {
  Dims d;
  if (shape.size() > (size_t)MAXR) throw std::runtime_error("tensor rank above 8 is not supported by the CUDA device");
  d.rank = (int)shape.size();
  for (size_t k = 0; k < shape.size(); ++k) {
    d.d[k] = (long long)shape[k];
    d.st[k] = (long long)st[k];
  }
  return d;
}

// ---- control flow inside CUDA graph capture ----

bool capturing(cudaStream_t s) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  return cudaStreamIsCapturing(s, &st) == cudaSuccess && st == cudaStreamCaptureStatusActive;
}

// Adds a conditional node (type, `bodies` body graphs) after the work captured on `s` so far, makes
// it the capture's only dependency, and returns its handle and body graphs. `prologue` runs on
// `s` before the node is added and receives the handle (to set the condition on the device).
std::vector<cudaGraph_t> add_conditional(cudaStream_t s, cudaGraphConditionalNodeType type, unsigned bodies,
                                         const std::function<void(cudaGraphConditionalHandle)>& prologue) {
  cudaStreamCaptureStatus cs;
  cudaGraph_t graph = nullptr;
  const cudaGraphNode_t* deps = nullptr;
  size_t nd = 0;
  ck(cudaStreamGetCaptureInfo(s, &cs, nullptr, &graph, &deps, &nd), "cudaStreamGetCaptureInfo");
  cudaGraphConditionalHandle h;
  ck(cudaGraphConditionalHandleCreate(&h, graph, 0, 0), "cudaGraphConditionalHandleCreate");
  prologue(h);
  ck(cudaStreamGetCaptureInfo(s, &cs, nullptr, &graph, &deps, &nd), "cudaStreamGetCaptureInfo");
  // Zeroed storage: the parameter union has members with non-trivial constructors in C++.
  alignas(cudaGraphNodeParams) unsigned char storage[sizeof(cudaGraphNodeParams)] = {};
  cudaGraphNodeParams& params = *reinterpret_cast<cudaGraphNodeParams*>(storage);
  params.type = cudaGraphNodeTypeConditional;
  params.conditional.handle = h;
  params.conditional.type = type;
  params.conditional.size = bodies;
  cudaGraphNode_t node;
  ck(cudaGraphAddNode(&node, graph, deps, nd, &params), "cudaGraphAddNode(conditional)");
  ck(cudaStreamUpdateCaptureDependencies(s, &node, 1, cudaStreamSetCaptureDependencies), "cudaStreamUpdateCaptureDependencies");
  return std::vector<cudaGraph_t>(params.conditional.phGraph_out, params.conditional.phGraph_out + bodies);
}

// Captures `fill(side)` into `graph` on the stream `side`.
void capture_into(cudaGraph_t graph, cudaStream_t side, const std::function<void(cudaStream_t)>& fill) {
  ck(cudaStreamBeginCaptureToGraph(side, graph, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCaptureToGraph");
  try {
    fill(side);
  } catch (...) {
    cudaGraph_t g;
    cudaStreamEndCapture(side, &g);
    throw;
  }
  cudaGraph_t g;
  ck(cudaStreamEndCapture(side, &g), "cudaStreamEndCapture(conditional body)");
}

// ---- lowering of one instruction ----

struct Builder {
  Program* p;
  std::vector<FDims> bcs;  // broadcast descriptors, uploaded once per program
  std::vector<Dims> bcs64;
  size_t scratch = 0;

  Lowered elementwise(const ElemSpec& spec, std::vector<size_t> in_slots, std::vector<size_t> out_slots) {
    std::string name;
    {
      std::lock_guard<std::mutex> lk(jit_mu());
      name = jit().add(spec);
    }
    size_t bc0 = bcs.size();
    bool small = spec.n < (1ull << 31);
    // Descriptors in the order of the inputs' `bc` indices (broadcast inputs and full inputs read
    // through their broadcast's source, in input order).
    for (auto& in : spec.inputs)
      if (in.kind == rg::ArgKind::Broadcast || in.via) {
        Dims d = dims_of(spec.shape, rg::bstrides(in.shape, spec.shape.size()));
        bool ok = false;
        bcs.push_back(fast_dims(d, &ok));
        bcs64.push_back(d);
        small = small && ok;
      }
    int vw = spec.dtype == DType::F64 ? 2 : 4;
    bool vec_ok = spec.n % (size_t)vw == 0;
    std::vector<FDiv> rows;
    for (auto& in : spec.inputs)
      rows.push_back(in.kind == rg::ArgKind::Row && in.row > 0 ? make_fdiv(in.row) : in.col ? make_fdiv(in.col) : FDiv{});
    long long n = (long long)spec.n;
    Program* prog = p;
    // The 32-bit-index kernel, or its 64-bit twin (`name_w`) when some index may not fit.
    auto fn = std::make_shared<CUfunction>(nullptr);
    Lowered l;
    l.run = [=](Ctx& c) {
      if (!*fn) {
        std::lock_guard<std::mutex> lk(jit_mu());
        *fn = jit().function(small ? name : name + "_w");
      }
      ElemArgs a;
      std::memset(&a, 0, sizeof a);
      a.n = n;
      a.vec = vec_ok ? 1 : 0;
      a.small = small ? 1 : 0;
      for (size_t k = 0; k < in_slots.size(); ++k) {
        a.in[k] = c.f->ptr[in_slots[k]];
        a.row[k] = rows[k];
      }
      for (size_t q = 0; q < out_slots.size(); ++q) a.out[q] = c.f->ptr[out_slots[q]];
      a.bc = prog->bc_dev + bc0;
      a.bc64 = prog->bc64_dev + bc0;
      if (n > 0) Jit::launch(*fn, a, n, vw, c.s);
    };
    if (in_slots.size() > (size_t)JIT_MAX_IN || out_slots.size() > (size_t)JIT_MAX_OUT)
      throw std::runtime_error("fused group has too many operands for one kernel");
    return l;
  }

  // A row chain as one generated kernel (rowkernel.h).
  Lowered rows(const RowKernel& rk) {
    {
      std::lock_guard<std::mutex> lk(jit_mu());
      jit().add_source(rk.name, rk.source);
    }
    size_t bc0 = bcs.size();
    for (auto& f : rk.bcs) {
      bcs.push_back(f);
      bcs64.push_back(Dims{});  // kept index-aligned with bcs; row kernels use the 32-bit form only
    }
    Program* prog = p;
    auto fn = std::make_shared<CUfunction>(nullptr);
    const std::string name = rk.name;
    const auto ins = rk.in_slots, outs = rk.out_slots;
    const auto divs = rk.in_div;
    const long long rows = rk.rows, blocks = (rk.rows + rk.rows_per_block - 1) / rk.rows_per_block;
    const size_t smem = rk.smem;
    Lowered l;
    l.run = [=](Ctx& c) {
      if (!*fn) {
        std::lock_guard<std::mutex> lk(jit_mu());
        *fn = jit().function(name);
      }
      ElemArgs a;
      std::memset(&a, 0, sizeof a);
      a.n = rows;
      for (size_t k = 0; k < ins.size(); ++k) {
        a.in[k] = c.f->ptr[ins[k]];
        a.row[k] = divs[k];
      }
      for (size_t q = 0; q < outs.size(); ++q) a.out[q] = c.f->ptr[outs[q]];
      a.bc = prog->bc_dev + bc0;
      a.bc64 = prog->bc64_dev + bc0;
      if (rows > 0) Jit::launch_rows(*fn, a, blocks, smem, c.s);
    };
    return l;
  }

  Lowered lower(const Instr& i) {
    Lowered l;
    const auto& a = i.args;
    size_t dst = i.dst;
    EType t = et(i.dtype);
    long long n = (long long)i.n;
    OpKind k = i.op.kind;
    if (i.op.is_unary_elementwise() || i.op.is_binary_elementwise() || k == OpKind::Where) {
      return elementwise(spec_from_instr(i), a, {dst});
    }
    switch (k) {
      case OpKind::Cast: {
        EType st = et(p->plan.slots[a[0]].first);
        l.run = [=](Ctx& c) { cast(c.f->ptr[dst], t, c.f->ptr[a[0]], st, n, c.s); };
        return l;
      }
      case OpKind::Transpose: {
        const auto& perm = i.op.shape;
        size_t r = perm.size();
        bool last2 = r >= 2 && perm[r - 1] == r - 2 && perm[r - 2] == r - 1;
        for (size_t d = 0; last2 && d + 2 < r; ++d) last2 = perm[d] == d;
        if (last2) {
          long long rows = (long long)i.arg_shapes[0][r - 2], cols = (long long)i.arg_shapes[0][r - 1];
          long long batch = rows * cols ? n / (rows * cols) : 0;
          l.run = [=](Ctx& c) { transpose_last2(c.f->ptr[dst], c.f->ptr[a[0]], t, batch, rows, cols, c.s); };
          return l;
        }
        auto src = rg::strides(i.arg_shapes[0]);
        std::vector<size_t> mapped;
        for (size_t q : perm) mapped.push_back(src[q]);
        Dims d = dims_of(i.shape, mapped);
        l.run = [=](Ctx& c) { strided_gather(c.f->ptr[dst], c.f->ptr[a[0]], t, d, 0, n, c.s); };
        return l;
      }
      case OpKind::BroadcastTo: {
        Dims d = dims_of(i.shape, rg::bstrides(i.arg_shapes[0], i.shape.size()));
        l.run = [=](Ctx& c) { strided_gather(c.f->ptr[dst], c.f->ptr[a[0]], t, d, 0, n, c.s); };
        return l;
      }
      case OpKind::Slice: {
        auto src = rg::strides(i.arg_shapes[0]);
        long long base = 0;
        for (size_t q = 0; q < src.size(); ++q) base += (long long)(i.op.starts[q] * src[q]);
        Dims d = dims_of(i.shape, src);
        l.run = [=](Ctx& c) { strided_gather(c.f->ptr[dst], c.f->ptr[a[0]], t, d, base, n, c.s); };
        return l;
      }
      case OpKind::Pad: {
        auto ds = rg::strides(i.shape);
        long long base = 0;
        for (size_t q = 0; q < ds.size(); ++q) base += (long long)(i.op.starts[q] * ds[q]);
        Dims d = dims_of(i.arg_shapes[0], ds);
        long long nin = (long long)rg::product(i.arg_shapes[0]);
        size_t bytes = (size_t)n * esize(t);
        l.kernels = 2;
        l.run = [=](Ctx& c) {
          fill_zero(c.f->ptr[dst], bytes, c.s);
          strided_scatter(c.f->ptr[dst], c.f->ptr[a[0]], t, d, base, nin, c.s);
        };
        return l;
      }
      case OpKind::Concat: {
        auto ds = rg::strides(i.shape);
        size_t axis = i.op.index;
        std::vector<std::pair<Dims, long long>> parts;
        std::vector<long long> counts;
        size_t at = 0;
        for (size_t q = 0; q < a.size(); ++q) {
          parts.emplace_back(dims_of(i.arg_shapes[q], ds), (long long)(at * ds[axis]));
          counts.push_back((long long)rg::product(i.arg_shapes[q]));
          at += i.arg_shapes[q][axis];
        }
        l.kernels = (int)a.size();
        l.run = [=](Ctx& c) {
          for (size_t q = 0; q < a.size(); ++q) strided_scatter(c.f->ptr[dst], c.f->ptr[a[q]], t, parts[q].first, parts[q].second, counts[q], c.s);
        };
        return l;
      }
      case OpKind::Take: {
        const auto& xs = i.arg_shapes[0];
        size_t axis = i.op.index;
        long long block = 1, outer = 1;
        for (size_t q = axis + 1; q < xs.size(); ++q) block *= (long long)xs[q];
        for (size_t q = 0; q < axis; ++q) outer *= (long long)xs[q];
        long long dim = (long long)xs[axis], n_idx = (long long)rg::product(i.arg_shapes[1]);
        l.run = [=](Ctx& c) { take_rows(c.f->ptr[dst], c.f->ptr[a[0]], (const int32_t*)c.f->ptr[a[1]], t, outer, dim, n_idx, block, c.s); };
        return l;
      }
      case OpKind::TakeAlong: {
        long long v = (long long)i.arg_shapes[0].back(), kk = (long long)i.arg_shapes[1].back();
        l.run = [=](Ctx& c) { take_along(c.f->ptr[dst], c.f->ptr[a[0]], (const int32_t*)c.f->ptr[a[1]], t, n, v, kk, c.s); };
        return l;
      }
      case OpKind::TakeGrad: {
        const auto& shape = i.op.shape;
        size_t axis = i.op.index;
        long long block = 1, outer = 1;
        for (size_t q = axis + 1; q < shape.size(); ++q) block *= (long long)shape[q];
        for (size_t q = 0; q < axis; ++q) outer *= (long long)shape[q];
        long long dim = (long long)shape[axis], n_idx = (long long)rg::product(i.arg_shapes[1]);
        scratch = std::max(scratch, take_grad_scratch_bytes(dim, n_idx));
        l.kernels = 5;
        l.run = [=](Ctx& c) {
          take_grad(c.f->ptr[dst], c.f->ptr[a[0]], (const int32_t*)c.f->ptr[a[1]], t, outer, dim, n_idx, block, c.f->scratch, c.s);
        };
        return l;
      }
      case OpKind::TakeAlongGrad: {
        long long v = (long long)i.op.shape.back(), kk = (long long)i.arg_shapes[1].back();
        long long rows = v ? n / v : 0;
        l.run = [=](Ctx& c) { take_along_grad(c.f->ptr[dst], c.f->ptr[a[0]], (const int32_t*)c.f->ptr[a[1]], t, rows, v, kk, c.s); };
        return l;
      }
      case OpKind::MatMul:
      case OpKind::MatMulT:
        return matmul(i, k == OpKind::MatMulT && i.op.flag_a, k == OpKind::MatMulT && i.op.flag_b);
      case OpKind::Reduce:
        return reduce(i);
      case OpKind::Cumsum: {
        long long v = (long long)i.shape.back();
        long long rows = v ? n / v : 0;
        bool rev = i.op.flag_a;
        l.run = [=](Ctx& c) { cumsum(c.f->ptr[dst], c.f->ptr[a[0]], t, rows, v, rev, c.s); };
        return l;
      }
      case OpKind::Argmax: {
        EType st = et(p->plan.slots[a[0]].first);
        long long v = (long long)i.arg_shapes[0].back();
        l.run = [=](Ctx& c) { argmax((int32_t*)c.f->ptr[dst], c.f->ptr[a[0]], st, n, v, c.s); };
        return l;
      }
      case OpKind::ArgTopK: {
        EType st = et(p->plan.slots[a[0]].first);
        long long v = (long long)i.arg_shapes[0].back(), kk = (long long)i.op.index;
        long long rows = kk ? n / kk : 0;
        l.run = [=](Ctx& c) { arg_top_k((int32_t*)c.f->ptr[dst], c.f->ptr[a[0]], st, rows, v, kk, c.s); };
        return l;
      }
      case OpKind::RandUniform:
        l.run = [=](Ctx& c) { rand_uniform(c.f->ptr[dst], (const int32_t*)c.f->ptr[a[0]], t, n, c.s); };
        return l;
      case OpKind::RandNormal:
        l.run = [=](Ctx& c) { rand_normal(c.f->ptr[dst], (const int32_t*)c.f->ptr[a[0]], t, n, c.s); };
        return l;
      case OpKind::KeySplit:
        l.run = [=](Ctx& c) { key_split((int32_t*)c.f->ptr[dst], (const int32_t*)c.f->ptr[a[0]], n / 2, c.s); };
        return l;
      case OpKind::AttnFwd:
      case OpKind::AttnBwd:
        return attention(i);
      case OpKind::Scan:
      case OpKind::While:
      case OpKind::Cond:
        return control(i);
      default:
        throw std::runtime_error(std::string("the CUDA device has no kernel for ") + i.op.name());
    }
  }

  // The device's fused attention (graph.h AttnFwd / AttnBwd; attention.cuh).
  // Whether slot `s` holds a constant (T, T) matrix that is nonzero exactly where j <= i (the
  // causal mask of an attention layer; constants are uploaded once and never rewritten).
  bool causal_constant(size_t s, int T) const {
    for (const auto& [slot, t] : p->plan.consts) {
      if (slot != s) continue;
      if (t->n() != (size_t)T * (size_t)T) return false;
      for (int r = 0; r < T; ++r)
        for (int c = 0; c < T; ++c)
          if ((t->data.get((size_t)r * T + c) != 0.0) != (c <= r)) return false;
      return true;
    }
    return false;
  }

  Lowered attention(const Instr& i) {
    Lowered l;
    const auto& qs = i.arg_shapes[0];
    const size_t r = qs.size();
    const bool packed = i.op.value->n() == 3;  // q, k, v as one (B, T, 3, H, d) tensor (graph.h)
    AttnShape as;
    if (packed) {
      as.heads = (int)i.op.value->data.get(2);
      as.t = (int)qs[1];
      as.d = as.dv = (int)qs[4];
      as.batch = (long long)(qs[0] * qs[3]);
    } else {
      as.t = (int)qs[r - 2];
      as.d = (int)qs[r - 1];
      as.dv = (int)i.arg_shapes[2][r - 1];
      as.batch = (long long)(rg::product(qs) / (qs[r - 2] * qs[r - 1]));
    }
    as.c = (float)i.op.value->data.get(0);
    as.fill = (float)i.op.value->data.get(1);
    if (i.dtype != DType::F32 || (!attention_tc_supported(as) && (as.t > 1024 || packed)))
      throw std::runtime_error(std::string("the CUDA device has no kernel for ") + i.op.name() + " of this dtype, length or layout");
    attention_init();
    const auto a = i.args;
    // Argument slots: q, k, v, mask, fwd, dO; packed: the one qkv slot three times (each part at
    // its offset), then mask, fwd, dO.
    const size_t part = packed ? (size_t)as.heads * as.d : 0;
    const std::vector<size_t> slot = packed ? std::vector<size_t>{a[0], a[0], a[0], a[1], i.op.kind == OpKind::AttnBwd ? a[2] : 0,
                                                                  i.op.kind == OpKind::AttnBwd ? a[3] : 0}
                                            : std::vector<size_t>(a.begin(), a.end());
    as.causal = causal_constant(slot[3], as.t);
    const size_t dst = i.dst;
    if (i.op.kind == OpKind::AttnFwd) {
      l.run = [=](Ctx& c) {
        const float* q = (const float*)c.f->ptr[slot[0]];
        attention_fwd((float*)c.f->ptr[dst], q, (const float*)c.f->ptr[slot[1]] + part, (const float*)c.f->ptr[slot[2]] + 2 * part,
                      (const float*)c.f->ptr[slot[3]], as, c.f->prog->tc_error, c.s);
      };
    } else {
      l.kernels = 2;
      scratch = std::max(scratch, attention_bwd_scratch_bytes(as));
      l.run = [=](Ctx& c) {
        const float* q = (const float*)c.f->ptr[slot[0]];
        attention_bwd((float*)c.f->ptr[dst], q, (const float*)c.f->ptr[slot[1]] + part, (const float*)c.f->ptr[slot[2]] + 2 * part,
                      (const float*)c.f->ptr[slot[3]], (const float*)c.f->ptr[slot[4]], (const float*)c.f->ptr[slot[5]], as, c.f->scratch,
                      c.f->prog->tc_error, c.s);
      };
    }
    return l;
  }

  // plan.rs:1453-1493
  Lowered matmul(const Instr& i, bool ta, bool tb) {
    Lowered l;
    const auto &sa = i.arg_shapes[0], &sb = i.arg_shapes[1];
    size_t ar = sa.size(), br = sb.size();
    long long m, kk, n;
    if (ar >= 2) {
      m = (long long)(ta ? sa[ar - 1] : sa[ar - 2]);
      kk = (long long)(ta ? sa[ar - 2] : sa[ar - 1]);
    } else {
      m = 1;
      kk = (long long)sa[0];
    }
    n = br >= 2 ? (long long)(tb ? sb[br - 2] : sb[br - 1]) : 1;
    std::vector<size_t> ba(sa.begin(), sa.end() - std::min<size_t>(2, ar));
    std::vector<size_t> bb(sb.begin(), sb.end() - std::min<size_t>(2, br));
    GemmBatch bt;
    long long count = 1;
    if (bb.empty() && !ta) {
      m *= (long long)rg::product(ba);  // row-major batches of A form one matrix
    } else {
      std::vector<size_t> batch;
      rg::broadcast_shapes(ba, bb, &batch);
      if (batch.size() > (size_t)MAXR) throw std::runtime_error("matmul batch rank above 8");
      auto st_a = rg::bstrides(ba, batch.size()), st_b = rg::bstrides(bb, batch.size());
      bt.rank = (int)batch.size();
      for (size_t d = 0; d < batch.size(); ++d) {
        bt.d[d] = (long long)batch[d];
        bt.sa[d] = (long long)st_a[d] * m * kk;
        bt.sb[d] = (long long)st_b[d] * kk * n;
      }
      count = (long long)rg::product(batch);
    }
    EType t = et(i.dtype);
    bool exact = m * n * kk * count <= exact_gemm_limit();
    size_t dst = i.dst, A = i.args[0], B = i.args[1];
    // Large fp32 products run on the tensor cores (3xTF32) when their batch folds into one
    // strided dimension; small ones keep rg's exact loop arithmetic on the SIMT cores.
    TcGemm tg;
    tg.m = m;
    tg.n = n;
    tg.k = kk;
    tg.ta = ta;
    tg.tb = tb;
    bool foldable = true;
    if (bt.rank == 0) {
      tg.batch = 1;
    } else {
      // Fold adjacent batch dims whose strides chain for both operands.
      long long d = bt.d[bt.rank - 1], sa_ = bt.sa[bt.rank - 1], sb_ = bt.sb[bt.rank - 1];
      for (int q = bt.rank - 2; q >= 0 && foldable; --q) {
        bool chain_a = bt.sa[q] == sa_ * d || (bt.sa[q] == 0 && sa_ == 0);
        bool chain_b = bt.sb[q] == sb_ * d || (bt.sb[q] == 0 && sb_ == 0);
        foldable = chain_a && chain_b;
        d *= bt.d[q];
      }
      tg.batch = count;
      tg.batch_a = sa_;
      tg.batch_b = sb_;
    }
    bool use_tc = !tc_disabled() && t == EType::F32 && !exact && foldable && tc_gemm_supported(tg);
    if (use_tc) {
      tc_gemm_init();
      scratch = std::max(scratch, tc_gemm_scratch_bytes(tg));
      l.kernels = tc_gemm_launches(tg);
      l.run = [=](Ctx& c) {
        TcGemm g = tg;
        g.a = (const float*)c.f->ptr[A];
        g.b = (const float*)c.f->ptr[B];
        g.c = (float*)c.f->ptr[dst];
        tc_gemm(g, c.f->scratch, c.f->prog->tc_error, c.s);
      };
      return l;
    }
    l.run = [=](Ctx& c) { gemm(c.f->ptr[dst], c.f->ptr[A], c.f->ptr[B], t, m, n, kk, ta, tb, bt, count, exact, c.s); };
    return l;
  }

  // plan.rs:1549-1622, routed by the shape of the reduced axis set.
  Lowered reduce(const Instr& i) {
    Lowered l;
    const auto& in_shape = i.arg_shapes[0];
    std::vector<size_t> axes = i.op.shape;
    std::sort(axes.begin(), axes.end());
    size_t r = in_shape.size();
    EType t = et(i.dtype);
    Red op = i.op.reduce == rg::ReduceKind::Sum ? Red::Sum : i.op.reduce == rg::ReduceKind::Max ? Red::Max : Red::Min;
    size_t dst = i.dst, src = i.args[0];
    long long n_in = (long long)rg::product(in_shape);
    if (op == Red::Sum && axes.size() == r) {
      scratch = std::max(scratch, full_sum_scratch_bytes(n_in, t));
      l.kernels = n_in > 32768 ? 2 : 1;
      l.run = [=](Ctx& c) { reduce_full_sum(c.f->ptr[dst], c.f->ptr[src], t, n_in, c.f->scratch, c.s); };
      return l;
    }
    // Dims of extent 1 do not change the memory order; drop them before matching patterns.
    std::vector<bool> red(r, false);
    for (size_t ax : axes) red[ax] = true;
    std::vector<size_t> keep_idx, red_idx;
    for (size_t d = 0; d < r; ++d)
      if (in_shape[d] != 1) (red[d] ? red_idx : keep_idx).push_back(d);
    long long n_out = (long long)i.n;
    auto contiguous = [](const std::vector<size_t>& v) {
      for (size_t q = 1; q < v.size(); ++q)
        if (v[q] < v[q - 1]) return false;
      return true;
    };
    bool trailing = !red_idx.empty() && (keep_idx.empty() || keep_idx.back() < red_idx.front()) && contiguous(red_idx);
    bool leading = !red_idx.empty() && !keep_idx.empty() && red_idx.back() < keep_idx.front();
    long long n_red = 1;
    for (size_t d : red_idx) n_red *= (long long)in_shape[d];
    if (red_idx.empty()) {
      // Reducing only extent-1 axes: an elementwise combine with the identity.
      long long nn = n_out;
      l.run = [=](Ctx& c) { reduce_rows(c.f->ptr[dst], c.f->ptr[src], t, op, nn, 1, c.s); };
      return l;
    }
    if (trailing) {
      long long rows = n_out, len = n_red;
      l.run = [=](Ctx& c) { reduce_rows(c.f->ptr[dst], c.f->ptr[src], t, op, rows, len, c.s); };
      return l;
    }
    if (leading) {
      long long rows = n_red, cols = n_out;
      // rg's parallel path chunks only when every axis but the last is reduced (plan.rs:1593).
      const bool chunked = axes.size() + 1 == r && !red[r - 1];
      scratch = std::max(scratch, cols_scratch_bytes(rows, cols, t));
      l.kernels = 2;
      l.run = [=](Ctx& c) { reduce_cols(c.f->ptr[dst], c.f->ptr[src], t, op, rows, cols, chunked, c.f->scratch, c.s); };
      return l;
    }
    auto st = rg::strides(in_shape);
    std::vector<size_t> kd, ks, rd, rs;
    for (size_t d : keep_idx) {
      kd.push_back(in_shape[d]);
      ks.push_back(st[d]);
    }
    for (size_t d : red_idx) {
      rd.push_back(in_shape[d]);
      rs.push_back(st[d]);
    }
    Dims kept = dims_of(kd, ks), reduced = dims_of(rd, rs);
    l.run = [=](Ctx& c) { reduce_generic(c.f->ptr[dst], c.f->ptr[src], t, op, kept, reduced, n_out, c.s); };
    return l;
  }

  // plan.rs:737-831 on device buffers; the host only sequences the iterations.
  Lowered control(const Instr& i) {
    Lowered l;
    Program* parent = p;
    if (i.op.kind == OpKind::Scan) {
      p->subs.push_back(make_program(*i.body_plan, p->device));
      Program* body = p->subs.back().get();
      size_t c = i.op.n_carry, x = i.op.n_x, length = i.op.length;
      bool reverse = i.op.flag_a;
      auto args = i.args;
      auto outs = i.outs;
      size_t n_y = body->plan.outputs.size() - c;
      std::vector<size_t> es;
      for (size_t q = 0; q < body->plan.input_slots.size(); ++q) es.push_back(rg::dtype_size(body->plan.slots[body->plan.input_slots[q]].first));
      l.capturable = body->capturable;
      l.kernels = 0;
      size_t carry_bytes = 0;
      for (size_t k = 0; k < c; ++k) carry_bytes += align_up(body->plan.outputs[k].n * es[k]);
      l.prepare = [=](Frame* f, cudaStream_t st) { body_frame(f, body, st, carry_bytes); };
      l.run = [=](Ctx& cx) {
        Frame* bf = body_frame(cx.f, body, cx.s, carry_bytes);
        const Plan& bp = body->plan;
        auto cp = [&](void* d, const void* s, size_t bytes) {
          if (bytes) ck(cudaMemcpyAsync(d, s, bytes, cudaMemcpyDeviceToDevice, cx.s), "scan copy");
        };
        for (size_t k = 0; k < args.size(); ++k)
          if (k < c || k >= c + x) cp(bf->ptr[bp.input_slots[k]], cx.f->ptr[args[k]], bp.input_ns[k] * es[k]);
        Ctx inner{cx.s, bf};
        for (size_t st = 0; st < length; ++st) {
          size_t at = reverse ? length - 1 - st : st;
          for (size_t k = c; k < c + x; ++k) {
            size_t m = bp.input_ns[k] * es[k];
            cp(bf->ptr[bp.input_slots[k]], cx.f->ptr[args[k]] + at * m, m);
          }
          for (auto& [index, slot] : outs) {
            if (index >= c + n_y) {
              size_t k = index - c - n_y;
              size_t m = bp.input_ns[k] * es[k];
              cp(cx.f->ptr[slot] + at * m, bf->ptr[bp.input_slots[k]], m);
            }
          }
          run_steps(body, inner);
          for (auto& [index, slot] : outs) {
            if (index >= c && index < c + n_y) {
              const auto& o = bp.outputs[index];
              size_t eb = rg::dtype_size(bp.slots[o.slot].first);
              cp(cx.f->ptr[slot] + at * o.n * eb, bf->ptr[o.slot], o.n * eb);
            }
          }
          // Body outputs feed the carries through staging: an output may be another carry's input.
          size_t off = 0;
          for (size_t k = 0; k < c; ++k) {
            cp(bf->staging + off, bf->ptr[bp.outputs[k].slot], bp.outputs[k].n * es[k]);
            off += align_up(bp.outputs[k].n * es[k]);
          }
          off = 0;
          for (size_t k = 0; k < c; ++k) {
            cp(bf->ptr[bp.input_slots[k]], bf->staging + off, bp.outputs[k].n * es[k]);
            off += align_up(bp.outputs[k].n * es[k]);
          }
        }
        for (auto& [index, slot] : outs)
          if (index < c) cp(cx.f->ptr[slot], bf->ptr[bp.input_slots[index]], bp.input_ns[index] * es[index]);
      };
      (void)parent;
      return l;
    }
    if (i.op.kind == OpKind::While) {
      p->subs.push_back(make_program(*i.body_plan, p->device));
      Program* cond = p->subs.back().get();
      p->subs.push_back(make_program(*i.body2_plan, p->device));
      Program* body = p->subs.back().get();
      auto args = i.args;
      auto outs = i.outs;
      size_t n_carry = i.op.n_carry, max_it = i.op.max_iterations;
      // Inside graph capture the loop becomes a conditional WHILE node whose condition a kernel
      // sets on the device; run directly, the host reads the condition each iteration.
      l.capturable = cond->capturable && body->capturable;
      l.kernels = 0;
      auto bytes_of = [](const Plan& pl, size_t k) { return pl.input_ns[k] * rg::dtype_size(pl.slots[pl.input_slots[k]].first); };
      size_t carry_bytes = 0;
      for (size_t k = 0; k < n_carry; ++k) carry_bytes += align_up(bytes_of(body->plan, k));
      l.prepare = [=](Frame* f, cudaStream_t st) {
        body_frame(f, cond, st);
        body_frame(f, body, st, carry_bytes, true);
      };
      l.run = [=](Ctx& cx) {
        Frame* cf = body_frame(cx.f, cond, cx.s);
        Frame* bf = body_frame(cx.f, body, cx.s, carry_bytes, true);
        const Plan& cp_ = cond->plan;
        const Plan& bp = body->plan;
        auto cp_on = [&](cudaStream_t st, void* d, const void* s, size_t bytes) {
          if (bytes) ck(cudaMemcpyAsync(d, s, bytes, cudaMemcpyDeviceToDevice, st), "while copy");
        };
        auto cp = [&](void* d, const void* s, size_t bytes) { cp_on(cx.s, d, s, bytes); };
        for (size_t k = 0; k < args.size(); ++k) {
          cp(cf->ptr[cp_.input_slots[k]], cx.f->ptr[args[k]], bytes_of(cp_, k));
          cp(bf->ptr[bp.input_slots[k]], cx.f->ptr[args[k]], bytes_of(bp, k));
        }
        const auto& co = cp_.outputs[0];
        const EType ct = et(cp_.slots[co.slot].first);
        if (capturing(cx.s)) {
          auto graphs = add_conditional(cx.s, cudaGraphCondTypeWhile, 1, [&](cudaGraphConditionalHandle h) {
            ck(cudaMemsetAsync(bf->counter, 0, sizeof(long long), cx.s), "while counter");
            Ctx ci{cx.s, cf};
            run_steps(cond, ci);
            set_conditional(h, cf->ptr[co.slot], ct, bf->counter, (long long)max_it, false, cx.s);
            bf->ctl_handle = h;
          });
          const cudaGraphConditionalHandle h = bf->ctl_handle;
          capture_into(graphs[0], bf->side, [&](cudaStream_t st) {
            Ctx bi{st, bf}, ci{st, cf};
            run_steps(body, bi);
            size_t off = 0;
            for (size_t k = 0; k < n_carry; ++k) {
              cp_on(st, bf->staging + off, bf->ptr[bp.outputs[k].slot], bytes_of(bp, k));
              off += align_up(bytes_of(bp, k));
            }
            off = 0;
            for (size_t k = 0; k < n_carry; ++k) {
              cp_on(st, bf->ptr[bp.input_slots[k]], bf->staging + off, bytes_of(bp, k));
              cp_on(st, cf->ptr[cp_.input_slots[k]], bf->staging + off, bytes_of(bp, k));
              off += align_up(bytes_of(bp, k));
            }
            run_steps(cond, ci);
            set_conditional(h, cf->ptr[co.slot], ct, bf->counter, (long long)max_it, true, st);
          });
          for (auto& [index, slot] : outs) {
            if (index < n_carry) cp(cx.f->ptr[slot], bf->ptr[bp.input_slots[index]], bytes_of(bp, index));
            else write_count((int32_t*)cx.f->ptr[slot], bf->counter, cx.s);
          }
          return;
        }
        Ctx ci{cx.s, cf}, bi{cx.s, bf};
        size_t count = 0;
        for (;;) {
          run_steps(cond, ci);
          const auto& o = cp_.outputs[0];
          double v = 0;
          DType d = cp_.slots[o.slot].first;
          v = read_scalar(cx.f, cf->ptr[o.slot], d, cx.s, "while condition");
          if (v == 0.0) break;
          if (count == max_it) break;
          run_steps(body, bi);
          size_t off = 0;
          for (size_t k = 0; k < n_carry; ++k) {
            cp(bf->staging + off, bf->ptr[bp.outputs[k].slot], bytes_of(bp, k));
            off += align_up(bytes_of(bp, k));
          }
          off = 0;
          for (size_t k = 0; k < n_carry; ++k) {
            cp(bf->ptr[bp.input_slots[k]], bf->staging + off, bytes_of(bp, k));
            cp(cf->ptr[cp_.input_slots[k]], bf->staging + off, bytes_of(bp, k));
            off += align_up(bytes_of(bp, k));
          }
          count += 1;
        }
        for (auto& [index, slot] : outs) {
          if (index < n_carry) {
            cp(cx.f->ptr[slot], bf->ptr[bp.input_slots[index]], bytes_of(bp, index));
          } else {
            int32_t cnt = (int32_t)count;
            ck(cudaMemcpyAsync(cx.f->ptr[slot], &cnt, 4, cudaMemcpyHostToDevice, cx.s), "while count");
            ck(cudaStreamSynchronize(cx.s), "while count");
          }
        }
      };
      return l;
    }
    // Cond
    p->subs.push_back(make_program(*i.body_plan, p->device));
    Program* then_p = p->subs.back().get();
    p->subs.push_back(make_program(*i.body2_plan, p->device));
    Program* else_p = p->subs.back().get();
    auto args = i.args;
    auto outs = i.outs;
    DType pd = p->plan.slots[args[0]].first;
    // Inside graph capture: a conditional IF node with an else body; run directly, the host
    // reads the predicate.
    l.capturable = then_p->capturable && else_p->capturable;
    l.kernels = 0;
    l.prepare = [=](Frame* f, cudaStream_t st) {
      body_frame(f, then_p, st, 0, true);
      body_frame(f, else_p, st, 0, true);
    };
    l.run = [=](Ctx& cx) {
      auto branch = [&](Program* body, cudaStream_t st) {
        Frame* bf = body_frame(cx.f, body, cx.s, 0, true);
        const Plan& bp = body->plan;
        for (size_t k = 0; k + 1 < args.size(); ++k) {
          size_t bytes = bp.input_ns[k] * rg::dtype_size(bp.slots[bp.input_slots[k]].first);
          if (bytes) ck(cudaMemcpyAsync(bf->ptr[bp.input_slots[k]], cx.f->ptr[args[k + 1]], bytes, cudaMemcpyDeviceToDevice, st), "cond copy");
        }
        Ctx inner{st, bf};
        run_steps(body, inner);
        for (auto& [index, slot] : outs) {
          const auto& o = bp.outputs[index];
          size_t bytes = o.n * rg::dtype_size(bp.slots[o.slot].first);
          if (bytes) ck(cudaMemcpyAsync(cx.f->ptr[slot], bf->ptr[o.slot], bytes, cudaMemcpyDeviceToDevice, st), "cond copy");
        }
      };
      if (capturing(cx.s)) {
        auto graphs = add_conditional(cx.s, cudaGraphCondTypeIf, 2, [&](cudaGraphConditionalHandle h) {
          set_conditional(h, cx.f->ptr[args[0]], et(pd), nullptr, 0, false, cx.s);
        });
        capture_into(graphs[0], body_frame(cx.f, then_p, cx.s, 0, true)->side, [&](cudaStream_t st) { branch(then_p, st); });
        capture_into(graphs[1], body_frame(cx.f, else_p, cx.s, 0, true)->side, [&](cudaStream_t st) { branch(else_p, st); });
        return;
      }
      double v = read_scalar(cx.f, cx.f->ptr[args[0]], pd, cx.s, "cond predicate");
      Program* body = v != 0.0 ? then_p : else_p;
      Frame* bf = body_frame(cx.f, body, cx.s);
      const Plan& bp = body->plan;
      for (size_t k = 0; k + 1 < args.size(); ++k) {
        size_t bytes = bp.input_ns[k] * rg::dtype_size(bp.slots[bp.input_slots[k]].first);
        if (bytes) ck(cudaMemcpyAsync(bf->ptr[bp.input_slots[k]], cx.f->ptr[args[k + 1]], bytes, cudaMemcpyDeviceToDevice, cx.s), "cond copy");
      }
      Ctx inner{cx.s, bf};
      run_steps(body, inner);
      for (auto& [index, slot] : outs) {
        const auto& o = bp.outputs[index];
        size_t bytes = o.n * rg::dtype_size(bp.slots[o.slot].first);
        if (bytes) ck(cudaMemcpyAsync(cx.f->ptr[slot], bf->ptr[o.slot], bytes, cudaMemcpyDeviceToDevice, cx.s), "cond copy");
      }
    };
    return l;
  }
};

std::unique_ptr<Program> make_program(const Plan& plan, int device) {
  auto p = std::make_unique<Program>();
  p->device = device;
  p->plan = plan;
  ck(cudaMalloc((void**)&p->tc_error, sizeof(int)), "cudaMalloc(error flag)");
  ck(cudaMemset(p->tc_error, 0, sizeof(int)), "cudaMemset(error flag)");
  p->offsets.resize(plan.slots.size());
  size_t off = 0;
  for (size_t s = 0; s < plan.slots.size(); ++s) {
    p->offsets[s] = off;
    off += align_up(std::max<size_t>(1, plan.slots[s].second) * rg::dtype_size(plan.slots[s].first));
  }
  p->arena_bytes = off;
  Builder b{p.get()};
  // The plan step that last wrote each slot, as steps are lowered in order. A full input of an
  // elementwise step whose slot holds a BroadcastTo of a constant or an input (pinned slots, never
  // rewritten during a step) is read from the broadcast's source through broadcast indexing: the
  // same values without reading the full-size copy (an attention layer's causal mask and fill
  // constants, read again by every layer). The BroadcastTo steps themselves still run, so every
  // slot holds what the plan says it holds.
  std::vector<long> last_writer(plan.slots.size(), -1);
  auto note_writes = [&](size_t k) {
    const auto& st = plan.steps[k];
    if (st.fused) {
      for (auto& o : st.group.outputs) last_writer[o.second] = (long)k;
      return;
    }
    if (st.instr.dst < last_writer.size()) last_writer[st.instr.dst] = (long)k;
    for (auto& [index, slot] : st.instr.outs) {
      (void)index;
      if (slot < last_writer.size()) last_writer[slot] = (long)k;
    }
  };
  auto read_broadcast_sources = [&](ElemSpec& spec, std::vector<size_t>& ins) {
    bool any = false;
    for (size_t j = 0; j < spec.inputs.size() && j < ins.size(); ++j) {
      auto& in = spec.inputs[j];
      if (in.kind != rg::ArgKind::Full || last_writer[ins[j]] < 0) continue;
      const rg::Step& w = plan.steps[(size_t)last_writer[ins[j]]];
      if (w.fused || w.instr.op.kind != OpKind::BroadcastTo || w.instr.args.size() != 1) continue;
      const size_t src = w.instr.args[0];
      if (src >= plan.pinned.size() || !plan.pinned[src] || plan.slots[src].first != spec.dtype || w.instr.shape != spec.shape) continue;
      in.via = true;
      in.shape = w.instr.arg_shapes[0];
      in.col = column_of(in.shape, spec.shape);
      ins[j] = src;
      any = true;
    }
    if (!any) return;
    int nbc = 0;
    for (auto& in : spec.inputs)
      if (in.kind == rg::ArgKind::Broadcast || in.via) in.bc = nbc++;
  };
  // One step that is neither an all-reduce nor part of a row chain.
  auto lower_one = [&](size_t k) -> Lowered {
    const auto& st = plan.steps[k];
    if (st.fused) {
      std::vector<size_t> ins, outs;
      for (auto& in : st.group.inputs) ins.push_back(in.slot);
      for (auto& o : st.group.outputs) outs.push_back(o.second);
      ElemSpec spec = spec_from_group(st.group);
      read_broadcast_sources(spec, ins);
      return b.elementwise(spec, ins, outs);
    }
    if (st.instr.op.is_unary_elementwise() || st.instr.op.is_binary_elementwise() || st.instr.op.kind == OpKind::Where) {
      std::vector<size_t> ins = st.instr.args;
      ElemSpec spec = spec_from_instr(st.instr);
      read_broadcast_sources(spec, ins);
      return b.elementwise(spec, ins, {st.instr.dst});
    }
    return b.lower(st.instr);
  };
  const std::vector<rg::RowChain> chains = rg::find_row_chains(plan, true);
  size_t next_chain = 0;
  for (size_t k = 0; k < plan.steps.size(); ++k) {
    const auto& st = plan.steps[k];
    if (next_chain < chains.size() && chains[next_chain].first == k) {
      const rg::RowChain& c = chains[next_chain++];
      RowKernel rk;
      std::string why;
      if (make_row_kernel(plan, c, &rk, &why)) {
        // The steps of the range in plan order (so that broadcast sources resolve as they would
        // step by step): the ones that run before the chain, the chain, the ones that run after.
        std::vector<Lowered> pre, post;
        for (size_t q = c.first; q <= c.last; ++q) {
          if (std::find(c.before.begin(), c.before.end(), q) != c.before.end()) pre.push_back(lower_one(q));
          else if (std::find(c.after.begin(), c.after.end(), q) != c.after.end()) post.push_back(lower_one(q));
          note_writes(q);
        }
        Lowered chain = b.rows(rk);
        Lowered all;
        all.kernels = chain.kernels;
        all.capturable = true;
        std::vector<std::function<void(Frame*, cudaStream_t)>> preps;
        for (auto* part : {&pre, &post})
          for (auto& l : *part) {
            all.kernels += l.kernels;
            all.capturable = all.capturable && l.capturable;
            if (l.prepare) preps.push_back(l.prepare);
          }
        all.run = [pre, chain, post](Ctx& cx) {
          for (auto& l : pre) l.run(cx);
          chain.run(cx);
          for (auto& l : post) l.run(cx);
        };
        if (!preps.empty())
          all.prepare = [preps](Frame* f, cudaStream_t s) {
            for (auto& pf : preps) pf(f, s);
          };
        p->steps.push_back(std::move(all));
        // The chain stands for every step of its range: keep step indices aligned.
        for (size_t q = c.first + 1; q <= c.last; ++q) {
          Lowered empty;
          empty.kernels = 0;
          empty.run = [](Ctx&) {};
          p->steps.push_back(std::move(empty));
        }
        k = c.last;
        continue;
      }
    }
    if (!st.fused && st.instr.op.kind == OpKind::AllReduce) {
      // Consecutive all-reduces (a model's gradients): the f32 ones are gathered into one
      // contiguous buffer (the frame's scratch, 256-byte aligned segments), all-reduced as one
      // NCCL operation and scattered to their destinations; one operation of 150 MB runs at
      // link bandwidth, while a group of 150 small ones pays a latency per operation. Sources
      // are all read before any destination is written, so slots the plan reuses between the
      // steps (a later destination in an earlier source's slot) are safe; a run is cut before
      // a destination that meets an earlier destination of the run. f64 items reduce alone.
      struct Item {
        size_t src, dst, n;
        bool f64;
      };
      std::vector<Item> all;
      while (k < plan.steps.size() && !plan.steps[k].fused && plan.steps[k].instr.op.kind == OpKind::AllReduce) {
        const Instr& i = plan.steps[k].instr;
        all.push_back(Item{i.args[0], i.dst, i.n, i.dtype == DType::F64});
        note_writes(k);
        ++k;
      }
      --k;
      auto emit = [&](std::vector<Item> items, bool staged) {
        if (items.empty()) return;
        std::vector<size_t> offsets;  // staged: each item's place in the contiguous buffer (floats)
        size_t total = 0;
        for (auto& it : items) {
          offsets.push_back(total);
          total += (it.n + 63) / 64 * 64;
        }
        if (staged) b.scratch = std::max(b.scratch, total * sizeof(float));
        Lowered l;
        l.kernels = (int)items.size();
        l.collective = true;
        l.run = [items, offsets, total, staged](Ctx& c) {
          if (dist_aborted()) throw std::runtime_error("the data-parallel communicator was aborted after a stalled collective");
          if (!dist_active()) {
            for (auto& it : items)
              ck(cudaMemcpyAsync(c.f->ptr[it.dst], c.f->ptr[it.src], it.n * (it.f64 ? 8 : 4), cudaMemcpyDeviceToDevice, c.s), "all_reduce copy");
            return;
          }
          if (!staged) {
            for (auto& it : items) dist_all_reduce_into(c.f->ptr[it.dst], c.f->ptr[it.src], it.n, it.f64, c.s);
            return;
          }
          float* stage = (float*)c.f->scratch;
          for (int pass = 0; pass < 2; ++pass) {  // gather, then (after the all-reduce) scatter
            if (pass == 1) dist_all_reduce(stage, total, false, c.s);
            for (size_t q = 0; q < items.size(); q += SEGMENTS_MAX) {
              Segments g;
              g.n = (int)std::min<size_t>(SEGMENTS_MAX, items.size() - q);
              for (int j = 0; j < g.n; ++j) {
                float* dev = (float*)c.f->ptr[pass ? items[q + j].dst : items[q + j].src];
                g.src[j] = pass ? stage + offsets[q + j] : dev;
                g.dst[j] = pass ? dev : stage + offsets[q + j];
                g.count[j] = (long long)items[q + j].n;
              }
              ck(copy_segments(g, c.s), pass ? "all_reduce scatter" : "all_reduce gather");
            }
          }
        };
        p->steps.push_back(std::move(l));
        // The grouped step stands for several plan steps: keep step indices aligned.
        for (size_t q = 1; q < items.size(); ++q) {
          Lowered empty;
          empty.kernels = 0;
          empty.run = [](Ctx&) {};
          p->steps.push_back(std::move(empty));
        }
      };
      std::vector<Item> run;
      std::vector<size_t> dsts;
      for (auto& it : all) {
        if (it.f64) {
          emit(std::move(run), true);
          run.clear();
          dsts.clear();
          emit({it}, false);
          continue;
        }
        if (std::find(dsts.begin(), dsts.end(), it.dst) != dsts.end()) {
          emit(std::move(run), true);
          run.clear();
          dsts.clear();
        }
        run.push_back(it);
        dsts.push_back(it.dst);
      }
      emit(std::move(run), true);
      continue;
    }
    p->steps.push_back(lower_one(k));
    note_writes(k);
  }
  {
    std::lock_guard<std::mutex> lk(jit_mu());
    jit().build();
  }
  if (!b.bcs.empty()) {
    ck(cudaMalloc(&p->bc_dev, b.bcs.size() * sizeof(FDims)), "cudaMalloc(broadcast descriptors)");
    ck(cudaMemcpy(p->bc_dev, b.bcs.data(), b.bcs.size() * sizeof(FDims), cudaMemcpyHostToDevice), "upload broadcast descriptors");
    ck(cudaMalloc(&p->bc64_dev, b.bcs64.size() * sizeof(Dims)), "cudaMalloc(broadcast descriptors)");
    ck(cudaMemcpy(p->bc64_dev, b.bcs64.data(), b.bcs64.size() * sizeof(Dims), cudaMemcpyHostToDevice), "upload broadcast descriptors");
  }
  p->scratch_bytes = b.scratch;
  p->capturable = true;
  p->kernels_per_step = 0;
  for (auto& st : p->steps) {
    p->capturable = p->capturable && st.capturable;
    p->kernels_per_step += st.kernels;
  }
  return p;
}

bool graphs_enabled() {
  static bool on = [] {
    const char* e = getenv("RGC_NO_GRAPH");
    return !(e && std::string(e) == "1");
  }();
  return on;
}

}  // namespace

}  // namespace rgc

// ---------------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------------

using namespace rgc;

struct rgc_program {
  std::unique_ptr<Program> p;
};

struct rgc_exec {
  rgc_program* owner = nullptr;
  std::unique_ptr<Frame> f;
};

namespace {

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

template <typename F> int guard(F f) {
  try {
    g_last_error.clear();
    return f();
  } catch (const CudaError& e) {
    return fail(RGC_ERR_CUDA, e.what());
  } catch (const std::exception& e) {
    return fail(RGC_ERR_INVALID, e.what());
  }
}

void mark_failed(rgc_exec* e, const std::string& why) {
  if (!e->f->failed) {
    e->f->failed = true;
    e->f->error = why;
  }
}

// Launches one plan step sequence on the frame's stream with the current layout.
void launch_plan(rgc_exec* e) {
  Program* p = e->owner->p.get();
  Ctx c{e->f->stream, e->f.get()};
  run_steps(p, c);
  p->launches += (uint64_t)p->kernels_per_step;
}

// A tensor-core GEMM whose pipeline wait gave up leaves a code in the program's error flag.
void check_tc_error(rgc_exec* e) {
  int code = 0;
  if (cudaMemcpy(&code, e->owner->p->tc_error, sizeof code, cudaMemcpyDeviceToHost) == cudaSuccess && code)
    mark_failed(e, "tensor-core kernel pipeline wait timed out (stage " + std::to_string(code) + ")");
}

void check_async(rgc_exec* e) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) mark_failed(e, std::string("kernel launch failed: ") + cudaGetErrorString(err));
}

cudaGraphExec_t capture(cudaStream_t s, const std::function<void(cudaStream_t)>& body) {
  cudaGraph_t graph;
  ck(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  try {
    body(s);
  } catch (...) {
    cudaGraph_t g2;
    cudaStreamEndCapture(s, &g2);
    if (g2) cudaGraphDestroy(g2);
    throw;
  }
  ck(cudaStreamEndCapture(s, &graph), "cudaStreamEndCapture");
  cudaGraphExec_t exec;
  ck(cudaGraphInstantiate(&exec, graph, 0), "cudaGraphInstantiate");
  cudaGraphDestroy(graph);
  return exec;
}

}  // namespace

// For entry points defined in other files of this library: sets (or, with an empty message,
// clears) what rgc_last_error reports on this thread, and returns `code`.
namespace rgc {
int set_last_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
}  // namespace rgc

extern "C" {

__attribute__((visibility("default"))) int rgc_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  return major == 10 ? 1 : 0;
}

__attribute__((visibility("default"))) const char* rgc_last_error(void) { return g_last_error.c_str(); }

__attribute__((visibility("default"))) int rgc_program_create(const uint8_t* blob, size_t len, int device, rgc_program** out) {
  return guard([&] {
    if (!blob || !out) return fail(RGC_ERR_INVALID, "null argument");
    if (!rgc_available()) return fail(RGC_ERR_UNAVAILABLE, "no sm_100 CUDA device is available");
    int dev = device;
    if (dev < 0) ck(cudaGetDevice(&dev), "cudaGetDevice");
    // Makes the device's primary context current: the JIT loads modules through the driver API.
    ck(cudaSetDevice(dev), "cudaSetDevice");
    ck(cudaFree(nullptr), "CUDA context initialisation");
    Plan plan = rg::decode_plan(blob, len);
    auto p = make_program(plan, dev);
    *out = new rgc_program{std::move(p)};
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) void rgc_program_destroy(rgc_program* p) {
  if (!p) return;
  cudaDeviceSynchronize();
  delete p;
}

__attribute__((visibility("default"))) size_t rgc_program_allocated_bytes(const rgc_program* p) {
  if (!p) return 0;
  return (p->p->arena_bytes + p->p->scratch_bytes) * p->p->frames_allocated.load();
}

__attribute__((visibility("default"))) uint64_t rgc_program_launches(const rgc_program* p) { return p ? p->p->launches.load() : 0; }

__attribute__((visibility("default"))) void rgc_program_inject_failure(rgc_program* p) {
  if (p) p->p->inject = true;
}

__attribute__((visibility("default"))) int rgc_exec_acquire(rgc_program* p, rgc_exec** out) {
  return guard([&] {
    if (!p || !out) return fail(RGC_ERR_INVALID, "null argument");
    ck(cudaSetDevice(p->p->device), "cudaSetDevice");
    std::unique_ptr<Frame> f;
    {
      std::lock_guard<std::mutex> lk(p->p->mu);
      if (!p->p->pool.empty()) {
        f = std::move(p->p->pool.back());
        p->p->pool.pop_back();
      }
    }
    if (!f) {
      f = make_frame(p->p.get(), nullptr);
      prepare_frame(p->p.get(), f.get(), f->stream);
      ck(cudaStreamSynchronize(f->stream), "prepare frame");
    }
    f->failed = false;
    f->error.clear();
    auto e = new rgc_exec;
    e->owner = p;
    e->f = std::move(f);
    *out = e;
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) void rgc_exec_release(rgc_exec* e) {
  if (!e) return;
  if (e->f) {
    cudaStreamSynchronize(e->f->stream);
    cudaError_t err = cudaGetLastError();
    // A frame that saw a device error is not reused.
    if (!e->f->failed && err == cudaSuccess) {
      std::lock_guard<std::mutex> lk(e->owner->p->mu);
      e->owner->p->pool.push_back(std::move(e->f));
    }
  }
  delete e;
}

__attribute__((visibility("default"))) int rgc_exec_load(rgc_exec* e, size_t input, const void* host, size_t bytes) {
  return guard([&] {
    const Plan& plan = e->owner->p->plan;
    if (input >= plan.input_slots.size()) return fail(RGC_ERR_INVALID, "input index out of range");
    size_t slot = plan.input_slots[input];
    size_t cap = plan.slots[slot].second * rg::dtype_size(plan.slots[slot].first);
    if (bytes > cap) return fail(RGC_ERR_INVALID, "input larger than its slot");
    if (bytes) {
      ck(cudaMemcpyAsync(e->f->ptr[slot], host, bytes, cudaMemcpyHostToDevice, e->f->stream), "load input");
      ck(cudaStreamSynchronize(e->f->stream), "load input");
    }
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_step(rgc_exec* e) {
  return guard([&] {
    if (e->f->failed) return fail(RGC_ERR_DEVICE, e->f->error);
    if (e->owner->p->inject.exchange(false)) {
      mark_failed(e, "injected failure for test");
      return fail(RGC_ERR_DEVICE, e->f->error);
    }
    launch_plan(e);
    check_async(e);
    return e->f->failed ? fail(RGC_ERR_DEVICE, e->f->error) : RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_step_at(rgc_exec* e, size_t k) {
  return guard([&] {
    Program* p = e->owner->p.get();
    if (k >= p->steps.size()) return fail(RGC_ERR_INVALID, "step index out of range");
    if (e->f->failed) return fail(RGC_ERR_DEVICE, e->f->error);
    Ctx c{e->f->stream, e->f.get()};
    p->steps[k].run(c);
    p->launches += (uint64_t)p->steps[k].kernels;
    check_async(e);
    return e->f->failed ? fail(RGC_ERR_DEVICE, e->f->error) : RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_swap(rgc_exec* e, size_t a, size_t b) {
  return guard([&] {
    if (a >= e->f->ptr.size() || b >= e->f->ptr.size()) return fail(RGC_ERR_INVALID, "slot out of range");
    std::swap(e->f->ptr[a], e->f->ptr[b]);
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_prefix(rgc_exec* e, size_t slot, void* host, size_t bytes) {
  return guard([&] {
    const Plan& plan = e->owner->p->plan;
    if (slot >= plan.slots.size()) return fail(RGC_ERR_INVALID, "slot out of range");
    if (bytes > plan.slots[slot].second * rg::dtype_size(plan.slots[slot].first)) return fail(RGC_ERR_INVALID, "read beyond the slot");
    std::string why;
    cudaError_t err = cudaSuccess;
    if (!dist_active()) {
      if (bytes) ck(cudaMemcpyAsync(host, e->f->ptr[slot], bytes, cudaMemcpyDeviceToHost, e->f->stream), "read slot");
      err = cudaStreamSynchronize(e->f->stream);
    } else {
      // Through pinned memory in chunks, so that the wait is the polled one that can give up on
      // a collective stalled earlier in the stream.
      const size_t chunk = size_t(16) << 20;
      size_t off = 0;
      do {
        const size_t b = std::min(chunk, bytes - off);
        void* stage = e->f->host_buffer(std::max<size_t>(b, 1));
        if (b) ck(cudaMemcpyAsync(stage, e->f->ptr[slot] + off, b, cudaMemcpyDeviceToHost, e->f->stream), "read slot");
        err = dist_sync(e->f->stream, &why);
        if (err != cudaSuccess) break;
        std::memcpy((char*)host + off, stage, b);
        off += b;
      } while (off < bytes);
    }
    if (err != cudaSuccess) {
      mark_failed(e, why.empty() ? std::string(cudaGetErrorString(err)) : why);
      return fail(RGC_ERR_DEVICE, e->f->error);
    }
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_write_prefix(rgc_exec* e, size_t slot, const void* host, size_t bytes) {
  return guard([&] {
    const Plan& plan = e->owner->p->plan;
    if (slot >= plan.slots.size()) return fail(RGC_ERR_INVALID, "slot out of range");
    if (bytes > plan.slots[slot].second * rg::dtype_size(plan.slots[slot].first)) return fail(RGC_ERR_INVALID, "write beyond the slot");
    if (bytes) {
      ck(cudaMemcpyAsync(e->f->ptr[slot], host, bytes, cudaMemcpyHostToDevice, e->f->stream), "write slot");
      ck(cudaStreamSynchronize(e->f->stream), "write slot");
    }
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_scalar(rgc_exec* e, size_t slot, double* out) {
  return guard([&] {
    const Plan& plan = e->owner->p->plan;
    if (slot >= plan.slots.size()) return fail(RGC_ERR_INVALID, "slot out of range");
    DType d = plan.slots[slot].first;
    char buf[8] = {0};
    int rc = rgc_exec_prefix(e, slot, buf, rg::dtype_size(d));
    if (rc) return rc;
    *out = d == DType::F32 ? (double)*(float*)buf : d == DType::F64 ? *(double*)buf : (double)*(int32_t*)buf;
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_failure(rgc_exec* e, char* buf, size_t cap) {
  if (!e || !e->f) return 0;
  if (!e->f->failed) {
    std::string why;
    cudaError_t err = dist_sync(e->f->stream, &why);
    if (err == cudaSuccess) err = cudaGetLastError();
    if (err != cudaSuccess) mark_failed(e, why.empty() ? std::string("device error: ") + cudaGetErrorString(err) : why);
  }
  if (!e->f->failed) check_tc_error(e);
  if (!e->f->failed) return 0;
  if (buf && cap) {
    std::strncpy(buf, e->f->error.c_str(), cap - 1);
    buf[cap - 1] = 0;
  }
  return 1;
}

__attribute__((visibility("default"))) int rgc_exec_slot_pointer(rgc_exec* e, size_t slot, void** out) {
  if (!e || slot >= e->f->ptr.size()) return fail(RGC_ERR_INVALID, "slot out of range");
  *out = e->f->ptr[slot];
  return RGC_OK;
}

// validate.rs:290-363 on the device. Steps run in chunks without host synchronisation; every
// step's history scalars go to a device array and the first non-finite step is recorded on the
// device. State is snapshotted at each chunk start, so a chunk that went past a non-finite step
// is restored and replayed (every kernel is deterministic) up to that step, which is where rg's
// loop stops.
__attribute__((visibility("default"))) int rgc_exec_run(rgc_exec* e, const rgc_run_spec* spec, const void* const* state, const void* const* batches,
                                                        size_t n_batches, size_t steps, double* history, void* const* outputs, const size_t* output_bytes,
                                                        size_t* steps_done, int64_t* nonfinite_step, double* seconds) {
  return guard([&] {
    Program* p = e->owner->p.get();
    const Plan& plan = p->plan;
    Frame* f = e->f.get();
    cudaStream_t s = f->stream;
    *steps_done = 0;
    *nonfinite_step = -1;
    *seconds = 0;
    if (f->failed) return fail(RGC_ERR_DEVICE, f->error);
    // RGC_TRACE_RUN=1 prints where a run's wall time goes (set-up, capture, loop, read-back).
    using Clock = std::chrono::steady_clock;
    static const bool trace = [] {
      const char* v = getenv("RGC_TRACE_RUN");
      return v && std::string(v) == "1";
    }();
    const auto t_start = Clock::now();
    auto slot_bytes = [&](size_t slot) { return plan.slots[slot].second * rg::dtype_size(plan.slots[slot].first); };
    auto in_bytes = [&](size_t input) { return plan.input_ns[input] * rg::dtype_size(plan.slots[plan.input_slots[input]].first); };
    for (size_t k = 0; k < spec->n_state; ++k) {
      if (spec->state_inputs[k] >= plan.input_slots.size() || spec->state_outputs[k] >= plan.outputs.size()) return fail(RGC_ERR_INVALID, "run spec index out of range");
      size_t b = in_bytes(spec->state_inputs[k]);
      if (b && state) ck(cudaMemcpyAsync(f->ptr[plan.input_slots[spec->state_inputs[k]]], state[k], b, cudaMemcpyHostToDevice, s), "load state");
    }
    for (size_t d = 0; d < spec->n_data; ++d)
      if (spec->data_inputs[d] >= plan.input_slots.size()) return fail(RGC_ERR_INVALID, "run spec index out of range");
    for (size_t h = 0; h < spec->n_history; ++h)
      if (spec->history_outputs[h] >= plan.outputs.size()) return fail(RGC_ERR_INVALID, "run spec index out of range");
    // Batches: one batch is loaded once; several live on the device and a kernel picks one per step.
    // Device buffers of the run (batches, history, counters, copy staging, snapshot) are the
    // frame's, grown when a run needs more and kept for the next run.
    Frame::RunCache& rc = f->run;
    auto grow = [](auto*& ptr, size_t& cap, size_t want, const char* what) {
      using T = std::remove_reference_t<decltype(*ptr)>;
      if (want <= cap) return;
      if (ptr) cudaFree((void*)ptr);
      ptr = nullptr;
      cap = 0;
      ck(cudaMalloc((void**)&ptr, want * sizeof(T)), what);
      cap = want;
    };
    std::vector<char*> batch_dev(spec->n_data, nullptr);
    if (n_batches == 1) {
      for (size_t d = 0; d < spec->n_data; ++d) {
        size_t b = in_bytes(spec->data_inputs[d]);
        if (b) ck(cudaMemcpyAsync(f->ptr[plan.input_slots[spec->data_inputs[d]]], batches[d], b, cudaMemcpyHostToDevice, s), "load batch");
      }
    } else if (n_batches > 1) {
      if (rc.batch.size() < spec->n_data) {
        rc.batch.resize(spec->n_data, nullptr);
        rc.batch_cap.resize(spec->n_data, 0);
      }
      for (size_t d = 0; d < spec->n_data; ++d) {
        size_t b = in_bytes(spec->data_inputs[d]);
        grow(rc.batch[d], rc.batch_cap[d], std::max<size_t>(1, b * n_batches), "cudaMalloc(batches)");
        batch_dev[d] = rc.batch[d];
        for (size_t q = 0; q < n_batches; ++q)
          if (b) ck(cudaMemcpyAsync(batch_dev[d] + q * b, batches[q * spec->n_data + d], b, cudaMemcpyHostToDevice, s), "upload batches");
      }
    }
    // Swaps and copies exactly as rg decides them (validate.rs:303-318).
    std::vector<size_t> out_slots;
    for (size_t k = 0; k < spec->n_state; ++k) out_slots.push_back(plan.outputs[spec->state_outputs[k]].slot);
    std::vector<std::pair<size_t, size_t>> swaps;
    std::vector<std::tuple<size_t, size_t, size_t>> copies;  // (input slot, output slot, bytes)
    for (size_t k = 0; k < spec->n_state; ++k) {
      size_t is = plan.input_slots[spec->state_inputs[k]], os = out_slots[k];
      if (is == os) continue;
      size_t users = std::count(out_slots.begin(), out_slots.end(), os);
      if (!plan.pinned[os] && users == 1 && plan.slots[os].second == plan.slots[is].second) swaps.emplace_back(is, os);
      else copies.emplace_back(is, os, plan.outputs[spec->state_outputs[k]].n * rg::dtype_size(plan.slots[os].first));
    }
    size_t nh = spec->n_history;
    size_t staging_bytes = 0;
    for (auto& c : copies) staging_bytes += align_up(std::get<2>(c));
    // History capacity: at least 2^16 steps, so that runs of different lengths share one capture.
    grow(rc.hist, rc.hist_cap, std::max<size_t>(1, nh * std::max<size_t>(steps, size_t(1) << 16)), "cudaMalloc(history)");
    size_t ctr_cap = rc.ctr ? 2 : 0;
    grow(rc.ctr, ctr_cap, 2, "cudaMalloc(counters)");
    if (staging_bytes) grow(rc.staging, rc.staging_cap, staging_bytes, "cudaMalloc(copy staging)");
    double* hist_dev = rc.hist;
    long long* ctr = rc.ctr;  // [0] = step counter, [1] = first non-finite step
    char* staging = staging_bytes ? rc.staging : nullptr;
    // History slot pointers per layout, and types.
    std::vector<int> types(nh);
    for (size_t h = 0; h < nh; ++h) {
      DType d = plan.slots[plan.outputs[spec->history_outputs[h]].slot].first;
      types[h] = d == DType::F32 ? 0 : d == DType::F64 ? 1 : 2;
    }
    int* types_dev = nullptr;
    void** hptr_dev = nullptr;  // [2][nh]
    if (nh) {
      if (nh > rc.nh_cap) {
        size_t tcap = rc.nh_cap, pcap = 2 * rc.nh_cap;
        grow(rc.types, tcap, nh, "cudaMalloc(types)");
        grow(rc.hptr, pcap, 2 * nh, "cudaMalloc(history pointers)");
        rc.nh_cap = nh;
      }
      types_dev = rc.types;
      hptr_dev = rc.hptr;
      ck(cudaMemcpyAsync(types_dev, types.data(), nh * sizeof(int), cudaMemcpyHostToDevice, s), "upload types");
    }
    // The two layouts: the current one, and the one after applying every swap.
    std::vector<char*> layout[2];
    layout[0] = f->ptr;
    layout[1] = f->ptr;
    for (auto& sw : swaps) std::swap(layout[1][sw.first], layout[1][sw.second]);
    bool alternating = !swaps.empty();
    bool use_graphs = graphs_enabled() && p->capturable;
    const bool split = dist_active();
    // What a captured step depends on besides the layouts.
    std::vector<uintptr_t> key;
    auto put = [&](uintptr_t v) { key.push_back(v); };
    put(spec->n_state);
    for (size_t k = 0; k < spec->n_state; ++k) {
      put(spec->state_inputs[k]);
      put(spec->state_outputs[k]);
    }
    put(spec->n_data);
    for (size_t d = 0; d < spec->n_data; ++d) {
      put(spec->data_inputs[d]);
      put((uintptr_t)batch_dev[d]);
    }
    put(nh);
    for (size_t h = 0; h < nh; ++h) put(spec->history_outputs[h]);
    put(n_batches);
    for (const void* q : {(const void*)hist_dev, (const void*)ctr, (const void*)staging, (const void*)types_dev, (const void*)hptr_dev}) put((uintptr_t)q);
    put(split);
    // The loop starts in layout `L`; a cached capture whose layouts are this run's in the other
    // order is replayed with the layouts renamed to its order.
    int L = 0;
    bool reuse = false;
    if (use_graphs && rc.captured && rc.key == key && rc.alternating == alternating) {
      if (rc.layout[0] == layout[0] && rc.layout[1] == layout[1]) {
        reuse = true;
      } else if (alternating && rc.layout[0] == layout[1] && rc.layout[1] == layout[0]) {
        reuse = true;
        std::swap(layout[0], layout[1]);
        L = 1;
      }
    }
    if (!reuse) rc.drop_graphs();
    if (nh) {
      std::vector<void*> hp(2 * nh);
      for (int LL = 0; LL < 2; ++LL)
        for (size_t h = 0; h < nh; ++h) hp[LL * nh + h] = layout[LL][plan.outputs[spec->history_outputs[h]].slot];
      ck(cudaMemcpyAsync(hptr_dev, hp.data(), hp.size() * sizeof(void*), cudaMemcpyHostToDevice, s), "upload history pointers");
    }
    long long init[2] = {0, -1};
    ck(cudaMemcpyAsync(ctr, init, sizeof init, cudaMemcpyHostToDevice, s), "reset counters");

    // One step with layout L: batch load, the plan's steps [first, last), history, copies
    // (through staging), counter. The batch load belongs to the first piece of a step and the
    // rest to the last.
    auto step_part = [&](int LL, cudaStream_t st, size_t first, size_t last) {
      f->ptr = layout[LL];
      if (first == 0 && n_batches > 1)
        for (size_t d = 0; d < spec->n_data; ++d)
          load_batch(f->ptr[plan.input_slots[spec->data_inputs[d]]], batch_dev[d], in_bytes(spec->data_inputs[d]), (long long)n_batches, ctr, st);
      Ctx c{st, f};
      for (size_t k = first; k < last; ++k) p->steps[k].run(c);
      if (last < p->steps.size()) return;
      if (nh) record_history(hist_dev, (const void* const*)(hptr_dev + LL * nh), types_dev, (int)nh, ctr, ctr + 1, st);
      size_t off = 0;
      for (auto& cp : copies) {
        ck(cudaMemcpyAsync(staging + off, layout[LL][std::get<1>(cp)], std::get<2>(cp), cudaMemcpyDeviceToDevice, st), "state copy");
        off += align_up(std::get<2>(cp));
      }
      off = 0;
      for (auto& cp : copies) {
        ck(cudaMemcpyAsync(layout[alternating ? 1 - LL : LL][std::get<0>(cp)], staging + off, std::get<2>(cp), cudaMemcpyDeviceToDevice, st), "state copy");
        off += align_up(std::get<2>(cp));
      }
      bump_counter(ctr, st);
    };
    // A step replays as pieces: CUDA graphs for the runs of steps between collectives, and under
    // data parallelism each collective launched directly (so that a stalled one can be aborted).
    std::vector<Frame::RunPiece>& pieces = rc.pieces;
    const auto t_setup = Clock::now();
    if (use_graphs && !reuse) {
      size_t start = 0;
      for (size_t k = 0; k <= p->steps.size(); ++k) {
        const bool cut = k == p->steps.size() || (split && p->steps[k].collective);
        if (!cut) continue;
        Frame::RunPiece pc;
        pc.first = start;
        pc.last = k;
        pieces.push_back(pc);
        if (k < p->steps.size()) {
          Frame::RunPiece d;
          d.first = k;
          d.last = k + 1;
          d.direct = true;
          pieces.push_back(d);
        }
        start = k + 1;
      }
      // The last graph piece carries the step's epilogue, even when the plan ends in a collective.
      if (pieces.back().direct) {
        Frame::RunPiece tail;
        tail.first = tail.last = p->steps.size();
        pieces.push_back(tail);
      }
      for (auto& pc : pieces) {
        if (pc.direct) continue;
        for (int LL = 0; LL < (alternating ? 2 : 1); ++LL)
          pc.g[LL] = capture(s, [&](cudaStream_t st) { step_part(LL, st, pc.first, pc.last); });
        if (!alternating) pc.g[1] = pc.g[0];
      }
      rc.key = key;
      rc.alternating = alternating;
      rc.layout[0] = layout[0];
      rc.layout[1] = layout[1];
      rc.captured = true;
    }
    const auto t_capture = Clock::now();
    uint64_t per_step = (uint64_t)p->kernels_per_step + (nh ? 1 : 0) + 1 + (n_batches > 1 ? spec->n_data : 0);
    // State snapshot buffers (chunk starts), sized by the state inputs.
    std::vector<std::pair<size_t, size_t>> snap_items;  // (input slot, bytes)
    size_t snap_bytes = 0;
    for (size_t k = 0; k < spec->n_state; ++k) {
      size_t is = plan.input_slots[spec->state_inputs[k]];
      snap_items.emplace_back(is, in_bytes(spec->state_inputs[k]));
      snap_bytes += align_up(in_bytes(spec->state_inputs[k]));
    }
    char* snap = nullptr;
    if (snap_bytes) {
      grow(rc.snap, rc.snap_cap, snap_bytes, "cudaMalloc(snapshot)");
      snap = rc.snap;
    }
    const char* env_chunk = getenv("RGC_RUN_CHUNK");
    size_t chunk = env_chunk ? (size_t)std::max(1, atoi(env_chunk)) : 64;
    size_t done = 0;
    long long bad = -1;
    ck(cudaStreamSynchronize(s), "run setup");
    // Device time of the loop, from events on the stream every step runs on.
    cudaEvent_t ev0, ev1;
    ck(cudaEventCreate(&ev0), "cudaEventCreate");
    ck(cudaEventCreate(&ev1), "cudaEventCreate");
    struct EventCleanup {
      cudaEvent_t a, b;
      ~EventCleanup() {
        cudaEventDestroy(a);
        cudaEventDestroy(b);
      }
    } event_cleanup{ev0, ev1};
    ck(cudaEventRecord(ev0, s), "cudaEventRecord");
    auto snapshot = [&](int LL, bool restore) {
      size_t off = 0;
      for (auto& [slot, bytes] : snap_items) {
        if (bytes) {
          if (restore) ck(cudaMemcpyAsync(layout[LL][slot], snap + off, bytes, cudaMemcpyDeviceToDevice, s), "restore state");
          else ck(cudaMemcpyAsync(snap + off, layout[LL][slot], bytes, cudaMemcpyDeviceToDevice, s), "snapshot state");
        }
        off += align_up(bytes);
      }
    };
    auto launch = [&](int LL) {
      if (!use_graphs) {
        step_part(LL, s, 0, p->steps.size());
      } else {
        for (auto& pc : pieces) {
          if (!pc.direct) {
            ck(cudaGraphLaunch(pc.g[LL], s), "cudaGraphLaunch");
            continue;
          }
          f->ptr = layout[LL];
          Ctx c{s, f};
          p->steps[pc.first].run(c);
        }
      }
      p->launches += per_step;
    };
    while (done < steps) {
      if (p->inject.exchange(false)) {
        mark_failed(e, "injected failure for test");
        break;
      }
      size_t n = std::min(chunk, steps - done);
      if (snap) snapshot(L, false);
      int L0 = L;
      for (size_t q = 0; q < n; ++q) {
        launch(L);
        if (alternating) L = 1 - L;
      }
      long long* host_ctr = (long long*)f->host_buffer(2 * sizeof(long long));
      ck(cudaMemcpyAsync(host_ctr, ctr, 2 * sizeof(long long), cudaMemcpyDeviceToHost, s), "read counters");
      std::string why;
      cudaError_t err = dist_sync(s, &why);
      if (err != cudaSuccess) {
        mark_failed(e, why.empty() ? std::string("device error: ") + cudaGetErrorString(err) : why);
        break;
      }
      if (host_ctr[1] >= 0) {
        bad = host_ctr[1];
        // Replay the chunk up to and including the bad step from the snapshot.
        if (snap) snapshot(L0, true);
        L = L0;
        long long rewind[1] = {(long long)done};
        ck(cudaMemcpyAsync(ctr, rewind, sizeof(long long), cudaMemcpyHostToDevice, s), "rewind counter");
        for (long long q = (long long)done; q <= bad; ++q) {
          launch(L);
          if (alternating) L = 1 - L;
        }
        ck(cudaStreamSynchronize(s), "replay");
        done = (size_t)bad + 1;
        break;
      }
      done += n;
    }
    ck(cudaEventRecord(ev1, s), "cudaEventRecord");
    ck(cudaStreamSynchronize(s), "run");
    const auto t_loop = Clock::now();
    float ms = 0;
    ck(cudaEventElapsedTime(&ms, ev0, ev1), "cudaEventElapsedTime");
    *seconds = ms * 1e-3;
    *steps_done = done;
    *nonfinite_step = bad;
    if (history && nh && done) {
      std::vector<double> hv(nh * done);
      ck(cudaMemcpy(hv.data(), hist_dev, hv.size() * sizeof(double), cudaMemcpyDeviceToHost), "read history");
      for (size_t h = 0; h < nh; ++h)
        for (size_t k = 0; k < done; ++k) history[h * steps + k] = hv[k * nh + h];
    }
    // Outputs of the last completed step live in the layout that step ran with.
    int last_L = alternating && done ? 1 - L : L;
    if (outputs && done) {
      for (size_t o = 0; o < plan.outputs.size(); ++o) {
        size_t b = std::min(output_bytes[o], slot_bytes(plan.outputs[o].slot));
        if (b && outputs[o]) ck(cudaMemcpy(outputs[o], layout[last_L][plan.outputs[o].slot], b, cudaMemcpyDeviceToHost), "read outputs");
      }
    }
    // The frame keeps the layout after the last step's swaps: the state is in the input slots.
    f->ptr = layout[L];
    if (trace) {
      auto ms_between = [](Clock::time_point a, Clock::time_point b) { return std::chrono::duration<double, std::milli>(b - a).count(); };
      fprintf(stderr, "[rgc run] steps %zu: setup %.3f ms, capture %.3f ms (%s), loop %.3f ms (device %.3f ms), read-back %.3f ms\n", done,
              ms_between(t_start, t_setup), ms_between(t_setup, t_capture), !use_graphs ? "no graphs" : reuse ? "cached" : "captured",
              ms_between(t_capture, t_loop), (double)ms, ms_between(t_loop, Clock::now()));
    }
    if (!f->failed) check_tc_error(e);
    if (f->failed) return fail(RGC_ERR_DEVICE, f->error);
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_step_checked(rgc_exec* e, int32_t* flags, size_t n_flags) {
  return guard([&] {
    if (e->f->failed) return fail(RGC_ERR_DEVICE, e->f->error);
    Program* p = e->owner->p.get();
    const Plan& plan = p->plan;
    const size_t n = plan.steps.size();
    if (!flags || n_flags < 2 * n) return fail(RGC_ERR_INVALID, "flags array shorter than twice the plan's steps");
    cudaStream_t s = e->f->stream;
    int* dflags = nullptr;
    ck(cudaMallocAsync((void**)&dflags, std::max<size_t>(1, 2 * n) * sizeof(int), s), "cudaMallocAsync(check flags)");
    ck(cudaMemsetAsync(dflags, 0, std::max<size_t>(1, 2 * n) * sizeof(int), s), "cudaMemsetAsync(check flags)");
    Ctx c{s, e->f.get()};
    auto check = [&](size_t slot, size_t count, int* flag) {
      DType d = plan.slots[slot].first;
      if (d != DType::I32 && count) any_nonfinite(e->f->ptr[slot], et(d), (long long)count, flag, s);
    };
    for (size_t k = 0; k < n; ++k) {
      const rg::Step& st = plan.steps[k];
      if (!st.fused && (st.instr.op.kind == OpKind::Take || st.instr.op.kind == OpKind::TakeAlong)) {
        const Instr& i = st.instr;
        const size_t dim = i.op.kind == OpKind::Take ? i.arg_shapes[0][i.op.index] : i.arg_shapes[0].back();
        index_outside((const int32_t*)e->f->ptr[i.args[1]], (long long)rg::product(i.arg_shapes[1]), (long long)dim, dflags + n + k, s);
      }
      p->steps[k].run(c);
      if (st.fused) {
        for (auto& o : st.group.outputs) check(o.second, st.group.n, dflags + k);
      } else if (st.instr.op.is_control_flow()) {
        for (auto& [index, slot] : st.instr.outs) {
          (void)index;
          check(slot, plan.slots[slot].second, dflags + k);
        }
      } else if (st.instr.op.kind != OpKind::AllReduce || !st.instr.args.empty()) {
        check(st.instr.dst, st.instr.n, dflags + k);
      }
    }
    int* host = (int*)e->f->host_buffer(std::max<size_t>(1, 2 * n) * sizeof(int));
    if (n) ck(cudaMemcpyAsync(host, dflags, 2 * n * sizeof(int), cudaMemcpyDeviceToHost, s), "read check flags");
    ck(cudaFreeAsync(dflags, s), "cudaFreeAsync(check flags)");
    std::string why;
    cudaError_t err = dist_sync(s, &why);
    if (err != cudaSuccess) {
      mark_failed(e, why.empty() ? std::string("device error: ") + cudaGetErrorString(err) : why);
      return fail(RGC_ERR_DEVICE, e->f->error);
    }
    for (size_t q = 0; q < 2 * n; ++q) flags[q] = host[q];
    p->launches += (uint64_t)p->kernels_per_step;
    return RGC_OK;
  });
}

namespace {
// Pinned staging for checkpoint streaming: two buffers, so that one chunk's device copy overlaps
// the file I/O of the other.
struct Pinned {
  static constexpr size_t CHUNK = size_t(64) << 20;
  void* buf[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  Pinned() {
    for (int i = 0; i < 2; ++i) {
      ck(cudaMallocHost(&buf[i], CHUNK), "cudaMallocHost(checkpoint staging)");
      ck(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming), "cudaEventCreate");
    }
  }
  ~Pinned() {
    for (int i = 0; i < 2; ++i) {
      if (buf[i]) cudaFreeHost(buf[i]);
      if (done[i]) cudaEventDestroy(done[i]);
    }
  }
};
}  // namespace

__attribute__((visibility("default"))) int rgc_exec_save_slots(rgc_exec* e, const char* path, const char* header, size_t header_len,
                                                             const size_t* slots, const size_t* sizes, size_t n) {
  return guard([&] {
    if (e->f->failed) return fail(RGC_ERR_DEVICE, e->f->error);
    const Plan& plan = e->owner->p->plan;
    if (!path || (header_len && !header) || (n && (!slots || !sizes))) return fail(RGC_ERR_INVALID, "null argument");
    for (size_t k = 0; k < n; ++k) {
      if (slots[k] >= plan.slots.size()) return fail(RGC_ERR_INVALID, "slot out of range");
      if (sizes[k] > plan.slots[slots[k]].second * rg::dtype_size(plan.slots[slots[k]].first)) return fail(RGC_ERR_INVALID, "read beyond the slot");
    }
    cudaStream_t s = e->f->stream;
    std::string tmp = std::string(path) + ".tmp." + std::to_string(getpid());
    FILE* fp = std::fopen(tmp.c_str(), "wb");
    if (!fp) return fail(RGC_ERR_INVALID, std::string("cannot open ") + tmp + " for writing");
    bool ok = true;
    try {
      uint64_t len = header_len;
      unsigned char le[8];
      for (int i = 0; i < 8; ++i) le[i] = (unsigned char)(len >> (8 * i));
      ok = std::fwrite(le, 1, 8, fp) == 8 && std::fwrite(header, 1, header_len, fp) == header_len;
      Pinned pin;
      // Chunks of every slot in order, double-buffered: copy chunk c + 1 while writing chunk c.
      std::vector<std::tuple<size_t, size_t, size_t>> chunks;  // (slot, offset, bytes)
      for (size_t k = 0; k < n; ++k)
        for (size_t off = 0; off < sizes[k]; off += Pinned::CHUNK) chunks.emplace_back(slots[k], off, std::min(Pinned::CHUNK, sizes[k] - off));
      auto issue = [&](size_t c) {
        auto [slot, off, bytes] = chunks[c];
        ck(cudaMemcpyAsync(pin.buf[c & 1], e->f->ptr[slot] + off, bytes, cudaMemcpyDeviceToHost, s), "checkpoint read");
        ck(cudaEventRecord(pin.done[c & 1], s), "cudaEventRecord");
      };
      if (!chunks.empty()) issue(0);
      for (size_t c = 0; c < chunks.size() && ok; ++c) {
        if (c + 1 < chunks.size()) issue(c + 1);
        ck(cudaEventSynchronize(pin.done[c & 1]), "checkpoint read");
        size_t bytes = std::get<2>(chunks[c]);
        ok = std::fwrite(pin.buf[c & 1], 1, bytes, fp) == bytes;
      }
      ck(cudaStreamSynchronize(s), "checkpoint read");
      ok = ok && std::fflush(fp) == 0 && fsync(fileno(fp)) == 0;
    } catch (...) {
      std::fclose(fp);
      std::remove(tmp.c_str());
      throw;
    }
    ok = (std::fclose(fp) == 0) && ok;
    if (!ok || std::rename(tmp.c_str(), path) != 0) {
      std::remove(tmp.c_str());
      return fail(RGC_ERR_INVALID, std::string("writing the checkpoint ") + path + " failed");
    }
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_load_slots(rgc_exec* e, const char* path, const uint64_t* offsets, const size_t* slots,
                                                             const size_t* sizes, size_t n) {
  return guard([&] {
    if (e->f->failed) return fail(RGC_ERR_DEVICE, e->f->error);
    const Plan& plan = e->owner->p->plan;
    if (!path || (n && (!offsets || !slots || !sizes))) return fail(RGC_ERR_INVALID, "null argument");
    for (size_t k = 0; k < n; ++k) {
      if (slots[k] >= plan.slots.size()) return fail(RGC_ERR_INVALID, "slot out of range");
      if (sizes[k] > plan.slots[slots[k]].second * rg::dtype_size(plan.slots[slots[k]].first)) return fail(RGC_ERR_INVALID, "write beyond the slot");
    }
    FILE* fp = std::fopen(path, "rb");
    if (!fp) return fail(RGC_ERR_INVALID, std::string("cannot open ") + path);
    struct Closer {
      FILE* f;
      ~Closer() { std::fclose(f); }
    } closer{fp};
    cudaStream_t s = e->f->stream;
    Pinned pin;
    size_t c = 0;
    for (size_t k = 0; k < n; ++k) {
      if (std::fseek(fp, (long)offsets[k], SEEK_SET) != 0) return fail(RGC_ERR_INVALID, std::string(path) + ": offset beyond the file");
      for (size_t off = 0; off < sizes[k]; off += Pinned::CHUNK, ++c) {
        const size_t bytes = std::min(Pinned::CHUNK, sizes[k] - off);
        // The buffer's previous copy must be done before it is refilled.
        ck(cudaEventSynchronize(pin.done[c & 1]), "checkpoint write");
        if (std::fread(pin.buf[c & 1], 1, bytes, fp) != bytes) return fail(RGC_ERR_INVALID, std::string(path) + ": file shorter than its header says");
        ck(cudaMemcpyAsync(e->f->ptr[slots[k]] + off, pin.buf[c & 1], bytes, cudaMemcpyHostToDevice, s), "checkpoint write");
        ck(cudaEventRecord(pin.done[c & 1], s), "cudaEventRecord");
      }
    }
    ck(cudaStreamSynchronize(s), "checkpoint write");
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_step_timed(rgc_exec* e, double* seconds, size_t n_steps) {
  return guard([&] {
    Program* p = e->owner->p.get();
    if (n_steps < p->steps.size()) return fail(RGC_ERR_INVALID, "seconds array too short");
    cudaStream_t s = e->f->stream;
    std::vector<cudaEvent_t> ev(p->steps.size() + 1);
    for (auto& x : ev) ck(cudaEventCreate(&x), "cudaEventCreate");
    ck(cudaEventRecord(ev[0], s), "cudaEventRecord");
    Ctx c{s, e->f.get()};
    for (size_t k = 0; k < p->steps.size(); ++k) {
      p->steps[k].run(c);
      ck(cudaEventRecord(ev[k + 1], s), "cudaEventRecord");
    }
    ck(cudaStreamSynchronize(s), "step_timed");
    for (size_t k = 0; k < p->steps.size(); ++k) {
      float ms = 0;
      cudaEventElapsedTime(&ms, ev[k], ev[k + 1]);
      seconds[k] += ms * 1e-3;
    }
    for (auto& x : ev) cudaEventDestroy(x);
    p->launches += (uint64_t)p->kernels_per_step;
    return RGC_OK;
  });
}

__attribute__((visibility("default"))) int rgc_exec_breakdown_json(rgc_exec* e, size_t repeats, char* buf, size_t cap) {
  return guard([&] {
    Program* p = e->owner->p.get();
    cudaStream_t s = e->f->stream;
    repeats = std::max<size_t>(1, repeats);
    cudaEvent_t a, b;
    ck(cudaEventCreate(&a), "cudaEventCreate");
    ck(cudaEventCreate(&b), "cudaEventCreate");
    auto t0 = std::chrono::steady_clock::now();
    ck(cudaEventRecord(a, s), "cudaEventRecord");
    for (size_t r = 0; r < repeats; ++r) launch_plan(e);
    ck(cudaEventRecord(b, s), "cudaEventRecord");
    auto t1 = std::chrono::steady_clock::now();
    ck(cudaStreamSynchronize(s), "breakdown");
    auto t2 = std::chrono::steady_clock::now();
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    char tmp[512];
    snprintf(tmp, sizeof tmp,
             "{\"repeats\":%zu,\"plan_steps\":%zu,\"kernels_per_step\":%d,\"gpu_seconds_per_step\":%.9g,\"launch_seconds_per_step\":%.9g,"
             "\"wall_seconds_per_step\":%.9g,\"graph_capturable\":%s}",
             repeats, p->steps.size(), p->kernels_per_step, ms * 1e-3 / repeats,
             std::chrono::duration<double>(t1 - t0).count() / repeats, std::chrono::duration<double>(t2 - t0).count() / repeats,
             p->capturable ? "true" : "false");
    if (buf && cap) {
      std::strncpy(buf, tmp, cap - 1);
      buf[cap - 1] = 0;
    }
    return RGC_OK;
  });
}

}  // extern "C"

// Not part of include/rgc.h: test support. Builds the row-chain kernels the device would generate
// for a plan blob and compiles them for sm_100a with NVRTC without loading them (no GPU or CUDA
// context is needed). Returns the number of kernels, or -1 with the compiler's log in `log`;
// chains that fall back to step-by-step lowering are listed in `log` either way.
extern "C" __attribute__((visibility("default"))) int rgc_debug_row_kernels(const void* blob, size_t size, char* log, size_t cap) {
  std::string msg;
  int result = -1;
  try {
    rg::Plan plan = rg::decode_plan((const uint8_t*)blob, size);
    std::vector<std::string> sources, names;
    for (auto& c : rg::find_row_chains(plan, true)) {
      rgc::RowKernel rk;
      std::string why;
      if (!rgc::make_row_kernel(plan, c, &rk, &why)) {
        msg += "chain at step " + std::to_string(c.first) + " lowered step by step: " + why + "\n";
        continue;
      }
      // Chains of the same structure (one per layer) share a kernel, as in the JIT.
      if (std::find(names.begin(), names.end(), rk.name) == names.end()) {
        names.push_back(rk.name);
        sources.push_back(rk.source);
      }
    }
    if (const char* dump = getenv("RGC_ROW_DUMP")) {
      FILE* f = fopen(dump, "w");
      if (f) {
        for (auto& src : sources) fprintf(f, "%s\n", src.c_str());
        fclose(f);
      }
    }
    std::string err = sources.empty() ? std::string() : rgc::Jit::compile_check(sources);
    if (err.empty()) {
      result = (int)sources.size();
    } else {
      msg = err;
    }
  } catch (const std::exception& e) {
    msg = e.what();
  }
  if (log && cap) {
    size_t n = std::min(cap - 1, msg.size());
    std::memcpy(log, msg.data(), n);
    log[n] = '\0';
  }
  return result;
}

// Not part of include/rgc.h: test support. Describes the kernel of row chain `index` of a plan
// blob as JSON (the chain's steps, the slots bound to its parameters, periods, broadcast
// descriptors, rows, rows per block, shared memory) and writes the prelude and its source to
// `source_path`, so that tests can compile it for the host and run it against the CPU
// interpreter. Returns 0, 1 when the plan has no such chain or it falls back to step-by-step
// lowering, or -1 with the reason in `json`.
extern "C" __attribute__((visibility("default"))) int rgc_debug_row_kernel(const void* blob, size_t size, int index, char* json, size_t cap,
                                                                           const char* source_path) {
  std::string out;
  int result = -1;
  try {
    rg::Plan plan = rg::decode_plan((const uint8_t*)blob, size);
    auto chains = rg::find_row_chains(plan, true);
    rgc::RowKernel rk;
    std::string why;
    if (index < 0 || (size_t)index >= chains.size() || !rgc::make_row_kernel(plan, chains[(size_t)index], &rk, &why)) {
      out = why;
      result = 1;
    } else {
      const rg::RowChain& c = chains[(size_t)index];
      auto list = [](const std::vector<size_t>& v) {
        std::string r = "[";
        for (size_t i = 0; i < v.size(); ++i) r += (i ? "," : "") + std::to_string(v[i]);
        return r + "]";
      };
      auto fdiv = [](const FDiv& f) { return "[" + std::to_string(f.d) + "," + std::to_string(f.m) + "," + std::to_string(f.s) + "]"; };
      out = "{\"name\":\"" + rk.name + "\",\"first\":" + std::to_string(c.first) + ",\"last\":" + std::to_string(c.last) +
            ",\"members\":" + list(c.members) + ",\"before\":" + list(c.before) + ",\"after\":" + list(c.after) +
            ",\"in_slots\":" + list(rk.in_slots) + ",\"out_slots\":" + list(rk.out_slots) + ",\"rows\":" + std::to_string(rk.rows) +
            ",\"rows_per_block\":" + std::to_string(rk.rows_per_block) + ",\"smem\":" + std::to_string(rk.smem) + ",\"in_div\":[";
      for (size_t i = 0; i < rk.in_div.size(); ++i) out += (i ? "," : "") + fdiv(rk.in_div[i]);
      out += "],\"bcs\":[";
      for (size_t i = 0; i < rk.bcs.size(); ++i) {
        const FDims& f = rk.bcs[i];
        out += std::string(i ? "," : "") + "{\"rank\":" + std::to_string(f.rank) + ",\"d\":[";
        for (int q = 0; q < MAXR; ++q) out += (q ? "," : "") + fdiv(f.d[q]);
        out += "],\"st\":[";
        for (int q = 0; q < MAXR; ++q) out += (q ? "," : "") + std::to_string(f.st[q]);
        out += "]}";
      }
      out += "]}";
      FILE* f = fopen(source_path, "w");
      if (!f) throw std::runtime_error("cannot write the kernel source");
      fprintf(f, "%s\n%s\n", rgc::Jit::prelude().c_str(), rk.source.c_str());
      fclose(f);
      result = 0;
    }
  } catch (const std::exception& e) {
    out = e.what();
    result = -1;
  }
  if (json && cap) {
    size_t n = std::min(cap - 1, out.size());
    std::memcpy(json, out.data(), n);
    json[n] = '\0';
  }
  return result;
}
