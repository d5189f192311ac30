// TEST INFRASTRUCTURE — runs a generated row-chain kernel (its CUDA source, unchanged apart from
// the griddepcontrol lines, which order launches and have no effect inside one) on the host: one
// OS thread per CUDA thread of a block, `__syncthreads` as a block barrier and `__shfl_sync` as a
// warp exchange between two warp barriers, blocks one after another. The host's libm gives the
// transcendental functions glibc's results, which is what rg and the CPU interpreter compute, so
// results compare bit for bit with the interpreter. Compiled with -ffp-contract=off.
#pragma once
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#define __global__
#define __device__
#define __forceinline__ inline
#define __launch_bounds__(n)
#define __shared__
#define __align__(n) __attribute__((aligned(n)))

struct rg_dim3 {
  unsigned x = 0, y = 0, z = 0;
};
inline thread_local rg_dim3 threadIdx, blockIdx;
inline rg_dim3 gridDim, blockDim;

struct float4 {
  float x, y, z, w;
};
struct double2 {
  double x, y;
};
struct int4 {
  int x, y, z, w;
};

inline unsigned __umulhi(unsigned a, unsigned b) { return (unsigned)(((unsigned long long)a * b) >> 32); }
inline float __int_as_float(int v) {
  float f;
  std::memcpy(&f, &v, 4);
  return f;
}
inline int __float_as_int(float f) {
  int v;
  std::memcpy(&v, &f, 4);
  return v;
}
inline double __longlong_as_double(long long v) {
  double f;
  std::memcpy(&f, &v, 8);
  return f;
}
inline long long __double_as_longlong(double f) {
  long long v;
  std::memcpy(&v, &f, 8);
  return v;
}

class RgBarrier {
 public:
  explicit RgBarrier(int n) : n_(n) {}
  void wait() {
    std::unique_lock<std::mutex> lk(mu_);
    const unsigned long gen = gen_;
    if (++count_ == n_) {
      count_ = 0;
      ++gen_;
      cv_.notify_all();
      return;
    }
    cv_.wait(lk, [&] { return gen_ != gen; });
  }

 private:
  std::mutex mu_;
  std::condition_variable cv_;
  int n_, count_ = 0;
  unsigned long gen_ = 0;
};

struct RgBlock {
  RgBarrier block{256};
  std::vector<RgBarrier*> warps;
  unsigned long long exchange[8][32];
  RgBlock() {
    for (int w = 0; w < 8; ++w) warps.push_back(new RgBarrier(32));
  }
  ~RgBlock() {
    for (auto* w : warps) delete w;
  }
};
inline RgBlock* rg_block = nullptr;

inline void __syncthreads() { rg_block->block.wait(); }

template <typename T> T __shfl_sync(unsigned, T v, int src) {
  const int warp = (int)threadIdx.x / 32, lane = (int)threadIdx.x % 32;
  unsigned long long bits = 0;
  std::memcpy(&bits, &v, sizeof(T));
  rg_block->exchange[warp][lane] = bits;
  rg_block->warps[warp]->wait();
  T r;
  bits = rg_block->exchange[warp][src & 31];
  std::memcpy(&r, &bits, sizeof(T));
  rg_block->warps[warp]->wait();
  return r;
}

// Block shared memory: blocks run one after another, so one buffer serves them all.
alignas(16) inline unsigned char rg_smem_store[256 * 1024];
#define rg_smem rg_smem_store
