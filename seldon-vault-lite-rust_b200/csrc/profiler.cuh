// profiler.cuh -- optional per-kernel-category CUDA-event timing and launch
// counting for a model or index handle (bench.py reads it through
// svl_gpu_testing.h to put live kernel times beside the roofline).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <vector>

namespace svl {

enum ProfCategory : int {
  kProfGemm = 0,       // tcgen05 TF32 GEMMs of the encoder
  kProfAttention = 1,  // attention
  kProfNorm = 2,       // RMSNorm / residual / q-k-v norm + RoPE
  kProfOther = 3,      // embedding gather, pooling, index bookkeeping, copies
  kProfScreen = 4,     // search: tensor-core screen + candidate epilogue
  kProfRescore = 5,    // search: exact f64 rescoring and selection
  kProfCount = 6
};

struct Profiler {
  bool enabled = false;
  std::atomic<uint64_t> launches[kProfCount] = {};  // counted from any host thread
  struct Mark {
    int cat;
    cudaEvent_t a, b;
  };
  std::vector<Mark> marks;
  std::vector<cudaEvent_t> pool;

  cudaEvent_t ev() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
  }
  // Brackets one launch of category `cat` on stream `st`.
  struct Scope {
    Profiler* p;
    int cat;
    cudaStream_t st;
    cudaEvent_t b = nullptr;
    Scope(Profiler* prof, int c, cudaStream_t s) : p(prof), cat(c), st(s) {
      p->launches[c].fetch_add(1, std::memory_order_relaxed);
      if (p->enabled) {
        cudaEvent_t a = p->ev();
        b = p->ev();
        cudaEventRecord(a, st);
        p->marks.push_back({c, a, b});
      }
    }
    ~Scope() {
      if (b) cudaEventRecord(b, st);
    }
  };
  // Sums elapsed ms per category since the last read (caller synchronised).
  void read(double* ms, uint64_t* counts) {
    for (int c = 0; c < kProfCount; ++c) {
      if (ms) ms[c] = 0.0;
      const uint64_t n = launches[c].exchange(0, std::memory_order_relaxed);
      if (counts) counts[c] = n;
    }
    for (auto& m : marks) {
      float t = 0.0f;
      if (cudaEventElapsedTime(&t, m.a, m.b) == cudaSuccess && ms) ms[m.cat] += t;
      pool.push_back(m.a);
      pool.push_back(m.b);
    }
    marks.clear();
  }
  ~Profiler() {
    for (auto& m : marks) {
      cudaEventDestroy(m.a);
      cudaEventDestroy(m.b);
    }
    for (auto e : pool) cudaEventDestroy(e);
  }
};

}  // namespace svl
