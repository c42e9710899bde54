// runtime.cu -- error reporting, version, per-device scratch of the
// kernel-level fused entries.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <new>
#include <vector>

#include "common.cuh"
#include "matvec.cuh"

namespace qasr {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return QASR_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? QASR_ERR_ALLOC : QASR_ERR_CUDA;
}

int launch_status(const char *what) { return cuda_status(cudaGetLastError(), what); }

struct NormScratch {
  float *buf = nullptr;
  size_t cap = 0;
};
static NormScratch g_norm_scratch[64];
static std::mutex g_scratch_mu;

int mv_norm_scratch(float **buf, size_t n_floats) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return QASR_ERR_INVALID;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  NormScratch &s = g_norm_scratch[dev];
  if (s.cap < n_floats) {
    if (s.buf) {
      cudaDeviceSynchronize();
      cudaFree(s.buf);
      s.buf = nullptr;
      s.cap = 0;
    }
    size_t want = n_floats < 65536 ? 65536 : n_floats;
    if (cudaMalloc(&s.buf, want * sizeof(float)) != cudaSuccess) {
      set_error("kernel-level scratch: cudaMalloc(%zu) failed", want * sizeof(float));
      return QASR_ERR_ALLOC;
    }
    s.cap = want;
  }
  *buf = s.buf;
  return QASR_OK;
}

// Per-device, per-purpose scratch for the kernel-level entries: grown on
// demand, zero-filled when (re)allocated.  Kernels that use counters in it
// leave them at zero again when they finish.
struct DevScratch {
  void *buf = nullptr;
  size_t cap = 0;
};
static DevScratch g_dev_scratch[64][kScratchSlots];

// Scratch owned by one engine.  While an ArenaScope of the engine is active
// on the calling thread, dev_scratch hands out the engine's buffers instead
// of the per-device ones, so engines driven from different host threads
// (the transcription lanes) never share a buffer.  A buffer that grows is
// retired, not freed: kernels still in flight on the engine's streams may
// read it, and freeing would synchronise the whole device under another
// thread's graph capture.  Retired buffers go with the arena.
struct ScratchArena {
  int device = 0;
  DevScratch slot[kScratchSlots];
  std::vector<void *> retired;
};

static thread_local ScratchArena *t_arena = nullptr;

ScratchArena *arena_create(int device) {
  ScratchArena *a = new (std::nothrow) ScratchArena;
  if (a) a->device = device;
  return a;
}

void arena_free(ScratchArena *a) {
  if (!a) return;
  for (auto &s : a->slot)
    if (s.buf) cudaFree(s.buf);
  for (void *p : a->retired) cudaFree(p);
  delete a;
}

ArenaScope::ArenaScope(ScratchArena *a) : prev(t_arena) {
  if (a) t_arena = a;
}
ArenaScope::~ArenaScope() { t_arena = prev; }

static int scratch_fill(void *buf, size_t bytes) {
  // zero on the legacy stream and wait for it: the engines' streams are
  // non-blocking and would not order behind it
  if (cudaMemset(buf, 0, bytes) != cudaSuccess || cudaStreamSynchronize(cudaStreamLegacy) != cudaSuccess) {
    set_error("kernel-level scratch: zero fill failed");
    return QASR_ERR_CUDA;
  }
  return QASR_OK;
}

int dev_scratch(int slot, size_t bytes, void **out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || slot < 0 || slot >= kScratchSlots) return QASR_ERR_INVALID;
  if (ScratchArena *a = t_arena; a && a->device == dev) {
    DevScratch &s = a->slot[slot];
    if (s.cap < bytes) {
      size_t want = bytes < 4096 ? 4096 : bytes;
      if (want < s.cap + s.cap / 2) want = s.cap + s.cap / 2;
      void *buf = nullptr;
      if (cudaMalloc(&buf, want) != cudaSuccess) {
        set_error("engine scratch: cudaMalloc(%zu) failed", want);
        return QASR_ERR_ALLOC;
      }
      if (int rc = scratch_fill(buf, want)) {
        cudaFree(buf);
        return rc;
      }
      if (s.buf) a->retired.push_back(s.buf);
      s.buf = buf;
      s.cap = want;
    }
    *out = s.buf;
    return QASR_OK;
  }
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  DevScratch &s = g_dev_scratch[dev][slot];
  if (s.cap < bytes) {
    if (s.buf) {
      cudaDeviceSynchronize();
      cudaFree(s.buf);
      s.buf = nullptr;
      s.cap = 0;
    }
    size_t want = bytes < 4096 ? 4096 : bytes;
    if (cudaMalloc(&s.buf, want) != cudaSuccess) {
      set_error("kernel-level scratch: cudaMalloc(%zu) failed", want);
      return QASR_ERR_ALLOC;
    }
    if (int rc = scratch_fill(s.buf, want)) return rc;
    s.cap = want;
  }
  *out = s.buf;
  return QASR_OK;
}

}  // namespace qasr

extern "C" const char *qasr_last_error(void) { return qasr::g_err; }
extern "C" const char *qasr_version(void) { return "qwenasr_b200 0.1.0 (sm_100a)"; }
