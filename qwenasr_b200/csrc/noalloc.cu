// noalloc.cu -- final RMSNorm + INT8 lm head + argmax without any device
// allocation.
//
// qasr_final_norm_lmhead_argmax keeps the cross-CTA argmax keys and the
// arrival counter in scratch that it cudaMalloc's on first use.  Some callers
// cannot allow that: a host whose device memory is handed out by its own pool
// (a serving runtime that forbids allocations after warm-up, or one that
// records its work into a CUDA graph and must not allocate while recording),
// or a process that has set a hard memory budget.  This variant keeps that
// scratch in a fixed file-scope __device__ array instead, so a call performs
// no allocation of any kind.
//
// The array holds the keys of at most kNoAllocMaxRows token rows, one
// arrival counter and one error word.  Every call first clears it with a
// 256-byte cudaMemsetAsync on the caller's stream (ordered before the
// kernel; a memset allocates nothing), so a call never depends on what the
// previous one left there.  If a bounded wait inside the kernel gives up, the
// kernel sets the error word and writes -1 as every id.  Because there is one
// array per device, calls that overlap in time on one device (two streams,
// two host threads) race on it and may return wrong ids: serialise them.
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "matvec.cuh"

namespace qasr {

constexpr int kNoAllocMaxRows = 8;
constexpr int kNoAllocCounterWord = 16;  // counter at byte 128, after 8 keys (64 B) and padding
constexpr int kNoAllocErrWord = 17;      // error word at byte 136
constexpr int kNoAllocWords = 32;        // 256 bytes

static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocWords];

struct NoAllocSlot {
  unsigned long long *base = nullptr;
};
static NoAllocSlot g_noalloc_slots[64];
static std::mutex g_noalloc_mu;

// Resolve the device address of the array for the current device, once.  In
// host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory, so only the address returned here may be handed to a kernel.
static int noalloc_scratch(unsigned long long **base) {
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "qasr_final_norm_lmhead_argmax_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) {
    set_error("qasr_final_norm_lmhead_argmax_noalloc: device %d out of range", dev);
    return QASR_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocSlot &s = g_noalloc_slots[dev];
  if (!s.base) {
    void *p = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                     "qasr_final_norm_lmhead_argmax_noalloc: cudaGetSymbolAddress");
    if (rc) return rc;
    s.base = static_cast<unsigned long long *>(p);
  }
  *base = s.base;
  return QASR_OK;
}

}  // namespace qasr

using namespace qasr;

extern "C" int qasr_final_norm_lmhead_argmax_noalloc(int32_t *ids_out, float *logits_out, const float *x,
                                                     const float *norm_w, const int8_t *w, const float *scales, int M,
                                                     int hidden, int vocab, float eps, void *stream) {
  const char *fn = "qasr_final_norm_lmhead_argmax_noalloc";
  if (!ids_out || !x || !norm_w || !w || !scales || M < 0 || hidden <= 0 || vocab <= 0) {
    set_error("%s: invalid arguments", fn);
    return QASR_ERR_INVALID;
  }
  if (M > kNoAllocMaxRows) {
    set_error("%s: M=%d exceeds the fixed scratch (at most %d token rows per call)", fn, M, kNoAllocMaxRows);
    return QASR_ERR_INVALID;
  }
  // Shapes the allocation-free path covers: one K slice (no split-K
  // partials), x rows staged whole in shared memory.
  if (hidden % 512 || (size_t)kNoAllocMaxRows * hidden * 4 > 96 * 1024) {
    set_error("%s: hidden=%d must be a multiple of 512 and at most 3072", fn, hidden);
    return QASR_ERR_UNSUPPORTED;
  }
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(norm_w)) & 15) {
    set_error("%s: x, w and norm_w must be 16-byte aligned", fn);
    return QASR_ERR_UNSUPPORTED;
  }
  if (M == 0) return QASR_OK;
  Mv2Params p{};
  p.x = x;
  p.x_stride = hidden;
  p.norm_w = norm_w;
  p.eps = eps;
  p.w = w;
  p.scales = scales;
  p.y = logits_out;
  p.y_stride = vocab;
  p.M = M;
  p.K = hidden;
  p.N = vocab;
  p.S = 1;
  p.KS = hidden;
  p.KC = 512;
  p.ids = ids_out;
  unsigned long long *base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  p.keys = base;
  p.counter = reinterpret_cast<unsigned *>(base + kNoAllocCounterWord);
  p.err = reinterpret_cast<int *>(base + kNoAllocErrWord);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = cuda_status(cudaMemsetAsync(base, 0, sizeof(g_noalloc_scratch), st), "qasr_final_norm_lmhead_argmax_noalloc: clear scratch");
  if (rc) return rc;
  rc = mv2_launch(p, MvEpi::Argmax, st, false);
  return rc ? rc : launch_status(fn);
}
