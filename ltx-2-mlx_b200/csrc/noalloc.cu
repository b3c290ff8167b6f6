// noalloc.cu -- ltxq_adaln_qlinear_noalloc: the AdaLN-prologue quantized
// linear without a workspace argument and without any device allocation.
//
// Some hosts cannot let a library allocate device memory: a serving runtime
// that reserves all of the GPU's memory up front and hands out only its own
// pool, a plugin running inside another framework's allocator whose
// accounting would break behind its back, or a latency-critical loop where a
// cudaMalloc / cudaFree (which may synchronize the device and stall every
// stream) is not acceptable.  This entry point serves them: its one piece of
// scratch -- the modulated activations that ltxq_adaln_qlinear keeps in the
// caller's workspace -- lives in a fixed-size array that is part of the
// library's device image instead.
//
// Properties a caller must know:
//  * the array holds at most kNoAllocScratchElems bf16 values (8 MiB): M * K
//    up to 4,194,304 (for example 1024 tokens x 4096 channels); larger
//    requests are rejected with LTXQ_ERR_UNSUPPORTED and launch nothing;
//  * every GPU that loads the library keeps these 8 MiB reserved until the
//    process exits;
//  * every call uses the same array, which keeps whatever the previous call
//    left in it.  Nothing has to start at zero: each call overwrites the
//    M x K values it reads.  Calls whose work overlaps on the GPU (different
//    streams without ordering between them, or several host threads) race on
//    the array, so callers must serialize them;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, once per device, with that device current) and
//    caches it.  Make that first call before any stream capture.  The cache
//    is keyed by the CUDA context as well: after a cudaDeviceReset the next
//    call looks the address up again in the new context (again outside any
//    capture).
//  * no cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "common.cuh"

namespace ltxq {

ltxq_status launch_adaln_modulate(const void* x, int x_dtype, int64_t rows, int64_t C, const ltxq_prologue& pro,
                                  void* out, cudaStream_t stream, const ltxq_mx_act* out_mx);
ltxq_status launch_qlinear(const void* x, int64_t M, const ltxq_qweight& w, const ltxq_epilogue* epi, void* out,
                           cudaStream_t stream, void* workspace, size_t workspace_bytes);

constexpr size_t kNoAllocScratchElems = size_t(4) << 20;  // bf16 values (8 MiB)

// The scratch itself.  In host code this name is only a handle for the
// runtime's symbol lookup, never a device address.
static __device__ __align__(256) uint16_t g_noalloc_scratch[kNoAllocScratchElems];

// Device address of g_noalloc_scratch on the current device: looked up once
// per device and context, cached, and looked up again when the calling
// thread's current context is not the one the address came from.
static ltxq_status noalloc_scratch(void** out) {
  struct Entry {
    void* ctx;
    void* addr;
  };
  static Entry cache[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (ltxq_status st = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return st;
  if (dev < 0 || dev >= 64) return fail(LTXQ_ERR_UNSUPPORTED, "adaln_qlinear_noalloc: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(mu);
  Entry& e = cache[dev];
  const void* ctx = current_cu_context();
  if (!e.addr || !ctx || e.ctx != ctx) {
    void* p = nullptr;
    if (ltxq_status st = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)"))
      return st;
    e.ctx = current_cu_context();  // the lookup binds the device's context if none was current
    e.addr = p;
  }
  *out = e.addr;
  return LTXQ_OK;
}

}  // namespace ltxq

extern "C" ltxq_status ltxq_adaln_qlinear_noalloc(const void* x, int64_t M, const ltxq_prologue* pro,
                                                  const ltxq_qweight* w, const ltxq_epilogue* epi, void* out,
                                                  void* stream) {
  using namespace ltxq;
  if (!w || !pro || !x || !out) return fail(LTXQ_ERR_INVALID, "adaln_qlinear_noalloc: NULL argument");
  if (M < 0 || w->k_in <= 0) return fail(LTXQ_ERR_INVALID, "adaln_qlinear_noalloc: bad shape");
  if (M > 0 && static_cast<uint64_t>(M) * static_cast<uint64_t>(w->k_in) > kNoAllocScratchElems)
    return fail(LTXQ_ERR_UNSUPPORTED,
                "adaln_qlinear_noalloc: M * K exceeds the 4194304-element (8 MiB) static scratch; use "
                "ltxq_adaln_qlinear with a caller workspace");
  if (M == 0) return LTXQ_OK;
  void* scratch = nullptr;
  if (ltxq_status st = noalloc_scratch(&scratch)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ltxq_status st = launch_adaln_modulate(x, LTXQ_BF16, M, w->k_in, *pro, scratch, s, nullptr)) return st;
  return launch_qlinear(scratch, M, *w, epi, out, s, nullptr, 0);  // unsplit: no partials
}
