// capi.cu -- library-level entry points and host helpers: thread-local error
// text, CUDA status checks, the tensor-map encoder, the device error word.
#include <atomic>
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"

namespace ltxq {

__device__ unsigned int g_dev_error = 0;

static PFN_cuCtxGetCurrent_v4000 g_ctx_get = nullptr;
static std::once_flag g_ctx_once;

void* current_cu_context() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  });
  CUcontext c = nullptr;
  if (g_ctx_get && g_ctx_get(&c) == CUDA_SUCCESS) return c;
  return nullptr;
}

// The error word's address per device, looked up again whenever the calling
// thread's current context differs from the one it was looked up in.
unsigned int* dev_error_word() {
  struct Entry {
    void* ctx;
    unsigned int* addr;
  };
  static Entry cache[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  Entry& e = cache[dev];
  const void* ctx = current_cu_context();
  if (e.addr && ctx && e.ctx == ctx) return e.addr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_dev_error) != cudaSuccess) return nullptr;
  e.ctx = current_cu_context();  // the lookup binds the device's context if none was current
  e.addr = static_cast<unsigned int*>(p);
  return e.addr;
}

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

ltxq_status launch_check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) note_launch();
  return cuda_check(e, what);
}

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

ltxq_status fail(ltxq_status code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

ltxq_status cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LTXQ_OK;
  return fail(LTXQ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static ltxq_status encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                               const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                               CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(LTXQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the CUDA driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(LTXQ_ERR_INVALID, "TMA base address must be 16-byte aligned");
  cuuint64_t d[3];
  cuuint64_t st[2];
  cuuint32_t bx[3];
  cuuint32_t estr[3] = {1, 1, 1};
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    if (i + 1 < rank) {
      if (strides[i] % 16 != 0) return fail(LTXQ_ERR_INVALID, "TMA strides must be multiples of 16 bytes");
      st[i] = strides[i];
    }
  }
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[200];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d) rank %u dims=(%llu,%llu,%llu) box=(%u,%u,%u)",
             (int)r, rank, (unsigned long long)dims[0], (unsigned long long)dims[1],
             (unsigned long long)(rank > 2 ? dims[2] : 1), box[0], box[1], rank > 2 ? box[2] : 1u);
    return fail(LTXQ_ERR_CUDA, buf);
  }
  return LTXQ_OK;
}

ltxq_status encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner_elems,
                           uint64_t outer_rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                           CUtensorMapSwizzle swizzle) {
  const uint64_t dims[2] = {inner_elems, outer_rows};
  const uint64_t strides[1] = {row_stride_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return encode_tmap(map, dtype, 2, base, dims, strides, box, swizzle);
}

ltxq_status encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
                           const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle) {
  return encode_tmap(map, dtype, 3, base, dims, strides_bytes, box, swizzle);
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// One warp: lane 0 waits, through the bounded mbarrier wait of the GEMM
// kernels, for phase 0 of a barrier that expects one arrival and never gets
// it.  The wait gives up after limit_ns, raises the device error word and the
// kernel returns normally (no trap, no fault): the failure-detection path of
// every kernel, exercised on its own.
__global__ void wait_selftest_kernel(unsigned int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err, limit_ns);
  __syncthreads();
}

}  // namespace ltxq

extern "C" {

const char* ltxq_last_error(void) { return ltxq::t_last_error.c_str(); }

uint64_t ltxq_launch_count(void) { return ltxq::g_launches.load(std::memory_order_relaxed); }

const char* ltxq_version(void) { return "ltxq 0.1 (sm_100a)"; }

ltxq_status ltxq_device_error(int32_t* code_out) {
  if (!code_out) return ltxq::fail(LTXQ_ERR_INVALID, "code_out is NULL");
  ltxq_status st = ltxq::cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (st) return st;
  unsigned int v = 0, zero = 0;
  st = ltxq::cuda_check(cudaMemcpyFromSymbol(&v, ltxq::g_dev_error, sizeof(v)), "read device error");
  if (st) return st;
  st = ltxq::cuda_check(cudaMemcpyToSymbol(ltxq::g_dev_error, &zero, sizeof(zero)), "clear device error");
  if (st) return st;
  *code_out = static_cast<int32_t>(v);
  return LTXQ_OK;
}

ltxq_status ltxq_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  if (limit_ns < 1000ull || limit_ns > 1000000000ull)
    return ltxq::fail(LTXQ_ERR_INVALID, "selftest_wait_timeout: limit_ns must be within [1 us, 1 s]");
  unsigned int* err = ltxq::dev_error_word();
  if (!err) return ltxq::fail(LTXQ_ERR_CUDA, "selftest_wait_timeout: device error word unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ltxq::wait_selftest_kernel<<<1, 32, 0, s>>>(err, limit_ns);
  if (ltxq_status st = ltxq::launch_check("wait self-test launch")) return st;
  if (ltxq_status st = ltxq::cuda_check(cudaStreamSynchronize(s), "wait self-test")) return st;
  unsigned int v = 0;
  if (ltxq_status st = ltxq::cuda_check(cudaMemcpyFromSymbol(&v, ltxq::g_dev_error, sizeof(v)), "read device error"))
    return st;
  if (v == 0) return ltxq::fail(LTXQ_ERR_CUDA, "selftest_wait_timeout: the wait did not report its expiry");
  char buf[160];
  snprintf(buf, sizeof(buf), "bounded wait expired after %llu ns as designed (device error word = %u)",
           static_cast<unsigned long long>(limit_ns), v);
  return ltxq::fail(LTXQ_ERR_DEVICE, buf);
}

}  // extern "C"
