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

unsigned int* dev_error_word() {
  static unsigned int* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_error) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<unsigned int*>(p);
  }
  return addr[dev];
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

ltxq_status encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner_elems,
                           uint64_t outer_rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
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
  if (row_stride_bytes % 16 != 0) return fail(LTXQ_ERR_INVALID, "TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner_elems, outer_rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d) dims=(%llu,%llu) box=(%u,%u)", (int)r,
             (unsigned long long)inner_elems, (unsigned long long)outer_rows, box_inner, box_outer);
    return fail(LTXQ_ERR_CUDA, buf);
  }
  return LTXQ_OK;
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
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

}  // extern "C"
