// Host plumbing implementation and the small library-wide C-ABI functions.
#include <stdio.h>
#include <string.h>

#include "ffa_host.h"

namespace ffa {

static thread_local char g_last_error[256] = "";
static thread_local unsigned long long g_wait_limit_ns = 2000000000ull;

void set_last_error(const char* msg) {
  strncpy(g_last_error, msg ? msg : "", sizeof(g_last_error) - 1);
  g_last_error[sizeof(g_last_error) - 1] = 0;
}

unsigned long long wait_limit_ns() { return g_wait_limit_ns; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes, uint64_t d0,
                 uint64_t d1, uint64_t d2, uint64_t d3, uint64_t s1_bytes, uint64_t s2_bytes, uint64_t s3_bytes,
                 uint32_t b0, uint32_t b1) {
  // The driver-level encode needs the device's primary context current on
  // this thread (host threads such as autograd workers may not have it yet).
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled entry point unavailable");
    return FFA_ERR_CUDA;
  }
  // Degenerate outer dims may carry any stride; TMA still wants a valid one.
  if (d2 == 1) s2_bytes = s1_bytes * d1;
  if (d3 == 1) s3_bytes = s2_bytes * d2;
  if ((s1_bytes % 16) || (s2_bytes % 16) || (s3_bytes % 16) || !aligned16(base)) {
    set_last_error("TMA operand needs 16-byte aligned base and strides");
    return FFA_ERR_INVALID_ARG;
  }
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {s1_bytes, s2_bytes, s3_bytes};
  cuuint32_t box[4] = {b0, b1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  (void)elem_bytes;
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "cuTensorMapEncodeTiled failed (%d): dims {%llu,%llu,%llu,%llu} byte strides {%llu,%llu,%llu} base %p",
             (int)r, (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
             (unsigned long long)d3, (unsigned long long)s1_bytes, (unsigned long long)s2_bytes,
             (unsigned long long)s3_bytes, base);
    set_last_error(msg);
    return FFA_ERR_INVALID_ARG;
  }
  return FFA_OK;
}

}  // namespace ffa

extern "C" {

int ffa_version(void) { return 10000; }

const char* ffa_last_error(void) { return ffa::g_last_error; }

void ffa_set_wait_limit_ns(unsigned long long ns) { ffa::g_wait_limit_ns = ns ? ns : 2000000000ull; }

int ffa_read_error(const uint32_t* dev_err, uint32_t* out, void* stream) {
  if (!dev_err || !out) return FFA_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = ffa::cuda_status(cudaMemcpyAsync(out, dev_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  if (st) return st;
  return ffa::cuda_status(cudaStreamSynchronize(s));
}

}  // extern "C"
