// ffa_bwd_noalloc: the backward of ffa_bwd for callers that cannot allocate
// device memory.
//
// ffa_bwd needs a scratch workspace (the padded base-2 LSE and Delta rows).
// Some callers have no way to provide one: code running inside a framework
// whose memory is owned by a pool they cannot reach, plugins that are handed
// only their input and output buffers, or hosts where calling cudaMalloc
// mid-step is forbidden because it synchronises the device.  This entry point
// uses a fixed scratch array compiled into the library instead, so it calls
// no cudaMalloc, cudaFree or other allocating routine.
//
// Limits and sharing rules:
//  * The scratch holds FFA_BWD_NOALLOC_MAX_ROWS (batch x query heads x query
//    length rounded up to 128) rows; larger problems are rejected with
//    FFA_ERR_UNSUPPORTED.  Every GPU that loads the library keeps this array
//    (8 MiB + 256 B) for the life of the process.
//  * Only D == Dv is served (query/key and value head dims equal); the
//    MLA training shape (192, 128) needs ffa_bwd with a workspace.
//  * All calls on a device share the one array.  Each call overwrites every
//    scratch row it later reads, so nothing needs clearing between calls, but
//    calls whose kernels overlap on the GPU (different streams, or different
//    host threads on one device without ordering) race on it.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make that
//    first call before any stream capture.
#include <mutex>

#include "ffa_common.cuh"
#include "ffa_host.h"

namespace ffa {

constexpr size_t BWD_NOALLOC_BYTES = 2ull * FFA_BWD_NOALLOC_MAX_ROWS * sizeof(float) + 256;

// Device-side scratch.  In host code this name is only a stand-in for the
// symbol, never a usable device address: the address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_bwd_scratch[BWD_NOALLOC_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
static void* g_scratch_ptr[NOALLOC_MAX_DEVICES] = {};
static std::mutex g_scratch_mu;

// Returns the device address of g_bwd_scratch on the current device.
static int scratch_address(void** out) {
  int dev = 0;
  int st = cuda_status(cudaGetDevice(&dev));
  if (st) return st;
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) {
    set_last_error("ffa_bwd_noalloc: device index beyond the supported range");
    return FFA_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    st = cuda_status(cudaGetSymbolAddress(&p, g_bwd_scratch));
    if (st) return st;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FFA_OK;
}

}  // namespace ffa

extern "C" int ffa_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v, const void* o,
                               const float* lse, void* dq, void* dk, void* dv, int dtype, int B, int Hq, int Hkv,
                               int Sq, int Skv, int D, const int64_t* q_strides, const int64_t* k_strides,
                               const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                               const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                               float scale, int causal, int q_offset, int window, float softcap, uint32_t* dev_err,
                               void* stream) {
  using namespace ffa;
  if (B <= 0 || Hq <= 0 || Sq <= 0) return FFA_ERR_INVALID_ARG;
  const size_t rows = (size_t)B * Hq * (((size_t)Sq + 127) / 128 * 128);
  if (rows > (size_t)FFA_BWD_NOALLOC_MAX_ROWS) {
    set_last_error("ffa_bwd_noalloc: B * Hq * round_up(Sq, 128) exceeds FFA_BWD_NOALLOC_MAX_ROWS");
    return FFA_ERR_UNSUPPORTED;
  }
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st) return st;
  return ffa_bwd(dout, q, k, v, o, lse, dq, dk, dv, dtype, B, Hq, Hkv, Sq, Skv, D, D, q_strides, k_strides, v_strides,
                 o_strides, do_strides, dq_strides, dk_strides, dv_strides, scale, causal, q_offset, window, softcap,
                 scratch, BWD_NOALLOC_BYTES, dev_err, stream);
}
