// Host-side plumbing shared by the C-ABI entry points: CUDA error capture,
// the per-thread wait limit, and TMA tensor-map encoding through the driver
// entry point (so the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "ffa_b200.h"

namespace ffa {

void set_last_error(const char* msg);
unsigned long long wait_limit_ns();

// Records the CUDA error string (if any) and maps it to a status.
inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return FFA_OK;
  set_last_error(cudaGetErrorString(e));
  return FFA_ERR_CUDA;
}

// Status of the most recent launch on this thread.
inline int launch_status() { return cuda_status(cudaGetLastError()); }

// Encodes a 4-D tiled TMA map over a row-major tensor whose innermost dim is
// contiguous: dims {d0 (contiguous), d1, d2, d3}, byte strides for d1..d3,
// box {b0, b1, 1, 1}, 128-byte swizzle, zero fill out of bounds.
int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes, uint64_t d0,
                 uint64_t d1, uint64_t d2, uint64_t d3, uint64_t s1_bytes, uint64_t s2_bytes, uint64_t s3_bytes,
                 uint32_t b0, uint32_t b1);

// Raises a kernel's dynamic shared-memory limit once per device.  The
// attribute belongs to the device's context, so the "done" record is a bit
// per device; the record is atomic because entry points may be called from
// several host threads (setting the attribute twice is harmless).
template <typename Kernel>
int smem_attr_once(Kernel kern, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  int s = cuda_status(cudaGetDevice(&dev));
  if (s) return s;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return FFA_OK;
  s = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (s) return s;
  if (bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return FFA_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// fp32 kernels on the CUDA cores (ffa_f32.cu), reached through ffa_fwd /
// ffa_bwd / ffa_bwd_masked with dtype FFA_DTYPE_F32.
int f32_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv, int Sq,
            int Skv, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
            const int64_t* o_strides, float scale, int causal, int q_offset, int window, float softcap,
            const uint8_t* block_mask, int n_br, int n_bc, int mask_bq, int mask_bkv, void* stream);
int f32_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
            void* dq, void* dk, void* dv, int B, int Hq, int Hkv, int Sq, int Skv, int D, int Dv,
            const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
            const int64_t* o_strides, const int64_t* do_strides, const int64_t* dq_strides,
            const int64_t* dk_strides, const int64_t* dv_strides, float scale, int causal, int q_offset,
            int window, float softcap, const uint8_t* block_mask, int n_br, int n_bc, int mask_bq, int mask_bkv,
            void* workspace, void* stream);

}  // namespace ffa
