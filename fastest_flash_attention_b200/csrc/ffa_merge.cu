// Merge of a partial attention result into a running one, by log-sum-exp:
//   L = logaddexp(L_acc, L_part)
//   O_acc = O_acc * e^(L_acc - L) + O_part * e^(L_part - L)
// used by the sequence-sharded ring (each step attends the local queries to
// one rank's K/V block).  One warp per row, fp32 running state, 16-bit or
// fp32 partials; rows whose partial saw no key (L_part = -inf) are left as
// they are.  HBM-bound: reads O_acc and O_part once, writes O_acc once.
#include "ffa_common.cuh"
#include "ffa_host.h"

namespace ffa {

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T>
__global__ void ffa_merge_partial_kernel(float* __restrict__ o_acc, float* __restrict__ lse_acc,
                                         const T* __restrict__ o_part, const float* __restrict__ lse_part,
                                         int64_t rows, int D) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= rows) return;
  const float la = lse_acc[w], lp = lse_part[w];
  if (lp == -INFINITY) return;
  const float m = fmaxf(la, lp);
  const float wa = la == -INFINITY ? 0.f : __expf(la - m);
  const float wp = __expf(lp - m);
  const float inv = 1.f / (wa + wp);
  float* acc = o_acc + w * D;
  const T* part = o_part + w * D;
  for (int d = lane; d < D; d += 32) acc[d] = (acc[d] * wa + to_f<T>(part[d]) * wp) * inv;
  if (lane == 0) lse_acc[w] = m + __logf(wa + wp);
}

}  // namespace ffa

extern "C" int ffa_merge_partial(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part, int dtype,
                                 int64_t rows, int D, void* stream) {
  using namespace ffa;
  if (!o_acc || !lse_acc || !o_part || !lse_part || rows < 0 || D <= 0) return FFA_ERR_INVALID_ARG;
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16) return FFA_ERR_UNSUPPORTED;
  if (rows == 0) return FFA_OK;
  const int64_t threads = rows * 32;
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FFA_DTYPE_BF16)
    ffa_merge_partial_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        o_acc, lse_acc, static_cast<const __nv_bfloat16*>(o_part), lse_part, rows, D);
  else
    ffa_merge_partial_kernel<__half><<<blocks, 256, 0, s>>>(o_acc, lse_acc, static_cast<const __half*>(o_part),
                                                             lse_part, rows, D);
  return launch_status();
}
