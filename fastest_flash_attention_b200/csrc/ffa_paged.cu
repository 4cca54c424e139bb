// Paged KV-cache append: one warp per (token, kv head) copies a D-element
// row of K and of V into its page slot with 16-byte vector stores.
// Replaces the per-token Python loop of ops/kv_cache.py:192-204.
#include "ffa_common.cuh"
#include "ffa_host.h"

namespace ffa {

__global__ void ffa_paged_append_kernel(const uint16_t* __restrict__ k_new, const uint16_t* __restrict__ v_new,
                                        uint16_t* __restrict__ k_pages, uint16_t* __restrict__ v_pages,
                                        const int* __restrict__ slots, int n_tokens, int Hkv, int D, int page_size,
                                        int num_pages, int64_t s_head, int64_t s_tok) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= n_tokens * Hkv) return;
  const int tok = w / Hkv, h = w % Hkv;
  const int slot = slots[tok];
  const int page = slot / page_size, off = slot % page_size;
  if (slot < 0 || page >= num_pages) return;  // rejected on the host; never write outside the pool
  const int64_t dst = (((int64_t)page * Hkv + h) * page_size + off) * D;
  const int64_t src = (int64_t)h * s_head + (int64_t)tok * s_tok;
  for (int d = lane * 8; d < D; d += 256) {
    *reinterpret_cast<uint4*>(k_pages + dst + d) = *reinterpret_cast<const uint4*>(k_new + src + d);
    *reinterpret_cast<uint4*>(v_pages + dst + d) = *reinterpret_cast<const uint4*>(v_new + src + d);
  }
}

}  // namespace ffa

extern "C" int ffa_paged_append(const void* k_new, const void* v_new, void* k_pages, void* v_pages,
                                const int* slots, int dtype, int n_tokens, int Hkv, int D, int page_size,
                                int num_pages, const int64_t* new_strides, void* stream) {
  using namespace ffa;
  if (!k_new || !v_new || !k_pages || !v_pages || !slots || !new_strides) return FFA_ERR_INVALID_ARG;
  if (n_tokens < 0 || Hkv <= 0 || D <= 0 || page_size <= 0 || num_pages <= 0) return FFA_ERR_INVALID_ARG;
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16) return FFA_ERR_UNSUPPORTED;
  if (D % 8 || new_strides[0] % 8 || new_strides[1] % 8 || !aligned16(k_new) || !aligned16(v_new) ||
      !aligned16(k_pages) || !aligned16(v_pages))
    return FFA_ERR_INVALID_ARG;
  if (n_tokens == 0) return FFA_OK;
  const int warps = n_tokens * Hkv;
  ffa_paged_append_kernel<<<(warps * 32 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(k_new), static_cast<const uint16_t*>(v_new), static_cast<uint16_t*>(k_pages),
      static_cast<uint16_t*>(v_pages), slots, n_tokens, Hkv, D, page_size, num_pages, new_strides[0],
      new_strides[1]);
  return launch_status();
}
