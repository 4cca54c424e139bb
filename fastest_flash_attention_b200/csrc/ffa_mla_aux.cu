// The projections around the MLA absorbed decode, fused per side of the
// attention (modules/flash_mla.py:133-152 builds them with separate
// projections, a RoPE module and up-projected K/V; the absorbed decode needs
// instead):
//   * ffa_mla_q_absorb: q = [q_nope . W_UK (latent) | rope(q_rope, pos)] per
//     request and head, the decode kernel's query [R, H, L + rope];
//   * ffa_mla_o_absorb: o = o_lat . W_UV^T per head, written as the rows of
//     o_proj's input [R, H * (d + rope)] with the reference's zero value
//     columns for the rope part (flash_mla.py:152);
//   * ffa_mla_latent_append: cache rows [c_kv | rope(k_rope, pos)] scattered
//     into their page slots.
// These are small, HBM-bound products (the weights are read once per call);
// each is one launch in place of a chain of eager ops and a per-request
// Python loop.  Activations and weights may be fp32, bf16 or fp16; the
// latent side (decode query, latent output, cache) is bf16 or fp16.
// RoPE is the half-split rotation with fp32 angles pos * inv_freq[i].
#include <type_traits>

#include "ffa_common.cuh"
#include "ffa_host.h"

namespace ffa {

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  if constexpr (std::is_same<T, float>::value)
    return *p;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __bfloat162float(*p);
  else
    return __half2float(*p);
}

template <typename T>
__device__ __forceinline__ T cvt(float x) {
  if constexpr (std::is_same<T, float>::value)
    return x;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __float2bfloat16_rn(x);
  else
    return __float2half_rn(x);
}

// Rotation of the pair (x1 = x[i], x2 = x[i + rope/2]) by angle pos * inv_freq[i].
__device__ __forceinline__ float2 rope_pair(float x1, float x2, int pos, float inv_freq) {
  float s, c;
  sincosf((float)pos * inv_freq, &s, &c);
  return make_float2(x1 * c - x2 * s, x2 * c + x1 * s);
}

constexpr int QA_COLS = 64;   // latent columns per CTA
constexpr int QA_RTILE = 32;  // requests staged in smem at a time

// grid (L / 64 + 1, H): x < L / 64 computes 64 latent columns of head h for
// every request; the last x rotates head h's rope part.
template <typename TI, typename TL>
__global__ void __launch_bounds__(256) ffa_mla_q_absorb_kernel(
    const TI* __restrict__ q_nope, int64_t qn_sr, int64_t qn_sh, const TI* __restrict__ q_rope, int64_t qr_sr,
    int64_t qr_sh, const TI* __restrict__ w_uk, int64_t w_sh, int64_t w_sj, const int* __restrict__ pos,
    const float* __restrict__ inv_freq, TL* __restrict__ out, int64_t o_sr, int64_t o_sh, int R, int d, int L,
    int rope) {
  __shared__ float sq[QA_RTILE * 192];
  const int h = blockIdx.y;
  if (blockIdx.x == L / QA_COLS) {  // rope part: pairs (i, i + rope/2)
    const int half = rope / 2;
    for (int e = threadIdx.x; e < R * half; e += blockDim.x) {
      const int r = e / half, i = e % half;
      const TI* src = q_rope + (int64_t)r * qr_sr + (int64_t)h * qr_sh;
      const float2 y = rope_pair(ldf(src + i), ldf(src + i + half), pos[r], inv_freq[i]);
      TL* dst = out + (int64_t)r * o_sr + (int64_t)h * o_sh + L;
      dst[i] = cvt<TL>(y.x);
      dst[i + half] = cvt<TL>(y.y);
    }
    return;
  }
  const int c = blockIdx.x * QA_COLS + threadIdx.x % QA_COLS;  // latent column of this thread
  const int rg = threadIdx.x / QA_COLS;                          // request group 0..3
  const TI* wcol = w_uk + (int64_t)h * w_sh + c;
  for (int r0 = 0; r0 < R; r0 += QA_RTILE) {
    const int nr = min(QA_RTILE, R - r0);
    __syncthreads();
    for (int e = threadIdx.x; e < nr * d; e += blockDim.x) {
      const int r = e / d, j = e % d;
      sq[r * d + j] = ldf(q_nope + (int64_t)(r0 + r) * qn_sr + (int64_t)h * qn_sh + j);
    }
    __syncthreads();
    float acc[QA_RTILE / 4];
#pragma unroll
    for (int k = 0; k < QA_RTILE / 4; ++k) acc[k] = 0.f;
    for (int j = 0; j < d; ++j) {
      const float w = ldf(wcol + (int64_t)j * w_sj);
#pragma unroll
      for (int k = 0; k < QA_RTILE / 4; ++k) {
        const int r = rg + 4 * k;
        if (r < nr) acc[k] = fmaf(sq[r * d + j], w, acc[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < QA_RTILE / 4; ++k) {
      const int r = rg + 4 * k;
      if (r < nr) out[(int64_t)(r0 + r) * o_sr + (int64_t)h * o_sh + c] = cvt<TL>(acc[k]);
    }
  }
}

// grid (H, d / 32): warp w of the CTA computes output dims 4 w .. 4 w + 3 of
// head h (of the CTA's 32) for every request; lanes split the latent sum.
template <typename TL, typename TI>
__global__ void __launch_bounds__(256) ffa_mla_o_absorb_kernel(const TL* __restrict__ o_lat, int64_t ol_sr,
                                                               int64_t ol_sh, const TI* __restrict__ w_uv,
                                                               int64_t w_sh, int64_t w_si, TI* __restrict__ out,
                                                               int64_t o_sr, int R, int d, int L, int rope) {
  const int h = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int seg = L / 32;  // latent elements per lane (16 at L = 512)
  for (int ii = 0; ii < 4; ++ii) {
    const int i = blockIdx.y * 32 + warp * 4 + ii;
    if (i >= d) break;
    float w[32];
    const TI* wr = w_uv + (int64_t)h * w_sh + (int64_t)i * w_si + lane * seg;
#pragma unroll
    for (int e = 0; e < 32; ++e) w[e] = e < seg ? ldf(wr + e) : 0.f;
    for (int r = 0; r < R; ++r) {
      const TL* xr = o_lat + (int64_t)r * ol_sr + (int64_t)h * ol_sh + lane * seg;
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (e < seg) acc = fmaf(ldf(xr + e), w[e], acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) out[(int64_t)r * o_sr + (int64_t)h * (d + rope) + i] = cvt<TI>(acc);
    }
  }
  // the rope columns of this head's output are zero (the reference pads V)
  if (blockIdx.y == 0)
    for (int e = threadIdx.x; e < R * rope; e += blockDim.x)
      out[(int64_t)(e / rope) * o_sr + (int64_t)h * (d + rope) + d + e % rope] = cvt<TI>(0.f);
}

// One CTA per token: row [lat (L) | rope(kr, pos) (rope)] -> page slot.
template <typename TI, typename TL>
__global__ void __launch_bounds__(128) ffa_mla_latent_append_kernel(const TI* __restrict__ lat, int64_t lat_s,
                                                                    const TI* __restrict__ kr, int64_t kr_s,
                                                                    const int* __restrict__ pos,
                                                                    const int* __restrict__ slots,
                                                                    const float* __restrict__ inv_freq,
                                                                    TL* __restrict__ rows, int64_t n_slots, int L,
                                                                    int rope) {
  const int t = blockIdx.x;
  const int slot = slots[t];
  if (slot < 0 || slot >= n_slots) return;  // checked on the host; never write outside the cache
  TL* dst = rows + (int64_t)slot * (L + rope);
  const TI* src = lat + (int64_t)t * lat_s;
  for (int e = threadIdx.x; e < L; e += blockDim.x) dst[e] = cvt<TL>(ldf(src + e));
  const int half = rope / 2;
  const TI* k = kr + (int64_t)t * kr_s;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float2 y = rope_pair(ldf(k + i), ldf(k + i + half), pos[t], inv_freq[i]);
    dst[L + i] = cvt<TL>(y.x);
    dst[L + i + half] = cvt<TL>(y.y);
  }
}

// Calls f with the C++ types of (activation/weight dtype, latent dtype).
template <typename F>
static int dispatch2(int in_dtype, int lat_dtype, F f) {
  if (lat_dtype != FFA_DTYPE_BF16 && lat_dtype != FFA_DTYPE_F16) return FFA_ERR_UNSUPPORTED;
  auto with_lat = [&](auto ti) -> int {
    using TI = decltype(ti);
    if (lat_dtype == FFA_DTYPE_BF16) return f(TI{}, __nv_bfloat16{});
    return f(TI{}, __half{});
  };
  if (in_dtype == FFA_DTYPE_F32) return with_lat(float{});
  if (in_dtype == FFA_DTYPE_BF16) return with_lat(__nv_bfloat16{});
  if (in_dtype == FFA_DTYPE_F16) return with_lat(__half{});
  return FFA_ERR_UNSUPPORTED;
}

}  // namespace ffa

extern "C" int ffa_mla_q_absorb(const void* q_nope, const int64_t* qn_strides, const void* q_rope,
                                const int64_t* qr_strides, const void* w_uk, const int64_t* w_strides,
                                const int* pos, const float* inv_freq, void* out, const int64_t* o_strides,
                                int in_dtype, int lat_dtype, int R, int H, int d, int L, int rope, void* stream) {
  using namespace ffa;
  if (!q_nope || !q_rope || !w_uk || !pos || !inv_freq || !out || !qn_strides || !qr_strides || !w_strides ||
      !o_strides)
    return FFA_ERR_INVALID_ARG;
  if (R < 0 || H <= 0 || d <= 0 || L <= 0 || rope <= 0 || rope % 2) return FFA_ERR_INVALID_ARG;
  if (L % QA_COLS || d > 192 || H > 65535) return FFA_ERR_UNSUPPORTED;
  if (R == 0) return FFA_OK;
  return dispatch2(in_dtype, lat_dtype, [&](auto ti, auto tl) -> int {
    using TI = decltype(ti);
    using TL = decltype(tl);
    ffa_mla_q_absorb_kernel<TI, TL><<<dim3(L / QA_COLS + 1, H), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const TI*>(q_nope), qn_strides[0], qn_strides[1], static_cast<const TI*>(q_rope),
        qr_strides[0], qr_strides[1], static_cast<const TI*>(w_uk), w_strides[0], w_strides[1], pos, inv_freq,
        static_cast<TL*>(out), o_strides[0], o_strides[1], R, d, L, rope);
    return launch_status();
  });
}

extern "C" int ffa_mla_o_absorb(const void* o_lat, const int64_t* ol_strides, const void* w_uv,
                                const int64_t* w_strides, void* out, int64_t out_row_stride, int in_dtype,
                                int lat_dtype, int R, int H, int d, int L, int rope, void* stream) {
  using namespace ffa;
  if (!o_lat || !w_uv || !out || !ol_strides || !w_strides) return FFA_ERR_INVALID_ARG;
  if (R < 0 || H <= 0 || d <= 0 || L <= 0 || rope < 0) return FFA_ERR_INVALID_ARG;
  if (L % 32 || L > 1024) return FFA_ERR_UNSUPPORTED;
  if (R == 0) return FFA_OK;
  return dispatch2(in_dtype, lat_dtype, [&](auto ti, auto tl) -> int {
    using TI = decltype(ti);
    using TL = decltype(tl);
    ffa_mla_o_absorb_kernel<TL, TI><<<dim3(H, (d + 31) / 32), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const TL*>(o_lat), ol_strides[0], ol_strides[1], static_cast<const TI*>(w_uv), w_strides[0],
        w_strides[1], static_cast<TI*>(out), out_row_stride, R, d, L, rope);
    return launch_status();
  });
}

extern "C" int ffa_mla_latent_append(const void* lat, int64_t lat_row_stride, const void* kr, int64_t kr_row_stride,
                                     const int* pos, const int* slots, const float* inv_freq, void* rows,
                                     int64_t n_slots, int in_dtype, int lat_dtype, int n_tokens, int L, int rope,
                                     void* stream) {
  using namespace ffa;
  if (!lat || !kr || !pos || !slots || !inv_freq || !rows) return FFA_ERR_INVALID_ARG;
  if (n_tokens < 0 || L <= 0 || rope <= 0 || rope % 2 || n_slots <= 0) return FFA_ERR_INVALID_ARG;
  if (n_tokens == 0) return FFA_OK;
  return dispatch2(in_dtype, lat_dtype, [&](auto ti, auto tl) -> int {
    using TI = decltype(ti);
    using TL = decltype(tl);
    ffa_mla_latent_append_kernel<TI, TL><<<n_tokens, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const TI*>(lat), lat_row_stride, static_cast<const TI*>(kr), kr_row_stride, pos, slots,
        inv_freq, static_cast<TL*>(rows), n_slots, L, rope);
    return launch_status();
  });
}
