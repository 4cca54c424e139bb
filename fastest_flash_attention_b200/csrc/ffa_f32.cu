// fp32 attention on the CUDA cores: forward, Delta preprocess, dK/dV and dQ.
//
// The reference computes fp32 inputs in fp32 (kernels/cpu_reference.py:132-312
// forward, :319-427 backward; _to_compute_dtype at :28-32 leaves fp32 alone when
// no compute_dtype is given), and its own tests hold fp32 results to 1e-5
// (tests/test_fastest_flash.py).  The tensor cores have no fp32 operand type
// (tf32 keeps 10 mantissa bits, an error near 1e-3), so fp32 callers are served
// here by FFMA register tiles with fp32 accumulation, the same arithmetic as the
// reference's fp32 matmuls up to summation order.
//
// Tiles: 64 queries x 64 keys per step, 256 threads; thread (ty, tx) = (t / 16,
// t % 16) holds rows 4*ty .. 4*ty+3 and score columns tx + 16*j (j < 4), and
// output columns 4*tx + 64*c .. +3 (c < width / 64).  Operand tiles sit in
// shared memory row-major with 4 floats of padding per row, so the 16-byte loads
// of the 16 threads of a row group hit distinct banks.  Masks (bounds, causal,
// window, block mask) are applied per element; key / query tiles outside the
// causal / window band are not visited.  The backward is deterministic: dK / dV
// and dQ are summed in a fixed order by the one CTA that owns each output tile.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "ffa_b200.h"
#include "ffa_host.h"

namespace ffa {
namespace {

constexpr int F_BM = 64;  // queries per tile
constexpr int F_BN = 64;  // keys per tile
constexpr int F_THREADS = 256;

struct F32Params {
  const float* q;
  const float* k;
  const float* v;
  const float* o;      // backward: the forward's output
  const float* dout;   // backward
  float* out;          // forward output
  float* lse;          // forward: may be null; backward: natural-log LSE [B, Hq, Sq]
  float* dq;
  float* dk;
  float* dv;
  float* delta;        // backward scratch [B, Hq, Sq]
  int64_t q_s[3], k_s[3], v_s[3], o_s[3], do_s[3], out_s[3], dq_s[3], dk_s[3], dv_s[3];
  int B, Hq, Hkv, Sq, Skv, q_offset, causal, window;
  float scale, softcap;
  const uint8_t* bm;
  int n_br, n_bc, mbq, mbk;
};

// Whether key j is visible to query i (both in range).
__device__ __forceinline__ bool f32_visible(const F32Params& p, int i, int j) {
  if (i >= p.Sq || j >= p.Skv) return false;
  if (p.causal && j > i + p.q_offset) return false;
  if (p.window > 0 && j < i + p.q_offset - p.window + 1) return false;
  if (p.bm && !p.bm[(size_t)(i / p.mbq) * p.n_bc + j / p.mbk]) return false;
  return true;
}

// Keys [lo, hi) that queries [i0, i1] can see under causal / window.
__device__ __forceinline__ void f32_key_range(const F32Params& p, int i0, int i1, int& lo, int& hi) {
  lo = 0;
  hi = p.Skv;
  if (p.causal) hi = min(hi, i1 + p.q_offset + 1);
  if (p.window > 0) lo = max(lo, i0 + p.q_offset - p.window + 1);
}

// Queries [lo, hi) that can see keys [j0, j1].
__device__ __forceinline__ void f32_query_range(const F32Params& p, int j0, int j1, int& lo, int& hi) {
  lo = 0;
  hi = p.Sq;
  if (p.causal) lo = max(lo, j0 - p.q_offset);
  if (p.window > 0) hi = min(hi, j1 - p.q_offset + p.window);
}

// Copies rows [r0, r0 + 64) of a [*, W] fp32 matrix (row stride `rs` elements)
// into smem rows of pitch W + 4; rows at or past `nrows` become zero.
template <int W>
__device__ __forceinline__ void f32_load_tile(float* dst, const float* src, int64_t rs, int r0, int nrows) {
  constexpr int V4 = W / 4;
  for (int idx = threadIdx.x; idx < 64 * V4; idx += F_THREADS) {
    const int r = idx / V4, c = idx % V4;
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < nrows) val = *reinterpret_cast<const float4*>(src + (int64_t)(r0 + r) * rs + 4 * c);
    *reinterpret_cast<float4*>(dst + r * (W + 4) + 4 * c) = val;
  }
}

// f32_load_tile through cp.async (16-byte copies, rows past `nrows` zero-filled):
// the copies are in flight until cp_async_wait; a commit groups them.
template <int W>
__device__ __forceinline__ void f32_load_tile_async(float* dst, const float* src, int64_t rs, int r0, int nrows) {
  constexpr int V4 = W / 4;
  for (int idx = threadIdx.x; idx < 64 * V4; idx += F_THREADS) {
    const int r = idx / V4, c = idx % V4;
    const bool in = r0 + r < nrows;
    const float* g = in ? src + (int64_t)(r0 + r) * rs + 4 * c : src;
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(dst + r * (W + 4) + 4 * c);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(g), "r"(in ? 16 : 0) : "memory");
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// acc[i][j] = sum_d A[4*ty + i][d] * Bm[tx + 16*j][d] over d < W (tiles of pitch W + 4).
template <int W>
__device__ __forceinline__ void f32_scores(const float* A, const float* Bm, int ty, int tx, float acc[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
  for (int d = 0; d < W; d += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(A + (4 * ty + i) * (W + 4) + d);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(Bm + (tx + 16 * j) * (W + 4) + d);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
        acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
        acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
        acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
      }
  }
}

// acc[i][c] (4 floats each) += sum_k P[4*ty + i][k] * M[k][4*tx + 64*c ..] over
// k < 64: P has pitch 68, M has pitch W + 4.
template <int W>
__device__ __forceinline__ void f32_accumulate(const float* P, const float* M, int ty, int tx,
                                               float4 acc[4][W / 64]) {
#pragma unroll 2
  for (int k = 0; k < 64; k += 4) {
    float4 pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = *reinterpret_cast<const float4*>(P + (4 * ty + i) * 68 + k);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int c = 0; c < W / 64; ++c) {
        const float4 m = *reinterpret_cast<const float4*>(M + (k + kk) * (W + 4) + 4 * tx + 64 * c);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float pv = kk == 0 ? pr[i].x : kk == 1 ? pr[i].y : kk == 2 ? pr[i].z : pr[i].w;
          acc[i][c].x = fmaf(pv, m.x, acc[i][c].x);
          acc[i][c].y = fmaf(pv, m.y, acc[i][c].y);
          acc[i][c].z = fmaf(pv, m.z, acc[i][c].z);
          acc[i][c].w = fmaf(pv, m.w, acc[i][c].w);
        }
      }
    }
  }
}

__device__ __forceinline__ float half_warp_max(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float half_warp_sum(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Score transform of the reference: s = (q.k) * scale, then softcap * tanh(s / softcap).
__device__ __forceinline__ float f32_score(const F32Params& p, float dot, float* th) {
  float s = dot * p.scale;
  if (p.softcap > 0.f) {
    const float t = tanhf(s / p.softcap);
    *th = t;
    s = p.softcap * t;
  }
  return s;
}

template <int DQ, int DV>
struct F32Smem {
  // forward: Q, P and NKV buffers of {K, V} (two, so the next tile loads
  // during this one's math, where they fit)
  static constexpr int NKV = (3 * 64 * (DQ + 4) + 2 * 64 * (DV + 4) + 64 * 68) * 4 <= 227 * 1024 ? 2 : 1;
  static constexpr int FWD = (64 * (DQ + 4) + NKV * 64 * (DQ + DV + 8) + 64 * 68) * 4;
  static constexpr int DKDV = (2 * 64 * (DQ + 4) + 2 * 64 * (DV + 4) + 2 * 64 * 68 + 2 * 64) * 4;
  static constexpr int DQK = (2 * 64 * (DQ + 4) + 2 * 64 * (DV + 4) + 64 * 68) * 4;
};

// Forward: one CTA per (64-query tile, query head, batch).
template <int DQ, int DV>
__global__ void __launch_bounds__(F_THREADS) ffa_f32_fwd_kernel(const F32Params p) {
  constexpr int NKV = F32Smem<DQ, DV>::NKV;
  extern __shared__ float4 f32_smem4[];
  float* sQ = reinterpret_cast<float*>(f32_smem4);
  float* sP = sQ + 64 * (DQ + 4);
  float* sKV = sP + 64 * 68;  // buffer u: K at u * KV_STRIDE, V after it
  constexpr int KV_STRIDE = 64 * (DQ + DV + 8);
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
  const int i0 = qt * F_BM, i1 = min(i0 + F_BM, p.Sq) - 1;
  const float* qb = p.q + b * p.q_s[0] + h * p.q_s[1];
  const float* kb = p.k + b * p.k_s[0] + hk * p.k_s[1];
  const float* vb = p.v + b * p.v_s[0] + hk * p.v_s[1];
  f32_load_tile_async<DQ>(sQ, qb, p.q_s[2], i0, p.Sq);

  float m[4], l[4];
  float4 acc[4][DV / 64];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < DV / 64; ++c) acc[i][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int klo, khi;
  f32_key_range(p, i0, i1, klo, khi);
  const int kt0 = max(klo, 0) / F_BN;
  if (kt0 * F_BN < khi) {
    f32_load_tile_async<DQ>(sKV, kb, p.k_s[2], kt0 * F_BN, p.Skv);
    f32_load_tile_async<DV>(sKV + 64 * (DQ + 4), vb, p.v_s[2], kt0 * F_BN, p.Skv);
  }
  cp_async_commit();  // Q and the first K / V tile
  for (int kt = kt0; kt * F_BN < khi; ++kt) {
    const int j0 = kt * F_BN;
    float* sK = sKV + ((kt - kt0) % NKV) * KV_STRIDE;
    float* sV = sK + 64 * (DQ + 4);
    __syncthreads();  // the previous tile's reads (of sP and of the buffer refilled next) are done
    if (NKV == 2 && (kt + 1) * F_BN < khi) {
      float* nK = sKV + ((kt + 1 - kt0) % 2) * KV_STRIDE;
      f32_load_tile_async<DQ>(nK, kb, p.k_s[2], j0 + F_BN, p.Skv);
      f32_load_tile_async<DV>(nK + 64 * (DQ + 4), vb, p.v_s[2], j0 + F_BN, p.Skv);
      cp_async_commit();
      cp_async_wait<1>();  // all but the tile just requested
    } else {
      if (NKV == 1 && kt > kt0) {
        f32_load_tile_async<DQ>(sK, kb, p.k_s[2], j0, p.Skv);
        f32_load_tile_async<DV>(sV, vb, p.v_s[2], j0, p.Skv);
        cp_async_commit();
      }
      cp_async_wait<0>();
    }
    __syncthreads();
    float s[4][4];
    f32_scores<DQ>(sQ, sK, ty, tx, s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = i0 + 4 * ty + i;
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float th;
        const float x = f32_score(p, s[i][j], &th);
        s[i][j] = f32_visible(p, qi, j0 + tx + 16 * j) ? x : -INFINITY;
        rmax = fmaxf(rmax, s[i][j]);
      }
      rmax = half_warp_max(rmax);
      const float mn = fmaxf(m[i], rmax);
      const float base = mn == -INFINITY ? 0.f : mn;
      const float alpha = expf(m[i] - base);  // 0 when m was -inf
      m[i] = mn;
      l[i] *= alpha;
#pragma unroll
      for (int c = 0; c < DV / 64; ++c) {
        acc[i][c].x *= alpha;
        acc[i][c].y *= alpha;
        acc[i][c].z *= alpha;
        acc[i][c].w *= alpha;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pr = expf(s[i][j] - base);
        l[i] += pr;
        sP[(4 * ty + i) * 68 + tx + 16 * j] = pr;
      }
    }
    __syncthreads();
    f32_accumulate<DV>(sP, sV, ty, tx, acc);
  }
  cp_async_wait<0>();  // no copy may still target shared memory when the CTA exits
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = i0 + 4 * ty + i;
    const float lt = half_warp_sum(l[i]);
    if (qi >= p.Sq) continue;
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    float* orow = p.out + b * p.out_s[0] + h * p.out_s[1] + (int64_t)qi * p.out_s[2];
#pragma unroll
    for (int c = 0; c < DV / 64; ++c)
      *reinterpret_cast<float4*>(orow + 4 * tx + 64 * c) =
          make_float4(acc[i][c].x * inv, acc[i][c].y * inv, acc[i][c].z * inv, acc[i][c].w * inv);
    if (p.lse && tx == 0)
      p.lse[((int64_t)b * p.Hq + h) * p.Sq + qi] = lt > 0.f ? m[i] + logf(lt) : -INFINITY;
  }
}

// Delta = rowsum(dO * O): one warp per row.
template <int DV>
__global__ void __launch_bounds__(256) ffa_f32_delta_kernel(const F32Params p) {
  const int64_t row = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= (int64_t)p.B * p.Hq * p.Sq) return;
  const int i = (int)(row % p.Sq);
  const int h = (int)((row / p.Sq) % p.Hq);
  const int b = (int)(row / ((int64_t)p.Sq * p.Hq));
  const float* o = p.o + b * p.o_s[0] + h * p.o_s[1] + (int64_t)i * p.o_s[2];
  const float* d = p.dout + b * p.do_s[0] + h * p.do_s[1] + (int64_t)i * p.do_s[2];
  float acc = 0.f;
  for (int c = lane; c < DV; c += 32) acc = fmaf(o[c], d[c], acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) p.delta[row] = acc;
}

// dK / dV: one CTA per (64-key tile, kv head, batch); it walks the query
// heads of the GQA group and their visible 64-query tiles in order.
template <int DQ, int DV>
__global__ void __launch_bounds__(F_THREADS) ffa_f32_dkdv_kernel(const F32Params p) {
  extern __shared__ float4 f32_smem4[];
  float* sK = reinterpret_cast<float*>(f32_smem4);
  float* sV = sK + 64 * (DQ + 4);
  float* sQ = sV + 64 * (DV + 4);
  float* sDO = sQ + 64 * (DQ + 4);
  float* sPT = sDO + 64 * (DV + 4);
  float* sDST = sPT + 64 * 68;
  float* sLse = sDST + 64 * 68;
  float* sDelta = sLse + 64;
  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int group = p.Hq / p.Hkv;
  const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
  const int j0 = kt * F_BN, j1 = min(j0 + F_BN, p.Skv) - 1;
  f32_load_tile<DQ>(sK, p.k + b * p.k_s[0] + hk * p.k_s[1], p.k_s[2], j0, p.Skv);
  f32_load_tile<DV>(sV, p.v + b * p.v_s[0] + hk * p.v_s[1], p.v_s[2], j0, p.Skv);
  float4 adk[4][DQ / 64], adv[4][DV / 64];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int c = 0; c < DQ / 64; ++c) adk[i][c] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int c = 0; c < DV / 64; ++c) adv[i][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int qlo, qhi;
  f32_query_range(p, j0, j1, qlo, qhi);
  for (int g = 0; g < group; ++g) {
    const int h = hk * group + g;
    const float* qb = p.q + b * p.q_s[0] + h * p.q_s[1];
    const float* db = p.dout + b * p.do_s[0] + h * p.do_s[1];
    const int64_t rb = ((int64_t)b * p.Hq + h) * p.Sq;
    for (int qt = max(qlo, 0) / F_BM; qt * F_BM < qhi; ++qt) {
      const int i0 = qt * F_BM;
      __syncthreads();
      f32_load_tile<DQ>(sQ, qb, p.q_s[2], i0, p.Sq);
      f32_load_tile<DV>(sDO, db, p.do_s[2], i0, p.Sq);
      if (threadIdx.x < 64) {
        const int qi = i0 + threadIdx.x;
        sLse[threadIdx.x] = qi < p.Sq ? p.lse[rb + qi] : 0.f;
        sDelta[threadIdx.x] = qi < p.Sq ? p.delta[rb + qi] : 0.f;
      }
      __syncthreads();
      float s[4][4], dp[4][4];
      f32_scores<DQ>(sK, sQ, ty, tx, s);   // S^T: rows = keys, columns = queries
      f32_scores<DV>(sV, sDO, ty, tx, dp);  // dP^T
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kj = j0 + 4 * ty + i;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int ql = tx + 16 * jj, qi = i0 + ql;
          float th = 0.f;
          const float x = f32_score(p, s[i][jj], &th);
          const bool vis = f32_visible(p, qi, kj);
          const float pr = vis ? expf(x - sLse[ql]) : 0.f;
          float ds = pr * (dp[i][jj] - sDelta[ql]);
          if (p.softcap > 0.f) ds *= 1.f - th * th;
          sPT[(4 * ty + i) * 68 + ql] = pr;
          sDST[(4 * ty + i) * 68 + ql] = ds;
        }
      }
      __syncthreads();
      f32_accumulate<DV>(sPT, sDO, ty, tx, adv);
      f32_accumulate<DQ>(sDST, sQ, ty, tx, adk);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kj = j0 + 4 * ty + i;
    if (kj >= p.Skv) continue;
    float* krow = p.dk + b * p.dk_s[0] + hk * p.dk_s[1] + (int64_t)kj * p.dk_s[2];
    float* vrow = p.dv + b * p.dv_s[0] + hk * p.dv_s[1] + (int64_t)kj * p.dv_s[2];
#pragma unroll
    for (int c = 0; c < DQ / 64; ++c)
      *reinterpret_cast<float4*>(krow + 4 * tx + 64 * c) = make_float4(
          adk[i][c].x * p.scale, adk[i][c].y * p.scale, adk[i][c].z * p.scale, adk[i][c].w * p.scale);
#pragma unroll
    for (int c = 0; c < DV / 64; ++c) *reinterpret_cast<float4*>(vrow + 4 * tx + 64 * c) = adv[i][c];
  }
}

// dQ: one CTA per (64-query tile, query head, batch); it walks the visible key tiles in order.
template <int DQ, int DV>
__global__ void __launch_bounds__(F_THREADS) ffa_f32_dq_kernel(const F32Params p) {
  extern __shared__ float4 f32_smem4[];
  float* sQ = reinterpret_cast<float*>(f32_smem4);
  float* sDO = sQ + 64 * (DQ + 4);
  float* sK = sDO + 64 * (DV + 4);
  float* sV = sK + 64 * (DQ + 4);
  float* sDS = sV + 64 * (DV + 4);
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
  const int i0 = qt * F_BM, i1 = min(i0 + F_BM, p.Sq) - 1;
  const float* kb = p.k + b * p.k_s[0] + hk * p.k_s[1];
  const float* vb = p.v + b * p.v_s[0] + hk * p.v_s[1];
  f32_load_tile<DQ>(sQ, p.q + b * p.q_s[0] + h * p.q_s[1], p.q_s[2], i0, p.Sq);
  f32_load_tile<DV>(sDO, p.dout + b * p.do_s[0] + h * p.do_s[1], p.do_s[2], i0, p.Sq);
  const int64_t rb = ((int64_t)b * p.Hq + h) * p.Sq;
  float lse[4], dl[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = i0 + 4 * ty + i;
    lse[i] = qi < p.Sq ? p.lse[rb + qi] : 0.f;
    dl[i] = qi < p.Sq ? p.delta[rb + qi] : 0.f;
  }
  float4 adq[4][DQ / 64];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < DQ / 64; ++c) adq[i][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  int klo, khi;
  f32_key_range(p, i0, i1, klo, khi);
  for (int kt = max(klo, 0) / F_BN; kt * F_BN < khi; ++kt) {
    const int j0 = kt * F_BN;
    __syncthreads();
    f32_load_tile<DQ>(sK, kb, p.k_s[2], j0, p.Skv);
    f32_load_tile<DV>(sV, vb, p.v_s[2], j0, p.Skv);
    __syncthreads();
    float s[4][4], dp[4][4];
    f32_scores<DQ>(sQ, sK, ty, tx, s);
    f32_scores<DV>(sDO, sV, ty, tx, dp);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = i0 + 4 * ty + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kl = tx + 16 * j;
        float th = 0.f;
        const float x = f32_score(p, s[i][j], &th);
        const float pr = f32_visible(p, qi, j0 + kl) ? expf(x - lse[i]) : 0.f;
        float ds = pr * (dp[i][j] - dl[i]);
        if (p.softcap > 0.f) ds *= 1.f - th * th;
        sDS[(4 * ty + i) * 68 + kl] = ds;
      }
    }
    __syncthreads();
    f32_accumulate<DQ>(sDS, sK, ty, tx, adq);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = i0 + 4 * ty + i;
    if (qi >= p.Sq) continue;
    float* row = p.dq + b * p.dq_s[0] + h * p.dq_s[1] + (int64_t)qi * p.dq_s[2];
#pragma unroll
    for (int c = 0; c < DQ / 64; ++c)
      *reinterpret_cast<float4*>(row + 4 * tx + 64 * c) = make_float4(
          adq[i][c].x * p.scale, adq[i][c].y * p.scale, adq[i][c].z * p.scale, adq[i][c].w * p.scale);
  }
}

bool f32_strides_ok(const void* ptr, const int64_t* s) {
  return ptr && s && aligned16(ptr) && s[0] % 4 == 0 && s[1] % 4 == 0 && s[2] % 4 == 0;
}

void f32_copy_strides(int64_t* dst, const int64_t* s) {
  dst[0] = s[0];
  dst[1] = s[1];
  dst[2] = s[2];
}

template <typename Kernel>
int f32_launch(Kernel kern, dim3 grid, int smem, const F32Params& p, cudaStream_t stream,
               std::atomic<uint64_t>& attr_done) {
  if (int st = smem_attr_once(kern, smem, attr_done)) return st;
  kern<<<grid, F_THREADS, smem, stream>>>(p);
  return launch_status();
}

template <int DQ, int DV>
int f32_fwd_launch(const F32Params& p, cudaStream_t s) {
  static std::atomic<uint64_t> done{0};
  const dim3 grid((p.Sq + F_BM - 1) / F_BM, p.Hq, p.B);
  return f32_launch(ffa_f32_fwd_kernel<DQ, DV>, grid, F32Smem<DQ, DV>::FWD, p, s, done);
}

template <int DQ, int DV>
int f32_bwd_launch(const F32Params& p, cudaStream_t s) {
  const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
  ffa_f32_delta_kernel<DV><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(p);
  if (int st = launch_status()) return st;
  static std::atomic<uint64_t> done_kv{0}, done_q{0};
  int st = f32_launch(ffa_f32_dkdv_kernel<DQ, DV>, dim3((p.Skv + F_BN - 1) / F_BN, p.Hkv, p.B),
                      F32Smem<DQ, DV>::DKDV, p, s, done_kv);
  if (st) return st;
  return f32_launch(ffa_f32_dq_kernel<DQ, DV>, dim3((p.Sq + F_BM - 1) / F_BM, p.Hq, p.B), F32Smem<DQ, DV>::DQK, p,
                    s, done_q);
}

bool f32_dims_ok(int D, int Dv) { return (D == 64 && Dv == 64) || (D == 128 && Dv == 128) || (D == 192 && Dv == 128); }

void f32_common(F32Params& p, int B, int Hq, int Hkv, int Sq, int Skv, float scale, int causal, int q_offset,
                int window, float softcap, const uint8_t* block_mask, int n_br, int n_bc, int mask_bq,
                int mask_bkv) {
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Sq = Sq;
  p.Skv = Skv;
  p.scale = scale;
  p.causal = causal;
  p.q_offset = q_offset;
  p.window = window > 0 ? window : 0;
  p.softcap = softcap > 0.f ? softcap : 0.f;
  p.bm = block_mask;
  p.n_br = n_br;
  p.n_bc = n_bc;
  p.mbq = mask_bq > 0 ? mask_bq : 1;
  p.mbk = mask_bkv > 0 ? mask_bkv : 1;
}

}  // namespace

// fp32 forward behind ffa_fwd (dtype FFA_DTYPE_F32); same argument checks.
int f32_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv, int Sq,
            int Skv, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
            const int64_t* o_strides, float scale, int causal, int q_offset, int window, float softcap,
            const uint8_t* block_mask, int n_br, int n_bc, int mask_bq, int mask_bkv, void* stream) {
  if (!f32_dims_ok(D, Dv)) return FFA_ERR_UNSUPPORTED;
  if (!f32_strides_ok(q, q_strides) || !f32_strides_ok(k, k_strides) || !f32_strides_ok(v, v_strides) ||
      !f32_strides_ok(o, o_strides))
    return FFA_ERR_INVALID_ARG;
  if ((int64_t)Sq > 65535LL * 64 * 32768 || Hq > 65535 || B > 65535) return FFA_ERR_UNSUPPORTED;
  F32Params p{};
  p.q = static_cast<const float*>(q);
  p.k = static_cast<const float*>(k);
  p.v = static_cast<const float*>(v);
  p.out = static_cast<float*>(o);
  p.lse = lse;
  f32_copy_strides(p.q_s, q_strides);
  f32_copy_strides(p.k_s, k_strides);
  f32_copy_strides(p.v_s, v_strides);
  f32_copy_strides(p.out_s, o_strides);
  f32_common(p, B, Hq, Hkv, Sq, Skv, scale, causal, q_offset, window, softcap, block_mask, n_br, n_bc, mask_bq,
             mask_bkv);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 64) return f32_fwd_launch<64, 64>(p, s);
  if (D == 128) return f32_fwd_launch<128, 128>(p, s);
  return f32_fwd_launch<192, 128>(p, s);
}

// fp32 backward behind ffa_bwd / ffa_bwd_masked (dtype FFA_DTYPE_F32).  The
// workspace holds Delta ([B, Hq, Sq] fp32, within ffa_bwd_workspace_size).
int f32_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
            void* dq, void* dk, void* dv, int B, int Hq, int Hkv, int Sq, int Skv, int D, int Dv,
            const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
            const int64_t* o_strides, const int64_t* do_strides, const int64_t* dq_strides,
            const int64_t* dk_strides, const int64_t* dv_strides, float scale, int causal, int q_offset,
            int window, float softcap, const uint8_t* block_mask, int n_br, int n_bc, int mask_bq, int mask_bkv,
            void* workspace, void* stream) {
  if (!f32_dims_ok(D, Dv)) return FFA_ERR_UNSUPPORTED;
  if (!f32_strides_ok(q, q_strides) || !f32_strides_ok(k, k_strides) || !f32_strides_ok(v, v_strides) ||
      !f32_strides_ok(o, o_strides) || !f32_strides_ok(dout, do_strides) || !f32_strides_ok(dq, dq_strides) ||
      !f32_strides_ok(dk, dk_strides) || !f32_strides_ok(dv, dv_strides) || !lse)
    return FFA_ERR_INVALID_ARG;
  if (Hq > 65535 || Hkv > 65535 || B > 65535) return FFA_ERR_UNSUPPORTED;
  F32Params p{};
  p.q = static_cast<const float*>(q);
  p.k = static_cast<const float*>(k);
  p.v = static_cast<const float*>(v);
  p.o = static_cast<const float*>(o);
  p.dout = static_cast<const float*>(dout);
  p.lse = const_cast<float*>(lse);
  p.dq = static_cast<float*>(dq);
  p.dk = static_cast<float*>(dk);
  p.dv = static_cast<float*>(dv);
  p.delta = static_cast<float*>(workspace);
  f32_copy_strides(p.q_s, q_strides);
  f32_copy_strides(p.k_s, k_strides);
  f32_copy_strides(p.v_s, v_strides);
  f32_copy_strides(p.o_s, o_strides);
  f32_copy_strides(p.do_s, do_strides);
  f32_copy_strides(p.dq_s, dq_strides);
  f32_copy_strides(p.dk_s, dk_strides);
  f32_copy_strides(p.dv_s, dv_strides);
  f32_common(p, B, Hq, Hkv, Sq, Skv, scale, causal, q_offset, window, softcap, block_mask, n_br, n_bc, mask_bq,
             mask_bkv);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 64) return f32_bwd_launch<64, 64>(p, s);
  if (D == 128) return f32_bwd_launch<128, 128>(p, s);
  return f32_bwd_launch<192, 128>(p, s);
}

}  // namespace ffa
