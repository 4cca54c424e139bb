// Backward attention for B200 (sm_100a): deterministic, recompute-based.
//
// Replaces kernels/cpu_reference.py:319 flash_attn_cpu_backward,
// kernels/cpu_fa4.py:445 fa4_backward and kernels/triton_bwd.py behind
// ffa_bwd().  Three launches, no atomics, fixed summation order (so results
// are bit-identical run to run):
//   1. preprocess: Delta = rowsum(dO * O) and NLSE2 = -LSE in base-2 units,
//      both padded to whole 128-row tiles (padding rows get NLSE2 = -inf, so
//      P = 0 there);
//   2. dK/dV: one CTA per (batch, kv head, 128-key tile).  It streams 64-row
//      query sub-tiles of every query head of the GQA group that sees the keys:
//        S^T = K Q^T, dP^T = V dO^T        (tensor cores, fp32 in TMEM)
//        P^T = 2^(S^T*scale*log2e + NLSE2), dS^T = P^T (dP^T - Delta) [* softcap']
//        dV += P^T dO,  dK += dS^T Q      (P^T / dS^T as 16-bit A operands in TMEM)
//   3. dQ: one CTA per (batch, query head, 128-row query tile), streaming
//      key units (128 keys for D <= 128, 64 for D = 192):
//        S = Q K^T, dP = dO V^T, dS as above, dQ += dS K.
// The dK/dV kernel double-buffers the score tiles in TMEM (alternate sub-tiles
// go to alternate buffers); the dQ kernel has one buffer of a wider unit.  A compute warpgroup loads its S / dP columns into
// registers and releases the TMEM buffer at once, then writes the 16-bit P^T /
// dS tiles to shared memory (128-byte swizzled, K-major: the A operands of the
// accumulation MMAs).  So the next S / dP MMAs into a buffer never wait for
// the accumulation MMAs of the sub-tile before, and the tensor core runs
// S(u+1), dV/dK(u) while unit u+1's compute overlaps them.
//   warps 0-15  compute warpgroups 0-3.  dK/dV (and dQ at D = 192):
//               warpgroup w serves alternate units (w % 2) and columns
//               [32 (w / 2), 32 (w / 2) + 32) of a 64-column sub-tile.  dQ at
//               D <= 128: every warpgroup serves every 128-key unit, columns
//               [32 w, 32 w + 32).  One TMEM lane = one row.
//   warp 16     TMA producer
//   warp 17     S / dP MMA issuer, TMEM owner
//   warp 18     accumulation MMA issuer
// dK and dQ are multiplied by the softmax scale in their epilogues.
// TMEM: the kept tile (16-bit A operands), then the score buffers (S or S^T,
// then dP or dP^T), then the fp32 accumulators; offsets in DkdvCfg / DqCfg.
#include "ffa_common.cuh"
#include "ffa_host.h"

#include <cstdlib>
#include <type_traits>

namespace ffa {

constexpr int BWD_BT = 128;       // rows of the tile a CTA keeps (keys in dK/dV, queries in dQ)
constexpr int BWD_BS = 64;        // rows of a streamed sub-tile
constexpr int BWD_NWG = 4;         // compute warpgroups: two per TMEM buffer, 32 columns each
constexpr int BWD_THREADS = BWD_NWG * 128 + 96;  // + TMA warp + two MMA-issuing warps
constexpr int BWD_WARP_LOAD = BWD_NWG * 4;
constexpr int BWD_WARP_MMA = BWD_NWG * 4 + 1;    // S / dP MMAs; TMEM owner
constexpr int BWD_WARP_ACC = BWD_NWG * 4 + 2;    // accumulation MMAs

struct BwdParams {
  // dK/dV kernel outputs
  void* dk;
  void* dv;
  int64_t dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  // dQ kernel output
  void* dq;
  int64_t dq_sb, dq_sh, dq_ss;
  const float* nlse2;  // [B*Hq, Sq_pad] minus the base-2 LSE, -inf on padding rows
  const float* delta;  // [B*Hq, Sq_pad]
  int Sq_pad;
  int B, Hq, Hkv, Sq, Skv, q_offset;
  float scale;         // softmax scale (applied to dK / dQ in the epilogue)
  float scale_log2;
  float sc_pre, sc_post;
  float sc_small;      // |raw score| below which softcap_small2 holds (0.5 / sc_pre)
  float sc_poly[3];    // softcap_small2 coefficients for k = sc_pre
  int use_softcap;
  int causal, window;
  // optional tile mask [n_br, n_bc] of (mask_bq x mask_bkv) blocks, the one
  // the forward was given: masked pairs get P = 0 (nullptr: none)
  const uint8_t* block_mask;
  int n_br, n_bc, mask_bq, mask_bkv;
  // CTA order: (b, kv head) pairs per group in dK/dV, (b, q head) pairs per
  // group in dQ (whole GQA groups); see bwd_head_groups
  int grp_kv, grp_q;
  ErrCtx ec;
};

enum : uint32_t {
  SITE_BWD_LOAD = 0x201,
  SITE_BWD_SP = 0x202,
  SITE_BWD_DS = 0x203,
  SITE_BWD_EMPTY = 0x204,
  SITE_BWD_DONE = 0x205,
  SITE_BWD_DRAIN = 0x206,
};

// 64-row query sub-tiles [i_lo, i_hi) that interact with 128-key tile j.
__device__ __forceinline__ void q_range_for_key_tile(const BwdParams& p, int j, int& i_lo, int& i_hi) {
  const int n_q = (p.Sq + BWD_BS - 1) / BWD_BS;
  const int k_lo = j * BWD_BT, k_hi = min(k_lo + BWD_BT, p.Skv) - 1;
  i_lo = 0;
  i_hi = n_q;
  if (p.causal) {  // need some q_abs >= k_lo  ->  q >= k_lo - q_offset
    const int qmin = k_lo - p.q_offset;
    i_lo = qmin > 0 ? min(qmin / BWD_BS, n_q) : 0;
  }
  if (p.window > 0) {  // need some q_abs <= k_hi + window - 1
    const int qmax = k_hi + p.window - 1 - p.q_offset;
    i_hi = qmax < 0 ? 0 : min(n_q, qmax / BWD_BS + 1);
  }
  if (i_lo > i_hi) i_lo = i_hi;
}

// 64-key sub-tiles [j_lo, j_hi) that interact with 128-row query tile i.
__device__ __forceinline__ void k_range_for_q_tile(const BwdParams& p, int i, int& j_lo, int& j_hi) {
  const int n_kv = (p.Skv + BWD_BS - 1) / BWD_BS;
  const int a_lo = i * BWD_BT + p.q_offset;
  const int a_hi = min(i * BWD_BT + BWD_BT, p.Sq) - 1 + p.q_offset;
  j_hi = n_kv;
  if (p.causal) j_hi = min(n_kv, a_hi >= 0 ? a_hi / BWD_BS + 1 : 0);
  j_lo = 0;
  if (p.window > 0) {
    const int lo_col = a_lo - p.window + 1;
    if (lo_col > 0) j_lo = min(lo_col / BWD_BS, j_hi);
  }
}

// Bits of the 32 columns [0, 32) that fall inside [lo, hi] (columns are
// relative to the unit's first column).
__device__ __forceinline__ uint32_t range_bits32(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 31);
  return hi >= lo ? ((2u << (hi - lo)) - 1u) << lo : 0u;
}

// Block-mask keep bits of 32 consecutive positions [x0, x0 + 32) along one
// mask axis (blocks of `bs`, `nb` of them), the other axis fixed: `cell(i)`
// is the mask byte of block i.  Positions past the mask's end are kept (the
// range test already drops them).
template <typename Cell>
__device__ __forceinline__ uint32_t block_mask_bits32(int x0, int bs, int nb, Cell cell) {
  uint32_t bits = ~0u;
#pragma unroll 1
  for (int i = max(x0, 0) / bs; i * bs < x0 + 32 && i < nb; ++i)
    if (!cell(i)) bits &= ~range_bits32(i * bs - x0, (i + 1) * bs - 1 - x0);
  return bits;
}

// P and dS for 16 columns of one TMEM row.  s: raw Q.K scores, dp: dO.V
// values.  Minus the base-2 LSE and Delta of each column come from smem
// (COL_STATS, dK/dV kernel: cnl2 / cdl, 16-byte aligned) or are the row's
// (rnl2 / rdl, dQ kernel).  With MASKED, columns c with (uint)(c - lo) >= cnt
// are dropped, and with BITS also those whose bit c of `bits` is clear (the
// block mask).  MODE 0: no softcap; 1: softcap with tanh by softcap_small2 (FMA
// pipe); 2: softcap with tanh through ex2 / rcp.  Columns are processed in
// pairs with packed fp32x2 instructions (per lane the same IEEE operations as
// the scalar forms: dp - dl is computed as dp + dl * -1, and
// (dp - dl)(1 - th^2) as (dl - dp)(th^2 - 1), both exact rewrites).
template <typename T, bool WRITE_P, bool COL_STATS, int MODE, bool MASKED, bool BITS>
__device__ __forceinline__ void bwd_chunk16(const BwdParams& p, const uint32_t* s, const uint32_t* dp,
                                            const float* cnl2, const float* cdl, float rnl2, float rdl, int lo,
                                            uint32_t cnt, uint32_t bits, uint32_t* pk_p, uint32_t* pk_ds) {
#pragma unroll
  for (int c4 = 0; c4 < 16; c4 += 4) {
    float2 nl2[2], dl[2];
    if (COL_STATS) {
      const float4 a = *reinterpret_cast<const float4*>(cnl2 + c4);
      const float4 z = *reinterpret_cast<const float4*>(cdl + c4);
      nl2[0] = make_float2(a.x, a.y);
      nl2[1] = make_float2(a.z, a.w);
      dl[0] = make_float2(z.x, z.y);
      dl[1] = make_float2(z.z, z.w);
    } else {
      nl2[0] = nl2[1] = f2(rnl2);
      dl[0] = dl[1] = f2(rdl);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = c4 + 2 * h;
      const float2 raw = make_float2(__uint_as_float(s[c]), __uint_as_float(s[c + 1]));
      const float2 dpv = make_float2(__uint_as_float(dp[c]), __uint_as_float(dp[c + 1]));
      float2 x, g;
      if (MODE == 0) {
        x = ffma2(raw, f2(p.scale_log2), nl2[h]);
        g = ffma2(dl[h], f2(-1.f), dpv);
      } else if (MODE == 1) {
        const float2 y = softcap_small2(raw, p.sc_poly[0], p.sc_poly[1], p.sc_poly[2]);
        x = ffma2(y, f2(p.scale_log2), nl2[h]);
        const float2 th = fmul2(y, f2(p.sc_pre));
        g = fmul2(ffma2(dpv, f2(-1.f), dl[h]), ffma2(th, th, f2(-1.f)));
      } else {
        const float t0 = tanh_acc(raw.x * p.sc_pre), t1 = tanh_acc(raw.y * p.sc_pre);
        x = make_float2(fmaf(t0, p.sc_post, nl2[h].x), fmaf(t1, p.sc_post, nl2[h].y));
        g = make_float2((dpv.x - dl[h].x) * fmaf(-t0, t0, 1.f), (dpv.y - dl[h].y) * fmaf(-t1, t1, 1.f));
      }
      float2 pr = make_float2(ex2(x.x), ex2(x.y));
      if (MASKED) {
        pr.x = ((uint32_t)(c - lo) < cnt) ? pr.x : 0.f;
        pr.y = ((uint32_t)(c + 1 - lo) < cnt) ? pr.y : 0.f;
        if (BITS) {
          pr.x = ((bits >> c) & 1u) ? pr.x : 0.f;
          pr.y = ((bits >> (c + 1)) & 1u) ? pr.y : 0.f;
        }
      }
      const float2 dv = fmul2(pr, g);
      if (WRITE_P) pk_p[c / 2] = pack2<T>(pr.x, pr.y);
      pk_ds[c / 2] = pack2<T>(dv.x, dv.y);
    }
  }
}

template <typename T, bool WRITE_P, bool COL_STATS, bool MASKED, bool BITS>
__device__ __forceinline__ void bwd_chunk16_mode(const BwdParams& p, const uint32_t* s, const uint32_t* dp,
                                                 const float* cnl2, const float* cdl, float rnl2, float rdl,
                                                 int lo, uint32_t cnt, uint32_t bits, uint32_t* pk_p,
                                                 uint32_t* pk_ds) {
  if (!p.use_softcap) {
    bwd_chunk16<T, WRITE_P, COL_STATS, 0, MASKED, BITS>(p, s, dp, cnl2, cdl, rnl2, rdl, lo, cnt, bits, pk_p, pk_ds);
    return;
  }
  // The cap is usually far above the scores, so tanh's argument is small:
  // then the polynomial on the FMA pipe (error 2e-7) spares the MUFU.
  float mx = 0.f;
#pragma unroll
  for (int c = 0; c < 16; c += 2) mx = fmax3(mx, fabsf(__uint_as_float(s[c])), fabsf(__uint_as_float(s[c + 1])));
  if (__all_sync(0xffffffffu, mx <= p.sc_small))
    bwd_chunk16<T, WRITE_P, COL_STATS, 1, MASKED, BITS>(p, s, dp, cnl2, cdl, rnl2, rdl, lo, cnt, bits, pk_p, pk_ds);
  else
    bwd_chunk16<T, WRITE_P, COL_STATS, 2, MASKED, BITS>(p, s, dp, cnl2, cdl, rnl2, rdl, lo, cnt, bits, pk_p, pk_ds);
}

// Stores 16-byte chunk `chunk` of row `row` of a 128-byte-swizzled K-major
// tile (the layout TMA's SWIZZLE_128B writes and the MMA descriptors read):
// chunk j of row r sits at r * 128 + 16 * (j ^ (r % 8)).  Rows 0-7 of the
// eight threads that store one chunk fall into distinct bank groups.
__device__ __forceinline__ void st_sw128(uint8_t* tile, int row, int chunk, uint32_t a, uint32_t b, uint32_t c,
                                         uint32_t d) {
  *reinterpret_cast<uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4)) = make_uint4(a, b, c, d);
}

// P / dS for this thread's 32 columns of a unit (one TMEM row = tile row
// `row`).  tS / tDP address the first of the 32 columns; the TMEM buffer is
// released (arrive on `tmem_free`) as soon as the values are in registers.
// (Releasing S before dP is read was measured slower: the two loads then
// no longer overlap.)
// Column statistics come from smem (COL_STATS: cnl2 / cdl for the first
// column) or are the row's (rnl2, rdl).  The row keeps columns
// [keep_lo, keep_hi] of the 32 (and, with BM, only those whose bit is set in
// `bm_bits`, from the block mask); `masked` (warp-uniform) is false when no
// row of the warp drops any column.  Before storing, waits (if pt_parity >= 0)
// for `pt_free` to show that the smem tiles' previous contents were consumed;
// then P^T (WRITE_P) goes to sP and dS to sDS, as 16-byte chunks
// 4*half .. 4*half+3 of the row.  Returns false if that wait gave up.
template <typename T, bool WRITE_P, bool COL_STATS, bool BM>
__device__ __forceinline__ bool bwd_unit(const BwdParams& p, uint32_t tS, uint32_t tDP, uint64_t* tmem_free,
                                         const float* cnl2, const float* cdl, float rnl2, float rdl, int keep_lo,
                                         int keep_hi, uint32_t bm_bits, bool masked, uint64_t* pt_free, int pt_parity,
                                         volatile int* abort_flag, uint8_t* sP, uint8_t* sDS, int row, int half) {
  uint32_t s[32], d[32];
  tmem_ld32(tS, s);
  tmem_ld32(tDP, d);
  tmem_ld_wait32(s);
  tmem_ld_wait32(d);
  tc_fence_before();
  __syncwarp();
  if (lane_id() == 0) mbar_arrive(tmem_free);
  uint32_t pp[16], pd[16];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float* n2 = COL_STATS ? cnl2 + 16 * k : nullptr;
    const float* d2 = COL_STATS ? cdl + 16 * k : nullptr;
    if (masked) {
      const int lo = max(keep_lo - 16 * k, 0);
      const int z = min(keep_hi - 16 * k, 15);
      const uint32_t cnt = z >= lo ? (uint32_t)(z - lo + 1) : 0u;
      bwd_chunk16_mode<T, WRITE_P, COL_STATS, true, BM>(p, s + 16 * k, d + 16 * k, n2, d2, rnl2, rdl, lo, cnt,
                                                        bm_bits >> (16 * k), pp + 8 * k, pd + 8 * k);
    } else {
      bwd_chunk16_mode<T, WRITE_P, COL_STATS, false, false>(p, s + 16 * k, d + 16 * k, n2, d2, rnl2, rdl, 0, 16u,
                                                            0u, pp + 8 * k, pd + 8 * k);
    }
  }
  if (pt_parity >= 0 &&
      !__all_sync(0xffffffffu, mbar_wait(pt_free, (uint32_t)pt_parity, p.ec, abort_flag, SITE_BWD_EMPTY)))
    return false;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (WRITE_P) st_sw128(sP, row, 4 * half + q, pp[4 * q], pp[4 * q + 1], pp[4 * q + 2], pp[4 * q + 3]);
    st_sw128(sDS, row, 4 * half + q, pd[4 * q], pd[4 * q + 1], pd[4 * q + 2], pd[4 * q + 3]);
  }
  fence_async_smem();  // the generic-proxy stores -> visible to the tensor core
  __syncwarp();
  return true;
}

// Stores 16 fp32 accumulator columns of one row (times mul) as T.
template <typename T>
__device__ __forceinline__ void store_row16(T* dst, const uint32_t* v, float mul, bool store) {
  uint32_t pk[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) pk[e] = pack2<T>(__uint_as_float(v[2 * e]) * mul, __uint_as_float(v[2 * e + 1]) * mul);
  if (store) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    d[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    d[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
}

__device__ __forceinline__ float2 load2f(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ float2 load2f(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Stores 32 fp32 accumulator columns of one row (times mul) as T.
template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const uint32_t* v, float mul, bool store) {
  uint32_t pk[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) pk[e] = pack2<T>(__uint_as_float(v[2 * e]) * mul, __uint_as_float(v[2 * e + 1]) * mul);
  if (store) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
  }
}

// K-major smem descriptor offset of the ks-th 16-column K step in a tile of
// `rows` rows stored as 64-column (128-byte) swizzled chunks.
__device__ __forceinline__ uint64_t kstep(int ks, int rows) {
  return (uint64_t)(((ks / 4) * rows * 128 + (ks % 4) * 32) >> 4);
}

// ---------------------------------------------------------------------------
// 1. preprocess: Delta and minus the base-2 LSE, padded to whole tiles
// ---------------------------------------------------------------------------
template <typename T>
__global__ void ffa_bwd_pre_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                   const float* __restrict__ lse, float* __restrict__ nlse2,
                                   float* __restrict__ delta, int Hq, int Sq, int Sq_pad, int D, int64_t o_sb,
                                   int64_t o_sh, int64_t o_ss, int64_t d_sb, int64_t d_sh, int64_t d_ss,
                                   int n_rows) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp_global >= n_rows) return;
  const int bh = warp_global / Sq_pad;
  const int q = warp_global % Sq_pad;
  const int b = bh / Hq, h = bh % Hq;
  float acc = 0.f;
  if (q < Sq) {
    const T* orow = o + b * o_sb + h * o_sh + (int64_t)q * o_ss;
    const T* drow = dout + b * d_sb + h * d_sh + (int64_t)q * d_ss;
    for (int d = lane * 2; d < D; d += 64) {
      const float2 ov = load2f(orow + d);
      const float2 dv = load2f(drow + d);
      acc += ov.x * dv.x + ov.y * dv.y;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const int64_t idx = (int64_t)bh * Sq_pad + q;
    delta[idx] = acc;
    const float l = (q < Sq) ? lse[(int64_t)bh * Sq + q] : INFINITY;
    // A row that saw no key has LSE = -inf: P is 0 for it, so any finite
    // offset works; -inf keeps 2^(x + NLSE2) at exactly 0.
    nlse2[idx] = (q < Sq && l != -INFINITY) ? l * -1.4426950408889634f : -INFINITY;
  }
}


// The same with 16-byte loads: TPR = D / 8 lanes per row, 32 / TPR rows per
// warp (rows and bases 16-byte aligned).  One load each of O and dO per lane
// keeps enough bytes in flight to stream at HBM rate.
template <typename T, int TPR>
__global__ void __launch_bounds__(256) ffa_bwd_pre_vec_kernel(
    const T* __restrict__ o, const T* __restrict__ dout, const float* __restrict__ lse, float* __restrict__ nlse2,
    float* __restrict__ delta, int Hq, int Sq, int Sq_pad, int64_t o_sb, int64_t o_sh, int64_t o_ss, int64_t d_sb,
    int64_t d_sh, int64_t d_ss, int n_rows) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int row_g = t / TPR;
  const int sub = t % TPR;
  const bool live = row_g < n_rows;
  const int bh = live ? row_g / Sq_pad : 0;
  const int q = live ? row_g % Sq_pad : Sq;
  const int b = bh / Hq, h = bh % Hq;
  float acc = 0.f;
  if (q < Sq) {
    const uint4 ov = __ldg(reinterpret_cast<const uint4*>(o + b * o_sb + h * o_sh + (int64_t)q * o_ss) + sub);
    const uint4 dv = __ldg(reinterpret_cast<const uint4*>(dout + b * d_sb + h * d_sh + (int64_t)q * d_ss) + sub);
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = load2f(reinterpret_cast<const T*>(&ow[e]));
      const float2 c = load2f(reinterpret_cast<const T*>(&dw[e]));
      acc = fmaf(a.x, c.x, fmaf(a.y, c.y, acc));
    }
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (live && sub == 0) {
    const int64_t idx = (int64_t)bh * Sq_pad + q;
    delta[idx] = acc;
    const float l = (q < Sq) ? lse[(int64_t)bh * Sq + q] : INFINITY;
    nlse2[idx] = (q < Sq && l != -INFINITY) ? l * -1.4426950408889634f : -INFINITY;
  }
}

// ---------------------------------------------------------------------------
// shared pieces of the dK/dV and dQ kernels
// ---------------------------------------------------------------------------
struct BwdBars {
  uint64_t fixed_full;    // TMA of the tile the CTA keeps (K/V or Q/dO) landed
  uint64_t fixed_tmem;    // ... and was copied into TMEM (one arrival per warp of warpgroups 0-1)
  uint64_t st_full[8];
  uint64_t st_empty[8];
  uint64_t sp_full[2];    // S and dP of unit u computed (index u % 2)
  uint64_t tmem_free[2];  // S and dP of unit u read out of TMEM (one arrival per consuming warp)
  uint64_t ds_ready[2];   // P / dS of unit u stored to smem (one arrival per warp of its pair)
  uint64_t pt_free[2];    // accumulation MMAs of unit u done with its P / dS smem tiles
  uint64_t acc_done;      // all accumulation MMAs done
  uint64_t s_done;        // all S / dP MMAs done
  uint32_t tmem_base;
  int abort;
};

// TMEM columns (per kernel, in its Cfg): the kept tile as 16-bit A operands
// of the S / dP MMAs, then the score buffers (128 columns each: S or S^T, then
// dP or dP^T), then the fp32 accumulators.

// `consumers`: warps that read each unit's scores and store its P / dS.
__device__ __forceinline__ void bwd_init_bars(BwdBars* bars, int ns, int consumers) {
  mbar_init(&bars->fixed_full, 1);
  mbar_init(&bars->fixed_tmem, 2 * 4);
  for (int s = 0; s < ns; ++s) {
    mbar_init(&bars->st_full[s], 1);
    mbar_init(&bars->st_empty[s], 1);
  }
  for (int t = 0; t < 2; ++t) {
    mbar_init(&bars->sp_full[t], 1);
    mbar_init(&bars->tmem_free[t], consumers);
    mbar_init(&bars->ds_ready[t], consumers);
    mbar_init(&bars->pt_free[t], 1);
  }
  mbar_init(&bars->acc_done, 1);
  mbar_init(&bars->s_done, 1);
  bars->abort = 0;
  fence_mbar_init();
}

// Copies row `row` of a 128-row, D-column 16-bit tile from swizzled smem
// (64-column chunks of 128 rows, as TMA wrote it) into TMEM columns
// [tcol, tcol + D/2) of this thread's lane: the layout of a K-major A operand.
template <int D>
__device__ __forceinline__ void tile_row_to_tmem(const uint8_t* tile, int row, uint32_t tcol) {
#pragma unroll
  for (int c = 0; c < D / 64; ++c) {
    uint32_t w[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(tile + c * BWD_BT * 128 + row * 128 + ((j ^ (row & 7)) << 4));
      w[4 * j] = v.x;
      w[4 * j + 1] = v.y;
      w[4 * j + 2] = v.z;
      w[4 * j + 3] = v.w;
    }
    tmem_st32(tcol + 32 * c, w);
  }
}

// The MMAs are issued by two threads in different warps, so that one never
// waits behind the other's issue (an issuing thread stalls while the tensor
// core's queue is full):
//  * bwd_issue_scores: S / dP of unit u (into TMEM score buffer u % NBUF) once
//    u's streamed operands have landed and unit u-NBUF is done with the
//    buffer (`buf_free`: its scores read out, or, when P / dS are kept in the
//    buffer, its accumulation MMAs done);
//  * bwd_issue_acc: the accumulation MMAs of unit u once its P / dS are in
//    smem, in unit order, so the sums are deterministic.
// Streamed operands: one ring of ns_stages slots (st_full / st_empty[0, ns)),
// released when the unit's accumulation is done; or, with nsv > 0, a second
// ring (st_full / st_empty[4, 4 + nsv)) that the S / dP MMAs alone read and
// that is released as soon as they are done (the dQ kernel's V).  A unit's
// accumulation starts after its S / dP MMAs completed (its P / dS derive from
// them), so the first ring's slot is free once the accumulation is done.
template <int NBUF, typename IssueS, typename IssueDP>
__device__ __forceinline__ bool bwd_issue_scores(BwdBars* bars, uint64_t* buf_free, int n, int ns_stages, int nsv,
                                                 const ErrCtx& ec, volatile int* abort_flag, IssueS issue_s,
                                                 IssueDP issue_dp) {
  for (int u = 0; u < n; ++u) {
    if (!mbar_wait_mma(&bars->st_full[u % ns_stages], (u / ns_stages) & 1, ec, abort_flag, SITE_BWD_LOAD))
      return false;
    if (nsv && !mbar_wait_mma(&bars->st_full[4 + u % nsv], (u / nsv) & 1, ec, abort_flag, SITE_BWD_LOAD))
      return false;
    if (u >= NBUF && !mbar_wait_mma(&buf_free[(u - NBUF) & 1], ((u - NBUF) >> 1) & 1, ec, abort_flag, SITE_BWD_DS))
      return false;
    tc_fence_after();
    issue_s(u);
    issue_dp(u);
    mma_commit(&bars->sp_full[u & 1]);
    if (nsv) mma_commit(&bars->st_empty[4 + u % nsv]);
  }
  return true;
}

template <typename IssueAcc>
__device__ __forceinline__ bool bwd_issue_acc(BwdBars* bars, int n, int ns_stages, const ErrCtx& ec,
                                              volatile int* abort_flag, IssueAcc issue_acc) {
  for (int u = 0; u < n; ++u) {
    if (!mbar_wait_mma(&bars->ds_ready[u & 1], (u >> 1) & 1, ec, abort_flag, SITE_BWD_DS)) return false;
    tc_fence_after();
    issue_acc(u);
    mma_commit(&bars->st_empty[u % ns_stages]);
    mma_commit(&bars->pt_free[u & 1]);
  }
  return true;
}

// ---------------------------------------------------------------------------
// 2. dK / dV
// ---------------------------------------------------------------------------
// D = query/key head dim, DV = value head dim.  TMEM holds the score
// buffers (S^T 64 + dP^T 64 columns each), the accumulators (dV, dK) and,
// where the columns allow, K and V as 16-bit A operands (else the S^T / dP^T
// MMAs read them from smem):
//   D = 64:  K + V (64 columns each) + two score buffers + dV 64 + dK 64; two
//            buffers let unit u+1's S / dP MMAs run while unit u's scores are
//            still being read out;
//   D = 128: K + V + one buffer + dV 128 + dK 128 (a second buffer would push
//            K and V to smem and cost a {Q, dO} stage: measured slower);
//   D = 192 (the MLA training shape): V + one buffer + dV 128 + dK 192.
// P^T / dS^T go through smem.  (Writing them back over their TMEM score
// columns, so the accumulation MMAs read them from TMEM, with two buffers at
// D = 128, measured no faster.)
template <int D, int DV>
struct DkdvCfg {
  static constexpr int NBUF = D == 64 ? 2 : 1;
  // TMEM columns left for K / V (64 each) after the score buffers and dV, dK
  static constexpr int KV_COLS = 512 - 128 * NBUF - (D + DV);
  static constexpr bool V_TMEM = KV_COLS >= 64;   // V kept in TMEM as an A operand
  static constexpr bool K_TMEM = KV_COLS >= 128;  // K kept in TMEM as an A operand
  static constexpr uint32_t TM_K = 0;
  static constexpr uint32_t TM_V = K_TMEM ? 64 : 0;
  static constexpr uint32_t TM_SC = (K_TMEM ? 64 : 0) + (V_TMEM ? 64 : 0);  // buffer b at TM_SC + 128 b
  static constexpr uint32_t TM_AC = TM_SC + 128 * NBUF;  // dV (DV columns) then dK (D columns)
  static_assert(TM_AC + DV + D <= 512, "dK/dV TMEM budget");
  static constexpr int TILE_K = BWD_BT * D * 2;     // K tile (128 rows)
  static constexpr int TILE_V = BWD_BT * DV * 2;    // V tile
  static constexpr int SUB_Q = BWD_BS * D * 2;      // Q sub-tile (64 rows)
  static constexpr int SUB_DO = BWD_BS * DV * 2;    // dO sub-tile
  static constexpr int STAGE = SUB_Q + SUB_DO;
  static constexpr int PT = BWD_BT * BWD_BS * 2;  // one P^T or dS^T tile (128 x 64, 16-bit)
  // With K and V both in TMEM their smem is free once copied: the four P^T /
  // dS^T tiles reuse it, which leaves room for one more {Q, dO} stage.
  // smem P^T / dS^T tiles reuse the K / V smem when both are in TMEM by then
  static constexpr bool PT_ALIAS = K_TMEM && V_TMEM && 4 * PT <= TILE_K + TILE_V;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE_K;
  static constexpr int STAGE_OFF = TILE_K + TILE_V + (PT_ALIAS ? 0 : 4 * PT);  // Q at s*STAGE, dO after
  static constexpr int PT_OFF = PT_ALIAS ? 0 : TILE_K + TILE_V;  // pair b: P^T at b*PT, dS^T at (2+b)*PT
  static constexpr int STAT = 2 * BWD_BS * 4;                    // nlse2[64], delta[64]
  static constexpr int NS_FIT = (227 * 1024 - 256 - 1024 - STAGE_OFF) / (STAGE + STAT);
  static constexpr int NS = NS_FIT > 8 ? 8 : NS_FIT;  // stages of {Q, dO, stats}
  static_assert(NS >= 2, "dK/dV smem budget");
  static constexpr int STAT_OFF = STAGE_OFF + NS * STAGE;  // stage s: stats at s*STAT
  static constexpr int BAR_OFF = STAT_OFF + NS * STAT;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
};

// The dK/dV epilogue at D = DV = 128 stages 16 warp boxes of 4 KB in the stage smem.
static_assert(DkdvCfg<128, 128>::NS * DkdvCfg<128, 128>::STAGE >= 16 * 32 * 128, "dK/dV store staging");

template <typename T, int D, int DV, bool BM>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    ffa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmDK, const __grid_constant__ CUtensorMap tmDV,
                        const BwdParams p) {
  using Cfg = DkdvCfg<D, DV>;
  constexpr int NS = Cfg::NS;
  constexpr int NBUF = Cfg::NBUF;
  constexpr uint32_t TM_ACC = Cfg::TM_AC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + Cfg::K_OFF;
  uint8_t* sV = smem + Cfg::V_OFF;
  uint8_t* sStage = smem + Cfg::STAGE_OFF;
  uint8_t* sPT = smem + Cfg::PT_OFF;
  float* sStat = reinterpret_cast<float*>(smem + Cfg::STAT_OFF);
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + Cfg::BAR_OFF);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // Key-tile-major order: under causal masking the first key tiles see the
  // most queries, so they are dispatched first.
  const int BHk = p.B * p.Hkv;
  const int n_j = (p.Skv + BWD_BT - 1) / BWD_BT;
  // (b, kv head) pairs in groups of p.grp_kv whose Q / dO stay in L2 while
  // the group's key tiles stream them; within a group key tiles go in order
  // (under causal masking the first ones see the most queries).
  const int g0 = (int)(blockIdx.x / ((unsigned)p.grp_kv * n_j)) * p.grp_kv;
  const int gn = min(p.grp_kv, BHk - g0);
  const int rem = (int)blockIdx.x - g0 * n_j;
  const int j = rem / gn;
  const int bhk = g0 + rem % gn;
  const int b = bhk / p.Hkv, hkv = bhk % p.Hkv;
  const int group = p.Hq / p.Hkv;
  int i_lo, i_hi;
  q_range_for_key_tile(p, j, i_lo, i_hi);
  const int n_i = i_hi - i_lo;
  const int n = n_i * group;  // units: (query head of the group, 64-row query sub-tile), head-major
  constexpr uint32_t FMT = DtypeFmt<T>::value;

  if (threadIdx.x == 0) bwd_init_bars(bars, NS, 2 * 4);
  if (warp == BWD_WARP_MMA) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == BWD_WARP_LOAD) {
    if (lane == 0 && n > 0) {
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(&bars->fixed_full, Cfg::TILE_K + Cfg::TILE_V);
      for (int hf = 0; hf < 2; ++hf) {
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(&tmK, &bars->fixed_full, sK + c * BWD_BT * 128 + hf * BWD_BS * 128, c * 64,
                      j * BWD_BT + hf * BWD_BS, hkv, b, pol);
        for (int c = 0; c < DV / 64; ++c)
          tma_load_4d(&tmV, &bars->fixed_full, sV + c * BWD_BT * 128 + hf * BWD_BS * 128, c * 64,
                      j * BWD_BT + hf * BWD_BS, hkv, b, pol);
      }
      int issued = 0;
      for (int u = 0; u < n; ++u) {
        const int s = u % NS, use = u / NS;
        if (use > 0 && !mbar_wait(&bars->st_empty[s], (use - 1) & 1, p.ec, abort_flag, SITE_BWD_EMPTY)) break;
        const int g = u / n_i, i = i_lo + u % n_i;
        const int h = hkv * group + g;
        mbar_arrive_expect_tx(&bars->st_full[s], Cfg::STAGE + 2 * BWD_BS * 4);
        uint8_t* dst = sStage + s * Cfg::STAGE;
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(&tmQ, &bars->st_full[s], dst + c * BWD_BS * 128, c * 64, i * BWD_BS, h, b, pol);
        for (int c = 0; c < DV / 64; ++c)
          tma_load_4d(&tmDO, &bars->st_full[s], dst + Cfg::SUB_Q + c * BWD_BS * 128, c * 64, i * BWD_BS, h, b, pol);
        const int64_t row0 = (int64_t)(b * p.Hq + h) * p.Sq_pad + i * BWD_BS;
        bulk_load(sStat + 2 * BWD_BS * s, p.nlse2 + row0, BWD_BS * 4, &bars->st_full[s]);
        bulk_load(sStat + 2 * BWD_BS * s + BWD_BS, p.delta + row0, BWD_BS * 4, &bars->st_full[s]);
        ++issued;
      }
      if (*abort_flag) {  // let copies in flight land before the CTA exits
        mbar_wait(&bars->fixed_full, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
        for (int u = max(0, issued - NS); u < issued; ++u)
          mbar_wait(&bars->st_full[u % NS], (u / NS) & 1, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      }
    }
    __syncwarp();
  } else if (warp == BWD_WARP_MMA || warp == BWD_WARP_ACC) {
    if (lane == 0 && n > 0) {
      const uint32_t idesc_t = make_idesc_f16(128, BWD_BS, FMT, 0, 0);  // S^T, dP^T (K-major A x K-major B)
      const uint32_t idesc_dv = make_idesc_f16(128, DV, FMT, 0, 1);     // dV (K-major A x MN-major B)
      const uint32_t idesc_dk = make_idesc_f16(128, D, FMT, 0, 1);      // dK
      const uint64_t st_kdesc = make_sdesc_sw128(smem_u32(sStage), 16, 1024);
      const uint64_t st_mdesc = make_sdesc_sw128(smem_u32(sStage), BWD_BS * 128, 1024);
      const uint64_t pt_desc = make_sdesc_sw128(smem_u32(sPT), 16, 1024);
      const uint64_t k_desc = make_sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t v_desc = make_sdesc_sw128(smem_u32(sV), 16, 1024);
      const uint32_t tK = tmem + Cfg::TM_K, tV = tmem + Cfg::TM_V;
      const uint32_t tDV = tmem + TM_ACC, tDK = tmem + TM_ACC + DV;
      auto issue_s = [&](int u) {
        const int s = u % NS;
        const uint32_t tS = tmem + Cfg::TM_SC + 128 * (u % NBUF);
        const uint64_t q_k = st_kdesc + (uint64_t)((s * Cfg::STAGE) >> 4);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          if constexpr (Cfg::K_TMEM)
            mma_ts(tS, tK + 8 * ks, q_k + kstep(ks, BWD_BS), idesc_t, ks > 0);
          else
            mma_ss(tS, k_desc + kstep(ks, BWD_BT), q_k + kstep(ks, BWD_BS), idesc_t, ks > 0);
        }
      };
      auto issue_dp = [&](int u) {
        const int s = u % NS;
        const uint32_t tDP = tmem + Cfg::TM_SC + 128 * (u % NBUF) + 64;
        const uint64_t do_k = st_kdesc + (uint64_t)((s * Cfg::STAGE + Cfg::SUB_Q) >> 4);
#pragma unroll
        for (int ks = 0; ks < DV / 16; ++ks) {
          if constexpr (Cfg::V_TMEM)
            mma_ts(tDP, tV + 8 * ks, do_k + kstep(ks, BWD_BS), idesc_t, ks > 0);
          else
            mma_ss(tDP, v_desc + kstep(ks, BWD_BT), do_k + kstep(ks, BWD_BS), idesc_t, ks > 0);
        }
      };
      auto issue_acc = [&](int v) {
        const int bb = v & 1, s = v % NS;
        const uint64_t q_m = st_mdesc + (uint64_t)((s * Cfg::STAGE) >> 4);
        const uint64_t do_m = st_mdesc + (uint64_t)((s * Cfg::STAGE + Cfg::SUB_Q) >> 4);
        const uint64_t p_k = pt_desc + (uint64_t)((bb * Cfg::PT) >> 4);
        const uint64_t ds_k = pt_desc + (uint64_t)(((2 + bb) * Cfg::PT) >> 4);
#pragma unroll
        for (int ks = 0; ks < BWD_BS / 16; ++ks)
          mma_ss(tDV, p_k + kstep(ks, BWD_BT), do_m + (uint64_t)((ks * 16 * 128) >> 4), idesc_dv,
                 (v > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < BWD_BS / 16; ++ks)
          mma_ss(tDK, ds_k + kstep(ks, BWD_BT), q_m + (uint64_t)((ks * 16 * 128) >> 4), idesc_dk,
                 (v > 0 || ks > 0) ? 1u : 0u);
      };
      if (warp == BWD_WARP_MMA) {
        bool ok = mbar_wait(&bars->fixed_tmem, 0, p.ec, abort_flag, SITE_BWD_LOAD);
        if (ok) ok = bwd_issue_scores<NBUF>(bars, bars->tmem_free, n, NS, 0, p.ec, abort_flag, issue_s, issue_dp);
        mma_commit(&bars->s_done);
        if (!ok) mbar_wait(&bars->s_done, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      } else {
        const bool ok = bwd_issue_acc(bars, n, NS, p.ec, abort_flag, issue_acc);
        mma_commit(&bars->acc_done);
        if (!ok) mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      }
    }
    __syncwarp();
  } else {
    // ------------------------- compute (key rows) -------------------------
    const int wg = warp / 4, pair = wg % 2, half = wg / 2;
    const int r = threadIdx.x % 128;  // key row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
    // units alternate between the pairs, and (NBUF = 2) between the buffers
    const uint32_t tS = tmem + lane_off + Cfg::TM_SC + 128 * (pair % NBUF) + 32 * half, tDP = tS + 64;
    const int key = j * BWD_BT + r;
    bool ok = true;
    if (n > 0 && wg < 2) {  // K (warpgroup 0) / V (warpgroup 1) into TMEM as the A operand
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->fixed_full, 0, p.ec, abort_flag, SITE_BWD_LOAD));
      if (ok) {
        if (wg == 1 && Cfg::V_TMEM)
          tile_row_to_tmem<DV>(sV, r, tmem + lane_off + Cfg::TM_V);
        else if (wg == 0 && Cfg::K_TMEM)
          tile_row_to_tmem<D>(sK, r, tmem + lane_off + Cfg::TM_K);
        tmem_st_wait();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->fixed_tmem);
    }
    // Kept query columns of this key, in absolute query positions minus q_offset:
    // causal keeps q >= key - q_offset, the window keeps q <= key + window - 1 - q_offset.
    const int q_keep_lo = p.causal ? key - p.q_offset : -0x3fffffff;
    const int q_keep_hi = key >= p.Skv ? -0x40000000 : (p.window > 0 ? key + p.window - 1 - p.q_offset : 0x3fffffff);
    for (int u = pair; u < n && ok; u += 2) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->sp_full[pair], (u >> 1) & 1, p.ec, abort_flag, SITE_BWD_SP));
      if (!ok) break;
      tc_fence_after();
      const int s = u % NS;
      const int q0 = (i_lo + u % n_i) * BWD_BS + 32 * half;
      const int keep_lo = q_keep_lo - q0, keep_hi = q_keep_hi - q0;
      uint32_t bm_bits = ~0u;
      if (BM && key < p.Skv) {  // queries are the block mask's rows here
        const uint8_t* mcol = p.block_mask + key / p.mask_bkv;
        bm_bits = block_mask_bits32(q0, p.mask_bq, p.n_br, [&](int br) { return mcol[(size_t)br * p.n_bc] != 0; });
      }
      const bool masked = !__all_sync(0xffffffffu, keep_lo <= 0 && keep_hi >= 31 && (!BM || bm_bits == ~0u));
      const float* nl2 = sStat + 2 * BWD_BS * s + 32 * half;
      // this pair's P^T / dS^T smem tiles are free once unit u-2's accumulation MMAs are done
      ok = bwd_unit<T, true, true, BM>(p, tS, tDP, &bars->tmem_free[pair], nl2, nl2 + BWD_BS, 0.f, 0.f, keep_lo,
                                       keep_hi, bm_bits, masked, &bars->pt_free[pair], u >= 2 ? ((u - 2) >> 1) & 1 : -1,
                                   abort_flag, sPT + pair * Cfg::PT, sPT + (2 + pair) * Cfg::PT, r, half);
      if (lane == 0) mbar_arrive(&bars->ds_ready[pair]);
    }
    // ------------------------------ epilogue ------------------------------
    // warpgroups 0 / 2 store dV, 1 / 3 dK (times the softmax scale), each half of the columns
    const bool have = ok && n > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DONE));
    if (have) tc_fence_after();
    const bool store = key < p.Skv;
    T* row = pair == 0
                 ? reinterpret_cast<T*>(p.dv) + (size_t)b * p.dv_sb + (size_t)hkv * p.dv_sh + (size_t)key * p.dv_ss
                 : reinterpret_cast<T*>(p.dk) + (size_t)b * p.dk_sb + (size_t)hkv * p.dk_sh + (size_t)key * p.dk_ss;
    const uint32_t tacc = tmem + lane_off + TM_ACC + pair * DV;
    const float mul = pair ? p.scale : 1.f;
    const int ncol = pair ? D : DV;
    if (D == 128 && DV == 128 && (have || n == 0)) {
      // Each warp packs its 32 rows x 64 columns into the (now idle) stage
      // smem in the 128-byte-swizzled layout and hands them to one TMA store,
      // so the CTA leaves once the copy has read the smem instead of once
      // every row's global stores have been issued.
      uint8_t* tile = sStage + (size_t)(wg * 4 + warp % 4) * (32 * 128);
      const int lr = r % 32;
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        uint32_t v[32];
        if (have) {
          tmem_ld32(tacc + half * 64 + c, v);
          tmem_ld_wait32(v);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0u;
        }
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = pack2<T>(__uint_as_float(v[2 * e]) * mul, __uint_as_float(v[2 * e + 1]) * mul);
#pragma unroll
        for (int q = 0; q < 4; ++q) st_sw128(tile, lr, c / 8 + q, pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_4d(pair == 0 ? &tmDV : &tmDK, tile, half * 64, j * BWD_BT + (warp % 4) * 32, hkv, b);
        tma_store_commit();
        tma_store_wait_read();
      }
      __syncwarp();
    } else {
#pragma unroll 1
      for (int c = half * (ncol / 2); c < (half + 1) * (ncol / 2); c += 32) {
        uint32_t v[32];
        if (have) {
          tmem_ld32(tacc + c, v);
          tmem_ld_wait32(v);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0u;
        }
        store_row32<T>(row + c, v, mul, store);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == BWD_WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// 3. dQ
// ---------------------------------------------------------------------------
// (D, DV) = (192, 128): Q and dO (160 packed columns) and dQ (192) leave TMEM
// room for one score buffer.
// A unit is UK keys.  D <= 128: UK = 128; the TMEM (Q 16-bit + dO 16-bit,
// one score buffer S 128 + dP 128 columns, dQ) holds exactly one score buffer,
// and all four compute warpgroups share each unit, 32 columns each.  The two
// dS tiles (128 x 128) reuse the smem of Q / dO once those are in TMEM.
// D = 192: UK = 64 with one score buffer; the warpgroup pairs alternate units.
template <int D, int DV>
struct DqCfg {
  static constexpr int UK = D <= 128 ? 128 : 64;
  static constexpr bool WIDE = UK == 128;
  static constexpr int NBUF = 1;
  static constexpr uint32_t TM_Q = 0;
  static constexpr uint32_t TM_DO = D <= 128 ? 64 : D / 2;
  static constexpr uint32_t TM_SC = D <= 128 ? 128 : 160;  // S at TM_SC, dP at TM_SC + UK
  static constexpr uint32_t TM_AC = TM_SC + 2 * UK * NBUF; // dQ (D columns)
  static_assert(TM_AC + D <= 512, "dQ TMEM budget");
  static constexpr int TILE_Q = BWD_BT * D * 2;     // Q tile (128 rows)
  static constexpr int TILE_DO = BWD_BT * DV * 2;   // dO tile
  static constexpr int SUB_K = UK * D * 2;          // K sub-tile (UK rows)
  static constexpr int SUB_V = UK * DV * 2;         // V sub-tile
  static constexpr int STAGE = SUB_K + SUB_V;
  static constexpr int DS = BWD_BT * UK * 2;        // one dS tile (128 x UK, 16-bit)
  static constexpr bool DS_ALIAS = 2 * DS <= TILE_Q + TILE_DO;  // dS tiles over Q / dO
  static constexpr int Q_OFF = 0;
  static constexpr int DO_OFF = TILE_Q;
  static constexpr int STAGE_OFF = TILE_Q + TILE_DO + (DS_ALIAS ? 0 : 2 * DS);
  static constexpr int DS_OFF = DS_ALIAS ? 0 : TILE_Q + TILE_DO;  // tile b at b*DS
  static constexpr int BUDGET = 227 * 1024 - 256 - 1024 - STAGE_OFF;
  // WIDE: K and V in separate rings (V is released when the S / dP MMAs are
  // done, K when the dQ accumulation is).  Otherwise NS stages of {K, V}.
  static constexpr bool SPLIT = WIDE && D == DV;
  static constexpr int SLOTS = BUDGET / SUB_K;
  static constexpr int NSV = SPLIT ? (SLOTS / 2 < 4 ? SLOTS / 2 : 4) : 0;
  static constexpr int NSK = SPLIT ? (SLOTS - NSV < 4 ? SLOTS - NSV : 4) : (BUDGET / STAGE > 4 ? 4 : BUDGET / STAGE);
  static_assert(NSK >= 2 && (!SPLIT || NSV >= 2), "dQ smem budget");
  __host__ __device__ static constexpr int k_off(int u) { return SPLIT ? (u % NSK) * SUB_K : (u % NSK) * STAGE; }
  __host__ __device__ static constexpr int v_off(int u) {
    return SPLIT ? NSK * SUB_K + (u % NSV) * SUB_V : (u % NSK) * STAGE + SUB_K;
  }
  static constexpr int BAR_OFF = STAGE_OFF + (SPLIT ? NSK * SUB_K + NSV * SUB_V : NSK * STAGE);
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
};

template <typename T, int D, int DV, bool BM>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    ffa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                      const BwdParams p) {
  using Cfg = DqCfg<D, DV>;
  constexpr int NSK = Cfg::NSK, NSV = Cfg::NSV;
  constexpr int NBUF = Cfg::NBUF;
  constexpr int UK = Cfg::UK;
  constexpr uint32_t TM_ACC = Cfg::TM_AC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Cfg::Q_OFF;
  uint8_t* sDO = smem + Cfg::DO_OFF;
  uint8_t* sStage = smem + Cfg::STAGE_OFF;
  uint8_t* sDS = smem + Cfg::DS_OFF;
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + Cfg::BAR_OFF);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_q = (p.Sq + BWD_BT - 1) / BWD_BT;
  // (b, q head) pairs in groups of p.grp_q whose K / V stay in L2 while the
  // group's query tiles stream them; within a group query tiles go heaviest
  // (latest, under causal masking) first.
  const int BH = p.B * p.Hq;
  const int g0 = (int)(blockIdx.x / ((unsigned)p.grp_q * n_q)) * p.grp_q;
  const int gn = min(p.grp_q, BH - g0);
  const int rem = (int)blockIdx.x - g0 * n_q;
  const int ii = rem / gn;
  const int i = p.causal ? (n_q - 1 - ii) : ii;
  const int bh = g0 + rem % gn;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hkv = h / (p.Hq / p.Hkv);
  int j_lo, j_hi;
  k_range_for_q_tile(p, i, j_lo, j_hi);
  // units of UK keys covering the 64-key sub-tiles [j_lo, j_hi); keys of a
  // unit outside the row's range are masked per column
  constexpr int R = UK / BWD_BS;
  j_lo = j_lo / R;
  j_hi = (j_hi + R - 1) / R;
  const int n = max(0, j_hi - j_lo);
  constexpr uint32_t FMT = DtypeFmt<T>::value;

  if (threadIdx.x == 0) bwd_init_bars(bars, 8, Cfg::WIDE ? 4 * 4 : 2 * 4);
  if (warp == BWD_WARP_MMA) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == BWD_WARP_LOAD) {
    if (lane == 0 && n > 0) {
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();
      mbar_arrive_expect_tx(&bars->fixed_full, Cfg::TILE_Q + Cfg::TILE_DO);
      for (int hf = 0; hf < 2; ++hf) {
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(&tmQ, &bars->fixed_full, sQ + c * BWD_BT * 128 + hf * BWD_BS * 128, c * 64,
                      i * BWD_BT + hf * BWD_BS, h, b, pol_q);
        for (int c = 0; c < DV / 64; ++c)
          tma_load_4d(&tmDO, &bars->fixed_full, sDO + c * BWD_BT * 128 + hf * BWD_BS * 128, c * 64,
                      i * BWD_BT + hf * BWD_BS, h, b, pol_q);
      }
      // unit u: V (SPLIT) into its own ring first, since its slot frees first;
      // then K (or {K, V}) into slot u % NSK
      int issued_k = 0, issued_v = 0;
      for (int u = 0; u < n; ++u) {
        const int jj = j_lo + u;
        if (Cfg::SPLIT) {
          const int sv = 4 + u % NSV, usev = u / NSV;
          if (usev > 0 && !mbar_wait(&bars->st_empty[sv], (usev - 1) & 1, p.ec, abort_flag, SITE_BWD_EMPTY)) break;
          mbar_arrive_expect_tx(&bars->st_full[sv], Cfg::SUB_V);
          uint8_t* dv = sStage + Cfg::v_off(u);
          for (int hf = 0; hf < R; ++hf)
            for (int c = 0; c < DV / 64; ++c)
              tma_load_4d(&tmV, &bars->st_full[sv], dv + c * UK * 128 + hf * BWD_BS * 128, c * 64,
                          jj * UK + hf * BWD_BS, hkv, b, pol_kv);
          ++issued_v;
        }
        const int s = u % NSK, use = u / NSK;
        if (use > 0 && !mbar_wait(&bars->st_empty[s], (use - 1) & 1, p.ec, abort_flag, SITE_BWD_EMPTY)) break;
        mbar_arrive_expect_tx(&bars->st_full[s], Cfg::SPLIT ? Cfg::SUB_K : Cfg::STAGE);
        uint8_t* dk = sStage + Cfg::k_off(u);
        uint8_t* dv = sStage + Cfg::v_off(u);
        for (int hf = 0; hf < R; ++hf) {
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(&tmK, &bars->st_full[s], dk + c * UK * 128 + hf * BWD_BS * 128, c * 64,
                        jj * UK + hf * BWD_BS, hkv, b, pol_kv);
          if (!Cfg::SPLIT)
            for (int c = 0; c < DV / 64; ++c)
              tma_load_4d(&tmV, &bars->st_full[s], dv + c * UK * 128 + hf * BWD_BS * 128, c * 64,
                          jj * UK + hf * BWD_BS, hkv, b, pol_kv);
        }
        ++issued_k;
      }
      if (*abort_flag) {
        mbar_wait(&bars->fixed_full, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
        for (int u = max(0, issued_k - NSK); u < issued_k; ++u)
          mbar_wait(&bars->st_full[u % NSK], (u / NSK) & 1, p.ec, abort_flag, SITE_BWD_DRAIN, true);
        if (Cfg::SPLIT)
          for (int u = max(0, issued_v - NSV); u < issued_v; ++u)
            mbar_wait(&bars->st_full[4 + u % NSV], (u / NSV) & 1, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      }
    }
    __syncwarp();
  } else if (warp == BWD_WARP_MMA || warp == BWD_WARP_ACC) {
    if (lane == 0 && n > 0) {
      const uint32_t idesc_s = make_idesc_f16(128, UK, FMT, 0, 0);  // S, dP (TMEM A x K-major B)
      const uint32_t idesc_dq = make_idesc_f16(128, D, FMT, 0, 1);  // dQ (K-major A x MN-major B)
      const uint64_t st_kdesc = make_sdesc_sw128(smem_u32(sStage), 16, 1024);
      const uint64_t st_mdesc = make_sdesc_sw128(smem_u32(sStage), UK * 128, 1024);
      const uint64_t ds_desc = make_sdesc_sw128(smem_u32(sDS), 16, 1024);
      const uint32_t tQ = tmem + Cfg::TM_Q, tDO = tmem + Cfg::TM_DO;
      const uint32_t tDQ = tmem + TM_ACC;
      auto issue_s = [&](int u) {
        const uint32_t tS = tmem + Cfg::TM_SC + 2 * UK * (u % NBUF);
        const uint64_t k_k = st_kdesc + (uint64_t)(Cfg::k_off(u) >> 4);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) mma_ts(tS, tQ + 8 * ks, k_k + kstep(ks, UK), idesc_s, ks > 0);
      };
      auto issue_dp = [&](int u) {
        const uint32_t tDP = tmem + Cfg::TM_SC + 2 * UK * (u % NBUF) + UK;
        const uint64_t v_k = st_kdesc + (uint64_t)(Cfg::v_off(u) >> 4);
#pragma unroll
        for (int ks = 0; ks < DV / 16; ++ks) mma_ts(tDP, tDO + 8 * ks, v_k + kstep(ks, UK), idesc_s, ks > 0);
      };
      auto issue_acc = [&](int v) {
        const int bb = v & 1;
        const uint64_t k_m = st_mdesc + (uint64_t)(Cfg::k_off(v) >> 4);
        const uint64_t ds_k = ds_desc + (uint64_t)((bb * Cfg::DS) >> 4);
#pragma unroll
        for (int ks = 0; ks < UK / 16; ++ks)
          mma_ss(tDQ, ds_k + kstep(ks, BWD_BT), k_m + (uint64_t)((ks * 16 * 128) >> 4), idesc_dq,
                 (v > 0 || ks > 0) ? 1u : 0u);
      };
      if (warp == BWD_WARP_MMA) {
        bool ok = mbar_wait(&bars->fixed_tmem, 0, p.ec, abort_flag, SITE_BWD_LOAD);
        if (ok) ok = bwd_issue_scores<NBUF>(bars, bars->tmem_free, n, NSK, NSV, p.ec, abort_flag, issue_s, issue_dp);
        mma_commit(&bars->s_done);
        if (!ok) mbar_wait(&bars->s_done, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      } else {
        const bool ok = bwd_issue_acc(bars, n, NSK, p.ec, abort_flag, issue_acc);
        mma_commit(&bars->acc_done);
        if (!ok) mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      }
    }
    __syncwarp();
  } else {
    // ------------------------- compute (query rows) -----------------------
    const int wg = warp / 4, pair = wg % 2, half = wg / 2;
    const int r = threadIdx.x % 128;
    const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
    // this warpgroup's 32 columns of a unit: WIDE, all warpgroups share each
    // unit (columns 32 wg); otherwise pairs alternate units (columns 32 half)
    const int colw = Cfg::WIDE ? 32 * wg : 32 * half;
    const uint32_t tS = tmem + lane_off + Cfg::TM_SC + colw, tDP = tS + UK;
    uint8_t* const sDSw = sDS + (colw / 64) * BWD_BT * 128;
    const int chunk_half = (colw / 32) & 1;
    const int row = i * BWD_BT + r;
    const int q_abs = row + p.q_offset;
    const int64_t sidx = (int64_t)(b * p.Hq + h) * p.Sq_pad + row;
    const float row_nl2 = p.nlse2[sidx], row_dl = p.delta[sidx];
    bool ok = true;
    if (n > 0 && wg < 2) {  // Q (warpgroup 0) / dO (warpgroup 1) into TMEM as the A operand
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->fixed_full, 0, p.ec, abort_flag, SITE_BWD_LOAD));
      if (ok) {
        if (wg == 0)
          tile_row_to_tmem<D>(sQ, r, tmem + lane_off + Cfg::TM_Q);
        else
          tile_row_to_tmem<DV>(sDO, r, tmem + lane_off + Cfg::TM_DO);
        tmem_st_wait();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->fixed_tmem);
    }
    // kept keys of this row: [q_abs - window + 1, min(q_abs, Skv - 1)]
    const int k_keep_lo = p.window > 0 ? q_abs - p.window + 1 : -0x3fffffff;
    const int k_keep_hi = min(p.causal ? q_abs : 0x3fffffff, p.Skv - 1);
    // unit u: barriers u % 2 with phase (u / 2) % 2, dS tile u % 2
    for (int u = Cfg::WIDE ? 0 : pair; u < n && ok; u += Cfg::WIDE ? 1 : 2) {
      const int bb = u & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->sp_full[bb], (u >> 1) & 1, p.ec, abort_flag, SITE_BWD_SP));
      if (!ok) break;
      tc_fence_after();
      const int c0 = (j_lo + u) * UK + colw;
      const int keep_lo = k_keep_lo - c0, keep_hi = k_keep_hi - c0;
      uint32_t bm_bits = ~0u;
      if (BM) {  // keys are the block mask's columns here
        const uint8_t* mrow = p.block_mask + (size_t)(min(row, p.Sq - 1) / p.mask_bq) * p.n_bc;
        bm_bits = block_mask_bits32(c0, p.mask_bkv, p.n_bc, [&](int bc) { return mrow[bc] != 0; });
      }
      const bool masked = !__all_sync(0xffffffffu, keep_lo <= 0 && keep_hi >= 31 && (!BM || bm_bits == ~0u));
      ok = bwd_unit<T, false, false, BM>(p, tS, tDP, &bars->tmem_free[bb], nullptr, nullptr, row_nl2, row_dl,
                                         keep_lo, keep_hi, bm_bits, masked, &bars->pt_free[bb],
                                     u >= 2 ? ((u - 2) >> 1) & 1 : -1, abort_flag, nullptr, sDSw + bb * Cfg::DS, r,
                                     chunk_half);
      if (lane == 0) mbar_arrive(&bars->ds_ready[bb]);
    }
    // epilogue: warpgroup w stores dQ columns [w D/4, (w+1) D/4)
    const bool have = ok && n > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DONE));
    if (have) tc_fence_after();
    const bool store = row < p.Sq;
    T* dqrow = reinterpret_cast<T*>(p.dq) + (size_t)b * p.dq_sb + (size_t)h * p.dq_sh + (size_t)row * p.dq_ss;
#pragma unroll
    for (int c = wg * (D / 4); c < (wg + 1) * (D / 4); c += 16) {
      uint32_t v[16];
      if (have) {
        tmem_ld16(tmem + lane_off + TM_ACC + c, v);
        tmem_ld_wait16(v);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0u;
      }
      store_row16<T>(dqrow + c, v, p.scale, store);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == BWD_WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// CTA-order group sizes (see the kernels' block mapping): groups whose
// streamed operands fit in about 48 MB of L2 together, so each streamed tile
// is read from HBM once per group instead of once per CTA that reads it.
// Sliding windows keep the plain order (a tile's readers are then near each
// other in it anyway).  FFA_BWD_HEAD_GROUP in the environment overrides it
// (0: the plain order; N > 0: N kv heads per group; for measurements).
static void bwd_head_groups(BwdParams& p, int D, int DV) {
  static const int forced = [] {
    const char* e = getenv("FFA_BWD_HEAD_GROUP");
    return e ? atoi(e) : -1;
  }();
  const int G = p.Hq / p.Hkv;
  const int BHk = p.B * p.Hkv, BH = p.B * p.Hq;
  if (forced > 0) {  // kv heads per group
    p.grp_kv = forced > BHk ? BHk : forced;
    p.grp_q = p.grp_kv * G;
    return;
  }
  if (forced == 0 || (p.window > 0 && p.window < p.Skv)) {
    p.grp_kv = BHk;
    p.grp_q = BH;
    return;
  }
  const double budget = 48.0 * 1024 * 1024;
  const double qdo = (double)p.Sq * (D + DV) * 2.0 * G;  // Q and dO of a GQA group
  const double kv = (double)p.Skv * (D + DV) * 2.0;      // K and V of a kv head
  const int nk = (int)(budget / (qdo > 1 ? qdo : 1));
  const int nq = (int)(budget / (kv > 1 ? kv : 1));
  p.grp_kv = nk < 1 ? 1 : (nk > BHk ? BHk : nk);
  p.grp_q = nq < 1 ? G : ((long long)nq * G > BH ? BH : nq * G);
  // Short grids (under 10 waves) keep the plain order, as the forward does:
  // the heaviest tiles of the last group would otherwise start near the end.
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if ((long long)(p.Skv + BWD_BT - 1) / BWD_BT * BHk < 10LL * sms) p.grp_kv = BHk;
  if ((long long)(p.Sq + BWD_BT - 1) / BWD_BT * BH < 10LL * sms) p.grp_q = BH;
}

template <typename T, int D, int DV, bool BM>
static int launch_bwd(const CUtensorMap* maps, const BwdParams& p, const void* o, const void* dout,
                      const float* lse, float* lse2, float* delta, const int64_t* o_str, const int64_t* do_str,
                      cudaStream_t st) {
  // 1. preprocess
  const int64_t n_rows64 = (int64_t)p.B * p.Hq * p.Sq_pad;
  const int threads = 256;
  // The scalar preprocess spends a warp per row: its grid is the larger one.
  if (n_rows64 * 32 / threads + 1 > 0x7fffffffLL) {
    set_last_error("ffa_bwd: B * Hq * round_up(Sq, 128) rows exceed the preprocess grid limit");
    return FFA_ERR_UNSUPPORTED;
  }
  const int n_rows = (int)n_rows64;
  const bool vec = ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(dout)) & 15) == 0 &&
                   o_str[0] % 8 == 0 && o_str[1] % 8 == 0 && o_str[2] % 8 == 0 && do_str[0] % 8 == 0 &&
                   do_str[1] % 8 == 0 && do_str[2] % 8 == 0;
  if (vec) {
    constexpr int TPR = DV / 8;
    const int blocks = (int)(((int64_t)n_rows * TPR + threads - 1) / threads);
    ffa_bwd_pre_vec_kernel<T, TPR><<<blocks, threads, 0, st>>>(
        reinterpret_cast<const T*>(o), reinterpret_cast<const T*>(dout), lse, lse2, delta, p.Hq, p.Sq, p.Sq_pad,
        o_str[0], o_str[1], o_str[2], do_str[0], do_str[1], do_str[2], n_rows);
  } else {
    const int blocks = (int)(((int64_t)n_rows * 32 + threads - 1) / threads);
    ffa_bwd_pre_kernel<T><<<blocks, threads, 0, st>>>(
        reinterpret_cast<const T*>(o), reinterpret_cast<const T*>(dout), lse, lse2, delta, p.Hq, p.Sq, p.Sq_pad,
        DV, o_str[0], o_str[1], o_str[2], do_str[0], do_str[1], do_str[2], n_rows);
  }
  int s = launch_status();
  if (s) return s;
  // 2. dK / dV
  {
    auto kern = ffa_bwd_dkdv_kernel<T, D, DV, BM>;
    static std::atomic<uint64_t> done{0};
    if ((s = smem_attr_once(kern, DkdvCfg<D, DV>::SMEM, done))) return s;
    const int grid = (p.Skv + BWD_BT - 1) / BWD_BT * p.B * p.Hkv;
    kern<<<grid, BWD_THREADS, DkdvCfg<D, DV>::SMEM, st>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p);
    if ((s = launch_status())) return s;
  }
  // 3. dQ
  {
    auto kern = ffa_bwd_dq_kernel<T, D, DV, BM>;
    static std::atomic<uint64_t> done{0};
    if ((s = smem_attr_once(kern, DqCfg<D, DV>::SMEM, done))) return s;
    const int grid = (p.Sq + BWD_BT - 1) / BWD_BT * p.B * p.Hq;
    kern<<<grid, BWD_THREADS, DqCfg<D, DV>::SMEM, st>>>(maps[0], maps[1], maps[2], maps[3], p);
    if ((s = launch_status())) return s;
  }
  return FFA_OK;
}

}  // namespace ffa

extern "C" size_t ffa_bwd_workspace_size(int B, int Hq, int Sq) {
  const size_t sq_pad = ((size_t)Sq + 127) / 128 * 128;
  return 2 * (size_t)B * Hq * sq_pad * sizeof(float) + 256;
}

extern "C" int ffa_bwd_masked(const void* dout, const void* q, const void* k, const void* v, const void* o,
                              const float* lse, void* dq, void* dk, void* dv, int dtype, int B, int Hq, int Hkv,
                              int Sq, int Skv, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                              const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                              float scale, int causal, int q_offset, int window, float softcap,
                              const uint8_t* block_mask, int n_br, int n_bc, int mask_bq, int mask_bkv,
                              void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  using namespace ffa;
  if (!dout || !q || !k || !v || !o || !lse || !dq || !dk || !dv) return FFA_ERR_INVALID_ARG;
  if (block_mask && (n_br <= 0 || n_bc <= 0 || mask_bq <= 0 || mask_bkv <= 0 ||
                     (int64_t)n_br * mask_bq < Sq || (int64_t)n_bc * mask_bkv < Skv))
    return FFA_ERR_INVALID_ARG;
  if (!q_strides || !k_strides || !v_strides || !o_strides || !do_strides || !dq_strides || !dk_strides ||
      !dv_strides)
    return FFA_ERR_INVALID_ARG;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Skv <= 0 || Hq % Hkv != 0) return FFA_ERR_INVALID_ARG;
  if (!((D == 64 && Dv == 64) || (D == 128 && Dv == 128) || (D == 192 && Dv == 128))) return FFA_ERR_UNSUPPORTED;
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16 && dtype != FFA_DTYPE_F32) return FFA_ERR_UNSUPPORTED;
  const size_t need = ffa_bwd_workspace_size(B, Hq, Sq);
  if (!workspace || workspace_bytes < need) return FFA_ERR_WORKSPACE;
  if (dtype == FFA_DTYPE_F32)
    return f32_bwd(dout, q, k, v, o, lse, dq, dk, dv, B, Hq, Hkv, Sq, Skv, D, Dv, q_strides, k_strides, v_strides,
                   o_strides, do_strides, dq_strides, dk_strides, dv_strides, scale, causal, q_offset, window,
                   softcap, block_mask, n_br, n_bc, mask_bq, mask_bkv,
                   reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 127) & ~uintptr_t(127)), stream);
  const int64_t* outs[3] = {dq_strides, dk_strides, dv_strides};
  for (auto* st : outs)
    if ((st[0] % 8) || (st[1] % 8) || (st[2] % 8)) return FFA_ERR_INVALID_ARG;
  if (!aligned16(dq) || !aligned16(dk) || !aligned16(dv) || (o_strides[2] % 2) || (do_strides[2] % 2) ||
      (reinterpret_cast<uintptr_t>(o) & 3) || (reinterpret_cast<uintptr_t>(dout) & 3))
    return FFA_ERR_INVALID_ARG;

  BwdParams p{};
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.dq_sb = dq_strides[0];
  p.dq_sh = dq_strides[1];
  p.dq_ss = dq_strides[2];
  p.dk_sb = dk_strides[0];
  p.dk_sh = dk_strides[1];
  p.dk_ss = dk_strides[2];
  p.dv_sb = dv_strides[0];
  p.dv_sh = dv_strides[1];
  p.dv_ss = dv_strides[2];
  p.Sq_pad = (Sq + 127) / 128 * 128;
  uintptr_t ws = (reinterpret_cast<uintptr_t>(workspace) + 127) & ~uintptr_t(127);
  float* lse2 = reinterpret_cast<float*>(ws);
  float* delta = lse2 + (size_t)B * Hq * p.Sq_pad;
  p.nlse2 = lse2;
  p.delta = delta;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Sq = Sq;
  p.Skv = Skv;
  p.q_offset = q_offset;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.use_softcap = softcap > 0.f;
  p.sc_pre = p.use_softcap ? scale / softcap : 0.f;
  p.sc_post = p.use_softcap ? softcap * 1.4426950408889634f : 0.f;
  p.sc_small = p.use_softcap ? 0.5f * softcap / scale : 0.f;
  softcap_poly_coeffs(p.sc_pre, p.sc_poly);
  p.causal = causal;
  p.window = window > 0 ? window : 0;
  p.block_mask = block_mask;
  p.n_br = n_br;
  p.n_bc = n_bc;
  p.mask_bq = mask_bq;
  p.mask_bkv = mask_bkv;
  p.ec.err = dev_err;
  p.ec.limit_ns = wait_limit_ns();
  bwd_head_groups(p, D, Dv);

  const CUtensorMapDataType dt =
      dtype == FFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap maps[6];
  int st = make_tmap_4d(&maps[0], q, dt, 2, D, Sq, Hq, B, q_strides[2] * 2, q_strides[1] * 2, q_strides[0] * 2, 64,
                        BWD_BS);
  if (!st)
    st = make_tmap_4d(&maps[1], k, dt, 2, D, Skv, Hkv, B, k_strides[2] * 2, k_strides[1] * 2, k_strides[0] * 2, 64,
                      BWD_BS);
  if (!st)
    st = make_tmap_4d(&maps[2], v, dt, 2, Dv, Skv, Hkv, B, v_strides[2] * 2, v_strides[1] * 2, v_strides[0] * 2, 64,
                      BWD_BS);
  if (!st)
    st = make_tmap_4d(&maps[3], dout, dt, 2, Dv, Sq, Hq, B, do_strides[2] * 2, do_strides[1] * 2, do_strides[0] * 2,
                      64, BWD_BS);
  // dK / dV stores: one 32-row x 64-column box per warp
  if (!st)
    st = make_tmap_4d(&maps[4], dk, dt, 2, D, Skv, Hkv, B, dk_strides[2] * 2, dk_strides[1] * 2, dk_strides[0] * 2,
                      64, 32);
  if (!st)
    st = make_tmap_4d(&maps[5], dv, dt, 2, Dv, Skv, Hkv, B, dv_strides[2] * 2, dv_strides[1] * 2, dv_strides[0] * 2,
                      64, 32);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto bm) -> int {
    constexpr bool BM = decltype(bm)::value;
    if (dtype == FFA_DTYPE_BF16) {
      if (D == 64)
        return launch_bwd<__nv_bfloat16, 64, 64, BM>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
      if (D == 128)
        return launch_bwd<__nv_bfloat16, 128, 128, BM>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
      return launch_bwd<__nv_bfloat16, 192, 128, BM>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
    }
    if (D == 64) return launch_bwd<__half, 64, 64, BM>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
    if (D == 128)
      return launch_bwd<__half, 128, 128, BM>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
    return launch_bwd<__half, 192, 128, BM>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
  };
  // Block-mask support is compiled into its own kernels, so the unmasked
  // kernels carry none of its per-unit work.
  return block_mask ? run(std::true_type{}) : run(std::false_type{});
}

extern "C" int ffa_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o,
                       const float* lse, void* dq, void* dk, void* dv, int dtype, int B, int Hq, int Hkv, int Sq,
                       int Skv, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                       const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                       const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                       float scale, int causal, int q_offset, int window, float softcap, void* workspace,
                       size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  return ffa_bwd_masked(dout, q, k, v, o, lse, dq, dk, dv, dtype, B, Hq, Hkv, Sq, Skv, D, Dv, q_strides, k_strides,
                        v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, scale, causal, q_offset,
                        window, softcap, nullptr, 0, 0, 0, 0, workspace, workspace_bytes, dev_err, stream);
}
