// Backward attention for B200 (sm_100a): deterministic, recompute-based.
//
// Replaces kernels/cpu_reference.py:319 flash_attn_cpu_backward,
// kernels/cpu_fa4.py:445 fa4_backward and kernels/triton_bwd.py behind
// ffa_bwd().  Three launches, no atomics, fixed summation order (so results
// are bit-identical run to run):
//   1. preprocess: Delta = rowsum(dO * O) and LSE in base-2 units, both padded
//      to whole 128-row tiles (padding rows get LSE = +inf, so P = 0 there);
//   2. dK/dV: one CTA per (batch, kv head, 128-key tile).  For every query
//      head of the GQA group and every 128-row query tile that sees the keys:
//        S^T = K Q^T, dP^T = V dO^T        (tensor cores, fp32 in TMEM)
//        P^T = 2^(S^T*scale*log2e - LSE2), dS^T = P^T (dP^T - Delta) [* softcap']
//        dV += P^T dO,  dK += dS^T Q      (P^T / dS^T as 16-bit A operands in TMEM)
//   3. dQ: one CTA per (batch, query head, 128-row query tile):
//        S = Q K^T, dP = dO V^T, dS as above, dQ += dS K.
// dK and dQ are multiplied by the softmax scale in their epilogues.
// TMEM (dK/dV kernel): [0,128) S^T/P^T, [128,256) dP^T/dS^T, then dV, dK.
// TMEM (dQ kernel):    [0,128) S/dS,    [128,256) dP,        then dQ.
#include "ffa_common.cuh"
#include "ffa_host.h"

namespace ffa {

constexpr int BWD_BM = 128;  // query rows per tile
constexpr int BWD_BN = 128;  // keys per tile
constexpr int BWD_THREADS = 192;  // warps 0-3 compute, 4 TMA producer, 5 MMA issuer + TMEM owner
constexpr int BWD_WARP_LOAD = 4;
constexpr int BWD_WARP_MMA = 5;

struct BwdParams {
  // dK/dV kernel outputs
  void* dk;
  void* dv;
  int64_t dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  // dQ kernel output
  void* dq;
  int64_t dq_sb, dq_sh, dq_ss;
  const float* lse2;   // [B*Hq, Sq_pad] base-2 LSE, +inf on padding rows
  const float* delta;  // [B*Hq, Sq_pad]
  int Sq_pad;
  int B, Hq, Hkv, Sq, Skv, q_offset;
  float scale;         // softmax scale (applied to dK / dQ in the epilogue)
  float scale_log2;
  float sc_pre, sc_post;
  int use_softcap;
  int causal, window;
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

// Query-tile range [i_lo, i_hi) that interacts with key tile j.
__device__ __forceinline__ void q_range_for_key_tile(const BwdParams& p, int j, int& i_lo, int& i_hi) {
  const int n_q = (p.Sq + BWD_BM - 1) / BWD_BM;
  const int k_lo = j * BWD_BN, k_hi = min(k_lo + BWD_BN, p.Skv) - 1;
  i_lo = 0;
  i_hi = n_q;
  if (p.causal) {  // need some q_abs >= k_lo  ->  q >= k_lo - q_offset
    const int qmin = k_lo - p.q_offset;
    i_lo = qmin > 0 ? qmin / BWD_BM : 0;
  }
  if (p.window > 0) {  // need some q_abs <= k_hi + window - 1
    const int qmax = k_hi + p.window - 1 - p.q_offset;
    i_hi = qmax < 0 ? 0 : min(n_q, qmax / BWD_BM + 1);
  }
  if (i_lo > i_hi) i_lo = i_hi;
}

// Key-tile range [j_lo, j_hi) that interacts with query tile i.
__device__ __forceinline__ void k_range_for_q_tile(const BwdParams& p, int i, int& j_lo, int& j_hi) {
  const int n_kv = (p.Skv + BWD_BN - 1) / BWD_BN;
  const int a_lo = i * BWD_BM + p.q_offset;
  const int a_hi = min(i * BWD_BM + BWD_BM, p.Sq) - 1 + p.q_offset;
  j_hi = n_kv;
  if (p.causal) j_hi = min(n_kv, a_hi >= 0 ? a_hi / BWD_BN + 1 : 0);
  j_lo = 0;
  if (p.window > 0) {
    const int lo_col = a_lo - p.window + 1;
    if (lo_col > 0) j_lo = min(lo_col / BWD_BN, j_hi);
  }
}

__device__ __forceinline__ bool pair_visible(const BwdParams& p, int q_abs, int key) {
  bool keep = key < p.Skv;
  if (p.causal) keep = keep && key <= q_abs;
  if (p.window > 0) keep = keep && key >= q_abs - p.window + 1;
  return keep;
}

// P and dS for one 32-wide chunk of a TMEM row.  `s` holds raw Q.K scores,
// `dp` holds dO.V values.  `lse2`/`delta` give the per-column (dK/dV kernel)
// or per-row (dQ kernel, broadcast) statistics.
template <typename T, bool COLS_ARE_QUERIES>
__device__ __forceinline__ void bwd_chunk(const BwdParams& p, const uint32_t* s, const uint32_t* dp,
                                          const float* lse2_col, const float* delta_col, float lse2_row,
                                          float delta_row, int row_pos, int col0, bool need_mask,
                                          uint32_t* pk_p, uint32_t* pk_ds) {
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    float pv[2], dv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = e + u;
      const float raw = __uint_as_float(s[c]);
      float x, dsc = 1.f;
      if (p.use_softcap) {
        const float th = tanh_acc(raw * p.sc_pre);
        x = th * p.sc_post;
        dsc = 1.f - th * th;
      } else {
        x = raw * p.scale_log2;
      }
      const float l2 = COLS_ARE_QUERIES ? lse2_col[c] : lse2_row;
      const float dl = COLS_ARE_QUERIES ? delta_col[c] : delta_row;
      float pr = ex2(x - l2);
      if (need_mask) {
        const int q_abs = COLS_ARE_QUERIES ? (col0 + c + p.q_offset) : row_pos;
        const int key = COLS_ARE_QUERIES ? row_pos : (col0 + c);
        if (!pair_visible(p, q_abs, key)) pr = 0.f;
      }
      pv[u] = pr;
      dv[u] = pr * (__uint_as_float(dp[c]) - dl) * dsc;
    }
    if (pk_p) pk_p[e / 2] = pack2<T>(pv[0], pv[1]);
    pk_ds[e / 2] = pack2<T>(dv[0], dv[1]);
  }
}

__device__ __forceinline__ float2 load2f(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ float2 load2f(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}

// ---------------------------------------------------------------------------
// 1. preprocess: Delta and base-2 LSE, padded to whole tiles
// ---------------------------------------------------------------------------
template <typename T>
__global__ void ffa_bwd_pre_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                   const float* __restrict__ lse, float* __restrict__ lse2,
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
    // offset works; +inf keeps 2^(x - LSE2) at exactly 0.
    lse2[idx] = (q < Sq && l != -INFINITY) ? l * 1.4426950408889634f : INFINITY;
  }
}

// ---------------------------------------------------------------------------
// 2. dK / dV
// ---------------------------------------------------------------------------
template <int D>
struct DkdvCfg {
  static constexpr int TILE = 128 * D * 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int STAGE_OFF = 2 * TILE;                // 2 stages of {Q, dO}
  static constexpr int STAT_OFF = STAGE_OFF + 4 * TILE;     // 2 stages of {lse2[128], delta[128]}
  static constexpr int BAR_OFF = STAT_OFF + 2 * 2 * 128 * 4;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
};

struct DkdvBars {
  uint64_t kv_full;
  uint64_t st_full[2];
  uint64_t st_empty[2];
  uint64_t sp_full;
  uint64_t ds_ready;
  uint64_t acc_done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <typename T, int D>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    ffa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const BwdParams p) {
  using Cfg = DkdvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + Cfg::K_OFF;
  uint8_t* sV = smem + Cfg::V_OFF;
  uint8_t* sStage = smem + Cfg::STAGE_OFF;  // stage s: Q at 2*s*TILE, dO at (2*s+1)*TILE
  float* sStat = reinterpret_cast<float*>(smem + Cfg::STAT_OFF);  // stage s: lse2 at 256*s, delta at 256*s+128
  DkdvBars* bars = reinterpret_cast<DkdvBars*>(smem + Cfg::BAR_OFF);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int j = blockIdx.x;
  const int bhk = blockIdx.y;
  const int b = bhk / p.Hkv, hkv = bhk % p.Hkv;
  const int group = p.Hq / p.Hkv;
  int i_lo, i_hi;
  q_range_for_key_tile(p, j, i_lo, i_hi);
  const int n_i = i_hi - i_lo;
  const int n_pairs = n_i * group;  // (query head of the group, query tile) pairs, head-major
  constexpr uint32_t FMT = DtypeFmt<T>::value;

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->st_full[s], 1);
      mbar_init(&bars->st_empty[s], 1);
    }
    mbar_init(&bars->sp_full, 1);
    mbar_init(&bars->ds_ready, 128);
    mbar_init(&bars->acc_done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == BWD_WARP_MMA) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == BWD_WARP_LOAD) {
    if (lane == 0 && n_pairs > 0) {
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(&bars->kv_full, 2 * Cfg::TILE);
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(&tmK, &bars->kv_full, sK + c * 128 * 128, c * 64, j * BWD_BN, hkv, b, pol);
        tma_load_4d(&tmV, &bars->kv_full, sV + c * 128 * 128, c * 64, j * BWD_BN, hkv, b, pol);
      }
      int issued = 0;
      for (int pi = 0; pi < n_pairs; ++pi) {
        const int s = pi & 1, use = pi >> 1;
        if (use > 0 && !mbar_wait(&bars->st_empty[s], (use - 1) & 1, p.ec, abort_flag, SITE_BWD_EMPTY)) break;
        const int g = pi / n_i, i = i_lo + pi % n_i;
        const int h = hkv * group + g;
        mbar_arrive_expect_tx(&bars->st_full[s], 2 * Cfg::TILE + 2 * 128 * 4);
        uint8_t* dst = sStage + 2 * s * Cfg::TILE;
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(&tmQ, &bars->st_full[s], dst + c * 128 * 128, c * 64, i * BWD_BM, h, b, pol);
          tma_load_4d(&tmDO, &bars->st_full[s], dst + Cfg::TILE + c * 128 * 128, c * 64, i * BWD_BM, h, b, pol);
        }
        const int64_t row0 = (int64_t)(b * p.Hq + h) * p.Sq_pad + i * BWD_BM;
        bulk_load(sStat + 256 * s, p.lse2 + row0, 128 * 4, &bars->st_full[s]);
        bulk_load(sStat + 256 * s + 128, p.delta + row0, 128 * 4, &bars->st_full[s]);
        ++issued;
      }
      if (*abort_flag) {
        mbar_wait(&bars->kv_full, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
        for (int q = max(0, issued - 2); q < issued; ++q)
          mbar_wait(&bars->st_full[q & 1], (q >> 1) & 1, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      }
    }
    __syncwarp();
  } else if (warp == BWD_WARP_MMA) {
    if (lane == 0 && n_pairs > 0) {
      const uint32_t idesc_t = make_idesc_f16(128, 128, FMT, 0, 0);  // S^T, dP^T (K-major x K-major)
      const uint32_t idesc_acc = make_idesc_f16(128, D, FMT, 0, 1);  // dV, dK (TMEM A x MN-major B)
      const uint64_t k_desc = make_sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t v_desc = make_sdesc_sw128(smem_u32(sV), 16, 1024);
      const uint64_t st_kdesc = make_sdesc_sw128(smem_u32(sStage), 16, 1024);
      const uint64_t st_mdesc = make_sdesc_sw128(smem_u32(sStage), 128 * 128, 1024);
      const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + D;
      bool ok = mbar_wait(&bars->kv_full, 0, p.ec, abort_flag, SITE_BWD_LOAD);
      for (int pi = 0; pi < n_pairs && ok; ++pi) {
        const int s = pi & 1;
        if (!(ok = mbar_wait(&bars->st_full[s], (pi >> 1) & 1, p.ec, abort_flag, SITE_BWD_LOAD))) break;
        tc_fence_after();
        const uint64_t q_k = st_kdesc + (uint64_t)((2 * s * Cfg::TILE) >> 4);
        const uint64_t do_k = st_kdesc + (uint64_t)(((2 * s + 1) * Cfg::TILE) >> 4);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = ((ks / 4) * (128 * 128) + (ks % 4) * 32) >> 4;
          mma_ss(tS, k_desc + off, q_k + off, idesc_t, ks > 0);
        }
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = ((ks / 4) * (128 * 128) + (ks % 4) * 32) >> 4;
          mma_ss(tDP, v_desc + off, do_k + off, idesc_t, ks > 0);
        }
        mma_commit(&bars->sp_full);
        if (!(ok = mbar_wait(&bars->ds_ready, pi & 1, p.ec, abort_flag, SITE_BWD_DS))) break;
        tc_fence_after();
        const uint64_t q_m = st_mdesc + (uint64_t)((2 * s * Cfg::TILE) >> 4);
        const uint64_t do_m = st_mdesc + (uint64_t)(((2 * s + 1) * Cfg::TILE) >> 4);
#pragma unroll
        for (int ks = 0; ks < BWD_BM / 16; ++ks) {
          const uint32_t off = (ks * 16 * 128) >> 4;
          mma_ts(tDV, tS + ks * 8, do_m + off, idesc_acc, (pi > 0 || ks > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int ks = 0; ks < BWD_BM / 16; ++ks) {
          const uint32_t off = (ks * 16 * 128) >> 4;
          mma_ts(tDK, tDP + ks * 8, q_m + off, idesc_acc, (pi > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&bars->st_empty[s]);
      }
      mma_commit(&bars->acc_done);
      if (!ok) mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
    }
    __syncwarp();
  } else {
    // ------------------------- compute (key rows) -------------------------
    const int r = threadIdx.x;  // key row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
    const uint32_t tS = tmem + lane_off, tDP = tmem + lane_off + 128;
    const int key = j * BWD_BN + r;
    bool ok = true;
    for (int pi = 0; pi < n_pairs; ++pi) {
      const int s = pi & 1;
      const int i = i_lo + pi % n_i;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->sp_full, pi & 1, p.ec, abort_flag, SITE_BWD_SP));
      if (!ok) break;
      tc_fence_after();
      const int q0 = i * BWD_BM;
      // masks are needed where the tile straddles a causal / window / length edge
      const int qa_lo = q0 + p.q_offset, qa_hi = q0 + BWD_BM - 1 + p.q_offset;
      const int k_lo = j * BWD_BN, k_hi = k_lo + BWD_BN - 1;
      const bool need_mask = (p.causal && k_hi > qa_lo) || (p.window > 0 && k_lo < qa_hi - p.window + 1) ||
                             (k_hi >= p.Skv);
      const float* lse2 = sStat + 256 * s;
      const float* delta = lse2 + 128;
#pragma unroll 1
      for (int cb = 0; cb < BWD_BM; cb += 32) {
        uint32_t sv[32], dpv[32];
        tmem_ld32(tS + cb, sv);
        tmem_ld32(tDP + cb, dpv);
        tmem_ld_wait32(sv);
        tmem_ld_wait32(dpv);
        uint32_t pk_p[16], pk_ds[16];
        bwd_chunk<T, true>(p, sv, dpv, lse2 + cb, delta + cb, 0.f, 0.f, key, q0 + cb, need_mask, pk_p, pk_ds);
        tmem_st16(tS + cb / 2, pk_p);
        tmem_st16(tDP + cb / 2, pk_ds);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->ds_ready);
    }
    // ------------------------------ epilogue ------------------------------
    const bool have = ok && n_pairs > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DONE));
    if (have) tc_fence_after();
    const bool store = key < p.Skv;
    T* dvrow = reinterpret_cast<T*>(p.dv) + (size_t)b * p.dv_sb + (size_t)hkv * p.dv_sh + (size_t)key * p.dv_ss;
    T* dkrow = reinterpret_cast<T*>(p.dk) + (size_t)b * p.dk_sb + (size_t)hkv * p.dk_sh + (size_t)key * p.dk_ss;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const uint32_t tacc = tmem + lane_off + 256 + which * D;
      const float mul = which ? p.scale : 1.f;
      T* dst_row = which ? dkrow : dvrow;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t v[32];
        if (have) {
          tmem_ld32(tacc + c, v);
          tmem_ld_wait32(v);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0u;
        }
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = pack2<T>(__uint_as_float(v[2 * e]) * mul, __uint_as_float(v[2 * e + 1]) * mul);
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(dst_row + c);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
        }
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
template <int D>
struct DqCfg {
  static constexpr int TILE = 128 * D * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int DO_OFF = TILE;
  static constexpr int KV_OFF = 2 * TILE;  // 2 stages of {K, V}
  static constexpr int BAR_OFF = KV_OFF + 4 * TILE;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
};

struct DqBars {
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t sp_full;
  uint64_t ds_ready;
  uint64_t acc_done;
  uint32_t tmem_base;
  int abort;
};

template <typename T, int D>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    ffa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                      const BwdParams p) {
  using Cfg = DqCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Cfg::Q_OFF;
  uint8_t* sDO = smem + Cfg::DO_OFF;
  uint8_t* sKV = smem + Cfg::KV_OFF;  // stage s: K at 2*s*TILE, V at (2*s+1)*TILE
  DqBars* bars = reinterpret_cast<DqBars*>(smem + Cfg::BAR_OFF);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_q = (p.Sq + BWD_BM - 1) / BWD_BM;
  // heavier (later) query tiles first under causal masking
  const int i = p.causal ? (n_q - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hkv = h / (p.Hq / p.Hkv);
  int j_lo, j_hi;
  k_range_for_q_tile(p, i, j_lo, j_hi);
  const int n = max(0, j_hi - j_lo);
  constexpr uint32_t FMT = DtypeFmt<T>::value;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    mbar_init(&bars->sp_full, 1);
    mbar_init(&bars->ds_ready, 128);
    mbar_init(&bars->acc_done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
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
      mbar_arrive_expect_tx(&bars->q_full, 2 * Cfg::TILE);
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(&tmQ, &bars->q_full, sQ + c * 128 * 128, c * 64, i * BWD_BM, h, b, pol_q);
        tma_load_4d(&tmDO, &bars->q_full, sDO + c * 128 * 128, c * 64, i * BWD_BM, h, b, pol_q);
      }
      int issued = 0;
      for (int it = 0; it < n; ++it) {
        const int s = it & 1, use = it >> 1;
        if (use > 0 && !mbar_wait(&bars->kv_empty[s], (use - 1) & 1, p.ec, abort_flag, SITE_BWD_EMPTY)) break;
        const int j = j_lo + it;
        mbar_arrive_expect_tx(&bars->kv_full[s], 2 * Cfg::TILE);
        uint8_t* dst = sKV + 2 * s * Cfg::TILE;
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(&tmK, &bars->kv_full[s], dst + c * 128 * 128, c * 64, j * BWD_BN, hkv, b, pol_kv);
          tma_load_4d(&tmV, &bars->kv_full[s], dst + Cfg::TILE + c * 128 * 128, c * 64, j * BWD_BN, hkv, b, pol_kv);
        }
        ++issued;
      }
      if (*abort_flag) {
        mbar_wait(&bars->q_full, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
        for (int q = max(0, issued - 2); q < issued; ++q)
          mbar_wait(&bars->kv_full[q & 1], (q >> 1) & 1, p.ec, abort_flag, SITE_BWD_DRAIN, true);
      }
    }
    __syncwarp();
  } else if (warp == BWD_WARP_MMA) {
    if (lane == 0 && n > 0) {
      const uint32_t idesc_s = make_idesc_f16(128, 128, FMT, 0, 0);
      const uint32_t idesc_dq = make_idesc_f16(128, D, FMT, 0, 1);
      const uint64_t q_desc = make_sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t do_desc = make_sdesc_sw128(smem_u32(sDO), 16, 1024);
      const uint64_t kv_kdesc = make_sdesc_sw128(smem_u32(sKV), 16, 1024);
      const uint64_t kv_mdesc = make_sdesc_sw128(smem_u32(sKV), 128 * 128, 1024);
      const uint32_t tS = tmem, tDP = tmem + 128, tDQ = tmem + 256;
      bool ok = mbar_wait(&bars->q_full, 0, p.ec, abort_flag, SITE_BWD_LOAD);
      for (int it = 0; it < n && ok; ++it) {
        const int s = it & 1;
        if (!(ok = mbar_wait(&bars->kv_full[s], (it >> 1) & 1, p.ec, abort_flag, SITE_BWD_LOAD))) break;
        tc_fence_after();
        const uint64_t k_k = kv_kdesc + (uint64_t)((2 * s * Cfg::TILE) >> 4);
        const uint64_t v_k = kv_kdesc + (uint64_t)(((2 * s + 1) * Cfg::TILE) >> 4);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = ((ks / 4) * (128 * 128) + (ks % 4) * 32) >> 4;
          mma_ss(tS, q_desc + off, k_k + off, idesc_s, ks > 0);
        }
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = ((ks / 4) * (128 * 128) + (ks % 4) * 32) >> 4;
          mma_ss(tDP, do_desc + off, v_k + off, idesc_s, ks > 0);
        }
        mma_commit(&bars->sp_full);
        if (!(ok = mbar_wait(&bars->ds_ready, it & 1, p.ec, abort_flag, SITE_BWD_DS))) break;
        tc_fence_after();
        const uint64_t k_m = kv_mdesc + (uint64_t)((2 * s * Cfg::TILE) >> 4);
#pragma unroll
        for (int ks = 0; ks < BWD_BN / 16; ++ks)
          mma_ts(tDQ, tS + ks * 8, k_m + (uint64_t)((ks * 16 * 128) >> 4), idesc_dq, (it > 0 || ks > 0) ? 1u : 0u);
        mma_commit(&bars->kv_empty[s]);
      }
      mma_commit(&bars->acc_done);
      if (!ok) mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DRAIN, true);
    }
    __syncwarp();
  } else {
    // ------------------------- compute (query rows) -----------------------
    const int r = threadIdx.x;
    const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
    const uint32_t tS = tmem + lane_off, tDP = tmem + lane_off + 128;
    const int row = i * BWD_BM + r;
    const int q_abs = row + p.q_offset;
    const int64_t sidx = (int64_t)(b * p.Hq + h) * p.Sq_pad + row;
    const float lse2_r = p.lse2[sidx];
    const float delta_r = p.delta[sidx];
    const int a_lo = i * BWD_BM + p.q_offset, a_hi = min(i * BWD_BM + BWD_BM, p.Sq) - 1 + p.q_offset;
    bool ok = true;
    for (int it = 0; it < n; ++it) {
      const int j = j_lo + it;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->sp_full, it & 1, p.ec, abort_flag, SITE_BWD_SP));
      if (!ok) break;
      tc_fence_after();
      const int c0 = j * BWD_BN;
      const bool need_mask = (p.causal && c0 + BWD_BN - 1 > a_lo) || (p.window > 0 && c0 < a_hi - p.window + 1) ||
                             (c0 + BWD_BN > p.Skv);
#pragma unroll 1
      for (int cb = 0; cb < BWD_BN; cb += 32) {
        uint32_t sv[32], dpv[32];
        tmem_ld32(tS + cb, sv);
        tmem_ld32(tDP + cb, dpv);
        tmem_ld_wait32(sv);
        tmem_ld_wait32(dpv);
        uint32_t pk_ds[16];
        bwd_chunk<T, false>(p, sv, dpv, nullptr, nullptr, lse2_r, delta_r, q_abs, c0 + cb, need_mask, nullptr,
                            pk_ds);
        tmem_st16(tS + cb / 2, pk_ds);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->ds_ready);
    }
    const bool have = ok && n > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&bars->acc_done, 0, p.ec, abort_flag, SITE_BWD_DONE));
    if (have) tc_fence_after();
    const bool store = row < p.Sq;
    T* dqrow = reinterpret_cast<T*>(p.dq) + (size_t)b * p.dq_sb + (size_t)h * p.dq_sh + (size_t)row * p.dq_ss;
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      uint32_t v[32];
      if (have) {
        tmem_ld32(tmem + lane_off + 256 + c, v);
        tmem_ld_wait32(v);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0u;
      }
      uint32_t pk[16];
#pragma unroll
      for (int e = 0; e < 16; ++e)
        pk[e] = pack2<T>(__uint_as_float(v[2 * e]) * p.scale, __uint_as_float(v[2 * e + 1]) * p.scale);
      if (store) {
        uint4* dst = reinterpret_cast<uint4*>(dqrow + c);
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
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

template <typename K>
static int set_smem(K kern, int bytes) {
  return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

template <typename T, int D>
static int launch_bwd(const CUtensorMap* maps, const BwdParams& p, const void* o, const void* dout,
                      const float* lse, float* lse2, float* delta, const int64_t* o_str, const int64_t* do_str,
                      cudaStream_t st) {
  // 1. preprocess
  const int n_rows = p.B * p.Hq * p.Sq_pad;
  const int threads = 256;
  const int blocks = (n_rows * 32 + threads - 1) / threads;
  ffa_bwd_pre_kernel<T><<<blocks, threads, 0, st>>>(
      reinterpret_cast<const T*>(o), reinterpret_cast<const T*>(dout), lse, lse2, delta, p.Hq, p.Sq, p.Sq_pad, D,
      o_str[0], o_str[1], o_str[2], do_str[0], do_str[1], do_str[2], n_rows);
  int s = launch_status();
  if (s) return s;
  // 2. dK / dV
  {
    auto kern = ffa_bwd_dkdv_kernel<T, D>;
    static bool set = false;
    if (!set) {
      if ((s = set_smem(kern, DkdvCfg<D>::SMEM))) return s;
      set = true;
    }
    dim3 grid((p.Skv + BWD_BN - 1) / BWD_BN, p.B * p.Hkv);
    kern<<<grid, BWD_THREADS, DkdvCfg<D>::SMEM, st>>>(maps[0], maps[1], maps[2], maps[3], p);
    if ((s = launch_status())) return s;
  }
  // 3. dQ
  {
    auto kern = ffa_bwd_dq_kernel<T, D>;
    static bool set = false;
    if (!set) {
      if ((s = set_smem(kern, DqCfg<D>::SMEM))) return s;
      set = true;
    }
    dim3 grid((p.Sq + BWD_BM - 1) / BWD_BM, p.B * p.Hq);
    kern<<<grid, BWD_THREADS, DqCfg<D>::SMEM, st>>>(maps[0], maps[1], maps[2], maps[3], p);
    if ((s = launch_status())) return s;
  }
  return FFA_OK;
}

}  // namespace ffa

extern "C" size_t ffa_bwd_workspace_size(int B, int Hq, int Sq) {
  const size_t sq_pad = ((size_t)Sq + 127) / 128 * 128;
  return 2 * (size_t)B * Hq * sq_pad * sizeof(float) + 256;
}

extern "C" int ffa_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o,
                       const float* lse, void* dq, void* dk, void* dv, int dtype, int B, int Hq, int Hkv, int Sq,
                       int Skv, int D, const int64_t* q_strides, const int64_t* k_strides,
                       const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                       const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                       float scale, int causal, int q_offset, int window, float softcap, void* workspace,
                       size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  using namespace ffa;
  if (!dout || !q || !k || !v || !o || !lse || !dq || !dk || !dv) return FFA_ERR_INVALID_ARG;
  if (!q_strides || !k_strides || !v_strides || !o_strides || !do_strides || !dq_strides || !dk_strides ||
      !dv_strides)
    return FFA_ERR_INVALID_ARG;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Skv <= 0 || Hq % Hkv != 0) return FFA_ERR_INVALID_ARG;
  if (D != 64 && D != 128) return FFA_ERR_UNSUPPORTED;
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16) return FFA_ERR_UNSUPPORTED;
  const size_t need = ffa_bwd_workspace_size(B, Hq, Sq);
  if (!workspace || workspace_bytes < need) return FFA_ERR_WORKSPACE;
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
  p.lse2 = lse2;
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
  p.causal = causal;
  p.window = window > 0 ? window : 0;
  p.ec.err = dev_err;
  p.ec.limit_ns = wait_limit_ns();

  const CUtensorMapDataType dt =
      dtype == FFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap maps[4];
  int st = make_tmap_4d(&maps[0], q, dt, 2, D, Sq, Hq, B, q_strides[2] * 2, q_strides[1] * 2, q_strides[0] * 2, 64,
                        BWD_BM);
  if (!st)
    st = make_tmap_4d(&maps[1], k, dt, 2, D, Skv, Hkv, B, k_strides[2] * 2, k_strides[1] * 2, k_strides[0] * 2, 64,
                      BWD_BN);
  if (!st)
    st = make_tmap_4d(&maps[2], v, dt, 2, D, Skv, Hkv, B, v_strides[2] * 2, v_strides[1] * 2, v_strides[0] * 2, 64,
                      BWD_BN);
  if (!st)
    st = make_tmap_4d(&maps[3], dout, dt, 2, D, Sq, Hq, B, do_strides[2] * 2, do_strides[1] * 2, do_strides[0] * 2,
                      64, BWD_BM);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FFA_DTYPE_BF16) {
    if (D == 64) return launch_bwd<__nv_bfloat16, 64>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
    return launch_bwd<__nv_bfloat16, 128>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
  }
  if (D == 64) return launch_bwd<__half, 64>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
  return launch_bwd<__half, 128>(maps, p, o, dout, lse, lse2, delta, o_strides, do_strides, s);
}
