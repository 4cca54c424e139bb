// Prefill / training forward attention for B200 (sm_100a).
//
// Replaces the reference's forward kernels (kernels/cpu_reference.py:132
// flash_attn_cpu_forward, kernels/cpu_fa4.py:219 fa4_forward and the Triton
// kernels in kernels/triton_fwd.py / triton_ffpa.py) behind ffa_fwd().
//
// One CTA owns two 128-row query tiles of one (batch, head) and walks the key
// tiles (128 keys each) its masks leave active:
//   warp 8      TMA producer: Q once, then K_j / V_j into a ring of smem slots
//   warp 9      MMA issuer:   S_t = Q_t K_j^T (smem x smem -> TMEM),
//                             O_t += P_t V_j  (P from TMEM x V from smem)
//   warps 0-3   softmax for query tile 0, warps 4-7 for query tile 1: each
//               thread owns one query row (= one TMEM lane), reads its S row,
//               applies scale / softcap / masks, runs the online softmax in
//               base 2 and writes P (16-bit) back over S in TMEM.
// The two tiles ping-pong: while one softmax group works on its scores the
// tensor core runs the other tile's P·V and next Q·K^T.
// Rescaling of O is lazy: the running max only moves (and O in TMEM is
// rescaled) when a row's max grows by more than 2^8; the result is exact
// because numerator and denominator always share the same stale max.
// TMEM columns: [0,128) S_0/P_0, [128,256) S_1/P_1, [256,384) O_0, [384,512) O_1.
#include "ffa_common.cuh"
#include "ffa_host.h"

namespace ffa {

constexpr int FWD_BM = 128;   // rows per query tile (= TMEM lanes)
constexpr int FWD_NQT = 2;    // query tiles per CTA
constexpr int FWD_BN = 128;   // keys per key tile
constexpr int FWD_THREADS = 256;  // two softmax warpgroups; no separate TMA / MMA warps
constexpr int FWD_WARP_TMEM = 1;  // allocates / frees TMEM
constexpr int FWD_MAX_LIST = 2048;  // key tiles recorded per CTA when a block mask filters them
constexpr float RESCALE_LOG2 = 8.0f;

// D = query/key head dim, DV = value head dim (DV <= 128; D = 192 with
// DV = 128 is the MLA prefill shape: 128 "nope" + 64 rotary dims).
template <int D, int DV>
struct FwdCfg {
  static constexpr int TILE = FWD_BM * D * 2;     // one 128-row Q (or K) tile
  static constexpr int VTILE = FWD_BN * DV * 2;   // one 128-row V tile
  static constexpr int BUF = TILE > VTILE ? TILE : VTILE;  // ring slot (holds a K or a V tile)
  static constexpr int NBUF = (D == 64) ? 8 : (D == 128 ? 4 : 2);
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = FWD_NQT * TILE;
  static constexpr int BAR_OFF = KV_OFF + NBUF * BUF;
  static constexpr int LIST_OFF = BAR_OFF + 512;
  static constexpr int SMEM = LIST_OFF + FWD_MAX_LIST * 2 + 1024;  // + alignment slack
};

struct FwdParams {
  void* o;
  float* lse;
  int64_t o_sb, o_sh, o_ss;
  int B, Hq, Hkv, Sq, Skv, q_offset;
  int n_qblk;
  float scale_log2;   // scale * log2(e)
  float sc_pre;       // scale / softcap
  float sc_post;      // softcap * log2(e)
  int use_softcap;
  int causal, window;
  const uint8_t* block_mask;
  int n_br, n_bc, mask_bq, mask_bkv;
  ErrCtx ec;
};

struct FwdBars {
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done[2];
  uint64_t drain[2];
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint32_t tmem_base;
  int abort;
  int n_tiles;
  int j_lo;
  int use_list;
};

enum : uint32_t {
  SITE_FWD_Q = 0x101,
  SITE_FWD_KV_EMPTY = 0x102,
  SITE_FWD_KV_FULL = 0x103,
  SITE_FWD_P_FULL = 0x104,
  SITE_FWD_S_FULL = 0x105,
  SITE_FWD_O_DONE = 0x106,
  SITE_FWD_DRAIN = 0x107,
};

__device__ __forceinline__ bool mask_entry(const FwdParams& p, int row, int col) {
  return p.block_mask[(size_t)(row / p.mask_bq) * p.n_bc + (col / p.mask_bkv)] != 0;
}

template <typename T, int D, int DV>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    ffa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using Cfg = FwdCfg<D, DV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Cfg::Q_OFF;
  uint8_t* sKV = smem + Cfg::KV_OFF;
  FwdBars* bars = reinterpret_cast<FwdBars*>(smem + Cfg::BAR_OFF);
  uint16_t* list = reinterpret_cast<uint16_t*>(smem + Cfg::LIST_OFF);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int BH = p.B * p.Hq;
  const int bid = blockIdx.x;
  // LPT order: with causal masking the last query blocks carry the most key
  // tiles, so they are dispatched first; heads vary fastest so that the query
  // heads of one GQA group (which share K/V) run side by side.
  const int qblk = p.causal ? (p.n_qblk - 1 - bid / BH) : (bid / BH);
  const int bh = bid % BH;
  const int b = bh / p.Hq;
  const int h = bh % p.Hq;
  const int hkv = h / (p.Hq / p.Hkv);

  const int q_lo = qblk * (FWD_BM * FWD_NQT);
  const int q_hi = min(q_lo + FWD_BM * FWD_NQT, p.Sq) - 1;
  const int a_lo = q_lo + p.q_offset;
  const int a_hi = q_hi + p.q_offset;
  const int n_kv = (p.Skv + FWD_BN - 1) / FWD_BN;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], FWD_BM);
      mbar_init(&bars->o_done[t], 1);
      mbar_init(&bars->drain[t], 1);
    }
    for (int i = 0; i < Cfg::NBUF; ++i) {
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], FWD_NQT);  // released once by each query tile's issuer
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == FWD_WARP_TMEM) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  if (warp == 0) {
    // Key-tile range allowed by causal / window masks, then filtered by the
    // block mask (a tile stays if any of its (row, col) pairs is kept).
    int j_hi = n_kv;
    if (p.causal) j_hi = min(n_kv, a_hi >= 0 ? a_hi / FWD_BN + 1 : 0);
    int j_lo = 0;
    if (p.window > 0) {
      const int lo_col = a_lo - p.window + 1;
      if (lo_col > 0) j_lo = min(lo_col / FWD_BN, j_hi);
    }
    if (p.block_mask == nullptr) {
      if (lane == 0) {
        bars->j_lo = j_lo;
        bars->n_tiles = max(0, j_hi - j_lo);
        bars->use_list = 0;
      }
    } else {
      int count = 0;
      const int br_lo = q_lo / p.mask_bq, br_hi = q_hi / p.mask_bq;
      for (int j0 = j_lo; j0 < j_hi; j0 += 32) {
        const int j = j0 + lane;
        bool keep = false;
        if (j < j_hi) {
          const int bc_lo = (j * FWD_BN) / p.mask_bkv;
          const int bc_hi = min(j * FWD_BN + FWD_BN, p.Skv) - 1;
          for (int br = br_lo; br <= br_hi && !keep; ++br)
            for (int bc = bc_lo; bc <= bc_hi / p.mask_bkv && !keep; ++bc)
              keep = p.block_mask[(size_t)br * p.n_bc + bc] != 0;
        }
        const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
        const int pos = count + __popc(ballot & ((1u << lane) - 1u));
        if (keep && pos < FWD_MAX_LIST) list[pos] = (uint16_t)j;
        count += __popc(ballot);
      }
      if (lane == 0) {
        bars->j_lo = 0;
        bars->n_tiles = min(count, FWD_MAX_LIST);
        bars->use_list = 1;
        if (count > FWD_MAX_LIST && p.ec.err) atomicCAS(p.ec.err, 0u, 0x1FFu);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem = bars->tmem_base;
  const int n = bars->n_tiles;
  const int j_lo = bars->j_lo;
  const bool use_list = bars->use_list != 0;
  auto tile_at = [&](int it) -> int { return use_list ? (int)list[it] : j_lo + it; };
  constexpr uint32_t FMT = DtypeFmt<T>::value;

  const int t = warp / 4;           // query tile of this warpgroup
  const int r = threadIdx.x % FWD_BM;
  const bool issuer = (r == 0);     // issues this tile's MMAs
  const bool loader = (threadIdx.x == 0);  // also streams Q, K, V with TMA

  // ------------------------------- loader ----------------------------------
  // Thread 0 keeps the K/V ring full without ever blocking on it: `pump`
  // issues every load whose slot has been released, and every wait this
  // thread performs keeps pumping.
  const uint64_t pol_kv = policy_evict_last();
  int ld_next = 0;  // next K/V slot (2 per key tile: K then V)
  auto pump = [&]() {
    while (ld_next < 2 * n) {
      const int s = ld_next, buf = s % Cfg::NBUF, use = s / Cfg::NBUF;
      if (use > 0 && !mbar_test(&bars->kv_empty[buf], (use - 1) & 1)) break;
      const int kv = s & 1, j = tile_at(s >> 1);
      mbar_arrive_expect_tx(&bars->kv_full[buf], kv ? Cfg::VTILE : Cfg::TILE);
      uint8_t* dst = sKV + buf * Cfg::BUF;
      for (int c = 0; c < (kv ? DV : D) / 64; ++c)
        tma_load_4d(kv ? &tmV : &tmK, &bars->kv_full[buf], dst + c * (FWD_BN * 128), c * 64, j * FWD_BN, hkv, b,
                    pol_kv);
      ++ld_next;
    }
  };
  auto wait = [&](uint64_t* bar, uint32_t par, uint32_t site) -> bool {
    if (!loader) return mbar_wait(bar, par, p.ec, abort_flag, site);
    if (mbar_test(bar, par)) return true;
    const long long t0 = clock64(), limit = (long long)(p.ec.limit_ns * 2ull);
    while (true) {
      pump();
      if (mbar_test(bar, par)) return true;
      if (*abort_flag) return false;
      if (clock64() - t0 > limit) {
        *abort_flag = 1;
        if (p.ec.err) atomicCAS(p.ec.err, 0u, site);
        return false;
      }
    }
  };
  if (loader && n > 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    const uint64_t pol_q = policy_evict_first();
    mbar_arrive_expect_tx(&bars->q_full, FWD_NQT * Cfg::TILE);
    for (int tq = 0; tq < FWD_NQT; ++tq)
      for (int c = 0; c < D / 64; ++c)
        tma_load_4d(&tmQ, &bars->q_full, sQ + tq * Cfg::TILE + c * (FWD_BM * 128), c * 64, q_lo + tq * FWD_BM, h, b,
                    pol_q);
    pump();
  }

  // ------------------------------- MMA issue -------------------------------
  const uint32_t idesc_qk = make_idesc_f16(FWD_BM, FWD_BN, FMT, 0, 0);
  const uint32_t idesc_pv = make_idesc_f16(FWD_BM, DV, FMT, 0, 1);
  const uint32_t tS0 = tmem + t * 128;        // lane-0 TMEM addresses of this tile's S/P and O
  const uint32_t tO0 = tmem + 256 + t * 128;
  auto issue_qk = [&](int buf) {
    const uint64_t qa = make_sdesc_sw128(smem_u32(sQ + t * Cfg::TILE), 16, 1024);
    const uint64_t kb = make_sdesc_sw128(smem_u32(sKV + buf * Cfg::BUF), 16, 1024);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const uint32_t off = ((ks / 4) * (FWD_BM * 128) + (ks % 4) * 32) >> 4;
      mma_ss(tS0, qa + off, kb + off, idesc_qk, ks > 0);
    }
  };
  auto issue_pv = [&](int buf, bool acc) {
    const uint64_t vb = make_sdesc_sw128(smem_u32(sKV + buf * Cfg::BUF), FWD_BN * 128, 1024);
#pragma unroll
    for (int ks = 0; ks < FWD_BN / 16; ++ks)
      mma_ts(tO0, tS0 + ks * 8, vb + (uint64_t)((ks * 16 * 128) >> 4), idesc_pv, (acc || ks > 0) ? 1u : 0u);
  };
  if (issuer && n > 0) {
    if (wait(&bars->q_full, 0, SITE_FWD_Q) && wait(&bars->kv_full[0], 0, SITE_FWD_KV_FULL)) {
      tc_fence_after();
      issue_qk(0);
      mma_commit(&bars->s_full[t]);
      mma_commit(&bars->kv_empty[0]);
    }
  }
  __syncwarp();

  // -------------------------------- softmax --------------------------------
  const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
  const uint32_t tS = tmem + lane_off + t * 128;
  const uint32_t tO = tmem + lane_off + 256 + t * 128;
  const int row = q_lo + t * FWD_BM + r;
  const int arow = row + p.q_offset;
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  for (int it = 0; it < n; ++it) {
    const int j = tile_at(it);
    ok = __all_sync(0xffffffffu, wait(&bars->s_full[t], it & 1, SITE_FWD_S_FULL));
    if (!ok) break;
    tc_fence_after();
    uint32_t s[FWD_BN];
#pragma unroll
    for (int c = 0; c < FWD_BN; c += 32) tmem_ld32(tS + c, s + c);
#pragma unroll
    for (int c = 0; c < FWD_BN; c += 32) tmem_ld_wait32(s + c);
    // Scores in base-2 units: s * scale*log2(e), or with a softcap
    // softcap*tanh(s*scale/softcap)*log2(e) computed in place (then mul = 1).
    float mul = p.scale_log2;
    if (p.use_softcap) {
#pragma unroll
      for (int c = 0; c < FWD_BN; ++c)
        s[c] = __float_as_uint(tanh_acc(__uint_as_float(s[c]) * p.sc_pre) * p.sc_post);
      mul = 1.f;
    }
    const int c0 = j * FWD_BN;
    const bool need_mask = (p.causal && c0 + FWD_BN - 1 > a_lo) || (p.window > 0 && c0 < a_hi - p.window + 1) ||
                           (c0 + FWD_BN > p.Skv) || (p.block_mask != nullptr);
    if (need_mask) {
      // Visible keys of this row form one range [lo, hi] (causal / window /
      // sequence end); one unsigned compare per element, no branches.
      const int hi = min(p.causal ? arow : 0x7ffffffe, p.Skv - 1) - c0;
      const int lo_c = p.window > 0 ? max(arow - p.window + 1 - c0, 0) : 0;
      const uint32_t span = hi >= lo_c ? (uint32_t)(hi - lo_c) : 0xffffffffu;
      const uint32_t ninf = __float_as_uint(-INFINITY);
#pragma unroll
      for (int c = 0; c < FWD_BN; ++c) {
        const bool keep = span != 0xffffffffu && (uint32_t)(c - lo_c) <= span;
        s[c] = keep ? s[c] : ninf;
      }
      if (p.block_mask != nullptr) {
        // Column keep-bits of this row from the block mask (a runtime loop over
        // the mask blocks the tile touches), then applied with an unrolled
        // bit test so s[] stays in registers.
        const uint8_t* mrow = p.block_mask + (size_t)(min(row, p.Sq - 1) / p.mask_bq) * p.n_bc;
        uint32_t kb[4] = {~0u, ~0u, ~0u, ~0u};
#pragma unroll 1
        for (int bc = c0 / p.mask_bkv; bc * p.mask_bkv < c0 + FWD_BN && bc < p.n_bc; ++bc) {
          if (mrow[bc]) continue;
          const int clo = max(bc * p.mask_bkv - c0, 0), chi = min((bc + 1) * p.mask_bkv - c0, FWD_BN);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const int a = max(clo, 32 * w), e = min(chi, 32 * w + 32);
            if (a < e) {
              const uint32_t len = e - a;
              const uint32_t bits = (len == 32 ? ~0u : ((1u << len) - 1u)) << (a - 32 * w);
              kb[w] &= ~bits;
            }
          }
        }
#pragma unroll
        for (int c = 0; c < FWD_BN; ++c) s[c] = ((kb[c / 32] >> (c % 32)) & 1u) ? s[c] : ninf;
      }
    }
    // Row max: eight independent 3-input max chains, then a small tree.
    float mx[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mx[i] = __uint_as_float(s[i]);
#pragma unroll
    for (int c = 8; c < FWD_BN; c += 16)
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], __uint_as_float(s[c + i]), __uint_as_float(s[c + 8 + i]));
    const float mraw = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
    const float m_new = fmaxf(m, mraw * mul);
    const bool warp_resc = __any_sync(0xffffffffu, m_new > m + RESCALE_LOG2);
    float alpha = 1.f;
    if (warp_resc) {
      alpha = (m_new == -INFINITY) ? 1.f : ex2(m - m_new);
      l *= alpha;
      m = m_new;
    }
    // O must carry the new max before this tile's P.V accumulates into it.
    // P.V of the previous tile was issued before this tile's Q.K^T by the same
    // thread, so it retired before S became ready: the wait is immediate.
    if (warp_resc && it > 0) {
      ok = __all_sync(0xffffffffu, wait(&bars->o_done[t], (it - 1) & 1, SITE_FWD_O_DONE));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < DV; c += 32) {
        uint32_t ov[32];
        tmem_ld32(tO + c, ov);
        tmem_ld_wait32(ov);
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
        tmem_st32(tO + c, ov);
      }
    }
    const float mu = (m == -INFINITY) ? 0.f : m;
    const float2 mul2 = make_float2(mul, mul);
    const float2 nmu2 = make_float2(-mu, -mu);
    // p = 2^(s*mul - mu), packed to 16-bit pairs and written over S in TMEM.
    float2 acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);
    uint32_t pk[FWD_BN / 2];
#pragma unroll
    for (int c = 0; c < FWD_BN / 2; ++c) {
      const float2 a = ffma2(make_float2(__uint_as_float(s[2 * c]), __uint_as_float(s[2 * c + 1])), mul2, nmu2);
      float2 pv;
      pv.x = ex2(a.x);
      pv.y = ex2(a.y);
      acc[c & 3] = fadd2(acc[c & 3], pv);
      pk[c] = pack2<T>(pv.x, pv.y);
    }
    const float2 acct = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
    l += acct.x + acct.y;
    tmem_st32(tS, pk);
    tmem_st32(tS + 32, pk + 32);
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive(&bars->p_full[t]);
    // The issuer waits for the whole group's P, then issues P.V for this tile
    // and Q.K^T for the next (which overwrites S/P: the tensor core executes
    // one thread's MMAs in issue order).
    if (issuer) {
      const int vs = 2 * it + 1, vb = vs % Cfg::NBUF;
      if (wait(&bars->p_full[t], it & 1, SITE_FWD_P_FULL) &&
          wait(&bars->kv_full[vb], (vs / Cfg::NBUF) & 1, SITE_FWD_KV_FULL)) {
        tc_fence_after();
        issue_pv(vb, it > 0);
        mma_commit(&bars->o_done[t]);
        mma_commit(&bars->kv_empty[vb]);
        if (it + 1 < n) {
          const int ks_ = 2 * (it + 1), kb = ks_ % Cfg::NBUF;
          if (wait(&bars->kv_full[kb], (ks_ / Cfg::NBUF) & 1, SITE_FWD_KV_FULL)) {
            tc_fence_after();
            issue_qk(kb);
            mma_commit(&bars->s_full[t]);
            mma_commit(&bars->kv_empty[kb]);
          }
        }
      }
    }
    if (loader) pump();
    __syncwarp();
  }
  if (issuer) {
    // Every MMA of this tile retires before TMEM is released.
    mma_commit(&bars->drain[t]);
    mbar_wait(&bars->drain[t], 0, p.ec, abort_flag, SITE_FWD_DRAIN, true);
  }
  if (loader && *abort_flag) {
    // Let copies still in flight land before the CTA gives up its smem.
    if (n > 0) mbar_wait(&bars->q_full, 0, p.ec, abort_flag, SITE_FWD_DRAIN, true);
    for (int s2 = max(0, ld_next - Cfg::NBUF); s2 < ld_next; ++s2)
      mbar_wait(&bars->kv_full[s2 % Cfg::NBUF], (s2 / Cfg::NBUF) & 1, p.ec, abort_flag, SITE_FWD_DRAIN, true);
  }
  __syncwarp();
  // ------------------------------ epilogue --------------------------------
  const bool have_o = ok && n > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&bars->o_done[t], (n - 1) & 1, p.ec, abort_flag, SITE_FWD_O_DONE));
  if (have_o) tc_fence_after();
  const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
  T* orow = reinterpret_cast<T*>(p.o) + (size_t)b * p.o_sb + (size_t)h * p.o_sh + (size_t)row * p.o_ss;
  const bool store = row < p.Sq;
#pragma unroll
  for (int c = 0; c < DV; c += 32) {
    uint32_t ov[32];
    if (have_o) {
      tmem_ld32(tO + c, ov);
      tmem_ld_wait32(ov);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) ov[e] = 0u;
    }
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 16; ++e)
      pk[e] = pack2<T>(__uint_as_float(ov[2 * e]) * inv_l, __uint_as_float(ov[2 * e + 1]) * inv_l);
    if (store) {
      uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
    }
  }
  if (store && p.lse != nullptr) {
    const float mu = (m == -INFINITY) ? 0.f : m;
    const float lse = (l > 0.f) ? (mu + lg2(l)) * 0.6931471805599453f : -INFINITY;
    p.lse[((size_t)b * p.Hq + h) * p.Sq + row] = lse;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == FWD_WARP_TMEM) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename T, int D, int DV>
static int launch_fwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FwdParams& p,
                      int grid, cudaStream_t stream) {
  using Cfg = FwdCfg<D, DV>;
  auto kern = ffa_fwd_kernel<T, D, DV>;
  static bool attr_set = false;
  if (!attr_set) {
    int st = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    if (st) return st;
    attr_set = true;
  }
  kern<<<grid, FWD_THREADS, Cfg::SMEM, stream>>>(mq, mk, mv, p);
  return launch_status();
}

}  // namespace ffa

extern "C" int ffa_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int dtype, int B,
                       int Hq, int Hkv, int Sq, int Skv, int D, int Dv, const int64_t* q_strides,
                       const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides, float scale,
                       int causal, int q_offset, int window, float softcap, const uint8_t* block_mask, int n_br,
                       int n_bc, int mask_bq, int mask_bkv, uint32_t* dev_err, void* stream) {
  using namespace ffa;
  if (!q || !k || !v || !o || !q_strides || !k_strides || !v_strides || !o_strides) return FFA_ERR_INVALID_ARG;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Skv < 0 || Hq % Hkv != 0) return FFA_ERR_INVALID_ARG;
  if (!((D == 64 && Dv == 64) || (D == 128 && Dv == 128) || (D == 192 && Dv == 128))) return FFA_ERR_UNSUPPORTED;
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16) return FFA_ERR_UNSUPPORTED;
  if (Skv > 65535 * FWD_BN) return FFA_ERR_UNSUPPORTED;
  if (block_mask && (n_br <= 0 || n_bc <= 0 || mask_bq <= 0 || mask_bkv <= 0 ||
                     (int64_t)n_br * mask_bq < Sq || (int64_t)n_bc * mask_bkv < Skv))
    return FFA_ERR_INVALID_ARG;
  if (!aligned16(o) || (o_strides[2] % 8) || (o_strides[1] % 8) || (o_strides[0] % 8)) return FFA_ERR_INVALID_ARG;

  FwdParams p{};
  p.o = o;
  p.lse = lse;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Sq = Sq;
  p.Skv = Skv;
  p.q_offset = q_offset;
  p.n_qblk = (Sq + FWD_BM * FWD_NQT - 1) / (FWD_BM * FWD_NQT);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.use_softcap = softcap > 0.f;
  p.sc_pre = p.use_softcap ? scale / softcap : 0.f;
  p.sc_post = p.use_softcap ? softcap * 1.4426950408889634f : 0.f;
  p.causal = causal;
  p.window = window > 0 ? window : 0;
  p.block_mask = block_mask;
  p.n_br = n_br;
  p.n_bc = n_bc;
  p.mask_bq = mask_bq;
  p.mask_bkv = mask_bkv;
  p.ec.err = dev_err;
  p.ec.limit_ns = wait_limit_ns();

  const CUtensorMapDataType dt =
      dtype == FFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv;
  const int skv_map = Skv > 0 ? Skv : 1;
  int st = make_tmap_4d(&mq, q, dt, 2, D, Sq, Hq, B, q_strides[2] * 2, q_strides[1] * 2, q_strides[0] * 2, 64,
                        FWD_BM);
  if (!st)
    st = make_tmap_4d(&mk, k, dt, 2, D, skv_map, Hkv, B, k_strides[2] * 2, k_strides[1] * 2, k_strides[0] * 2, 64,
                      FWD_BN);
  if (!st)
    st = make_tmap_4d(&mv, v, dt, 2, Dv, skv_map, Hkv, B, v_strides[2] * 2, v_strides[1] * 2, v_strides[0] * 2, 64,
                      FWD_BN);
  if (st) return st;

  const long long grid = (long long)p.n_qblk * B * Hq;
  if (grid > 0x7fffffffLL) return FFA_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FFA_DTYPE_BF16) {
    if (D == 64) return launch_fwd<__nv_bfloat16, 64, 64>(mq, mk, mv, p, (int)grid, s);
    if (D == 128) return launch_fwd<__nv_bfloat16, 128, 128>(mq, mk, mv, p, (int)grid, s);
    return launch_fwd<__nv_bfloat16, 192, 128>(mq, mk, mv, p, (int)grid, s);
  }
  if (D == 64) return launch_fwd<__half, 64, 64>(mq, mk, mv, p, (int)grid, s);
  if (D == 128) return launch_fwd<__half, 128, 128>(mq, mk, mv, p, (int)grid, s);
  return launch_fwd<__half, 192, 128>(mq, mk, mv, p, (int)grid, s);
}
