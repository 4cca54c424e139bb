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

#include <cstdlib>

namespace ffa {

constexpr int FWD_BM = 128;   // rows per query tile (= TMEM lanes)
constexpr int FWD_BN = 128;   // keys per key tile
#ifndef FFA_FWD_NQT1_MAX_COLS
#define FFA_FWD_NQT1_MAX_COLS 2048
#endif
constexpr long long FWD_NQT1_MAX_COLS = FFA_FWD_NQT1_MAX_COLS;  // rows this short use one query tile per CTA

// CTA shapes.  NQT = 2 (one CTA per SM): two query tiles whose softmax groups
// ping-pong inside the CTA.  NQT = 1 (two CTAs per SM, each half the TMEM
// and under half the shared memory): one query tile per CTA, and the two
// resident CTAs interleave on the SM's tensor core the way the two groups of
// an NQT = 2 CTA do, while one CTA's set-up (barriers, TMEM, the first Q / K
// loads) and epilogue overlap the other's main loop.  That matters when a CTA
// walks few key tiles (sliding windows, short rows), where set-up and
// epilogue are a large share of a CTA's time.
template <int NQT>
struct FwdShape;
template <>
struct FwdShape<2> {
  static constexpr int THREADS = 384;  // 2 softmax warpgroups + 1 warpgroup for TMA / MMA (2 warps idle)
  static constexpr int MIN_BLOCKS = 1;
  // Register budgets after the split: 2 x 128 x 200 + 128 x 104 = 384 x 168 (the launch allocation).
  // (208 / 88 spilled more in the TMA / MMA warps: config 2 2.06 -> 1.98-2.01 ms with 200 / 104.)
  static constexpr uint32_t REGS_SOFTMAX = 200, REGS_OTHER = 104;
  static constexpr int TMEM_COLS = 512;
};
template <>
struct FwdShape<1> {
  static constexpr int THREADS = 256;  // 1 softmax warpgroup + 1 warpgroup for TMA / MMA (2 warps idle)
  static constexpr int MIN_BLOCKS = 2;
  // 128 x 200 + 128 x 56 = 256 x 128 (the launch allocation at two CTAs per SM).
  static constexpr uint32_t REGS_SOFTMAX = 200, REGS_OTHER = 56;
  static constexpr int TMEM_COLS = 256;
};
constexpr int FWD_MAX_LIST = 2048;  // key tiles recorded per CTA when a block mask filters them
constexpr float RESCALE_LOG2 = 8.0f;
#ifndef FFA_FWD_PCH
#define FFA_FWD_PCH 2
#endif
constexpr int FWD_PCH = FFA_FWD_PCH;  // P is handed to the MMA warp in FWD_PCH chunks of 128 / FWD_PCH keys (2: each
// hand-over costs the MMA warp a barrier wait, and fewer waits measured faster)

// D = query/key head dim, DV = value head dim (DV <= 128; D = 192 with
// DV = 128 is the MLA prefill shape: 128 "nope" + 64 rotary dims).
template <int D, int DV, int NQT = 2>
struct FwdCfg {
  static constexpr int TILE = FWD_BM * D * 2;     // one 128-row Q (or K) tile
  static constexpr int VTILE = FWD_BN * DV * 2;   // one 128-row V tile
  // D <= 128: one ring of NBUF equal slots, K and V of each key tile in turn,
  // fed by one producer warp.  D = 192: the two Q tiles take 96 KB, which
  // leaves room for one K and one V slot of a shared ring; instead K and V
  // get rings of their own (two 48 KB K slots, one 32 KB V slot), each fed by
  // its own producer warp, so the next-but-one K tile loads a whole key tile
  // ahead (config 5 prefill 3.61 -> 3.26 ms).
  static constexpr bool SPLIT = NQT == 2 && D == 192;
  static constexpr int BUF = TILE > VTILE ? TILE : VTILE;  // shared-ring slot (holds a K or a V tile)
  static constexpr int NBUF = NQT == 2 ? ((D == 64) ? 8 : (D == 128 ? 4 : 2)) : (D == 64 ? 4 : 2);
  static constexpr int NK = 2, NV = 1;  // SPLIT: K slots (barriers [0, NK)), V slots (barriers [4, 4 + NV))
  // key tiles recorded per CTA when a block mask filters them (D = 192: what
  // the shared memory left over holds)
  static constexpr int MAX_LIST = SPLIT ? 512 : FWD_MAX_LIST;
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = NQT * TILE;                           // shared ring, or the K ring
  static constexpr int V_OFF = SPLIT ? KV_OFF + NK * TILE : KV_OFF;   // the V ring
  static constexpr int BAR_OFF = SPLIT ? V_OFF + NV * VTILE : KV_OFF + NBUF * BUF;
  static constexpr int LIST_OFF = BAR_OFF + 512;
  static constexpr int SMEM = LIST_OFF + MAX_LIST * 2 + 1024;  // + alignment slack
  static_assert(SMEM <= 227 * 1024, "forward shared memory budget");
};

struct FwdParams {
  void* o;
  float* lse;
  int64_t o_sb, o_sh, o_ss;
  int B, Hq, Hkv, Sq, Skv, q_offset;
  int n_qblk;
  int head_group;     // (b, h) pairs per CTA-order group (see the kernel's block mapping)
  float scale_log2;   // scale * log2(e)
  float sc_pre;       // scale / softcap
  float sc_post;      // softcap * log2(e)
  float sc_poly[3];   // softcap_small2 coefficients for k = sc_pre
  int use_softcap;
  int causal, window;
  const uint8_t* block_mask;
  int n_br, n_bc, mask_bq, mask_bkv;
  ErrCtx ec;
};

struct FwdBars {
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t p_full[2][FWD_PCH];
  uint64_t o_done[2];
  uint64_t drain;
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


template <typename T, int D, int DV, int NQT>
__global__ void __launch_bounds__(FwdShape<NQT>::THREADS, FwdShape<NQT>::MIN_BLOCKS)
    ffa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using Cfg = FwdCfg<D, DV, NQT>;
  using Shape = FwdShape<NQT>;
  constexpr int FWD_NQT = NQT;
  constexpr int FWD_WARP_LOAD = 4 * NQT;     // the warpgroup after the softmax groups
  constexpr int FWD_WARP_MMA = 4 * NQT + 1;
  constexpr uint32_t O_COL = NQT * 128;      // TMEM: S_t/P_t at [128 t, ...), O_t at O_COL + 128 t
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Cfg::Q_OFF;
  uint8_t* sKV = smem + Cfg::KV_OFF;
  uint8_t* sV = smem + Cfg::V_OFF;
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
  // Heads are taken in groups of p.head_group (consecutive (b, h), so a GQA
  // group's query heads stay together) whose K/V fit in L2 together; within a
  // group, query blocks go heaviest first.
  const int gsz = p.head_group;
  const int grp = bid / (gsz * p.n_qblk);
  const int g0 = grp * gsz;
  const int gn = min(gsz, BH - g0);  // heads in this (possibly last, smaller) group
  const int rem = bid - g0 * p.n_qblk;
  const int qblk = p.causal ? (p.n_qblk - 1 - rem / gn) : (rem / gn);
  const int bh = g0 + rem % gn;
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
    for (int t = 0; t < NQT; ++t) {
      mbar_init(&bars->s_full[t], 1);
      for (int k = 0; k < FWD_PCH; ++k) mbar_init(&bars->p_full[t][k], FWD_BM / 32);  // one arrival per warp
      mbar_init(&bars->o_done[t], 1);
    }
    mbar_init(&bars->drain, 1);
    for (int i = 0; i < 8; ++i) {  // shared ring [0, NBUF); split rings: K [0, NK), V [4, 4 + NV)
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == FWD_WARP_MMA) {
    tmem_alloc(&bars->tmem_base, Shape::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == FWD_WARP_LOAD) {
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
        if (keep && pos < Cfg::MAX_LIST) list[pos] = (uint16_t)j;
        count += __popc(ballot);
      }
      if (lane == 0) {
        bars->j_lo = 0;
        bars->n_tiles = min(count, Cfg::MAX_LIST);
        bars->use_list = 1;
        if (count > Cfg::MAX_LIST && p.ec.err) atomicCAS(p.ec.err, 0u, 0x1FFu);
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

  if (warp >= 4 * NQT) {
   regs_dec<Shape::REGS_OTHER>();
   if (Cfg::SPLIT && (warp == FWD_WARP_LOAD || warp == FWD_WARP_LOAD + 2)) {
    // --------------------------- split-ring producers -----------------------
    // warp FWD_WARP_LOAD: Q, then the K ring; warp FWD_WARP_LOAD + 2: the V ring.
    if (lane == 0) {
      const bool is_v = warp != FWD_WARP_LOAD;
      const CUtensorMap* tm = is_v ? &tmV : &tmK;
      tma_prefetch_desc(tm);
      const uint64_t pol_kv = policy_evict_last();
      if (!is_v) {
        tma_prefetch_desc(&tmQ);
        const uint64_t pol_q = policy_evict_first();
        mbar_arrive_expect_tx(&bars->q_full, FWD_NQT * Cfg::TILE);
        for (int t = 0; t < FWD_NQT; ++t)
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(&tmQ, &bars->q_full, sQ + t * Cfg::TILE + c * (FWD_BM * 128), c * 64, q_lo + t * FWD_BM,
                        h, b, pol_q);
      }
      const int nslot = is_v ? Cfg::NV : Cfg::NK;
      const int bar0 = is_v ? 4 : 0;
      const int bytes = is_v ? Cfg::VTILE : Cfg::TILE;
      uint8_t* ring = is_v ? sV : sKV;
      int issued = 0;  // slots armed so far
      for (int it = 0; it < n; ++it) {
        const int j = tile_at(it);
        const int buf = it % nslot, use = it / nslot;
        if (use > 0 &&
            !mbar_wait(&bars->kv_empty[bar0 + buf], (use - 1) & 1, p.ec, abort_flag, SITE_FWD_KV_EMPTY))
          break;
        mbar_arrive_expect_tx(&bars->kv_full[bar0 + buf], bytes);
        ++issued;
        uint8_t* dst = ring + buf * bytes;
        for (int c = 0; c < (is_v ? DV : D) / 64; ++c)
          tma_load_4d(tm, &bars->kv_full[bar0 + buf], dst + c * (FWD_BN * 128), c * 64, j * FWD_BN, hkv, b, pol_kv);
      }
      if (*abort_flag) {
        // Let copies still in flight land before the CTA gives up its smem.
        if (!is_v) mbar_wait(&bars->q_full, 0, p.ec, abort_flag, SITE_FWD_DRAIN, true);
        for (int s = max(0, issued - nslot); s < issued; ++s)
          mbar_wait(&bars->kv_full[bar0 + s % nslot], (s / nslot) & 1, p.ec, abort_flag, SITE_FWD_DRAIN, true);
      }
    }
    __syncwarp();
   } else if (!Cfg::SPLIT && warp == FWD_WARP_LOAD) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();
      mbar_arrive_expect_tx(&bars->q_full, FWD_NQT * Cfg::TILE);
      for (int t = 0; t < FWD_NQT; ++t)
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(&tmQ, &bars->q_full, sQ + t * Cfg::TILE + c * (FWD_BM * 128), c * 64, q_lo + t * FWD_BM,
                      h, b, pol_q);
      int issued = 0;  // key/value slots armed so far
      for (int it = 0; it < n; ++it) {
        const int j = tile_at(it);
        bool ok = true;
        for (int kv = 0; kv < 2 && ok; ++kv) {
          const int s = 2 * it + kv;
          const int buf = s % Cfg::NBUF;
          const int use = s / Cfg::NBUF;
          if (use > 0 && !mbar_wait(&bars->kv_empty[buf], (use - 1) & 1, p.ec, abort_flag, SITE_FWD_KV_EMPTY)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->kv_full[buf], kv ? Cfg::VTILE : Cfg::TILE);
          ++issued;
          uint8_t* dst = sKV + buf * Cfg::BUF;
          for (int c = 0; c < (kv ? DV : D) / 64; ++c)
            tma_load_4d(kv ? &tmV : &tmK, &bars->kv_full[buf], dst + c * (FWD_BN * 128), c * 64, j * FWD_BN,
                        hkv, b, pol_kv);
        }
        if (!ok) break;
      }
      if (*abort_flag) {
        // Let copies still in flight land before the CTA gives up its smem.
        mbar_wait(&bars->q_full, 0, p.ec, abort_flag, SITE_FWD_DRAIN, true);
        for (int s = max(0, issued - Cfg::NBUF); s < issued; ++s)
          mbar_wait(&bars->kv_full[s % Cfg::NBUF], (s / Cfg::NBUF) & 1, p.ec, abort_flag, SITE_FWD_DRAIN, true);
      }
    }
    __syncwarp();
  } else if (warp == FWD_WARP_MMA) {
    // ---------------------------- MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc_qk = make_idesc_f16(FWD_BM, FWD_BN, FMT, 0, 0);
      const uint32_t idesc_pv = make_idesc_f16(FWD_BM, DV, FMT, 0, 1);
      // Descriptors are built once; every MMA then only adds a constant
      // (address >> 4) offset to the low bits, keeping this single issuing
      // thread's instruction count (and so its issue-slot needs) minimal.
      const uint64_t q_base = make_sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_base = make_sdesc_sw128(smem_u32(sKV), 16, 1024);
      const uint64_t v_base = make_sdesc_sw128(smem_u32(sV), FWD_BN * 128, 1024);
      constexpr int KSLOT = Cfg::SPLIT ? Cfg::TILE : Cfg::BUF, VSLOT = Cfg::SPLIT ? Cfg::VTILE : Cfg::BUF;
      auto issue_qk = [&](int t, int buf) {
        const uint32_t d = tmem + t * 128;
        const uint64_t qa = q_base + (uint64_t)((t * Cfg::TILE) >> 4);
        const uint64_t kb = k_base + (uint64_t)((buf * KSLOT) >> 4);
        // Fully unrolled at D <= 128; at D = 192 a full unroll of the 12 k-steps
        // made the issuing warp spill (184-byte stack frame) and ran ~2 % slower.
#pragma unroll(D > 128 ? 4 : D / 16)
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = ((ks / 4) * (FWD_BM * 128) + (ks % 4) * 32) >> 4;
          mma_ss(d, qa + off, kb + off, idesc_qk, ks > 0);
        }
      };
      // P·V for one chunk of keys (k-steps of 16 keys); chunks are issued as
      // the softmax group releases them.
      auto issue_pv = [&](int t, int buf, bool acc, int chunk) {
        const uint32_t d = tmem + O_COL + t * 128;
        const uint32_t a = tmem + t * 128;
        const uint64_t vb = v_base + (uint64_t)((buf * VSLOT) >> 4);
        constexpr int KS_PER = FWD_BN / 16 / FWD_PCH;
#pragma unroll
        for (int kk = 0; kk < KS_PER; ++kk) {
          const int ks = chunk * KS_PER + kk;
          mma_ts(d, a + ks * 8, vb + (uint64_t)((ks * 16 * 128) >> 4), idesc_pv, (acc || ks > 0) ? 1u : 0u);
        }
      };
      bool ok = n == 0 || mbar_wait_mma(&bars->q_full, 0, p.ec, abort_flag, SITE_FWD_Q);
      if (ok && n > 0) {
        ok = mbar_wait_mma(&bars->kv_full[0], 0, p.ec, abort_flag, SITE_FWD_KV_FULL);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < NQT; ++t) {
            issue_qk(t, 0);
            mma_commit(&bars->s_full[t]);
          }
          mma_commit(&bars->kv_empty[0]);
        }
      }
      for (int it = 0; it < n && ok; ++it) {
        // slot (vb: V of tile it, kb: K of tile it + 1), its barrier and phase
        int vb, kb, vbar, kbar;
        uint32_t vph, kph;
        if constexpr (Cfg::SPLIT) {
          vb = it % Cfg::NV, kb = (it + 1) % Cfg::NK;
          vbar = 4 + vb, kbar = kb;
          vph = (it / Cfg::NV) & 1, kph = ((it + 1) / Cfg::NK) & 1;
        } else {
          const int vs = 2 * it + 1, ks_ = 2 * (it + 1);
          vb = vbar = vs % Cfg::NBUF, kb = kbar = ks_ % Cfg::NBUF;
          vph = (vs / Cfg::NBUF) & 1, kph = (ks_ / Cfg::NBUF) & 1;
        }
        const bool has_next = it + 1 < n;
        if (!mbar_wait_mma(&bars->kv_full[vbar], vph, p.ec, abort_flag, SITE_FWD_KV_FULL)) break;
        for (int t = 0; t < FWD_NQT && ok; ++t) {
          for (int k = 0; k < FWD_PCH; ++k) {
            if (!mbar_wait_mma(&bars->p_full[t][k], it & 1, p.ec, abort_flag, SITE_FWD_P_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, vb, it > 0, k);
          }
          if (!ok) break;
          mma_commit(&bars->o_done[t]);
          // With two slots or a V ring of one, V of tile it is released as soon
          // as the last query tile's P·V retires (before the next S), so its
          // refill starts earlier; deeper shared rings release it below.
          if ((Cfg::SPLIT || Cfg::NBUF == 2) && t == FWD_NQT - 1) mma_commit(&bars->kv_empty[vbar]);
          if (has_next) {
            if (t == 0 && !mbar_wait_mma(&bars->kv_full[kbar], kph, p.ec, abort_flag, SITE_FWD_KV_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk(t, kb);
            mma_commit(&bars->s_full[t]);
          }
        }
        if (!ok) break;
        if (!(Cfg::SPLIT || Cfg::NBUF == 2)) mma_commit(&bars->kv_empty[vbar]);
        if (has_next) mma_commit(&bars->kv_empty[kbar]);
      }
      // Every MMA must retire before TMEM is released.
      mma_commit(&bars->drain);
      mbar_wait_mma(&bars->drain, 0, p.ec, abort_flag, SITE_FWD_DRAIN, true);
    }
    __syncwarp();
   }
  } else {
    regs_inc<Shape::REGS_SOFTMAX>();
    // ------------------------------ softmax -------------------------------
    const int t = warp / 4;
    const int r = threadIdx.x % FWD_BM;
    const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + O_COL + t * 128;
    const int row = q_lo + t * FWD_BM + r;
    const int arow = row + p.q_offset;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int it = 0; it < n; ++it) {
      const int j = tile_at(it);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[t], it & 1, p.ec, abort_flag, SITE_FWD_S_FULL));
      if (!ok) break;
      tc_fence_after();
      uint32_t s[FWD_BN];
#pragma unroll
      for (int c = 0; c < FWD_BN; c += 32) tmem_ld32(tS + c, s + c);
#pragma unroll
      for (int c = 0; c < FWD_BN; c += 32) tmem_ld_wait32(s + c);
      // Scores in base-2 units are  s * mul  (mul = scale*log2 e), or, with a
      // softcap, tanh(s*scale/softcap) computed in place (mul = softcap*log2 e).
      float mul = p.scale_log2;
      if (p.use_softcap) {
        // tanh(s*scale/softcap): the FMA-pipe polynomial when every argument
        // of the warp's tile is within 1/2 (the usual case, softcap >> scores;
        // s becomes y with tanh = k y, and the exponent keeps mul =
        // scale*log2 e), else the exact exp-based form (two MUFU ops per
        // score, mul = softcap*log2 e).
        float amax = 0.f;
#pragma unroll
        for (int c = 0; c < FWD_BN; c += 2)
          amax = fmax3(amax, fabsf(__uint_as_float(s[c])), fabsf(__uint_as_float(s[c + 1])));
        if (__all_sync(0xffffffffu, amax * fabsf(p.sc_pre) <= 0.5f)) {
          // pairs with packed instructions (per lane the same operations)
#pragma unroll
          for (int c = 0; c < FWD_BN; c += 2) {
            const float2 y = softcap_small2(make_float2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])),
                                            p.sc_poly[0], p.sc_poly[1], p.sc_poly[2]);
            s[c] = __float_as_uint(y.x);
            s[c + 1] = __float_as_uint(y.y);
          }
        } else {
#pragma unroll
          for (int c = 0; c < FWD_BN; ++c)
            s[c] = __float_as_uint(tanh_acc(__uint_as_float(s[c]) * p.sc_pre));
          mul = p.sc_post;  // softcap*log2(e) > 0: applied in the exponent's FMA
        }
      }
      const int c0 = j * FWD_BN;
      const bool need_mask = (p.causal && c0 + FWD_BN - 1 > a_lo) ||
                             (p.window > 0 && c0 < a_hi - p.window + 1) || (c0 + FWD_BN > p.Skv) ||
                             (p.block_mask != nullptr);
      if (need_mask) {
        // Visible keys of this row form one range [lo_c, hi] (causal, window
        // and sequence end): one unsigned compare per element, no branches.
        // (A branchy per-element form made the compiler keep s[] in local
        // memory and ran ~30x slower on these diagonal tiles.)
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
          // Column keep-bits of this row from the block mask (a runtime loop
          // over the mask blocks the tile touches), applied with an unrolled
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
                kb[w] &= ~((len == 32 ? ~0u : ((1u << len) - 1u)) << (a - 32 * w));
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
      // O must carry the new max before this tile's P·V accumulates into it.
      // P·V of the previous tile retired before this tile's S was produced
      // (the tensor core runs in issue order), so the wait below is immediate.
      if (warp_resc && it > 0) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&bars->o_done[t], (it - 1) & 1, p.ec, abort_flag, SITE_FWD_O_DONE));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < DV; c += 32) {
          uint32_t ov[32];
          tmem_ld32(tO + c, ov);
          tmem_ld_wait32(ov);
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 v = fmul2(make_float2(__uint_as_float(ov[e]), __uint_as_float(ov[e + 1])), f2(alpha));
            ov[e] = __float_as_uint(v.x);
            ov[e + 1] = __float_as_uint(v.y);
          }
          tmem_st32(tO + c, ov);
        }
      }
      const float mu = (m == -INFINITY) ? 0.f : m;
      const float2 mul2 = make_float2(mul, mul);
      const float2 nmu2 = make_float2(-mu, -mu);
      // p = 2^(s*mul - mu), written over S as 16-bit pairs one 32-key chunk at
      // a time; each chunk is released to the MMA warp as soon as it is in
      // TMEM so P·V overlaps the rest of the exponentials.
      float2 acc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < FWD_PCH; ++k) {
#pragma unroll
        for (int g = 0; g < 4 / FWD_PCH; ++g) {  // 16 packed pairs (32 keys) per group
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int c = (k * (4 / FWD_PCH) + g) * 16 + e;
            const float2 a =
                ffma2(make_float2(__uint_as_float(s[2 * c]), __uint_as_float(s[2 * c + 1])), mul2, nmu2);
            float2 pv;
            pv.x = ex2(a.x);
            pv.y = ex2(a.y);
            acc[e & 3] = fadd2(acc[e & 3], pv);
            pk[e] = pack2<T>(pv.x, pv.y);
          }
          tmem_st16(tS + (k * (4 / FWD_PCH) + g) * 16, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[t][k]);
      }
      const float2 acct = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
      l += acct.x + acct.y;
    }
    // ------------------------------ epilogue ------------------------------
    const bool have_o =
        ok && n > 0 &&
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
      for (int e = 0; e < 16; ++e) {
        const float2 v = fmul2(make_float2(__uint_as_float(ov[2 * e]), __uint_as_float(ov[2 * e + 1])), f2(inv_l));
        pk[e] = pack2<T>(v.x, v.y);
      }
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
  }

  tc_fence_before();
  __syncthreads();
  if (warp == FWD_WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, Shape::TMEM_COLS);
  }
}

template <typename T, int D, int DV, int NQT>
static int launch_fwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FwdParams& p,
                      int grid, cudaStream_t stream) {
  using Cfg = FwdCfg<D, DV, NQT>;
  auto kern = ffa_fwd_kernel<T, D, DV, NQT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int st = smem_attr_once(kern, Cfg::SMEM, attr_done)) return st;
  kern<<<grid, FwdShape<NQT>::THREADS, Cfg::SMEM, stream>>>(mq, mk, mv, p);
  return launch_status();
}

// CTAs walk (b, h) pairs in groups whose K/V fit in L2 together (about
// 48 MB, a good part of the 126 MB L2, the rest left to the streaming Q and O),
// so that the query blocks of a head find its K/V tiles in L2 instead of
// refetching them from HBM; whole GQA groups per group.  FFA_FWD_HEAD_GROUP in
// the environment overrides the group size (for measurements; 0 = all heads
// in one group, the plain heaviest-first order).
static int fwd_head_group(int BH, int G, int Skv, int D, int Dv, int window, long long ctas) {
  static const int forced = [] {
    const char* e = getenv("FFA_FWD_HEAD_GROUP");
    return e ? atoi(e) : -1;
  }();
  if (forced == 0) return BH;
  if (forced > 0) return forced;
  // Under a sliding window a query block reads only its window's keys, which
  // the same query block of every head together keeps within L2: the plain
  // order (measured 0.486-0.491 ms on config 3 against 0.495 grouped).
  if (window > 0 && window < Skv) return BH;
  // A short grid keeps the plain order too: with few waves, the heaviest
  // query blocks of the last group would start near the end and set the
  // tail (qk 192, B=2: 1024 CTAs, 0.385 ms plain against 0.422 grouped; B=4,
  // 2048 CTAs: 0.779 against 0.740).
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (ctas < 10LL * sms) return BH;
  const double kv_per_group = (double)Skv * (D + Dv) * 2.0;  // one kv head's K and V
  int kv_heads = (int)(48.0 * 1024 * 1024 / (kv_per_group > 1 ? kv_per_group : 1));
  if (kv_heads < 1) kv_heads = 1;
  const long long heads = (long long)kv_heads * G;
  return heads >= BH ? BH : (int)heads;
}

// Query tiles per CTA.  One tile per CTA (two CTAs per SM) when a CTA would
// walk few key tiles, so that set-up and epilogue are hidden behind the
// other resident CTA; two tiles per CTA otherwise.  D = 192 has only the
// two-tile shape (its tiles do not fit twice in shared memory).
// FFA_FWD_NQT=1|2 in the environment forces a shape (for measurements).
static int fwd_query_tiles(int D, int Sq, int Skv, int causal, int window, bool masked) {
  static const int forced = [] {
    const char* e = getenv("FFA_FWD_NQT");
    return e ? atoi(e) : 0;
  }();
  if (D == 192) return 2;
  if (forced == 1 || forced == 2) return forced;
  // average key columns a query row attends to (upper bound under masks)
  long long cols = Skv;
  if (causal) cols = (Skv + 1) / 2 + (Skv > Sq ? Skv - Sq : 0);
  if (window > 0 && window < cols) cols = window;
  (void)masked;
  // Measured (B=8 H=16 S=4096): at D = 64 with a 512-key window one tile per
  // CTA ran 0.237 ms against 0.296 ms; at D = 128 it was slower in every case
  // tried (its register budget at two CTAs per SM spills, and its K/V ring
  // holds only one key tile), so D = 128 keeps two tiles per CTA.
  return (D == 64 && cols <= FWD_NQT1_MAX_COLS) ? 1 : 2;
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
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16 && dtype != FFA_DTYPE_F32) return FFA_ERR_UNSUPPORTED;
  if (Skv > 65535 * FWD_BN) return FFA_ERR_UNSUPPORTED;
  // with a block mask a CTA records its kept key tiles in shared memory
  if (block_mask && D == 192 && (Skv + FWD_BN - 1) / FWD_BN > FwdCfg<192, 128>::MAX_LIST) return FFA_ERR_UNSUPPORTED;
  if (block_mask && (n_br <= 0 || n_bc <= 0 || mask_bq <= 0 || mask_bkv <= 0 ||
                     (int64_t)n_br * mask_bq < Sq || (int64_t)n_bc * mask_bkv < Skv))
    return FFA_ERR_INVALID_ARG;
  if (dtype == FFA_DTYPE_F32)
    return f32_fwd(q, k, v, o, lse, B, Hq, Hkv, Sq, Skv, D, Dv, q_strides, k_strides, v_strides, o_strides, scale,
                   causal, q_offset, window, softcap, block_mask, n_br, n_bc, mask_bq, mask_bkv, stream);
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
  const int nqt = fwd_query_tiles(D, Sq, Skv, causal, window, block_mask != nullptr);
  p.n_qblk = (Sq + FWD_BM * nqt - 1) / (FWD_BM * nqt);
  p.head_group = fwd_head_group(B * Hq, Hq / Hkv, Skv, D, Dv, window, (long long)p.n_qblk * B * Hq);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.use_softcap = softcap > 0.f;
  p.sc_pre = p.use_softcap ? scale / softcap : 0.f;
  p.sc_post = p.use_softcap ? softcap * 1.4426950408889634f : 0.f;
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
    if (D == 64)
      return nqt == 1 ? launch_fwd<__nv_bfloat16, 64, 64, 1>(mq, mk, mv, p, (int)grid, s)
                      : launch_fwd<__nv_bfloat16, 64, 64, 2>(mq, mk, mv, p, (int)grid, s);
    if (D == 128)
      return nqt == 1 ? launch_fwd<__nv_bfloat16, 128, 128, 1>(mq, mk, mv, p, (int)grid, s)
                      : launch_fwd<__nv_bfloat16, 128, 128, 2>(mq, mk, mv, p, (int)grid, s);
    return launch_fwd<__nv_bfloat16, 192, 128, 2>(mq, mk, mv, p, (int)grid, s);
  }
  if (D == 64)
    return nqt == 1 ? launch_fwd<__half, 64, 64, 1>(mq, mk, mv, p, (int)grid, s)
                    : launch_fwd<__half, 64, 64, 2>(mq, mk, mv, p, (int)grid, s);
  if (D == 128)
    return nqt == 1 ? launch_fwd<__half, 128, 128, 1>(mq, mk, mv, p, (int)grid, s)
                    : launch_fwd<__half, 128, 128, 2>(mq, mk, mv, p, (int)grid, s);
  return launch_fwd<__half, 192, 128, 2>(mq, mk, mv, p, (int)grid, s);
}
