// Paged-KV split decode for B200 (sm_100a).
//
// Replaces the reference's decode path — PagedKVCache.get_kv
// (ops/kv_cache.py:208-232) gathering pages into a contiguous tensor, then
// fastest_flash_attn_forward (ops/attention_forward.py:23) with one query
// token — by attention computed straight from the page pool.
//
// Page pool layout is the reference's: k_pages/v_pages [P, Hkv, page_size, D]
// (kv_cache.py:142-149); block_table [R, max_pages] int32, ctx_lens [R] int32.
//
// Kernel 1 (split): one CTA per (split, request, kv head).  A producer warp
// streams the split's 16-token chunks of K and V through a ring of smem
// slots with TMA (the pool is one tensor of rows, encoded as a 4-D map with
// unit outer dims; each chunk is a
// 16-row box at row (page*Hkv + h)*page_size + offset, 128-byte swizzled).
// Four consumer warps take chunks round-robin; each computes, for the whole
// GQA group of query heads at once (rows of an m16n8k16 tile), S = Q K^T and
// O += P V with warp-level tensor-core MMAs fed by ldmatrix, and keeps its
// own online-softmax state.  The warps' states are merged in smem and the
// split writes (O_split, LSE_split).
// Kernel 2 (merge): one warp per (request, query head) combines the splits
// with LSE weights.
// HBM traffic is the K/V bytes of the context, read once per kv head.
#include "ffa_common.cuh"
#include "ffa_host.h"

#include <type_traits>

namespace ffa {

constexpr int DEC_CHUNK = 16;     // tokens per chunk (one MMA K-step of P V)
constexpr int DEC_CONSUMERS = 4;  // consumer warps
constexpr int DEC_THREADS = (DEC_CONSUMERS + 1) * 32;
// Stages of the K/V ring.  Consumer w takes chunks w, w + C, w + 2C, ... and
// waits on stage idx % STAGES with parity (idx / STAGES) & 1.  With STAGES a
// multiple of C the stage's previous chunk is the same warp's own, so the
// barrier can never be two phases behind a waiting warp (where the parity
// test would pass on the stale phase).  8 stages keep a CTA at 65 KB of smem:
// three CTAs per SM (the register limit too), which measured 0.655 ms on
// config 4 against 0.80 ms at 12 stages (two CTAs per SM) and 1.47 ms at 16
// (one).
constexpr int DEC_STAGES = 8;
static_assert(DEC_STAGES % DEC_CONSUMERS == 0, "a stage's previous chunk must be the same consumer's");

struct DecParams {
  const void* q;      // [R, Hq, D]
  int64_t q_sr, q_sh;
  const int* block_table;
  int64_t bt_stride;  // elements between requests' rows of the block table
  const int* ctx_lens;
  int num_pages;      // valid page ids are [0, num_pages)
  int max_ctx;        // max_pages_per_req * page_size
  float* o_part;      // [R, max_splits, Hq, D]
  float* lse_part;    // [R, max_splits, Hq] (base 2)
  int R, Hq, Hkv, G, page_size, max_splits, chunks_per_split;
  float scale_log2;
  float sc_pre, sc_post;
  int use_softcap;
  ErrCtx ec;
};

enum : uint32_t { SITE_DEC_FULL = 0x301, SITE_DEC_EMPTY = 0x302 };
// Invalid paging data (not expired waits): a context length outside
// [0, max_pages_per_req * page_size], or a block-table entry outside
// [0, num_pages).  The offending CTA records the code and loads nothing.
enum : uint32_t { SITE_DEC_BAD_CTX = 0x3E0, SITE_DEC_BAD_PAGE = 0x3E1 };

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// smem address of 16-byte chunk `ch` of row `row` in a 128-byte-swizzled
// half tile (TMA SWIZZLE_128B, 1024-byte aligned base).
__device__ __forceinline__ uint32_t sw128(uint32_t base, int row, int ch) {
  return base + row * 128 + ((ch ^ (row & 7)) << 4);
}

template <int D>
struct DecCfg {
  static constexpr int HALF = DEC_CHUNK * 128;           // 16 rows x 64 elements
  static constexpr int KV_BYTES = DEC_CHUNK * D * 2;     // one chunk of K (or V)
  static constexpr int STAGE = 2 * KV_BYTES;
  // per-warp m, l, O for the CTA merge: over the stage ring, which is idle by
  // then (a separate area would cost a third CTA per SM)
  static constexpr int MERGE_OFF = 0;
  static constexpr int MERGE_BYTES = DEC_CONSUMERS * 16 * (D + 2) * 4;
  static constexpr int RING = DEC_STAGES * STAGE;
  static constexpr int BAR_OFF = RING > MERGE_BYTES ? RING : MERGE_BYTES;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
};

template <typename T, int D>
__global__ void __launch_bounds__(DEC_THREADS)
    ffa_paged_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                            const DecParams p) {
  using Cfg = DecCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* empty = full + DEC_STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + DEC_STAGES);
  float* mrg = reinterpret_cast<float*>(smem + Cfg::MERGE_OFF);

  const int split = blockIdx.x, r = blockIdx.y, h = blockIdx.z;
  const int ctx = p.ctx_lens[r];
  if (ctx < 0 || ctx > p.max_ctx) {
    if (split == 0 && h == 0 && threadIdx.x == 0 && p.ec.err) atomicCAS(p.ec.err, 0u, SITE_DEC_BAD_CTX);
    return;
  }
  const int n_chunks = (ctx + DEC_CHUNK - 1) / DEC_CHUNK;
  const int c_begin = split * p.chunks_per_split;
  if (c_begin >= n_chunks) return;  // this request has fewer splits
  const int c_end = min(n_chunks, c_begin + p.chunks_per_split);
  const int n = c_end - c_begin;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int sub_per_page = p.page_size / DEC_CHUNK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < DEC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == DEC_CONSUMERS) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();  // every byte is read once
      const int* table = p.block_table + (int64_t)r * p.bt_stride;
      int issued = 0;
      for (int idx = 0; idx < n; ++idx) {
        const int s = idx % DEC_STAGES, use = idx / DEC_STAGES;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, p.ec, abort_flag, SITE_DEC_EMPTY)) break;
        const int c = c_begin + idx;
        const int page = table[c / sub_per_page];
        if ((unsigned)page >= (unsigned)p.num_pages) {
          if (p.ec.err) atomicCAS(p.ec.err, 0u, SITE_DEC_BAD_PAGE);
          *abort_flag = 1;
          break;
        }
        const int row = (page * p.Hkv + h) * p.page_size + (c % sub_per_page) * DEC_CHUNK;
        mbar_arrive_expect_tx(&full[s], Cfg::STAGE);
        uint8_t* dst = smem + s * Cfg::STAGE;
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf) {
          tma_load_4d(&tmK, &full[s], dst + hf * Cfg::HALF, hf * 64, row, 0, 0, pol);
          tma_load_4d(&tmV, &full[s], dst + Cfg::KV_BYTES + hf * Cfg::HALF, hf * 64, row, 0, 0, pol);
        }
        ++issued;
      }
      if (*abort_flag)
        for (int q = max(0, issued - DEC_STAGES); q < issued; ++q)
          mbar_wait(&full[q % DEC_STAGES], (q / DEC_STAGES) & 1, p.ec, abort_flag, SITE_DEC_FULL, true);
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int g = lane >> 2, t = lane & 3;  // mma fragment coordinates
  // Q as the A operand: rows = query heads of the group (rows >= G are zero).
  uint32_t qa[D / 16][4];
  {
    const T* qbase = reinterpret_cast<const T*>(p.q) + (int64_t)r * p.q_sr;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int row = g + 8 * hi;
        if (row < p.G) {
          const T* qr = qbase + (int64_t)(h * p.G + row) * p.q_sh + kk * 16 + 2 * t;
          qa[kk][hi] = *reinterpret_cast<const uint32_t*>(qr);
          qa[kk][2 + hi] = *reinterpret_cast<const uint32_t*>(qr + 8);
        } else {
          qa[kk][hi] = qa[kk][2 + hi] = 0u;
        }
      }
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY;  // rows g and g + 8 (base-2 units)
  float l_lo = 0.f, l_hi = 0.f;               // this lane's partial row sums
  const int mi = lane >> 3, mr = lane & 7;    // ldmatrix: matrix index / row within it

  for (int idx = warp; idx < n; idx += DEC_CONSUMERS) {
    const int s = idx % DEC_STAGES;
    const bool ok =
        __all_sync(0xffffffffu, mbar_wait(&full[s], (idx / DEC_STAGES) & 1, p.ec, abort_flag, SITE_DEC_FULL));
    if (!ok) break;
    const uint32_t kbase = smem_u32(smem + s * Cfg::STAGE);
    const uint32_t vbase = kbase + Cfg::KV_BYTES;
    // S = Q K^T for the chunk's 16 tokens (two n-tiles of 8 tokens)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int hf = kk / 4, ch = 2 * (kk % 4) + (mi & 1);
      const int tok = mr + 8 * (mi >> 1);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(sw128(kbase + hf * Cfg::HALF, tok, ch), b00, b01, b10, b11);
      mma16816<T>(sc[0], qa[kk], b00, b01);
      mma16816<T>(sc[1], qa[kk], b10, b11);
    }
    // scale, softcap, mask tokens beyond the context
    const int tok0 = (c_begin + idx) * DEC_CHUNK;
    float x[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = sc[nt][e];
        v = p.use_softcap ? tanh_acc(v * p.sc_pre) * p.sc_post : v * p.scale_log2;
        const int tok = tok0 + nt * 8 + 2 * t + (e & 1);
        x[nt][e] = tok < ctx ? v : -INFINITY;
      }
    float mx_lo = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
    float mx_hi = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    // lazy rescale: only when a row max grows by more than 2^8
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    if (__any_sync(0xffffffffu, mn_lo > m_lo + 8.f || mn_hi > m_hi + 8.f)) {
      const float a_lo = (mn_lo == -INFINITY) ? 1.f : ex2(m_lo - mn_lo);
      const float a_hi = (mn_hi == -INFINITY) ? 1.f : ex2(m_hi - mn_hi);
      l_lo *= a_lo;
      l_hi *= a_hi;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][0] *= a_lo;
        o[i][1] *= a_lo;
        o[i][2] *= a_hi;
        o[i][3] *= a_hi;
      }
      m_lo = mn_lo;
      m_hi = mn_hi;
    }
    const float u_lo = (m_lo == -INFINITY) ? 0.f : m_lo, u_hi = (m_hi == -INFINITY) ? 0.f : m_hi;
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      pr[nt][0] = ex2(x[nt][0] - u_lo);
      pr[nt][1] = ex2(x[nt][1] - u_lo);
      pr[nt][2] = ex2(x[nt][2] - u_hi);
      pr[nt][3] = ex2(x[nt][3] - u_hi);
      l_lo += pr[nt][0] + pr[nt][1];
      l_hi += pr[nt][2] + pr[nt][3];
    }
    // P as the A operand of P V (the S accumulator layout of two n-tiles is
    // exactly the A layout of one k = 16 step)
    const uint32_t pa[4] = {pack2<T>(pr[0][0], pr[0][1]), pack2<T>(pr[0][2], pr[0][3]),
                            pack2<T>(pr[1][0], pr[1][1]), pack2<T>(pr[1][2], pr[1][3])};
#pragma unroll
    for (int nt = 0; nt < D / 8; nt += 2) {
      const int hf = nt / 8, ch = (nt % 8) + (mi >> 1);
      const int tok = mr + 8 * (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sw128(vbase + hf * Cfg::HALF, tok, ch), b0, b1, b2, b3);
      mma16816<T>(o[nt], pa, b0, b1);
      mma16816<T>(o[nt + 1], pa, b2, b3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // -------------------- merge the consumer warps' states -------------------
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  // The merge area overlays the stage ring: every consumer must be done with
  // its last chunk first.  After an abort, copies may still be landing in the
  // ring (the producer drains them), so nothing is written.
  asm volatile("bar.sync 1, %0;" ::"n"(DEC_CONSUMERS * 32) : "memory");
  if (*abort_flag) return;
  float* wm = mrg + warp * 16 * (D + 2);  // per warp: 16 rows x (m, l, O[D])
  if (t == 0) {
    wm[g * (D + 2) + 0] = m_lo;
    wm[g * (D + 2) + 1] = l_lo;
    wm[(g + 8) * (D + 2) + 0] = m_hi;
    wm[(g + 8) * (D + 2) + 1] = l_hi;
  }
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) {
    const int d = nt * 8 + 2 * t;
    wm[g * (D + 2) + 2 + d] = o[nt][0];
    wm[g * (D + 2) + 2 + d + 1] = o[nt][1];
    wm[(g + 8) * (D + 2) + 2 + d] = o[nt][2];
    wm[(g + 8) * (D + 2) + 2 + d + 1] = o[nt][3];
  }
  asm volatile("bar.sync 1, %0;" ::"n"(DEC_CONSUMERS * 32) : "memory");
  const int tid = threadIdx.x;
  for (int item = tid; item < p.G * (D / 4); item += DEC_CONSUMERS * 32) {
    const int row = item / (D / 4), d0 = (item % (D / 4)) * 4;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < DEC_CONSUMERS; ++w) M = fmaxf(M, mrg[w * 16 * (D + 2) + row * (D + 2)]);
    float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < DEC_CONSUMERS; ++w) {
      const float* wr = mrg + w * 16 * (D + 2) + row * (D + 2);
      const float mw = wr[0];
      const float f = (mw == -INFINITY) ? 0.f : ex2(mw - M);
      L += wr[1] * f;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] += wr[2 + d0 + e] * f;
    }
    const int head = h * p.G + row;
    const int64_t pidx = ((int64_t)r * p.max_splits + split) * p.Hq + head;
    const float inv = L > 0.f ? 1.f / L : 0.f;
    *reinterpret_cast<float4*>(p.o_part + pidx * D + d0) =
        make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    if (d0 == 0) p.lse_part[pidx] = (L > 0.f) ? M + lg2(L) : -INFINITY;
  }
}

// One warp per (request, query head): combine the splits.
template <typename T, int D>
__global__ void ffa_decode_merge_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part,
                                        const int* __restrict__ ctx_lens, void* out, float* lse_out, int R, int Hq,
                                        int max_splits, int chunks_per_split, int64_t o_sr, int64_t o_sh) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (wid >= R * Hq) return;
  const int r = wid / Hq, head = wid % Hq;
  const int n_chunks = (ctx_lens[r] + DEC_CHUNK - 1) / DEC_CHUNK;
  // clamped: an out-of-range length (reported by the split kernel) never
  // makes the merge read past the request's partials
  const int ns = min(max((n_chunks + chunks_per_split - 1) / chunks_per_split, 0), max_splits);
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, lse_part[((int64_t)r * max_splits + s) * Hq + head]);
  float L = 0.f;
  float acc[D / 32];
#pragma unroll
  for (int e = 0; e < D / 32; ++e) acc[e] = 0.f;
  for (int s = 0; s < ns; ++s) {
    const int64_t pidx = ((int64_t)r * max_splits + s) * Hq + head;
    const float ls = lse_part[pidx];
    const float f = (ls == -INFINITY) ? 0.f : ex2(ls - M);
    L += f;
#pragma unroll
    for (int e = 0; e < D / 32; ++e) acc[e] += f * o_part[pidx * D + lane + 32 * e];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* orow = reinterpret_cast<T*>(out) + (int64_t)r * o_sr + (int64_t)head * o_sh;
#pragma unroll
  for (int e = 0; e < D / 32; ++e) {
    const float v = acc[e] * inv;
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
      orow[lane + 32 * e] = __float2bfloat16_rn(v);
    else
      orow[lane + 32 * e] = __float2half_rn(v);
  }
  if (lane == 0 && lse_out)
    lse_out[(int64_t)r * Hq + head] = (L > 0.f) ? (M + lg2(L)) * 0.6931471805599453f : -INFINITY;
}

template <typename T, int D>
static int launch_decode(const CUtensorMap& mk, const CUtensorMap& mv, const DecParams& p, void* out,
                         float* lse, int64_t o_sr, int64_t o_sh, cudaStream_t st) {
  using Cfg = DecCfg<D>;
  auto kern = ffa_paged_decode_kernel<T, D>;
  static std::atomic<uint64_t> done{0};
  if (int s = smem_attr_once(kern, Cfg::SMEM, done)) return s;
  dim3 grid(p.max_splits, p.R, p.Hkv);
  kern<<<grid, DEC_THREADS, Cfg::SMEM, st>>>(mk, mv, p);
  int s = launch_status();
  if (s) return s;
  const int warps = p.R * p.Hq;
  ffa_decode_merge_kernel<T, D><<<(warps * 32 + 255) / 256, 256, 0, st>>>(
      p.o_part, p.lse_part, p.ctx_lens, out, lse, p.R, p.Hq, p.max_splits, p.chunks_per_split, o_sr, o_sh);
  return launch_status();
}

// ---------------------------------------------------------------------------
// MLA absorbed decode.
//
// The latent cache holds, per token, [c_kv (LAT) | k_rope (ROPE)] (576 values
// for DeepSeek-style 512 + 64).  With the up-projections absorbed into the
// query (q_lat = q_nope W_UK per head) and applied after attention
// (out = o_lat W_UV^T), decoding is multi-query attention of every head over
// the shared latent keys [c_kv | k_rope] with values c_kv.  One CTA per
// (split, request), splits merged by LSE.
// ---------------------------------------------------------------------------
constexpr int MLA_LAT = 512, MLA_ROPE = 64, MLA_DK = MLA_LAT + MLA_ROPE;
constexpr int MLA_HEADS = 32;  // query heads: the N dimension of both tensor-core products
constexpr int MLA_BOXES = MLA_DK / 64;  // 9 swizzled 64-column boxes per token row

struct MlaParams {
  const void* q;  // [R, H, 576] = [q_lat | q_rope]
  int64_t q_sr, q_sh;
  const int* block_table;
  int64_t bt_stride;
  const int* ctx_lens;
  int num_pages;  // valid page ids are [0, num_pages)
  int max_ctx;    // max_pages_per_req * page_size
  float* o_part;    // [R, max_splits, H, 512]
  float* lse_part;  // [R, max_splits, H] (base 2)
  int R, H, page_size, max_splits, chunks_per_split;
  int box_rows;  // token rows per TMA box of the latent decode kernel: gcd(page_size, 128)
  float scale_log2;
  ErrCtx ec;
};

// ---------------------------------------------------------------------------
// MLA absorbed decode on the 5th-generation tensor cores.
//
// Tokens are the M dimension of both products, so 32 heads fit the MMA shape
// without padding:
//   S^T [128 tokens x 32 heads] = C [128 x 576] . Q^T          (K = 576)
//   O^T [512 dims x 32 heads]  += C_lat^T [512 x 128] . P^T     (K = 128 tokens)
// C is read once per tile of 128 tokens and serves both products: the latent
// part (512 dims) as the M-major A operand of the second.  Roles:
//   warps 0-7  softmax (thread r % 128 = token r of the tile; warpgroup g
//              takes heads [16 g, 16 g + 16)): per-head maximum over the
//              tile's tokens by a transposing butterfly of warp shuffles plus
//              a cross-warp exchange in smem, P^T = 2^(s*scale*log2e - m)
//              stored to smem as the B operand of O^T, running row sums; O^T
//              is rescaled (exactly, numerator and denominator alike) only
//              when a head's maximum grows by more than 2^8.
//   warp 8     TMA producer: boxes of gcd(page_size, 128) tokens through the
//              block table into a ring of 5 slots (4 slots of 2 latent
//              boxes, 1 rope box).
//   warp 9     MMA issuer, TMEM owner.
// TMEM: O^T in columns [0, 128) (block m of 128 dims at 32 m), S^T double
// buffered at [128, 192).
// ---------------------------------------------------------------------------
constexpr int MLT_TILE = 128;                 // tokens per tile (MMA M)
constexpr int MLT_BOX = MLT_TILE * 128;       // one 64-dim box of the tile: 16 KB
constexpr int MLT_SLOT = 2 * MLT_BOX;         // 32 KB
constexpr int MLT_NSLOT = 5;
constexpr int MLT_Q_OFF = MLT_NSLOT * MLT_SLOT;               // 9 boxes of [32 heads x 64 dims]
constexpr int MLT_QBOX = MLA_HEADS * 128;                     // 4 KB
constexpr int MLT_P_OFF = MLT_Q_OFF + MLA_BOXES * MLT_QBOX;  // 2 buffers of P^T [32 x 128]
constexpr int MLT_PBUF = MLA_HEADS * MLT_TILE * 2;            // 8 KB
constexpr int MLT_RED_OFF = MLT_P_OFF + 2 * MLT_PBUF;         // [2][4 warps][32] floats
constexpr int MLT_BAR_OFF = MLT_RED_OFF + 2 * 4 * 32 * 4;
constexpr int MLT_SMEM = MLT_BAR_OFF + 256 + 1024;
constexpr int MLT_THREADS = 320;
constexpr float MLT_RESCALE = 8.0f;

struct MltBars {
  uint64_t slot_full[MLT_NSLOT];
  uint64_t slot_empty[MLT_NSLOT];
  uint64_t q_ready;     // Q stored to smem (one arrival per softmax warp)
  uint64_t s_full[2];   // S^T of tile t computed
  uint64_t p_ready[2];  // P^T of tile t stored (one arrival per softmax warp)
  uint64_t o_done[2];   // O^T MMAs of tile t retired
  uint64_t red_full[2]; // per-warp partial maxima / sums of a tile exchanged
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Transposing butterfly over 16 columns: lanes i and i + 16 end with the
// maximum (MAX) or sum over the 32 lanes of v[i % 16].  16 shuffles.
template <bool MAX>
__device__ __forceinline__ float warp_colreduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float keep = up ? v[i + o] : v[i];
      const float give = up ? v[i] : v[i + o];
      const float got = __shfl_xor_sync(0xffffffffu, give, o);
      v[i] = MAX ? fmaxf(keep, got) : keep + got;
    }
  }
  const float other = __shfl_xor_sync(0xffffffffu, v[0], 16);
  return MAX ? fmaxf(v[0], other) : v[0] + other;
}

template <typename T>
__global__ void __launch_bounds__(128) ffa_mla_merge_kernel(const float* __restrict__ o_part,
                                                            const float* __restrict__ lse_part,
                                                            const int* __restrict__ ctx_lens, void* out,
                                                            float* lse_out, int H, int max_splits,
                                                            int chunks_per_split, int64_t o_sr, int64_t o_sh) {
  const int r = blockIdx.x / H, head = blockIdx.x % H;
  const int n_chunks = (ctx_lens[r] + DEC_CHUNK - 1) / DEC_CHUNK;
  const int ns = min(max((n_chunks + chunks_per_split - 1) / chunks_per_split, 0), max_splits);
  const int64_t base = (int64_t)r * max_splits * H + head;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, lse_part[base + (int64_t)s * H]);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int s = 0; s < ns; ++s) {
    const int64_t pidx = base + (int64_t)s * H;
    const float ls = lse_part[pidx];
    const float f = (ls == -INFINITY) ? 0.f : ex2(ls - M);
    const float4 v = reinterpret_cast<const float4*>(o_part + pidx * MLA_LAT)[threadIdx.x];
    L += f;
    acc.x += f * v.x;
    acc.y += f * v.y;
    acc.z += f * v.z;
    acc.w += f * v.w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* orow = reinterpret_cast<T*>(out) + (int64_t)r * o_sr + (int64_t)head * o_sh + 4 * threadIdx.x;
  const uint32_t lo = pack2<T>(acc.x * inv, acc.y * inv), hi = pack2<T>(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(orow) = make_uint2(lo, hi);
  if (threadIdx.x == 0 && lse_out)
    lse_out[(int64_t)r * H + head] = (L > 0.f) ? (M + lg2(L)) * 0.6931471805599453f : -INFINITY;
}

template <typename T>
__global__ void __launch_bounds__(MLT_THREADS, 1)
    ffa_mla_decode_tc_kernel(const __grid_constant__ CUtensorMap tmC, const MlaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  MltBars* bars = reinterpret_cast<MltBars*>(smem + MLT_BAR_OFF);
  float* red = reinterpret_cast<float*>(smem + MLT_RED_OFF);
  volatile int* abort_flag = &bars->abort;

  const int split = blockIdx.x, r = blockIdx.y;
  const int ctx = p.ctx_lens[r];
  if (ctx < 0 || ctx > p.max_ctx) {
    if (split == 0 && threadIdx.x == 0 && p.ec.err) atomicCAS(p.ec.err, 0u, SITE_DEC_BAD_CTX);
    return;
  }
  const int n_chunks = (ctx + DEC_CHUNK - 1) / DEC_CHUNK;
  const int c_begin = split * p.chunks_per_split;
  if (c_begin >= n_chunks) return;
  const int c_end = min(n_chunks, c_begin + p.chunks_per_split);
  const int tok_end = min(ctx, c_end * DEC_CHUNK);  // tokens of this split: [c_begin*16, tok_end)
  const int n_tiles = (c_end - c_begin + 7) / 8;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr uint32_t FMT = DtypeFmt<T>::value;

  if (threadIdx.x == 0) {
    for (int s = 0; s < MLT_NSLOT; ++s) {
      mbar_init(&bars->slot_full[s], 1);
      mbar_init(&bars->slot_empty[s], 1);
    }
    mbar_init(&bars->q_ready, 8);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_ready[b], 8);
      mbar_init(&bars->o_done[b], 1);
      mbar_init(&bars->red_full[b], 8);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 8) {
    // ------------------------------ producer ------------------------------
    // The split's page ids are read 32 at a time, one per lane, and handed to
    // the issuing lane by shuffles, so no TMA issue waits on a global load.
    const uint64_t pol = policy_evict_first();
    const int* table = p.block_table + (int64_t)r * p.bt_stride;
    const int br = p.box_rows;
    const int page0 = c_begin * DEC_CHUNK / p.page_size;
    const int n_pages_req = (ctx + p.page_size - 1) / p.page_size;
    const int n_blk = (ctx + br - 1) / br;  // br-row blocks holding the request's tokens
    int win = -1, pid = 0;  // page window [32 win, 32 win + 32) held by the lanes
    int issued = 0;
    // Every page id this split will read is checked before the first copy is
    // armed (independent loads, one latency); a bad id stops the CTA.
    const int page_last = min(n_pages_req, (c_begin * DEC_CHUNK + n_tiles * MLT_TILE + p.page_size - 1) / p.page_size);
    bool bad = false;
    for (int i = page0 + lane; i < page_last; i += 32) bad |= (unsigned)table[i] >= (unsigned)p.num_pages;
    bool ok = !__any_sync(0xffffffffu, bad);
    if (!ok) {
      if (lane == 0 && p.ec.err) atomicCAS(p.ec.err, 0u, SITE_DEC_BAD_PAGE);
      *abort_flag = 1;
    }
    for (int t = 0; t < n_tiles && ok; ++t) {
      for (int kk = 0; kk < MLT_NSLOT && ok; ++kk) {
        const int k = (kk + MLT_NSLOT - 1) % MLT_NSLOT;  // the rope slot first: it frees earliest
        if (t > 0)
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->slot_empty[k], (t - 1) & 1, p.ec, abort_flag, SITE_DEC_EMPTY));
        if (!ok) break;
        const int nbox = k < 4 ? 2 : 1;
        if (lane == 0) mbar_arrive_expect_tx(&bars->slot_full[k], nbox * MLT_BOX);
        uint8_t* dst = smem + k * MLT_SLOT;
        for (int sub = 0; sub < MLT_TILE / br; ++sub) {
          // blocks past the request reload its last block: finite values, masked by P = 0
          const int blk = min((c_begin * DEC_CHUNK + t * MLT_TILE) / br + sub, n_blk - 1);
          const int pg = blk * br / p.page_size - page0;
          if (pg / 32 != win) {
            win = pg / 32;
            const int idx = page0 + 32 * win + lane;
            pid = idx < n_pages_req ? table[idx] : 0;
          }
          const int page = __shfl_sync(0xffffffffu, pid, pg % 32);
          const int row = page * p.page_size + (blk * br) % p.page_size;
          if (lane == 0)
            for (int bx = 0; bx < nbox; ++bx) {
              const int box = k < 4 ? 2 * k + bx : 8;
              tma_load_4d(&tmC, &bars->slot_full[k], dst + bx * MLT_BOX + sub * br * 128, box * 64, row, 0, 0, pol);
            }
        }
        ++issued;
      }
    }
    if (lane == 0 && *abort_flag)  // copies in flight must land before the CTA exits
      for (int q = max(0, issued - MLT_NSLOT); q < issued; ++q)
        mbar_wait(&bars->slot_full[(q % MLT_NSLOT + MLT_NSLOT - 1) % MLT_NSLOT], (q / MLT_NSLOT) & 1, p.ec,
                  abort_flag, SITE_DEC_FULL, true);
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_f16(128, MLA_HEADS, FMT, 0, 0);  // C (K-major) x Q (K-major)
      const uint32_t idesc_o = make_idesc_f16(128, MLA_HEADS, FMT, 1, 0);  // C_lat^T (M-major) x P^T (K-major)
      const uint64_t c_kdesc = make_sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t c_mdesc = make_sdesc_sw128(smem_u32(smem), MLT_BOX, 1024);
      const uint64_t q_desc = make_sdesc_sw128(smem_u32(smem + MLT_Q_OFF), 16, 1024);
      const uint64_t p_desc = make_sdesc_sw128(smem_u32(smem + MLT_P_OFF), 16, 1024);
      bool ok = mbar_wait(&bars->q_ready, 0, p.ec, abort_flag, SITE_DEC_FULL);
      auto issue_o = [&](int t) -> bool {
        if (!mbar_wait(&bars->p_ready[t & 1], (t >> 1) & 1, p.ec, abort_flag, SITE_DEC_FULL)) return false;
        tc_fence_after();
        const uint64_t pb = p_desc + (uint64_t)(((t & 1) * MLT_PBUF) >> 4);
        for (int m = 0; m < 4; ++m) {
          const uint64_t a = c_mdesc + (uint64_t)((m * MLT_SLOT) >> 4);
#pragma unroll
          for (int ks = 0; ks < MLT_TILE / 16; ++ks)
            mma_ss(tmem + 32 * m, a + (uint64_t)((ks * 16 * 128) >> 4),
                   pb + (uint64_t)(((ks / 4) * (MLA_HEADS * 128) + (ks % 4) * 32) >> 4), idesc_o,
                   (t > 0 || ks > 0) ? 1u : 0u);
          mma_commit(&bars->slot_empty[m]);
        }
        mma_commit(&bars->o_done[t & 1]);
        return true;
      };
      // O^T(t-1) goes before S^T(t): the loads of tile t wait for the slots
      // that O^T(t-1) releases.
      for (int t = 0; t < n_tiles && ok; ++t) {
        if (t > 0 && !(ok = issue_o(t - 1))) break;
        const uint32_t dS = tmem + 128 + 32 * (t & 1);
        bool first = true;
        for (int kk = 0; kk < MLT_NSLOT && ok; ++kk) {
          const int k = (kk + MLT_NSLOT - 1) % MLT_NSLOT;
          if (!(ok = mbar_wait(&bars->slot_full[k], t & 1, p.ec, abort_flag, SITE_DEC_FULL))) break;
          tc_fence_after();
          const int nbox = k < 4 ? 2 : 1;
          for (int bx = 0; bx < nbox; ++bx) {
            const int box = k < 4 ? 2 * k + bx : 8;
            const uint64_t a = c_kdesc + (uint64_t)((k * MLT_SLOT + bx * MLT_BOX) >> 4);
            const uint64_t b = q_desc + (uint64_t)((box * MLT_QBOX) >> 4);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              mma_ss(dS, a + (uint64_t)(ks * 2), b + (uint64_t)(ks * 2), idesc_s, first ? 0u : 1u);
              first = false;
            }
          }
        }
        if (!ok) break;
        mma_commit(&bars->slot_empty[4]);  // the rope box is not needed by O^T
        mma_commit(&bars->s_full[t & 1]);
      }
      if (ok && n_tiles > 0) ok = issue_o(n_tiles - 1);
      if (!ok) {  // let issued MMAs retire before TMEM is released
        mma_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, p.ec, abort_flag, SITE_DEC_FULL, true);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ softmax -------------------------------
    // warpgroup hh handles heads [16 hh, 16 hh + 16) of every token
    const int tr = threadIdx.x % 128;  // token row of the tile = TMEM lane
    const int hh = warp / 4;
    const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
    // Q -> smem as 9 K-major swizzled boxes of [32 heads x 64 dims]
    {
      const T* qr = reinterpret_cast<const T*>(p.q) + (int64_t)r * p.q_sr;
      for (int c = threadIdx.x; c < MLA_HEADS * (MLA_DK / 8); c += 256) {
        const int h = c / (MLA_DK / 8), j = c % (MLA_DK / 8);
        const uint4 v = *reinterpret_cast<const uint4*>(qr + (int64_t)h * p.q_sh + j * 8);
        const int box = j / 8, jj = j % 8;
        *reinterpret_cast<uint4*>(smem + MLT_Q_OFF + box * MLT_QBOX + h * 128 + ((jj ^ (h & 7)) << 4)) = v;
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->q_ready);
    }
    float m_run[16], l_part[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      m_run[h] = -INFINITY;
      l_part[h] = 0.f;
    }
    // this warpgroup's 4 per-warp partials of head j: red[buf][4 hh + w][j]
    auto wg_reduce = [&](const float* rb, float (&out)[16], bool is_max) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 acc = reinterpret_cast<const float4*>(rb + (4 * hh) * 16)[q];
#pragma unroll
        for (int w = 1; w < 4; ++w) {
          const float4 v = reinterpret_cast<const float4*>(rb + (4 * hh + w) * 16)[q];
          acc.x = is_max ? fmaxf(acc.x, v.x) : acc.x + v.x;
          acc.y = is_max ? fmaxf(acc.y, v.y) : acc.y + v.y;
          acc.z = is_max ? fmaxf(acc.z, v.z) : acc.z + v.z;
          acc.w = is_max ? fmaxf(acc.w, v.w) : acc.w + v.w;
        }
        out[4 * q] = acc.x;
        out[4 * q + 1] = acc.y;
        out[4 * q + 2] = acc.z;
        out[4 * q + 3] = acc.w;
      }
    };
    bool ok = true;
    for (int t = 0; t < n_tiles && ok; ++t) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[t & 1], (t >> 1) & 1, p.ec, abort_flag, SITE_DEC_FULL));
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[16];
      tmem_ld16(tmem + lane_off + 128 + 32 * (t & 1) + 16 * hh, sv);
      tmem_ld_wait16(sv);
      const bool valid = c_begin * DEC_CHUNK + t * MLT_TILE + tr < tok_end;
      float x[16], v[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        x[h] = valid ? __uint_as_float(sv[h]) * p.scale_log2 : -INFINITY;
        v[h] = x[h];
      }
      // per-head tile maximum: warp butterfly, then the warpgroup's 4 warps through smem
      float* rb = red + (t & 1) * 128;
      const float wm = warp_colreduce16<true>(v, lane);
      if (lane < 16) rb[warp * 16 + lane] = wm;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->red_full[t & 1]);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->red_full[t & 1], (t >> 1) & 1, p.ec, abort_flag, SITE_DEC_FULL));
      if (!ok) break;
      // heads whose maximum grew past the threshold move it, and rescale
      float mt[16], alpha[16];
      wg_reduce(rb, mt, true);
      bool resc = false;
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        alpha[h] = 1.f;
        if (mt[h] > m_run[h] + MLT_RESCALE) {
          alpha[h] = m_run[h] == -INFINITY ? 0.f : ex2(m_run[h] - mt[h]);
          m_run[h] = mt[h];
          l_part[h] *= alpha[h];
          resc = true;
        }
      }
      // O^T and this buffer of P^T must be done with tile t-1 / t-2: both
      // follow from O^T(t-1) having retired (the tensor core runs in order).
      if (t > 0) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&bars->o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, p.ec, abort_flag, SITE_DEC_FULL));
        if (!ok) break;
        tc_fence_after();
        if (resc) {
          // thread tr owns dim tr of each 128-dim block of O^T
#pragma unroll 1
          for (int m = 0; m < 4; ++m) {
            uint32_t ov[16];
            tmem_ld16(tmem + lane_off + 32 * m + 16 * hh, ov);
            tmem_ld_wait16(ov);
#pragma unroll
            for (int h = 0; h < 16; ++h) ov[h] = __float_as_uint(__uint_as_float(ov[h]) * alpha[h]);
            tmem_st16(tmem + lane_off + 32 * m + 16 * hh, ov);
          }
          tmem_st_wait();
        }
      }
      // P^T[h][tr] (K-major B of O^T: head rows, token columns in two 64-token chunks)
      uint8_t* pb = smem + MLT_P_OFF + (t & 1) * MLT_PBUF + (tr / 64) * (MLA_HEADS * 128);
      const int tc = tr % 64;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int h = 16 * hh + j;
        const float pv = ex2(x[j] - (m_run[j] == -INFINITY ? 0.f : m_run[j]));
        l_part[j] += pv;
        T hv;
        if constexpr (std::is_same<T, __nv_bfloat16>::value)
          hv = __float2bfloat16_rn(pv);
        else
          hv = __float2half_rn(pv);
        *reinterpret_cast<T*>(pb + h * 128 + (((tc / 8) ^ (h & 7)) << 4) + (tc % 8) * 2) = hv;
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_ready[t & 1]);
    }
    // ------------------------------ epilogue ------------------------------
    // row sums per head over all 128 token threads (exchange slot n_tiles & 1)
    if (ok && n_tiles > 0) {
      float* rb = red + (n_tiles & 1) * 128;
      const float ws = warp_colreduce16<false>(l_part, lane);
      if (lane < 16) rb[warp * 16 + lane] = ws;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->red_full[n_tiles & 1]);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->red_full[n_tiles & 1], (n_tiles >> 1) & 1, p.ec, abort_flag,
                                             SITE_DEC_FULL)) &&
           __all_sync(0xffffffffu, mbar_wait(&bars->o_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, p.ec,
                                             abort_flag, SITE_DEC_FULL));
      if (ok) {
        tc_fence_after();
        float L[16], inv[16];
        wg_reduce(rb, L, false);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          inv[j] = L[j] > 0.f ? 1.f / L[j] : 0.f;
          if (tr == j) {
            const int64_t pidx = ((int64_t)r * p.max_splits + split) * p.H + 16 * hh + j;
            p.lse_part[pidx] = L[j] > 0.f ? m_run[j] + lg2(L[j]) : -INFINITY;
          }
        }
#pragma unroll 1
        for (int m = 0; m < 4; ++m) {
          uint32_t ov[16];
          tmem_ld16(tmem + lane_off + 32 * m + 16 * hh, ov);
          tmem_ld_wait16(ov);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t pidx = ((int64_t)r * p.max_splits + split) * p.H + 16 * hh + j;
            p.o_part[pidx * MLA_LAT + 128 * m + tr] = __uint_as_float(ov[j]) * inv[j];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace ffa

extern "C" size_t ffa_paged_decode_workspace_size(int R, int Hq, int D, int max_pages_per_req, int page_size,
                                                  int chunks_per_split) {
  if (R <= 0 || Hq <= 0 || D <= 0 || max_pages_per_req <= 0 || page_size <= 0 || chunks_per_split <= 0) return 0;
  const int max_chunks = max_pages_per_req * (page_size / ffa::DEC_CHUNK);
  const int max_splits = (max_chunks + chunks_per_split - 1) / chunks_per_split;
  return (size_t)R * max_splits * Hq * (D + 1) * sizeof(float) + 256;
}

extern "C" int ffa_paged_decode(const void* q, const void* k_pages, const void* v_pages, const int* block_table,
                                const int* ctx_lens, void* out, float* lse, int dtype, int R, int Hq, int Hkv,
                                int D, int num_pages, int page_size, int max_pages_per_req,
                                const int64_t* q_strides, const int64_t* o_strides, float scale, float softcap,
                                int chunks_per_split, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                                void* stream) {
  using namespace ffa;
  if (!q || !k_pages || !v_pages || !block_table || !ctx_lens || !out || !q_strides || !o_strides)
    return FFA_ERR_INVALID_ARG;
  if (R <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || num_pages <= 0 || max_pages_per_req <= 0)
    return FFA_ERR_INVALID_ARG;
  if (D != 64 && D != 128) return FFA_ERR_UNSUPPORTED;
  if (Hq / Hkv > 16) return FFA_ERR_UNSUPPORTED;
  if (page_size <= 0 || page_size % DEC_CHUNK != 0) return FFA_ERR_UNSUPPORTED;
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16) return FFA_ERR_UNSUPPORTED;
  if (chunks_per_split <= 0) chunks_per_split = 32;
  if ((q_strides[1] % 2) || (q_strides[0] % 2) || (reinterpret_cast<uintptr_t>(q) & 3)) return FFA_ERR_INVALID_ARG;
  const size_t need = ffa_paged_decode_workspace_size(R, Hq, D, max_pages_per_req, page_size, chunks_per_split);
  if (!workspace || workspace_bytes < need) return FFA_ERR_WORKSPACE;

  DecParams p{};
  p.q = q;
  p.q_sr = q_strides[0];
  p.q_sh = q_strides[1];
  p.block_table = block_table;
  p.bt_stride = max_pages_per_req;
  p.ctx_lens = ctx_lens;
  p.num_pages = num_pages;
  if ((int64_t)max_pages_per_req * page_size > 0x7fffffffLL) return FFA_ERR_UNSUPPORTED;
  p.max_ctx = max_pages_per_req * page_size;
  const int max_chunks = max_pages_per_req * (page_size / DEC_CHUNK);
  p.max_splits = (max_chunks + chunks_per_split - 1) / chunks_per_split;
  uintptr_t ws = (reinterpret_cast<uintptr_t>(workspace) + 127) & ~uintptr_t(127);
  p.o_part = reinterpret_cast<float*>(ws);
  p.lse_part = p.o_part + (size_t)R * p.max_splits * Hq * D;
  p.R = R;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.page_size = page_size;
  p.chunks_per_split = chunks_per_split;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.use_softcap = softcap > 0.f;
  p.sc_pre = p.use_softcap ? scale / softcap : 0.f;
  p.sc_post = p.use_softcap ? softcap * 1.4426950408889634f : 0.f;
  p.ec.err = dev_err;
  p.ec.limit_ns = wait_limit_ns();
  if (p.max_splits > 65535 || R > 65535 || Hkv > 65535) return FFA_ERR_UNSUPPORTED;

  const CUtensorMapDataType dt =
      dtype == FFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // The pool as a 2-D tensor of rows: [num_pages * Hkv * page_size, D].
  const uint64_t rows = (uint64_t)num_pages * Hkv * page_size;
  CUtensorMap mk, mv;
  int st = make_tmap_4d(&mk, k_pages, dt, 2, D, rows, 1, 1, (uint64_t)D * 2, rows * D * 2, rows * D * 2, 64,
                        DEC_CHUNK);
  if (!st)
    st = make_tmap_4d(&mv, v_pages, dt, 2, D, rows, 1, 1, (uint64_t)D * 2, rows * D * 2, rows * D * 2, 64,
                      DEC_CHUNK);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FFA_DTYPE_BF16) {
    if (D == 64) return launch_decode<__nv_bfloat16, 64>(mk, mv, p, out, lse, o_strides[0], o_strides[1], s);
    return launch_decode<__nv_bfloat16, 128>(mk, mv, p, out, lse, o_strides[0], o_strides[1], s);
  }
  if (D == 64) return launch_decode<__half, 64>(mk, mv, p, out, lse, o_strides[0], o_strides[1], s);
  return launch_decode<__half, 128>(mk, mv, p, out, lse, o_strides[0], o_strides[1], s);
}

extern "C" size_t ffa_mla_decode_workspace_size(int R, int H, int max_pages_per_req, int page_size,
                                                int chunks_per_split) {
  return ffa_paged_decode_workspace_size(R, H, ffa::MLA_LAT, max_pages_per_req, page_size, chunks_per_split);
}

extern "C" int ffa_mla_decode(const void* q, const void* ckv_pages, const int* block_table, const int* ctx_lens,
                              void* out_lat, float* lse, int dtype, int R, int H, int num_pages, int page_size,
                              int max_pages_per_req, const int64_t* q_strides, const int64_t* o_strides, float scale,
                              int chunks_per_split, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                              void* stream) {
  using namespace ffa;
  if (!q || !ckv_pages || !block_table || !ctx_lens || !out_lat || !q_strides || !o_strides)
    return FFA_ERR_INVALID_ARG;
  if (R <= 0 || num_pages <= 0 || max_pages_per_req <= 0) return FFA_ERR_INVALID_ARG;
  if (H != MLA_HEADS) return FFA_ERR_UNSUPPORTED;
  if (page_size <= 0 || page_size % DEC_CHUNK != 0) return FFA_ERR_UNSUPPORTED;
  if (dtype != FFA_DTYPE_BF16 && dtype != FFA_DTYPE_F16) return FFA_ERR_UNSUPPORTED;
  if (chunks_per_split <= 0) chunks_per_split = 32;
  if ((q_strides[1] % 8) || (q_strides[0] % 8) || (reinterpret_cast<uintptr_t>(q) & 15)) return FFA_ERR_INVALID_ARG;
  if ((o_strides[1] % 4) || (o_strides[0] % 4) || (reinterpret_cast<uintptr_t>(out_lat) & 7)) return FFA_ERR_INVALID_ARG;
  const size_t need = ffa_mla_decode_workspace_size(R, H, max_pages_per_req, page_size, chunks_per_split);
  if (!workspace || workspace_bytes < need) return FFA_ERR_WORKSPACE;
  // Splits are whole 128-token tiles (8 chunks); rounding up only lowers the
  // number of splits, so the workspace sized for the caller's value suffices.
  chunks_per_split = (chunks_per_split + 7) / 8 * 8;
  MlaParams p{};
  p.q = q;
  p.q_sr = q_strides[0];
  p.q_sh = q_strides[1];
  p.block_table = block_table;
  p.bt_stride = max_pages_per_req;
  p.ctx_lens = ctx_lens;
  p.num_pages = num_pages;
  if ((int64_t)max_pages_per_req * page_size > 0x7fffffffLL) return FFA_ERR_UNSUPPORTED;
  p.max_ctx = max_pages_per_req * page_size;
  const int max_chunks = max_pages_per_req * (page_size / DEC_CHUNK);
  p.max_splits = (max_chunks + chunks_per_split - 1) / chunks_per_split;
  if (p.max_splits > 65535 || R > 65535) return FFA_ERR_UNSUPPORTED;
  uintptr_t ws = (reinterpret_cast<uintptr_t>(workspace) + 127) & ~uintptr_t(127);
  p.o_part = reinterpret_cast<float*>(ws);
  p.lse_part = p.o_part + (size_t)R * p.max_splits * H * MLA_LAT;
  p.R = R;
  p.H = H;
  p.page_size = page_size;
  p.chunks_per_split = chunks_per_split;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.ec.err = dev_err;
  p.ec.limit_ns = wait_limit_ns();
  const CUtensorMapDataType dt =
      dtype == FFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t rows = (uint64_t)num_pages * page_size;
  // Boxes as tall as a page allows (and dividing the 128-token tile): fewer,
  // larger TMA requests.
  int br = 128;
  while (page_size % br) br /= 2;
  p.box_rows = br;
  CUtensorMap mc;
  int st = make_tmap_4d(&mc, ckv_pages, dt, 2, MLA_DK, rows, 1, 1, (uint64_t)MLA_DK * 2, rows * MLA_DK * 2,
                        rows * MLA_DK * 2, 64, br);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kern, auto merge) -> int {
    static std::atomic<uint64_t> done_b{0}, done_h{0};
    if (int e = smem_attr_once(kern, MLT_SMEM, dtype == FFA_DTYPE_BF16 ? done_b : done_h)) return e;
    kern<<<dim3(p.max_splits, R), MLT_THREADS, MLT_SMEM, s>>>(mc, p);
    int e = launch_status();
    if (e) return e;
    merge<<<R * H, 128, 0, s>>>(p.o_part, p.lse_part, ctx_lens, out_lat, lse, H, p.max_splits, chunks_per_split,
                                o_strides[0], o_strides[1]);
    return launch_status();
  };
  if (dtype == FFA_DTYPE_BF16)
    return launch(ffa_mla_decode_tc_kernel<__nv_bfloat16>, ffa_mla_merge_kernel<__nv_bfloat16>);
  return launch(ffa_mla_decode_tc_kernel<__half>, ffa_mla_merge_kernel<__half>);
}
