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
constexpr int DEC_STAGES = 8;

struct DecParams {
  const void* q;      // [R, Hq, D]
  int64_t q_sr, q_sh;
  const int* block_table;
  int64_t bt_stride;  // elements between requests' rows of the block table
  const int* ctx_lens;
  float* o_part;      // [R, max_splits, Hq, D]
  float* lse_part;    // [R, max_splits, Hq] (base 2)
  int R, Hq, Hkv, G, page_size, max_splits, chunks_per_split;
  float scale_log2;
  float sc_pre, sc_post;
  int use_softcap;
  ErrCtx ec;
};

enum : uint32_t { SITE_DEC_FULL = 0x301, SITE_DEC_EMPTY = 0x302 };

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
  static constexpr int MERGE_OFF = DEC_STAGES * STAGE;   // per-warp m, l, O for the CTA merge
  static constexpr int MERGE_BYTES = DEC_CONSUMERS * 16 * (D + 2) * 4;
  static constexpr int BAR_OFF = MERGE_OFF + MERGE_BYTES;
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
  const int ns = (n_chunks + chunks_per_split - 1) / chunks_per_split;
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
  static bool set = false;
  if (!set) {
    int s = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    if (s) return s;
    set = true;
  }
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
// (split, request); the chunk of 16 tokens x 576 values is loaded once and
// serves as both K and V.  The 4 consumer warps split Q.K^T over the key
// dims (partial scores summed through smem in MMA-fragment order, so no
// layout change) and split O over the value dims.
// ---------------------------------------------------------------------------
constexpr int MLA_LAT = 512, MLA_ROPE = 64, MLA_DK = MLA_LAT + MLA_ROPE;
constexpr int MLA_HEADS = 32;  // two m16 tiles of query heads per CTA
constexpr int MLA_STAGES = 4;
constexpr int MLA_BOXES = MLA_DK / 64;           // 9 swizzled 64-column boxes per chunk
constexpr int MLA_STAGE = MLA_BOXES * DEC_CHUNK * 128;  // 18 KB
constexpr int MLA_KSTEPS = MLA_DK / 16 / DEC_CONSUMERS;  // 9 k-steps of the scores per warp
constexpr int MLA_XS_OFF = MLA_STAGES * MLA_STAGE;
constexpr int MLA_XS_BYTES = 2 * DEC_CONSUMERS * 32 * 16 * 4;
constexpr int MLA_BAR_OFF = MLA_XS_OFF + MLA_XS_BYTES;
constexpr int MLA_SMEM = MLA_BAR_OFF + 256 + 1024;

struct MlaParams {
  const void* q;  // [R, H, 576] = [q_lat | q_rope]
  int64_t q_sr, q_sh;
  const int* block_table;
  int64_t bt_stride;
  const int* ctx_lens;
  float* o_part;    // [R, max_splits, H, 512]
  float* lse_part;  // [R, max_splits, H] (base 2)
  int R, H, page_size, max_splits, chunks_per_split;
  float scale_log2;
  ErrCtx ec;
};

template <typename T>
__global__ void __launch_bounds__(DEC_THREADS)
    ffa_mla_decode_kernel(const __grid_constant__ CUtensorMap tmC, const MlaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + MLA_BAR_OFF);
  uint64_t* empty = full + MLA_STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + MLA_STAGES);
  float* xs = reinterpret_cast<float*>(smem + MLA_XS_OFF);

  const int split = blockIdx.x, r = blockIdx.y;
  const int ctx = p.ctx_lens[r];
  const int n_chunks = (ctx + DEC_CHUNK - 1) / DEC_CHUNK;
  const int c_begin = split * p.chunks_per_split;
  if (c_begin >= n_chunks) return;
  const int n = min(n_chunks, c_begin + p.chunks_per_split) - c_begin;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int sub_per_page = p.page_size / DEC_CHUNK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < MLA_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], DEC_CONSUMERS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == DEC_CONSUMERS) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const int* table = p.block_table + (int64_t)r * p.bt_stride;
      int issued = 0;
      for (int idx = 0; idx < n; ++idx) {
        const int s = idx % MLA_STAGES, use = idx / MLA_STAGES;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, p.ec, abort_flag, SITE_DEC_EMPTY)) break;
        const int c = c_begin + idx;
        const int row = table[c / sub_per_page] * p.page_size + (c % sub_per_page) * DEC_CHUNK;
        mbar_arrive_expect_tx(&full[s], MLA_STAGE);
        uint8_t* dst = smem + s * MLA_STAGE;
#pragma unroll
        for (int bx = 0; bx < MLA_BOXES; ++bx)
          tma_load_4d(&tmC, &full[s], dst + bx * DEC_CHUNK * 128, bx * 64, row, 0, 0, pol);
        ++issued;
      }
      if (*abort_flag)
        for (int q = max(0, issued - MLA_STAGES); q < issued; ++q)
          mbar_wait(&full[q % MLA_STAGES], (q / MLA_STAGES) & 1, p.ec, abort_flag, SITE_DEC_FULL, true);
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, mr = lane & 7;
  // This warp's slice of Q (k-steps 9w .. 9w+8) for both 16-head row tiles.
  uint32_t qa[MLA_KSTEPS][2][4];
  {
    const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)r * p.q_sr;
#pragma unroll
    for (int i = 0; i < MLA_KSTEPS; ++i) {
      const int d = (warp * MLA_KSTEPS + i) * 16 + 2 * t;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const T* qr = qb + (int64_t)(mt * 16 + g + 8 * hi) * p.q_sh + d;
          qa[i][mt][hi] = *reinterpret_cast<const uint32_t*>(qr);
          qa[i][mt][2 + hi] = *reinterpret_cast<const uint32_t*>(qr + 8);
        }
    }
  }
  float o[2][16][4];  // [row tile][8-dim n-tile of this warp's 128 value dims][frag]
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < 16; ++i) o[mt][i][0] = o[mt][i][1] = o[mt][i][2] = o[mt][i][3] = 0.f;
  float m_r[2][2] = {{-INFINITY, -INFINITY}, {-INFINITY, -INFINITY}};  // [row tile][lo/hi]
  float l_r[2][2] = {{0.f, 0.f}, {0.f, 0.f}};

  bool ok = true;
  for (int idx = 0; idx < n; ++idx) {
    const int s = idx % MLA_STAGES;
    // No early exit: every consumer warp must reach the named barrier below
    // once per chunk.  After an expired wait (abort) the waits return at
    // once and the stale smem is only read, so the loop drains quickly; the
    // error word reports the failure.
    ok = mbar_wait(&full[s], (idx / MLA_STAGES) & 1, p.ec, abort_flag, SITE_DEC_FULL) && ok;
    __syncwarp();
    const uint32_t cbase = smem_u32(smem + s * MLA_STAGE);
    float sc[2][2][4];  // [row tile][token n-tile][frag]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.f;
#pragma unroll
    for (int i = 0; i < MLA_KSTEPS; ++i) {
      const int kk = warp * MLA_KSTEPS + i;
      const int bx = kk / 4, ch = 2 * (kk % 4) + (mi & 1), tok = mr + 8 * (mi >> 1);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(sw128(cbase + bx * DEC_CHUNK * 128, tok, ch), b00, b01, b10, b11);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        mma16816<T>(sc[mt][0], qa[i][mt], b00, b01);
        mma16816<T>(sc[mt][1], qa[i][mt], b10, b11);
      }
    }
    // Sum the four warps' partial scores (same fragment positions in every warp).
    float* xw = xs + ((idx & 1) * DEC_CONSUMERS + warp) * 32 * 16 + lane * 16;
#pragma unroll
    for (int e = 0; e < 16; ++e) xw[e] = sc[e / 8][(e / 4) % 2][e % 4];
    asm volatile("bar.sync 1, %0;" ::"n"(DEC_CONSUMERS * 32) : "memory");
    float x[2][2][4];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < DEC_CONSUMERS; ++w) v += xs[((idx & 1) * DEC_CONSUMERS + w) * 32 * 16 + lane * 16 + e];
      const int nt = (e / 4) % 2;
      const int tok = (c_begin + idx) * DEC_CHUNK + nt * 8 + 2 * t + (e & 1);
      x[e / 8][nt][e % 4] = tok < ctx ? v * p.scale_log2 : -INFINITY;
    }
    // online softmax per row (identical in every warp)
    uint32_t pa[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float mx_lo = fmaxf(fmaxf(x[mt][0][0], x[mt][0][1]), fmaxf(x[mt][1][0], x[mt][1][1]));
      float mx_hi = fmaxf(fmaxf(x[mt][0][2], x[mt][0][3]), fmaxf(x[mt][1][2], x[mt][1][3]));
#pragma unroll
      for (int off = 1; off < 4; off <<= 1) {
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
        mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
      }
      const float mn_lo = fmaxf(m_r[mt][0], mx_lo), mn_hi = fmaxf(m_r[mt][1], mx_hi);
      if (__any_sync(0xffffffffu, mn_lo > m_r[mt][0] + 8.f || mn_hi > m_r[mt][1] + 8.f)) {
        const float a_lo = (mn_lo == -INFINITY) ? 1.f : ex2(m_r[mt][0] - mn_lo);
        const float a_hi = (mn_hi == -INFINITY) ? 1.f : ex2(m_r[mt][1] - mn_hi);
        l_r[mt][0] *= a_lo;
        l_r[mt][1] *= a_hi;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[mt][i][0] *= a_lo;
          o[mt][i][1] *= a_lo;
          o[mt][i][2] *= a_hi;
          o[mt][i][3] *= a_hi;
        }
        m_r[mt][0] = mn_lo;
        m_r[mt][1] = mn_hi;
      }
      const float u_lo = (m_r[mt][0] == -INFINITY) ? 0.f : m_r[mt][0];
      const float u_hi = (m_r[mt][1] == -INFINITY) ? 0.f : m_r[mt][1];
      float pr[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        pr[nt][0] = ex2(x[mt][nt][0] - u_lo);
        pr[nt][1] = ex2(x[mt][nt][1] - u_lo);
        pr[nt][2] = ex2(x[mt][nt][2] - u_hi);
        pr[nt][3] = ex2(x[mt][nt][3] - u_hi);
        l_r[mt][0] += pr[nt][0] + pr[nt][1];
        l_r[mt][1] += pr[nt][2] + pr[nt][3];
      }
      pa[mt][0] = pack2<T>(pr[0][0], pr[0][1]);
      pa[mt][1] = pack2<T>(pr[0][2], pr[0][3]);
      pa[mt][2] = pack2<T>(pr[1][0], pr[1][1]);
      pa[mt][3] = pack2<T>(pr[1][2], pr[1][3]);
    }
    // O[:, 128w .. 128w+127] += P V  (V = the chunk's latent columns)
#pragma unroll
    for (int nt = 0; nt < 16; nt += 2) {
      const int d = warp * 128 + nt * 8;
      const int bx = d / 64, ch = (d % 64) / 8 + (mi >> 1), tok = mr + 8 * (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sw128(cbase + bx * DEC_CHUNK * 128, tok, ch), b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        mma16816<T>(o[mt][nt], pa[mt], b0, b1);
        mma16816<T>(o[mt][nt + 1], pa[mt], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // Full row sums, then this warp's value dims of the split result.
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hi = 0; hi < 2; ++hi)
#pragma unroll
      for (int off = 1; off < 4; off <<= 1) l_r[mt][hi] += __shfl_xor_sync(0xffffffffu, l_r[mt][hi], off);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      const int head = mt * 16 + g + 8 * hi;
      const int64_t pidx = ((int64_t)r * p.max_splits + split) * p.H + head;
      const float L = l_r[mt][hi];
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float* dst = p.o_part + pidx * MLA_LAT + warp * 128;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
        *reinterpret_cast<float2*>(dst + nt * 8 + 2 * t) =
            make_float2(o[mt][nt][2 * hi] * inv, o[mt][nt][2 * hi + 1] * inv);
      if (warp == 0 && t == 0) p.lse_part[pidx] = (L > 0.f) ? m_r[mt][hi] + lg2(L) : -INFINITY;
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
  if ((q_strides[1] % 2) || (q_strides[0] % 2) || (reinterpret_cast<uintptr_t>(q) & 3)) return FFA_ERR_INVALID_ARG;
  const size_t need = ffa_mla_decode_workspace_size(R, H, max_pages_per_req, page_size, chunks_per_split);
  if (!workspace || workspace_bytes < need) return FFA_ERR_WORKSPACE;
  MlaParams p{};
  p.q = q;
  p.q_sr = q_strides[0];
  p.q_sh = q_strides[1];
  p.block_table = block_table;
  p.bt_stride = max_pages_per_req;
  p.ctx_lens = ctx_lens;
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
  CUtensorMap mc;
  int st = make_tmap_4d(&mc, ckv_pages, dt, 2, MLA_DK, rows, 1, 1, (uint64_t)MLA_DK * 2, rows * MLA_DK * 2,
                        rows * MLA_DK * 2, 64, DEC_CHUNK);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kern, auto merge) -> int {
    static bool set_b = false, set_h = false;
    bool& set = (dtype == FFA_DTYPE_BF16) ? set_b : set_h;
    if (!set) {
      int e = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MLA_SMEM));
      if (e) return e;
      set = true;
    }
    kern<<<dim3(p.max_splits, R), DEC_THREADS, MLA_SMEM, s>>>(mc, p);
    int e = launch_status();
    if (e) return e;
    merge<<<(R * H * 32 + 255) / 256, 256, 0, s>>>(p.o_part, p.lse_part, ctx_lens, out_lat, lse, R, H, p.max_splits,
                                                  chunks_per_split, o_strides[0], o_strides[1]);
    return launch_status();
  };
  if (dtype == FFA_DTYPE_BF16)
    return launch(ffa_mla_decode_kernel<__nv_bfloat16>, ffa_decode_merge_kernel<__nv_bfloat16, MLA_LAT>);
  return launch(ffa_mla_decode_kernel<__half>, ffa_decode_merge_kernel<__half, MLA_LAT>);
}
