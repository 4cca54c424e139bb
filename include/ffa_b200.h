/*
 * ffa_b200.h — C ABI of the B200 (sm_100a) flash-attention kernels.
 *
 * Every entry point takes raw device pointers, element strides and sizes,
 * launches on the given CUDA stream (cudaStream_t passed as void*), never
 * throws, never allocates device memory, and returns an ffa_status.  Tensors
 * are row-major in their last dimension (stride 1); the other strides are in
 * elements.  The library is loaded by the Python package through ctypes and
 * can be bound the same way from any FFI (ctypes, cgo, JNI, N-API).
 *
 * Reference interfaces replaced (MindIntels/fastest_flash_attention, paths
 * relative to the project root):
 *   ffa_fwd            <- ops/attention_forward.py:23  fastest_flash_attn_forward
 *                         kernels/cpu_reference.py:132 flash_attn_cpu_forward
 *                         kernels/cpu_fa4.py:219       fa4_forward
 *                         kernels/triton_fwd.py:144, kernels/triton_ffpa.py:217
 *   ffa_bwd*           <- ops/attention_backward.py:19 fastest_flash_attn_backward
 *                         kernels/cpu_reference.py:319 flash_attn_cpu_backward
 *                         kernels/cpu_fa4.py:445       fa4_backward
 *                         kernels/triton_bwd.py:122
 *   ffa_paged_*        <- ops/kv_cache.py:170 PagedKVCache.append_tokens and
 *                         ops/kv_cache.py:208 get_kv + the forward it feeds
 *   ffa_mla_*          <- modules/flash_mla.py:116 FastestFlashMLA.forward
 *                         (absorbed latent form of the same attention)
 */
#ifndef FFA_B200_H_
#define FFA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  FFA_OK = 0,
  FFA_ERR_INVALID_ARG = 1,     /* bad shape / stride / alignment / pointer */
  FFA_ERR_UNSUPPORTED = 2,     /* valid request outside what the kernels cover */
  FFA_ERR_CUDA = 3,            /* a CUDA runtime/driver call failed */
  FFA_ERR_DEVICE_TIMEOUT = 4,  /* a bounded in-kernel wait expired (see ffa_read_error) */
  FFA_ERR_WORKSPACE = 5        /* workspace missing or too small */
} ffa_status;

/* F32 is accepted only where an entry point says so (ffa_fwd / ffa_bwd /
 * ffa_bwd_masked, and the MLA projections). */
typedef enum { FFA_DTYPE_F16 = 0, FFA_DTYPE_BF16 = 1, FFA_DTYPE_F32 = 2 } ffa_dtype;

/* Library version (major*10000 + minor*100 + patch). */
int ffa_version(void);

/* Last CUDA error string seen by the library on this thread (static storage). */
const char* ffa_last_error(void);

/* Device error word helpers: kernels record the site code of an expired wait
 * into a caller-provided uint32 in device memory (nullptr disables it), and
 * invalid data they find: 0x3E0 a decode context length outside
 * [0, max_pages_per_req * page_size], 0x3E1 a block-table page id outside
 * [0, num_pages), 0x1FF a block mask keeping more key tiles than the forward's
 * tile list holds (the offending loads are skipped; treat the call as failed).
 * ffa_read_error copies it to *out (synchronising `stream`). */
int ffa_read_error(const uint32_t* dev_err, uint32_t* out, void* stream);

/* Wall-clock limit (nanoseconds) applied to every in-kernel wait of later
 * launches on this host thread; default 2e9 (2 s). */
void ffa_set_wait_limit_ns(unsigned long long ns);

/* ----------------------------------------------------------------------------
 * Prefill / training forward.
 *   q  [B, Hq,  Sq,  D ]   k [B, Hkv, Skv, D]   v [B, Hkv, Skv, Dv]
 *   o  [B, Hq,  Sq,  Dv]   lse [B, Hq, Sq] fp32 (natural log), may be NULL
 * Strides are given as {batch, head, seq} in elements for each tensor.
 * GQA/MQA: Hq % Hkv == 0, query head h reads kv head h / (Hq / Hkv).
 * causal: key j is visible to query i iff j <= i + q_offset.
 * window > 0: key j visible iff j >= i + q_offset - window + 1.
 * softcap > 0: scores become softcap * tanh(score * scale / softcap).
 * block_mask (uint8 [n_br, n_bc], 1 = keep) masks every (query, key) pair whose
 *   (i / mask_bq, j / mask_bkv) entry is 0; NULL disables it.
 * D is the query/key head dim, Dv the value (and output) head dim.
 * Supported (D, Dv): (64, 64), (128, 128), (192, 128) — the last is the MLA
 * prefill shape (modules/flash_mla.py:96-152: 128 + 64 rotary dims, values
 * not padded).  dtype f16/bf16 (tensor cores), or f32: computed in fp32 on the
 * CUDA cores (FFMA register tiles, fp32 accumulation), as the reference
 * computes fp32 inputs (kernels/cpu_reference.py:28-32); q/k/v/o then need
 * 16-byte aligned bases and strides that are multiples of 4 elements.
 * ------------------------------------------------------------------------- */
int ffa_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int dtype, int B, int Hq,
            int Hkv, int Sq, int Skv, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
            const int64_t* v_strides, const int64_t* o_strides, float scale, int causal, int q_offset,
            int window, float softcap, const uint8_t* block_mask, int n_br, int n_bc, int mask_bq,
            int mask_bkv, uint32_t* dev_err, void* stream);

/* ----------------------------------------------------------------------------
 * Backward (deterministic: fixed summation order, no atomics; bit-identical
 * results run to run).  Replaces ops/attention_backward.py:19
 * fastest_flash_attn_backward -> kernels/cpu_reference.py:319 and
 * kernels/cpu_fa4.py:445.
 *   q, dq [B, Hq, Sq, D]; k, dk [B, Hkv, Skv, D]; v, dv [B, Hkv, Skv, Dv]
 *   dout, o [B, Hq, Sq, Dv]; lse [B, Hq, Sq] fp32 (natural log, from ffa_fwd)
 *   (GQA groups summed in order into dk / dv).  (D, Dv) in {(64, 64),
 *   (128, 128), (192, 128)}; the last is the MLA training shape.
 * Same mask / softcap semantics as ffa_fwd (no block mask: the reference
 * backward has none).  dtype f32 runs the fp32 CUDA-core backward (same
 * determinism; the workspace then holds Delta).  `workspace` must hold ffa_bwd_workspace_size() bytes
 * of device memory (padded base-2 LSE and Delta = rowsum(dO*O)).
 * Three kernel launches on `stream`: preprocess, dK/dV, dQ.
 * ------------------------------------------------------------------------- */
size_t ffa_bwd_workspace_size(int B, int Hq, int Sq);

int ffa_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
            void* dq, void* dk, void* dv, int dtype, int B, int Hq, int Hkv, int Sq, int Skv, int D, int Dv,
            const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
            const int64_t* o_strides, const int64_t* do_strides, const int64_t* dq_strides,
            const int64_t* dk_strides, const int64_t* dv_strides, float scale, int causal, int q_offset,
            int window, float softcap, void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream);

/* Backward with a block mask: ffa_bwd's arguments plus the forward's tile
 * mask (block_mask [n_br, n_bc] uint8, blocks of mask_bq queries x mask_bkv
 * keys, nonzero = kept; the same arguments ffa_fwd takes).  Masked (query,
 * key) pairs get P = 0, so the gradients are those of the masked forward.
 * The reference backward (kernels/cpu_reference.py:319-427) ignores the mask;
 * this defines it as the derivative of its masked forward (:220-224).
 * ffa_bwd is this call with block_mask = NULL. */
int ffa_bwd_masked(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
                   void* dq, void* dk, void* dv, int dtype, int B, int Hq, int Hkv, int Sq, int Skv, int D, int Dv,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                   const int64_t* o_strides, const int64_t* do_strides, const int64_t* dq_strides,
                   const int64_t* dk_strides, const int64_t* dv_strides, float scale, int causal, int q_offset,
                   int window, float softcap, const uint8_t* block_mask, int n_br, int n_bc, int mask_bq,
                   int mask_bkv, void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream);

/* ----------------------------------------------------------------------------
 * Allocation-free backward.  No counterpart in the reference: this entry
 * point exists for callers that cannot allocate device memory (code handed
 * only its input/output buffers by a host framework, or hosts that forbid a
 * device-synchronising cudaMalloc in the middle of a step).  Same arguments
 * and bit-identical results as ffa_bwd without the workspace and with Dv
 * fixed to D (so only D == Dv; the MLA shape D=192, Dv=128 is rejected with
 * FFA_ERR_UNSUPPORTED and needs ffa_bwd): the scratch rows live in an
 * array compiled into the library (8 MiB + 256 B held by every GPU that loads
 * it, until process exit).  Limit: B * Hq * round_up(Sq, 128) <=
 * FFA_BWD_NOALLOC_MAX_ROWS, else FFA_ERR_UNSUPPORTED.  All calls on a device
 * share the array, so calls whose kernels overlap on the GPU race.  The first
 * call on a device looks up the array's address; make it before any stream
 * capture.
 * ------------------------------------------------------------------------- */
#define FFA_BWD_NOALLOC_MAX_ROWS (1 << 20)

int ffa_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v, const void* o,
                    const float* lse, void* dq, void* dk, void* dv, int dtype, int B, int Hq, int Hkv, int Sq,
                    int Skv, int D, const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                    const int64_t* o_strides, const int64_t* do_strides, const int64_t* dq_strides,
                    const int64_t* dk_strides, const int64_t* dv_strides, float scale, int causal, int q_offset,
                    int window, float softcap, uint32_t* dev_err, void* stream);

/* ----------------------------------------------------------------------------
 * Paged-KV decode (one query token per request), split over the context and
 * merged by LSE.  Replaces ops/kv_cache.py:208 PagedKVCache.get_kv (page
 * gather) followed by ops/attention_forward.py:23 on the gathered K/V.
 *   q [R, Hq, D] (strides {request, head} in elements)
 *   k_pages, v_pages [num_pages, Hkv, page_size, D] contiguous (the
 *     reference's page pool layout, ops/kv_cache.py:142-149)
 *   block_table [R, max_pages_per_req] int32 page ids; ctx_lens [R] int32
 *   out [R, Hq, D] (strides {request, head}); lse [R, Hq] fp32 natural log
 *     (may be NULL)
 * page_size must be a multiple of 16; Hq / Hkv <= 16; D in {64, 128}.
 * chunks_per_split (16-token chunks per CTA; <= 0 selects 32) sets the split
 * size; `workspace` must hold ffa_paged_decode_workspace_size() bytes.
 * Two launches on `stream`: split kernel and merge kernel.
 * ------------------------------------------------------------------------- */
size_t ffa_paged_decode_workspace_size(int R, int Hq, int D, int max_pages_per_req, int page_size,
                                       int chunks_per_split);

int ffa_paged_decode(const void* q, const void* k_pages, const void* v_pages, const int* block_table,
                     const int* ctx_lens, void* out, float* lse, int dtype, int R, int Hq, int Hkv, int D,
                     int num_pages, int page_size, int max_pages_per_req, const int64_t* q_strides,
                     const int64_t* o_strides, float scale, float softcap, int chunks_per_split, void* workspace,
                     size_t workspace_bytes, uint32_t* dev_err, void* stream);

/* ----------------------------------------------------------------------------
 * MLA absorbed decode.  Replaces modules/flash_mla.py:116 FastestFlashMLA
 * forward for one new token per request (the reference re-runs the whole
 * prefix through up-projections; here W_UK is folded into the query and
 * W_UV applied to the latent output by the caller).  Multi-query attention
 * of H = 32 heads over a paged latent cache:
 *   q [R, H, 576] = [q_nope W_UK (512) | rope(q_rope) (64)] per head
 *   ckv_pages [num_pages, page_size, 576] = [c_kv (512) | rope(k_rope) (64)]
 *   out_lat [R, H, 512] = softmax(q . k * scale) c_kv; lse [R, H] (or NULL)
 * page_size multiple of 16; workspace from ffa_mla_decode_workspace_size().
 * ------------------------------------------------------------------------- */
size_t ffa_mla_decode_workspace_size(int R, int H, int max_pages_per_req, int page_size, int chunks_per_split);

int ffa_mla_decode(const void* q, const void* ckv_pages, const int* block_table, const int* ctx_lens, void* out_lat,
                   float* lse, int dtype, int R, int H, int num_pages, int page_size, int max_pages_per_req,
                   const int64_t* q_strides, const int64_t* o_strides, float scale, int chunks_per_split,
                   void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream);

/* ----------------------------------------------------------------------------
 * The projections on either side of the MLA absorbed decode, one launch each.
 * Replace modules/flash_mla.py:133-152 (q/k RoPE through the RotaryEmbedding
 * module, kv_up_proj of the whole prefix) for one new token per request:
 * W_UK / W_UV are the two halves of kv_up_proj.weight viewed [H, 2d, L].
 * in_dtype (activations, weights, o_absorb output): F32, BF16 or F16;
 * lat_dtype (decode query, latent output, cache rows): BF16 or F16.
 * RoPE is half-split with fp32 angles pos * inv_freq[i], i < rope/2.
 *
 * ffa_mla_q_absorb: out[r, h, :] = [q_nope[r, h] . W_UK[h] (L) |
 *   rope(q_rope[r, h], pos[r]) (rope)].  q_nope [R, H, d] strides {r, h};
 *   q_rope [R, H, rope] strides {r, h}; w_uk [H, d, L] strides {h, j};
 *   out [R, H, L + rope] strides {r, h}.  L multiple of 64, d <= 192.
 * ffa_mla_o_absorb: out[r, h (d + rope) + i] = o_lat[r, h] . W_UV[h, i] for
 *   i < d, and 0 for the rope columns (the reference's zero-padded V):
 *   o_proj's input rows.  o_lat [R, H, L] strides {r, h}; w_uv [H, d, L]
 *   strides {h, i}; out rows of stride out_row_stride.  L multiple of 32,
 *   L <= 1024.
 * ffa_mla_latent_append: rows[slots[t]] = [lat[t] (L) | rope(kr[t], pos[t])]
 *   for n_tokens tokens; rows [n_slots, L + rope] contiguous (the latent
 *   cache's pages viewed as rows); slots outside [0, n_slots) are skipped.
 * ------------------------------------------------------------------------- */
int ffa_mla_q_absorb(const void* q_nope, const int64_t* qn_strides, const void* q_rope, const int64_t* qr_strides,
                     const void* w_uk, const int64_t* w_strides, const int* pos, const float* inv_freq, void* out,
                     const int64_t* o_strides, int in_dtype, int lat_dtype, int R, int H, int d, int L, int rope,
                     void* stream);

int ffa_mla_o_absorb(const void* o_lat, const int64_t* ol_strides, const void* w_uv, const int64_t* w_strides,
                     void* out, int64_t out_row_stride, int in_dtype, int lat_dtype, int R, int H, int d, int L,
                     int rope, void* stream);

int ffa_mla_latent_append(const void* lat, int64_t lat_row_stride, const void* kr, int64_t kr_row_stride,
                          const int* pos, const int* slots, const float* inv_freq, void* rows, int64_t n_slots,
                          int in_dtype, int lat_dtype, int n_tokens, int L, int rope, void* stream);

/* ----------------------------------------------------------------------------
 * Paged-KV append: scatter new K/V tokens into their (page, offset) slots.
 * Replaces the per-token loop of ops/kv_cache.py:170-206
 * PagedKVCache.append_tokens (slot assignment stays on the host, where the
 * reference's FIFO page allocator lives).
 *   k_new, v_new [Hkv, n_tokens, D] (strides {head, token} in elements)
 *   slots [n_tokens] int32 = page * page_size + offset
 * ------------------------------------------------------------------------- */
int ffa_paged_append(const void* k_new, const void* v_new, void* k_pages, void* v_pages, const int* slots,
                     int dtype, int n_tokens, int Hkv, int D, int page_size, int num_pages,
                     const int64_t* new_strides, void* stream);

/* ----------------------------------------------------------------------------
 * Log-sum-exp merge of a partial attention result into a running one, for
 * the sequence-sharded ring (each step attends the local queries to one
 * rank's K/V block; the reference has no multi-GPU path, so this has no
 * counterpart there).  In place on (o_acc, lse_acc):
 *   L = logaddexp(L_acc, L_part);  O_acc = O_acc e^(L_acc-L) + O_part e^(L_part-L)
 *   o_acc [rows, D] fp32, lse_acc [rows] fp32 natural log (-inf = empty)
 *   o_part [rows, D] dtype (f16/bf16), lse_part [rows] fp32 natural log
 * ------------------------------------------------------------------------- */
int ffa_merge_partial(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part, int dtype,
                      int64_t rows, int D, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FFA_B200_H_ */
