/*
 * flashdllm_b200.h -- C ABI of the B200 (sm_100a) Flash-Cache / Flash-Verify
 * hot path for LLaDA-style masked-diffusion decoding.
 *
 * Every entry point takes raw device pointers, plain integer sizes and a
 * cudaStream_t, launches asynchronously on that stream and returns an
 * fdllm status code (0 = success).  Host-side argument checks return
 * FDLLM_ERR_ARG before anything is launched.  Device-side problems (a cache
 * slot or key index out of range, a malformed block table, a bounded wait
 * that ran out) skip the offending access and are recorded in a per-process
 * device status word that fdllm_status_read() returns and clears.
 *
 * Tensors are row-major and contiguous unless a leading dimension is given.
 * "bf16" means __nv_bfloat16 / torch.bfloat16.  The library allocates no
 * device memory: callers pass workspaces sized by the *_workspace_bytes()
 * queries.  A QKV workspace is zero-filled once before first use and the
 * kernels leave it ready for the next call, except after a call whose device
 * status reported an error: zero it again before reusing it.
 *
 * Citations "ref file:line" name the reference interface each entry point
 * replaces (VILA-Lab/Flash-dLLM).
 */
#ifndef FLASHDLLM_B200_H
#define FLASHDLLM_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FDLLM_OK 0
#define FDLLM_ERR_ARG 1       /* invalid size, pointer or unsupported shape (host check) */
#define FDLLM_ERR_CUDA 2      /* a CUDA runtime call or kernel launch failed */
#define FDLLM_ERR_INDEX 3     /* device: cache slot / key / row index out of range */
#define FDLLM_ERR_TIMEOUT 4   /* device: a bounded wait ran out */
#define FDLLM_ERR_TABLE 5     /* device: malformed block table */
#define FDLLM_ERR_WORKSPACE 6 /* workspace too small */
#define FDLLM_ERR_DRIVER 7    /* TMA descriptor encode unavailable or failed */
#define FDLLM_ERR_SCRATCH_LIMIT 8 /* request needs more scratch than the library's fixed array holds */
#define FDLLM_ERR_RANGE 9     /* device: an attention-score column sum non-finite or beyond 2^24 in magnitude */

/* Library version string. */
const char* fdllm_version(void);

/* Human-readable name of a status code. */
const char* fdllm_error_string(int code);

/* Synchronise `stream`, copy the device status word of the current device
 * into out[0..3] = {first error code, info, kernel id, 0} and clear it.
 * No reference counterpart (the reference has no error reporting). */
int fdllm_status_read(int32_t out[4], cudaStream_t stream);

/* RMSNorm as the reference's RMSLayerNorm: y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))),
 * x/w/y bf16, rows x dim.  ref llada/model/modeling_llada.py:389-403 (called as
 * self.attn_norm(x) at llada/flash_cache_triton.py:494). */
int fdllm_rmsnorm(const void* x, const void* weight, void* y, int32_t rows, int32_t dim, float eps,
                  cudaStream_t stream);

/* Residual add fused with the next RMSNorm: y = bf16(x + residual), h = RMSNorm(y) with the rounding
 * points of fdllm_rmsnorm; x, residual, y, h bf16 [rows, dim] (dim <= 4096).
 * ref llada/flash_cache_triton.py:618-627 (x + dropout(att); ff_norm(x)). */
int fdllm_add_rmsnorm(const void* x, const void* residual, const void* weight, void* y, void* h, int32_t rows,
                      int32_t dim, float eps, cudaStream_t stream);

/* SwiGLU product out = bf16(silu(gate)) * up (silu in fp32): gate and up are [rows, cols] bf16 with row
 * stride ld_in elements (e.g. the two column halves of one [rows, 2*cols] GEMM output), out is contiguous
 * [rows, cols]; cols and ld_in multiples of 8.
 * ref llada/flash_cache_triton.py:628-633 (act(ff_proj(x)) * up_proj(x)). */
int fdllm_swiglu(const void* gate, const void* up, void* out, int64_t rows, int32_t cols, int64_t ld_in,
                 cudaStream_t stream);

/* Override the QKV kernel's plan (tuning and tests; not thread-safe against concurrent calls).
 * impl -1 = automatic (the stream-K GEMM at every row count), 0 = the stream-K GEMM (tile width and ring
 * from fdllm_gemm_set_plan), 1 = the earlier whole-tile kernels, where bn = tile width 64 or 128 columns (0: automatic), splits = K splits
 * (0 or 1: none), ksub = 64-wide K sub-tiles per ring slot 1 or 2 (0: automatic), pair = CTA-pair
 * kernel above 128 rows: 1 on, 0 off, -1 automatic.  The initial values come from the
 * FDLLM_QKV_IMPL / _BN / _SPLITS / _KSUB / _PAIR environment variables, read once.  The workspace
 * query follows the current plan.  No reference counterpart (the reference's tile sizes are Triton
 * constexprs). */
int fdllm_qkv_set_plan(int32_t impl, int32_t bn, int32_t splits, int32_t ksub, int32_t pair);

/* Override the stream-K GEMM's plan (tuning and tests): bn = single-CTA tile width 128 or 256
 * columns, ksub = 64-wide K sub-tiles per ring stage 1 or 2, grid = CTAs or CTA pairs (at most
 * what is resident at once), pair = CTA-pair kernel with 256 x 256 tiles: 1 on, 0 off, -1
 * automatic (pairs above 128 rows); dp = 1: one whole tile per CTA (no stream-K pieces) when the
 * tiles fit the grid, 2: every tile split stream-K, 0 = automatic (whole-tile waves after a
 * stream-K region of the remaining tiles when there are at least as many tiles as CTAs, else
 * stream-K).  Initial values from FDLLM_GEMM_BN / _KSUB / _GRID / _PAIR / _DP, read once.  No
 * reference counterpart. */
int fdllm_gemm_set_plan(int32_t bn, int32_t ksub, int32_t grid, int32_t pair, int32_t dp);

/* Workspace (bytes) of fdllm_gemm_bf16 (swiglu = 0; n_cols = output columns) or
 * fdllm_gemm_swiglu (swiglu = 1; n_cols = 2 * hidden): stream-K flags and one fp32 partial
 * accumulator per CTA.  Zero-filled once before first use; the kernel leaves it ready for the next
 * call (after a call whose device status reported an error, zero it again). */
size_t fdllm_gemm_workspace_bytes(int32_t n_rows, int32_t n_cols, int32_t k_dim, int32_t swiglu);

/* out[r, c] = bf16(sum_k a[r, k] * w[c, k] (+ residual[r, c])) for r < n_rows, c < n_cols:
 * a bf16 [n_rows, k_dim] (row stride k_dim), w bf16 [n_cols, k_dim] (nn.Linear weight, no bias),
 * out / residual bf16 with row strides ld_out / ld_res elements (residual may be NULL).  The sum
 * is fp32 and rounded once (as torch.addmm).  n_cols a multiple of 32, k_dim of 64.  Persistent
 * stream-K tcgen05 GEMM (one CTA per SM).
 * ref llada/flash_cache_triton.py:618-627, 634-636 (attn_out + residual, ff_out + residual) and
 * llada/model/modeling_llada.py:1484 (the LM head, no residual). */
int fdllm_gemm_bf16(const void* a, const void* w, void* out, const void* residual, int32_t n_rows, int32_t n_cols,
                    int32_t k_dim, int64_t ld_out, int64_t ld_res, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream);

/* SwiGLU MLP input projection in one GEMM: w_gate_up bf16 [2 * hidden, k_dim] is ff_proj's weight
 * stacked over up_proj's; out bf16 [n_rows, hidden] (row stride ld_out) =
 * bf16(bf16(silu(bf16(a W_gate^T))) * bf16(a W_up^T)), silu in fp32 -- the rounding points of
 * act(ff_proj(x)) * up_proj(x) in bf16.  hidden a multiple of 128, k_dim of 64.  The gate and up
 * activations stay in TMEM.  ref llada/flash_cache_triton.py:628-633. */
int fdllm_gemm_swiglu(const void* a, const void* w_gate_up, void* out, int32_t n_rows, int32_t hidden, int32_t k_dim,
                      int64_t ld_out, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Workspace (bytes) fdllm_qkv_rope_cache / fdllm_verify_qkv need for n_rows query rows. */
size_t fdllm_qkv_workspace_bytes(int32_t n_rows, int32_t d_model, int32_t n_heads);

/* Fused QKV projection + RoPE + KV-cache scatter (tcgen05/TMEM GEMM fed by TMA).
 *   xn        bf16 [n_rows, d_model]   RMS-normed hidden states of the query rows
 *   wq,wk,wv  bf16 [d_model, d_model]  nn.Linear weights (out, in), no bias
 *   pos       int64 [n_rows]           flat cache slot of each query row
 *   rope_sin, rope_cos  fp32 [n_slots, head_dim]  tables indexed by flat slot
 *   q_out     bf16 [n_rows, d_model]   RoPE'd Q, row-indexed
 *   k_cache, v_cache  bf16 [n_slots, d_model]  RoPE'd K and plain V are written to row pos[r]
 * head_dim = d_model / n_heads must be 128.  Rows [0, n_rows) are processed:
 * the caller passes the row span its block table covers.
 * ref llada/flash_cache_triton.py:15-100 (_flash_qkv_proj_cache_fwd) and its launch at :541-559. */
int fdllm_qkv_rope_cache(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                         const float* rope_sin, const float* rope_cos, void* q_out, void* k_cache, void* v_cache,
                         int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream);

/* fdllm_qkv_rope_cache for callers that cannot allocate device memory (for example a runtime
 * whose device memory is owned by another component, or a plugin that may not call cudaMalloc
 * once loaded): same arguments and results minus the workspace, whose role is taken by a fixed
 * 24 MiB array inside the library (held on every GPU that loads it until exit).  No counterpart
 * in the reference.  Calls needing more split-K scratch than that (d_model 4096: more than 128
 * rows with a requested K split) return FDLLM_ERR_SCRATCH_LIMIT without launching; the partial
 * sums of the CTA-pair kernel (129-256 rows, one 128 KB slot per CTA) fit.  The first call on a
 * device looks up the array's address; make it before any stream capture.  Calls share the
 * array; its counter / flag region (split-K tile counters, CTA-pair handoff flags) is zeroed on
 * entry of every call that uses it, so a call that ended on a device error leaves nothing stale
 * behind.  Calls that overlap on the GPU race on the array: serialise them.  Allocates nothing. */
int fdllm_qkv_rope_cache_noalloc(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                                 const float* rope_sin, const float* rope_cos, void* q_out, void* k_cache,
                                 void* v_cache, int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots,
                                 cudaStream_t stream);

/* Verify-query projection: same math as fdllm_qkv_rope_cache, but Q, K and V are all written
 * row-indexed to q_out/k_out/v_out (bf16 [n_rows, d_model]); the cache is not touched.
 * ref llada/flash_cache_triton.py:255-338 (_flash_verify_qkv_proj_fwd) and its launch at :505-519. */
int fdllm_verify_qkv(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                     const float* rope_sin, const float* rope_cos, void* q_out, void* k_out, void* v_out,
                     int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace,
                     size_t workspace_bytes, cudaStream_t stream);

/* Work-item capacity of an attention plan for n_rows query rows of batch_size sequences
 * (ceil(n_rows/64) + batch_size), and its size in bytes (header, items, and a per-sequence
 * section the score reduction reads). */
int fdllm_attn_plan_capacity(int32_t n_rows, int32_t batch_size);
size_t fdllm_attn_plan_bytes(int32_t n_rows, int32_t batch_size);

/* Build the attention work list from the reference's block tables (device int64 [n, 4] rows
 * (seq, k_end, q_start, q_end); masked tiles first in the row space, then tracked tiles).
 * Each work item is up to 64 query rows of one sequence (its masked rows first), so one pass
 * over the sequence's K/V serves masked and tracked rows together.  Malformed tables
 * (k_end outside (0, seqlen_max], a tile taller than block_m, more than one masked tile per
 * sequence, tracked tiles of a sequence not contiguous, tiles of one sequence with different
 * k_end) are reported as FDLLM_ERR_TABLE and yield an empty plan.
 * ref llada/generate.py:52-58,146-163,439-465 (make_blocks / block tables) as consumed by
 * llada/flash_cache_triton.py:561-607. */
int fdllm_plan_cache_attention(const int64_t* masked_blocks, int32_t n_masked, const int64_t* tracked_blocks,
                               int32_t n_tracked, int32_t n_rows, int32_t batch_size, int32_t block_m,
                               int32_t seqlen_max, void* plan, size_t plan_bytes, cudaStream_t stream);

/* Workspace (bytes) fdllm_attn_cache needs when it accumulates attn_scores: a 64-bit fixed-point
 * accumulator of seqlen_max entries and an arrival counter per sequence (max_items =
 * fdllm_attn_plan_capacity(...) bounds the batch).  Zero-filled once before first use; every call
 * leaves it zeroed again (after a call whose device status reported an error, zero it again). */
size_t fdllm_attn_workspace_bytes(int32_t max_items, int32_t n_heads, int32_t seqlen_max);

/* Block-table scheduled attention over the KV cache for masked + tracked rows.
 *   q          bf16 [n_rows, d_model];  o  bf16 [n_rows, d_model]
 *   k_cache, v_cache  bf16 [n_slots, d_model].  Without a page table, sequence b owns rows
 *              [b*seqlen_max, b*seqlen_max + k_end) (the reference's layout).  With one
 *              (page_table int32 [batch, pages_per_seq], pages_per_seq * 64 >= seqlen_max), key n
 *              of sequence b is row page_table[b*pages_per_seq + n/64]*64 + n%64; a page outside
 *              the cache is reported as FDLLM_ERR_INDEX and read as row 0.
 *   plan       from fdllm_plan_cache_attention; max_items = fdllm_attn_plan_capacity(...)
 *   attn_scores  fp32 [batch*seqlen_max] (logical slots) or NULL: when given, for every key n of
 *              sequence b, attn_scores[b*seqlen_max + n] += score_scale * sum over masked rows and
 *              heads of the raw (unscaled) q.k logit -- the reference's S tensor + S.mean((0,1))
 *              fused.  Per (item, head) column sums (fp32, from the tensor cores) are added in
 *              2^-32 fixed point with 64-bit integer atomics -- exact and order-independent, so the
 *              scores are the same on every run -- and converted once per sequence by the last
 *              CTA to finish it.  A column sum that is non-finite or reaches 2^24 in magnitude is
 *              reported as FDLLM_ERR_RANGE (and left out).
 *   kv_splits  split of each item's key range over CTAs: 1 = none; 2, 4 or 8 (other counts round
 *              down) run as one cluster of CTAs per item pair, merged in distributed shared memory
 * ref llada/flash_cache_triton.py:103-252 (_flash_masked_attention_fwd, _flash_tracked_attention_fwd)
 * and :538, :614-615 (S and attn_scores); the page table has no reference counterpart (the reference
 * addresses start_n = batch_id * SEQLEN_MAX, :122 and :202). */
int fdllm_attn_cache(const void* q, void* o, const void* k_cache, const void* v_cache, const void* plan,
                     int32_t max_items, float* attn_scores, float score_scale, int32_t d_model, int32_t n_heads,
                     int32_t seqlen_max, int64_t n_slots, float softmax_scale, int32_t kv_splits,
                     const int32_t* page_table, int32_t pages_per_seq, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream);

/* Flash-Verify attention: rows [q_s, q_e) of verify block row b = (k_s, k_e, q_s, q_e) (int32
 * [n_blocks, 4]) attend to cache rows pos_k[k_s:k_e] (gathered) and to their own block's fresh
 * k1/v1 rows under attn_mask (bool/uint8 [n_blocks*block_rows, block_rows]); block_rows = 2*block_m.
 * The in-block part is merged with a re-stabilised online softmax (the reference reuses the
 * cache part's running max, which yields NaN rows when a sequence has no cache keys).  kv_splits
 * as for fdllm_attn_cache; workspace / workspace_bytes are reserved (may be NULL / 0).
 * ref llada/flash_cache_triton.py:341-428 (_flash_verify_attention_fwd) and its launch at :521-535. */
int fdllm_verify_attn(const void* q1, const void* k1, const void* v1, void* o, const void* k_cache,
                      const void* v_cache, const int64_t* pos_k, int64_t n_pos_k, const uint8_t* attn_mask,
                      const int32_t* verify_blocks, int32_t n_blocks, int32_t block_rows, int32_t n_rows,
                      int32_t d_model, int32_t n_heads, int64_t n_slots, float softmax_scale, int32_t kv_splits,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* fp64 softmax statistics of logit rows (bf16 [n_rows, ld], vocab used columns): for row r
 * p_max[r] = max_v softmax(row)_v computed in fp64, argmax[r] = first index of the maximum, and
 * when p_tok != NULL, p_tok[r] = softmax(row)[tokens[r]].
 * ref llada/generate.py:218-219, 320-321, 337-338 (F.softmax(logits.to(float64)) + max / gather). */
int fdllm_row_stats(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab, const int64_t* tokens,
                    double* p_max, int64_t* argmax, double* p_tok, cudaStream_t stream);

/* Confidence acceptance of the masked window, batched over sequences (one warp each).
 * full_pos is int64 [batch_slots, lmax]; x and x_draft hold batch_slots * lmax tokens.
 * seq_info int64 [batch, 4] = (row offset into p/tok/window, window length n <= 256, flat index
 * slot * lmax + num_decoded into full_pos, predicted_length as a flat slot).  For sequence j:
 * probabilities of window slots >= predicted_length are zeroed
 * when eos_known[j]; the window is ordered by descending probability (ties keep window order);
 * keep = min(n, max(#(p >= threshold), min_keep)); full_pos row at the given flat index receives
 * the ordered window slots;
 * x[slot] = token for the first keep slots; x_draft[slot] = token for every window slot when
 * x_draft != NULL.  Outputs keep_out, length_out (slots before predicted_length) and eos_out (largest
 * committed slot holding eos_id, else -1).
 * ref llada/generate.py:215-251 (verify stage 1) and :335-361 (Flash-Cache acceptance). */
int fdllm_window_accept(const double* p, const int64_t* tok, const int64_t* window, const int64_t* seq_info,
                        const int32_t* eos_known, int32_t batch, int64_t batch_slots, int64_t lmax, double threshold,
                        int32_t min_keep, int64_t eos_id, int64_t* full_pos, int64_t* x, int64_t* x_draft,
                        int32_t* keep_out, int32_t* length_out, int64_t* eos_out, cudaStream_t stream);

/* Flash-Verify acceptance scan, batched over sequences.  seq_info int64 [batch, 4] = (row offset
 * into p/draft_tok/draft_slot, number of drafts S, unused, predicted_length); x holds n_slots tokens.  p[i] is the
 * mask-view probability of draft i; drafts at slots >= predicted_length count as 0 when
 * eos_known[j]; keep = #(cumprod(p) >= gamma) with the product taken sequentially; the first keep
 * drafts are committed to x.  ref llada/generate.py:312-333, 352-361. */
int fdllm_verify_accept(const double* p, const int64_t* draft_tok, const int64_t* draft_slot,
                        const int64_t* seq_info, const int32_t* eos_known, int32_t batch, int64_t n_slots,
                        double gamma, int64_t eos_id, int64_t* x, int32_t* keep_out, int64_t* eos_out,
                        cudaStream_t stream);

/* Flash-Cache forward inputs of one step, built on the device from per-sequence scalars.
 * seq int64 [n_seq, 16] = (slot row j, k_end, num decoded nd, predicted length, masked range start,
 * masked count, tracked range 1 start, count, tracked range 2 start, count, masked row offset,
 * tracked row offset, masked tile offset, tracked tile offset, 0, 0); range starts index row j of
 * full_pos (int64 [n_seq rows of lmax], the slot order); x int64 [n_slots].  Writes the sequence's
 * query rows to qpos / xq (slots and tokens; masked rows at the masked row offset, tracked rows,
 * range 1 then 2, at the tracked row offset), its block-table rows (seq, k_end, row begin, row end)
 * as tiles of bm rows at the tile offsets of tables int64 [tiles, 4], and seq_info int64 [n_seq, 4] =
 * (masked row offset, masked count, j * lmax + nd, predicted length) for fdllm_window_accept.
 * Positions outside row j are reported as FDLLM_ERR_INDEX.
 * ref llada/generate.py:52-58 (make_blocks), :146-163 and :439-465 (masked / tracked block tables). */
int fdllm_cache_build(const int64_t* seq, int32_t n_seq, int32_t bm, int64_t lmax, int64_t n_slots,
                      const int64_t* full_pos, const int64_t* x, int64_t* tables, int64_t* qpos, int64_t* xq,
                      int64_t* seq_info, cudaStream_t stream);

/* Flash-Verify forward inputs of one step, built on the device from per-sequence scalars.
 * seq int64 [n_seq, 8] = (slot row j, drafts s <= bm, num decoded nd, seqlen_k, predicted length,
 * key offset, draft offset, unused); the offsets are the running sums of the key counts
 * max(nd - t, 0) + max(seqlen_k - nd - s, 0) (t = 2 bm - 2 s) and of s.  full_pos int64 [n_seq rows of
 * lmax] (the slot order), x / x_draft int64 [n_slots].  Writes per sequence k: qpos / xv int64
 * [k * 2bm .. + 2bm) (verify rows' slots and tokens: t decoded slots before nd, the s drafts from
 * x_draft, the same s slots from x), mask uint8 [2bm rows x 2bm] (the verify mask), kpos int64 (its
 * keys: slots full_pos[j, 0:nd - t] and full_pos[j, nd + s:seqlen_k]), dslot / lidx int64 [s] (the
 * drafts' slots and logit rows), vblocks int32 [4] (key begin, key end, row begin, row end) and
 * info2 int64 [4] (draft offset, s, 0, predicted length).  Indices outside the sequence's row are
 * reported as FDLLM_ERR_INDEX.  ref llada/generate.py:254-292 (verify inputs), :262-269 (mask). */
int fdllm_verify_build(const int64_t* seq, int32_t n_seq, int32_t bm, int64_t lmax, int64_t n_slots,
                       const int64_t* full_pos, const int64_t* x, const int64_t* x_draft, int64_t* qpos, int64_t* xv,
                       uint8_t* mask, int64_t* kpos, int64_t* dslot, int64_t* lidx, int32_t* vblocks, int64_t* info2,
                       cudaStream_t stream);

/* Top-k selective refresh order: for each sequence j, stably sort full_pos[j, 0:counts[j]]
 * (int64 [batch, lmax]) ascending by scores[full_pos[j, i]] in place (counts[j] <= 8192).
 * ref llada/generate.py:364-366. */
int fdllm_refresh_sort(int64_t* full_pos, int32_t batch, int64_t lmax, const int64_t* counts, const float* scores,
                       int64_t n_slots, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHDLLM_B200_H */
