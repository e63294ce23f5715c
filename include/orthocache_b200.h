/*
 * orthocache_b200.h - C ABI of the B200 (sm_100a) fused spectral-eviction
 * decode-attention library (liborthocache_b200.so).
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * launches on the given CUDA stream (a cudaStream_t passed as void*; NULL is
 * the legacy default stream), never allocates memory and never synchronises.
 * Returns OC_OK or an OC_ERR_* code; oc_status_string() names a code.
 *
 * Reference interfaces replaced (paths are in j-arndt/orthocache-gpu,
 * src/orthocache_gpu/triton_kernels/):
 *   oc_fwht_eviction          fwht_fused_prototype.py:255-322  triton_fwht_eviction
 *   oc_fused_attention_v1     fused_eviction.py:698-800        fused_orthocache_attention
 *   oc_fused_attention_v2     fused_eviction.py:573-691        fused_orthocache_attention_v2
 *   oc_fused_attention_v3_gqa gqa_eviction.py:511-639          fused_orthocache_attention_v3_gqa
 *   oc_fused_attention_paged  paged_eviction.py:323-445        fused_orthocache_attention_paged
 *   oc_lse_merge              fused_eviction.py:316-373        _splitk_reduce_kernel (as a
 *                             stand-alone merge of split partials, used across GPUs)
 *
 * Dtype codes: OC_F32, OC_F16, OC_BF16 for queries, values and outputs;
 * keys may also be OC_F8E4M3 (k_scale is folded into q by the caller, as the
 * reference does).  K and V must have the same dtype unless K is OC_F8E4M3.
 * head_dim: 16, 32, 64, 128 or 256 (float32 keys: up to 128).  Tile size 64.
 * Base pointers and token / head / block strides must be multiples of 16
 * bytes (the tiles are moved by the bulk-copy engine).
 *
 * Thresholds are given in double precision and compared exactly as the
 * reference's CPU path compares them (see the notes at each function).
 *
 * Workspace: a fixed header (the per-unit tile prefix, written by every
 * launch for the merge kernel) followed by the split partial states; its size
 * depends only on the query group and head_dim.  Size it with
 * oc_workspace_bytes(); it needs no initialisation.  Launches that share a
 * workspace must not overlap on the GPU.
 *
 * Status word: launches OR error bits (OC_STATUS_*) into *status and never
 * clear it, so a non-zero word means that some launch since the caller last
 * cleared it produced invalid outputs.  Callers that check after every call
 * clear it after reading; callers that batch launches check it once.
 */
#ifndef ORTHOCACHE_B200_H
#define ORTHOCACHE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OC_F32 = 0, OC_F16 = 1, OC_BF16 = 2, OC_F8E4M3 = 3 };

enum {
  OC_OK = 0,
  OC_ERR_INVALID = 1,     /* bad pointer, size, stride or alignment */
  OC_ERR_UNSUPPORTED = 2, /* dtype / head_dim combination not compiled */
  OC_ERR_WORKSPACE = 3,   /* workspace too small */
  OC_ERR_CUDA = 4,        /* the launch failed; see cudaGetLastError */
  OC_ERR_TOO_LARGE = 5    /* beyond the fixed scratch of oc_fused_attention_v2_noalloc */
};

/* bits of the device status word */
enum { OC_STATUS_TIMEOUT = 1, OC_STATUS_BAD_PAGE = 2, OC_STATUS_BAD_SEQLEN = 4 };

/* gate selector of oc_fused_attention_paged */
enum { OC_GATE_ZETA = 0, OC_GATE_CAUCHY_SCHWARZ = 2 };

const char* oc_status_string(int code);

/* Library version, e.g. 100 for 0.1.0. */
int oc_version(void);

/* Diagnostics: a device buffer of unsigned 64-bit words that decode launches
 * fill with per-team timelines (8 words a team: %globaltimer at entry, after
 * the first copies were issued, at the first arrival and at exit; first and
 * last flattened tile; K and V tiles processed) followed by 3 words per merge
 * block (timer before and after its grid dependency wait).  Written only by
 * a library built with OC_TRACE; NULL disables.  No counterpart in the
 * reference. */
void oc_debug_set_trace(void* buffer);

/* Bytes of workspace for an attention call over `num_groups` (sequence,
 * kv-head) pairs with `group` query heads each, at most `num_tiles` 64-token
 * tiles per sequence, and `head_dim`.  The mask-only call needs none. */
size_t oc_workspace_bytes(int64_t num_groups, int group, int64_t num_tiles, int head_dim);

/* The reference's split heuristic: min(num_sms, max(1, num_tiles/4), num_tiles),
 * at least 1 (fused_eviction.py:556-570). */
int oc_auto_num_splits(int64_t num_tiles, int num_sms);

/* ζ mask for one head: keys (num_tokens, head_dim), token stride in elements.
 * mask_out[t] = (ζ_t <= float32(zeta_max)) as 0/1 bytes (fwht_fused_prototype.py:246;
 * a NaN ζ is evicted); zeta_out (nullable) receives ζ_t as float32. */
int oc_fwht_eviction(const void* keys, int k_dtype, int64_t num_tokens, int head_dim,
                     int64_t k_tok_stride, double zeta_max, uint8_t* mask_out, float* zeta_out,
                     uint32_t* status, void* stream);

/* Multi-head ζ-gated decode (V2).  q (num_heads, head_dim); keys / values
 * (num_heads, seq_len, head_dim) with the given element strides; out
 * (num_heads, head_dim) with out_head_stride.  A tile is evicted iff
 * ζ > zeta_max in double precision (fused_eviction.py:428-432), so a NaN ζ
 * is retained.  mask_out (nullable): (num_heads, seq_len/64) retain flags.
 * retained (nullable): set to the number of retained tiles of the call
 * (written on the stream by the launch itself; no zeroing needed).
 * num_splits <= 0 selects
 * oc_auto_num_splits(num_tiles, num_sms). */
int oc_fused_attention_v2(const void* q, int q_dtype, int64_t q_head_stride,
                          const void* keys, int k_dtype, int64_t k_head_stride, int64_t k_tok_stride,
                          const void* values, int v_dtype, int64_t v_head_stride, int64_t v_tok_stride,
                          int num_heads, int64_t seq_len, int head_dim, double zeta_max,
                          int num_splits, int num_sms, void* out, int out_dtype, int64_t out_head_stride,
                          uint8_t* mask_out, uint32_t* retained, uint32_t* status,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Single-head ζ-gated decode (V1): oc_fused_attention_v2 with num_heads = 1;
 * q (1, head_dim), keys / values (seq_len, head_dim). */
int oc_fused_attention_v1(const void* q, int q_dtype, const void* keys, int k_dtype, int64_t k_tok_stride,
                          const void* values, int v_dtype, int64_t v_tok_stride, int64_t seq_len,
                          int head_dim, double zeta_max, int num_sms, void* out, int out_dtype,
                          uint8_t* mask_out, uint32_t* retained, uint32_t* status, void* workspace,
                          size_t workspace_bytes, void* stream);

/* GQA decode with the Cauchy-Schwarz gate (V3), with an optional leading
 * batch of `num_seqs` independent sequences (num_seqs = 1 is the reference's
 * layout).  q (num_seqs, num_kv_heads*group, head_dim); keys / values
 * (num_seqs, num_kv_heads, seq_len, head_dim); out like q.  Query heads
 * [h*group, (h+1)*group) share kv head h.  A tile is evicted iff
 * max_g(|q_g| * |K_high|_F) <= tau in double precision, norms below 1e-38
 * read as 0 (gqa_eviction.py:216-239). */
int oc_fused_attention_v3_gqa(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                              const void* keys, int k_dtype, int64_t k_seq_stride, int64_t k_head_stride,
                              int64_t k_tok_stride, const void* values, int v_dtype, int64_t v_seq_stride,
                              int64_t v_head_stride, int64_t v_tok_stride, int num_seqs, int num_kv_heads,
                              int group, int64_t seq_len, int head_dim, double tau, int num_splits,
                              int num_sms, void* out, int out_dtype, int64_t out_seq_stride,
                              int64_t out_head_stride, uint8_t* mask_out, uint32_t* retained,
                              uint32_t* status, void* workspace, size_t workspace_bytes, void* stream);

/* Paged-KV decode.  q (num_seqs, num_kv_heads*group, head_dim); caches
 * (num_blocks, num_kv_heads, block_size, head_dim) addressed through element
 * strides; block_tables (num_seqs, max_blocks) int32 with row stride
 * bt_seq_stride.  seq_lens (nullable, int32, multiples of 64): tokens of each
 * sequence; NULL means max_blocks*block_size for every sequence, the
 * reference's behaviour.  gate = OC_GATE_ZETA (threshold = zeta_max, the
 * reference's paged path) or OC_GATE_CAUCHY_SCHWARZ (threshold = tau).
 * block_size: power of two.  group = 1 with OC_GATE_ZETA is exactly the
 * reference's MHA paged kernel.  num_splits is accepted for compatibility:
 * the tiles of each (sequence, kv head) are processed in sequence order so
 * that the block table is read in windows.  k_scale applies to float8 key caches only
 * (other dtypes: pass 1.0 and fold any scale into q): every key element is
 * de-quantised into q's dtype as round(float(k) * float(k_scale)) before the
 * gate and the logits, which is the reference's k_cache.to(q.dtype) * k_scale
 * (paged_eviction.py:355-357). */
int oc_fused_attention_paged(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                             const void* k_cache, int k_dtype, int64_t k_blk_stride, int64_t k_head_stride,
                             int64_t k_tok_stride, const void* v_cache, int v_dtype, int64_t v_blk_stride,
                             int64_t v_head_stride, int64_t v_tok_stride, int num_blocks, int block_size,
                             const int32_t* block_tables, int64_t bt_seq_stride, int max_blocks,
                             const int32_t* seq_lens, int num_seqs, int num_kv_heads, int group,
                             int head_dim, int gate, double threshold, double k_scale, int num_splits,
                             int num_sms,
                             void* out, int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
                             uint8_t* mask_out, uint32_t* retained, uint32_t* status, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Log-sum-exp merge of partial softmax states: for each of num_units rows,
 * m (num_units, num_parts), l (num_units, num_parts) and acc (num_units,
 * num_parts, head_dim), all float32 contiguous, m in log2 units as written
 * by this library.  out[u] = sum_p acc[u,p] 2^(m[u,p]-M) / max(sum_p l[u,p]
 * 2^(m[u,p]-M), 1e-9).  Used to combine sequence shards computed on
 * different GPUs. */
int oc_lse_merge(const float* m, const float* l, const float* acc, int64_t num_units, int num_parts,
                 int head_dim, void* out, int out_dtype, void* stream);

/* Sequence-shard decode: like oc_fused_attention_v3_gqa (num_seqs = 1) but
 * instead of the final output it writes this shard's merged partial state
 * m_out (units), l_out (units), acc_out (units, head_dim), units =
 * num_kv_heads*group, for oc_lse_merge across shards.  The tau gate and the
 * tile grid are those of the full sequence restricted to this shard.
 * seq_len_dev (nullable, one device int32, a multiple of 64 <= seq_len):
 * the number of tokens to decode, read by the kernel, so that a launch
 * captured in a CUDA graph can follow a growing cache (seq_len is then the
 * capacity). */
int oc_fused_attention_v3_shard(const void* q, int q_dtype, int64_t q_head_stride, const void* keys,
                                int k_dtype, int64_t k_head_stride, int64_t k_tok_stride,
                                const void* values, int v_dtype, int64_t v_head_stride,
                                int64_t v_tok_stride, int num_kv_heads, int group, int64_t seq_len,
                                int head_dim, double tau, int num_splits, int num_sms, float* m_out,
                                float* l_out, float* acc_out, uint8_t* mask_out, const int32_t* seq_len_dev,
                                uint32_t* retained, uint32_t* status, void* workspace, size_t workspace_bytes,
                                void* stream);

/* ---- spectral norm cache and the O(1) decode gate ----------------------
 * Reference: src/orthocache_gpu/norm_cache.py:21-146 (SpectralNormCache),
 * triton_kernels/decode_gate.py:54-300 (compute_q_high_norm_exact,
 * decode_gate, _pytorch_decode_gate), eval/perplexity_eval.py:554-674 (the
 * decode path that consumes them). */

/* Per 64-token tile of each head: |(W K_tile)[high_start:high_end]|_F, W the
 * natural-order 64-point Walsh matrix / 8 applied along the tokens, norms
 * below 1e-38 written as 0 (norm_cache.py:58-88 update_prefill).  keys
 * (num_heads, num_tokens, head_dim) with element strides; out[h *
 * out_head_stride + t].  Replaces SpectralNormCache.update_prefill /
 * populate_from_keys (norm_cache.py:58-117); the default band of the
 * reference's model path is [48, 64) (eval/perplexity_eval.py:436). */
int oc_tile_high_norms(const void* keys, int k_dtype, int num_heads, int64_t num_tokens, int head_dim,
                       int64_t k_head_stride, int64_t k_tok_stride, int high_start, int high_end, float* out,
                       int64_t out_head_stride, void* stream);

/* Decode gate (decode_gate.py:188-300).  q (num_kv_heads*group, head_dim);
 * norms (num_kv_heads, >= max_tiles) float32 with norm_head_stride.  Per kv
 * head s = max (q_stat 0) or sorted(...)[group/2] (q_stat 1, the model
 * path's median, perplexity_eval.py:612-616) over its query heads of
 * |q_high|_2 = sqrt(max(0, |q|^2 - sum_i S_i^2 / bs)) with S_i the sums of
 * low_band contiguous blocks of bs = head_dim/low_band dims (tight = 1,
 * compute_q_high_norm_exact) or |q|_2 (tight = 0).  evict_out (nullable,
 * (num_kv_heads, max_tiles) bytes): 1 iff float32(s * norm[t]) <=
 * float32(tau * 64 * head_dim) for t < num_tiles, 0 beyond.  q_norms_out
 * (nullable): s per kv head. */
int oc_decode_gate(const void* q, int q_dtype, int64_t q_head_stride, int num_kv_heads, int group, int head_dim,
                   const float* norms, int64_t norm_head_stride, int num_tiles, int max_tiles, double tau,
                   int tight, int low_band, int q_stat, uint8_t* evict_out, float* q_norms_out, void* stream);

/* Bytes of workspace for oc_fused_attention_cached. */
size_t oc_cached_workspace_bytes(int64_t num_groups, int group, int64_t num_tiles, int head_dim);

/* Decode attention gated by cached key norms: oc_decode_gate (low_band 8)
 * per (sequence, kv head), then attention over the retained tiles only --
 * an evicted tile costs no K and no V read.  Shapes as
 * oc_fused_attention_v3_gqa; norms (num_seqs, num_kv_heads, >= seq_len/64)
 * with element strides.  evict_out (nullable, (num_seqs, num_kv_heads,
 * seq_len/64)): the gate's evict flags.  The reference evaluates this gate
 * and masks the logits of the dense product (perplexity_eval.py:554-674);
 * the output is the same softmax over the retained tiles.  With m_out, l_out
 * and acc_out (all or none; (num_seqs*num_kv_heads*group) and that x
 * head_dim floats) the merged softmax state of each query head is written
 * instead of out (as oc_fused_attention_v3_shard), e.g. to merge with a
 * ragged tail of tokens through oc_lse_merge. */
int oc_fused_attention_cached(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                              const void* keys, int k_dtype, int64_t k_seq_stride, int64_t k_head_stride,
                              int64_t k_tok_stride, const void* values, int v_dtype, int64_t v_seq_stride,
                              int64_t v_head_stride, int64_t v_tok_stride, int num_seqs, int num_kv_heads,
                              int group, int64_t seq_len, int head_dim, const float* norms,
                              int64_t norm_seq_stride, int64_t norm_head_stride, double tau, int tight,
                              int q_stat, int num_sms, void* out, int out_dtype, int64_t out_seq_stride,
                              int64_t out_head_stride, float* m_out, float* l_out, float* acc_out,
                              uint8_t* evict_out, float* q_norms_out, uint32_t* retained, uint32_t* status,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Attention over explicit tile lists (no gate): each (sequence, kv head) g
 * attends to the 64-token tiles tile_list[g * list_stride + k], k <
 * list_count[g] (device int32 arrays; list_stride 0 shares one list).
 * Entries must lie in [0, seq_len/64); an out-of-range entry reads a
 * zero-filled tile (no access outside the tensor).  Shapes and the optional
 * merged-state outputs as oc_fused_attention_cached.  Replaces the
 * compacted-block attention of the reference's 'compact' pipeline mode
 * (adaptive_attention.py:159-205, compaction.py:150-220), with 512-token
 * blocks given as their 8 tiles. */
int oc_fused_attention_tiles(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                             const void* keys, int k_dtype, int64_t k_seq_stride, int64_t k_head_stride,
                             int64_t k_tok_stride, const void* values, int v_dtype, int64_t v_seq_stride,
                             int64_t v_head_stride, int64_t v_tok_stride, int num_seqs, int num_kv_heads,
                             int group, int64_t seq_len, int head_dim, const int32_t* tile_list,
                             int64_t list_stride, const int32_t* list_count, int num_sms, void* out, int out_dtype,
                             int64_t out_seq_stride, int64_t out_head_stride, float* m_out, float* l_out,
                             float* acc_out, uint32_t* retained, uint32_t* status, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Decoder-step helpers of the model driver (orthocache_gpu_b200/model.py),
 * the per-layer operations around the decode attention of a Llama-shaped
 * model.  The reference runs them as PyTorch ops inside HF Llama (its
 * evaluation harness, eval/perplexity_eval.py:320-745); here each is one
 * launch so that a decode step is a short graph.  dtype: OC_BF16 or OC_F16.
 *
 * oc_add_rms_norm: per row of x (rows, n): x += y when y is not NULL (the
 * residual add, rounded to dtype), then h = (x * rsqrt(mean(x^2) + eps))
 * rounded to dtype, times weight (n), rounded to dtype. */
int oc_add_rms_norm(void* x, const void* y, const void* weight, void* h, int64_t rows, int64_t n, float eps,
                    int dtype, void* stream);

/* oc_rope_cache_append: qkv (1, (heads + 2 kv_heads) head_dim) holds one
 * token's q | k | v.  Writes the rotate-half rotary embedding of q (with the
 * fp32 tables cos_tab / sin_tab (max_len, head_dim) at row *pos) to q_out
 * (heads, head_dim), that of k to k_cache[*pos] and v to v_cache[*pos]; the
 * caches are token-major (max_len, kv_heads, head_dim) with the given token
 * stride.  *pos (int64) is read on the device. */
int oc_rope_cache_append(const void* qkv, int heads, int kv_heads, int head_dim, const float* cos_tab,
                         const float* sin_tab, const int64_t* pos, void* q_out, void* k_cache, void* v_cache,
                         int64_t cache_token_stride, int dtype, void* stream);

/* oc_tail_merge: decode attention of q (heads, head_dim) over the ragged
 * tail of the caches, tokens [full, n) with n = *pos + 1 and full = n rounded
 * down to 64, merged by log-sum-exp with the state (m in log2 units, l,
 * unnormalised acc (heads, head_dim), float32) that the fused kernel returned
 * for tokens [0, full) (oc_fused_attention_v3_shard).  scale_log2 =
 * log2(e) / sqrt(head_dim).  out (heads, head_dim) in dtype.  The launch is a
 * programmatic dependent of the kernel before it on the stream (the one that
 * wrote m / l / acc): q and the caches are read before it waits, so they must
 * be complete by the time that kernel starts. */
int oc_tail_merge(const void* q, int heads, int kv_heads, int head_dim, const void* k_cache, const void* v_cache,
                  int64_t cache_token_stride, int64_t max_len, const int64_t* pos, const float* m, const float* l,
                  const float* acc, float scale_log2, void* out, int dtype, void* stream);

/* oc_gemv: one decode token's projection out[n] = sum_k h[k] W[n, k], W in
 * the (out_features, in_features) layout of a linear layer (N rows of K
 * contiguous 16-bit elements, leading dimension ldw; K and ldw multiples of
 * 8, K <= 8192, N even, W 16-byte aligned), fp32 accumulation.  With
 * norm_w == NULL, h = x.  With norm_w, the residual add and RMSNorm of
 * oc_add_rms_norm run first, inside the same launch: v = round(x + y) (y may
 * be NULL), written to x_out when x_out is not NULL (it must not alias x or
 * y), and h = rmsnorm(v, eps) * norm_w (x / y / x_out 16-byte aligned).
 * epilogue OC_GEMV_PLAIN: out (N) = round(h W^T).  OC_GEMV_SILU_MUL: W's
 * rows interleave two projections, row 2j = a_j and row 2j + 1 = b_j, and
 * out (N / 2) = round(round(silu(round(a))) * round(b)).  The launch is a
 * programmatic dependent of the kernel before it on the stream.  The
 * reference runs these products as PyTorch linear layers inside HF Llama
 * (eval/perplexity_eval.py:320-745). */
enum { OC_GEMV_PLAIN = 0, OC_GEMV_SILU_MUL = 1 };
int oc_gemv(const void* x, const void* y, const void* norm_w, float eps, void* x_out, const void* W, int64_t ldw,
            int64_t K, int64_t N, void* out, int epilogue, int dtype, void* stream);

/* oc_gemv_qkv_rope: oc_gemv with N = (heads + 2 kv_heads) head_dim rows
 * (q | k | v) whose epilogue is oc_rope_cache_append's: the rotary embedding
 * of the q and k rows at position *pos, q to q_out (heads, head_dim), k and v
 * written to the token-major caches at *pos (head_dim even). */
int oc_gemv_qkv_rope(const void* x, const void* y, const void* norm_w, float eps, void* x_out, const void* W,
                     int64_t ldw, int64_t K, int heads, int kv_heads, int head_dim, const float* cos_tab,
                     const float* sin_tab, const int64_t* pos, void* q_out, void* k_cache, void* v_cache,
                     int64_t cache_token_stride, int dtype, void* stream);

/* Allocation-free variant of oc_fused_attention_v2 (no counterpart in the
 * reference).  For callers that cannot allocate device memory: code running
 * inside another framework's allocator, under a memory budget, or from a
 * plugin interface that hands over only inputs and outputs.  Same arguments
 * and results as oc_fused_attention_v2 minus the workspace: the split-K
 * scratch lives in a 2 MiB array that this library reserves statically on
 * every GPU that loads it, held until the process exits.  The scratch does
 * not grow with the number of heads or tokens (about 0.03 MiB + 10 KiB *
 * (head_dim + 16)): head_dim up to 128 fits, and a call whose scratch would
 * exceed 2 MiB (head_dim 256) returns OC_ERR_TOO_LARGE.  It calls no cudaMalloc or
 * cudaFree.  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture.  Every launch writes the parts of the
 * array it later reads, so nothing needs clearing between calls; all calls
 * share the one array: calls that overlap on the GPU (different streams, or
 * different host threads) race and give wrong results. */
int oc_fused_attention_v2_noalloc(const void* q, int q_dtype, int64_t q_head_stride,
                                  const void* keys, int k_dtype, int64_t k_head_stride, int64_t k_tok_stride,
                                  const void* values, int v_dtype, int64_t v_head_stride, int64_t v_tok_stride,
                                  int num_heads, int64_t seq_len, int head_dim, double zeta_max,
                                  int num_splits, int num_sms, void* out, int out_dtype, int64_t out_head_stride,
                                  uint8_t* mask_out, uint32_t* retained, uint32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ORTHOCACHE_B200_H */
