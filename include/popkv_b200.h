/*
 * popkv_b200.h -- C ABI of the B200 (sm_100a) Pop-KV retrieval library.
 *
 * Plain pointers and sizes only: every pointer argument is a device pointer
 * unless stated otherwise, every call is asynchronous on `stream`
 * (a cudaStream_t, passed as void*; NULL = legacy default stream), and every
 * call returns POPKV_OK or an error code (see popkv_error_string /
 * popkv_last_error).  Argument checks happen on the host before anything is
 * launched, so an error return means nothing was enqueued.
 *
 * Packed key cache (identical to the reference layout, csrc/popkv_ext.cu:204-208):
 *   k_sign, k_mag : int32  [cache_heads, capacity, words]   bit i of word w = channel 32w+i
 *   low, delta    : fp16   [cache_heads, capacity, words]   (passed as uint16 bit patterns)
 *   words = ceil(head_dim / 32); element (h, t, w) at (h*capacity + t)*words + w.
 *
 * Batched caches (an extension of the reference, whose batch rows share one cache):
 * with cache_per_batch != 0 the cache heads are [batch, kv_heads] flattened,
 * and sequence b owns heads b*kv_heads .. b*kv_heads+kv_heads-1.
 *
 * Sequence lengths: calls take a host `tokens` (the prefix length L, or an upper
 * bound) and an optional device `seq_len` array [batch] (int32).  When seq_len is
 * given, row b uses min(seq_len[b], tokens) -- this keeps launches identical from
 * step to step, so a whole decode step can be captured once in a CUDA graph.
 */
#ifndef POPKV_B200_H
#define POPKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* popkv_stream_t;

enum popkv_status {
    POPKV_OK = 0,
    POPKV_ERR_INVALID_ARGUMENT = 1,
    POPKV_ERR_CAPACITY = 2,
    POPKV_ERR_UNSUPPORTED = 3,
    POPKV_ERR_ALIGNMENT = 4,
    POPKV_ERR_CUDA = 5,
    POPKV_ERR_WORKSPACE = 6
};

enum popkv_dtype { POPKV_F32 = 0, POPKV_F16 = 1, POPKV_BF16 = 2 };

/* Flags for pack / append / score. */
enum popkv_flags {
    /* Divide the representative sums with the PTX div.full.ftz.f32 instruction and
     * scale scores by rsqrtf(D), as a --use_fast_math build of the reference
     * extension does (popkv_cuda.py:20).  Default: IEEE division, 1/sqrt(D)
     * correctly rounded on the host. */
    POPKV_FLAG_REFERENCE_DIVISION = 1,
    /* popkv_score_select: take the two-kernel path (score buffer + select) even where
     * the fused kernel applies. */
    POPKV_FLAG_UNFUSED_SELECT = 2
};

/* Static description of an error code. */
const char* popkv_error_string(int status);
/* Detail message of the last error raised by a call on this host thread. */
const char* popkv_last_error(void);
/* Library version (major*10000 + minor*100 + patch). */
int popkv_version(void);

/*
 * (a) Key packer.  Replaces popkv_pack_cuda / popkv_pack_into_cuda
 * (csrc/popkv_ext.cu:198-227, bound as `pack` / `pack_into` in csrc/popkv_ext.cpp:13-14).
 *
 * keys: [heads, tokens, head_dim] rows of `dtype`, head h starting at
 *       keys + h*key_head_stride elements (key_head_stride >= tokens*head_dim).
 * Tokens are grouped in 32s from the first input row; input row t is written to
 * packed row token_offset + t of every head.  Requires token_offset + tokens <= capacity.
 * thresholds (nullable): fp32 [heads, ceil(tokens/32), head_dim, 2] = (min*0.5, max*0.5).
 */
int popkv_pack(const void* keys, int dtype, int64_t heads, int64_t tokens, int64_t head_dim,
               int64_t key_head_stride, int32_t* k_sign, int32_t* k_mag, uint16_t* low,
               uint16_t* delta, int64_t capacity, int64_t token_offset, float* thresholds,
               int flags, popkv_stream_t stream);

/*
 * (b) Incremental append with open-group re-pack.  Replaces append_popkv + the static
 * cache write (popkv.py:270-280, popkv.py:487-495): one launch per layer, no host copies.
 *
 * For every cache head h (sequence b = h / kv_heads_per_seq) with position
 * P = seq_len ? seq_len[b] : position:
 *   key_cache[h, P] = new_keys[h], value_cache[h, P] = new_values[h]   (when non-NULL),
 *   then re-packs the open group rows floor(P/32)*32 .. P of the packed cache from
 *   key_cache (row P taken from new_keys), exactly as pack_keys_into of the open group.
 * key_cache/value_cache: [heads, kv_capacity, head_dim]; new_keys/new_values: [heads, head_dim].
 * new_keys may be NULL when row P of key_cache already holds the new key
 * (then value arguments are ignored).  Heads whose P >= min(capacity, kv_capacity) are
 * skipped on the device (callers check capacity on the host).
 */
int popkv_append(void* key_cache, void* value_cache, int dtype, int64_t heads,
                 int64_t kv_capacity, int64_t head_dim, const void* new_keys,
                 const void* new_values, int32_t* k_sign, int32_t* k_mag, uint16_t* low,
                 uint16_t* delta, int64_t capacity, const int32_t* seq_len, int64_t position,
                 int64_t kv_heads_per_seq, int flags, popkv_stream_t stream);

/*
 * (c)+(d) Query packer fused with the popcount scorer.  Replaces popkv_score_cuda
 * (csrc/popkv_ext.cu:229-254, bound as `score` in csrc/popkv_ext.cpp:15).
 *
 * queries: [batch, q_heads, head_dim] of q_dtype; head_to_kv: int64 [q_heads] (device).
 * scores: fp32 [batch, q_heads, score_stride]; tokens 0..L-1 of every row are written.
 * Requires tokens <= capacity and tokens <= score_stride.
 * select_workspace (nullable): a select workspace (popkv_select_workspace_bytes for
 * batch*q_heads rows, zero-filled once after allocation); the scorer adds each
 * row's histogram of the top 11 bits of the scores' order keys to it (rows of a
 * KV head with more than 8 query heads are skipped), and popkv_select with the
 * same workspace uses and re-zeroes it.
 */
int popkv_score(const void* queries, int q_dtype, int64_t batch, int64_t q_heads,
                int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                const uint16_t* low, const uint16_t* delta, int64_t kv_heads, int64_t capacity,
                int cache_per_batch, const int64_t* head_to_kv, int64_t tokens,
                const int32_t* seq_len, float* scores, int64_t score_stride,
                void* select_workspace, int flags, popkv_stream_t stream);

/*
 * (e) Per-row top-(budget-1) with the newest token reserved.  Replaces
 * torch.topk(sorted=False) + _append_current (popkv.py:594-600, 141-145).
 *
 * scores: fp32 [rows, score_stride]; row r (sequence r / rows_per_seq) has L tokens.
 * indices: int32 [rows, budget]: the k = min(budget-1, L) largest scores' token
 * indices in ascending index order (ties -> lowest index; -0.0 == +0.0), then L,
 * then -1 padding.
 * head_masks (nullable): also OR the selection into the per-KV-head token bitmask
 * of an attention workspace (see popkv_sparse_attention_masks): row r = b*QH + qh
 * sets bit qh % heads_per_kv of token t in mask row b*(QH/heads_per_kv) + qh/heads_per_kv,
 * with rows_per_seq = QH.  popkv_sparse_attention_premasked then skips its own scatter.
 * select_workspace (nullable, select_workspace_bytes long): the workspace popkv_score
 * filled for these rows.  With it, the selection runs as two kernels spread over the
 * whole GPU and leaves the workspace ready for the next step.  A histogram row
 * that does not add up to L is ignored (the result is the same, only slower).
 * Calls that share a select workspace must not overlap on the GPU.
 */
size_t popkv_select_workspace_bytes(int64_t rows, int64_t tokens);
int popkv_select(const float* scores, int64_t rows, int64_t score_stride, int64_t tokens,
                 const int32_t* seq_len, int64_t rows_per_seq, int64_t budget,
                 int32_t* indices, uint16_t* head_masks, int64_t mask_stride,
                 int64_t heads_per_kv, void* select_workspace, size_t select_workspace_bytes,
                 popkv_stream_t stream);

/*
 * (c)+(d)+(e) fused: score and select in one launch.  Replaces the pair
 * popkv_score_cuda + torch.topk/_append_current of one decode step
 * (popkv.py:587-600, csrc/popkv_ext.cu:229-254).
 *
 * Arguments as popkv_score (queries, packed cache, head_to_kv, tokens, seq_len,
 * flags) and popkv_select (budget, indices, head_masks, mask_stride, heads_per_kv)
 * with rows = batch*q_heads, rows_per_seq = q_heads.  The indices (and head masks)
 * are identical to popkv_score followed by popkv_select.
 * With head_dim 128, bf16/fp16 queries and 16-byte aligned packed words, one
 * cluster of CTAs per row scores its slices into shared memory and selects from
 * there: no score buffer, no histogram workspace; scores / select_workspace may
 * then be NULL and are not touched.  Other sizes (or POPKV_FLAG_UNFUSED_SELECT)
 * run popkv_score + popkv_select and need both (POPKV_ERR_UNSUPPORTED without).
 */
int popkv_score_select(const void* queries, int q_dtype, int64_t batch, int64_t q_heads,
                       int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                       const uint16_t* low, const uint16_t* delta, int64_t kv_heads,
                       int64_t capacity, int cache_per_batch, const int64_t* head_to_kv,
                       int64_t tokens, const int32_t* seq_len, int64_t budget, int32_t* indices,
                       uint16_t* head_masks, int64_t mask_stride, int64_t heads_per_kv,
                       float* scores, int64_t score_stride, void* select_workspace,
                       size_t select_workspace_bytes, int flags, popkv_stream_t stream);

/*
 * (f) Fused gather + exact split-K decode attention.  Replaces gather_selected_kv +
 * selected_attention (popkv.py:341-368) without materialising the gathered rows.
 *
 * queries/out: [batch, q_heads, head_dim]; key_cache/value_cache: [cache_heads,
 * kv_capacity, head_dim]; all of `dtype`.  Query head qh reads KV head qh / G with
 * G = q_heads / kv_heads (the decoder's head_to_kv = arange(QH) // G, popkv.py:427);
 * G must be <= 16.  current_keys/current_values ([batch, kv_heads, head_dim],
 * nullable): the rows used for token index L (the newest token, not yet in the
 * cache); when NULL row L is read from the caches.
 * indices: int32 [batch*q_heads, index_stride]; the first min(budget-1, L)+1 entries
 * of each row are the attended tokens (any order, entries outside 0..L ignored), e.g.
 * the output of popkv_select.  indices == NULL selects dense attention over 0..L.
 * Scale 1/sqrt(head_dim), softmax and accumulation in fp32.
 * workspace: device buffer of popkv_sparse_attention_workspace_bytes(); it must be
 * zero-filled once after allocation, and again before it is used with other
 * (batch, q_heads, kv_heads, head_dim, tokens, splits): every call leaves it ready
 * for the next call of the same sizes.  Calls that share a workspace must not
 * overlap on the GPU.
 * splits: number of token segments per (sequence, KV head); 0 = automatic.
 */
size_t popkv_sparse_attention_workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                              int64_t head_dim, int64_t tokens, int64_t splits);
int popkv_sparse_attention(const void* queries, int dtype, int64_t batch, int64_t q_heads,
                           int64_t head_dim, const void* key_cache, const void* value_cache,
                           int64_t kv_heads, int64_t kv_capacity, int cache_per_batch,
                           const void* current_keys, const void* current_values,
                           const int32_t* indices, int64_t index_stride, int64_t budget,
                           int64_t tokens, const int32_t* seq_len, void* out, void* workspace,
                           size_t workspace_bytes, int64_t splits, popkv_stream_t stream);

/*
 * popkv_sparse_attention over the token bitmask already written into `workspace`
 * by popkv_select(head_masks = popkv_sparse_attention_masks(workspace, ...)) for the
 * same sizes; saves the scatter of the index lists.  Same arguments otherwise.
 */
int popkv_sparse_attention_premasked(const void* queries, int dtype, int64_t batch,
                                     int64_t q_heads, int64_t head_dim, const void* key_cache,
                                     const void* value_cache, int64_t kv_heads,
                                     int64_t kv_capacity, int cache_per_batch,
                                     const void* current_keys, const void* current_values,
                                     int64_t tokens, const int32_t* seq_len, void* out,
                                     void* workspace, size_t workspace_bytes, int64_t splits,
                                     popkv_stream_t stream);
/*
 * popkv_sparse_attention_premasked whose output rows are also all-gathered over
 * NVLink peer memory, in place of a separate collective after it (the reference
 * runs one GPU and has no counterpart; this serves the KV-head-sharded decode).
 * Rank `rank` of `world` (<= 8, one process per GPU) writes its out row r into row
 * rank * batch * q_heads + r of every rank's gathered buffer (peer_out[j]: rank j's
 * buffer, [world * batch * q_heads, head_dim], mapped into this process; 16-byte
 * aligned), then stores this layer's epoch into word `rank` of every rank's arrival
 * words (peer_flags[j]: rank j's [world] uint32, zero-initialised once).
 *   defer_wait == 0: the call then waits until all `world` of its own words hold the
 *     epoch: on return of the stream work the gathered buffer is complete on this rank.
 *   defer_wait != 0: the call does not wait; popkv_peer_gather_wait, queued later on
 *     the same stream, waits for this and every other layer of the step at once.
 * sync_words: this rank's [3] uint32 (zeroed once): CTA ticket, epoch, error (1 after
 * a wait ran out, ~2 s; the gathered rows are then incomplete and must not be used).
 * Every rank must make the same sequence of calls for a given set of buffers.  A
 * rank may write a peer's gathered rows while that peer still reads them from an
 * earlier call of the same layer: reuse a gathered buffer no sooner than every
 * second step (alternate two buffers), and consume a step's rows on the stream
 * before the next step's work is queued.
 */
int popkv_sparse_attention_premasked_gather(
    const void* queries, int dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* key_cache, const void* value_cache, int64_t kv_heads, int64_t kv_capacity,
    int cache_per_batch, const void* current_keys, const void* current_values, int64_t tokens,
    const int32_t* seq_len, void* out, void* workspace, size_t workspace_bytes, int64_t splits,
    int world, int rank, void* const* peer_out, uint32_t* const* peer_flags, uint32_t* sync_words,
    int defer_wait, popkv_stream_t stream);
/*
 * Peer all-gather of one layer's output rows by a separate push (no counterpart in
 * the reference, which runs on one GPU): one CTA stores `bytes` (a multiple of 16)
 * from `rows` to peer_dst[j] for every rank j < world (each rank's gathered buffer
 * at this rank's row offset, peer-mapped), makes the stores visible system-wide and
 * stores the layer's next epoch (sync_words[1] + 1, also written back) into
 * peer_flags[j][rank].  Queued on a side stream after the layer's attention, it keeps
 * NVLink off the compute stream; popkv_peer_gather_wait then waits for every layer.
 */
int popkv_peer_push(const void* rows, int64_t bytes, void* const* peer_dst,
                    uint32_t* const* peer_flags, int rank, int world, uint32_t* sync_words,
                    popkv_stream_t stream);
/*
 * Deferred wait of the peer all-gather (no counterpart in the reference): for every
 * layer l < layers, waits until this rank's arrival words own_flags[l*world ..
 * l*world + world-1] all reach the epoch that the layer's last
 * popkv_sparse_attention_premasked_gather(defer_wait != 0) call stored in
 * sync_words[3*l + 1].  sync_words is the [layers, 3] array of those calls' sync
 * words; a wait that runs out (~2 s) sets sync_words[3*l + 2] to 1.
 */
int popkv_peer_gather_wait(const uint32_t* own_flags, uint32_t* sync_words, int layers, int world,
                           popkv_stream_t stream);
/* Token-bitmask region of an attention workspace (for popkv_select's head_masks). */
int popkv_sparse_attention_masks(void* workspace, int64_t batch, int64_t q_heads,
                                 int64_t kv_heads, int64_t head_dim, int64_t tokens,
                                 int64_t splits, uint16_t** masks, int64_t* mask_stride);

/*
 * Allocation-free variant of popkv_sparse_attention (no counterpart in the
 * reference).  For callers that may not allocate device memory -- a plugin whose
 * host engine owns every allocation, or code that must not call cudaMalloc while
 * the engine holds its allocator -- the scratch comes from a fixed array of
 * POPKV_NOALLOC_SCRATCH_BYTES built into the library (held on every GPU that
 * loads it, until exit) instead of a caller workspace.  Arguments as for
 * popkv_sparse_attention, minus the workspace.  Sizes whose scratch exceeds the
 * array are rejected with POPKV_ERR_WORKSPACE (about 1.2 MB covers one
 * Llama-3.1-8B layer at 32K tokens).  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) and should come before any stream
 * capture.  Every call clears the parts that must start at zero; all calls share
 * the one array, so calls that overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller.
 */
#define POPKV_NOALLOC_SCRATCH_BYTES (8u << 20)
int popkv_sparse_attention_noalloc(const void* queries, int dtype, int64_t batch, int64_t q_heads,
                                   int64_t head_dim, const void* key_cache,
                                   const void* value_cache, int64_t kv_heads,
                                   int64_t kv_capacity, int cache_per_batch,
                                   const void* current_keys, const void* current_values,
                                   const int32_t* indices, int64_t index_stride, int64_t budget,
                                   int64_t tokens, const int32_t* seq_len, void* out,
                                   int64_t splits, popkv_stream_t stream);

/* Adds `increment` to seq_len[0..batch-1] on the device (end of a decode step). */
int popkv_advance(int32_t* seq_len, int64_t batch, int32_t increment, popkv_stream_t stream);

/*
 * Decoder plumbing (fp16/bf16).  No retrieval-path counterpart in the reference; they
 * fuse the elementwise steps the reference's decoder runs as transformers module
 * calls (LlamaRMSNorm, apply_rotary_pos_emb, LlamaMLP act_fn * up; popkv.py:529-616)
 * so that a graphed decode step needs one launch per step.
 *
 * popkv_rmsnorm: out[r] = weight * round(x[r] * rsqrt(mean(x[r]^2) + eps)), rows x n.
 * popkv_rope_qkv: qkv [rows, (q_heads + 2 kv_heads) * head_dim] (a fused projection);
 *   row r is rotated at position positions_of_rows[r] (device int32, clamped to the
 *   table) with cos/sin tables [positions, head_dim]; q [rows, q_heads, head_dim],
 *   k and v [rows, kv_heads, head_dim] are written.
 * popkv_silu_mul: gate_up [rows, 2 ffn] = [gate | up] -> out [rows, ffn] =
 *   round(silu(gate)) * up.
 */
int popkv_rmsnorm(const void* x, const void* weight, void* out, int dtype, int64_t rows, int64_t n,
                  float eps, popkv_stream_t stream);
int popkv_rope_qkv(const void* qkv, const void* cos_table, const void* sin_table,
                   const int32_t* positions_of_rows, int64_t positions, int dtype, int64_t rows,
                   int64_t q_heads, int64_t kv_heads, int64_t head_dim, void* q, void* k, void* v,
                   popkv_stream_t stream);
int popkv_silu_mul(const void* gate_up, void* out, int dtype, int64_t rows, int64_t ffn,
                   popkv_stream_t stream);
/*
 * Decoder weight streams (replaces torch.matmul / torch.addmm with one activation
 * row, the projections of LlamaSparseDecoder.decode, popkv.py:613-616):
 * out[j] = round(round(sum_i x[i] * weight[j, i]) + residual[j]) (the product rounded
 * before the residual add, as `h + o_proj(x)`), weight [n_out, k] row-major (an
 * nn.Linear weight), x [k], residual [n_out] or NULL; fp32 accumulation.
 * k a multiple of 8; fp16/bf16; x and weight 16-byte aligned.
 */
int popkv_gemv(const void* x, const void* weight, const void* residual, void* out, int dtype,
               int64_t n_out, int64_t k, popkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* POPKV_B200_H */
