// (c) Query packer fused with (d) the popcount scorer.
//
// Semantics follow popkv_score_kernel (csrc/popkv_ext.cu:93-178): each query row
// is packed with per-row thresholds max*0.5 / min*0.5, per-word fp32 low/delta
// representatives summed in channel order; each token's score is the sum over
// words, in word order, of
//   fmaf(ql*kl, Cs, fmaf(dq*kl, Cq, fmaf(ql*dk, Ck, dq*dk*Cqk)))
// with Cs/Cq/Ck/Cqk = 2*popc(match & x) - popc(x), then multiplied by 1/sqrt(D).
//
// B200 layout of the work: one CTA per (sequence, KV head, token tile of at most
// 1024 tokens, sized so that every SM holds two CTAs) serves every query head
// mapped to that KV head, so each packed row (48 B at D = 128) is read from HBM once
// for the whole GQA group (the reference re-reads it once per query head).  Each
// thread owns four tokens and fetches their sign/mag words with 16-byte loads and
// low/delta with 8-byte loads, issued before the query pack so that the HBM latency
// overlaps it.  The query pack is warp-parallel (ballots for the bit words) with the
// sequential channel-order sums kept on one lane per word.
#include <cmath>

#include "score_core.cuh"

namespace popkv {
namespace {

constexpr int kScoreThreads = 256;
#ifndef POPKV_SCORE_TOKENS_PER_THREAD
#define POPKV_SCORE_TOKENS_PER_THREAD 4
#endif
#ifndef POPKV_SCORE_HIST_AGG
#define POPKV_SCORE_HIST_AGG 0
#endif
#ifndef POPKV_SCORE_CTAS_PER_SM
#define POPKV_SCORE_CTAS_PER_SM 2
#endif
constexpr int kTokensPerThread = POPKV_SCORE_TOKENS_PER_THREAD;
constexpr int kScoreCtasPerSm = POPKV_SCORE_CTAS_PER_SM;
constexpr int kTile = kScoreThreads * kTokensPerThread;
constexpr int kBins = 2048;     // histogram of the top 11 bits of each score's order key
constexpr int kHistHeads = 8;   // query heads per KV head covered by the in-CTA histogram

template <typename TQ, int W, bool VEC, bool FULL>
__global__ void __launch_bounds__(kScoreThreads, kScoreCtasPerSm)
score_kernel(const TQ* __restrict__ queries, int q_heads, int D,
             const int32_t* __restrict__ k_sign, const int32_t* __restrict__ k_mag,
             const uint16_t* __restrict__ k_low, const uint16_t* __restrict__ k_delta,
             int kv_heads, int64_t capacity, bool per_batch,
             const int64_t* __restrict__ head_to_kv, int64_t tokens,
             const int32_t* __restrict__ seq_len, float* __restrict__ scores, int64_t stride,
             float scale, bool ref_div, uint32_t* __restrict__ score_hist, int hist_heads,
             int tile) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t* s_hist = reinterpret_cast<uint32_t*>(smem_raw);         // [hist_heads][kBins]
    float* s_abs = reinterpret_cast<float*>(s_hist + hist_heads * kBins);  // [warps][W*33]
    int* s_heads = reinterpret_cast<int*>(s_abs + (kScoreThreads / 32) * W * 33);  // [q_heads]
    uint32_t* s_qs = reinterpret_cast<uint32_t*>(s_heads + q_heads);  // [q_heads][W]
    uint32_t* s_qm = s_qs + q_heads * W;
    float* s_ql = reinterpret_cast<float*>(s_qm + q_heads * W);
    float* s_qd = s_ql + q_heads * W;
    __shared__ int s_nh;

    const int b = blockIdx.y / kv_heads;
    const int kvh = blockIdx.y - b * kv_heads;
    int64_t L = seq_len ? static_cast<int64_t>(seq_len[b]) : tokens;
    L = L < tokens ? L : tokens;
    const int64_t t_base = static_cast<int64_t>(blockIdx.x) * tile;  // tile <= kTile tokens
    if (t_base >= L) return;  // uniform over the CTA
    const int64_t t_end = t_base + tile < L ? t_base + tile : L;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    // 1. Issue the packed-row loads first.
    const int64_t cache_head = (per_batch ? static_cast<int64_t>(b) * kv_heads : 0) + kvh;
    PackedRow<W, VEC> rows[kTokensPerThread];
#pragma unroll
    for (int j = 0; j < kTokensPerThread; ++j) {
        const int64_t t = t_base + j * kScoreThreads + tid;
        if (t < t_end) rows[j].load(k_sign, k_mag, k_low, k_delta, (cache_head * capacity + t) * W);
    }

    // 2. Query heads of this KV head, in ascending head order.
    if (warp == 0) {
        int count = 0;
        for (int q0 = 0; q0 < q_heads; q0 += 32) {
            const int qh = q0 + lane;
            const bool mine = qh < q_heads && head_to_kv[qh] == kvh;
            const unsigned bal = __ballot_sync(0xffffffffu, mine);
            if (mine) s_heads[count + __popc(bal & ((1u << lane) - 1u))] = qh;
            count += __popc(bal);
        }
        if (lane == 0) s_nh = count;
    }
    __syncthreads();
    const int nh = s_nh;
    const bool use_hist = score_hist != nullptr && nh <= hist_heads;

    // 3. Warp-parallel query pack, one warp per query head.
    if (use_hist)
        for (int i = tid; i < nh * kBins; i += kScoreThreads) s_hist[i] = 0u;
    pack_query_heads<TQ, W, kScoreThreads / 32>(queries, b, q_heads, D, s_heads, nh, s_abs, s_qs,
                                                 s_qm, s_ql, s_qd, ref_div);
    __syncthreads();

    const uint32_t last_valid = (D & 31) ? ((1u << (D & 31)) - 1u) : 0xffffffffu;
    const float sc = ref_div ? rsqrtf(static_cast<float>(D)) : scale;
    // popc of each token's magnitude words does not depend on the query head: counted
    // once per token (one byte per word, W <= 4) instead of once per head.
    const int last_bits = __popc(last_valid);
    uint32_t pkm[kTokensPerThread];
    float klf[kTokensPerThread][W], kdf[kTokensPerThread][W];
#pragma unroll
    for (int j = 0; j < kTokensPerThread; ++j) {
        pkm[j] = mag_popcounts<W>(rows[j].m, last_valid);
        half_words<W>(rows[j].l, klf[j]);
        half_words<W>(rows[j].d, kdf[j]);
    }
    for (int slot = 0; slot < nh; ++slot) {
        float* out = scores + (static_cast<int64_t>(b) * q_heads + s_heads[slot]) * stride;
        uint32_t* hist = s_hist + slot * kBins;
        uint32_t qs[W], qm[W];
        float ql[W], dq[W];
        int pq[W];
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const uint32_t valid = (w == W - 1) ? last_valid : 0xffffffffu;
            qs[w] = s_qs[slot * W + w];
            qm[w] = s_qm[slot * W + w] & valid;
            ql[w] = s_ql[slot * W + w];
            dq[w] = s_qd[slot * W + w];
            pq[w] = __popc(qm[w]);
        }
#pragma unroll
        for (int j = 0; j < kTokensPerThread; ++j) {
            const int64_t t = t_base + j * kScoreThreads + tid;
#if POPKV_SCORE_HIST_AGG
            // Warp-aggregated histogram update: lanes whose scores share a bin add once.
            const bool valid = t < t_end;
            float v = 0.0f;
            if (valid) {
                const float score = token_score<W, FULL>(rows[j].s, rows[j].m, klf[j], kdf[j],
                                                         pkm[j], qs, qm, ql, dq, pq, last_valid,
                                                         last_bits);
                v = __fmul_rn(score, sc);
                out[t] = v;
            }
            if (use_hist) {
                const uint32_t bin = valid ? (order_key(v) >> 21) : 0xffffffffu;
                const uint32_t peers = __match_any_sync(0xffffffffu, bin);
                if (valid && (peers & ((1u << lane) - 1u)) == 0u) atomicAdd(hist + bin, __popc(peers));
            }
#else
            if (t >= t_end) continue;
            const float score = token_score<W, FULL>(rows[j].s, rows[j].m, klf[j], kdf[j], pkm[j],
                                               qs, qm, ql, dq, pq, last_valid, last_bits);
            const float v = __fmul_rn(score, sc);
            out[t] = v;
            if (use_hist) atomicAdd(hist + (order_key(v) >> 21), 1u);
#endif
        }
    }
    if (use_hist) {
        __syncthreads();
        for (int i = tid; i < nh * kBins; i += kScoreThreads) {
            const uint32_t c = s_hist[i];
            if (c) atomicAdd(score_hist + (static_cast<int64_t>(b) * q_heads + s_heads[i / kBins]) * kBins +
                                 (i % kBins), c);
        }
    }
}

template <typename TQ, int W>
int launch_score_t(const void* q, int64_t batch, int64_t q_heads, int D, const int32_t* sg,
                   const int32_t* mg, const uint16_t* lo, const uint16_t* de, int64_t kv_heads,
                   int64_t cap, bool per_batch, const int64_t* h2k, int64_t tokens,
                   const int32_t* seq_len, float* scores, int64_t stride, float scale,
                   bool ref_div, bool vec, uint32_t* hist, cudaStream_t st) {
    // Tiles of at most kTile tokens, as many as keep two CTAs on every SM busy, so
    // that no SM gets a larger share of the tokens than the others.
    int64_t ntiles = (tokens + kTile - 1) / kTile;
    const int64_t fill = (kScoreCtasPerSm * num_sms()) / (batch * kv_heads);
    if (fill > ntiles) ntiles = fill < tokens ? fill : tokens;
    const int tile = (int)((tokens + ntiles - 1) / ntiles);
    ntiles = (tokens + tile - 1) / tile;
    const dim3 grid((unsigned)ntiles, (unsigned)(batch * kv_heads));
    // Histogram rows in shared memory for the expected heads per KV head (a KV head
    // with more skips the histogram; select then counts the top digit itself).
    const int64_t per_kv = (q_heads + kv_heads - 1) / kv_heads;
    const int hist_heads = hist ? (int)(per_kv < kHistHeads ? per_kv : kHistHeads) : 0;
    const size_t smem = (size_t)hist_heads * kBins * 4 + (size_t)(kScoreThreads / 32) * W * 33 * 4 +
                        (size_t)q_heads * (sizeof(int) + (size_t)W * 16);
    auto run = [&](auto kern) {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        launch_pdl(kern, grid, dim3(kScoreThreads), smem, st,

            static_cast<const TQ*>(q), (int)q_heads, D, sg, mg, lo, de, (int)kv_heads, cap,
            per_batch, h2k, tokens, seq_len, scores, stride, scale, ref_div, hist, hist_heads, tile);
    };
    const bool full = D % 32 == 0;
    if (vec && full) run(score_kernel<TQ, W, true, true>);
    else if (vec) run(score_kernel<TQ, W, true, false>);
    else if (full) run(score_kernel<TQ, W, false, true>);
    else run(score_kernel<TQ, W, false, false>);
    return check_launch("popkv_score");
}

template <typename TQ, typename... A>
int score_words(int W, A... a) {
    switch (W) {
        case 1: return launch_score_t<TQ, 1>(a...);
        case 2: return launch_score_t<TQ, 2>(a...);
        case 3: return launch_score_t<TQ, 3>(a...);
        case 4: return launch_score_t<TQ, 4>(a...);
        case 5: return launch_score_t<TQ, 5>(a...);
        case 6: return launch_score_t<TQ, 6>(a...);
        case 7: return launch_score_t<TQ, 7>(a...);
        case 8: return launch_score_t<TQ, 8>(a...);
        default: return fail(POPKV_ERR_UNSUPPORTED, "head_dim above 256 is not supported");
    }
}

}  // namespace
}  // namespace popkv

using namespace popkv;

extern "C" int popkv_score(const void* queries, int q_dtype, int64_t batch, int64_t q_heads,
                           int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                           const uint16_t* low, const uint16_t* delta, int64_t kv_heads,
                           int64_t capacity, int cache_per_batch, const int64_t* head_to_kv,
                           int64_t tokens, const int32_t* seq_len, float* scores,
                           int64_t score_stride, void* select_workspace, int flags,
                           popkv_stream_t stream) {
    // The select workspace starts with the [rows][2048] uint32 histogram.
    uint32_t* score_hist = static_cast<uint32_t*>(select_workspace);
    if (dtype_size(q_dtype) == 0)
        return fail(POPKV_ERR_UNSUPPORTED, "queries dtype %d is not fp32/fp16/bf16", q_dtype);
    if (batch < 0 || q_heads <= 0 || head_dim <= 0 || kv_heads <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "queries must be [batch, q_heads, head_dim]");
    if (head_dim > 256) return fail(POPKV_ERR_UNSUPPORTED, "head_dim %lld > 256", (long long)head_dim);
    if (tokens <= 0 || tokens > capacity)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid score token count %lld (capacity %lld)",
                    (long long)tokens, (long long)capacity);
    if (score_stride < tokens)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "score_stride %lld < tokens %lld",
                    (long long)score_stride, (long long)tokens);
    if (q_heads > 4096 || batch * kv_heads > 65535)
        return fail(POPKV_ERR_UNSUPPORTED, "too many heads for one launch");
    if (batch == 0) return POPKV_OK;
    if (!queries || !k_sign || !k_mag || !low || !delta || !head_to_kv || !scores)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    const int W = (int)((head_dim + 31) / 32);
    const bool vec = aligned(k_sign, 16) && aligned(k_mag, 16) && aligned(low, 8) && aligned(delta, 8);
    const float scale = (float)(1.0 / std::sqrt((double)head_dim));
    const bool ref_div = (flags & POPKV_FLAG_REFERENCE_DIVISION) != 0;
    const cudaStream_t st = as_stream(stream);
    switch (q_dtype) {
        case POPKV_F32:
            return score_words<float>(W, queries, batch, q_heads, (int)head_dim, k_sign, k_mag, low,
                                      delta, kv_heads, capacity, cache_per_batch != 0, head_to_kv,
                                      tokens, seq_len, scores, score_stride, scale, ref_div, vec, score_hist, st);
        case POPKV_F16:
            return score_words<__half>(W, queries, batch, q_heads, (int)head_dim, k_sign, k_mag, low,
                                       delta, kv_heads, capacity, cache_per_batch != 0, head_to_kv,
                                       tokens, seq_len, scores, score_stride, scale, ref_div, vec, score_hist, st);
        default:
            return score_words<__nv_bfloat16>(W, queries, batch, q_heads, (int)head_dim, k_sign,
                                              k_mag, low, delta, kv_heads, capacity,
                                              cache_per_batch != 0, head_to_kv, tokens, seq_len,
                                              scores, score_stride, scale, ref_div, vec, score_hist, st);
    }
}
