// (e) Per-row top-(budget-1) selection with the newest token reserved.
//
// Contract (replaces torch.topk(scores, k=min(budget-1, L), sorted=False) +
// _append_current, popkv.py:594-600 and 141-145): output row = the k largest
// scores' token indices in ascending index order, ties at the threshold broken
// towards the lowest index, then L (the newest token), then -1 padding.
//
// B200 design: one 1024-thread CTA per row, exact in every case.
//  1. Threshold guess.  With the scorer's histogram of the top 11 key bits, the
//     bin holding the k-th largest score gives an exact lower bound T0.  Without
//     it, rows longer than the candidate buffer draw 1024 evenly
//     spaced scores, sort them in shared memory (bitonic) and take the sample
//     whose rank corresponds to ~1.15 k of the row plus a margin: a lower bound
//     T0 that almost surely leaves at least k scores at or above it.
//  2. Candidates.  One pass over the row (16-byte loads, L2-resident scores)
//     counts the scores >= T0 per warp with ballots, a second pass compacts them
//     -- in index order -- into shared memory (about 1.3 k entries).
//  3. Exact radix select (11/11/10-bit digits, warp-aggregated histograms with
//     match.any) over the candidates only.
//  4. Ranking with warp ballots over the index-ordered candidates writes the
//     picks in ascending index order, plus -- optionally -- the per-KV-head token
//     bitmask the fused attention consumes.
// If the guess leaves fewer than k candidates, or more than the buffer holds
// (heavy ties), steps 3-4 run over the whole row read from global memory instead:
// slower, same result.  No CTA waits on another.
#include "common.cuh"

namespace popkv {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kBins = 2048;
constexpr int kCandMax = 16384;  // candidates kept in shared memory (key + index: 128 KB)
constexpr int kSample = 1024;

struct SelectShared {
    uint32_t hist[kBins];
    uint32_t wsum[kSelWarps];
    uint32_t wa[kSelWarps], wb[kSelWarps];
    uint32_t sel_bin, sel_above;
    uint32_t count;
};

struct SelectArgs {
    const float* scores;
    int64_t stride;
    int64_t tokens;
    const int32_t* seq_len;
    int64_t rows_per_seq;
    int64_t budget;
    int32_t* indices;
    uint16_t* masks;       // optional [rows / heads_per_kv][mask_stride] head bitmask
    int64_t mask_stride;
    int heads_per_kv;
    uint32_t* hist;        // optional [rows][kBins] top-digit histogram from the scorer
    bool vec;
};

// Finds the bin of sh.hist where the count from the top first reaches `remaining`:
// sh.sel_bin, sh.sel_above (count strictly above it) and sh.count (total).
__device__ void find_bin(SelectShared& sh, uint32_t remaining) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int kPer = kBins / kSelThreads;
    uint32_t local = 0u;
#pragma unroll
    for (int j = 0; j < kPer; ++j) local += sh.hist[tid * kPer + j];
    uint32_t suffix = local;  // sum over lanes >= lane
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_down_sync(0xffffffffu, suffix, o);
        if (lane + o < 32) suffix += y;
    }
    if (lane == 0) sh.wsum[warp] = suffix;
    __syncthreads();
    uint32_t above = suffix - local;
    for (int w = warp + 1; w < kSelWarps; ++w) above += sh.wsum[w];
    if (tid == 0) sh.count = above + local;
#pragma unroll
    for (int j = kPer - 1; j >= 0; --j) {
        const uint32_t cnt = sh.hist[tid * kPer + j];
        if (above < remaining && above + cnt >= remaining) {
            sh.sel_bin = static_cast<uint32_t>(tid * kPer + j);
            sh.sel_above = above;
        }
        above += cnt;
    }
    __syncthreads();
}

// Exact k-th largest key among n keys given by `get` (3 radix passes); returns the
// threshold key and how many keys equal to it are taken (the lowest-indexed ones).
template <typename Get>
__device__ void radix_threshold(Get get, int64_t n, uint32_t k, SelectShared& sh,
                                uint32_t& thr, uint32_t& need) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t prefix = 0u, pmask = 0u, remaining = k;
#pragma unroll 1
    for (int pass = 0; pass < 3; ++pass) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const uint32_t dmask = pass == 2 ? 0x3ffu : 0x7ffu;
        for (int i = tid; i < kBins; i += kSelThreads) sh.hist[i] = 0u;
        __syncthreads();
        for (int64_t i0 = 0; i0 < n; i0 += kSelThreads) {
            const int64_t i = i0 + tid;
            const bool active = i < n;
            const uint32_t key = active ? get(i) : 0u;
            const bool want = active && (key & pmask) == prefix;
            if (!__any_sync(0xffffffffu, want)) continue;
            const uint32_t digit = (key >> shift) & dmask;
            const unsigned peers = __match_any_sync(0xffffffffu, want ? digit : 0xffffffffu);
            if (want && lane == __ffs(peers) - 1) atomicAdd(&sh.hist[digit], __popc(peers));
        }
        __syncthreads();
        find_bin(sh, remaining);
        remaining -= sh.sel_above;
        prefix |= sh.sel_bin << shift;
        pmask |= dmask << shift;
        __syncthreads();
    }
    thr = prefix;
    need = remaining;
}

// Writes the picks (keys > thr, and the first `need` keys == thr) of n index-ordered
// elements at their rank; idx(i) gives the token index of element i.
template <typename Get, typename Idx>
__device__ void rank_and_write(Get get, Idx idx, int64_t n, uint32_t thr, uint32_t need,
                               SelectShared& sh, int32_t* out, uint32_t* mask_words, uint32_t bit) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t seg = ((n + kSelWarps - 1) / kSelWarps + 31) / 32 * 32;
    const int64_t w_lo = warp * seg;
    const int64_t w_hi = imin64(n, w_lo + seg);
    uint32_t gt = 0u, eq = 0u;
    for (int64_t e = w_lo; e < w_hi; e += 32) {
        const int64_t i = e + lane;
        const uint32_t key = i < w_hi ? get(i) : 0u;
        gt += __popc(__ballot_sync(0xffffffffu, i < w_hi && key > thr));
        eq += __popc(__ballot_sync(0xffffffffu, i < w_hi && key == thr));
    }
    if (lane == 0) { sh.wa[warp] = gt; sh.wb[warp] = eq; }
    __syncthreads();
    if (tid == 0) {
        uint32_t a = 0u, b = 0u;
        for (int w = 0; w < kSelWarps; ++w) {
            const uint32_t x = sh.wa[w], y = sh.wb[w];
            sh.wa[w] = a; sh.wb[w] = b;
            a += x; b += y;
        }
    }
    __syncthreads();
    uint32_t gt_run = sh.wa[warp], eq_run = sh.wb[warp];
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int64_t e = w_lo; e < w_hi; e += 32) {
        const int64_t i = e + lane;
        const uint32_t key = i < w_hi ? get(i) : 0u;
        const bool is_gt = i < w_hi && key > thr;
        const bool is_eq = i < w_hi && key == thr;
        const unsigned bg = __ballot_sync(0xffffffffu, is_gt);
        const unsigned be = __ballot_sync(0xffffffffu, is_eq);
        const uint32_t g_before = gt_run + __popc(bg & lt_mask);
        const uint32_t e_before = eq_run + __popc(be & lt_mask);
        const bool take = is_gt || (is_eq && e_before < need);
        if (take) {
            const int32_t t = idx(i);
            out[g_before + min(e_before, need)] = t;
            if (mask_words) atomicOr(mask_words + (t >> 1), bit << ((t & 1) * 16));
        }
        gt_run += __popc(bg);
        eq_run += __popc(be);
    }
}

__global__ void __launch_bounds__(kSelThreads, 1) select_kernel(SelectArgs a) {
    extern __shared__ __align__(16) uint32_t s_dyn[];
    uint32_t* cand_key = s_dyn;                                          // [kCandMax]
    int32_t* cand_idx = reinterpret_cast<int32_t*>(s_dyn + kCandMax);     // [kCandMax]
    __shared__ SelectShared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t row = blockIdx.x;
    int64_t L = a.seq_len ? static_cast<int64_t>(a.seq_len[row / a.rows_per_seq]) : a.tokens;
    L = L < a.tokens ? (L < 0 ? 0 : L) : a.tokens;
    const int64_t k = a.budget - 1 < L ? a.budget - 1 : L;
    int32_t* out = a.indices + row * a.budget;
    const float* src = a.scores + row * a.stride;
    uint32_t* mask_words = nullptr;
    uint32_t bit = 0u;
    if (a.masks != nullptr) {
        const int64_t b = row / a.rows_per_seq;
        const int64_t qh = row - b * a.rows_per_seq;
        const int64_t kv_per_seq = a.rows_per_seq / a.heads_per_kv;
        mask_words = reinterpret_cast<uint32_t*>(
            a.masks + (b * kv_per_seq + qh / a.heads_per_kv) * a.mask_stride);
        bit = 1u << (qh % a.heads_per_kv);
    }
    bool hist_ok = false;
    if (a.hist != nullptr) {  // the scorer's top-digit histogram of this row (zeroed for next use)
        uint32_t* hrow = a.hist + row * kBins;
        for (int i = tid; i < kBins; i += kSelThreads) {
            sh.hist[i] = hrow[i];
            hrow[i] = 0u;
        }
        __syncthreads();
        if (k > 0 && k < L) {
            find_bin(sh, static_cast<uint32_t>(k));
            hist_ok = sh.count == static_cast<uint32_t>(L);
        }
    }
    if (tid == 0) {
        out[k] = static_cast<int32_t>(L);
        if (mask_words) atomicOr(mask_words + (L >> 1), bit << ((L & 1) * 16));
    }
    for (int64_t j = k + 1 + tid; j < a.budget; j += kSelThreads) out[j] = -1;
    if (k == 0) return;
    if (k == L) {
        for (int64_t i = tid; i < L; i += kSelThreads) {
            out[i] = static_cast<int32_t>(i);
            if (mask_words) atomicOr(mask_words + (i >> 1), bit << ((i & 1) * 16));
        }
        return;
    }

    // 1. Lower-bound threshold from a sorted sample (rows that do not fit whole).
    uint32_t t0 = 0u;
    if (hist_ok) {
        t0 = sh.sel_bin << 21;  // lowest key of the bin holding the k-th largest score
        __syncthreads();
    } else if (L > kCandMax) {
        uint32_t* s = cand_key;
        s[tid] = order_key(__ldg(src + (static_cast<int64_t>(tid) * L) / kSample));
        for (int size = 2; size <= kSample; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                __syncthreads();
                const int j = tid ^ stride;
                if (j > tid) {
                    const uint32_t x = s[tid], y = s[j];
                    if ((x < y) == ((tid & size) == 0)) { s[tid] = y; s[j] = x; }
                }
            }
        }
        __syncthreads();
        int64_t r = (kSample * k * 115) / (L * 100) + 25;  // rank ~1.15 k/L of the sample + margin
        if (r > kSample) r = kSample;
        t0 = s[r - 1];
        __syncthreads();
    }

    // 2. Count and compact the scores >= t0 in index order (warp-contiguous segments).
    const int64_t seg = ((L + kSelWarps - 1) / kSelWarps + 127) / 128 * 128;
    const int64_t w_lo = imin64(warp * seg, L);
    const int64_t w_hi = imin64(w_lo + seg, L);
    auto flags4 = [&](int64_t i4, uint32_t (&key)[4]) -> uint32_t {
        uint32_t f = 0u;
        if (a.vec && i4 + 3 < w_hi) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(src + i4));
            key[0] = order_key(v.x); key[1] = order_key(v.y); key[2] = order_key(v.z); key[3] = order_key(v.w);
#pragma unroll
            for (int j = 0; j < 4; ++j) f |= static_cast<uint32_t>(key[j] >= t0) << j;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool in = i4 + j < w_hi;
                key[j] = in ? order_key(__ldg(src + i4 + j)) : 0u;
                f |= static_cast<uint32_t>(in && key[j] >= t0) << j;
            }
        }
        return f;
    };
    uint32_t wc = 0u;
    for (int64_t e = w_lo; e < w_hi; e += 128) {
        uint32_t key[4];
        wc += __reduce_add_sync(0xffffffffu, __popc(flags4(e + 4 * lane, key)));
    }
    if (lane == 0) sh.wa[warp] = wc;
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0u;
        for (int w = 0; w < kSelWarps; ++w) { const uint32_t x = sh.wa[w]; sh.wa[w] = acc; acc += x; }
        sh.count = acc;
    }
    __syncthreads();
    const uint32_t nc = sh.count;
    const bool fallback = nc < static_cast<uint32_t>(k) || nc > static_cast<uint32_t>(kCandMax);
    if (!fallback) {
        uint32_t base = sh.wa[warp];
        for (int64_t e = w_lo; e < w_hi; e += 128) {
            uint32_t key[4];
            const uint32_t f = flags4(e + 4 * lane, key);
            const uint32_t c = __popc(f);
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            uint32_t pos = base + incl - c;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if ((f >> j) & 1u) {
                    cand_key[pos] = key[j];
                    cand_idx[pos] = static_cast<int32_t>(e + 4 * lane + j);
                    ++pos;
                }
            }
            base += __shfl_sync(0xffffffffu, incl, 31);
        }
        __syncthreads();
        uint32_t thr, need;
        auto get = [&](int64_t i) { return cand_key[i]; };
        auto idx = [&](int64_t i) { return cand_idx[i]; };
        radix_threshold(get, nc, static_cast<uint32_t>(k), sh, thr, need);
        rank_and_write(get, idx, nc, thr, need, sh, out, mask_words, bit);
    } else {
        uint32_t thr, need;
        auto get = [&](int64_t i) { return order_key(__ldg(src + i)); };
        auto idx = [&](int64_t i) { return static_cast<int32_t>(i); };
        radix_threshold(get, L, static_cast<uint32_t>(k), sh, thr, need);
        rank_and_write(get, idx, L, thr, need, sh, out, mask_words, bit);
    }
}

}  // namespace
}  // namespace popkv

using namespace popkv;

extern "C" int popkv_select(const float* scores, int64_t rows, int64_t score_stride,
                            int64_t tokens, const int32_t* seq_len, int64_t rows_per_seq,
                            int64_t budget, int32_t* indices, uint16_t* head_masks,
                            int64_t mask_stride, int64_t heads_per_kv, uint32_t* score_hist,
                            popkv_stream_t stream) {
    if (rows < 0 || tokens < 0 || score_stride < tokens)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid select shape (rows %lld, tokens %lld, stride %lld)",
                    (long long)rows, (long long)tokens, (long long)score_stride);
    if (budget <= 1)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "budget must reserve at least one retrieved and one current token");
    if (tokens > 0x7ffffffeLL) return fail(POPKV_ERR_UNSUPPORTED, "row too long");
    if (rows > 0x7fffffffLL) return fail(POPKV_ERR_UNSUPPORTED, "too many rows");
    if (seq_len != nullptr && rows_per_seq <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "rows_per_seq must be positive");
    if (head_masks != nullptr) {
        if (heads_per_kv <= 0 || heads_per_kv > 16 || rows_per_seq <= 0 || rows_per_seq % heads_per_kv != 0)
            return fail(POPKV_ERR_INVALID_ARGUMENT, "head masks need 0 < heads_per_kv <= 16 dividing rows_per_seq");
        if (mask_stride < tokens + 1 || mask_stride % 2 != 0 || !aligned(head_masks, 4))
            return fail(POPKV_ERR_INVALID_ARGUMENT, "mask_stride must be even and >= tokens + 1");
    }
    if (rows == 0) return POPKV_OK;
    if (!indices || (tokens > 0 && !scores)) return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    SelectArgs a;
    a.scores = scores; a.stride = score_stride; a.tokens = tokens; a.seq_len = seq_len;
    a.rows_per_seq = rows_per_seq > 0 ? rows_per_seq : rows;
    a.budget = budget; a.indices = indices; a.masks = head_masks; a.mask_stride = mask_stride;
    a.heads_per_kv = (int)(heads_per_kv > 0 ? heads_per_kv : 1);
    a.hist = score_hist;
    a.vec = aligned(scores, 16) && score_stride % 4 == 0;
    const size_t smem = (size_t)kCandMax * 8;
    cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    select_kernel<<<(unsigned)rows, kSelThreads, smem, as_stream(stream)>>>(a);
    return check_launch("popkv_select");
}
