// (e) Per-row top-(budget-1) selection with the newest token reserved.
//
// Contract (replaces torch.topk(scores, k=min(budget-1, L), sorted=False) +
// _append_current, popkv.py:594-600 and 141-145): output row = the k largest
// scores' token indices in ascending index order, ties at the threshold broken
// towards the lowest index, then L (the newest token), then -1 padding.
//
// Two exact paths, both built on one idea: find a lower bound T0 for the k-th
// largest score, compact the scores >= T0 (about 1.1-1.3 k of them) in index
// order, run the exact radix select (11/11/10-bit digits, warp-aggregated
// shared-memory histograms with match.any) over those candidates only, and rank
// them with warp ballots so the picks come out in index order without a sort.
//
//  * With a select workspace (the decode pipeline): the scorer has already
//    built each row's histogram of the top 11 key bits, which fixes the first
//    radix digit exactly.  Kernel 1 (one 256-thread CTA per row and 4096-token
//    chunk, i.e. the whole GPU) reads the histogram, derives T0 and compacts its
//    chunk's candidates into the workspace; kernel 2 (one 1024-thread CTA per
//    row) stitches the chunk lists, finishes digits 2-3, ranks and writes, and
//    zeroes the histogram for the next step.
//  * Without one: a single 1024-thread CTA per row sorts 1024 evenly spaced
//    samples (bitonic, shared memory) to pick T0 at ~1.15 k plus a margin, then
//    compacts and selects as above.
// Either way, if the candidates turn out fewer than k or more than the shared
// buffer holds (heavy ties), the radix select and ranking run over the whole row
// instead: slower, same result.  Optionally the selection is also OR-ed into the
// per-KV-head token bitmask the fused attention consumes.  No CTA waits on another.
#include <cmath>
#include <cooperative_groups.h>

#include "score_core.cuh"

namespace popkv {
namespace {

constexpr int kBins = 2048;
constexpr int kCandMax = 16384;   // candidates kept in shared memory (key + index: 128 KB)
constexpr int kSample = 1024;
constexpr int kChunk = 4096;      // tokens per candidate-compaction CTA
constexpr int kChunkThreads = 256;
constexpr int kMaxChunks = 1024;  // rows up to 4M tokens on the workspace path
constexpr int kRowThreads = 1024;

struct SelectShared {
    uint32_t hist[kBins];
    uint32_t wsum[32], wabove[32], wgt[32], weq[32];
    uint32_t total;
    uint32_t sel_bin, sel_above;
    uint32_t count;
    uint32_t chunk_off[kMaxChunks];
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
    bool vec;
    // select workspace (nullable)
    uint32_t* hist;        // [rows][kBins]
    uint32_t* counts;      // [rows][kMaxChunks]
    uint32_t* ckey;        // [rows][tokens_pad]
    int32_t* cidx;         // [rows][tokens_pad]
    int64_t tokens_pad;
};

struct SelectWorkspace {
    size_t hist, counts, ckey, cidx, total;
    int64_t tokens_pad;
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

SelectWorkspace select_layout(int64_t rows, int64_t tokens) {
    SelectWorkspace w;
    w.tokens_pad = (tokens + kChunk - 1) / kChunk * kChunk;
    w.hist = 0;
    w.counts = align256(sizeof(uint32_t) * rows * kBins);
    w.ckey = w.counts + align256(sizeof(uint32_t) * rows * kMaxChunks);
    w.cidx = w.ckey + align256(sizeof(uint32_t) * rows * w.tokens_pad);
    w.total = w.cidx + align256(sizeof(int32_t) * rows * w.tokens_pad);
    return w;
}

__device__ __forceinline__ int64_t row_length(const SelectArgs& a, int64_t row) {
    int64_t L = a.seq_len ? static_cast<int64_t>(a.seq_len[row / a.rows_per_seq]) : a.tokens;
    return L < a.tokens ? (L < 0 ? 0 : L) : a.tokens;
}

// Sum of `local` over the threads above this one (higher tid) and over all threads.
template <int THREADS>
__device__ __forceinline__ void block_suffix(uint32_t local, SelectShared& sh, uint32_t& above,
                                             uint32_t& total) {
    constexpr int NW = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t suffix = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_down_sync(0xffffffffu, suffix, o);
        if (lane + o < 32) suffix += y;
    }
    if (lane == 0) sh.wsum[warp] = suffix;
    __syncthreads();
    if (warp == 0) {
        const uint32_t v = lane < NW ? sh.wsum[lane] : 0u;
        uint32_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_down_sync(0xffffffffu, x, o);
            if (lane + o < 32) x += y;
        }
        sh.wabove[lane] = x - v;
        if (lane == 0) sh.total = x;
    }
    __syncthreads();
    above = suffix - local + sh.wabove[warp];
    total = sh.total;
}

// Sum of `local` over the threads below this one, and over all threads.
template <int THREADS>
__device__ __forceinline__ void block_prefix(uint32_t local, SelectShared& sh, uint32_t& before,
                                             uint32_t& total) {
    constexpr int NW = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) sh.wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t v = lane < NW ? sh.wsum[lane] : 0u;
        uint32_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        sh.wabove[lane] = x - v;
        if (lane == 31) sh.total = x;
    }
    __syncthreads();
    before = incl - local + sh.wabove[warp];
    total = sh.total;
}

// The bin of sh.hist where the count from the top first reaches `remaining`:
// sh.sel_bin, sh.sel_above (count strictly above it) and sh.count (all bins).
template <int THREADS>
__device__ void find_bin(SelectShared& sh, uint32_t remaining) {
    constexpr int kPer = kBins / THREADS;
    const int tid = threadIdx.x;
    if (tid == 0) {  // a bin is always found when remaining <= total; keep indices in range otherwise
        sh.sel_bin = 0u;
        sh.sel_above = 0u;
    }
    uint32_t local = 0u;
#pragma unroll
    for (int j = 0; j < kPer; ++j) local += sh.hist[tid * kPer + j];
    uint32_t above, total;
    block_suffix<THREADS>(local, sh, above, total);
#pragma unroll
    for (int j = kPer - 1; j >= 0; --j) {
        const uint32_t cnt = sh.hist[tid * kPer + j];
        if (above < remaining && above + cnt >= remaining) {
            sh.sel_bin = static_cast<uint32_t>(tid * kPer + j);
            sh.sel_above = above;
        }
        above += cnt;
    }
    if (tid == 0) sh.count = total;
    __syncthreads();
}

// Exact k-th largest key among n keys given by `get`; returns the threshold key and
// how many keys equal to it are taken (the lowest-indexed ones).  Passes before
// `first_pass` are given by (prefix, pmask).
template <int THREADS, typename Get>
__device__ void radix_threshold(Get get, int64_t n, uint32_t k, SelectShared& sh, uint32_t& thr,
                                uint32_t& need, int first_pass = 0, uint32_t prefix = 0u,
                                uint32_t pmask = 0u) {
    const int tid = threadIdx.x, lane = tid & 31;
    uint32_t remaining = k;
#pragma unroll 1
    for (int pass = first_pass; pass < 3; ++pass) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const uint32_t dmask = pass == 2 ? 0x3ffu : 0x7ffu;
        for (int i = tid; i < kBins; i += THREADS) sh.hist[i] = 0u;
        __syncthreads();
        for (int64_t i0 = 0; i0 < n; i0 += THREADS) {
            const int64_t i = i0 + tid;
            const bool active = i < n;
            const uint32_t key = active ? get(i) : 0u;
            const bool want = active && (key & pmask) == prefix;
            const uint32_t digit = (key >> shift) & dmask;
            if (pass > 0) {  // within one top-digit bin the lower digits spread out
                if (want) atomicAdd(&sh.hist[digit], 1u);
                continue;
            }
            if (!__any_sync(0xffffffffu, want)) continue;
            const unsigned peers = __match_any_sync(0xffffffffu, want ? digit : 0xffffffffu);
            if (want && lane == __ffs(peers) - 1) atomicAdd(&sh.hist[digit], __popc(peers));
        }
        __syncthreads();
        find_bin<THREADS>(sh, remaining);
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
template <int THREADS, typename Get, typename Idx>
__device__ void rank_and_write(Get get, Idx idx, int64_t n, uint32_t thr, uint32_t need,
                               SelectShared& sh, int32_t* out, uint32_t* mask_words, uint32_t bit) {
    constexpr int NW = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t seg = ((n + NW - 1) / NW + 31) / 32 * 32;
    const int64_t w_lo = warp * seg;
    const int64_t w_hi = imin64(n, w_lo + seg);
    uint32_t gt = 0u, eq = 0u;
    for (int64_t e = w_lo; e < w_hi; e += 32) {
        const int64_t i = e + lane;
        const uint32_t key = i < w_hi ? get(i) : 0u;
        gt += __popc(__ballot_sync(0xffffffffu, i < w_hi && key > thr));
        eq += __popc(__ballot_sync(0xffffffffu, i < w_hi && key == thr));
    }
    if (lane == 0) { sh.wgt[warp] = gt; sh.weq[warp] = eq; }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the per-warp counts
        uint32_t a = lane < NW ? sh.wgt[lane] : 0u, b = lane < NW ? sh.weq[lane] : 0u;
        uint32_t ia = a, ib = b;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t ya = __shfl_up_sync(0xffffffffu, ia, o);
            const uint32_t yb = __shfl_up_sync(0xffffffffu, ib, o);
            if (lane >= o) { ia += ya; ib += yb; }
        }
        if (lane < NW) { sh.wgt[lane] = ia - a; sh.weq[lane] = ib - b; }
    }
    __syncthreads();
    uint32_t gt_run = sh.wgt[warp], eq_run = sh.weq[warp];
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
        if (is_gt || (is_eq && e_before < need)) {
            const int32_t t = idx(i);
            out[g_before + min(e_before, need)] = t;
            if (mask_words) atomicOr(mask_words + (t >> 1), bit << ((t & 1) * 16));
        }
        gt_run += __popc(bg);
        eq_run += __popc(be);
    }
}

struct RowOut {
    int32_t* out;
    uint32_t* mask_words;
    uint32_t bit;
};

__device__ __forceinline__ RowOut row_output(const SelectArgs& a, int64_t row) {
    RowOut r;
    r.out = a.indices + row * a.budget;
    r.mask_words = nullptr;
    r.bit = 0u;
    if (a.masks != nullptr) {
        const int64_t b = row / a.rows_per_seq;
        const int64_t qh = row - b * a.rows_per_seq;
        const int64_t kv_per_seq = a.rows_per_seq / a.heads_per_kv;
        r.mask_words = reinterpret_cast<uint32_t*>(
            a.masks + (b * kv_per_seq + qh / a.heads_per_kv) * a.mask_stride);
        r.bit = 1u << (qh % a.heads_per_kv);
    }
    return r;
}

// Newest token, padding and the all/nothing cases; returns true when the row is done.
__device__ bool write_trivial(const SelectArgs& a, const RowOut& r, int64_t L, int64_t k,
                              int threads) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        r.out[k] = static_cast<int32_t>(L);
        if (r.mask_words) atomicOr(r.mask_words + (L >> 1), r.bit << ((L & 1) * 16));
    }
    for (int64_t j = k + 1 + tid; j < a.budget; j += threads) r.out[j] = -1;
    if (k == 0) return true;
    if (k == L) {
        for (int64_t i = tid; i < L; i += threads) {
            r.out[i] = static_cast<int32_t>(i);
            if (r.mask_words) atomicOr(r.mask_words + (i >> 1), r.bit << ((i & 1) * 16));
        }
        return true;
    }
    return false;
}

// Exact selection of the whole row read from global memory (the fallback).
__device__ void select_whole_row(const float* src, int64_t L, int64_t k, SelectShared& sh,
                                 const RowOut& r) {
    uint32_t thr, need;
    auto get = [&](int64_t i) { return order_key(__ldg(src + i)); };
    auto idx = [&](int64_t i) { return static_cast<int32_t>(i); };
    radix_threshold<kRowThreads>(get, L, static_cast<uint32_t>(k), sh, thr, need);
    rank_and_write<kRowThreads>(get, idx, L, thr, need, sh, r.out, r.mask_words, r.bit);
}

// ---------------------------------------------------------------- one kernel
__global__ void __launch_bounds__(kRowThreads, 1) select_kernel(SelectArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) uint32_t s_dyn[];
    uint32_t* cand_key = s_dyn;                                          // [kCandMax]
    int32_t* cand_idx = reinterpret_cast<int32_t*>(s_dyn + kCandMax);     // [kCandMax]
    __shared__ SelectShared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t row = blockIdx.x;
    const int64_t L = row_length(a, row);
    const int64_t k = a.budget - 1 < L ? a.budget - 1 : L;
    const float* src = a.scores + row * a.stride;
    const RowOut r = row_output(a, row);
    if (write_trivial(a, r, L, k, kRowThreads)) return;

    // 1. Lower-bound threshold from a sorted sample (rows that do not fit whole).
    uint32_t t0 = 0u;
    if (L > kCandMax) {
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
        int64_t rk = (kSample * k * 115) / (L * 100) + 25;  // rank ~1.15 k/L of the sample + margin
        if (rk > kSample) rk = kSample;
        t0 = s[rk - 1];
        __syncthreads();
    }

    // 2. Count and compact the scores >= t0 in index order (warp-contiguous segments).
    const int64_t seg = ((L + 31) / 32 + 127) / 128 * 128;
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
    uint32_t wbase, nc;
    block_prefix<kRowThreads>(lane == 0 ? wc : 0u, sh, wbase, nc);
    wbase = __shfl_sync(0xffffffffu, wbase, 0);
    if (nc < static_cast<uint32_t>(k) || nc > static_cast<uint32_t>(kCandMax)) {
        select_whole_row(src, L, k, sh, r);
        return;
    }
    uint32_t base = wbase;
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
    radix_threshold<kRowThreads>(get, nc, static_cast<uint32_t>(k), sh, thr, need);
    rank_and_write<kRowThreads>(get, idx, nc, thr, need, sh, r.out, r.mask_words, r.bit);
}

// ------------------------------------------------- workspace path: kernel 1
// One CTA per (row, 4096-token chunk): threshold bin from the scorer's histogram,
// then the chunk's scores >= T0 compacted in index order into the workspace.
__global__ void __launch_bounds__(kChunkThreads) select_candidates_kernel(SelectArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ SelectShared sh;
    const int tid = threadIdx.x;
    const int64_t row = blockIdx.y;
    const int64_t c = blockIdx.x;
    const int64_t L = row_length(a, row);
    const int64_t k = a.budget - 1 < L ? a.budget - 1 : L;
    const int64_t lo = c * kChunk;
    uint32_t* count_out = a.counts + row * kMaxChunks + c;
    if (k == 0 || k == L || lo >= L) {
        if (tid == 0) *count_out = 0u;
        return;
    }
    const int64_t hi = imin64(lo + kChunk, L);
    const float* src = a.scores + row * a.stride;
    constexpr int PER = kChunk / kChunkThreads;  // 16 consecutive scores per thread
    const int64_t first = lo + static_cast<int64_t>(tid) * PER;
    uint32_t key[PER];
    bool in[PER];
    if (a.vec && first + PER <= hi) {  // score loads first: they do not need the threshold
#pragma unroll
        for (int q = 0; q < PER / 4; ++q) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src + first) + q);
            key[4 * q] = order_key(v.x); key[4 * q + 1] = order_key(v.y);
            key[4 * q + 2] = order_key(v.z); key[4 * q + 3] = order_key(v.w);
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) in[j] = true;
    } else {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            in[j] = first + j < hi;
            key[j] = in[j] ? order_key(__ldcg(src + first + j)) : 0u;
        }
    }
    const uint32_t* hrow = a.hist + row * kBins;
    for (int i = tid; i < kBins; i += kChunkThreads) sh.hist[i] = __ldcg(hrow + i);
    __syncthreads();
    find_bin<kChunkThreads>(sh, static_cast<uint32_t>(k));
    // A histogram that does not add up to L (heads the scorer skipped) makes every
    // score a candidate; the finishing kernel then works from the whole row.
    const uint32_t t0 = sh.count == static_cast<uint32_t>(L) ? (sh.sel_bin << 21) : 0u;
    uint32_t f = 0u;
#pragma unroll
    for (int j = 0; j < PER; ++j) f |= static_cast<uint32_t>(in[j] && key[j] >= t0) << j;
    uint32_t before, total;
    block_prefix<kChunkThreads>(__popc(f), sh, before, total);
    uint32_t* ck = a.ckey + row * a.tokens_pad + lo;
    int32_t* ci = a.cidx + row * a.tokens_pad + lo;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        if ((f >> j) & 1u) {
            ck[before] = key[j];
            ci[before] = static_cast<int32_t>(first + j);
            ++before;
        }
    }
    if (tid == 0) *count_out = total;
}

// ------------------------------------------------- workspace path: kernel 2
__global__ void __launch_bounds__(kRowThreads, 1) select_finish_kernel(SelectArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) uint32_t s_dyn[];
    uint32_t* cand_key = s_dyn;
    int32_t* cand_idx = reinterpret_cast<int32_t*>(s_dyn + kCandMax);
    __shared__ SelectShared sh;
    const int tid = threadIdx.x;
    const int64_t row = blockIdx.x;
    const int64_t L = row_length(a, row);
    const int64_t k = a.budget - 1 < L ? a.budget - 1 : L;
    const float* src = a.scores + row * a.stride;
    const RowOut r = row_output(a, row);
    uint32_t* hrow = a.hist + row * kBins;
    const int64_t nchunks = (L + kChunk - 1) / kChunk;
    const uint32_t cnt = tid < nchunks ? __ldcg(a.counts + row * kMaxChunks + tid) : 0u;
    for (int i = tid; i < kBins; i += kRowThreads) {  // read, and zero for the next step
        sh.hist[i] = __ldcg(hrow + i);
        hrow[i] = 0u;
    }
    __syncthreads();
    if (write_trivial(a, r, L, k, kRowThreads)) return;
    find_bin<kRowThreads>(sh, static_cast<uint32_t>(k));
    const bool hist_ok = sh.count == static_cast<uint32_t>(L);
    const uint32_t bin = sh.sel_bin, above = sh.sel_above;
    uint32_t off, nc;
    block_prefix<kRowThreads>(cnt, sh, off, nc);
    if (tid < nchunks) sh.chunk_off[tid] = off;
    __syncthreads();
    if (nc < static_cast<uint32_t>(k) || nc > static_cast<uint32_t>(kCandMax)) {
        select_whole_row(src, L, k, sh, r);
        return;
    }
    // Stitch the chunk lists: every candidate position finds its chunk by binary
    // search, so all loads are independent.
    {
        constexpr int kUnroll = 4;
        const uint32_t* ck = a.ckey + row * a.tokens_pad;
        const int32_t* ci = a.cidx + row * a.tokens_pad;
        for (uint32_t p0 = 0; p0 < nc; p0 += kRowThreads * kUnroll) {
            uint32_t kv[kUnroll];
            int32_t iv[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const uint32_t p = p0 + u * kRowThreads + tid;
                if (p < nc) {
                    int lo = 0, hi = static_cast<int>(nchunks) - 1;  // last chunk with offset <= p
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (sh.chunk_off[mid] <= p) lo = mid; else hi = mid - 1;
                    }
                    const int64_t src = static_cast<int64_t>(lo) * kChunk + (p - sh.chunk_off[lo]);
                    kv[u] = __ldcg(ck + src);
                    iv[u] = __ldcg(ci + src);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const uint32_t p = p0 + u * kRowThreads + tid;
                if (p < nc) { cand_key[p] = kv[u]; cand_idx[p] = iv[u]; }
            }
        }
    }
    __syncthreads();
    uint32_t thr, need;
    auto get = [&](int64_t i) { return cand_key[i]; };
    auto idx = [&](int64_t i) { return cand_idx[i]; };
    if (hist_ok)  // the histogram fixed the top digit: start at the second pass
        radix_threshold<kRowThreads>(get, nc, static_cast<uint32_t>(k) - above, sh, thr, need, 1,
                                     bin << 21, 0x7ffu << 21);
    else
        radix_threshold<kRowThreads>(get, nc, static_cast<uint32_t>(k), sh, thr, need);
    rank_and_write<kRowThreads>(get, idx, nc, thr, need, sh, r.out, r.mask_words, r.bit);
}


// ------------------------------- workspace path: one cluster of C CTAs per row
// For rows of up to C * kRowThreads * kRowMaxPer tokens.  CTA c of a row's cluster
// stages the order keys of the row's c-th slice in shared memory with coalesced
// 16-byte loads (from L2, where the scorer left them); thread t then owns the `per`
// consecutive keys from t * per on (per odd: the strided shared-memory reads are free
// of bank conflicts).  The scorer's histogram fixes the top digit in every CTA alike;
// digits 2 and 3 take a local shared-memory histogram per CTA, which one warp per CTA
// reduces over the cluster by reading its peers' per-lane sums and then the 64 bins
// that hold the threshold (distributed shared memory, no remote atomics).  The picks
// are ranked by a block scan of packed (> thr, == thr) per-thread counts plus the
// totals of the lower-ranked CTAs, and written in index order.
namespace cg = cooperative_groups;
constexpr int kRowMaxPer = 45;

// Histogram bin b lives at b + b / 64: a lane scanning 64 consecutive bins then
// reads a different bank from its neighbours.
constexpr int kPaddedBins = kBins + kBins / 64;
__device__ __forceinline__ int hidx(uint32_t b) { return static_cast<int>(b + (b >> 6)); }

struct RowShared {
    uint32_t hist[3][kPaddedBins];  // top digit, digit 2, digit 3 (this CTA's counts)
    uint32_t lane_sum[3][32];  // per-lane sums of each histogram, read by peers
    uint32_t wsum[32];
    uint32_t total;            // this CTA's packed (> thr) << 16 | (== thr), read by peers
    uint32_t sel_bin, sel_above, count;
    uint32_t sel_count;        // cluster total of the selected bin
    uint32_t base_gt, base_eq;
    uint64_t bar;              // completion of the bulk copy of this CTA's scores
};

__device__ unsigned int g_select_wait_timeouts = 0;

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Where the running count from the top reaches `remaining` in the sum over the
// cluster's C copies of sh.hist[slot] (nbins = 2048 or 1024): sh.sel_bin,
// sh.sel_above (count above the bin) and sh.count (all bins).  Called by every
// thread after its CTA's histogram is complete; includes the cluster barrier that
// publishes the histograms.
template <int C>
__device__ void cluster_find_bin(RowShared& sh, int slot, int nbins, uint32_t remaining) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = nbins / 32;  // bins per lane at level 1 (64 or 32)
    __syncthreads();
    if (warp == 0) {
        const uint32_t* h = sh.hist[slot] + hidx(lane * per);  // per <= 64: no padding inside
        uint32_t l0 = 0u, l1 = 0u;
#pragma unroll 8
        for (int j = 0; j < per; j += 2) {
            l0 += h[j];
            l1 += h[j + 1];
        }
        sh.lane_sum[slot][lane] = l0 + l1;
    }
    if constexpr (C > 1) { cluster_arrive(); cluster_wait(); } else { __syncthreads(); }
    if (warp == 0) {
        cg::cluster_group cluster = cg::this_cluster();
        uint32_t local = 0u;
#pragma unroll
        for (int q = 0; q < C; ++q) {
            const RowShared* peer = C > 1 ? cluster.map_shared_rank(&sh, q) : &sh;
            local += peer->lane_sum[slot][lane];
        }
        uint32_t suffix = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_down_sync(0xffffffffu, suffix, o);
            if (lane + o < 32) suffix += y;
        }
        const uint32_t total = __shfl_sync(0xffffffffu, suffix, 0);
        const unsigned hit = __ballot_sync(0xffffffffu, suffix - local < remaining && suffix >= remaining);
        const int l1 = hit ? __ffs(hit) - 1 : 0;
        const uint32_t above1 = __shfl_sync(0xffffffffu, suffix - local, l1);
        // Level 2: lane l takes bins l1 * per + [l * sub, l * sub + sub).
        const int sub = per / 32;  // 2 or 1
        const int b0 = l1 * per + lane * sub;
        uint32_t c0 = 0u, c1 = 0u;
#pragma unroll
        for (int q = 0; q < C; ++q) {
            const RowShared* peer = C > 1 ? cluster.map_shared_rank(&sh, q) : &sh;
            c0 += peer->hist[slot][hidx(b0)];
            if (sub == 2) c1 += peer->hist[slot][hidx(b0 + 1)];
        }
        const uint32_t l2 = c0 + c1;
        uint32_t s2 = l2;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_down_sync(0xffffffffu, s2, o);
            if (lane + o < 32) s2 += y;
        }
        const uint32_t ab = above1 + s2 - l2;  // count above this lane's bins
        if (lane == 0) {
            sh.count = total;
            if (!hit) { sh.sel_bin = 0u; sh.sel_above = 0u; sh.sel_count = 0u; }
        }
        if (hit && ab < remaining && ab + l2 >= remaining) {  // exactly one lane
            if (sub == 2 && ab + c1 >= remaining) { sh.sel_bin = b0 + 1; sh.sel_above = ab; sh.sel_count = c1; }
            else { sh.sel_bin = b0; sh.sel_above = ab + (sub == 2 ? c1 : 0u); sh.sel_count = sub == 2 ? c0 : l2; }
        }
    }
    __syncthreads();
}

// Inputs of the fused score + select path: the packed cache and the queries, scored
// inside select_row_kernel instead of read back from a score buffer.
struct ScoreIn {
    const void* queries;
    int q_heads, D;
    const int32_t* k_sign;
    const int32_t* k_mag;
    const uint16_t* k_low;
    const uint16_t* k_delta;
    int kv_heads;
    int64_t capacity;
    bool per_batch;
    const int64_t* head_to_kv;
    float scale;
    bool ref_div, vec;
};

// Scores of this CTA's slice [lo, lo + n) of row `row` (query head row % QH of
// sequence row / QH) into s_keys as order keys, counted into sh.hist[0] by their top
// 11 bits.  Bit-identical to score_kernel: the same packed-row loads, query packing
// and token_score arithmetic.  Every thread calls it; it ends with a barrier.
template <typename TQ, int W, int NT>
__device__ void score_slice(const SelectArgs& a, const ScoreIn& in, int64_t row, int64_t lo, int n,
                            uint32_t* s_keys, RowShared& sh) {
    __shared__ float s_abs[W * 33];
    __shared__ uint32_t s_qs[W], s_qm[W];
    __shared__ float s_ql[W], s_qd[W];
    __shared__ int s_head;
    const int tid = threadIdx.x;
    const int64_t b = row / a.rows_per_seq;
    const int qh = static_cast<int>(row - b * a.rows_per_seq);
    const int64_t kvh = in.head_to_kv[qh];
    const int64_t cache_head = (in.per_batch ? b * in.kv_heads : 0) + kvh;
    const int64_t base = cache_head * in.capacity + lo;
    // The slice's packed rows towards L2 in four bulk prefetches, and this thread's
    // first two rows into registers, all before the query pack.
    if (tid == 32 && n >= 4) {
        const uint32_t wb = static_cast<uint32_t>(n) * W * 4u & ~15u, hb = static_cast<uint32_t>(n) * W * 2u & ~15u;
        prefetch_l2(in.k_sign + base * W, wb);
        prefetch_l2(in.k_mag + base * W, wb);
        prefetch_l2(in.k_low + base * W, hb);
        prefetch_l2(in.k_delta + base * W, hb);
    }
    PackedRow<W, true> r0, r1;
    if (tid < n) r0.load(in.k_sign, in.k_mag, in.k_low, in.k_delta, (base + tid) * W);
    if (tid + NT < n) r1.load(in.k_sign, in.k_mag, in.k_low, in.k_delta, (base + tid + NT) * W);
    if (tid < 32) {
        if (tid == 0) s_head = qh;
        __syncwarp();
        pack_query_heads<TQ, W, 1>(static_cast<const TQ*>(in.queries), b, in.q_heads, in.D, &s_head, 1,
                                   s_abs, s_qs, s_qm, s_ql, s_qd, in.ref_div);
    }
    __syncthreads();
    constexpr bool kFull = true;  // W * 32 == D on this path
    uint32_t qs[W], qm[W];
    float ql[W], dq[W];
    int pq[W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
        qs[w] = s_qs[w];
        qm[w] = s_qm[w];
        ql[w] = s_ql[w];
        dq[w] = s_qd[w];
        pq[w] = __popc(qm[w]);
    }
    const float sc = in.ref_div ? rsqrtf(static_cast<float>(in.D)) : in.scale;
    auto one = [&](const PackedRow<W, true>& r) {
        float klf[W], kdf[W];
        half_words<W>(r.l, klf);
        half_words<W>(r.d, kdf);
        const uint32_t pkm = mag_popcounts<W>(r.m, 0xffffffffu);
        const float score = token_score<W, kFull>(r.s, r.m, klf, kdf, pkm, qs, qm, ql, dq, pq,
                                                  0xffffffffu, 32);
        return order_key(__fmul_rn(score, sc));
    };
    // With 512-thread CTAs (two per SM, long rows) odd lanes count into a second copy
    // of the top-digit histogram (fewer lanes of a warp on one address); the copies
    // are added after the slice.  (Measured: helps there, not with 1024 threads.)
    constexpr bool kTwoCopies = NT < kRowThreads;
    uint32_t* hist0 = (kTwoCopies && (threadIdx.x & 1)) ? sh.hist[1] : sh.hist[0];
    int i = tid;
    for (; i + NT < n; i += 2 * NT) {
        if (i != tid) {
            r0.load(in.k_sign, in.k_mag, in.k_low, in.k_delta, (base + i) * W);
            r1.load(in.k_sign, in.k_mag, in.k_low, in.k_delta, (base + i + NT) * W);
        }
        const uint32_t k0 = one(r0), k1 = one(r1);
        s_keys[i] = k0;
        s_keys[i + NT] = k1;
        atomicAdd(&hist0[hidx(k0 >> 21)], 1u);
        atomicAdd(&hist0[hidx(k1 >> 21)], 1u);
    }
    if (i < n) {
        if (i != tid) r0.load(in.k_sign, in.k_mag, in.k_low, in.k_delta, (base + i) * W);
        const uint32_t k0 = one(r0);
        s_keys[i] = k0;
        atomicAdd(&hist0[hidx(k0 >> 21)], 1u);
    }
    __syncthreads();
    if constexpr (kTwoCopies) {
        for (int j = tid; j < kPaddedBins; j += NT) {
            sh.hist[0][j] += sh.hist[1][j];
            sh.hist[1][j] = 0u;
        }
        __syncthreads();
    }
}

// FUSE_W == 0: keys from the score buffer (and the scorer's histogram when given).
// FUSE_W > 0: the slice is scored here (score_slice, head_dim = 32 * FUSE_W, queries
// of type TQ) and no score buffer or histogram workspace is used.
template <int C, int NT, int FUSE_W = 0, typename TQ = float>
__global__ void __launch_bounds__(NT, kRowThreads / NT) select_row_kernel(SelectArgs a, int per, ScoreIn in) {
    pdl_trigger();
    pdl_wait();
    __shared__ __align__(16) RowShared sh;
    extern __shared__ __align__(16) uint32_t s_keys[];  // [NT * per]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int crank = C > 1 ? static_cast<int>(cg::this_cluster().block_rank()) : 0;
    const int64_t row = blockIdx.y;
    const int64_t L = row_length(a, row);
    const int64_t k = a.budget - 1 < L ? a.budget - 1 : L;
    const RowOut r = row_output(a, row);
    // This CTA's slice [lo, lo + n); slice starts are multiples of 4 tokens.
    const int64_t chunk = ((L + C - 1) / C + 3) / 4 * 4;
    const int64_t lo = imin64(static_cast<int64_t>(crank) * chunk, L);
    const int n = static_cast<int>(imin64(lo + chunk, L) - lo);
    uint32_t* hrow = a.hist + row * kBins;

    // Newest token, padding, and the all/nothing cases (uniform over the cluster).
    if (crank == 0) {
        if (tid == 0) {
            if (r.out) r.out[k] = static_cast<int32_t>(L);
            if (r.mask_words) atomicOr(r.mask_words + (L >> 1), r.bit << ((L & 1) * 16));
        }
        if (r.out)
            for (int64_t j = k + 1 + tid; j < a.budget; j += NT) r.out[j] = -1;
    }
    if (k == 0 || k == L) {
        if (k == L)
            for (int i = tid; i < n; i += NT) {
                const int32_t t = static_cast<int32_t>(lo + i);
                if (r.out) r.out[t] = t;
                if (r.mask_words) atomicOr(r.mask_words + (t >> 1), r.bit << ((t & 1) * 16));
            }
        if constexpr (C > 1) { cluster_arrive(); cluster_wait(); }  // every CTA has read the histogram
        if (crank == 0 && a.hist != nullptr)
            for (int i = tid; i < kBins; i += NT) hrow[i] = 0u;
        return;
    }
    uint32_t remaining = static_cast<uint32_t>(k);
    const int first = tid * per;
    const int nvalid = n - first <= 0 ? 0 : (n - first < per ? n - first : per);
    const uint32_t* mine = s_keys + first;
    if constexpr (FUSE_W > 0) {
        for (int i = tid; i < kPaddedBins; i += NT) {
            sh.hist[0][i] = 0u;
            sh.hist[1][i] = 0u;
            sh.hist[2][i] = 0u;
        }
        __syncthreads();
        score_slice<TQ, FUSE_W, NT>(a, in, row, lo, n, s_keys, sh);
        cluster_find_bin<C>(sh, 0, kBins, remaining);
    } else {

    // 1. The slice's scores into shared memory by one bulk copy (the TMA engine
    // streams it while the threads set up the histograms), then turned into order
    // keys in place; the scorer's histogram beside them.
    const float* src = a.scores + row * a.stride + lo;
    const int n4 = a.vec ? (n >> 2) : 0;  // slices start on 4-token boundaries
    if (tid == 0) {
        mbar_init(&sh.bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && n4 > 0) {
        mbar_expect_tx(&sh.bar, static_cast<uint32_t>(n4) * 16u);
        bulk_load(s_keys, src, static_cast<uint32_t>(n4) * 16u, &sh.bar);
    }
    uint32_t hv[(kBins + NT - 1) / NT];
#pragma unroll
    for (int j = 0; j < (kBins + NT - 1) / NT; ++j) {
        const int i = tid + j * NT;
        hv[j] = i < kBins ? __ldcg(hrow + i) : 0u;
    }
    for (int i = tid; i < kPaddedBins; i += NT) {
        sh.hist[1][i] = 0u;
        sh.hist[2][i] = 0u;
        if (i % 65 == 64) sh.hist[0][i] = 0u;  // padding slots
    }
#pragma unroll
    for (int j = 0; j < (kBins + NT - 1) / NT; ++j) {
        const int i = tid + j * NT;
        if (i < kBins) sh.hist[0][hidx(i)] = hv[j];
    }
    if (n4 > 0 && !mbar_wait_bounded(&sh.bar, 0u) && tid == 0) atomicAdd(&g_select_wait_timeouts, 1u);
    for (int i = tid; i < n4; i += NT) {
        uint4 v = reinterpret_cast<uint4*>(s_keys)[i];
        v.x = order_key(__uint_as_float(v.x)); v.y = order_key(__uint_as_float(v.y));
        v.z = order_key(__uint_as_float(v.z)); v.w = order_key(__uint_as_float(v.w));
        reinterpret_cast<uint4*>(s_keys)[i] = v;
    }
    for (int i = (n4 << 2) + tid; i < n; i += NT) s_keys[i] = order_key(__ldg(src + i));
    __syncthreads();

    // 2. Top digit: the scorer's histogram when it counted this row's L scores (the
    // same answer in every CTA of the cluster), else counted here.
    if (warp == 0) {
        uint32_t local = 0u;
#pragma unroll 8
        for (int i = lane; i < kPaddedBins; i += 32) local += sh.hist[0][i];  // padding is 0
        local = __reduce_add_sync(0xffffffffu, local);
        if (lane == 0) sh.count = local;
    }
    __syncthreads();
    if (sh.count == static_cast<uint32_t>(L)) {
        cluster_find_bin<1>(sh, 0, kBins, remaining);  // local: every CTA holds the totals
    } else {
        for (int i = tid; i < kPaddedBins; i += NT) sh.hist[0][i] = 0u;
        __syncthreads();
        for (int i = tid; i < n; i += NT) {
            const uint32_t d = s_keys[i] >> 21;
            const unsigned peers = __match_any_sync(__activemask(), d);
            if (lane == __ffs(peers) - 1) atomicAdd(&sh.hist[0][hidx(d)], __popc(peers));
        }
        cluster_find_bin<C>(sh, 0, kBins, remaining);
    }
    }  // FUSE_W == 0
    uint32_t prefix = sh.sel_bin << 21;
    remaining -= sh.sel_above;

    // 3. One sweep over this thread's keys sorts them by the top digit: above the
    // threshold bin (certain picks, bitmap gt_bits) or in it (bitmap bin_bits,
    // counted into the digit-2 histogram).  Bit j stands for token lo + first + j.
    const uint32_t d1 = prefix >> 21;
    uint32_t gt_w[2] = {0u, 0u}, bin_w[2] = {0u, 0u};  // bitmap halves: keys 0-31, 32-63
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int jn = nvalid - 32 * h < 32 ? nvalid - 32 * h : 32;
        uint32_t g = 0u, bn = 0u;
        for (int j = 0; j < jn; ++j) {
            const uint32_t x = mine[32 * h + j];
            const uint32_t top = x >> 21;
            g |= static_cast<uint32_t>(top > d1) << j;
            if (top == d1) {
                bn |= 1u << j;
                atomicAdd(&sh.hist[1][hidx((x >> 10) & 0x7ffu)], 1u);
            }
        }
        gt_w[h] = g;
        bin_w[h] = bn;
    }
    uint64_t gt_bits = (static_cast<uint64_t>(gt_w[1]) << 32) | gt_w[0];
    const uint64_t bin_bits = (static_cast<uint64_t>(bin_w[1]) << 32) | bin_w[0];
    cluster_find_bin<C>(sh, 1, kBins, remaining);
    // Every CTA of the cluster has now read the scorer's histogram: zero it for the next step.
    if (crank == 0 && a.hist != nullptr)
        for (int i = tid; i < kBins; i += NT) hrow[i] = 0u;
    const uint32_t d2 = sh.sel_bin;
    prefix |= d2 << 10;
    remaining -= sh.sel_above;
    // When every key of the digit-2 bin is a pick (the common case: a 22-bit prefix
    // holds one or two keys), the third digit is not needed: the threshold goes just
    // below the bin.  The test reads cluster totals, so every CTA takes the same branch.
    const bool whole_bin = sh.sel_count == remaining && prefix != 0u;
    uint32_t thr, need;
    uint64_t eq_bits = 0u;
    if (whole_bin) {
        for (uint64_t m = bin_bits; m != 0u; m &= m - 1) {
            const int j = __ffsll(static_cast<long long>(m)) - 1;
            if (((mine[j] >> 10) & 0x7ffu) >= d2) gt_bits |= 1ull << j;
        }
        thr = prefix - 1u;
        need = 0u;
    } else {
        // Digit 3 over the keys of the digit-2 bin, visiting only the top-digit bin.
        uint64_t bin2_bits = 0u;
        for (uint64_t m = bin_bits; m != 0u; m &= m - 1) {
            const int j = __ffsll(static_cast<long long>(m)) - 1;
            const uint32_t x = mine[j];
            const uint32_t dx = (x >> 10) & 0x7ffu;
            if (dx > d2) {
                gt_bits |= 1ull << j;
            } else if (dx == d2) {
                bin2_bits |= 1ull << j;
                atomicAdd(&sh.hist[2][hidx(x & 0x3ffu)], 1u);
            }
        }
        cluster_find_bin<C>(sh, 2, 1024, remaining);
        thr = prefix | sh.sel_bin;
        need = remaining - sh.sel_above;
        for (uint64_t m = bin2_bits; m != 0u; m &= m - 1) {
            const int j = __ffsll(static_cast<long long>(m)) - 1;
            const uint32_t x = mine[j];
            if (x > thr) gt_bits |= 1ull << j;
            else if (x == thr) eq_bits |= 1ull << j;
        }
    }

    // 4. Rank: (> thr) << 16 | (== thr) counts per thread (slice totals < 2^16), one
    // exclusive block scan, the lower-ranked CTAs' totals, then the picks in index
    // order: every key above thr and the first `need` keys equal to it.
    const uint32_t cnt = (static_cast<uint32_t>(__popcll(gt_bits)) << 16) |
                         static_cast<uint32_t>(__popcll(eq_bits));
    uint32_t incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) sh.wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t v = lane < NT / 32 ? sh.wsum[lane] : 0u;
        uint32_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        sh.wsum[lane] = x - v;
        if (lane == 31) sh.total = x;
    }
    if constexpr (C > 1) {
        cluster_arrive();
        cluster_wait();
        if (warp == 0) {  // lane q < crank reads CTA q's totals; all loads in flight at once
            cg::cluster_group cluster = cg::this_cluster();
            const uint32_t t = lane < crank ? cluster.map_shared_rank(&sh, lane)->total : 0u;
            const uint32_t g = __reduce_add_sync(0xffffffffu, t >> 16);
            const uint32_t e = __reduce_add_sync(0xffffffffu, t & 0xffffu);
            if (lane == 0) {
                sh.base_gt = g;
                sh.base_eq = e;
            }
        }
        cluster_arrive();  // this CTA is done reading its peers
    } else if (tid == 0) {
        sh.base_gt = 0u;
        sh.base_eq = 0u;
    }
    __syncthreads();
    const uint32_t before = incl - cnt + sh.wsum[warp];
    // This CTA's picks take out[P0, P0 + n_c) (index order, the slice is contiguous):
    // each thread writes its picks' token indices compacted into shared memory (over
    // the keys, no longer needed), and the CTA stores them coalesced.
    const uint32_t need_left = need;
    const uint32_t eq_c = sh.total & 0xffffu, gt_c = sh.total >> 16;
    const uint32_t p0 = sh.base_gt + min(sh.base_eq, need_left);
    const uint32_t n_c = gt_c + min(sh.base_eq + eq_c, need_left) - min(sh.base_eq, need_left);
    uint32_t gb = sh.base_gt + (before >> 16), eb = sh.base_eq + (before & 0xffffu);
    const uint32_t p_start = gb + min(eb, need_left) - p0;
    uint64_t picks = gt_bits;
    for (uint64_t m = eq_bits; m != 0u && eb < need_left; m &= m - 1, ++eb)
        picks |= m & (~m + 1);  // lowest remaining tie
    // (every key was read before the scan's barriers: s_keys may be overwritten)
    int32_t* s_out = reinterpret_cast<int32_t*>(s_keys);
    uint32_t pos = p_start;
    while (picks != 0u) {
        const int j = __ffsll(static_cast<long long>(picks)) - 1;
        picks &= picks - 1;
        s_out[pos++] = static_cast<int32_t>(lo + first + j);
    }
    __syncthreads();
    for (uint32_t i = tid; i < n_c; i += NT) {
        const int32_t t = s_out[i];
        if (r.out) r.out[p0 + i] = t;
        if (r.mask_words) atomicOr(r.mask_words + (t >> 1), r.bit << ((t & 1) * 16));
    }
    if constexpr (C > 1) cluster_wait();  // peers are done reading this CTA's shared memory
}

}  // namespace
}  // namespace popkv

using namespace popkv;


extern "C" size_t popkv_select_workspace_bytes(int64_t rows, int64_t tokens) {
    if (rows <= 0 || tokens < 0) return 0;
    return select_layout(rows, tokens).total;
}

extern "C" int popkv_select(const float* scores, int64_t rows, int64_t score_stride,
                            int64_t tokens, const int32_t* seq_len, int64_t rows_per_seq,
                            int64_t budget, int32_t* indices, uint16_t* head_masks,
                            int64_t mask_stride, int64_t heads_per_kv, void* select_workspace,
                            size_t select_workspace_bytes, popkv_stream_t stream) {
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
    SelectArgs a = {};
    a.scores = scores; a.stride = score_stride; a.tokens = tokens; a.seq_len = seq_len;
    a.rows_per_seq = rows_per_seq > 0 ? rows_per_seq : rows;
    a.budget = budget; a.indices = indices; a.masks = head_masks; a.mask_stride = mask_stride;
    a.heads_per_kv = (int)(heads_per_kv > 0 ? heads_per_kv : 1);
    a.vec = aligned(scores, 16) && score_stride % 4 == 0;
    const size_t smem = (size_t)kCandMax * 8;
    const cudaStream_t st = as_stream(stream);
    if (select_workspace != nullptr) {
        const SelectWorkspace w = select_layout(rows, tokens);
        if (select_workspace_bytes < w.total)
            return fail(POPKV_ERR_WORKSPACE, "select workspace of %zu bytes, %zu needed",
                        select_workspace_bytes, w.total);
        if (!aligned(select_workspace, 256)) return fail(POPKV_ERR_ALIGNMENT, "select workspace needs 256-byte alignment");
        if (tokens > (int64_t)kMaxChunks * kChunk) return fail(POPKV_ERR_UNSUPPORTED, "row too long for the select workspace");
        unsigned char* base = static_cast<unsigned char*>(select_workspace);
        a.hist = reinterpret_cast<uint32_t*>(base + w.hist);
        a.counts = reinterpret_cast<uint32_t*>(base + w.counts);
        a.ckey = reinterpret_cast<uint32_t*>(base + w.ckey);
        a.cidx = reinterpret_cast<int32_t*>(base + w.cidx);
        a.tokens_pad = w.tokens_pad;
        // Cluster size: the smallest power of two whose slices fit shared memory,
        // raised while the rows still leave SMs idle.  Rows that fill the GPU many
        // times over (long batched contexts) take 512-thread CTAs instead, so that
        // two rows' latency chains overlap on every SM.
        int C = 1;
        while (C < 8 && (tokens + C - 1) / C > (int64_t)kRowThreads * kRowMaxPer) C *= 2;
        while (C < 8 && rows * C * 2 <= num_sms() && (tokens + 2 * C - 1) / (2 * C) >= 2048) C *= 2;
        int NT = kRowThreads;
        if (rows * C > 2 * (int64_t)num_sms()) {
            int C2 = 1;
            while (C2 < 8 && (tokens + C2 - 1) / C2 > (int64_t)(kRowThreads / 2) * kRowMaxPer) C2 *= 2;
            if ((tokens + C2 - 1) / C2 <= (int64_t)(kRowThreads / 2) * kRowMaxPer) { C = C2; NT = kRowThreads / 2; }
        }
        const int64_t chunk = ((tokens + C - 1) / C + 3) / 4 * 4;
        if (chunk <= (int64_t)NT * kRowMaxPer && rows <= 65535) {
            const int per = (int)((chunk + NT - 1) / NT) | 1;  // odd
            const size_t smem_keys = (size_t)per * NT * 4;
            auto go = [&](auto kern) {
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_keys);
                if (C > 1) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
                launch_pdl_cluster(kern, dim3((unsigned)C, (unsigned)rows), dim3(NT), smem_keys,
                                   st, (unsigned)C, a, per, ScoreIn{});
            };
            if (NT == kRowThreads) {
                switch (C) {
                    case 1: go(select_row_kernel<1, kRowThreads>); break;
                    case 2: go(select_row_kernel<2, kRowThreads>); break;
                    case 4: go(select_row_kernel<4, kRowThreads>); break;
                    default: go(select_row_kernel<8, kRowThreads>); break;
                }
            } else {
                switch (C) {
                    case 1: go(select_row_kernel<1, kRowThreads / 2>); break;
                    case 2: go(select_row_kernel<2, kRowThreads / 2>); break;
                    case 4: go(select_row_kernel<4, kRowThreads / 2>); break;
                    default: go(select_row_kernel<8, kRowThreads / 2>); break;
                }
            }
            return check_launch("popkv_select (row)");
        }
        const int64_t chunks = (tokens + kChunk - 1) / kChunk;
        if (chunks > 0) {
            launch_pdl(select_candidates_kernel, dim3((unsigned)chunks, (unsigned)rows), dim3(kChunkThreads), 0, st, a);
            const int rc = check_launch("popkv_select (candidates)");
            if (rc != POPKV_OK) return rc;
        }
        cudaFuncSetAttribute(select_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        launch_pdl(select_finish_kernel, dim3((unsigned)rows), dim3(kRowThreads), smem, st, a);
        return check_launch("popkv_select");
    }
    cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(select_kernel, dim3((unsigned)rows), dim3(kRowThreads), smem, st, a);
    return check_launch("popkv_select");
}

extern "C" int popkv_score_select(const void* queries, int q_dtype, int64_t batch, int64_t q_heads,
                                  int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                                  const uint16_t* low, const uint16_t* delta, int64_t kv_heads,
                                  int64_t capacity, int cache_per_batch, const int64_t* head_to_kv,
                                  int64_t tokens, const int32_t* seq_len, int64_t budget,
                                  int32_t* indices, uint16_t* head_masks, int64_t mask_stride,
                                  int64_t heads_per_kv, float* scores, int64_t score_stride,
                                  void* select_workspace, size_t select_workspace_bytes, int flags,
                                  popkv_stream_t stream) {
    if (batch < 0 || q_heads <= 0 || head_dim <= 0 || kv_heads <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "queries must be [batch, q_heads, head_dim]");
    if (tokens <= 0 || tokens > capacity)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid score token count %lld (capacity %lld)",
                    (long long)tokens, (long long)capacity);
    if (budget <= 1)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "budget must reserve at least one retrieved and one current token");
    if (head_masks != nullptr) {
        if (heads_per_kv <= 0 || heads_per_kv > 16 || q_heads % heads_per_kv != 0)
            return fail(POPKV_ERR_INVALID_ARGUMENT, "head masks need 0 < heads_per_kv <= 16 dividing q_heads");
        if (mask_stride < tokens + 1 || mask_stride % 2 != 0 || !aligned(head_masks, 4))
            return fail(POPKV_ERR_INVALID_ARGUMENT, "mask_stride must be even and >= tokens + 1");
    }
    if (batch == 0) return POPKV_OK;
    if (!queries || !k_sign || !k_mag || !low || !delta || !head_to_kv || !indices)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    const int64_t rows = batch * q_heads;
    // The fused kernel: head_dim 128, 16-bit queries, rows that fit one cluster.
    int C = 1;
    while (C < 8 && (tokens + C - 1) / C > (int64_t)kRowThreads * kRowMaxPer) C *= 2;
    while (C < 8 && rows * C * 2 <= num_sms() && (tokens + 2 * C - 1) / (2 * C) >= 2048) C *= 2;
    int NT = kRowThreads;
    if (rows * C > 2 * (int64_t)num_sms()) {
        int C2 = 1;
        while (C2 < 8 && (tokens + C2 - 1) / C2 > (int64_t)(kRowThreads / 2) * kRowMaxPer) C2 *= 2;
        if ((tokens + C2 - 1) / C2 <= (int64_t)(kRowThreads / 2) * kRowMaxPer) { C = C2; NT = kRowThreads / 2; }
    }
    const int64_t chunk = ((tokens + C - 1) / C + 3) / 4 * 4;
    const bool vec = aligned(k_sign, 16) && aligned(k_mag, 16) && aligned(low, 8) && aligned(delta, 8);
    const bool fused = head_dim == 128 && (q_dtype == POPKV_BF16 || q_dtype == POPKV_F16) && vec &&
                       chunk <= (int64_t)NT * kRowMaxPer && rows <= 65535 &&
                       (flags & POPKV_FLAG_UNFUSED_SELECT) == 0;
    if (!fused) {
        if (!scores || !select_workspace)
            return fail(POPKV_ERR_UNSUPPORTED,
                        "these sizes need the two-kernel path: pass a score buffer and a select workspace");
        int rc = popkv_score(queries, q_dtype, batch, q_heads, head_dim, k_sign, k_mag, low, delta,
                             kv_heads, capacity, cache_per_batch, head_to_kv, tokens, seq_len, scores,
                             score_stride, select_workspace, flags, stream);
        if (rc != POPKV_OK) return rc;
        return popkv_select(scores, rows, score_stride, tokens, seq_len, q_heads, budget, indices,
                            head_masks, mask_stride, heads_per_kv, select_workspace,
                            select_workspace_bytes, stream);
    }
    SelectArgs a = {};
    a.tokens = tokens; a.seq_len = seq_len; a.rows_per_seq = q_heads;
    a.budget = budget; a.indices = indices; a.masks = head_masks; a.mask_stride = mask_stride;
    a.heads_per_kv = (int)(heads_per_kv > 0 ? heads_per_kv : 1);
    ScoreIn in = {};
    in.queries = queries; in.q_heads = (int)q_heads; in.D = (int)head_dim;
    in.k_sign = k_sign; in.k_mag = k_mag; in.k_low = low; in.k_delta = delta;
    in.kv_heads = (int)kv_heads; in.capacity = capacity; in.per_batch = cache_per_batch != 0;
    in.head_to_kv = head_to_kv; in.scale = (float)(1.0 / std::sqrt((double)head_dim));
    in.ref_div = (flags & POPKV_FLAG_REFERENCE_DIVISION) != 0; in.vec = vec;
    const int per = (int)((chunk + NT - 1) / NT) | 1;  // odd
    const size_t smem_keys = (size_t)per * NT * 4;
    const cudaStream_t st = as_stream(stream);
    auto go = [&](auto kern) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_keys);
        if (C > 1) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
        launch_pdl_cluster(kern, dim3((unsigned)C, (unsigned)rows), dim3(NT), smem_keys, st,
                           (unsigned)C, a, per, in);
    };
    auto by_c = [&](auto tq) {
        using TQ = decltype(tq);
        if (NT == kRowThreads) {
            switch (C) {
                case 1: go(select_row_kernel<1, kRowThreads, 4, TQ>); break;
                case 2: go(select_row_kernel<2, kRowThreads, 4, TQ>); break;
                case 4: go(select_row_kernel<4, kRowThreads, 4, TQ>); break;
                default: go(select_row_kernel<8, kRowThreads, 4, TQ>); break;
            }
        } else {
            switch (C) {
                case 1: go(select_row_kernel<1, kRowThreads / 2, 4, TQ>); break;
                case 2: go(select_row_kernel<2, kRowThreads / 2, 4, TQ>); break;
                case 4: go(select_row_kernel<4, kRowThreads / 2, 4, TQ>); break;
                default: go(select_row_kernel<8, kRowThreads / 2, 4, TQ>); break;
            }
        }
    };
    if (q_dtype == POPKV_BF16) by_c(__nv_bfloat16{});
    else by_c(__half{});
    return check_launch("popkv_score_select");
}
