// (e) Per-row top-(budget-1) selection with the newest token reserved.
//
// Contract (replaces torch.topk(scores, k=min(budget-1, L), sorted=False) +
// _append_current, popkv.py:594-600 and 141-145): output row = the k largest
// scores' token indices in ascending index order, ties at the threshold broken
// towards the lowest index, then L (the newest token), then -1 padding.
//
// B200 design: one thread-block cluster of C CTAs per row (C <= 8, the smallest
// that lets each CTA hold its slice: rows up to 32K tokens run as one CTA with the
// whole row in shared memory).  Each CTA stages its slice as order-preserving uint32 keys
// and the cluster runs an exact 3-pass radix select (11/11/10-bit digits): each
// CTA builds a histogram of its candidates (warp-aggregated with match.any), the
// cluster reads all histograms through distributed shared memory, and every CTA
// derives the same threshold digit.  A final pass ranks the keys above the
// threshold and the lowest-indexed ties with warp ballots and a cluster-wide
// prefix over CTA counts, so the selection is written in index order without a
// sort.  Rows longer than 8 x 32768 keys are re-read from global memory (L2) in
// every pass instead of being staged.  Cluster barriers are hardware barriers;
// no CTA spins on memory.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace popkv {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kBins = 2048;
constexpr int kResidentMax = 32768;  // keys staged per CTA (128 KB)

struct SelectShared {
    uint32_t hist[2][kBins];
    uint32_t total[kBins];
    uint32_t wsum[kSelWarps];
    uint32_t wgt[kSelWarps], weq[kSelWarps];
    uint32_t cta_gt, cta_eq;
    uint32_t gt_before, eq_before;
    uint32_t sel_bin, sel_above;
};

template <bool RESIDENT, int C>
__global__ void __launch_bounds__(kSelThreads)
select_kernel(const float* __restrict__ scores, int64_t stride, int64_t tokens,
              const int32_t* __restrict__ seq_len, int64_t rows_per_seq, int64_t budget,
              int32_t* __restrict__ indices, bool vec) {
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = C == 1 ? 0 : static_cast<int>(cluster.block_rank());
    const int64_t row = blockIdx.y;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    extern __shared__ __align__(16) uint32_t s_keys[];
    __shared__ SelectShared sh;

    int64_t L = seq_len ? static_cast<int64_t>(seq_len[row / rows_per_seq]) : tokens;
    L = L < tokens ? (L < 0 ? 0 : L) : tokens;
    const int64_t k = budget - 1 < L ? budget - 1 : L;
    int32_t* out = indices + row * budget;
    // Chunks are multiples of 4 keys so that every CTA's slice starts 16-byte aligned.
    const int64_t chunk = (((L + C - 1) / C) + 3) / 4 * 4;
    const int64_t lo = imin64(static_cast<int64_t>(crank) * chunk, L);
    const int64_t hi = imin64(lo + chunk, L);
    const int n = static_cast<int>(hi - lo);

    if (k == L || k == 0) {  // all or nothing selected: no ranking needed (uniform per cluster)
        if (k == L)
            for (int i = tid; i < n; i += kSelThreads) out[lo + i] = static_cast<int32_t>(lo + i);
        if (crank == 0) {
            if (tid == 0) out[k] = static_cast<int32_t>(L);
            for (int64_t j = k + 1 + tid; j < budget; j += kSelThreads) out[j] = -1;
        }
        return;
    }

    const float* src = scores + row * stride + lo;
    if constexpr (RESIDENT) {
        if (vec) {
            const int n4 = n / 4;
            for (int i = tid; i < n4; i += kSelThreads) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(src) + i);
                uint4 u;
                u.x = order_key(f.x); u.y = order_key(f.y); u.z = order_key(f.z); u.w = order_key(f.w);
                reinterpret_cast<uint4*>(s_keys)[i] = u;
            }
            for (int i = n4 * 4 + tid; i < n; i += kSelThreads) s_keys[i] = order_key(__ldg(src + i));
        } else {
            for (int i = tid; i < n; i += kSelThreads) s_keys[i] = order_key(__ldg(src + i));
        }
    }
    auto key_at = [&](int i) -> uint32_t {
        if constexpr (RESIDENT) return s_keys[i];
        else return order_key(__ldg(src + i));
    };

    uint32_t prefix = 0u, pmask = 0u;
    uint32_t remaining = static_cast<uint32_t>(k);
#pragma unroll 1
    for (int pass = 0; pass < 3; ++pass) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const uint32_t dmask = pass == 2 ? 0x3ffu : 0x7ffu;
        uint32_t* hist = sh.hist[pass & 1];
        for (int i = tid; i < kBins; i += kSelThreads) hist[i] = 0u;
        __syncthreads();
        for (int i0 = 0; i0 < n; i0 += kSelThreads) {
            const int i = i0 + tid;
            const bool active = i < n;
            const uint32_t key = active ? key_at(i) : 0u;
            const bool want = active && (key & pmask) == prefix;
            if (!__any_sync(0xffffffffu, want)) continue;
            const uint32_t digit = (key >> shift) & dmask;
            const unsigned peers = __match_any_sync(0xffffffffu, want ? digit : 0xffffffffu);
            if (want && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
        }
        if constexpr (C == 1) {
            __syncthreads();
            for (int bin = tid; bin < kBins; bin += kSelThreads) sh.total[bin] = hist[bin];
        } else {
            cluster.sync();
            for (int bin = tid; bin < kBins; bin += kSelThreads) {
                uint32_t part[C];
#pragma unroll
                for (int r = 0; r < C; ++r) part[r] = cluster.map_shared_rank(hist, r)[bin];
                uint32_t s = 0u;
#pragma unroll
                for (int r = 0; r < C; ++r) s += part[r];
                sh.total[bin] = s;
            }
        }
        __syncthreads();
        // Threshold digit: the bin where the count from the top first reaches `remaining`.
        constexpr int kPer = kBins / kSelThreads;
        uint32_t local = 0u;
#pragma unroll
        for (int j = 0; j < kPer; ++j) local += sh.total[tid * kPer + j];
        uint32_t suffix = local;  // sum over lanes >= lane within the warp
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_down_sync(0xffffffffu, suffix, o);
            if (lane + o < 32) suffix += y;
        }
        if (lane == 0) sh.wsum[warp] = suffix;
        __syncthreads();
        uint32_t above = suffix - local;
        for (int w = warp + 1; w < kSelWarps; ++w) above += sh.wsum[w];
#pragma unroll
        for (int j = kPer - 1; j >= 0; --j) {
            const int bin = tid * kPer + j;
            const uint32_t cnt = sh.total[bin];
            if (above < remaining && above + cnt >= remaining) {
                sh.sel_bin = static_cast<uint32_t>(bin);
                sh.sel_above = above;
            }
            above += cnt;
        }
        __syncthreads();
        remaining -= sh.sel_above;
        prefix |= sh.sel_bin << shift;
        pmask |= dmask << shift;
        __syncthreads();  // sel_* are rewritten by the next pass
    }
    const uint32_t thr = prefix;
    const uint32_t need = remaining;

    // Rank pass 1: per-warp counts over warp-contiguous segments.
    const int seg = ((n + kSelWarps - 1) / kSelWarps + 31) / 32 * 32;
    const int w_lo = warp * seg;
    const int w_hi = min(n, w_lo + seg);
    uint32_t gt = 0u, eq = 0u;
    for (int e = w_lo; e < w_hi; e += 32) {
        const int i = e + lane;
        const uint32_t key = i < w_hi ? key_at(i) : 0u;
        gt += __popc(__ballot_sync(0xffffffffu, i < w_hi && key > thr));
        eq += __popc(__ballot_sync(0xffffffffu, i < w_hi && key == thr));
    }
    if (lane == 0) { sh.wgt[warp] = gt; sh.weq[warp] = eq; }
    __syncthreads();
    if (tid == 0) {
        uint32_t a = 0u, b = 0u;
        for (int w = 0; w < kSelWarps; ++w) {
            const uint32_t x = sh.wgt[w], y = sh.weq[w];
            sh.wgt[w] = a; sh.weq[w] = b;
            a += x; b += y;
        }
        sh.cta_gt = a;
        sh.cta_eq = b;
    }
    if constexpr (C == 1) __syncthreads(); else cluster.sync();
    if (tid == 0) {
        uint32_t a = 0u, b = 0u;
        for (int r = 0; r < crank; ++r) {
            const SelectShared* remote = cluster.map_shared_rank(&sh, r);
            a += remote->cta_gt;
            b += remote->cta_eq;
        }
        sh.gt_before = a;
        sh.eq_before = b;
    }
    __syncthreads();
    // Rank pass 2: write the picks at their rank in index order.
    uint32_t gt_run = sh.gt_before + sh.wgt[warp];
    uint32_t eq_run = sh.eq_before + sh.weq[warp];
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int e = w_lo; e < w_hi; e += 32) {
        const int i = e + lane;
        const uint32_t key = i < w_hi ? key_at(i) : 0u;
        const bool is_gt = i < w_hi && key > thr;
        const bool is_eq = i < w_hi && key == thr;
        const unsigned bg = __ballot_sync(0xffffffffu, is_gt);
        const unsigned be = __ballot_sync(0xffffffffu, is_eq);
        const uint32_t g_before = gt_run + __popc(bg & lt_mask);
        const uint32_t e_before = eq_run + __popc(be & lt_mask);
        if (is_gt) out[g_before + min(e_before, need)] = static_cast<int32_t>(lo + i);
        if (is_eq && e_before < need) out[g_before + e_before] = static_cast<int32_t>(lo + i);
        gt_run += __popc(bg);
        eq_run += __popc(be);
    }
    if (crank == 0) {
        if (tid == 0) out[k] = static_cast<int32_t>(L);
        for (int64_t j = k + 1 + tid; j < budget; j += kSelThreads) out[j] = -1;
    }
    if constexpr (C > 1) cluster.sync();  // keep shared memory alive until every peer has read it
}

}  // namespace
}  // namespace popkv

using namespace popkv;

extern "C" int popkv_select(const float* scores, int64_t rows, int64_t score_stride,
                            int64_t tokens, const int32_t* seq_len, int64_t rows_per_seq,
                            int64_t budget, int32_t* indices, popkv_stream_t stream) {
    if (rows < 0 || tokens < 0 || score_stride < tokens)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid select shape (rows %lld, tokens %lld, stride %lld)",
                    (long long)rows, (long long)tokens, (long long)score_stride);
    if (budget <= 1)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "budget must reserve at least one retrieved and one current token");
    if (tokens > 0x7fffffffLL - 1) return fail(POPKV_ERR_UNSUPPORTED, "row too long");
    if (rows > 65535) return fail(POPKV_ERR_UNSUPPORTED, "more than 65535 rows in one launch");
    if (seq_len != nullptr && rows_per_seq <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "rows_per_seq must be positive");
    if (rows == 0) return POPKV_OK;
    if (!indices || (tokens > 0 && !scores)) return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    // Cluster size: the smallest power of two (<= 8) whose per-CTA slice fits in
    // shared memory; longer rows use 8 CTAs re-reading their slice from L2.
    int C = 1;
    while (C < 8 && (tokens + C - 1) / C > kResidentMax) C <<= 1;
    const int64_t chunk = (((tokens + C - 1) / C) + 3) / 4 * 4;
    const bool resident = chunk <= kResidentMax;
    const bool vec = aligned(scores, 16) && score_stride % 4 == 0;
    const size_t smem = resident ? (size_t)chunk * sizeof(uint32_t) : 0;
    const int64_t rps = rows_per_seq > 0 ? rows_per_seq : rows;
    cudaError_t e = cudaSuccess;
    auto launch = [&](auto kern, int cluster) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)cluster, (unsigned)rows, 1);
        cfg.blockDim = dim3(kSelThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = as_stream(stream);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)cluster;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (smem > 0) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        e = cudaLaunchKernelEx(&cfg, kern, scores, score_stride, tokens, seq_len, rps, budget,
                               indices, vec);
    };
    if (resident) {
        switch (C) {
            case 1: launch(select_kernel<true, 1>, 1); break;
            case 2: launch(select_kernel<true, 2>, 2); break;
            case 4: launch(select_kernel<true, 4>, 4); break;
            default: launch(select_kernel<true, 8>, 8); break;
        }
    } else {
        launch(select_kernel<false, 8>, 8);
    }
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_select launch: %s", cudaGetErrorString(e));
    return check_launch("popkv_select");
}
