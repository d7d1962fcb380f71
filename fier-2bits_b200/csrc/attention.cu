// (f) Fused gather + exact split-K decode attention over the selected tokens.
//
// Semantics: for every query head, softmax(q . K_sel^T / sqrt(D)) . V_sel over the
// head's selected tokens, the newest token (index L) read from the current k/v
// rows -- the reference's gather_selected_kv + selected_attention
// (popkv.py:341-368) -- without materialising the gathered rows.
//
// B200 layout of the work:
//  * a scatter kernel turns the [rows, budget] index lists into a per-token bitmask
//    of the query heads (of one KV head) that selected the token;
//  * one CTA per (sequence, KV head, token segment) reads the segment's bitmask
//    (and clears it for the next call), compacts the UNION of its G query heads'
//    selections, and streams those K/V rows once from HBM with 16-byte cp.async
//    copies into a per-warp double-buffered shared-memory ring; the G heads share
//    every row read (GQA);
//  * each warp runs a flash-decoding tile of 16 rows on the tensor cores
//    (mma.m16n8k16, bf16/fp16 in, fp32 accumulate) with the query heads packed
//    into the M dimension, masking every (head, row) pair the head did not select;
//  * partial (max, sum, acc) per (head, segment) go to the workspace and a
//    combine kernel (one CTA per query head) merges them.
// fp32 caches and head_dim outside {64, 96, 128} take a SIMT variant of the same
// segment kernel.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace popkv {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxGroup = 16;
constexpr int kSegMax = 2048;   // tokens per segment (multiple of 8)
constexpr int kTileRows = 16;
constexpr int kMaxSplits = 1024;
constexpr int kMaxPeers = 8;       // ranks of one NVLink domain in a peer all-gather

struct AttnParams {
    const void* q;
    const void* kc;
    const void* vc;
    const void* cur_k;
    const void* cur_v;
    void* out;
    const int32_t* indices;
    int64_t index_stride;
    int64_t budget;
    uint16_t* masks;       // [B*KVH][mask_stride]
    int64_t mask_stride;   // multiple of 8
    float* ws_m;           // [B*QH][S]
    float* ws_l;           // [B*QH][S]
    float* ws_acc;         // [B*QH][S][D]
    uint32_t* tickets;     // [B*KVH]
    int B, QH, KVH, G, D;
    int64_t kv_cap;
    int per_batch;
    int64_t tokens;
    const int32_t* seq_len;
    int S;
    float sl2;       // 1/sqrt(D) * log2(e)
    int work_bytes;  // scratch bytes before the token list (SIMT kernel)
    int dense;       // attend every token 0..L (no head masks)
    // Peer all-gather of the output (world > 1): row r of this rank's out also goes
    // to row rank * B * QH + r of every rank's gathered buffer, then the ranks
    // exchange arrival flags (see combine_kernel).
    int world, rank;
    void* peer_out[kMaxPeers];        // gathered buffer base on each rank
    uint32_t* peer_flags[kMaxPeers];  // each rank's [world] arrival words of this layer
    uint32_t* sync;                   // this rank's [3]: CTA ticket, epoch, error
    int peer_defer;                   // publish arrival only; popkv_peer_gather_wait waits
};

__device__ __forceinline__ int64_t seq_length(const AttnParams& p, int b) {
    int64_t L = p.seq_len ? static_cast<int64_t>(p.seq_len[b]) : p.tokens;
    return L < p.tokens ? (L < 0 ? 0 : L) : p.tokens;
}

__device__ __forceinline__ int64_t segment_len(int64_t L, int S) {
    return ((L + 1 + S - 1) / S + 7) / 8 * 8;
}

// ------------------------------------------------------------- scatter kernel
__global__ void scatter_kernel(AttnParams p) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.y;  // b*QH + qh
    const int b = row / p.QH;
    const int qh = row - b * p.QH;
    const int kvh = qh / p.G;
    const int bit = qh - kvh * p.G;
    const int64_t L = seq_length(p, b);
    const int64_t count = (p.budget - 1 < L ? p.budget - 1 : L) + 1;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= count) return;
    const int64_t t = p.indices[row * p.index_stride + j];
    if (t < 0 || t > L) return;
    uint32_t* words = reinterpret_cast<uint32_t*>(p.masks + (static_cast<int64_t>(b) * p.KVH + kvh) * p.mask_stride);
    atomicOr(words + (t >> 1), (1u << bit) << ((t & 1) * 16));
}

// ------------------------------------------------------ union of one segment
// Reads the bitmask of tokens [lo, lo+n) (n <= kSegMax, lo multiple of 8), clears
// it, and writes the selected tokens (ascending) and their head masks to shared
// memory.  Returns the union size (same value in every thread).
template <typename TokT>
__device__ int build_union(const AttnParams& p, int b, int kvh, int64_t lo, int n, TokT* s_tok,
                           uint16_t* s_msk, int* s_scan, bool dense) {
    // int lists hold token indices; uint16 lists hold offsets from lo (n <= kSegMax).
    const int64_t tok_base = sizeof(TokT) == 2 ? lo : 0;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    if (dense) {
        const uint16_t full = static_cast<uint16_t>((1u << p.G) - 1u);
        for (int i = tid; i < n; i += kAttnThreads) {
            s_tok[i] = static_cast<TokT>(lo + i - tok_base);
            s_msk[i] = full;
        }
        __syncthreads();
        return n;
    }
    constexpr int PER = kSegMax / kAttnThreads;  // 16 tokens = two 16-byte words
    uint16_t* mrow = p.masks + (static_cast<int64_t>(b) * p.KVH + kvh) * p.mask_stride + lo;
    const int first = tid * PER;
    uint16_t m[PER];
    if (first + PER <= n) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(mrow + first);
        const uint4 w1 = *reinterpret_cast<const uint4*>(mrow + first + 8);
        const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            m[2 * j] = static_cast<uint16_t>(ws[j] & 0xffffu);
            m[2 * j + 1] = static_cast<uint16_t>(ws[j] >> 16);
        }
        if ((w0.x | w0.y | w0.z | w0.w | w1.x | w1.y | w1.z | w1.w) != 0u) {
            *reinterpret_cast<uint4*>(mrow + first) = make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(mrow + first + 8) = make_uint4(0u, 0u, 0u, 0u);
        }
    } else {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            m[j] = (first + j < n) ? mrow[first + j] : static_cast<uint16_t>(0);
            if (m[j]) mrow[first + j] = 0;
        }
    }
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) cnt += m[j] != 0;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_scan[warp] = incl;
    __syncthreads();
    int base = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
        base += (w < warp) ? s_scan[w] : 0;
        total += s_scan[w];
    }
    int pos = base + incl - cnt;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        if (m[j]) {
            s_tok[pos] = static_cast<TokT>(lo + first + j - tok_base);
            s_msk[pos] = m[j];
            ++pos;
        }
    }
    __syncthreads();
    return total;
}

// ------------------------------------------------------- peer all-gather
// The combine of a rank writes each output row straight into every rank's gathered
// buffer over NVLink (16-byte stores to peer memory), so no separate collective runs.
// Completion: every CTA makes its stores visible system-wide and takes a ticket; the
// last CTA bumps this layer's epoch and stores it (release, system scope) into its
// slot of every rank's arrival words.  Then either that CTA waits (acquire) until
// every rank's word for this layer reaches the epoch -- the gathered rows are
// complete here when the kernel ends, as after an all-gather -- or, with a deferred
// wait, the kernel ends at once and a later peer_wait_kernel does the waiting for
// all layers of a step together, so no layer is held up by the slowest rank.  Every
// wait is bounded (~2 s); running out of it sets the error word and returns.  Epochs
// only grow, so no flag is ever reset.
//
// A rank can write into a peer's gathered buffer while that peer still reads the
// same rows from an earlier call; callers that reuse buffers alternate two of them
// (the Python stack does, by step parity).
constexpr long long kPeerWaitNs = 2000000000ll;

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits (bounded) until all `world` words at `flags` reach `epoch`; false on timeout.
__device__ bool wait_arrivals(const uint32_t* flags, int world, uint32_t epoch) {
    const unsigned long long t0 = global_ns();
    for (int j = 0; j < world; ++j) {
        while (static_cast<int32_t>(load_acquire_sys(flags + j) - epoch) < 0) {
            if (global_ns() - t0 > static_cast<unsigned long long>(kPeerWaitNs)) return false;
            __nanosleep(256);
        }
    }
    return true;
}

template <int DPT, typename T>
__device__ void peer_gather_rows(const AttnParams& p, int64_t row, const float (&o)[DPT], float inv) {
    // Stage the row in shared memory, then store it to every rank as 16-byte chunks
    // (head_dim is a multiple of 8, so a row is a whole number of chunks).
    __shared__ __align__(16) T s_row[256];
#pragma unroll
    for (int c = 0; c < DPT; ++c) {
        const int d = threadIdx.x + 128 * c;
        if (d < p.D) s_row[d] = from_float<T>(o[c] * inv);
    }
    __syncthreads();
    const int chunks = p.D * static_cast<int>(sizeof(T)) / 16;
    const int64_t dst_row = static_cast<int64_t>(p.rank) * p.B * p.QH + row;
    const uint4* src = reinterpret_cast<const uint4*>(s_row);
    for (int i = threadIdx.x; i < p.world * chunks; i += blockDim.x) {
        const int j = i / chunks;
        const int c = i - j * chunks;
        uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(p.peer_out[j]) + dst_row * p.D);
        dst[c] = src[c];
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    const uint32_t t = atomicAdd(p.sync, 1u);
    if (t != gridDim.x - 1) return;
    __threadfence_system();  // the other CTAs' stores, seen through their tickets, come first
    p.sync[0] = 0u;           // every CTA has taken its ticket: ready for the next call
    const uint32_t epoch = p.sync[1] + 1u;
    p.sync[1] = epoch;
    for (int j = 0; j < p.world; ++j) store_release_sys(p.peer_flags[j] + p.rank, epoch);
    if (p.peer_defer) return;
    if (!wait_arrivals(p.peer_flags[p.rank], p.world, epoch)) atomicExch(p.sync + 2, 1u);
}

// All-gather by a separate push (deferred-wait mode): one CTA, queued on a side
// stream after the layer's combine, stores this rank's `bytes` of output rows at
// byte offset `dst_off` of every rank's gathered buffer (16-byte stores over NVLink),
// makes them visible system-wide and publishes the layer's next epoch into its slot
// of every rank's arrival words.  The compute stream never waits on NVLink.
struct PushArgs {
    const uint4* src;
    uint4* dst[kMaxPeers];
    uint32_t* flags[kMaxPeers];
    uint32_t* sync;  // this rank's [3] words of the layer: ticket (unused), epoch, error
    int64_t chunks;  // 16-byte chunks
    int world, rank;
};

__global__ void __launch_bounds__(256) peer_push_kernel(PushArgs a) {
    pdl_trigger();
    pdl_wait();
    for (int64_t i = threadIdx.x; i < a.world * a.chunks; i += blockDim.x) {
        const int j = static_cast<int>(i / a.chunks);
        const int64_t c = i - static_cast<int64_t>(j) * a.chunks;
        a.dst[j][c] = a.src[c];
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    const uint32_t epoch = a.sync[1] + 1u;
    a.sync[1] = epoch;
    for (int j = 0; j < a.world; ++j) store_release_sys(a.flags[j] + a.rank, epoch);
}

// Deferred wait of the peer all-gather: thread l waits until every rank's arrival
// word of layer l (own_flags + l * world) reaches that layer's epoch (sync + 3 l + 1,
// written by the combine kernels queued before this one); a wait that runs out sets
// the layer's error word.
__global__ void peer_wait_kernel(const uint32_t* own_flags, uint32_t* sync, int layers, int world) {
    pdl_trigger();
    pdl_wait();
    for (int l = threadIdx.x; l < layers; l += blockDim.x) {
        const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(sync + 3 * l + 1);
        if (!wait_arrivals(own_flags + static_cast<int64_t>(l) * world, world, epoch))
            atomicExch(sync + 3 * l + 2, 1u);
    }
}

// ----------------------------------------------------------------- combine
// One CTA per (sequence, query head): merges the S segment partials (max, sum,
// acc) into the output.  Every warp walks the splits in chunks of 32 with an online
// rescale (one max, one sum per chunk by warp shuffles, no block barrier), and all
// loads of a chunk -- max, sum and the thread's accumulator channels -- are issued
// together, so a chunk costs one L2 round trip.
template <typename T, int CH>  // CH = splits per chunk: 64 (head_dim <= 128) or 32
__global__ void __launch_bounds__(128) combine_kernel(AttnParams p) {
    pdl_trigger();
    pdl_wait();
    constexpr int DPT = CH == 64 ? 1 : 2;  // channels per thread (tid, tid + 128)
    const int64_t row = blockIdx.x;        // b*QH + qh
    const int S = p.S, D = p.D;
    const int tid = threadIdx.x, lane = tid & 31;
    const float* mrow = p.ws_m + row * S;
    const float* lrow = p.ws_l + row * S;
    const float* arow = p.ws_acc + row * static_cast<int64_t>(S) * D;
    float M = -INFINITY, lsum = 0.0f, o[DPT];
#pragma unroll
    for (int c = 0; c < DPT; ++c) o[c] = 0.0f;
    for (int s0 = 0; s0 < S; s0 += CH) {
        const int n = S - s0 < CH ? S - s0 : CH;
        float m_l[CH / 32], l_l[CH / 32];
#pragma unroll
        for (int h = 0; h < CH / 32; ++h) {
            const int j = h * 32 + lane;
            m_l[h] = j < n ? __ldcg(mrow + s0 + j) : -INFINITY;
            l_l[h] = j < n ? __ldcg(lrow + s0 + j) : 0.0f;
        }
        float a[DPT][CH];
#pragma unroll
        for (int j = 0; j < CH; ++j) {
            const float* src = arow + static_cast<int64_t>(s0 + j) * D;
#pragma unroll
            for (int c = 0; c < DPT; ++c) {
                const int d = tid + 128 * c;
                a[c][j] = (j < n && d < D) ? __ldcg(src + d) : 0.0f;
            }
        }
        float cmax = m_l[0];
#pragma unroll
        for (int h = 1; h < CH / 32; ++h) cmax = fmaxf(cmax, m_l[h]);
#pragma unroll
        for (int x = 16; x > 0; x >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, x));
        const float m_new = fmaxf(M, cmax);
        if (m_new == -INFINITY) continue;  // uniform: no token in these splits yet
        const float scale = exp2f(M - m_new);  // 0 while M is still -inf
        lsum *= scale;
#pragma unroll
        for (int c = 0; c < DPT; ++c) o[c] *= scale;
        float w_l[CH / 32], wl = 0.0f;
#pragma unroll
        for (int h = 0; h < CH / 32; ++h) {
            w_l[h] = m_l[h] == -INFINITY ? 0.0f : exp2f(m_l[h] - m_new);
            wl = fmaf(w_l[h], l_l[h], wl);
        }
#pragma unroll
        for (int x = 16; x > 0; x >>= 1) wl += __shfl_xor_sync(0xffffffffu, wl, x);
        lsum += wl;
#pragma unroll
        for (int j = 0; j < CH; ++j) {
            const float w = __shfl_sync(0xffffffffu, w_l[j / 32], j & 31);
#pragma unroll
            for (int c = 0; c < DPT; ++c) o[c] = fmaf(w, a[c][j], o[c]);
        }
        M = m_new;
    }
    const float inv = 1.0f / lsum;
    T* out = static_cast<T*>(p.out);
#pragma unroll
    for (int c = 0; c < DPT; ++c) {
        const int d = tid + 128 * c;
        if (d < D) out[row * D + d] = from_float<T>(o[c] * inv);
    }
    if (p.world > 1) peer_gather_rows<DPT, T>(p, row, o, inv);
}

template <typename T>
void launch_combine(const AttnParams& p, cudaStream_t st) {
    if (p.D <= 128) launch_pdl(combine_kernel<T, 64>, dim3((unsigned)(p.B * p.QH)), dim3(128), 0, st, p);
    else launch_pdl(combine_kernel<T, 32>, dim3((unsigned)(p.B * p.QH)), dim3(128), 0, st, p);
}

// -------------------------------------------------------------- PTX helpers
__device__ __forceinline__ void cp_async16_s(uint32_t s, const void* gmem, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* smem) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* smem) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
    static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&v);
    }
};
template <> struct MmaOp<__half> {
    static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        const __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&v);
    }
};

// Shared-memory plan of the tensor-core kernel (bytes).
#ifndef POPKV_ATTN_CTAS_PER_SM
#define POPKV_ATTN_CTAS_PER_SM 3
#endif
constexpr int kMmaCtasPerSm = POPKV_ATTN_CTAS_PER_SM;
constexpr int kMmaStages = kMmaCtasPerSm >= 3 ? 2 : 3;  // cp.async ring depth per warp

template <typename T, int D>
struct MmaPlan {
    // Rows of 8 or 16 sixteen-byte chunks are stored unpadded with chunk c of row r
    // at c ^ (r & 7) (conflict-free ldmatrix); other widths are padded by 16 bytes.
    static constexpr int CPR = D * (int)sizeof(T) / 16;
#ifdef POPKV_ATTN_NO_SWIZZLE
    static constexpr bool SWZ = false;
#else
    static constexpr bool SWZ = CPR % 8 == 0;
#endif
    static constexpr int LDS = SWZ ? D : D + 8;
    static constexpr int kStageBytes = 2 * kTileRows * LDS * (int)sizeof(T);
    static constexpr int kRingBytes = kAttnWarps * kMmaStages * kStageBytes;
    static constexpr int kMergeBytes = kAttnWarps * kMaxGroup * (D + 2) * 4;
    static constexpr int kWorkBytes = kRingBytes > kMergeBytes ? kRingBytes : kMergeBytes;
    static constexpr int kListBytes = kSegMax * 2 + kSegMax * 2;  // uint16 offsets + head masks
};

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}

// Tokens in M, query heads in N.  Per 16-row tile a warp computes
// S^T = K_tile Q^T (16 tokens x 8 heads per n-tile, K_tile straight from the ring
// as the A operand, Q^T preloaded as B fragments), runs the online softmax per head
// column (reductions over the 8 lanes that share a column), turns P^T into B
// fragments with movmatrix, and accumulates O^T += V_tile^T P^T (head_dim in M,
// V^T read with ldmatrix.trans).  NHT = n-tiles of 8 query heads (G <= 8 * NHT).
// Q^T fragments (B operand) of the heads 8 nh + g of this CTA's KV head, channels
// 16 kk + 2 t (+1, +8, +9).  The queries are never written by this library's
// kernels, so the loads may run before griddepcontrol.wait.
template <typename T, int D, int NHT>
__device__ __forceinline__ void prefetch_q_fragments(uint32_t (&qb)[NHT][D / 16][2], const AttnParams& p) {
    const int b = blockIdx.y / p.KVH;
    const int kvh = blockIdx.y - b * p.KVH;
    const int g = (threadIdx.x & 31) >> 2, tig = threadIdx.x & 3;
    const int64_t qrow0 = static_cast<int64_t>(b) * p.QH + static_cast<int64_t>(kvh) * p.G;
    const T* q = static_cast<const T*>(p.q);
#pragma unroll
    for (int nh = 0; nh < NHT; ++nh) {
        const int h = 8 * nh + g;
        const uint32_t* qr = reinterpret_cast<const uint32_t*>(q + (qrow0 + (h < p.G ? h : 0)) * D);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            qb[nh][kk][0] = h < p.G ? __ldg(qr + 8 * kk + tig) : 0u;
            qb[nh][kk][1] = h < p.G ? __ldg(qr + 8 * kk + 4 + tig) : 0u;
        }
    }
}

template <typename T, int D, int NHT>
__global__ void __launch_bounds__(kAttnThreads, kMmaCtasPerSm) attention_mma_kernel(AttnParams p) {
    pdl_trigger();
    uint32_t qb[NHT][D / 16][2];
    prefetch_q_fragments<T, D, NHT>(qb, p);
    pdl_wait();
    using Plan = MmaPlan<T, D>;
    constexpr int LDS = Plan::LDS;
    constexpr int KS = D / 16;   // k-steps of QK^T
    constexpr int MT = D / 16;   // m-tiles of O^T
    constexpr int kStages = kMmaStages;
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* work = smem;
    uint16_t* s_tok = reinterpret_cast<uint16_t*>(smem + Plan::kWorkBytes);  // offsets from lo
    uint16_t* s_msk = s_tok + kSegMax;
    __shared__ int s_scan[kAttnWarps];

    const int s = blockIdx.x;
    const int b = blockIdx.y / p.KVH;
    const int kvh = blockIdx.y - b * p.KVH;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int g = lane >> 2;
    const int tig = lane & 3;
    const int64_t L = seq_length(p, b);
    const int64_t seg = segment_len(L, p.S);
    const int64_t lo = imin64(static_cast<int64_t>(s) * seg, L + 1);
    const int64_t hi = imin64(lo + seg, L + 1);
    const int64_t qrow0 = static_cast<int64_t>(b) * p.QH + static_cast<int64_t>(kvh) * p.G;
    const int n_union = build_union(p, b, kvh, lo, static_cast<int>(hi - lo), s_tok, s_msk, s_scan,
                                    p.dense != 0);

    const T* kc = static_cast<const T*>(p.kc);
    const T* vc = static_cast<const T*>(p.vc);
    const T* cur_k = static_cast<const T*>(p.cur_k);
    const T* cur_v = static_cast<const T*>(p.cur_v);
    const int64_t cache_head = (p.per_batch ? static_cast<int64_t>(b) * p.KVH : 0) + kvh;
    const int64_t cur_row = (static_cast<int64_t>(b) * p.KVH + kvh) * D;
    T* ring = reinterpret_cast<T*>(work) + warp * kStages * 2 * kTileRows * LDS;
    const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
    const T* kb = kc + (cache_head * p.kv_cap + lo) * D;  // row of offset 0
    const T* vb = vc + (cache_head * p.kv_cap + lo) * D;
    const T* ckr = cur_k != nullptr ? cur_k + cur_row : nullptr;
    const T* cvr = cur_v != nullptr ? cur_v + cur_row : nullptr;
    const int cur_off = static_cast<int>(L - lo);  // offset of the newest token

    // Copies of tile `tile` (16 union rows of K and V) into ring stage `st`; rows past
    // the union are zero-filled.
    auto issue = [&](int tile, int st) {
        constexpr int CPR = D * (int)sizeof(T) / 16;
        constexpr int EPC = 16 / (int)sizeof(T);
        constexpr uint32_t kStageB = 2 * kTileRows * LDS * sizeof(T);
        const uint32_t kd = ring_s + st * kStageB;
        const uint32_t vd = kd + kTileRows * LDS * sizeof(T);
#pragma unroll
        for (int c = lane; c < kTileRows * CPR; c += 32) {
            const int r = c / CPR;
            const int ch = c - r * CPR;
            const int e = tile * kTileRows + r;
            const bool in = e < n_union;
            const int t = in ? static_cast<int>(s_tok[e]) : 0;
            const bool cur = t == cur_off && ckr != nullptr;
            const T* ks = (cur ? ckr : kb + static_cast<int64_t>(t) * D) + ch * EPC;
            const T* vs = (cur ? cvr : vb + static_cast<int64_t>(t) * D) + ch * EPC;
            const int pch = Plan::SWZ ? (ch ^ (r & 7)) : ch;
            const uint32_t off = static_cast<uint32_t>((r * LDS + pch * EPC) * sizeof(T));
            cp_async16_s(kd + off, ks, in ? 16 : 0);
            cp_async16_s(vd + off, vs, in ? 16 : 0);
        }
    };

    float acc[MT][NHT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nh = 0; nh < NHT; ++nh) acc[mt][nh][0] = acc[mt][nh][1] = acc[mt][nh][2] = acc[mt][nh][3] = 0.0f;
    float m_run[NHT][2], l_run[NHT][2];  // heads 8 nh + 2 tig + j (l: this lane's tokens only)
#pragma unroll
    for (int nh = 0; nh < NHT; ++nh) {
        m_run[nh][0] = m_run[nh][1] = -INFINITY;
        l_run[nh][0] = l_run[nh][1] = 0.0f;
    }

    const int n_tiles = (n_union + kTileRows - 1) / kTileRows;
    const int my_tiles = n_tiles > warp ? (n_tiles - warp + kAttnWarps - 1) / kAttnWarps : 0;
#pragma unroll
    for (int st = 0; st < kStages - 1; ++st) {
        if (st < my_tiles) issue(warp + kAttnWarps * st, st);
        cp_async_commit();
    }
    for (int i = 0; i < my_tiles; ++i) {
        const int nxt = i + kStages - 1;
        if (nxt < my_tiles) issue(warp + kAttnWarps * nxt, nxt % kStages);
        cp_async_commit();
        cp_async_wait<kStages - 1>();
        __syncwarp();
        const int tile = warp + kAttnWarps * i;
        const T* Ks = ring + (i % kStages) * 2 * kTileRows * LDS;
        const T* Vs = Ks + kTileRows * LDS;

        // S^T = K Q^T: rows g, g + 8 of the tile, head columns 2 tig, 2 tig + 1.
        float sc[NHT][4];
#pragma unroll
        for (int nh = 0; nh < NHT; ++nh) sc[nh][0] = sc[nh][1] = sc[nh][2] = sc[nh][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            uint32_t a[4];
            const int r = lane & 15;
            const int kch = 2 * kk + (lane >> 4);
            ldmatrix_x4(a, Ks + r * LDS + (Plan::SWZ ? (kch ^ (r & 7)) : kch) * 8);
#pragma unroll
            for (int nh = 0; nh < NHT; ++nh) MmaOp<T>::run(sc[nh], a, qb[nh][kk][0], qb[nh][kk][1]);
        }
        const int e0 = tile * kTileRows + g;
        const uint32_t mk0 = e0 < n_union ? s_msk[e0] : 0u;
        const uint32_t mk1 = e0 + 8 < n_union ? s_msk[e0 + 8] : 0u;
        uint32_t pb[NHT][2];
        bool rescale = false;
        float corr[NHT][2];
#pragma unroll
        for (int nh = 0; nh < NHT; ++nh) {
            float pr[4];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int h = 8 * nh + 2 * tig + j;
                const float x0 = ((mk0 >> h) & 1u) ? sc[nh][j] * p.sl2 : -INFINITY;      // row g
                const float x1 = ((mk1 >> h) & 1u) ? sc[nh][2 + j] * p.sl2 : -INFINITY;  // row g + 8
                float tmax = fmaxf(x0, x1);
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
                const float m_new = fmaxf(m_run[nh][j], tmax);
                const float cr = (m_new == -INFINITY || m_new == m_run[nh][j]) ? 1.0f
                                                                               : exp2f(m_run[nh][j] - m_new);
                const float p0 = x0 == -INFINITY ? 0.0f : exp2f(x0 - m_new);
                const float p1 = x1 == -INFINITY ? 0.0f : exp2f(x1 - m_new);
                pr[j] = p0;
                pr[2 + j] = p1;
                l_run[nh][j] = fmaf(l_run[nh][j], cr, p0 + p1);
                m_run[nh][j] = m_new;
                corr[nh][j] = cr;
                rescale |= cr != 1.0f;
            }
            pb[nh][0] = movmatrix_trans(MmaOp<T>::pack(pr[0], pr[1]));  // tokens 0-7
            pb[nh][1] = movmatrix_trans(MmaOp<T>::pack(pr[2], pr[3]));  // tokens 8-15
        }
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int nh = 0; nh < NHT; ++nh) {
                    acc[mt][nh][0] *= corr[nh][0];
                    acc[mt][nh][1] *= corr[nh][1];
                    acc[mt][nh][2] *= corr[nh][0];
                    acc[mt][nh][3] *= corr[nh][1];
                }
        }
        // O^T += V^T P^T: head_dim rows 16 mt + g (+8), head columns 2 tig (+1).
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            uint32_t a[4];
            const int r = (lane & 7) + ((lane >> 4) << 3);
            const int vch = 2 * mt + ((lane >> 3) & 1);
            ldmatrix_x4_trans(a, Vs + r * LDS + (Plan::SWZ ? (vch ^ (r & 7)) : vch) * 8);
#pragma unroll
            for (int nh = 0; nh < NHT; ++nh) MmaOp<T>::run(acc[mt][nh], a, pb[nh][0], pb[nh][1]);
        }
        __syncwarp();
    }
    cp_async_wait<0>();
#pragma unroll
    for (int nh = 0; nh < NHT; ++nh)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            l_run[nh][j] += __shfl_xor_sync(0xffffffffu, l_run[nh][j], 4);
            l_run[nh][j] += __shfl_xor_sync(0xffffffffu, l_run[nh][j], 8);
            l_run[nh][j] += __shfl_xor_sync(0xffffffffu, l_run[nh][j], 16);
        }
    __syncthreads();  // ring no longer needed: reuse it for the warp merge
    float* s_wm = reinterpret_cast<float*>(work);            // [warps][16]
    float* s_wl = s_wm + kAttnWarps * kMaxGroup;              // [warps][16]
    float* s_wacc = s_wl + kAttnWarps * kMaxGroup;            // [warps][16][D]
#pragma unroll
    for (int nh = 0; nh < NHT; ++nh) {
        if (g == 0) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                s_wm[warp * kMaxGroup + 8 * nh + 2 * tig + j] = m_run[nh][j];
                s_wl[warp * kMaxGroup + 8 * nh + 2 * tig + j] = l_run[nh][j];
            }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            float* r0 = s_wacc + (warp * kMaxGroup + 8 * nh + 2 * tig) * D + 16 * mt + g;
            r0[0] = acc[mt][nh][0];
            r0[D] = acc[mt][nh][1];
            r0[8] = acc[mt][nh][2];
            r0[D + 8] = acc[mt][nh][3];
        }
    }
    __syncthreads();
    for (int i = tid; i < p.G * D; i += kAttnThreads) {
        const int h = i / D;
        const int d = i - h * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_wm[w * kMaxGroup + h]);
        float a = 0.0f, l = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                const float mw = s_wm[w * kMaxGroup + h];
                const float f = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
                a += f * s_wacc[(w * kMaxGroup + h) * D + d];
                l += f * s_wl[w * kMaxGroup + h];
            }
        }
        const int64_t prow = (qrow0 + h) * p.S + s;
        p.ws_acc[prow * D + d] = a;
        if (d == 0) {
            p.ws_m[prow] = M;
            p.ws_l[prow] = l;
        }
    }
}

// SIMT variant (fp32 caches, or head_dim outside the tensor-core instances).
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) attention_simt_kernel(AttnParams p) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(128) unsigned char smem[];
    // [0, work_bytes): merge / combine scratch; then token list and masks.
    int* s_tok = reinterpret_cast<int*>(smem + p.work_bytes);
    uint16_t* s_msk = reinterpret_cast<uint16_t*>(s_tok + kSegMax);
    __shared__ int s_scan[kAttnWarps];
    float* s_wm = reinterpret_cast<float*>(smem);
    float* s_wl = s_wm + kAttnWarps;
    float* s_wacc = s_wl + kAttnWarps;  // [warps][D]

    const int s = blockIdx.x;
    const int b = blockIdx.y / p.KVH;
    const int kvh = blockIdx.y - b * p.KVH;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int D = p.D;
    const int64_t L = seq_length(p, b);
    const int64_t seg = segment_len(L, p.S);
    const int64_t lo = imin64(static_cast<int64_t>(s) * seg, L + 1);
    const int64_t hi = imin64(lo + seg, L + 1);
    const int n_union = build_union(p, b, kvh, lo, static_cast<int>(hi - lo), s_tok, s_msk, s_scan,
                                    p.dense != 0);
    const T* q = static_cast<const T*>(p.q);
    const T* kc = static_cast<const T*>(p.kc);
    const T* vc = static_cast<const T*>(p.vc);
    const T* cur_k = static_cast<const T*>(p.cur_k);
    const T* cur_v = static_cast<const T*>(p.cur_v);
    const int64_t cache_head = (p.per_batch ? static_cast<int64_t>(b) * p.KVH : 0) + kvh;
    const int64_t cur_row = (static_cast<int64_t>(b) * p.KVH + kvh) * D;
    const int64_t qrow0 = static_cast<int64_t>(b) * p.QH + static_cast<int64_t>(kvh) * p.G;
    const float sl2 = p.sl2;

    for (int h = 0; h < p.G; ++h) {
        float qv[8], av[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = lane + 32 * j;
            qv[j] = c < D ? to_float<T>(q[(qrow0 + h) * D + c]) : 0.0f;
            av[j] = 0.0f;
        }
        float m_run = -INFINITY, l_run = 0.0f;
        for (int e = warp; e < n_union; e += kAttnWarps) {
            if (!((s_msk[e] >> h) & 1u)) continue;
            const int64_t t = s_tok[e];
            const T* kr = (t == L && cur_k) ? cur_k + cur_row : kc + (cache_head * p.kv_cap + t) * D;
            const T* vr = (t == L && cur_v) ? cur_v + cur_row : vc + (cache_head * p.kv_cap + t) * D;
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = lane + 32 * j;
                if (c < D) dot += qv[j] * to_float<T>(kr[c]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            const float xv = dot * sl2;
            const float m_new = fmaxf(m_run, xv);
            const float corr = exp2f(m_run - m_new);
            const float pe = exp2f(xv - m_new);
            l_run = l_run * corr + pe;
            m_run = m_new;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = lane + 32 * j;
                av[j] = av[j] * corr + (c < D ? pe * to_float<T>(vr[c]) : 0.0f);
            }
        }
        if (lane == 0) {
            s_wm[warp] = m_run;
            s_wl[warp] = l_run;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = lane + 32 * j;
            if (c < D) s_wacc[warp * D + c] = av[j];
        }
        __syncthreads();
        for (int d = tid; d < D; d += kAttnThreads) {
            float M = -INFINITY;
            for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_wm[w]);
            float a = 0.0f, l = 0.0f;
            if (M != -INFINITY) {
                for (int w = 0; w < kAttnWarps; ++w) {
                    const float f = (s_wm[w] == -INFINITY) ? 0.0f : exp2f(s_wm[w] - M);
                    a += f * s_wacc[w * D + d];
                    l += f * s_wl[w];
                }
            }
            const int64_t prow = (qrow0 + h) * p.S + s;
            p.ws_acc[prow * D + d] = a;
            if (d == 0) {
                p.ws_m[prow] = M;
                p.ws_l[prow] = l;
            }
        }
        __syncthreads();
    }
}

struct WorkspaceLayout {
    size_t tickets, masks, m, l, acc, total;
    int64_t mask_stride;
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

WorkspaceLayout layout(int64_t B, int64_t QH, int64_t KVH, int64_t D, int64_t tokens, int64_t S) {
    WorkspaceLayout w;
    w.mask_stride = (tokens + 1 + 7) / 8 * 8;
    w.tickets = 0;
    w.masks = w.tickets + align256(sizeof(uint32_t) * B * KVH);
    w.m = w.masks + align256(sizeof(uint16_t) * B * KVH * w.mask_stride);
    w.l = w.m + align256(sizeof(float) * B * QH * S);
    w.acc = w.l + align256(sizeof(float) * B * QH * S);
    w.total = w.acc + align256(sizeof(float) * B * QH * S * D);
    return w;
}

int64_t auto_splits(int64_t B, int64_t KVH, int64_t tokens) {
    const int64_t min_s = (tokens + 1 + (kSegMax - 8) - 1) / (kSegMax - 8);
    // One wave: every CTA resident at once (a partly filled second wave costs a
    // whole extra segment time).
    int64_t fill = (int64_t)kMmaCtasPerSm * num_sms() / (B * KVH);
    if (fill < 1) fill = 1;
    int64_t S = min_s > fill ? min_s : fill;
    const int64_t max_useful = (tokens + 1 + 63) / 64;  // keep >= 64 tokens per segment
    if (S > max_useful && max_useful >= min_s) S = max_useful;
    if (S < 1) S = 1;
    return S;
}

template <typename T, int D>
int launch_mma(const AttnParams& p, cudaStream_t st) {
    using Plan = MmaPlan<T, D>;
    const size_t smem = (size_t)Plan::kWorkBytes + Plan::kListBytes;
    if (smem > 227 * 1024) return fail(POPKV_ERR_UNSUPPORTED, "too many splits for shared memory");
    auto kern = p.G <= 8 ? attention_mma_kernel<T, D, 1> : attention_mma_kernel<T, D, 2>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(kern, dim3((unsigned)p.S, (unsigned)(p.B * p.KVH)), dim3(kAttnThreads), smem, st, p);
    const int rc = check_launch("popkv_sparse_attention");
    if (rc != POPKV_OK) return rc;
    launch_combine<T>(p, st);
    return check_launch("popkv_sparse_attention (combine)");
}

template <typename T>
int launch_simt(AttnParams p, cudaStream_t st) {
    const int merge = (2 * kAttnWarps + kAttnWarps * p.D) * 4;
    p.work_bytes = (merge + 15) / 16 * 16;
    const size_t smem = (size_t)p.work_bytes + kSegMax * 6;
    if (smem > 227 * 1024) return fail(POPKV_ERR_UNSUPPORTED, "too many splits for shared memory");
    auto kern = attention_simt_kernel<T>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(kern, dim3((unsigned)p.S, (unsigned)(p.B * p.KVH)), dim3(kAttnThreads), smem, st, p);
    const int rc = check_launch("popkv_sparse_attention");
    if (rc != POPKV_OK) return rc;
    launch_combine<T>(p, st);
    return check_launch("popkv_sparse_attention (combine)");
}

}  // namespace
}  // namespace popkv

using namespace popkv;


extern "C" size_t popkv_sparse_attention_workspace_bytes(int64_t batch, int64_t q_heads,
                                                         int64_t kv_heads, int64_t head_dim,
                                                         int64_t tokens, int64_t splits) {
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || tokens < 0) return 0;
    const int64_t S = splits > 0 ? splits : auto_splits(batch, kv_heads, tokens);
    return layout(batch, q_heads, kv_heads, head_dim, tokens, S).total;
}

enum AttnMode { kFromIndices = 0, kDense = 1, kPremasked = 2 };

static int attention_impl(const void* queries, int dtype, int64_t batch, int64_t q_heads,
                          int64_t head_dim, const void* key_cache, const void* value_cache,
                          int64_t kv_heads, int64_t kv_capacity, int cache_per_batch,
                          const void* current_keys, const void* current_values,
                          const int32_t* indices, int64_t index_stride, int64_t budget,
                          int64_t tokens, const int32_t* seq_len, void* out, void* workspace,
                          size_t workspace_bytes, int64_t splits, popkv_stream_t stream,
                          int mode, int world = 1, int rank = 0, void* const* peer_out = nullptr,
                          uint32_t* const* peer_flags = nullptr, uint32_t* sync_words = nullptr,
                          int peer_defer = 0, bool check_only = false) {
    const size_t es = dtype_size(dtype);
    if (es == 0) return fail(POPKV_ERR_UNSUPPORTED, "dtype %d is not fp32/fp16/bf16", dtype);
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid attention shape");
    if (q_heads % kv_heads != 0 || q_heads / kv_heads > kMaxGroup)
        return fail(POPKV_ERR_UNSUPPORTED, "q_heads/kv_heads must be an integer <= %d", kMaxGroup);
    if (head_dim > 256 || head_dim % 8 != 0)
        return fail(POPKV_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and <= 256");
    if (tokens < 0 || tokens >= kv_capacity + (current_keys ? 1 : 0))
        return fail(POPKV_ERR_CAPACITY, "tokens %lld do not fit the KV capacity %lld",
                    (long long)tokens, (long long)kv_capacity);
    if ((current_keys == nullptr) != (current_values == nullptr))
        return fail(POPKV_ERR_INVALID_ARGUMENT, "current_keys and current_values go together");
    if (indices != nullptr && (budget <= 1 || index_stride < budget))
        return fail(POPKV_ERR_INVALID_ARGUMENT, "indices need budget > 1 and index_stride >= budget");
    if (!queries || !key_cache || !value_cache || !out || !workspace)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    if (!aligned(key_cache, 16) || !aligned(value_cache, 16) || !aligned(queries, 16) ||
        !aligned(workspace, 256) || (current_keys && (!aligned(current_keys, 16) || !aligned(current_values, 16))))
        return fail(POPKV_ERR_ALIGNMENT, "caches, queries and current rows need 16-byte alignment, workspace 256");
    const int64_t S = splits > 0 ? splits : auto_splits(batch, kv_heads, tokens);
    if (S > kMaxSplits) return fail(POPKV_ERR_UNSUPPORTED, "splits %lld > %d", (long long)S, kMaxSplits);
    if (((tokens + 1 + S - 1) / S + 7) / 8 * 8 > kSegMax)
        return fail(POPKV_ERR_UNSUPPORTED, "segment longer than %d tokens: raise splits", kSegMax);
    if (batch * kv_heads > 65535) return fail(POPKV_ERR_UNSUPPORTED, "too many (batch, kv head) pairs");
    const WorkspaceLayout w = layout(batch, q_heads, kv_heads, head_dim, tokens, S);
    if (workspace_bytes < w.total)
        return fail(POPKV_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", workspace_bytes, w.total);

    AttnParams p;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    p.q = queries; p.kc = key_cache; p.vc = value_cache;
    p.cur_k = current_keys; p.cur_v = current_values; p.out = out;
    p.indices = indices; p.index_stride = index_stride; p.budget = budget;
    p.masks = reinterpret_cast<uint16_t*>(ws + w.masks);
    p.mask_stride = w.mask_stride;
    p.ws_m = reinterpret_cast<float*>(ws + w.m);
    p.ws_l = reinterpret_cast<float*>(ws + w.l);
    p.ws_acc = reinterpret_cast<float*>(ws + w.acc);
    p.tickets = reinterpret_cast<uint32_t*>(ws + w.tickets);
    p.B = (int)batch; p.QH = (int)q_heads; p.KVH = (int)kv_heads;
    p.G = (int)(q_heads / kv_heads); p.D = (int)head_dim;
    p.kv_cap = kv_capacity; p.per_batch = cache_per_batch != 0;
    p.tokens = tokens; p.seq_len = seq_len; p.S = (int)S;
    p.sl2 = (float)((1.0 / std::sqrt((double)head_dim)) * 1.4426950408889634);
    p.work_bytes = 0;
    p.dense = mode == kDense;
    p.world = 1;
    p.rank = 0;
    p.sync = nullptr;
    p.peer_defer = 0;
    for (int j = 0; j < kMaxPeers; ++j) { p.peer_out[j] = nullptr; p.peer_flags[j] = nullptr; }
    if (world > 1) {
        if (world > kMaxPeers || rank < 0 || rank >= world || !peer_out || !peer_flags || !sync_words)
            return fail(POPKV_ERR_INVALID_ARGUMENT, "peer gather needs 1 < world <= %d, rank < world, peer "
                        "pointers and sync words", kMaxPeers);
        for (int j = 0; j < world; ++j) {
            if (!peer_out[j] || !peer_flags[j] || !aligned(peer_out[j], 16) || !aligned(peer_flags[j], 4))
                return fail(POPKV_ERR_INVALID_ARGUMENT, "peer %d: null or misaligned gather pointer", j);
            p.peer_out[j] = peer_out[j];
            p.peer_flags[j] = peer_flags[j];
        }
        p.world = world;
        p.rank = rank;
        p.sync = sync_words;
        p.peer_defer = peer_defer != 0;
    }
    if (check_only) return POPKV_OK;  // every argument check passed; nothing launched
    const cudaStream_t st = as_stream(stream);

    if (mode == kFromIndices) {
        const int64_t per_row = (budget < tokens + 1 ? budget : tokens + 1);
        const dim3 grid((unsigned)((per_row + 255) / 256), (unsigned)(batch * q_heads));
        launch_pdl(scatter_kernel, grid, dim3(256), 0, st, p);
        const int rc = check_launch("popkv_sparse_attention (scatter)");
        if (rc != POPKV_OK) return rc;
    }
    if (dtype == POPKV_BF16) {
        if (head_dim == 128) return launch_mma<__nv_bfloat16, 128>(p, st);
        if (head_dim == 64) return launch_mma<__nv_bfloat16, 64>(p, st);
        if (head_dim == 96) return launch_mma<__nv_bfloat16, 96>(p, st);
        return launch_simt<__nv_bfloat16>(p, st);
    }
    if (dtype == POPKV_F16) {
        if (head_dim == 128) return launch_mma<__half, 128>(p, st);
        if (head_dim == 64) return launch_mma<__half, 64>(p, st);
        if (head_dim == 96) return launch_mma<__half, 96>(p, st);
        return launch_simt<__half>(p, st);
    }
    return launch_simt<float>(p, st);
}

extern "C" int popkv_sparse_attention(const void* queries, int dtype, int64_t batch,
                                      int64_t q_heads, int64_t head_dim, const void* key_cache,
                                      const void* value_cache, int64_t kv_heads,
                                      int64_t kv_capacity, int cache_per_batch,
                                      const void* current_keys, const void* current_values,
                                      const int32_t* indices, int64_t index_stride,
                                      int64_t budget, int64_t tokens, const int32_t* seq_len,
                                      void* out, void* workspace, size_t workspace_bytes,
                                      int64_t splits, popkv_stream_t stream) {
    return attention_impl(queries, dtype, batch, q_heads, head_dim, key_cache, value_cache,
                          kv_heads, kv_capacity, cache_per_batch, current_keys, current_values,
                          indices, index_stride, budget, tokens, seq_len, out, workspace,
                          workspace_bytes, splits, stream, indices ? kFromIndices : kDense);
}

extern "C" int popkv_sparse_attention_premasked(
    const void* queries, int dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* key_cache, const void* value_cache, int64_t kv_heads, int64_t kv_capacity,
    int cache_per_batch, const void* current_keys, const void* current_values, int64_t tokens,
    const int32_t* seq_len, void* out, void* workspace, size_t workspace_bytes, int64_t splits,
    popkv_stream_t stream) {
    return attention_impl(queries, dtype, batch, q_heads, head_dim, key_cache, value_cache,
                          kv_heads, kv_capacity, cache_per_batch, current_keys, current_values,
                          nullptr, 0, 2, tokens, seq_len, out, workspace, workspace_bytes, splits,
                          stream, kPremasked);
}

extern "C" int popkv_sparse_attention_premasked_gather(
    const void* queries, int dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* key_cache, const void* value_cache, int64_t kv_heads, int64_t kv_capacity,
    int cache_per_batch, const void* current_keys, const void* current_values, int64_t tokens,
    const int32_t* seq_len, void* out, void* workspace, size_t workspace_bytes, int64_t splits,
    int world, int rank, void* const* peer_out, uint32_t* const* peer_flags, uint32_t* sync_words,
    int defer_wait, popkv_stream_t stream) {
    return attention_impl(queries, dtype, batch, q_heads, head_dim, key_cache, value_cache,
                          kv_heads, kv_capacity, cache_per_batch, current_keys, current_values,
                          nullptr, 0, 2, tokens, seq_len, out, workspace, workspace_bytes, splits,
                          stream, kPremasked, world, rank, peer_out, peer_flags, sync_words,
                          defer_wait);
}

extern "C" int popkv_peer_push(const void* rows, int64_t bytes, void* const* peer_dst,
                               uint32_t* const* peer_flags, int rank, int world,
                               uint32_t* sync_words, popkv_stream_t stream) {
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "peer push needs 1 <= world <= %d and 0 <= rank < world", kMaxPeers);
    if (bytes <= 0 || bytes % 16 != 0 || !aligned(rows, 16))
        return fail(POPKV_ERR_ALIGNMENT, "peer push moves 16-byte aligned rows in whole 16-byte chunks");
    if (!peer_dst || !peer_flags || !sync_words) return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    PushArgs a = {};
    a.src = static_cast<const uint4*>(rows);
    for (int j = 0; j < world; ++j) {
        if (!peer_dst[j] || !aligned(peer_dst[j], 16) || !peer_flags[j])
            return fail(POPKV_ERR_ALIGNMENT, "peer buffers must be 16-byte aligned");
        a.dst[j] = static_cast<uint4*>(peer_dst[j]);
        a.flags[j] = peer_flags[j];
    }
    a.sync = sync_words;
    a.chunks = bytes / 16;
    a.world = world;
    a.rank = rank;
    launch_pdl(peer_push_kernel, dim3(1), dim3(256), 0, as_stream(stream), a);
    return check_launch("popkv_peer_push");
}

extern "C" int popkv_peer_gather_wait(const uint32_t* own_flags, uint32_t* sync_words, int layers,
                                      int world, popkv_stream_t stream) {
    if (layers <= 0 || world < 2 || world > kMaxPeers || !own_flags || !sync_words)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "peer wait needs layers > 0, 1 < world <= %d and "
                    "flag / sync pointers", kMaxPeers);
    if (!aligned(own_flags, 4) || !aligned(sync_words, 4))
        return fail(POPKV_ERR_ALIGNMENT, "flag and sync words need 4-byte alignment");
    const int threads = layers < 256 ? (layers + 31) / 32 * 32 : 256;
    launch_pdl(peer_wait_kernel, dim3(1), dim3((unsigned)threads), 0, as_stream(stream), own_flags,
               sync_words, layers, world);
    return check_launch("popkv_peer_gather_wait");
}

extern "C" int popkv_sparse_attention_masks(void* workspace, int64_t batch, int64_t q_heads,
                                            int64_t kv_heads, int64_t head_dim, int64_t tokens,
                                            int64_t splits, uint16_t** masks,
                                            int64_t* mask_stride) {
    if (!workspace || !masks || !mask_stride) return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || tokens < 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid attention shape");
    const int64_t S = splits > 0 ? splits : auto_splits(batch, kv_heads, tokens);
    const WorkspaceLayout w = layout(batch, q_heads, kv_heads, head_dim, tokens, S);
    *masks = reinterpret_cast<uint16_t*>(static_cast<unsigned char*>(workspace) + w.masks);
    *mask_stride = w.mask_stride;
    return POPKV_OK;
}

// ----------------------------------------------------------------------------
// Allocation-free variant of popkv_sparse_attention.
//
// Some callers cannot allocate device memory at all: plugins that run inside a
// host engine owning every allocation through its own pool, code paths that must
// not call cudaMalloc while the engine holds its allocator lock, or embedders with
// no allocator they may call.  For them this entry point takes its scratch from a
// fixed array compiled into the library instead of a caller workspace.  The array
// lives in every GPU that loads the library until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = POPKV_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once per
// device (the host-side symbol is not a device address).
int noalloc_scratch(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(POPKV_ERR_UNSUPPORTED, "device index %d", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(POPKV_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        g_noalloc_ptr[dev] = ptr;
    }
    *out = g_noalloc_ptr[dev];
    return POPKV_OK;
}

}  // namespace

extern "C" int popkv_sparse_attention_noalloc(
    const void* queries, int dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* key_cache, const void* value_cache, int64_t kv_heads, int64_t kv_capacity,
    int cache_per_batch, const void* current_keys, const void* current_values,
    const int32_t* indices, int64_t index_stride, int64_t budget, int64_t tokens,
    const int32_t* seq_len, void* out, int64_t splits, popkv_stream_t stream) {
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || tokens < 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid attention shape");
    const int64_t S = splits > 0 ? splits : auto_splits(batch, kv_heads, tokens);
    const WorkspaceLayout w = layout(batch, q_heads, kv_heads, head_dim, tokens, S);
    if (w.total > kNoAllocScratchBytes)
        return fail(POPKV_ERR_WORKSPACE,
                    "popkv_sparse_attention_noalloc needs %zu bytes of scratch for these sizes; "
                    "its fixed scratch holds %zu (use popkv_sparse_attention with a workspace)",
                    w.total, kNoAllocScratchBytes);
    void* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc != POPKV_OK) return rc;
    // Run every argument check first, so that a rejected call leaves the shared
    // scratch (and the stream) untouched.
    rc = attention_impl(queries, dtype, batch, q_heads, head_dim, key_cache, value_cache, kv_heads,
                        kv_capacity, cache_per_batch, current_keys, current_values, indices,
                        index_stride, budget, tokens, seq_len, out, scratch, kNoAllocScratchBytes, S,
                        stream, indices ? kFromIndices : kDense, 1, 0, nullptr, nullptr, nullptr, 0,
                        /*check_only=*/true);
    if (rc != POPKV_OK) return rc;
    // The tickets and head masks must start at zero; the array keeps whatever the
    // previous call (of any sizes) left there.
    const cudaError_t e = cudaMemsetAsync(scratch, 0, w.m, as_stream(stream));
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "clearing scratch: %s", cudaGetErrorString(e));
    return popkv_sparse_attention(queries, dtype, batch, q_heads, head_dim, key_cache, value_cache,
                                  kv_heads, kv_capacity, cache_per_batch, current_keys,
                                  current_values, indices, index_stride, budget, tokens, seq_len,
                                  out, scratch, kNoAllocScratchBytes, S, stream);
}
