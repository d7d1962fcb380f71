// (a) Key packer and (b) incremental append / open-group re-pack.
//
// Semantics follow the reference packer popkv_pack_g32_kernel
// (csrc/popkv_ext.cu:29-91): per 32-token group and channel, thresholds
// max*0.5 / min*0.5; per token, a sign bit (v >= 0) and a magnitude bit
// (v > max/2 for v >= 0, v < min/2 otherwise) per channel, packed 32 channels
// to a word with channel 32w+i at bit i; per (token, word) the mean |v| of the
// low and high lanes, summed in __shfl_down tree order (offsets 16..1), stored
// as fp16 low and fp16 (high - low).
//
// B200 layout of the work: one CTA of 32*W threads per (head, group) instead of
// one warp per (head, group, word).  The 32 x D group tile is read from HBM once
// with 16-byte loads into shared memory (the reference walks it twice with
// 2-byte loads), thresholds come from a channel-per-thread pass, and the
// (token, word) outputs are computed one per thread and written back as
// contiguous runs.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"

namespace popkv {
namespace {

constexpr int kGroup = 32;

__host__ __device__ constexpr int tile_ld(int d) { return (d % 2 == 0) ? d + 1 : d; }

struct PackSmem {
    float* tile;      // [32][ld]
    float* neg;       // [D]
    float* pos;       // [D]
    uint32_t* sign;   // [32*W]
    uint32_t* mag;    // [32*W]
    uint16_t* low;    // [32*W]
    uint16_t* delta;  // [32*W]
};

template <int W>
__device__ __forceinline__ PackSmem carve(unsigned char* raw, int D) {
    PackSmem s;
    s.tile = reinterpret_cast<float*>(raw);
    s.neg = s.tile + kGroup * tile_ld(D);
    s.pos = s.neg + D;
    s.sign = reinterpret_cast<uint32_t*>(s.pos + D);
    s.mag = s.sign + kGroup * W;
    s.low = reinterpret_cast<uint16_t*>(s.mag + kGroup * W);
    s.delta = s.low + kGroup * W;
    return s;
}

inline size_t pack_smem_bytes(int D, int W) {
    return sizeof(float) * (size_t)(kGroup * tile_ld(D) + 2 * D) +
           sizeof(uint32_t) * 2 * kGroup * W + sizeof(uint16_t) * 2 * kGroup * W;
}

// Loads row t (t < n) of the tile.  `row` maps a tile row to its source pointer.
template <typename T, typename RowFn>
__device__ __forceinline__ void load_tile(float* tile, int ld, int n, int D, bool vec_ok,
                                          RowFn row) {
    constexpr int VEC = 16 / sizeof(T);
    if (vec_ok) {
        const int vpr = D / VEC;
        for (int i = threadIdx.x; i < n * vpr; i += blockDim.x) {
            const int t = i / vpr;
            const int c0 = (i - t * vpr) * VEC;
            const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row(t) + c0));
            const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
            for (int j = 0; j < VEC; ++j) tile[t * ld + c0 + j] = to_float<T>(v[j]);
        }
    } else {
        for (int i = threadIdx.x; i < n * D; i += blockDim.x) {
            const int t = i / D;
            const int c = i - t * D;
            tile[t * ld + c] = to_float<T>(row(t)[c]);
        }
    }
}

// Packs a loaded tile of n (1..32) tokens and writes packed rows out_row0 .. out_row0+n-1.
template <int W>
__device__ __forceinline__ void pack_tile(const PackSmem& s, int n, int D, int64_t out_row0,
                                          int32_t* __restrict__ k_sign,
                                          int32_t* __restrict__ k_mag,
                                          uint16_t* __restrict__ low_out,
                                          uint16_t* __restrict__ delta_out,
                                          float* __restrict__ thresholds, bool ref_div) {
    const int ld = tile_ld(D);
    const int tid = threadIdx.x;
    // Thresholds: one thread per channel, min/max over the group's tokens.
    if (tid < D) {
        float mn = s.tile[tid], mx = mn;
        for (int t = 1; t < n; ++t) {
            const float v = s.tile[t * ld + tid];
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
        s.neg[tid] = mn * 0.5f;
        s.pos[tid] = mx * 0.5f;
        if (thresholds != nullptr) {
            thresholds[2 * tid] = s.neg[tid];
            thresholds[2 * tid + 1] = s.pos[tid];
        }
    }
    __syncthreads();
    // One thread per (token, word): warp w = word, lane = token.
    const int w = tid >> 5;
    const int t = tid & 31;
    if (t < n) {
        uint32_t sw = 0u, mw = 0u;
        float lo[32], hi[32];
        int lc = 0, hc = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int c = w * 32 + i;
            const bool valid = c < D;
            const float v = valid ? s.tile[t * ld + c] : 0.0f;
            const bool sg = valid && v >= 0.0f;
            const bool mg = valid && (sg ? (v > s.pos[c]) : (v < s.neg[c]));
            sw |= static_cast<uint32_t>(sg) << i;
            mw |= static_cast<uint32_t>(mg) << i;
            lo[i] = (!mg && valid) ? fabsf(v) : 0.0f;
            hi[i] = (mg && valid) ? fabsf(v) : 0.0f;
            lc += (!mg && valid);
            hc += mg;
        }
        // Lane-0 result of a shfl_down tree with offsets 16, 8, 4, 2, 1.
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
            for (int i = 0; i < off; ++i) {
                lo[i] = lo[i] + lo[i + off];
                hi[i] = hi[i] + hi[i + off];
            }
        }
        float low, high;
        representatives(lo[0], lc, hi[0], hc, ref_div, low, high);
        s.sign[t * W + w] = sw;
        s.mag[t * W + w] = mw;
        s.low[t * W + w] = __half_as_ushort(__float2half_rn(low));
        s.delta[t * W + w] = __half_as_ushort(__float2half_rn(high - low));
    }
    __syncthreads();
    const int64_t base = out_row0 * W;
    for (int i = tid; i < n * W; i += blockDim.x) {
        k_sign[base + i] = static_cast<int32_t>(s.sign[i]);
        k_mag[base + i] = static_cast<int32_t>(s.mag[i]);
        low_out[base + i] = s.low[i];
        delta_out[base + i] = s.delta[i];
    }
}

template <typename T, int W>
__global__ void __launch_bounds__(32 * W)
pack_kernel(const T* __restrict__ keys, int64_t tokens, int D, int64_t head_stride,
            int64_t groups, int32_t* __restrict__ k_sign, int32_t* __restrict__ k_mag,
            uint16_t* __restrict__ low, uint16_t* __restrict__ delta, int64_t capacity,
            int64_t token_offset, float* __restrict__ thresholds, bool vec_ok, bool ref_div) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const PackSmem s = carve<W>(smem_raw, D);
    const int64_t h = blockIdx.x / groups;
    const int64_t g = blockIdx.x - h * groups;
    const int64_t t0 = g * kGroup;
    const int n = static_cast<int>(imin64(kGroup, tokens - t0));
    const T* src = keys + h * head_stride + t0 * D;
    load_tile<T>(s.tile, tile_ld(D), n, D, vec_ok, [&](int t) { return src + (int64_t)t * D; });
    __syncthreads();
    float* thr = thresholds ? thresholds + (h * groups + g) * (int64_t)D * 2 : nullptr;
    pack_tile<W>(s, n, D, h * capacity + token_offset + t0, k_sign, k_mag, low, delta, thr,
                 ref_div);
}

// ------------------------------------------------------------------ streaming packer
// Prefill packing of whole heads (rows a multiple of 128 bytes: head_dim % 64 == 0
// for 16-bit keys, % 32 for fp32): a grid of a few CTAs per SM walks the
// (head, group) list; each CTA keeps kPackStages group tiles in flight, each brought
// in by TMA tensor copies of [32 tokens x 128 bytes] boxes with the 128-byte swizzle
// (16-byte chunk c of token row r lands at chunk c ^ (r & 7), so a warp reading the
// same word of 32 rows hits distinct banks), completed on the stage's "full"
// mbarrier.  Tokens past the end of a head arrive as zeros and are not used.
// Warp w owns word w: it first reduces the word's 32 channels over the group's
// tokens (the warp's own thresholds), then lane t packs token t's word and stores
// it.  Warps meet only on the stage's "empty" mbarrier, which warp 0 waits on before
// refilling the stage with the group kPackStages ahead; no block barrier.
//
// 16-bit keys are compared two channels at a time: with max, min and v all
// bf16/fp16 values, v > max*0.5 <=> v+v > max and v < min*0.5 <=> v+v < min exactly
// (max*0.5 is exact in fp32, doubling a 16-bit value is exact or overflows to an
// infinity on the same side), and (v >= 0 ? v > pos : v < neg) equals
// (v > pos || v < neg) because pos >= 0 whenever some v >= 0 and neg <= v whenever
// v >= 0.
constexpr int kPackStages = 4;
constexpr int kBoxBytes = kGroup * 128;  // one [32 x 128 B] swizzled box
__device__ unsigned int g_pack_wait_timeouts = 0;

template <typename T, int W>
struct StreamSmem {
    static constexpr int kBoxes = 32 * W * (int)sizeof(T) / 128;
    static constexpr int kTile = kBoxes * kBoxBytes;
    static constexpr size_t bytes() {
        return 1024 + (size_t)kPackStages * kTile + (size_t)W * 64 * sizeof(float) +
               2 * kPackStages * sizeof(uint64_t);
    }
};

// Shared-memory address of byte `off` (within the 16-byte chunk) of token row t.
__device__ __forceinline__ int swz(int t, int off) {
    const int b = off >> 7, c = (off & 127) >> 4;
    return b * kBoxBytes + t * 128 + ((c ^ (t & 7)) << 4) + (off & 15);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
    using T2 = __nv_bfloat162;
    static __device__ __forceinline__ float lo_f(uint32_t bits) { return __uint_as_float(bits << 16); }
    static __device__ __forceinline__ float hi_f(uint32_t bits) { return __uint_as_float(bits & 0xffff0000u); }
};
template <> struct Pair<__half> {
    using T2 = __half2;
    static __device__ __forceinline__ float lo_f(uint32_t bits) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xffffu)));
    }
    static __device__ __forceinline__ float hi_f(uint32_t bits) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(bits >> 16)));
    }
};

template <typename T2> __device__ __forceinline__ T2 as_pair(uint32_t u) { return *reinterpret_cast<T2*>(&u); }
template <typename T2> __device__ __forceinline__ uint32_t pair_bits(T2 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Bits 0..15 of x to the even bits of the result.
__device__ __forceinline__ uint32_t spread_even(uint32_t x) {
    x &= 0xffffu;
    x = (x | (x << 8)) & 0x00ff00ffu;
    x = (x | (x << 4)) & 0x0f0f0f0fu;
    x = (x | (x << 2)) & 0x33333333u;
    x = (x | (x << 1)) & 0x55555555u;
    return x;
}

// Lane-0 result of a shfl_down tree (offsets 16..1) over lo[] and hi[], both sums
// carried in one f32x2 register per channel.
__device__ __forceinline__ float2 tree_sums(float2 (&v)[32]) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int c = 0; c < off; ++c) v[c] = __fadd2_rn(v[c], v[c + off]);
    }
    return v[0];
}

template <typename T, int W>
__global__ void __launch_bounds__(32 * W)
pack_stream_kernel(const __grid_constant__ CUtensorMap key_map, int64_t tokens, int64_t groups,
                   int64_t total, int32_t* __restrict__ k_sign, int32_t* __restrict__ k_mag,
                   uint16_t* __restrict__ low, uint16_t* __restrict__ delta, int64_t capacity,
                   int64_t token_offset, float* __restrict__ thresholds, bool ref_div) {
    pdl_trigger();
    pdl_wait();
    using S = StreamSmem<T, W>;
    constexpr int D = 32 * W;
    constexpr int kWordBytes = 32 * (int)sizeof(T);
    constexpr int kBoxElems = 128 / (int)sizeof(T);
    constexpr bool kPaired = sizeof(T) == 2;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // 1024-byte aligned for the swizzled boxes (pointer arithmetic on the shared array
    // keeps the loads in the shared window).
    unsigned char* tiles = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    float* thr = reinterpret_cast<float*>(tiles + kPackStages * S::kTile);  // [W][64]
    uint64_t* full = reinterpret_cast<uint64_t*>(thr + W * 64);
    uint64_t* empty = full + kPackStages;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int w = tid >> 5;

    auto group_of = [&](int64_t i, int64_t& h, int64_t& t0, int& n) {
        h = i / groups;
        t0 = (i - h * groups) * kGroup;
        n = static_cast<int>(imin64(kGroup, tokens - t0));
    };
    // One thread fills stage s with group i.
    auto issue = [&](int64_t i, int s) {
        int64_t h, t0;
        int n;
        group_of(i, h, t0, n);
        mbar_expect_tx(&full[s], (uint32_t)S::kTile);
#pragma unroll
        for (int bx = 0; bx < S::kBoxes; ++bx)
            tma_load_3d(tiles + s * S::kTile + bx * kBoxBytes, &key_map, bx * kBoxElems, (int)t0,
                        (int)h, &full[s]);
    };
    if (tid == 0) {
        for (int s = 0; s < kPackStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const int64_t first = blockIdx.x, step = gridDim.x;
    if (tid == 0)
        for (int s = 0; s < kPackStages; ++s)
            if (first + s * step < total) issue(first + s * step, s);

    int it = 0;
    for (int64_t i = first; i < total; i += step, ++it) {
        const int s = it % kPackStages;
        const uint32_t parity = (uint32_t)(it / kPackStages) & 1u;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], parity))) {
            // A copy never completed: record it and leave; warp 0 first waits (bounded)
            // for the copies it still has in flight.
            if (lane == 0) atomicAdd(&g_pack_wait_timeouts, 1u);
            if (tid == 0)
                for (int k = 1; k < kPackStages; ++k)
                    if (i + (int64_t)k * step < total)
                        mbar_wait_bounded(&full[(it + k) % kPackStages],
                                          (uint32_t)((it + k) / kPackStages) & 1u);
            return;
        }
        int64_t h, t0;
        int n;
        group_of(i, h, t0, n);
        const unsigned char* tile = tiles + s * S::kTile;
        float* wthr = thr + w * 64;
        const int64_t grp = h * groups + t0 / kGroup;
        const int64_t out = (h * capacity + token_offset + t0 + lane) * W + w;
        float2 sums[32];  // (low-lane sum, high-lane sum) per channel, before the tree
        uint32_t sw = 0u, mw = 0u;
        if constexpr (kPaired) {
            using P2 = typename Pair<T>::T2;
            uint32_t* wmm = reinterpret_cast<uint32_t*>(wthr);  // [16] max pairs, [16] min pairs
            {
                // Lane (pair p, half) reduces channels 2p, 2p+1 over tokens 16*half..+15
                // (tokens past n repeat token 0).
                const int p = lane & 15, half = lane >> 4;
                const int off = w * kWordBytes + 4 * p;
                P2 mx = as_pair<P2>(*reinterpret_cast<const uint32_t*>(tile + swz(0, off))), mn = mx;
                if (n == kGroup) {
                    // Row 16*half+k sits at k*128 past row 16*half, its chunk XOR-ed with k&7.
                    const unsigned char* base = tile + swz(16 * half, off);
                    const int cx = (off & 127) >> 4;
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int d = (((cx ^ (k & 7)) - cx) << 4) + k * 128;
                        const P2 x = as_pair<P2>(*reinterpret_cast<const uint32_t*>(base + d));
                        mx = __hmax2(mx, x);
                        mn = __hmin2(mn, x);
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int t = 16 * half + k;
                        const P2 x = as_pair<P2>(*reinterpret_cast<const uint32_t*>(tile + swz(t < n ? t : 0, off)));
                        mx = __hmax2(mx, x);
                        mn = __hmin2(mn, x);
                    }
                }
                mx = __hmax2(mx, as_pair<P2>(__shfl_xor_sync(0xffffffffu, pair_bits(mx), 16)));
                mn = __hmin2(mn, as_pair<P2>(__shfl_xor_sync(0xffffffffu, pair_bits(mn), 16)));
                if (half == 0) {
                    wmm[p] = pair_bits(mx);
                    wmm[16 + p] = pair_bits(mn);
                    if (thresholds != nullptr) {
                        float4* tg = reinterpret_cast<float4*>(thresholds + grp * (int64_t)D * 2) + (32 * w + 2 * p) / 2;
                        *tg = make_float4(Pair<T>::lo_f(pair_bits(mn)) * 0.5f, Pair<T>::lo_f(pair_bits(mx)) * 0.5f,
                                          Pair<T>::hi_f(pair_bits(mn)) * 0.5f, Pair<T>::hi_f(pair_bits(mx)) * 0.5f);
                    }
                }
            }
            __syncwarp();
            if (lane < n) {
                uint32_t r[16], mxv[16], mnv[16];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint4 a = *reinterpret_cast<const uint4*>(tile + swz(lane, w * kWordBytes + 16 * j));
                    const uint4 b = reinterpret_cast<const uint4*>(wmm)[j];
                    const uint4 c = reinterpret_cast<const uint4*>(wmm + 16)[j];
                    r[4 * j] = a.x; r[4 * j + 1] = a.y; r[4 * j + 2] = a.z; r[4 * j + 3] = a.w;
                    mxv[4 * j] = b.x; mxv[4 * j + 1] = b.y; mxv[4 * j + 2] = b.z; mxv[4 * j + 3] = b.w;
                    mnv[4 * j] = c.x; mnv[4 * j + 1] = c.y; mnv[4 * j + 2] = c.z; mnv[4 * j + 3] = c.w;
                }
                uint32_t am = 0u, as = 0u;  // bit p: channel 2p, bit 16+p: channel 2p+1
                const P2 zero = as_pair<P2>(0u);
                float2 lo2[16], hi2[16];      // (channel 2p, channel 2p+1)
#pragma unroll
                for (int p = 0; p < 16; ++p) {
                    const P2 x = as_pair<P2>(r[p]);
                    const P2 x2 = __hadd2(x, x);
                    const uint32_t m = __hgt2_mask(x2, as_pair<P2>(mxv[p])) | __hlt2_mask(x2, as_pair<P2>(mnv[p]));
                    am |= m & (0x00010001u << p);
                    as |= __hge2_mask(x, zero) & (0x00010001u << p);
                    const uint32_t rm = r[p] & m & 0x7fff7fffu, rn = r[p] & ~m & 0x7fff7fffu;
                    lo2[p] = make_float2(Pair<T>::lo_f(rn), Pair<T>::hi_f(rn));
                    hi2[p] = make_float2(Pair<T>::lo_f(rm), Pair<T>::hi_f(rm));
                }
                // The shfl_down tree on channel pairs: level 16 adds pair p and p+8, ...,
                // level 2 pairs 0 and 1, level 1 the two halves of pair 0.
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) {
#pragma unroll
                    for (int q = 0; q < off; ++q) {
                        lo2[q] = __fadd2_rn(lo2[q], lo2[q + off]);
                        hi2[q] = __fadd2_rn(hi2[q], hi2[q + off]);
                    }
                }
                mw = spread_even(am) | (spread_even(am >> 16) << 1);
                sw = spread_even(as) | (spread_even(as >> 16) << 1);
                sums[0] = make_float2(lo2[0].x + lo2[0].y, hi2[0].x + hi2[0].y);
            }
        } else {
            {
                // Thresholds of channel 32w+lane over the group's tokens.
                const int off = w * kWordBytes + (int)sizeof(T) * lane;
                auto at = [&](int t) { return to_float<T>(*reinterpret_cast<const T*>(tile + swz(t, off))); };
                float mn = at(0), mx = mn;
#pragma unroll 8
                for (int t = 1; t < n; ++t) { const float v = at(t); mn = fminf(mn, v); mx = fmaxf(mx, v); }
                wthr[lane] = mn * 0.5f;
                wthr[32 + lane] = mx * 0.5f;
                if (thresholds != nullptr) {
                    float* tg = thresholds + grp * (int64_t)D * 2;
                    tg[2 * (32 * w + lane)] = mn * 0.5f;
                    tg[2 * (32 * w + lane) + 1] = mx * 0.5f;
                }
            }
            __syncwarp();
            if (lane < n) {
                constexpr int kVec = 16 / (int)sizeof(T);
#pragma unroll
                for (int j = 0; j < 32; j += kVec) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(tile + swz(lane, w * kWordBytes + (int)sizeof(T) * j));
                    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
                    for (int k = 0; k < kVec; ++k) {
                        const int c = j + k;
                        const float v = to_float<T>(e[k]);
                        const bool mg = (v > wthr[32 + c]) | (v < wthr[c]);
                        if (v >= 0.0f) sw |= 1u << c;
                        if (mg) mw |= 1u << c;
                        sums[c] = make_float2(mg ? 0.0f : fabsf(v), mg ? fabsf(v) : 0.0f);
                    }
                }
            }
        }
        if (lane < n) {
            const float2 tot = kPaired ? sums[0] : tree_sums(sums);
            const int hc = __popc(mw);
            float lv, hv;
            representatives(tot.x, 32 - hc, tot.y, hc, ref_div, lv, hv);
            k_sign[out] = static_cast<int32_t>(sw);
            k_mag[out] = static_cast<int32_t>(mw);
            low[out] = __half_as_ushort(__float2half_rn(lv));
            delta[out] = __half_as_ushort(__float2half_rn(hv - lv));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (w == 0 && i + kPackStages * step < total) {
            // Refill once every warp has released the stage.
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&empty[s], parity))) {
                if (lane == 0) atomicAdd(&g_pack_wait_timeouts, 1u);
                return;
            }
            if (lane == 0) issue(i + kPackStages * step, s);
        }
    }
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no
// link against libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Tensor map of keys [heads][tokens][D] (head stride in elements) in [32 x 128 B]
// boxes with the 128-byte swizzle; false if it cannot be made.
template <typename T>
bool key_tensor_map(CUtensorMap* map, const void* keys, int64_t heads, int64_t tokens, int D,
                    int64_t head_stride) {
    const EncodeTiledFn enc = encode_tiled();
    if (enc == nullptr) return false;
    const CUtensorMapDataType dt = sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)tokens, (cuuint64_t)heads};
    const cuuint64_t strides[2] = {(cuuint64_t)D * sizeof(T), (cuuint64_t)head_stride * sizeof(T)};
    const cuuint32_t box[3] = {128u / (cuuint32_t)sizeof(T), (cuuint32_t)kGroup, 1u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return enc(map, dt, 3, const_cast<void*>(keys), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int W>
__global__ void __launch_bounds__(32 * W)
append_kernel(T* __restrict__ key_cache, T* __restrict__ value_cache, int64_t kv_capacity, int D,
              const T* __restrict__ new_keys, const T* __restrict__ new_values,
              int32_t* __restrict__ k_sign, int32_t* __restrict__ k_mag,
              uint16_t* __restrict__ low, uint16_t* __restrict__ delta, int64_t capacity,
              const int32_t* __restrict__ seq_len, int64_t position, int64_t heads_per_seq,
              bool vec_ok, bool ref_div) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const PackSmem s = carve<W>(smem_raw, D);
    const int64_t h = blockIdx.x;
    const int64_t P = seq_len ? static_cast<int64_t>(seq_len[h / heads_per_seq]) : position;
    if (P < 0 || P >= capacity || P >= kv_capacity) return;
    const int64_t g0 = (P / kGroup) * kGroup;
    const int n = static_cast<int>(P - g0 + 1);
    T* head_keys = key_cache + h * kv_capacity * D;
    const T* new_row = new_keys ? new_keys + h * D : head_keys + P * D;
    if (new_keys != nullptr) {
        for (int c = threadIdx.x; c < D; c += blockDim.x) {
            head_keys[P * D + c] = new_keys[h * D + c];
            if (value_cache != nullptr && new_values != nullptr)
                value_cache[(h * kv_capacity + P) * D + c] = new_values[h * D + c];
        }
    }
    load_tile<T>(s.tile, tile_ld(D), n, D, vec_ok, [&](int t) -> const T* {
        return (t == n - 1) ? new_row : head_keys + (g0 + t) * D;
    });
    __syncthreads();
    pack_tile<W>(s, n, D, h * capacity + g0, k_sign, k_mag, low, delta, nullptr, ref_div);
}

template <typename T, int W>
int launch_pack_t(const void* keys, int64_t heads, int64_t tokens, int D, int64_t stride,
                  int32_t* sg, int32_t* mg, uint16_t* lo, uint16_t* de, int64_t cap,
                  int64_t off, float* thr, bool vec_ok, bool ref_div, cudaStream_t st) {
    const int64_t groups = (tokens + kGroup - 1) / kGroup;
    CUtensorMap map;
    if (D == 32 * W && (D * (int)sizeof(T)) % 128 == 0 && vec_ok && (thr == nullptr || aligned(thr, 16)) &&
        tokens < (1ll << 31) && heads < (1ll << 31) &&
        key_tensor_map<T>(&map, keys, heads, tokens, D, heads > 1 ? stride : tokens * D)) {
        // Streaming packer: TMA boxes of whole 128-byte row slices.
        using SS = StreamSmem<T, W>;
        auto sk = pack_stream_kernel<T, W>;
        const size_t ssm = SS::bytes();
        if (ssm > 48 * 1024) cudaFuncSetAttribute(sk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm);
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sk, 32 * W, ssm) != cudaSuccess ||
            per_sm < 1)
            per_sm = 1;
        const int64_t total = heads * groups;
        const int64_t grid = imin64(total, (int64_t)per_sm * num_sms());
        launch_pdl(sk, dim3((unsigned)grid), dim3(32 * W), ssm, st,

            map, tokens, groups, total, sg, mg, lo, de, cap, off, thr, ref_div);
        return check_launch("popkv_pack");
    }
    const size_t smem = pack_smem_bytes(D, W);
    auto kern = pack_kernel<T, W>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(kern, dim3((unsigned)(heads * groups)), dim3(32 * W), smem, st,

        static_cast<const T*>(keys), tokens, D, stride, groups, sg, mg, lo, de, cap, off, thr,
        vec_ok, ref_div);
    return check_launch("popkv_pack");
}

template <typename T, int W>
int launch_append_t(void* kc, void* vc, int64_t heads, int64_t kv_cap, int D, const void* nk,
                    const void* nv, int32_t* sg, int32_t* mg, uint16_t* lo, uint16_t* de,
                    int64_t cap, const int32_t* seq_len, int64_t pos, int64_t hps, bool vec_ok,
                    bool ref_div, cudaStream_t st) {
    const size_t smem = pack_smem_bytes(D, W);
    auto kern = append_kernel<T, W>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(kern, dim3((unsigned)heads), dim3(32 * W), smem, st,

        static_cast<T*>(kc), static_cast<T*>(vc), kv_cap, D, static_cast<const T*>(nk),
        static_cast<const T*>(nv), sg, mg, lo, de, cap, seq_len, pos, hps, vec_ok, ref_div);
    return check_launch("popkv_append");
}

// Dispatch over (dtype, words) at run time to the template instances.
template <template <typename, int> class F, typename... Args>
int dispatch_dtype_words(int dtype, int W, Args... args) {
#define POPKV_W_CASES(T)                                  \
    switch (W) {                                          \
        case 1: return F<T, 1>::run(args...);             \
        case 2: return F<T, 2>::run(args...);             \
        case 3: return F<T, 3>::run(args...);             \
        case 4: return F<T, 4>::run(args...);             \
        case 5: return F<T, 5>::run(args...);             \
        case 6: return F<T, 6>::run(args...);             \
        case 7: return F<T, 7>::run(args...);             \
        case 8: return F<T, 8>::run(args...);             \
        default: return fail(POPKV_ERR_UNSUPPORTED, "head_dim above 256 is not supported"); \
    }
    switch (dtype) {
        case POPKV_F32: POPKV_W_CASES(float)
        case POPKV_F16: POPKV_W_CASES(__half)
        case POPKV_BF16: POPKV_W_CASES(__nv_bfloat16)
        default: return fail(POPKV_ERR_UNSUPPORTED, "dtype %d is not fp32/fp16/bf16", dtype);
    }
#undef POPKV_W_CASES
}

template <typename T, int W>
struct PackRun {
    template <typename... A>
    static int run(A... a) { return launch_pack_t<T, W>(a...); }
};
template <typename T, int W>
struct AppendRun {
    template <typename... A>
    static int run(A... a) { return launch_append_t<T, W>(a...); }
};

}  // namespace
}  // namespace popkv

using namespace popkv;

extern "C" int popkv_pack(const void* keys, int dtype, int64_t heads, int64_t tokens,
                          int64_t head_dim, int64_t key_head_stride, int32_t* k_sign,
                          int32_t* k_mag, uint16_t* low, uint16_t* delta, int64_t capacity,
                          int64_t token_offset, float* thresholds, int flags,
                          popkv_stream_t stream) {
    const size_t es = dtype_size(dtype);
    if (es == 0) return fail(POPKV_ERR_UNSUPPORTED, "keys dtype %d is not fp32/fp16/bf16", dtype);
    if (heads < 0 || tokens < 0 || head_dim <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "keys must be [heads, tokens, head_dim] with head_dim > 0");
    if (head_dim > 256) return fail(POPKV_ERR_UNSUPPORTED, "head_dim %lld > 256", (long long)head_dim);
    if (token_offset < 0 || token_offset + tokens > capacity)
        return fail(POPKV_ERR_CAPACITY, "Pop-KV cache capacity exceeded: offset %lld + tokens %lld > capacity %lld",
                    (long long)token_offset, (long long)tokens, (long long)capacity);
    if (heads > 1 && key_head_stride < tokens * head_dim)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "key_head_stride smaller than tokens*head_dim");
    if (heads == 0 || tokens == 0) return POPKV_OK;
    if (!keys || !k_sign || !k_mag || !low || !delta)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    if (heads * ((tokens + 31) / 32) > 0x7fffffffLL)
        return fail(POPKV_ERR_UNSUPPORTED, "too many groups for one launch");
    const int W = (int)((head_dim + 31) / 32);
    const bool vec_ok = aligned(keys, 16) && (head_dim * es) % 16 == 0 &&
                        (key_head_stride * es) % 16 == 0;
    return dispatch_dtype_words<PackRun>(dtype, W, keys, heads, tokens, (int)head_dim,
                                         key_head_stride, k_sign, k_mag, low, delta, capacity,
                                         token_offset, thresholds, vec_ok,
                                         (flags & POPKV_FLAG_REFERENCE_DIVISION) != 0,
                                         as_stream(stream));
}

extern "C" int popkv_append(void* key_cache, void* value_cache, int dtype, int64_t heads,
                            int64_t kv_capacity, int64_t head_dim, const void* new_keys,
                            const void* new_values, int32_t* k_sign, int32_t* k_mag,
                            uint16_t* low, uint16_t* delta, int64_t capacity,
                            const int32_t* seq_len, int64_t position, int64_t kv_heads_per_seq,
                            int flags, popkv_stream_t stream) {
    const size_t es = dtype_size(dtype);
    if (es == 0) return fail(POPKV_ERR_UNSUPPORTED, "cache dtype %d is not fp32/fp16/bf16", dtype);
    if (heads < 0 || head_dim <= 0 || kv_capacity <= 0 || capacity <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid append shape");
    if (head_dim > 256) return fail(POPKV_ERR_UNSUPPORTED, "head_dim %lld > 256", (long long)head_dim);
    if (!key_cache || !k_sign || !k_mag || !low || !delta)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    if (seq_len == nullptr && (position < 0 || position >= capacity || position >= kv_capacity))
        return fail(POPKV_ERR_CAPACITY, "Pop-KV cache reserve exhausted: position %lld, capacity %lld, kv capacity %lld",
                    (long long)position, (long long)capacity, (long long)kv_capacity);
    if (seq_len != nullptr && kv_heads_per_seq <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "kv_heads_per_seq must be positive");
    if (heads == 0) return POPKV_OK;
    const int W = (int)((head_dim + 31) / 32);
    const bool vec_ok = aligned(key_cache, 16) && (head_dim * es) % 16 == 0 &&
                        (new_keys == nullptr || aligned(new_keys, 16));
    return dispatch_dtype_words<AppendRun>(
        dtype, W, key_cache, value_cache, heads, kv_capacity, (int)head_dim, new_keys, new_values,
        k_sign, k_mag, low, delta, capacity, seq_len, position,
        kv_heads_per_seq > 0 ? kv_heads_per_seq : heads,
        vec_ok, (flags & POPKV_FLAG_REFERENCE_DIVISION) != 0, as_stream(stream));
}
