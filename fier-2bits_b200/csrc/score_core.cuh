// Device pieces of the popcount scorer shared by the scorer kernel (score.cu) and
// the fused score + select kernel (select.cu): packed-row loads, the query packer
// and the per-token score (popkv_ext.cu:93-178).
#pragma once

#include "common.cuh"

namespace popkv {
namespace {

// Exact float of a small integer (|n| < 2^22) with two full-rate ALU operations:
// 1.5 * 2^23 + n has n in its low mantissa bits, and subtracting 1.5 * 2^23 is exact.
__device__ __forceinline__ float small_int_to_float(int n) {
    return __fsub_rn(__int_as_float(0x4B400000 + n), 12582912.0f);
}

template <int W, bool VEC>
struct PackedRow {
    uint32_t s[W], m[W];
    uint16_t l[W], d[W];

    __device__ __forceinline__ void load(const int32_t* __restrict__ sg,
                                         const int32_t* __restrict__ mg,
                                         const uint16_t* __restrict__ lo,
                                         const uint16_t* __restrict__ de, int64_t base) {
        if constexpr (VEC && W % 4 == 0) {
#pragma unroll
            for (int j = 0; j < W; j += 4) {
                const uint4 a = __ldg(reinterpret_cast<const uint4*>(sg + base + j));
                const uint4 b = __ldg(reinterpret_cast<const uint4*>(mg + base + j));
                const uint2 c = __ldg(reinterpret_cast<const uint2*>(lo + base + j));
                const uint2 e = __ldg(reinterpret_cast<const uint2*>(de + base + j));
                s[j] = a.x; s[j + 1] = a.y; s[j + 2] = a.z; s[j + 3] = a.w;
                m[j] = b.x; m[j + 1] = b.y; m[j + 2] = b.z; m[j + 3] = b.w;
                l[j] = c.x & 0xffffu; l[j + 1] = c.x >> 16; l[j + 2] = c.y & 0xffffu; l[j + 3] = c.y >> 16;
                d[j] = e.x & 0xffffu; d[j + 1] = e.x >> 16; d[j + 2] = e.y & 0xffffu; d[j + 3] = e.y >> 16;
            }
        } else if constexpr (VEC && W % 2 == 0) {
#pragma unroll
            for (int j = 0; j < W; j += 2) {
                const uint2 a = __ldg(reinterpret_cast<const uint2*>(sg + base + j));
                const uint2 b = __ldg(reinterpret_cast<const uint2*>(mg + base + j));
                const uint32_t c = __ldg(reinterpret_cast<const unsigned int*>(lo + base + j));
                const uint32_t e = __ldg(reinterpret_cast<const unsigned int*>(de + base + j));
                s[j] = a.x; s[j + 1] = a.y; m[j] = b.x; m[j + 1] = b.y;
                l[j] = c & 0xffffu; l[j + 1] = c >> 16; d[j] = e & 0xffffu; d[j + 1] = e >> 16;
            }
        } else {
#pragma unroll
            for (int j = 0; j < W; ++j) {
                s[j] = static_cast<uint32_t>(__ldg(sg + base + j));
                m[j] = static_cast<uint32_t>(__ldg(mg + base + j));
                l[j] = __ldg(lo + base + j);
                d[j] = __ldg(de + base + j);
            }
        }
    }
};

// One token's score against one packed query head: the word-ordered sum of
//   fmaf(ql*kl, Cs, fmaf(dq*kl, Cq, fmaf(ql*dk, Ck, dq*dk*Cqk)))
// (popkv_ext.cu:155-176).  pkm holds popc of the token's magnitude words (a byte per
// word, W <= 4).  FULL: every word holds 32 channels (head_dim % 32 == 0), so no
// lane mask is applied.
template <int W, bool FULL>
__device__ __forceinline__ float token_score(const uint32_t (&ks)[W], const uint32_t (&km_raw)[W],
                                             const float (&klf)[W], const float (&kdf)[W],
                                             uint32_t pkm, const uint32_t (&qs)[W],
                                             const uint32_t (&qm)[W], const float (&ql)[W],
                                             const float (&dq)[W], const int (&pq)[W],
                                             uint32_t last_valid, int last_bits) {
    float score = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
        const bool edge = !FULL && w == W - 1;
        const uint32_t km = edge ? (km_raw[w] & last_valid) : km_raw[w];
        const uint32_t match = edge ? (~(qs[w] ^ ks[w]) & last_valid) : ~(qs[w] ^ ks[w]);
        const uint32_t both = qm[w] & km;
        const int cs = 2 * __popc(match) - (edge ? last_bits : 32);
        const int pk = W <= 4 ? static_cast<int>((pkm >> (8 * w)) & 0xffu) : __popc(km);
        const int ck = 2 * __popc(match & km) - pk;
        const int cq = 2 * __popc(match & qm[w]) - pq[w];
        const int cqk = 2 * __popc(match & both) - __popc(both);
        const float kl = klf[w];
        const float dk = kdf[w];
        const float inner = __fmul_rn(__fmul_rn(dq[w], dk), small_int_to_float(cqk));
        const float gs = fmaf(__fmul_rn(ql[w], kl), small_int_to_float(cs),
                              fmaf(__fmul_rn(dq[w], kl), small_int_to_float(cq),
                                   fmaf(__fmul_rn(ql[w], dk), small_int_to_float(ck), inner)));
        score = __fadd_rn(score, gs);
    }
    return score;
}

template <int W>
__device__ __forceinline__ void half_words(const uint16_t (&bits)[W], float (&out)[W]) {
#pragma unroll
    for (int w = 0; w < W; ++w) out[w] = __half2float(__ushort_as_half(bits[w]));
}

template <int W>
__device__ __forceinline__ uint32_t mag_popcounts(const uint32_t (&km)[W], uint32_t last_valid) {
    uint32_t p = 0u;
    if constexpr (W <= 4) {
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const uint32_t valid = (w == W - 1) ? last_valid : 0xffffffffu;
            p |= static_cast<uint32_t>(__popc(km[w] & valid)) << (8 * w);
        }
    }
    return p;
}

// Packs the nh query heads listed in s_heads (one warp per head): ballots give the
// sign/magnitude words; lane j then sums word j's magnitudes in channel order (the
// reference's sequential query sums, popkv_ext.cu:129-138) from a conflict-free
// shared scratch.  Caller synchronises before and after.
template <typename TQ, int W, int NWARPS>
__device__ __forceinline__ void pack_query_heads(const TQ* __restrict__ queries, int64_t b,
                                                 int q_heads, int D, const int* s_heads, int nh,
                                                 float* s_abs, uint32_t* s_qs, uint32_t* s_qm,
                                                 float* s_ql, float* s_qd, bool ref_div) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    float* my_abs = s_abs + warp * (W * 33);  // word j at 33 j: conflict-free column reads
    for (int slot = warp; slot < nh; slot += NWARPS) {
        const TQ* q = queries + (b * q_heads + s_heads[slot]) * D;
        float v[W];
        float mn = INFINITY, mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < W; ++j) {
            const int c = 32 * j + lane;
            v[j] = c < D ? to_float<TQ>(q[c]) : 0.0f;
            if (c < D) { mn = fminf(mn, v[j]); mx = fmaxf(mx, v[j]); }
            my_abs[33 * j + lane] = fabsf(v[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        const float neg = mn * 0.5f, pos = mx * 0.5f;
        uint32_t my_sw = 0u, my_mw = 0u;
#pragma unroll
        for (int j = 0; j < W; ++j) {
            const bool valid = 32 * j + lane < D;
            const bool sg = valid && v[j] >= 0.0f;
            const bool mg = valid && (sg ? v[j] > pos : v[j] < neg);
            const uint32_t sw = __ballot_sync(0xffffffffu, sg);
            const uint32_t mw = __ballot_sync(0xffffffffu, mg);
            if (lane == j) { my_sw = sw; my_mw = mw; }
        }
        __syncwarp();
        if (lane < W) {
            // Channel-order sums without branches: each magnitude goes to both sums, as
            // itself or as +0 (which leaves a sum of magnitudes unchanged); channels past
            // D hold 0.
            float ls = 0.0f, hs = 0.0f;
            const int n = min(32, D - 32 * lane);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float x = my_abs[33 * lane + i];
                const bool high = (my_mw >> i) & 1u;
                hs += high ? x : 0.0f;
                ls += high ? 0.0f : x;
            }
            const int hc = __popc(my_mw), lc = n - hc;
            float low, high;
            representatives(ls, lc, hs, hc, ref_div, low, high);
            s_qs[slot * W + lane] = my_sw;
            s_qm[slot * W + lane] = my_mw;
            s_ql[slot * W + lane] = low;
            s_qd[slot * W + lane] = high - low;
        }
        __syncwarp();
    }
}

}  // namespace
}  // namespace popkv
