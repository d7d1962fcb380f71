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
