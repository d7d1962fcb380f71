// Decoder plumbing around the retrieval path: the elementwise steps of a Llama
// decode step fused into one kernel each, so that a CUDA-graphed token step is a
// few launches per layer instead of dozens of small tensor ops.
//
//  * rmsnorm:   out = weight * bf16(x * rsqrt(mean(x^2) + eps))   (LlamaRMSNorm)
//  * rope_qkv:  split a fused [q | k | v] projection row, rotate q and k at the
//               sequence's current position (rotate-half form, popkv.py:389-398),
//               write q, k, v to the retrieval stack's input buffers
//  * silu_mul:  out = bf16(silu(gate)) * up                       (LlamaMLP)
//
// Rounding follows the transformers modules step by step in the storage dtype
// (every product and sum of two 16-bit values rounded once), so outputs match
// them up to the order of the fp32 sum of squares in rmsnorm.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace popkv {
namespace {

constexpr int kNormThreads = 256;

template <typename T>
__device__ __forceinline__ T round_to(float v) { return from_float<T>(v); }

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const T* __restrict__ x,
                                                              const T* __restrict__ weight,
                                                              T* __restrict__ out, int n, float eps) {
    pdl_trigger();
    pdl_wait();
    const T* row = x + static_cast<int64_t>(blockIdx.x) * n;
    T* orow = out + static_cast<int64_t>(blockIdx.x) * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += kNormThreads) {
        const float v = to_float<T>(row[i]);
        ss = fmaf(v, v, ss);
    }
    __shared__ float s_part[kNormThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) total += s_part[w];
    const float inv = rsqrtf(total / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += kNormThreads) {
        const float h = to_float<T>(round_to<T>(to_float<T>(row[i]) * inv));
        orow[i] = round_to<T>(to_float<T>(weight[i]) * h);
    }
}

// One CTA per sequence row b: qkv [B, (QH + 2 KVH) * D]; cos/sin [positions, D];
// position of row b = pos[b] (device) -> q [B, QH, D], k [B, KVH, D], v [B, KVH, D].
template <typename T>
__global__ void __launch_bounds__(kNormThreads) rope_qkv_kernel(const T* __restrict__ qkv,
                                                               const T* __restrict__ cos_t,
                                                               const T* __restrict__ sin_t,
                                                               const int32_t* __restrict__ pos,
                                                               int64_t positions, int qh, int kvh,
                                                               int D, T* __restrict__ q,
                                                               T* __restrict__ k, T* __restrict__ v) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    int64_t p = pos[b];
    p = p < 0 ? 0 : (p >= positions ? positions - 1 : p);
    const T* c = cos_t + p * D;
    const T* s = sin_t + p * D;
    const int width = (qh + 2 * kvh) * D;
    const T* row = qkv + static_cast<int64_t>(b) * width;
    const int half = D / 2;
    for (int i = threadIdx.x; i < width; i += kNormThreads) {
        const int head = i / D;
        const int d = i - head * D;
        if (head >= qh + kvh) {  // value: copied as is
            v[(static_cast<int64_t>(b) * kvh + (head - qh - kvh)) * D + d] = row[i];
            continue;
        }
        // x * cos + rotate_half(x) * sin, each product and the sum rounded to T.
        const float x = to_float<T>(row[i]);
        const float partner = to_float<T>(row[head * D + (d < half ? d + half : d - half)]);
        const float rot = d < half ? -partner : partner;
        const float a = to_float<T>(round_to<T>(x * to_float<T>(c[d])));
        const float r = to_float<T>(round_to<T>(rot * to_float<T>(s[d])));
        const T y = round_to<T>(a + r);
        if (head < qh) q[(static_cast<int64_t>(b) * qh + head) * D + d] = y;
        else k[(static_cast<int64_t>(b) * kvh + (head - qh)) * D + d] = y;
    }
}

// gate_up [rows, 2F] = [gate | up] -> out [rows, F].
template <typename T>
__global__ void __launch_bounds__(kNormThreads) silu_mul_kernel(const T* __restrict__ gate_up,
                                                               T* __restrict__ out, int F,
                                                               int64_t total) {
    pdl_trigger();
    pdl_wait();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kNormThreads + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * kNormThreads) {
        const int64_t r = i / F;
        const int64_t j = i - r * F;
        const float g = to_float<T>(gate_up[r * 2 * F + j]);
        const float u = to_float<T>(gate_up[r * 2 * F + F + j]);
        const float act = to_float<T>(round_to<T>(g / (1.0f + expf(-g))));
        out[i] = round_to<T>(act * u);
    }
}

// ------------------------------------------------------------------ GEMV
// out[j] = round(round(sum_i x[i] * W[j, i]) + residual[j]) for one activation row
// (batch-1 decode; the product is rounded before the residual add, as
// `h + o_proj(x)` is): W is [n_out, k] row-major (an nn.Linear weight).  HBM-bound
// on W.  One 256-thread CTA per kGemvRows rows; warp w takes the w-th eighth of k
// (split-K), every lane keeps kGemvRows 16-byte weight loads per step in flight,
// fp32 partial sums meet in shared memory.
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvRows = 4;

template <typename T>
__device__ __forceinline__ void fma8(float& a, const uint4& wv, const uint4& xv) {
    const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w}, xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const T* we = reinterpret_cast<const T*>(&wa[j]);
        const T* xe = reinterpret_cast<const T*>(&xa[j]);
        a = fmaf(to_float<T>(we[0]), to_float<T>(xe[0]), a);
        a = fmaf(to_float<T>(we[1]), to_float<T>(xe[1]), a);
    }
}

template <typename T>
__global__ void __launch_bounds__(kGemvThreads)
gemv_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ residual,
            T* __restrict__ out, int64_t n_out, int k) {
    pdl_trigger();
    pdl_wait();
    __shared__ float s_part[kGemvWarps][kGemvRows];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kGemvRows;
    const int chunks = k / 8;
    const int per_warp = (chunks + kGemvWarps - 1) / kGemvWarps;
    const int c0 = warp * per_warp;
    const int c1 = min(chunks, c0 + per_warp);
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const uint4* wr[kGemvRows];
    float acc[kGemvRows];
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) {
        acc[r] = 0.0f;
        const int64_t row = r0 + r < n_out ? r0 + r : n_out - 1;
        wr[r] = reinterpret_cast<const uint4*>(w + row * k);
    }
    int c = c0 + lane;
    for (; c + 32 < c1; c += 64) {
        uint4 wa[kGemvRows], wb[kGemvRows];
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
            wa[r] = __ldcs(wr[r] + c);
            wb[r] = __ldcs(wr[r] + c + 32);
        }
        const uint4 xa = __ldg(xv + c), xb = __ldg(xv + c + 32);
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
            fma8<T>(acc[r], wa[r], xa);
            fma8<T>(acc[r], wb[r], xb);
        }
    }
    if (c < c1) {
        const uint4 xa = __ldg(xv + c);
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) fma8<T>(acc[r], __ldcs(wr[r] + c), xa);
    }
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        if (lane == 0) s_part[warp][r] = acc[r];
    }
    __syncthreads();
    if (threadIdx.x < kGemvRows && r0 + threadIdx.x < n_out) {
        float v = 0.0f;
#pragma unroll
        for (int q = 0; q < kGemvWarps; ++q) v += s_part[q][threadIdx.x];
        T o = from_float<T>(v);
        if (residual != nullptr) o = from_float<T>(to_float<T>(o) + to_float<T>(residual[r0 + threadIdx.x]));
        out[r0 + threadIdx.x] = o;
    }
}

}  // namespace
}  // namespace popkv

using namespace popkv;

extern "C" int popkv_rmsnorm(const void* x, const void* weight, void* out, int dtype, int64_t rows,
                             int64_t n, float eps, popkv_stream_t stream) {
    if (rows < 0 || n <= 0 || n > (1 << 24)) return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid rmsnorm shape");
    if (rows == 0) return POPKV_OK;
    if (!x || !weight || !out) return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    const cudaStream_t st = as_stream(stream);
    const dim3 grid((unsigned)rows), block(kNormThreads);
    switch (dtype) {
        case POPKV_BF16:
            launch_pdl(rmsnorm_kernel<__nv_bfloat16>, grid, block, 0, st, static_cast<const __nv_bfloat16*>(x),
                       static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out), (int)n, eps);
            break;
        case POPKV_F16:
            launch_pdl(rmsnorm_kernel<__half>, grid, block, 0, st, static_cast<const __half*>(x),
                       static_cast<const __half*>(weight), static_cast<__half*>(out), (int)n, eps);
            break;
        default:
            return fail(POPKV_ERR_UNSUPPORTED, "rmsnorm dtype %d is not fp16/bf16", dtype);
    }
    return check_launch("popkv_rmsnorm");
}

extern "C" int popkv_rope_qkv(const void* qkv, const void* cos_table, const void* sin_table,
                              const int32_t* positions_of_rows, int64_t positions, int dtype,
                              int64_t rows, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                              void* q, void* k, void* v, popkv_stream_t stream) {
    if (rows < 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 || positions <= 0)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid rope shape");
    if (rows == 0) return POPKV_OK;
    if (!qkv || !cos_table || !sin_table || !positions_of_rows || !q || !k || !v)
        return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    const cudaStream_t st = as_stream(stream);
    const dim3 grid((unsigned)rows), block(kNormThreads);
    switch (dtype) {
        case POPKV_BF16: {
            using T = __nv_bfloat16;
            launch_pdl(rope_qkv_kernel<T>, grid, block, 0, st, static_cast<const T*>(qkv),
                       static_cast<const T*>(cos_table), static_cast<const T*>(sin_table), positions_of_rows,
                       positions, (int)q_heads, (int)kv_heads, (int)head_dim, static_cast<T*>(q),
                       static_cast<T*>(k), static_cast<T*>(v));
            break;
        }
        case POPKV_F16: {
            using T = __half;
            launch_pdl(rope_qkv_kernel<T>, grid, block, 0, st, static_cast<const T*>(qkv),
                       static_cast<const T*>(cos_table), static_cast<const T*>(sin_table), positions_of_rows,
                       positions, (int)q_heads, (int)kv_heads, (int)head_dim, static_cast<T*>(q),
                       static_cast<T*>(k), static_cast<T*>(v));
            break;
        }
        default:
            return fail(POPKV_ERR_UNSUPPORTED, "rope dtype %d is not fp16/bf16", dtype);
    }
    return check_launch("popkv_rope_qkv");
}

extern "C" int popkv_silu_mul(const void* gate_up, void* out, int dtype, int64_t rows, int64_t ffn,
                              popkv_stream_t stream) {
    if (rows < 0 || ffn <= 0) return fail(POPKV_ERR_INVALID_ARGUMENT, "invalid silu_mul shape");
    if (rows == 0) return POPKV_OK;
    if (!gate_up || !out) return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    const int64_t total = rows * ffn;
    const int64_t blocks64 = (total + kNormThreads - 1) / kNormThreads;
    const dim3 grid((unsigned)(blocks64 < 4 * num_sms() ? blocks64 : 4 * num_sms())), block(kNormThreads);
    const cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case POPKV_BF16:
            launch_pdl(silu_mul_kernel<__nv_bfloat16>, grid, block, 0, st,
                       static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), (int)ffn, total);
            break;
        case POPKV_F16:
            launch_pdl(silu_mul_kernel<__half>, grid, block, 0, st, static_cast<const __half*>(gate_up),
                       static_cast<__half*>(out), (int)ffn, total);
            break;
        default:
            return fail(POPKV_ERR_UNSUPPORTED, "silu_mul dtype %d is not fp16/bf16", dtype);
    }
    return check_launch("popkv_silu_mul");
}

extern "C" int popkv_gemv(const void* x, const void* weight, const void* residual, void* out,
                          int dtype, int64_t n_out, int64_t k, popkv_stream_t stream) {
    if (n_out <= 0 || k <= 0) return fail(POPKV_ERR_INVALID_ARGUMENT, "gemv needs n_out > 0 and k > 0");
    if (k % 8 != 0 || k > (1 << 24)) return fail(POPKV_ERR_UNSUPPORTED, "gemv needs k a multiple of 8");
    if (!x || !weight || !out) return fail(POPKV_ERR_INVALID_ARGUMENT, "null pointer argument");
    if (!aligned(x, 16) || !aligned(weight, 16)) return fail(POPKV_ERR_ALIGNMENT, "gemv x and weight need 16-byte alignment");
    const cudaStream_t st = as_stream(stream);
    const int64_t grid = (n_out + kGemvRows - 1) / kGemvRows;
    if (grid > 0x7fffffffLL) return fail(POPKV_ERR_UNSUPPORTED, "gemv: too many rows");
    auto go = [&](auto kern, auto* tp) {
        using T = std::remove_pointer_t<decltype(tp)>;
        launch_pdl(kern, dim3((unsigned)grid), dim3(kGemvThreads), 0, st, static_cast<const T*>(x),
                   static_cast<const T*>(weight), static_cast<const T*>(residual), static_cast<T*>(out),
                   n_out, (int)k);
    };
    switch (dtype) {
        case POPKV_BF16: go(gemv_kernel<__nv_bfloat16>, (__nv_bfloat16*)nullptr); break;
        case POPKV_F16: go(gemv_kernel<__half>, (__half*)nullptr); break;
        default: return fail(POPKV_ERR_UNSUPPORTED, "gemv dtype %d is not fp16/bf16", dtype);
    }
    return check_launch("popkv_gemv");
}
