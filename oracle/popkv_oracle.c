/*
 * popkv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the Pop-KV decode-time retrieval path, used as the
 * checker for the CUDA kernels.  Nothing in the shipped library links or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg load it (through oracle/popkv_oracle.py).
 *
 * Every function restates the reference algorithm (kw78999/FIER-2bits) step
 * by step, with the arithmetic order the reference's CUDA kernel uses, so
 * that packing, scores and selections can be compared bit for bit:
 *
 *   oracle_pack_keys     csrc/popkv_ext.cu:29-91   (group-of-32 key packer)
 *   oracle_pack_queries  csrc/popkv_ext.cu:117-149 (per-row query packer)
 *   oracle_score         csrc/popkv_ext.cu:150-177 (popcount scorer)
 *   oracle_select        popkv.py:594-600, 141-145 (top-(budget-1) + newest);
 *                        ties resolved towards the lowest index
 *   oracle_attention     popkv.py:341-368 (gather + exact SDPA, fp64 accum.)
 *
 * Division: the kernels here use IEEE round-to-nearest division; the
 * reference extension is built with --use_fast_math, so its fp16
 * representatives may differ from these by one fp16 ulp in rare cases.
 * Build with -ffp-contract=off so that no multiply-add is fused unless the
 * reference writes fmaf explicitly.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* IEEE binary16 round-to-nearest-even of a float, as __float2half_rn does. */
static uint16_t f32_to_f16_rn(float x) {
    _Float16 h = (_Float16)x;
    uint16_t bits;
    memcpy(&bits, &h, sizeof bits);
    return bits;
}

static uint32_t popc32(uint32_t x) { return (uint32_t)__builtin_popcount(x); }

/* Sum of 32 lane values in the order of a __shfl_down_sync tree with
 * offsets 16, 8, 4, 2, 1 read back at lane 0 (csrc/popkv_ext.cu:69-75). */
static float shfl_down_tree_sum(float a[32]) {
    for (int off = 16; off > 0; off >>= 1)
        for (int i = 0; i < off; ++i) a[i] = a[i] + a[i + off];
    return a[0];
}

/* Representative rule shared by keys and queries (popkv_ext.cu:77-83,139-145). */
static void representatives(float low_sum, int low_count, float high_sum, int high_count,
                            float* low_out, float* high_out) {
    float low, high;
    if (low_count == 0) {
        low = high_count ? high_sum / (float)high_count : 0.0f;
        high = low;
    } else {
        low = low_sum / (float)low_count;
        high = high_count ? high_sum / (float)high_count : low;
    }
    *low_out = low;
    *high_out = high;
}

/*
 * keys: float32 values of the key rows; row t of head h at
 *       keys + h*head_stride + t*head_dim.
 * Output rows (h, token_offset + t) of the [heads, capacity, words] arrays.
 * thresholds (nullable): [heads, groups, head_dim, 2] = (min*0.5, max*0.5).
 * Groups are formed relative to the first input token, as in the reference.
 */
void oracle_pack_keys(const float* keys, int64_t heads, int64_t tokens, int64_t head_dim,
                      int64_t head_stride, int64_t capacity, int64_t token_offset,
                      int32_t* k_sign, int32_t* k_mag, uint16_t* low_mean, uint16_t* delta_mean,
                      float* thresholds) {
    const int64_t words = (head_dim + 31) / 32;
    const int64_t groups = (tokens + 31) / 32;
    float* neg = (float*)malloc(sizeof(float) * (size_t)head_dim);
    float* pos = (float*)malloc(sizeof(float) * (size_t)head_dim);
    for (int64_t h = 0; h < heads; ++h) {
        const float* hk = keys + h * head_stride;
        for (int64_t g = 0; g < groups; ++g) {
            int64_t t0 = g * 32, t1 = t0 + 32 < tokens ? t0 + 32 : tokens;
            for (int64_t d = 0; d < head_dim; ++d) {
                float mn = hk[t0 * head_dim + d], mx = mn;
                for (int64_t t = t0 + 1; t < t1; ++t) {
                    float v = hk[t * head_dim + d];
                    mn = fminf(mn, v);
                    mx = fmaxf(mx, v);
                }
                neg[d] = mn * 0.5f;
                pos[d] = mx * 0.5f;
                if (thresholds) {
                    float* th = thresholds + ((h * groups + g) * head_dim + d) * 2;
                    th[0] = neg[d];
                    th[1] = pos[d];
                }
            }
            for (int64_t t = t0; t < t1; ++t) {
                for (int64_t w = 0; w < words; ++w) {
                    uint32_t sw = 0, mw = 0;
                    float lo[32], hi[32];
                    int lc = 0, hc = 0;
                    for (int i = 0; i < 32; ++i) {
                        int64_t d = w * 32 + i;
                        int valid = d < head_dim;
                        float v = valid ? hk[t * head_dim + d] : 0.0f;
                        int s = valid && v >= 0.0f;
                        int m = valid && (s ? (v > pos[d]) : (v < neg[d]));
                        if (s) sw |= 1u << i;
                        if (m) mw |= 1u << i;
                        lo[i] = (!m && valid) ? fabsf(v) : 0.0f;
                        hi[i] = (m && valid) ? fabsf(v) : 0.0f;
                        lc += (!m && valid);
                        hc += (m && valid);
                    }
                    float ls = shfl_down_tree_sum(lo), hs = shfl_down_tree_sum(hi);
                    float low, high;
                    representatives(ls, lc, hs, hc, &low, &high);
                    int64_t out = (h * capacity + token_offset + t) * words + w;
                    k_sign[out] = (int32_t)sw;
                    k_mag[out] = (int32_t)mw;
                    low_mean[out] = f32_to_f16_rn(low);
                    delta_mean[out] = f32_to_f16_rn(high - low);
                }
            }
        }
    }
    free(neg);
    free(pos);
}

/* queries: [rows, head_dim] float32.  Outputs [rows, words]. */
void oracle_pack_queries(const float* queries, int64_t rows, int64_t head_dim,
                         uint32_t* q_sign, uint32_t* q_mag, float* q_low, float* q_delta) {
    const int64_t words = (head_dim + 31) / 32;
    for (int64_t r = 0; r < rows; ++r) {
        const float* q = queries + r * head_dim;
        float mn = q[0], mx = mn;
        for (int64_t d = 1; d < head_dim; ++d) {
            mn = fminf(mn, q[d]);
            mx = fmaxf(mx, q[d]);
        }
        float neg = mn * 0.5f, pos = mx * 0.5f;
        for (int64_t w = 0; w < words; ++w) {
            uint32_t sw = 0, mw = 0;
            float ls = 0.0f, hs = 0.0f;
            int lc = 0, hc = 0;
            int64_t d0 = w * 32, d1 = d0 + 32 < head_dim ? d0 + 32 : head_dim;
            for (int64_t d = d0; d < d1; ++d) {
                float v = q[d];
                int s = v >= 0.0f;
                int m = s ? (v > pos) : (v < neg);
                uint32_t bit = 1u << (uint32_t)(d - d0);
                if (s) sw |= bit;
                if (m) { mw |= bit; hs += fabsf(v); ++hc; }
                else { ls += fabsf(v); ++lc; }
            }
            float low, high;
            representatives(ls, lc, hs, hc, &low, &high);
            q_sign[r * words + w] = sw;
            q_mag[r * words + w] = mw;
            q_low[r * words + w] = low;
            q_delta[r * words + w] = high - low;
        }
    }
}

static float f16_bits_to_f32(uint16_t bits) {
    _Float16 h;
    memcpy(&h, &bits, sizeof h);
    return (float)h;
}

/*
 * queries [batch, q_heads, head_dim] float32; packed cache [cache_heads, capacity, words]
 * where the KV head of (b, qh) is (cache_per_batch ? b*kv_heads : 0) + head_to_kv[qh].
 * scores [batch, q_heads, row_stride]; tokens [0, lengths[b]) are written.
 */
void oracle_score(const float* queries, int64_t batch, int64_t q_heads, int64_t head_dim,
                  const int32_t* k_sign, const int32_t* k_mag, const uint16_t* low_mean,
                  const uint16_t* delta_mean, int64_t kv_heads, int64_t capacity,
                  int cache_per_batch, const int64_t* head_to_kv, const int64_t* lengths,
                  float scale, float* scores, int64_t row_stride) {
    const int64_t words = (head_dim + 31) / 32;
    uint32_t* qs = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(batch * q_heads * words));
    uint32_t* qm = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(batch * q_heads * words));
    float* ql = (float*)malloc(sizeof(float) * (size_t)(batch * q_heads * words));
    float* qd = (float*)malloc(sizeof(float) * (size_t)(batch * q_heads * words));
    oracle_pack_queries(queries, batch * q_heads, head_dim, qs, qm, ql, qd);
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t h = 0; h < q_heads; ++h) {
            int64_t row = b * q_heads + h;
            int64_t kvh = (cache_per_batch ? b * kv_heads : 0) + head_to_kv[h];
            for (int64_t t = 0; t < lengths[b]; ++t) {
                int64_t base = (kvh * capacity + t) * words;
                float score = 0.0f;
                for (int64_t w = 0; w < words; ++w) {
                    uint32_t valid = 0xffffffffu;
                    if (w == words - 1 && (head_dim & 31)) valid = (1u << (uint32_t)(head_dim & 31)) - 1u;
                    uint32_t qmw = qm[row * words + w] & valid;
                    uint32_t kmw = (uint32_t)k_mag[base + w] & valid;
                    uint32_t match = ~(qs[row * words + w] ^ (uint32_t)k_sign[base + w]) & valid;
                    uint32_t both = qmw & kmw;
                    int cs = 2 * (int)popc32(match) - (int)popc32(valid);
                    int cq = 2 * (int)popc32(match & qmw) - (int)popc32(qmw);
                    int ck = 2 * (int)popc32(match & kmw) - (int)popc32(kmw);
                    int cqk = 2 * (int)popc32(match & both) - (int)popc32(both);
                    float l = ql[row * words + w], dq = qd[row * words + w];
                    float kl = f16_bits_to_f32(low_mean[base + w]);
                    float dk = f16_bits_to_f32(delta_mean[base + w]);
                    float inner = dq * dk;
                    inner = inner * (float)cqk;
                    float gs = fmaf(l * kl, (float)cs,
                                    fmaf(dq * kl, (float)cq, fmaf(l * dk, (float)ck, inner)));
                    score += gs;
                }
                scores[row * row_stride + t] = score * scale;
            }
        }
    }
    free(qs); free(qm); free(ql); free(qd);
}

typedef struct { float v; int32_t i; } scored_t;

static int by_score_then_index(const void* pa, const void* pb) {
    const scored_t* a = (const scored_t*)pa;
    const scored_t* b = (const scored_t*)pb;
    if (a->v > b->v) return -1;
    if (a->v < b->v) return 1;
    return (a->i > b->i) - (a->i < b->i);
}

static int by_index(const void* pa, const void* pb) {
    int32_t a = *(const int32_t*)pa, b = *(const int32_t*)pb;
    return (a > b) - (a < b);
}

/*
 * scores [rows, row_stride]; row r considers tokens [0, lengths[r]).
 * Output [rows, budget]: the k = min(budget-1, L) best tokens sorted by index
 * ascending, then L (the newest token), then -1 padding.
 */
void oracle_select(const float* scores, int64_t rows, int64_t row_stride, const int64_t* lengths,
                   int64_t budget, int32_t* indices) {
    for (int64_t r = 0; r < rows; ++r) {
        int64_t L = lengths[r];
        int64_t k = budget - 1 < L ? budget - 1 : L;
        int32_t* out = indices + r * budget;
        scored_t* items = (scored_t*)malloc(sizeof(scored_t) * (size_t)(L > 0 ? L : 1));
        for (int64_t t = 0; t < L; ++t) {
            float v = scores[r * row_stride + t];
            items[t].v = v == 0.0f ? 0.0f : v; /* -0.0 and +0.0 tie */
            items[t].i = (int32_t)t;
        }
        qsort(items, (size_t)L, sizeof(scored_t), by_score_then_index);
        for (int64_t j = 0; j < k; ++j) out[j] = items[j].i;
        qsort(out, (size_t)k, sizeof(int32_t), by_index);
        out[k] = (int32_t)L;
        for (int64_t j = k + 1; j < budget; ++j) out[j] = -1;
        free(items);
    }
}

/*
 * Exact attention over the selected rows, accumulated in double precision.
 * queries [batch, q_heads, D]; caches [cache_heads, kv_capacity, D] where the
 * head of (b, qh) is (cache_per_batch ? b*kv_heads : 0) + head_to_kv[qh].
 * current (nullable) [batch, kv_heads, D]: used for index == lengths[b].
 * indices [batch*q_heads, budget] (count = min(budget-1, L)+1 valid entries),
 * or NULL for dense attention over tokens 0..L (inclusive).
 */
void oracle_attention(const float* queries, int64_t batch, int64_t q_heads, int64_t head_dim,
                      const float* key_cache, const float* value_cache, int64_t kv_heads,
                      int64_t kv_capacity, int cache_per_batch, const float* cur_keys,
                      const float* cur_values, const int64_t* head_to_kv, const int32_t* indices,
                      int64_t budget, const int64_t* lengths, float* out) {
    const double scale = 1.0 / sqrt((double)head_dim);
    for (int64_t b = 0; b < batch; ++b) {
        int64_t L = lengths[b];
        for (int64_t h = 0; h < q_heads; ++h) {
            int64_t row = b * q_heads + h;
            int64_t kv = head_to_kv[h];
            int64_t ch = (cache_per_batch ? b * kv_heads : 0) + kv;
            const float* q = queries + row * head_dim;
            int64_t n = indices ? ((budget - 1 < L ? budget - 1 : L) + 1) : L + 1;
            double* logits = (double*)malloc(sizeof(double) * (size_t)n);
            double mx = -INFINITY;
            for (int64_t j = 0; j < n; ++j) {
                int64_t t = indices ? indices[row * budget + j] : j;
                const float* k = (t == L && cur_keys) ? cur_keys + (b * kv_heads + kv) * head_dim
                                                      : key_cache + (ch * kv_capacity + t) * head_dim;
                double s = 0.0;
                for (int64_t d = 0; d < head_dim; ++d) s += (double)q[d] * (double)k[d];
                logits[j] = s * scale;
                if (logits[j] > mx) mx = logits[j];
            }
            double denom = 0.0;
            for (int64_t j = 0; j < n; ++j) { logits[j] = exp(logits[j] - mx); denom += logits[j]; }
            for (int64_t d = 0; d < head_dim; ++d) {
                double acc = 0.0;
                for (int64_t j = 0; j < n; ++j) {
                    int64_t t = indices ? indices[row * budget + j] : j;
                    const float* v = (t == L && cur_values) ? cur_values + (b * kv_heads + kv) * head_dim
                                                            : value_cache + (ch * kv_capacity + t) * head_dim;
                    acc += logits[j] * (double)v[d];
                }
                out[row * head_dim + d] = (float)(acc / denom);
            }
            free(logits);
        }
    }
}
