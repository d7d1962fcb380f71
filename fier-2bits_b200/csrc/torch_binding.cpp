// Thin torch extension over the C ABI (include/popkv_b200.h).
//
// Mirrors the reference's pybind surface (csrc/popkv_ext.cpp:12-16: pack,
// pack_into, score) and adds the rest of the retrieval path (append, select,
// sparse_attention, advance).  Every function validates with TORCH_CHECK, hands
// raw device pointers and the current CUDA stream to the C ABI, and turns a
// non-zero status into a RuntimeError carrying the library's message.  No
// computation happens here.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <vector>

#include "popkv_b200.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIGUOUS(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_DTYPE(x, t) TORCH_CHECK((x).scalar_type() == (t), #x " has the wrong dtype")

void check_status(int rc, const char* what) {
    TORCH_CHECK(rc == POPKV_OK, what, " failed (", popkv_error_string(rc), "): ", popkv_last_error());
}

int dtype_code(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kFloat: return POPKV_F32;
        case at::kHalf: return POPKV_F16;
        case at::kBFloat16: return POPKV_BF16;
        default: TORCH_CHECK(false, "expected an fp32/fp16/bf16 tensor, got ", t.scalar_type());
    }
    return -1;
}

void* stream_of(const at::Tensor& t) {
    return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void check_packed(const std::vector<at::Tensor>& packed) {
    TORCH_CHECK(packed.size() == 4, "packed cache is (k_sign, k_mag, low, delta)");
    for (const auto& t : packed) { CHECK_CUDA(t); CHECK_CONTIGUOUS(t); }
    CHECK_DTYPE(packed[0], at::kInt);
    CHECK_DTYPE(packed[1], at::kInt);
    TORCH_CHECK(packed[2].scalar_type() == at::kHalf && packed[3].scalar_type() == at::kHalf,
                "Pop-KV representative metadata must be float16");
    for (int i = 1; i < 4; ++i)
        TORCH_CHECK(packed[i].sizes() == packed[0].sizes(), "packed tensors must share one shape");
    TORCH_CHECK(packed[0].dim() == 3 || packed[0].dim() == 4,
                "packed tensors are [KVH, capacity, words] or [B, KVH, capacity, words]");
}

void* select_ws_ptr(const c10::optional<at::Tensor>& ws, int64_t rows, int64_t tokens) {
    if (!ws) return nullptr;
    CHECK_CUDA(*ws); CHECK_CONTIGUOUS(*ws);
    TORCH_CHECK((size_t)ws->nbytes() >= popkv_select_workspace_bytes(rows, tokens),
                "select workspace too small for ", rows, " rows of ", tokens, " tokens");
    return ws->data_ptr();
}

std::vector<at::Tensor> pack(const at::Tensor& keys, int64_t token_capacity, int64_t flags,
                             bool with_thresholds) {
    CHECK_CUDA(keys); CHECK_CONTIGUOUS(keys);
    TORCH_CHECK(keys.dim() == 3, "keys must be [KVH, T, D]");
    TORCH_CHECK(token_capacity >= keys.size(1), "token capacity is too small");
    c10::cuda::CUDAGuard guard(keys.device());
    const int64_t heads = keys.size(0), tokens = keys.size(1), dim = keys.size(2);
    const int64_t words = (dim + 31) / 32;
    auto opts = keys.options();
    auto k_sign = at::empty({heads, token_capacity, words}, opts.dtype(at::kInt));
    auto k_mag = at::empty({heads, token_capacity, words}, opts.dtype(at::kInt));
    auto low = at::empty({heads, token_capacity, words}, opts.dtype(at::kHalf));
    auto delta = at::empty({heads, token_capacity, words}, opts.dtype(at::kHalf));
    at::Tensor thr;
    if (with_thresholds) thr = at::empty({heads, (tokens + 31) / 32, dim, 2}, opts.dtype(at::kFloat));
    const int rc = popkv_pack(keys.data_ptr(), dtype_code(keys), heads, tokens, dim, tokens * dim,
                              k_sign.data_ptr<int32_t>(), k_mag.data_ptr<int32_t>(),
                              reinterpret_cast<uint16_t*>(low.data_ptr<at::Half>()),
                              reinterpret_cast<uint16_t*>(delta.data_ptr<at::Half>()),
                              token_capacity, 0, with_thresholds ? thr.data_ptr<float>() : nullptr,
                              (int)flags, stream_of(keys));
    check_status(rc, "popkv_pack");
    std::vector<at::Tensor> out{k_sign, k_mag, low, delta};
    if (with_thresholds) out.push_back(thr);
    return out;
}

void pack_into(const at::Tensor& keys, const at::Tensor& k_sign, const at::Tensor& k_mag,
               const at::Tensor& low, const at::Tensor& delta, int64_t token_offset,
               int64_t flags) {
    CHECK_CUDA(keys); CHECK_CONTIGUOUS(keys);
    TORCH_CHECK(keys.dim() == 3, "keys must be [KVH, T, D]");
    check_packed({k_sign, k_mag, low, delta});
    TORCH_CHECK(k_sign.dim() == 3 && k_sign.size(0) == keys.size(0), "packed cache heads mismatch");
    TORCH_CHECK(token_offset >= 0 && token_offset + keys.size(1) <= k_sign.size(1),
                "Pop-KV cache capacity exceeded");
    c10::cuda::CUDAGuard guard(keys.device());
    const int rc = popkv_pack(keys.data_ptr(), dtype_code(keys), keys.size(0), keys.size(1),
                              keys.size(2), keys.size(1) * keys.size(2), k_sign.data_ptr<int32_t>(),
                              k_mag.data_ptr<int32_t>(),
                              reinterpret_cast<uint16_t*>(low.data_ptr<at::Half>()),
                              reinterpret_cast<uint16_t*>(delta.data_ptr<at::Half>()),
                              k_sign.size(1), token_offset, nullptr, (int)flags, stream_of(keys));
    check_status(rc, "popkv_pack");
}

void append(const at::Tensor& key_cache, const c10::optional<at::Tensor>& value_cache,
            const c10::optional<at::Tensor>& new_keys, const c10::optional<at::Tensor>& new_values,
            const at::Tensor& k_sign, const at::Tensor& k_mag, const at::Tensor& low,
            const at::Tensor& delta, int64_t position, const c10::optional<at::Tensor>& seq_len,
            int64_t kv_heads_per_seq, int64_t flags) {
    CHECK_CUDA(key_cache); CHECK_CONTIGUOUS(key_cache);
    check_packed({k_sign, k_mag, low, delta});
    TORCH_CHECK(key_cache.dim() >= 3, "key cache is [..., heads, capacity, D]");
    const int64_t dim = key_cache.size(-1), kv_cap = key_cache.size(-2);
    const int64_t heads = key_cache.numel() / (kv_cap * dim);
    const int64_t cap = k_sign.size(-2);
    TORCH_CHECK(k_sign.numel() / (cap * k_sign.size(-1)) == heads, "packed cache heads mismatch");
    const void* nk = nullptr;
    const void* nv = nullptr;
    void* vc = nullptr;
    if (new_keys) {
        CHECK_CUDA(*new_keys); CHECK_CONTIGUOUS(*new_keys);
        TORCH_CHECK(new_keys->numel() == heads * dim && new_keys->scalar_type() == key_cache.scalar_type(),
                    "new_keys must hold one row per cache head, in the cache dtype");
        nk = new_keys->data_ptr();
    }
    if (value_cache && new_values) {
        CHECK_CUDA(*value_cache); CHECK_CONTIGUOUS(*value_cache);
        CHECK_CUDA(*new_values); CHECK_CONTIGUOUS(*new_values);
        TORCH_CHECK(value_cache->sizes() == key_cache.sizes() && new_values->numel() == heads * dim,
                    "value cache / new values shape mismatch");
        vc = value_cache->data_ptr();
        nv = new_values->data_ptr();
    }
    const int32_t* sl = nullptr;
    if (seq_len) { CHECK_CUDA(*seq_len); CHECK_DTYPE(*seq_len, at::kInt); sl = seq_len->data_ptr<int32_t>(); }
    c10::cuda::CUDAGuard guard(key_cache.device());
    const int rc = popkv_append(key_cache.data_ptr(), vc, dtype_code(key_cache), heads, kv_cap, dim,
                                nk, nv, k_sign.data_ptr<int32_t>(), k_mag.data_ptr<int32_t>(),
                                reinterpret_cast<uint16_t*>(low.data_ptr<at::Half>()),
                                reinterpret_cast<uint16_t*>(delta.data_ptr<at::Half>()), cap, sl,
                                position, kv_heads_per_seq, (int)flags, stream_of(key_cache));
    check_status(rc, "popkv_append");
}

at::Tensor score(const at::Tensor& queries, const at::Tensor& k_sign, const at::Tensor& k_mag,
                 const at::Tensor& low, const at::Tensor& delta, const at::Tensor& head_to_kv,
                 int64_t tokens, int64_t flags, const c10::optional<at::Tensor>& seq_len,
                 const c10::optional<at::Tensor>& out, const c10::optional<at::Tensor>& hist) {
    CHECK_CUDA(queries); CHECK_CONTIGUOUS(queries);
    TORCH_CHECK(queries.dim() == 3, "queries must be [B, QH, D]");
    check_packed({k_sign, k_mag, low, delta});
    CHECK_CUDA(head_to_kv); CHECK_CONTIGUOUS(head_to_kv);
    TORCH_CHECK(head_to_kv.scalar_type() == at::kLong, "head mapping must be int64");
    TORCH_CHECK(head_to_kv.numel() == queries.size(1), "head mapping needs one entry per query head");
    const int64_t batch = queries.size(0), q_heads = queries.size(1), dim = queries.size(2);
    const bool per_batch = k_sign.dim() == 4;
    if (per_batch) TORCH_CHECK(k_sign.size(0) == batch, "batched packed cache must match the batch");
    const int64_t kv_heads = per_batch ? k_sign.size(1) : k_sign.size(0);
    const int64_t cap = k_sign.size(-2);
    TORCH_CHECK(k_sign.size(-1) == (dim + 31) / 32, "packed words do not match head_dim");
    TORCH_CHECK(tokens > 0 && tokens <= cap, "invalid score token count");
    const int32_t* sl = nullptr;
    if (seq_len) { CHECK_CUDA(*seq_len); CHECK_DTYPE(*seq_len, at::kInt); sl = seq_len->data_ptr<int32_t>(); }
    c10::cuda::CUDAGuard guard(queries.device());
    at::Tensor scores;
    if (out) {
        scores = *out;
        CHECK_CUDA(scores); CHECK_CONTIGUOUS(scores); CHECK_DTYPE(scores, at::kFloat);
        TORCH_CHECK(scores.dim() == 3 && scores.size(0) == batch && scores.size(1) == q_heads &&
                    scores.size(2) >= tokens, "scores out must be [B, QH, >= tokens]");
    } else {
        scores = at::empty({batch, q_heads, tokens}, queries.options().dtype(at::kFloat));
    }
    const int rc = popkv_score(queries.data_ptr(), dtype_code(queries), batch, q_heads, dim,
                               k_sign.data_ptr<int32_t>(), k_mag.data_ptr<int32_t>(),
                               reinterpret_cast<const uint16_t*>(low.data_ptr<at::Half>()),
                               reinterpret_cast<const uint16_t*>(delta.data_ptr<at::Half>()),
                               kv_heads, cap, per_batch ? 1 : 0, head_to_kv.data_ptr<int64_t>(),
                               tokens, sl, scores.data_ptr<float>(), scores.size(2),
                               select_ws_ptr(hist, batch * q_heads, tokens), (int)flags, stream_of(queries));
    check_status(rc, "popkv_score");
    return scores;
}

at::Tensor select_topk(const at::Tensor& scores, int64_t budget, int64_t tokens,
                       const c10::optional<at::Tensor>& seq_len, int64_t rows_per_seq,
                       const c10::optional<at::Tensor>& out,
                       const c10::optional<at::Tensor>& attn_workspace,
                       std::vector<int64_t> attn_sizes, const c10::optional<at::Tensor>& hist) {
    CHECK_CUDA(scores); CHECK_DTYPE(scores, at::kFloat);
    TORCH_CHECK(scores.stride(-1) == 1, "scores rows must be contiguous");
    const int64_t stride = scores.dim() > 1 ? scores.stride(-2) : scores.size(-1);
    const int64_t rows = scores.numel() / std::max<int64_t>(scores.size(-1), 1);
    TORCH_CHECK(scores.dim() <= 2 || scores.is_contiguous(), "scores must be contiguous or a 2-D row view");
    TORCH_CHECK(tokens <= scores.size(-1), "tokens exceed the score row length");
    const int32_t* sl = nullptr;
    if (seq_len) { CHECK_CUDA(*seq_len); CHECK_DTYPE(*seq_len, at::kInt); sl = seq_len->data_ptr<int32_t>(); }
    c10::cuda::CUDAGuard guard(scores.device());
    at::Tensor idx;
    if (out) {
        idx = *out;
        CHECK_CUDA(idx); CHECK_CONTIGUOUS(idx); CHECK_DTYPE(idx, at::kInt);
        TORCH_CHECK(idx.numel() == rows * budget, "indices out must hold rows x budget entries");
    } else {
        idx = at::empty({rows, budget}, scores.options().dtype(at::kInt));
    }
    uint16_t* masks = nullptr;
    int64_t mask_stride = 0, heads_per_kv = 0;
    if (attn_workspace) {
        // attn_sizes = (batch, q_heads, kv_heads, head_dim, tokens, splits) of the attention call.
        TORCH_CHECK(attn_sizes.size() == 6, "attn_sizes = (batch, q_heads, kv_heads, head_dim, tokens, splits)");
        CHECK_CUDA(*attn_workspace); CHECK_CONTIGUOUS(*attn_workspace);
        const size_t need = popkv_sparse_attention_workspace_bytes(attn_sizes[0], attn_sizes[1], attn_sizes[2],
                                                                   attn_sizes[3], attn_sizes[4], attn_sizes[5]);
        TORCH_CHECK((size_t)attn_workspace->nbytes() >= need, "attention workspace too small");
        check_status(popkv_sparse_attention_masks(attn_workspace->data_ptr(), attn_sizes[0], attn_sizes[1],
                                                  attn_sizes[2], attn_sizes[3], attn_sizes[4], attn_sizes[5],
                                                  &masks, &mask_stride),
                     "popkv_sparse_attention_masks");
        heads_per_kv = attn_sizes[1] / attn_sizes[2];
        TORCH_CHECK(rows_per_seq == attn_sizes[1], "rows_per_seq must equal q_heads with head masks");
    }
    const int rc = popkv_select(scores.data_ptr<float>(), rows, stride, tokens, sl, rows_per_seq,
                                budget, idx.data_ptr<int32_t>(), masks, mask_stride, heads_per_kv,
                                select_ws_ptr(hist, rows, tokens), hist ? (size_t)hist->nbytes() : 0,
                                stream_of(scores));
    check_status(rc, "popkv_select");
    return idx;
}

// Score + select in one call (popkv_score_select): indices [B*QH, budget], optionally
// the attention workspace's head bitmask; `scores`/`hist` serve the two-kernel
// fallback only.
at::Tensor score_select(const at::Tensor& queries, const at::Tensor& k_sign, const at::Tensor& k_mag,
                        const at::Tensor& low, const at::Tensor& delta, const at::Tensor& head_to_kv,
                        int64_t budget, int64_t tokens, int64_t flags,
                        const c10::optional<at::Tensor>& seq_len, const c10::optional<at::Tensor>& out,
                        const c10::optional<at::Tensor>& attn_workspace, std::vector<int64_t> attn_sizes,
                        const c10::optional<at::Tensor>& scores, const c10::optional<at::Tensor>& hist) {
    CHECK_CUDA(queries); CHECK_CONTIGUOUS(queries);
    TORCH_CHECK(queries.dim() == 3, "queries must be [B, QH, D]");
    check_packed({k_sign, k_mag, low, delta});
    CHECK_CUDA(head_to_kv); CHECK_CONTIGUOUS(head_to_kv);
    TORCH_CHECK(head_to_kv.scalar_type() == at::kLong, "head mapping must be int64");
    TORCH_CHECK(head_to_kv.numel() == queries.size(1), "head mapping needs one entry per query head");
    const int64_t batch = queries.size(0), q_heads = queries.size(1), dim = queries.size(2);
    const bool per_batch = k_sign.dim() == 4;
    if (per_batch) TORCH_CHECK(k_sign.size(0) == batch, "batched packed cache must match the batch");
    const int64_t kv_heads = per_batch ? k_sign.size(1) : k_sign.size(0);
    const int64_t cap = k_sign.size(-2);
    TORCH_CHECK(k_sign.size(-1) == (dim + 31) / 32, "packed words do not match head_dim");
    TORCH_CHECK(tokens > 0 && tokens <= cap, "invalid score token count");
    const int32_t* sl = nullptr;
    if (seq_len) { CHECK_CUDA(*seq_len); CHECK_DTYPE(*seq_len, at::kInt); sl = seq_len->data_ptr<int32_t>(); }
    c10::cuda::CUDAGuard guard(queries.device());
    const int64_t rows = batch * q_heads;
    at::Tensor idx;
    if (out) {
        idx = *out;
        CHECK_CUDA(idx); CHECK_CONTIGUOUS(idx); CHECK_DTYPE(idx, at::kInt);
        TORCH_CHECK(idx.numel() == rows * budget, "indices out must hold rows x budget entries");
    } else {
        idx = at::empty({rows, budget}, queries.options().dtype(at::kInt));
    }
    uint16_t* masks = nullptr;
    int64_t mask_stride = 0, heads_per_kv = 0;
    if (attn_workspace) {
        TORCH_CHECK(attn_sizes.size() == 6, "attn_sizes = (batch, q_heads, kv_heads, head_dim, tokens, splits)");
        CHECK_CUDA(*attn_workspace); CHECK_CONTIGUOUS(*attn_workspace);
        const size_t need = popkv_sparse_attention_workspace_bytes(attn_sizes[0], attn_sizes[1], attn_sizes[2],
                                                                   attn_sizes[3], attn_sizes[4], attn_sizes[5]);
        TORCH_CHECK((size_t)attn_workspace->nbytes() >= need, "attention workspace too small");
        check_status(popkv_sparse_attention_masks(attn_workspace->data_ptr(), attn_sizes[0], attn_sizes[1],
                                                  attn_sizes[2], attn_sizes[3], attn_sizes[4], attn_sizes[5],
                                                  &masks, &mask_stride),
                     "popkv_sparse_attention_masks");
        heads_per_kv = attn_sizes[1] / attn_sizes[2];
        TORCH_CHECK(q_heads == attn_sizes[1], "attention sizes must match the queries");
    }
    float* sp = nullptr;
    int64_t sstride = tokens;
    if (scores) {
        CHECK_CUDA(*scores); CHECK_CONTIGUOUS(*scores); CHECK_DTYPE(*scores, at::kFloat);
        TORCH_CHECK(scores->numel() >= rows * tokens && scores->numel() % rows == 0, "scores buffer too small");
        sp = scores->data_ptr<float>();
        sstride = scores->numel() / rows;
    }
    const int rc = popkv_score_select(
        queries.data_ptr(), dtype_code(queries), batch, q_heads, dim, k_sign.data_ptr<int32_t>(),
        k_mag.data_ptr<int32_t>(), reinterpret_cast<const uint16_t*>(low.data_ptr<at::Half>()),
        reinterpret_cast<const uint16_t*>(delta.data_ptr<at::Half>()), kv_heads, cap, per_batch ? 1 : 0,
        head_to_kv.data_ptr<int64_t>(), tokens, sl, budget, idx.data_ptr<int32_t>(), masks, mask_stride,
        heads_per_kv, sp, sstride, select_ws_ptr(hist, rows, tokens), hist ? (size_t)hist->nbytes() : 0,
        (int)flags, stream_of(queries));
    check_status(rc, "popkv_score_select");
    return idx;
}

std::mutex g_ws_mutex;
std::map<std::vector<int64_t>, at::Tensor> g_workspaces;

// One zero-initialised workspace per (device, shape) layout: the kernels keep a
// workspace clean for the layout it was used with, not for a different one.
at::Tensor default_workspace(const at::Device& dev, std::vector<int64_t> key, size_t bytes) {
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    key.push_back(dev.index());
    auto& ws = g_workspaces[key];
    if (!ws.defined() || (size_t)ws.numel() < bytes)
        ws = at::zeros({(int64_t)bytes}, at::TensorOptions().device(dev).dtype(at::kByte));
    return ws;
}

int64_t workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                        int64_t tokens, int64_t splits) {
    return (int64_t)popkv_sparse_attention_workspace_bytes(batch, q_heads, kv_heads, head_dim,
                                                           tokens, splits);
}

at::Tensor sparse_attention(const at::Tensor& queries, const at::Tensor& key_cache,
                            const at::Tensor& value_cache,
                            const c10::optional<at::Tensor>& indices, int64_t budget,
                            int64_t tokens, const c10::optional<at::Tensor>& current_keys,
                            const c10::optional<at::Tensor>& current_values,
                            const c10::optional<at::Tensor>& seq_len,
                            const c10::optional<at::Tensor>& workspace, int64_t splits,
                            const c10::optional<at::Tensor>& out) {
    CHECK_CUDA(queries); CHECK_CONTIGUOUS(queries);
    CHECK_CUDA(key_cache); CHECK_CONTIGUOUS(key_cache);
    CHECK_CUDA(value_cache); CHECK_CONTIGUOUS(value_cache);
    TORCH_CHECK(queries.dim() == 3, "queries must be [B, QH, D]");
    TORCH_CHECK(key_cache.sizes() == value_cache.sizes(), "key and value caches differ in shape");
    TORCH_CHECK(key_cache.scalar_type() == queries.scalar_type() &&
                value_cache.scalar_type() == queries.scalar_type(),
                "queries and caches must share one dtype");
    const int64_t batch = queries.size(0), q_heads = queries.size(1), dim = queries.size(2);
    TORCH_CHECK(key_cache.dim() == 3 || key_cache.dim() == 4,
                "caches are [KVH, capacity, D] (shared) or [B, KVH, capacity, D]");
    TORCH_CHECK(key_cache.size(-1) == dim, "cache head_dim mismatch");
    const bool per_batch = key_cache.dim() == 4;
    const int64_t kv_heads = key_cache.dim() == 4 ? key_cache.size(1) : key_cache.size(0);
    if (key_cache.dim() == 4) TORCH_CHECK(key_cache.size(0) == batch, "batched caches must match the batch");
    const int64_t kv_cap = key_cache.size(-2);
    const void* ck = nullptr;
    const void* cv = nullptr;
    if (current_keys || current_values) {
        TORCH_CHECK(current_keys && current_values, "current_keys and current_values go together");
        CHECK_CUDA(*current_keys); CHECK_CONTIGUOUS(*current_keys);
        CHECK_CUDA(*current_values); CHECK_CONTIGUOUS(*current_values);
        TORCH_CHECK(current_keys->numel() == batch * kv_heads * dim &&
                    current_values->numel() == batch * kv_heads * dim,
                    "current rows must be [B, KVH, D]");
        TORCH_CHECK(current_keys->scalar_type() == queries.scalar_type() &&
                    current_values->scalar_type() == queries.scalar_type(), "current rows dtype");
        ck = current_keys->data_ptr();
        cv = current_values->data_ptr();
    }
    const int32_t* idx = nullptr;
    int64_t idx_stride = 0;
    if (indices) {
        CHECK_CUDA(*indices); CHECK_CONTIGUOUS(*indices); CHECK_DTYPE(*indices, at::kInt);
        TORCH_CHECK(indices->numel() % (batch * q_heads) == 0, "indices must be [B*QH, n]");
        idx_stride = indices->numel() / (batch * q_heads);
        TORCH_CHECK(idx_stride >= budget, "indices rows shorter than budget");
        idx = indices->data_ptr<int32_t>();
    }
    const int32_t* sl = nullptr;
    if (seq_len) { CHECK_CUDA(*seq_len); CHECK_DTYPE(*seq_len, at::kInt); sl = seq_len->data_ptr<int32_t>(); }
    c10::cuda::CUDAGuard guard(queries.device());
    const size_t need = popkv_sparse_attention_workspace_bytes(batch, q_heads, kv_heads, dim, tokens, splits);
    at::Tensor ws;
    if (workspace) {
        ws = *workspace;
        CHECK_CUDA(ws); CHECK_CONTIGUOUS(ws);
        TORCH_CHECK((size_t)ws.nbytes() >= need, "workspace too small: ", ws.nbytes(), " < ", need);
    } else {
        ws = default_workspace(queries.device(), {batch, q_heads, kv_heads, dim, tokens, splits}, need);
    }
    at::Tensor o = out ? *out : at::empty_like(queries);
    if (out) {
        CHECK_CUDA(o); CHECK_CONTIGUOUS(o);
        TORCH_CHECK(o.sizes() == queries.sizes() && o.scalar_type() == queries.scalar_type(), "out shape/dtype");
    }
    const int rc = popkv_sparse_attention(
        queries.data_ptr(), dtype_code(queries), batch, q_heads, dim, key_cache.data_ptr(),
        value_cache.data_ptr(), kv_heads, kv_cap, per_batch ? 1 : 0, ck, cv, idx, idx_stride,
        budget, tokens, sl, o.data_ptr(), ws.data_ptr(), (size_t)ws.nbytes(), splits,
        stream_of(queries));
    check_status(rc, "popkv_sparse_attention");
    return o;
}

at::Tensor sparse_attention_premasked(const at::Tensor& queries, const at::Tensor& key_cache,
                                     const at::Tensor& value_cache, int64_t tokens,
                                     const at::Tensor& current_keys, const at::Tensor& current_values,
                                     const c10::optional<at::Tensor>& seq_len,
                                     const at::Tensor& workspace, int64_t splits, const at::Tensor& out,
                                     std::vector<int64_t> peer_out, std::vector<int64_t> peer_flags,
                                     int64_t rank, const c10::optional<at::Tensor>& sync_words,
                                     bool defer_wait) {
    for (const at::Tensor* t : {&queries, &key_cache, &value_cache, &current_keys, &current_values, &workspace, &out}) {
        CHECK_CUDA(*t); CHECK_CONTIGUOUS(*t);
    }
    TORCH_CHECK(queries.dim() == 3 && out.sizes() == queries.sizes(), "queries/out must be [B, QH, D]");
    TORCH_CHECK(key_cache.sizes() == value_cache.sizes() && key_cache.dim() == 4, "caches are [B, KVH, capacity, D]");
    const int64_t batch = queries.size(0), q_heads = queries.size(1), dim = queries.size(2);
    const int64_t kv_heads = key_cache.size(1);
    const int32_t* sl = nullptr;
    if (seq_len) { CHECK_CUDA(*seq_len); CHECK_DTYPE(*seq_len, at::kInt); sl = seq_len->data_ptr<int32_t>(); }
    c10::cuda::CUDAGuard guard(queries.device());
    int rc;
    if (peer_out.empty()) {
        rc = popkv_sparse_attention_premasked(
            queries.data_ptr(), dtype_code(queries), batch, q_heads, dim, key_cache.data_ptr(),
            value_cache.data_ptr(), kv_heads, key_cache.size(2), 1, current_keys.data_ptr(),
            current_values.data_ptr(), tokens, sl, out.data_ptr(), workspace.data_ptr(),
            (size_t)workspace.nbytes(), splits, stream_of(queries));
    } else {
        // Peer all-gather: device addresses of every rank's gathered buffer and arrival
        // words (mapped into this process), this rank's sync words.
        TORCH_CHECK(sync_words && peer_flags.size() == peer_out.size(), "peer gather needs flags and sync words");
        CHECK_CUDA(*sync_words); CHECK_DTYPE(*sync_words, at::kInt);
        TORCH_CHECK(sync_words->numel() >= 3, "sync words hold 3 entries");
        std::vector<void*> outs;
        std::vector<uint32_t*> flags;
        for (int64_t a : peer_out) outs.push_back(reinterpret_cast<void*>(a));
        for (int64_t a : peer_flags) flags.push_back(reinterpret_cast<uint32_t*>(a));
        rc = popkv_sparse_attention_premasked_gather(
            queries.data_ptr(), dtype_code(queries), batch, q_heads, dim, key_cache.data_ptr(),
            value_cache.data_ptr(), kv_heads, key_cache.size(2), 1, current_keys.data_ptr(),
            current_values.data_ptr(), tokens, sl, out.data_ptr(), workspace.data_ptr(),
            (size_t)workspace.nbytes(), splits, (int)outs.size(), (int)rank, outs.data(), flags.data(),
            reinterpret_cast<uint32_t*>(sync_words->data_ptr<int32_t>()), defer_wait ? 1 : 0,
            stream_of(queries));
    }
    check_status(rc, "popkv_sparse_attention_premasked");
    return out;
}

// Deferred wait of the peer all-gather: flags = this rank's [layers, world] arrival
// words, sync = its [layers, 3] sync words.
void peer_wait(const at::Tensor& flags, const at::Tensor& sync) {
    CHECK_CUDA(flags); CHECK_CONTIGUOUS(flags); CHECK_DTYPE(flags, at::kInt);
    CHECK_CUDA(sync); CHECK_CONTIGUOUS(sync); CHECK_DTYPE(sync, at::kInt);
    TORCH_CHECK(flags.dim() == 2 && sync.dim() == 2 && sync.size(1) == 3 && sync.size(0) == flags.size(0),
                "flags are [layers, world] and sync words [layers, 3]");
    c10::cuda::CUDAGuard guard(flags.device());
    check_status(popkv_peer_gather_wait(reinterpret_cast<const uint32_t*>(flags.data_ptr<int32_t>()),
                                        reinterpret_cast<uint32_t*>(sync.data_ptr<int32_t>()),
                                        (int)flags.size(0), (int)flags.size(1), stream_of(flags)),
                 "popkv_peer_gather_wait");
}

void peer_push(const at::Tensor& rows, std::vector<int64_t> peer_dst, std::vector<int64_t> peer_flags,
               int64_t rank, const at::Tensor& sync_words) {
    CHECK_CUDA(rows); CHECK_CONTIGUOUS(rows); CHECK_CUDA(sync_words); CHECK_CONTIGUOUS(sync_words);
    CHECK_DTYPE(sync_words, at::kInt);
    TORCH_CHECK(peer_dst.size() == peer_flags.size() && !peer_dst.empty() && peer_dst.size() <= 8,
                "one destination and one flag pointer per rank (at most 8)");
    TORCH_CHECK(sync_words.numel() == 3, "sync words are the layer's [3] words");
    std::vector<void*> dst(peer_dst.size());
    std::vector<uint32_t*> flg(peer_flags.size());
    for (size_t j = 0; j < dst.size(); ++j) {
        dst[j] = reinterpret_cast<void*>(peer_dst[j]);
        flg[j] = reinterpret_cast<uint32_t*>(peer_flags[j]);
    }
    c10::cuda::CUDAGuard guard(rows.device());
    check_status(popkv_peer_push(rows.data_ptr(), rows.numel() * rows.element_size(), dst.data(), flg.data(),
                                 (int)rank, (int)dst.size(),
                                 reinterpret_cast<uint32_t*>(sync_words.data_ptr<int32_t>()),
                                 stream_of(rows)),
                 "popkv_peer_push");
}

void advance(const at::Tensor& seq_len, int64_t increment) {
    CHECK_CUDA(seq_len); CHECK_CONTIGUOUS(seq_len); CHECK_DTYPE(seq_len, at::kInt);
    c10::cuda::CUDAGuard guard(seq_len.device());
    check_status(popkv_advance(seq_len.data_ptr<int32_t>(), seq_len.numel(), (int32_t)increment,
                               stream_of(seq_len)),
                 "popkv_advance");
}

void gemv(const at::Tensor& x, const at::Tensor& weight, const c10::optional<at::Tensor>& residual,
          const at::Tensor& out) {
    CHECK_CUDA(x); CHECK_CONTIGUOUS(x); CHECK_CUDA(weight); CHECK_CONTIGUOUS(weight);
    CHECK_CUDA(out); CHECK_CONTIGUOUS(out);
    TORCH_CHECK(weight.dim() == 2 && x.numel() == weight.size(1) && out.numel() == weight.size(0),
                "gemv: x [k], weight [n, k], out [n]");
    TORCH_CHECK(x.scalar_type() == weight.scalar_type() && out.scalar_type() == x.scalar_type(),
                "gemv tensors must share a dtype");
    const void* res = nullptr;
    if (residual) {
        CHECK_CUDA(*residual); CHECK_CONTIGUOUS(*residual);
        TORCH_CHECK(residual->numel() == out.numel() && residual->scalar_type() == x.scalar_type(), "gemv residual");
        res = residual->data_ptr();
    }
    c10::cuda::CUDAGuard guard(x.device());
    check_status(popkv_gemv(x.data_ptr(), weight.data_ptr(), res, out.data_ptr(), dtype_code(x),
                            weight.size(0), weight.size(1), stream_of(x)),
                 "popkv_gemv");
}

void rmsnorm(const at::Tensor& x, const at::Tensor& weight, double eps, const at::Tensor& out) {
    for (const at::Tensor* t : {&x, &weight, &out}) { CHECK_CUDA((*t)); CHECK_CONTIGUOUS((*t)); }
    TORCH_CHECK(x.scalar_type() == weight.scalar_type() && x.scalar_type() == out.scalar_type(),
                "rmsnorm tensors must share a dtype");
    const int64_t n = x.size(-1);
    TORCH_CHECK(weight.numel() == n && out.numel() == x.numel(), "rmsnorm shapes");
    c10::cuda::CUDAGuard guard(x.device());
    check_status(popkv_rmsnorm(x.data_ptr(), weight.data_ptr(), out.data_ptr(), dtype_code(x),
                               x.numel() / n, n, (float)eps, stream_of(x)),
                 "popkv_rmsnorm");
}

void rope_qkv(const at::Tensor& qkv, const at::Tensor& cos, const at::Tensor& sin,
              const at::Tensor& positions_of_rows, int64_t q_heads, int64_t kv_heads,
              const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
    for (const at::Tensor* t : {&qkv, &cos, &sin, &positions_of_rows, &q, &k, &v}) {
        CHECK_CUDA((*t)); CHECK_CONTIGUOUS((*t));
    }
    CHECK_DTYPE(positions_of_rows, at::kInt);
    const int64_t D = cos.size(-1);
    const int64_t rows = qkv.numel() / ((q_heads + 2 * kv_heads) * D);
    TORCH_CHECK(rows * (q_heads + 2 * kv_heads) * D == qkv.numel() && positions_of_rows.numel() >= rows,
                "qkv must be [rows, (q_heads + 2 kv_heads) * head_dim]");
    TORCH_CHECK(q.numel() == rows * q_heads * D && k.numel() == rows * kv_heads * D &&
                v.numel() == rows * kv_heads * D && sin.sizes() == cos.sizes(), "rope output shapes");
    c10::cuda::CUDAGuard guard(qkv.device());
    check_status(popkv_rope_qkv(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                positions_of_rows.data_ptr<int32_t>(), cos.size(0), dtype_code(qkv), rows,
                                q_heads, kv_heads, D, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                stream_of(qkv)),
                 "popkv_rope_qkv");
}

void silu_mul(const at::Tensor& gate_up, const at::Tensor& out) {
    CHECK_CUDA(gate_up); CHECK_CONTIGUOUS(gate_up); CHECK_CUDA(out); CHECK_CONTIGUOUS(out);
    const int64_t ffn = out.size(-1);
    TORCH_CHECK(gate_up.size(-1) == 2 * ffn && gate_up.numel() == 2 * out.numel(), "gate_up is [rows, 2 ffn]");
    c10::cuda::CUDAGuard guard(out.device());
    check_status(popkv_silu_mul(gate_up.data_ptr(), out.data_ptr(), dtype_code(out), out.numel() / ffn, ffn,
                                stream_of(out)),
                 "popkv_silu_mul");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "Pop-KV retrieval on B200 (sm_100a): torch front end of the C ABI";
    m.def("pack", &pack, py::arg("keys"), py::arg("token_capacity"), py::arg("flags") = 0,
          py::arg("with_thresholds") = false);
    m.def("pack_into", &pack_into, py::arg("keys"), py::arg("k_sign"), py::arg("k_mag"),
          py::arg("low"), py::arg("delta"), py::arg("token_offset"), py::arg("flags") = 0);
    m.def("append", &append, py::arg("key_cache"), py::arg("value_cache"), py::arg("new_keys"),
          py::arg("new_values"), py::arg("k_sign"), py::arg("k_mag"), py::arg("low"),
          py::arg("delta"), py::arg("position"), py::arg("seq_len") = py::none(),
          py::arg("kv_heads_per_seq") = 0, py::arg("flags") = 0);
    m.def("score", &score, py::arg("queries"), py::arg("k_sign"), py::arg("k_mag"), py::arg("low"),
          py::arg("delta"), py::arg("head_to_kv"), py::arg("tokens"), py::arg("flags") = 0,
          py::arg("seq_len") = py::none(), py::arg("out") = py::none(), py::arg("hist") = py::none());
    m.def("select", &select_topk, py::arg("scores"), py::arg("budget"), py::arg("tokens"),
          py::arg("seq_len") = py::none(), py::arg("rows_per_seq") = 0, py::arg("out") = py::none(),
          py::arg("attn_workspace") = py::none(), py::arg("attn_sizes") = std::vector<int64_t>{},
          py::arg("hist") = py::none());
    m.def("score_select", &score_select, py::arg("queries"), py::arg("k_sign"), py::arg("k_mag"),
          py::arg("low"), py::arg("delta"), py::arg("head_to_kv"), py::arg("budget"), py::arg("tokens"),
          py::arg("flags"), py::arg("seq_len"), py::arg("out"), py::arg("attn_workspace"),
          py::arg("attn_sizes"), py::arg("scores"), py::arg("hist"));
    m.def("sparse_attention_premasked", &sparse_attention_premasked, py::arg("queries"), py::arg("key_cache"),
          py::arg("value_cache"), py::arg("tokens"), py::arg("current_keys"), py::arg("current_values"),
          py::arg("seq_len"), py::arg("workspace"), py::arg("splits"), py::arg("out"),
          py::arg("peer_out") = std::vector<int64_t>{}, py::arg("peer_flags") = std::vector<int64_t>{},
          py::arg("rank") = 0, py::arg("sync_words") = py::none(), py::arg("defer_wait") = false);
    m.def("peer_wait", &peer_wait, py::arg("flags"), py::arg("sync"));
    m.def("sparse_attention", &sparse_attention, py::arg("queries"), py::arg("key_cache"),
          py::arg("value_cache"), py::arg("indices"), py::arg("budget"), py::arg("tokens"),
          py::arg("current_keys") = py::none(), py::arg("current_values") = py::none(),
          py::arg("seq_len") = py::none(), py::arg("workspace") = py::none(),
          py::arg("splits") = 0, py::arg("out") = py::none());
    m.def("workspace_bytes", &workspace_bytes);
    m.def("select_workspace_bytes", [](int64_t rows, int64_t tokens) {
        return (int64_t)popkv_select_workspace_bytes(rows, tokens);
    });
    m.def("advance", &advance);
    m.def("peer_push", &peer_push);
    m.def("rmsnorm", &rmsnorm);
    m.def("gemv", &gemv);
    m.def("rope_qkv", &rope_qkv);
    m.def("silu_mul", &silu_mul);
    m.def("version", &popkv_version);
}
