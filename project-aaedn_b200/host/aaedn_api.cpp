// aaedn_api.cpp — the reference's C++ API (namespace aaedn, the headers in
// host/include/aaedn/) as a thin layer over the C ABI (include/aaedn_b200.h).
//
// The signatures are the reference's, so they return void; failures leave
// the outputs as the reference leaves them (zeros / zeroed structs) and
// record the reason in aaedn_last_error(). Compute calls are asynchronous on
// the legacy default stream; transformer_forward synchronises because it
// returns host logits.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "aaedn/arena.hpp"
#include "aaedn/attention.hpp"
#include "aaedn/dequant.hpp"
#include "aaedn/ffn.hpp"
#include "aaedn/fused_matmul.hpp"
#include "aaedn/kvcache.hpp"
#include "aaedn/quant.hpp"
#include "aaedn/rmsnorm.hpp"
#include "aaedn/rope.hpp"
#include "aaedn/transformer.hpp"
#include "aaedn_b200.h"
#include "host_common.hpp"

using aaedn_host::set_error;

namespace aaedn
{

namespace
{
size_t align_up(size_t v, size_t a) { return a ? (v + a - 1) / a * a : v; }
constexpr size_t kHostArenaBytes = 1 << 20; // least host part of an arena
} // namespace

// ---- arena (src/arena.cpp) ------------------------------------------------
Arena arena_create(size_t bytes, size_t align)
{
    Arena a{};
    void* d = nullptr;
    if (bytes && aaedn_dev_alloc(&d, bytes) == AAEDN_OK)
    {
        a.base = static_cast<uint8_t*>(d);
        a.capacity = bytes;
    }
    const size_t hal = align < 64 ? 64 : align;
    // host tables (KV branch and segment tables, tokenizer tables): as large
    // as the device part, at least 1 MB (pages are only touched when used)
    const size_t hbytes = bytes > kHostArenaBytes ? bytes : kHostArenaBytes;
    a.host_base = static_cast<uint8_t*>(std::aligned_alloc(hal, align_up(hbytes, hal)));
    a.host_capacity = a.host_base ? hbytes : 0;
    return a;
}

void* arena_alloc(Arena* a, size_t bytes, size_t align)
{
    if (!a || !a->base || (align & (align - 1)))
    {
        set_error(AAEDN_EINVAL, "arena_alloc: no device arena");
        return nullptr;
    }
    const size_t off = align_up(a->used, align ? align : 1);
    if (off + bytes > a->capacity) // src/arena.cpp:17 asserts here
    {
        set_error(AAEDN_ENOMEM, "arena_alloc: %zu bytes do not fit (%zu of %zu used)", bytes, a->used, a->capacity);
        return nullptr;
    }
    a->used = off + bytes;
    return a->base + off;
}

void* arena_alloc_host(Arena* a, size_t bytes, size_t align)
{
    if (!a || !a->host_base || (align & (align - 1)))
        return nullptr;
    const size_t off = align_up(a->host_used, align ? align : 1);
    if (off + bytes > a->host_capacity)
    {
        set_error(AAEDN_ENOMEM, "arena_alloc_host: %zu bytes do not fit", bytes);
        return nullptr;
    }
    a->host_used = off + bytes;
    return a->host_base + off;
}

void arena_destroy(Arena* a)
{
    if (!a)
        return;
    if (a->base)
        aaedn_dev_free(a->base);
    std::free(a->host_base);
    *a = Arena{};
}

// ---- quant (src/quant.cpp:31-129) ------------------------------------------
QuantBlock quant_load(Arena* arena, const char* path)
{
    QuantBlock q{};
    aaedn_abn_header h{};
    if (aaedn_abn_read_header(path, &h) != AAEDN_OK)
        return q;
    const size_t hd = h.hidden_dim;
    const size_t data_bytes = hd * hd / 2, scale_bytes = hd * hd / 32 * 2;
    std::vector<uint8_t> data(data_bytes);
    std::vector<uint16_t> scales(scale_bytes / 2);
    if (aaedn_abn_read_payload(path, &h, data.data(), scales.data()) != AAEDN_OK)
        return q;
    const size_t used0 = arena ? arena->used : 0;
    auto* d_data = static_cast<uint8_t*>(arena_alloc(arena, data_bytes, 32));
    auto* d_scales = static_cast<uint16_t*>(arena_alloc(arena, scale_bytes, 32));
    if (!d_data || !d_scales || aaedn_memcpy_h2d(d_data, data.data(), data_bytes, nullptr) != AAEDN_OK ||
        aaedn_memcpy_h2d(d_scales, scales.data(), scale_bytes, nullptr) != AAEDN_OK ||
        aaedn_stream_sync(nullptr) != AAEDN_OK)
    {
        if (arena)
            arena->used = used0;
        return q;
    }
    q.data = d_data;
    q.scales = d_scales;
    q.num_blocks = data_bytes / 32; // src/quant.cpp:85 (counts 32-byte groups)
    q.block_size = 32;
    q.type = h.quant_type == static_cast<uint8_t>(QuantType::INT8) ? QuantType::INT8 : QuantType::INT4;
    q.format_version = h.version;
    q.checksum = h.payload_checksum;
    return q;
}

void quant_unload(QuantBlock* q)
{
    if (!q)
        return;
    q->data = nullptr;
    q->scales = nullptr;
    q->num_blocks = 0;
    q->block_size = 0;
    q->format_version = 0;
    q->checksum = 0;
}

// ---- kernels ---------------------------------------------------------------
void dequant_4bit(const uint8_t* data, const uint16_t* scales, float* output, size_t n)
{
    aaedn_cu_dequant_4bit(data, scales, output, n, AAEDN_SCALE_U16INT, nullptr);
}

void fused_matmul_init(Arena*) {}
void fused_matmul_destroy() {}

void fused_matmul(const float* input, const uint8_t* weights, const uint16_t* scales, float* output, size_t M, size_t N,
                  size_t K, size_t lda, size_t ldb, size_t ldc)
{
    aaedn_cu_fused_matmul(input, weights, scales, output, M, N, K, lda, ldb, ldc, AAEDN_SCALE_F16, nullptr);
}

void rmsnorm(const float* input, float* output, const float* weight, size_t n, float eps)
{
    aaedn_cu_rmsnorm(input, output, weight, n, eps, nullptr);
}

RoPETables rope_init(Arena* arena, size_t max_seq_len, size_t head_dim)
{
    RoPETables t{};
    t.max_seq_len = max_seq_len;
    t.head_dim = head_dim;
    const size_t n = max_seq_len * (head_dim / 2);
    std::vector<float> c(n), s(n);
    if (aaedn_rope_table(c.data(), s.data(), max_seq_len, head_dim, 10000.0, 0) != AAEDN_OK)
        return t;
    auto* dc = static_cast<float*>(arena_alloc(arena, n * 4, 32));
    auto* ds = static_cast<float*>(arena_alloc(arena, n * 4, 32));
    if (!dc || !ds || aaedn_memcpy_h2d(dc, c.data(), n * 4, nullptr) != AAEDN_OK ||
        aaedn_memcpy_h2d(ds, s.data(), n * 4, nullptr) != AAEDN_OK || aaedn_stream_sync(nullptr) != AAEDN_OK)
        return t;
    t.cos_table = dc;
    t.sin_table = ds;
    return t;
}

void rope_apply(float* q, float* k, size_t seq_len, size_t head_dim, const RoPETables* tables)
{
    if (!tables || !tables->cos_table || !tables->sin_table) // src/rope.cpp:38-39
        return;
    if (seq_len > tables->max_seq_len)
        seq_len = tables->max_seq_len;
    aaedn_cu_rope_apply(q, k, seq_len, head_dim, tables->cos_table, tables->sin_table, nullptr);
}

void attention(const float* q, const float* k_cache, const float* v_cache, const Segment* segments, size_t num_segments,
               float* output, size_t n_heads, size_t head_dim, float scale)
{
    static_assert(sizeof(Segment) == 8, "Segment is two u32");
    aaedn_cu_attention(q, k_cache, v_cache, reinterpret_cast<const uint32_t*>(segments), num_segments, output,
                       n_heads, head_dim, scale, nullptr);
}

void ffn_swiglu(const float* input, float* output, size_t batch_size, size_t hidden_dim, size_t ffn_dim,
                const QuantBlock* gate_w, const QuantBlock* up_w, const QuantBlock* down_w, const uint16_t* gate_scales,
                const uint16_t* up_scales, const uint16_t* down_scales)
{
    aaedn_cu_ffn_swiglu(input, output, batch_size, hidden_dim, ffn_dim, gate_w ? gate_w->data : nullptr,
                        up_w ? up_w->data : nullptr, down_w ? down_w->data : nullptr, gate_scales, up_scales,
                        down_scales, AAEDN_FFN_REFERENCE, nullptr);
}

// ---- KV cache (src/kvcache.cpp) --------------------------------------------
void kvcache_init(KVCache* kv, Arena* arena, size_t max_tokens, size_t n_layers, size_t n_heads, size_t head_dim,
                  size_t max_agents)
{
    if (!kv)
        return;
    kv->base = nullptr;
    kv->max_tokens = max_tokens;
    kv->n_layers = n_layers;
    kv->n_heads = n_heads;
    kv->head_dim = head_dim;
    kv->stride = n_heads * head_dim * sizeof(float);
    kv->branch_table = nullptr;
    kv->max_branches = 0;
    kv->max_agents = 0;
    kv->fill = nullptr;
    for (size_t i = 0; i < KV_MAX_AGENTS; ++i)
    {
        kv->segment_tables[i] = nullptr;
        kv->segment_counts[i] = 0;
    }
    kv->generation_counter.store(0, std::memory_order_release);
    if (max_agents > KV_MAX_AGENTS)
    {
        set_error(AAEDN_EINVAL, "kvcache_init: at most %zu agents", KV_MAX_AGENTS);
        return;
    }
    const size_t slab = max_tokens * n_layers * kv->stride; // one of K, V
    kv->base = static_cast<uint8_t*>(arena_alloc(arena, 2 * slab, 256));
    kv->max_branches = 256; // src/kvcache.cpp:27
    kv->branch_table = static_cast<BranchNode*>(arena_alloc_host(arena, sizeof(BranchNode) * 256, 32));
    kv->fill = static_cast<uint32_t*>(arena_alloc_host(arena, n_layers * n_heads * sizeof(uint32_t), 32));
    if (!kv->base || !kv->branch_table || !kv->fill)
    {
        kv->base = nullptr;
        return;
    }
    for (size_t i = 0; i < 256; ++i)
    {
        BranchNode& b = kv->branch_table[i];
        b.parent_branch_id = 0;
        b.divergence_token_idx = 0;
        b.branch_length = 0;
        b.valence_hint = 0;
        b.prune_flag.store(0, std::memory_order_relaxed);
    }
    std::memset(kv->fill, 0, n_layers * n_heads * sizeof(uint32_t));
    for (size_t i = 0; i < max_agents; ++i)
    {
        kv->segment_tables[i] =
            static_cast<Segment*>(arena_alloc_host(arena, KV_MAX_SEGMENTS * sizeof(Segment), 32));
        if (!kv->segment_tables[i])
        {
            kv->base = nullptr;
            return;
        }
        kv->segment_counts[i] = 0; // an agent starts with an empty view
    }
    kv->max_agents = max_agents;
}

float* kvcache_layer_k(const KVCache* kv, size_t layer)
{
    if (!kv || !kv->base || layer >= kv->n_layers)
        return nullptr;
    return reinterpret_cast<float*>(kv->base + layer * kv->max_tokens * kv->stride);
}

float* kvcache_layer_v(const KVCache* kv, size_t layer)
{
    if (!kv || !kv->base || layer >= kv->n_layers)
        return nullptr;
    return reinterpret_cast<float*>(kv->base + (kv->n_layers + layer) * kv->max_tokens * kv->stride);
}

void kvcache_append(KVCache* kv, int agent_id, size_t layer, size_t head, const float* k, const float* v)
{
    if (!kv || !kv->base || !k || !v || layer >= kv->n_layers || head >= kv->n_heads || agent_id < 0 ||
        (size_t)agent_id >= kv->max_agents)
    {
        set_error(AAEDN_EINVAL, "kvcache_append: bad arguments");
        return;
    }
    uint32_t& f = kv->fill[layer * kv->n_heads + head];
    if (f >= kv->max_tokens)
    {
        set_error(AAEDN_ESTATE, "kvcache_append: cache full (%zu tokens)", kv->max_tokens);
        return;
    }
    const size_t row = (size_t)f * kv->n_heads + head;
    const size_t bytes = kv->head_dim * sizeof(float);
    if (aaedn_memcpy_d2d(kvcache_layer_k(kv, layer) + row * kv->head_dim, k, bytes, nullptr) != AAEDN_OK ||
        aaedn_memcpy_d2d(kvcache_layer_v(kv, layer) + row * kv->head_dim, v, bytes, nullptr) != AAEDN_OK)
        return;
    if (layer == 0 && head == 0)
    {
        // the agent's view grows by this token
        Segment* seg = kv->segment_tables[agent_id];
        uint32_t& n = kv->segment_counts[agent_id];
        if (n > 0 && seg[n - 1].start_token + seg[n - 1].length == f)
            ++seg[n - 1].length;
        else if (n < KV_MAX_SEGMENTS)
            seg[n++] = Segment{f, 1u};
        else
            set_error(AAEDN_ESTATE, "kvcache_append: agent %d has %zu segments", agent_id, KV_MAX_SEGMENTS);
    }
    ++f;
}

bool kvcache_fork(KVCache* kv, int parent_agent, int child_agent)
{
    if (!kv || parent_agent < 0 || child_agent < 0 || (size_t)parent_agent >= kv->max_agents ||
        (size_t)child_agent >= kv->max_agents || parent_agent == child_agent)
        return false;
    const uint32_t n = kv->segment_counts[parent_agent];
    std::memcpy(kv->segment_tables[child_agent], kv->segment_tables[parent_agent], n * sizeof(Segment));
    kv->segment_counts[child_agent] = n;
    return true;
}

const Segment* kvcache_segments(const KVCache* kv, int agent_id, size_t* count)
{
    if (!kv || agent_id < 0 || (size_t)agent_id >= kv->max_agents)
    {
        if (count)
            *count = 0;
        return nullptr;
    }
    if (count)
        *count = kv->segment_counts[agent_id];
    return kv->segment_tables[agent_id];
}

void kvcache_compact(KVCache* kv, uint16_t pruned_branch)
{
    if (!kv || !kv->branch_table || pruned_branch >= kv->max_branches)
        return;
    kv->branch_table[pruned_branch].prune_flag.store(1, std::memory_order_release); // src/kvcache.cpp:58-59
    kv->generation_counter.fetch_add(1, std::memory_order_release);
}

// ---- transformer (src/transformer.cpp) -------------------------------------
void transformer_init(Transformer* tf, Arena* arena, const char* model_path)
{
    if (!tf)
        return;
    *tf = Transformer{};
    tf->arena = arena;
    // src/transformer.cpp:37-43 unless the file's header gives the shape
    aaedn_model_config c{};
    c.dim = 1024;
    c.n_layers = 24;
    c.n_heads = 16;
    c.n_kv_heads = 16;
    c.head_dim = 64;
    c.ffn_dim = 4096;
    c.vocab = 32768;
    c.max_seq = 16384;
    c.rope_theta = 10000.0f;
    c.eps = 1e-6f;
    aaedn_abn_header h{};
    aaedn_model_config fc{};
    const bool whole = model_path && aaedn_abn_model_read_header(model_path, &h, &fc) == AAEDN_OK;
    if (whole)
    {
        // a whole-model file: its shape and, below, its weights
        fc.max_seq = c.max_seq;
        c = fc;
    }
    else if (model_path && aaedn_abn_read_header(model_path, &h) == AAEDN_OK && h.n_layers && h.n_heads &&
             h.head_dim && h.vocab_size && h.hidden_dim && h.ffn_dim)
    {
        c.dim = h.hidden_dim;
        c.n_layers = h.n_layers;
        c.n_heads = c.n_kv_heads = h.n_heads;
        c.head_dim = h.head_dim;
        c.ffn_dim = h.ffn_dim;
        c.vocab = h.vocab_size;
    }
    aaedn_model* m = nullptr;
    if (aaedn_model_create(&c, &m) != AAEDN_OK)
        return;
    if ((whole ? aaedn_model_load_abn(m, model_path) : aaedn_model_synthesize(m, 1234)) != AAEDN_OK)
    {
        aaedn_model_destroy(m);
        return;
    }
    tf->model = m;
    tf->n_layers = c.n_layers;
    tf->n_heads = c.n_heads;
    tf->head_dim = c.head_dim;
    tf->hidden_dim = c.dim;
    tf->ffn_dim = c.ffn_dim;
    tf->vocab_size = c.vocab;
    tf->max_seq_len = c.max_seq;
}

void transformer_forward(Transformer* tf, const uint32_t* token_ids, size_t seq_len, float* logits)
{
    if (!tf)
        return;
    auto zero = [&]() {
        if (logits)
            std::memset(logits, 0, (size_t)tf->vocab_size * sizeof(float));
    };
    if (seq_len == 0 || !token_ids || !logits || !tf->model) // src/transformer.cpp:130-135
    {
        zero();
        return;
    }
    for (size_t i = 0; i < seq_len; ++i)
        if (token_ids[i] >= tf->vocab_size) // src/transformer.cpp:137-142
        {
            zero();
            return;
        }
    // the reference wraps its position at max_seq_len (src/transformer.cpp:240-242)
    if ((size_t)aaedn_model_pos(tf->model) + seq_len > tf->max_seq_len)
        aaedn_model_reset(tf->model);
    if (aaedn_model_forward(tf->model, token_ids, seq_len, logits) != AAEDN_OK)
        zero();
}

void transformer_destroy(Transformer* tf)
{
    if (!tf)
        return;
    if (tf->model)
        aaedn_model_destroy(tf->model);
    tf->model = nullptr;
}

} // namespace aaedn
