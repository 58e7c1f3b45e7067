// kvcache.hpp — mirror of the reference include/kvcache.hpp, with the
// branch-aware view made real.
//
// K and V live in the arena (device): per layer, token-major rows of
// n_heads * head_dim floats, so a layer's slab (kvcache_layer_k/_v) is
// exactly what attention() reads. Tokens are handed out by one fill counter
// per (layer, head): kvcache_append writes the next free row (the reference
// always writes row 0, src/kvcache.cpp:43). Each agent (branch) sees the
// cache through its Segment table (host memory): appending for agent a at
// layer 0, head 0 extends a's last segment or opens a new one, and
// kvcache_fork gives a child branch its parent's segments, so a shared
// prefix is stored once and read through both views. The branch table and
// kvcache_compact keep the reference's bookkeeping (prune flag, generation
// counter, src/kvcache.cpp:56-60).
#ifndef AAEDN_B200_KVCACHE_HPP
#define AAEDN_B200_KVCACHE_HPP

#include <atomic>
#include <cstddef>
#include <cstdint>

namespace aaedn
{

struct Arena;

struct BranchNode
{
    uint16_t parent_branch_id;
    uint16_t divergence_token_idx;
    uint16_t branch_length;
    uint8_t valence_hint;
    std::atomic<uint8_t> prune_flag;
};

struct Segment
{
    uint32_t start_token;
    uint32_t length;
};

constexpr size_t KV_MAX_AGENTS = 6;    // segment_tables[6] of the reference
constexpr size_t KV_MAX_SEGMENTS = 32; // per agent (src/kvcache.cpp:33)

struct KVCache
{
    uint8_t* base; // device: K slab then V slab
    size_t max_tokens;
    size_t n_layers;
    size_t n_heads;
    size_t head_dim;
    size_t stride; // bytes of one token row of one layer (n_heads * head_dim * 4)

    BranchNode* branch_table; // host
    size_t max_branches;

    Segment* segment_tables[KV_MAX_AGENTS]; // host, KV_MAX_SEGMENTS each
    size_t max_agents;

    std::atomic<uint32_t> generation_counter;

    // B200 additions
    uint32_t* fill;                              // host [n_layers][n_heads]: rows in use
    uint32_t segment_counts[KV_MAX_AGENTS];      // segments in use per agent
};

void kvcache_init(KVCache* kv, Arena* arena, size_t max_tokens, size_t n_layers, size_t n_heads, size_t head_dim,
                  size_t max_agents);
void kvcache_append(KVCache* kv, int agent_id, size_t layer, size_t head, const float* k, const float* v);
void kvcache_compact(KVCache* kv, uint16_t pruned_branch);

// B200 additions
float* kvcache_layer_k(const KVCache* kv, size_t layer); // device [max_tokens][n_heads][head_dim]
float* kvcache_layer_v(const KVCache* kv, size_t layer);
// child sees parent's tokens (no copy); returns false if an id is out of range
bool kvcache_fork(KVCache* kv, int parent_agent, int child_agent);
// the agent's segments (host) and their count
const Segment* kvcache_segments(const KVCache* kv, int agent_id, size_t* count);

} // namespace aaedn

#endif
