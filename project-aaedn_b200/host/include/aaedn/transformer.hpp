// transformer.hpp — mirror of the reference include/transformer.hpp.
//
// transformer_init builds a device-resident model from the file at
// model_path: a whole-model .abn file (aaedn_abn_model_read_header) gives the
// shape and every weight; otherwise the shape comes from an .abn v2 header
// (src/quant.cpp's checks; the reference's hard-coded shape,
// src/transformer.cpp:37-43, when the file is missing or rejected) and the
// weights are seeded N(0, 0.02) values quantized with the reference
// quantizer (the reference fills its weights with rand() and constants,
// src/transformer.cpp:54-121; real weights also go in through
// aaedn_model_set_layer). The context is 16384 tokens. transformer_forward runs the token loop on
// the B200 for all seq_len tokens at the model's current position and copies
// the last token's logits to the HOST array `logits` (vocab_size floats).
// kv_cache and rope_tables stay null: the model keeps its paged cache and
// tables in its own arena.
#ifndef AAEDN_B200_TRANSFORMER_HPP
#define AAEDN_B200_TRANSFORMER_HPP

#include <cstddef>
#include <cstdint>

struct aaedn_model;

namespace aaedn
{

struct Arena;
struct KVCache;
struct RoPETables;
struct QuantBlock;

struct Transformer
{
    Arena* arena;
    KVCache* kv_cache;
    RoPETables* rope_tables;

    QuantBlock* qkv_weight;
    QuantBlock* out_proj_weight;
    QuantBlock* ffn_gate_weight;
    QuantBlock* ffn_up_weight;
    QuantBlock* ffn_down_weight;

    float* qkv_bias;
    float* out_proj_bias;
    float* ffn_bias;

    float* input_embedding;
    float* lm_head;

    uint32_t n_layers;
    uint32_t n_heads;
    uint32_t head_dim;
    uint32_t hidden_dim;
    uint32_t ffn_dim;
    uint32_t vocab_size;
    uint32_t max_seq_len;

    aaedn_model* model; // B200: the device model behind this transformer
};

void transformer_init(Transformer* tf, Arena* arena, const char* model_path);
void transformer_forward(Transformer* tf, const uint32_t* token_ids, size_t seq_len, float* logits);
// B200 addition: releases the device model
void transformer_destroy(Transformer* tf);

} // namespace aaedn

#endif
