// abn_file.cpp — the .abn v2 model-file reader behind quant_load
// (src/quant.cpp:31-119; the writer is tools/convert_model.py:130-150), and
// the reader of whole-model files (at the end of this file).
//
// The header is read field by field, little-endian, in the order of the
// format string "<8sIQI6IB15s" (64 bytes). The checks are the reference's:
// magic "AAEDNMDL", version 2, payload_size == hidden^2/2 + hidden^2/16 (one
// hidden x hidden block-quantized matrix: codes, then u16 scales), and the
// FNV-1a 32 checksum of codes followed by scales.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include "aaedn_b200.h"
#include "host_common.hpp"

using aaedn_host::set_error;

namespace
{

constexpr uint32_t kAbnVersion = 2; // src/quant.cpp:10

struct File
{
    FILE* f = nullptr;
    explicit File(const char* path) : f(path ? std::fopen(path, "rb") : nullptr) {}
    ~File()
    {
        if (f)
            std::fclose(f);
    }
    bool read(void* dst, size_t n) { return std::fread(dst, 1, n, f) == n; }
};

uint32_t le32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
uint64_t le64(const uint8_t* p) { return (uint64_t)le32(p) | (uint64_t)le32(p + 4) << 32; }

// The 64 header bytes, unchecked beyond the magic; raw keeps them (the full
// model format keeps more fields in the reserved bytes).
int parse_raw(File& file, aaedn_abn_header* h, uint8_t* raw)
{
    if (!file.read(raw, 64))
        return set_error(AAEDN_EFORMAT, "abn: header shorter than 64 bytes");
    if (std::memcmp(raw, "AAEDNMDL", 8) != 0)
        return set_error(AAEDN_EFORMAT, "abn: bad magic");
    h->version = le32(raw + 8);
    h->payload_size = le64(raw + 12);
    h->payload_checksum = le32(raw + 20);
    h->n_layers = le32(raw + 24);
    h->n_heads = le32(raw + 28);
    h->head_dim = le32(raw + 32);
    h->vocab_size = le32(raw + 36);
    h->hidden_dim = le32(raw + 40);
    h->ffn_dim = le32(raw + 44);
    h->quant_type = raw[48];
    return AAEDN_OK;
}

int parse(File& file, aaedn_abn_header* h)
{
    uint8_t raw[64];
    if (int rc = parse_raw(file, h, raw))
        return rc;
    if (h->version != kAbnVersion)
        return set_error(AAEDN_EFORMAT, "abn: version %u (want %u)", h->version, kAbnVersion);
    const uint64_t hd = h->hidden_dim;
    const uint64_t expect = hd * hd / 2 + hd * hd / 32 * 2;
    if (h->payload_size != expect)
        return set_error(AAEDN_EFORMAT, "abn: payload_size %llu, a %u x %u matrix needs %llu",
                         (unsigned long long)h->payload_size, h->hidden_dim, h->hidden_dim,
                         (unsigned long long)expect);
    return AAEDN_OK;
}

} // namespace

extern "C" int aaedn_abn_read_header(const char* path, aaedn_abn_header* h_out)
{
    if (!path || !h_out)
        return set_error(AAEDN_EINVAL, "aaedn_abn_read_header: null argument");
    std::memset(h_out, 0, sizeof *h_out);
    File file(path);
    if (!file.f)
        return set_error(AAEDN_EFORMAT, "abn: cannot open %s", path);
    return parse(file, h_out);
}

extern "C" int aaedn_abn_read_payload(const char* path, const aaedn_abn_header* h_hdr, uint8_t* h_data,
                                      uint16_t* h_scales)
{
    if (!path || !h_hdr || !h_data || !h_scales)
        return set_error(AAEDN_EINVAL, "aaedn_abn_read_payload: null argument");
    File file(path);
    if (!file.f)
        return set_error(AAEDN_EFORMAT, "abn: cannot open %s", path);
    aaedn_abn_header h{};
    int rc = parse(file, &h);
    if (rc)
        return rc;
    if (h.payload_size != h_hdr->payload_size || h.payload_checksum != h_hdr->payload_checksum)
        return set_error(AAEDN_EFORMAT, "abn: header changed since it was read");
    const size_t hd = h.hidden_dim;
    const size_t data_bytes = hd * hd / 2, scale_bytes = hd * hd / 32 * 2;
    if (!file.read(h_data, data_bytes) || !file.read(h_scales, scale_bytes))
        return set_error(AAEDN_EFORMAT, "abn: payload shorter than %zu bytes", data_bytes + scale_bytes);
    uint32_t c = aaedn_fnv1a32(h_data, data_bytes, 0x811C9DC5u);
    c = aaedn_fnv1a32(reinterpret_cast<const uint8_t*>(h_scales), scale_bytes, c);
    if (c != h.payload_checksum)
        return set_error(AAEDN_EFORMAT, "abn: checksum %08x, header says %08x", c, h.payload_checksum);
    return AAEDN_OK;
}

// ---------------------------------------------------------------------------
// Full-model files: the layout of docs/mpd.md:497-499 (per layer, in order:
// RMSNorm scale, QKV weight, QKV bias, O weight, FFN gate, FFN up, FFN down,
// RMSNorm 2 scale; a weight is its row-major 4-bit codes, then its u16
// scales), which the reference's converter does not write yet
// (tools/convert_model.py:121-126 writes one matrix). Stored as version 3
// with what the documented header lacks in its reserved bytes, and the
// model's remaining tensors after the layers.
namespace
{

constexpr uint32_t kAbnModelVersion = 3;

struct ModelDims
{
    uint64_t D, qkv, qdim, F, V;
};

ModelDims dims_of(const aaedn_model_config& c)
{
    return {c.dim, (uint64_t)(c.n_heads + 2 * c.n_kv_heads) * c.head_dim, (uint64_t)c.n_heads * c.head_dim,
            c.ffn_dim, c.vocab};
}

uint64_t q4_bytes(uint64_t rows, uint64_t cols) { return rows * cols / 2 + rows * cols / 32 * 2; }

uint64_t layer_bytes(const ModelDims& d)
{
    return d.D * 4 + q4_bytes(d.qkv, d.D) + d.qkv * 4 + q4_bytes(d.D, d.qdim) + 2 * q4_bytes(d.F, d.D) +
           q4_bytes(d.D, d.F) + d.D * 4;
}

uint64_t model_payload_bytes(const aaedn_model_config& c)
{
    const ModelDims d = dims_of(c);
    return (uint64_t)c.n_layers * layer_bytes(d) + d.D * 4 + 2 * d.V * d.D * 4;
}

float lef32(const uint8_t* p)
{
    const uint32_t u = le32(p);
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

int parse_model(File& file, aaedn_abn_header* h, aaedn_model_config* c)
{
    uint8_t raw[64];
    if (int rc = parse_raw(file, h, raw))
        return rc;
    if (h->version != kAbnModelVersion)
        return set_error(AAEDN_EFORMAT, "abn: version %u is not a full-model file (%u)", h->version,
                         kAbnModelVersion);
    if (h->quant_type != 0)
        return set_error(AAEDN_EUNSUPPORTED, "abn: quant_type %u (only 0, 4-bit blocks)", h->quant_type);
    *c = aaedn_model_config{};
    c->dim = h->hidden_dim;
    c->n_layers = h->n_layers;
    c->n_heads = h->n_heads;
    c->n_kv_heads = le32(raw + 49);
    c->head_dim = h->head_dim;
    c->ffn_dim = h->ffn_dim;
    c->vocab = h->vocab_size;
    c->rope_theta = lef32(raw + 53);
    c->eps = lef32(raw + 57);
    if (!c->dim || !c->n_layers || !c->n_heads || !c->n_kv_heads || !c->head_dim || !c->ffn_dim || !c->vocab ||
        c->n_heads % c->n_kv_heads || c->dim % 32 || c->ffn_dim % 32 || (c->n_heads * c->head_dim) % 32 ||
        !(c->rope_theta > 0.0f) || !(c->eps > 0.0f))
        return set_error(AAEDN_EFORMAT, "abn: model dimensions in the header do not describe a model");
    if (h->payload_size != model_payload_bytes(*c))
        return set_error(AAEDN_EFORMAT, "abn: payload_size %llu, the header's dimensions need %llu",
                         (unsigned long long)h->payload_size, (unsigned long long)model_payload_bytes(*c));
    return AAEDN_OK;
}

} // namespace

extern "C" int aaedn_abn_model_read_header(const char* path, aaedn_abn_header* h_out, aaedn_model_config* cfg_out)
{
    if (!path || !h_out || !cfg_out)
        return set_error(AAEDN_EINVAL, "aaedn_abn_model_read_header: null argument");
    std::memset(h_out, 0, sizeof *h_out);
    File file(path);
    if (!file.f)
        return set_error(AAEDN_EFORMAT, "abn: cannot open %s", path);
    return parse_model(file, h_out, cfg_out);
}

extern "C" int aaedn_model_load_abn(aaedn_model* m, const char* path)
{
    if (!m || !path)
        return set_error(AAEDN_EINVAL, "aaedn_model_load_abn: null argument");
    aaedn_model_config mc{}, fc{};
    if (int rc = aaedn_model_config_get(m, &mc))
        return rc;
    aaedn_abn_header h{};
    // one open handle for both passes
    File file(path);
    if (!file.f)
        return set_error(AAEDN_EFORMAT, "abn: cannot open %s", path);
    {
        if (int rc = parse_model(file, &h, &fc))
            return rc;
        if (fc.dim != mc.dim || fc.n_layers != mc.n_layers || fc.n_heads != mc.n_heads ||
            fc.n_kv_heads != mc.n_kv_heads || fc.head_dim != mc.head_dim || fc.ffn_dim != mc.ffn_dim ||
            fc.vocab != mc.vocab)
            return set_error(AAEDN_EINVAL, "aaedn_model_load_abn: the file's model shape differs from the model's");
        // pass 1: the checksum, before any weight reaches the model
        std::vector<uint8_t> buf(64u << 20);
        uint32_t c = 0x811C9DC5u;
        for (uint64_t left = h.payload_size; left > 0;)
        {
            const size_t n = (size_t)std::min<uint64_t>(left, buf.size());
            if (!file.read(buf.data(), n))
                return set_error(AAEDN_EFORMAT, "abn: payload shorter than %llu bytes",
                                 (unsigned long long)h.payload_size);
            c = aaedn_fnv1a32(buf.data(), n, c);
            left -= n;
        }
        if (c != h.payload_checksum)
            return set_error(AAEDN_EFORMAT, "abn: checksum %08x, header says %08x", c, h.payload_checksum);
    }
    // pass 2: layer by layer into the model, from the same handle rewound to
    // the payload; the checksum is taken again over the bytes this pass
    // reads, and a file that changed between the passes is refused before
    // the embedding and lm_head are set (the layers already set then hold a
    // mix: reload the model)
    if (std::fseek(file.f, 64, SEEK_SET) != 0)
        return set_error(AAEDN_EFORMAT, "abn: cannot rewind %s", path);
    const ModelDims d = dims_of(fc);
    const uint64_t qrows = d.qdim, krows = (uint64_t)fc.n_kv_heads * fc.head_dim;
    std::vector<float> an(d.D), fn(d.D), bias(d.qkv);
    std::vector<uint8_t> qkv_c(d.qkv * d.D / 2), o_c(d.D * d.qdim / 2), g_c(d.F * d.D / 2), u_c(d.F * d.D / 2),
        d_c(d.D * d.F / 2);
    std::vector<uint16_t> qkv_s(d.qkv * d.D / 32), o_s(d.D * d.qdim / 32), g_s(d.F * d.D / 32), u_s(d.F * d.D / 32),
        d_s(d.D * d.F / 32);
    uint32_t c2 = 0x811C9DC5u;
    auto rd = [&](void* dst, size_t n) {
        if (!file.read(dst, n))
            return false;
        c2 = aaedn_fnv1a32(static_cast<const uint8_t*>(dst), n, c2);
        return true;
    };
    for (uint32_t l = 0; l < fc.n_layers; ++l)
    {
        const bool ok = rd(an.data(), d.D * 4) && rd(qkv_c.data(), qkv_c.size()) && rd(qkv_s.data(), qkv_s.size() * 2) &&
                        rd(bias.data(), d.qkv * 4) && rd(o_c.data(), o_c.size()) && rd(o_s.data(), o_s.size() * 2) &&
                        rd(g_c.data(), g_c.size()) && rd(g_s.data(), g_s.size() * 2) && rd(u_c.data(), u_c.size()) &&
                        rd(u_s.data(), u_s.size() * 2) && rd(d_c.data(), d_c.size()) &&
                        rd(d_s.data(), d_s.size() * 2) && rd(fn.data(), d.D * 4);
        if (!ok)
            return set_error(AAEDN_EFORMAT, "abn: layer %u cut short", l);
        for (float b : bias)
            if (b != 0.0f) // decision D8: the model has no bias (src/transformer.cpp:112-117 zeroes it)
                return set_error(AAEDN_EUNSUPPORTED, "abn: layer %u has a nonzero QKV bias", l);
        // QKV rows are q, then k, then v: each matrix is a contiguous run of
        // the codes and of the scales
        aaedn_layer_host w{};
        w.wq = qkv_c.data();
        w.wk = qkv_c.data() + qrows * d.D / 2;
        w.wv = qkv_c.data() + (qrows + krows) * d.D / 2;
        w.sq = qkv_s.data();
        w.sk = qkv_s.data() + qrows * d.D / 32;
        w.sv = qkv_s.data() + (qrows + krows) * d.D / 32;
        w.wo = o_c.data();
        w.so = o_s.data();
        w.wg = g_c.data();
        w.sg = g_s.data();
        w.wu = u_c.data();
        w.su = u_s.data();
        w.wd = d_c.data();
        w.sd = d_s.data();
        w.attn_norm = an.data();
        w.ffn_norm = fn.data();
        if (int rc = aaedn_model_set_layer(m, l, &w))
            return rc;
    }
    std::vector<float> final_norm(d.D), emb(d.V * d.D), lm(d.V * d.D);
    if (!rd(final_norm.data(), d.D * 4) || !rd(emb.data(), emb.size() * 4) || !rd(lm.data(), lm.size() * 4))
        return set_error(AAEDN_EFORMAT, "abn: embedding or lm_head cut short");
    if (c2 != h.payload_checksum)
        return set_error(AAEDN_EFORMAT, "abn: %s changed while it was read (checksum %08x, header says %08x)", path,
                         c2, h.payload_checksum);
    return aaedn_model_set_globals(m, emb.data(), final_norm.data(), lm.data());
}

// ---------------------------------------------------------------------------
// Writer of whole-model files (the layout aaedn_model_load_abn reads): the
// header is written last, once the payload's FNV-1a checksum is known.
namespace
{

struct WFile
{
    FILE* f = nullptr;
    uint32_t hash = 0x811C9DC5u;
    uint64_t bytes = 0;
    explicit WFile(const char* path) : f(path ? std::fopen(path, "wb") : nullptr) {}
    ~WFile()
    {
        if (f)
            std::fclose(f);
    }
    bool put(const void* p, size_t n)
    {
        if (!n)
            return true;
        if (std::fwrite(p, 1, n, f) != n)
            return false;
        hash = aaedn_fnv1a32(static_cast<const uint8_t*>(p), n, hash);
        bytes += n;
        return true;
    }
    bool zeros(size_t n)
    {
        static const uint8_t z[4096] = {};
        for (size_t left = n; left > 0;)
        {
            const size_t k = std::min(left, sizeof z);
            if (!put(z, k))
                return false;
            left -= k;
        }
        return true;
    }
};

void le32w(uint8_t* p, uint32_t v)
{
    for (int i = 0; i < 4; ++i)
        p[i] = (uint8_t)(v >> (8 * i));
}

} // namespace

extern "C" int aaedn_abn_model_write(const char* path, const aaedn_model_config* cfg, const aaedn_layer_host* layers,
                                     const float* h_embedding, const float* h_final_norm, const float* h_lm_head)
{
    if (!path || !cfg || !layers || !h_embedding || !h_lm_head)
        return set_error(AAEDN_EINVAL, "aaedn_abn_model_write: null argument");
    const aaedn_model_config& c = *cfg;
    if (!c.dim || !c.n_layers || !c.n_heads || !c.n_kv_heads || !c.head_dim || !c.ffn_dim || !c.vocab ||
        c.n_heads % c.n_kv_heads || c.dim % 32 || c.ffn_dim % 32 || (c.n_heads * c.head_dim) % 32 ||
        !(c.rope_theta > 0.0f) || !(c.eps > 0.0f))
        return set_error(AAEDN_EINVAL, "aaedn_abn_model_write: the config does not describe a model");
    const ModelDims d = dims_of(c);
    const uint64_t qrows = d.qdim, krows = (uint64_t)c.n_kv_heads * c.head_dim;
    WFile file(path);
    if (!file.f)
        return set_error(AAEDN_EFORMAT, "abn: cannot create %s", path);
    uint8_t hdr[64] = {};
    if (std::fwrite(hdr, 1, 64, file.f) != 64) // placeholder, rewritten at the end
        return set_error(AAEDN_EFORMAT, "abn: write to %s failed", path);
    std::vector<float> ones(d.D, 1.0f);
    bool ok = true;
    for (uint32_t l = 0; l < c.n_layers && ok; ++l)
    {
        const aaedn_layer_host& w = layers[l];
        if (!w.wq || !w.wk || !w.wv || !w.wo || !w.wg || !w.wu || !w.wd || !w.sq || !w.sk || !w.sv || !w.so ||
            !w.sg || !w.su || !w.sd)
            return set_error(AAEDN_EINVAL, "aaedn_abn_model_write: layer %u has a null tensor", l);
        const float* an = w.attn_norm ? w.attn_norm : ones.data();
        const float* fn = w.ffn_norm ? w.ffn_norm : ones.data();
        // RMSNorm | QKV codes (q, k, v rows) | QKV scales | QKV bias (zero) |
        // O | gate | up | down (codes, then scales) | RMSNorm 2
        ok = file.put(an, d.D * 4) && file.put(w.wq, qrows * d.D / 2) && file.put(w.wk, krows * d.D / 2) &&
             file.put(w.wv, krows * d.D / 2) && file.put(w.sq, qrows * d.D / 32 * 2) &&
             file.put(w.sk, krows * d.D / 32 * 2) && file.put(w.sv, krows * d.D / 32 * 2) &&
             file.zeros(d.qkv * 4) && file.put(w.wo, d.D * d.qdim / 2) && file.put(w.so, d.D * d.qdim / 32 * 2) &&
             file.put(w.wg, d.F * d.D / 2) && file.put(w.sg, d.F * d.D / 32 * 2) && file.put(w.wu, d.F * d.D / 2) &&
             file.put(w.su, d.F * d.D / 32 * 2) && file.put(w.wd, d.D * d.F / 2) &&
             file.put(w.sd, d.D * d.F / 32 * 2) && file.put(fn, d.D * 4);
    }
    ok = ok && file.put(h_final_norm ? h_final_norm : ones.data(), d.D * 4) && file.put(h_embedding, d.V * d.D * 4) &&
         file.put(h_lm_head, d.V * d.D * 4);
    if (!ok)
        return set_error(AAEDN_EFORMAT, "abn: write to %s failed", path);
    if (file.bytes != model_payload_bytes(c))
        return set_error(AAEDN_EFORMAT, "abn: wrote %llu payload bytes, the layout has %llu",
                         (unsigned long long)file.bytes, (unsigned long long)model_payload_bytes(c));
    // "<8sIQI6IB15s": magic, version 3, payload size, checksum, the six dims,
    // quant_type 0; reserved bytes: n_kv_heads, rope_theta, eps
    std::memcpy(hdr, "AAEDNMDL", 8);
    le32w(hdr + 8, kAbnModelVersion);
    le32w(hdr + 12, (uint32_t)file.bytes);
    le32w(hdr + 16, (uint32_t)(file.bytes >> 32));
    le32w(hdr + 20, file.hash);
    const uint32_t dims6[6] = {c.n_layers, c.n_heads, c.head_dim, c.vocab, c.dim, c.ffn_dim};
    for (int i = 0; i < 6; ++i)
        le32w(hdr + 24 + 4 * i, dims6[i]);
    hdr[48] = 0;
    le32w(hdr + 49, c.n_kv_heads);
    uint32_t tb, eb;
    std::memcpy(&tb, &c.rope_theta, 4);
    std::memcpy(&eb, &c.eps, 4);
    le32w(hdr + 53, tb);
    le32w(hdr + 57, eb);
    if (std::fseek(file.f, 0, SEEK_SET) != 0 || std::fwrite(hdr, 1, 64, file.f) != 64 || std::fflush(file.f) != 0)
        return set_error(AAEDN_EFORMAT, "abn: header write to %s failed", path);
    return AAEDN_OK;
}
