// abn_file.cpp — the .abn v2 model-file reader behind quant_load
// (src/quant.cpp:31-119; the writer is tools/convert_model.py:130-150).
//
// The header is read field by field, little-endian, in the order of the
// format string "<8sIQI6IB15s" (64 bytes). The checks are the reference's:
// magic "AAEDNMDL", version 2, payload_size == hidden^2/2 + hidden^2/16 (one
// hidden x hidden block-quantized matrix: codes, then u16 scales), and the
// FNV-1a 32 checksum of codes followed by scales.
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

int parse(File& file, aaedn_abn_header* h)
{
    uint8_t raw[64];
    if (!file.read(raw, sizeof raw))
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
