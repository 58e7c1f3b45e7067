// The reference's tests/test_startup_failure.cpp checks, against this
// library's C++ API: quant_load rejects a file with a bad magic and one with
// a bad checksum, returning a zeroed block. Added: a short header, a short
// payload, a wrong version and a wrong payload size are rejected; a valid
// file's header and payload are accepted by the reader (the upload itself
// needs a GPU and is covered by test_api_gpu). Runs without a GPU.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "aaedn/arena.hpp"
#include "aaedn/quant.hpp"
#include "aaedn_b200.h"
#include "abn_writer.hpp"

static int fails = 0;
#define CHECK(cond)                                                                                                   \
    do                                                                                                                \
    {                                                                                                                 \
        if (!(cond))                                                                                                  \
        {                                                                                                             \
            std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #cond);                                                \
            ++fails;                                                                                                  \
        }                                                                                                             \
    } while (0)

static bool zeroed(const aaedn::QuantBlock& q) { return !q.data && !q.scales && q.num_blocks == 0; }

int main(int argc, char** argv)
{
    const std::string dir = argc > 1 ? argv[1] : "/tmp";
    using namespace abn_test;
    Dims d;
    const std::string bad_magic = dir + "/fail_magic.abn", bad_sum = dir + "/fail_checksum.abn",
                      short_hdr = dir + "/fail_short.abn", bad_ver = dir + "/fail_version.abn",
                      bad_size = dir + "/fail_size.abn", short_pay = dir + "/fail_payload.abn",
                      bad_payload_sum = dir + "/fail_payload_checksum.abn", good = dir + "/good.abn";
    write_file(bad_magic, std::vector<uint8_t>(64, 0xAA)); // the reference test's invalid_magic_file
    {
        // the reference test's bad_checksum_model: 10-byte payload, checksum 0xDEADBEEF
        Dims r;
        r.n_layers = 24, r.n_heads = 16, r.head_dim = 64, r.vocab = 32768, r.hidden = 4, r.ffn = 16;
        auto f = header(2, 10, 0xDEADBEEF, r);
        f.insert(f.end(), 10, 0x11);
        write_file(bad_sum, f);
    }
    write_file(short_hdr, std::vector<uint8_t>{'A', 'A', 'E', 'D', 'N', 'M', 'D', 'L', 2, 0});
    {
        auto f = valid_model(d);
        f[8] = 3; // version 3
        write_file(bad_ver, f);
        auto g = valid_model(d);
        g[12] ^= 1; // payload size
        write_file(bad_size, g);
        auto s = valid_model(d);
        s.resize(s.size() - 5);
        write_file(short_pay, s);
        write_file(good, valid_model(d));
        auto c = valid_model(d);
        c[64 + 7] ^= 0x10; // one payload bit: the checksum no longer matches
        write_file(bad_payload_sum, c);
    }

    aaedn::Arena arena = aaedn::arena_create(8 * 1024 * 1024, 64);
    for (const std::string& p : {bad_magic, bad_sum, short_hdr, bad_ver, bad_size, short_pay, bad_payload_sum})
    {
        aaedn::QuantBlock q = aaedn::quant_load(&arena, p.c_str());
        CHECK(zeroed(q));
    }
    aaedn::QuantBlock none = aaedn::quant_load(&arena, (dir + "/missing.abn").c_str());
    CHECK(zeroed(none));

    // the reader's decisions and error codes
    aaedn_abn_header h{};
    CHECK(aaedn_abn_read_header(bad_magic.c_str(), &h) == AAEDN_EFORMAT);
    CHECK(std::strstr(aaedn_last_error(), "magic") != nullptr);
    CHECK(aaedn_abn_read_header(bad_ver.c_str(), &h) == AAEDN_EFORMAT);
    CHECK(aaedn_abn_read_header(bad_size.c_str(), &h) == AAEDN_EFORMAT);
    CHECK(aaedn_abn_read_header(short_hdr.c_str(), &h) == AAEDN_EFORMAT);
    CHECK(aaedn_abn_read_header(good.c_str(), &h) == AAEDN_OK);
    CHECK(h.version == 2 && h.hidden_dim == d.hidden && h.n_layers == d.n_layers && h.vocab_size == d.vocab);
    std::vector<uint8_t> codes(d.hidden * d.hidden / 2), want_codes;
    std::vector<uint16_t> scales(d.hidden * d.hidden / 32), want_scales;
    valid_model(d, &want_codes, &want_scales);
    CHECK(aaedn_abn_read_payload(good.c_str(), &h, codes.data(), scales.data()) == AAEDN_OK);
    CHECK(codes == want_codes && scales == want_scales);
    aaedn_abn_header hs{};
    CHECK(aaedn_abn_read_header(short_pay.c_str(), &hs) == AAEDN_OK); // header intact
    CHECK(aaedn_abn_read_payload(short_pay.c_str(), &hs, codes.data(), scales.data()) == AAEDN_EFORMAT);
    aaedn_abn_header hp{};
    CHECK(aaedn_abn_read_header(bad_payload_sum.c_str(), &hp) == AAEDN_OK);
    CHECK(aaedn_abn_read_payload(bad_payload_sum.c_str(), &hp, codes.data(), scales.data()) == AAEDN_EFORMAT);
    CHECK(std::strstr(aaedn_last_error(), "checksum") != nullptr);
    aaedn_abn_header hc{};
    CHECK(aaedn_abn_read_header(bad_sum.c_str(), &hc) == AAEDN_EFORMAT); // 10 bytes is no 4x4 payload

    // quant_unload zeroes (src/quant.cpp:121-129)
    aaedn::QuantBlock q{};
    q.num_blocks = 3;
    q.block_size = 32;
    aaedn::quant_unload(&q);
    CHECK(zeroed(q) && q.block_size == 0);

    aaedn::arena_destroy(&arena);
    std::printf("%s\n", fails ? "FAILED" : "PASSED");
    return fails ? 1 : 0;
}
