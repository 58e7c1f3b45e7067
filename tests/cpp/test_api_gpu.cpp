// The reference's C++ API (namespace aaedn) on a B200, end to end: arena,
// quant_load upload, dequant_4bit, fused_matmul, rmsnorm, rope_init/apply,
// attention, ffn_swiglu, the branch-aware KV cache and transformer_forward.
// Expected values are computed here on the host with plain loops that follow
// the reference sources (cited per check); fp32 results are compared with a
// relative bound, integer/bit work exactly.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
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
#include "abn_writer.hpp"

static int fails = 0;
#define CHECK(cond)                                                                                                   \
    do                                                                                                                \
    {                                                                                                                 \
        if (!(cond))                                                                                                  \
        {                                                                                                             \
            std::printf("FAIL %s:%d %s (%s)\n", __FILE__, __LINE__, #cond, aaedn_last_error());                       \
            ++fails;                                                                                                  \
        }                                                                                                             \
    } while (0)

namespace
{
uint64_t rng = 88172645463325252ull;
float frand() // xorshift, uniform [-1, 1)
{
    rng ^= rng << 13;
    rng ^= rng >> 7;
    rng ^= rng << 17;
    return (float)((rng >> 40) & 0xFFFFFF) / 8388608.0f - 1.0f;
}
template <class T> T* up(aaedn::Arena* a, const std::vector<T>& h)
{
    T* d = static_cast<T*>(aaedn::arena_alloc(a, h.size() * sizeof(T), 256));
    aaedn_memcpy_h2d(d, h.data(), h.size() * sizeof(T), nullptr);
    return d;
}
template <class T> std::vector<T> down(const T* d, size_t n)
{
    std::vector<T> h(n);
    aaedn_memcpy_d2h(h.data(), d, n * sizeof(T), nullptr);
    aaedn_stream_sync(nullptr);
    return h;
}
float* dev_f(aaedn::Arena* a, size_t n) { return static_cast<float*>(aaedn::arena_alloc(a, n * 4, 256)); }
bool close(const std::vector<float>& got, const std::vector<float>& want, const std::vector<float>& mag, float rel)
{
    for (size_t i = 0; i < got.size(); ++i)
        if (!(std::fabs(got[i] - want[i]) <= rel * mag[i] + 1e-6f))
        {
            std::printf("  mismatch at %zu: %g vs %g (mag %g)\n", i, got[i], want[i], mag[i]);
            return false;
        }
    return true;
}
float half_to_float(uint16_t h)
{
    const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
    float v = e == 0 ? std::ldexp((float)m, -24) : std::ldexp((float)(m | 1024), (int)e - 25);
    return s ? -v : v;
}
} // namespace

int main(int argc, char** argv)
{
    const std::string dir = argc > 1 ? argv[1] : "/tmp";
    aaedn::Arena arena = aaedn::arena_create(512ull << 20, 64);
    CHECK(arena.base != nullptr);

    // ---- quant_load: a valid file lands on the device unchanged
    abn_test::Dims d;
    std::vector<uint8_t> codes;
    std::vector<uint16_t> scales;
    abn_test::write_file(dir + "/good.abn", abn_test::valid_model(d, &codes, &scales));
    aaedn::QuantBlock q = aaedn::quant_load(&arena, (dir + "/good.abn").c_str());
    CHECK(q.data && q.scales && q.format_version == 2 && q.block_size == 32);
    CHECK(q.num_blocks == codes.size() / 32); // src/quant.cpp:85
    CHECK(down(q.data, codes.size()) == codes && down(q.scales, scales.size()) == scales);

    // ---- dequant_4bit: src/dequant.cpp:16-27, integer scale cast, bit-exact
    {
        const size_t n = codes.size() * 2;
        float* out = dev_f(&arena, n);
        aaedn::dequant_4bit(q.data, q.scales, out, n);
        auto got = down(out, n);
        bool ok = true;
        for (size_t i = 0; i < n && ok; ++i)
        {
            const int c = (codes[i / 2] >> ((i & 1) * 4)) & 15;
            const float want = (float)c * (float)scales[i / 32];
            ok = std::memcmp(&want, &got[i], 4) == 0;
        }
        CHECK(ok);
    }

    // ---- fused_matmul: out = x W^T with fp16 block scales (model semantics)
    {
        const size_t M = 3, N = d.hidden, K = d.hidden;
        std::vector<float> x(M * K);
        for (auto& v : x)
            v = frand();
        float* dx = up(&arena, x);
        float* dy = dev_f(&arena, M * N);
        aaedn::fused_matmul_init(&arena);
        aaedn::fused_matmul(dx, q.data, q.scales, dy, M, N, K, K, K, N);
        aaedn::fused_matmul_destroy();
        auto got = down(dy, M * N);
        std::vector<float> want(M * N), mag(M * N);
        for (size_t m = 0; m < M; ++m)
            for (size_t n = 0; n < N; ++n)
            {
                double s = 0, a = 0;
                for (size_t k = 0; k < K; ++k)
                {
                    const size_t e = n * K + k;
                    const double w = ((codes[e / 2] >> ((e & 1) * 4)) & 15) * (double)half_to_float(scales[e / 32]);
                    s += x[m * K + k] * w;
                    a += std::fabs(x[m * K + k] * w);
                }
                want[m * N + n] = (float)s;
                mag[m * N + n] = (float)a;
            }
        CHECK(close(got, want, mag, 2e-5f));
    }

    // ---- rmsnorm: src/rmsnorm.cpp:8-51
    {
        const size_t n = 1000;
        std::vector<float> x(n), w(n);
        for (size_t i = 0; i < n; ++i)
            x[i] = frand(), w[i] = 1.0f + 0.5f * frand();
        float* dx = up(&arena, x);
        float* dw = up(&arena, w);
        float* dy = dev_f(&arena, n);
        aaedn::rmsnorm(dx, dy, dw, n);
        auto got = down(dy, n);
        double ss = 0;
        for (float v : x)
            ss += (double)v * v;
        const double r = 1.0 / std::sqrt(ss / n + 1e-6);
        std::vector<float> want(n), mag(n);
        for (size_t i = 0; i < n; ++i)
            want[i] = (float)(x[i] * r * w[i]), mag[i] = std::fabs(want[i]);
        CHECK(close(got, want, mag, 1e-5f));
    }

    // ---- rope: the reference table (src/rope.cpp:20-29) and rotation (:44-61)
    {
        const size_t S = 40, hd = 64, half = hd / 2;
        aaedn::RoPETables t = aaedn::rope_init(&arena, 128, hd);
        CHECK(t.cos_table && t.sin_table && t.max_seq_len == 128);
        std::vector<float> qh(S * hd), kh(S * hd);
        for (auto& v : qh)
            v = frand();
        for (auto& v : kh)
            v = frand();
        float* dq = up(&arena, qh);
        float* dk = up(&arena, kh);
        aaedn::rope_apply(dq, dk, S, hd, &t);
        auto gq = down(dq, S * hd), gk = down(dk, S * hd);
        auto tc = down(t.cos_table, 128 * half), ts = down(t.sin_table, 128 * half);
        std::vector<float> wq(S * hd), mq(S * hd, 1.0f);
        bool ok = true;
        for (size_t p = 0; p < S; ++p)
            for (size_t i = 0; i < half; ++i)
            {
                const float c = tc[p * half + i], s = ts[p * half + i];
                const float q0 = qh[p * hd + i], q1 = qh[p * hd + i + half];
                wq[p * hd + i] = c * q0 - s * q1;
                wq[p * hd + i + half] = s * q0 + c * q1;
                const float k0 = kh[p * hd + i], k1 = kh[p * hd + i + half];
                ok = ok && std::fabs(gk[p * hd + i] - (c * k0 - s * k1)) < 1e-6f;
            }
        CHECK(ok && close(gq, wq, mq, 1e-6f));
        aaedn::rope_apply(dq, dk, S, hd, nullptr); // no tables: no-op (src/rope.cpp:38-39)
        CHECK(down(dq, S * hd) == gq);
    }

    // ---- KV cache: appends, branch views, fork, attention over a view
    {
        const size_t L = 2, H = 4, hd = 32, T = 50;
        aaedn::KVCache kv;
        aaedn::kvcache_init(&kv, &arena, 256, L, H, hd, 3);
        CHECK(kv.base && kv.max_agents == 3 && kv.max_branches == 256);
        std::vector<float> hk(T * H * hd), hv(T * H * hd);
        for (auto& v : hk)
            v = frand();
        for (auto& v : hv)
            v = frand();
        float* dk = up(&arena, hk);
        float* dv = up(&arena, hv);
        // agent 0: tokens 0..29 (shared prefix); fork into agent 1; both then
        // append their own tokens
        auto app = [&](int agent, size_t t) {
            for (size_t l = 0; l < L; ++l)
                for (size_t h = 0; h < H; ++h)
                    aaedn::kvcache_append(&kv, agent, l, h, dk + (t * H + h) * hd, dv + (t * H + h) * hd);
        };
        for (size_t t = 0; t < 30; ++t)
            app(0, t);
        CHECK(aaedn::kvcache_fork(&kv, 0, 1));
        for (size_t t = 30; t < 40; ++t)
            app(0, t);
        for (size_t t = 40; t < 50; ++t)
            app(1, t);
        size_t n0 = 0, n1 = 0;
        const aaedn::Segment* s0 = aaedn::kvcache_segments(&kv, 0, &n0);
        const aaedn::Segment* s1 = aaedn::kvcache_segments(&kv, 1, &n1);
        CHECK(n0 == 1 && s0[0].start_token == 0 && s0[0].length == 40);
        CHECK(n1 == 2 && s1[0].start_token == 0 && s1[0].length == 30 && s1[1].start_token == 40 &&
              s1[1].length == 10);
        // rows landed in order in layer 1
        CHECK(down(aaedn::kvcache_layer_k(&kv, 1), T * H * hd) == hk);
        CHECK(down(aaedn::kvcache_layer_v(&kv, 1), T * H * hd) == hv);
        // attention of agent 1 over its view (src/attention.cpp:10-84 per head)
        std::vector<float> qh(H * hd);
        for (auto& v : qh)
            v = frand();
        float* dq = up(&arena, qh);
        float* dout = dev_f(&arena, H * hd);
        const float scale = 1.0f / std::sqrt((float)hd);
        aaedn::attention(dq, aaedn::kvcache_layer_k(&kv, 1), aaedn::kvcache_layer_v(&kv, 1), s1, n1, dout, H, hd,
                         scale);
        auto got = down(dout, H * hd);
        std::vector<float> want(H * hd), mag(H * hd, 1.0f);
        for (size_t h = 0; h < H; ++h)
        {
            std::vector<size_t> toks;
            for (size_t i = 0; i < n1; ++i)
                for (uint32_t j = 0; j < s1[i].length; ++j)
                    toks.push_back(s1[i].start_token + j);
            std::vector<double> sc(toks.size());
            double mx = -1e300;
            for (size_t j = 0; j < toks.size(); ++j)
            {
                double dot = 0;
                for (size_t e = 0; e < hd; ++e)
                    dot += (double)qh[h * hd + e] * hk[(toks[j] * H + h) * hd + e];
                sc[j] = dot * scale;
                mx = std::max(mx, sc[j]);
            }
            double den = 0;
            for (auto& v : sc)
                den += (v = std::exp(v - mx));
            for (size_t e = 0; e < hd; ++e)
            {
                double o = 0;
                for (size_t j = 0; j < toks.size(); ++j)
                    o += sc[j] * hv[(toks[j] * H + h) * hd + e];
                want[h * hd + e] = (float)(o / den);
            }
        }
        CHECK(close(got, want, mag, 2e-5f));
        aaedn::kvcache_compact(&kv, 7);
        CHECK(kv.branch_table[7].prune_flag.load() == 1 && kv.generation_counter.load() == 1);
    }

    // ---- ffn_swiglu: src/ffn.cpp:29-76 (row-group integer scales, g*silu(g)*u)
    {
        const size_t B = 2, h = 64, f = 96;
        std::vector<uint8_t> wg(f * h / 2), wu(f * h / 2), wd(h * f / 2);
        for (auto* w : {&wg, &wu, &wd})
            for (auto& b : *w)
                b = (uint8_t)(rng = rng * 6364136223846793005ull + 1442695040888963407ull, rng >> 56);
        std::vector<uint16_t> sg(f / 32 + 1), su(f / 32 + 1), sd(h / 32 + 1);
        for (auto* s : {&sg, &su, &sd})
            for (auto& v : *s)
                v = (uint16_t)(1 + (rng >> 60));
        std::vector<float> x(B * h);
        for (auto& v : x)
            v = 0.01f * frand();
        aaedn::QuantBlock G{}, U{}, Dn{};
        G.data = up(&arena, wg);
        U.data = up(&arena, wu);
        Dn.data = up(&arena, wd);
        uint16_t* dsg = up(&arena, sg);
        uint16_t* dsu = up(&arena, su);
        uint16_t* dsd = up(&arena, sd);
        float* dx = up(&arena, x);
        float* dy = dev_f(&arena, B * h);
        aaedn::ffn_swiglu(dx, dy, B, h, f, &G, &U, &Dn, dsg, dsu, dsd);
        auto got = down(dy, B * h);
        std::vector<float> want(B * h), mag(B * h);
        for (size_t b = 0; b < B; ++b)
        {
            std::vector<double> act(f);
            for (size_t j = 0; j < f; ++j)
            {
                double g = 0, u = 0;
                for (size_t i = 0; i < h; ++i)
                {
                    const int cg = (wg[j * h / 2 + i / 2] >> ((i % 2) * 4)) & 15;
                    const int cu = (wu[j * h / 2 + i / 2] >> ((i % 2) * 4)) & 15;
                    g += x[b * h + i] * (double)cg * sg[j / 32];
                    u += x[b * h + i] * (double)cu * su[j / 32];
                }
                act[j] = g * (g / (1.0 + std::exp(-g))) * u;
            }
            for (size_t i = 0; i < h; ++i)
            {
                double o = 0, a = 0;
                for (size_t j = 0; j < f; ++j)
                {
                    const int c = (wd[i * f / 2 + j / 2] >> ((j % 2) * 4)) & 15;
                    o += act[j] * c * sd[i / 32];
                    a += std::fabs(act[j] * c * sd[i / 32]);
                }
                want[b * h + i] = (float)o;
                mag[b * h + i] = (float)a;
            }
        }
        CHECK(close(got, want, mag, 1e-4f));
        aaedn::ffn_swiglu(dx, dy, B, h, f, nullptr, &U, &Dn, dsg, dsu, dsd); // src/ffn.cpp:22-27
        auto z = down(dy, B * h);
        bool allz = true;
        for (float v : z)
            allz = allz && v == 0.0f;
        CHECK(allz);
    }

    // ---- transformer: dims from the .abn header, forward twice, rejects bad ids
    {
        abn_test::Dims md;
        md.n_layers = 2, md.n_heads = 4, md.head_dim = 32, md.vocab = 1000, md.hidden = 128, md.ffn = 256;
        abn_test::write_file(dir + "/model.abn", abn_test::valid_model(md));
        aaedn::Transformer tf;
        aaedn::transformer_init(&tf, &arena, (dir + "/model.abn").c_str());
        CHECK(tf.model && tf.n_layers == 2 && tf.hidden_dim == 128 && tf.vocab_size == 1000);
        std::vector<float> l1(md.vocab), l2(md.vocab), l3(md.vocab, 5.0f);
        const uint32_t ids[3] = {5, 17, 999};
        aaedn::transformer_forward(&tf, ids, 3, l1.data());
        aaedn::transformer_forward(&tf, ids, 1, l2.data());
        bool finite = true, nonzero = false;
        for (float v : l1)
            finite = finite && std::isfinite(v), nonzero = nonzero || v != 0.0f;
        CHECK(finite && nonzero && l1 != l2);
        CHECK(aaedn_model_pos(tf.model) == 4);
        const uint32_t bad[1] = {1000};
        aaedn::transformer_forward(&tf, bad, 1, l3.data()); // src/transformer.cpp:137-142
        bool allz = true;
        for (float v : l3)
            allz = allz && v == 0.0f;
        CHECK(allz);
        // the same model through the C ABI gives the same logits
        aaedn_model_config c{};
        aaedn_model_config_get(tf.model, &c);
        aaedn_model* m2 = nullptr;
        CHECK(aaedn_model_create(&c, &m2) == AAEDN_OK && aaedn_model_synthesize(m2, 1234) == AAEDN_OK);
        std::vector<float> r1(md.vocab);
        CHECK(aaedn_model_forward(m2, ids, 3, r1.data()) == AAEDN_OK);
        CHECK(r1 == l1);
        aaedn_model_destroy(m2);
        aaedn::transformer_destroy(&tf);
        CHECK(tf.model == nullptr);
    }

    // ---- transformer_init from a whole-model file: the same logits as the
    // same weights handed to a model through the C ABI
    {
        abn_test::Dims md;
        md.n_layers = 2, md.n_heads = 4, md.head_dim = 32, md.vocab = 1000, md.hidden = 128, md.ffn = 256;
        const uint32_t KV = 2, D = md.hidden, F = md.ffn, V = md.vocab, QR = md.n_heads * md.head_dim,
                       KR = KV * md.head_dim;
        auto q4 = [&](size_t rows, size_t cols, std::vector<uint8_t>& c, std::vector<uint16_t>& s) {
            std::vector<float> x(rows * cols);
            for (auto& v : x)
                v = 0.02f * frand();
            c.resize(rows * cols / 2);
            s.resize(rows * cols / 32);
            aaedn_quantize_q4(x.data(), x.size(), c.data(), s.data());
        };
        struct Layer
        {
            std::vector<uint8_t> c[7];
            std::vector<uint16_t> s[7];
            std::vector<float> an, fn;
        };
        const size_t rows[7] = {QR, KR, KR, D, F, F, D}, cols[7] = {D, D, D, QR, D, D, F};
        std::vector<Layer> L(md.n_layers);
        std::vector<uint8_t> payload;
        for (auto& l : L)
        {
            for (int i = 0; i < 7; ++i)
                q4(rows[i], cols[i], l.c[i], l.s[i]);
            l.an.assign(D, 1.0f);
            l.fn.assign(D, 1.0f);
            for (size_t i = 0; i < D; ++i)
                l.an[i] += 0.1f * frand(), l.fn[i] += 0.1f * frand();
            abn_test::append(payload, l.an);
            for (int i = 0; i < 3; ++i) // QKV codes: q rows, k rows, v rows
                abn_test::append(payload, l.c[i]);
            for (int i = 0; i < 3; ++i) // then their scales
                abn_test::append(payload, l.s[i]);
            abn_test::append(payload, std::vector<float>(QR + 2 * KR, 0.0f)); // QKV bias
            for (int i = 3; i < 7; ++i)
            {
                abn_test::append(payload, l.c[i]);
                abn_test::append(payload, l.s[i]);
            }
            abn_test::append(payload, l.fn);
        }
        std::vector<float> fnorm(D, 1.0f), emb((size_t)V * D), lm((size_t)V * D);
        for (auto& v : emb)
            v = 0.02f * frand();
        for (auto& v : lm)
            v = 0.02f * frand();
        abn_test::append(payload, fnorm);
        abn_test::append(payload, emb);
        abn_test::append(payload, lm);
        std::vector<uint8_t> file = abn_test::whole_model_header(md, KV, 10000.0f, 1e-6f, payload);
        file.insert(file.end(), payload.begin(), payload.end());
        abn_test::write_file(dir + "/whole.abn", file);

        aaedn::Transformer tf;
        aaedn::transformer_init(&tf, &arena, (dir + "/whole.abn").c_str());
        const bool shaped = tf.model && tf.n_layers == 2 && tf.hidden_dim == D && tf.vocab_size == V;
        CHECK(shaped);
        aaedn_model_config c{};
        aaedn_model_config_get(tf.model, &c);
        CHECK(c.n_kv_heads == KV && c.rope_theta == 10000.0f);
        if (!shaped || c.n_kv_heads != KV) // the weights below only fit that shape
        {
            aaedn::transformer_destroy(&tf);
            aaedn::arena_destroy(&arena);
            std::printf("FAILED\n");
            return 1;
        }
        const uint32_t ids[3] = {3, 141, 592};
        std::vector<float> got(V), want(V);
        aaedn::transformer_forward(&tf, ids, 3, got.data());
        aaedn_model* m2 = nullptr;
        CHECK(aaedn_model_create(&c, &m2) == AAEDN_OK);
        for (uint32_t li = 0; li < md.n_layers; ++li)
        {
            const Layer& l = L[li];
            aaedn_layer_host w{};
            w.wq = l.c[0].data(), w.wk = l.c[1].data(), w.wv = l.c[2].data(), w.wo = l.c[3].data();
            w.wg = l.c[4].data(), w.wu = l.c[5].data(), w.wd = l.c[6].data();
            w.sq = l.s[0].data(), w.sk = l.s[1].data(), w.sv = l.s[2].data(), w.so = l.s[3].data();
            w.sg = l.s[4].data(), w.su = l.s[5].data(), w.sd = l.s[6].data();
            w.attn_norm = l.an.data(), w.ffn_norm = l.fn.data();
            CHECK(aaedn_model_set_layer(m2, li, &w) == AAEDN_OK);
        }
        CHECK(aaedn_model_set_globals(m2, emb.data(), fnorm.data(), lm.data()) == AAEDN_OK);
        CHECK(aaedn_model_forward(m2, ids, 3, want.data()) == AAEDN_OK);
        CHECK(got == want);
        aaedn_model_destroy(m2);
        aaedn::transformer_destroy(&tf);
    }

    aaedn::arena_destroy(&arena);
    std::printf("%s\n", fails ? "FAILED" : "PASSED");
    return fails ? 1 : 0;
}
