"""The .abt tokenizer (host code, no GPU): the library's C ABI, its C++ API
and the oracle against the reference's own answers
(tests/golden/tokenizer_golden.npz, made by make_tokenizer_golden.py from
src/tokenizer.cpp compiled from source), and the library against the oracle
and (where oracle/_ref is built) the reference on fresh seeded cases."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import aaedn_b200 as ab
from aaedn_b200.tokenizer import Tokenizer, abt_bytes, from_hf

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import tok_oracle  # noqa: E402

G = np.load(os.path.join(HERE, "golden", "tokenizer_golden.npz"))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libaaedn_ref.so")


def _split(flat, lens):
    out, o = [], 0
    for n in lens:
        out.append(flat[o:o + n])
        o += n
    return out


TEXTS = [bytes(t) for t in _split(G["text_bytes"], G["text_len"])]


def _golden(name, bos):
    ids = _split(G[f"{name}_bos{bos}_ids"], G[f"{name}_bos{bos}_n"])
    dec = [bytes(d) for d in _split(G[f"{name}_bos{bos}_dec"], G[f"{name}_bos{bos}_dec_n"])]
    return ids, dec


def _declists(name):
    ids = _split(G[f"{name}_declist_ids"], G[f"{name}_declist_n"])
    dec = [bytes(d) for d in _split(G[f"{name}_declist_dec"], G[f"{name}_declist_dec_n"])]
    return ids, dec


@pytest.mark.parametrize("name", ["seeded", "roundtrip"])
def test_oracle_matches_reference_golden(name):
    tok = tok_oracle.load(G[f"tok_{name}"].tobytes())
    info = G[f"{name}_info"]
    assert [tok["vocab_size"], tok["merge_count"], tok["max_token_bytes"], tok["format_version"],
            tok["payload_checksum"]] == [int(v) for v in info]
    for bos in (0, 1):
        ids, dec = _golden(name, bos)
        for t, want, wd in zip(TEXTS, ids, dec):
            got = tok_oracle.encode(tok, t, bos)
            assert got == [int(v) for v in want], t
            assert tok_oracle.decode(tok, got) == wd
    for L, wd in zip(*_declists(name)):
        assert tok_oracle.decode(tok, [int(v) for v in L]) == wd


def test_oracle_load_decisions_match_reference():
    for name, ok in zip(G["case_names"], G["case_ok"]):
        got = tok_oracle.load(G[f"case_{name}"].tobytes())
        assert (got is not None) == bool(ok), name


@pytest.mark.parametrize("name", ["seeded", "roundtrip"])
def test_library_matches_reference_golden(name):
    t = Tokenizer(data=G[f"tok_{name}"].tobytes())
    assert [t.vocab_size, t.merge_count, t.max_token_bytes, t.format_version,
            t.payload_checksum] == [int(v) for v in G[f"{name}_info"]]
    for bos in (0, 1):
        ids, dec = _golden(name, bos)
        for text, want, wd in zip(TEXTS, ids, dec):
            got = t.encode(text, add_bos=bool(bos))
            np.testing.assert_array_equal(got, want)
            assert t.decode(got) == wd
    for L, wd in zip(*_declists(name)):
        assert t.decode(L) == wd


def test_library_load_decisions_match_reference(tmp_path):
    for name, ok, info in zip(G["case_names"], G["case_ok"], G["case_info"]):
        img = G[f"case_{name}"].tobytes()
        p = tmp_path / f"{name}.abt"
        p.write_bytes(img)
        for kw in (dict(path=p), dict(data=img)):
            if ok:
                t = Tokenizer(**kw)
                assert [t.vocab_size, t.merge_count, t.max_token_bytes, t.format_version,
                        t.payload_checksum] == [int(v) for v in info], name
            else:
                with pytest.raises(ab.AaednError) as e:
                    Tokenizer(**kw)
                assert e.value.rc == ab.EFORMAT, name
    with pytest.raises(ab.AaednError):
        Tokenizer(path=tmp_path / "missing.abt")


def _random_tokenizer(rng, n_rules, alpha=b"abcde "):
    tokens = [bytes([i]) for i in range(256)] + [bytes(alpha[int(k)] for k in rng.integers(0, len(alpha), 3))
                                                  for _ in range(int(rng.integers(0, 40)))]
    vocab = len(tokens)
    merges = []
    for _ in range(n_rules):
        r = rng.random()
        if r < 0.55 or not merges:
            a, b = (int(alpha[int(k)]) for k in rng.integers(0, len(alpha), 2))
        elif r < 0.9:
            a = vocab + int(rng.integers(0, len(merges)))
            b = int(alpha[int(rng.integers(0, len(alpha)))]) if rng.random() < 0.5 else vocab + int(
                rng.integers(0, len(merges)))
        else:
            a, b = merges[int(rng.integers(0, len(merges)))]
        merges.append((a & 0xFFFF, b & 0xFFFF))
    return tokens, merges


def test_library_matches_oracle_fuzz():
    rng = np.random.default_rng(99)
    for case in range(12):
        tokens, merges = _random_tokenizer(rng, int(rng.integers(1, 120)))
        img = abt_bytes(tokens, merges)
        t = Tokenizer(data=img)
        o = tok_oracle.load(img)
        for _ in range(15):
            text = bytes(b"abcde "[int(k)] for k in rng.integers(0, 6, int(rng.integers(0, 90))))
            bos = bool(rng.integers(0, 2))
            got = t.encode(text, add_bos=bos)
            assert [int(v) for v in got] == tok_oracle.encode(o, text, bos), (case, text)
            assert t.decode(got) == tok_oracle.decode(o, [int(v) for v in got])


def test_encode_stops_at_nul_and_sizes():
    t = Tokenizer(data=abt_bytes([bytes([i]) for i in range(256)], [(97, 98)]))
    np.testing.assert_array_equal(t.encode(b"ab\0ab"), [256])
    assert t.encode(b"").size == 0
    np.testing.assert_array_equal(t.encode("", add_bos=True), [32765])
    # the C ABI's size query and too-small buffers. "abab": both (a, b) pairs
    # are queued under rule 0; the one at position 0 leaves the queue first,
    # which moves the second pair off its queued position, so it stays
    # unmerged (the reference's discipline): 3 ids
    n = ctypes.c_size_t()
    assert ab.lib().aaedn_tokenizer_encode(t._h, b"abab", 0, None, 0, ctypes.byref(n)) == ab.OK and n.value == 3
    np.testing.assert_array_equal(t.encode(b"abab"), [256, 97, 98])
    out = np.zeros(1, np.uint32)
    assert ab.lib().aaedn_tokenizer_encode(t._h, b"abab", 0, out.ctypes.data, 1, ctypes.byref(n)) == ab.EINVAL
    ids = np.array([97, 98], np.uint32)
    buf = ctypes.create_string_buffer(2)
    assert ab.lib().aaedn_tokenizer_decode(t._h, ids.ctypes.data, 2, buf, 2, ctypes.byref(n)) == ab.EINVAL
    assert n.value == 2


def test_out_of_block_offset_decodes_empty():
    img = bytearray(abt_bytes([b"a", b"b"], []))
    # offset of token 1 -> far outside the 4-byte string block, checksum redone
    import struct
    struct.pack_into("<I", img, 64 + 16 + 4 + 4, 1000)
    struct.pack_into("<I", img, 20, ab.fnv1a32(bytes(img[64:])))
    t = Tokenizer(data=bytes(img))
    assert t.decode([0, 1, 0]) == b"aa"


def test_from_hf_reads_vocab_and_merges():
    class Fake:
        merges = ["a b", "ab c", "x##y", "bad", 7]

        def get_vocab(self):
            return {"a": 0, "b": 1, "c": 2, "ab": 3, "x": 4}

    tokens, merges = from_hf(Fake())
    assert tokens == ["a", "b", "c", "ab", "x"]
    assert merges == [(0, 1), (3, 2), (4, 0)]
    t = Tokenizer(data=abt_bytes(tokens, merges))
    assert (t.vocab_size, t.merge_count, t.max_token_bytes) == (5, 3, 2)


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref (the reference compiled here) is not built")
def test_library_matches_compiled_reference_fuzz(tmp_path):
    lib = ctypes.CDLL(REF_SO)
    sz = ctypes.c_size_t
    lib.ref_tokenizer.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                  sz, ctypes.POINTER(sz), ctypes.c_void_p, sz, ctypes.POINTER(sz)]
    lib.ref_tokenizer.restype = ctypes.c_int
    rng = np.random.default_rng(7)
    for case in range(20):
        tokens, merges = _random_tokenizer(rng, int(rng.integers(1, 300)))
        img = abt_bytes(tokens, merges)
        p = str(tmp_path / "t.abt")
        with open(p, "wb") as f:
            f.write(img)
        t = Tokenizer(path=p)
        for _ in range(10):
            text = bytes(b"abcde "[int(k)] for k in rng.integers(0, 6, int(rng.integers(0, 400))))
            bos = int(rng.integers(0, 2))
            info = np.zeros(5, np.uint32)
            ids = np.zeros(len(text) + 2, np.uint32)
            buf = ctypes.create_string_buffer(8 * len(text) + 64)
            ni, nb = sz(), sz()
            assert lib.ref_tokenizer(p.encode(), text, bos, info.ctypes.data, ids.ctypes.data, ids.size,
                                     ctypes.byref(ni), buf, len(buf), ctypes.byref(nb)) == 1
            got = t.encode(text, add_bos=bool(bos))
            np.testing.assert_array_equal(got, ids[:ni.value])
            assert t.decode(got) == buf.raw[:nb.value]


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref (the reference compiled here) is not built")
def test_long_text_matches_compiled_reference(tmp_path):
    """A 40 KB text (tens of thousands of merges, many of them chained and
    tied) against the reference compiled from source."""
    lib = ctypes.CDLL(REF_SO)
    sz = ctypes.c_size_t
    lib.ref_tokenizer.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                  sz, ctypes.POINTER(sz), ctypes.c_void_p, sz, ctypes.POINTER(sz)]
    lib.ref_tokenizer.restype = ctypes.c_int
    rng = np.random.default_rng(11)
    tokens, merges = _random_tokenizer(rng, 250)
    alpha = b"abcde "
    merges = [(x, y) for x in alpha for y in alpha] + merges  # every byte pair has a rule
    p = str(tmp_path / "t.abt")
    with open(p, "wb") as f:
        f.write(abt_bytes(tokens, merges))
    text = bytes(b"abcde "[int(k)] for k in rng.integers(0, 6, 40000))
    ids = np.zeros(len(text) + 2, np.uint32)
    buf = ctypes.create_string_buffer(8 * len(text))
    info = np.zeros(5, np.uint32)
    ni, nb = sz(), sz()
    assert lib.ref_tokenizer(p.encode(), text, 1, info.ctypes.data, ids.ctypes.data, ids.size, ctypes.byref(ni),
                             buf, len(buf), ctypes.byref(nb)) == 1
    got = Tokenizer(path=p).encode(text, add_bos=True)
    assert len(text) + 1 - got.size > 500  # a thousand merges (most queued entries go stale as positions shift)
    np.testing.assert_array_equal(got, ids[:ni.value])


def _chain_tokenizer(k):
    """Byte tokens and the chain (a, a) -> X0, (X0, a) -> X1, ...: a run of
    'a' merges over and over near its start."""
    toks = [bytes([i]) for i in range(256)]
    return toks, [(97, 97)] + [(256 + i, 97) for i in range(k - 1)]


def test_encode_scales_to_megabytes():
    """Encode is O((n + merges) log n): a 1 MB run of one byte under a
    30000-rule chain (hundreds of thousands of merges near the start, where
    erasing from a vector, as the reference does, moves the whole tail each
    time) stays well under a few seconds."""
    import time
    t = Tokenizer(data=abt_bytes(*_chain_tokenizer(30000)))
    text = b"a" * (1 << 20)
    t0 = time.perf_counter()
    ids = t.encode(text)
    dt = time.perf_counter() - t0
    assert len(text) - ids.size > 100000, ids.size
    assert dt < 10.0, dt


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref (the reference compiled here) is not built")
def test_merge_chain_matches_compiled_reference(tmp_path):
    """The chained merges of a 20 KB run of one byte against the reference."""
    lib = ctypes.CDLL(REF_SO)
    sz = ctypes.c_size_t
    lib.ref_tokenizer.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                  sz, ctypes.POINTER(sz), ctypes.c_void_p, sz, ctypes.POINTER(sz)]
    lib.ref_tokenizer.restype = ctypes.c_int
    p = str(tmp_path / "chain.abt")
    with open(p, "wb") as f:
        f.write(abt_bytes(*_chain_tokenizer(3000)))
    text = b"a" * 20000
    ids = np.zeros(len(text) + 2, np.uint32)
    buf = ctypes.create_string_buffer(8 * len(text))
    info = np.zeros(5, np.uint32)
    ni, nb = sz(), sz()
    assert lib.ref_tokenizer(p.encode(), text, 0, info.ctypes.data, ids.ctypes.data, ids.size, ctypes.byref(ni),
                             buf, len(buf), ctypes.byref(nb)) == 1
    got = Tokenizer(path=p).encode(text)
    assert len(text) - got.size > 5000
    np.testing.assert_array_equal(got, ids[:ni.value])


CPP = r'''
#include <cstdio>
#include <cstring>
#include "aaedn/arena.hpp"
#include "aaedn/tokenizer.hpp"
int main(int argc, char** argv)
{
    aaedn::Arena a = aaedn::arena_create(1 << 16, 64);
    aaedn::Tokenizer t = aaedn::tokenizer_load(&a, argv[1]);
    if (!t.strings) { std::printf("rejected\n"); aaedn::arena_destroy(&a); return 0; }
    std::printf("%u %u %u %u %u\n", t.vocab_size, t.merge_count, t.max_token_bytes, t.format_version,
                t.payload_checksum);
    for (int i = 2; i < argc; ++i)
    {
        std::vector<uint32_t> ids = aaedn::tokenizer_encode(&t, argv[i], i % 2 == 1);
        for (uint32_t v : ids) std::printf("%u ", v);
        std::printf("| %s\n", aaedn::tokenizer_decode(&t, ids).c_str());
    }
    aaedn::arena_destroy(&a);
    return 0;
}
'''


def test_cpp_api_tokenizer(tmp_path):
    """The reference-shaped C++ API (tokenizer_load into the arena's host part,
    encode, decode), compiled against the mirror headers."""
    pkg = os.path.join(ROOT, "project-aaedn_b200")
    src = tmp_path / "tok.cpp"
    src.write_text(CPP)
    exe = tmp_path / "tok"
    libdir = os.path.join(pkg, "aaedn_b200")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I" + os.path.join(pkg, "host", "include"), str(src), "-o", str(exe),
                    "-L" + libdir, "-laaedn_b200", "-Wl,-rpath," + libdir], check=True)
    name = "seeded"
    p = tmp_path / "t.abt"
    p.write_bytes(G[f"tok_{name}"].tobytes())
    texts = [t for t in TEXTS[:30] if t and 0 not in t and all(32 <= c < 127 for c in t)]
    r = subprocess.run([str(exe), str(p)] + [t.decode() for t in texts], capture_output=True, check=True)
    lines = r.stdout.decode().splitlines()
    assert lines[0].split() == [str(int(v)) for v in G[f"{name}_info"]]
    ref = {bytes(t): (i, d) for t, i, d in zip(TEXTS, *_golden(name, 0))}
    ref_b = {bytes(t): (i, d) for t, i, d in zip(TEXTS, *_golden(name, 1))}
    for k, (t, line) in enumerate(zip(texts, lines[1:])):
        ids_s, dec = line.split(" | ", 1) if " | " in line else (line.rstrip(" |"), "")
        want_ids, want_dec = (ref_b if (k + 2) % 2 == 1 else ref)[t]
        assert [int(v) for v in ids_s.split()] == [int(v) for v in want_ids]
        assert dec.encode() == want_dec
    bad = tmp_path / "bad.abt"
    bad.write_bytes(G["case_bad_magic"].tobytes())
    r = subprocess.run([str(exe), str(bad)], capture_output=True, check=True)
    assert r.stdout.decode().strip() == "rejected"
