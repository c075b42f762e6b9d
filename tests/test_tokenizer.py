"""The native WordPiece tokenizer (include/futon_tokenizer.h) against the
reference's conformance fixtures and the CPU restatement (no GPU needed).

Pins, in order: the committed fixtures are the reference's (sha256); the
oracle reproduces every fixture id list (native/tokenizer_test.go:
TestTokenizerConformance, TestTokenizerSpecials); the native tokenizer
reproduces them too and equals the oracle bit for bit on seeded random text
(controls, invalid UTF-8, special literals, CJK, accents, combining-mark runs,
every truncation edge), for every thread count and batch shape; vocab parsing
and configuration follow NewTokenizer; FuzzTokenizerEncode's invariants hold.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import random

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from futon_b200 import FutonError, _lib
from futon_b200.tokenizer import Tokenizer, TokenizerConfig, pack_texts
from oracle import tokenizer as OT

TOKDIR = ROOT / "tests" / "golden" / "tokenizer"
VOCAB = TOKDIR / "vocab_bert_uncased.txt"
# native/tokenizer_test.go:18 (expectedVocabSHA256).
VOCAB_SHA256 = "07eced375cec144d27c900241f3e339478dec958f92fddbc551f295c992038a3"
BERT_CFG = dict(do_lower_case=True, tokenize_chinese_chars=True)  # defaultTokCfg


@pytest.fixture(scope="module")
def vocab_bytes():
    return VOCAB.read_bytes()


@pytest.fixture(scope="module")
def fixtures():
    return json.loads((TOKDIR / "tokenizer_fixtures.json").read_text())


@pytest.fixture(scope="module")
def native(vocab_bytes):
    return Tokenizer(vocab_bytes, TokenizerConfig(**BERT_CFG))


@pytest.fixture(scope="module")
def oracle(vocab_bytes):
    return OT.Tokenizer(vocab_bytes, OT.TokenizerConfig(**BERT_CFG))


def _fixture_cases(fx):
    for model, m in fx["models"].items():
        for c in m["cases"]:
            yield model, c["name"], c["text"], m["max_seq_len"], c["ids"]
            yield model, c["name"], c["text"], 16, c["ids_max16"]


def test_fixtures_are_the_references():
    sums = json.loads((TOKDIR / "SHA256SUMS.json").read_text())
    for name, want in sums.items():
        assert hashlib.sha256((TOKDIR / name).read_bytes()).hexdigest() == want, name
    assert sums["vocab_bert_uncased.txt"] == VOCAB_SHA256


def test_oracle_matches_reference_fixtures(fixtures, oracle):
    n = 0
    for model, name, text, max_len, want in _fixture_cases(fixtures):
        assert oracle.encode(text, max_len) == want, (model, name, max_len)
        n += 1
    assert n == 168 and len(fixtures["models"]) == 3


def test_native_matches_reference_fixtures(fixtures, native):
    for model, name, text, max_len, want in _fixture_cases(fixtures):
        assert native.encode(text, max_len) == want, (model, name, max_len)


def test_native_batch_matches_reference_fixtures(fixtures, native):
    for model, m in fixtures["models"].items():
        texts = [c["text"] for c in m["cases"]]
        for max_len, key in ((m["max_seq_len"], "ids"), (16, "ids_max16")):
            ids, cu = native.encode_batch(texts, max_len, threads=3)
            for i, c in enumerate(m["cases"]):
                assert ids[cu[i]:cu[i + 1]].tolist() == c[key], (model, c["name"], max_len)


def test_specials_and_vocab_size(native, oracle):
    """TestTokenizerSpecials: [PAD] is 0; empty and whitespace-only text
    reduce to [CLS][SEP]."""
    assert native.pad_id() == 0 == oracle.pad_id
    assert native.vocab_size() == 30522 == oracle.vocab_size()
    for text in ("", "   \t\n "):
        assert native.encode(text, 512) == [101, 102]


def test_missing_vocab_errors():
    """TestTokenizerMissingVocab."""
    with pytest.raises(FutonError, match="tokenizer: open vocab"):
        Tokenizer.from_file(TOKDIR / "does-not-exist.txt", TokenizerConfig(**BERT_CFG))


# ---- native == oracle on seeded random text ----------------------------------

POOL = ([chr(c) for c in range(32, 127)] * 4
        + list("\u00c9\u00e9\u00e8\u00c0\u00c2\u00e7\u00f1\u00d1\u00fc\u00dc\u00f6\u00d8"
               "\u00df\u0110\u1eb7\u1eab\u01c5\u0130\u212a\u03a3\u017f")
        + [chr(0x300 + i) for i in range(0x70)]
        + list("\u81ea\u7136\u8a00\u8a9e\u51e6\u7406\u673a\u5668\u5b66\u4e60"
               "\uc790\uc5f0\uc5b4\ucc98\ub9ac")
        + ["\u00a0", "\u2003", "\u3000", "\t", "\n", "\r", "\v", "\x00", "\x07", "\x85",
           "\ufffd", "\u2028", "\u2029", "\u200b", "\ue000", "\U0001F680", "\U0001D165",
           "\U0001D16D", "\uf900", "\u0344", "\u0f73", "\u1e9b\u0323"]
        + ["[CLS]", "[SEP]", "[MASK]", "[PAD]", "[UNK]", "[unused0]", "[CLS", "SEP]"])


def _random_texts(seed, n, words):
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        parts = []
        for _ in range(rng.randint(0, 50)):
            r = rng.random()
            if r < 0.45:
                w = rng.choice(words)
                parts.append((w.upper() if rng.random() < 0.1 else w.capitalize()
                               if rng.random() < 0.2 else w) + " ")
            elif r < 0.9:
                parts.append(rng.choice(POOL))
            else:
                parts.append("".join(rng.choice(POOL) for _ in range(rng.randint(1, 150))))
        out.append("".join(parts))
    out += [bytes(rng.randrange(256) for _ in range(rng.randint(0, 60))) for _ in range(n // 5)]
    out += ["a" + "\u0301" * 45 + "b", "x" + "\u0301\u0345" * 20 + "\U0001D165\u0300" * 20,
            "word" * 30, "\u00e9" * 120, "ab" * 50, "ab" * 51, "\xe9" * 101, "[CLS]" * 600]
    return out


@pytest.fixture(scope="module")
def random_texts(vocab_bytes):
    words = [w for w in vocab_bytes.decode().split("\n")[1000:12000] if w.isalpha()]
    return _random_texts(1234, 1200, words)


@pytest.mark.parametrize("max_len", [0, 1, 2, 3, 16, 128, 512])
def test_native_matches_oracle_random(native, oracle, random_texts, max_len):
    for t in random_texts:
        assert native.encode(t, max_len) == oracle.encode(t, max_len), (max_len, t)


@pytest.mark.parametrize("threads", [1, 3, 0])
def test_batch_equals_single_for_every_thread_count(native, oracle, random_texts, threads):
    texts = random_texts[:777]  # not a multiple of the 64-text chunk
    ids, cu = native.encode_batch(texts, 64, threads=threads)
    want_ids, want_cu = oracle.encode_batch(texts, 64)
    assert np.array_equal(cu, want_cu) and np.array_equal(ids, want_ids)


def test_batch_shapes(native):
    ids, cu = native.encode_batch([], 512)
    assert ids.size == 0 and cu.tolist() == [0]
    ids, cu = native.encode_batch(["", "", "hello"], 512)
    assert cu.tolist() == [0, 2, 4, 7] and ids.tolist() == [101, 102, 101, 102, 101, 7592, 102]


def test_batch_reports_total_when_ids_do_not_fit(native):
    """A short ids buffer fails with FUTON_EINVAL after writing cu_seqlens,
    so the caller can size it exactly (the Python wrapper retries)."""
    data, off = pack_texts(["hello world", "the cat sat"])
    cu = np.zeros(3, dtype=np.int32)
    ids = np.zeros(3, dtype=np.int32)
    with pytest.raises(FutonError, match="do not fit"):
        _lib.call("futon_tokenizer_encode_batch", native._h, data, off.ctypes.data, 2, 512, 1,
                  ids.ctypes.data, 3, cu.ctypes.data)
    assert cu.tolist() == [0, 4, 9]
    got, gcu = native.encode_packed_bytes(data, off, 512)
    assert gcu.tolist() == [0, 4, 9] and got.size == 9


def test_batch_rejects_bad_offsets(native):
    data, off = pack_texts(["abc", "def"])
    bad = np.array([0, 4, 3], dtype=np.int64)
    cu = np.zeros(3, dtype=np.int32)
    ids = np.zeros(16, dtype=np.int32)
    with pytest.raises(FutonError, match="decrease"):
        _lib.call("futon_tokenizer_encode_batch", native._h, data, bad.ctypes.data, 2, 512, 1,
                  ids.ctypes.data, 16, cu.ctypes.data)
    with pytest.raises(FutonError, match="null"):
        _lib.call("futon_tokenizer_encode_batch", None, data, off.ctypes.data, 2, 512, 1,
                  ids.ctypes.data, 16, cu.ctypes.data)


def test_single_encode_reports_needed_count(native):
    out = (C.c_int32 * 2)()
    n = C.c_int(0)
    text = b"hello world"
    with pytest.raises(FutonError, match="do not fit"):
        _lib.call("futon_tokenizer_encode", native._h, text, len(text), 512, out, 2, C.byref(n))
    assert n.value == 4


def test_fuzz_invariants(native, vocab_bytes):
    """FuzzTokenizerEncode: [CLS] … [SEP] within [2, maxLen], every id in
    the vocab, the same ids on re-encoding; over its seeds and seeded byte
    soup."""
    seeds = [b"", b" ", b"hello world", "\u00c9lodie caf\u00e9 \u2603".encode(),
             "\u81ea\u7136\u8a00\u8a9e\u51e6\u7406".encode(),
             b"(((([[{{}}]]))))", b"a\x00b\x07c", b"\xff\xfe invalid utf8",
             b"buffalo buffalo buffalo", b"x", b"[CLS] injected [SEP]"]
    rng = random.Random(7)
    soup = [bytes(rng.randrange(256) for _ in range(rng.randint(0, 300))) for _ in range(400)]
    for i, text in enumerate(seeds + soup):
        max_len = (rng.randrange(1 << 16) % 1024) + 2
        ids = native.encode(text, max_len)
        assert 2 <= len(ids) <= max_len
        assert ids[0] == 101 and ids[-1] == 102
        assert all(0 <= t < native.vocab_size() for t in ids)
        assert native.encode(text, max_len) == ids


# ---- vocab parsing and configuration (NewTokenizer) --------------------------

SPECIALS = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"]


def _both(vocab: bytes, **cfg):
    return Tokenizer(vocab, TokenizerConfig(**cfg)), OT.Tokenizer(vocab, OT.TokenizerConfig(**cfg))


def test_vocab_crlf_duplicates_and_final_line():
    """Lines split at LF with trailing CR trimmed; a repeated token keeps
    its last id and counts once; an empty line is the token ""; a final line
    without LF counts."""
    body = "\r\n".join(SPECIALS + ["hello", "world", "hello", "##s", "", "cat"])
    for vocab in (body.encode(), (body + "\r\n").encode()):
        n, o = _both(vocab, do_lower_case=True)
        assert n.vocab_size() == o.vocab_size() == 10
        for text in ("hello worlds", "Cats", "hello  cat", "x"):
            assert n.encode(text, 32) == o.encode(text, 32)
        assert n.encode("hello cat", 32) == [2, 7, 10, 3]


def test_vocab_errors():
    with pytest.raises(FutonError, match="vocab is empty"):
        Tokenizer(b"", TokenizerConfig())
    with pytest.raises(FutonError, match='special token "\\[MASK\\]" not in vocab'):
        Tokenizer("\n".join(SPECIALS[:4]).encode(), TokenizerConfig())
    with pytest.raises(FutonError, match="token too long"):
        Tokenizer(b"x" * (1 << 20) + b"\n" + "\n".join(SPECIALS).encode(), TokenizerConfig())
    with pytest.raises(OT.TokenizerError, match="token too long"):
        OT.Tokenizer(b"x" * (1 << 20) + b"\n" + "\n".join(SPECIALS).encode())
    # The largest line bufio.Scanner accepts (LF included) loads.
    Tokenizer(b"x" * ((1 << 20) - 1) + b"\n" + "\n".join(SPECIALS).encode(), TokenizerConfig())


@pytest.mark.parametrize("cfg", [
    dict(do_lower_case=False, tokenize_chinese_chars=True),
    dict(do_lower_case=True, tokenize_chinese_chars=False),
    dict(do_lower_case=True, tokenize_chinese_chars=True, max_input_chars_per_word=4),
    dict(do_lower_case=True, cls_token="<s>", sep_token="</s>", unk_token="<unk>",
         pad_token="<pad>", mask_token="<mask>"),
])
def test_config_variants_match_oracle(vocab_bytes, random_texts, cfg):
    vocab = vocab_bytes + b"\n<s>\n</s>\n<unk>\n<pad>\n<mask>\nHello\n##World\n"
    n, o = _both(vocab, **cfg)
    for t in random_texts[:300] + ["Hello World <s> x</s>", "HelloWorld",
                                   "\u81ea\u7136 \u00dcber"]:
        assert n.encode(t, 96) == o.encode(t, 96), (cfg, t)


def test_stream_safe_nfd_order():
    """NFD in the Stream-Safe Text Format (x/text norm, UAX #15 §13): after
    30 non-starters a CGJ barrier stops canonical reordering, which is
    visible through the two kept (Mc) non-starters U+1D16D (class 226) and
    U+1D165 (class 216) around a run of U+0301 (class 230, stripped)."""
    a, b = "\U0001D165", "\U0001D16D"
    vocab = "\n".join(SPECIALS + ["x", "##" + a, "##" + b]).encode()
    n, o = _both(vocab, do_lower_case=True)
    short = "x" + b + "\u0301" * 28 + a  # 30 non-starters: one run, sorted
    long = "x" + b + "\u0301" * 30 + a   # the 31st starts a new segment
    assert n.encode(short, 16) == o.encode(short, 16) == [2, 5, 6, 7, 3]
    assert n.encode(long, 16) == o.encode(long, 16) == [2, 5, 7, 6, 3]
    # An ASCII control inside the run is removed before NFD: it neither ends
    # the run nor resets the count, while a kept ASCII character ends both.
    ctrl = "x" + b + "\x07" + "\u0301" * 30 + "\x01" + a
    assert n.encode(ctrl, 16) == o.encode(ctrl, 16) == [2, 5, 7, 6, 3]
    kept = "x" + b + "\u0301" * 15 + "x" + "\u0301" * 15 + a
    assert n.encode(kept, 16) == o.encode(kept, 16)


def test_toy_pack_text_ids(toy_expected):
    """The toy packs' text cases (native/testdata/toy/expected.json) tokenise
    to the ids the upstream HF tokenizer gave, with the pack's own vocab and
    tokenizer config."""
    from futon_b200.pack import load_pack_config
    pack = GOLDEN / "toy-absolute-gelu"
    cfg = load_pack_config(pack)
    tok = Tokenizer.from_file(pack / "vocab.txt", TokenizerConfig.from_dict(cfg.tokenizer))
    for c in toy_expected["packs"]["toy-absolute-gelu"]["text_cases"]:
        assert tok.encode(c["text"], cfg.effective_max_seq_len()) == c["ids"], c["text"]


# ---- property-based: arbitrary text and bytes (FuzzTokenizerEncode's input) --

from hypothesis import given, settings, strategies as st  # noqa: E402

# Every Unicode category, weighted towards what the pipeline treats specially:
# ASCII, Latin with accents, combining marks, CJK, whitespace and controls.
_ALPHABET = st.one_of(
    st.characters(min_codepoint=0, max_codepoint=0x7F),
    st.characters(min_codepoint=0xC0, max_codepoint=0x24F),
    st.characters(min_codepoint=0x300, max_codepoint=0x36F),
    st.sampled_from(list("\u3000\u00a0\u2028\u2003\u0085\u200b\ufffd\u0130\u212a\u03a3"
                         "\u81ea\u7136\uac00\ud55c\U0001D165\U0001D16D\u0f73\u0344")),
    st.characters(blacklist_categories=("Cs",)),
)
_TEXT = st.one_of(
    st.text(_ALPHABET, max_size=120),
    st.binary(max_size=120),
    st.lists(st.sampled_from(["[CLS]", "[SEP]", "[PAD]", "hello", "World", " ", "\u0301",
                              "##", "[", "]", "\xe9t\xe9"]), max_size=20).map("".join),
)


@settings(max_examples=600, deadline=None, derandomize=True)
@given(text=_TEXT, max_len=st.integers(min_value=-3, max_value=600))
def test_native_matches_oracle_property(native, oracle, text, max_len):
    got = native.encode(text, max_len)
    assert got == oracle.encode(text, max_len)
    assert 2 <= len(got) <= max(2, max_len)
    assert got[0] == 101 and got[-1] == 102


def test_huge_max_len_allocates_by_text(native):
    """encode sizes its buffer by the text, not by max_seq_len."""
    assert native.encode("hello world", 2**31 - 1) == [101, 7592, 2088, 102]
    ids, cu = native.encode_batch(["hello world", ""], 2**31 - 1)
    assert ids.tolist() == [101, 7592, 2088, 102, 101, 102] and cu.tolist() == [0, 4, 6]


# ---- the compiled port timed as the text path's CPU baseline ---------------

def test_compiled_port_gives_the_reference_ids(fixtures, native, random_texts):
    """oracle/tokenizer_port.cpp (the reference tokenizer's structure,
    compiled; bench.py's CPU baseline) reproduces the fixtures and equals the
    library on seeded random text, for one and several threads."""
    from oracle.tokport import TokenizerPort
    port = TokenizerPort(VOCAB.read_bytes())
    for model, name, text, max_len, want in _fixture_cases(fixtures):
        assert port.encode(text, max_len) == want, (model, name, max_len)
    data, off = pack_texts(random_texts)
    for threads in (1, 4):
        for max_len in (16, 512):
            ids, cu = port.encode_packed_bytes(data, off, max_len, threads)
            want_ids, want_cu = native.encode_packed_bytes(data, off, max_len)
            assert np.array_equal(cu, want_cu) and np.array_equal(ids, want_ids)
