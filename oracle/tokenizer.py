"""CPU restatement of futon's WordPiece tokenizer — TEST INFRASTRUCTURE ONLY.

The checker for the native tokenizer in libfuton_cuda (include/
futon_tokenizer.h): tests and bench.py's CPU-baseline leg call it, nothing in
futon_b200/ does. It follows native/tokenizer.go step by step, with Go's
library semantics spelled out where Python's differ:

  * Go's `unicode` tables (Go 1.23, Unicode 15.0.0) for the categories Mn,
    Zs, C (= Cc ∪ Cf ∪ Co ∪ Cs: Go has no table for unassigned code points,
    so Cn is NOT control) and P*;
  * `strings.ToLower` = the simple (one-to-one) lowercase mapping per rune,
    so U+0130 lowercases to U+0069 (Python's full mapping gives two runes)
    and capital sigma always to U+03C3;
  * `strings.Fields` splits on Go's `unicode.IsSpace` (the White_Space
    property), which after the cleaning step leaves U+2028 and U+2029 as
    separators besides the space;
  * `norm.NFD` from golang.org/x/text v0.21.0 (absent from the reference
    tree; Unicode 15.0.0): canonical decomposition and canonical ordering
    (UAX #15), in the Stream-Safe Text Format of UAX #15 §13 — after 30
    consecutive non-starters a U+034F COMBINING GRAPHEME JOINER is inserted,
    which stops reordering across it. CGJ is Mn, so accent stripping removes
    it again; the rule changes results only for runs of more than 30
    combining marks. Decomposition and reordering come from CPython's
    unicodedata (Unicode 15.0.0), independently of the native tables;
  * Go's UTF-8 decoding: an invalid byte decodes to U+FFFD, which the
    cleaning step drops (Python's replacement may merge several invalid
    bytes into one U+FFFD; dropped either way).

Pinned by the reference's conformance fixtures (native/testdata/
tokenizer_fixtures.json, HF fast-tokenizer ids for 28 texts × 3 packs at
their max length and at 16) in tests/test_tokenizer.py.
"""
from __future__ import annotations

import dataclasses
import unicodedata
from typing import Dict, List, Optional, Sequence, Tuple

assert unicodedata.unidata_version == "15.0.0", unicodedata.unidata_version

CGJ = "\u034f"
MAX_NON_STARTERS = 30
# Go unicode.IsSpace (White_Space, Unicode 15.0.0 PropList).
GO_SPACE = frozenset("\t\n\v\f\r \x85\xa0\u1680\u2028\u2029\u202f\u205f\u3000"
                     + "".join(chr(c) for c in range(0x2000, 0x200B)))
SCAN_MAX_TOKEN = 1 << 20  # bufio.Scanner buffer limit set at tokenizer.go:101


class TokenizerError(ValueError):
    pass


@dataclasses.dataclass
class TokenizerConfig:
    """TokenizerConfig (tokenizer.go:15-32) with applyDefaults (:34-55)."""

    do_lower_case: bool = False
    tokenize_chinese_chars: bool = False
    max_input_chars_per_word: int = 0
    cls_token: str = ""
    sep_token: str = ""
    unk_token: str = ""
    pad_token: str = ""
    mask_token: str = ""

    @classmethod
    def from_dict(cls, d: dict) -> "TokenizerConfig":
        kw = {f.name: d[f.name] for f in dataclasses.fields(cls) if f.name in d}
        return cls(**kw)

    def with_defaults(self) -> "TokenizerConfig":
        c = dataclasses.replace(self)
        if c.max_input_chars_per_word == 0:
            c.max_input_chars_per_word = 100
        c.cls_token = c.cls_token or "[CLS]"
        c.sep_token = c.sep_token or "[SEP]"
        c.unk_token = c.unk_token or "[UNK]"
        c.pad_token = c.pad_token or "[PAD]"
        c.mask_token = c.mask_token or "[MASK]"
        return c


def parse_vocab(data: bytes) -> Tuple[Dict[bytes, int], int]:
    """NewTokenizer's scan (tokenizer.go:98-113): bufio.Scanner lines (split
    at LF, one trailing CR dropped, a final line without LF kept if
    non-empty), each trimmed of trailing CR/LF; line number = id, a repeated
    token keeps its last id. Returns (vocab, number of lines)."""
    lines = data.split(b"\n")
    if lines and lines[-1] == b"":
        lines.pop()
    for i, ln in enumerate(lines):
        terminated = i < len(lines) - 1 or data.endswith(b"\n")
        if len(ln) + (1 if terminated else 0) > SCAN_MAX_TOKEN:
            raise TokenizerError("tokenizer: scan vocab: bufio.Scanner: token too long")
    vocab: Dict[bytes, int] = {}
    for i, ln in enumerate(lines):
        vocab[ln.rstrip(b"\r\n")] = i
    return vocab, len(lines)


def go_lower(c: str) -> str:
    """unicode.ToLower: the simple lowercase mapping."""
    if c == "\u0130":
        return "i"
    lo = c.lower()
    return lo if len(lo) == 1 else c


def is_mn(c: str) -> bool:
    return unicodedata.category(c) == "Mn"


def is_whitespace(c: str) -> bool:
    """isWhitespace (tokenizer.go:318-326)."""
    return c in " \t\n\r" or unicodedata.category(c) == "Zs"


def is_control(c: str) -> bool:
    """isControl (tokenizer.go:328-337) over Go's category C."""
    if c in "\t\n\r":
        return False
    return unicodedata.category(c) in ("Cc", "Cf", "Co", "Cs")


def is_punct(c: str) -> bool:
    """isPunct (tokenizer.go:339-346)."""
    r = ord(c)
    if 33 <= r <= 47 or 58 <= r <= 64 or 91 <= r <= 96 or 123 <= r <= 126:
        return True
    return unicodedata.category(c).startswith("P")


def is_cjk(c: str) -> bool:
    """isCJK (tokenizer.go:348-361)."""
    r = ord(c)
    return (0x4E00 <= r <= 0x9FFF or 0x3400 <= r <= 0x4DBF or 0x20000 <= r <= 0x2A6DF
            or 0x2A700 <= r <= 0x2B73F or 0x2B740 <= r <= 0x2B81F or 0x2B820 <= r <= 0x2CEAF
            or 0xF900 <= r <= 0xFAFF or 0x2F800 <= r <= 0x2FA1F)


def _non_starters(c: str) -> Tuple[int, int]:
    """(leading, trailing) non-starter counts of c's canonical decomposition."""
    d = unicodedata.normalize("NFD", c)
    lead = 0
    while lead < len(d) and unicodedata.combining(d[lead]):
        lead += 1
    trail = 0
    while trail < len(d) and unicodedata.combining(d[len(d) - 1 - trail]):
        trail += 1
    return lead, trail


def nfd_stream_safe(s: str) -> str:
    """norm.NFD.String: NFD in the Stream-Safe Text Format (UAX #15 §13)."""
    out: List[str] = []
    start, ss = 0, 0
    for i, c in enumerate(s):
        lead, trail = _non_starters(c)
        if ss + lead > MAX_NON_STARTERS:
            out.append(unicodedata.normalize("NFD", s[start:i]))
            out.append(CGJ)
            start, ss = i, 0
        if lead == 0:
            ss = trail
        else:
            ss += lead
    out.append(unicodedata.normalize("NFD", s[start:]))
    return "".join(out)


def strip_accents(s: str) -> str:
    """stripAccents (tokenizer.go:304-316)."""
    return "".join(c for c in nfd_stream_safe(s) if not is_mn(c))


class Tokenizer:
    """Tokenizer (tokenizer.go:57-88) built like NewTokenizer (:90-136)."""

    def __init__(self, vocab_bytes: bytes, cfg: Optional[TokenizerConfig] = None):
        self.cfg = (cfg or TokenizerConfig()).with_defaults()
        self.vocab, nlines = parse_vocab(vocab_bytes)
        if nlines == 0:
            raise TokenizerError("tokenizer: vocab is empty")
        self.specials: List[Tuple[bytes, int]] = []
        ids = []
        for name in (self.cfg.cls_token, self.cfg.sep_token, self.cfg.unk_token,
                     self.cfg.pad_token, self.cfg.mask_token):
            key = name.encode()
            if key not in self.vocab:
                raise TokenizerError(f"tokenizer: special token {name!r} not in vocab")
            ids.append(self.vocab[key])
            self.specials.append((key, self.vocab[key]))
        self.cls_id, self.sep_id, self.unk_id, self.pad_id, self.mask_id = ids

    @classmethod
    def from_file(cls, path, cfg: Optional[TokenizerConfig] = None) -> "Tokenizer":
        with open(path, "rb") as f:
            return cls(f.read(), cfg)

    def vocab_size(self) -> int:
        """VocabSize (tokenizer.go:138): distinct tokens."""
        return len(self.vocab)

    def split_specials(self, text: bytes) -> List[Tuple[bytes, int]]:
        """splitSpecials (tokenizer.go:186-216) on the raw bytes."""
        segs: List[Tuple[bytes, int]] = []
        while text:
            best, best_id, best_len = -1, -1, 0
            for lit, sid in self.specials:
                i = text.find(lit)
                if i >= 0 and (best < 0 or i < best or (i == best and len(lit) > best_len)):
                    best, best_id, best_len = i, sid, len(lit)
            if best < 0:
                segs.append((text, -1))
                break
            if best > 0:
                segs.append((text[:best], -1))
            segs.append((b"", best_id))
            text = text[best + best_len:]
        return segs

    def basic_tokenize(self, text: bytes) -> List[str]:
        """basicTokenize (tokenizer.go:218-266)."""
        sb: List[str] = []
        for c in text.decode("utf-8", errors="replace"):
            if c == "\x00" or c == "\ufffd" or is_control(c):
                continue
            if is_whitespace(c):
                sb.append(" ")
            elif self.cfg.tokenize_chinese_chars and is_cjk(c):
                sb.append(" " + c + " ")
            else:
                sb.append(c)
        cleaned = "".join(sb)
        if self.cfg.do_lower_case:
            cleaned = strip_accents("".join(go_lower(c) for c in cleaned))
        words: List[str] = []

        def fields(s: str):
            cur: List[str] = []
            for c in s:
                if c in GO_SPACE:
                    if cur:
                        yield "".join(cur)
                        cur = []
                else:
                    cur.append(c)
            if cur:
                yield "".join(cur)

        for chunk_s in fields(cleaned):
            start = -1
            for i, c in enumerate(chunk_s):
                if is_punct(c):
                    if start >= 0:
                        words.append(chunk_s[start:i])
                        start = -1
                    words.append(c)
                elif start < 0:
                    start = i
            if start >= 0:
                words.append(chunk_s[start:])
        return words

    def word_piece(self, word: str) -> List[int]:
        """wordPiece (tokenizer.go:268-302): greedy longest match."""
        if len(word) > self.cfg.max_input_chars_per_word:
            return [self.unk_id]
        out: List[int] = []
        start = 0
        while start < len(word):
            end = len(word)
            cur = -1
            while end > start:
                sub = word[start:end].encode()
                if start > 0:
                    sub = b"##" + sub
                if sub in self.vocab:
                    cur = self.vocab[sub]
                    break
                end -= 1
            if cur < 0:
                return [self.unk_id]
            out.append(cur)
            start = end
        return out

    def encode(self, text, max_seq_len: int) -> List[int]:
        """Encode (tokenizer.go:143-184): [CLS] … [SEP], head-truncated so
        that len(ids) <= max(max_seq_len, 2)."""
        if isinstance(text, str):
            text = text.encode("utf-8", "surrogatepass")
        if max_seq_len < 2:
            max_seq_len = 2
        ids = [self.cls_id]
        budget = max_seq_len - 2
        done = False
        for seg, sid in self.split_specials(text):
            if sid >= 0:
                if len(ids) - 1 >= budget:
                    break
                ids.append(sid)
                continue
            for w in self.basic_tokenize(seg):
                if len(ids) - 1 >= budget:
                    done = True
                    break
                for p in self.word_piece(w):
                    if len(ids) - 1 >= budget:
                        done = True
                        break
                    ids.append(p)
                if done:
                    break
            if done:
                break
        ids.append(self.sep_id)
        return ids

    def encode_batch(self, texts: Sequence, max_seq_len: int):
        """Packed (ids int32 [Σ L], cu_seqlens int32 [n+1]) of Encode per text."""
        import numpy as np
        seqs = [self.encode(t, max_seq_len) for t in texts]
        cu = np.zeros(len(seqs) + 1, dtype=np.int32)
        cu[1:] = np.cumsum([len(s) for s in seqs])
        ids = np.fromiter((i for s in seqs for i in s), dtype=np.int32, count=int(cu[-1]))
        return ids, cu
