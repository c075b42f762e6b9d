// Native WordPiece tokenizer: the text side of futon's native Provider
// (native/tokenizer.go), producing the packed ids + cu_seqlens that the
// encoder entry points take.
//
// Per text segment, one pass over the bytes does what the reference does in
// several string passes (tokenizer.go:218-266). ASCII bytes (most of any
// text) go through a 128-entry class table: no decoding, no Unicode tables.
// Each run of other bytes is decoded and cleaned on its own — NUL, U+FFFD
// and category-C runes but TAB/LF/CR dropped, whitespace (those three,
// space, Zs) turned into a space, CJK ideographs isolated, lowercased (simple
// mapping) — and, with lowercasing on, put through NFD + removal of Mn,
// skipped when no code point is at or above U+00C0 (none below decomposes or
// is a combining mark). The ASCII characters between runs are starters
// without decompositions, so NFD never reaches across them. Words are split
// on Go's unicode.IsSpace and on punctuation, and each word goes through
// greedy longest-match WordPiece (tokenizer.go:268-302) against two
// open-addressing tables: word-initial keys, and "##" continuation keys
// stored without the prefix, so no lookup builds a string. Candidate pieces
// longer than the table's longest key are skipped without a lookup (they
// cannot match).
//
// Unicode data (categories, lowercase, canonical decompositions, combining
// classes; Unicode 15.0.0 as in Go 1.23 and golang.org/x/text v0.21.0) comes
// from unicode_tables.h, generated at build time by gen_unicode_tables.py.
// NFD follows UAX #15 including its Stream-Safe Text Format (a U+034F
// barrier after 30 consecutive non-starters), as x/text's norm.NFD does.
//
// A batch is cut into chunks of 64 consecutive texts handed out to host
// threads through an atomic counter; each chunk's ids land in one buffer,
// and after the lengths' prefix sum every chunk is one contiguous copy into
// the caller's packed output. Results do not depend on the thread count.

#include "futon_cuda.h"
#include "futon_tokenizer.h"
#include "unicode_tables.h"

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <exception>
#include <limits>
#include <string_view>
#include <new>
#include <string>
#include <thread>
#include <vector>

using namespace futon_uni;

namespace {

void set_err(char* err, size_t errlen, const char* fmt, ...) {
  if (!err || errlen == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, errlen, fmt, ap);
  va_end(ap);
}

// ---- Unicode lookups -------------------------------------------------------

inline uint8_t uflags(uint32_t cp) {
  const uint32_t blk = kUniStage1[cp >> kBlockShift];
  return kUniStage2[(blk << kBlockShift) | (cp & ((1u << kBlockShift) - 1))];
}

template <size_t N>
inline uint32_t pair_lookup(const uint32_t (&tab)[N][2], uint32_t cp, uint32_t miss) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (tab[mid][0] < cp) lo = mid + 1; else hi = mid;
  }
  return (lo < N && tab[lo][0] == cp) ? tab[lo][1] : miss;
}

// unicode.ToLower (simple mapping).
inline uint32_t to_lower(uint32_t cp, uint8_t f) {
  if (cp < 0x80) return (cp >= 'A' && cp <= 'Z') ? cp + 32 : cp;
  return (f & F_LOWER) ? pair_lookup(kUniLower, cp, cp) : cp;
}

inline uint8_t ccc_of(uint32_t cp) {
  return (uflags(cp) & F_CCC) ? (uint8_t)pair_lookup(kUniCcc, cp, 0) : 0;
}

// Full canonical decomposition of cp into d (at most kUniMaxDecomp runes;
// Hangul syllables arithmetically, Unicode §3.12). Returns the rune count.
inline int decompose(uint32_t cp, uint32_t* d) {
  constexpr uint32_t kS = 0xAC00, kL = 0x1100, kV = 0x1161, kT = 0x11A7;
  constexpr uint32_t kVCount = 21, kTCount = 28, kSCount = 11172;
  if (cp - kS < kSCount) {
    const uint32_t s = cp - kS, t = s % kTCount;
    d[0] = kL + s / (kVCount * kTCount);
    d[1] = kV + (s % (kVCount * kTCount)) / kTCount;
    if (t == 0) return 2;
    d[2] = kT + t;
    return 3;
  }
  if (uflags(cp) & F_DECOMP) {
    const size_t n = sizeof(kUniDecomp) / sizeof(kUniDecomp[0]);
    size_t lo = 0, hi = n;
    while (lo < hi) {
      const size_t mid = (lo + hi) / 2;
      if (kUniDecomp[mid].cp < cp) lo = mid + 1; else hi = mid;
    }
    const Decomp& e = kUniDecomp[lo];
    for (int i = 0; i < e.len; ++i) d[i] = kUniDecompData[e.off + i];
    return e.len;
  }
  d[0] = cp;
  return 1;
}

inline bool is_cjk(uint32_t r) {
  return (r >= 0x4E00 && r <= 0x9FFF) || (r >= 0x3400 && r <= 0x4DBF) ||
         (r >= 0x20000 && r <= 0x2A6DF) || (r >= 0x2A700 && r <= 0x2B73F) ||
         (r >= 0x2B740 && r <= 0x2B81F) || (r >= 0x2B820 && r <= 0x2CEAF) ||
         (r >= 0xF900 && r <= 0xFAFF) || (r >= 0x2F800 && r <= 0x2FA1F);
}

// One rune of UTF-8 by Go's rules (utf8.DecodeRune): an invalid or truncated
// sequence yields U+FFFD and consumes one byte.
inline uint32_t decode_utf8(const uint8_t* s, size_t n, size_t* width) {
  const uint32_t b0 = s[0];
  *width = 1;
  if (b0 < 0x80) return b0;
  auto cont = [&](size_t i, uint32_t lo = 0x80, uint32_t hi = 0xBF) {
    return i < n && s[i] >= lo && s[i] <= hi;
  };
  if (b0 >= 0xC2 && b0 <= 0xDF) {
    if (!cont(1)) return 0xFFFD;
    *width = 2;
    return ((b0 & 0x1F) << 6) | (s[1] & 0x3F);
  }
  if (b0 >= 0xE0 && b0 <= 0xEF) {
    const uint32_t lo = b0 == 0xE0 ? 0xA0 : 0x80, hi = b0 == 0xED ? 0x9F : 0xBF;
    if (!cont(1, lo, hi) || !cont(2)) return 0xFFFD;
    *width = 3;
    return ((b0 & 0x0F) << 12) | ((s[1] & 0x3F) << 6) | (s[2] & 0x3F);
  }
  if (b0 >= 0xF0 && b0 <= 0xF4) {
    const uint32_t lo = b0 == 0xF0 ? 0x90 : 0x80, hi = b0 == 0xF4 ? 0x8F : 0xBF;
    if (!cont(1, lo, hi) || !cont(2) || !cont(3)) return 0xFFFD;
    *width = 4;
    return ((b0 & 0x07) << 18) | ((s[1] & 0x3F) << 12) | ((s[2] & 0x3F) << 6) | (s[3] & 0x3F);
  }
  return 0xFFFD;
}

inline void append_utf8(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out.push_back((char)cp);
  } else if (cp < 0x800) {
    out.push_back((char)(0xC0 | (cp >> 6)));
    out.push_back((char)(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out.push_back((char)(0xE0 | (cp >> 12)));
    out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (cp & 0x3F)));
  } else {
    out.push_back((char)(0xF0 | (cp >> 18)));
    out.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
    out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (cp & 0x3F)));
  }
}

// ---- Vocabulary table --------------------------------------------------------

// Open addressing over byte-string keys; linear probing.
class VocabTable {
 public:
  void reserve(size_t n) {
    size_t cap = 16;
    while (cap < 2 * n) cap <<= 1;
    slots_.assign(cap, Slot{0, -1, 0, {}});
    mask_ = cap - 1;
  }

  // Later inserts of the same key replace its id (a repeated vocab line
  // keeps the last id, like a Go map assignment).
  void assign(const char* p, size_t n, int32_t id) {
    const uint64_t h = hash(p, n);
    for (size_t i = h & mask_;; i = (i + 1) & mask_) {
      Slot& s = slots_[i];
      if (s.id < 0) {
        s.h = h;
        s.id = id;
        s.len = (uint32_t)n;
        if (n <= kInline) {
          memcpy(s.key, p, n);
        } else {
          const uint32_t off = (uint32_t)arena_.size();
          memcpy(s.key, &off, sizeof(off));
          arena_.append(p, n);
        }
        ++count_;
        max_len_ = std::max(max_len_, n);
        return;
      }
      if (same(s, h, p, n)) {
        s.id = id;
        return;
      }
    }
  }

  int32_t find(const char* p, size_t n) const {
    if (n > max_len_) return -1;
    const uint64_t h = hash(p, n);
    for (size_t i = h & mask_;; i = (i + 1) & mask_) {
      const Slot& s = slots_[i];
      if (s.id < 0) return -1;
      if (same(s, h, p, n)) return s.id;
    }
  }

  size_t count() const { return count_; }
  size_t max_len() const { return max_len_; }

 private:
  // Keys of up to kInline bytes sit in the slot itself (one cache line per
  // probe); longer ones in the arena, the slot holding their offset.
  static constexpr size_t kInline = 16;
  struct Slot {
    uint64_t h;
    int32_t id;
    uint32_t len;
    char key[kInline];
  };

  bool same(const Slot& s, uint64_t h, const char* p, size_t n) const {
    if (s.h != h || s.len != n) return false;
    if (n <= kInline) return memcmp(s.key, p, n) == 0;
    uint32_t off;
    memcpy(&off, s.key, sizeof(off));
    return memcmp(arena_.data() + off, p, n) == 0;
  }

  // The last n < 8 bytes as one word, from fixed-size loads (a variable-size
  // copy would be a library call per lookup). For a given n the value
  // determines the bytes: two overlapping 4-byte loads cover n = 4..7, and
  // bytes 0, n/2 and n-1 cover n = 1..3.
  static uint64_t tail(const char* p, size_t n) {
    if (n >= 4) {
      uint32_t a, b;
      memcpy(&a, p, 4);
      memcpy(&b, p + n - 4, 4);
      return (uint64_t)a | ((uint64_t)b << 32);
    }
    if (n == 0) return 0;
    return (uint64_t)(uint8_t)p[0] | ((uint64_t)(uint8_t)p[n >> 1] << 8) |
           ((uint64_t)(uint8_t)p[n - 1] << 16);
  }

  // One multiply-xorshift per 8 bytes; the final fold brings the high bits
  // into the low ones that index the slots. Lookups compare whole keys, so
  // the hash only has to spread them.
  static uint64_t hash(const char* p, size_t n) {
    uint64_t h = 0x9E3779B97F4A7C15ull ^ ((uint64_t)n << 56);
    while (n >= 8) {
      uint64_t v;
      memcpy(&v, p, 8);
      h = (h ^ v) * 0xBF58476D1CE4E5B9ull;
      h ^= h >> 29;
      p += 8;
      n -= 8;
    }
    h = (h ^ tail(p, n)) * 0x94D049BB133111EBull;
    return h ^ (h >> 32);
  }

  std::vector<Slot> slots_;
  std::string arena_;
  size_t mask_ = 0, count_ = 0, max_len_ = 0;
};

// ---- Tokenizer -----------------------------------------------------------------

constexpr int kMaxNonStarters = 30;  // UAX #15 Stream-Safe Text Format
constexpr uint32_t kCGJ = 0x034F;
constexpr size_t kScanMaxToken = (size_t)1 << 20;  // bufio.Scanner limit, tokenizer.go:101

struct Scratch {
  std::vector<uint32_t> cps, nfd;
  std::vector<uint8_t> ccc;
  std::string word;
  std::vector<uint32_t> bounds;  // byte offset of each rune of `word`, plus its end
  std::vector<int32_t> pieces;
};

struct Special {
  std::string lit;
  int32_t id;
};

// What the cleaning step and the split make of an ASCII byte: dropped (NUL
// and the other C0 controls but TAB/LF/CR, and DEL), a word separator
// (space, TAB, LF, CR), a punctuation word of its own (the four ASCII
// symbol/punctuation ranges of isPunct), or a word character. ASCII text
// has nothing to decompose and no combining marks, so NFD is the identity.
enum AsciiClass : uint8_t { kDrop, kSep, kPunct, kWordChar };

struct AsciiTable {
  uint8_t cls[128];
  char lower[128];  // unicode.ToLower on ASCII
  constexpr AsciiTable() : cls{}, lower{} {
    for (int c = 0; c < 128; ++c) {
      if (c == ' ' || c == '\t' || c == '\n' || c == '\r') cls[c] = kSep;
      else if (c < 32 || c == 127) cls[c] = kDrop;
      else if ((c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) ||
               (c >= 123 && c <= 126)) cls[c] = kPunct;
      else cls[c] = kWordChar;
      lower[c] = (char)((c >= 'A' && c <= 'Z') ? c + 32 : c);
    }
  }
};
constexpr AsciiTable kAscii;

}  // namespace

struct futon_tokenizer {
  bool lower = false, cjk = false;
  int max_chars = 100;
  VocabTable initial, cont;
  int32_t cls = 0, sep = 0, unk = 0, pad = 0, mask = 0;
  std::vector<Special> specials;

  void nfd_strip(Scratch& sc) const;
  void word_piece(const char* w, const uint32_t* b, size_t nr,
                  std::vector<int32_t>& pieces) const;
  bool emit_word(const char* w, const uint32_t* b, size_t nr, Scratch& sc,
                 std::vector<int32_t>& ids, size_t budget) const;
  bool clean_run(const uint8_t* s, size_t n, Scratch& sc) const;
  bool encode_text(const uint8_t* s, size_t n, Scratch& sc, std::vector<int32_t>& ids,
                   size_t budget) const;
  void encode(const uint8_t* s, size_t n, int max_seq_len, Scratch& sc,
              std::vector<int32_t>& ids) const;
};

// stripAccents (tokenizer.go:304-316): NFD of sc.cps, then every Mn rune
// removed. Canonical ordering is a stable sort of each run of non-starters
// by combining class; the stream-safe barrier ends a run after 30
// non-starters (counted per input rune from its decomposition's leading and
// trailing non-starters).
void futon_tokenizer::nfd_strip(Scratch& sc) const {
  std::vector<uint32_t>& out = sc.nfd;
  std::vector<uint8_t>& cc = sc.ccc;
  out.clear();
  cc.clear();
  size_t run = SIZE_MAX;
  auto close_run = [&]() {
    if (run == SIZE_MAX) return;
    for (size_t i = run + 1; i < out.size(); ++i) {
      const uint32_t v = out[i];
      const uint8_t c = cc[i];
      size_t j = i;
      while (j > run && cc[j - 1] > c) {
        out[j] = out[j - 1];
        cc[j] = cc[j - 1];
        --j;
      }
      out[j] = v;
      cc[j] = c;
    }
    run = SIZE_MAX;
  };
  int ss = 0;
  uint32_t d[4];
  uint8_t c[4];
  static_assert(kUniMaxDecomp <= 4, "decomposition buffer");
  for (uint32_t cp : sc.cps) {
    const int n = decompose(cp, d);
    for (int i = 0; i < n; ++i) c[i] = ccc_of(d[i]);
    int lead = 0, trail = 0;
    while (lead < n && c[lead]) ++lead;
    while (trail < n && c[n - 1 - trail]) ++trail;
    if (ss + lead > kMaxNonStarters) {
      close_run();
      out.push_back(kCGJ);
      cc.push_back(0);
      ss = 0;
    }
    ss = lead == 0 ? trail : ss + lead;
    for (int i = 0; i < n; ++i) {
      if (c[i] == 0) {
        close_run();
      } else if (run == SIZE_MAX) {
        run = out.size();
      }
      out.push_back(d[i]);
      cc.push_back(c[i]);
    }
  }
  close_run();
  size_t k = 0;
  for (uint32_t cp : out)
    if (!(uflags(cp) & F_MN)) out[k++] = cp;
  out.resize(k);
  sc.cps.swap(out);
}

// wordPiece (tokenizer.go:268-302) of the nr-rune word w into pieces. b holds
// the byte offset of each rune plus the word's end; b == nullptr means one
// byte per rune (an ASCII word).
void futon_tokenizer::word_piece(const char* w, const uint32_t* b, size_t nr,
                                 std::vector<int32_t>& pieces) const {
  pieces.clear();
  if (nr > (size_t)max_chars) {
    pieces.push_back(unk);
    return;
  }
  auto off = [b](size_t i) -> size_t { return b ? b[i] : i; };
  size_t start = 0;
  while (start < nr) {
    const VocabTable& tab = start > 0 ? cont : initial;
    const size_t lim = tab.max_len();
    size_t end = nr;
    while (end > start && off(end) - off(start) > lim) --end;
    int32_t id = -1;
    for (; end > start; --end) {
      id = tab.find(w + off(start), off(end) - off(start));
      if (id >= 0) break;
    }
    if (id < 0) {
      pieces.clear();
      pieces.push_back(unk);
      return;
    }
    pieces.push_back(id);
    start = end;
  }
}

// The per-word step of Encode's loop (tokenizer.go:166-176): stop before the
// word, or before any of its pieces, once the id budget is spent. Returns
// false then.
bool futon_tokenizer::emit_word(const char* w, const uint32_t* b, size_t nr, Scratch& sc,
                                std::vector<int32_t>& ids, size_t budget) const {
  if (ids.size() - 1 >= budget) return false;
  word_piece(w, b, nr, sc.pieces);
  for (int32_t p : sc.pieces) {
    if (ids.size() - 1 >= budget) return false;
    ids.push_back(p);
  }
  return true;
}

// Cleaning (tokenizer.go:224-239) and lowercasing of the code points of
// s[0, n) into sc.cps: NUL, U+FFFD and category-C runes but TAB/LF/CR are
// dropped, TAB/LF/CR/space/Zs become a space, CJK ideographs are isolated
// by spaces. Returns whether a code point at or above U+00C0 was kept (none
// below decomposes or is a combining mark, so NFD can be skipped without).
bool futon_tokenizer::clean_run(const uint8_t* s, size_t n, Scratch& sc) const {
  std::vector<uint32_t>& cps = sc.cps;
  cps.clear();
  bool wide = false;
  for (size_t i = 0; i < n;) {
    size_t w;
    const uint32_t r = decode_utf8(s + i, n - i, &w);
    i += w;
    if (r == 0 || r == 0xFFFD) continue;
    const uint8_t f = uflags(r);
    const bool tnr = r == '\t' || r == '\n' || r == '\r';
    if ((f & F_CTRL) && !tnr) continue;
    if (tnr || r == ' ' || (f & F_ZS)) {
      cps.push_back(' ');
    } else if (cjk && is_cjk(r)) {
      cps.push_back(' ');
      cps.push_back(r);
      cps.push_back(' ');
      wide = true;
    } else {
      const uint32_t v = lower ? to_lower(r, f) : r;
      wide |= v >= 0xC0;
      cps.push_back(v);
    }
  }
  return wide;
}

// basicTokenize + the WordPiece loop of Encode (tokenizer.go:158-178) for one
// text segment, in one pass over its bytes. ASCII bytes go through a
// 128-entry class table (no decoding, no Unicode tables; words are built
// in place). A run of other bytes, together with any ASCII controls inside
// it (the cleaning step removes those before NFD sees the text), is
// decoded and cleaned by clean_run and, with lowercasing on, put through
// NFD and Mn removal on its own: every ASCII character that survives
// cleaning is a starter without a decomposition, so NFD's reordering and
// its stream-safe count cannot reach across one. Words are then split on
// Go's unicode.IsSpace and on punctuation. Returns false once the id budget
// is spent.
bool futon_tokenizer::encode_text(const uint8_t* s, size_t n, Scratch& sc,
                                  std::vector<int32_t>& ids, size_t budget) const {
  std::string& word = sc.word;
  std::vector<uint32_t>& bounds = sc.bounds;
  word.clear();
  bounds.clear();
  bool multi = false;  // the word holds a multi-byte rune: bounds are kept
  auto flush = [&]() -> bool {
    if (word.empty()) return true;
    bool ok;
    if (multi) {
      bounds.push_back((uint32_t)word.size());
      ok = emit_word(word.data(), bounds.data(), bounds.size() - 1, sc, ids, budget);
    } else {
      ok = emit_word(word.data(), nullptr, word.size(), sc, ids, budget);
    }
    word.clear();
    bounds.clear();
    multi = false;
    return ok;
  };
  auto append_rune = [&](uint32_t cp) {
    if (cp < 0x80 && !multi) {
      word.push_back((char)cp);
      return;
    }
    if (!multi) {  // the ASCII prefix so far: one rune per byte
      bounds.resize(word.size());
      for (size_t k = 0; k < word.size(); ++k) bounds[k] = (uint32_t)k;
      multi = true;
    }
    bounds.push_back((uint32_t)word.size());
    append_utf8(word, cp);
  };
  for (size_t i = 0; i < n;) {
    const uint8_t c = s[i];
    if (c < 0x80) {
      const uint8_t k = kAscii.cls[c];
      if (k == kWordChar) {
        size_t j = i + 1;
        while (j < n && s[j] < 0x80 && kAscii.cls[s[j]] == kWordChar) ++j;
        if (!multi) {
          const size_t old = word.size();
          word.resize(old + (j - i));
          char* d = &word[old];
          if (lower) {
            for (size_t t = i; t < j; ++t) *d++ = kAscii.lower[s[t]];
          } else {
            memcpy(d, s + i, j - i);
          }
        } else {
          for (size_t t = i; t < j; ++t) {
            bounds.push_back((uint32_t)word.size());
            word.push_back(lower ? kAscii.lower[s[t]] : (char)s[t]);
          }
        }
        i = j;
        continue;
      }
      ++i;
      if (k == kDrop) continue;
      if (!flush()) return false;
      if (k == kPunct) {
        word.push_back((char)c);
        if (!flush()) return false;
      }
      continue;
    }
    size_t j = i + 1;
    while (j < n && (s[j] >= 0x80 || kAscii.cls[s[j]] == kDrop)) ++j;
    if (clean_run(s + i, j - i, sc) && lower) nfd_strip(sc);
    for (uint32_t cp : sc.cps) {
      const uint8_t f = uflags(cp);
      if (f & F_SPACE) {
        if (!flush()) return false;
      } else if (f & F_PUNCT) {
        if (!flush()) return false;
        append_rune(cp);
        if (!flush()) return false;
      } else {
        append_rune(cp);
      }
    }
    i = j;
  }
  return flush();
}

// Encode (tokenizer.go:143-184) with splitSpecials (:186-216) over the raw
// bytes: leftmost literal match, the longer literal at a tie; each literal's
// next occurrence is cached until the scan passes it.
void futon_tokenizer::encode(const uint8_t* s, size_t n, int max_seq_len, Scratch& sc,
                             std::vector<int32_t>& ids) const {
  if (max_seq_len < 2) max_seq_len = 2;
  const size_t budget = (size_t)max_seq_len - 2;
  ids.clear();
  ids.push_back(cls);
  const std::string_view text((const char*)s, n);
  size_t next[5];
  const size_t nsp = specials.size();
  for (size_t k = 0; k < nsp; ++k) next[k] = text.find(specials[k].lit);
  size_t pos = 0;
  while (pos < n) {
    size_t best = std::string_view::npos, best_len = 0;
    int32_t best_id = -1;
    for (size_t k = 0; k < nsp; ++k) {
      if (next[k] != std::string_view::npos && next[k] < pos) next[k] = text.find(specials[k].lit, pos);
      const size_t i = next[k];
      const size_t len = specials[k].lit.size();
      if (i != std::string_view::npos && (best == std::string_view::npos || i < best ||
                                          (i == best && len > best_len))) {
        best = i;
        best_len = len;
        best_id = specials[k].id;
      }
    }
    if (best == std::string_view::npos) {
      encode_text(s + pos, n - pos, sc, ids, budget);
      break;
    }
    if (best > pos && !encode_text(s + pos, best - pos, sc, ids, budget)) break;
    if (ids.size() - 1 >= budget) break;
    ids.push_back(best_id);
    pos = best + best_len;
  }
  ids.push_back(sep);
}

extern "C" {

int futon_tokenizer_create(const char* vocab, size_t vocab_len, const futon_tokenizer_cfg* cfg,
                           futon_tokenizer** out, char* err, size_t errlen) {
  if (!out || (!vocab && vocab_len)) {
    set_err(err, errlen, "tokenizer: null argument");
    return FUTON_EINVAL;
  }
  *out = nullptr;
  try {
    auto* t = new futon_tokenizer();
    futon_tokenizer_cfg c = cfg ? *cfg : futon_tokenizer_cfg{};
    t->lower = c.do_lower_case != 0;
    t->cjk = c.tokenize_chinese_chars != 0;
    t->max_chars = c.max_input_chars_per_word != 0 ? c.max_input_chars_per_word : 100;
    // bufio.Scanner lines: split at LF; a final line without LF counts if
    // non-empty; each token is the line with trailing CR/LF trimmed.
    std::vector<std::pair<size_t, size_t>> lines;
    size_t p = 0;
    while (p < vocab_len) {
      const char* nl = (const char*)memchr(vocab + p, '\n', vocab_len - p);
      const size_t e = nl ? (size_t)(nl - vocab) : vocab_len;
      if (e - p + (nl ? 1 : 0) > kScanMaxToken) {
        delete t;
        set_err(err, errlen, "tokenizer: scan vocab: bufio.Scanner: token too long");
        return FUTON_EINVAL;
      }
      size_t q = e;
      while (q > p && (vocab[q - 1] == '\r' || vocab[q - 1] == '\n')) --q;
      lines.emplace_back(p, q - p);
      p = e + 1;
    }
    if (lines.empty()) {
      delete t;
      set_err(err, errlen, "tokenizer: vocab is empty");
      return FUTON_EINVAL;
    }
    t->initial.reserve(lines.size());
    t->cont.reserve(lines.size());
    for (size_t id = 0; id < lines.size(); ++id) {
      const char* k = vocab + lines[id].first;
      const size_t n = lines[id].second;
      t->initial.assign(k, n, (int32_t)id);
      if (n >= 2 && k[0] == '#' && k[1] == '#') t->cont.assign(k + 2, n - 2, (int32_t)id);
    }
    const char* names[5] = {c.cls_token, c.sep_token, c.unk_token, c.pad_token, c.mask_token};
    const char* defaults[5] = {"[CLS]", "[SEP]", "[UNK]", "[PAD]", "[MASK]"};
    int32_t* dst[5] = {&t->cls, &t->sep, &t->unk, &t->pad, &t->mask};
    for (int i = 0; i < 5; ++i) {
      const char* nm = (names[i] && names[i][0]) ? names[i] : defaults[i];
      const int32_t id = t->initial.find(nm, strlen(nm));
      if (id < 0) {
        delete t;
        set_err(err, errlen, "tokenizer: special token \"%s\" not in vocab", nm);
        return FUTON_EINVAL;
      }
      *dst[i] = id;
      t->specials.push_back(Special{nm, id});
    }
    *out = t;
    return FUTON_OK;
  } catch (const std::bad_alloc&) {
    set_err(err, errlen, "tokenizer: out of host memory");
    return FUTON_ENOMEM;
  }
}

void futon_tokenizer_destroy(futon_tokenizer* tok) { delete tok; }

int futon_tokenizer_vocab_size(const futon_tokenizer* tok) {
  return tok ? (int)tok->initial.count() : -1;
}

int futon_tokenizer_pad_id(const futon_tokenizer* tok) { return tok ? tok->pad : -1; }

int futon_tokenizer_encode(const futon_tokenizer* tok, const char* text, size_t len,
                           int max_seq_len, int32_t* ids, int cap, int* n_ids, char* err,
                           size_t errlen) {
  if (!tok || (!text && len) || !n_ids || (!ids && cap > 0) || cap < 0) {
    set_err(err, errlen, "tokenizer: null or negative argument");
    return FUTON_EINVAL;
  }
  try {
    Scratch sc;
    std::vector<int32_t> out;
    tok->encode((const uint8_t*)text, len, max_seq_len, sc, out);
    *n_ids = (int)out.size();
    if (out.size() > (size_t)cap) {
      set_err(err, errlen, "tokenizer: %zu ids do not fit in cap %d", out.size(), cap);
      return FUTON_EINVAL;
    }
    memcpy(ids, out.data(), out.size() * sizeof(int32_t));
    return FUTON_OK;
  } catch (const std::bad_alloc&) {
    set_err(err, errlen, "tokenizer: out of host memory");
    return FUTON_ENOMEM;
  }
}

int futon_tokenizer_encode_batch(const futon_tokenizer* tok, const char* text,
                                 const int64_t* text_offsets, int ntexts, int max_seq_len,
                                 int nthreads, int32_t* ids, int64_t ids_cap,
                                 int32_t* cu_seqlens, char* err, size_t errlen) {
  if (!tok || ntexts < 0 || !cu_seqlens || (ntexts > 0 && !text_offsets) || ids_cap < 0 ||
      (!ids && ids_cap > 0)) {
    set_err(err, errlen, "tokenizer: null or negative argument");
    return FUTON_EINVAL;
  }
  if (ntexts > 0 && text_offsets[0] < 0) {
    set_err(err, errlen, "tokenizer: text_offsets[0] = %lld < 0", (long long)text_offsets[0]);
    return FUTON_EINVAL;
  }
  for (int i = 0; i < ntexts; ++i) {
    if (text_offsets[i + 1] < text_offsets[i]) {
      set_err(err, errlen, "tokenizer: text_offsets decrease at text %d", i);
      return FUTON_EINVAL;
    }
  }
  if (ntexts > 0 && !text && text_offsets[ntexts] > text_offsets[0]) {
    set_err(err, errlen, "tokenizer: null text with non-empty offsets");
    return FUTON_EINVAL;
  }
  cu_seqlens[0] = 0;
  if (ntexts == 0) return FUTON_OK;

  constexpr int kChunk = 64;
  const int nchunks = (ntexts + kChunk - 1) / kChunk;
  int hw = nthreads > 0 ? nthreads : (int)std::thread::hardware_concurrency();
  const int workers = std::max(1, std::min(hw, nchunks));
  try {
    std::vector<std::vector<int32_t>> chunk_ids(nchunks);
    std::vector<int32_t> lens(ntexts);
    std::atomic<int> next{0};
    std::atomic<bool> oom{false};
    auto tokenize = [&]() {
      try {
        Scratch sc;
        std::vector<int32_t> one;
        for (int c; (c = next.fetch_add(1)) < nchunks;) {
          std::vector<int32_t>& dst = chunk_ids[c];
          const int lo = c * kChunk, hi = std::min(ntexts, lo + kChunk);
          for (int i = lo; i < hi; ++i) {
            const int64_t a = text_offsets[i], b = text_offsets[i + 1];
            tok->encode((const uint8_t*)text + a, (size_t)(b - a), max_seq_len, sc, one);
            lens[i] = (int32_t)one.size();
            dst.insert(dst.end(), one.begin(), one.end());
          }
        }
      } catch (const std::bad_alloc&) {
        oom = true;
        next = nchunks;
      }
    };
    // The calling thread works too, and the atomic counter hands out every
    // chunk, so a thread that cannot be started only leaves fewer workers.
    auto run = [&](auto&& body) {
      std::vector<std::thread> pool;
      try {
        pool.reserve(workers - 1);
        for (int w = 1; w < workers; ++w) pool.emplace_back(body);
      } catch (const std::exception&) {
      }
      body();
      for (auto& th : pool) th.join();
    };
    run(tokenize);
    if (oom) {
      set_err(err, errlen, "tokenizer: out of host memory");
      return FUTON_ENOMEM;
    }
    int64_t total = 0;
    for (int i = 0; i < ntexts; ++i) total += lens[i];
    if (total > std::numeric_limits<int32_t>::max()) {
      set_err(err, errlen, "tokenizer: %lld ids exceed the int32 cu_seqlens range",
              (long long)total);
      return FUTON_EINVAL;
    }
    for (int i = 0; i < ntexts; ++i) cu_seqlens[i + 1] = cu_seqlens[i] + lens[i];
    if (total > ids_cap) {
      set_err(err, errlen, "tokenizer: %lld ids do not fit in ids_cap %lld", (long long)total,
              (long long)ids_cap);
      return FUTON_EINVAL;
    }
    next = 0;
    run([&]() {
      for (int c; (c = next.fetch_add(1)) < nchunks;) {
        const std::vector<int32_t>& src = chunk_ids[c];
        if (!src.empty())
          memcpy(ids + cu_seqlens[c * kChunk], src.data(), src.size() * sizeof(int32_t));
      }
    });
    return FUTON_OK;
  } catch (const std::bad_alloc&) {
    set_err(err, errlen, "tokenizer: out of host memory");
    return FUTON_ENOMEM;
  }
}

}  // extern "C"
