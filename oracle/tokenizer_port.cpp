// Compiled port of futon's WordPiece tokenizer — TEST INFRASTRUCTURE ONLY.
//
// The CPU baseline that bench.py times beside the library's tokenizer: the
// reference's algorithm in the reference's own structure (native/
// tokenizer.go), compiled, so its speed stands in for the Go tokenizer that
// cannot be built here (no Go toolchain). Like the Go code it makes separate
// passes that each build a new string (clean + CJK isolation, ToLower, NFD
// with x/text's quick check for text already in NFD, Mn removal), splits by
// substrings (Fields, punctuation), keeps the vocab in a hash map with
// string keys, and builds a new string for every WordPiece candidate. A batch
// runs on host threads that take texts from a shared counter, as EmbedBatch's
// workers do (provider.go:152-202). Its ids are checked against the
// reference's fixtures and the library's tokenizer in tests/test_tokenizer.py.
//
// Unicode data: unicode_tables.h from futon_b200/csrc/gen_unicode_tables.py
// (CPython unicodedata, Unicode 15.0.0), generated into _build/ by the
// Makefile. NFD as UAX #15 with its Stream-Safe Text Format, as
// golang.org/x/text v0.21.0's norm does.

#include "unicode_tables.h"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <string>
#include <string_view>
#include <thread>
#include <unordered_map>
#include <vector>

using namespace futon_uni;

namespace {

uint8_t flags(uint32_t r) {
  return kUniStage2[((uint32_t)kUniStage1[r >> kBlockShift] << kBlockShift) |
                    (r & ((1u << kBlockShift) - 1))];
}

template <size_t N>
uint32_t lookup(const uint32_t (&tab)[N][2], uint32_t r, uint32_t miss) {
  auto it = std::lower_bound(&tab[0], &tab[0] + N, r,
                             [](const uint32_t (&e)[2], uint32_t v) { return e[0] < v; });
  return (it != &tab[0] + N && (*it)[0] == r) ? (*it)[1] : miss;
}

uint8_t ccc(uint32_t r) { return (flags(r) & F_CCC) ? (uint8_t)lookup(kUniCcc, r, 0) : 0; }

// unicode.ToLower.
uint32_t to_lower(uint32_t r) {
  if (r < 0x80) return (r >= 'A' && r <= 'Z') ? r + 32 : r;
  return (flags(r) & F_LOWER) ? lookup(kUniLower, r, r) : r;
}

// utf8.DecodeRune: U+FFFD and width 1 for an invalid sequence.
uint32_t decode(std::string_view s, size_t i, size_t* w) {
  const uint8_t b0 = (uint8_t)s[i];
  *w = 1;
  if (b0 < 0x80) return b0;
  auto c = [&](size_t k, uint8_t lo = 0x80, uint8_t hi = 0xBF) {
    return i + k < s.size() && (uint8_t)s[i + k] >= lo && (uint8_t)s[i + k] <= hi;
  };
  if (b0 >= 0xC2 && b0 <= 0xDF && c(1)) {
    *w = 2;
    return ((b0 & 0x1Fu) << 6) | ((uint8_t)s[i + 1] & 0x3Fu);
  }
  if (b0 >= 0xE0 && b0 <= 0xEF && c(1, b0 == 0xE0 ? 0xA0 : 0x80, b0 == 0xED ? 0x9F : 0xBF) &&
      c(2)) {
    *w = 3;
    return ((b0 & 0x0Fu) << 12) | (((uint8_t)s[i + 1] & 0x3Fu) << 6) | ((uint8_t)s[i + 2] & 0x3Fu);
  }
  if (b0 >= 0xF0 && b0 <= 0xF4 && c(1, b0 == 0xF0 ? 0x90 : 0x80, b0 == 0xF4 ? 0x8F : 0xBF) &&
      c(2) && c(3)) {
    *w = 4;
    return ((b0 & 0x07u) << 18) | (((uint8_t)s[i + 1] & 0x3Fu) << 12) |
           (((uint8_t)s[i + 2] & 0x3Fu) << 6) | ((uint8_t)s[i + 3] & 0x3Fu);
  }
  return 0xFFFD;
}

std::vector<uint32_t> runes(std::string_view s) {
  std::vector<uint32_t> out;
  for (size_t i = 0, w; i < s.size(); i += w) out.push_back(decode(s, i, &w));
  return out;
}

void put(std::string& out, uint32_t r) {
  if (r < 0x80) {
    out += (char)r;
  } else if (r < 0x800) {
    out += (char)(0xC0 | (r >> 6));
    out += (char)(0x80 | (r & 0x3F));
  } else if (r < 0x10000) {
    out += (char)(0xE0 | (r >> 12));
    out += (char)(0x80 | ((r >> 6) & 0x3F));
    out += (char)(0x80 | (r & 0x3F));
  } else {
    out += (char)(0xF0 | (r >> 18));
    out += (char)(0x80 | ((r >> 12) & 0x3F));
    out += (char)(0x80 | ((r >> 6) & 0x3F));
    out += (char)(0x80 | (r & 0x3F));
  }
}

// Canonical decomposition of one rune (Hangul arithmetically).
std::vector<uint32_t> decomposition(uint32_t r) {
  if (r >= 0xAC00 && r <= 0xD7A3) {
    const uint32_t s = r - 0xAC00;
    std::vector<uint32_t> d{0x1100 + s / 588, 0x1161 + (s % 588) / 28};
    if (s % 28) d.push_back(0x11A7 + s % 28);
    return d;
  }
  if (flags(r) & F_DECOMP) {
    const size_t n = sizeof(kUniDecomp) / sizeof(kUniDecomp[0]);
    auto it = std::lower_bound(kUniDecomp, kUniDecomp + n, r,
                               [](const Decomp& e, uint32_t v) { return e.cp < v; });
    return std::vector<uint32_t>(kUniDecompData + it->off, kUniDecompData + it->off + it->len);
  }
  return {r};
}

// norm.NFD.String: decomposition, canonical ordering of each run of
// non-starters, a U+034F barrier once 30 non-starters follow a starter.
std::string nfd(std::string_view s) {
  bool done = true;  // the quick check: nothing decomposes, nothing combines
  for (size_t i = 0, w; i < s.size() && done; i += w) {
    const uint32_t r = decode(s, i, &w);
    done = !(flags(r) & (F_DECOMP | F_CCC)) && !(r >= 0xAC00 && r <= 0xD7A3);
  }
  if (done) return std::string(s);
  std::vector<uint32_t> out;
  size_t run = std::string::npos;
  auto close = [&]() {
    if (run != std::string::npos)
      std::stable_sort(out.begin() + run, out.end(),
                       [](uint32_t a, uint32_t b) { return ccc(a) < ccc(b); });
    run = std::string::npos;
  };
  int ss = 0;
  for (uint32_t r : runes(s)) {
    std::vector<uint32_t> d = decomposition(r);
    int lead = 0, trail = 0;
    while (lead < (int)d.size() && ccc(d[lead])) ++lead;
    while (trail < (int)d.size() && ccc(d[d.size() - 1 - trail])) ++trail;
    if (ss + lead > 30) {
      close();
      out.push_back(0x034F);
      ss = 0;
    }
    ss = lead == 0 ? trail : ss + lead;
    for (uint32_t x : d) {
      if (ccc(x) == 0) {
        close();
      } else if (run == std::string::npos) {
        run = out.size();
      }
      out.push_back(x);
    }
  }
  close();
  std::string res;
  for (uint32_t r : out) put(res, r);
  return res;
}

bool is_cjk(uint32_t r) {
  return (r >= 0x4E00 && r <= 0x9FFF) || (r >= 0x3400 && r <= 0x4DBF) ||
         (r >= 0x20000 && r <= 0x2A6DF) || (r >= 0x2A700 && r <= 0x2B73F) ||
         (r >= 0x2B740 && r <= 0x2B81F) || (r >= 0x2B820 && r <= 0x2CEAF) ||
         (r >= 0xF900 && r <= 0xFAFF) || (r >= 0x2F800 && r <= 0x2FA1F);
}

}  // namespace

struct TpTokenizer {
  std::unordered_map<std::string, int> vocab;
  bool lower = false, cjk = false;
  int max_chars = 100;
  int cls = -1, sep = -1, unk = -1;
  std::vector<std::pair<std::string, int>> specials;

  // basicTokenize (tokenizer.go:218-266).
  std::vector<std::string> basic_tokenize(std::string_view text) const {
    std::string sb;
    sb.reserve(text.size() + text.size() / 4);
    for (size_t i = 0, w; i < text.size(); i += w) {
      const uint32_t r = decode(text, i, &w);
      const uint8_t f = flags(r);
      const bool tnr = r == '\t' || r == '\n' || r == '\r';
      if (r == 0 || r == 0xFFFD || ((f & F_CTRL) && !tnr)) continue;
      if (tnr || r == ' ' || (f & F_ZS)) {
        sb += ' ';
      } else if (cjk && is_cjk(r)) {
        sb += ' ';
        put(sb, r);
        sb += ' ';
      } else {
        put(sb, r);
      }
    }
    std::string cleaned = sb;
    if (lower) {
      // strings.ToLower: ASCII lowered byte by byte, anything else rune by rune.
      std::string low;
      low.reserve(cleaned.size());
      for (size_t i = 0, w; i < cleaned.size(); i += w) {
        const uint32_t r = decode(cleaned, i, &w);
        put(low, to_lower(r));
      }
      const std::string d = nfd(low);  // stripAccents
      std::string stripped;
      stripped.reserve(d.size());
      for (size_t i = 0, w; i < d.size(); i += w) {
        const uint32_t r = decode(d, i, &w);
        if (!(flags(r) & F_MN)) stripped.append(d, i, w);
      }
      cleaned = std::move(stripped);
    }
    std::vector<std::string_view> chunks;  // strings.Fields: substrings
    const std::string_view cv(cleaned);
    size_t from = std::string_view::npos;
    for (size_t i = 0, w; i < cv.size(); i += w) {
      const uint32_t r = decode(cv, i, &w);
      if (flags(r) & F_SPACE) {
        if (from != std::string_view::npos) chunks.push_back(cv.substr(from, i - from));
        from = std::string_view::npos;
      } else if (from == std::string_view::npos) {
        from = i;
      }
    }
    if (from != std::string_view::npos) chunks.push_back(cv.substr(from));
    std::vector<std::string> words;
    for (std::string_view chunk : chunks) {
      size_t start = std::string_view::npos;
      for (size_t i = 0, w; i < chunk.size(); i += w) {
        const uint32_t r = decode(chunk, i, &w);
        if (flags(r) & F_PUNCT) {
          if (start != std::string_view::npos) words.emplace_back(chunk.substr(start, i - start));
          start = std::string_view::npos;
          words.emplace_back(chunk.substr(i, w));
        } else if (start == std::string_view::npos) {
          start = i;
        }
      }
      if (start != std::string_view::npos) words.emplace_back(chunk.substr(start));
    }
    return words;
  }

  // wordPiece (tokenizer.go:268-302).
  std::vector<int> word_piece(const std::string& word) const {
    const std::vector<uint32_t> rs = runes(word);
    if ((int)rs.size() > max_chars) return {unk};
    std::vector<int> out;
    size_t start = 0;
    while (start < rs.size()) {
      size_t end = rs.size();
      int id = -1;
      while (end > start) {
        std::string sub = start > 0 ? "##" : "";
        for (size_t k = start; k < end; ++k) put(sub, rs[k]);
        auto it = vocab.find(sub);
        if (it != vocab.end()) {
          id = it->second;
          break;
        }
        --end;
      }
      if (id < 0) return {unk};
      out.push_back(id);
      start = end;
    }
    return out;
  }

  // Encode (tokenizer.go:143-184) with splitSpecials (:186-216).
  std::vector<int> encode(std::string_view text, int max_seq_len) const {
    if (max_seq_len < 2) max_seq_len = 2;
    const size_t budget = (size_t)max_seq_len - 2;
    std::vector<int> ids{cls};
    std::vector<std::pair<std::string_view, int>> segs;
    while (!text.empty()) {
      size_t best = std::string_view::npos, best_len = 0;
      int best_id = -1;
      for (const auto& sp : specials) {
        const size_t i = text.find(sp.first);
        if (i != std::string_view::npos &&
            (best == std::string_view::npos || i < best || (i == best && sp.first.size() > best_len))) {
          best = i;
          best_len = sp.first.size();
          best_id = sp.second;
        }
      }
      if (best == std::string_view::npos) {
        segs.emplace_back(text, -1);
        break;
      }
      if (best > 0) segs.emplace_back(text.substr(0, best), -1);
      segs.emplace_back(std::string_view(), best_id);
      text = text.substr(best + best_len);
    }
    for (const auto& seg : segs) {
      if (seg.second >= 0) {
        if (ids.size() - 1 >= budget) break;
        ids.push_back(seg.second);
        continue;
      }
      for (const std::string& w : basic_tokenize(seg.first)) {
        if (ids.size() - 1 >= budget) goto done;
        for (int p : word_piece(w)) {
          if (ids.size() - 1 >= budget) goto done;
          ids.push_back(p);
        }
      }
    }
  done:
    ids.push_back(sep);
    return ids;
  }
};

extern "C" {

// NewTokenizer over vocab.txt's bytes with the default special tokens;
// returns NULL when the vocab is empty or lacks one of them.
TpTokenizer* tp_create(const char* vocab, size_t len, int lower, int cjk) {
  auto* t = new TpTokenizer();
  t->lower = lower != 0;
  t->cjk = cjk != 0;
  std::string_view v(vocab, len);
  int id = 0;
  while (!v.empty()) {
    const size_t nl = v.find('\n');
    std::string_view line = v.substr(0, nl);
    while (!line.empty() && (line.back() == '\r' || line.back() == '\n')) line.remove_suffix(1);
    t->vocab[std::string(line)] = id++;
    if (nl == std::string_view::npos) break;
    v.remove_prefix(nl + 1);
  }
  const char* names[5] = {"[CLS]", "[SEP]", "[UNK]", "[PAD]", "[MASK]"};
  int ids[5];
  for (int i = 0; i < 5; ++i) {
    auto it = t->vocab.find(names[i]);
    if (id == 0 || it == t->vocab.end()) {
      delete t;
      return nullptr;
    }
    ids[i] = it->second;
    t->specials.emplace_back(names[i], it->second);
  }
  t->cls = ids[0];
  t->sep = ids[1];
  t->unk = ids[2];
  return t;
}

void tp_destroy(TpTokenizer* t) { delete t; }

// Encode of every text on `threads` host threads; text i is
// text[off[i], off[i+1]). Writes cu[0..n] and the packed ids; returns the
// total, or -1 when it exceeds cap.
long long tp_encode_batch(const TpTokenizer* t, const char* text, const int64_t* off, int n,
                          int max_seq_len, int threads, int32_t* ids, long long cap,
                          int32_t* cu) {
  std::vector<std::vector<int>> res(n);
  std::atomic<int> next{0};
  auto work = [&]() {
    for (int i; (i = next.fetch_add(1)) < n;)
      res[i] = t->encode(std::string_view(text + off[i], (size_t)(off[i + 1] - off[i])),
                         max_seq_len);
  };
  std::vector<std::thread> pool;
  for (int k = 1; k < std::max(1, threads); ++k) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
  long long total = 0;
  cu[0] = 0;
  for (int i = 0; i < n; ++i) {
    total += (long long)res[i].size();
    cu[i + 1] = (int32_t)total;
  }
  if (total > cap) return -1;
  for (int i = 0; i < n; ++i) std::copy(res[i].begin(), res[i].end(), ids + cu[i]);
  return total;
}

}  // extern "C"
