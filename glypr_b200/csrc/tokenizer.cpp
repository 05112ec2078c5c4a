// Text front end: glypr's GGUF tokenizer and task prompts, on the host in C++.
//
// The reference tokenises on the host with the `tokenizers` crate 0.22.2 (Cargo.lock:3151-3153),
// configured by GlyprTokenizer::from_gguf_metadata (crates/glypr-core/src/tokenizer.rs:77-138):
// a byte-level-fallback BPE over the GGUF vocabulary (`tokenizer.ggml.tokens`) and merges
// (`tokenizer.ggml.merges`), unknown token "<unk>" with consecutive unknowns fused, the
// normaliser Replace(' ' -> U+2581) and the pre-tokeniser Split(' ', MergedWithPrevious) — which
// finds no ' ' once the normaliser has run, so every text is one BPE word.  This file restates
// the crate's published algorithm:
//
//   * build (models/bpe/model.rs BPE::build): vocabulary token -> index (a later duplicate
//     wins, as in the reference's hash-map insert), merge map (left id, right id) ->
//     (rank = position in the list, id of the concatenation), a later duplicate pair winning;
//     a merge part or concatenation missing from the vocabulary fails the build;
//   * merge_word: one symbol per code point; a code point without a token falls back to its
//     UTF-8 bytes as "<0xXX>" tokens when all exist, else becomes the unknown token, consecutive
//     unknowns fused into one (a byte fallback leaves a pending unknown pending: it is emitted
//     at the next known code point or at the end, as the crate does);
//   * Word::merge_all (models/bpe/word.rs): a min-heap of candidate merges keyed by (rank,
//     position); an entry whose position no longer holds a mergeable pair with the same result
//     is dropped; each merge pushes the new pairs with its left and right neighbours.
//
// On top of it, the three sequence forms the reference builds from a text (glp_tokenize), the
// batch form with its per-item limit (encode_batch_padded_with_limit, tokenizer.rs:182-222),
// and the prompt formatters (tokenizer.rs:13-64, 144-160; task.rs:21-73) with Rust's
// str::to_lowercase (Unicode full lowercase + Final_Sigma; tables in unicode_case.inc).
//
// Strings crossing the C ABI are UTF-8 (Rust &str): invalid UTF-8 is rejected.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>
#include <string_view>
#include <thread>
#include <unordered_map>
#include <vector>

#include "glypr_cuda.h"
#include "gguf.h"

namespace glp {
void set_last_error(const std::string& msg);  // glypr_cuda.cu: this thread's glp_last_error()
}

namespace {

constexpr int32_t kTokenPad = 0, kTokenEos = 1, kTokenBos = 2;  // tokenizer.rs:588-590

// ------------------------------------------------------------------------------------- UTF-8
// Decodes one code point; returns its byte length, or 0 for an ill-formed sequence (overlong,
// surrogate, above U+10FFFF, truncated), the set Rust's &str excludes.
int utf8_decode(const unsigned char* p, size_t n, uint32_t* cp) {
  const unsigned c = p[0];
  if (c < 0x80) {
    *cp = c;
    return 1;
  }
  int len;
  uint32_t v, min;
  if ((c & 0xE0) == 0xC0) {
    len = 2, v = c & 0x1F, min = 0x80;
  } else if ((c & 0xF0) == 0xE0) {
    len = 3, v = c & 0x0F, min = 0x800;
  } else if ((c & 0xF8) == 0xF0) {
    len = 4, v = c & 0x07, min = 0x10000;
  } else {
    return 0;
  }
  if (n < static_cast<size_t>(len)) return 0;
  for (int i = 1; i < len; ++i) {
    if ((p[i] & 0xC0) != 0x80) return 0;
    v = (v << 6) | (p[i] & 0x3F);
  }
  if (v < min || v > 0x10FFFF || (v >= 0xD800 && v <= 0xDFFF)) return 0;
  *cp = v;
  return len;
}

bool utf8_valid(const char* s, size_t n) {
  const auto* p = reinterpret_cast<const unsigned char*>(s);
  for (size_t i = 0; i < n;) {
    uint32_t cp;
    const int l = utf8_decode(p + i, n - i, &cp);
    if (!l) return false;
    i += l;
  }
  return true;
}

void utf8_append(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out.push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
    out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
    out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
    out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

std::vector<uint32_t> utf8_code_points(std::string_view s) {
  std::vector<uint32_t> cps;
  cps.reserve(s.size());
  const auto* p = reinterpret_cast<const unsigned char*>(s.data());
  for (size_t i = 0; i < s.size();) {
    uint32_t cp = 0xFFFD;
    const int l = utf8_decode(p + i, s.size() - i, &cp);
    cps.push_back(cp);
    i += l ? l : 1;
  }
  return cps;
}

// ------------------------------------------------------------------ Rust str::to_lowercase
struct LowerRun {
  uint32_t first;
  uint16_t count, stride;
  int32_t delta;
};
struct CpRange {
  uint32_t first, last;
};
#include "unicode_case.inc"

template <size_t N>
bool in_ranges(const CpRange (&r)[N], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (r[mid].last < cp)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo < N && r[lo].first <= cp;
}

uint32_t lower_simple(uint32_t cp) {
  size_t lo = 0, hi = sizeof(kLowerRuns) / sizeof(kLowerRuns[0]);
  while (lo < hi) {  // last run with first <= cp
    const size_t mid = (lo + hi) / 2;
    if (kLowerRuns[mid].first <= cp)
      lo = mid + 1;
    else
      hi = mid;
  }
  if (lo == 0) return cp;
  const LowerRun& r = kLowerRuns[lo - 1];
  const uint32_t off = cp - r.first;
  if (off % r.stride || off / r.stride >= r.count) return cp;
  return static_cast<uint32_t>(static_cast<int64_t>(cp) + r.delta);
}

bool case_ignorable(uint32_t cp) { return in_ranges(kCaseIgnorable, cp); }
bool cased(uint32_t cp) { return in_ranges(kCased, cp); }

std::string to_lowercase(std::string_view s) {
  const std::vector<uint32_t> cps = utf8_code_points(s);
  std::string out;
  out.reserve(s.size());
  const auto preceded_by_cased = [&](size_t i) {  // case-ignorables skipped, then a cased one
    while (i > 0 && case_ignorable(cps[i - 1])) --i;
    return i > 0 && cased(cps[i - 1]);
  };
  const auto followed_by_cased = [&](size_t i) {
    ++i;
    while (i < cps.size() && case_ignorable(cps[i])) ++i;
    return i < cps.size() && cased(cps[i]);
  };
  for (size_t i = 0; i < cps.size(); ++i) {
    const uint32_t cp = cps[i];
    if (cp == 0x3A3) {  // Final_Sigma
      utf8_append(out, preceded_by_cased(i) && !followed_by_cased(i) ? 0x3C2 : 0x3C3);
    } else if (cp == 0x130) {  // the one multi-code-point lowercase
      utf8_append(out, 0x69);
      utf8_append(out, 0x307);
    } else {
      utf8_append(out, lower_simple(cp));
    }
  }
  return out;
}

// name.to_lowercase().replace(['-', '_', ' '], "")  (task.rs:55, tokenizer.rs:145)
std::string task_key(std::string_view name) {
  std::string low = to_lowercase(name), key;
  for (char c : low)
    if (c != '-' && c != '_' && c != ' ') key.push_back(c);
  return key;
}

// ----------------------------------------------------------------------------- hash tables
// Open addressing over 64-bit keys (merge pairs, single-code-point tokens).
class FlatMap {
 public:
  void reserve(size_t n) {
    size_t cap = 16;
    while (cap < 2 * n) cap <<= 1;
    keys_.assign(cap, kEmpty);
    vals_.assign(cap, 0);
    mask_ = cap - 1;
  }
  void put(uint64_t k, uint64_t v) {
    size_t i = slot(k);
    while (keys_[i] != kEmpty && keys_[i] != k) i = (i + 1) & mask_;
    keys_[i] = k;
    vals_[i] = v;
  }
  const uint64_t* get(uint64_t k) const {
    if (keys_.empty()) return nullptr;
    for (size_t i = slot(k);; i = (i + 1) & mask_) {
      if (keys_[i] == k) return &vals_[i];
      if (keys_[i] == kEmpty) return nullptr;
    }
  }

 private:
  static constexpr uint64_t kEmpty = ~0ull;
  size_t slot(uint64_t k) const { return static_cast<size_t>((k * 0x9E3779B97F4A7C15ull) >> 17) & mask_; }
  std::vector<uint64_t> keys_, vals_;
  size_t mask_ = 0;
};

struct Symbol {
  uint32_t c;
  int32_t prev, next;
  uint32_t len;  // bytes of the normalised text; 0 = merged away
};

struct Merge {
  uint32_t rank, pos, new_id;
};
// std::push_heap keeps the "largest" on top: lowest rank, then lowest position, wins
struct MergeLater {
  bool operator()(const Merge& a, const Merge& b) const {
    return a.rank != b.rank ? a.rank > b.rank : a.pos > b.pos;
  }
};

struct EncodeFailure {
  std::string msg;
};

}  // namespace

struct glp_tokenizer {
  std::string pool;  // all token strings, back to back (the vocabulary's keys view into it)
  std::unordered_map<std::string_view, uint32_t> vocab;
  FlatMap merges;      // (left << 32 | right) -> (rank << 32 | new id)
  FlatMap single_cp;   // code point -> id of its one-code-point token
  int32_t ascii[128];  // the same for ASCII, -1 when absent
  int32_t byte_tok[256];
  int64_t unk_id = -1;
  int n_tokens = 0;
  int n_merges = 0;

  // builds from the two GGUF string arrays; returns "" or the build error
  std::string build(const std::vector<std::string_view>& tokens, const std::vector<std::string_view>& merge_strs) {
    size_t bytes = 0;
    for (auto t : tokens) bytes += t.size();
    pool.reserve(bytes);
    std::vector<std::pair<size_t, size_t>> spans;
    spans.reserve(tokens.size());
    for (auto t : tokens) {
      spans.emplace_back(pool.size(), t.size());
      pool.append(t.data(), t.size());
    }
    vocab.reserve(tokens.size());
    for (size_t i = 0; i < spans.size(); ++i)  // tokenizer.rs:96-101: a later duplicate wins
      vocab[std::string_view(pool.data() + spans[i].first, spans[i].second)] = static_cast<uint32_t>(i);
    n_tokens = static_cast<int>(tokens.size());

    std::fill(ascii, ascii + 128, -1);
    single_cp.reserve(vocab.size());
    for (const auto& kv : vocab) {
      uint32_t cp;
      const int l = utf8_decode(reinterpret_cast<const unsigned char*>(kv.first.data()), kv.first.size(), &cp);
      if (l && static_cast<size_t>(l) == kv.first.size()) {
        single_cp.put(cp, kv.second);
        if (cp < 128) ascii[cp] = static_cast<int32_t>(kv.second);
      }
    }
    char name[8];
    for (int b = 0; b < 256; ++b) {
      std::snprintf(name, sizeof(name), "<0x%02X>", b);
      auto it = vocab.find(std::string_view(name, 6));
      byte_tok[b] = it == vocab.end() ? -1 : static_cast<int32_t>(it->second);
    }
    auto u = vocab.find("<unk>");
    unk_id = u == vocab.end() ? -1 : static_cast<int64_t>(u->second);

    // tokenizer.rs:103-111: "left right", exactly two parts; then BPE::build's merge map
    merges.reserve(merge_strs.size());
    uint32_t rank = 0;
    std::string joined;
    for (auto m : merge_strs) {
      const size_t sp = m.find(' ');
      if (sp == std::string_view::npos || m.find(' ', sp + 1) != std::string_view::npos) continue;
      const std::string_view a = m.substr(0, sp), b = m.substr(sp + 1);
      joined.assign(a.data(), a.size());
      joined.append(b.data(), b.size());
      for (std::string_view part : {a, b, std::string_view(joined)})
        if (!vocab.count(part)) return "BPE build error: Token `" + std::string(part) + "` out of vocabulary";
      const uint64_t key = (static_cast<uint64_t>(vocab[a]) << 32) | vocab[b];
      merges.put(key, (static_cast<uint64_t>(rank) << 32) | vocab[std::string_view(joined)]);
      ++rank;
    }
    n_merges = static_cast<int>(rank);
    return "";
  }

  const uint64_t* merge_of(uint32_t l, uint32_t r) const { return merges.get((static_cast<uint64_t>(l) << 32) | r); }

  // Tokenizer::encode(text, _): BPE ids of the one word the normaliser leaves
  void bpe(std::string_view text, std::vector<int32_t>& ids, std::vector<Symbol>& sym, std::vector<Merge>& heap) const {
    ids.clear();
    sym.clear();
    heap.clear();
    const auto add = [&](uint32_t c, uint32_t len) {
      const int32_t n = static_cast<int32_t>(sym.size());
      if (n) sym.back().next = n;
      sym.push_back(Symbol{c, n - 1, -1, len});
    };
    // merge_word, with ' ' read as U+2581 (3 bytes of the normalised text)
    bool unk_pending = false;
    uint32_t unk_len = 0;
    const auto* p = reinterpret_cast<const unsigned char*>(text.data());
    for (size_t i = 0; i < text.size();) {
      uint32_t cp;
      int blen = utf8_decode(p + i, text.size() - i, &cp);  // the caller validated the text
      const unsigned char* bytes = p + i;
      i += blen;
      if (cp == ' ') {
        cp = 0x2581;
        blen = 3;
        static const unsigned char kLowLine[3] = {0xE2, 0x96, 0x81};
        bytes = kLowLine;
      }
      int64_t id = -1;
      if (cp < 128) {
        id = ascii[cp];
      } else if (const uint64_t* v = single_cp.get(cp)) {
        id = static_cast<int64_t>(*v);
      }
      if (id >= 0) {
        if (unk_pending) {
          add(static_cast<uint32_t>(unk_id), unk_len);
          unk_pending = false;
        }
        add(static_cast<uint32_t>(id), static_cast<uint32_t>(blen));
        continue;
      }
      bool all_bytes = true;
      for (int k = 0; k < blen; ++k) all_bytes = all_bytes && byte_tok[bytes[k]] >= 0;
      if (all_bytes) {
        for (int k = 0; k < blen; ++k) add(static_cast<uint32_t>(byte_tok[bytes[k]]), 1);
        continue;
      }
      if (unk_pending) {
        unk_len += blen;
      } else {
        if (unk_id < 0) throw EncodeFailure{"Unk token `<unk>` not found in the vocabulary"};
        unk_pending = true;
        unk_len = blen;
      }
    }
    if (unk_pending) add(static_cast<uint32_t>(unk_id), unk_len);

    // Word::merge_all
    for (size_t i = 0; i + 1 < sym.size(); ++i)
      if (const uint64_t* m = merge_of(sym[i].c, sym[i + 1].c))
        heap.push_back(Merge{static_cast<uint32_t>(*m >> 32), static_cast<uint32_t>(i), static_cast<uint32_t>(*m)});
    std::make_heap(heap.begin(), heap.end(), MergeLater());
    const int32_t n_sym = static_cast<int32_t>(sym.size());
    while (!heap.empty()) {
      std::pop_heap(heap.begin(), heap.end(), MergeLater());
      const Merge top = heap.back();
      heap.pop_back();
      Symbol& cur = sym[top.pos];
      if (cur.len == 0 || cur.next == -1) continue;
      const int32_t nxt = cur.next;
      const Symbol right = sym[nxt];
      const uint64_t* m = merge_of(cur.c, right.c);
      if (!m || static_cast<uint32_t>(*m) != top.new_id) continue;  // stale entry
      cur.c = top.new_id;
      cur.len += right.len;
      cur.next = right.next;
      sym[nxt].len = 0;
      if (right.next > -1 && right.next < n_sym) sym[right.next].prev = static_cast<int32_t>(top.pos);
      if (cur.prev >= 0) {
        if (const uint64_t* pm = merge_of(sym[cur.prev].c, cur.c)) {
          heap.push_back(Merge{static_cast<uint32_t>(*pm >> 32), static_cast<uint32_t>(cur.prev), static_cast<uint32_t>(*pm)});
          std::push_heap(heap.begin(), heap.end(), MergeLater());
        }
      }
      if (cur.next > -1 && cur.next < n_sym) {
        if (const uint64_t* nm = merge_of(cur.c, sym[cur.next].c)) {
          heap.push_back(Merge{static_cast<uint32_t>(*nm >> 32), top.pos, static_cast<uint32_t>(*nm)});
          std::push_heap(heap.begin(), heap.end(), MergeLater());
        }
      }
    }
    for (const Symbol& s : sym)
      if (s.len) ids.push_back(static_cast<int32_t>(s.c));
  }

  // the three sequence forms of a text (GLP_TOKENS_*)
  void encode(std::string_view text, int form, std::vector<int32_t>& out, std::vector<Symbol>& sym,
              std::vector<Merge>& heap) const {
    std::vector<int32_t> ids;
    try {
      bpe(text, ids, sym, heap);
    } catch (EncodeFailure& f) {
      throw EncodeFailure{(form == GLP_TOKENS_SEQUENCE ? "Encode text part error: " : "Encode error: ") + f.msg};
    }
    out.clear();
    if (form == GLP_TOKENS_SEQUENCE) {  // tokenizer.rs:454-566, one text part
      out.push_back(kTokenBos);
      out.insert(out.end(), ids.begin(), ids.end());
      out.push_back(kTokenEos);
    } else if (form == GLP_TOKENS_SINGLE) {  // tokenizer.rs:162-177
      if (ids.empty() || ids.front() != kTokenBos) out.push_back(kTokenBos);
      out.insert(out.end(), ids.begin(), ids.end());
      if (out.back() != kTokenEos) out.push_back(kTokenEos);
    } else {
      out = std::move(ids);
    }
  }
};

namespace {

int fail(int code, const std::string& msg) {
  glp::set_last_error(msg);
  return code;
}

int make_tokenizer(const std::vector<std::string_view>& tokens, const std::vector<std::string_view>& merges,
                   glp_tokenizer** out) {
  auto* t = new glp_tokenizer();
  const std::string err = t->build(tokens, merges);
  if (!err.empty()) {
    delete t;
    return fail(GLP_ERR_FORMAT, err);
  }
  *out = t;
  return GLP_OK;
}

int write_string(const std::string& s, char* out, size_t cap, size_t* n_out) {
  if (n_out) *n_out = s.size();
  if (!out || cap < s.size() + 1)
    return fail(GLP_ERR_INVALID_ARG, "output buffer too small: " + std::to_string(s.size() + 1) + " bytes needed");
  std::memcpy(out, s.data(), s.size());
  out[s.size()] = '\0';
  return GLP_OK;
}

bool valid_cstr(const char* s) { return !s || utf8_valid(s, std::strlen(s)); }

// tokenizer.rs:13-64
const char* default_prompt(const std::string& key) {
  static const std::pair<const char*, const char*> kPrompts[] = {
      {"searchquery", "task: search result | query: "},
      {"retrieval", "task: search result | query: "},
      {"coderetrieval", "task: code retrieval | query: "},
      {"questionanswering", "task: question answering | query: "},
      {"factchecking", "task: fact checking | query: "},
      {"sentencesimilarity", "task: sentence similarity | query: "},
      {"sts", "task: sentence similarity | query: "},
      {"summarization", "task: sentence similarity | query: "},
      {"classification", "task: classification | query: "},
      {"clustering", "task: clustering | query: "},
      {"reranking", "task: search result | query: "},
      {"bitextmining", "task: search result | query: "},
      {"document", "title: none | text: "},
  };
  for (const auto& p : kPrompts)
    if (key == p.first) return p.second;
  return nullptr;
}

// Task::from_name_and_title(name, title).prompt_prefix() (task.rs:21-44, 54-73); false = Task::Raw
bool task_prefix(const char* name, const char* title, std::string* prefix) {
  if (!name) return false;
  const std::string key = task_key(name);
  static const std::pair<const char*, const char*> kTasks[] = {
      {"searchquery", "task: search result | query: "},
      {"retrieval", "task: search result | query: "},
      {"retrievalquery", "task: search result | query: "},
      {"query", "task: search result | query: "},
      {"coderetrieval", "task: code retrieval | query: "},
      {"code", "task: code retrieval | query: "},
      {"classification", "task: classification | query: "},
      {"multilabelclassification", "task: classification | query: "},
      {"clustering", "task: clustering | query: "},
      {"questionanswering", "task: question answering | query: "},
      {"qa", "task: question answering | query: "},
      {"factchecking", "task: fact checking | query: "},
      {"sentencesimilarity", "task: sentence similarity | query: "},
      {"sts", "task: sentence similarity | query: "},
      {"pairclassification", "task: sentence similarity | query: "},
      {"summarization", "task: sentence similarity | query: "},
  };
  if (key == "raw" || key == "none") return false;
  if (key == "document" || key == "retrievaldocument") {
    *prefix = title ? "title: " + std::string(title) + " | text: " : "title: none | text: ";
    return true;
  }
  for (const auto& t : kTasks)
    if (key == t.first) {
      *prefix = t.second;
      return true;
    }
  const std::string n(name);  // Task::Custom
  *prefix = (n.find(':') != std::string::npos || n.find('|') != std::string::npos) ? n : "task: " + n + " | query: ";
  return true;
}

}  // namespace

namespace glp {
// Tokenises one text in a sequence form; "" on success, else the error (used by the engine).
std::string tokenize_text(const glp_tokenizer* tok, std::string_view text, int form, std::vector<int32_t>* ids) {
  std::vector<Symbol> sym;
  std::vector<Merge> heap;
  try {
    tok->encode(text, form, *ids, sym, heap);
  } catch (EncodeFailure& f) {
    return f.msg;
  }
  return "";
}

// Task::from_name_and_title(task, title).format_text(text) (used by the engine)
std::string format_task(const char* task, const char* title, std::string_view text) {
  std::string s;
  task_prefix(task, title, &s);
  s.append(text.data(), text.size());
  return s;
}

bool valid_utf8(const char* s, size_t n) { return utf8_valid(s, n); }
}  // namespace glp

extern "C" {

int glp_tokenizer_from_gguf(const char* gguf_path, glp_tokenizer** out) {
  if (!gguf_path || !out) return fail(GLP_ERR_INVALID_ARG, "gguf_path and out must not be NULL");
  *out = nullptr;
  glp::GgufFile f;
  std::string err;
  if (!f.open(gguf_path, &err)) return fail(GLP_ERR_IO, err);
  // tokenizer.rs:80-94
  const glp::GgufValue* tv = f.find("tokenizer.ggml.tokens");
  if (!tv) return fail(GLP_ERR_FORMAT, "Missing tokenizer.ggml.tokens in GGUF metadata");
  const glp::GgufValue* mv = f.find("tokenizer.ggml.merges");
  if (!mv) return fail(GLP_ERR_FORMAT, "Missing tokenizer.ggml.merges in GGUF metadata");
  if (tv->type != 9) return fail(GLP_ERR_FORMAT, "tokenizer.ggml.tokens must be an Array");
  if (mv->type != 9) return fail(GLP_ERR_FORMAT, "tokenizer.ggml.merges must be an Array");
  // only string elements are read (a non-string array contributes nothing)
  return make_tokenizer(tv->strs, mv->strs, out);
}

int glp_tokenizer_from_vocab(const char* const* tokens, int n_tokens, const char* const* merges, int n_merges,
                             glp_tokenizer** out) {
  if (!out || n_tokens < 0 || n_merges < 0 || (n_tokens && !tokens) || (n_merges && !merges))
    return fail(GLP_ERR_INVALID_ARG, "bad vocabulary arguments");
  *out = nullptr;
  std::vector<std::string_view> t(n_tokens), m(n_merges);
  for (int i = 0; i < n_tokens; ++i) {
    if (!tokens[i] || !utf8_valid(tokens[i], std::strlen(tokens[i])))
      return fail(GLP_ERR_INVALID_ARG, "token " + std::to_string(i) + " is NULL or not UTF-8");
    t[i] = tokens[i];
  }
  for (int i = 0; i < n_merges; ++i) {
    if (!merges[i] || !utf8_valid(merges[i], std::strlen(merges[i])))
      return fail(GLP_ERR_INVALID_ARG, "merge " + std::to_string(i) + " is NULL or not UTF-8");
    m[i] = merges[i];
  }
  return make_tokenizer(t, m, out);
}

void glp_tokenizer_free(glp_tokenizer* tok) { delete tok; }

int glp_tokenizer_info(const glp_tokenizer* tok, int* n_tokens, int* n_merges) {
  if (!tok) return fail(GLP_ERR_INVALID_ARG, "tokenizer is NULL");
  if (n_tokens) *n_tokens = tok->n_tokens;
  if (n_merges) *n_merges = tok->n_merges;
  return GLP_OK;
}

int glp_tokenize(const glp_tokenizer* tok, const char* text, size_t text_len, int form, int32_t* ids, int cap,
                 int* n_ids) {
  if (!tok || (text_len && !text) || !n_ids || form < GLP_TOKENS_BARE || form > GLP_TOKENS_SEQUENCE || cap < 0)
    return fail(GLP_ERR_INVALID_ARG, "bad glp_tokenize arguments");
  if (!utf8_valid(text, text_len)) return fail(GLP_ERR_INVALID_ARG, "text is not valid UTF-8");
  std::vector<int32_t> out;
  const std::string err = glp::tokenize_text(tok, std::string_view(text, text_len), form, &out);
  if (!err.empty()) return fail(GLP_ERR_INVALID_ARG, err);
  *n_ids = static_cast<int>(out.size());
  if (static_cast<int>(out.size()) > cap || (!out.empty() && !ids))
    return fail(GLP_ERR_INVALID_ARG, "ids buffer too small: " + std::to_string(out.size()) + " ids");
  std::copy(out.begin(), out.end(), ids);
  return GLP_OK;
}

int glp_tokenize_batch(const glp_tokenizer* tok, const char* const* texts, const size_t* text_lens, int n_texts,
                       int form, int limit, int n_threads, int32_t* ids, size_t ids_cap, int64_t* offsets) {
  if (!tok || n_texts <= 0 || !texts || !text_lens || !offsets || form < GLP_TOKENS_BARE ||
      form > GLP_TOKENS_SEQUENCE)
    return fail(GLP_ERR_INVALID_ARG, n_texts == 0 ? "Cannot encode an empty batch" : "bad glp_tokenize_batch arguments");
  size_t total_bytes = 0;
  for (int i = 0; i < n_texts; ++i) {
    if (text_lens[i] && !texts[i]) return fail(GLP_ERR_INVALID_ARG, "text " + std::to_string(i) + " is NULL");
    if (!utf8_valid(texts[i], text_lens[i]))
      return fail(GLP_ERR_INVALID_ARG, "text " + std::to_string(i) + " is not valid UTF-8");
    total_bytes += text_lens[i];
  }
  std::vector<std::vector<int32_t>> rows(n_texts);
  std::vector<std::string> errs(n_texts);
  unsigned nt = n_threads > 0 ? static_cast<unsigned>(n_threads) : std::max(1u, std::thread::hardware_concurrency());
  nt = static_cast<unsigned>(std::min<size_t>({nt, static_cast<size_t>(n_texts), total_bytes / 4096 + 1, 64}));
  std::atomic<int> next{0};
  auto work = [&] {
    std::vector<Symbol> sym;
    std::vector<Merge> heap;
    for (int i; (i = next.fetch_add(1)) < n_texts;) {
      try {
        tok->encode(std::string_view(texts[i], text_lens[i]), form, rows[i], sym, heap);
      } catch (EncodeFailure& f) {
        errs[i] = f.msg;
      }
    }
  };
  if (nt <= 1) {
    work();
  } else {
    std::vector<std::thread> pool;
    try {
      for (unsigned k = 0; k < nt; ++k) pool.emplace_back(work);
    } catch (const std::exception&) {  // fewer threads than asked: the calling thread helps
    }
    if (pool.size() < nt) work();
    for (auto& th : pool) th.join();
  }
  // the first failing item in order, as the reference's sequential loop reports it
  offsets[0] = 0;
  for (int i = 0; i < n_texts; ++i) {
    if (!errs[i].empty()) return fail(GLP_ERR_INVALID_ARG, errs[i]);
    const size_t len = rows[i].size();
    if (limit > 0 && len > static_cast<size_t>(limit))
      return fail(GLP_ERR_CONTEXT_LIMIT, "Batch item " + std::to_string(i) + " sequence length (" + std::to_string(len) +
                                             " tokens) exceeds maximum context limit (" + std::to_string(limit) +
                                             " tokens)");
    offsets[i + 1] = offsets[i] + static_cast<int64_t>(len);
  }
  if (static_cast<size_t>(offsets[n_texts]) > ids_cap || (offsets[n_texts] && !ids))
    return fail(GLP_ERR_INVALID_ARG, "ids buffer too small: " + std::to_string(offsets[n_texts]) + " ids");
  for (int i = 0; i < n_texts; ++i) std::copy(rows[i].begin(), rows[i].end(), ids + offsets[i]);
  return GLP_OK;
}

int glp_format_query(const char* query, size_t query_len, const char* task, char* out, size_t cap, size_t* n_out) {
  if ((query_len && !query) || !task) return fail(GLP_ERR_INVALID_ARG, "query and task must not be NULL");
  if (!utf8_valid(query, query_len) || !valid_cstr(task)) return fail(GLP_ERR_INVALID_ARG, "not valid UTF-8");
  const char* p = default_prompt(task_key(task));  // tokenizer.rs:144-152
  std::string s = p ? std::string(p) : "task: " + to_lowercase(task) + " | query: ";
  s.append(query, query_len);
  return write_string(s, out, cap, n_out);
}

int glp_format_document(const char* content, size_t content_len, const char* title, char* out, size_t cap,
                        size_t* n_out) {
  if (content_len && !content) return fail(GLP_ERR_INVALID_ARG, "content must not be NULL");
  if (!utf8_valid(content, content_len) || !valid_cstr(title)) return fail(GLP_ERR_INVALID_ARG, "not valid UTF-8");
  std::string s = "title: " + std::string(title ? title : "none") + " | text: ";  // tokenizer.rs:154-160
  s.append(content, content_len);
  return write_string(s, out, cap, n_out);
}

int glp_task_format(const char* task, const char* title, const char* text, size_t text_len, char* out, size_t cap,
                    size_t* n_out) {
  if (text_len && !text) return fail(GLP_ERR_INVALID_ARG, "text must not be NULL");
  if (!utf8_valid(text, text_len) || !valid_cstr(task) || !valid_cstr(title))
    return fail(GLP_ERR_INVALID_ARG, "not valid UTF-8");
  std::string s;
  task_prefix(task, title, &s);  // task.rs:46-52: prefix + text, or the text alone for Raw
  s.append(text, text_len);
  return write_string(s, out, cap, n_out);
}

}  // extern "C"

namespace {

// One slice [lo, hi) of glp_embed_texts' batch, tokenised into packed ids + offsets.
struct TextPart {
  int lo = 0, hi = 0;
  std::vector<int32_t> packed;
  std::vector<int64_t> off;
  int rc = GLP_OK;
  std::string err;  // glp_last_error() of the thread that tokenised the part
};

void tokenize_part(const glp_tokenizer* tok, const char* const* texts, const size_t* text_lens, int form,
                   TextPart* P) {
  size_t cap = 2 * static_cast<size_t>(P->hi - P->lo);
  for (int i = P->lo; i < P->hi; ++i) cap += 3 * text_lens[i];  // a space may take 3 byte tokens
  P->packed.assign(std::max<size_t>(cap, 1), 0);
  P->off.assign(static_cast<size_t>(P->hi - P->lo) + 1, 0);
  P->rc = glp_tokenize_batch(tok, texts + P->lo, text_lens + P->lo, P->hi - P->lo, form, 0, 0, P->packed.data(),
                             cap, P->off.data());
  if (P->rc != GLP_OK) P->err = glp_last_error();
}

// The preflight length check of the reference path the form stands for, over one part (item
// indices are the batch's).
int preflight_part(const TextPart& P, int n_texts, int form, int64_t limit) {
  for (int i = P.lo; i < P.hi; ++i) {
    const int64_t len = P.off[i - P.lo + 1] - P.off[i - P.lo];
    if (len <= limit) continue;
    const std::string n = std::to_string(len), l = std::to_string(limit);
    std::string msg;
    if (form == GLP_TOKENS_SEQUENCE && n_texts == 1)  // embed_batch of one -> embed_interleaved, lib.rs:551-558
      msg = "Interleaved multimodal sequence length (" + n + " tokens) exceeds maximum context limit (" + l +
            " tokens). Preflight check failed before neural encoding (parts: 1).";
    else if (form == GLP_TOKENS_SEQUENCE)  // embed_batch_inner, lib.rs:837-844
      msg = "Batch item " + std::to_string(i) + " sequence length (" + n + ") exceeds maximum context limit (" + l + ")";
    else if (n_texts == 1)  // encode_single_text, lib.rs:969-976
      msg = "Text sequence length (" + n + " tokens) exceeds maximum context limit (" + l + " tokens)";
    else  // encode_batch_padded_with_limit, tokenizer.rs:195-203
      msg = "Batch item " + std::to_string(i) + " sequence length (" + n + " tokens) exceeds maximum context limit (" +
            l + " tokens)";
    return fail(GLP_ERR_CONTEXT_LIMIT, msg);
  }
  return GLP_OK;
}

int embed_part(glp_ctx* ctx, const TextPart& P, int out_dim, int row_dim, float* out) {
  const int n = P.hi - P.lo;
  int64_t width = 1;
  for (int i = 0; i < n; ++i) width = std::max(width, P.off[i + 1] - P.off[i]);
  std::vector<int32_t> ids(static_cast<size_t>(n) * width, kTokenPad), lengths(n);
  for (int i = 0; i < n; ++i) {
    lengths[i] = static_cast<int32_t>(P.off[i + 1] - P.off[i]);
    std::copy(P.packed.begin() + P.off[i], P.packed.begin() + P.off[i + 1], ids.begin() + static_cast<size_t>(i) * width);
  }
  return glp_embed_tokens(ctx, ids.data(), lengths.data(), n, static_cast<int>(width), out_dim,
                          out + static_cast<size_t>(P.lo) * row_dim, nullptr);
}

}  // namespace

extern "C" {

// Texts -> embeddings: tokenise (all host threads), run the reference's preflight length
// check, embed.  A large batch is cut into up to four parts of about 64 k estimated ids, and
// the next part is tokenised on a helper thread while the current one is embedded: a
// sequence's embedding does not depend on the batch it is in, so the output is the same.
// Errors keep the unsplit order -- every tokenisation error before every preflight error
// before an embedding error, each the first in batch order: when a part fails, the later
// parts are tokenised and checked before its error is returned.  Parts are used only where
// glp_embed_tokens cannot fail on ids or out_dim (valid out_dim, every token id inside the
// model's vocabulary).
int glp_embed_texts(glp_ctx* ctx, const glp_tokenizer* tok, const char* const* texts, const size_t* text_lens,
                    int n_texts, int form, int max_seq_len, int out_dim, float* out) {
  if (!ctx || !tok || n_texts <= 0 || !texts || !text_lens || !out || form < GLP_TOKENS_BARE ||
      form > GLP_TOKENS_SEQUENCE || max_seq_len < 0)
    return fail(GLP_ERR_INVALID_ARG, "bad glp_embed_texts arguments");
  const int64_t limit = max_seq_len > 0 ? max_seq_len : GLP_DEFAULT_MAX_SEQ_LEN;
  glp_model_info_t info{};
  int rc = glp_model_info(ctx, &info);
  if (rc != GLP_OK) return rc;
  int n_tok = 0;
  rc = glp_tokenizer_info(tok, &n_tok, nullptr);
  if (rc != GLP_OK) return rc;
  size_t bytes = 0;
  for (int i = 0; i < n_texts; ++i) bytes += text_lens[i];
  constexpr size_t kPartBytes = 3 * 65536;  // about 64 k ids at 3 bytes per id
  int parts = static_cast<int>(std::min<size_t>(4, bytes / kPartBytes));
  const bool splittable = out_dim >= 0 && out_dim <= info.embedding_dim && n_tok <= info.vocab;
  if (!splittable || parts < 2 || n_texts < 2 * parts) parts = 1;
  if (parts > 1) {
    // glp_tokenize_batch's argument errors, with the batch's item indices
    for (int i = 0; i < n_texts; ++i) {
      if (text_lens[i] && !texts[i]) return fail(GLP_ERR_INVALID_ARG, "text " + std::to_string(i) + " is NULL");
      if (!utf8_valid(texts[i], text_lens[i]))
        return fail(GLP_ERR_INVALID_ARG, "text " + std::to_string(i) + " is not valid UTF-8");
    }
  }
  const int row_dim = out_dim > 0 ? out_dim : info.embedding_dim;
  // parts embed into a private buffer, copied out only when the whole batch succeeded (no
  // partial outputs on failure)
  std::vector<float> staged(parts > 1 ? static_cast<size_t>(n_texts) * row_dim : 0);
  float* dst = parts > 1 ? staged.data() : out;
  std::vector<TextPart> ps(parts);
  for (int p = 0; p < parts; ++p) {
    ps[p].lo = static_cast<int>(static_cast<int64_t>(n_texts) * p / parts);
    ps[p].hi = static_cast<int>(static_cast<int64_t>(n_texts) * (p + 1) / parts);
  }
  auto over_positions = [&](const TextPart& P) {  // glp_embed_tokens' max_position_embeddings check
    for (size_t i = 0; i + 1 < P.off.size(); ++i)
      if (P.off[i + 1] - P.off[i] > info.max_position) return true;
    return false;
  };
  tokenize_part(tok, texts, text_lens, form, &ps[0]);
  for (int p = 0; p < parts; ++p) {
    std::thread next;
    if (p + 1 < parts) {
      try {
        next = std::thread(tokenize_part, tok, texts, text_lens, form, &ps[p + 1]);
      } catch (const std::exception&) {  // no thread to be had: tokenise it here, unoverlapped
        tokenize_part(tok, texts, text_lens, form, &ps[p + 1]);
      }
    }
    if (ps[p].rc != GLP_OK) {  // the batch's first tokenisation error
      if (next.joinable()) next.join();
      return fail(ps[p].rc, ps[p].err);
    }
    rc = preflight_part(ps[p], n_texts, form, limit);
    const bool embed_fails = rc == GLP_OK && over_positions(ps[p]);
    if (rc != GLP_OK || embed_fails) {
      // an earlier error class may still come from a later part
      const std::string own = glp_last_error();
      if (next.joinable()) next.join();
      for (int q = p + 2; q < parts; ++q) tokenize_part(tok, texts, text_lens, form, &ps[q]);
      for (int q = p + 1; q < parts; ++q)
        if (ps[q].rc != GLP_OK) return fail(ps[q].rc, ps[q].err);
      if (rc != GLP_OK) return fail(rc, own);
      for (int q = p + 1; q < parts; ++q) {
        rc = preflight_part(ps[q], n_texts, form, limit);
        if (rc != GLP_OK) return rc;
      }
    }
    rc = embed_part(ctx, ps[p], out_dim, row_dim, dst);
    if (next.joinable()) next.join();
    if (rc != GLP_OK) return rc;
  }
  if (parts > 1) std::memcpy(out, staged.data(), staged.size() * sizeof(float));
  return GLP_OK;
}

}  // extern "C"
