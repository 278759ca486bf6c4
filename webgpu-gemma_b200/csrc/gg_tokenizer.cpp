// gg_tokenizer.cpp -- the reference's greedy longest-match tokenizer (src/tokenizer.ts) in C++.
//
// The reference works on JavaScript strings, i.e. UTF-16 code units: token lengths, the
// longest-prefix search and the one-unit skip over unknown input are all counted in code
// units (tokenizer.ts:77-104). This implementation converts its UTF-8 input to UTF-16 and
// follows the same steps on code units, so it produces the reference's ids for any text,
// characters outside the BMP included; output text is converted back to UTF-8 (a lone
// surrogate becomes U+FFFD, as TextEncoder does).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include "gemma_b200.h"

namespace {

// UTF-8 -> UTF-16 with U+FFFD for every byte that does not start a valid sequence (the
// WHATWG decoder's replacement behaviour for the common cases).
std::u16string utf8_to_utf16(const char* s, size_t n) {
  std::u16string out;
  out.reserve(n);
  const auto* p = reinterpret_cast<const unsigned char*>(s);
  size_t i = 0;
  while (i < n) {
    const unsigned c = p[i];
    uint32_t cp = 0xFFFD;
    size_t len = 1;
    if (c < 0x80) {
      cp = c;
    } else if (c >= 0xC2 && c <= 0xDF && i + 1 < n && (p[i + 1] & 0xC0) == 0x80) {
      cp = ((c & 0x1F) << 6) | (p[i + 1] & 0x3F);
      len = 2;
    } else if (c >= 0xE0 && c <= 0xEF && i + 2 < n && (p[i + 1] & 0xC0) == 0x80 && (p[i + 2] & 0xC0) == 0x80) {
      const uint32_t v = ((c & 0x0F) << 12) | ((p[i + 1] & 0x3F) << 6) | (p[i + 2] & 0x3F);
      if (v >= 0x800 && (v < 0xD800 || v > 0xDFFF)) {
        cp = v;
        len = 3;
      }
    } else if (c >= 0xF0 && c <= 0xF4 && i + 3 < n && (p[i + 1] & 0xC0) == 0x80 && (p[i + 2] & 0xC0) == 0x80 &&
               (p[i + 3] & 0xC0) == 0x80) {
      const uint32_t v = ((c & 0x07) << 18) | ((p[i + 1] & 0x3F) << 12) | ((p[i + 2] & 0x3F) << 6) | (p[i + 3] & 0x3F);
      if (v >= 0x10000 && v <= 0x10FFFF) {
        cp = v;
        len = 4;
      }
    }
    if (cp >= 0x10000) {
      cp -= 0x10000;
      out.push_back(static_cast<char16_t>(0xD800 + (cp >> 10)));
      out.push_back(static_cast<char16_t>(0xDC00 + (cp & 0x3FF)));
    } else {
      out.push_back(static_cast<char16_t>(cp));
    }
    i += len;
  }
  return out;
}

void append_utf8(std::string& out, uint32_t cp) {
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

void utf16_to_utf8(std::u16string_view s, std::string& out) {
  for (size_t i = 0; i < s.size(); i++) {
    const uint32_t u = s[i];
    if (u >= 0xD800 && u <= 0xDBFF && i + 1 < s.size() && s[i + 1] >= 0xDC00 && s[i + 1] <= 0xDFFF) {
      append_utf8(out, 0x10000 + ((u - 0xD800) << 10) + (s[i + 1] - 0xDC00u));
      i++;
    } else if (u >= 0xD800 && u <= 0xDFFF) {
      append_utf8(out, 0xFFFD);
    } else {
      append_utf8(out, u);
    }
  }
}

constexpr char16_t kSpaceMark = u'\u2581';  // '▁', the space marker of the vocabulary

// SPECIAL_TOKENS and FUNC_TOKEN_NAMES (tokenizer.ts:3-16).
const std::pair<const char*, int32_t> kSpecial[] = {
    {"<start_of_turn>", 105}, {"<end_of_turn>", 106}, {"<eos>", 1}, {"<bos>", 2}};
const char* const kFuncNames[] = {"<start_function_declaration>", "<end_function_declaration>",
                                  "<start_function_call>",        "<end_function_call>",
                                  "<start_function_response>",    "<end_function_response>",
                                  "<escape>"};

}  // namespace

struct gg_tokenizer {
  std::vector<std::u16string> vocab;
  std::unordered_map<std::u16string, int32_t> by_text;  // tokenByText: first id wins
  size_t max_len = 0;                                   // maxTokenLen (code units)
  std::vector<uint16_t> max_len_from;                   // longest token starting with each code unit
  // specialTokens in the reference's key order, then sorted longest first (stable), the order
  // in which its alternation regex tries them (tokenizer.ts:70-75)
  std::vector<std::pair<std::u16string, int32_t>> special;
  std::vector<std::pair<std::string, int32_t>> func;    // funcTokens found in the vocabulary

  int32_t find(std::u16string_view t) const {
    auto it = by_text.find(std::u16string(t));
    return it == by_text.end() ? -1 : it->second;
  }

  // encodeSegment (tokenizer.ts:77-104): spaces -> '▁', optional leading '▁', then repeatedly
  // the longest vocabulary prefix, skipping one code unit where none matches.
  void encode_segment(std::u16string_view text, bool add_prefix, std::vector<int32_t>& out) const {
    std::u16string rem;
    rem.reserve(text.size() + 1);
    if (add_prefix) rem.push_back(kSpaceMark);
    for (char16_t c : text) rem.push_back(c == u' ' ? kSpaceMark : c);
    std::u16string key;
    size_t i = 0;
    while (i < rem.size()) {
      const size_t left = rem.size() - i;
      const size_t top = std::min(left, (size_t)max_len_from[rem[i]]);
      int32_t best = -1;
      size_t best_len = 0;
      for (size_t len = top; len >= 1; len--) {
        key.assign(rem, i, len);
        auto it = by_text.find(key);
        if (it != by_text.end()) {
          best = it->second;
          best_len = len;
          break;
        }
      }
      if (best_len == 0) {
        i += 1;
      } else {
        out.push_back(best);
        i += best_len;
      }
    }
  }

  // encode (tokenizer.ts:106-126): BOS, then the text split on special-token names (leftmost
  // match; at one position the longest name first), each piece encoded on its own.
  void encode(std::u16string_view text, std::vector<int32_t>& out) const {
    out.push_back(2);
    size_t last = 0;
    bool after_special = false;
    size_t i = 0;
    while (i < text.size()) {
      int32_t id = -1;
      size_t mlen = 0;
      if (text[i] == u'<') {
        for (const auto& sp : special) {
          if (text.compare(i, sp.first.size(), sp.first) == 0) {
            id = sp.second;
            mlen = sp.first.size();
            break;
          }
        }
      }
      if (mlen == 0) {
        i++;
        continue;
      }
      if (i > last) encode_segment(text.substr(last, i - last), !after_special, out);
      out.push_back(id);
      i += mlen;
      last = i;
      after_special = true;
    }
    if (last < text.size()) encode_segment(text.substr(last), !after_special, out);
  }
};

extern "C" int gg_tokenizer_create(const char* const* tokens, const size_t* lens, int n, gg_tokenizer** out) {
  if (!out || n < 0 || (n > 0 && (!tokens || !lens))) return GG_E_ARG;
  *out = nullptr;
  gg_tokenizer* t = new (std::nothrow) gg_tokenizer();
  if (!t) return GG_E_NOMEM;
  try {
    t->vocab.resize((size_t)n);
    t->max_len_from.assign(65536, 0);
    t->by_text.reserve((size_t)n * 2);
    for (int i = 0; i < n; i++) {  // buildTokenIndex (tokenizer.ts:43-57)
      if (!tokens[i] && lens[i]) {
        delete t;
        return GG_E_ARG;
      }
      t->vocab[i] = utf8_to_utf16(tokens[i] ? tokens[i] : "", lens[i]);
      const std::u16string& s = t->vocab[i];
      if (s.empty()) continue;
      t->by_text.emplace(s, i);
      t->max_len = std::max(t->max_len, s.size());
      uint16_t& m = t->max_len_from[s[0]];
      m = (uint16_t)std::min<size_t>(65535, std::max<size_t>(m, s.size()));
    }
    std::vector<std::pair<std::u16string, int32_t>> sp;
    for (const auto& s : kSpecial) sp.emplace_back(utf8_to_utf16(s.first, std::strlen(s.first)), s.second);
    for (const char* name : kFuncNames) {  // initFunctionTokens (tokenizer.ts:59-68)
      const std::u16string u = utf8_to_utf16(name, std::strlen(name));
      const int32_t id = t->find(u);
      if (id < 0) continue;
      t->func.emplace_back(name, id);
      bool replaced = false;
      for (auto& e : sp)
        if (e.first == u) {
          e.second = id;
          replaced = true;
        }
      if (!replaced) sp.emplace_back(u, id);
    }
    std::stable_sort(sp.begin(), sp.end(), [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
    t->special = std::move(sp);
  } catch (const std::bad_alloc&) {
    delete t;
    return GG_E_NOMEM;
  }
  *out = t;
  return GG_OK;
}

extern "C" int gg_tokenizer_encode(const gg_tokenizer* t, const char* text, size_t len, int32_t* ids, int cap,
                                   int* n_out) {
  if (!t || (!text && len) || !n_out || cap < 0 || (cap > 0 && !ids)) return GG_E_ARG;
  try {
    std::vector<int32_t> out;
    t->encode(utf8_to_utf16(text ? text : "", len), out);
    *n_out = (int)out.size();
    std::copy_n(out.begin(), std::min<size_t>(out.size(), (size_t)cap), ids);
  } catch (const std::bad_alloc&) {
    return GG_E_NOMEM;
  }
  return GG_OK;
}

extern "C" int gg_tokenizer_decode(const gg_tokenizer* t, const int32_t* ids, int n, char* text, size_t cap,
                                   size_t* len_out) {
  if (!t || n < 0 || (n > 0 && !ids) || !len_out || (cap > 0 && !text)) return GG_E_ARG;
  try {
    std::string out;
    for (int i = 0; i < n; i++) {  // decodeToken (tokenizer.ts:128-133)
      const int32_t id = ids[i];
      if (id >= 0 && (size_t)id < t->vocab.size() && !t->vocab[id].empty()) {
        std::u16string s = t->vocab[id];
        std::replace(s.begin(), s.end(), kSpaceMark, u' ');
        utf16_to_utf8(s, out);
      } else {
        out += "<unk:" + std::to_string(id) + ">";
      }
    }
    *len_out = out.size();
    if (cap > 0) std::memcpy(text, out.data(), std::min(out.size(), cap));
  } catch (const std::bad_alloc&) {
    return GG_E_NOMEM;
  }
  return GG_OK;
}

extern "C" int gg_tokenizer_token_id(const gg_tokenizer* t, const char* name, int32_t* id) {
  if (!t || !name || !id) return GG_E_ARG;
  *id = t->find(utf8_to_utf16(name, std::strlen(name)));
  return GG_OK;
}

extern "C" void gg_tokenizer_destroy(gg_tokenizer* t) { delete t; }
