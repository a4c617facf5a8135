// C entry points onto the reference's OWN tag tokenizer — TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/build_oracle.py (when the reference tree is present) from the reference's
// header src/io/tokenizer.hpp where it lies, into oracle/_ref/libref_tokenizer.so.  The golden
// generator (tests/golden/make_tokenizer_vectors.py) runs it on a synthetic vocabulary to record
// what the reference's Tokenizer (encode / encode_text / decode / tag_to_id, tokenizer.hpp:60-250)
// returns, and the vocabulary checks it rejects (tokenizer.hpp:487-527).
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "io/tokenizer.hpp"

namespace {
thread_local std::string g_err;
}

extern "C" {

const char* ref_tok_error() { return g_err.c_str(); }

void* ref_tok_create(const char* vocab_path) {
  try {
    return new dollama::Tokenizer(vocab_path);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void ref_tok_destroy(void* h) { delete static_cast<dollama::Tokenizer*>(h); }

int ref_tok_vocab_size(void* h) { return static_cast<int>(static_cast<dollama::Tokenizer*>(h)->vocab_size()); }

int ref_tok_tag_to_id(void* h, const char* tag) { return static_cast<dollama::Tokenizer*>(h)->tag_to_id(tag); }

// tags: n NUL-terminated strings; writes at most cap ids, returns the id count
int ref_tok_encode(void* h, const char* const* tags, int n, int max_len, int* out, int cap) {
  std::vector<std::string> v(tags, tags + n);
  const std::vector<int> ids = static_cast<dollama::Tokenizer*>(h)->encode(v, max_len);
  const int m = static_cast<int>(ids.size());
  for (int i = 0; i < m && i < cap; ++i) out[i] = ids[i];
  return m;
}

int ref_tok_encode_text(void* h, const char* text, int max_len, int* out, int cap) {
  const std::vector<int> ids = static_cast<dollama::Tokenizer*>(h)->encode_text(text, max_len);
  const int m = static_cast<int>(ids.size());
  for (int i = 0; i < m && i < cap; ++i) out[i] = ids[i];
  return m;
}

// decoded tokens joined by '\n' into buf (cap bytes); returns the joined length
int ref_tok_decode(void* h, const int* ids, int n, char* buf, int cap) {
  const std::vector<std::string> toks = static_cast<dollama::Tokenizer*>(h)->decode(std::vector<int>(ids, ids + n));
  std::string s;
  for (size_t i = 0; i < toks.size(); ++i) {
    if (i) s.push_back('\n');
    s += toks[i];
  }
  if (cap > 0) {
    const size_t k = s.size() < static_cast<size_t>(cap - 1) ? s.size() : static_cast<size_t>(cap - 1);
    std::memcpy(buf, s.data(), k);
    buf[k] = '\0';
  }
  return static_cast<int>(s.size());
}

// normalize (static) into buf; returns the length
int ref_tok_normalize(const char* s, char* buf, int cap) {
  const std::string r = dollama::Tokenizer::normalize(s);
  if (cap > 0) {
    const size_t k = r.size() < static_cast<size_t>(cap - 1) ? r.size() : static_cast<size_t>(cap - 1);
    std::memcpy(buf, r.data(), k);
    buf[k] = '\0';
  }
  return static_cast<int>(r.size());
}

}  // extern "C"
