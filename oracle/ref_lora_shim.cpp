// C entry points onto the reference's OWN kohya LoRA loader — TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/build_oracle.py (when the reference tree is present) from the reference's
// headers src/infer/lora.hpp and src/io/safetensors.hpp where they lie, into
// oracle/_ref/libref_lora.so.  The tests run the reference's load_lora_modules (lora.hpp:300-455)
// on safetensors files they write, and compare its modules, scales, fp16 bits and report
// counters with the library's loader (dollama_b200/lora.py).
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "infer/lora.hpp"

namespace {
struct Loaded {
  std::vector<dollama::LoraModule> mods;
  dollama::LoraLoadReport rep;
};
thread_local std::string g_err;
}  // namespace

extern "C" {

const char* ref_lora_error() { return g_err.c_str(); }

// returns a handle (nullptr on error, message in ref_lora_error)
void* ref_lora_load(const char* base_path, const char* lora_path, float strength) {
  try {
    dollama::SafeTensors base(base_path);
    dollama::SafeTensors lora(lora_path);
    auto* l = new Loaded;
    l->mods = dollama::load_lora_modules(base, lora, strength, &l->rep);
    return l;
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void ref_lora_free(void* h) { delete static_cast<Loaded*>(h); }

int ref_lora_count(void* h) { return static_cast<int>(static_cast<Loaded*>(h)->mods.size()); }

// report: te_skipped, other_keys, incomplete, modules
void ref_lora_report(void* h, long long* out) {
  const auto& r = static_cast<Loaded*>(h)->rep;
  out[0] = static_cast<long long>(r.te_skipped);
  out[1] = static_cast<long long>(r.other_keys);
  out[2] = static_cast<long long>(r.incomplete);
  out[3] = static_cast<long long>(r.modules);
}

// module i: key (NUL-terminated, keycap bytes), dims, scale; A / B fp16 bits when a / b are given
int ref_lora_module(void* h, int i, char* key, int keycap, int* dims, float* scale, uint16_t* a,
                    uint16_t* b) {
  const auto& m = static_cast<Loaded*>(h)->mods[static_cast<size_t>(i)];
  const size_t k = m.base_key.size() < static_cast<size_t>(keycap - 1) ? m.base_key.size()
                                                                        : static_cast<size_t>(keycap - 1);
  std::memcpy(key, m.base_key.data(), k);
  key[k] = '\0';
  dims[0] = m.rank;
  dims[1] = m.in_flat;
  dims[2] = m.out_dim;
  *scale = m.scale;
  if (a) std::memcpy(a, m.a_fp16.data(), m.a_fp16.size() * sizeof(uint16_t));
  if (b) std::memcpy(b, m.b_fp16.data(), m.b_fp16.size() * sizeof(uint16_t));
  return 0;
}

}  // extern "C"
