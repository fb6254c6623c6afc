// manifest.cu — the converted-checkpoint loader behind the C ABI
// (llm/weights-q8-io.ts:14-128, llm/weights.ts:95-115): a manifest (the JSON
// `llm/tools/convert_weights.py` and `gen_fixture_q8.py` write: "config" and
// "weights" entries) plus the three buffers it indexes — int8 codes, f32
// scales, f32 norms — become a resident engine, with every offset checked
// against the buffers before any device work.  Also the RoPE row
// permutation the converter applies to HF wq/wk weights.
#include <string.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"

namespace xpu {
namespace {

// ------------------------------------------------------------------ JSON --
// A small recursive-descent parser for the manifest: objects, arrays,
// strings (with the standard escapes), numbers, true/false/null.
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* key) const {
    if (kind != Obj) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* end;
  std::string err;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail(const char* what) {
    if (err.empty()) err = what;
    return false;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(end - p) < n || memcmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  bool str(std::string& out) {
    if (p >= end || *p != '"') return fail("expected a string");
    ++p;
    while (p < end && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= end) return fail("bad escape");
        const char e = *p++;
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (end - p < 4) return fail("bad \\u escape");
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              v = v * 16 + (unsigned)(h >= '0' && h <= '9' ? h - '0' : (h | 32) - 'a' + 10);
            }
            // Names here are ASCII; other code points are kept as UTF-8.
            if (v < 0x80) {
              out += (char)v;
            } else if (v < 0x800) {
              out += (char)(0xC0 | (v >> 6));
              out += (char)(0x80 | (v & 0x3F));
            } else {
              out += (char)(0xE0 | (v >> 12));
              out += (char)(0x80 | ((v >> 6) & 0x3F));
              out += (char)(0x80 | (v & 0x3F));
            }
            break;
          }
          default: return fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool value(JVal& v) {
    if (++depth > 64) return fail("nesting too deep");
    ws();
    if (p >= end) return fail("unexpected end");
    bool ok = true;
    if (*p == '{') {
      ++p;
      v.kind = JVal::Obj;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        for (;;) {
          ws();
          std::string key;
          JVal item;
          if (!str(key)) return false;
          ws();
          if (p >= end || *p != ':') return fail("expected ':'");
          ++p;
          if (!value(item)) return false;
          v.obj.emplace_back(std::move(key), std::move(item));
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == '}') {
            ++p;
            break;
          }
          return fail("expected ',' or '}'");
        }
      }
    } else if (*p == '[') {
      ++p;
      v.kind = JVal::Arr;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        for (;;) {
          JVal item;
          if (!value(item)) return false;
          v.arr.push_back(std::move(item));
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == ']') {
            ++p;
            break;
          }
          return fail("expected ',' or ']'");
        }
      }
    } else if (*p == '"') {
      v.kind = JVal::Str;
      ok = str(v.str);
    } else if (lit("true")) {
      v.kind = JVal::Bool;
      v.b = true;
    } else if (lit("false")) {
      v.kind = JVal::Bool;
    } else if (lit("null")) {
      v.kind = JVal::Null;
    } else {
      char* q = nullptr;
      const std::string tok(p, (size_t)std::min<ptrdiff_t>(end - p, 64));
      v.num = strtod(tok.c_str(), &q);
      if (q == tok.c_str()) return fail("bad value");
      v.kind = JVal::Num;
      p += q - tok.c_str();
    }
    --depth;
    return ok;
  }
};

// An integer field of `obj` in [lo, hi]; false (with the message) if absent,
// not an integer or out of range.
bool int_field(const JVal& obj, const char* key, int64_t lo, int64_t hi, int64_t* out) {
  const JVal* v = obj.get(key);
  if (!v || v->kind != JVal::Num || v->num != std::floor(v->num) || v->num < (double)lo || v->num > (double)hi) {
    set_error("manifest: %s must be an integer in [%lld, %lld]", key, (long long)lo, (long long)hi);
    return false;
  }
  *out = (int64_t)v->num;
  return true;
}

}  // namespace
}  // namespace xpu

using namespace xpu;

extern "C" {

int xpu_llama_create_from_manifest(const char* manifest_json, const int8_t* codes, int64_t codes_len,
                                   const float* scales, int64_t scales_len, const float* norms, int64_t norms_len,
                                   int32_t max_seq_len, int32_t device, xpu_llama** engine) {
  XPU_REQUIRE(manifest_json && engine, XPU_EINVAL, "manifest: null pointer");
  *engine = nullptr;
  XPU_REQUIRE(codes_len >= 0 && scales_len >= 0 && norms_len >= 0 && (codes || !codes_len) &&
                  (scales || !scales_len) && (norms || !norms_len),
              XPU_EINVAL, "manifest: buffer pointers and lengths do not match");
  JParser ps{manifest_json, manifest_json + strlen(manifest_json)};
  JVal root;
  if (!ps.value(root)) {
    set_error("manifest: JSON parse error (%s) at byte %lld", ps.err.c_str(), (long long)(ps.p - manifest_json));
    return XPU_EINVAL;
  }
  const JVal* cfg = root.get("config");
  const JVal* ents = root.get("weights");
  XPU_REQUIRE(cfg && cfg->kind == JVal::Obj && ents && ents->kind == JVal::Arr, XPU_EINVAL,
              "manifest: needs a \"config\" object and a \"weights\" array (llm/weights-q8-io.ts)");

  // llm/weights-q8-io.ts:36-55: the manifest config plus maxSeqLen.
  xpu_llama_config c{};
  int64_t v;
  const int64_t big = 1 << 30;
  if (!int_field(*cfg, "numLayers", 1, big, &v)) return XPU_EINVAL;
  c.num_layers = (int32_t)v;
  if (!int_field(*cfg, "hiddenSize", 1, big, &v)) return XPU_EINVAL;
  c.hidden_size = (int32_t)v;
  if (!int_field(*cfg, "numHeads", 1, big, &v)) return XPU_EINVAL;
  c.num_heads = (int32_t)v;
  if (!int_field(*cfg, "numKvHeads", 1, big, &v)) return XPU_EINVAL;
  c.num_kv_heads = (int32_t)v;
  if (!int_field(*cfg, "headDim", 1, big, &v)) return XPU_EINVAL;
  c.head_dim = (int32_t)v;
  if (!int_field(*cfg, "ffnHidden", 1, big, &v)) return XPU_EINVAL;
  c.ffn_hidden = (int32_t)v;
  if (!int_field(*cfg, "vocabSize", 1, big, &v)) return XPU_EINVAL;
  c.vocab_size = (int32_t)v;
  const JVal* theta = cfg->get("ropeTheta");
  const JVal* eps = cfg->get("rmsNormEps");
  XPU_REQUIRE(theta && theta->kind == JVal::Num && eps && eps->kind == JVal::Num, XPU_EINVAL,
              "manifest: ropeTheta and rmsNormEps must be numbers");
  c.rope_theta = theta->num;
  c.rms_norm_eps = eps->num;
  const JVal* tie = cfg->get("tieEmbeddings");
  c.tie_embeddings = tie && tie->kind == JVal::Bool && tie->b ? 1 : 0;
  c.max_seq_len = max_seq_len;

  // llm/weights-q8-io.ts:76-128: views into the three buffers, by name.
  std::map<std::string, xpu_q8_linear> quant;
  std::map<std::string, const float*> norm_by_name;
  std::map<std::string, int64_t> norm_len;
  for (const JVal& e : ents->arr) {
    const JVal* name = e.get("name");
    const JVal* kind = e.get("kind");
    const JVal* shape = e.get("shape");
    XPU_REQUIRE(name && name->kind == JVal::Str && kind && kind->kind == JVal::Str && shape &&
                    shape->kind == JVal::Arr && !shape->arr.empty(),
                XPU_EINVAL, "manifest: every weight entry needs a name, a kind and a shape");
    int64_t elems = 1;
    for (const JVal& d : shape->arr) {
      XPU_REQUIRE(d.kind == JVal::Num && d.num >= 0 && d.num == std::floor(d.num) && d.num < (double)big, XPU_EINVAL,
                  "manifest: bad shape of %s", name->str.c_str());
      elems *= (int64_t)d.num;
    }
    if (kind->str == "quant") {
      XPU_REQUIRE(shape->arr.size() == 2, XPU_EINVAL, "manifest: %s: a quant entry has shape [N, K]",
                  name->str.c_str());
      const int64_t n = (int64_t)shape->arr[0].num, k = (int64_t)shape->arr[1].num;
      int64_t co, so;
      if (!int_field(e, "codesOffset", 0, (int64_t)1 << 60, &co) || !int_field(e, "scaleOffset", 0, (int64_t)1 << 60, &so))
        return XPU_EINVAL;
      XPU_REQUIRE(co + n * k <= codes_len && so + n <= scales_len, XPU_EINVAL,
                  "manifest: %s reaches past the codes (%lld) or scales (%lld) buffer", name->str.c_str(),
                  (long long)codes_len, (long long)scales_len);
      quant[name->str] = xpu_q8_linear{codes + co, scales + so, n, k};
    } else if (kind->str == "norm") {
      int64_t off;
      if (!int_field(e, "offset", 0, (int64_t)1 << 60, &off)) return XPU_EINVAL;
      XPU_REQUIRE(off + elems <= norms_len, XPU_EINVAL, "manifest: %s reaches past the norms buffer (%lld)",
                  name->str.c_str(), (long long)norms_len);
      norm_by_name[name->str] = norms + off;
      norm_len[name->str] = elems;
    } else {
      set_error("manifest: %s has unknown kind \"%s\"", name->str.c_str(), kind->str.c_str());
      return XPU_EINVAL;
    }
  }
  auto q = [&](const std::string& n, xpu_q8_linear* out) {
    auto it = quant.find(n);
    if (it == quant.end()) {
      set_error("buildLlamaWeightsQ8: no quantized weight named \"%s\"", n.c_str());
      return false;
    }
    *out = it->second;
    return true;
  };
  auto nm = [&](const std::string& n, const float** out) {
    auto it = norm_by_name.find(n);
    if (it == norm_by_name.end()) {
      set_error("buildLlamaWeightsQ8: no norm weight named \"%s\"", n.c_str());
      return false;
    }
    if (norm_len[n] != c.hidden_size) {
      set_error("manifest: %s has %lld elements, hiddenSize is %d", n.c_str(), (long long)norm_len[n], c.hidden_size);
      return false;
    }
    *out = it->second;
    return true;
  };
  std::vector<xpu_llama_layer_q8> layers((size_t)c.num_layers);
  xpu_llama_weights_q8 w{};
  bool ok = q("embedTokens", &w.embed_tokens) && q("lmHead", &w.lm_head) && nm("finalNorm", &w.final_norm);
  for (int i = 0; ok && i < c.num_layers; ++i) {
    const std::string p = "layers." + std::to_string(i) + ".";
    xpu_llama_layer_q8& L = layers[(size_t)i];
    ok = nm(p + "attnNorm", &L.attn_norm) && q(p + "wq", &L.wq) && q(p + "wk", &L.wk) && q(p + "wv", &L.wv) &&
         q(p + "wo", &L.wo) && nm(p + "ffnNorm", &L.ffn_norm) && q(p + "wGate", &L.w_gate) &&
         q(p + "wUp", &L.w_up) && q(p + "wDown", &L.w_down);
  }
  if (!ok) return XPU_EINVAL;
  w.layers = layers.data();
  w.num_layers = c.num_layers;
  return xpu_llama_create(&c, &w, device, engine);
}

// llm/weights.ts:95-115 permuteRopeChannels: within each head, HF rows i and
// i + headDim/2 become rows 2i and 2i + 1 (the adjacent-pair RoPE layout).
int xpu_permute_rope_channels(const float* weight, int64_t heads, int64_t head_dim, int64_t in_features,
                              float* out) {
  XPU_REQUIRE(heads >= 0 && head_dim >= 0 && in_features >= 0 && head_dim % 2 == 0, XPU_EINVAL,
              "permuteRopeChannels: sizes must be >= 0 and headDim even");
  const int64_t n = heads * head_dim * in_features;
  if (n == 0) return XPU_OK;
  XPU_REQUIRE(weight && out && weight != out, XPU_EINVAL, "permuteRopeChannels: null or aliased pointer");
  const int64_t half = head_dim / 2;
  for (int64_t h = 0; h < heads; ++h) {
    const int64_t base = h * head_dim * in_features;
    for (int64_t i = 0; i < half; ++i) {
      memcpy(out + base + 2 * i * in_features, weight + base + i * in_features, (size_t)in_features * sizeof(float));
      memcpy(out + base + (2 * i + 1) * in_features, weight + base + (i + half) * in_features,
             (size_t)in_features * sizeof(float));
    }
  }
  return XPU_OK;
}

}  // extern "C"
