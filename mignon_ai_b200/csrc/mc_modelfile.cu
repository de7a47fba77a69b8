// Host-side reader of the INT8 model file: quant.Decode (internal/quant/checkpoint.go:162-212).
//
// Binary files: binfmt (internal/binfmt/binfmt.go:1-14, Decode :88-107, Fill :111-144) — "MGNN",
// version 1, kind 2 (INT8), the checkpoint JSON without arrays, then the arrays in the order of
// CheckpointJSON.arrays (checkpoint.go:77-89). Legacy JSON files carry the arrays inline. The
// shape check is checkBlockShapes (:216-225).
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "mc_host.h"

namespace mc {

struct HostTensor {
  std::vector<int8_t> data;
  float scale = 0.f;
};

struct HostBlock {
  int steps = 0, dilation_base = 0, initial_dilation = 0;
  HostTensor w1, w2, wsel;
  std::vector<float> b1, b2, gamma;
  bool has_attn = false;
  std::vector<float> attn_norm;
  HostTensor qkv, out;
};

struct HostModel {
  int vocab = 0, state = 0, hidden = 0;
  bool tied = false;
  HostTensor embed, head_w;
  std::vector<HostBlock> blocks;
  std::vector<float> final_norm, head_b;
  int context_size = 0, attn_heads = 0, attn_window = 0;
};

namespace json {

struct Value {
  enum Type { Null, Bool, Num, Str, Arr, Obj } type = Null;
  bool b = false;
  double num = 0;
  float f32 = 0;  // the number parsed directly to float32 (strconv.ParseFloat(s, 32))
  std::string str;
  std::vector<std::unique_ptr<Value>> items;
  std::vector<std::string> keys;
  const Value* get(const char* k) const {
    if (type != Obj) return nullptr;
    for (size_t i = 0; i < keys.size(); ++i)
      if (keys[i] == k) return items[i].get();
    return nullptr;
  }
  double number(const char* k, double d) const {
    const Value* v = get(k);
    return v && v->type == Num ? v->num : d;
  }
};

class Parser {
 public:
  Parser(const char* s, size_t n) : s_(s), n_(n) {}
  std::unique_ptr<Value> parse() {
    auto v = value(0);
    ws();
    if (i_ != n_) ok_ = false;
    return ok_ ? std::move(v) : nullptr;
  }

 private:
  const char* s_;
  size_t n_, i_ = 0;
  bool ok_ = true;
  void ws() {
    while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  bool string(std::string& out) {
    if (i_ >= n_ || s_[i_] != '"') return false;
    ++i_;
    while (i_ < n_ && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\' && i_ < n_) {
        char e = s_[i_++];
        switch (e) {
          case 'n': c = '\n'; break;
          case 't': c = '\t'; break;
          case 'r': c = '\r'; break;
          case 'b': c = '\b'; break;
          case 'f': c = '\f'; break;
          case 'u': i_ += 4; c = '?'; break;
          default: c = e;
        }
      }
      out.push_back(c);
    }
    if (i_ >= n_) return false;
    ++i_;
    return true;
  }
  std::unique_ptr<Value> value(int depth) {
    auto v = std::make_unique<Value>();
    ws();
    if (depth > 64 || i_ >= n_) {
      ok_ = false;
      return v;
    }
    const char c = s_[i_];
    if (c == '{') {
      v->type = Value::Obj;
      ++i_;
      ws();
      if (i_ < n_ && s_[i_] == '}') {
        ++i_;
        return v;
      }
      while (ok_) {
        ws();
        std::string k;
        if (!string(k)) {
          ok_ = false;
          break;
        }
        ws();
        if (i_ >= n_ || s_[i_] != ':') {
          ok_ = false;
          break;
        }
        ++i_;
        v->keys.push_back(k);
        v->items.push_back(value(depth + 1));
        ws();
        if (i_ < n_ && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < n_ && s_[i_] == '}') {
          ++i_;
          break;
        }
        ok_ = false;
      }
      return v;
    }
    if (c == '[') {
      v->type = Value::Arr;
      ++i_;
      ws();
      if (i_ < n_ && s_[i_] == ']') {
        ++i_;
        return v;
      }
      while (ok_) {
        v->items.push_back(value(depth + 1));
        ws();
        if (i_ < n_ && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < n_ && s_[i_] == ']') {
          ++i_;
          break;
        }
        ok_ = false;
      }
      return v;
    }
    if (c == '"') {
      v->type = Value::Str;
      if (!string(v->str)) ok_ = false;
      return v;
    }
    if (n_ - i_ >= 4 && !strncmp(s_ + i_, "null", 4)) {
      i_ += 4;
      return v;
    }
    if (n_ - i_ >= 4 && !strncmp(s_ + i_, "true", 4)) {
      i_ += 4;
      v->type = Value::Bool;
      v->b = true;
      return v;
    }
    if (n_ - i_ >= 5 && !strncmp(s_ + i_, "false", 5)) {
      i_ += 5;
      v->type = Value::Bool;
      return v;
    }
    std::string num;
    while (i_ < n_ && strchr("+-0123456789.eE", s_[i_]) && num.size() < 64) num.push_back(s_[i_++]);
    if (num.empty()) {
      ok_ = false;
      return v;
    }
    char* end = nullptr;
    v->num = strtod(num.c_str(), &end);
    if (*end) ok_ = false;
    v->f32 = strtof(num.c_str(), nullptr);
    v->type = Value::Num;
    return v;
  }
};

}  // namespace json

namespace {

struct ArrRef {
  std::vector<int8_t>* i8 = nullptr;
  std::vector<float>* f32 = nullptr;
  const json::Value* inline_src = nullptr;
};

float scale_of(const json::Value* t) {
  const json::Value* v = t ? t->get("scale") : nullptr;
  return v && v->type == json::Value::Num ? v->f32 : 0.f;
}

const json::Value* data_of(const json::Value* t) { return t ? t->get("data") : nullptr; }

}  // namespace

// Parses a model file; returns kOk or kBadModel with the reason recorded.
int parse_model_file(const uint8_t* data, size_t n, HostModel& m) {
  const bool binary = n >= 4 && !memcmp(data, "MGNN", 4);
  const char* hdr = reinterpret_cast<const char*>(data);
  size_t hlen = n;
  const uint8_t* rest = nullptr;
  size_t rest_n = 0;
  if (binary) {
    if (n < 12) return set_error(kBadModel, "binary model file is truncated");
    const uint16_t ver = (uint16_t)(data[4] | (data[5] << 8));
    if (ver != 1) return set_error(kBadModel, "binary model file version " + std::to_string(ver) + " is not supported");
    if (data[6] != 1 && data[6] != 2) return set_error(kBadModel, "unknown model kind " + std::to_string(data[6]));
    if (data[6] != 2) return set_error(kBadModel, "not an INT8 model file");
    const uint32_t h = (uint32_t)data[8] | ((uint32_t)data[9] << 8) | ((uint32_t)data[10] << 16) | ((uint32_t)data[11] << 24);
    if ((uint64_t)h + 12 > n) return set_error(kBadModel, "binary model file is truncated (header)");
    hdr = reinterpret_cast<const char*>(data) + 12;
    hlen = h;
    rest = data + 12 + h;
    rest_n = n - 12 - h;
  }
  json::Parser p(hdr, hlen);
  auto root = p.parse();
  if (!root || root->type != json::Value::Obj) return set_error(kBadModel, "malformed model header JSON");
  m.vocab = (int)root->number("vocab_size", 0);
  m.state = (int)root->number("state_size", 0);
  m.hidden = (int)root->number("hidden_size", 0);
  const json::Value* te = root->get("tied_embed");
  m.tied = te && te->type == json::Value::Bool && te->b;
  const json::Value* meta = root->get("metadata");
  if (meta) {
    m.context_size = (int)meta->number("context_size", 0);
    m.attn_heads = (int)meta->number("attn_heads", 0);
    m.attn_window = (int)meta->number("attn_window", 0);
  }
  const json::Value* jembed = root->get("embed");
  m.embed.scale = scale_of(jembed);
  const json::Value* jblocks = root->get("blocks");
  const size_t nb = (jblocks && jblocks->type == json::Value::Arr) ? jblocks->items.size() : 0;
  m.blocks.resize(nb);
  std::vector<ArrRef> arrs;
  arrs.push_back({&m.embed.data, nullptr, data_of(jembed)});
  for (size_t b = 0; b < nb; ++b) {
    const json::Value* jb = jblocks->items[b].get();
    HostBlock& bl = m.blocks[b];
    bl.steps = (int)jb->number("steps", 0);
    bl.dilation_base = (int)jb->number("dilation_base", 0);
    bl.initial_dilation = (int)jb->number("initial_dilation", 0);
    bl.w1.scale = scale_of(jb->get("rule_w1"));
    bl.w2.scale = scale_of(jb->get("rule_w2"));
    bl.wsel.scale = scale_of(jb->get("rule_w_select"));
    arrs.push_back({&bl.w1.data, nullptr, data_of(jb->get("rule_w1"))});
    arrs.push_back({nullptr, &bl.b1, jb->get("rule_b1")});
    arrs.push_back({&bl.w2.data, nullptr, data_of(jb->get("rule_w2"))});
    arrs.push_back({nullptr, &bl.b2, jb->get("rule_b2")});
    arrs.push_back({nullptr, &bl.gamma, jb->get("gamma")});
    arrs.push_back({&bl.wsel.data, nullptr, data_of(jb->get("rule_w_select"))});
    const json::Value* ja = jb->get("attn");
    if (ja && ja->type == json::Value::Obj) {
      bl.has_attn = true;
      bl.qkv.scale = scale_of(ja->get("qkv"));
      bl.out.scale = scale_of(ja->get("out"));
      arrs.push_back({nullptr, &bl.attn_norm, ja->get("norm")});
      arrs.push_back({&bl.qkv.data, nullptr, data_of(ja->get("qkv"))});
      arrs.push_back({&bl.out.data, nullptr, data_of(ja->get("out"))});
    }
  }
  m.head_w.scale = scale_of(root->get("head_w"));
  arrs.push_back({nullptr, &m.final_norm, root->get("final_norm")});
  arrs.push_back({&m.head_w.data, nullptr, data_of(root->get("head_w"))});
  arrs.push_back({nullptr, &m.head_b, root->get("head_b")});

  if (binary) {
    size_t off = 0;
    for (size_t i = 0; i < arrs.size(); ++i) {
      if (rest_n - off < 4) return set_error(kBadModel, "binary model file is truncated (array " + std::to_string(i) + ")");
      const uint32_t cnt = (uint32_t)rest[off] | ((uint32_t)rest[off + 1] << 8) | ((uint32_t)rest[off + 2] << 16) |
                           ((uint32_t)rest[off + 3] << 24);
      off += 4;
      if (arrs[i].i8) {
        if (cnt > rest_n - off) return set_error(kBadModel, "binary model file is truncated (array " + std::to_string(i) + ")");
        arrs[i].i8->assign(reinterpret_cast<const int8_t*>(rest + off), reinterpret_cast<const int8_t*>(rest + off) + cnt);
        off += cnt;
      } else {
        if (cnt > (rest_n - off) / 4) return set_error(kBadModel, "binary model file is truncated (array " + std::to_string(i) + ")");
        arrs[i].f32->resize(cnt);
        if (cnt) memcpy(arrs[i].f32->data(), rest + off, (size_t)cnt * 4);
        off += (size_t)cnt * 4;
      }
    }
    if (off != rest_n)
      return set_error(kBadModel, "binary model file has " + std::to_string(rest_n - off) + " unexpected trailing bytes");
  } else {
    for (auto& a : arrs) {
      const json::Value* v = a.inline_src;
      if (!v || v->type == json::Value::Null) continue;
      if (v->type != json::Value::Arr) return set_error(kBadModel, "malformed array in JSON model file");
      for (auto& it : v->items)
        if (it->type != json::Value::Num) return set_error(kBadModel, "malformed array in JSON model file");
      if (a.i8) {
        a.i8->resize(v->items.size());
        for (size_t j = 0; j < v->items.size(); ++j) (*a.i8)[j] = (int8_t)v->items[j]->num;
      } else {
        a.f32->resize(v->items.size());
        for (size_t j = 0; j < v->items.size(); ++j) (*a.f32)[j] = v->items[j]->f32;
      }
    }
  }
  // checkBlockShapes and the sizes the engine relies on
  const size_t D = m.state, H = m.hidden, V = m.vocab;
  if (D == 0 || H == 0 || V == 0) return set_error(kBadModel, "model has a zero dimension");
  if (m.embed.data.size() != V * D) return set_error(kBadModel, "embedding has the wrong size");
  for (size_t b = 0; b < nb; ++b) {
    const HostBlock& bl = m.blocks[b];
    if (bl.w1.data.size() != 2 * H * 3 * D)
      return set_error(kBadModel, "block " + std::to_string(b) + " rule_w1 has " + std::to_string(bl.w1.data.size()) +
                                      " weights, want " + std::to_string(2 * H * 3 * D) +
                                      " (2*hidden*3*state): trained with a different CA neighbourhood");
    if (bl.w2.data.size() != 2 * D * H || bl.wsel.data.size() != D * D || bl.b1.size() != 2 * H || bl.b2.size() != 2 * D)
      return set_error(kBadModel, "block " + std::to_string(b) + " has tensors of the wrong size");
    if (bl.has_attn && (bl.qkv.data.size() != 3 * D * D || bl.out.data.size() != D * D || bl.attn_norm.size() != D))
      return set_error(kBadModel, "block " + std::to_string(b) + " attention tensors have the wrong size");
  }
  if (!m.tied && m.head_w.data.size() != V * D) return set_error(kBadModel, "head weights have the wrong size");
  if (m.head_b.size() != V) return set_error(kBadModel, "head bias has the wrong size");
  return kOk;
}

}  // namespace mc
