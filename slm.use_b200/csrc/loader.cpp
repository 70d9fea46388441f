// Model files: config.json (reference src/config.rs:20-106) and f32
// model.safetensors (src/model.rs:32-61).  A small JSON reader covers both.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "common.cuh"
#include "loader.hpp"

namespace slm {

namespace {

struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char* p;
  const char* end;
  [[noreturn]] void bad(const char* what) { fail(SLM_ERR_IO, std::string("malformed JSON: ") + what); }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  Json value() {
    ws();
    if (p >= end) bad("unexpected end");
    Json j;
    if (*p == '{') {
      j.kind = Json::OBJ;
      p++;
      ws();
      if (p < end && *p == '}') {
        p++;
        return j;
      }
      for (;;) {
        ws();
        if (p >= end || *p != '"') bad("expected key");
        std::string k = string();
        ws();
        if (p >= end || *p != ':') bad("expected ':'");
        p++;
        j.obj.emplace_back(k, value());
        ws();
        if (p < end && *p == ',') {
          p++;
          continue;
        }
        if (p < end && *p == '}') {
          p++;
          return j;
        }
        bad("expected ',' or '}'");
      }
    }
    if (*p == '[') {
      j.kind = Json::ARR;
      p++;
      ws();
      if (p < end && *p == ']') {
        p++;
        return j;
      }
      for (;;) {
        j.arr.push_back(value());
        ws();
        if (p < end && *p == ',') {
          p++;
          continue;
        }
        if (p < end && *p == ']') {
          p++;
          return j;
        }
        bad("expected ',' or ']'");
      }
    }
    if (*p == '"') {
      j.kind = Json::STR;
      j.str = string();
      return j;
    }
    if (end - p >= 4 && !std::strncmp(p, "true", 4)) {
      p += 4;
      j.kind = Json::BOOL;
      j.b = true;
      return j;
    }
    if (end - p >= 5 && !std::strncmp(p, "false", 5)) {
      p += 5;
      j.kind = Json::BOOL;
      return j;
    }
    if (end - p >= 4 && !std::strncmp(p, "null", 4)) {
      p += 4;
      return j;
    }
    char* stop = nullptr;
    std::string tmp(p, std::min<size_t>(end - p, 64));
    j.num = std::strtod(tmp.c_str(), &stop);
    if (stop == tmp.c_str()) bad("unexpected character");
    p += stop - tmp.c_str();
    j.kind = Json::NUM;
    return j;
  }
  std::string string() {
    std::string s;
    p++;  // opening quote
    while (p < end && *p != '"') {
      if (*p == '\\') {
        p++;
        if (p >= end) bad("bad escape");
        char c = *p;
        if (c == 'n') s += '\n';
        else if (c == 't') s += '\t';
        else if (c == 'u') {
          if (end - p < 5) bad("bad \\u escape");
          s += '?';
          p += 4;
        } else s += c;
        p++;
        continue;
      }
      s += *p++;
    }
    if (p >= end) bad("unterminated string");
    p++;
    return s;
  }
};

Json parse(const std::string& text) {
  Parser ps{text.data(), text.data() + text.size()};
  Json j = ps.value();
  return j;
}

std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail(SLM_ERR_IO, "reading " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

double num(const Json& j, const char* key, double dflt, bool required) {
  const Json* v = j.get(key);
  if (!v || v->kind == Json::NUL) {
    if (required) fail(SLM_ERR_IO, std::string("config.json: missing ") + key);
    return dflt;
  }
  if (v->kind == Json::BOOL) return v->b ? 1 : 0;
  if (v->kind != Json::NUM) fail(SLM_ERR_IO, std::string("config.json: ") + key + " is not a number");
  return v->num;
}

std::string str(const Json& j, const char* key) {
  const Json* v = j.get(key);
  if (!v || v->kind != Json::STR) fail(SLM_ERR_IO, std::string("config.json: missing ") + key);
  return v->str;
}

}  // namespace

Config load_config(const std::string& dir) {
  std::string path = dir + "/config.json";
  Json j = parse(read_file(path));
  if (j.kind != Json::OBJ) fail(SLM_ERR_IO, "parsing " + path);
  Config c;
  c.vocab = (size_t)num(j, "vocab_size", 0, true);
  c.d = (size_t)num(j, "d_model", 0, true);
  c.heads = (size_t)num(j, "n_heads", 0, true);
  c.kv_heads = (size_t)num(j, "global_kv_heads", 4, false);  // default_kv_heads, src/config.rs:54-56
  c.logn = (uint32_t)num(j, "global_logn", 0, false);
  c.kshift = (uint32_t)num(j, "global_kshift", 0, false);
  c.emb = (uint32_t)num(j, "global_emb", 0, false);
  c.far = (uint32_t)num(j, "global_far", 0, false);
  c.prelude = str(j, "prelude");
  c.core = str(j, "core");
  c.coda = str(j, "coda");
  c.window = (size_t)num(j, "window", 0, true);
  c.max_loops = (size_t)num(j, "max_loops", 0, true);
  c.default_loops = (size_t)num(j, "default_loops", 0, true);
  c.damp = (float)num(j, "damp", 1.0, false);  // default_damp, src/config.rs:58-60
  c.rope_base = (float)num(j, "rope_base", 0, true);
  c.eps = (float)num(j, "norm_eps", 0, true);
  // Options the reference rejects at load (src/config.rs:69-77).
  if (num(j, "loop_lora", 0, false) != 0) fail(SLM_ERR_INVALID, "loop_lora models are not supported");
  if (num(j, "state_loops", 0, false) != 0) fail(SLM_ERR_INVALID, "state_loops models are not supported");
  if (num(j, "global_rope_base", 0, false) != 0) fail(SLM_ERR_INVALID, "global_rope_base is not supported");
  if (c.heads == 0 || c.d % c.heads != 0) fail(SLM_ERR_INVALID, "d_model must be a multiple of n_heads");
  return c;
}

Tensors load_safetensors(const std::string& dir) {
  std::string path = dir + "/model.safetensors";
  auto blob = std::make_shared<std::string>(read_file(path));
  const std::string& raw = *blob;
  if (raw.size() < 8) fail(SLM_ERR_IO, path + ": too short");
  uint64_t n = 0;
  std::memcpy(&n, raw.data(), 8);
  if (n > raw.size() - 8) fail(SLM_ERR_IO, path + ": bad header size");
  Json h = parse(raw.substr(8, n));
  if (h.kind != Json::OBJ) fail(SLM_ERR_IO, path + ": bad header");
  Tensors out;
  out.blob = blob;
  size_t base = 8 + n;
  for (auto& kv : h.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& t = kv.second;
    const Json* dt = t.get("dtype");
    const Json* shape = t.get("shape");
    const Json* offs = t.get("data_offsets");
    if (!dt || !shape || !offs || offs->arr.size() != 2) fail(SLM_ERR_IO, path + ": bad entry " + kv.first);
    if (dt->str != "F32") fail(SLM_ERR_IO, kv.first + ": expected f32 weights");
    TensorView tv;
    for (auto& s : shape->arr) tv.shape.push_back((size_t)s.num);
    size_t a = (size_t)offs->arr[0].num, b = (size_t)offs->arr[1].num;
    size_t count = 1;
    for (size_t s : tv.shape) count *= s;
    if (b < a || base + b > raw.size() || b - a != count * 4) fail(SLM_ERR_IO, path + ": bad offsets for " + kv.first);
    tv.data = reinterpret_cast<const float*>(raw.data() + base + a);  // little-endian host
    tv.count = count;
    out.map[kv.first] = tv;
  }
  return out;
}

}  // namespace slm
