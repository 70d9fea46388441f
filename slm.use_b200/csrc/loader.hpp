// Model configuration and weight files.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace slm {

// config.json (reference src/config.rs:22-52).
struct Config {
  size_t vocab = 0, d = 0, heads = 0, kv_heads = 4, window = 0, max_loops = 0, default_loops = 0;
  uint32_t logn = 0, kshift = 0, emb = 0, far = 0;
  float damp = 1.0f, rope_base = 10000.0f, eps = 1e-6f;
  std::string prelude, core, coda;
  size_t dh() const { return d / heads; }
};

struct TensorView {
  std::vector<size_t> shape;
  const float* data = nullptr;
  size_t count = 0;
};

struct Tensors {
  std::shared_ptr<std::string> blob;
  std::map<std::string, TensorView> map;
};

Config load_config(const std::string& dir);
Tensors load_safetensors(const std::string& dir);

}  // namespace slm
