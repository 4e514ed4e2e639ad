// mxmoe.hpp -- C++ mirror of burn-extended's `moe` / `quant` / `loader::mxfp4`
// API over the C ABI of include/mxmoe.h (header only).
//
//   quant::QuantLinearMxFp4Desc   src/quant/mod.rs:3-11
//   quant::MoeQuantLayerHost      src/quant/mod.rs:13-21
//   moe::MoeConfig / init         src/moe/mod.rs:22-33, :60-91
//   moe::MoeGatedSwiGLU           src/moe/mod.rs:35-57 (set_resident :95-97,
//                                 forward :99-115)
//   loader::mxfp4::dequant_mxfp4_bytes  src/loader/mxfp4.rs:57-79 (device)
//
// The reference panics on failure (e.g. src/moe/mod.rs:111-113); this mirror
// throws mxmoe::Error carrying the library status and message.  Exceptions are
// raised on the caller's side of the boundary only -- the C ABI itself never
// throws.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "mxmoe.h"

namespace burn_extended {

class Error : public std::runtime_error {
 public:
  Error(int status, const std::string& msg) : std::runtime_error(msg), status_(status) {}
  int status() const { return status_; }

 private:
  int status_;
};

inline void check(int status) {
  if (status != MXMOE_OK) {
    char buf[1024];
    mxmoe_last_error(buf, sizeof(buf));
    throw Error(status, std::string("mxmoe: ") + buf);
  }
}

namespace quant {

struct QuantLinearMxFp4Desc {
  uint64_t experts = 0, rows = 0, cols = 0, bpr = 0, gpr = 0;
  int32_t ue8_offset = 0;

  static QuantLinearMxFp4Desc for_shape(uint64_t experts, uint64_t rows, uint64_t cols, int32_t ue8 = 0) {
    return {experts, rows, cols, (cols + 1) / 2, (cols + 31) / 32, ue8};
  }
  mxmoe_quant_desc c() const { return {experts, rows, cols, bpr, gpr, ue8_offset}; }
};

struct MoeQuantLayerHost {
  QuantLinearMxFp4Desc w1_desc, w2_desc;
  std::vector<uint8_t> w1_blocks, w1_scales, w2_blocks, w2_scales;
};

}  // namespace quant

namespace moe {

class MoeGatedSwiGLU;

struct MoeConfig {
  uint32_t d_model = 0;
  uint32_t ffn_hidden = 0;
  uint32_t num_experts = 0;
  uint32_t experts_per_token = 0;
  float swiglu_alpha = 1.702f;
  float swiglu_limit = 7.0f;
  bool disabled = false;
  bool verbose = false;
  float rms_eps = 1e-5f;
  uint32_t flags = 0;  // MXMOE_FLAG_INTERLEAVED_GLU, MXMOE_FLAG_BIAS_PER_FTILE, ...

  MoeGatedSwiGLU init(int device = 0) const;
};

class MoeGatedSwiGLU {
 public:
  MoeGatedSwiGLU(const MoeConfig& cfg, int device) : cfg_(cfg) {
    mxmoe_config c{cfg.d_model, cfg.ffn_hidden, cfg.num_experts, cfg.experts_per_token, cfg.swiglu_alpha,
                   cfg.swiglu_limit, cfg.rms_eps, cfg.flags | (cfg.disabled ? MXMOE_FLAG_DISABLED : 0u), device};
    check(mxmoe_create(&c, &layer_));
  }
  // Takes ownership of a layer the library created (the model.bin loader).
  MoeGatedSwiGLU(const MoeConfig& cfg, mxmoe_layer* adopted) : cfg_(cfg), layer_(adopted) {}
  MoeGatedSwiGLU(const MoeGatedSwiGLU&) = delete;
  MoeGatedSwiGLU& operator=(const MoeGatedSwiGLU&) = delete;
  MoeGatedSwiGLU(MoeGatedSwiGLU&& o) noexcept : cfg_(o.cfg_), layer_(std::exchange(o.layer_, nullptr)) {}
  ~MoeGatedSwiGLU() {
    if (layer_) mxmoe_destroy(layer_);
  }

  const MoeConfig& config() const { return cfg_; }
  mxmoe_layer* raw() const { return layer_; }

  // RmsNorm gain [d], gate weight [E][d], gate bias [E] (host, f32).
  void set_router(const float* gamma, const float* gate_w, const float* gate_b) {
    check(mxmoe_set_router(layer_, gamma, gate_w, gate_b, MXMOE_F32, nullptr));
  }

  // MoeQuantLayerResident::new + set_resident; biases [E][2f] and [E][d] (f32).
  void set_resident(const quant::MoeQuantLayerHost& h, const float* mlp1_bias, const float* mlp2_bias) {
    const mxmoe_quant_desc d1 = h.w1_desc.c(), d2 = h.w2_desc.c();
    check(mxmoe_upload_experts(layer_, &d1, h.w1_blocks.data(), h.w1_scales.data(), &d2, h.w2_blocks.data(),
                               h.w2_scales.data(), mlp1_bias, mlp2_bias, MXMOE_F32, nullptr));
  }

  // forward on device buffers [n_tokens][d] (stream-ordered, asynchronous).
  void forward(const void* x, mxmoe_dtype x_dtype, void* y, mxmoe_dtype y_dtype, uint32_t n_tokens,
               void* stream = nullptr) {
    check(mxmoe_forward(layer_, x, x_dtype, y, y_dtype, n_tokens, stream));
  }

  // forward on host buffers; returns after y is written.
  void forward_host(const void* x, mxmoe_dtype x_dtype, void* y, mxmoe_dtype y_dtype, uint32_t n_tokens,
                    void* stream = nullptr) {
    check(mxmoe_forward_host(layer_, x, x_dtype, y, y_dtype, n_tokens, stream));
  }

 private:
  MoeConfig cfg_;
  mxmoe_layer* layer_ = nullptr;
};

inline MoeGatedSwiGLU MoeConfig::init(int device) const { return MoeGatedSwiGLU(*this, device); }

}  // namespace moe

namespace loader {
namespace modelbin {

// parse_modelbin (src/loader/modelbin.rs:153-156).
inline mxmoe_modelbin_header parse_modelbin(const char* path) {
  mxmoe_modelbin_header h{};
  check(mxmoe_modelbin_info(path, &h));
  return h;
}

// The MoE part of load_modelbin_into (src/loader/modelbin.rs:158-462) for one
// layer; expert_count == 0 loads every expert.
inline moe::MoeGatedSwiGLU load_moe_layer(const char* path, uint32_t layer, int device = 0, uint32_t flags = 0,
                                          uint32_t expert_begin = 0, uint32_t expert_count = 0) {
  const mxmoe_modelbin_header h = parse_modelbin(path);
  mxmoe_layer* raw = nullptr;
  check(mxmoe_modelbin_load_layer(path, layer, device, flags, expert_begin, expert_count, nullptr, &raw));
  moe::MoeConfig cfg;
  cfg.d_model = h.embedding_dim;
  cfg.ffn_hidden = h.mlp_dim;
  cfg.num_experts = h.num_experts;
  cfg.experts_per_token = h.num_active_experts;
  cfg.swiglu_limit = h.swiglu_limit;
  cfg.rms_eps = h.rms_eps;
  cfg.flags = flags;
  return moe::MoeGatedSwiGLU(cfg, raw);
}

}  // namespace modelbin

namespace mxfp4 {

// Device-side dequant_mxfp4_bytes: blocks [rows][b], scales [rows], out [rows][2b].
inline void dequant_mxfp4_bytes(const uint8_t* blocks_dev, uint64_t rows, uint64_t b, const uint8_t* scales_dev,
                                float* out_dev, void* stream = nullptr) {
  check(mxmoe_dequant_mxfp4_bytes(blocks_dev, rows, b, scales_dev, out_dev, stream));
}

}  // namespace mxfp4
}  // namespace loader

}  // namespace burn_extended
