// model.bin reader: the MoE part of burn-extended's loader
// (src/loader/modelbin.rs) on top of the library's own C ABI.
//
// File layout (what parse_headers and load_modelbin_into walk,
// src/loader/modelbin.rs:75-151 and :158-462; written by
// src/bin/gptoss_export.rs):
//   magic[16] ("GPT-OSS v1.0" in the first 12 bytes), model uuid[16]
//   u32 context_length, num_blocks, num_experts, num_active_experts,
//       embedding_dim, mlp_dim; f32 swiglu_limit; u32 head_dim, num_heads,
//       num_kv_heads, attention_window; f32 rope_theta, interpolation_scale,
//       yarn_offset, yarn_scale, yarn_multiplier, rms_eps; layout uuid[16]
//   tokenizer uuid[16]; u32 num_special, num_text, regex_size, tokens_size;
//       special-token uuids [num_special][16]; regex; token blob
//   pad to 16 KiB
//   bf16 embedding [num_text + num_special][d]
//   per layer, every segment starting 16-byte aligned: attention norm [d];
//       qkv weight [hd*(nh+2*kv)][d] followed by its bias; sinks [nh];
//       attention out weight [d][nh*hd] followed by its bias [d];
//       MoE norm [d]; gate weight [E][d] followed by its bias [E]
//   final norm [d]; unembedding [num_text + num_special][d] (16-byte aligned)
//   per layer, padded to 16 KiB, per expert, each segment 16-byte aligned:
//       mlp1 blocks [2f][ceil(d/2)], mlp1 scales [2f][ceil(d/32)] (E8M0 + 14),
//       mlp1 bias bf16 [2f], mlp2 blocks [d][ceil(f/2)],
//       mlp2 scales [d][ceil(f/32)] (E8M0 + 14), mlp2 bias bf16 [d]
// Offsets are computed from the header, every read is bounds-checked against
// the file size, and the expert bytes go straight to mxmoe_upload_experts,
// which repacks them into the tensor-core layout on the device.

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "../../include/mxmoe.h"

namespace mxmoe {
int set_last_error(int code, const char* msg);
}

namespace {

constexpr uint64_t kSectionAlign = 16;
constexpr uint64_t kPageAlign = 16384;
constexpr int kModelBinUe8Offset = 14;      // src/loader/modelbin.rs:452-453
constexpr float kGptOssSwigluAlpha = 1.702f;  // src/activation/mod.rs:6

int bail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return mxmoe::set_last_error(code, buf);
}

uint64_t align_up(uint64_t off, uint64_t a) { return (off + a - 1) / a * a; }

// Owns one read-only descriptor; every read is a positioned read checked
// against the file size.
struct File {
  int fd = -1;
  uint64_t size = 0;
  const char* path = "";
  ~File() {
    if (fd >= 0) close(fd);
  }
  int open_path(const char* p) {
    path = p;
    fd = ::open(p, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return bail(MXMOE_ERR_INVALID_ARG, "model.bin: cannot open %s: %s", p, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) return bail(MXMOE_ERR_INVALID_ARG, "model.bin: stat %s failed", p);
    size = uint64_t(st.st_size);
    return MXMOE_OK;
  }
  int read_at(uint64_t off, void* dst, uint64_t n, const char* what) const {
    if (off > size || n > size - off)
      return bail(MXMOE_ERR_INVALID_ARG, "model.bin %s: %s [%llu, +%llu) lies past the end of the file (%llu bytes)",
                  path, what, (unsigned long long)off, (unsigned long long)n, (unsigned long long)size);
    char* p = static_cast<char*>(dst);
    while (n > 0) {
      ssize_t got = pread(fd, p, n > (1u << 30) ? (1u << 30) : size_t(n), off_t(off));
      if (got <= 0)
        return bail(MXMOE_ERR_INVALID_ARG, "model.bin %s: read of %s failed: %s", path, what,
                    got < 0 ? strerror(errno) : "short read");
      p += got;
      off += uint64_t(got);
      n -= uint64_t(got);
    }
    return MXMOE_OK;
  }
};

#define MB_TRY(expr)               \
  do {                             \
    int _rc = (expr);              \
    if (_rc != MXMOE_OK) return _rc; \
  } while (0)

// Little-endian scalar fields, read in file order.
struct Cursor {
  const File& f;
  uint64_t off;
  int rc = MXMOE_OK;
  template <typename T>
  T next(const char* what) {
    T v{};
    if (rc == MXMOE_OK) {
      rc = f.read_at(off, &v, sizeof(T), what);
      off += sizeof(T);
    }
    return v;
  }
  void skip(uint64_t n) { off += n; }
};

// Byte offsets of one expert's six segments inside a layer payload.
struct ExpertSegs {
  uint64_t w1_blocks, w1_scales, w1_bias, w2_blocks, w2_scales, w2_bias;
};

struct Plan {
  mxmoe_modelbin_header info{};
  uint64_t w1_blocks_bytes = 0, w1_scales_bytes = 0, w1_bias_bytes = 0;
  uint64_t w2_blocks_bytes = 0, w2_scales_bytes = 0, w2_bias_bytes = 0;
  uint64_t bpr1 = 0, gpr1 = 0, bpr2 = 0, gpr2 = 0;
  std::vector<uint64_t> mlp_norm, gate_w;  // per layer
  uint64_t expert_stride = 0;              // bytes between consecutive experts
  uint64_t expert0_rel[6] = {};            // expert 0's segments, relative to the payload start

  uint64_t payload(uint32_t layer) const { return info.moe_offset + uint64_t(layer) * info.moe_layer_stride; }
  ExpertSegs expert(uint32_t layer, uint32_t e) const {
    uint64_t b = payload(layer) + uint64_t(e) * expert_stride;
    return {b + expert0_rel[0], b + expert0_rel[1], b + expert0_rel[2],
            b + expert0_rel[3], b + expert0_rel[4], b + expert0_rel[5]};
  }
};

int parse(const File& f, Plan& P) {
  char magic[16];
  MB_TRY(f.read_at(0, magic, sizeof(magic), "magic"));
  if (memcmp(magic, "GPT-OSS v1.0", 12) != 0)
    return bail(MXMOE_ERR_INVALID_ARG, "model.bin %s: invalid magic header", f.path);
  mxmoe_modelbin_header& I = P.info;
  Cursor c{f, 32};  // after magic + model uuid
  I.context_length = c.next<uint32_t>("context_length");
  I.num_blocks = c.next<uint32_t>("num_blocks");
  I.num_experts = c.next<uint32_t>("num_experts");
  I.num_active_experts = c.next<uint32_t>("num_active_experts");
  I.embedding_dim = c.next<uint32_t>("embedding_dim");
  I.mlp_dim = c.next<uint32_t>("mlp_dim");
  I.swiglu_limit = c.next<float>("swiglu_limit");
  I.head_dim = c.next<uint32_t>("head_dim");
  I.num_heads = c.next<uint32_t>("num_heads");
  I.num_kv_heads = c.next<uint32_t>("num_kv_heads");
  I.attention_window = c.next<uint32_t>("attention_window");
  c.skip(5 * sizeof(float));  // rope_theta, interpolation_scale, yarn offset / scale / multiplier
  I.rms_eps = c.next<float>("rms_eps");
  c.skip(16 + 16);  // layout uuid, tokenizer uuid
  I.num_special_tokens = c.next<uint32_t>("num_special");
  I.num_text_tokens = c.next<uint32_t>("num_text");
  uint32_t regex_size = c.next<uint32_t>("regex_size");
  uint32_t tokens_size = c.next<uint32_t>("tokens_size");
  MB_TRY(c.rc);
  c.skip(uint64_t(I.num_special_tokens) * 16 + regex_size + tokens_size);
  I.dense_offset = align_up(c.off, kPageAlign);
  I.file_bytes = f.size;

  if (I.embedding_dim == 0 || I.mlp_dim == 0 || I.num_experts == 0 || I.num_active_experts == 0 ||
      I.num_active_experts > I.num_experts)
    return bail(MXMOE_ERR_INVALID_ARG, "model.bin %s: bad MoE header (d=%u f=%u E=%u k=%u)", f.path,
                I.embedding_dim, I.mlp_dim, I.num_experts, I.num_active_experts);

  const uint64_t d = I.embedding_dim, f2 = 2ull * I.mlp_dim, fh = I.mlp_dim, E = I.num_experts;
  const uint64_t included = uint64_t(I.num_text_tokens) + I.num_special_tokens;
  const uint64_t qkv_rows = uint64_t(I.head_dim) * (uint64_t(I.num_heads) + 2ull * I.num_kv_heads);
  const uint64_t attn_cols = uint64_t(I.num_heads) * I.head_dim;

  uint64_t off = I.dense_offset + included * d * 2;  // embedding
  P.mlp_norm.resize(I.num_blocks);
  P.gate_w.resize(I.num_blocks);
  for (uint32_t l = 0; l < I.num_blocks; ++l) {
    off = align_up(off, kSectionAlign) + d * 2;                                // attention norm
    off = align_up(off, kSectionAlign) + qkv_rows * d * 2 + qkv_rows * 2;      // qkv weight + bias
    off = align_up(off, kSectionAlign) + uint64_t(I.num_heads) * 2;            // sinks
    off = align_up(off, kSectionAlign) + d * attn_cols * 2 + d * 2;            // out weight + bias
    P.mlp_norm[l] = align_up(off, kSectionAlign);
    off = P.mlp_norm[l] + d * 2;
    P.gate_w[l] = align_up(off, kSectionAlign);
    off = P.gate_w[l] + E * d * 2 + E * 2;                                     // gate weight + bias
  }
  off = align_up(off, kSectionAlign) + d * 2;              // final norm
  off = align_up(off, kSectionAlign) + included * d * 2;   // unembedding

  P.bpr1 = (d + 1) / 2;
  P.gpr1 = (d + 31) / 32;
  P.bpr2 = (fh + 1) / 2;
  P.gpr2 = (fh + 31) / 32;
  P.w1_blocks_bytes = f2 * P.bpr1;
  P.w1_scales_bytes = f2 * P.gpr1;
  P.w1_bias_bytes = f2 * 2;
  P.w2_blocks_bytes = d * P.bpr2;
  P.w2_scales_bytes = d * P.gpr2;
  P.w2_bias_bytes = d * 2;

  // One expert's segments from a payload start; the payload start is 16 KiB
  // aligned, so every expert after the first sits at the same relative
  // alignment and the walk is periodic with a 16-byte-aligned stride.
  const uint64_t seg_bytes[6] = {P.w1_blocks_bytes, P.w1_scales_bytes, P.w1_bias_bytes,
                                 P.w2_blocks_bytes, P.w2_scales_bytes, P.w2_bias_bytes};
  uint64_t rel = 0;
  for (int s = 0; s < 6; ++s) {
    rel = align_up(rel, kSectionAlign);
    P.expert0_rel[s] = rel;
    rel += seg_bytes[s];
  }
  P.expert_stride = align_up(rel, kSectionAlign);
  const uint64_t layer_bytes = (E - 1) * P.expert_stride + rel;
  I.moe_offset = align_up(off, kPageAlign);
  I.moe_layer_stride = align_up(layer_bytes, kPageAlign);
  return MXMOE_OK;
}

}  // namespace

extern "C" {

int mxmoe_modelbin_info(const char* path, mxmoe_modelbin_header* out) {
  if (!path || !out) return bail(MXMOE_ERR_INVALID_ARG, "mxmoe_modelbin_info: null argument");
  File f;
  MB_TRY(f.open_path(path));
  Plan P;
  MB_TRY(parse(f, P));
  *out = P.info;
  return MXMOE_OK;
}

int mxmoe_modelbin_load_layer(const char* path, uint32_t layer, int32_t device, uint32_t flags,
                              uint32_t expert_begin, uint32_t expert_count, void* stream, mxmoe_layer** out) {
  if (!path || !out) return bail(MXMOE_ERR_INVALID_ARG, "mxmoe_modelbin_load_layer: null argument");
  *out = nullptr;
  File f;
  MB_TRY(f.open_path(path));
  Plan P;
  MB_TRY(parse(f, P));
  const mxmoe_modelbin_header& I = P.info;
  if (layer >= I.num_blocks)
    return bail(MXMOE_ERR_INVALID_ARG, "model.bin %s: layer %u out of range (num_blocks %u)", path, layer,
                I.num_blocks);
  const bool shard = expert_count != 0;
  const uint32_t e0 = shard ? expert_begin : 0;
  const uint32_t ne = shard ? expert_count : I.num_experts;
  if (uint64_t(e0) + ne > I.num_experts)
    return bail(MXMOE_ERR_INVALID_ARG, "model.bin %s: experts [%u, +%u) outside num_experts %u", path, e0, ne,
                I.num_experts);
  // The last byte this layer's payload uses must be inside the file.
  const ExpertSegs last = P.expert(layer, I.num_experts - 1);
  if (last.w2_bias + P.w2_bias_bytes > f.size)
    return bail(MXMOE_ERR_INVALID_ARG,
                "model.bin %s: layer %u expert payload ends at byte %llu, past the end of the file (%llu bytes)",
                path, layer, (unsigned long long)(last.w2_bias + P.w2_bias_bytes), (unsigned long long)f.size);

  const uint64_t d = I.embedding_dim, E = I.num_experts;
  std::vector<uint16_t> gamma(d), gate_w(E * d), gate_b(E);
  MB_TRY(f.read_at(P.mlp_norm[layer], gamma.data(), d * 2, "mlp.norm.scale"));
  MB_TRY(f.read_at(P.gate_w[layer], gate_w.data(), E * d * 2, "mlp.gate.weight"));
  MB_TRY(f.read_at(P.gate_w[layer] + E * d * 2, gate_b.data(), E * 2, "mlp.gate.bias"));

  std::vector<uint8_t> w1b(ne * P.w1_blocks_bytes), w1s(ne * P.w1_scales_bytes);
  std::vector<uint8_t> w2b(ne * P.w2_blocks_bytes), w2s(ne * P.w2_scales_bytes);
  std::vector<uint8_t> b1(ne * P.w1_bias_bytes), b2(ne * P.w2_bias_bytes);
  for (uint32_t i = 0; i < ne; ++i) {
    const ExpertSegs s = P.expert(layer, e0 + i);
    MB_TRY(f.read_at(s.w1_blocks, &w1b[i * P.w1_blocks_bytes], P.w1_blocks_bytes, "mlp1 blocks"));
    MB_TRY(f.read_at(s.w1_scales, &w1s[i * P.w1_scales_bytes], P.w1_scales_bytes, "mlp1 scales"));
    MB_TRY(f.read_at(s.w1_bias, &b1[i * P.w1_bias_bytes], P.w1_bias_bytes, "mlp1 bias"));
    MB_TRY(f.read_at(s.w2_blocks, &w2b[i * P.w2_blocks_bytes], P.w2_blocks_bytes, "mlp2 blocks"));
    MB_TRY(f.read_at(s.w2_scales, &w2s[i * P.w2_scales_bytes], P.w2_scales_bytes, "mlp2 scales"));
    MB_TRY(f.read_at(s.w2_bias, &b2[i * P.w2_bias_bytes], P.w2_bias_bytes, "mlp2 bias"));
  }

  mxmoe_config cfg{};
  cfg.d_model = I.embedding_dim;
  cfg.ffn_hidden = I.mlp_dim;
  cfg.num_experts = I.num_experts;
  cfg.experts_per_token = I.num_active_experts;
  cfg.swiglu_alpha = kGptOssSwigluAlpha;
  cfg.swiglu_limit = I.swiglu_limit;
  cfg.rms_eps = I.rms_eps;
  cfg.flags = flags;
  cfg.device = device;
  mxmoe_layer* L = nullptr;
  MB_TRY(mxmoe_create(&cfg, &L));
  const mxmoe_quant_desc d1{ne, 2ull * I.mlp_dim, d, P.bpr1, P.gpr1, kModelBinUe8Offset};
  const mxmoe_quant_desc d2{ne, d, I.mlp_dim, P.bpr2, P.gpr2, kModelBinUe8Offset};
  int rc = MXMOE_OK;
  if (shard) rc = mxmoe_set_expert_shard(L, e0, ne);
  if (rc == MXMOE_OK)
    rc = mxmoe_set_router(L, gamma.data(), gate_w.data(), gate_b.data(), MXMOE_BF16, stream);
  if (rc == MXMOE_OK)
    rc = mxmoe_upload_experts(L, &d1, w1b.data(), w1s.data(), &d2, w2b.data(), w2s.data(), b1.data(), b2.data(),
                              MXMOE_BF16, stream);
  if (rc != MXMOE_OK) {
    // Keep the failing call's message: destroy does not overwrite it on success.
    mxmoe_destroy(L);
    return rc;
  }
  *out = L;
  return MXMOE_OK;
}

}  // extern "C"
