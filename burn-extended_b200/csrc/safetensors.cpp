// Safetensors MoE loader: the GPT-OSS checkpoint's MoE tensors straight into
// a device-resident layer.
//
// Replaces load_gptoss_moe (src/loader/gpt_oss.rs:369-423), which dequantizes
// the MXFP4 blocks to f32 on the CPU (src/loader/mxfp4.rs:82-125) and targets
// `layers.{l}.mlp.mlp1_weight`, a parameter path MoeGatedSwiGLU does not have
// (src/moe/mod.rs:40-45).  Here the packed bytes are uploaded as they are
// (mxmoe_upload_experts repacks them for the tensor cores) into the layer
// object itself, with W1 read in the checkpoint's interleaved row order
// [glu0, lin0, glu1, lin1, ...] (src/activation/mod.rs:8-13), not the
// split-half order the reference's resident kernel assumes
// (src/quant/gpu.rs:108-113).
//
// Tensors of layer l (names as build_gptoss_moe_mxfp4_specs and the bias map
// use, src/loader/gpt_oss.rs:351-366, :393-414):
//   block.{l}.mlp.norm.scale            [d]                 bf16 | f32
//   block.{l}.mlp.gate.weight / .bias   [E][d] / [E]        bf16 | f32
//   block.{l}.mlp.mlp1_weight.blocks    [E][2f][d/32][16]   u8 (two E2M1 codes per byte)
//   block.{l}.mlp.mlp1_weight.scales    [E][2f][d/32]       u8 (E8M0, bias 127)
//   block.{l}.mlp.mlp1_bias             [E][2f]             bf16 | f32
//   block.{l}.mlp.mlp2_weight.blocks    [E][d][f/32][16]    u8
//   block.{l}.mlp.mlp2_weight.scales    [E][d][f/32]        u8
//   block.{l}.mlp.mlp2_bias             [E][d]              bf16 | f32
// A checkpoint may be split over several files; each tensor is looked up in
// all of them.
//
// File format: u64 little-endian header length N, N bytes of JSON
// {name: {"dtype": s, "shape": [..], "data_offsets": [begin, end]}, ...,
// "__metadata__": {..}}, then the data section the offsets index.

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/mxmoe.h"

namespace mxmoe {
int set_last_error(int code, const char* msg);
}

namespace {

constexpr uint64_t kMaxHeaderBytes = 100ull << 20;  // the format's own limit is 100 MB

int bail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return mxmoe::set_last_error(code, buf);
}

#define ST_TRY(expr)                 \
  do {                               \
    int _rc = (expr);                \
    if (_rc != MXMOE_OK) return _rc; \
  } while (0)

struct TensorInfo {
  std::string dtype;
  std::vector<uint64_t> shape;
  uint64_t begin = 0, end = 0;  // relative to the data section
};

// A JSON reader for the safetensors header: objects, arrays, strings,
// non-negative integers and the literals.  Entries other than tensor records
// (__metadata__) are parsed and dropped.
class HeaderParser {
 public:
  HeaderParser(const std::string& s, const char* path) : s_(s), path_(path) {}

  int parse(std::map<std::string, TensorInfo>& out) {
    ws();
    if (!eat('{')) return err("expected '{'");
    ws();
    if (eat('}')) return MXMOE_OK;
    for (;;) {
      std::string name;
      ST_TRY(string(name));
      ws();
      if (!eat(':')) return err("expected ':'");
      ws();
      if (name == "__metadata__") {
        ST_TRY(skip_value());
      } else {
        TensorInfo t;
        ST_TRY(tensor(t));
        out[name] = t;
      }
      ws();
      if (eat(',')) {
        ws();
        continue;
      }
      if (eat('}')) return MXMOE_OK;
      return err("expected ',' or '}'");
    }
  }

 private:
  const std::string& s_;
  const char* path_;
  size_t i_ = 0;

  int err(const char* what) {
    return bail(MXMOE_ERR_INVALID_ARG, "safetensors %s: bad header at byte %zu: %s", path_, i_, what);
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  bool eat(char c) {
    if (i_ < s_.size() && s_[i_] == c) {
      ++i_;
      return true;
    }
    return false;
  }
  int string(std::string& out) {
    if (!eat('"')) return err("expected a string");
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) break;
        char e = s_[i_++];
        switch (e) {
          case 'n': c = '\n'; break;
          case 't': c = '\t'; break;
          case 'r': c = '\r'; break;
          case 'b': c = '\b'; break;
          case 'f': c = '\f'; break;
          case 'u':  // tensor names are ASCII; keep the escape's low byte
            if (i_ + 4 > s_.size()) return err("short \\u escape");
            c = char(strtoul(s_.substr(i_, 4).c_str(), nullptr, 16) & 0xFF);
            i_ += 4;
            break;
          default: c = e;
        }
      }
      out.push_back(c);
    }
    if (!eat('"')) return err("unterminated string");
    return MXMOE_OK;
  }
  int integer(uint64_t& v) {
    if (i_ >= s_.size() || s_[i_] < '0' || s_[i_] > '9') return err("expected a non-negative integer");
    v = 0;
    while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') {
      uint64_t nv = v * 10 + uint64_t(s_[i_] - '0');
      if (nv / 10 != v) return err("integer overflow");
      v = nv;
      ++i_;
    }
    return MXMOE_OK;
  }
  int int_array(std::vector<uint64_t>& out) {
    if (!eat('[')) return err("expected '['");
    ws();
    if (eat(']')) return MXMOE_OK;
    for (;;) {
      uint64_t v;
      ST_TRY(integer(v));
      out.push_back(v);
      ws();
      if (eat(',')) {
        ws();
        continue;
      }
      if (eat(']')) return MXMOE_OK;
      return err("expected ',' or ']'");
    }
  }
  int tensor(TensorInfo& t) {
    if (!eat('{')) return err("expected a tensor record");
    bool have_dtype = false, have_shape = false, have_offsets = false;
    ws();
    if (!eat('}')) {
      for (;;) {
        std::string key;
        ST_TRY(string(key));
        ws();
        if (!eat(':')) return err("expected ':'");
        ws();
        if (key == "dtype") {
          ST_TRY(string(t.dtype));
          have_dtype = true;
        } else if (key == "shape") {
          ST_TRY(int_array(t.shape));
          have_shape = true;
        } else if (key == "data_offsets") {
          std::vector<uint64_t> o;
          ST_TRY(int_array(o));
          if (o.size() != 2 || o[1] < o[0]) return err("data_offsets must be [begin, end]");
          t.begin = o[0];
          t.end = o[1];
          have_offsets = true;
        } else {
          ST_TRY(skip_value());
        }
        ws();
        if (eat(',')) {
          ws();
          continue;
        }
        if (eat('}')) break;
        return err("expected ',' or '}'");
      }
    }
    if (!have_dtype || !have_shape || !have_offsets) return err("tensor record lacks dtype, shape or data_offsets");
    return MXMOE_OK;
  }
  int skip_value() {
    ws();
    if (i_ >= s_.size()) return err("unexpected end");
    char c = s_[i_];
    if (c == '"') {
      std::string tmp;
      return string(tmp);
    }
    if (c == '{' || c == '[') {
      const char close = c == '{' ? '}' : ']';
      ++i_;
      ws();
      if (eat(close)) return MXMOE_OK;
      for (;;) {
        if (c == '{') {
          std::string k;
          ST_TRY(string(k));
          ws();
          if (!eat(':')) return err("expected ':'");
        }
        ST_TRY(skip_value());
        ws();
        if (eat(',')) {
          ws();
          continue;
        }
        if (eat(close)) return MXMOE_OK;
        return err("unbalanced brackets");
      }
    }
    // number or literal
    size_t j = i_;
    while (i_ < s_.size() && strchr(",}] \n\r\t", s_[i_]) == nullptr) ++i_;
    if (i_ == j) return err("empty value");
    return MXMOE_OK;
  }
};

struct StFile {
  int fd = -1;
  std::string path;
  uint64_t size = 0, data_start = 0;
  std::map<std::string, TensorInfo> tensors;
  ~StFile() {
    if (fd >= 0) close(fd);
  }

  int open_parse(const char* p) {
    path = p;
    fd = ::open(p, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return bail(MXMOE_ERR_INVALID_ARG, "safetensors: cannot open %s: %s", p, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) return bail(MXMOE_ERR_INVALID_ARG, "safetensors: stat %s failed", p);
    size = uint64_t(st.st_size);
    uint8_t lenb[8];
    ST_TRY(read_raw(0, lenb, 8, "header length"));
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | lenb[i];
    if (n > kMaxHeaderBytes || n > size - 8)
      return bail(MXMOE_ERR_INVALID_ARG, "safetensors %s: header length %llu does not fit the file", p,
                  (unsigned long long)n);
    std::string hdr(n, '\0');
    ST_TRY(read_raw(8, hdr.data(), n, "header"));
    data_start = 8 + n;
    ST_TRY(HeaderParser(hdr, p).parse(tensors));
    for (const auto& kv : tensors)
      if (kv.second.end > size - data_start)
        return bail(MXMOE_ERR_INVALID_ARG, "safetensors %s: tensor %s [%llu, %llu) lies past the end of the file",
                    p, kv.first.c_str(), (unsigned long long)kv.second.begin, (unsigned long long)kv.second.end);
    return MXMOE_OK;
  }

  int read_raw(uint64_t off, void* dst, uint64_t n, const char* what) const {
    if (off > size || n > size - off)
      return bail(MXMOE_ERR_INVALID_ARG, "safetensors %s: %s lies past the end of the file", path.c_str(), what);
    char* p = static_cast<char*>(dst);
    while (n > 0) {
      ssize_t got = pread(fd, p, n > (1u << 30) ? (1u << 30) : size_t(n), off_t(off));
      if (got <= 0)
        return bail(MXMOE_ERR_INVALID_ARG, "safetensors %s: read of %s failed: %s", path.c_str(), what,
                    got < 0 ? strerror(errno) : "short read");
      p += got;
      off += uint64_t(got);
      n -= uint64_t(got);
    }
    return MXMOE_OK;
  }
};

uint64_t elem_bytes(const std::string& dt) {
  if (dt == "U8" || dt == "I8") return 1;
  if (dt == "BF16" || dt == "F16") return 2;
  if (dt == "F32") return 4;
  return 0;
}

float bf16_to_f32(uint16_t b) {
  uint32_t u = uint32_t(b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

struct Checkpoint {
  std::vector<std::unique_ptr<StFile>> files;

  int find(const std::string& name, const StFile** f, const TensorInfo** t) const {
    for (const auto& file : files) {
      auto it = file->tensors.find(name);
      if (it != file->tensors.end()) {
        *f = file.get();
        *t = &it->second;
        return MXMOE_OK;
      }
    }
    return bail(MXMOE_ERR_INVALID_ARG, "safetensors: tensor %s not found in the %zu file(s) given", name.c_str(),
                files.size());
  }

  // Looks a tensor up and checks its dtype (one of `dtypes`, "|"-separated)
  // and shape.
  int lookup(const std::string& name, const char* dtypes, const std::vector<uint64_t>& shape, const StFile** f,
             const TensorInfo** t) const {
    ST_TRY(find(name, f, t));
    const TensorInfo& ti = **t;
    std::string allowed = std::string("|") + dtypes + "|";
    if (allowed.find("|" + ti.dtype + "|") == std::string::npos)
      return bail(MXMOE_ERR_INVALID_ARG, "safetensors: %s has dtype %s, want %s", name.c_str(), ti.dtype.c_str(),
                  dtypes);
    if (ti.shape != shape) {
      std::string got, want;
      for (uint64_t v : ti.shape) got += std::to_string(v) + ",";
      for (uint64_t v : shape) want += std::to_string(v) + ",";
      return bail(MXMOE_ERR_INVALID_ARG, "safetensors: %s has shape [%s], want [%s]", name.c_str(), got.c_str(),
                  want.c_str());
    }
    uint64_t n = elem_bytes(ti.dtype);
    for (uint64_t v : shape) n *= v;
    if (ti.end - ti.begin != n)
      return bail(MXMOE_ERR_INVALID_ARG, "safetensors: %s spans %llu bytes, its shape needs %llu", name.c_str(),
                  (unsigned long long)(ti.end - ti.begin), (unsigned long long)n);
    return MXMOE_OK;
  }

  // Bytes [skip, skip + n) of a tensor's data.
  static int read(const StFile* f, const TensorInfo* t, uint64_t skip, void* dst, uint64_t n, const char* what) {
    return f->read_raw(f->data_start + t->begin + skip, dst, n, what);
  }

  // A float tensor (bf16 or f32) as f32, elements [first, first + count).
  static int read_f32(const StFile* f, const TensorInfo* t, uint64_t first, uint64_t count, std::vector<float>& out,
                      const char* what) {
    out.resize(count);
    if (t->dtype == "F32") return read(f, t, first * 4, out.data(), count * 4, what);
    std::vector<uint16_t> tmp(count);
    ST_TRY(read(f, t, first * 2, tmp.data(), count * 2, what));
    for (uint64_t i = 0; i < count; ++i) out[i] = bf16_to_f32(tmp[i]);
    return MXMOE_OK;
  }
};

}  // namespace

extern "C" {

int mxmoe_safetensors_load_layer(const char* const* paths, uint32_t n_paths, uint32_t layer,
                                 const mxmoe_config* cfg_in, uint32_t expert_begin, uint32_t expert_count,
                                 void* stream, mxmoe_layer** out) {
  if (!paths || n_paths == 0 || !cfg_in || !out)
    return bail(MXMOE_ERR_INVALID_ARG, "mxmoe_safetensors_load_layer: null argument");
  *out = nullptr;
  Checkpoint ck;
  for (uint32_t i = 0; i < n_paths; ++i) {
    if (!paths[i]) return bail(MXMOE_ERR_INVALID_ARG, "mxmoe_safetensors_load_layer: paths[%u] is null", i);
    ck.files.emplace_back(new StFile());
    ST_TRY(ck.files.back()->open_parse(paths[i]));
  }
  const std::string pre = "block." + std::to_string(layer) + ".mlp.";

  // Shapes come from the gate weight and the mlp1 blocks; the config's
  // non-zero d_model / ffn_hidden / num_experts must agree with them.
  const StFile *fg, *f1b;
  const TensorInfo *tg, *t1b;
  ST_TRY(ck.find(pre + "gate.weight", &fg, &tg));
  ST_TRY(ck.find(pre + "mlp1_weight.blocks", &f1b, &t1b));
  if (tg->shape.size() != 2 || t1b->shape.size() != 4 || t1b->shape[3] != 16 || t1b->shape[1] % 2 != 0)
    return bail(MXMOE_ERR_INVALID_ARG, "safetensors: %sgate.weight must be [E][d] and %smlp1_weight.blocks "
                "[E][2f][d/32][16]", pre.c_str(), pre.c_str());
  const uint64_t E = tg->shape[0], d = tg->shape[1], f = t1b->shape[1] / 2;
  mxmoe_config cfg = *cfg_in;
  if ((cfg.d_model && cfg.d_model != d) || (cfg.ffn_hidden && cfg.ffn_hidden != f) ||
      (cfg.num_experts && cfg.num_experts != E))
    return bail(MXMOE_ERR_INVALID_ARG, "safetensors: checkpoint layer is d=%llu f=%llu E=%llu, config says "
                "d=%u f=%u E=%u", (unsigned long long)d, (unsigned long long)f, (unsigned long long)E,
                cfg.d_model, cfg.ffn_hidden, cfg.num_experts);
  if (d % 32 != 0 || f % 32 != 0)
    return bail(MXMOE_ERR_INVALID_ARG, "safetensors: d=%llu and f=%llu must be multiples of 32", (unsigned long long)d,
                (unsigned long long)f);
  cfg.d_model = uint32_t(d);
  cfg.ffn_hidden = uint32_t(f);
  cfg.num_experts = uint32_t(E);
  cfg.flags |= MXMOE_FLAG_INTERLEAVED_GLU;  // the checkpoint's W1 row order

  const bool shard = expert_count != 0;
  const uint64_t e0 = shard ? expert_begin : 0, ne = shard ? expert_count : E;
  if (e0 + ne > E)
    return bail(MXMOE_ERR_INVALID_ARG, "safetensors: experts [%llu, +%llu) outside num_experts %llu",
                (unsigned long long)e0, (unsigned long long)ne, (unsigned long long)E);

  const char* kFloat = "BF16|F32";
  const StFile *fn, *fgb, *f1s, *f1bias, *f2b, *f2s, *f2bias;
  const TensorInfo *tn, *tgb, *t1s, *t1bias, *t2b, *t2s, *t2bias;
  ST_TRY(ck.lookup(pre + "norm.scale", kFloat, {d}, &fn, &tn));
  ST_TRY(ck.lookup(pre + "gate.weight", kFloat, {E, d}, &fg, &tg));
  ST_TRY(ck.lookup(pre + "gate.bias", kFloat, {E}, &fgb, &tgb));
  ST_TRY(ck.lookup(pre + "mlp1_weight.blocks", "U8", {E, 2 * f, d / 32, 16}, &f1b, &t1b));
  ST_TRY(ck.lookup(pre + "mlp1_weight.scales", "U8", {E, 2 * f, d / 32}, &f1s, &t1s));
  ST_TRY(ck.lookup(pre + "mlp1_bias", kFloat, {E, 2 * f}, &f1bias, &t1bias));
  ST_TRY(ck.lookup(pre + "mlp2_weight.blocks", "U8", {E, d, f / 32, 16}, &f2b, &t2b));
  ST_TRY(ck.lookup(pre + "mlp2_weight.scales", "U8", {E, d, f / 32}, &f2s, &t2s));
  ST_TRY(ck.lookup(pre + "mlp2_bias", kFloat, {E, d}, &f2bias, &t2bias));

  std::vector<float> gamma, gate_w, gate_b, b1, b2;
  ST_TRY(Checkpoint::read_f32(fn, tn, 0, d, gamma, "norm.scale"));
  ST_TRY(Checkpoint::read_f32(fg, tg, 0, E * d, gate_w, "gate.weight"));
  ST_TRY(Checkpoint::read_f32(fgb, tgb, 0, E, gate_b, "gate.bias"));
  ST_TRY(Checkpoint::read_f32(f1bias, t1bias, e0 * 2 * f, ne * 2 * f, b1, "mlp1_bias"));
  ST_TRY(Checkpoint::read_f32(f2bias, t2bias, e0 * d, ne * d, b2, "mlp2_bias"));
  const uint64_t w1b_e = 2 * f * (d / 2), w1s_e = 2 * f * (d / 32), w2b_e = d * (f / 2), w2s_e = d * (f / 32);
  std::vector<uint8_t> w1b(ne * w1b_e), w1s(ne * w1s_e), w2b(ne * w2b_e), w2s(ne * w2s_e);
  ST_TRY(Checkpoint::read(f1b, t1b, e0 * w1b_e, w1b.data(), w1b.size(), "mlp1_weight.blocks"));
  ST_TRY(Checkpoint::read(f1s, t1s, e0 * w1s_e, w1s.data(), w1s.size(), "mlp1_weight.scales"));
  ST_TRY(Checkpoint::read(f2b, t2b, e0 * w2b_e, w2b.data(), w2b.size(), "mlp2_weight.blocks"));
  ST_TRY(Checkpoint::read(f2s, t2s, e0 * w2s_e, w2s.data(), w2s.size(), "mlp2_weight.scales"));

  mxmoe_layer* L = nullptr;
  ST_TRY(mxmoe_create(&cfg, &L));
  const mxmoe_quant_desc d1{ne, 2 * f, d, d / 2, d / 32, 0};
  const mxmoe_quant_desc d2{ne, d, f, f / 2, f / 32, 0};
  int rc = MXMOE_OK;
  if (shard) rc = mxmoe_set_expert_shard(L, uint32_t(e0), uint32_t(ne));
  if (rc == MXMOE_OK) rc = mxmoe_set_router(L, gamma.data(), gate_w.data(), gate_b.data(), MXMOE_F32, stream);
  if (rc == MXMOE_OK)
    rc = mxmoe_upload_experts(L, &d1, w1b.data(), w1s.data(), &d2, w2b.data(), w2s.data(), b1.data(), b2.data(),
                              MXMOE_F32, stream);
  if (rc != MXMOE_OK) {
    mxmoe_destroy(L);
    return rc;
  }
  *out = L;
  return MXMOE_OK;
}

}  // extern "C"
