// moe_forward.cpp -- host program on the C++ mirror (include/mxmoe.hpp):
// reads a layer and a token batch from raw little-endian files in a
// directory, runs MoeGatedSwiGLU::forward_host and writes y.
//
//   moe_forward <dir>         dir/meta.txt: d f E k n interleaved
//                             dir/{x,gamma,gate_w,gate_b,b1,b2}.f32
//                             dir/{w1_blocks,w1_scales,w2_blocks,w2_scales}.u8
//                             -> dir/y.f32
//   moe_forward --check-errors   exercises argument validation only (no GPU)
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <string>
#include <vector>

#include "mxmoe.hpp"

namespace be = burn_extended;

template <typename T>
static std::vector<T> read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  std::vector<T> out(raw.size() / sizeof(T));
  std::memcpy(out.data(), raw.data(), out.size() * sizeof(T));
  return out;
}

static int check_errors() {
  int caught = 0;
  try {
    be::moe::MoeConfig bad;
    bad.d_model = 0;
    bad.ffn_hidden = 256;
    bad.num_experts = 2;
    bad.experts_per_token = 2;
    auto layer = bad.init(0);
  } catch (const be::Error& e) {
    caught += e.status() == MXMOE_ERR_INVALID_ARG;
  }
  try {
    be::moe::MoeConfig bad{250, 256, 2, 2};
    auto layer = bad.init(0);
  } catch (const be::Error& e) {
    caught += e.status() == MXMOE_ERR_UNSUPPORTED;
  }
  std::printf("errors caught: %d\n", caught);
  return caught == 2 ? 0 : 1;
}

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: moe_forward <dir> | --check-errors\n");
    return 2;
  }
  if (std::string(argv[1]) == "--check-errors") return check_errors();
  try {
    const std::string dir = argv[1];
    std::ifstream meta(dir + "/meta.txt");
    uint32_t d, f, E, k, n, inter;
    meta >> d >> f >> E >> k >> n >> inter;
    be::moe::MoeConfig cfg{d, f, E, k};
    if (inter) cfg.flags |= MXMOE_FLAG_INTERLEAVED_GLU;
    auto layer = cfg.init(0);
    auto gamma = read_file<float>(dir + "/gamma.f32"), gw = read_file<float>(dir + "/gate_w.f32"),
         gb = read_file<float>(dir + "/gate_b.f32"), b1 = read_file<float>(dir + "/b1.f32"),
         b2 = read_file<float>(dir + "/b2.f32"), x = read_file<float>(dir + "/x.f32");
    layer.set_router(gamma.data(), gw.data(), gb.data());
    be::quant::MoeQuantLayerHost host;
    host.w1_desc = be::quant::QuantLinearMxFp4Desc::for_shape(E, 2ull * f, d);
    host.w2_desc = be::quant::QuantLinearMxFp4Desc::for_shape(E, d, f);
    host.w1_blocks = read_file<uint8_t>(dir + "/w1_blocks.u8");
    host.w1_scales = read_file<uint8_t>(dir + "/w1_scales.u8");
    host.w2_blocks = read_file<uint8_t>(dir + "/w2_blocks.u8");
    host.w2_scales = read_file<uint8_t>(dir + "/w2_scales.u8");
    layer.set_resident(host, b1.data(), b2.data());
    std::vector<float> y(x.size());
    layer.forward_host(x.data(), MXMOE_F32, y.data(), MXMOE_F32, n);
    std::ofstream out(dir + "/y.f32", std::ios::binary);
    out.write(reinterpret_cast<const char*>(y.data()), y.size() * sizeof(float));
    std::printf("ok %u tokens\n", n);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
}
