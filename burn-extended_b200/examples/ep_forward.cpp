// ep_forward.cpp -- the expert-parallel step through the C ABI alone
// (mxmoe_ep_reserve / mxmoe_ep_attach / mxmoe_ep_forward): `world` ranks,
// each a layer holding E / world experts, driven by its own host thread and
// CUDA stream, meet through a host barrier.  All ranks live on one GPU here
// (peer buffers are plain device pointers of this process); ranks on
// different GPUs would pass pointers opened with mxmoe_ipc_open instead.
// Every rank's output is compared with the full single-GPU layer
// (mxmoe_forward) on the same tokens, over several steps.
//
//   ep_forward [world] [tokens per rank] [steps]      exit 0 = every step within tolerance
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <thread>
#include <vector>

#include "mxmoe.h"

namespace {

#define CK(expr)                                                                                  \
  do {                                                                                            \
    const int rc_ = (expr);                                                                       \
    if (rc_ != MXMOE_OK) {                                                                        \
      char msg_[512];                                                                             \
      mxmoe_last_error(msg_, sizeof(msg_));                                                       \
      std::fprintf(stderr, "%s:%d %s -> %d: %s\n", __FILE__, __LINE__, #expr, rc_, msg_);          \
      std::exit(1);                                                                               \
    }                                                                                             \
  } while (0)
#define CU(expr)                                                                                  \
  do {                                                                                            \
    const cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess) {                                                                      \
      std::fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #expr, cudaGetErrorString(e_));   \
      std::exit(1);                                                                               \
    }                                                                                             \
  } while (0)

struct Rng {
  uint64_t s;
  uint32_t next() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return static_cast<uint32_t>(s >> 11);
  }
  float normal() {  // sum of uniforms, mean 0, unit variance
    float a = 0.0f;
    for (int i = 0; i < 12; ++i) a += static_cast<float>(next() & 0xFFFFFF) / 16777216.0f;
    return a - 6.0f;
  }
};

// The caller's barrier: each rank's stream work before the call is complete
// (stream synchronize), then all ranks meet on the host.
struct HostBarrier {
  std::mutex m;
  std::condition_variable cv;
  int world = 0, arrived = 0;
  uint64_t gen = 0;
  static int call(void* ctx, void* stream) {
    auto* b = static_cast<HostBarrier*>(ctx);
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return 1;
    std::unique_lock<std::mutex> lk(b->m);
    const uint64_t g = b->gen;
    if (++b->arrived == b->world) {
      b->arrived = 0;
      ++b->gen;
      b->cv.notify_all();
    } else {
      b->cv.wait(lk, [&] { return b->gen != g; });
    }
    return 0;
  }
};

}  // namespace

int main(int argc, char** argv) {
  const uint32_t world = argc > 1 ? std::atoi(argv[1]) : 2;
  const uint32_t n = argc > 2 ? std::atoi(argv[2]) : 48;
  const int steps = argc > 3 ? std::atoi(argv[3]) : 2;
  const uint32_t d = 256, f = 256, E = 8, k = 2;
  if (world == 0 || E % world != 0) {
    std::fprintf(stderr, "world must divide %u experts\n", E);
    return 2;
  }
  const uint32_t epr = E / world;
  Rng rng{0x9E3779B97F4A7C15ull};
  // synthetic MXFP4 layer: random E2M1 codes, E8M0 scales 2^-9 .. 2^3 (+127), small biases
  const uint64_t w1r = 2ull * f, w1b = d / 2, w1g = d / 32, w2r = d, w2b = f / 2, w2g = f / 32;
  std::vector<uint8_t> w1q(E * w1r * w1b), w1s(E * w1r * w1g), w2q(E * w2r * w2b), w2s(E * w2r * w2g);
  for (auto& v : w1q) v = rng.next() & 0xFF;
  for (auto& v : w1s) v = 118 + rng.next() % 13;
  for (auto& v : w2q) v = rng.next() & 0xFF;
  for (auto& v : w2s) v = 118 + rng.next() % 13;
  std::vector<float> b1(E * w1r), b2(E * d), gamma(d, 1.0f), gate_w(E * d), gate_b(E);
  for (auto& v : b1) v = 0.02f * rng.normal();
  for (auto& v : b2) v = 0.02f * rng.normal();
  for (auto& v : gate_w) v = 0.02f * rng.normal();
  for (auto& v : gate_b) v = 0.02f * rng.normal();

  auto make_layer = [&](uint32_t begin, uint32_t count) {
    mxmoe_config cfg{d, f, E, k, 1.702f, 7.0f, 1e-5f, 0u, 0};
    mxmoe_layer* L = nullptr;
    CK(mxmoe_create(&cfg, &L));
    CK(mxmoe_set_router(L, gamma.data(), gate_w.data(), gate_b.data(), MXMOE_F32, nullptr));
    if (count != E) CK(mxmoe_set_expert_shard(L, begin, count));
    const mxmoe_quant_desc d1{count, w1r, d, w1b, w1g, 0}, d2{count, w2r, f, w2b, w2g, 0};
    CK(mxmoe_upload_experts(L, &d1, w1q.data() + begin * w1r * w1b, w1s.data() + begin * w1r * w1g, &d2,
                            w2q.data() + begin * w2r * w2b, w2s.data() + begin * w2r * w2g, b1.data() + begin * w1r,
                            b2.data() + begin * d, MXMOE_F32, nullptr));
    return L;
  };
  mxmoe_layer* full = make_layer(0, E);
  std::vector<mxmoe_layer*> ranks(world);
  std::vector<void*> bufs(3 * world), ret(world);
  std::vector<int32_t*> counts(world);
  std::vector<char> handles(3 * MXMOE_IPC_HANDLE_BYTES);
  for (uint32_t r = 0; r < world; ++r) {
    ranks[r] = make_layer(r * epr, epr);
    CK(mxmoe_ep_reserve(ranks[r], n, world, handles.data()));
    void* b[3];
    CK(mxmoe_ep_buffers(ranks[r], b));
    for (int i = 0; i < 3; ++i) bufs[i * world + r] = b[i];
    CU(cudaMalloc(&ret[r], static_cast<size_t>(n) * k * d * 2));
    CU(cudaMalloc(reinterpret_cast<void**>(&counts[r]), static_cast<size_t>(world) * E * 4));
  }
  HostBarrier bar;
  bar.world = static_cast<int>(world);
  for (uint32_t r = 0; r < world; ++r)
    CK(mxmoe_ep_attach(ranks[r], r, world, bufs.data(), ret.data(), counts.data(), &HostBarrier::call, &bar));

  std::vector<cudaStream_t> streams(world);
  std::vector<float*> xd(world), yd(world), yref(world);
  for (uint32_t r = 0; r < world; ++r) {
    CU(cudaStreamCreateWithFlags(&streams[r], cudaStreamNonBlocking));
    CU(cudaMalloc(reinterpret_cast<void**>(&xd[r]), static_cast<size_t>(n) * d * 4));
    CU(cudaMalloc(reinterpret_cast<void**>(&yd[r]), static_cast<size_t>(n) * d * 4));
    CU(cudaMalloc(reinterpret_cast<void**>(&yref[r]), static_cast<size_t>(n) * d * 4));
  }
  int failures = 0;
  for (int step = 0; step < steps; ++step) {
    // new tokens per rank and step; the last rank gets none on odd steps
    std::vector<uint32_t> nr(world, n);
    if (step % 2 == 1) nr[world - 1] = 0;
    for (uint32_t r = 0; r < world; ++r) {
      std::vector<float> x(static_cast<size_t>(n) * d);
      for (auto& v : x) v = rng.normal();
      CU(cudaMemcpy(xd[r], x.data(), x.size() * 4, cudaMemcpyHostToDevice));
      if (nr[r] > 0) CK(mxmoe_forward(full, xd[r], MXMOE_F32, yref[r], MXMOE_F32, nr[r], nullptr));
    }
    CU(cudaDeviceSynchronize());
    std::vector<std::thread> th;
    std::vector<int> rc(world, 0);
    for (uint32_t r = 0; r < world; ++r)
      th.emplace_back([&, r] {
        rc[r] = mxmoe_ep_forward(ranks[r], xd[r], MXMOE_F32, nr[r], yd[r], MXMOE_F32, streams[r]);
        if (rc[r] == MXMOE_OK) rc[r] = mxmoe_sync_status(ranks[r], streams[r]);
      });
    for (auto& t : th) t.join();
    for (uint32_t r = 0; r < world; ++r) {
      if (rc[r] != MXMOE_OK) {
        char msg[512];
        mxmoe_last_error(msg, sizeof(msg));
        std::fprintf(stderr, "step %d rank %u: status %d (%s)\n", step, r, rc[r], msg);
        return 1;
      }
      if (nr[r] == 0) continue;
      std::vector<float> y(static_cast<size_t>(nr[r]) * d), yr(y.size());
      CU(cudaMemcpy(y.data(), yd[r], y.size() * 4, cudaMemcpyDeviceToHost));
      CU(cudaMemcpy(yr.data(), yref[r], yr.size() * 4, cudaMemcpyDeviceToHost));
      double mx = 0, mref = 0, num = 0, den = 0;
      for (size_t i = 0; i < y.size(); ++i) {
        const double e = std::fabs(static_cast<double>(y[i]) - yr[i]);
        mx = std::max(mx, e);
        mref = std::max(mref, std::fabs(static_cast<double>(yr[i])));
        num += e * e;
        den += static_cast<double>(yr[i]) * yr[i];
      }
      const double max_rel = mx / std::max(mref, 1e-30), rel_l2 = std::sqrt(num / std::max(den, 1e-30));
      const bool ok = max_rel <= 2e-2 && rel_l2 <= 1e-2;
      failures += ok ? 0 : 1;
      std::printf("step %d rank %u/%u tokens %u: max_abs/max %.3e rel_l2 %.3e %s\n", step, r, world, nr[r], max_rel,
                  rel_l2, ok ? "ok" : "FAIL");
    }
  }
  for (uint32_t r = 0; r < world; ++r) {
    CK(mxmoe_destroy(ranks[r]));
    cudaFree(ret[r]);
    cudaFree(counts[r]);
    cudaFree(xd[r]);
    cudaFree(yd[r]);
    cudaFree(yref[r]);
    cudaStreamDestroy(streams[r]);
  }
  CK(mxmoe_destroy(full));
  std::printf(failures ? "FAILED\n" : "ep_forward ok\n");
  return failures ? 1 : 0;
}
