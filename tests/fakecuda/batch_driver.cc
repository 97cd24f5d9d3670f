// Drives the C ABI's batch mode (go-infer_b200/csrc/capi.cu, compiled
// against the fake runtime of this folder) through the call patterns of
// go-infer's prefill: every chain is run call by call and inside one batch,
// and the results must agree bit for bit.  Prints "ok" or the first failure.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "cuda_runtime.h"  // the fake runtime of this folder
#include "goinfer_cuda.h"

float fake_weight(int qtype, const uint8_t* row, int64_t c);
float fake_silu_mul(float g, float u);

#define CHECK(c)                                                                        \
  do {                                                                                  \
    if (!(c)) {                                                                         \
      std::printf("FAIL line %d: %s (%s)\n", __LINE__, #c, gi_cuda_last_error());       \
      return 1;                                                                         \
    }                                                                                   \
  } while (0)

namespace {

uint32_t rng_state = 12345;
float frand() {
  rng_state = rng_state * 1664525u + 1013904223u;
  return ((rng_state >> 8) & 0xFFFF) / 32768.0f - 1.0f;
}
std::vector<float> vec(size_t n) {
  std::vector<float> v(n);
  for (auto& x : v) x = frand();
  return v;
}
std::vector<uint8_t> bytes(size_t n) {
  std::vector<uint8_t> v(n);
  for (auto& b : v) b = (uint8_t)(rng_state = rng_state * 1664525u + 1013904223u, rng_state >> 24);
  return v;
}
bool same(const std::vector<float>& a, const std::vector<float>& b) {
  return a.size() == b.size() && std::memcmp(a.data(), b.data(), sizeof(float) * a.size()) == 0;
}
bool all_nan_free_equal(const std::vector<float>& a, float v) {
  for (float x : a)
    if (x != v) return false;
  return true;
}

std::vector<gi_cuda_buffer_t> all_buffers;  // released at the end of main

struct Mat {
  int qtype;
  int rows, cols;
  std::vector<uint8_t> host;
  gi_cuda_buffer_t buf;
};

Mat make_mat(int qtype, int rows, int cols) {
  Mat m{qtype, rows, cols, {}, nullptr};
  const size_t rb = (size_t)gi_quant_row_bytes(qtype, cols);
  if (qtype == GI_TYPE_F32) {
    std::vector<float> f = vec((size_t)rows * cols);
    m.host.resize(rb * rows);
    std::memcpy(m.host.data(), f.data(), m.host.size());
  } else {
    m.host = bytes(rb * rows);
  }
  m.buf = gi_cuda_create_buffer(m.host.data(), m.host.size());
  all_buffers.push_back(m.buf);
  return m;
}

// y = W x on the host with the fake kernels' arithmetic (index order).
std::vector<float> host_gemv(const Mat& m, const float* x) {
  const size_t rb = (size_t)gi_quant_row_bytes(m.qtype, m.cols);
  std::vector<float> y(m.rows);
  for (int r = 0; r < m.rows; ++r) {
    float s = 0.f;
    for (int c = 0; c < m.cols; ++c) s += fake_weight(m.qtype, m.host.data() + r * rb, c) * x[c];
    y[r] = s;
  }
  return y;
}

}  // namespace

int main() {
  CHECK(gi_cuda_init() == 0);
  const int B = 3, D = 256, H = 512;

  // ---- A: the prefill FFN with gate, up and SwiGLU apart (forward.go:604-642) ----
  {
    Mat wg = make_mat(GI_TYPE_F32, H, D), wu = make_mat(GI_TYPE_F32, H, D), wd = make_mat(GI_TYPE_F32, D, H);
    const std::vector<float> x = vec((size_t)B * D), r0 = vec((size_t)B * D);
    auto chain = [&](std::vector<float>& g, std::vector<float>& u, std::vector<float>& d, std::vector<float>& r,
                     bool batch) -> int {
      g.assign((size_t)B * H, -7.f);
      u.assign((size_t)B * H, -7.f);
      d.assign((size_t)B * D, -7.f);
      r = r0;
      if (batch) gi_cuda_begin_batch();
      CHECK(gi_cuda_gemm_buf(GI_TYPE_F32, g.data(), x.data(), wg.buf, B, H, D) == 0);
      CHECK(gi_cuda_gemm_buf(GI_TYPE_F32, u.data(), x.data(), wu.buf, B, H, D) == 0);
      CHECK(gi_cuda_swiglu(g.data(), u.data(), B * H) == 0);
      CHECK(gi_cuda_gemm_buf(GI_TYPE_F32, d.data(), g.data(), wd.buf, B, D, H) == 0);
      CHECK(gi_cuda_add_residual(r.data(), d.data(), B * D) == 0);
      if (batch) {
        // Metal's contract: nothing reaches the host slices before end_batch
        CHECK(all_nan_free_equal(g, -7.f) && all_nan_free_equal(d, -7.f) && same(r, r0));
        gi_cuda_end_batch();
      }
      return 0;
    };
    std::vector<float> g1, u1, d1, r1, g2, u2, d2, r2;
    CHECK(chain(g1, u1, d1, r1, false) == 0);
    CHECK(chain(g2, u2, d2, r2, true) == 0);
    CHECK(same(g1, g2) && same(u1, u2) && same(d1, d2) && same(r1, r2));
    // and against the host arithmetic
    for (int b = 0; b < B; ++b) {
      std::vector<float> g = host_gemv(wg, x.data() + b * D), u = host_gemv(wu, x.data() + b * D);
      for (int i = 0; i < H; ++i) g[i] = fake_silu_mul(g[i], u[i]);
      std::vector<float> d = host_gemv(wd, g.data());
      for (int i = 0; i < D; ++i) CHECK(r1[b * D + i] == r0[b * D + i] + d[i]);
      CHECK(std::memcmp(g1.data() + b * H, g.data(), sizeof(float) * H) == 0);
    }
  }

  // ---- B: fused gate/up (Q4_K) feeding down and the residual in one batch ----
  {
    Mat qg = make_mat(GI_TYPE_Q4_K, H, D), qu = make_mat(GI_TYPE_Q4_K, H, D), qd = make_mat(GI_TYPE_Q4_K, D, H);
    for (int batch : {1, B}) {
      const std::vector<float> x = vec((size_t)batch * D), r0 = vec((size_t)batch * D);
      std::vector<float> g[2], d[2], r[2];
      for (int pass = 0; pass < 2; ++pass) {
        g[pass].assign((size_t)batch * H, 0.f);
        d[pass].assign((size_t)batch * D, 0.f);
        r[pass] = r0;
        if (pass) gi_cuda_begin_batch();
        CHECK(gi_cuda_gemm_fused_gate_up_buf(GI_TYPE_Q4_K, g[pass].data(), x.data(), qg.buf, qu.buf, batch, H, D) ==
              0);
        CHECK(gi_cuda_gemm_buf(GI_TYPE_Q4_K, d[pass].data(), g[pass].data(), qd.buf, batch, D, H) == 0);
        CHECK(gi_cuda_add_residual(r[pass].data(), d[pass].data(), batch * D) == 0);
        if (pass) gi_cuda_end_batch();
      }
      CHECK(same(g[0], g[1]) && same(d[0], d[1]) && same(r[0], r[1]));
    }
  }

  // ---- C: an input straddling two outputs of the batch ----
  {
    Mat w1 = make_mat(GI_TYPE_F32, H, D), w2 = make_mat(GI_TYPE_F32, D, H);
    const std::vector<float> xa = vec(D), xb = vec(D);
    std::vector<float> h[2], y[2];
    for (int pass = 0; pass < 2; ++pass) {
      h[pass].assign(2 * H, 0.f);
      y[pass].assign(D, 0.f);
      if (pass) gi_cuda_begin_batch();
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, h[pass].data(), xa.data(), w1.buf, H, D) == 0);
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, h[pass].data() + H, xb.data(), w1.buf, H, D) == 0);
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, y[pass].data(), h[pass].data() + H / 2, w2.buf, D, H) == 0);
      if (pass) gi_cuda_end_batch();
    }
    CHECK(same(h[0], h[1]) && same(y[0], y[1]));
  }

  // ---- D: a newer output inside an older one, then reads of both ranges ----
  {
    Mat wbig = make_mat(GI_TYPE_F32, 2 * H, D), wsmall = make_mat(GI_TYPE_F32, H / 2, D);
    Mat wr = make_mat(GI_TYPE_F32, D, 2 * H), wq = make_mat(GI_TYPE_F32, D, H / 2);
    const std::vector<float> x = vec(D), x2 = vec(D);
    std::vector<float> big[2], y1[2], y2[2];
    for (int pass = 0; pass < 2; ++pass) {
      big[pass].assign(2 * H, 0.f);
      y1[pass].assign(D, 0.f);
      y2[pass].assign(D, 0.f);
      if (pass) gi_cuda_begin_batch();
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, big[pass].data(), x.data(), wbig.buf, 2 * H, D) == 0);
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, big[pass].data() + H / 2, x2.data(), wsmall.buf, H / 2, D) == 0);
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, y2[pass].data(), big[pass].data() + H / 2, wq.buf, D, H / 2) == 0);
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, y1[pass].data(), big[pass].data(), wr.buf, D, 2 * H) == 0);
      if (pass) gi_cuda_end_batch();
    }
    CHECK(same(big[0], big[1]) && same(y1[0], y1[1]) && same(y2[0], y2[1]));
  }

  // ---- E: repeated in-place updates of one output ----
  {
    Mat w = make_mat(GI_TYPE_F32, H, D);
    const std::vector<float> x = vec(D), r0 = vec(H);
    std::vector<float> p[2], r[2];
    for (int pass = 0; pass < 2; ++pass) {
      p[pass].assign(H, 0.f);
      r[pass] = r0;
      if (pass) gi_cuda_begin_batch();
      CHECK(gi_cuda_gemv_buf(GI_TYPE_F32, p[pass].data(), x.data(), w.buf, H, D) == 0);
      CHECK(gi_cuda_add_residual(r[pass].data(), p[pass].data(), H) == 0);
      CHECK(gi_cuda_add_residual(r[pass].data(), p[pass].data(), H) == 0);
      CHECK(gi_cuda_swiglu(p[pass].data(), r[pass].data(), H) == 0);
      CHECK(gi_cuda_add_residual(r[pass].data(), p[pass].data(), H) == 0);
      if (pass) gi_cuda_end_batch();
    }
    CHECK(same(p[0], p[1]) && same(r[0], r[1]));
  }

  // ---- F: a batch larger than the activation arena (overflow blocks) ----
  {
    const int R = 4096, C = 256, BB = 64;  // each output 1 MiB, each input 64 KiB
    Mat w = make_mat(GI_TYPE_F32, R, C), w2 = make_mat(GI_TYPE_F32, C, R);
    const std::vector<float> x = vec((size_t)BB * C);
    std::vector<float> o[2][12], z[2];
    for (int pass = 0; pass < 2; ++pass) {
      if (pass) gi_cuda_begin_batch();
      for (int i = 0; i < 12; ++i) {
        o[pass][i].assign((size_t)BB * R, 0.f);
        CHECK(gi_cuda_gemm_buf(GI_TYPE_F32, o[pass][i].data(), x.data(), w.buf, BB, R, C) == 0);
      }
      z[pass].assign((size_t)BB * C, 0.f);
      CHECK(gi_cuda_gemm_buf(GI_TYPE_F32, z[pass].data(), o[pass][11].data(), w2.buf, BB, C, R) == 0);
      if (pass) gi_cuda_end_batch();
    }
    for (int i = 0; i < 12; ++i) CHECK(same(o[0][i], o[1][i]));
    CHECK(same(z[0], z[1]));
    // the next batch of the same size fits the grown arena
    gi_cuda_begin_batch();
    std::vector<float> again((size_t)BB * R, 0.f);
    CHECK(gi_cuda_gemm_buf(GI_TYPE_F32, again.data(), x.data(), w.buf, BB, R, C) == 0);
    gi_cuda_end_batch();
    CHECK(same(again, o[0][0]));
  }

  // ---- G: status codes of the new entry points ----
  {
    Mat q = make_mat(GI_TYPE_Q4_K, 16, 256);
    std::vector<float> y(16), x(256), a(8, 1.f);
    CHECK(gi_cuda_gemm_fused_gate_up_buf(GI_TYPE_Q6_K, y.data(), x.data(), q.buf, q.buf, 1, 16, 256) == -2);
    CHECK(gi_cuda_gemm_fused_gate_up_buf(GI_TYPE_Q4_K, y.data(), x.data(), nullptr, q.buf, 1, 16, 256) == -1);
    CHECK(gi_cuda_gemm_fused_gate_up_buf(GI_TYPE_Q4_K, y.data(), x.data(), q.buf, q.buf, 1, 32, 256) == -4);
    CHECK(gi_cuda_add_residual(a.data(), a.data(), 0) == -4);
    CHECK(gi_cuda_swiglu(nullptr, a.data(), 8) == -4);
    CHECK(gi_cuda_add_residual(a.data(), a.data(), 8) == 0 && a[0] == 2.f && a[7] == 2.f);
    CHECK(gi_cuda_model_set_persistent(nullptr, 1) == -4);
    CHECK(gi_cuda_set_q6k_mma(1) == 0 && gi_cuda_set_q6k_mma(0) == 0);
  }

  // ---- H: the no-alloc prefill against gi_cuda_gemm_dev, device pointers ----
  {
    Mat q = make_mat(GI_TYPE_Q4_K, 64, 512);
    const int BB = 20;
    const std::vector<float> x = vec((size_t)BB * 512);
    float *xd = nullptr, *y1 = nullptr, *y2 = nullptr;
    CHECK(cudaMalloc(&xd, sizeof(float) * x.size()) == cudaSuccess);
    CHECK(cudaMalloc(&y1, sizeof(float) * BB * 64) == cudaSuccess);
    CHECK(cudaMalloc(&y2, sizeof(float) * BB * 64) == cudaSuccess);
    CHECK(cudaMemcpy(xd, x.data(), sizeof(float) * x.size(), cudaMemcpyHostToDevice) == cudaSuccess);
    const void* wd = gi_cuda_buffer_device_ptr(q.buf);
    CHECK(wd != nullptr);
    CHECK(gi_cuda_gemm_dev(GI_TYPE_Q4_K, y1, xd, wd, q.host.size(), BB, 64, 512, nullptr) == 0);
    std::vector<float> a((size_t)BB * 64), b((size_t)BB * 64);
    CHECK(cudaMemcpy(a.data(), y1, sizeof(float) * a.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
    for (int call = 0; call < 2; ++call) {
      CHECK(cudaMemset(y2, 0xFF, sizeof(float) * b.size()) == cudaSuccess);
      CHECK(gi_cuda_gemm_dev_noalloc(GI_TYPE_Q4_K, y2, xd, wd, q.host.size(), BB, 64, 512, nullptr) == 0);
      CHECK(cudaMemcpy(b.data(), y2, sizeof(float) * b.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
      CHECK(same(a, b));
    }
    CHECK(gi_cuda_gemm_dev_noalloc(GI_TYPE_Q6_K, y2, xd, wd, q.host.size(), BB, 64, 512, nullptr) == -4);
    cudaFree(xd);
    cudaFree(y1);
    cudaFree(y2);
  }

  for (gi_cuda_buffer_t b : all_buffers) gi_cuda_release_buffer(b);
  std::printf("ok\n");
  return 0;
}
