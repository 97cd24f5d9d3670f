// quantize.cu -- quantisers that produce GGUF Q8_0 / Q4_K / Q6_K rows, on the
// host and (for the synthetic benchmark models) on the device.
//
// Model-preparation tooling (the counterpart of go-infer's cmd/quantize),
// not part of the GEMV path.  Q8_0 follows go-infer's own QuantizeQ8_0
// (pkg/quant/quant.go:407-455) including its truncating fp16 conversion
// (pkg/quant/fp16.go:38-69).  go-infer ships no Q4_K or Q6_K quantiser, so
// those two are this library's own min/max fits written from the block
// formats that DequantizeQ4_K / DequantizeQ6_K decode
// (pkg/quant/quant.go:215-291).  Every step is a single IEEE float32
// operation (host code built with -ffp-contract=off, device code with
// -fmad=false), so host and device quantise a block identically.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "gemv.cuh"

#define GI_HD __host__ __device__ inline

namespace gi {
namespace {

GI_HD uint32_t f2u(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
GI_HD float u2f(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// fp32 -> fp16 by truncation of the mantissa, as go-infer's FP32ToFP16.
GI_HD uint16_t f32_to_f16_trunc(float val) {
  const uint32_t bits = f2u(val);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  int exp = (int)((bits >> 23) & 0xFF);
  uint32_t mant = bits & 0x007FFFFFu;
  if (exp == 255) return (uint16_t)(sign | (mant ? 0x7E00u : 0x7C00u));
  exp = exp - 127 + 15;
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant = (mant | 0x00800000u) >> (1 - exp);
    return (uint16_t)(sign | (mant >> 13));
  }
  return (uint16_t)(sign | ((uint32_t)exp << 10) | (mant >> 13));
}

// Exact fp16 -> fp32 for every finite value.
GI_HD float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1F, mant = h & 0x3FFu;
  if (exp == 0) {
    if (mant == 0) return u2f(sign);
    exp = 1;
    while (!(mant & 0x400u)) {
      mant <<= 1;
      exp--;
    }
    mant &= 0x3FFu;
    return u2f(sign | ((exp + 112) << 23) | (mant << 13));
  }
  if (exp == 0x1F) return u2f(sign | 0x7F800000u | (mant << 13));
  return u2f(sign | ((exp + 112) << 23) | (mant << 13));
}

GI_HD void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[1] = (uint8_t)(v >> 8);
}

// QuantizeQ8_0 for one row of `n` floats (n a multiple of 32).
GI_HD void q8_0_row(const float* src, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const float* s = src + 32 * b;
    float maxv = 0.f;
    for (int i = 0; i < 32; ++i) {
      const float v = fabsf(s[i]);
      if (v > maxv) maxv = v;
    }
    float scale = maxv / 127.0f;
    uint16_t h = 0;
    if (scale > 0) {
      h = f32_to_f16_trunc(scale);
      scale = f16_to_f32(h);
    }
    const float inv = scale > 0 ? 1.0f / scale : 0.f;
    uint8_t* o = out + 34 * b;
    put16(o, h);
    for (int i = 0; i < 32; ++i) {
      int8_t q = 0;
      if (inv > 0) {
        float v = s[i] * inv;
        if (v > 127) v = 127;
        else if (v < -128) v = -128;
        q = (int8_t)roundf(v);
      }
      o[2 + i] = (uint8_t)q;
    }
  }
}

GI_HD float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Q4_K super-block fit: per 32-weight sub-block j, w ~ d*sc_j*q - dmin*m_j
// with q in [0,15] and 6-bit sc_j, m_j.  The offset m_j*dmin covers the
// sub-block minimum (clipped at 0), the step d*sc_j its range / 15; d and
// dmin put the largest step / offset at 63 and go through the truncating
// fp16 conversion the repository uses for every block scale.
GI_HD void q4_k_block(const float* w, uint8_t* out) {
  float step[8], off[8];
  float max_step = 0.f, max_off = 0.f;
  for (int j = 0; j < 8; ++j) {
    float lo = 0.f, hi = w[32 * j];
    for (int i = 0; i < 32; ++i) {
      const float v = w[32 * j + i];
      if (v < lo) lo = v;
      if (v > hi) hi = v;
    }
    step[j] = (hi - lo) / 15.0f;
    off[j] = -lo;
    if (step[j] > max_step) max_step = step[j];
    if (off[j] > max_off) max_off = off[j];
  }
  const uint16_t dh = f32_to_f16_trunc(max_step / 63.0f);
  const uint16_t mh = f32_to_f16_trunc(max_off / 63.0f);
  const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  uint8_t sc[8], mn[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = d > 0 ? (uint8_t)clampf(roundf(step[j] / d), 0.f, 63.f) : 0;
    mn[j] = dmin > 0 ? (uint8_t)clampf(roundf(off[j] / dmin), 0.f, 63.f) : 0;
  }
  put16(out, dh);
  put16(out + 2, mh);
  uint8_t* scales = out + 4;
  // Inverse of getScaleMin (pkg/quant/quant.go:228-235).
  for (int j = 0; j < 4; ++j) {
    scales[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    scales[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    scales[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; ++j) {
    const float ds = d * (float)sc[j];
    const float dm = dmin * (float)mn[j];
    for (int i = 0; i < 32; ++i) {
      float v = 0.f;
      if (ds > 0) v = clampf(roundf((w[32 * j + i] + dm) / ds), 0.f, 15.f);
      q[32 * j + i] = (uint8_t)v;
    }
  }
  // Nibble order of DequantizeQ4_K (pkg/quant/quant.go:237-249).
  uint8_t* qs = out + 16;
  for (int c = 0; c < 4; ++c)
    for (int l = 0; l < 32; ++l)
      qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

// Q6_K super-block fit: per 16-weight sub-block s, w ~ d*sc_s*q with
// q in [-32,31] and int8 sc_s; step = max|w| / 31, d puts the largest step
// at 127.  Layout of DequantizeQ6_K (pkg/quant/quant.go:263-286).
GI_HD void q6_k_block(const float* w, uint8_t* out) {
  float step[16], max_step = 0.f;
  for (int s = 0; s < 16; ++s) {
    float amax = 0.f;
    for (int i = 0; i < 16; ++i) {
      const float v = fabsf(w[16 * s + i]);
      if (v > amax) amax = v;
    }
    step[s] = amax / 31.0f;
    if (step[s] > max_step) max_step = step[s];
  }
  const uint16_t dh = f32_to_f16_trunc(max_step / 127.0f);
  const float d = f16_to_f32(dh);
  int8_t sc[16];
  for (int s = 0; s < 16; ++s)
    sc[s] = d > 0 ? (int8_t)clampf(roundf(step[s] / d), -128.f, 127.f) : 0;
  uint8_t q[256];  // stored as q + 32
  for (int s = 0; s < 16; ++s) {
    const float ds = d * (float)sc[s];
    for (int i = 0; i < 16; ++i) {
      float v = 0.f;
      if (ds > 0) v = clampf(roundf(w[16 * s + i] / ds), -32.f, 31.f);
      q[16 * s + i] = (uint8_t)((int)v + 32);
    }
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  for (int i = 0; i < 210; ++i) out[i] = 0;
  for (int n = 0; n < 2; ++n)
    for (int l = 0; l < 32; ++l) {
      const int b = 128 * n + l;
      const uint8_t q1 = q[b], q2 = q[b + 32], q3 = q[b + 64], q4 = q[b + 96];
      ql[64 * n + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[64 * n + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  for (int s = 0; s < 16; ++s) out[192 + s] = (uint8_t)sc[s];
  put16(out + 208, dh);
}

}  // namespace

// Quantise rows x cols floats into `dst` (rows * row_bytes(qtype, cols)
// bytes), splitting rows over `threads` host threads.
int quantize_host(int qtype, const float* src, int64_t rows, int64_t cols, uint8_t* dst,
                  int threads) {
  const int64_t block = qtype == kTypeQ8_0 ? 32 : 256;
  if (qtype != kTypeQ8_0 && qtype != kTypeQ4_K && qtype != kTypeQ6_K) return -2;
  if (rows < 1 || cols < block || cols % block) return -4;
  const int64_t rb = row_bytes(qtype, cols);
  auto work = [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      const float* s = src + r * cols;
      uint8_t* o = dst + r * rb;
      if (qtype == kTypeQ8_0) {
        q8_0_row(s, cols, o);
      } else {
        for (int64_t b = 0; b < cols / 256; ++b) {
          if (qtype == kTypeQ4_K) q4_k_block(s + 256 * b, o + 144 * b);
          else q6_k_block(s + 256 * b, o + 210 * b);
        }
      }
    }
  };
  if (threads < 1) threads = 1;
  if (threads > rows) threads = (int)rows;
  if (threads == 1) {
    work(0, rows);
    return 0;
  }
  std::vector<std::thread> pool;
  const int64_t chunk = (rows + threads - 1) / threads;
  for (int i = 0; i < threads; ++i) {
    const int64_t r0 = i * chunk, r1 = r0 + chunk < rows ? r0 + chunk : rows;
    if (r0 < r1) pool.emplace_back(work, r0, r1);
  }
  for (auto& th : pool) th.join();
  return 0;
}

// Seeded N(0, std) weights, quantised row by row without holding the fp32
// matrix.  Every 256-column block of row r draws from its own splitmix64
// stream keyed by (seed, r, block), so any rows and any 256-aligned column
// range can be generated on their own (tensor-parallel shards) and the
// bytes do not depend on the thread count.  The normal deviates come from
// the Marsaglia polar method in double precision, with the logarithm
// written out below: every step is an integer operation or one correctly
// rounded double add, multiply, divide or square root, so the host
// (gi_quantize_seeded) and the device (gi_synth_weights) produce the same
// bytes.  F32 writes the float32 values themselves.
namespace {
GI_HD uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Correctly rounded double operations, spelled out so that the device
// compiler cannot contract them (the host build uses -ffp-contract=off).
GI_HD double dadd(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dadd_rn(a, b);
#else
  return a + b;
#endif
}
GI_HD double dmul(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dmul_rn(a, b);
#else
  return a * b;
#endif
}
GI_HD double ddiv(double a, double b) {
#ifdef __CUDA_ARCH__
  return __ddiv_rn(a, b);
#else
  return a / b;
#endif
}
GI_HD double dsqrt(double a) {
#ifdef __CUDA_ARCH__
  return __dsqrt_rn(a);
#else
  return std::sqrt(a);
#endif
}

// Natural logarithm of a positive normal double: s = m * 2^k with m in
// [sqrt(1/2), sqrt(2)), ln m = 2 atanh(t) = 2 (t + t^3/3 + t^5/5 + ...) with
// t = (m - 1) / (m + 1), |t| < 0.172, summed to t^23 (the next term is
// below 2^-60 of the total).
GI_HD double log_pos(double s) {
  uint64_t bits;
  std::memcpy(&bits, &s, 8);
  int k = (int)((bits >> 52) & 0x7FF) - 1023;
  bits = (bits & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull;
  double m;
  std::memcpy(&m, &bits, 8);
  if (m > 1.4142135623730951) {
    m = dmul(m, 0.5);
    ++k;
  }
  const double t = ddiv(dadd(m, -1.0), dadd(m, 1.0));
  const double r = dmul(t, t);
  double p = 2.0 / 23.0;
  p = dadd(dmul(p, r), 2.0 / 21.0);
  p = dadd(dmul(p, r), 2.0 / 19.0);
  p = dadd(dmul(p, r), 2.0 / 17.0);
  p = dadd(dmul(p, r), 2.0 / 15.0);
  p = dadd(dmul(p, r), 2.0 / 13.0);
  p = dadd(dmul(p, r), 2.0 / 11.0);
  p = dadd(dmul(p, r), 2.0 / 9.0);
  p = dadd(dmul(p, r), 2.0 / 7.0);
  p = dadd(dmul(p, r), 2.0 / 5.0);
  p = dadd(dmul(p, r), 2.0 / 3.0);
  const double lnm = dadd(dmul(2.0, t), dmul(dmul(t, r), p));
  return dadd(dmul((double)k, 0.6931471805599453), lnm);  // + k ln 2
}

GI_HD uint64_t block_stream(uint64_t seed, int64_t row, int64_t blk) {
  return seed * 0xD1B54A32D192ED03ull ^ (uint64_t)row * 0x8CB92BA72F3D8DD7ull ^
         (uint64_t)blk * 0xA0761D6478BD642Full;
}

// The first n (<= 256) deviates of N(0, stddev) of one block's stream.
GI_HD void normal_block(uint64_t seed, int64_t row, int64_t blk, float stddev, float* out, int64_t n) {
  uint64_t s = block_stream(seed, row, blk);
  for (int64_t i = 0; i < n; i += 2) {
    double u, v, q;
    do {  // a point uniform in the unit disc (minus the centre)
      u = dadd(dmul((double)(splitmix64(s) >> 11), 0x1.0p-52), -1.0);  // [-1, 1)
      v = dadd(dmul((double)(splitmix64(s) >> 11), 0x1.0p-52), -1.0);
      q = dadd(dmul(u, u), dmul(v, v));
    } while (q >= 1.0 || q == 0.0);
    const double f = dmul(dsqrt(ddiv(dmul(-2.0, log_pos(q)), q)), (double)stddev);
    out[i] = (float)dmul(u, f);
    if (i + 1 < n) out[i + 1] = (float)dmul(v, f);
  }
}
}  // namespace

// Rows [row0, row0 + rows) and columns [col0, col0 + cols) of the seeded
// matrix (col0 a multiple of 256).
int quantize_seeded(int qtype, uint64_t seed, float stddev, int64_t row0, int64_t rows, int64_t col0, int64_t cols,
                    uint8_t* dst, int threads) {
  const bool f32 = qtype == kTypeF32;
  const int64_t block = qtype == kTypeQ8_0 ? 32 : (f32 ? 1 : 256);
  if (!f32 && qtype != kTypeQ8_0 && qtype != kTypeQ4_K && qtype != kTypeQ6_K) return -2;
  if (rows < 1 || row0 < 0 || col0 < 0 || col0 % 256 || cols < block || cols % block) return -4;
  const int64_t rb = f32 ? cols * 4 : row_bytes(qtype, cols);
  auto work = [&](int64_t r0, int64_t r1) {
    std::vector<float> buf((size_t)cols);
    for (int64_t r = r0; r < r1; ++r) {
      for (int64_t c = 0; c < cols; c += 256)
        normal_block(seed, row0 + r, (col0 + c) / 256, stddev, buf.data() + c, std::min<int64_t>(256, cols - c));
      uint8_t* o = dst + r * rb;
      if (f32) {
        std::memcpy(o, buf.data(), (size_t)cols * 4);
      } else if (qtype == kTypeQ8_0) {
        q8_0_row(buf.data(), cols, o);
      } else {
        for (int64_t b = 0; b < cols / 256; ++b) {
          if (qtype == kTypeQ4_K) q4_k_block(buf.data() + 256 * b, o + 144 * b);
          else q6_k_block(buf.data() + 256 * b, o + 210 * b);
        }
      }
    }
  };
  if (threads < 1) threads = 1;
  if (threads > rows) threads = (int)rows;
  std::vector<std::thread> pool;
  const int64_t chunk = (rows + threads - 1) / threads;
  for (int i = 0; i < threads; ++i) {
    const int64_t r0 = i * chunk, r1 = r0 + chunk < rows ? r0 + chunk : rows;
    if (r0 < r1) pool.emplace_back(work, r0, r1);
  }
  for (auto& th : pool) th.join();
  return 0;
}

// ---- device generator of the synthetic benchmark models --------------------
// gi_quantize_seeded's generator and block quantisers on the device, one
// thread per 256-column block: the same bytes as the host, in a fraction of
// a second for a 70B-shaped model.
namespace {
__global__ void synth_kernel(int qtype, uint64_t seed, float stddev, int64_t row0, int64_t rows, int64_t col0,
                             int64_t nblk, uint8_t* __restrict__ dst, int64_t rb) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nblk) return;
  const int64_t r = i / nblk, b = i - r * nblk;
  float w[256];
  normal_block(seed, row0 + r, col0 / 256 + b, stddev, w, 256);
  uint8_t* o = dst + r * rb;
  if (qtype == kTypeQ4_K) {
    q4_k_block(w, o + 144 * b);
  } else if (qtype == kTypeQ6_K) {
    q6_k_block(w, o + 210 * b);
  } else if (qtype == kTypeQ8_0) {
    q8_0_row(w, 256, o + 8 * 34 * b);
  } else {
    float* f = reinterpret_cast<float*>(o) + 256 * b;
    for (int k = 0; k < 256; ++k) f[k] = w[k];
  }
}
}  // namespace

int synth_device(int qtype, uint64_t seed, float stddev, int64_t row0, int64_t rows, int64_t col0, int64_t cols,
                 void* dst, size_t dst_bytes, cudaStream_t stream) {
  if (qtype != kTypeF32 && qtype != kTypeQ8_0 && qtype != kTypeQ4_K && qtype != kTypeQ6_K) return -2;
  if (rows < 1 || row0 < 0 || col0 < 0 || col0 % 256 || cols < 256 || cols % 256) return -4;
  const int64_t rb = qtype == kTypeF32 ? cols * 4 : row_bytes(qtype, cols);
  if (dst_bytes < (size_t)(rb * rows)) return -4;
  if (qtype == kTypeF32 && (reinterpret_cast<uintptr_t>(dst) & 3)) return -4;
  const int64_t n = rows * (cols / 256);
  synth_kernel<<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(qtype, seed, stddev, row0, rows, col0, cols / 256,
                                                                 static_cast<uint8_t*>(dst), rb);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -5;
}

}  // namespace gi
