// Device sampling with the reference's random numbers.
//
// The reference draws every generated token with torch.multinomial(prob.cpu(), 1, generator=g) on a CPU generator
// seeded once per call (asrn/nucleo.py:1962, :1996). For one sample torch takes the argmax of prob / q over each row,
// q = an Exp(1) draw per element of prob, made by the CPU exponential_ kernel: one MT19937 64-bit value (two 32-bit
// outputs, the first one high) per element in memory order, u = (value & (2^53 - 1)) * 2^-53, q = (float)(-log1p(-u)).
// So step k of a call with a (B, V) probability matrix reads the generator's outputs [2 B V k, 2 B V (k + 1)).
// Those numbers do not depend on the logits, only on the seed and the step, so they can be made on the device ahead
// of time and the draw becomes an argmax on the device: no probability matrix crosses PCIe.
//
// MT19937 (Matsumoto and Nishimura, 1998) is linear over GF(2): the 624-word window S_n = (x_n, ..., x_{n+623}) of
// its untempered word stream advances by a linear map A whose characteristic polynomial phi has degree 19937, so
// S_{n+J} = g(A) S_n = XOR over the set coefficients i of g of S_{n+i}, with g = x^J mod phi (the jump-ahead of
// Haramoto et al., 2008). The host finds phi once per process with the Berlekamp-Massey algorithm on one bit of the
// stream and raises x to the needed powers modulo phi; the device kernel gives one block to each step of a window of
// steps: the block jumps from the window's start state to its step (one jump per set bit of the step index, with the
// polynomials x^(2^l J) mod phi), then runs the recurrence over the step's 2 B V words and writes q.
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "layout.h"

namespace asrn {
namespace mt {

constexpr int kN = 624;                      // words in the state window
constexpr int kShift = 227;                  // kN - 397: the recurrence's distance to its middle term, from the end
constexpr int kDeg = 19937;                  // degree of phi
constexpr int kPolyWords = kN;               // 624 x 32 bits >= 19937 coefficients
constexpr uint32_t kMatrixA = 0x9908b0dfu;
constexpr int kJumpWords = kN + kDeg - 1;    // x_n .. x_{n + 19936 + 623}
constexpr int kRing = 4096;                  // generation ring (power of two, > kN + kGen)
constexpr int kGen = 3120;                   // words made between two consumption passes (even, <= kRing - kN)
constexpr int kThreads = 1024;

__host__ __device__ __forceinline__ uint32_t twist(uint32_t a, uint32_t b) {   // a = x_k, b = x_{k+1}
  const uint32_t y = (a & 0x80000000u) | (b & 0x7fffffffu);
  return (y >> 1) ^ ((b & 1u) ? kMatrixA : 0u);
}

__host__ __device__ __forceinline__ uint32_t temper(uint32_t y) {
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

// ---- host: phi and powers of x modulo phi ------------------------------------------------------------------------

using Poly = std::vector<uint64_t>;

inline bool bit(const Poly& p, int64_t i) { return (p[i >> 6] >> (i & 63)) & 1u; }

// p ^= q << s (bit shift), q of nq words
inline void xor_shifted(uint64_t* p, size_t np, const uint64_t* q, size_t nq, int64_t s) {
  const int64_t ws = s >> 6;
  const int bs = static_cast<int>(s & 63);
  for (size_t j = 0; j < nq; ++j) {
    const uint64_t w = q[j];
    if (!w) continue;
    const size_t k = j + ws;
    if (k < np) p[k] ^= w << bs;
    if (bs && k + 1 < np) p[k + 1] ^= w >> (64 - bs);
  }
}

// Minimal polynomial of the stream (monic, degree kDeg), found by Berlekamp-Massey on bit 0 of the untempered words
// of one seeded generator. Fails (empty result) unless the degree is 19937.
Poly characteristic() {
  constexpr int64_t n_bits = 2 * kDeg + 256;
  std::vector<uint32_t> x(kN + n_bits + 1024);
  x[0] = 5489u;
  for (int i = 1; i < kN; ++i) x[i] = 1812433253u * (x[i - 1] ^ (x[i - 1] >> 30)) + static_cast<uint32_t>(i);
  for (size_t a = kN; a < x.size(); ++a) x[a] = x[a - kShift] ^ twist(x[a - kN], x[a - kN + 1]);
  const int64_t W = n_bits / 64 + 4;
  Poly rev(W, 0);                              // bit j = s[n_bits - 1 - j]
  for (int64_t t = 0; t < n_bits; ++t)
    if (x[1000 + t] & 1u) rev[(n_bits - 1 - t) >> 6] |= 1ull << ((n_bits - 1 - t) & 63);
  Poly C(W, 0), B(W, 0), T;
  C[0] = B[0] = 1;
  int64_t L = 0, m = 1;
  for (int64_t n = 0; n < n_bits; ++n) {
    // d = parity(sum_{i=0..L} C_i s_{n-i}); s_{n-i} = rev bit (n_bits - 1 - n + i)
    const int64_t off = n_bits - 1 - n;
    const int64_t ow = off >> 6;
    const int ob = static_cast<int>(off & 63);
    uint64_t acc = 0;
    for (int64_t j = 0; j <= (L >> 6); ++j) {
      uint64_t r = rev[ow + j] >> ob;
      if (ob && ow + j + 1 < W) r |= rev[ow + j + 1] << (64 - ob);
      acc ^= C[j] & r;
    }
    if (!__builtin_parityll(acc)) {
      ++m;
      continue;
    }
    if (2 * L <= n) {
      T = C;
      xor_shifted(C.data(), W, B.data(), W, m);
      L = n + 1 - L;
      B.swap(T);
      m = 1;
    } else {
      xor_shifted(C.data(), W, B.data(), W, m);
      ++m;
    }
  }
  if (L != kDeg) return Poly();
  Poly phi(kDeg / 64 + 1, 0);                  // phi(x) = x^L C(1/x)
  for (int64_t i = 0; i <= L; ++i)
    if (bit(C, i)) phi[(L - i) >> 6] |= 1ull << ((L - i) & 63);
  return phi;
}

struct PolyMod {
  Poly phi;                                    // 312 words, bit kDeg set
  size_t nw() const { return phi.size(); }

  void mulx(Poly& r) const {
    uint64_t carry = 0;
    for (auto& w : r) {
      const uint64_t c = w >> 63;
      w = (w << 1) | carry;
      carry = c;
    }
    if (bit(r, kDeg))
      for (size_t j = 0; j < nw(); ++j) r[j] ^= phi[j];
  }

  void reduce(Poly& t) const {                 // t (any length) -> t mod phi, nw() words
    for (int64_t w = static_cast<int64_t>(t.size()) - 1; w >= 0; --w) {
      while (true) {
        const uint64_t v = t[w];
        if (!v) break;
        const int64_t top = w * 64 + 63 - __builtin_clzll(v);
        if (top < kDeg) break;
        xor_shifted(t.data(), t.size(), phi.data(), nw(), top - kDeg);
      }
    }
    t.resize(nw());
  }

  void sqr(Poly& r) const {
    Poly t(2 * nw(), 0);
    for (size_t j = 0; j < nw(); ++j) {
      const uint64_t w = r[j];
      uint64_t lo = 0, hi = 0;
      for (int b = 0; b < 32; ++b) {
        lo |= ((w >> b) & 1ull) << (2 * b);
        hi |= ((w >> (b + 32)) & 1ull) << (2 * b);
      }
      t[2 * j] = lo;
      t[2 * j + 1] = hi;
    }
    reduce(t);
    r.swap(t);
  }

  Poly pow_x(uint64_t J) const {               // x^J mod phi
    Poly r(nw(), 0);
    r[0] = 1;
    for (int b = 63; b >= 0; --b) {
      sqr(r);
      if ((J >> b) & 1u) mulx(r);
    }
    return r;
  }
};

const PolyMod* poly_mod() {
  static std::once_flag once;
  static PolyMod pm;
  std::call_once(once, [] { pm.phi = characteristic(); });
  return pm.phi.empty() ? nullptr : &pm;
}

void to_words(const Poly& p, uint32_t* out) {
  for (int w = 0; w < kPolyWords; ++w) {
    const uint64_t v = (static_cast<size_t>(w >> 1) < p.size()) ? p[w >> 1] : 0;
    out[w] = static_cast<uint32_t>((w & 1) ? v >> 32 : v);
  }
}

// ---- device ------------------------------------------------------------------------------------------------------

// buf[a] for a in [from, to) from the recurrence x_a = x_{a-227} ^ twist(x_{a-624}, x_{a-623}); 227 words at a time
__device__ __forceinline__ void extend_linear(uint32_t* buf, int from, int to) {
  for (int base = from; base < to; base += kShift) {
    const int a = base + static_cast<int>(threadIdx.x);
    if (threadIdx.x < kShift && a < to) buf[a] = buf[a - kShift] ^ twist(buf[a - kN], buf[a - kN + 1]);
    __syncthreads();
  }
}

// buf[0, 624) = S_n -> S_{n+J}, poly = x^J mod phi (624 words, global)
__device__ void jump(uint32_t* buf, const uint32_t* __restrict__ poly) {
  extend_linear(buf, kN, kJumpWords);
  const int t = threadIdx.x;
  uint32_t acc = 0;
  if (t < kN) {
    for (int w = 0; w < kPolyWords; ++w) {
      uint32_t g = __ldg(poly + w);
      while (g) {
        const int b = __ffs(g) - 1;
        g &= g - 1;
        acc ^= buf[32 * w + b + t];
      }
    }
  }
  __syncthreads();
  if (t < kN) buf[t] = acc;
  __syncthreads();
}

// Block k: the Exp(1) draws of step k of the window, q[k * draws + i] for i < draws.
__global__ void __launch_bounds__(kThreads) k_mt_fill(int64_t draws, int64_t steps, int levels,
                                                     const uint32_t* __restrict__ start,
                                                     const uint32_t* __restrict__ polys, float* __restrict__ q,
                                                     uint32_t* __restrict__ end_state) {
  extern __shared__ uint32_t buf[];            // kJumpWords words; the first kRing serve as the generation ring
  const int64_t k = blockIdx.x;
  const int t = threadIdx.x;
  if (t < kN) buf[t] = start[t];
  __syncthreads();
  for (int l = 0; l < levels; ++l)
    if ((k >> l) & 1) jump(buf, polys + static_cast<int64_t>(l) * kPolyWords);
  // ring[a & (kRing - 1)] = x_{n+a}; words a in [0, 624) are in place
  constexpr int64_t M = kRing - 1;
  const int64_t total = kN + 2 * draws;
  float* qk = q + k * draws;
  for (int64_t a0 = kN; a0 < total; a0 += kGen) {
    const int64_t a1 = (a0 + kGen < total) ? a0 + kGen : total;
    for (int64_t base = a0; base < a1; base += kShift) {
      const int64_t a = base + t;
      if (t < kShift && a < a1) buf[a & M] = buf[(a - kShift) & M] ^ twist(buf[(a - kN) & M], buf[(a - kN + 1) & M]);
      __syncthreads();
    }
    for (int64_t d = (a0 - kN) / 2 + t; d < (a1 - kN) / 2; d += kThreads) {
      const uint32_t hi = temper(buf[(kN + 2 * d) & M]);
      const uint32_t lo = temper(buf[(kN + 2 * d + 1) & M]);
      const uint64_t v = ((static_cast<uint64_t>(hi) << 32) | lo) & ((1ull << 53) - 1);
      const double u = static_cast<double>(v) * 0x1.0p-53;
      qk[d] = static_cast<float>(-log1p(-u));
    }
    __syncthreads();
  }
  if (end_state && k == steps - 1 && t < kN) end_state[t] = buf[(total - kN + t) & M];
}

// argmax over a row with torch's rule: NaN wins, equal values keep the lower index
__device__ __forceinline__ bool better(float a, int64_t ia, float b, int64_t ib) {
  if (isnan(a)) return !isnan(b) || ia < ib;
  if (isnan(b)) return false;
  return a > b || (a == b && ia < ib);
}

constexpr int kArgThreads = 512;

__global__ void __launch_bounds__(kArgThreads) k_sample_argmax(int64_t V, const float* __restrict__ prob,
                                                              const float* __restrict__ q, int64_t* __restrict__ out,
                                                              int* status) {
  const int64_t row = blockIdx.x;
  const float* p = prob + row * V;
  const float* qr = q + row * V;
  float bv = -INFINITY;
  int64_t bi = V;
  bool bad = false, pos = false;
  for (int64_t j = threadIdx.x; j < V; j += kArgThreads) {
    const float pj = __ldg(p + j);
    bad |= !(pj >= 0.f) || isinf(pj);
    pos |= pj > 0.f;
    const float r = __fdiv_rn(pj, __ldg(qr + j));
    if (better(r, j, bv, bi)) {
      bv = r;
      bi = j;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float sv[kArgThreads / 32];
  __shared__ int64_t si[kArgThreads / 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  bad = __syncthreads_or(bad);
  pos = __syncthreads_or(pos);
  if (threadIdx.x == 0) {
    for (int i = 1; i < kArgThreads / 32; ++i)
      if (better(sv[i], si[i], bv, bi)) {
        bv = sv[i];
        bi = si[i];
      }
    out[row] = bi < V ? bi : 0;
    if ((bad || !pos) && status) atomicCAS(status, 0, ASRN_ERR_DATA);
  }
}

// Plain argmax of each row with torch.argmax's rule (the greedy token of a step): T = float or bf16, rows of V values;
// bf16 rows with V % 8 == 0 are read 16 bytes at a time.
template <typename T>
__global__ void __launch_bounds__(kArgThreads) k_argmax_rows(int64_t V, const T* __restrict__ x,
                                                             int64_t* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * V;
  float bv = -INFINITY;
  int64_t bi = V;
  if constexpr (sizeof(T) == 2) {
    if (V % 8 == 0) {
      const uint4* v8 = reinterpret_cast<const uint4*>(xr);
      for (int64_t c = threadIdx.x; c < V / 8; c += kArgThreads) {
        const uint4 u = __ldg(v8 + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float f = __uint_as_float((k & 1) ? (w[k >> 1] & 0xFFFF0000u) : (w[k >> 1] << 16));
          if (better(f, 8 * c + k, bv, bi)) {
            bv = f;
            bi = 8 * c + k;
          }
        }
      }
    } else {
      for (int64_t j = threadIdx.x; j < V; j += kArgThreads) {
        const float f = __bfloat162float(xr[j]);
        if (better(f, j, bv, bi)) {
          bv = f;
          bi = j;
        }
      }
    }
  } else {
    for (int64_t j = threadIdx.x; j < V; j += kArgThreads) {
      const float f = __ldg(reinterpret_cast<const float*>(xr) + j);
      if (better(f, j, bv, bi)) {
        bv = f;
        bi = j;
      }
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float sv[kArgThreads / 32];
  __shared__ int64_t si[kArgThreads / 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < kArgThreads / 32; ++i)
      if (better(sv[i], si[i], bv, bi)) {
        bv = sv[i];
        bi = si[i];
      }
    out[row] = bi < V ? bi : 0;
  }
}

}  // namespace mt
}  // namespace asrn

extern "C" {

int asrn_argmax_rows(int64_t rows, int64_t V, const void* x, int32_t dtype, int64_t* out, void* stream) {
  using namespace asrn::mt;
  if (rows < 0 || V <= 0 || rows > 0x7fffffff || (dtype != 0 && dtype != 1)) return ASRN_ERR_ARG;
  if (rows == 0) return ASRN_OK;
  if (!x || !out) return ASRN_ERR_ARG;
  if (dtype == 1 && (reinterpret_cast<uintptr_t>(x) & 15)) return ASRN_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == 1)
    k_argmax_rows<__nv_bfloat16><<<static_cast<unsigned>(rows), kArgThreads, 0, s>>>(
        V, reinterpret_cast<const __nv_bfloat16*>(x), out);
  else
    k_argmax_rows<float><<<static_cast<unsigned>(rows), kArgThreads, 0, s>>>(V, reinterpret_cast<const float*>(x),
                                                                            out);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}


int asrn_sampler_seed_state(uint64_t seed, uint32_t* state) {
  if (!state) return ASRN_ERR_ARG;
  state[0] = static_cast<uint32_t>(seed);
  for (int i = 1; i < asrn::mt::kN; ++i)
    state[i] = 1812433253u * (state[i - 1] ^ (state[i - 1] >> 30)) + static_cast<uint32_t>(i);
  return ASRN_OK;
}

int asrn_sampler_jump_poly(uint64_t distance, uint32_t* poly) {
  using namespace asrn::mt;
  if (!poly) return ASRN_ERR_ARG;
  const PolyMod* pm = poly_mod();
  if (!pm) return ASRN_ERR_UNSUPPORTED;
  static std::mutex mu;
  static std::map<uint64_t, Poly> cache;
  Poly p;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(distance);
    if (it != cache.end()) p = it->second;
  }
  if (p.empty()) {
    Poly half;                                 // x^(2m) = (x^m)^2: one squaring when the half distance is known
    if (distance % 2 == 0) {
      std::lock_guard<std::mutex> lock(mu);
      auto it = cache.find(distance / 2);
      if (it != cache.end()) half = it->second;
    }
    if (!half.empty()) {
      pm->sqr(half);
      p.swap(half);
    } else {
      p = pm->pow_x(distance);
    }
    std::lock_guard<std::mutex> lock(mu);
    cache.emplace(distance, p);
  }
  to_words(p, poly);
  return ASRN_OK;
}

int asrn_sampler_fill(int64_t draws, int64_t steps, int32_t levels, const uint32_t* state, const uint32_t* polys,
                      float* q, uint32_t* end_state, void* stream) {
  using namespace asrn::mt;
  if (draws <= 0 || steps <= 0 || levels < 0 || levels > 30 || steps > (int64_t(1) << levels) || !state ||
      (levels && !polys) || !q)
    return ASRN_ERR_ARG;
  if (steps > 0x7fffffff || draws > (int64_t(1) << 40)) return ASRN_ERR_ARG;
  const size_t smem = static_cast<size_t>(kJumpWords) * sizeof(uint32_t);
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_mt_fill, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return ASRN_ERR_CUDA;
    attr = true;
  }
  k_mt_fill<<<static_cast<unsigned>(steps), kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      draws, steps, levels, state, polys, q, end_state);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int asrn_sample_argmax(int64_t rows, int64_t V, const float* prob, const float* q, int64_t* out, int* status,
                       void* stream) {
  using namespace asrn::mt;
  if (rows < 0 || V <= 0 || rows > 0x7fffffff) return ASRN_ERR_ARG;
  if (rows == 0) return ASRN_OK;
  if (!prob || !q || !out) return ASRN_ERR_ARG;
  k_sample_argmax<<<static_cast<unsigned>(rows), kArgThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      V, prob, q, out, status);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // extern "C"
