// Per-token kernels of the generation step for the stages whose whole-sequence kernels are tiled for long inputs
// (128-token tensor-core tiles, weights streamed through one tile): with one new token per sequence, B rows, those
// kernels run a handful of CTAs through the full weight matrices. These spread the weights over many CTAs instead.
//
// k_gen_front: one block per sequence computes, for its new token, the context stage (LN(h), Qc, Kc, the clock
//   projection -> beta / log_alfa, g(h), the signature) and the sign-hash projection (both MLP layers, the bucket ids),
//   with the rounding chains of k_context and k_hash_simt (asrn/estable.py:153-194, asrn/nucleo.py:639-664).
// The gate of the new tokens (k_gen_gate_tc) is in gate.cu, beside the gate's other kernels.
#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

namespace {

constexpr int kFrontThreads = 512;
constexpr int kDotWays = 4;   // dot products a warp advances together (independent loads in flight)

// Element e of a 16-byte chunk of weights as fp32.
template <typename W>
__device__ __forceinline__ float chunk_elem(const uint4& raw, int e) {
  if constexpr (sizeof(W) == 2) {
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(&raw);
    return __bfloat162float(p[e]);
  } else {
    const float* p = reinterpret_cast<const float*>(&raw);
    return p[e];
  }
}

// r[k] = sum_j x_k[j] * w_k[j] for kDotWays rows of length d at once (x in shared memory, w in global memory, rows
// 16-byte aligned and d a multiple of 16 / sizeof(W)); nrows <= kDotWays rows are valid. Results in every lane.
template <typename W>
__device__ __forceinline__ void dot_rows(const float* const* x, const W* const* w, int nrows, int d, int lane,
                                         float* r) {
  constexpr int VW = 16 / sizeof(W);
  float acc[kDotWays];
#pragma unroll
  for (int k = 0; k < kDotWays; ++k) acc[k] = 0.f;
  const int nv = d / VW;
  for (int v = lane; v < nv; v += 32) {
    uint4 raw[kDotWays];
#pragma unroll
    for (int k = 0; k < kDotWays; ++k)
      raw[k] = k < nrows ? __ldg(reinterpret_cast<const uint4*>(w[k]) + v) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < kDotWays; ++k) {
      float xv[VW];
#pragma unroll
      for (int e4 = 0; e4 < VW / 4; ++e4) {     // 16-byte shared-memory reads
        const float4 q = *reinterpret_cast<const float4*>(x[k] + v * VW + 4 * e4);
        xv[4 * e4] = q.x; xv[4 * e4 + 1] = q.y; xv[4 * e4 + 2] = q.z; xv[4 * e4 + 3] = q.w;
      }
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[k] = fmaf(xv[e], chunk_elem<W>(raw[k], e), acc[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < kDotWays; ++k) r[k] = warp_sum(acc[k]);
}

// sum_j x[j] * w[j], both in shared memory (w: act-typed row of d values, 16-byte aligned); result in every lane.
template <typename W>
__device__ __forceinline__ float dot_row_smem(const float* x, const W* w, int d, int lane) {
  constexpr int VW = 16 / sizeof(W);
  float acc = 0.f;
  for (int v = lane; v < d / VW; v += 32) {
    const uint4 raw = *reinterpret_cast<const uint4*>(w + v * VW);
    float xv[VW];
#pragma unroll
    for (int e4 = 0; e4 < VW / 4; ++e4) {
      const float4 q = *reinterpret_cast<const float4*>(x + v * VW + 4 * e4);
      xv[4 * e4] = q.x; xv[4 * e4 + 1] = q.y; xv[4 * e4 + 2] = q.z; xv[4 * e4 + 3] = q.w;
    }
#pragma unroll
    for (int e = 0; e < VW; ++e) acc = fmaf(xv[e], chunk_elem<W>(raw, e), acc);
  }
  return warp_sum(acc);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
  return s;
}

}  // namespace

template <bool Half>
__global__ void __launch_bounds__(kFrontThreads) k_gen_front(GenFrontArgs a) {
  using A = Act<Half>;
  using AT = typename A::T;
  extern __shared__ __align__(16) float sm[];
  const int d = a.d, cf = a.cf, m = a.m, P = a.P, nb = a.nb, T = a.T;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = kFrontThreads / 32;
  float* s_h = sm;                 // raw h row
  float* s_hn = s_h + d;           // LN(h), fp32
  float* s_hna = s_hn + d;         // act(LN(h))
  float* s_e = s_hna + d;          // act(E_t)
  float* s_p = s_e + d;            // act(E_{t-1})
  const int nq = 2 * cf + 3 + 3 * m;
  float* s_dot = s_p + d;          // nq dot products
  float* s_hid = s_dot + ((nq + 3) & ~3);   // 2m hidden (after GELU), 16-byte aligned
  float* s_phi = s_hid + 2 * m;    // P
  float* s_red = s_phi + ((P + 3) & ~3);   // 32, then the weight double buffer (16-byte aligned)

  const float* hrow = a.h + b * d;
  const AT* yrow = a.y ? reinterpret_cast<const AT*>(a.y) + b * d : nullptr;
  float s = 0.f;
  for (int j = tid; j < d; j += kFrontThreads) {
    const float x = yrow ? __fadd_rn(hrow[j], A::load(yrow + j)) : hrow[j];   // the residual h + y of the block
    if (a.h_sum) a.h_sum[b * d + j] = x;
    s_h[j] = x;
    s += x;
    s_e[j] = act<Half>(a.e_t[b * d + j]);
    s_p[j] = act<Half>(a.e_prev[b * d + j]);
  }
  const float mean = block_sum(s, s_red) / (float)d;
  float v = 0.f;
  for (int j = tid; j < d; j += kFrontThreads) {
    const float c = s_h[j] - mean;
    v += c * c;
  }
  const float rstd = 1.f / sqrtf(block_sum(v, s_red) / (float)d + 1e-5f);
  for (int j = tid; j < d; j += kFrontThreads) {
    const float hn = (s_h[j] - mean) * rstd * a.ln_w[j] + a.ln_b[j];
    s_hn[j] = hn;
    s_hna[j] = act<Half>(hn);
  }
  __syncthreads();

  // dot products: [0, 2cf) Qc / Kc; 2cf, 2cf + 1 the clock projection; 2cf + 2 g(h); then the 3m hidden sums
  // hp = act(E_t) . pal0, ca = act(E_t) . ctx0[:, :d], cb = act(E_{t-1}) . ctx0[:, d:]. The act-typed weight rows
  // ([cq; ck] then the 3m hidden rows) stream through a double buffer of kFrontRows-row chunks (48 KB) by bulk copies
  // on an mbarrier per buffer (bounded waits), a chunk in flight while the previous one is consumed (warp w: rows w and
  // w + 16 of the chunk); block b starts at chunk b % (number of chunks). The three fp32 rows are read directly by
  // the last warp during the first chunk.
  const AT* wctx = reinterpret_cast<const AT*>(a.wctx);
  const AT* w1 = reinterpret_cast<const AT*>(a.w1);
  const int nact = 2 * cf + 3 * m;                        // act-typed rows: Qc/Kc then the hidden sums
  constexpr int kFrontRows = Half ? 32 : 16;
  AT* s_w = reinterpret_cast<AT*>(s_red + 32);            // [2][kFrontRows][d] act weights
  const int nch = (nact + kFrontRows - 1) / kFrontRows;
  const int vpr = d * (int)sizeof(AT) / 16;               // 16-byte chunks per row
  const int rot = (int)(blockIdx.x % nch);
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_w + 2 * kFrontRows * d);     // [2] buffer-full barriers, [2] W2
  AT* s_w2 = reinterpret_cast<AT*>(bar + 4);                                    // (P, m) second hash layer
  const uint32_t w2_bytes = (uint32_t)(P * m * sizeof(AT));
  if (tid == 0) {
    umma::mbar_init(bar, 1);
    umma::mbar_init(bar + 1, 1);
    umma::mbar_init(bar + 2, 1);
    umma::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {            // the second hash layer's weights arrive while the first layer streams
    umma::mbar_expect_tx(bar + 2, w2_bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"((uint32_t)__cvta_generic_to_shared(s_w2)), "l"(a.w2), "r"(w2_bytes),
                 "r"((uint32_t)__cvta_generic_to_shared(bar + 2))
                 : "memory");
  }
  // chunk c (rows of the rotated order) into buffer c & 1: one or two bulk copies (the rows of [cq; ck] and of w1
  // are contiguous in the prepared buffer), counted on bar[c & 1]
  auto issue = [&](int c) {
    if (tid != 0) return;
    const int r0 = ((c + rot) % nch) * kFrontRows;
    const int r1 = min(r0 + kFrontRows, nact);
    AT* dst = s_w + (c & 1) * kFrontRows * d;
    const uint32_t row_bytes = (uint32_t)d * sizeof(AT);
    umma::mbar_expect_tx(bar + (c & 1), (uint32_t)(r1 - r0) * row_bytes);
    const int a0 = r0, a1 = min(r1, 2 * cf);
    if (a1 > a0)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(wctx + (int64_t)a0 * d),
                   "r"((uint32_t)(a1 - a0) * row_bytes), "r"((uint32_t)__cvta_generic_to_shared(bar + (c & 1)))
                   : "memory");
    const int b0 = max(r0, 2 * cf), b1 = r1;
    if (b1 > b0)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"((uint32_t)__cvta_generic_to_shared(dst + (b0 - r0) * d)),
                   "l"(w1 + (int64_t)(b0 - 2 * cf) * d), "r"((uint32_t)(b1 - b0) * row_bytes),
                   "r"((uint32_t)__cvta_generic_to_shared(bar + (c & 1)))
                   : "memory");
  };
  issue(0);
  if (nch > 1) issue(1);
  if (wid == nw - 1) {       // the three fp32 rows (global loads), overlapping the first chunk's copy
    const float* xs[kDotWays] = {s_hn, s_hn, s_h, s_h};
    const float* ws[kDotWays] = {a.w_reloj, a.w_reloj + d, a.g_w, a.g_w};
    float r[kDotWays];
    dot_rows<float>(xs, ws, 3, d, lane, r);
    if (lane == 0) {
      s_dot[2 * cf] = r[0];
      s_dot[2 * cf + 1] = r[1];
      s_dot[2 * cf + 2] = r[2];
    }
  }
  for (int c = 0; c < nch; ++c) {
    umma::mbar_wait(bar + (c & 1), (uint32_t)((c >> 1) & 1), a.status);
    const AT* wbuf = s_w + (c & 1) * kFrontRows * d;
    for (int r = wid; r < kFrontRows; r += nw) {
      const int q = ((c + rot) % nch) * kFrontRows + r;
      if (q >= nact) break;
      const float* x = q < 2 * cf ? s_hna : ((q - 2 * cf) < 2 * m ? s_e : s_p);
      const float r0 = dot_row_smem<AT>(x, wbuf + r * d, d, lane);
      if (lane == 0) s_dot[q < 2 * cf ? q : q + 3] = r0;
    }
    __syncthreads();                       // buffer c & 1 consumed
    if (c + 2 < nch) issue(c + 2);
  }

  if (tid < 2 * cf) {
    AT* dst = reinterpret_cast<AT*>(tid < cf ? a.Qc : a.Kc);
    A::store(dst + b * cf + (tid < cf ? tid : tid - cf), s_dot[tid]);
  } else if (tid == 2 * cf) {
    const float u0 = s_dot[2 * cf] + a.b_reloj[0];
    const float u1 = s_dot[2 * cf + 1] + a.b_reloj[1];
    a.beta[b] = (double)fminf(softplus_t(u0), a.beta_max);
    a.log_alfa[b] = fmaxf(logsigmoid_t(u1) + 0.693147180559945309f, a.log_alfa_min);
    a.glogit[b] = s_dot[2 * cf + 2] + a.g_b[0];
    a.sig[b] = (float)a.tokens[b];
  }
  const float* y = s_dot + 2 * cf + 3;
  for (int i = tid; i < m; i += kFrontThreads) {
    s_hid[i] = act<Half>(gelu_t(act<Half>(y[i] + a.b1[i])));
    s_hid[m + i] = act<Half>(gelu_t(act<Half>((y[m + i] + y[2 * m + i]) + a.b1[m + i])));
  }
  __syncthreads();
  AT* phi = reinterpret_cast<AT*>(a.phi);
  umma::mbar_wait(bar + 2, 0, a.status);
  for (int o = wid; o < P; o += nw) {
    const float* src = (o / nb < a.Tw) ? s_hid : s_hid + m;
    const float acc = dot_row_smem<AT>(src, s_w2 + (int64_t)o * m, m, lane);
    if (lane == 0) {
      const float val = act<Half>(acc + a.b2[o]);
      s_phi[o] = val;
      A::store(phi + b * P + o, val);
    }
  }
  __syncthreads();
  if (tid < T) {
    uint32_t id = 0;
    for (int j = 0; j < nb; ++j) id |= (s_phi[tid * nb + j] > 0.f ? 1u : 0u) << j;
    a.ids[b * T + tid] = (uint16_t)id;
  }
}

// ---- the same front split over more blocks (with a scratch buffer of the dot products) ------------------------------
// k_gen_front_dots: block (b, slice) recomputes LN(h), act(E_t), act(E_{t-1}) of sequence b (cheap) and takes the
//   slice's kFrontRows act weight rows ([cq; ck] then the 3m hidden rows) in one bulk copy: B x ceil(nact / rows)
//   blocks instead of B, each streaming 1 / nch of the weights. Slice 0 also takes the three fp32 rows. The dot
//   products land in dots (B, nq) in the single-block kernel's order, with the same per-row arithmetic.
// k_gen_front_out: one block per sequence turns them into the outputs (the second hash layer, the ids).
constexpr int kF1Threads = 256;

template <bool Half>
__global__ void __launch_bounds__(kF1Threads) k_gen_front_dots(GenFrontArgs a) {
  using AT = typename Act<Half>::T;
  extern __shared__ __align__(16) float sm[];
  const int d = a.d, cf = a.cf, m = a.m;
  const int nq = 2 * cf + 3 + 3 * m, nact = 2 * cf + 3 * m;
  constexpr int kRows = Half ? 32 : 16;
  const int64_t b = blockIdx.x;
  const int slice = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = kF1Threads / 32;
  float* s_h = sm;
  float* s_hn = s_h + d;
  float* s_hna = s_hn + d;
  float* s_e = s_hna + d;
  float* s_p = s_e + d;
  float* s_red = s_p + d;                                   // 32
  AT* s_w = reinterpret_cast<AT*>(s_red + 32);              // [kRows][d]
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_w + kRows * d);
  const int r0 = slice * kRows, r1 = min(r0 + kRows, nact);
  if (tid == 0) {
    umma::mbar_init(bar, 1);
    umma::fence_mbar_init();
    const AT* wctx = reinterpret_cast<const AT*>(a.wctx);
    const AT* w1 = reinterpret_cast<const AT*>(a.w1);
    const uint32_t row_bytes = (uint32_t)d * sizeof(AT);
    umma::mbar_expect_tx(bar, (uint32_t)(r1 - r0) * row_bytes);
    const int a0 = r0, a1 = min(r1, 2 * cf);
    if (a1 > a0)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"((uint32_t)__cvta_generic_to_shared(s_w)), "l"(wctx + (int64_t)a0 * d),
                   "r"((uint32_t)(a1 - a0) * row_bytes), "r"((uint32_t)__cvta_generic_to_shared(bar))
                   : "memory");
    const int b0 = max(r0, 2 * cf), b1 = r1;
    if (b1 > b0)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"((uint32_t)__cvta_generic_to_shared(s_w + (b0 - r0) * d)),
                   "l"(w1 + (int64_t)(b0 - 2 * cf) * d), "r"((uint32_t)(b1 - b0) * row_bytes),
                   "r"((uint32_t)__cvta_generic_to_shared(bar))
                   : "memory");
  }
  const float* hrow = a.h + b * d;
  const AT* yrow = a.y ? reinterpret_cast<const AT*>(a.y) + b * d : nullptr;
  float s = 0.f;
  for (int j = tid; j < d; j += kF1Threads) {
    const float x = yrow ? __fadd_rn(hrow[j], Act<Half>::load(yrow + j)) : hrow[j];   // the residual h + y
    if (a.h_sum && slice == 0) a.h_sum[b * d + j] = x;
    s_h[j] = x;
    s += x;
    s_e[j] = act<Half>(a.e_t[b * d + j]);
    s_p[j] = act<Half>(a.e_prev[b * d + j]);
  }
  const float mean = block_sum(s, s_red) / (float)d;
  float v = 0.f;
  for (int j = tid; j < d; j += kF1Threads) {
    const float c = s_h[j] - mean;
    v += c * c;
  }
  const float rstd = 1.f / sqrtf(block_sum(v, s_red) / (float)d + 1e-5f);
  for (int j = tid; j < d; j += kF1Threads) {
    const float hn = (s_h[j] - mean) * rstd * a.ln_w[j] + a.ln_b[j];
    s_hn[j] = hn;
    s_hna[j] = act<Half>(hn);
  }
  __syncthreads();
  float* dots = a.dots + b * nq;
  if (slice == 0 && wid == nw - 1) {      // the three fp32 rows, while the copy is in flight
    const float* xs[kDotWays] = {s_hn, s_hn, s_h, s_h};
    const float* ws[kDotWays] = {a.w_reloj, a.w_reloj + d, a.g_w, a.g_w};
    float r[kDotWays];
    dot_rows<float>(xs, ws, 3, d, lane, r);
    if (lane == 0) {
      dots[2 * cf] = r[0];
      dots[2 * cf + 1] = r[1];
      dots[2 * cf + 2] = r[2];
    }
  }
  umma::mbar_wait(bar, 0u, a.status);
  for (int r = wid; r < r1 - r0; r += nw) {
    const int q = r0 + r;
    const float* x = q < 2 * cf ? s_hna : ((q - 2 * cf) < 2 * m ? s_e : s_p);
    const float rv = dot_row_smem<AT>(x, s_w + r * d, d, lane);
    if (lane == 0) dots[q < 2 * cf ? q : q + 3] = rv;
  }
}

template <bool Half>
__global__ void __launch_bounds__(kF1Threads) k_gen_front_out(GenFrontArgs a) {
  using A = Act<Half>;
  using AT = typename A::T;
  __shared__ __align__(16) float s_dot[2 * kMaxConfirm + 3 + 3 * 128 + 4];
  __shared__ __align__(16) float s_hid[2 * 128];
  __shared__ float s_phi[kMaxPhi];
  const int cf = a.cf, m = a.m, P = a.P, nb = a.nb, T = a.T;
  const int nq = 2 * cf + 3 + 3 * m;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = kF1Threads / 32;
  for (int i = tid; i < nq; i += kF1Threads) s_dot[i] = a.dots[b * nq + i];
  __syncthreads();
  if (tid < 2 * cf) {
    AT* dst = reinterpret_cast<AT*>(tid < cf ? a.Qc : a.Kc);
    A::store(dst + b * cf + (tid < cf ? tid : tid - cf), s_dot[tid]);
  } else if (tid == 2 * cf) {
    const float u0 = s_dot[2 * cf] + a.b_reloj[0];
    const float u1 = s_dot[2 * cf + 1] + a.b_reloj[1];
    a.beta[b] = (double)fminf(softplus_t(u0), a.beta_max);
    a.log_alfa[b] = fmaxf(logsigmoid_t(u1) + 0.693147180559945309f, a.log_alfa_min);
    a.glogit[b] = s_dot[2 * cf + 2] + a.g_b[0];
    a.sig[b] = (float)a.tokens[b];
  }
  const float* y = s_dot + 2 * cf + 3;
  for (int i = tid; i < m; i += kF1Threads) {
    s_hid[i] = act<Half>(gelu_t(act<Half>(y[i] + a.b1[i])));
    s_hid[m + i] = act<Half>(gelu_t(act<Half>((y[m + i] + y[2 * m + i]) + a.b1[m + i])));
  }
  __syncthreads();
  AT* phi = reinterpret_cast<AT*>(a.phi);
  const AT* w2 = reinterpret_cast<const AT*>(a.w2);
  for (int o = wid * kDotWays; o < P; o += nw * kDotWays) {
    const float* xs[kDotWays];
    const AT* ws[kDotWays];
#pragma unroll
    for (int k = 0; k < kDotWays; ++k) {
      const int oo = min(o + k, P - 1);
      xs[k] = (oo / nb < a.Tw) ? s_hid : s_hid + m;
      ws[k] = w2 + (int64_t)oo * m;
    }
    float r[kDotWays];
    dot_rows<AT>(xs, ws, min(kDotWays, P - o), m, lane, r);
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < kDotWays; ++k) {
        if (o + k >= P) break;
        const float val = act<Half>(r[k] + a.b2[o + k]);
        s_phi[o + k] = val;
        A::store(phi + b * P + o + k, val);
      }
    }
  }
  __syncthreads();
  if (tid < T) {
    uint32_t id = 0;
    for (int j = 0; j < nb; ++j) id |= (s_phi[tid * nb + j] > 0.f ? 1u : 0u) << j;
    a.ids[b * T + tid] = (uint16_t)id;
  }
}

size_t gen_front_smem(const GenFrontArgs& a, bool half) {
  const size_t f = sizeof(float) * (5 * (size_t)a.d + ((2 * a.cf + 3 + 3 * a.m + 3) & ~3) + 2 * a.m + ((a.P + 3) & ~3) + 32);
  const size_t rows = half ? 32 : 16, es = half ? 2 : 4;
  return ((f + 15) / 16) * 16 + 2 * rows * (size_t)a.d * es + 32 + (size_t)a.P * a.m * es;
}

int launch_gen_front(const GenFrontArgs& a, bool half, cudaStream_t s) {
  if (a.B == 0) return ASRN_OK;
  // 16-byte weight rows: d and m multiples of 8 (bf16) / 4 (fp32); the prepared buffer's rows are then aligned
  if (a.d % 8 != 0 || a.m % 8 != 0) return ASRN_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a.w_reloj) | reinterpret_cast<uintptr_t>(a.g_w)) & 15) return ASRN_ERR_ARG;
  if (a.dots) {             // split over (sequence, slice of weight rows) blocks
    if (a.m > 128 || a.cf > kMaxConfirm || a.P > kMaxPhi) return ASRN_ERR_UNSUPPORTED;
    const int rows = half ? 32 : 16, es = half ? 2 : 4;
    const int nact = 2 * a.cf + 3 * a.m;
    const size_t smem1 = sizeof(float) * (5 * (size_t)a.d + 32) + (size_t)rows * a.d * es + 16;
    const dim3 g1((unsigned)a.B, (unsigned)((nact + rows - 1) / rows));
    if (half) {
      cudaFuncSetAttribute(k_gen_front_dots<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
      k_gen_front_dots<true><<<g1, kF1Threads, smem1, s>>>(a);
      k_gen_front_out<true><<<(unsigned)a.B, kF1Threads, 0, s>>>(a);
    } else {
      cudaFuncSetAttribute(k_gen_front_dots<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
      k_gen_front_dots<false><<<g1, kF1Threads, smem1, s>>>(a);
      k_gen_front_out<false><<<(unsigned)a.B, kF1Threads, 0, s>>>(a);
    }
    return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
  }
  const size_t smem = gen_front_smem(a, half);
  if (smem > 220 * 1024) return ASRN_ERR_UNSUPPORTED;
  if (half) {
    cudaFuncSetAttribute(k_gen_front<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_gen_front<true><<<(unsigned)a.B, kFrontThreads, smem, s>>>(a);
  } else {
    cudaFuncSetAttribute(k_gen_front<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_gen_front<false><<<(unsigned)a.B, kFrontThreads, smem, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
