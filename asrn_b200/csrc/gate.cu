// Gate and output projection. Reference: CapaASRNEstable._combinar (asrn/estable.py:376-403), _senales
// (asrn/estable.py:294-300) and _respuesta_racha (asrn/nucleo.py:865-878):
//   pt = tables with candidates; mejor = max over those tables of their best score (else 0), clamped to +-mejor_max
//   logit = g(h) + g_conf([pt/T, mejor, pico/max(1,pt), pt_ctx/Tc]) + w_vistos . vistos + u_hawkes . log1p(hawkes)
//           + response(racha)                                     (all fp32; g_conf in bf16 under autocast)
//   h' = h + sigmoid(logit) * o(salida / max(1, pt))
// Here salida = W_v acc (acc = sum of att * Ea rows from the scoring kernel), so o(salida) = (W_o W_v) acc and the
// projection is one GEMM against the prepared W_ov.
#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

constexpr int kGateTM = 64, kGateTN = 64, kGateKC = 32;

// Gate of one token (sigmoid(logit), rounded to the compute type) and max(1, pt).
template <bool Half>
__device__ __forceinline__ void gate_of_token(const GateArgs& a, int64_t g, float* sigma, float* ptc) {
  const int T = a.T;
  float pt = 0.f, mejor = kProhibido, pico = 0.f, pctx = 0.f;
  for (int tau = 0; tau < T; ++tau) {
    const float hay = (float)a.sen_hay[g * T + tau];
    pt = __fadd_rn(pt, hay);
    if (hay > 0.f) mejor = fmaxf(mejor, a.sen_mx[g * T + tau]);
    pico = __fadd_rn(pico, __fmul_rn(a.sen_pk[g * T + tau], hay));
    if (tau >= T - a.Tc) pctx = __fadd_rn(pctx, hay);
  }
  mejor = fmaxf(mejor, kProhibido);
  mejor = (pt > 0.f) ? mejor : 0.f;
  mejor = fminf(fmaxf(mejor, -a.mejor_max), a.mejor_max);
  const float pt1 = fmaxf(pt, 1.f);
  float s[4] = {__fdiv_rn(pt, (float)T), mejor, __fdiv_rn(pico, pt1), __fdiv_rn(pctx, (float)a.Tc)};
  float gc = 0.f;
  for (int i = 0; i < 4; ++i) gc = fmaf(act<Half>(s[i]), a.gconf[i], gc);
  gc = act<Half>(__fadd_rn(gc, a.gconf[4]));
  float logit = __fadd_rn(a.glogit[g], gc);
  float sv = 0.f;
  for (int j = 0; j < a.n; ++j) sv = __fadd_rn(sv, __fmul_rn((float)a.vistos[g * a.n + j], a.w_vistos[j]));
  logit = __fadd_rn(logit, sv);
  float sh = 0.f;
  for (int j = 0; j < a.n; ++j) sh = __fadd_rn(sh, __fmul_rn(log1pf(a.hawkes[g * a.n + j]), a.u_hawkes[j]));
  logit = __fadd_rn(logit, sh);
  // response to the streak: linear interpolation of u_racha on x = log1p(racha) / paso, flat past the last node
  float x = __fdiv_rn(log1pf(a.racha[g]), a.racha_paso);
  x = fminf(x, (float)(a.nodes - 1));
  const float xf = (x != x) ? 0.f : x;
  int i = (int)floorf(xf);
  i = min(max(i, 0), a.nodes - 2);
  const float resp = __fadd_rn(a.u_racha[i], __fmul_rn(__fsub_rn(x, (float)i), a.d_racha[i + 1]));
  logit = __fadd_rn(logit, resp);
  if (a.tope > 0.f) logit = __fmul_rn(a.tope, tanhf(__fdiv_rn(logit, a.tope)));
  *sigma = act<Half>(1.f / (1.f + expf(-logit)));
  *ptc = pt1;
}

template <bool Half>
__global__ void __launch_bounds__(256) k_gate_simt(GateArgs a) {
  using A = Act<Half>;
  __shared__ float s_sigma[kGateTM], s_pt[kGateTM];
  __shared__ __align__(16) float As[kGateKC][kGateTM];
  __shared__ __align__(16) float Bs[kGateKC][kGateTN];
  const int64_t M = a.B * a.L;
  const int d = a.d;
  const int64_t t0 = (int64_t)blockIdx.y * kGateTM;
  const int n0 = blockIdx.x * kGateTN;
  const int tid = threadIdx.x;
  for (int r = tid; r < kGateTM; r += blockDim.x) {
    const int64_t g = t0 + r;
    float sg = 0.f, pt = 1.f;
    if (g < M) gate_of_token<Half>(a, g, &sg, &pt);
    s_sigma[r] = sg;
    s_pt[r] = pt;
  }
  __syncthreads();
  const int tr = tid >> 4, tc = tid & 15;
  float acc[4][4] = {};
  const typename A::T* W = reinterpret_cast<const typename A::T*>(a.wov);
  for (int k0 = 0; k0 < d; k0 += kGateKC) {
    for (int e = tid; e < kGateTM * kGateKC; e += blockDim.x) {
      const int r = e / kGateKC, kk = e % kGateKC;
      const int64_t g = t0 + r;
      const int k = k0 + kk;
      As[kk][r] = (g < M && k < d) ? act<Half>(__fdiv_rn(a.acc[g * d + k], s_pt[r])) : 0.f;
    }
    for (int e = tid; e < kGateTN * kGateKC; e += blockDim.x) {
      const int c = e / kGateKC, kk = e % kGateKC;
      const int k = k0 + kk;
      Bs[kk][c] = (n0 + c < d && k < d) ? A::load(W + (int64_t)(n0 + c) * d + k) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kGateKC; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&As[kk][tr * 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk][tc * 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w}, br[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = tr * 4 + i;
    const int64_t g = t0 + r;
    if (g >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tc * 4 + j;
      if (c >= d) continue;
      const float o = act<Half>(acc[i][j]);
      const float add = act<Half>(__fmul_rn(s_sigma[r], o));
      a.out[g * d + c] = __fadd_rn(a.h[g * d + c], add);
    }
  }
}

// ---- tensor-core version (bf16 autocast mode) -------------------------------------------------------------------
// Tile: 128 tokens (TMEM lanes) x NT output columns (TMEM columns), K = d in chunks of 64. A = bf16(acc / max(1,pt))
// built by the threads in the 128-byte-swizzled K-major layout; B = rows [n0, n0 + NT) of W_ov by TMA; the fp32
// accumulator in TMEM; the epilogue transposes 32 x 32 blocks through shared memory so that h is read and h'
// written in coalesced rows.
namespace {
constexpr int kGTM = 128, kGBK = 64, kGThreads = 256;
constexpr int kGStageA = kGTM * 128;
}  // namespace

template <int NT>
__global__ void __launch_bounds__(kGThreads, 2) k_gate_tc(const __grid_constant__ CUtensorMap tmap_wov, GateArgs a) {
  using namespace umma;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  constexpr int kStageB = NT * 128;
  uint8_t* sA = sm;
  uint8_t* sB = sm + 2 * kGStageA;
  uint8_t* tail = sB + 2 * kStageB;
  uint64_t* full_b = reinterpret_cast<uint64_t*>(tail);
  uint64_t* mma_done = full_b + 2;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(full_b + 4);
  int* abort_s = reinterpret_cast<int*>(tmem_base_s + 1);
  float* s_sigma = reinterpret_cast<float*>(tmem_base_s + 4);
  float* s_pt = s_sigma + kGTM;
  float* tr = reinterpret_cast<float*>(sm);          // epilogue: [8 warps][32][33], reuses the stage buffers

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int d = a.d;
  const int nk = d / kGBK;
  const int n0 = blockIdx.x * NT;
  const int64_t M = a.B * a.L;
  const int64_t m0 = (int64_t)blockIdx.y * kGTM;
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(full_b + i, 1);
    *abort_s = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_wov);
  }
  if (wid == 0) {
    tmem_alloc(tmem_base_s, NT < 32 ? 32 : NT);
    tmem_relinquish();
  }
  if (tid < kGTM) {
    float sg = 0.f, pt = 1.f;
    if (m0 + tid < M) gate_of_token<true>(a, m0 + tid, &sg, &pt);
    s_sigma[tid] = sg;
    s_pt[tid] = pt;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;

  const int ar = tid >> 1, ah = tid & 1;
  const int64_t ag = m0 + ar;
  const bool arow_ok = ag < M;
  const float* arow = a.acc + (arow_ok ? ag : 0) * (int64_t)d + ah * 32;
  const float pt_r = s_pt[ar];
  float4 pre[8];
  auto load_chunk = [&](int k) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      pre[i] = arow_ok ? __ldg(reinterpret_cast<const float4*>(arow + k * kGBK) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  load_chunk(0);
  const uint32_t idesc = idesc_bf16(kGTM, NT);
  bool ok = true;
  for (int k = 0; k < nk; ++k) {
    const int s = k & 1;
    if (k >= 2) ok = mbar_wait(mma_done + s, ((k - 2) >> 1) & 1, a.status) && ok;
    if (tid == 0 && ok) {
      mbar_expect_tx(full_b + s, (uint32_t)kStageB);
      tma_load_2d(sB + s * kStageB, &tmap_wov, k * kGBK, n0, full_b + s);
    }
    uint8_t* dstA = sA + s * kGStageA;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 x0 = pre[2 * c], x1 = pre[2 * c + 1];
      const uint4 q = make_uint4(pack_bf16x2(__fdiv_rn(x0.x, pt_r), __fdiv_rn(x0.y, pt_r)),
                                 pack_bf16x2(__fdiv_rn(x0.z, pt_r), __fdiv_rn(x0.w, pt_r)),
                                 pack_bf16x2(__fdiv_rn(x1.x, pt_r), __fdiv_rn(x1.y, pt_r)),
                                 pack_bf16x2(__fdiv_rn(x1.z, pt_r), __fdiv_rn(x1.w, pt_r)));
      *reinterpret_cast<uint4*>(dstA + umma::sw128_offset(ar, ah * 4 + c)) = q;
    }
    if (k + 1 < nk) load_chunk(k + 1);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (ok) ok = mbar_wait(full_b + s, (k >> 1) & 1, a.status);
      if (ok) {
        const uint32_t a0 = smem_u32(dstA), b0 = smem_u32(sB + s * kStageB);
#pragma unroll
        for (int j = 0; j < kGBK / 16; ++j)
          mma_bf16(tmem, desc_sw128(a0 + j * 32), desc_sw128(b0 + j * 32), idesc, (k > 0 || j > 0) ? 1u : 0u);
      }
      mma_commit(mma_done + s);
      if (!ok) *abort_s = 1;
    }
  }
  ok = mbar_wait(mma_done + ((nk - 1) & 1), ((nk - 1) >> 1) & 1, a.status) && ok;
  if (nk >= 2) ok = mbar_wait(mma_done + ((nk - 2) & 1), ((nk - 2) >> 1) & 1, a.status) && ok;
  tc_fence_after();
  __syncthreads();
  if (!ok) *abort_s = 1;
  __syncthreads();
  if (*abort_s == 0) {
    const int q4 = wid & 3, grp = wid >> 2;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    float* T = tr + wid * (32 * 33);
    for (int ch = grp; ch * 32 < NT; ch += 2) {
      float v[32];
      tmem_ld32(trow + ch * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) T[lane * 33 + i] = v[i];
      __syncwarp();
      const int col = n0 + ch * 32 + lane;
      for (int rr = 0; rr < 32; ++rr) {
        const int row = q4 * 32 + rr;
        const int64_t g = m0 + row;
        if (g >= M) break;
        const float o = round_bf16(T[rr * 33 + lane]);
        const float add = round_bf16(__fmul_rn(s_sigma[row], o));
        a.out[g * d + col] = __fadd_rn(a.h[g * d + col], add);
      }
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, NT < 32 ? 32 : NT);
  }
}

template <int NT>
static size_t gate_tc_smem() {
  const size_t stages = 2 * (size_t)kGStageA + 2 * (size_t)NT * 128;
  const size_t tr = 8 * 32 * 33 * 4;
  return 1024 + (stages > tr ? stages : tr) + 64 + 2 * kGTM * 4;
}

int gate_tc_tile(int d) {
  if (d % 256 == 0) return 256;
  if (d % 128 == 0) return 128;
  if (d % 64 == 0) return 64;
  return 0;
}

template <int NT>
static int launch_gate_tc_t(const GateArgs& a, const CUtensorMap& map, cudaStream_t s) {
  const size_t smem = gate_tc_smem<NT>();
  cudaFuncSetAttribute(k_gate_tc<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t M = a.B * a.L;
  dim3 grid((unsigned)(a.d / NT), (unsigned)((M + kGTM - 1) / kGTM));
  k_gate_tc<NT><<<grid, kGThreads, smem, s>>>(map, a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_gate_tc(const GateArgs& a, const CUtensorMap& map, int nt, cudaStream_t s) {
  switch (nt) {
    case 256: return launch_gate_tc_t<256>(a, map, s);
    case 128: return launch_gate_tc_t<128>(a, map, s);
    case 64: return launch_gate_tc_t<64>(a, map, s);
    default: return ASRN_ERR_UNSUPPORTED;
  }
}

int launch_gate(const GateArgs& a, bool half, cudaStream_t s) {
  const int64_t M = a.B * a.L;
  if (M == 0) return ASRN_OK;
  const int nt = gate_tc_tile(a.d);
  if (half && tensor_cores_enabled() && nt > 0) {
    CUtensorMap map;
    if (!make_tmap_bf16(&map, a.wov, (uint64_t)a.d, (uint64_t)a.d, (uint64_t)a.d * 2, 64, (uint32_t)nt))
      return ASRN_ERR_CUDA;
    return launch_gate_tc(a, map, nt, s);
  }
  dim3 grid((unsigned)((a.d + kGateTN - 1) / kGateTN), (unsigned)((M + kGateTM - 1) / kGateTM));
  if (half)
    k_gate_simt<true><<<grid, 256, 0, s>>>(a);
  else
    k_gate_simt<false><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
