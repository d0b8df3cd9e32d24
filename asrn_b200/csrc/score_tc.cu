// Candidate scoring on tensor cores (bf16 autocast mode). Same computation as k_score_simt (asrn/estable.py:204-300,
// asrn/nucleo.py:279-382), organised per sub-tile of 32 sorted query slots:
//   window = the 64 sorted slots [q0 - 32, q0 + 32) of the row (the previous sub-tile + the current one);
//   S = phi_q . phi_k and Qc . Kc (32 x 64 each) on mma.sync (fp32 accumulate), then the reference's rounding chain,
//   suffix weight, log_alfa_k and the fp64 time difference, the exact-mask softmax per query, and
//   out (32 x d_part) = att (32 x 64, bf16) . V (64 x d_part) on mma.sync, added into acc with vector L2 reductions.
// A value row Ea[pos + 1] is gathered only for slots some query can use (the next sorted slot is in the same bucket);
// other rows are zero-filled without reading memory.
//
// One block of 16 warps per (row, span of 512 slots), two warp groups working on consecutive sub-tiles at once:
// in iteration i group A (warps 0-7) scores sub-tile i + 1 and takes its softmax, while group B (warps 8-15)
// multiplies sub-tile i's weights by its value rows and reduces them into acc. The weights pass from A to B through
// a double buffer; one block barrier per iteration. Every load is cp.async: the sorted entries of sub-tile i + 3,
// the scalars and feature rows (phi, Qc, Kc) of sub-tile i + 2 into a 4-sub-tile feature ring, the value rows of
// sub-tile i + 1 into a 3-sub-tile value ring; all land while the current iteration computes. The value rows move
// by bulk copies (cp.async.bulk, one per used row) counted on an mbarrier per ring stage, so the largest transfers do
// not occupy the warps' load slots; value rows no query uses are not loaded and keep earlier finite contents (the
// ring is zeroed when the block starts), multiplied by zero weights. The feature rows and the small per-position
// gathers (clock, log_alfa, previous signatures, the sorted entries) are cp.async. d is split over two blocks only
// when d > 768.
#include <cuda.h>

#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

namespace {
constexpr int kQ = 32;           // queries per sub-tile
constexpr int kRF = 128;         // feature ring: 4 sub-tiles (score windows of i and i + 1, prefetch of i + 2)
constexpr int kRV = 96;          // value ring: 3 sub-tiles (window of i, prefetch of i + 1)
constexpr int kSpanTc = 512;     // sorted slots per block
constexpr int kThreadsTc = 512;  // 16 warps: two groups of 8
constexpr int kGroupWarps = 8;
constexpr int kMaxNt = 12;       // n8 value tiles per group-B warp (d_part <= 768)
constexpr int kStage = 3;        // staging buffers of sorted-row entries
constexpr int kStageIds = 40;    // ids staged per sub-tile: its 32 slots and the next 8 (the `used` test reads s + 1)

struct TcSmem {
  int* st_pos;          // [kStage][kQ] orden entries of a staged sub-tile
  uint16_t* st_id;      // [kStage][kStageIds] ids_o entries
  int* pos;             // [kRF]
  int* id;              // [kRF]
  int* used;            // [kRF]
  double* bt;           // [kRF]
  float* la;            // [kRF]
  float* pf;            // [kRF][kMaxSuffix]
  __nv_bfloat16* phi;   // [kRF][Pp]
  __nv_bfloat16* qc;    // [kRF][Cp]
  __nv_bfloat16* kc;    // [kRF][Cp]
  __nv_bfloat16* v;     // [kRV][Dp]
  float* sc;            // [32][65]
  __nv_bfloat16* att;   // [2][32][72]
  int* qhay;            // [2][32]
  float* wsuf;          // [kMaxSuffix + 1] suffix weights w_sufijo
  uint64_t* vbar;       // [3] value-stage mbarriers
  uint64_t* fbar;       // [4] feature-stage mbarriers (one per 32-row stage of the feature ring)
  int Pp, Cp, Dp;        // row pitches (elements)
  int Gp, Gc;            // 4-row group strides of the phi and Qc / Kc rings (elements)
  __device__ __forceinline__ int prow(int fr) const { return (fr >> 2) * Gp + (fr & 3) * Pp; }
  __device__ __forceinline__ int crow(int fr) const { return (fr >> 2) * Gc + (fr & 3) * Cp; }
};

__host__ __device__ inline int pad16(int x) { return (x + 15) / 16 * 16; }
// Feature rings: rows of the padded pitch (an odd number of 16-byte chunks: the 4 rows of a group fall in distinct
// bank groups) in groups of 4 rows -- one row gather -- each group starting on a 128-byte boundary.
__host__ __device__ inline int group_elems(int pitch) { return (4 * pitch * 2 + 127) / 128 * 128 / 2; }

__host__ __device__ inline size_t tc_smem_bytes(int P, int cf, int dpart) {
  const int Pp = pad16(P) + 8, Cp = pad16(cf) + 8, Dp = dpart + 8;
  size_t b = 128;                                // alignment slack of the dynamic shared memory base
  b += (size_t)(kRF / 4) * (group_elems(Pp) + 2 * group_elems(Cp)) * 2;
  b += kStage * kQ * 4 + kStage * kStageIds * 2;
  b = (b + 15) / 16 * 16;
  b += kRF * 8;                                  // bt
  b += kRF * 4 * (size_t)kMaxSuffix;             // pf
  b += kRF * 4 * 4;                              // pos, id, used, la
  b += (size_t)kRV * Dp * 2;
  b += (size_t)kQ * 65 * 4;
  b += 2 * (size_t)kQ * 72 * 2;
  b += 2 * kQ * 4;
  b += (kMaxSuffix + 8) * 4;
  b = (b + 15) / 16 * 16;
  b += 8 * 8;                                    // mbarriers
  return b + 16;
}

__device__ inline TcSmem carve_tc(char* base, int P, int cf, int dpart) {
  TcSmem s;
  s.Pp = pad16(P) + 8;
  s.Cp = pad16(cf) + 8;
  s.Dp = dpart + 8;
  s.Gp = group_elems(s.Pp);
  s.Gc = group_elems(s.Cp);
  base += (128 - (__cvta_generic_to_shared(base) & 127)) & 127;
  char* p = base;
  s.phi = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)(kRF / 4) * s.Gp * 2;
  s.qc = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)(kRF / 4) * s.Gc * 2;
  s.kc = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)(kRF / 4) * s.Gc * 2;
  s.st_pos = reinterpret_cast<int*>(p); p += kStage * kQ * 4;
  s.st_id = reinterpret_cast<uint16_t*>(p); p += kStage * kStageIds * 2;
  p = base + ((p - base) + 15) / 16 * 16;
  s.bt = reinterpret_cast<double*>(p); p += kRF * 8;
  s.pf = reinterpret_cast<float*>(p); p += kRF * 4 * kMaxSuffix;
  s.pos = reinterpret_cast<int*>(p); p += kRF * 4;
  s.id = reinterpret_cast<int*>(p); p += kRF * 4;
  s.used = reinterpret_cast<int*>(p); p += kRF * 4;
  s.la = reinterpret_cast<float*>(p); p += kRF * 4;
  s.v = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kRV * s.Dp * 2;
  s.sc = reinterpret_cast<float*>(p); p += kQ * 65 * 4;
  s.att = reinterpret_cast<__nv_bfloat16*>(p); p += 2 * kQ * 72 * 2;
  s.qhay = reinterpret_cast<int*>(p); p += 2 * kQ * 4;
  s.wsuf = reinterpret_cast<float*>(p); p += (kMaxSuffix + 8) * 4;
  p = base + ((p - base) + 15) / 16 * 16;
  s.vbar = reinterpret_cast<uint64_t*>(p);
  s.fbar = s.vbar + 3;
  return s;
}

// Ring rows by the slot's index in the block's window space: li = slot - (S0 - 32) >= 0.
__device__ __forceinline__ int frow(int li) { return li & (kRF - 1); }
__device__ __forceinline__ int vrow(int li) { return li % kRV; }

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Bulk copy of `bytes` (a multiple of 16, 16-byte aligned ends) from global to shared memory, counted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(su32(dst)), "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}
// Four rows (row coordinates y0..y3, column 0) of a 2-D tensor map into consecutive rows at dst (the map's box is one
// row of the ring's padded pitch), counted on `bar`; rows outside the tensor read zeros.
__device__ __forceinline__ void gather4_rows(void* dst, const CUtensorMap* map, int y0, int y1, int y2, int y3,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5, %6}], [%7];" ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y0), "r"(y1), "r"(y2),
      "r"(y3), "r"(su32(bar))
      : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bar_group_a() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Block context shared by the phases.
struct TcBlock {
  int64_t r, b, S0, S1;
  int tau, dp0, dpart, Ppad, Cpad;
  float tasa;
  float inv_temp;       // 1 / temperature: the scores' division becomes a product (within an fp32 ulp)
  bool write_signals;
};
}  // namespace

// Sorted entries of sub-tile t (slots [S0 + 32 t, + 32 / 40)) into staging buffer (t + 1) % kStage by 16-byte
// cp.async (zero-filled outside [0, L); rows are 16-byte aligned: L % 8 == 0). Threads 0-7 copy orden, 8-12 ids.
__device__ __forceinline__ void tc_stage1(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t) {
  const int tid = threadIdx.x;
  const int buf = (t + 1) % kStage;
  const int64_t s0 = k.S0 + (int64_t)t * kQ;
  if (tid < kQ / 4) {
    const int64_t s = s0 + 4 * tid;
    const bool ok = s >= 0 && s < a.L;
    cp_async16(S.st_pos + buf * kQ + 4 * tid, a.orden + k.r * a.L + (ok ? s : 0), ok);
  } else if (tid < kQ / 4 + kStageIds / 8) {
    const int c = tid - kQ / 4;
    const int64_t s = s0 + 8 * c;
    const bool ok = s >= 0 && s < a.L;
    cp_async16(S.st_id + buf * kStageIds + 8 * c, a.ids_o + k.r * a.L + (ok ? s : 0), ok);
  }
}

// Scalars and feature rows of sub-tile t, spread over the 16 warps. Warp w takes slots 2w and 2w + 1 (lanes 0 and 1):
// it derives (position, id, used) from the staging buffer, writes them to the feature ring and copies the slot's
// clock (8 B), log_alfa (4 B) and its kMaxSuffix previous signatures (4 B; NaN, never equal, before the text and past
// K) by cp.async. The phi, Qc and Kc rows move as tensor-map row gathers of four slots each: lane 0 of warps 0-7
// issues the three gathers of slots 4w .. 4w + 3, counted on the stage's mbarrier (its byte count is set by thread 0
// beforehand, expect_features); a slot outside the row reads zero rows (row coordinate -1), and the ring's padding
// columns beyond P / cf are zero-filled by the same copies.
__device__ __forceinline__ void tc_stage2_features(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t,
                                                   const CUtensorMap* tm_phi, const CUtensorMap* tm_qc,
                                                   const CUtensorMap* tm_kc) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int buf = (t + 1) % kStage;
  const int64_t s0 = k.S0 + (int64_t)t * kQ;
  if (lane < 2) {
    const int i = 2 * wid + lane;
    const int64_t s = s0 + i;
    const int fr = frow((t + 1) * kQ + i);
    const bool real = s >= 0 && s < a.L;
    const int pos = real ? S.st_pos[buf * kQ + i] : 0;
    const int id = real ? (int)S.st_id[buf * kStageIds + i] : -1;
    const bool used = real && s + 1 < a.L && (int)S.st_id[buf * kStageIds + i + 1] == id && pos + 1 < a.Lf;
    S.pos[fr] = pos;
    S.id[fr] = id;
    S.used[fr] = used ? 1 : 0;
    const int64_t g = k.b * a.Lf + pos;
    if (real) {
      cp_async8(S.bt + fr, a.Bt + g);
      cp_async4(S.la + fr, a.log_alfa + g);
    } else {
      S.bt[fr] = 0.0;
      S.la[fr] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < kMaxSuffix; ++c) {
      const int64_t tt = (int64_t)pos - 1 - c;
      if (real && c < a.K && tt >= 0) cp_async4(S.pf + fr * kMaxSuffix + c, a.sig + k.b * a.Lf + tt);
      else S.pf[fr * kMaxSuffix + c] = __int_as_float(0x7fc00000);
    }
  } else if (lane == 2 && wid < kQ / 4) {
    int y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * wid + j;
      const int64_t s = s0 + i;
      y[j] = (s >= 0 && s < a.L) ? (int)(k.b * a.Lf + S.st_pos[buf * kQ + i]) : -1;
    }
    uint64_t* bar = S.fbar + ((t + 1) & 3);
    const int fr0 = frow((t + 1) * kQ + 4 * wid);
    gather4_rows(S.phi + S.prow(fr0), tm_phi, y[0], y[1], y[2], y[3], bar);
    gather4_rows(S.qc + S.crow(fr0), tm_qc, y[0], y[1], y[2], y[3], bar);
    gather4_rows(S.kc + S.crow(fr0), tm_kc, y[0], y[1], y[2], y[3], bar);
  }
}

// Value rows Ea[pos + 1] of sub-tile t (its scalars already in the feature ring): one bulk copy per used row onto
// the stage's mbarrier, issued by lane 0 of warp slot % 16 (spread over the warps). Thread 0 first sets the stage's
// transaction count from the used flags (arrive.expect_tx); the copies follow a block barrier.
__device__ __forceinline__ int tc_value_bytes(const TcSmem& S, const TcBlock& k, int t) {
  int n = 0;
  for (int i = 0; i < kQ; ++i) n += S.used[frow((t + 1) * kQ + i)];
  return n * k.dpart * 2;
}
__device__ __forceinline__ void tc_stage2_values(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane != 0) return;
  uint64_t* bar = S.vbar + ((t + 1) % 3);
  const uint32_t bytes = (uint32_t)k.dpart * 2;
  for (int i = wid; i < kQ; i += nw) {
    const int li = (t + 1) * kQ + i;
    const int fr = frow(li), vr = vrow(li);
    if (S.used[fr]) {
      const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.Ea) + (k.b * a.Lf + S.pos[fr] + 1) *
                                 (int64_t)a.d + k.dp0;
      bulk_load(S.v + vr * S.Dp, src, bytes, bar);
    }
  }
}

// Group A: scores of sub-tile t (queries: window slots 32 .. 63; keys: 0 .. 63, slot q0 - 32 + key), the exact-mask
// softmax, the weights into att[t & 1] and the per-table gate signals. Warp w (0-7) owns n-tile w (keys 8w .. 8w + 7)
// of both m-tiles: the two MMA chains run interleaved on the same key fragments, then one epilogue pass over the
// warp's 8 elements per lane; the softmax takes the warp's 4 queries in one set of shuffle rounds.
template <bool kSuf4>
__device__ __forceinline__ void tc_scores(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int C = a.C;
  const int64_t q0 = k.S0 + (int64_t)t * kQ;
  const int lb = t * kQ;                        // window index of key 0 (li of slot q0 - 32)
  const int nt = wid;
  // band: keys [8 nt, 8 nt + 8) meet queries [16 mt, 16 mt + 16) only if some key is within C before one of them
  bool band[2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) band[mt] = nt * 8 + 7 >= mt * 16 + 32 - C && nt * 8 < mt * 16 + 16 + 32;
  float cphi[2][4] = {}, cqk[2][4] = {};
  if (band[0] || band[1]) {
    const int ka = (lane >> 4) * 8;
    const int rk = frow(lb + nt * 8 + (lane & 7));
    const int kb = ((lane >> 3) & 1) * 8;
    const int ra0 = frow(lb + kQ + (lane & 15)), ra1 = frow(lb + kQ + 16 + (lane & 15));
    const uint32_t phi_b = su32(S.phi) + 2u * (uint32_t)(S.prow(rk) + kb);
    const uint32_t kc_b = su32(S.kc) + 2u * (uint32_t)(S.crow(rk) + kb);
    const uint32_t phi_a0 = su32(S.phi) + 2u * (uint32_t)(S.prow(ra0) + ka);
    const uint32_t phi_a1 = su32(S.phi) + 2u * (uint32_t)(S.prow(ra1) + ka);
    const uint32_t qc_a0 = su32(S.qc) + 2u * (uint32_t)(S.crow(ra0) + ka);
    const uint32_t qc_a1 = su32(S.qc) + 2u * (uint32_t)(S.crow(ra1) + ka);
    for (int k0 = 0; k0 < k.Ppad; k0 += 16) {
      uint32_t b0, b1;
      ldsm_x2(phi_b + 2 * k0, b0, b1);
      if (band[0]) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(phi_a0 + 2 * k0, a0, a1, a2, a3);
        mma16816(cphi[0], a0, a1, a2, a3, b0, b1);
      }
      if (band[1]) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(phi_a1 + 2 * k0, a0, a1, a2, a3);
        mma16816(cphi[1], a0, a1, a2, a3, b0, b1);
      }
    }
    for (int k0 = 0; k0 < k.Cpad; k0 += 16) {
      uint32_t b0, b1;
      ldsm_x2(kc_b + 2 * k0, b0, b1);
      if (band[0]) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(qc_a0 + 2 * k0, a0, a1, a2, a3);
        mma16816(cqk[0], a0, a1, a2, a3, b0, b1);
      }
      if (band[1]) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(qc_a1 + 2 * k0, a0, a1, a2, a3);
        mma16816(cqk[1], a0, a1, a2, a3, b0, b1);
      }
    }
  }
  // this lane's four query rows (g, g + 8, 16 + g, 24 + g; g = lane / 4) and two key columns (kj0, kj0 + 1): their
  // ring-row scalars are read once; the suffix length is the count of leading equal previous signatures
  const int g4 = lane >> 2, kj0 = nt * 8 + (lane & 3) * 2;
  int q_id[4], k_id[2];
  float4 q_pf[4][2], k_pf[2][2];
  double q_bt[4], k_bt[2];
  float k_la[2];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int rq = frow(lb + kQ + g4 + 8 * u);
    q_id[u] = S.id[rq];
    q_pf[u][0] = *reinterpret_cast<const float4*>(S.pf + rq * kMaxSuffix);
    q_pf[u][1] = *reinterpret_cast<const float4*>(S.pf + rq * kMaxSuffix + 4);
    q_bt[u] = S.bt[rq];
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int rk = frow(lb + kj0 + u);
    k_id[u] = S.id[rk];
    k_pf[u][0] = *reinterpret_cast<const float4*>(S.pf + rk * kMaxSuffix);
    k_pf[u][1] = *reinterpret_cast<const float4*>(S.pf + rk * kMaxSuffix + 4);
    k_bt[u] = S.bt[rk];
    k_la[u] = S.la[rk];
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int uq = 2 * mt + (e >> 1), uk = e & 1;
      const int qi = g4 + 8 * uq;
      const int kj = kj0 + uk;
      const int64_t sq = q0 + qi, sk = q0 - kQ + kj;
      // every element is computed (no divergent branch) and masked at the end: outside the band, the row or the
      // bucket it is -inf
      const bool ok = band[mt] && kj < qi + 32 && kj >= qi + 32 - C && sq < a.L && sk >= 0 && k_id[uk] == q_id[uq];
      const float s1 = round_bf16(__fmul_rn(round_bf16(cphi[mt][e]), k.inv_temp));
      const float s2 = round_bf16(__fmul_rn(round_bf16(cqk[mt][e]), a.esc_c));
      float t1 = round_bf16(__fadd_rn(s1, s2));
      const float4 qa = q_pf[uq][0], ka = k_pf[uk][0];
      uint32_t eq = (qa.x == ka.x ? 1u : 0u) | (qa.y == ka.y ? 2u : 0u) | (qa.z == ka.z ? 4u : 0u) |
                    (qa.w == ka.w ? 8u : 0u);
      if (!kSuf4) {                             // entries 4 .. 7 are NaN (never equal) when K <= 4
        const float4 qb = q_pf[uq][1], kb = k_pf[uk][1];
        eq |= (qb.x == kb.x ? 16u : 0u) | (qb.y == kb.y ? 32u : 0u) | (qb.z == kb.z ? 64u : 0u) |
              (qb.w == kb.w ? 128u : 0u);
      }
      const int ln = __ffs(~eq) - 1;            // leading equal entries (entries past K are NaN: never equal)
      t1 = __fadd_rn(t1, S.wsuf[ln]);
      t1 = __fadd_rn(t1, k_la[uk]);
      const float dt = __double2float_rn(k_bt[uk] - q_bt[uq]);
      const float val = ok ? __fadd_rn(t1, __fmul_rn(dt, k.tasa)) : -INFINITY;
      S.sc[qi * 65 + kj] = val;
    }
  }
  bar_group_a();
  // softmax: warp w -> queries 4w .. 4w + 3 together; lane -> keys lane, lane + 32
  __nv_bfloat16* att = S.att + (t & 1) * kQ * 72;
  int* qhay = S.qhay + (t & 1) * kQ;
  const int qa = wid * 4;
  float x[4][2], m[4], sum[4], e[4][2];
  unsigned bal[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    x[u][0] = S.sc[(qa + u) * 65 + lane];
    x[u][1] = S.sc[(qa + u) * 65 + lane + 32];
    bal[u] = __ballot_sync(0xffffffffu, x[u][0] != -INFINITY || x[u][1] != -INFINITY);
    m[u] = fmaxf(x[u][0], x[u][1]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < 4; ++u) m[u] = fmaxf(m[u], __shfl_xor_sync(0xffffffffu, m[u], o));
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    e[u][0] = x[u][0] != -INFINITY ? __expf(__fsub_rn(x[u][0], m[u])) : 0.f;
    e[u][1] = x[u][1] != -INFINITY ? __expf(__fsub_rn(x[u][1], m[u])) : 0.f;
    sum[u] = e[u][0] + e[u][1];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < 4; ++u) sum[u] += __shfl_xor_sync(0xffffffffu, sum[u], o);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int qi = qa + u;
    const int64_t sq = q0 + qi;
    const bool anyv = bal[u] != 0;
    const int posq = S.pos[frow(lb + kQ + qi)];
    const bool mine = sq < k.S1 && posq >= a.q_lo && posq < a.q_hi;   // else a key only (another shard's position)
    const int64_t gq = k.b * (a.q_hi - a.q_lo) + (posq - a.q_lo);
    float w0 = 0.f, w1 = 0.f;
    if (anyv) {
      const float rs = __frcp_rn(sum[u]);
      w0 = __fmul_rn(e[u][0], rs);
      w1 = __fmul_rn(e[u][1], rs);
      // the largest weight is the maximum's: exp(0) / sum
      if (lane == 0 && k.write_signals && mine) {
        a.sen_hay[gq * a.T + k.tau] = 1;
        a.sen_mx[gq * a.T + k.tau] = m[u];
        a.sen_pk[gq * a.T + k.tau] = rs;
      }
    } else if (lane == 0 && k.write_signals && mine) {
      a.sen_hay[gq * a.T + k.tau] = 0;
      a.sen_mx[gq * a.T + k.tau] = kProhibido;
      a.sen_pk[gq * a.T + k.tau] = 0.f;
    }
    att[qi * 72 + lane] = __float2bfloat16_rn(w0);
    att[qi * 72 + lane + 32] = __float2bfloat16_rn(w1);
    if (lane == 0) qhay[qi] = (anyv && mine) ? 1 : 0;
  }
}

// Group B: out = att[t & 1] . V for sub-tile t on tensor cores, reduced into acc. Warp w (0-7 within the group) owns
// the n8 tiles w, w + 8, ... of the d_part columns.
__device__ __forceinline__ void tc_values(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t, int w) {
  const int lane = threadIdx.x & 31;
  const int lb = t * kQ;                        // window index of key 0 (li of slot q0 - 32)
  const __nv_bfloat16* att = S.att + (t & 1) * kQ * 72;
  const int* qhay = S.qhay + (t & 1) * kQ;
  const int ntiles = k.dpart / 8;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const int qbase = mt * 16;
    const bool any = qhay[qbase + (lane & 15)] != 0;
    if (!__any_sync(0xffffffffu, any)) continue;
    float acc[kMaxNt][4];
#pragma unroll
    for (int j = 0; j < kMaxNt; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    // queries of m-tile mt use window keys [qbase, qbase + 47]
    const uint32_t att_a = su32(att) + 2u * (uint32_t)((qbase + (lane & 15)) * 72 + (lane >> 4) * 8);
    for (int ks = mt; ks < mt + 3; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(att_a + 2u * (uint32_t)(ks * 16), a0, a1, a2, a3);
      const uint32_t v_row = su32(S.v) + 2u * (uint32_t)(vrow(lb + ks * 16 + (lane & 15)) * S.Dp);
#pragma unroll
      for (int j = 0; j < kMaxNt; ++j) {
        const int tile = w + kGroupWarps * j;
        if (tile < ntiles) {
          uint32_t b0, b1;
          ldsm_x2_t(v_row + 2u * (uint32_t)(tile * 8), b0, b1);
          mma16816(acc[j], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    // one 16-byte reduction per lane and tile: lanes q and q ^ 1 of a quad swap halves so that the even lane holds
    // columns 4 (q >> 1) .. + 3 of row r and the odd lane the same columns of row r + 8
    const int qd = lane & 3;
    const int rowq = qbase + (lane >> 2) + ((qd & 1) ? 8 : 0);
    const bool hasq = qhay[rowq] != 0;
    const int64_t gq = k.b * (a.q_hi - a.q_lo) + (S.pos[frow(lb + kQ + rowq)] - a.q_lo);
    float* dst = a.acc + gq * a.d + k.dp0 + (qd >> 1) * 4;
#pragma unroll
    for (int j = 0; j < kMaxNt; ++j) {
      const int tile = w + kGroupWarps * j;
      if (tile < ntiles) {
        const bool odd = qd & 1;
        const float s0 = odd ? acc[j][0] : acc[j][2], s1 = odd ? acc[j][1] : acc[j][3];
        const float r0 = __shfl_xor_sync(0xffffffffu, s0, 1), r1 = __shfl_xor_sync(0xffffffffu, s1, 1);
        const float v0 = odd ? r0 : acc[j][0], v1 = odd ? r1 : acc[j][1];
        const float v2 = odd ? acc[j][2] : r0, v3 = odd ? acc[j][3] : r1;
        if (hasq) red_add_v4(dst + tile * 8, v0, v1, v2, v3);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreadsTc, 1)
k_score_tc(const __grid_constant__ CUtensorMap tm_phi, const __grid_constant__ CUtensorMap tm_qc,
           const __grid_constant__ CUtensorMap tm_kc, ScoreArgs a, int nds, int dpart) {
  extern __shared__ __align__(16) char smem_raw[];
  const TcSmem S = carve_tc(smem_raw, a.P, a.cf, dpart);
  TcBlock k;
  k.r = blockIdx.y;
  k.b = k.r / a.T;
  k.tau = (int)(k.r % a.T);
  const int part = blockIdx.x % nds;
  k.S0 = (int64_t)(blockIdx.x / nds) * kSpanTc;
  k.S1 = min(min(k.S0 + kSpanTc, a.L), a.row_len ? a.row_len[k.r] : a.L);
  if (k.S0 >= k.S1) return;                     // a span past the row's used slots (sharded rows)
  k.dp0 = part * dpart;
  k.dpart = dpart;
  k.Ppad = pad16(a.P);
  k.Cpad = pad16(a.cf);
  k.tasa = a.tasa[k.tau];
  k.inv_temp = 1.f / a.inv_temp_div;
  k.write_signals = part == 0;
  const int wid = threadIdx.x >> 5;
  const bool group_a = wid < kGroupWarps;
  const int ntile = (int)((k.S1 - k.S0 + kQ - 1) / kQ);

  // zero both rings once (rows never loaded keep finite contents), set up the stage barriers
  {
    uint4* z0 = reinterpret_cast<uint4*>(S.phi);
    const int nz = (int)(((char*)(S.v + kRV * S.Dp) - (char*)S.phi) / 16);
    for (int i = threadIdx.x; i < nz; i += blockDim.x) z0[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x <= kMaxSuffix) S.wsuf[threadIdx.x] = threadIdx.x <= a.K ? a.w_suf[threadIdx.x] : 0.f;
    umma::fence_proxy_async();                 // the zeros precede the bulk copies into the same rows
    if (threadIdx.x == 0) {
      for (int i = 0; i < 7; ++i) umma::mbar_init(S.vbar + i, 1);   // 3 value stages, then 4 feature stages
      umma::fence_mbar_init();
    }
  }
  // bounded wait for the value bulk copies of a stage, by every thread (each observes the completed phase)
  auto wait_values = [&](int t) {
    umma::mbar_wait(S.vbar + ((t + 1) % 3), (uint32_t)(((t + 1) / 3) & 1), a.status);
  };
  // bounded wait for the feature rows of sub-tile t (stage (t + 1) % 4)
  auto wait_features = [&](int t) {
    umma::mbar_wait(S.fbar + ((t + 1) & 3), (uint32_t)(((t + 1) >> 2) & 1), a.status);
  };
  // the stages' transaction counts (the used value rows; the fixed feature rows) are set by thread 0 before any copy
  // of the stage is issued
  auto expect_values = [&](int t) {
    if (threadIdx.x == 0) umma::mbar_expect_tx(S.vbar + ((t + 1) % 3), (uint32_t)tc_value_bytes(S, k, t));
  };
  auto expect_features = [&](int t) {
    if (threadIdx.x == 0) umma::mbar_expect_tx(S.fbar + ((t + 1) & 3), (uint32_t)(kQ * (S.Pp + 2 * S.Cp) * 2));
  };

  // prologue: sub-tiles -1 (the first window half), 0 and 1 of the features, -1 and 0 of the values, the scores of
  // 0 taken; sub-tile 2's sorted entries on their way
  __syncthreads();
  tc_stage1(a, S, k, -1);
  tc_stage1(a, S, k, 0);
  if (ntile > 1) tc_stage1(a, S, k, 1);
  cp_async_commit();
  cp_async_wait_all();
  expect_features(-1);
  expect_features(0);
  if (ntile > 1) expect_features(1);
  __syncthreads();
  tc_stage2_features(a, S, k, -1, &tm_phi, &tm_qc, &tm_kc);
  tc_stage2_features(a, S, k, 0, &tm_phi, &tm_qc, &tm_kc);
  if (ntile > 1) tc_stage2_features(a, S, k, 1, &tm_phi, &tm_qc, &tm_kc);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  expect_values(-1);
  expect_values(0);
  if (ntile > 2) tc_stage1(a, S, k, 2);        // its buffer was read by sub-tile -1's feature stage above
  cp_async_commit();
  __syncthreads();
  tc_stage2_values(a, S, k, -1);
  tc_stage2_values(a, S, k, 0);
  wait_features(-1);
  wait_features(0);
  const bool suf4 = a.K <= 4;
  if (group_a) {
    if (suf4) tc_scores<true>(a, S, k, 0);
    else tc_scores<false>(a, S, k, 0);
  }
  cp_async_wait_all();
  wait_values(-1);
  wait_values(0);
  if (ntile > 1) wait_features(1);
  __syncthreads();

  for (int i = 0; i < ntile; ++i) {
    // value rows of i + 1 (their scalars arrived with the features in iteration i - 1) and feature rows of i + 2:
    // byte counts first, then the copies, issued by all warps
    if (i + 1 < ntile) expect_values(i + 1);
    if (i + 2 < ntile) expect_features(i + 2);
    if (i + 3 < ntile) tc_stage1(a, S, k, i + 3);
    if (i + 1 < ntile) {
      asm volatile("bar.sync 2, 512;" ::: "memory");   // the expect_tx precedes every copy of the stages
      if (i + 2 < ntile) tc_stage2_features(a, S, k, i + 2, &tm_phi, &tm_qc, &tm_kc);
      tc_stage2_values(a, S, k, i + 1);
    }
    cp_async_commit();
    if (group_a) {
      if (i + 1 < ntile) {
        if (suf4) tc_scores<true>(a, S, k, i + 1);
        else tc_scores<false>(a, S, k, i + 1);
      }
    } else {
      tc_values(a, S, k, i, wid - kGroupWarps);
    }
    cp_async_wait_all();
    if (i + 1 < ntile) wait_values(i + 1);
    if (i + 2 < ntile) wait_features(i + 2);
    __syncthreads();
  }
}

bool score_tc_supported(const ScoreArgs& a) {
  return a.d % 64 == 0 && a.d <= 1024 && a.C <= 32 && a.P <= kMaxPhi && a.P % 8 == 0 && pad16(a.P) + 8 <= 256 &&
         a.cf <= kMaxConfirm && a.cf % 8 == 0 && a.K <= kMaxSuffix && a.L % 8 == 0 && a.B * a.Lf < ((int64_t)1 << 31);
}

int launch_score_tc(const ScoreArgs& a, cudaStream_t s) {
  // the whole width in one block when its 96-row value ring fits next to the features (d <= 768), else halves
  int nds = (a.d + 767) / 768;
  while (a.d % (nds * 64) != 0) ++nds;
  const int dpart = a.d / nds;
  if (dpart / 8 > kGroupWarps * kMaxNt) return ASRN_ERR_UNSUPPORTED;
  const size_t smem = tc_smem_bytes(a.P, a.cf, dpart);
  if (smem > 227 * 1024) return ASRN_ERR_UNSUPPORTED;
  // feature rows as one-row boxes of the ring's padded pitch (the padding columns lie outside the tensor: zeros)
  CUtensorMap tm_phi, tm_qc, tm_kc;
  const uint64_t rows = (uint64_t)(a.B * a.Lf);
  if (!make_tmap_rows_bf16(&tm_phi, a.phi, (uint64_t)a.P, rows, (uint64_t)a.P * 2, (uint32_t)(pad16(a.P) + 8)) ||
      !make_tmap_rows_bf16(&tm_qc, a.Qc, (uint64_t)a.cf, rows, (uint64_t)a.cf * 2, (uint32_t)(pad16(a.cf) + 8)) ||
      !make_tmap_rows_bf16(&tm_kc, a.Kc, (uint64_t)a.cf, rows, (uint64_t)a.cf * 2, (uint32_t)(pad16(a.cf) + 8)))
    return ASRN_ERR_CUDA;
  cudaFuncSetAttribute(k_score_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)(((a.L + kSpanTc - 1) / kSpanTc) * nds), (unsigned)(a.B * a.T));
  k_score_tc<<<grid, kThreadsTc, smem, s>>>(tm_phi, tm_qc, tm_kc, a, nds, dpart);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
