// Candidate scoring on tensor cores (bf16 autocast mode). Same computation as k_score_simt (asrn/estable.py:204-300,
// asrn/nucleo.py:279-382), organised per sub-tile of 32 sorted query slots:
//   window = the 64 sorted slots [q0 - 32, q0 + 32) of the row (the previous sub-tile + the current one);
//   S = phi_q . phi_k and Qc . Kc on tcgen05 (fp32 accumulators in TMEM), then the reference's rounding chain,
//   suffix weight, log_alfa_k and the fp64 time difference, the exact-mask softmax per query, and
//   out^T (d_part x 32) = V^T (d_part x 64) . att^T (64 x 32) on tcgen05 (M = 128 rows of d per MMA, N = the 32
//   queries, K = the 64 window keys; the accumulators in TMEM), added into the bf16 accumulator acc by bf16 reductions
//   in L2.
// A value row Ea[pos + 1] is gathered only for slots some query can use (the next sorted slot is in the same bucket);
// other rows keep finite contents (zeros) and meet zero weights.
//
// One block of 20 warps per (row, span of 512-2048 slots), three warp groups working on consecutive sub-tiles at once:
// in iteration i group A (warps 0-7) scores sub-tile i + 1 (its S products were issued to the tensor cores an
// iteration earlier; the element epilogue by the four warps whose TMEM lanes hold the window's keys) and takes its
// softmax, while the load group's first thread issues the S products of i + 2; group B (warps 8-15) has the value products
// of sub-tile i computed by the tensor cores (lane 0 of warp m issues M-tile m) and reduces them into acc, and the
// load group (warps 16-19) issues the copies: the sorted entries of sub-tile i + 4 and the per-position scalars of
// i + 3 by cp.async, the phi / Qc / Kc rows of i + 3 by tensor-map row gathers (four rows per instruction) into a
// 4-sub-tile feature ring, the used value rows of i + 1 by 16-byte cp.async into a 3-sub-tile value ring kept
// in the MMA's MN-major 128-byte-swizzled layout (one 12 KB region per 64 columns of d). The weights pass from A to B
// through a double buffer in the MMA's K-major swizzled layout; one block barrier per iteration.
// The value epilogue stages each warp's 32 rows of d x 16 queries in shared memory and reads them back transposed, so
// that each lane adds 8 consecutive values of one query row with one 16-byte bf16 reduction (no lane shuffles). The
// table sum thus moves 2 bytes per value into L2 instead of 4: L2 sustains about 6 TB/s of reductions on B200, so the
// fp32 sum of 8 tables x d values per token would bound the kernel at about 1.1 ms for 32 x 8192 tokens at d = 768.
// d is split over blocks only when d > 768 (d_part a multiple of 128).
#include <cuda.h>

#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

namespace {
constexpr int kQ = 32;           // queries per sub-tile
constexpr int kRF = 128;         // feature ring: 4 sub-tiles (iteration i: i, i + 1 scored, i + 2 in the MMAs, i + 3 loaded)
constexpr int kRV = 96;          // value ring: 3 sub-tiles (window of i, prefetch of i + 1)
constexpr int kSpanTc = 512;     // sorted slots per block: the shortest span (longer ones when the grid stays large)
constexpr int kGroupWarps = 8;   // warps 0-7: scores (group A); 8-15: value products (group B)
constexpr int kLoadWarps = 4;    // warps 16-19: every copy into shared memory (the load group)
constexpr int kLoadThreads = kLoadWarps * 32;
constexpr int kThreadsTc = (2 * kGroupWarps + kLoadWarps) * 32;
constexpr int kMaxMt = 6;        // M = 128 tiles of d_part (d_part <= 768)
constexpr int kVRegion = kRV * 128;   // one 64-column region of the value ring (bytes)
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
  uint8_t* phi;         // [nbp][kRF rows][128 B]: column blocks of 64 features, 128-byte swizzle
  uint8_t* qc;          // [kRF rows][64 B], 64-byte swizzle
  uint8_t* kc;          // [kRF rows][64 B]
  uint8_t* v;           // [d_part / 64][kRV rows][128 B], MN-major 128-byte swizzle (1024-byte aligned)
  float* sc;            // [32][64], key column kj of query qi at kj ^ sc_swz(qi)
  uint8_t* att;         // [2][32 rows][128 B], K-major 128-byte swizzle (1024-byte aligned)
  int64_t* qoff;        // [2][32] acc element offset of the query's row, or -1 (no candidate / not this shard's)
  float* wsuf;          // [kMaxSuffix + 1] suffix weights w_sufijo
  uint64_t* fbar;       // [4] feature-stage mbarriers (one per 32-row stage of the feature ring)
  uint64_t* pvbar;      // value-product MMAs done
  uint64_t* sbar;       // [2] score MMAs of a sub-tile done (sub-tile t on t & 1)
  uint32_t* tmem;       // TMEM base address
  int nbp;               // phi column blocks
  int Dp;
};

__host__ __device__ inline int pad16(int x) { return (x + 15) / 16 * 16; }
// Feature rings, written by tensor-map row gathers with the map's swizzle so that the 8 rows of an ldmatrix fall in 8
// distinct bank groups (a gather's 4 rows start on a 128-byte boundary): phi in column blocks of 64 features, rows of
// 128 B with the 128-byte swizzle (16-byte chunk c of ring row r at chunk c ^ (r mod 8)); Qc / Kc (cf <= 32) in rows
// of 64 B with the 64-byte swizzle (chunk c of row r at c ^ ((r / 2) mod 4)).
__host__ __device__ inline int ring_blocks(int cols) { return (pad16(cols) * 2 + 127) / 128; }
__host__ __device__ inline int ring_bytes_phi(int P) { return ring_blocks(P) * kRF * 128; }
constexpr int kRingBytesC = kRF * 64;
__host__ __device__ inline int sc_swz(int qi) { return (qi & 1) | (((qi >> 1) & 3) << 3); }

__host__ __device__ inline size_t tc_smem_bytes(int P, int cf, int dpart) {
  size_t b = 1024;                               // alignment slack of the dynamic shared memory base
  b += (size_t)(dpart / 64) * kVRegion + 2 * kQ * 128;
  b += (size_t)ring_bytes_phi(P) + 2 * (size_t)kRingBytesC;
  b += kStage * kQ * 4 + kStage * kStageIds * 2;
  b = (b + 15) / 16 * 16;
  b += kRF * 8;                                  // bt
  b += kRF * 4 * (size_t)kMaxSuffix;             // pf
  b += kRF * 4 * 4;                              // pos, id, used, la
  b += (size_t)kQ * 64 * 4;
  b += 2 * kQ * 8;                               // qoff
  b += (kMaxSuffix + 8) * 4;
  b = (b + 15) / 16 * 16;
  b += 8 * 8 + 16;                               // mbarriers, TMEM address
  return b;
}

__device__ inline TcSmem carve_tc(char* base, int P, int cf, int dpart) {
  TcSmem s;
  s.nbp = ring_blocks(P);
  s.Dp = dpart;
  base += (1024 - (__cvta_generic_to_shared(base) & 1023)) & 1023;
  char* p = base;
  s.v = reinterpret_cast<uint8_t*>(p); p += (size_t)(dpart / 64) * kVRegion;
  s.att = reinterpret_cast<uint8_t*>(p); p += 2 * kQ * 128;
  s.phi = reinterpret_cast<uint8_t*>(p); p += ring_bytes_phi(P);
  s.qc = reinterpret_cast<uint8_t*>(p); p += kRingBytesC;
  s.kc = reinterpret_cast<uint8_t*>(p); p += kRingBytesC;
  s.st_pos = reinterpret_cast<int*>(p); p += kStage * kQ * 4;
  s.st_id = reinterpret_cast<uint16_t*>(p); p += kStage * kStageIds * 2;
  p = base + ((p - base) + 15) / 16 * 16;
  s.bt = reinterpret_cast<double*>(p); p += kRF * 8;
  s.pf = reinterpret_cast<float*>(p); p += kRF * 4 * kMaxSuffix;
  s.pos = reinterpret_cast<int*>(p); p += kRF * 4;
  s.id = reinterpret_cast<int*>(p); p += kRF * 4;
  s.used = reinterpret_cast<int*>(p); p += kRF * 4;
  s.la = reinterpret_cast<float*>(p); p += kRF * 4;
  s.sc = reinterpret_cast<float*>(p); p += kQ * 64 * 4;
  s.qoff = reinterpret_cast<int64_t*>(p); p += 2 * kQ * 8;
  s.wsuf = reinterpret_cast<float*>(p); p += (kMaxSuffix + 8) * 4;
  p = base + ((p - base) + 15) / 16 * 16;
  s.fbar = reinterpret_cast<uint64_t*>(p);
  s.pvbar = s.fbar + 4;
  s.sbar = s.fbar + 5;
  s.tmem = reinterpret_cast<uint32_t*>(s.fbar + 8);
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
// Four rows (row coordinates y0..y3, columns x .. x + box) of a 2-D tensor map into consecutive ring rows at dst
// (the map's box is one ring row), counted on `bar`; rows and columns outside the tensor read zeros.
__device__ __forceinline__ void gather4_rows(void* dst, const CUtensorMap* map, int x, int y0, int y1, int y2, int y3,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5, %6}], [%7];" ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2),
      "r"(y3), "r"(su32(bar))
      : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async16_s(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(su32(dst)), "l"(src) : "memory");
}
// 16-byte reduction into global memory with no compiler memory barrier (nothing in the kernel reads acc back, so
// the surrounding shared-memory loads may move across it).
__device__ __forceinline__ void red_add_v4_nc(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d));
}
// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Round two fp32 values to bf16 (nearest even) in one conversion, back as fp32.
__device__ __forceinline__ void round2_bf16(float& a, float& b) {
  const uint32_t u = pack2_bf16(a, b);           // a in the low half, b in the high half
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xFFFF0000u);
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_but_last() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void bar_group_a() { asm volatile("bar.sync 1, 256;" ::: "memory"); }


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
// cp.async (zero-filled outside [0, L); rows are 16-byte aligned: L % 8 == 0). Load threads 0-7 copy orden, 8-12 ids.
__device__ __forceinline__ void tc_stage1(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t, int tid) {
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

// Scalars and feature rows of sub-tile t, issued by the load group (thread pt of kLoadThreads). Thread pt < 64 takes
// slot pt / 2: even threads copy its kMaxSuffix previous signatures (4 B each by cp.async; NaN, never equal, before the
// text and past K), odd threads its clock (8 B) and log_alfa (4 B) and write (position, id, used) from the staging
// buffer. The phi, Qc and Kc rows move as tensor-map row gathers of four slots each: thread 64 + j, j < 8 (nbp + 2),
// issues gather j / 8 (phi column blocks, then Qc, then Kc) of slots 4 (j % 8) .. + 3, counted on the stage's mbarrier
// (its byte count is set beforehand, expect_features); a slot outside the row reads zero rows (row coordinate -1), and
// the columns past P / cf read zeros.
__device__ __forceinline__ void tc_stage2_features(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t, int pt,
                                                   const CUtensorMap* tm_phi, const CUtensorMap* tm_qc,
                                                   const CUtensorMap* tm_kc) {
  const int buf = (t + 1) % kStage;
  const int64_t s0 = k.S0 + (int64_t)t * kQ;
  if (pt < 2 * kQ) {
    const int i = pt >> 1;
    const int64_t s = s0 + i;
    const int fr = frow((t + 1) * kQ + i);
    const bool real = s >= 0 && s < a.L;
    const int pos = real ? S.st_pos[buf * kQ + i] : 0;
    if ((pt & 1) == 0) {
#pragma unroll
      for (int j = 0; j < kMaxSuffix; ++j) {
        const int64_t tt = (int64_t)pos - 1 - j;
        if (real && j < a.K && tt >= 0) cp_async4(S.pf + fr * kMaxSuffix + j, a.sig + k.b * a.Lf + tt);
        else S.pf[fr * kMaxSuffix + j] = __int_as_float(0x7fc00000);
      }
    } else {
      const int64_t g = k.b * a.Lf + pos;
      if (real) {
        cp_async8(S.bt + fr, a.Bt + g);
        cp_async4(S.la + fr, a.log_alfa + g);
      } else {
        S.bt[fr] = 0.0;
        S.la[fr] = 0.f;
      }
      const int id = real ? (int)S.st_id[buf * kStageIds + i] : -1;
      const bool used = real && s + 1 < a.L && (int)S.st_id[buf * kStageIds + i + 1] == id && pos + 1 < a.Lf;
      S.pos[fr] = pos;
      S.id[fr] = id;
      S.used[fr] = used ? 1 : 0;
    }
  }
  const int gp = pt - 2 * kQ;
  if (gp >= 0 && gp < 8 * (S.nbp + 2)) {
    const int grp = gp & 7, gi = gp >> 3;
    int y[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int iq = 4 * grp + q;
      const int64_t sq = s0 + iq;
      y[q] = (sq >= 0 && sq < a.L) ? (int)(k.b * a.Lf + S.st_pos[buf * kQ + iq]) : -1;
    }
    uint64_t* bar = S.fbar + ((t + 1) & 3);
    const int fr0 = frow((t + 1) * kQ + 4 * grp);
    const int nbp = S.nbp;
    const CUtensorMap* map = gi < nbp ? tm_phi : (gi == nbp ? tm_qc : tm_kc);
    uint8_t* dst = gi < nbp ? S.phi + ((gi * kRF + fr0) << 7) : (gi == nbp ? S.qc : S.kc) + (fr0 << 6);
    gather4_rows(dst, map, gi < nbp ? gi * 64 : 0, y[0], y[1], y[2], y[3], bar);
  }
}

// Value rows Ea[pos + 1] of sub-tile t (its scalars already in the feature ring) into the value ring, only the used
// rows, by the load group (thread pt) one iteration ahead of their MMAs: load warp w takes slots w, w + 4, ..., its
// lanes the row's 16-byte chunks by cp.async, each chunk at its place in the MN-major 128-byte-swizzled layout (region
// = 64 columns, row = key, chunk index XOR the key's row in its group of 8). (As tensor-map row gathers these take 12
// gathers per 4 rows, which makes the tensor-map unit the bottleneck of the loop.)
__device__ __forceinline__ void tc_stage2_values(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t, int pt) {
  const int lane = pt & 31, wb = pt >> 5;
  const int nch = k.dpart / 8;                 // 16-byte chunks per row (<= 96: chunks lane, lane + 32, lane + 64)
  // chunk c = lane + 32 u of a row sits in region c / 8 = lane / 8 + 4 u at chunk (c % 8) ^ (row % 8) = (lane % 8) ^ ...
  const uint32_t v_lane = su32(S.v) + (uint32_t)(lane >> 3) * kVRegion;
  const uint32_t x_lane = (uint32_t)(lane & 7) << 4;
  const bool c0 = lane < nch, c1 = lane + 32 < nch, c2 = lane + 64 < nch;
  // the value of position p is row p + 1 of Ea
  const __nv_bfloat16* ea = reinterpret_cast<const __nv_bfloat16*>(a.Ea) + (k.b * a.Lf + 1) * (int64_t)a.d + k.dp0 +
                            lane * 8;
  // the warp's 8 rows' flags and positions first: read inside the copy loop, each row's shared-memory loads wait
  // behind the previous row's copies (1.7 of a 4 us iteration)
  constexpr int kRows = kQ / kLoadWarps;
  int used[kRows], pos[kRows];
#pragma unroll
  for (int u = 0; u < kRows; ++u) {
    const int fr = frow((t + 1) * kQ + wb + kLoadWarps * u);
    used[u] = S.used[fr];
    pos[u] = S.pos[fr];
  }
#pragma unroll
  for (int u = 0; u < kRows; ++u) {
    if (!used[u]) continue;
    const int vr = vrow((t + 1) * kQ + wb + kLoadWarps * u);
    const __nv_bfloat16* src = ea + (int64_t)pos[u] * a.d;
    const uint32_t x = (uint32_t)(vr & 7);
    const uint32_t dst = v_lane + (uint32_t)(vr >> 3) * 1024 + (x << 7) + (x_lane ^ (x << 4));
    if (c0) cp_async16_s(dst, src);
    if (c1) cp_async16_s(dst + 4 * kVRegion, src + 256);
    if (c2) cp_async16_s(dst + 8 * kVRegion, src + 512);
  }
}

// Group A: the exact-mask softmax of sub-tile t's score tile (eight lanes per query), the weights into att[t & 1] in
// the K-major 128-byte-swizzled layout and the per-table gate signals.
__device__ __forceinline__ void tc_softmax(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t q0 = k.S0 + (int64_t)t * kQ;
  const int lb = t * kQ;
  bar_group_a();
  // softmax: warp w -> queries 4w .. 4w + 3, eight lanes per query; lane -> keys 8 kg .. 8 kg + 7 (kg = lane % 8) of
  // query qi = 4w + lane / 8. In the score tile these keys are the 8-aligned group 8 (kg ^ (swz / 8)) with adjacent
  // pairs swapped when bit 0 of the row's swizzle is set.
  uint8_t* att = S.att + (t & 1) * kQ * 128;
  int64_t* qoff = S.qoff + (t & 1) * kQ;
  const int qi = wid * 4 + (lane >> 3), kg = lane & 7;
  const int swz = sc_swz(qi);
  const float* srow = S.sc + qi * 64 + 8 * (kg ^ (swz >> 3));
  const float4 lo = *reinterpret_cast<const float4*>(srow), hi = *reinterpret_cast<const float4*>(srow + 4);
  float x[8];
  if (swz & 1) {
    x[0] = lo.y; x[1] = lo.x; x[2] = lo.w; x[3] = lo.z; x[4] = hi.y; x[5] = hi.x; x[6] = hi.w; x[7] = hi.z;
  } else {
    x[0] = lo.x; x[1] = lo.y; x[2] = lo.z; x[3] = lo.w; x[4] = hi.x; x[5] = hi.y; x[6] = hi.z; x[7] = hi.w;
  }
  float m = x[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) m = fmaxf(m, x[j]);
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const bool anyv = m != -INFINITY;             // the query has at least one candidate in this table
  float e[8], sum = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    e[j] = x[j] != -INFINITY ? __expf(__fsub_rn(x[j], m)) : 0.f;
    sum += e[j];
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const int64_t sq = q0 + qi;
  const int posq = S.pos[frow(lb + kQ + qi)];
  const bool mine = sq < k.S1 && posq >= a.q_lo && posq < a.q_hi;   // else a key only (another shard's position)
  const int64_t gq = k.b * (a.q_hi - a.q_lo) + (posq - a.q_lo);
  const float rs = anyv ? __frcp_rn(sum) : 0.f;
  if (kg == 0 && k.write_signals && mine) {
    // the largest weight is the maximum's: exp(0) / sum
    a.sen_hay[gq * a.T + k.tau] = anyv ? 1 : 0;
    a.sen_mx[gq * a.T + k.tau] = anyv ? m : kProhibido;
    a.sen_pk[gq * a.T + k.tau] = rs;
  }
  // the 8 weights as one 16-byte chunk (keys 8 kg .. + 7) of row qi of the swizzled K-major operand
  uint4 wv;
  wv.x = umma::pack_bf16x2(__fmul_rn(e[0], rs), __fmul_rn(e[1], rs));
  wv.y = umma::pack_bf16x2(__fmul_rn(e[2], rs), __fmul_rn(e[3], rs));
  wv.z = umma::pack_bf16x2(__fmul_rn(e[4], rs), __fmul_rn(e[5], rs));
  wv.w = umma::pack_bf16x2(__fmul_rn(e[6], rs), __fmul_rn(e[7], rs));
  *reinterpret_cast<uint4*>(att + (qi >> 3) * 1024 + (qi & 7) * 128 + ((kg ^ (qi & 7)) << 4)) = wv;
  if (kg == 0) qoff[qi] = (anyv && mine) ? gq * a.d + k.dp0 : -1;
  umma::fence_proxy_async();       // the weights are read by the tensor cores (async proxy) after the block barrier
}

// Group A: scores of sub-tile t (queries: window slots 32 .. 63; keys: 0 .. 63, slot q0 - 32 + key), the exact-mask
// softmax, the weights into att[t & 1] and the per-table gate signals.
// S^T = phi_k . phi_q^T and Kc . Qc^T on tcgen05, issued by lane 0 of warp 0 once the features are in: A = all 128 rows
// of the feature ring (the keys: lane r of the accumulator is ring row r), B = the sub-tile's 32 query rows (N = 32),
// K = P (phi, 64 features per 128-byte-swizzled column block) and cf (Qc / Kc, 64-byte swizzle); fp32 accumulators in
// TMEM columns kScol + 64 (t & 1) (phi) and + 32 (Qc . Kc). Rows of the ring that are not the window's (a sub-tile being
// loaded) give accumulator lanes nobody reads. The window's keys are two 32-row stages of the ring, i.e. two TMEM lane
// quadrants: the four warps of those quadrants (warp w reads lanes 32 (w % 4) .. + 31) take one key per lane and 16
// queries each (half w / 4) and write t1 (the bf16 rounding chain of the two products) into the score tile; then all
// eight warps add the suffix weight, log_alfa_k and the fp64 time difference and apply the masks in place, eight
// elements per lane.
constexpr uint32_t kScol = 256;     // TMEM columns of the score accumulators (the value products use 0 .. 191)

// The score MMAs of sub-tile t (one thread, once the sub-tile's feature rows are in the ring).
__device__ __forceinline__ void tc_issue_scores(const TcSmem& S, const TcBlock& k, int t, uint32_t tmem) {
  const int lb = t * kQ;
  const uint32_t scol = kScol + 64u * (uint32_t)(t & 1);
  umma::tc_fence_after();
  const uint32_t idesc = umma::idesc_bf16(128, kQ);
  const int rq0 = frow(lb + kQ);                 // first query row (a 32-row stage: 4 KB / 2 KB aligned)
  const uint32_t phi0 = su32(S.phi);
  for (int i = 0; 16 * i < k.Ppad; ++i) {
    const uint32_t blk = phi0 + (uint32_t)(i >> 2) * (kRF * 128), off = (uint32_t)(i & 3) * 32;
    umma::mma_bf16(tmem + scol, umma::desc_sw128(blk + off), umma::desc_sw128(blk + (uint32_t)rq0 * 128 + off), idesc,
                   i > 0 ? 1u : 0u);
  }
  for (int i = 0; 16 * i < k.Cpad; ++i)
    umma::mma_bf16(tmem + scol + kQ, umma::desc_sw64(su32(S.kc) + (uint32_t)i * 32),
                   umma::desc_sw64(su32(S.qc) + (uint32_t)rq0 * 64 + (uint32_t)i * 32), idesc, i > 0 ? 1u : 0u);
  umma::mma_commit(S.sbar + (t & 1));
}

template <bool kSuf4>
__device__ __forceinline__ void tc_scores(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t, uint32_t tmem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int C = a.C;
  const int64_t q0 = k.S0 + (int64_t)t * kQ;
  const int lb = t * kQ;                        // window index of key 0 (li of slot q0 - 32)
  const uint32_t scol = kScol + 64u * (uint32_t)(t & 1);
  const int q4 = wid & 3, hq = wid >> 2;
  const int qa = t & 3, qb = (t + 1) & 3;       // the quadrants (ring stages) of the window's two key halves
  if (q4 == qa || q4 == qb) {
    // t1 of the warp's 32 keys x 16 queries into the score tile (key kj of query qi at qi * 64 + (kj ^ sc_swz(qi)))
    const int kj = (q4 == qa ? 0 : kQ) + lane;   // this lane's key (window index)
    float sp[16], sq[16];
    umma::mbar_wait(S.sbar + (t & 1), (uint32_t)((t >> 1) & 1), a.status);
    __syncwarp();                                // lane 0 of warp 0 may have issued the MMAs: converge for tcgen05.ld
    umma::tc_fence_after();
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16) + scol + (uint32_t)(16 * hq);
    tmem_ld16(trow, sp);
    tmem_ld16(trow + kQ, sq);
    umma::tc_fence_before();                     // the TMEM reads precede the next MMA into this buffer
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      // the reference's rounding chain, two queries per conversion: s1 = bf16(bf16(phi.phi) / T),
      // s2 = bf16(bf16(Qc.Kc) * cf^-1/2), t1 = bf16(s1 + s2)
      float s1a = sp[j], s1b = sp[j + 1], s2a = sq[j], s2b = sq[j + 1];
      round2_bf16(s1a, s1b);
      round2_bf16(s2a, s2b);
      s1a = __fmul_rn(s1a, k.inv_temp);
      s1b = __fmul_rn(s1b, k.inv_temp);
      s2a = __fmul_rn(s2a, a.esc_c);
      s2b = __fmul_rn(s2b, a.esc_c);
      round2_bf16(s1a, s1b);
      round2_bf16(s2a, s2b);
      float t1a = __fadd_rn(s1a, s2a), t1b = __fadd_rn(s1b, s2b);
      round2_bf16(t1a, t1b);
      const int qi = 16 * hq + j;
      S.sc[qi * 64 + (kj ^ sc_swz(qi))] = t1a;
      S.sc[(qi + 1) * 64 + (kj ^ sc_swz(qi + 1))] = t1b;
    }
  }
  bar_group_a();
  // every warp: the rest of the score of 8 elements per lane (key columns kj0, kj0 + 1 of warp n-tile wid; query rows
  // g, g + 8, g + 16, g + 24): suffix weight, log_alfa_k, the fp64 time difference and the masks, in place
  {
    const int nt = wid;
    const int g4 = lane >> 2, kj0 = nt * 8 + (lane & 3) * 2;
    int k_id[2];
    float4 k_pf[2][2];
    double k_bt[2];
    float k_la[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int rk = frow(lb + kj0 + u);
      k_id[u] = S.id[rk];
      k_pf[u][0] = *reinterpret_cast<const float4*>(S.pf + rk * kMaxSuffix);
      k_pf[u][1] = *reinterpret_cast<const float4*>(S.pf + rk * kMaxSuffix + 4);
      k_bt[u] = S.bt[rk];
      k_la[u] = S.la[rk];
    }
    const int64_t rem = a.L - q0;
    const int qlim = rem < kQ ? (int)rem : kQ;
    const bool kv[2] = {q0 - kQ + kj0 >= 0, q0 - kQ + kj0 + 1 >= 0};
    const int wlo = kQ - C;                      // key kj is a candidate of query qi iff kj - qi in [32 - C, 32)
#pragma unroll
    for (int uq = 0; uq < 4; ++uq) {
      const int qi = g4 + 8 * uq;
      const int rq = frow(lb + kQ + qi);
      const int q_id = S.id[rq];
      const float4 qa4 = *reinterpret_cast<const float4*>(S.pf + rq * kMaxSuffix);
      const double q_bt = S.bt[rq];
      const bool qv = qi < qlim;
      const int row = qi * 64, swz = sc_swz(qi);
#pragma unroll
      for (int uk = 0; uk < 2; ++uk) {
        const int kj = kj0 + uk;
        float* cell = S.sc + row + (kj ^ swz);
        const bool ok = qv && kv[uk] && (unsigned)(kj - qi - wlo) < (unsigned)C && k_id[uk] == q_id;
        if (!ok) {
          *cell = -INFINITY;
          continue;
        }
        const float4 ka = k_pf[uk][0];
        int ln;
        if (kSuf4) {                             // entries past K are NaN (never equal)
          ln = qa4.x == ka.x ? (qa4.y == ka.y ? (qa4.z == ka.z ? (qa4.w == ka.w ? 4 : 3) : 2) : 1) : 0;
        } else {
          const float4 qb4 = *reinterpret_cast<const float4*>(S.pf + rq * kMaxSuffix + 4), kb = k_pf[uk][1];
          const uint32_t eq = (qa4.x == ka.x ? 1u : 0u) | (qa4.y == ka.y ? 2u : 0u) | (qa4.z == ka.z ? 4u : 0u) |
                              (qa4.w == ka.w ? 8u : 0u) | (qb4.x == kb.x ? 16u : 0u) | (qb4.y == kb.y ? 32u : 0u) |
                              (qb4.z == kb.z ? 64u : 0u) | (qb4.w == kb.w ? 128u : 0u);
          ln = __ffs(~eq) - 1;                   // leading equal entries
        }
        float v = __fadd_rn(*cell, S.wsuf[ln]);
        v = __fadd_rn(v, k_la[uk]);
        const float dt = __double2float_rn(k_bt[uk] - q_bt);
        v = __fadd_rn(v, __fmul_rn(dt, k.tasa));
        *cell = v;
      }
    }
  }
  tc_softmax(a, S, k, t);
}

// Group B: out^T = V^T . att^T for sub-tile t on tcgen05, reduced into the bf16 accumulator. Lane 0 of warp mm issues
// M-tile mm (rows 128 mm .. + 127 of d_part: two 64-column regions of the value ring, MN-major, 12 KB apart), K-step
// ks (window keys 16 ks .. + 15: two 8-key groups of the ring, 1024 B apart), N = the 32 queries (att rows, K-major);
// D in TMEM columns 32 mm .. + 31. Then warp w reads TMEM lanes 32 (w % 4) .. + 31 (32 rows of d) for M-tiles
// (w - 8) / 4, + 2, + 4, 16 query columns at a time: each lane holds one row of d for 16 queries and stores them into
// a 2 KB staging piece laid out [query][32 rows of d], the 16-byte granules of a query's row permuted by the query
// (granule g of query q at g ^ (q mod 8)) so that both the stores (one query row per instruction) and the reads
// (eight queries x four granule pairs per instruction) are free of bank conflicts. Each lane then reads 8 consecutive
// rows of d of one query and adds them, rounded to bf16, with one 16-byte bf16 reduction: a warp instruction covers
// 8 queries x 64 bytes. The pieces sit in the value ring's rows of sub-tile t - 1, which no MMA reads once sub-tile
// t's products are done; they are zeroed afterwards, since ring rows that are not reloaded must keep finite bf16
// contents (they meet zero weights).
__device__ __forceinline__ void tc_values(const ScoreArgs& a, const TcSmem& S, const TcBlock& k, int t, int w,
                                          uint32_t tmem) {
  const int lane = threadIdx.x & 31;
  const int lb = t * kQ;                        // window index of key 0 (li of slot q0 - 32)
  const int nM = k.dpart / 128;
  if (w < nM && lane == 0) {                    // warp w issues M-tile w (its own commit on the shared barrier)
    umma::tc_fence_after();
    const uint32_t idesc = umma::idesc_bf16(128, kQ) | (1u << 15);      // A (the value rows) MN-major
    const uint32_t v0 = su32(S.v) + (uint32_t)(2 * w) * kVRegion, a0 = su32(S.att + (t & 1) * kQ * 128);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int r0 = vrow(lb + ks * 16);
      const uint64_t adesc = umma::desc_mn_sw128(v0 + (uint32_t)(r0 >> 3) * 1024, (uint32_t)kVRegion);
      umma::mma_bf16(tmem + (uint32_t)(w * kQ), adesc, umma::desc_sw128(a0 + ks * 32), idesc, ks > 0 ? 1u : 0u);
    }
    umma::mma_commit(S.pvbar);
  }
  // this lane's reductions: query rq(hq, j) = 16 hq + 8 j + lane / 4, rows of d 8 (lane % 4) .. + 7 of the warp's 32
  // (granules 2 (lane % 4) and + 1 of the query's staged row, at g ^ (lane / 4))
  const int64_t* qoff_s = S.qoff + (t & 1) * kQ;
  const int kq = lane >> 2, kg = lane & 3;
  const int rd0 = kq * 32 + (((2 * kg) ^ kq) << 2), rd1 = kq * 32 + (((2 * kg + 1) ^ kq) << 2);
  int64_t qo[2][2];
#pragma unroll
  for (int hq = 0; hq < 2; ++hq)
#pragma unroll
    for (int j = 0; j < 2; ++j) qo[hq][j] = qoff_s[16 * hq + 8 * j + kq];
  // this warp's staging piece: 2 KB of the ring rows of sub-tile t - 1 (32 rows x 128 B per 64-column region; warp w
  // takes half w % 2 of region w / 2, so the 4 nM pieces of the active warps fit in the 2 nM regions)
  float* piece = reinterpret_cast<float*>(S.v + (w >> 1) * kVRegion + vrow(lb) * 128 + (w & 1) * 2048);
  __syncwarp();
  umma::mbar_wait(S.pvbar, (uint32_t)(t & 1), a.status);
  umma::tc_fence_after();
  const int q4 = w & 3;
  __nv_bfloat16* acc16 = reinterpret_cast<__nv_bfloat16*>(a.acc);
  bool staged = false;
  for (int mm = w >> 2; mm < nM; mm += 2) {
    __nv_bfloat16* dst_base = acc16 + mm * 128 + q4 * 32 + 8 * kg;
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(mm * kQ + hq * 16), v);
      __syncwarp();                             // the previous reads of the piece are done
#pragma unroll
      for (int c = 0; c < 16; ++c) piece[c * 32 + (lane ^ ((c & 7) << 2))] = v[c];
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float4 lo = *reinterpret_cast<const float4*>(piece + 256 * j + rd0);
        const float4 hi = *reinterpret_cast<const float4*>(piece + 256 * j + rd1);
        if (qo[hq][j] >= 0)
          red_add_bf16x8(dst_base + qo[hq][j], pack2_bf16(lo.x, lo.y), pack2_bf16(lo.z, lo.w),
                         pack2_bf16(hi.x, hi.y), pack2_bf16(hi.z, hi.w));
      }
      staged = true;
    }
  }
  if (staged) {
    __syncwarp();
    uint4* z = reinterpret_cast<uint4*>(piece);
#pragma unroll
    for (int i = 0; i < 4; ++i) z[lane + 32 * i] = make_uint4(0, 0, 0, 0);
    umma::fence_proxy_async();                  // the zeros precede later tensor-core reads of these rows
  }
  umma::tc_fence_before();
}

__global__ void __launch_bounds__(kThreadsTc, 1)
k_score_tc(const __grid_constant__ CUtensorMap tm_phi, const __grid_constant__ CUtensorMap tm_qc,
           const __grid_constant__ CUtensorMap tm_kc, ScoreArgs a, int nds, int dpart, int span) {
  extern __shared__ __align__(16) char smem_raw[];
  const TcSmem S = carve_tc(smem_raw, a.P, a.cf, dpart);
  TcBlock k;
  k.r = blockIdx.y;
  k.b = k.r / a.T;
  k.tau = (int)(k.r % a.T);
  const int part = blockIdx.x % nds;
  k.S0 = (int64_t)(blockIdx.x / nds) * span;
  k.S1 = min(min(k.S0 + span, a.L), a.row_len ? a.row_len[k.r] : a.L);
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

  // zero both rings once (rows never loaded keep finite contents), set up the barriers, TMEM for the value products
  {
    uint4* z0 = reinterpret_cast<uint4*>(S.v);
    const int nz = (int)((reinterpret_cast<char*>(S.st_pos) - reinterpret_cast<char*>(S.v)) / 16);
    for (int i = threadIdx.x; i < nz; i += blockDim.x) z0[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x <= kMaxSuffix) S.wsuf[threadIdx.x] = threadIdx.x <= a.K ? a.w_suf[threadIdx.x] : 0.f;
    umma::fence_proxy_async();                 // the zeros precede the tensor-map copies into the same rows
    if (threadIdx.x == 0) {
      for (int i = 0; i < 4; ++i) umma::mbar_init(S.fbar + i, 1);   // 4 feature stages
      umma::mbar_init(S.pvbar, (uint32_t)(k.dpart / 128));           // one commit per M-tile's issuing warp
      umma::mbar_init(S.sbar, 1);                                      // score MMAs of even / odd sub-tiles
      umma::mbar_init(S.sbar + 1, 1);
      umma::fence_mbar_init();
    }
    if (wid == kGroupWarps) {
      umma::tmem_alloc(S.tmem, 512);
      umma::tmem_relinquish();
    }
  }
  const bool loader = wid >= 2 * kGroupWarps;
  const int pt = threadIdx.x - 2 * kGroupWarps * 32;   // thread index within the load group
  // bounded wait for the feature rows of sub-tile t (stage (t + 1) % 4), by the thread that issues its score MMAs
  auto wait_features = [&](int t) {
    umma::mbar_wait(S.fbar + ((t + 1) & 3), (uint32_t)(((t + 1) >> 2) & 1), a.status);
  };
  // the stage's transaction count, set by load thread 0 before any copy of the stage is issued (bar_load)
  auto expect_features = [&](int t) {
    if (pt == 0) umma::mbar_expect_tx(S.fbar + ((t + 1) & 3), (uint32_t)(kQ * (S.nbp * 128 + 2 * 64)));
  };
  // this thread's cp.async copies complete (value rows: then made visible to the tensor cores)
  auto wait_copies = [&]() {
    cp_async_wait_all();
    umma::fence_proxy_async();
  };
  auto bar_load = []() { asm volatile("bar.sync 2, %0;" ::"n"(kLoadThreads) : "memory"); };

  // prologue: the load group copies sub-tiles -1 (the first window half), 0, 1 and 2 of the features, sub-tile 3's
  // sorted entries and the value rows of -1 and 0; then group A issues the score MMAs of sub-tiles 0 and 1 and scores
  // sub-tile 0
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *S.tmem;
  if (loader) {
    tc_stage1(a, S, k, -1, pt);
    tc_stage1(a, S, k, 0, pt);
    if (ntile > 1) tc_stage1(a, S, k, 1, pt);
    cp_async_commit();
    cp_async_wait_all();
    expect_features(-1);
    expect_features(0);
    if (ntile > 1) expect_features(1);
    bar_load();
    tc_stage2_features(a, S, k, -1, pt, &tm_phi, &tm_qc, &tm_kc);
    tc_stage2_features(a, S, k, 0, pt, &tm_phi, &tm_qc, &tm_kc);
    if (ntile > 1) tc_stage2_features(a, S, k, 1, pt, &tm_phi, &tm_qc, &tm_kc);
    cp_async_commit();
    cp_async_wait_all();
    bar_load();
    if (ntile > 2) {
      tc_stage1(a, S, k, 2, pt);                // its buffer was read by sub-tile -1's feature stage above
      cp_async_commit();
      cp_async_wait_all();
      expect_features(2);
      bar_load();
      tc_stage2_features(a, S, k, 2, pt, &tm_phi, &tm_qc, &tm_kc);
      if (ntile > 3) tc_stage1(a, S, k, 3, pt);  // its buffer was read by sub-tile 0's feature stage
    }
    tc_stage2_values(a, S, k, -1, pt);
    tc_stage2_values(a, S, k, 0, pt);
    cp_async_commit();
    wait_copies();
  }
  __syncthreads();
  const bool suf4 = a.K <= 4;
  if (group_a) {
    if (threadIdx.x == 0) {                     // the issuer of the score MMAs waits for the feature rows
      wait_features(-1);
      wait_features(0);
      tc_issue_scores(S, k, 0, tmem);
      if (ntile > 1) {
        wait_features(1);
        tc_issue_scores(S, k, 1, tmem);
      }
    }
    if (suf4) tc_scores<true>(a, S, k, 0, tmem);
    else tc_scores<false>(a, S, k, 0, tmem);
  }
  __syncthreads();

  // iteration i: group A scores sub-tile i + 1, group B takes the value products of i; meanwhile the load group copies
  // the value rows of i + 1 and the sorted entries of i + 4 (waited for at the end of the iteration), then the features
  // of i + 3 (into the ring stage of i - 1, which no score MMA or epilogue reads from here on; the scalar copies are
  // waited for in the next iteration, the rows by the stage's mbarrier), and its first thread issues the score MMAs of
  // i + 2 while its copies are in flight: their features arrived during the previous iteration, their TMEM buffer (sub-tile i's) was read by
  // group A in the previous iteration. (Issued by group A at the end of its epilogue, the six MMAs held its iteration
  // about 450 ns; issued at its start, where group B's value MMAs queue, about 1 us.)
  for (int i = 0; i < ntile; ++i) {
    if (loader) {
      if (i + 3 < ntile) expect_features(i + 3);
      if (i + 4 < ntile) tc_stage1(a, S, k, i + 4, pt);
      if (i + 1 < ntile) tc_stage2_values(a, S, k, i + 1, pt);
      cp_async_commit();                        // group 1: the value rows and sorted entries, used next iteration
      if (i + 3 < ntile) {
        bar_load();                             // the expect_tx precedes every copy of the stage
        tc_stage2_features(a, S, k, i + 3, pt, &tm_phi, &tm_qc, &tm_kc);
      }
      cp_async_commit();                        // group 2: the scalars of i + 3, first read in iteration i + 2
      // the score MMAs of sub-tile i + 2 while the copies are in flight
      if (i + 2 < ntile && pt == 0) {
        wait_features(i + 2);
        tc_issue_scores(S, k, i + 2, tmem);
      }
      __syncwarp();                             // the issuing warp converges before its next named barrier
      // group 1 and everything older (the previous iteration's group 2) complete; this iteration's scalars may land
      // during the next one. Value rows: then made visible to the tensor cores.
      cp_async_wait_but_last();
      umma::fence_proxy_async();
    } else if (group_a) {
      if (i + 1 < ntile) {
        if (suf4) tc_scores<true>(a, S, k, i + 1, tmem);
        else tc_scores<false>(a, S, k, i + 1, tmem);
      }
    } else {
      tc_values(a, S, k, i, wid - kGroupWarps, tmem);
    }
    __syncthreads();
  }
  if (wid == kGroupWarps) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, 512);
  }
}

bool score_tc_supported(const ScoreArgs& a) {
  return a.d % 128 == 0 && a.d <= 1536 && a.C <= 32 && a.P <= kMaxPhi && a.P % 8 == 0 &&
         a.cf <= kMaxConfirm && a.cf % 8 == 0 && a.K <= kMaxSuffix && a.L % 8 == 0 && a.B * a.Lf < ((int64_t)1 << 31);
}

int launch_score_tc(const ScoreArgs& a, cudaStream_t s) {
  // the whole width in one block when its 96-row value ring fits next to the features (d <= 768), else parts that are
  // multiples of 128 (the value MMAs' M)
  int nds = (a.d + 767) / 768;
  while (a.d % (nds * 128) != 0) ++nds;
  const int dpart = a.d / nds;
  if (dpart / 128 > kMaxMt) return ASRN_ERR_UNSUPPORTED;
  const size_t smem = tc_smem_bytes(a.P, a.cf, dpart);
  if (smem > 227 * 1024) return ASRN_ERR_UNSUPPORTED;
  // feature rows as one-row boxes of one ring row (64 phi features / 32 Qc, Kc features with the ring's swizzle;
  // columns past P / cf read zeros)
  CUtensorMap tm_phi, tm_qc, tm_kc;
  const uint64_t rows = (uint64_t)(a.B * a.Lf);
  if (!make_tmap_rows_bf16(&tm_phi, a.phi, (uint64_t)a.P, rows, (uint64_t)a.P * 2, 64, 128) ||
      !make_tmap_rows_bf16(&tm_qc, a.Qc, (uint64_t)a.cf, rows, (uint64_t)a.cf * 2, 32, 64) ||
      !make_tmap_rows_bf16(&tm_kc, a.Kc, (uint64_t)a.cf, rows, (uint64_t)a.cf * 2, 32, 64))
    return ASRN_ERR_CUDA;
  cudaFuncSetAttribute(k_score_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // each block pays a prologue of about 10 us (the first window half and two sub-tiles of latency): spans of 1024 or
  // 2048 slots while the grid keeps at least 4 blocks per SM (32 x 8192 tokens: 2048 slots, 6.9 waves of one block
  // per SM, 3.11 instead of 3.16 ms with the 8-per-SM rule's 1024)
  int span = kSpanTc;
  while (span < 2048 && ((a.L + 2 * span - 1) / (2 * span)) * nds * a.B * a.T >= 4 * 148) span *= 2;
  dim3 grid((unsigned)(((a.L + span - 1) / span) * nds), (unsigned)(a.B * a.T));
  k_score_tc<<<grid, kThreadsTc, smem, s>>>(tm_phi, tm_qc, tm_kc, a, nds, dpart, span);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
