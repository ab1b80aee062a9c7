// FlashEntropyAttention backward on tcgen05 / TMEM / TMA, D = 128 (reference semantics:
// video_monarch_attention/kernel.py:154-313, including the entropy-gradient term folded into the
// per-row constants c_i, g_i computed by fea_bwd_pre: dS = P (dP - c_i - g_i x_ij)).
//
// TMEM holds 512 fp32 columns per SM, too few for S^T, dP^T, dK, dV and dQ of one tile at once, so
// in general the backward is two kernels (7 MMAs per 128x64 tile pair instead of 5, but no atomics
// and a deterministic result):
//
// dkdv kernel: CTA = 128 keys of one sequence, walks the query tiles (64 rows):
//   S^T = K Q^T, dP^T = W dO^T                  (SS MMAs, M = 128 keys, N = 64 queries)
//   thread = key row: P^T = 2^(x - LSE2_q), dS^T = P^T (dP^T - c_q - g_q x) sm_scale
//     -> bf16 back into TMEM (double-buffered)
//   dK += dS^T Q;  dV += P^T dO                  (TS MMAs, A = P^T / dS^T from TMEM)
//   With V aliasing K (the VMonarch R step, W = [K | V2]) the value gradient of the K columns is
//   added into dK by one more TS MMA (dK += P^T dO[:, :128]) and dV holds the V2 columns.
//   TMEM: buffer b (query tile parity) S^T [128b, 128b+64) dP^T [128b+64, 128b+128),
//   dK [256,384), dV [384,512)
// dq kernel: CTA = 128 queries, walks the key tiles (128 rows):
//   S = Q K^T, dP = dO W^T (SS, double-buffered in TMEM), dS (thread = query row) -> TMEM,
//   dQ += dS K (TS).
// Both write their gradients directly (bf16, or added into fp32 accumulators in grad_mode 1).
//
// Fused dQ (FQ, V aliasing K with no V2, fp32 dQ, few key tiles per sequence: the first VMonarch R
// step): the dK kernel also stages dS^T (bf16) in shared memory and forms dQ^T = K^T dS^T
// (SS MMA, both operands M/N-major, M = 128 head dims, N = 64 queries) into the free dV columns
// (two buffers [384 + 64b, 448 + 64b)); the compute threads reduce-add it into the fp32 dQ
// (thread = head-dim row, a warp covers 128 contiguous bytes of one query row), and the dq kernel
// is not run: 5 MMAs per tile pair, at the price of n_kv / 128 fp32 reductions per dQ element
// (summation order varies between runs).
// Tails: rows past n_q / n_kv load as zeros (TMA), the folded statistics of queries past n_q are
// (-1e30, 0, 0) so their P and dS are 0; gradients are only stored for valid rows. Every wait is bounded (sm100.cuh).
#include <algorithm>

#include "common.cuh"
#include "fea_params.h"
#include "launch.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace vmb {

__device__ int g_bwd_err;

namespace {

using namespace sm100;

constexpr int kDqWarpgroups = 4;       // dQ kernel: compute warpgroups (32 key columns each)
constexpr int kDqThreads = 64 + 128 * kDqWarpgroups;
constexpr int kDkdvWarpgroups = 4;     // dK/dV kernel: two per query-tile stream (32 queries each)
constexpr int kDkdvThreads = 64 + 128 * kDkdvWarpgroups;
constexpr int kAtom128 = 128 * 128;  // swizzle-atom column block of 128 rows x 128 B
constexpr int kAtom64 = 64 * 128;    // ... of 64 rows x 128 B

struct Sm100BwdParams {
  CUtensorMap tm_a, tm_b, tm_c, tm_d;  // dkdv: K, X, Q, dO ; dq: Q, dO, K, X  (boxes of 64 cols x 64/128 rows)
  CUtensorMap tm_g0, tm_g1;            // gradient outputs (dkdv: dK, dV / dV2; dq: dQ): fp32 boxes of
                                       // 32 x 128 when added into (acc), else 16-bit boxes of 64 x 128
  const void* dout;  // dq kernel with dO in TMEM: [batch][n_q][DW] rows read directly (view dov)
  View dov;
  int n1, n2;        // batch split of every view and of the maps over caller tensors
  const float* nl;  // folded statistics planes [batch][n_pad] (fea_bwd_pre): -LSE2,
  const float* nc;  //   -sm_scale (c + g LSE2),
  const float* ng;  //   -sm_scale g
  int64_t n_pad;
  int n_q, n_kv, n_tiles;
  int k_split, kt_per;  // dQ kernel: key range split over k_split CTAs of kt_per 128-key tiles each
  int n_seq;            // sequences (batch) of the call
  int acc;       // 1: fp32 gradients added into (TMA reduce-add); 2: fp32 stores; 0: 16-bit stores;
                 // 3: 16-bit stores of (fp32 accumulator tile + this call's gradient)
  float scale_log2, sm_scale;
  float* dq;     // fused dQ: dense fp32 [batch][n_q][128] with batch stride dq_bs, added into
  int64_t dq_bs;
  CUtensorMap tm_f0, tm_f1;  // acc 3: the fp32 accumulators of tm_g0 / tm_g1 (boxes of 32 x 128)
  // d = 64 with V aliasing K and a second value tensor: the second atom of every K tile is V2,
  // loaded from tm_b (dK / dV kernel) or tm_d (dq kernel) at column 0, so the tile is [K | V2];
  // Q's second atom is zero, so S and dS are unchanged, dP = dO [K | V2]^T, and the dK
  // accumulator's second half is dV2 (stored through tm_g1)
  int k_hi_x;
  void* ds;                  // dK/dV kernel: dS^T out [batch][ds_rows][ds_ld] (16-bit), or null
  int64_t ds_ld, ds_bs;      // row stride (queries, padded to 64) and batch stride (elements)
};

// acc 3: out16 = 16-bit(TMEM accumulator + fp32 accumulator tile staged at `fin`), for the 32-column
// chunks [c_begin, c_end) of row `row`; fp32 staging as in stage_acc_rows, 16-bit output as two
// [128 rows][64 elements] boxes at out + a * 16 KB.
template <typename T>
__device__ __forceinline__ void finalize_rows(uint32_t taddr, uint32_t fin, uint32_t out, int row, int c_begin,
                                              int c_end) {
#pragma unroll 1
  for (int c = c_begin; c < c_end; ++c) {
    uint32_t v[32];
    tmem_ld32(taddr + c * 32, v);
    tmem_wait_ld();
    const uint32_t src = fin + c * 16384 + row * 128;
    uint32_t w[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float4 a;
      asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                   : "=f"(a.x), "=f"(a.y), "=f"(a.z), "=f"(a.w)
                   : "r"(src + ((k ^ (row & 7)) << 4)));
      w[2 * k] = Elem<T>::pack(__uint_as_float(v[4 * k]) + a.x, __uint_as_float(v[4 * k + 1]) + a.y);
      w[2 * k + 1] = Elem<T>::pack(__uint_as_float(v[4 * k + 2]) + a.z, __uint_as_float(v[4 * k + 3]) + a.w);
    }
    const uint32_t base = out + (c >> 1) * 16384 + row * 128;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int chunk = (c & 1) * 4 + k;
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((chunk ^ (row & 7)) << 4)), "r"(w[4 * k]),
                   "r"(w[4 * k + 1]), "r"(w[4 * k + 2]), "r"(w[4 * k + 3])
                   : "memory");
    }
  }
}

// Gradient epilogue. The 128 x 128 fp32 accumulator tile in TMEM (thread = row = TMEM lane) is
// staged in shared memory with the 128-byte swizzle and written by TMA: reduce-add into fp32
// gradients (acc), or stored as 16-bit values. The read-modify-write then runs in the memory system
// instead of stalling the SM on load latency, and rows past the map's extent are clipped.
// Staging layout: fp32 -> four [128 rows][32 floats] boxes at stage + c * 16 KB; 16-bit -> two
// [128 rows][64 elements] boxes at stage + a * 16 KB.
template <typename T>
__device__ __forceinline__ void stage_acc_rows(uint32_t taddr, uint32_t stage, int row, bool f32, int c_begin,
                                               int c_end) {
#pragma unroll 1
  for (int c = c_begin; c < c_end; ++c) {
    uint32_t v[32];
    tmem_ld32(taddr + c * 32, v);
    tmem_wait_ld();
    if (f32) {
      const uint32_t base = stage + c * 16384 + row * 128;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((k ^ (row & 7)) << 4)), "r"(v[4 * k]),
                     "r"(v[4 * k + 1]), "r"(v[4 * k + 2]), "r"(v[4 * k + 3])
                     : "memory");
    } else {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = Elem<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
      const uint32_t base = stage + (c >> 1) * 16384 + row * 128;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int chunk = (c & 1) * 4 + k;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((chunk ^ (row & 7)) << 4)),
                     "r"(w[4 * k]), "r"(w[4 * k + 1]), "r"(w[4 * k + 2]), "r"(w[4 * k + 3])
                     : "memory");
      }
    }
  }
}

// One thread, after the staging barrier: the whole 128-row tile starting at row0 of sequence bi.
// mode 1: fp32 reduce-add; 2: fp32 store; 0: 16-bit store.
__device__ __forceinline__ void issue_grad_tile(const CUtensorMap* tm, uint32_t stage, int row0, BIdx bi, int mode) {
  if (mode == 1) {
    for (int c = 0; c < 4; ++c) tma_reduce_add(tm, 32 * c, row0, bi, stage + c * 16384);
  } else if (mode == 2) {
    for (int c = 0; c < 4; ++c) tma_store(tm, 32 * c, row0, bi, stage + c * 16384);
  } else {
    for (int a = 0; a < 2; ++a) tma_store(tm, 64 * a, row0, bi, stage + a * 16384);
  }
}

// issue_grad_tile for a [lo | hi] tile of two 64-column tensors: columns [0, 64) through `lo`,
// [64, 128) through `hi` from its column 0 (modes 0, 1, 2).
__device__ __forceinline__ void issue_grad_tile_split(const CUtensorMap* lo, const CUtensorMap* hi, uint32_t stage,
                                                      int row0, BIdx bi, int mode) {
  if (mode == 1 || mode == 2) {
    for (int c = 0; c < 4; ++c) {
      const CUtensorMap* tm = c < 2 ? lo : hi;
      if (mode == 1)
        tma_reduce_add(tm, 32 * (c & 1), row0, bi, stage + c * 16384);
      else
        tma_store(tm, 32 * (c & 1), row0, bi, stage + c * 16384);
    }
  } else {
    tma_store(lo, 0, row0, bi, stage);
    tma_store(hi, 0, row0, bi, stage + 16384);
  }
}

// ================================================================================ dK / dV kernel
// XA: resident value atoms (V when !VK, V2 when VK); DW = width of W (and of dO).
// Folded per-query statistics (written by fea_bwd_pre). With t = s * scale_log2 - LSE2 (the log2-
// domain score minus the query's LSE2), P = 2^t and the reference's dS = sm_scale P (dP - c - g x),
// x = t + LSE2, becomes dS = P (sm_scale dP + nc + ng t) with nl = -LSE2, nc = -sm_scale (c + g LSE2),
// ng = -sm_scale g: two packed f32x2 FMAs and one multiply per pair of scores. Queries past n_q have
// nl = -1e30 (finite, so ng t = 0 with ng = 0), hence P = 0 and dS = 0.

// P and dS of two scores (s0, s1) with their dP (d0, d1), packed to the element type.
template <typename T, bool WANT_P>
__device__ __forceinline__ void prob_dscore(uint32_t s0, uint32_t s1, uint32_t d0, uint32_t d1, float2 sc2, float2 sm2,
                                            float2 nl2, float2 nc2, float2 ng2, uint32_t& p_out, uint32_t& ds_out) {
  const float2 t = __ffma2_rn(make_float2(__uint_as_float(s0), __uint_as_float(s1)), sc2, nl2);
  const float2 pr = make_float2(fast_exp2(t.x), fast_exp2(t.y));
  const float2 u = __ffma2_rn(ng2, t, __ffma2_rn(make_float2(__uint_as_float(d0), __uint_as_float(d1)), sm2, nc2));
  const float2 ds = __fmul2_rn(pr, u);
  if (WANT_P) p_out = Elem<T>::pack(pr.x, pr.y);
  ds_out = Elem<T>::pack(ds.x, ds.y);
}

template <int XA, bool VK, int NQS, bool FQ = false>
struct DkdvCfg {
  static constexpr int DW = VK ? 128 + 64 * XA : 64 * XA;
  static constexpr int RES = (2 + XA) * kAtom128;                 // resident K | X
  static constexpr int DS = FQ ? 2 * kAtom128 : 0;                // fused dQ: dS^T of both streams
  static constexpr int SLOT_T = (2 + DW / 64) * kAtom64;          // Q | dO tiles of one query tile
  static constexpr int SLOT = SLOT_T + 1024;                      // + statistics: LSE2, c, g x 64
  static constexpr int SMEM = 1024 + RES + DS + NQS * SLOT;
  static constexpr bool HAS_DV = XA > 0;
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(!FQ || (VK && XA == 0), "fused dQ needs the dV columns of TMEM");
};

__device__ __forceinline__ void red_add_f32(float* ptr, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(ptr), "f"(v) : "memory");
}

// 32 bytes to a 32-byte aligned global address (one 256-bit store, sm_100)
__device__ __forceinline__ void st_global_v8(void* ptr, const uint32_t* v) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

template <typename T, int XA, bool VK, int NQS, int NWG, bool FQ = false>
__global__ void __launch_bounds__(64 + 128 * NWG, 1) fea_bwd_dkdv_kernel(const __grid_constant__ Sm100BwdParams p) {
  using C = DkdvCfg<XA, VK, NQS, FQ>;
  constexpr bool kBf16 = Elem<T>::is_bf16;
  constexpr uint32_t IDESC_SP = idesc_f16(kBf16, 128, 64, false, false);   // S^T, dP^T
  constexpr uint32_t IDESC_SPK = idesc_f16(kBf16, 128, 128, false, false);  // [S^T | dP^T] = K [Q | dO_K]^T (V aliasing K)
  constexpr uint32_t IDESC_ACC = idesc_f16(kBf16, 128, 128, false, true);  // dK, dV (B MN-major)
  constexpr uint32_t IDESC_DQ = idesc_f16(kBf16, 128, 64, true, true);     // dQ^T = K^T dS^T (both MN-major)
  constexpr uint32_t IDESC_SP32 = idesc_f16(kBf16, 128, 32, false, false);  // a last tile of <= 32 queries
  constexpr uint32_t IDESC_DQ32 = idesc_f16(kBf16, 128, 32, true, true);
  static_assert(NWG == 2 || NWG == 4, "two or four compute warpgroups");
  static_assert(!FQ || NWG == 4, "fused dQ: two warpgroups per stream, 32 queries each");
  // Column of the packed P^T / dS^T of queries [16kk, 16kk + 16) inside a tile's S^T / dP^T:
  // two warpgroups (one per tile) write halves h at [16h, 16h + 16); four (two per tile, one per
  // 32-query half) write half h at [32h, 32h + 16), inside the range that warpgroup loaded itself.
  auto pcol = [](int kk) -> uint32_t { return NWG == 4 ? 32 * (kk >> 1) + 8 * (kk & 1) : 8 * kk; };

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[1 + 2 * NQS + 5 + 2 + 1 + 2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bi = blockIdx.x / p.n_tiles;
  const BIdx bx = bidx(bi, p.n1, p.n2);
  const int k0 = (blockIdx.x % p.n_tiles) * 128;
  const int nq = (p.n_q + 63) / 64;
  // Query tile of step i. With fused dQ the key tiles of a sequence start their walks at different
  // query tiles, so the concurrent reductions into one dQ row come from different steps.
  const int rot = FQ ? (2 * (blockIdx.x % p.n_tiles)) % nq : 0;
  auto qtile = [&](int i) { return FQ ? (i + rot < nq ? i + rot : i + rot - nq) : i; };
  // a last query tile of <= 32 queries: S^T, dP^T (and dQ^T) at N = 32, the query contractions over
  // its first 32 queries (the other columns are stale TMEM that no MMA reads)
  auto qtail = [&](int i) { return p.n_q - qtile(i) * 64 <= 32; };

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sRes = sbase;                       // K atoms, then X atoms
  const uint32_t sW = VK ? sRes : sRes + 2 * kAtom128;
  const uint32_t sDS = sbase + C::RES;               // fused dQ: dS^T of stream b at sDS + b * kAtom128
  const uint32_t sSlots = sbase + C::RES + C::DS;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t BAR_KV = bar0;
  auto BAR_QFULL = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_QEMPTY = [&](int s) { return bar0 + 8u * (1 + NQS + s); };
  auto BAR_SPFULL = [&](int b) { return bar0 + 8u * (1 + 2 * NQS + b); };
  auto BAR_PDSFULL = [&](int b) { return bar0 + 8u * (3 + 2 * NQS + b); };
  const uint32_t BAR_DONE = bar0 + 8u * (5 + 2 * NQS);
  // fused dQ: stream b has drained dQ^T of its previous tile and staged dS^T of the current one
  auto BAR_DQFREE = [&](int b) { return bar0 + 8u * (6 + 2 * NQS + b); };
  const uint32_t BAR_FIN = bar0 + 8u * (8 + 2 * NQS);  // acc 3: the fp32 accumulator tiles landed
  // fused dQ: dQ^T of stream b's latest tile complete (commit behind it). S^T / dP^T of tile i + 2
  // is issued before dQ^T(i), so its completion no longer implies dQ^T(i)'s: the stream waits here
  // before overwriting its dS^T staging and before draining dQ^T(i)
  auto BAR_DQDONE = [&](int b) { return bar0 + 8u * (9 + 2 * NQS + b); };
  volatile int* abort = &abort_sh;
  // Query slot: 64-query tiles of Q (2 atoms of 64 columns) and dO (DW / 64 atoms). With V aliasing
  // K the first two dO atoms interleave with Q's (Q0 dO0 Q1 dO1 [dO2 dO3]), so that Q atom a and
  // dO atom a form one 128-row K-major operand: S^T and the K part of dP^T are then one N = 128
  // MMA group, [S^T | dP^T] = K [Q | dO_K]^T, which reads the resident K once for both.
  auto q_atom = [&](int s, int a) -> uint32_t { return sSlots + s * C::SLOT + (VK ? 2 * a : a) * kAtom64; };
  auto do_atom = [&](int s, int a) -> uint32_t {
    return sSlots + s * C::SLOT + (VK ? (a < 2 ? 2 * a + 1 : a + 2) : 2 + a) * kAtom64;
  };
  constexpr uint32_t kQLbo = VK ? 2 * kAtom64 : kAtom64;  // distance between Q's (and dO_K's) two atoms
  auto slot_stats = [&](int s) { return sSlots + s * C::SLOT + C::SLOT_T; };  // shared address

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(BAR_KV, 1);
    for (int s = 0; s < NQS; ++s) {
      mbar_init(BAR_QFULL(s), 1);
      mbar_init(BAR_QEMPTY(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR_SPFULL(b), 1);
      mbar_init(BAR_PDSFULL(b), 64 * NWG);
      if (FQ) mbar_init(BAR_DQFREE(b), 64 * NWG);
      if (FQ) mbar_init(BAR_DQDONE(b), 1);
    }
    mbar_init(BAR_DONE, 1);
    mbar_init(BAR_FIN, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_base_sh), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (whole warp)
    int armed[NQS];
    for (int s = 0; s < NQS; ++s) armed[s] = 0;
    if (lane == 0) {
      prefetch_tmap(&p.tm_a);
      prefetch_tmap(&p.tm_c);
      prefetch_tmap(&p.tm_d);
      mbar_expect_tx(BAR_KV, C::RES);
      tma_load(sRes, &p.tm_a, 0, k0, bx, BAR_KV);
      tma_load(sRes + kAtom128, p.k_hi_x ? &p.tm_b : &p.tm_a, p.k_hi_x ? 0 : 64, k0, bx, BAR_KV);
      for (int a = 0; a < XA; ++a) tma_load(sRes + (2 + a) * kAtom128, &p.tm_b, 64 * a, k0, bx, BAR_KV);
    }
    for (int i = 0; i < nq; ++i) {
      const int s = i % NQS;
      if (i >= NQS &&
          !__all_sync(0xffffffffu, mbar_wait(BAR_QEMPTY(s), ((i / NQS) - 1) & 1, abort, &g_bwd_err, 1)))
        break;
      if (lane == 0) {
        const int q0 = qtile(i) * 64;
        mbar_expect_tx(BAR_QFULL(s), C::SLOT_T + 3 * 256);
        tma_load(q_atom(s, 0), &p.tm_c, 0, q0, bx, BAR_QFULL(s));
        tma_load(q_atom(s, 1), &p.tm_c, 64, q0, bx, BAR_QFULL(s));
        for (int a = 0; a < C::DW / 64; ++a) tma_load(do_atom(s, a), &p.tm_d, 64 * a, q0, bx, BAR_QFULL(s));
        // the 64 queries' folded statistics: one 256-byte copy per plane (rows padded to 128)
        const int64_t r0 = (int64_t)bi * p.n_pad + q0;
        bulk_load(slot_stats(s), p.nl + r0, 256, BAR_QFULL(s));
        bulk_load(slot_stats(s) + 256, p.nc + r0, 256, BAR_QFULL(s));
        bulk_load(slot_stats(s) + 512, p.ng + r0, 256, BAR_QFULL(s));
        // bring the tile NQS loads ahead into L2: a slot is reloaded only ~NQS - 2 tiles before
        // its use, less than a DRAM round trip under this kernel's load
        if (i + NQS < nq) {
          const int qa = qtile(i + NQS) * 64;
          tma_prefetch(&p.tm_c, 0, qa, bx);
          tma_prefetch(&p.tm_c, 64, qa, bx);
          for (int a = 0; a < C::DW / 64; ++a) tma_prefetch(&p.tm_d, 64 * a, qa, bx);
        }
        if (p.acc == 3 && i == nq - 1) {  // the accumulator tiles the epilogue reads, into L2
          for (int c = 0; c < 4; ++c) {
            tma_prefetch(&p.tm_f0, 32 * c, k0, bx);
            if (C::HAS_DV) tma_prefetch(&p.tm_f1, 32 * c, k0, bx);
          }
        }
      }
      armed[s] = i / NQS + 1;
    }
    if (lane == 0) {
      mbar_wait_drain(BAR_KV, 0);
      for (int s = 0; s < NQS; ++s)
        if (armed[s] > 0) mbar_wait_drain(BAR_QFULL(s), (armed[s] - 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // TMEM buffer b = query tile parity: S^T [128b, 128b+64), dP^T [128b+64, 128b+128); P^T and
    // dS^T (bf16) are written over the first 32 columns of S^T / dP^T. dK [256,384), dV [384,512).
    // The whole warp walks the schedule with warp-uniform waits; one elected lane issues.
    const uint32_t leader = elect_one() ? 1u : 0u;  // the lane that issues (warp converged here)
    auto wwait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_bwd_err, code));
    };
    {
      bool ok = wwait(BAR_KV, 0, 2);
      auto issue_sp = [&](int i) -> bool {
        const int s = i % NQS;
        if (!wwait(BAR_QFULL(s), (i / NQS) & 1, 2)) return false;
        tc_fence_after();
        {
          const uint32_t tb = tmem + 128 * (i & 1);
          int kd0 = 0;  // first step of dP^T = W dO^T still to issue (16 columns of W per step)
          if (VK && !qtail(i)) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {  // [S^T | dP^T] = K [Q | dO_K]^T over D: columns [0, 128) of the buffer
              const uint32_t offa = (kk >> 2) * kAtom128 + (kk & 3) * 32;
              mma_ss_if(leader, tb, smem_desc_sw128(sRes + offa, 16, 1024),
                        smem_desc_sw128(q_atom(s, kk >> 2) + (kk & 3) * 32, 16, 1024), IDESC_SPK, kk > 0);
            }
            kd0 = 8;
          } else {
            const uint32_t idesc = qtail(i) ? IDESC_SP32 : IDESC_SP;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {  // S^T = K Q^T over D
              const uint32_t offa = (kk >> 2) * kAtom128 + (kk & 3) * 32;
              mma_ss_if(leader, tb, smem_desc_sw128(sRes + offa, 16, 1024),
                        smem_desc_sw128(q_atom(s, kk >> 2) + (kk & 3) * 32, 16, 1024), idesc, kk > 0);
            }
          }
          const uint32_t idesc = qtail(i) ? IDESC_SP32 : IDESC_SP;
#pragma unroll
          for (int kk = 0; kk < C::DW / 16; ++kk) {  // dP^T (+)= W dO^T over the rest of DW
            if (kk < kd0) continue;
            const uint32_t offa = (kk >> 2) * kAtom128 + (kk & 3) * 32;
            mma_ss_if(leader, tb + 64, smem_desc_sw128(sW + offa, 16, 1024),
                      smem_desc_sw128(do_atom(s, kk >> 2) + (kk & 3) * 32, 16, 1024), idesc, kk > 0 ? 1u : 0u);
          }
          mma_commit_if(leader, BAR_SPFULL(i & 1));
        }
        return true;
      };
      if (ok) ok = issue_sp(0);
      if (ok && nq > 1) ok = issue_sp(1);
      for (int i = 0; ok && i < nq; ++i) {
        if (!wwait(BAR_PDSFULL(i & 1), (i >> 1) & 1, 4)) break;
        tc_fence_after();
        const int s = i % NQS;
        {
          const uint32_t pt = tmem + 128 * (i & 1), dst = pt + 64;
          const bool tail = qtail(i);
          const uint32_t qmask = tail ? 0x3u : 0xfu;  // 16-query steps of the tile
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // dK += dS^T Q   (K = 64 queries)
            mma_ts_if(leader & ((qmask >> kk) & 1u), tmem + 256, dst + pcol(kk),
                      smem_desc_sw128(q_atom(s, 0) + kk * 2048, kQLbo, 1024), IDESC_ACC, (i > 0 || kk > 0) ? 1u : 0u);
          if (VK) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // dK += P^T dO[:, :128]  (value gradient of the K columns)
              mma_ts_if(leader & ((qmask >> kk) & 1u), tmem + 256, pt + pcol(kk),
                        smem_desc_sw128(do_atom(s, 0) + kk * 2048, kQLbo, 1024), IDESC_ACC, 1u);
          }
          if (C::HAS_DV) {
            const uint32_t vb = do_atom(s, VK ? 2 : 0);  // the value columns of dO (contiguous atoms)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // dV += P^T dO[:, cols]
              mma_ts_if(leader & ((qmask >> kk) & 1u), tmem + 384, pt + pcol(kk),
                        smem_desc_sw128(vb + kk * 2048, kAtom64, 1024), IDESC_ACC, (i > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit_if(leader, BAR_QEMPTY(s));
          // the next S^T / dP^T of this buffer is issued after the MMAs that read its P^T / dS^T;
          // with fused dQ also ahead of dQ^T(i), which reads dS^T from shared memory, so the pipe
          // has that group's work while the stream drains dQ^T(i - 2)
          if (i + 2 < nq && !(ok = issue_sp(i + 2))) break;
          if (FQ) {
            // dQ^T = K^T dS^T over the 128 keys (A: the resident K read M-major; B: the staged dS^T),
            // once the stream has drained the dQ^T of its previous tile from this buffer
            if (!wwait(BAR_DQFREE(i & 1), (i >> 1) & 1, 5)) break;
            tc_fence_after();
            const uint32_t dqt = tmem + 384 + 64 * (i & 1), sds = sDS + (i & 1) * kAtom128;
            const uint32_t idq = tail ? IDESC_DQ32 : IDESC_DQ;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_ss_if(leader, dqt, smem_desc_sw128(sRes + kk * 2048, kAtom128, 1024),
                        smem_desc_sw128(sds + kk * 2048, kAtom128, 1024), idq, kk > 0);
            mma_commit_if(leader, BAR_DQDONE(i & 1));
          }
        }
      }
      if (elect_one()) {
        mma_commit(BAR_DONE);
        mbar_wait_drain(BAR_DONE, 0);
      }
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------------- compute: thread = key row
    // stream st = tile parity (TMEM buffer st); with four warpgroups two share a stream and each
    // takes one 32-query half of every tile
    const int wg = (warp - 2) >> 2;
    const int stm = NWG == 4 ? wg >> 1 : wg;
    const int h0 = NWG == 4 ? (wg & 1) : 0, h1 = NWG == 4 ? h0 + 1 : 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    auto warp_wait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      const bool mine = mbar_wait(bar, parity, abort, &g_bwd_err, code);
      return __all_sync(0xffffffffu, mine);
    };
    const uint32_t ts = tmem + lane_off + 128 * stm, tdp = ts + 64;
    // fused dQ: reduce-add this warpgroup's 32 queries of dQ^T(j) (thread = head-dim row) into dQ
    auto drain_dq = [&](int j) {
      uint32_t v[32];
      tmem_ld32(tmem + lane_off + 384 + 64 * (j & 1) + 32 * h0, v);
      tmem_wait_ld();
      const int q0 = qtile(j) * 64 + 32 * h0;
      // dQ is plain here (the host fuses only a dense [batch][n_q][128] dQ): batch stride dq_bs,
      // rows of 128 floats, so the 32 reductions take immediate offsets
      float* dst = p.dq + (int64_t)bi * p.dq_bs + (int64_t)q0 * 128 + row;
      const int nv = min(32, p.n_q - q0);
#pragma unroll
      for (int c = 0; c < 32; ++c)
        if (c < nv) red_add_f32(dst + c * 128, __uint_as_float(v[c]));
    };
    bool ok = true;
    for (int i = stm; i < nq; i += 2) {
      const int s = i % NQS;
      if (!warp_wait(BAR_SPFULL(stm), (i >> 1) & 1, 8)) { ok = false; break; }
      if (!warp_wait(BAR_QFULL(s), (i / NQS) & 1, 8)) { ok = false; break; }
      // fused dQ: dQ^T(i - 2) has finished reading this stream's dS^T staging (and may be drained)
      if (FQ && i >= 2 && !warp_wait(BAR_DQDONE(stm), ((i >> 1) - 1) & 1, 8)) { ok = false; break; }
      tc_fence_after();
      const uint32_t st = slot_stats(s);
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), sm2 = make_float2(p.sm_scale, p.sm_scale);
      // dS^T for the dQ GEMM (four warpgroups): the two 16-query chunks of this warpgroup's half
      // are 64 contiguous bytes of the key's row, held here and stored after the tile is handed
      // to the MMA warp, off the TMEM load -> exponentials -> TMEM store chain
      uint32_t ds_hold[2][8];
      // 16-query chunks of this warpgroup's half(s): P^T / dS^T of chunk qc go to columns pcol(qc) of
      // S^T / dP^T, which lie inside what this warpgroup has already loaded
#pragma unroll 1
      for (int qc = 2 * h0; qc < 2 * h1; ++qc) {  // 16-query chunks: P^T / dS^T of chunk qc -> pcol(qc)
        uint32_t sv[16], dv[16];
        tmem_ld16(ts + 16 * qc, sv);
        tmem_ld16(tdp + 16 * qc, dv);
        tmem_wait_ld();
        uint32_t pk[8], dk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
          const uint32_t so = st + 4 * (16 * qc + e);
          float4 l4, c4, g4;
          asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(l4.x), "=f"(l4.y), "=f"(l4.z), "=f"(l4.w) : "r"(so));
          asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(c4.x), "=f"(c4.y), "=f"(c4.z), "=f"(c4.w) : "r"(so + 256));
          asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(g4.x), "=f"(g4.y), "=f"(g4.z), "=f"(g4.w) : "r"(so + 512));
          prob_dscore<T, true>(sv[e], sv[e + 1], dv[e], dv[e + 1], sc2, sm2, make_float2(l4.x, l4.y),
                               make_float2(c4.x, c4.y), make_float2(g4.x, g4.y), pk[e >> 1], dk[e >> 1]);
          prob_dscore<T, true>(sv[e + 2], sv[e + 3], dv[e + 2], dv[e + 3], sc2, sm2, make_float2(l4.z, l4.w),
                               make_float2(c4.z, c4.w), make_float2(g4.z, g4.w), pk[(e >> 1) + 1], dk[(e >> 1) + 1]);
        }
        tmem_st8(ts + pcol(qc), pk);
        tmem_st8(tdp + pcol(qc), dk);
        if (NWG == 4 && p.ds) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (qc & 1)
              ds_hold[1][e] = dk[e];
            else
              ds_hold[0][e] = dk[e];
          }
        } else if (p.ds) {  // dS^T row (key k0 + row), queries [64 qtile + 16 qc, +16) for the dQ GEMM
          uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(p.ds) + (int64_t)bi * p.ds_bs + (int64_t)(k0 + row) * p.ds_ld +
                                                qtile(i) * 64 + 16 * qc);
          dst[0] = make_uint4(dk[0], dk[1], dk[2], dk[3]);
          dst[1] = make_uint4(dk[4], dk[5], dk[6], dk[7]);
        }
        if (FQ) {  // dS^T row (key) `row`, queries [16qc, 16qc + 16): 16-byte chunks 2qc, 2qc + 1, swizzled
          const uint32_t rb = sDS + stm * kAtom128 + row * 128;
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rb + (((2 * qc) ^ (row & 7)) << 4)), "r"(dk[0]),
                       "r"(dk[1]), "r"(dk[2]), "r"(dk[3])
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rb + (((2 * qc + 1) ^ (row & 7)) << 4)),
                       "r"(dk[4]), "r"(dk[5]), "r"(dk[6]), "r"(dk[7])
                       : "memory");
        }
      }
      tmem_wait_st();
      if (FQ) fence_proxy_async_smem();  // dS^T is read by the dQ^T MMA (async proxy)
      tc_fence_before();
      mbar_arrive(BAR_PDSFULL(stm));
      if (NWG == 4 && p.ds) {  // dS^T row (key k0 + row), queries [64 qtile + 32 h0, +32)
        uint8_t* dst = reinterpret_cast<uint8_t*>(static_cast<T*>(p.ds) + (int64_t)bi * p.ds_bs +
                                                  (int64_t)(k0 + row) * p.ds_ld + qtile(i) * 64 + 32 * h0);
        st_global_v8(dst, ds_hold[0]);
        st_global_v8(dst + 32, ds_hold[1]);
      }
      if (FQ) {
        // while the MMA warp runs this tile's dK MMAs and S^T / dP^T(i + 2): drain dQ^T(i - 2)
        // (complete: DQDONE was waited for above); then its buffer may take dQ^T(i)
        if (i >= 2) drain_dq(i - 2);
        tc_fence_before();
        mbar_arrive(BAR_DQFREE(stm));
      }
    }
    if (ok) ok = warp_wait(BAR_DONE, 0, 8);
    tc_fence_after();
    if (FQ && ok) {  // the stream's last tile
      const int last = stm + 2 * ((nq - 1 - stm) >> 1);
      if (stm < nq) drain_dq(last);
    }
    // epilogue: stage dK (and dV) in the idle query slots, one thread writes them with TMA. The
    // warpgroups split the 32-column chunks: with dV, the first half of them stages dK, the second
    // dV; without, all stage dK. acc 3: the fp32 accumulator tiles are loaded into those slots
    // and the 16-bit sums staged in the idle resident K | X tiles.
    const uint32_t stage0 = sSlots, stage1 = sSlots + 65536;
    const bool fin = p.acc == 3;
    bool fin_issued = false;
    if (fin) {
      if (warp == 2 && lane == 0 && ok) {
        fin_issued = true;
        mbar_expect_tx(BAR_FIN, (C::HAS_DV ? 2 : 1) * 65536);
        for (int c = 0; c < 4; ++c) {
          tma_load(stage0 + c * 16384, &p.tm_f0, 32 * c, k0, bx, BAR_FIN);
          if (C::HAS_DV) tma_load(stage1 + c * 16384, &p.tm_f1, 32 * c, k0, bx, BAR_FIN);
        }
      }
      if (ok) ok = warp_wait(BAR_FIN, 0, 8);
    }
    if (ok && fin) {
      constexpr int CPW = C::HAS_DV ? 8 / NWG : 4 / NWG;
      const int mat = C::HAS_DV ? wg / (NWG / 2) : 0, c0 = C::HAS_DV ? CPW * (wg % (NWG / 2)) : CPW * wg;
      finalize_rows<T>(tmem + lane_off + 256 + 128 * mat, mat ? stage1 : stage0, sRes + mat * 32768, row, c0, c0 + CPW);
    } else if (ok) {
      if (C::HAS_DV) {
        constexpr int CPW = 8 / NWG;  // chunks per warpgroup
        const int mat = wg / (NWG / 2), c0 = CPW * (wg % (NWG / 2));
        if (mat == 0) stage_acc_rows<T>(tmem + lane_off + 256, stage0, row, p.acc, c0, c0 + CPW);
        else stage_acc_rows<T>(tmem + lane_off + 384, stage1, row, p.acc, c0, c0 + CPW);
      } else {
        constexpr int CPW = 4 / NWG;
        stage_acc_rows<T>(tmem + lane_off + 256, stage0, row, p.acc, CPW * wg, CPW * (wg + 1));
      }
    }
    fence_proxy_async_smem();
    ok = named_bar_and(1, 128 * NWG, ok);
    if (warp == 2 && lane == 0 && ok && !*abort) {
      if (!C::HAS_DV && p.k_hi_x)  // [dK | dV2] (never with acc 3)
        issue_grad_tile_split(&p.tm_g0, &p.tm_g1, stage0, k0, bx, p.acc);
      else
        issue_grad_tile(&p.tm_g0, fin ? sRes : stage0, k0, bx, fin ? 0 : p.acc);
      if (C::HAS_DV) issue_grad_tile(&p.tm_g1, fin ? sRes + 32768 : stage1, k0, bx, fin ? 0 : p.acc);
      tma_store_commit_and_wait();
    }
    if (fin_issued) mbar_wait_drain(BAR_FIN, 0);  // loads still in flight after a timeout
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ================================================================================ dQ kernel, 128-key tiles
// CTA = 128 queries; walks 128-key tiles, so every MMA is a full-rate 128 x 128 x 16 instruction.
// Both compute warpgroups work on the same tile: WG w owns keys [64w, 64w+64) of it.
//   S = Q K^T (SS), dP = dO W^T (SS, or TS with dO resident in TMEM when DW = 256), dS (bf16)
//   written over the first half of the warpgroup's own S columns, dQ += dS K (TS).
// DOT = false: TMEM S0 [0,128) S1 [128,256) dP [256,384) dQ [384,512); S double-buffered, so
//   S(j+2) is queued behind dQ(j) while dP(j+1) is issued as soon as tile j's dP has been read.
// DOT = true (DW = 256): TMEM S [0,128) dP [128,256) dO [256,384) dQ [384,512); dO is staged into
//   TMEM once by the compute threads (dP is a TS MMA). S is single-buffered, so dS goes to shared
//   memory (K-major, thread = query row) and dQ += dS K is an SS MMA: S(j+1) and dP(j+1) are
//   issued as soon as tile j's S and dP are in registers and run under the dS math of tile j.
//   dS(j) is written into the V2 slot of tile j, which dP(j) has finished reading; the slot is
//   released after dQ(j), so no tile waits for the previous tile's dQ.
// K and X (V, or V2 when V aliases K) stream through separate rings: X(j) is released after dP(j)
// (DOT: after dQ(j), whose dS it holds), K(j) after dQ(j).
template <int XA, bool VK, bool DOT, int NK, int NX>
struct DqCfg2 {
  static constexpr int DW = VK ? 128 + 64 * XA : 64 * XA;
  static constexpr int NS = DOT ? 1 : 2;
  static constexpr int RES = 2 * kAtom128 + (DOT ? 0 : (DW / 64) * kAtom128);  // Q | dO
  static constexpr int KSLOT = 2 * kAtom128;
  static constexpr int XSLOT = XA * kAtom128;
  static constexpr int SMEM = 1024 + RES + NK * KSLOT + NX * XSLOT;
  static_assert(NK * KSLOT >= 4 * 16384, "the dQ epilogue stages 64 KB in the K ring");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(!DOT || (DW == 256 && XA == 2), "dO in TMEM is laid out for DW = 256; dS fills a V2 slot");
  static_assert((XA == 0) == (NX == 0), "X ring present exactly when there is an X tile");
};

template <typename T, int XA, bool VK, bool DOT, int NK, int NX, int NWG>
__global__ void __launch_bounds__(64 + 128 * NWG, 1) fea_bwd_dq128_kernel(const __grid_constant__ Sm100BwdParams p) {
  using C = DqCfg2<XA, VK, DOT, NK, NX>;
  constexpr int NS = C::NS;
  constexpr int NXB = NX > 0 ? NX : 1;
  constexpr bool kBf16 = Elem<T>::is_bf16;
  constexpr uint32_t IDESC_S = idesc_f16(kBf16, 128, 128, false, false);
  constexpr uint32_t IDESC_S32 = idesc_f16(kBf16, 128, 32, false, false);  // a last key tile of <= 32 keys
  constexpr uint32_t IDESC_DQ = idesc_f16(kBf16, 128, 128, false, true);
  constexpr uint32_t T_DP = DOT ? 128 : 256, T_DO = 256, T_DQ = 384;
  constexpr int CW = 128 / NWG;          // key columns of a tile per compute warpgroup
  constexpr int NCT = 128 * NWG;         // compute threads
  constexpr int B_Q = 0, B_KFULL = 1, B_KEMPTY = B_KFULL + NK, B_XFULL = B_KEMPTY + NK, B_XEMPTY = B_XFULL + NXB;
  constexpr int B_SFULL = B_XEMPTY + NXB, B_DSFULL = B_SFULL + NS, B_DPFULL = B_DSFULL + NS;
  constexpr int B_DPFREE = B_DPFULL + 1, B_DOT = B_DPFREE + 1, B_DONE = B_DOT + 1, B_FIN = B_DONE + 1;
  constexpr int NBARS = B_FIN + 1;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[NBARS];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // block -> (sequence, query tile, key chunk); chunks of one query tile add their partial dQ
  const int per_seq = p.n_tiles * p.k_split;
  const int bi = blockIdx.x / per_seq;
  const BIdx bx = bidx(bi, p.n1, p.n2);
  const int q0 = ((blockIdx.x % per_seq) / p.k_split) * 128;
  const int kt0 = (blockIdx.x % p.k_split) * p.kt_per;  // first key tile of this chunk
  const int nk = min((p.n_kv + 127) / 128 - kt0, p.kt_per);  // >= 1 by the host's choice of split

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = sbase, sDO = sbase + 2 * kAtom128;
  const uint32_t sK = sbase + C::RES, sX = sK + NK * C::KSLOT;
  // DOT: dS [128 queries][128 keys] bf16 (two K-major atoms) of tile j in V2 slot j % NX
  auto sDS = [&](int j) { return sX + (uint32_t)(j % NXB) * C::XSLOT; };
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  volatile int* abort = &abort_sh;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(BAR(B_Q), 1);
    for (int s = 0; s < NK; ++s) {
      mbar_init(BAR(B_KFULL + s), 1);
      mbar_init(BAR(B_KEMPTY + s), 1);
    }
    for (int s = 0; s < NXB; ++s) {
      mbar_init(BAR(B_XFULL + s), 1);
      mbar_init(BAR(B_XEMPTY + s), 1);
    }
    for (int b = 0; b < NS; ++b) {
      mbar_init(BAR(B_SFULL + b), 1);
      mbar_init(BAR(B_DSFULL + b), NCT);
    }
    mbar_init(BAR(B_DPFULL), 1);
    mbar_init(BAR(B_DPFREE), NCT);
    mbar_init(BAR(B_DOT), NCT);
    mbar_init(BAR(B_DONE), 1);
    mbar_init(BAR(B_FIN), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_base_sh), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tm_a);
      prefetch_tmap(&p.tm_c);
      if (!DOT) prefetch_tmap(&p.tm_b);
      if (XA > 0) prefetch_tmap(&p.tm_d);
      mbar_expect_tx(BAR(B_Q), C::RES);
      tma_load(sQ, &p.tm_a, 0, q0, bx, BAR(B_Q));
      tma_load(sQ + kAtom128, &p.tm_a, 64, q0, bx, BAR(B_Q));
      if (!DOT)
        for (int a = 0; a < C::DW / 64; ++a) tma_load(sDO + a * kAtom128, &p.tm_b, 64 * a, q0, bx, BAR(B_Q));
      int karmed[NK], xarmed[NXB];
      for (int s = 0; s < NK; ++s) karmed[s] = 0;
      for (int s = 0; s < NXB; ++s) xarmed[s] = 0;
      for (int j = 0; j < nk; ++j) {
        const int s = j % NK;
        if (j >= NK && !mbar_wait(BAR(B_KEMPTY + s), ((j / NK) - 1) & 1, abort, &g_bwd_err, 16)) break;
        mbar_expect_tx(BAR(B_KFULL + s), C::KSLOT);
        const CUtensorMap* khi = p.k_hi_x ? &p.tm_d : &p.tm_c;  // [K | V2] tiles (k_hi_x)
        const int xhi = p.k_hi_x ? 0 : 64;
        tma_load(sK + s * C::KSLOT, &p.tm_c, 0, (kt0 + j) * 128, bx, BAR(B_KFULL + s));
        tma_load(sK + s * C::KSLOT + kAtom128, khi, xhi, (kt0 + j) * 128, bx, BAR(B_KFULL + s));
        if (j + NK < nk) {  // the K tile NK loads ahead into L2
          tma_prefetch(&p.tm_c, 0, (kt0 + j + NK) * 128, bx);
          tma_prefetch(khi, xhi, (kt0 + j + NK) * 128, bx);
        }
        if (p.acc == 3 && j == nk - 1)  // the accumulator tile the epilogue reads, into L2
          for (int c = 0; c < 4; ++c) tma_prefetch(&p.tm_f0, 32 * c, q0, bx);
        karmed[s] = j / NK + 1;
        if (XA > 0) {
          const int x = j % NXB;
          if (j >= NXB && !mbar_wait(BAR(B_XEMPTY + x), ((j / NXB) - 1) & 1, abort, &g_bwd_err, 16)) break;
          mbar_expect_tx(BAR(B_XFULL + x), C::XSLOT);
          for (int a = 0; a < XA; ++a)
            tma_load(sX + x * C::XSLOT + a * kAtom128, &p.tm_d, 64 * a, (kt0 + j) * 128, bx, BAR(B_XFULL + x));
          if (j + NXB < nk)
            for (int a = 0; a < XA; ++a) tma_prefetch(&p.tm_d, 64 * a, (kt0 + j + NXB) * 128, bx);
          xarmed[x] = j / NXB + 1;
        }
      }
      mbar_wait_drain(BAR(B_Q), 0);
      for (int s = 0; s < NK; ++s)
        if (karmed[s] > 0) mbar_wait_drain(BAR(B_KFULL + s), (karmed[s] - 1) & 1);
      if (XA > 0)
        for (int s = 0; s < NXB; ++s)
          if (xarmed[s] > 0) mbar_wait_drain(BAR(B_XFULL + s), (xarmed[s] - 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp walks the schedule with warp-uniform waits; one elected lane issues.
    const uint32_t leader = elect_one() ? 1u : 0u;  // the lane that issues (warp converged here)
    auto wwait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_bwd_err, code));
    };
    {
      bool ok = wwait(BAR(B_Q), 0, 32);
      if (DOT && ok) ok = wwait(BAR(B_DOT), 0, 32);
      // a last key tile of <= 32 keys: S and dP at N = 32, dQ over its first 32 keys only (the
      // scores of the other columns are stale TMEM and never reach an MMA)
      auto tail32 = [&](int j) { return p.n_kv - (kt0 + j) * 128 <= 32; };
      auto issue_s = [&](int j) -> bool {
        const int s = j % NK;
        if (!wwait(BAR(B_KFULL + s), (j / NK) & 1, 32)) return false;
        tc_fence_after();
        {
          const uint32_t kb = sK + s * C::KSLOT;
          const uint32_t d = tmem + 128u * (uint32_t)(j % NS);
          const uint32_t idesc = tail32(j) ? IDESC_S32 : IDESC_S;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kAtom128 + (kk & 3) * 32;
            mma_ss_if(leader, d, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), idesc, kk > 0);
          }
          mma_commit_if(leader, BAR(B_SFULL + j % NS));
        }
        return true;
      };
      auto issue_dp = [&](int j) -> bool {
        const int s = j % NK, x = j % NXB;
        if (VK && !wwait(BAR(B_KFULL + s), (j / NK) & 1, 32)) return false;
        if (XA > 0 && !wwait(BAR(B_XFULL + x), (j / NXB) & 1, 32)) return false;
        tc_fence_after();
        {
          const uint32_t kb = sK + s * C::KSLOT, xb = sX + x * C::XSLOT;
          const uint32_t idesc = tail32(j) ? IDESC_S32 : IDESC_S;
#pragma unroll
          for (int kk = 0; kk < C::DW / 16; ++kk) {
            uint32_t boff;
            if (VK) boff = kk < 8 ? kb + (kk >> 2) * kAtom128 + (kk & 3) * 32
                                  : xb + ((kk - 8) >> 2) * kAtom128 + ((kk - 8) & 3) * 32;
            else boff = xb + (kk >> 2) * kAtom128 + (kk & 3) * 32;
            const uint64_t bd = smem_desc_sw128(boff, 16, 1024);
            if (DOT)
              mma_ts_if(leader, tmem + T_DP, tmem + T_DO + kk * 8, bd, idesc, kk > 0);
            else
              mma_ss_if(leader, tmem + T_DP, smem_desc_sw128(sDO + (kk >> 2) * kAtom128 + (kk & 3) * 32, 16, 1024), bd, idesc,
                     kk > 0);
          }
          mma_commit_if(leader, BAR(B_DPFULL));
          if (XA > 0 && !DOT) mma_commit_if(leader, BAR(B_XEMPTY + x));  // DOT: after dQ (dS lives there)
        }
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok) ok = issue_dp(0);
      if (ok && NS == 2 && nk > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nk; ++j) {
        if (j + 1 < nk) {
          if (!wwait(BAR(B_DPFREE), j & 1, 64)) break;
          // DOT: tile j's S is in registers and its dS goes to shared memory, so S(j + 1) may be
          // written into the one S buffer now
          if (DOT && !issue_s(j + 1)) break;
          if (!issue_dp(j + 1)) break;
        }
        if (!wwait(BAR(B_DSFULL + j % NS), (j / NS) & 1, 64)) break;
        tc_fence_after();
        {
          const uint32_t kb = sK + (j % NK) * C::KSLOT;
          const uint32_t sb = tmem + 128u * (uint32_t)(j % NS);
          const uint32_t kmask = tail32(j) ? 0x3u : 0xffu;  // key steps (16 keys each) of the tile
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // dQ += dS K ; keys [16kk, 16kk+16) of warpgroup 16kk/CW
            const uint64_t bd = smem_desc_sw128(kb + kk * 2048, kAtom128, 1024);
            const uint32_t on = leader & ((kmask >> kk) & 1u);
            if (DOT) {
              const uint32_t a_sm = sDS(j) + (kk >> 2) * kAtom128 + (kk & 3) * 32;
              mma_ss_if(on, tmem + T_DQ, smem_desc_sw128(a_sm, 16, 1024), bd, IDESC_DQ, (j > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint32_t a_tm = sb + CW * (16 * kk / CW) + (16 * kk % CW) / 2;
              mma_ts_if(on, tmem + T_DQ, a_tm, bd, IDESC_DQ, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit_if(leader, BAR(B_KEMPTY + j % NK));
          if (DOT) mma_commit_if(leader, BAR(B_XEMPTY + j % NXB));  // V2 slot, then dS of tile j
        }
        const int nxt = j + NS;  // the next tile that uses this S buffer (DOT: issued above)
        if (!DOT && nxt < nk) ok = issue_s(nxt);
      }
      if (elect_one()) {
        mma_commit(BAR(B_DONE));
        mbar_wait_drain(BAR(B_DONE), 0);
      }
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------------- compute: thread = query row
    const int wg = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int q = q0 + row;
    const bool qok = q < p.n_q;
    const int64_t fidx = (int64_t)bi * p.n_pad + q;  // q < n_pad (rows padded to 128)
    const float fl = p.nl[fidx], fc = p.nc[fidx], fg = p.ng[fidx];
    const float2 nl2 = make_float2(fl, fl), nc2 = make_float2(fc, fc), ng2 = make_float2(fg, fg);
    const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), sm2 = make_float2(p.sm_scale, p.sm_scale);
    auto warp_wait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      const bool mine = mbar_wait(bar, parity, abort, &g_bwd_err, code);
      return __all_sync(0xffffffffu, mine);
    };
    bool ok = true;
    if (DOT) {
      // dO row -> TMEM (bf16 pairs): warpgroup w stages elements [EW w, EW w + EW)
      constexpr int EW = C::DW / NWG;  // elements per warpgroup (EW / 2 TMEM columns)
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(p.dout) +
                                                        view_offset(p.dov, p.n1, p.n2, bi, qok ? q : 0) + EW * wg);
#pragma unroll
      for (int h = 0; h < EW / 64; ++h) {
        uint32_t w32[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 v = qok ? src[8 * h + i] : make_uint4(0, 0, 0, 0);
          w32[4 * i] = v.x;
          w32[4 * i + 1] = v.y;
          w32[4 * i + 2] = v.z;
          w32[4 * i + 3] = v.w;
        }
        tmem_st32(tmem + lane_off + T_DO + EW / 2 * wg + 32 * h, w32);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR(B_DOT));
    }
    for (int j = 0; j < nk; ++j) {
      const int b = j % NS;
      if (!warp_wait(BAR(B_SFULL + b), (j / NS) & 1, 128)) { ok = false; break; }
      if (!warp_wait(BAR(B_DPFULL), j & 1, 128)) { ok = false; break; }
      tc_fence_after();
      const uint32_t ts = tmem + lane_off + 128u * (uint32_t)b + CW * wg;
      const uint32_t tdp = tmem + lane_off + T_DP + CW * wg;
      uint32_t sv[CW], dv[CW];
#pragma unroll
      for (int c = 0; c < CW / 32; ++c) {
        tmem_ld32(ts + 32 * c, sv + 32 * c);
        tmem_ld32(tdp + 32 * c, dv + 32 * c);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(BAR(B_DPFREE));
      uint32_t pk[CW / 2];
#pragma unroll
      for (int e = 0; e < CW; e += 2) {
        uint32_t unused;
        prob_dscore<T, false>(sv[e], sv[e + 1], dv[e], dv[e + 1], sc2, sm2, nl2, nc2, ng2, unused, pk[e >> 1]);
      }
      if (DOT) {
        // dS row `row`, keys [CW wg, CW wg + CW) -> K-major atom (CW wg) / 64, 16-byte chunks from
        // ((CW wg) % 64) / 8, swizzled, into tile j's V2 slot (dP(j), its reader, has completed)
        const uint32_t rb = sDS(j) + ((CW * wg) >> 6) * kAtom128 + row * 128;
        const int c0 = ((CW * wg) & 63) >> 3;
#pragma unroll
        for (int t = 0; t < CW / 8; ++t)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rb + (((c0 + t) ^ (row & 7)) << 4)),
                       "r"(pk[4 * t]), "r"(pk[4 * t + 1]), "r"(pk[4 * t + 2]), "r"(pk[4 * t + 3])
                       : "memory");
        fence_proxy_async_smem();  // read by the dQ MMA (async proxy)
      } else {
        if (CW == 64) tmem_st32(ts, pk);
        else tmem_st16(ts, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(BAR(B_DSFULL + b));
    }
    if (ok) ok = warp_wait(BAR(B_DONE), 0, 128);
    tc_fence_after();
    // epilogue: stage dQ in the idle K ring (WG w: columns [CW w, CW w + CW)), one thread writes it.
    // acc 3: the fp32 accumulator tile is loaded into the K ring and the 16-bit sum staged in the
    // idle Q tile.
    const bool fin = p.acc == 3;
    bool fin_issued = false;
    if (fin) {
      if (warp == 2 && lane == 0 && ok) {
        fin_issued = true;
        mbar_expect_tx(BAR(B_FIN), 65536);
        for (int c = 0; c < 4; ++c) tma_load(sK + c * 16384, &p.tm_f0, 32 * c, q0, bx, BAR(B_FIN));
      }
      if (ok) ok = warp_wait(BAR(B_FIN), 0, 128);
      if (ok) finalize_rows<T>(tmem + lane_off + T_DQ, sK, sQ, row, (CW / 32) * wg, (CW / 32) * (wg + 1));
    } else if (ok) {
      stage_acc_rows<T>(tmem + lane_off + T_DQ, sK, row, p.acc != 0, (CW / 32) * wg, (CW / 32) * (wg + 1));
    }
    fence_proxy_async_smem();
    ok = named_bar_and(1, NCT, ok);
    if (warp == 2 && lane == 0 && ok && !*abort) {
      // a split key range writes its partial tile into its own slice: sequence index chunk * batch + bi
      issue_grad_tile(&p.tm_g0, fin ? sQ : sK, q0, p.k_split > 1 ? BIdx((kt0 / p.kt_per) * p.n_seq + bi) : bx,
                      fin ? 0 : p.acc);
      tma_store_commit_and_wait();
    }
    if (fin_issued) mbar_wait_drain(BAR(B_FIN), 0);  // loads still in flight after a timeout
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// dq[bi][q] (+)= sum over chunks c (in order) of part[c][bi][q]: the split key ranges' partial tiles
// (added into dq, or written over it in the store mode)
__global__ void dq_split_reduce_kernel(const float* part, int split, int64_t batch, int64_t n_pad, int n_q, float* dq,
                                       View dqv, int n1, int n2, int store, int c4n) {
  const int64_t total = batch * n_q * 32;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bi = idx / ((int64_t)n_q * 32), rem = idx % ((int64_t)n_q * 32);
    const int64_t q = rem / 32, c4 = rem % 32;
    if (c4 >= c4n) continue;  // columns past d (d = 64)
    float4* dst = reinterpret_cast<float4*>(dq + view_offset(dqv, n1, n2, bi, q)) + c4;
    float4 acc = store ? make_float4(0.f, 0.f, 0.f, 0.f) : *dst;
    for (int c = 0; c < split; ++c) {
      const float4 v = reinterpret_cast<const float4*>(part + (((int64_t)c * batch + bi) * n_pad + q) * 128)[c4];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    *dst = acc;
  }
}

// out16[bi][q] = 16-bit(fin[bi][q] + sum over chunks c (in order) of part[c][bi][q]) (acc 3)
template <typename T>
__global__ void dq_split_finalize_kernel(const float* part, int split, int64_t batch, int64_t n_pad, int n_q,
                                         const float* fin, View finv, T* out, View outv, int n1, int n2, int c4n) {
  const int64_t total = batch * n_q * 32;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bi = idx / ((int64_t)n_q * 32), rem = idx % ((int64_t)n_q * 32);
    const int64_t q = rem / 32, c4 = rem % 32;
    if (c4 >= c4n) continue;  // columns past d (d = 64)
    float4 acc = reinterpret_cast<const float4*>(fin + view_offset(finv, n1, n2, bi, q))[c4];
    for (int c = 0; c < split; ++c) {
      const float4 v = reinterpret_cast<const float4*>(part + (((int64_t)c * batch + bi) * n_pad + q) * 128)[c4];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    uint2 w;
    w.x = Elem<T>::pack(acc.x, acc.y);
    w.y = Elem<T>::pack(acc.z, acc.w);
    reinterpret_cast<uint2*>(out + view_offset(outv, n1, n2, bi, q))[c4] = w;
  }
}

// ================================================================================ dQ = dS K
// CTA = 128 queries of one sequence; streams the dS^T rows (keys) the dK/dV kernel stored and the
// K tile, 64 keys per stage: dQ += dS K with A = dS read M-major from the dS^T rows and B = K
// read N-major (M = N = 128, 4 MMAs of 16 keys per stage). HBM-bound (dS is read once); the
// epilogue writes dQ like the dq kernel (16-bit store, fp32 reduce-add or store). Three stages
// (96 KB) hold the epilogue's fp32 tile and keep two CTAs per SM, so one CTA's epilogue and
// pipeline fill overlap the other's stream of dS.
constexpr int kGemmStages = 3;
constexpr int kGemmStage = 4 * kAtom64;  // dS^T 2 atoms (64 queries x 64 keys) | K 2 atoms (64 d x 64 keys)

template <typename T, int NS>
__global__ void __launch_bounds__(192, NS <= 3 ? 2 : 1) dq_from_ds_kernel(const __grid_constant__ Sm100BwdParams p) {
  constexpr bool kBf16 = Elem<T>::is_bf16;
  constexpr uint32_t IDESC = idesc_f16(kBf16, 128, 128, true, true);
  static_assert(NS >= 3, "the epilogue stages 96 KB in the pipeline stages");
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * NS + 2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bi = blockIdx.x / p.n_tiles;
  const BIdx bx = bidx(bi, p.n1, p.n2);
  const int q0 = (blockIdx.x % p.n_tiles) * 128;
  const int nkc = (p.n_kv + 63) / 64;
  const uint32_t BAR_FIN_OFF = 8u * (2 * NS + 1);
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  auto stage = [&](int s) { return sbase + (uint32_t)s * kGemmStage; };
  const uint32_t bar0 = smem_u32(bars);
  auto BAR_FULL = [&](int s) { return bar0 + 8u * s; };
  auto BAR_EMPTY = [&](int s) { return bar0 + 8u * (NS + s); };
  const uint32_t BAR_DONE = bar0 + 8u * (2 * NS);
  volatile int* abort = &abort_sh;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(BAR_FULL(s), 1);
      mbar_init(BAR_EMPTY(s), 1);
    }
    mbar_init(BAR_DONE, 1);
    mbar_init(bar0 + BAR_FIN_OFF, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_base_sh), 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&p.tm_a);
      prefetch_tmap(&p.tm_c);
      int armed[NS];
      for (int s = 0; s < NS; ++s) armed[s] = 0;
      for (int c = 0; c < nkc; ++c) {
        const int s = c % NS;
        if (c >= NS && !mbar_wait(BAR_EMPTY(s), ((c / NS) - 1) & 1, abort, &g_bwd_err, 64)) break;
        mbar_expect_tx(BAR_FULL(s), kGemmStage);
        for (int a = 0; a < 2; ++a) {
          tma_load(stage(s) + a * kAtom64, &p.tm_a, q0 + 64 * a, 64 * c, bi, BAR_FULL(s));
          tma_load(stage(s) + (2 + a) * kAtom64, &p.tm_c, 64 * a, 64 * c, bx, BAR_FULL(s));
        }
        armed[s] = c / NS + 1;
        if (p.acc == 3 && c == nkc - 1)  // the accumulator tile the epilogue reads, into L2
          for (int x = 0; x < 4; ++x) tma_prefetch(&p.tm_f0, 32 * x, q0, bx);
      }
      for (int s = 0; s < NS; ++s)
        if (armed[s] > 0) mbar_wait_drain(BAR_FULL(s), (armed[s] - 1) & 1);
    }
  } else if (warp == 1) {
    const uint32_t leader = elect_one() ? 1u : 0u;
    bool ok = true;
    for (int c = 0; c < nkc; ++c) {
      const int s = c % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(BAR_FULL(s), (c / NS) & 1, abort, &g_bwd_err, 64))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_ss_if(leader, tmem, smem_desc_sw128(stage(s) + kk * 2048, kAtom64, 1024),
                  smem_desc_sw128(stage(s) + 2 * kAtom64 + kk * 2048, kAtom64, 1024), IDESC, (c > 0 || kk > 0) ? 1u : 0u);
      mma_commit_if(leader, BAR_EMPTY(s));
    }
    (void)ok;
    if (elect_one()) {
      mma_commit(BAR_DONE);
      mbar_wait_drain(BAR_DONE, 0);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3, row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    bool ok = __all_sync(0xffffffffu, mbar_wait(BAR_DONE, 0, abort, &g_bwd_err, 64));
    tc_fence_after();
    const uint32_t st = stage(0), out16 = stage(2);  // every stage is idle once DONE
    const bool fin = p.acc == 3;  // 16-bit dQ = fp32 accumulator tile + this call's dQ
    bool fin_issued = false;
    if (fin) {
      const uint32_t bfin = bar0 + BAR_FIN_OFF;
      if (warp == 2 && lane == 0 && ok) {
        fin_issued = true;
        mbar_expect_tx(bfin, 65536);
        for (int x = 0; x < 4; ++x) tma_load(st + x * 16384, &p.tm_f0, 32 * x, q0, bx, bfin);
      }
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bfin, 0, abort, &g_bwd_err, 64));
      if (ok) finalize_rows<T>(tmem + lane_off, st, out16, row, 0, 4);
    } else if (ok) {
      stage_acc_rows<T>(tmem + lane_off, st, row, p.acc != 0, 0, 4);
    }
    fence_proxy_async_smem();
    ok = named_bar_and(1, 128, ok);
    if (warp == 2 && lane == 0 && ok && !*abort) {
      issue_grad_tile(&p.tm_g0, fin ? out16 : st, q0, bx, fin ? 0 : p.acc);
      tma_store_commit_and_wait();
    }
    if (fin_issued) mbar_wait_drain(bar0 + BAR_FIN_OFF, 0);  // loads still in flight after a timeout
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ================================================================================ host side
template <typename Kern>
cudaError_t run(Kern kern, int smem, int64_t blocks, int threads, const Sm100BwdParams& p, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, threads, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_all(const BwdParams& b, int64_t batch, int dv, bool vk, cudaStream_t st) {
  const bool bf16 = Elem<T>::is_bf16;
  // d = 64 with V aliasing K: the K tiles are [K | V2] (dv = 128, k_hi_x) or [K | 0] (dv = 64), so
  // the kernels of V aliasing a 128-wide K run with no value atoms of their own
  const bool vk64 = vk && b.d == 64;
  const bool k_hi_x = vk64 && dv == 128;
  if (k_hi_x && (b.acc_kv == 3 || b.acc_q == 3)) return cudaErrorNotSupported;  // no [dK | dV2] finalize
  const int xa = vk ? (vk64 ? 0 : (dv - 128) / 64) : dv / 64;  // value atoms beyond K (vk) or V atoms
  const void* xsrc = vk ? b.v2 : b.v;
  const View xv = vk ? b.v2v : b.vv;
  const int n1 = b.n1, n2 = b.n2;
  // ---- dK / dV: 64-query tiles (two warpgroups on alternate tiles, double-buffered S^T / dP^T)
  const int qrows = 64;
  Sm100BwdParams pa{};
  pa.n1 = n1;
  pa.n2 = n2;
  // d = 64 (keys, queries and dQ / dK 64 wide): the maps are 64 columns wide, so the kernels' second
  // 64-column atom loads as zeros and stores nothing (the contraction over 128 columns is exact)
  const int d = b.d;
  if (!tma::make_map_view(&pa.tm_a, b.k, bf16, d, b.n_kv, batch, b.kv, n1, n2, 128)) return cudaErrorInvalidValue;
  if (xa > 0) {
    if (!tma::make_map_view(&pa.tm_b, xsrc, bf16, 64 * xa, b.n_kv, batch, xv, n1, n2, 128)) return cudaErrorInvalidValue;
  } else if (k_hi_x) {  // V2: the second atom of the resident K tile
    if (!tma::make_map_view(&pa.tm_b, b.v2, bf16, 64, b.n_kv, batch, b.v2v, n1, n2, 128)) return cudaErrorInvalidValue;
  } else {
    pa.tm_b = pa.tm_a;
  }
  pa.k_hi_x = k_hi_x ? 1 : 0;
  if (!tma::make_map_view(&pa.tm_c, b.q, bf16, d, b.n_q, batch, b.qv, n1, n2, qrows)) return cudaErrorInvalidValue;
  if (!tma::make_map_view(&pa.tm_d, b.dout, bf16, dv, b.n_q, batch, b.dov, n1, n2, qrows)) return cudaErrorInvalidValue;
  pa.nl = b.fold;
  pa.nc = b.fold + batch * b.n_pad;
  pa.ng = b.fold + 2 * batch * b.n_pad;
  pa.n_pad = b.n_pad;
  // gradient maps: dK, and dV (or dV2 when V aliases K) when the kernel has a value accumulator
  auto grad_map = [&](CUtensorMap* m, void* base, int64_t cols, int64_t rows, const View& v, bool f32) {
    return f32 ? tma::make_map_view_f32(m, base, cols, rows, batch, v, n1, n2, 128)
               : tma::make_map_view(m, base, bf16, cols, rows, batch, v, n1, n2, 128);
  };
  const int xcols = vk ? dv - 128 : dv;  // columns of the value gradient the kernel writes
  const bool f32_kv = b.acc_kv == 1 || b.acc_kv == 2;  // acc 3 writes 16-bit values
  if (!grad_map(&pa.tm_g0, b.dk, d, b.n_kv, b.dkv, f32_kv)) return cudaErrorInvalidValue;
  if (xa > 0 && !grad_map(&pa.tm_g1, vk ? b.dv2 : b.dv, xcols, b.n_kv, vk ? b.dv2v : b.dvv, f32_kv))
    return cudaErrorInvalidValue;
  if (k_hi_x && !grad_map(&pa.tm_g1, b.dv2, 64, b.n_kv, b.dv2v, f32_kv)) return cudaErrorInvalidValue;
  if (b.acc_kv == 3) {
    if (!tma::make_map_view_f32(&pa.tm_f0, b.fin_k, d, b.n_kv, batch, b.finkv, n1, n2, 128))
      return cudaErrorInvalidValue;
    if (xa > 0 && !tma::make_map_view_f32(&pa.tm_f1, vk ? b.fin_v2 : b.fin_v, xcols, b.n_kv, batch,
                                          vk ? b.finv2v : b.finvv, n1, n2, 128))
      return cudaErrorInvalidValue;
  }
  pa.n_q = b.n_q;
  pa.n_kv = b.n_kv;
  pa.n_tiles = (b.n_kv + 127) / 128;
  pa.acc = b.acc_kv;
  const bool ds_gemm = b.ds != nullptr && fea_bwd_ds_gemm(batch, b.n_q, b.n_kv, dv, vk, b.acc_q);
  if (ds_gemm) {
    pa.ds = b.ds;
    pa.ds_ld = (b.n_q + 63) / 64 * 64;
    pa.ds_bs = (int64_t)(b.n_kv + 127) / 128 * 128 * pa.ds_ld;
  }
  pa.scale_log2 = b.scale_log2;
  pa.sm_scale = b.sm_scale;
  cudaError_t e;
  const int64_t blocks_a = (int64_t)pa.n_tiles * batch;
  if (fea_bwd_fuses_dq(b.n_kv, d, dv, vk, b.acc_q, b.deterministic)) {
    // dQ comes from the dK kernel as reductions into fp32: clear it first in the overwrite mode
    if (b.acc_q == 2) {
      e = cudaMemset2DAsync(b.dq, b.dq_bs * 4, 0, (size_t)b.n_q * 128 * 4, batch, st);
      if (e != cudaSuccess) return e;
    }
    pa.dq = b.dq;
    pa.dq_bs = b.dq_bs;  // the host fuses only a uniform dQ view (one batch stride, rows of 128)
    return run(fea_bwd_dkdv_kernel<T, 0, true, 4, kDkdvWarpgroups, true>, DkdvCfg<0, true, 4, true>::SMEM, blocks_a,
               kDkdvThreads, pa, st);
  }
  if (vk && xa > 0) {
    e = run(fea_bwd_dkdv_kernel<T, 2, true, 3, kDkdvWarpgroups>, DkdvCfg<2, true, 3>::SMEM, blocks_a, kDkdvThreads, pa, st);
  } else if (vk) {
    e = run(fea_bwd_dkdv_kernel<T, 0, true, 5, kDkdvWarpgroups>, DkdvCfg<0, true, 5>::SMEM, blocks_a, kDkdvThreads, pa, st);
  } else {
    e = run(fea_bwd_dkdv_kernel<T, 2, false, 4, kDkdvWarpgroups>, DkdvCfg<2, false, 4>::SMEM, blocks_a, kDkdvThreads, pa, st);
  }
  if (e != cudaSuccess) return e;
  if (ds_gemm) {
    // ---- dQ = dS K from the dS^T rows the dK/dV kernel stored
    Sm100BwdParams pg{};
    if (!tma::make_map(&pg.tm_a, b.ds, bf16, pa.ds_ld, pa.ds_bs / pa.ds_ld, batch, pa.ds_bs, 64)) return cudaErrorInvalidValue;
    pg.n1 = n1;
    pg.n2 = n2;
    if (!tma::make_map_view(&pg.tm_c, b.k, bf16, d, b.n_kv, batch, b.kv, n1, n2, 64)) return cudaErrorInvalidValue;
    if (!grad_map(&pg.tm_g0, b.dq, d, b.n_q, b.dqv, b.acc_q == 1 || b.acc_q == 2)) return cudaErrorInvalidValue;
    if (b.acc_q == 3 && !tma::make_map_view_f32(&pg.tm_f0, b.fin_q, d, b.n_q, batch, b.finqv, n1, n2, 128))
      return cudaErrorInvalidValue;
    pg.n_q = b.n_q;
    pg.n_kv = b.n_kv;
    pg.n_tiles = (b.n_q + 127) / 128;
    pg.acc = b.acc_q;
    constexpr int smem = 1024 + kGemmStages * kGemmStage;
    return run(dq_from_ds_kernel<T, kGemmStages>, smem, (int64_t)pg.n_tiles * batch, 192, pg, st);
  }
  // ---- dQ: 128-key tiles (dO staged in TMEM when it is 256 wide)
  Sm100BwdParams pb{};
  pb.n1 = n1;
  pb.n2 = n2;
  if (!tma::make_map_view(&pb.tm_a, b.q, bf16, d, b.n_q, batch, b.qv, n1, n2, 128)) return cudaErrorInvalidValue;
  if (!tma::make_map_view(&pb.tm_b, b.dout, bf16, dv, b.n_q, batch, b.dov, n1, n2, 128)) return cudaErrorInvalidValue;
  if (!tma::make_map_view(&pb.tm_c, b.k, bf16, d, b.n_kv, batch, b.kv, n1, n2, 128)) return cudaErrorInvalidValue;
  if (xa > 0) {
    if (!tma::make_map_view(&pb.tm_d, xsrc, bf16, 64 * xa, b.n_kv, batch, xv, n1, n2, 128)) return cudaErrorInvalidValue;
  } else if (k_hi_x) {  // V2: the second atom of every K tile
    if (!tma::make_map_view(&pb.tm_d, b.v2, bf16, 64, b.n_kv, batch, b.v2v, n1, n2, 128)) return cudaErrorInvalidValue;
  } else {
    pb.tm_d = pb.tm_c;
  }
  pb.k_hi_x = k_hi_x ? 1 : 0;
  pb.dout = b.dout;
  pb.dov = b.dov;
  pb.nl = b.fold;
  pb.nc = b.fold + batch * b.n_pad;
  pb.ng = b.fold + 2 * batch * b.n_pad;
  pb.n_pad = b.n_pad;
  pb.n_seq = (int)batch;
  {
    const int nkt = (b.n_kv + 127) / 128;
    pb.k_split = fea_bwd_dq_split(batch, b.n_q, b.n_kv, b.acc_q != 0);
    pb.kt_per = (nkt + pb.k_split - 1) / pb.k_split;
  }
  if (pb.k_split > 1) {
    // each key chunk stores its partial dQ tile into slice [chunk][batch] of the workspace; a
    // fixed-order sum adds them into dQ afterwards (deterministic, unlike concurrent reduce-adds)
    if (!b.dq_part || !tma::make_map_f32(&pb.tm_g0, b.dq_part, 128, b.n_pad, (int64_t)pb.k_split * batch,
                                         b.n_pad * 128, 128))
      return cudaErrorInvalidValue;
  } else {
    if (!grad_map(&pb.tm_g0, b.dq, d, b.n_q, b.dqv, b.acc_q == 1 || b.acc_q == 2)) return cudaErrorInvalidValue;
    if (b.acc_q == 3 && !tma::make_map_view_f32(&pb.tm_f0, b.fin_q, d, b.n_q, batch, b.finqv, n1, n2, 128))
      return cudaErrorInvalidValue;
  }
  pb.n_q = b.n_q;
  pb.n_kv = b.n_kv;
  pb.n_tiles = (b.n_q + 127) / 128;
  pb.acc = pb.k_split > 1 ? 2 : b.acc_q;
  pb.scale_log2 = b.scale_log2;
  pb.sm_scale = b.sm_scale;
  const int64_t blocks_b = (int64_t)pb.n_tiles * pb.k_split * batch;
  if (vk && xa == 0)
    e = run(fea_bwd_dq128_kernel<T, 0, true, false, 5, 0, kDqWarpgroups>, DqCfg2<0, true, false, 5, 0>::SMEM, blocks_b,
            kDqThreads, pb, st);
  else if (vk)
    e = run(fea_bwd_dq128_kernel<T, 2, true, true, 3, 3, kDqWarpgroups>, DqCfg2<2, true, true, 3, 3>::SMEM, blocks_b,
            kDqThreads, pb, st);
  else
    e = run(fea_bwd_dq128_kernel<T, 2, false, false, 3, 2, kDqWarpgroups>, DqCfg2<2, false, false, 3, 2>::SMEM, blocks_b,
            kDqThreads, pb, st);
  if (e != cudaSuccess || pb.k_split == 1) return e;
  const int64_t total = batch * b.n_q * 32;  // threads: 32 per dQ row (lanes past d / 4 idle)
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  if (b.acc_q == 3)
    dq_split_finalize_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(b.dq_part, pb.k_split, batch, b.n_pad, b.n_q, b.fin_q,
                                                                  b.finqv, reinterpret_cast<T*>(b.dq), b.dqv, n1, n2,
                                                                  d / 4);
  else
    dq_split_reduce_kernel<<<(unsigned)blocks, 256, 0, st>>>(b.dq_part, pb.k_split, batch, b.n_pad, b.n_q, b.dq,
                                                             b.dqv, n1, n2, b.acc_q == 2, d / 4);
  return cudaGetLastError();
}

}  // namespace

int fea_bwd_dq_split(int64_t batch, int n_q, int n_kv, bool acc) {
  // Split the key range when the query tiles alone fill the GPU poorly (few, long CTAs). Chosen
  // to minimise waves x (key tiles per CTA + ~3 tiles of fixed cost); only the fp32-accumulate
  // mode splits (its partial tiles are summed into the fp32 gradient).
  if (!acc || batch <= 0 || n_q <= 0) return 1;
  const int64_t n_tiles = (n_q + 127) / 128;
  const int nkt = (n_kv + 127) / 128;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  int best = 1;
  int64_t best_cost = 0;
  for (int ks = 1; ks <= 8; ++ks) {
    const int per = (nkt + ks - 1) / ks;
    if ((ks - 1) * per >= nkt) break;  // every chunk owns at least one key tile
    const int64_t waves = (n_tiles * batch * ks + sms - 1) / sms;
    const int64_t cost = waves * (per + 3);
    if (ks == 1 || cost * 100 < best_cost * 90) {  // a split must gain 10 % (merge pass)
      best = ks;
      best_cost = cost;
    }
  }
  return best;
}

bool fea_bwd_fuses_dq(int n_kv, int d, int dv, bool vk, int acc_q, bool deterministic) {
  // dQ from the dK kernel (no dq kernel) when V aliases a 128-wide K without V2 (free TMEM columns;
  // its reductions address dQ rows of 128), dQ is fp32 (reductions) and each dQ element receives at
  // most 32 of them (<= 32 key tiles)
  return vk && d == 128 && dv == 128 && (acc_q == 1 || acc_q == 2) && !deterministic && (n_kv + 127) / 128 <= 32;
}

bool fea_bwd_ds_gemm(int64_t batch, int n_q, int n_kv, int dv, bool vk, int acc_q) {
  // One HBM round trip of dS^T (stored by the dK/dV kernel, read by dq_from_ds) instead of a dq
  // kernel that recomputes S and dP. Taken for the last VMonarch R step (V aliasing K with a
  // 256-wide dP, short sequences) and for separate-V calls with few queries per sequence (the exact
  // recompute: n_q = r rows against the whole sequence), where the dq kernel's recomputation outweighs the
  // dS^T bytes (measured: last R-step backward 4.57 -> 4.10 ms, recompute backward 3.63 -> 3.28
  // ms). The first R step (V aliasing K, dv = 128) fuses dQ into the dK/dV kernel instead.
  // Separate V also needs enough query tiles to fill the GPU (two GEMM CTAs per SM): with few
  // sequences (strong scaling, small batches) the dq kernel's key-range split balances better.
  (void)acc_q;  // every write mode, the finalize mode included
  if (vk) return dv == 256 && (n_kv + 127) / 128 <= 32 && n_q <= 4096;
  if (dv != 128 || n_q > 4096) return false;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  return batch * ((n_q + 127) / 128) >= 2 * (int64_t)sms;
}

int64_t fea_bwd_ds_bytes(int64_t batch, int n_q, int n_kv) {
  return batch * ((int64_t)(n_kv + 127) / 128 * 128) * ((int64_t)(n_q + 63) / 64 * 64) * 2;
}

bool fea_bwd_sm100_supported(int d, int dv, int dv1, bool vk) {
  // d = 64, dv = 64 or 128: the 128-column kernels over 64-column maps of the 64-wide tensors
  // (zero second atom); with V aliasing K, V2 (dv = 128) is the K tiles' second atom
  if (d == 64) return vk ? dv1 == 64 && (dv == 64 || dv == 128) : (dv == 64 || dv == 128) && dv1 == dv;
  if (d != 128) return false;
  if (vk) return dv1 == 128 && (dv == 128 || dv == 256);
  return dv == 128 && dv1 == 128;
}

cudaError_t fea_bwd_sm100(const BwdParams& p, int64_t batch, int dv, bool vk, bool bf16, cudaStream_t st) {
  return bf16 ? launch_all<__nv_bfloat16>(p, batch, dv, vk, st) : launch_all<__half>(p, batch, dv, vk, st);
}

cudaError_t fea_bwd_sm100_status(cudaStream_t st, int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_bwd_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && *out) e = cudaMemcpyToSymbolAsync(g_bwd_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e;
}

}  // namespace vmb
