// FlashEntropyAttention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), D = 128.
//
// Reference semantics: video_monarch_attention/kernel.py:32-151 (online softmax with the running
// entropy accumulator h = sum p (x - m), E = (log2 l - h / l) ln 2, LSE2 = m + log2 l).
//
// CTA = one 128-row query tile of one sequence; 10 warps:
//   warp 0   TMA producer (Q once, then K / V tiles into an NSLOT-deep ring) + TMEM allocator
//   warp 1   MMA issuer (one elected lane of the converged warp): S = Q K^T into a double-buffered
//            TMEM S, O += P V with P read from TMEM (the bf16 probabilities are written over the
//            first 64 columns of S)
//   warps 2-9 softmax + epilogue, two warpgroups: thread = one query row (TMEM lane) x one half
//            (64 keys) of each 128-key tile; the half-row maxima are exchanged once per tile.
// TMEM (512 columns): S0 [0,128), S1 [128,256), O [256, 256 + NV).
// The max is rescaled lazily: O, l and h keep a stale reference max m_ref until a tile's scores
// pass it (a 64-key half's sum of p above 2^14 on full tiles, its max above m_ref + 8 on first and
// ragged tiles and with e4m3 P), the only point where O is read back and rescaled. The entropy
// identity E = log l - h / l holds for any reference, so this is exact.
//
// Shared-memory ring slot = [K tile (2 swizzle atoms of 128 keys x 64 cols)][X tile]:
//   separate V   : X = V (NV/64 atoms); P V reads the X atoms                 (plain FEA, recompute)
//   V aliases K  : X = V2 (0 or 2 atoms); P V reads K and V2 as one contiguous (VMonarch R steps,
//                  N = 128 + 64*XA operand, so the non-last R steps load K only vmonarch.py:50)
// Tails: TMA zero-fills rows past n_q / n_kv per sequence (3-D maps [batch][rows][cols]); keys
// past n_kv are masked to p = 0; the O tile is written with a TMA store, which clips rows >= n_q.
// e4m3 instances (template flag F8, the opt-in FP8 R step): q, k and X arrive as e4m3 (one 128-byte
// swizzle atom per 128 columns, so a D = 128 tile is one atom), both products are
// tcgen05.mma.kind::f8f6f4 (K = 32 per instruction) and P is packed to e4m3 in TMEM, four keys per
// column; the statistics use the unrounded p and O is written in the 16-bit type as usual.
//
// Every mbarrier wait is bounded (sm100.cuh); a CTA that gives up records an error code in
// g_fwd_err (read by vmb_device_status) and drains its in-flight copies and MMAs before freeing
// TMEM, so a fault in the pipeline ends the kernel instead of hanging the GPU.
#include "common.cuh"
#include "fea_params.h"
#include "launch.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace vmb {

__device__ int g_fwd_err;

namespace {

using namespace sm100;

constexpr int kThreads = 320;
constexpr int kAtom = 128 * 128;  // bytes of one swizzle atom column block: 128 rows x 128 B
constexpr float kRescaleThreshold = 8.0f;
// Full tiles after a stream's first, 16-bit P: the exponentials go against the current reference
// and are kept unless a 64-key half's sum of p exceeds this (64 x 2^8). The test costs one compare
// per half instead of a running max beside every pair of exponentials. Kept halves hold
// p <= 2^14 (inside bf16 and fp16, and the fp32 accumulators' relative precision does not depend
// on the scale); a row whose max passed the reference by more than kRescaleThreshold + 6 always
// fails it. e4m3 P (max 448) keeps the max test against kRescaleThreshold (p <= 2^8).
constexpr float kSumThreshold = 16384.0f;

struct Sm100FwdParams {
  CUtensorMap tm_q, tm_k, tm_x, tm_o;
  CUtensorMap tm_po;  // key-range split: partial O tiles [split * batch][n_pad][128] fp32 (32 x 128 boxes)
  float* lse;
  float* ent;
  float* pst;         // key-range split: partial (m, l, h) planes, each [split * batch * n_pad]
  int n_q, n_kv, n_qtiles;
  int kv_split, kt_per, n_seq;  // split count, key tiles per chunk, sequences of the call
  int n1, n2;                   // batch split of the q / k / v / o maps (fea_params.h View)
  long long wait_limit;         // pipeline wait limit in cycles (0: kWaitCycles); shortened by tests
  int hold_loads;               // test of the timeout path: the producers issue no load
  // d = 64 with V aliasing K and a second value tensor: the K tile's second atom is loaded from
  // tm_x (V2) at column 0, so the tile holds [K | V2]; Q's second atom is zero, so S = Q K^T is
  // unchanged and P V over the tile gives [P K | P V2]
  int k_hi_x;
  int64_t n_pad;      // n_q rounded up to 128
  float scale_log2;
};

template <int XA, bool VK, int NSLOT, bool F8 = false>
struct FwdCfg {
  static constexpr int NV = VK ? 128 + 64 * XA : 64 * XA;  // N of the P V MMA = output columns
  // swizzle atoms per 128-row tile of q / k (D = 128) and of X (64 XA columns): a 128-byte atom row
  // holds 64 16-bit or 128 e4m3 elements
  static constexpr int KA = F8 ? 1 : 2;
  static constexpr int XAT = F8 ? XA / 2 : XA;
  static constexpr int SLOT = (KA + XAT) * kAtom;          // bytes per ring slot
  static constexpr int PV_OFF = VK ? 0 : KA * kAtom;       // start of the P V operand in a slot
  static constexpr int Q_BYTES = KA * kAtom;
  static constexpr int SMEM = 1024 + Q_BYTES + NSLOT * SLOT;
  static_assert(NV == 128 || NV == 256, "P V width must be 128 or 256");
  static_assert(!F8 || (VK && XA % 2 == 0), "e4m3: V aliasing K, whole X atoms");
  static_assert(NSLOT * SLOT >= NV * 256, "the epilogue stages the 16-bit O tile in the ring");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// P of one 64-key segment into TMEM: 32 columns of 16-bit pairs, or 16 columns of e4m3 quads.
template <bool F8>
__device__ __forceinline__ void tmem_st_p(uint32_t taddr, const uint32_t* pk) {
  if constexpr (F8) tmem_st16(taddr, pk);
  else tmem_st32(taddr, pk);
}

// Three-input max (sm_100: one instruction).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Max of the raw scores of one row segment of N keys (keys >= valid ignored when MASK). The scale
// is applied to the max afterwards, as the reference does (kernel.py:45: max(qk) * qk_scale).
// Four independent chains of three-input maxima.
template <int N, bool MASK>
__device__ __forceinline__ float row_max_raw(const uint32_t (&sr)[N], int valid) {
  auto at = [&](int i) { return (MASK && i >= valid) ? -1e30f : __uint_as_float(sr[i]); };
  float mr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) mr[k] = fmax3(at(3 * k), at(3 * k + 1), at(3 * k + 2));
#pragma unroll
  for (int i = 12; i < N; i += 2) mr[(i >> 1) & 3] = fmax3(mr[(i >> 1) & 3], at(i), at(i + 1));
  return fmax3(fmaxf(mr[0], mr[1]), mr[2], mr[3]);
}

// p = 2^(s * scale - m) for one row segment of N keys, packed to the element type, with the row
// sum l and the entropy sum h = sum p (x - m). Pairs of keys go through the packed f32x2 FMA / add
// (one instruction per pair) into two chains each. Keys >= valid (MASK) get x - m = -1e30, so
// p = 0 and p (x - m) = 0 exactly. MAXO (unmasked segments): also returns the segment's max of
// s * scale (four chains of three-input maxima beside the exponentials), else -1e30.
// F8: p packed as e4m3, four keys per 32-bit word (p <= 2^8 under the lazy rescale, inside the
// format's range); l and h sum the unrounded p.
template <typename T, int N, bool ENT, bool MASK, bool MAXO = false, bool F8 = false>
__device__ __forceinline__ float probs_row(const uint32_t (&sr)[N], uint32_t (&pk)[F8 ? N / 4 : N / 2], float sc,
                                           float m, int valid, float& l, float& h) {
  static_assert(!MASK || !MAXO, "masked segments take a separate max");
  float2 la[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float2 ha[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float mr[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
  const float2 sc2 = make_float2(sc, sc), nm2 = make_float2(-m, -m);
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    if (MAXO) mr[i & 3] = fmax3(mr[i & 3], __uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1]));
    float2 d = __ffma2_rn(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sc2, nm2);
    if (MASK) {
      if (2 * i >= valid) d.x = -1e30f;
      if (2 * i + 1 >= valid) d.y = -1e30f;
    }
    const float2 pp = make_float2(fast_exp2(d.x), fast_exp2(d.y));
    la[i & 1] = __fadd2_rn(la[i & 1], pp);
    if (ENT) ha[i & 1] = __ffma2_rn(pp, d, ha[i & 1]);
    if constexpr (F8) {
      const uint32_t b2 = pack_e4m3x2(pp.x, pp.y);
      if (i & 1) pk[i >> 1] |= b2 << 16;
      else pk[i >> 1] = b2;
    } else {
      pk[i] = Elem<T>::pack(pp.x, pp.y);
    }
  }
  l += (la[0].x + la[0].y) + (la[1].x + la[1].y);
  if (ENT) h += (ha[0].x + ha[0].y) + (ha[1].x + ha[1].y);
  return MAXO ? fmaxf(fmaxf(mr[0], mr[1]), fmaxf(mr[2], mr[3])) * sc : -1e30f;
}



template <typename T, int XA, bool VK, int NSLOT, bool ENT, bool F8 = false>
__global__ void __launch_bounds__(kThreads, 1) fea_fwd_sm100_kernel(const __grid_constant__ Sm100FwdParams p) {
  using C = FwdCfg<XA, VK, NSLOT, F8>;
  constexpr bool kBf16 = Elem<T>::is_bf16;
  // F8: q, k and X are e4m3 (kind::f8f6f4, K = 32 per MMA) and P is stored as e4m3; o stays T
  constexpr uint32_t IDESC_S = F8 ? idesc_e4m3(128, 128, false, false) : idesc_f16(kBf16, 128, 128, false, false);
  constexpr uint32_t IDESC_S32 =  // a last tile of <= 32 keys
      F8 ? idesc_e4m3(128, 32, false, false) : idesc_f16(kBf16, 128, 32, false, false);
  constexpr uint32_t IDESC_PV = F8 ? idesc_e4m3(128, C::NV, false, true) : idesc_f16(kBf16, 128, C::NV, false, true);
  constexpr int SK = F8 ? 4 : 8;              // S MMAs over D = 128 (32 bytes of each row per step)
  constexpr int PVS = F8 ? 4 : 8;             // P V MMAs over a 128-key tile
  constexpr int PVB = 128 / PVS * 128;        // bytes of X rows per P V step
  constexpr int PK = F8 ? 16 : 32;            // 32-bit words of P per 64-key segment

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[8 + 3 * NSLOT];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bi = blockIdx.x / p.n_qtiles;
  const BIdx bx = bidx(bi, p.n1, p.n2);
  const int q0 = (blockIdx.x % p.n_qtiles) * 128;
  const int n_kt = (p.n_kv + 127) / 128;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = sbase;
  const uint32_t sRing = sbase + C::Q_BYTES;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t BAR_Q = bar0;
  auto BAR_KFULL = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_VFULL = [&](int s) { return bar0 + 8u * (1 + NSLOT + s); };
  auto BAR_EMPTY = [&](int s) { return bar0 + 8u * (1 + 2 * NSLOT + s); };
  auto BAR_SFULL = [&](int b) { return bar0 + 8u * (1 + 3 * NSLOT + b); };
  auto BAR_PFULL = [&](int b) { return bar0 + 8u * (3 + 3 * NSLOT + b); };
  const uint32_t BAR_DONE = bar0 + 8u * (5 + 3 * NSLOT);
  // P V(j) complete (commit behind it, alternating by tile parity): a rescale of O at tile j waits
  // for P V(j - 1), the only one that can be in flight then, so no parity wait can be lapped
  auto BAR_PVD = [&](int b) { return bar0 + 8u * (6 + 3 * NSLOT + b); };
  volatile int* abort = &abort_sh;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(BAR_Q, 1);
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(BAR_KFULL(s), 1);
      mbar_init(BAR_VFULL(s), 1);
      mbar_init(BAR_EMPTY(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR_SFULL(b), 1);
      mbar_init(BAR_PFULL(b), 256);
      mbar_init(BAR_PVD(b), 1);
    }
    mbar_init(BAR_DONE, 1);
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
    // ------------------------------------------------------------------ TMA producer
    // (hold_loads, a test of the timeout path: no load is issued, so every consumer wait runs out)
    if (lane == 0 && !p.hold_loads) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      if (XA > 0) prefetch_tmap(&p.tm_x);
      constexpr int AX = F8 ? 128 : 64;  // columns per atom
      mbar_expect_tx(BAR_Q, C::Q_BYTES);
      for (int a = 0; a < C::KA; ++a) tma_load(sQ + a * kAtom, &p.tm_q, AX * a, q0, bx, BAR_Q);
      int armed[NSLOT];
      for (int s = 0; s < NSLOT; ++s) armed[s] = 0;
      for (int j = 0; j < n_kt; ++j) {
        const int s = j % NSLOT;
        if (j >= NSLOT && !mbar_wait(BAR_EMPTY(s), ((j / NSLOT) - 1) & 1, abort, &g_fwd_err, 1, p.wait_limit)) break;
        const uint32_t slot = sRing + s * C::SLOT;
        mbar_expect_tx(BAR_KFULL(s), C::KA * kAtom);
        for (int a = 0; a < C::KA; ++a) tma_load(slot + a * kAtom, &p.tm_k, AX * a, j * 128, bx, BAR_KFULL(s));
        if (XA > 0) {
          mbar_expect_tx(BAR_VFULL(s), C::XAT * kAtom);
          for (int a = 0; a < C::XAT; ++a)
            tma_load(slot + (C::KA + a) * kAtom, &p.tm_x, AX * a, j * 128, bx, BAR_VFULL(s));
        }
        if (j + NSLOT < n_kt) {  // the tiles one ring ahead into L2
          for (int a = 0; a < C::KA; ++a) tma_prefetch(&p.tm_k, AX * a, (j + NSLOT) * 128, bx);
          for (int a = 0; a < C::XAT; ++a) tma_prefetch(&p.tm_x, AX * a, (j + NSLOT) * 128, bx);
        }
        armed[s] = j / NSLOT + 1;
      }
      // drain: every armed phase must have landed before the CTA may exit
      mbar_wait_drain(BAR_Q, 0);
      for (int s = 0; s < NSLOT; ++s) {
        if (armed[s] > 0) {
          mbar_wait_drain(BAR_KFULL(s), (armed[s] - 1) & 1);
          if (XA > 0) mbar_wait_drain(BAR_VFULL(s), (armed[s] - 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the schedule (waits are made warp-uniform); one elected lane (always the
    // same one, so its commits track all MMAs) issues. Two commits per KV tile: S -> SFULL, and
    // P V -> EMPTY(slot), which both frees the ring slot and tells the softmax warps that O is done.
    const uint32_t leader = elect_one() ? 1u : 0u;  // the lane that issues (warp converged here)
    auto wwait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_fwd_err, code, p.wait_limit));
    };
    bool ok = wwait(BAR_Q, 0, 2);
    auto issue_s = [&](int j) -> bool {
      const int s = j % NSLOT;
      if (!wwait(BAR_KFULL(s), (j / NSLOT) & 1, 2)) return false;
      tc_fence_after();
      {
        const uint32_t kb = sRing + s * C::SLOT;
        const uint32_t d = tmem + (uint32_t)((j & 1) * 128);
        // a last tile of <= 32 keys: N = 32 (the softmax masks the columns past n_kv by index)
        const uint32_t idesc = p.n_kv - j * 128 <= 32 ? IDESC_S32 : IDESC_S;
#pragma unroll
        for (int kk = 0; kk < SK; ++kk) {
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          mmax_ss_if<F8>(leader, d, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), idesc,
                         kk > 0);
        }
        mma_commit_if(leader, BAR_SFULL(j & 1));
      }
      return true;
    };
    if (ok) ok = issue_s(0);
    if (ok && n_kt > 1) ok = issue_s(1);
    for (int j = 0; ok && j < n_kt; ++j) {
      const int s = j % NSLOT;
      if (!wwait(BAR_PFULL(j & 1), (j >> 1) & 1, 4)) break;
      if (XA > 0 && !wwait(BAR_VFULL(s), (j / NSLOT) & 1, 4)) break;
      tc_fence_after();
      {
        const uint32_t vb = sRing + s * C::SLOT + C::PV_OFF;
        const uint32_t a_tm = tmem + (uint32_t)((j & 1) * 128);
        const int ksteps = p.n_kv - j * 128 <= 32 ? 32 * PVS / 128 : PVS;  // keys of the tile, 128 / PVS per step
#pragma unroll
        for (int kk = 0; kk < PVS; ++kk)  // P of keys [64 h, 64 h + 64) sits in the first PK columns from 64 h
          mmax_ts_if<F8>(leader & (kk < ksteps ? 1u : 0u), tmem + 256,
                         a_tm + (kk / (PVS / 2)) * 64 + (kk % (PVS / 2)) * 8,
                         smem_desc_sw128(vb + kk * PVB, kAtom, 1024), IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit_if(leader, BAR_EMPTY(s));
        mma_commit_if(leader, BAR_PVD(j & 1));
      }
      if (j + 2 < n_kt) ok = issue_s(j + 2);
    }
    // drain: all issued MMAs complete before TMEM can be freed
    if (elect_one()) {
      mma_commit(BAR_DONE);
      mbar_wait_drain(BAR_DONE, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    // Two warpgroups split every 128-key tile by columns: warpgroup wg owns keys [64 wg, 64 wg + 64)
    // of each row and O columns [wg NV/2, (wg + 1) NV/2). Both hold the same m_ref and take
    // identical rescale decisions: on full tiles after the first, the exponentials run against
    // m_ref and one OR barrier (named barrier 1) confirms that no row's sum passed the limit; otherwise
    // they exchange the half-row maxima through TMEM (named barrier 1 again) and compute P against
    // the agreed reference. l and h are per-warpgroup partial sums, added in the epilogue. Every
    // named barrier is reached by all 256 threads and reduces their status, so a failed wait in
    // one warpgroup ends both at the same point.
    // Each warpgroup writes its P (bf16) over the first 32 columns of its own half of S (columns
    // [64 wg, 64 wg + 32), already loaded), so neither waits for the other before storing it; the
    // maxima are exchanged through column 64 wg + 32 of its half (not written by any P; the next S
    // MMA into this buffer waits for both warpgroups' P).
    const int wg = (warp - 2) >> 2;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    constexpr int OCH = C::NV / 64;  // 32-column O chunks per warpgroup
    float m_ref = -1e30f, l = 0.f, h = 0.f;
    bool ok = true;

    auto warp_wait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      const bool mine = mbar_wait(bar, parity, abort, &g_fwd_err, code, p.wait_limit);
      return __all_sync(0xffffffffu, mine);
    };

    for (int j = 0; j < n_kt; ++j) {
      bool good = ok && warp_wait(BAR_SFULL(j & 1), (j >> 1) & 1, 8);
      tc_fence_after();
      const uint32_t tS = tmem + lane_off + (uint32_t)((j & 1) * 128);
      uint32_t sr[64];
      const int valid = p.n_kv - j * 128 - wg * 64;  // keys of this half; uniform per warpgroup
      if (good) {
        tmem_ld32(tS + wg * 64, sr);
        tmem_ld32(tS + wg * 64 + 32, sr + 32);
        tmem_wait_ld();
      }
      uint32_t pk[PK];
      float lt = 0.f, ht = 0.f;
      // A full tile after the first: the exponentials against the current reference, P stored at
      // once. One barrier tells both warpgroups whether any row's half sum passed kSumThreshold
      // (e4m3: its max passed the reference by more than the threshold) or a wait failed. Otherwise
      // (first tile, ragged tile, or a row past the threshold) the half-row maxima are exchanged
      // as below and P is computed (again) against the agreed reference and stored.
      bool redo = true;
      const bool fast = j > 0 && p.n_kv - j * 128 >= 128;  // the same branch in both warpgroups (one barrier)
      if (fast) {
        float mh = -1e30f;
        if (good) {
          mh = probs_row<T, 64, ENT, false, F8, F8>(sr, pk, p.scale_log2, m_ref, 64, lt, ht);
          tmem_st_p<F8>(tS + wg * 64, pk);  // this warpgroup's own half of S (already loaded)
        }
        redo = named_bar_or(1, 256, !good || (F8 ? mh > m_ref + kRescaleThreshold : !(lt <= kSumThreshold)));
      }
      if (redo) {
        float mh = -1e30f;
        if (good) mh = valid < 64 ? row_max_raw<64, true>(sr, valid) : row_max_raw<64, false>(sr, 64);
        if (good) {
          tmem_st1(tS + 64 * wg + 32, __float_as_uint(mh));  // past this warpgroup's P columns
          tmem_wait_st();
        }
        tc_fence_before();
        if (!named_bar_and(1, 256, good)) { ok = false; break; }
        tc_fence_after();
        const float mo = __uint_as_float(tmem_ld1(tS + 64 * (wg ^ 1) + 32));
        tmem_wait_ld();
        const float mx = fmaxf(mh, mo) * p.scale_log2;
        bool fresh = !fast;  // P not yet computed against the reference
        if (j == 0) {
          m_ref = mx;
        } else if (__any_sync(0xffffffffu, mx > m_ref + kRescaleThreshold)) {
          // The rescale touches TMEM with warp-collective loads / stores and waits on a barrier, so
          // the decision is taken per warp: every lane whose max grew adopts it (alpha < 1), the
          // others keep their reference (alpha = 1). The twin warp of the other warpgroup sees the
          // same maxima and takes the same decision.
          if (!warp_wait(BAR_PVD((j - 1) & 1), ((j - 1) >> 1) & 1, 8)) ok = false;  // reported at the next barrier
          tc_fence_after();
          const float m_new = fmaxf(m_ref, mx);
          const float alpha = fast_exp2(m_ref - m_new);
#pragma unroll 1
          for (int c = wg * OCH; c < (wg + 1) * OCH; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
          tmem_wait_st();
          if (ENT) h = alpha * fmaf(m_ref - m_new, l, h);
          l *= alpha;
          m_ref = m_new;
          fresh = true;
        }
        if (fresh) {
          lt = 0.f;
          ht = 0.f;
          if (valid <= 0) {  // no key of this half (a ragged last tile): P = 0 with no exponentials
#pragma unroll
            for (int i = 0; i < PK; ++i) pk[i] = 0u;
          } else if (valid <= 32) {  // keys [0, 32) of the half only
            const uint32_t(&s32)[32] = *reinterpret_cast<const uint32_t(*)[32]>(&sr[0]);
            uint32_t(&p32)[PK / 2] = *reinterpret_cast<uint32_t(*)[PK / 2]>(&pk[0]);
            probs_row<T, 32, ENT, true, false, F8>(s32, p32, p.scale_log2, m_ref, valid, lt, ht);
#pragma unroll
            for (int i = PK / 2; i < PK; ++i) pk[i] = 0u;
          } else if (valid < 64) {
            probs_row<T, 64, ENT, true, false, F8>(sr, pk, p.scale_log2, m_ref, valid, lt, ht);
          } else {
            probs_row<T, 64, ENT, false, false, F8>(sr, pk, p.scale_log2, m_ref, 64, lt, ht);
          }
        }
        if (good) tmem_st_p<F8>(tS + wg * 64, pk);
      }
      l += lt;
      h += ht;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR_PFULL(j & 1));
    }

    if (ok) ok = warp_wait(BAR_PVD((n_kt - 1) & 1), ((n_kt - 1) >> 1) & 1, 8);  // the last P V
    tc_fence_after();
    // epilogue: add the partial sums (exchanged through the Q tile, idle once the last P V - and
    // with it every S MMA - has completed), O / l -> bf16 in the (now idle) ring, TMA store; LSE
    // and entropy per row
    float* xch = reinterpret_cast<float*>(smem_raw + (sQ - smem_u32(smem_raw)));
    xch[(2 * wg) * 128 + row] = l;
    xch[(2 * wg + 1) * 128 + row] = h;
    ok = named_bar_and(2, 256, ok);
    const uint32_t stage = sRing;
    if (ok) {
      l += xch[(2 * (wg ^ 1)) * 128 + row];
      h += xch[(2 * (wg ^ 1) + 1) * 128 + row];
      const float inv = 1.f / l;
#pragma unroll 1
      for (int c = wg * OCH; c < (wg + 1) * OCH; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = Elem<T>::pack(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        const int atom = c >> 1;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int chunk = (c & 1) * 4 + k;
          const uint32_t dst = stage + atom * kAtom + row * 128 + ((chunk ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[4 * k]), "r"(w[4 * k + 1]),
                       "r"(w[4 * k + 2]), "r"(w[4 * k + 3])
                       : "memory");
        }
      }
      const int grow = q0 + row;
      if (wg == 0 && grow < p.n_q) {
        const float lg = log2f(l);
        const int64_t idx = (int64_t)bi * p.n_q + grow;
        if (p.lse) p.lse[idx] = m_ref + lg;
        if (ENT && p.ent) p.ent[idx] = (lg - h / l) * kLn2;
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(3, 256);
    if (warp == 2 && lane == 0 && ok && !*abort) {
      for (int a = 0; a < C::NV / 64; ++a) tma_store(&p.tm_o, 64 * a, q0, bx, stage + a * kAtom);
      tma_store_commit_and_wait();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------- Dv = 128
// Two-stream forward for 128 output columns. CTA = two 128-row query tiles of one sequence; the two
// softmax warpgroups are two independent streams, stream w owning query tile w, each with its own
// TMEM S buffer, O accumulator and online statistics (m_ref, l, h), both walking the same key tiles:
// every K / V tile is loaded once for two query tiles. The streams never wait for each other, so
// one warpgroup's exponentials overlap the other's TMEM loads and the tensor work of its tile.
// TMEM: S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512). The MMA warp walks steps
// j = 2 t + w (stream w, key tile t).
// A tile's P goes out in two 64-key halves: BAR_PHALF after the first lets the MMA warp issue
// P V for those keys while the softmax works on the second (the chain softmax -> own P V -> next S
// bounds each stream's cycle). Full tiles after a stream's first skip the separate max pass: the
// exponentials run against the current reference m_ref, and a half whose sum of p passes
// kSumThreshold (e4m3: whose max, taken beside the exponentials, passes m_ref + threshold) is
// redone from its scores (still in registers)
// after the rescale; a redo in the second half first waits for BAR_PVH, the commit behind the
// first half's P V, which adds into O. The stream's first tile and a ragged last tile take the
// max first.
// One tcgen05.commit per step (S -> SFULL): S_w(t+1) is issued after P V_w(t) into the same buffers
// and the tensor pipe executes one thread's MMAs in order, so S_w(t+1) complete implies P V_w(t)
// complete. So a rescale of O_w at key tile t needs no wait beyond S_w(t), and each stream that
// observes S_w(t) arrives on the EMPTY barriers (two arrivals each) of the ring slots it is done
// with: the K slot of tile t (K read by the S MMAs only) and the V slot of tile t - 1 (read by
// P V(t - 1)); with V aliasing K the K slot of tile t - 1. The producer waits on those per-slot
// barriers, whose next phase needs a tile it has not loaded yet, so no parity wait can be lapped.
// NS = 1 (V aliasing K, short sequences): one stream and one query tile, S [0,128) and O [128,256),
// so two CTAs share an SM (96 KB of shared memory, 256 TMEM columns each) and one CTA's Q load and
// epilogue overlap the other's key loop; S goes out in two halves (HS, below).
template <bool VK, int NS = 2, bool F8 = false>
struct Fwd2Cfg {
  static_assert(NS == 2 || (NS == 1 && VK), "one stream only with V aliasing K");
  static_assert(!F8 || NS == 1, "e4m3: the one-stream instance");
  // a 128-row tile of q or k (D = 128) is two 128-byte swizzle atoms of 16-bit elements, one of e4m3
  static constexpr int TILE = (F8 ? 1 : 2) * kAtom;
  static constexpr int NK = NS == 1 ? (F8 ? 4 : 2) : (VK ? 5 : 3);  // K ring slots (V aliasing K: also the V operand)
  static constexpr int NVS = VK ? 0 : 2;                 // V ring slots
  static constexpr int Q_BYTES = NS * TILE;              // one 128-row query tile per stream
  static constexpr int SMEM = 1024 + Q_BYTES + (NK + NVS) * TILE;
  static_assert((NK + NVS) * TILE >= NS * 2 * kAtom, "the epilogue stages the 16-bit O tiles in the ring");
  static constexpr int THREADS = 64 + 128 * NS;
  static_assert(SMEM <= 232448 - 1024, "shared memory budget");
  static_assert(NS == 2 || 2 * (SMEM + 1024) <= 233472, "two CTAs per SM");
};

template <typename T, bool VK, bool ENT, int NS = 2, bool F8 = false>
__global__ void __launch_bounds__(64 + 128 * NS, 3 - NS) fea_fwd2_sm100_kernel(const __grid_constant__ Sm100FwdParams p) {
  using C = Fwd2Cfg<VK, NS, F8>;
  constexpr uint32_t kTmemCols = NS == 2 ? 512 : 256;
  constexpr int NK = C::NK, NVS = C::NVS;
  constexpr uint32_t TILE = C::TILE;
  constexpr bool kBf16 = Elem<T>::is_bf16;
  // F8: q and k are e4m3 (kind::f8f6f4, K = 32 per MMA) and P is stored as e4m3; o stays T
  constexpr uint32_t IDESC_S = F8 ? idesc_e4m3(128, 128, false, false) : idesc_f16(kBf16, 128, 128, false, false);
  constexpr uint32_t IDESC_S32 =  // a last tile of <= 32 keys
      F8 ? idesc_e4m3(128, 32, false, false) : idesc_f16(kBf16, 128, 32, false, false);
  constexpr uint32_t IDESC_S64 =  // one 64-key half of S
      F8 ? idesc_e4m3(128, 64, false, false) : idesc_f16(kBf16, 128, 64, false, false);
  constexpr uint32_t IDESC_PV = F8 ? idesc_e4m3(128, 128, false, true) : idesc_f16(kBf16, 128, 128, false, true);
  constexpr int SK = F8 ? 4 : 8;        // S MMAs over D = 128 (32 bytes of each row per step)
  constexpr int PVS = F8 ? 4 : 8;       // P V MMAs over a 128-key tile
  constexpr int PVB = 128 / PVS * 128;  // bytes of V rows per P V step
  constexpr int PK = F8 ? 16 : 32;      // 32-bit words of P per 64-key segment
  // HS (the one-stream instance): S in two 64-key halves, S_A = keys [0, 64) -> columns [0, 64) and
  // S_B = keys [64, 128) -> columns [64, 128), with P of each half over the first 32 columns of its
  // own half. S_A(j + NS) is issued right behind P V of the first half of tile j and S_B(j + NS)
  // behind the second, so the softmax finds each half of its next S ready instead of waiting for
  // P V(j) and the whole of S(j + NS) after finishing tile j.
  constexpr bool HS = NS == 1;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[14 + 2 * (NK + NVS)];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // block -> (sequence, NS query tiles, key chunk); with kv_split == 1 a CTA walks all key tiles.
  // Stream w owns query tile rows [q0 + 128 w, q0 + 128 w + 128) (past n_q: zero-filled, clipped).
  const int n_units = (p.n_qtiles + NS - 1) / NS;
  const int per_seq = n_units * p.kv_split;
  const int bi = blockIdx.x / per_seq;
  const BIdx bx = bidx(bi, p.n1, p.n2);
  const int q0 = ((blockIdx.x % per_seq) / p.kv_split) * 128 * NS;
  const int kchunk = blockIdx.x % p.kv_split;
  const int kt0 = kchunk * p.kt_per;                                  // first key tile of the chunk
  const int n_kt = min((p.n_kv + 127) / 128 - kt0, p.kt_per);       // >= 1 by the host's choice

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = sbase;
  const uint32_t sK = sbase + C::Q_BYTES;
  const uint32_t sV = sK + NK * TILE;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t BAR_Q = bar0;
  auto BAR_KFULL = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_VFULL = [&](int s) { return bar0 + 8u * (1 + NK + s); };
  auto BAR_KEMPTY = [&](int s) { return bar0 + 8u * (1 + NK + NVS + s); };
  auto BAR_VEMPTY = [&](int s) { return bar0 + 8u * (1 + 2 * NK + NVS + s); };
  auto BAR_SFULL = [&](int b) { return bar0 + 8u * (1 + 2 * (NK + NVS) + b); };
  auto BAR_PFULL = [&](int b) { return bar0 + 8u * (3 + 2 * (NK + NVS) + b); };
  const uint32_t BAR_DONE = bar0 + 8u * (5 + 2 * (NK + NVS));
  auto BAR_PHALF = [&](int b) { return bar0 + 8u * (6 + 2 * (NK + NVS) + b); };  // P of keys [0, 64) in TMEM
  auto BAR_PVH = [&](int b) { return bar0 + 8u * (8 + 2 * (NK + NVS) + b); };    // that half of P V complete
  auto BAR_SA = [&](int b) { return bar0 + 8u * (10 + 2 * (NK + NVS) + b); };    // HS: S_A complete
  auto BAR_PVB = [&](int b) { return bar0 + 8u * (12 + 2 * (NK + NVS) + b); };   // HS: P V of keys [64, 128) complete
  volatile int* abort = &abort_sh;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(BAR_Q, 1);
    // slot releases: one commit behind the last MMA reading the slot (HS), else one arrival per stream
    for (int s = 0; s < NK; ++s) {
      mbar_init(BAR_KFULL(s), 1);
      mbar_init(BAR_KEMPTY(s), HS ? 1 : NS);
    }
    for (int s = 0; s < NVS; ++s) {
      mbar_init(BAR_VFULL(s), 1);
      mbar_init(BAR_VEMPTY(s), HS ? 1 : NS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR_SFULL(b), 1);
      mbar_init(BAR_PFULL(b), 128);
      mbar_init(BAR_PHALF(b), 128);
      mbar_init(BAR_PVH(b), 1);
      mbar_init(BAR_SA(b), 1);
      mbar_init(BAR_PVB(b), 1);
    }
    mbar_init(BAR_DONE, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_base_sh), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producers
    // lane 0: Q, then the K ring; lane 1 (separate V only): the V ring. (hold_loads, a test of the
    // timeout path: no load is issued, so every consumer wait runs out)
    if ((lane == 0 || (!VK && lane == 1)) && !p.hold_loads) {
      const bool kl = lane == 0;
      const int nslot = kl ? NK : NVS;
      if (kl) {
        prefetch_tmap(&p.tm_q);
        prefetch_tmap(&p.tm_k);
        mbar_expect_tx(BAR_Q, C::Q_BYTES);
        for (int w = 0; w < NS; ++w) {
          tma_load(sQ + w * TILE, &p.tm_q, 0, q0 + 128 * w, bx, BAR_Q);
          if (!F8) tma_load(sQ + w * TILE + kAtom, &p.tm_q, 64, q0 + 128 * w, bx, BAR_Q);
        }
      } else {
        prefetch_tmap(&p.tm_x);
      }
      int armed[NK > NVS ? NK : NVS];
      for (int s = 0; s < nslot; ++s) armed[s] = 0;
      for (int j = 0; j < n_kt; ++j) {
        const int s = j % nslot;
        const uint32_t empty = kl ? BAR_KEMPTY(s) : BAR_VEMPTY(s);
        if (j >= nslot && !mbar_wait(empty, ((j / nslot) - 1) & 1, abort, &g_fwd_err, 1, p.wait_limit)) break;
        const uint32_t full = kl ? BAR_KFULL(s) : BAR_VFULL(s);
        const uint32_t slot = (kl ? sK : sV) + s * TILE;
        mbar_expect_tx(full, TILE);
        const bool hx = kl && p.k_hi_x;  // second atom of the K tile from V2
        const CUtensorMap* hi = (kl && !hx) ? &p.tm_k : &p.tm_x;
        tma_load(slot, kl ? &p.tm_k : &p.tm_x, 0, (kt0 + j) * 128, bx, full);
        if (!F8) tma_load(slot + kAtom, hi, hx ? 0 : 64, (kt0 + j) * 128, bx, full);
        if (j + nslot < n_kt) {  // the tile one ring ahead into L2
          tma_prefetch(kl ? &p.tm_k : &p.tm_x, 0, (kt0 + j + nslot) * 128, bx);
          if (!F8) tma_prefetch(hi, hx ? 0 : 64, (kt0 + j + nslot) * 128, bx);
        }
        armed[s] = j / nslot + 1;
      }
      // drain: every armed phase must have landed before the CTA may exit
      if (kl) mbar_wait_drain(BAR_Q, 0);
      for (int s = 0; s < nslot; ++s)
        if (armed[s] > 0) mbar_wait_drain(kl ? BAR_KFULL(s) : BAR_VFULL(s), (armed[s] - 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t leader = elect_one() ? 1u : 0u;  // the lane that issues (warp converged here)
    auto wwait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_fwd_err, code, p.wait_limit));
    };
    bool ok = wwait(BAR_Q, 0, 2);
    // Step j: stream w = j % NS (query tile w) with key tile t = j / NS.
    auto issue_s = [&](int j) -> bool {
      const int w = j % NS, t = j / NS, s = t % NK;
      if (!wwait(BAR_KFULL(s), (t / NK) & 1, 2)) return false;
      tc_fence_after();
      {
        const uint32_t kb = sK + s * TILE, qb = sQ + w * TILE;
        const uint32_t d = tmem + (uint32_t)(w * 128);
        // a last tile of <= 32 keys: N = 32 (the softmax masks the columns past n_kv by index)
        const uint32_t idesc = p.n_kv - (kt0 + t) * 128 <= 32 ? IDESC_S32 : IDESC_S;
#pragma unroll
        for (int kk = 0; kk < SK; ++kk) {
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          mmax_ss_if<F8>(leader, d, smem_desc_sw128(qb + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), idesc,
                         kk > 0);
        }
        mma_commit_if(leader, BAR_SFULL(w));
      }
      return true;
    };
    // HS: the two halves of S(j); S_B is skipped when no key of the tile lies in [64, 128), and the
    // K slot (and with separate V the V slot) is released by commits behind the last MMA reading it
    auto issue_sa = [&](int j) -> bool {  // NS = 1: key tile t = j
      const int s = j % NK;
      if (!wwait(BAR_KFULL(s), (j / NK) & 1, 2)) return false;
      tc_fence_after();
      const uint32_t kb = sK + s * TILE;
      const uint32_t d = tmem + (uint32_t)((j % NS) * 128);
      const uint32_t idesc = p.n_kv - (kt0 + j) * 128 <= 32 ? IDESC_S32 : IDESC_S64;
#pragma unroll
      for (int kk = 0; kk < SK; ++kk) {
        const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
        mmax_ss_if<F8>(leader, d, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), idesc,
                       kk > 0);
      }
      mma_commit_if(leader, BAR_SA(j % NS));
      return true;
    };
    auto issue_sb = [&](int j) {  // K(j) has landed (issue_sa)
      const int s = j % NK;
      const uint32_t kb = sK + s * TILE + 64 * 128;  // key rows [64, 128)
      const uint32_t d = tmem + (uint32_t)((j % NS) * 128) + 64;
      const uint32_t on = p.n_kv - (kt0 + j) * 128 > 64 ? leader : 0u;
#pragma unroll
      for (int kk = 0; kk < SK; ++kk) {
        const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
        mmax_ss_if<F8>(on, d, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), IDESC_S64,
                       kk > 0);
      }
      mma_commit_if(leader, BAR_SFULL(j % NS));
      if (!VK) mma_commit_if(leader, BAR_KEMPTY(s));  // separate V: K(j) is read by S(j) only
    };
    const int n_steps = NS * n_kt;
    if (HS) {
      if (ok) ok = issue_sa(0);
      if (ok) issue_sb(0);
    } else {
      for (int j = 0; ok && j < NS; ++j) ok = issue_s(j);  // key tile 0 of every stream
    }
    // P V in two 64-key halves: the first is issued once the softmax has stored P of keys [0, 64)
    // (BAR_PHALF), so it runs while the softmax computes the second half
    for (int j = 0; ok && j < n_steps; ++j) {
      const int w = j % NS, t = j / NS;
      const uint32_t vb = VK ? sK + (t % NK) * TILE : sV + (t % NVS) * TILE;
      const uint32_t a_tm = tmem + (uint32_t)(w * 128);
      const uint32_t o_tm = tmem + NS * 128 + (uint32_t)(w * 128);
      const int ksteps = p.n_kv - (kt0 + t) * 128 <= 32 ? 32 * PVS / 128 : PVS;  // keys of the tile, 128 / PVS per step
      if (!wwait(BAR_PHALF(w), t & 1, 4)) break;
      if (!VK && !wwait(BAR_VFULL(t % NVS), (t / NVS) & 1, 4)) break;
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < PVS / 2; ++kk)
        mmax_ts_if<F8>(leader & (kk < ksteps ? 1u : 0u), o_tm, a_tm + kk * 8,
                       smem_desc_sw128(vb + kk * PVB, kAtom, 1024), IDESC_PV, (t > 0 || kk > 0) ? 1u : 0u);
      mma_commit_if(leader, BAR_PVH(w));  // a softmax that rescales O mid-tile waits for it
      if (HS && j + NS < n_steps && !(ok = issue_sa(j + NS))) break;
      if (!wwait(BAR_PFULL(w), t & 1, 4)) break;
      tc_fence_after();
#pragma unroll
      for (int kk = PVS / 2; kk < PVS; ++kk)  // HS: P of keys [64, 128) sits in the first PK columns from 64
        mmax_ts_if<F8>(leader & (kk < ksteps ? 1u : 0u), o_tm, a_tm + (HS ? 64 + (kk - PVS / 2) * 8 : kk * 8),
                       smem_desc_sw128(vb + kk * PVB, kAtom, 1024), IDESC_PV, 1u);
      if (HS) {
        mma_commit_if(leader, BAR_PVB(w));
        mma_commit_if(leader, VK ? BAR_KEMPTY(t % NK) : BAR_VEMPTY(t % NVS));  // the slot P V(j) read
        if (j + NS < n_steps) issue_sb(j + NS);
      } else if (j + NS < n_steps) {
        ok = issue_s(j + NS);
      }
    }
    // DONE: every MMA complete (the epilogue reads O; TMEM may be freed)
    if (elect_one()) {
      mma_commit(BAR_DONE);
      mbar_wait_drain(BAR_DONE, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax streams + epilogue
    const int w = (warp - 2) >> 2;  // stream: query tile w, every key tile of the CTA's range
    const int quad = warp & 3;      // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + (uint32_t)(w * 128);
    float m_ref = -1e30f, l = 0.f, h = 0.f;
    bool ok = true;
    auto warp_wait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_fwd_err, code, p.wait_limit));
    };

    for (int t = 0; t < n_kt; ++t) {  // key tile t of this stream (step j = NS t + w)
      // HS: S_A first (S_B is waited for before the second half); otherwise all of S
      if (!warp_wait(HS ? BAR_SA(w) : BAR_SFULL(w), t & 1, 8)) { ok = false; break; }
      tc_fence_after();
      if (!HS && warp == 2 + 4 * w && lane == 0) {  // ring slots done with (see above)
        // S_w(t) complete: every stream's arrival frees the K slot of key tile t (separate V: read
        // by the S MMAs only) or of t - 1 (V aliasing K: read by P V too), and the V slot of t - 1
        if (VK) {
          if (t >= 1) mbar_arrive(BAR_KEMPTY((t - 1) % NK));
        } else {
          mbar_arrive(BAR_KEMPTY(t % NK));
          if (t >= 1) mbar_arrive(BAR_VEMPTY((t - 1) % NVS));
        }
      }
      const int valid = p.n_kv - (kt0 + t) * 128;  // same for every thread: the branches below are uniform
      // O, l, h to the reference max(m_ref, mx). Warp-uniform (warp-collective TMEM access): lanes
      // whose max grew adopt it. The caller guarantees no P V into O_w is in flight.
      auto rescale = [&](float mx) {
        const float m_new = fmaxf(m_ref, mx);
        const float alpha = fast_exp2(m_ref - m_new);
        const uint32_t tO = tmem + lane_off + NS * 128 + (uint32_t)(w * 128);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
        tmem_wait_st();
        if (ENT) h = alpha * fmaf(m_ref - m_new, l, h);
        l *= alpha;
        m_ref = m_new;
      };
      // P in two 64-key halves: keys [64 k, 64 k + 64) -> columns [32 k, 32 k + 32); BAR_PHALF
      // after the first lets P V of those keys start.
      if (t > 0 && valid >= 128) {
        // A full tile after the stream's first: the exponentials go against the current reference;
        // a half whose sum passes kSumThreshold (rare: the reference only grows) is redone after
        // the rescale to its max, from the scores still in registers.
        {
          uint32_t sa[64];
          tmem_ld32(tS + 0, sa);
          tmem_ld32(tS + 32, sa + 32);
          tmem_wait_ld();
          uint32_t pk[PK];
          float lt = 0.f, ht = 0.f;
          const float mx = probs_row<T, 64, ENT, false, F8, F8>(sa, pk, p.scale_log2, m_ref, 64, lt, ht);
          if (__any_sync(0xffffffffu, F8 ? mx > m_ref + kRescaleThreshold : !(lt <= kSumThreshold))) {
            // every earlier P V into O_w has completed (S_w(t) complete; HS: S_A(t) only follows the
            // first half of P V(t - 1), so wait for the second); P V(t) is not issued yet
            if (HS && !warp_wait(BAR_PVB(w), (t - 1) & 1, 16)) { ok = false; break; }
            tc_fence_after();
            rescale(F8 ? mx : row_max_raw<64, false>(sa, 64) * p.scale_log2);
            lt = 0.f;
            ht = 0.f;
            probs_row<T, 64, ENT, false, false, F8>(sa, pk, p.scale_log2, m_ref, 64, lt, ht);
          }
          l += lt;
          h += ht;
          tmem_st_p<F8>(tS + 0, pk);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(BAR_PHALF(w));
        }
        if (HS) {
          if (!warp_wait(BAR_SFULL(w), t & 1, 8)) { ok = false; break; }
          tc_fence_after();
        }
        {
          uint32_t sb[64];
          tmem_ld32(tS + 64, sb);
          tmem_ld32(tS + 96, sb + 32);
          tmem_wait_ld();
          uint32_t pk[PK];
          float lt = 0.f, ht = 0.f;
          const float mx = probs_row<T, 64, ENT, false, F8, F8>(sb, pk, p.scale_log2, m_ref, 64, lt, ht);
          if (__any_sync(0xffffffffu, F8 ? mx > m_ref + kRescaleThreshold : !(lt <= kSumThreshold))) {
            // the first half of P V(t) may still be adding into O_w: wait for its commit
            if (!warp_wait(BAR_PVH(w), t & 1, 16)) { ok = false; break; }
            tc_fence_after();
            rescale(F8 ? mx : row_max_raw<64, false>(sb, 64) * p.scale_log2);
            lt = 0.f;
            ht = 0.f;
            probs_row<T, 64, ENT, false, false, F8>(sb, pk, p.scale_log2, m_ref, 64, lt, ht);
          }
          l += lt;
          h += ht;
          tmem_st_p<F8>(tS + (HS ? 64 : 32), pk);
        }
      } else {
        // the stream's first tile (sets the reference) and the ragged last tile: the tile max first
        if (HS) {
          if (!warp_wait(BAR_SFULL(w), t & 1, 8)) { ok = false; break; }
          tc_fence_after();
        }
        uint32_t sr[128];
        tmem_ld32(tS + 0, sr);
        tmem_ld32(tS + 32, sr + 32);
        tmem_ld32(tS + 64, sr + 64);
        tmem_ld32(tS + 96, sr + 96);
        tmem_wait_ld();
        const float mx =
            (valid < 128 ? row_max_raw<128, true>(sr, valid) : row_max_raw<128, false>(sr, 128)) * p.scale_log2;
        if (t == 0) {
          m_ref = mx;
        } else if (__any_sync(0xffffffffu, mx > m_ref + kRescaleThreshold)) {
          // every earlier P V into O_w has completed (S_w(t) complete, see above; HS: the second
          // half of P V(t - 1) is waited for)
          if (HS && !warp_wait(BAR_PVB(w), (t - 1) & 1, 16)) { ok = false; break; }
          tc_fence_after();
          rescale(mx);
        }
        {  // the second half of S is loaded again from TMEM (its columns are only overwritten by the
           // second half of P), so the first half's scores are the only ones live through the exponentials
          const uint32_t(&sh)[64] = *reinterpret_cast<const uint32_t(*)[64]>(&sr[0]);
          uint32_t pk[PK];
          if (valid <= 32) {  // keys [0, 32) only (the S and P V MMAs of such a tile are N / K = 32)
            const uint32_t(&s32)[32] = *reinterpret_cast<const uint32_t(*)[32]>(&sr[0]);
            uint32_t(&p32)[PK / 2] = *reinterpret_cast<uint32_t(*)[PK / 2]>(&pk[0]);
            probs_row<T, 32, ENT, true, false, F8>(s32, p32, p.scale_log2, m_ref, valid, l, h);
#pragma unroll
            for (int i = PK / 2; i < PK; ++i) pk[i] = 0u;
          } else if (valid < 128) {
            probs_row<T, 64, ENT, true, false, F8>(sh, pk, p.scale_log2, m_ref, valid, l, h);
          } else {
            probs_row<T, 64, ENT, false, false, F8>(sh, pk, p.scale_log2, m_ref, 64, l, h);
          }
          tmem_st_p<F8>(tS + 0, pk);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(BAR_PHALF(w));
        }
        {
          uint32_t pk[PK];
          if (valid > 64) {
            uint32_t sh[64];
            tmem_ld32(tS + 64, sh);
            tmem_ld32(tS + 96, sh + 32);
            tmem_wait_ld();
            if (valid < 128) probs_row<T, 64, ENT, true, false, F8>(sh, pk, p.scale_log2, m_ref, valid - 64, l, h);
            else probs_row<T, 64, ENT, false, false, F8>(sh, pk, p.scale_log2, m_ref, 64, l, h);
          } else {
            // no key of the tile in [64, 128) (the R-step tails at b = 1560 hold 24): P = 0 with no
            // exponentials; P V reads these columns when the tile has more than 32 keys
#pragma unroll
            for (int i = 0; i < PK; ++i) pk[i] = 0u;
          }
          tmem_st_p<F8>(tS + (HS ? 64 : 32), pk);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR_PFULL(w));
    }

    // epilogue: wait for every MMA; each stream normalises its own O (O / l) into 16-bit (or, for a
    // key chunk, fp32 O / l plus (m, l, h)) in the idle ring, one thread stores every stream's tile
    // with TMA (rows past n_q / n_pad clipped); LSE and entropy per row
    if (ok) ok = warp_wait(BAR_DONE, 0, 8);
    tc_fence_after();
    const bool part = p.kv_split > 1;  // key chunk: fp32 O normalised by this chunk's l, plus (m, l, h)
    const uint32_t stage = sK + (uint32_t)w * (part ? 4 : 2) * kAtom;  // this stream's tile (fp32: 64 KB)
    const int grow = q0 + 128 * w + row;
    if (ok) {
      const float inv = 1.f / l;
      const uint32_t tO = tmem + lane_off + NS * 128 + (uint32_t)(w * 128);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
        if (part) {
          // [128 rows][32 floats] box c of the fp32 staging (128-byte swizzle)
          const uint32_t base = stage + c * 16384 + row * 128;
#pragma unroll
          for (int k4 = 0; k4 < 8; ++k4)
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((k4 ^ (row & 7)) << 4)),
                         "f"(__uint_as_float(o[4 * k4]) * inv), "f"(__uint_as_float(o[4 * k4 + 1]) * inv),
                         "f"(__uint_as_float(o[4 * k4 + 2]) * inv), "f"(__uint_as_float(o[4 * k4 + 3]) * inv)
                         : "memory");
          continue;
        }
        uint32_t wv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          wv[i] = Elem<T>::pack(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        const int atom = c >> 1;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int chunk = (c & 1) * 4 + k;
          const uint32_t dst = stage + atom * kAtom + row * 128 + ((chunk ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(wv[4 * k]), "r"(wv[4 * k + 1]),
                       "r"(wv[4 * k + 2]), "r"(wv[4 * k + 3])
                       : "memory");
        }
      }
      if (part) {
        if (grow < p.n_pad) {  // rows past n_q too (inside n_pad): never read by the merge
          const int64_t plane = (int64_t)p.kv_split * p.n_seq * p.n_pad;
          const int64_t idx = ((int64_t)kchunk * p.n_seq + bi) * p.n_pad + grow;
          p.pst[idx] = m_ref;
          p.pst[plane + idx] = l;
          p.pst[2 * plane + idx] = h;
        }
      } else if (grow < p.n_q) {
        const float lg = log2f(l);
        const int64_t idx = (int64_t)bi * p.n_q + grow;
        if (p.lse) p.lse[idx] = m_ref + lg;
        if (ENT && p.ent) p.ent[idx] = (lg - h / l) * kLn2;
      }
    }
    fence_proxy_async_smem();
    ok = named_bar_and(2, 128 * NS, ok);
    if (warp == 2 && lane == 0 && ok && !*abort) {
      for (int ws = 0; ws < NS; ++ws) {
        const uint32_t st = sK + (uint32_t)ws * (part ? 4 : 2) * kAtom;
        const int qr = q0 + 128 * ws;
        if (part) {
          for (int c = 0; c < 4; ++c) tma_store(&p.tm_po, 32 * c, qr, kchunk * p.n_seq + bi, st + c * 16384);
        } else {
          for (int a = 0; a < 2; ++a) tma_store(&p.tm_o, 64 * a, qr, bx, st + a * kAtom);
        }
      }
      tma_store_commit_and_wait();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// Merge of the key chunks of a split key range (one warp per query row, lane = 4 columns):
// m = max_c m_c, a_c = 2^(m_c - m), l = sum a_c l_c, h = sum a_c (h_c + (m_c - m) l_c),
// o = sum (a_c l_c / l) o_c with o_c normalised by its own l_c; LSE2 = m + log2 l,
// entropy = (log2 l - h / l) ln 2. Chunks are summed in order (deterministic).
template <typename T>
__global__ void __launch_bounds__(256) fwd_split_merge_kernel(const float* po, const float* pst, int split, int64_t n_seq,
                                                              int64_t n_pad, int n_q, T* o, View ov, int n1, int n2,
                                                              float* lse, float* ent) {
  const int64_t rg = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (rg >= n_seq * n_q) return;
  const int64_t bi = rg / n_q, r = rg % n_q;
  const int64_t plane = (int64_t)split * n_seq * n_pad;
  float m = -3.0e38f;
  for (int c = 0; c < split; ++c) m = fmaxf(m, pst[((int64_t)c * n_seq + bi) * n_pad + r]);
  float l = 0.f, h = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c = 0; c < split; ++c) {
    const int64_t idx = ((int64_t)c * n_seq + bi) * n_pad + r;
    const float mc = pst[idx], lc = pst[plane + idx], hc = pst[2 * plane + idx];
    const float a = fast_exp2(mc - m);
    l = fmaf(a, lc, l);
    h = fmaf(a, fmaf(mc - m, lc, hc), h);
    const float wgt = a * lc;
    const float4 v = reinterpret_cast<const float4*>(po + idx * 128)[lane];
    acc.x = fmaf(wgt, v.x, acc.x);
    acc.y = fmaf(wgt, v.y, acc.y);
    acc.z = fmaf(wgt, v.z, acc.z);
    acc.w = fmaf(wgt, v.w, acc.w);
  }
  const float inv = 1.f / l;
  uint2 w;
  w.x = Elem<T>::pack(acc.x * inv, acc.y * inv);
  w.y = Elem<T>::pack(acc.z * inv, acc.w * inv);
  reinterpret_cast<uint2*>(o + view_offset(ov, n1, n2, bi, r))[lane] = w;
  if (lane == 0) {
    const float lg = log2f(l);
    if (lse) lse[bi * n_q + r] = m + lg;
    if (ent) ent[bi * n_q + r] = (lg - h / l) * kLn2;
  }
}

// Key-range split of the d = dv = 128 kernel: minimise waves x (key tiles per CTA + ~5 tiles of
// fixed cost: Q load, TMEM set-up, merge and store), never leaving a chunk without a tile.
int fwd2_split(int64_t batch, int n_q, int n_kv) {
  if (batch <= 0 || n_q <= 0) return 1;
  const int64_t n_qt = (n_q + 255) / 256;  // CTAs per sequence and key chunk: two query tiles each
  const int nkt = (n_kv + 127) / 128;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  int best = 1;
  int64_t best_cost = 0;
  for (int ks = 1; ks <= 8; ++ks) {
    const int per = (nkt + ks - 1) / ks;
    if ((ks - 1) * per >= nkt) break;
    const int64_t waves = (n_qt * batch * ks + sms - 1) / sms;
    const int64_t cost = waves * (per + 5);
    if (ks == 1 || cost * 100 < best_cost * 90) {  // a split must gain 10 % (merge pass)
      best = ks;
      best_cost = cost;
    }
  }
  return best;
}

int64_t round_up256(int64_t x) { return (x + 255) / 256 * 256; }

// Workspace of a split: partial O [split][batch][n_pad][128] fp32, then the (m, l, h) planes.
int64_t split_bytes(int split, int64_t batch, int n_q) {
  if (split <= 1) return 0;
  const int64_t n_pad = (n_q + 127) / 128 * 128;
  return round_up256((int64_t)split * batch * n_pad * 128 * 4) + round_up256(3 * (int64_t)split * batch * n_pad * 4);
}

// ---------------------------------------------------------------------------------- host side
template <typename T, int XA, bool VK, int NSLOT, bool ENT, bool F8 = false>
cudaError_t launch(const Sm100FwdParams& p, int64_t batch, cudaStream_t st) {
  using C = FwdCfg<XA, VK, NSLOT, F8>;
  auto kern = fea_fwd_sm100_kernel<T, XA, VK, NSLOT, ENT, F8>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.n_qtiles * batch;
  if (blocks > 0x7fffffff || batch > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, kThreads, C::SMEM, st>>>(p);
  return cudaGetLastError();
}

template <typename T, bool VK, bool ENT, int NS = 2, bool F8 = false>
cudaError_t launch2(const Sm100FwdParams& p, int64_t batch, cudaStream_t st) {
  using C = Fwd2Cfg<VK, NS, F8>;
  auto kern = fea_fwd2_sm100_kernel<T, VK, ENT, NS, F8>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)((p.n_qtiles + NS - 1) / NS) * p.kv_split * batch;  // NS query tiles per CTA
  if (blocks > 0x7fffffff || batch > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, C::THREADS, C::SMEM, st>>>(p);
  return cudaGetLastError();
}

// V aliasing K: the one-stream kernel (two CTAs per SM, S in halves) hides the Q load and the
// epilogue of one CTA under the other's key loop; it runs every unsplit key range (measured faster
// than the two-stream kernel from 1560 to 32768 keys). A split key range keeps the two-stream kernel.
bool fwd_one_stream(int n_kv, int kv_split) { (void)n_kv; return kv_split == 1; }

template <typename T, bool ENT>
cudaError_t dispatch(const Sm100FwdParams& p, int64_t batch, int dv, int dv1, bool vk, bool e4m3, cudaStream_t st) {
  if (e4m3) {  // the R steps: V aliasing K, without (dv = 128) or with a second value tensor
    if (!vk || p.kv_split != 1) return cudaErrorNotSupported;
    if (dv == 128) return launch2<T, true, ENT, 1, true>(p, batch, st);
    if (dv == 256 && dv1 == 128) return launch<T, 2, true, 4, ENT, true>(p, batch, st);
    return cudaErrorNotSupported;
  }
  if (vk) {
    if (dv == 128 && fwd_one_stream(p.n_kv, p.kv_split)) return launch2<T, true, ENT, 1>(p, batch, st);
    if (dv == 128) return launch2<T, true, ENT>(p, batch, st);
    if (dv == 256 && dv1 == 128) return launch<T, 2, true, 3, ENT>(p, batch, st);
  } else {
    // d = 64: the 128-column kernel over 64-column q / k maps (their second atoms load as zeros);
    // with dv = 64 the v map loads zeros too and the second half of O is clipped on store
    if (dv == 128 || dv == 64) return launch2<T, false, ENT>(p, batch, st);
    if (dv == 256) return launch<T, 4, false, 2, ENT>(p, batch, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace

bool fea_fwd_sm100_supported(int d, int dv, int dv1, bool vk) {
  // d = 64: 64-column q / k maps (second atoms load as zeros), v and o 64 or 128 wide; with V
  // aliasing K, only [K | V2] (dv = 128): the K tile's second atom holds V2. No key-range split.
  if (d == 64) return vk ? dv == 128 && dv1 == 64 : (dv == 64 || dv == 128) && dv1 == dv;
  if (d != 128) return false;
  if (vk) return dv == 128 || (dv == 256 && dv1 == 128);
  return (dv == 128 || dv == 256) && dv1 == dv;
}

bool fea_fwd_sm100_e4m3_supported(int d, int dv, int dv1, bool vk) {
  // e4m3 operands: the VMonarch R-step forms (D = 128, V aliasing K, with or without [K | V2])
  return d == 128 && vk && (dv == 128 || (dv == 256 && dv1 == 128));
}

int64_t fea_fwd_sm100_workspace_bytes(int64_t batch, int n_q, int n_kv, int d, int dv, int dv1, bool vk) {
  if (d != 128 || !fea_fwd_sm100_supported(d, dv, dv1, vk) || dv != 128) return 0;  // only the two-stream kernel splits (d = 128)
  return split_bytes(fwd2_split(batch, n_q, n_kv), batch, n_q);
}

int fea_fwd_sm100_split(int64_t batch, int n_q, int n_kv, int d, int dv, const void* work, int64_t work_bytes) {
  if (d != 128 || dv != 128 || !work) return 1;
  const int ks = fwd2_split(batch, n_q, n_kv);
  return (ks > 1 && work_bytes >= split_bytes(ks, batch, n_q)) ? ks : 1;
}

cudaError_t fea_fwd_sm100(const FwdParams& fp, int64_t batch, int d, int dv, bool ent, bool bf16, bool vk,
                          cudaStream_t st) {
  Sm100FwdParams p;
  const int dv1 = fp.dv1;
  const int n1 = fp.n1, n2 = fp.n2;
  if (fp.e4m3) {
    // e4m3 operands: one 128-byte box per 128-column row segment; only the R-step forms
    if (d != 128 || !vk || !fea_fwd_sm100_e4m3_supported(d, dv, dv1, vk)) return cudaErrorNotSupported;
    if (!tma::make_map_view_e4m3(&p.tm_q, fp.q, d, fp.n_q, batch, fp.qv, n1, n2, 128) ||
        !tma::make_map_view_e4m3(&p.tm_k, fp.k, d, fp.n_kv, batch, fp.kv, n1, n2, 128))
      return cudaErrorInvalidValue;
    if (dv > dv1 && !tma::make_map_view_e4m3(&p.tm_x, fp.v2, dv - dv1, fp.n_kv, batch, fp.v2v, n1, n2, 128))
      return cudaErrorInvalidValue;
    if (dv == dv1) p.tm_x = p.tm_k;
  } else {
    if (!tma::make_map_view(&p.tm_q, fp.q, bf16, d, fp.n_q, batch, fp.qv, n1, n2, 128) ||
        !tma::make_map_view(&p.tm_k, fp.k, bf16, d, fp.n_kv, batch, fp.kv, n1, n2, 128))
      return cudaErrorInvalidValue;
    if (vk) {
      if (dv > dv1 && !tma::make_map_view(&p.tm_x, fp.v2, bf16, dv - dv1, fp.n_kv, batch, fp.v2v, n1, n2, 128))
        return cudaErrorInvalidValue;
      if (dv == dv1) p.tm_x = p.tm_k;
    } else if (!tma::make_map_view(&p.tm_x, fp.v, bf16, dv, fp.n_kv, batch, fp.vv, n1, n2, 128)) {
      return cudaErrorInvalidValue;
    }
  }
  if (!tma::make_map_view(&p.tm_o, fp.o, bf16, dv, fp.n_q, batch, fp.ov, n1, n2, 128)) return cudaErrorInvalidValue;
  p.n1 = n1;
  p.n2 = n2;
  p.wait_limit = fp.wait_limit;
  p.hold_loads = fp.hold_loads;
  p.k_hi_x = (d == 64 && vk && dv == 128) ? 1 : 0;
  p.lse = fp.lse;
  p.ent = fp.ent;
  p.n_q = fp.n_q;
  p.n_kv = fp.n_kv;
  p.n_qtiles = (fp.n_q + 127) / 128;
  p.scale_log2 = fp.scale_log2;
  // key-range split (two-stream kernel, with a large enough workspace)
  const int nkt = (fp.n_kv + 127) / 128;
  p.kv_split = fp.e4m3 ? 1 : fea_fwd_sm100_split(batch, fp.n_q, fp.n_kv, d, dv, fp.work, fp.work_bytes);
  p.kt_per = (nkt + p.kv_split - 1) / p.kv_split;
  p.n_seq = (int)batch;
  p.n_pad = (fp.n_q + 127) / 128 * 128;
  float* po = nullptr;
  p.pst = nullptr;
  if (p.kv_split > 1) {
    po = static_cast<float*>(fp.work);
    p.pst = reinterpret_cast<float*>(static_cast<char*>(fp.work) +
                                     round_up256((int64_t)p.kv_split * batch * p.n_pad * 128 * 4));
    if (!tma::make_map_f32(&p.tm_po, po, 128, p.n_pad, (int64_t)p.kv_split * batch, p.n_pad * 128, 128))
      return cudaErrorInvalidValue;
  }
  cudaError_t e;
  const bool f8 = fp.e4m3;
  if (bf16)
    e = ent ? dispatch<__nv_bfloat16, true>(p, batch, dv, dv1, vk, f8, st)
            : dispatch<__nv_bfloat16, false>(p, batch, dv, dv1, vk, f8, st);
  else
    e = ent ? dispatch<__half, true>(p, batch, dv, dv1, vk, f8, st)
            : dispatch<__half, false>(p, batch, dv, dv1, vk, f8, st);
  if (e != cudaSuccess || p.kv_split == 1) return e;
  const int64_t rows = batch * fp.n_q;
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  if (bf16)
    fwd_split_merge_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(
        po, p.pst, p.kv_split, batch, p.n_pad, fp.n_q, static_cast<__nv_bfloat16*>(fp.o), fp.ov, n1, n2, fp.lse,
        ent ? fp.ent : nullptr);
  else
    fwd_split_merge_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(po, p.pst, p.kv_split, batch, p.n_pad, fp.n_q,
                                                                      static_cast<__half*>(fp.o), fp.ov, n1, n2, fp.lse,
                                                                      ent ? fp.ent : nullptr);
  return cudaGetLastError();
}

cudaError_t fea_fwd_sm100_status(cudaStream_t st, int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_fwd_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && *out) e = cudaMemcpyToSymbolAsync(g_fwd_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e;
}

}  // namespace vmb
