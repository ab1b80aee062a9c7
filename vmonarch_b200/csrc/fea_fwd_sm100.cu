// FlashEntropyAttention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), D = 128.
//
// Reference semantics: video_monarch_attention/kernel.py:32-151 (online softmax with the running
// entropy accumulator h = sum p (x - m), E = (log2 l - h / l) ln 2, LSE2 = m + log2 l).
//
// CTA = one 128-row query tile of one sequence; 6 warps:
//   warp 0   TMA producer (Q once, then K / V tiles into an NSLOT-deep ring) + TMEM allocator
//   warp 1   MMA issuer (one elected lane of the converged warp): S = Q K^T into a double-buffered
//            TMEM S, O += P V with P read from TMEM (the bf16 probabilities are written over the
//            first 64 columns of S)
//   warps 2-5 softmax + epilogue: thread = one query row = one TMEM lane; the whole 128-key row of
//            S is in registers, so max / sum / entropy need no shuffles.
// TMEM (512 columns): S0 [0,128), S1 [128,256), O [256, 256 + NV).
// The max is rescaled lazily: O, l and h keep a stale reference max m_ref until a tile's max
// exceeds it by more than 8 (p <= 256), the only point where O is read back and rescaled. The
// entropy identity E = log l - h / l holds for any reference, so this is exact.
//
// Shared-memory ring slot = [K tile (2 swizzle atoms of 128 keys x 64 cols)][X tile]:
//   separate V   : X = V (NV/64 atoms); P V reads the X atoms                 (plain FEA, recompute)
//   V aliases K  : X = V2 (0 or 2 atoms); P V reads K and V2 as one contiguous (VMonarch R steps,
//                  N = 128 + 64*XA operand, so the non-last R steps load K only vmonarch.py:50)
// Tails: TMA zero-fills rows past n_q / n_kv per sequence (3-D maps [batch][rows][cols]); keys
// past n_kv are masked to p = 0; the O tile is written with a TMA store, which clips rows >= n_q.
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

constexpr int kThreads = 192;
constexpr int kAtom = 128 * 128;  // bytes of one swizzle atom column block: 128 rows x 128 B
constexpr float kRescaleThreshold = 8.0f;

struct Sm100FwdParams {
  CUtensorMap tm_q, tm_k, tm_x, tm_o;
  float* lse;
  float* ent;
  int n_q, n_kv, n_qtiles;
  float scale_log2;
};

template <int XA, bool VK, int NSLOT>
struct FwdCfg {
  static constexpr int NV = VK ? 128 + 64 * XA : 64 * XA;  // N of the P V MMA = output columns
  static constexpr int SLOT = (2 + XA) * kAtom;            // bytes per ring slot
  static constexpr int PV_OFF = VK ? 0 : 2 * kAtom;         // start of the P V operand in a slot
  static constexpr int Q_BYTES = 2 * kAtom;
  static constexpr int SMEM = 1024 + Q_BYTES + NSLOT * SLOT;
  static_assert(NV == 128 || NV == 256, "P V width must be 128 or 256");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Three-input max (sm_100: one instruction).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Max of the raw scores of one 128-key row (keys >= valid ignored when MASK). The scale is applied
// to the max afterwards, as the reference does (kernel.py:45: max(qk) * qk_scale). Four
// independent chains of three-input maxima: with one softmax warp per scheduler a single long
// chain is pure latency.
template <bool MASK>
__device__ __forceinline__ float row_max_raw(const uint32_t (&sr)[128], int valid) {
  auto at = [&](int i) { return (MASK && i >= valid) ? -1e30f : __uint_as_float(sr[i]); };
  float mr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) mr[k] = fmax3(at(3 * k), at(3 * k + 1), at(3 * k + 2));
#pragma unroll
  for (int i = 12; i < 128; i += 2) mr[(i >> 1) & 3] = fmax3(mr[(i >> 1) & 3], at(i), at(i + 1));
  return fmax3(fmaxf(mr[0], mr[1]), mr[2], mr[3]);
}

// p = 2^(s * scale - m) for one 128-key row, packed to the element type, with the row sum l and
// the entropy sum h = sum p (x - m). Pairs of keys go through the packed f32x2 FMA / add (one
// instruction per pair) into two chains each. Keys >= valid (MASK) get x - m = -1e30, so p = 0
// and p (x - m) = 0 exactly.
template <typename T, bool ENT, bool MASK>
__device__ __forceinline__ void probs_row(const uint32_t (&sr)[128], uint32_t (&pk)[64], float sc, float m, int valid,
                                          float& l, float& h) {
  float2 la[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float2 ha[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  const float2 sc2 = make_float2(sc, sc), nm2 = make_float2(-m, -m);
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    float2 d = __ffma2_rn(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sc2, nm2);
    if (MASK) {
      if (2 * i >= valid) d.x = -1e30f;
      if (2 * i + 1 >= valid) d.y = -1e30f;
    }
    const float2 pp = make_float2(fast_exp2(d.x), fast_exp2(d.y));
    la[i & 1] = __fadd2_rn(la[i & 1], pp);
    if (ENT) ha[i & 1] = __ffma2_rn(pp, d, ha[i & 1]);
    pk[i] = Elem<T>::pack(pp.x, pp.y);
  }
  l += (la[0].x + la[0].y) + (la[1].x + la[1].y);
  if (ENT) h += (ha[0].x + ha[0].y) + (ha[1].x + ha[1].y);
}

template <typename T, int XA, bool VK, int NSLOT, bool ENT>
__global__ void __launch_bounds__(kThreads, 1) fea_fwd_sm100_kernel(const __grid_constant__ Sm100FwdParams p) {
  using C = FwdCfg<XA, VK, NSLOT>;
  constexpr bool kBf16 = Elem<T>::is_bf16;
  constexpr uint32_t IDESC_S = idesc_f16(kBf16, 128, 128, false, false);
  constexpr uint32_t IDESC_PV = idesc_f16(kBf16, 128, C::NV, false, true);

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[6 + 3 * NSLOT];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bi = blockIdx.x / p.n_qtiles;
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
      mbar_init(BAR_PFULL(b), 128);
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
    if (lane == 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      if (XA > 0) prefetch_tmap(&p.tm_x);
      mbar_expect_tx(BAR_Q, C::Q_BYTES);
      tma_load_3d(sQ, &p.tm_q, 0, q0, bi, BAR_Q);
      tma_load_3d(sQ + kAtom, &p.tm_q, 64, q0, bi, BAR_Q);
      int armed[NSLOT];
      for (int s = 0; s < NSLOT; ++s) armed[s] = 0;
      for (int j = 0; j < n_kt; ++j) {
        const int s = j % NSLOT;
        if (j >= NSLOT && !mbar_wait(BAR_EMPTY(s), ((j / NSLOT) - 1) & 1, abort, &g_fwd_err, 1)) break;
        const uint32_t slot = sRing + s * C::SLOT;
        mbar_expect_tx(BAR_KFULL(s), 2 * kAtom);
        tma_load_3d(slot, &p.tm_k, 0, j * 128, bi, BAR_KFULL(s));
        tma_load_3d(slot + kAtom, &p.tm_k, 64, j * 128, bi, BAR_KFULL(s));
        if (XA > 0) {
          mbar_expect_tx(BAR_VFULL(s), XA * kAtom);
          for (int a = 0; a < XA; ++a) tma_load_3d(slot + (2 + a) * kAtom, &p.tm_x, 64 * a, j * 128, bi, BAR_VFULL(s));
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
    auto wwait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, &g_fwd_err, code));
    };
    bool ok = wwait(BAR_Q, 0, 2);
    auto issue_s = [&](int j) -> bool {
      const int s = j % NSLOT;
      if (!wwait(BAR_KFULL(s), (j / NSLOT) & 1, 2)) return false;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t kb = sRing + s * C::SLOT;
        const uint32_t d = tmem + (uint32_t)((j & 1) * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          mma_ss(d, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), IDESC_S, kk > 0);
        }
        mma_commit(BAR_SFULL(j & 1));
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = issue_s(0);
    if (ok && n_kt > 1) ok = issue_s(1);
    for (int j = 0; ok && j < n_kt; ++j) {
      const int s = j % NSLOT;
      if (!wwait(BAR_PFULL(j & 1), (j >> 1) & 1, 4)) break;
      if (XA > 0 && !wwait(BAR_VFULL(s), (j / NSLOT) & 1, 4)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t vb = sRing + s * C::SLOT + C::PV_OFF;
        const uint32_t a_tm = tmem + (uint32_t)((j & 1) * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts(tmem + 256, a_tm + kk * 8, smem_desc_sw128(vb + kk * 2048, kAtom, 1024), IDESC_PV,
                 (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(BAR_EMPTY(s));
      }
      __syncwarp();
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
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    float m_ref = -1e30f, l = 0.f, h = 0.f;
    int pv_waited = -1;
    bool ok = true;

    auto warp_wait = [&](uint32_t bar, uint32_t parity, int code) -> bool {
      const bool mine = mbar_wait(bar, parity, abort, &g_fwd_err, code);
      return __all_sync(0xffffffffu, mine);
    };
    // PV[t] is committed to EMPTY[t % NSLOT]. Waiting for every t in order keeps the wait at most
    // one phase behind: PV[t + NSLOT] needs P[t + NSLOT - 1], which this warpgroup has not written
    // when it waits for PV[t] (t <= j - 1 while it works on tile j).
    auto wait_pv = [&](int t) -> bool {
      while (pv_waited < t) {
        const int u = pv_waited + 1;
        if (!warp_wait(BAR_EMPTY(u % NSLOT), (u / NSLOT) & 1, 8)) return false;
        pv_waited = u;
      }
      return true;
    };

    for (int j = 0; j < n_kt; ++j) {
      if (!warp_wait(BAR_SFULL(j & 1), (j >> 1) & 1, 8)) { ok = false; break; }
      tc_fence_after();
      // S[j] complete implies PV[j-2] complete: consume that phase to keep the bookkeeping exact
      if (j >= 2 && !wait_pv(j - 2)) { ok = false; break; }
      const uint32_t tS = tmem + lane_off + (uint32_t)((j & 1) * 128);
      uint32_t sr[128];
      tmem_ld32(tS + 0, sr);
      tmem_ld32(tS + 32, sr + 32);
      tmem_ld32(tS + 64, sr + 64);
      tmem_ld32(tS + 96, sr + 96);
      tmem_wait_ld();
      const int valid = p.n_kv - j * 128;  // same for every thread: the branches below are uniform
      const float mx = (valid < 128 ? row_max_raw<true>(sr, valid) : row_max_raw<false>(sr, 128)) * p.scale_log2;
      if (j == 0) {
        m_ref = mx;
      } else if (__any_sync(0xffffffffu, mx > m_ref + kRescaleThreshold)) {
        // The rescale touches TMEM with warp-collective loads / stores and waits on a barrier, so
        // the decision is taken per warp: every lane whose max grew adopts it (alpha < 1), the
        // others keep their reference (alpha = 1).
        if (!wait_pv(j - 1)) { ok = false; break; }
        tc_fence_after();
        const float m_new = fmaxf(m_ref, mx);
        const float alpha = fast_exp2(m_ref - m_new);
#pragma unroll 1
        for (int c = 0; c < C::NV / 32; ++c) {
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
      }
      uint32_t pk[64];
      if (valid < 128) probs_row<T, ENT, true>(sr, pk, p.scale_log2, m_ref, valid, l, h);
      else probs_row<T, ENT, false>(sr, pk, p.scale_log2, m_ref, 128, l, h);
      tmem_st32(tS + 0, pk);
      tmem_st32(tS + 32, pk + 32);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR_PFULL(j & 1));
    }

    if (ok) ok = wait_pv(n_kt - 1);
    tc_fence_after();
    // epilogue: O / l -> bf16 in the (now idle) ring, TMA store; LSE and entropy per row
    const uint32_t stage = sRing;
    if (ok) {
      const float inv = 1.f / l;
#pragma unroll 1
      for (int c = 0; c < C::NV / 32; ++c) {
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
      if (grow < p.n_q) {
        const float lg = log2f(l);
        const int64_t idx = (int64_t)bi * p.n_q + grow;
        if (p.lse) p.lse[idx] = m_ref + lg;
        if (ENT && p.ent) p.ent[idx] = (lg - h / l) * kLn2;
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1, 128);
    if (warp == 2 && lane == 0 && !*abort) {
      for (int a = 0; a < C::NV / 64; ++a) tma_store_3d(&p.tm_o, 64 * a, q0, bi, stage + a * kAtom);
      tma_store_commit_and_wait();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------- host side
template <typename T, int XA, bool VK, int NSLOT, bool ENT>
cudaError_t launch(const Sm100FwdParams& p, int64_t batch, cudaStream_t st) {
  using C = FwdCfg<XA, VK, NSLOT>;
  auto kern = fea_fwd_sm100_kernel<T, XA, VK, NSLOT, ENT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.n_qtiles * batch;
  if (blocks > 0x7fffffff || batch > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, kThreads, C::SMEM, st>>>(p);
  return cudaGetLastError();
}

template <typename T, bool ENT>
cudaError_t dispatch(const Sm100FwdParams& p, int64_t batch, int dv, int dv1, bool vk, cudaStream_t st) {
  if (vk) {
    if (dv == 128) return launch<T, 0, true, 4, ENT>(p, batch, st);
    if (dv == 256 && dv1 == 128) return launch<T, 2, true, 3, ENT>(p, batch, st);
  } else {
    if (dv == 128) return launch<T, 2, false, 3, ENT>(p, batch, st);
    if (dv == 256) return launch<T, 4, false, 2, ENT>(p, batch, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace

bool fea_fwd_sm100_supported(int d, int dv, int dv1, bool vk) {
  if (d != 128) return false;
  if (vk) return dv == 128 || (dv == 256 && dv1 == 128);
  return (dv == 128 || dv == 256) && dv1 == dv;
}

cudaError_t fea_fwd_sm100(const FwdParams& fp, int64_t batch, int d, int dv, bool ent, bool bf16, bool vk,
                          cudaStream_t st) {
  Sm100FwdParams p;
  const int dv1 = fp.dv1;
  if (!tma::make_map(&p.tm_q, fp.q, bf16, d, fp.n_q, batch, fp.q_bs, 128)) return cudaErrorInvalidValue;
  if (!tma::make_map(&p.tm_k, fp.k, bf16, d, fp.n_kv, batch, fp.k_bs, 128)) return cudaErrorInvalidValue;
  if (vk) {
    if (dv > dv1 && !tma::make_map(&p.tm_x, fp.v2, bf16, dv - dv1, fp.n_kv, batch, fp.v2_bs, 128)) return cudaErrorInvalidValue;
    if (dv == dv1) p.tm_x = p.tm_k;
  } else {
    if (!tma::make_map(&p.tm_x, fp.v, bf16, dv, fp.n_kv, batch, fp.v_bs, 128)) return cudaErrorInvalidValue;
  }
  if (!tma::make_map(&p.tm_o, fp.o, bf16, dv, fp.n_q, batch, fp.o_bs, 128)) return cudaErrorInvalidValue;
  p.lse = fp.lse;
  p.ent = fp.ent;
  p.n_q = fp.n_q;
  p.n_kv = fp.n_kv;
  p.n_qtiles = (fp.n_q + 127) / 128;
  p.scale_log2 = fp.scale_log2;
  if (bf16)
    return ent ? dispatch<__nv_bfloat16, true>(p, batch, dv, dv1, vk, st)
               : dispatch<__nv_bfloat16, false>(p, batch, dv, dv1, vk, st);
  return ent ? dispatch<__half, true>(p, batch, dv, dv1, vk, st) : dispatch<__half, false>(p, batch, dv, dv1, vk, st);
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
