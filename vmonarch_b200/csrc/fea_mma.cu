// FlashEntropyAttention on warp-level MMA (mma.sync m16n8k16), every (D, Dv) the reference accepts:
// D, Dv in {16, 32, 64, 128, 256} with Dv % D == 0 (video_monarch_attention/kernel.py:260, 324).
//
// Forward  (reference: video_monarch_attention/kernel.py:32-67 inner loop, 106-151 kernel):
//   per query row i:  x_ij = s_ij * sm_scale * log2(e),  m = running max,  p = 2^(x - m)
//   l = sum p,  h = sum p * (x - m)   (rescaled online exactly like l, kernel.py:49-50)
//   o = sum p v / l,  LSE2 = m + log2 l,  E = (log2 l - h / l) * ln 2   (kernel.py:146-148)
// Backward (reference: kernel.py:154-313):
//   P = 2^(x - LSE2),  dP = dO V^T,  dS = P (dP - c_i - g_i x_ij) with
//   c_i = delta_i + dE_i (E_i - LSE_i),  g_i = dE_i ln 2   (kernel.py:165-167, 202, 241 folded
//   into one per-row constant), dV = P^T dO, dK = sm_scale dS^T Q, dQ = sm_scale dS K.
//   One CTA owns 64 keys and walks all query tiles: 5 MMAs per tile pair (the reference's
//   _attn_bwd recomputes S and dP in separate dK/dV and dQ halves: 7). dQ is accumulated in fp32
//   with vector atomics.
//
// Tails are handled in-kernel: rows past n_q / n_kv are zero-filled on load, keys past n_kv are
// masked to p = 0, so no padded copies of the inputs are made (the reference pads to 128,
// kernel.py:399-400).
#include "common.cuh"
#include "fea_params.h"
#include "launch.h"

namespace vmb {

// ============================================================================ forward
template <typename T, int D, int DV, bool ENT>
__global__ void __launch_bounds__(128) fea_fwd_mma_kernel(const FwdParams p) {
  constexpr int BM = 64, BN = 64;
  constexpr int DCH = D / 8, VCH = DV / 8;
  // shared-memory rows are at least 64 elements wide (the swizzle spans 8 chunks of 16 bytes);
  // for head dims 16 and 32 only the first D / DV columns are loaded and read
  constexpr int DP = D < 64 ? 64 : D, VP = DV < 64 ? 64 : DV;
  constexpr int DPCH = DP / 8, VPCH = VP / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  T* sQ = reinterpret_cast<T*>(smem_raw);
  T* sK = sQ + BM * DP;       // [2][BN*DP]
  T* sV = sK + 2 * BN * DP;   // [2][BN*VP]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bi = blockIdx.x / p.n_qtiles;
  const int q0 = (blockIdx.x % p.n_qtiles) * BM;
  const T* gq = static_cast<const T*>(p.q) + bi * p.q_bs;
  const T* gk = static_cast<const T*>(p.k) + bi * p.k_bs;
  const T* gv = static_cast<const T*>(p.v) + bi * p.v_bs;
  const T* gv2 = p.v2 ? static_cast<const T*>(p.v2) + bi * p.v2_bs : nullptr;
  const int dv1 = p.dv1, dv2 = DV - p.dv1;

  for (int c = tid; c < BM * DCH; c += 128) {
    const int r = c / DCH, ch = c % DCH, gr = q0 + r;
    const T* src = gq + (int64_t)min(gr, p.n_q - 1) * D + ch * 8;
    cp_async16(smem_u32(sQ + swz<DPCH>(r, ch)), src, gr < p.n_q ? 16 : 0);
  }
  auto load_kv = [&](int t, int stage) {
    const int k0 = t * BN;
    T* dK = sK + stage * BN * DP;
    T* dV = sV + stage * BN * VP;
    for (int c = tid; c < BN * DCH; c += 128) {
      const int r = c / DCH, ch = c % DCH, gr = k0 + r;
      const T* src = gk + (int64_t)min(gr, p.n_kv - 1) * D + ch * 8;
      cp_async16(smem_u32(dK + swz<DPCH>(r, ch)), src, gr < p.n_kv ? 16 : 0);
    }
    for (int c = tid; c < BN * VCH; c += 128) {
      const int r = c / VCH, ch = c % VCH, gr = min(k0 + r, p.n_kv - 1), col = ch * 8;
      const T* src = col < dv1 ? gv + (int64_t)gr * dv1 + col : gv2 + (int64_t)gr * dv2 + (col - dv1);
      cp_async16(smem_u32(dV + swz<VPCH>(r, ch)), src, k0 + r < p.n_kv ? 16 : 0);
    }
  };

  load_kv(0, 0);
  cp_async_commit();

  float o_acc[DV / 8][4];
#pragma unroll
  for (int j = 0; j < DV / 8; ++j) o_acc[j][0] = o_acc[j][1] = o_acc[j][2] = o_acc[j][3] = 0.f;
  float m_r[2] = {-1e30f, -1e30f}, l_r[2] = {0.f, 0.f}, h_r[2] = {0.f, 0.f};
  const int n_kt = (p.n_kv + BN - 1) / BN;

  for (int t = 0; t < n_kt; ++t) {
    if (t + 1 < n_kt) load_kv(t + 1, (t + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* cK = sK + (t & 1) * BN * DP;
    const T* cV = sV + (t & 1) * BN * VP;

    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(smem_u32(sQ + swz<DPCH>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4))), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(smem_u32(cK + swz<DPCH>(r, kk * 2 + ((lane >> 3) & 1))), b0, b1, b2, b3);
        mma16816<T>(s[2 * np], a, b0, b1);
        mma16816<T>(s[2 * np + 1], a, b2, b3);
      }
    }

    const bool tail = (t + 1) * BN > p.n_kv;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * p.scale_log2;
        if (tail && t * BN + j * 8 + (lane & 3) * 2 + (e & 1) >= p.n_kv) x = -1e30f;
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float alpha[2], lsum[2] = {0.f, 0.f}, hsum[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 2; ++i) alpha[i] = fast_exp2(m_r[i] - mx[i]);
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float d = s[j][e] - mx[e >> 1];
        const float pv = fast_exp2(d);
        s[j][e] = pv;
        lsum[e >> 1] += pv;
        if (ENT) hsum[e >> 1] = fmaf(pv, d, hsum[e >> 1]);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (ENT) h_r[i] = alpha[i] * fmaf(m_r[i] - mx[i], l_r[i], h_r[i]) + hsum[i];
      l_r[i] = fmaf(alpha[i], l_r[i], lsum[i]);
      m_r[i] = mx[i];
    }
#pragma unroll
    for (int j = 0; j < DV / 8; ++j) {
      o_acc[j][0] *= alpha[0];
      o_acc[j][1] *= alpha[0];
      o_acc[j][2] *= alpha[1];
      o_acc[j][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t a[4];
      a[0] = Elem<T>::pack(s[2 * kk][0], s[2 * kk][1]);
      a[1] = Elem<T>::pack(s[2 * kk][2], s[2 * kk][3]);
      a[2] = Elem<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = Elem<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < DV / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        ldsm_x4_t(smem_u32(cV + swz<VPCH>(r, np * 2 + (lane >> 4))), b0, b1, b2, b3);
        mma16816<T>(o_acc[2 * np], a, b0, b1);
        mma16816<T>(o_acc[2 * np + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }

  T* go = static_cast<T*>(p.o) + bi * p.o_bs;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float l = l_r[i], h = h_r[i];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (ENT) {
      h += __shfl_xor_sync(0xffffffffu, h, 1);
      h += __shfl_xor_sync(0xffffffffu, h, 2);
    }
    const int row = q0 + warp * 16 + (lane >> 2) + i * 8;
    if (row < p.n_q) {
      const float inv = 1.f / l;
      uint32_t* orow = reinterpret_cast<uint32_t*>(go + (int64_t)row * DV);
#pragma unroll
      for (int j = 0; j < DV / 8; ++j)
        orow[(j * 8 + (lane & 3) * 2) >> 1] = Elem<T>::pack(o_acc[j][2 * i] * inv, o_acc[j][2 * i + 1] * inv);
      if ((lane & 3) == 0) {
        const float lg = log2f(l);
        if (p.lse) p.lse[bi * p.n_q + row] = m_r[i] + lg;
        if (ENT && p.ent) p.ent[bi * p.n_q + row] = (lg - h / l) * kLn2;
      }
    }
  }
}

// ============================================================================ backward
// One CTA = 4 warps = 64 keys (16 per warp); walks all query tiles of BQ = 32 rows.
// VK: v aliases k (dv1 == D). Then the value-gradient of columns [0, D) is the same tensor as
// the key gradient and is accumulated straight into the dK accumulator.
template <typename T, int D, int DV, bool VK>
__global__ void __launch_bounds__(128) fea_bwd_mma_kernel(const BwdParams p) {
  constexpr int BN = 64, BQ = 32, SDS = BQ + 8;
  constexpr int DCH = D / 8, VCH = DV / 8;
  constexpr int DP = D < 64 ? 64 : D, VP = DV < 64 ? 64 : DV;  // shared-memory row widths (>= 64)
  constexpr int DPCH = DP / 8, VPCH = VP / 8;
  constexpr int DVA = VK ? DV - D : DV;  // columns held by the separate dV accumulator
  extern __shared__ __align__(128) uint8_t smem_raw[];
  T* sK = reinterpret_cast<T*>(smem_raw);     // BN*DP
  T* sV = sK + BN * DP;                       // BN*VP
  T* sQ = sV + BN * VP;                       // [2][BQ*DP]
  T* sO = sQ + 2 * BQ * DP;                   // [2][BQ*VP]  (dO)
  T* sS = sO + 2 * BQ * VP;                   // BN*SDS  dS^T (scaled)
  float* sL = reinterpret_cast<float*>(sS + BN * SDS);  // [2][BQ]
  float* sC = sL + 2 * BQ;
  float* sG = sC + 2 * BQ;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bi = blockIdx.x / p.n_ktiles;
  const int k0 = (blockIdx.x % p.n_ktiles) * BN;
  const T* gq = static_cast<const T*>(p.q) + bi * p.q_bs;
  const T* gk = static_cast<const T*>(p.k) + bi * p.k_bs;
  const T* gv = static_cast<const T*>(p.v) + bi * p.v_bs;
  const T* gv2 = p.v2 ? static_cast<const T*>(p.v2) + bi * p.v2_bs : nullptr;
  const T* gdo = static_cast<const T*>(p.dout) + bi * p.do_bs;
  const float* glse = p.lse + bi * p.n_q;
  const float* gcc = p.cc + bi * p.n_q;
  const float* ggg = p.gg + bi * p.n_q;
  float* gdq = p.dq + bi * p.dq_bs;
  const int dv1 = p.dv1, dv2 = DV - p.dv1;

  for (int c = tid; c < BN * DCH; c += 128) {
    const int r = c / DCH, ch = c % DCH, gr = k0 + r;
    cp_async16(smem_u32(sK + swz<DPCH>(r, ch)), gk + (int64_t)min(gr, p.n_kv - 1) * D + ch * 8, gr < p.n_kv ? 16 : 0);
  }
  for (int c = tid; c < BN * VCH; c += 128) {
    const int r = c / VCH, ch = c % VCH, gr = min(k0 + r, p.n_kv - 1), col = ch * 8;
    const T* src = col < dv1 ? gv + (int64_t)gr * dv1 + col : gv2 + (int64_t)gr * dv2 + (col - dv1);
    cp_async16(smem_u32(sV + swz<VPCH>(r, ch)), src, k0 + r < p.n_kv ? 16 : 0);
  }
  auto load_q = [&](int t, int stage) {
    const int q0 = t * BQ;
    T* dQ = sQ + stage * BQ * DP;
    T* dO = sO + stage * BQ * VP;
    for (int c = tid; c < BQ * DCH; c += 128) {
      const int r = c / DCH, ch = c % DCH, gr = q0 + r;
      cp_async16(smem_u32(dQ + swz<DPCH>(r, ch)), gq + (int64_t)min(gr, p.n_q - 1) * D + ch * 8, gr < p.n_q ? 16 : 0);
    }
    for (int c = tid; c < BQ * VCH; c += 128) {
      const int r = c / VCH, ch = c % VCH, gr = q0 + r;
      cp_async16(smem_u32(dO + swz<VPCH>(r, ch)), gdo + (int64_t)min(gr, p.n_q - 1) * DV + ch * 8, gr < p.n_q ? 16 : 0);
    }
    if (tid < BQ) {
      const int gr = q0 + tid;
      const bool ok = gr < p.n_q;
      sL[stage * BQ + tid] = ok ? glse[gr] : __int_as_float(0x7f800000);  // +inf -> P = 0
      sC[stage * BQ + tid] = ok ? gcc[gr] : 0.f;
      sG[stage * BQ + tid] = ok ? ggg[gr] : 0.f;
    }
  };

  load_q(0, 0);
  cp_async_commit();

  float dk_acc[D / 8][4];
  float dv_acc[DVA / 8 > 0 ? DVA / 8 : 1][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) dk_acc[j][0] = dk_acc[j][1] = dk_acc[j][2] = dk_acc[j][3] = 0.f;
#pragma unroll
  for (int j = 0; j < DVA / 8; ++j) dv_acc[j][0] = dv_acc[j][1] = dv_acc[j][2] = dv_acc[j][3] = 0.f;

  const int g = lane >> 2, tq = lane & 3;
  const bool key_ok0 = k0 + warp * 16 + g < p.n_kv;
  const bool key_ok1 = k0 + warp * 16 + g + 8 < p.n_kv;
  const int n_qt = (p.n_q + BQ - 1) / BQ;

  for (int t = 0; t < n_qt; ++t) {
    if (t + 1 < n_qt) load_q(t + 1, (t + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int st = t & 1;
    const T* cQ = sQ + st * BQ * DP;
    const T* cO = sO + st * BQ * VP;
    const float* cL = sL + st * BQ;
    const float* cC = sC + st * BQ;
    const float* cG = sG + st * BQ;

    // S^T = K Q^T  and  dP^T = V dO^T   (rows: this warp's 16 keys, cols: 32 queries)
    float s[BQ / 8][4], dp[BQ / 8][4];
#pragma unroll
    for (int j = 0; j < BQ / 8; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      dp[j][0] = dp[j][1] = dp[j][2] = dp[j][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(smem_u32(sK + swz<DPCH>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4))), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int np = 0; np < BQ / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(smem_u32(cQ + swz<DPCH>(r, kk * 2 + ((lane >> 3) & 1))), b0, b1, b2, b3);
        mma16816<T>(s[2 * np], a, b0, b1);
        mma16816<T>(s[2 * np + 1], a, b2, b3);
      }
    }
#pragma unroll
    for (int kk = 0; kk < DV / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(smem_u32(sV + swz<VPCH>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4))), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int np = 0; np < BQ / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(smem_u32(cO + swz<VPCH>(r, kk * 2 + ((lane >> 3) & 1))), b0, b1, b2, b3);
        mma16816<T>(dp[2 * np], a, b0, b1);
        mma16816<T>(dp[2 * np + 1], a, b2, b3);
      }
    }
    // P^T and dS^T (dS scaled by sm_scale, it feeds dK and dQ only)
#pragma unroll
    for (int j = 0; j < BQ / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = j * 8 + tq * 2 + (e & 1);
        const float x = s[j][e] * p.scale_log2;
        float pv = fast_exp2(x - cL[qc]);
        if (!((e >> 1) ? key_ok1 : key_ok0)) pv = 0.f;
        const float ds = pv * (dp[j][e] - cC[qc] - cG[qc] * x);
        s[j][e] = pv;
        dp[j][e] = ds * p.sm_scale;
      }
    }
    // dV += P^T dO ; dK += dS^T Q (+ P^T dO[:, :D] when v aliases k)
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      uint32_t ap[4], as[4];
      ap[0] = Elem<T>::pack(s[2 * kk][0], s[2 * kk][1]);
      ap[1] = Elem<T>::pack(s[2 * kk][2], s[2 * kk][3]);
      ap[2] = Elem<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      ap[3] = Elem<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      as[0] = Elem<T>::pack(dp[2 * kk][0], dp[2 * kk][1]);
      as[1] = Elem<T>::pack(dp[2 * kk][2], dp[2 * kk][3]);
      as[2] = Elem<T>::pack(dp[2 * kk + 1][0], dp[2 * kk + 1][1]);
      as[3] = Elem<T>::pack(dp[2 * kk + 1][2], dp[2 * kk + 1][3]);
      const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(cQ + swz<DPCH>(r, np * 2 + (lane >> 4))), b0, b1, b2, b3);
        mma16816<T>(dk_acc[2 * np], as, b0, b1);
        mma16816<T>(dk_acc[2 * np + 1], as, b2, b3);
        if (VK) {
          ldsm_x4_t(smem_u32(cO + swz<VPCH>(r, np * 2 + (lane >> 4))), b0, b1, b2, b3);
          mma16816<T>(dk_acc[2 * np], ap, b0, b1);
          mma16816<T>(dk_acc[2 * np + 1], ap, b2, b3);
        }
      }
#pragma unroll
      for (int np = 0; np < DVA / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int cb = (VK ? D / 8 : 0) + np * 2;
        ldsm_x4_t(smem_u32(cO + swz<VPCH>(r, cb + (lane >> 4))), b0, b1, b2, b3);
        mma16816<T>(dv_acc[2 * np], ap, b0, b1);
        mma16816<T>(dv_acc[2 * np + 1], ap, b2, b3);
      }
    }
    // dS^T -> shared, then dQ (+)= dS K over this CTA's 64 keys
#pragma unroll
    for (int j = 0; j < BQ / 8; ++j) {
      const int qc = j * 8 + tq * 2;
      const int kr = warp * 16 + g;
      *reinterpret_cast<uint32_t*>(sS + kr * SDS + qc) = Elem<T>::pack(dp[j][0], dp[j][1]);
      *reinterpret_cast<uint32_t*>(sS + (kr + 8) * SDS + qc) = Elem<T>::pack(dp[j][2], dp[j][3]);
    }
    __syncthreads();
    {
      // d columns per warp: two warps per query half split D; at D = 16 one warp takes all 16
      constexpr int DH = D >= 32 ? D / 2 : D;
      const int qw = (warp & 1) * 16, dw = (warp >> 1) * DH;
      if (D >= 32 || warp < 2) {
      float acc[DH / 8][4];
#pragma unroll
      for (int j = 0; j < DH / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t a[4];
        const int mi = lane >> 3;
        const int kr = kk * 16 + (lane & 7) + ((mi >> 1) << 3);
        const int qc = qw + ((mi & 1) << 3);
        ldsm_x4_t(smem_u32(sS + kr * SDS + qc), a[0], a[1], a[2], a[3]);
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
        for (int np = 0; np < DH / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(sK + swz<DPCH>(r, dw / 8 + np * 2 + (lane >> 4))), b0, b1, b2, b3);
          mma16816<T>(acc[2 * np], a, b0, b1);
          mma16816<T>(acc[2 * np + 1], a, b2, b3);
        }
      }
      const int qrow0 = t * BQ + qw + g;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int qrow = qrow0 + i * 8;
        if (qrow < p.n_q) {
          float* dst = gdq + (int64_t)qrow * D + dw + tq * 2;
#pragma unroll
          for (int j = 0; j < DH / 8; ++j)
            atomicAdd(reinterpret_cast<float2*>(dst + j * 8), make_float2(acc[j][2 * i], acc[j][2 * i + 1]));
        }
      }
      }
    }
  }

  // epilogue: this warp's 16 keys
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int key = k0 + warp * 16 + g + i * 8;
    if (key >= p.n_kv) continue;
    if (p.acc_kv) {
      float* dk = static_cast<float*>(p.dk) + bi * p.dk_bs + (int64_t)key * D + tq * 2;
#pragma unroll
      for (int j = 0; j < D / 8; ++j) {
        float2 v = *reinterpret_cast<float2*>(dk + j * 8);
        v.x += dk_acc[j][2 * i];
        v.y += dk_acc[j][2 * i + 1];
        *reinterpret_cast<float2*>(dk + j * 8) = v;
      }
#pragma unroll
      for (int j = 0; j < DVA / 8; ++j) {
        const int col = (VK ? D : 0) + j * 8 + tq * 2;
        float* dst = col < dv1 ? static_cast<float*>(p.dv) + bi * p.dv_bs + (int64_t)key * dv1 + col
                               : static_cast<float*>(p.dv2) + bi * p.dv2_bs + (int64_t)key * dv2 + (col - dv1);
        float2 v = *reinterpret_cast<float2*>(dst);
        v.x += dv_acc[j][2 * i];
        v.y += dv_acc[j][2 * i + 1];
        *reinterpret_cast<float2*>(dst) = v;
      }
    } else {
      uint32_t* dk = reinterpret_cast<uint32_t*>(static_cast<T*>(p.dk) + bi * p.dk_bs + (int64_t)key * D + tq * 2);
#pragma unroll
      for (int j = 0; j < D / 8; ++j) dk[j * 4] = Elem<T>::pack(dk_acc[j][2 * i], dk_acc[j][2 * i + 1]);
#pragma unroll
      for (int j = 0; j < DVA / 8; ++j) {
        const int col = (VK ? D : 0) + j * 8 + tq * 2;
        T* dst = col < dv1 ? static_cast<T*>(p.dv) + bi * p.dv_bs + (int64_t)key * dv1 + col
                           : static_cast<T*>(p.dv2) + bi * p.dv2_bs + (int64_t)key * dv2 + (col - dv1);
        *reinterpret_cast<uint32_t*>(dst) = Elem<T>::pack(dv_acc[j][2 * i], dv_acc[j][2 * i + 1]);
      }
    }
  }
}

// ============================================================================ launchers
template <typename T, int D, int DV, bool ENT>
static cudaError_t launch_fwd_t(const FwdParams& p0, int64_t batch, cudaStream_t st) {
  FwdParams p = p0;
  p.n_qtiles = (p.n_q + 63) / 64;
  constexpr int DP = D < 64 ? 64 : D, VP = DV < 64 ? 64 : DV;
  const size_t smem = (size_t)(64 * DP + 2 * 64 * DP + 2 * 64 * VP) * sizeof(T);
  auto kern = fea_fwd_mma_kernel<T, D, DV, ENT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.n_qtiles * batch;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, 128, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T, int D, int DV, bool VK>
static cudaError_t launch_bwd_t(const BwdParams& p0, int64_t batch, cudaStream_t st) {
  BwdParams p = p0;
  p.n_ktiles = (p.n_kv + 63) / 64;
  constexpr int DP = D < 64 ? 64 : D, VP = DV < 64 ? 64 : DV;
  const size_t smem = (size_t)(64 * DP + 64 * VP + 2 * 32 * DP + 2 * 32 * VP + 64 * 40) * sizeof(T) + 6 * 32 * sizeof(float);
  auto kern = fea_bwd_mma_kernel<T, D, DV, VK>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.n_ktiles * batch;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, 128, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t dispatch_fwd(const FwdParams& p, int64_t batch, int d, int dv, bool ent, cudaStream_t st) {
#define VMB_FWD(DD, VV)                                                                  \
  if (d == DD && dv == VV)                                                               \
    return ent ? launch_fwd_t<T, DD, VV, true>(p, batch, st) : launch_fwd_t<T, DD, VV, false>(p, batch, st);
  VMB_FWD(16, 16)
  VMB_FWD(16, 32)
  VMB_FWD(16, 64)
  VMB_FWD(16, 128)
  VMB_FWD(16, 256)
  VMB_FWD(32, 32)
  VMB_FWD(32, 64)
  VMB_FWD(32, 128)
  VMB_FWD(32, 256)
  VMB_FWD(64, 64)
  VMB_FWD(64, 128)
  VMB_FWD(64, 256)
  VMB_FWD(128, 128)
  VMB_FWD(128, 256)
  VMB_FWD(256, 256)
#undef VMB_FWD
  return cudaErrorNotSupported;
}

template <typename T>
static cudaError_t dispatch_bwd(const BwdParams& p, int64_t batch, int d, int dv, bool vk, cudaStream_t st) {
#define VMB_BWD(DD, VV)                                                                  \
  if (d == DD && dv == VV)                                                               \
    return vk ? launch_bwd_t<T, DD, VV, true>(p, batch, st) : launch_bwd_t<T, DD, VV, false>(p, batch, st);
  // values aliasing keys (the VMonarch R step) exist only with dv = d or 2 d
#define VMB_BWD_SEP(DD, VV)                                                              \
  if (d == DD && dv == VV && !vk) return launch_bwd_t<T, DD, VV, false>(p, batch, st);
  VMB_BWD(16, 16)
  VMB_BWD(16, 32)
  VMB_BWD_SEP(16, 64)
  VMB_BWD_SEP(16, 128)
  VMB_BWD_SEP(16, 256)
  VMB_BWD(32, 32)
  VMB_BWD(32, 64)
  VMB_BWD_SEP(32, 128)
  VMB_BWD_SEP(32, 256)
  VMB_BWD(64, 64)
  VMB_BWD(64, 128)
  VMB_BWD(64, 256)
  VMB_BWD(128, 128)
  VMB_BWD(128, 256)
  VMB_BWD(256, 256)
#undef VMB_BWD
#undef VMB_BWD_SEP
  return cudaErrorNotSupported;
}

cudaError_t fea_fwd_mma(const FwdParams& p, int64_t batch, int d, int dv, bool ent, bool bf16, cudaStream_t st) {
  return bf16 ? dispatch_fwd<__nv_bfloat16>(p, batch, d, dv, ent, st) : dispatch_fwd<__half>(p, batch, d, dv, ent, st);
}

cudaError_t fea_bwd_mma(const BwdParams& p, int64_t batch, int d, int dv, bool vk, bool bf16, cudaStream_t st) {
  return bf16 ? dispatch_bwd<__nv_bfloat16>(p, batch, d, dv, vk, st) : dispatch_bwd<__half>(p, batch, d, dv, vk, st);
}

}  // namespace vmb
