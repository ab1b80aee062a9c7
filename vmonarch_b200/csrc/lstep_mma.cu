// Monarch L step on warp-level tensor-core MMA (mma.sync m16n8k16, fp32 accumulate), m <= 128.
//
// Same mathematics as lstep.cu (reference video_monarch_attention/vmonarch.py:51-63 and its
// autograd backward); this is the fast path for the shapes VMonarch uses (Dv == D, m <= 128).
// For m <= 32 one warp owns one grid column j of one (batch, head) (for m <= 128, and the non-last
// steps with m > 16, one CTA of two to eight warps: see the kernels at the end): it gathers the m
// rows q_i = q[i*b + j]
// and out_k = out[k*b + j] (16-byte cp.async, rows padded to MP = 16, 32, 64 or 128 with zeros), and
// every m x m x D contraction is a handful of MMAs out of swizzled shared memory. The L step is
// HBM-bound (~10 flop/byte), so the tensor cores only serve to keep the arithmetic off the
// critical path; outputs are staged in shared memory and written with 16-byte stores.
//
// Forward: logits = scale * q out_D^T (+ ent_k), a = softmax_k (fp32 registers)
//   non-last: c_k = scale / max(sum_i a_ik, min_col_mass);  u_k = c_k * sum_i a_ik q_i
//   last:     z_i = sum_k a_ik y_k   (tokens < skip_rows are left to the exact recompute)
// Backward (non-last), with G = q du^T:
//   dc_k = sum_i a_ik G_ik,  dcm_k = [cs_k > min_col_mass] (-dc_k c_k / cm_k),
//   dA = c_k G_ik + dcm_k,   dlog = a (dA - rowsum(a dA)),
//   dq_i += sum_k a_ik c_k du_k + scale * sum_k dlog_ik out_k,  dout_k = scale * sum_i dlog_ik q_i
// Backward (last): dA = dz y^T, dlog as above, dq_i += scale * sum_k dlog_ik out_k,
//   dout_k[:D] = scale * sum_i dlog_ik q_i,  dout_k[D:] = sum_i a_ik dz_i
#include "common.cuh"
#include "launch.h"

namespace vmb {
namespace {

// Warps (= grid columns) per CTA. There is no block-level barrier, so CTAs are kept small: the
// per-warp shared memory (19-37 KB) then packs 6-11 warps per SM instead of one 4-warp CTA.
constexpr int kWarpsFwd = 2;
constexpr int kWarpsBwd = 1;

template <int MP>
struct Tile {
  static constexpr int SA = MP + 8;   // row stride (elements) of the m x m staging tile
};

// C[i][k] += sum_d X[i][d] * Y[k][d] over D (X, Y: MP rows, swizzled, XCH chunks per row; the
// contraction starts at chunk xc0 / yc0).
template <typename T, int MP, int D, int XCH, int YCH>
__device__ __forceinline__ void mm_rows(float (&acc)[MP / 16][MP / 8][4], const T* X, int xc0, const T* Y, int yc0,
                                        int zr, int lane) {
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a[MP / 16][4];
#pragma unroll
    for (int mt = 0; mt < MP / 16; ++mt)
      ldsm_x4(smem_u32(X + swz<XCH>(min(mt * 16 + (lane & 15), zr), xc0 + kk * 2 + (lane >> 4))), a[mt][0],
              a[mt][1], a[mt][2], a[mt][3]);
#pragma unroll
    for (int np = 0; np < MP / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(Y + swz<YCH>(min(np * 16 + (lane & 7) + ((lane >> 4) << 3), zr), yc0 + kk * 2 + ((lane >> 3) & 1))),
              b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < MP / 16; ++mt) {
        mma16816<T>(acc[mt][2 * np], a[mt], b0, b1);
        mma16816<T>(acc[mt][2 * np + 1], a[mt], b2, b3);
      }
    }
  }
}

// Packs rows (mt) x k-step (kk) of an accumulator-layout MP x MP fp32 matrix into an A fragment.
template <typename T, int MP>
__device__ __forceinline__ void frag_from_acc(const float (&v)[MP / 16][MP / 8][4], int mt, int kk, uint32_t (&a)[4]) {
  a[0] = Elem<T>::pack(v[mt][2 * kk][0], v[mt][2 * kk][1]);
  a[1] = Elem<T>::pack(v[mt][2 * kk][2], v[mt][2 * kk][3]);
  a[2] = Elem<T>::pack(v[mt][2 * kk + 1][0], v[mt][2 * kk + 1][1]);
  a[3] = Elem<T>::pack(v[mt][2 * kk + 1][2], v[mt][2 * kk + 1][3]);
}

// Writes an accumulator-layout MP x MP matrix to a row-major [MP][SA] staging tile (bf16/fp16).
template <typename T, int MP>
__device__ __forceinline__ void stage_mm(T* S, const float (&v)[MP / 16][MP / 8][4], int lane) {
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = mt * 16 + (lane >> 2) + h * 8, c = nt * 8 + (lane & 3) * 2;
        *reinterpret_cast<uint32_t*>(S + r * Tile<MP>::SA + c) = Elem<T>::pack(v[mt][nt][2 * h], v[mt][nt][2 * h + 1]);
      }
}

// out[r][n] (r: MP rows, n: 64 columns from chunk bc0 of B) = sum_i A[r][i] * B[i][n]
// where A comes from the [MP][SA] staging tile TRANSPOSED (A[r][i] = S[i][r]) and B rows are i.
template <typename T, int MP, int BCH>
__device__ __forceinline__ void mm_tn64(float (&acc)[MP / 16][8][4], const T* S, const T* B, int bc0, int zr, int lane) {
#pragma unroll
  for (int kk = 0; kk < MP / 16; ++kk) {
    uint32_t a[MP / 16][4];
    const int mi = lane >> 3;
#pragma unroll
    for (int mt = 0; mt < MP / 16; ++mt)
      ldsm_x4_t(smem_u32(S + (kk * 16 + (lane & 7) + ((mi >> 1) << 3)) * Tile<MP>::SA + mt * 16 + ((mi & 1) << 3)),
                a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
    const int r = min(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), zr);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(B + swz<BCH>(r, bc0 + np * 2 + (lane >> 4))), b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < MP / 16; ++mt) {
        mma16816<T>(acc[mt][2 * np], a[mt], b0, b1);
        mma16816<T>(acc[mt][2 * np + 1], a[mt], b2, b3);
      }
    }
  }
}

// Transpose of an 8 x 8 block of 16-bit values held one row per four lanes (row lane / 4, columns
// 2 (lane % 4) and 2 (lane % 4) + 1, low half first): the result holds the transposed block in
// the same layout.
__device__ __forceinline__ uint32_t movt(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// m16n8k16 A fragments of the TRANSPOSE of an accumulator-layout MP x MP matrix V (rows i, columns
// k): at[rt][kk] covers rows [16 rt, 16 rt + 16) (k) and columns [16 kk, 16 kk + 16) (i) of V^T.
// Each register is one packed 8 x 8 block of V moved across the lanes, so the fragments hold the
// same 16-bit values a transposed ldmatrix of V staged in shared memory would load.
template <typename T, int MP>
__device__ __forceinline__ void frag_t_from_acc(const float (&v)[MP / 16][MP / 8][4],
                                                uint32_t (&at)[MP / 16][MP / 16][4]) {
#pragma unroll
  for (int rt = 0; rt < MP / 16; ++rt)
#pragma unroll
    for (int kk = 0; kk < MP / 16; ++kk) {
      at[rt][kk][0] = movt(Elem<T>::pack(v[kk][2 * rt][0], v[kk][2 * rt][1]));
      at[rt][kk][1] = movt(Elem<T>::pack(v[kk][2 * rt + 1][0], v[kk][2 * rt + 1][1]));
      at[rt][kk][2] = movt(Elem<T>::pack(v[kk][2 * rt][2], v[kk][2 * rt][3]));
      at[rt][kk][3] = movt(Elem<T>::pack(v[kk][2 * rt + 1][2], v[kk][2 * rt + 1][3]));
    }
}

// mm_tn64 with the transposed A in registers (frag_t_from_acc) instead of a staging tile.
template <typename T, int MP, int BCH>
__device__ __forceinline__ void mm_tn64_reg(float (&acc)[MP / 16][8][4], const uint32_t (&at)[MP / 16][MP / 16][4],
                                            const T* B, int bc0, int zr, int lane) {
#pragma unroll
  for (int kk = 0; kk < MP / 16; ++kk) {
    const int r = min(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), zr);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(B + swz<BCH>(r, bc0 + np * 2 + (lane >> 4))), b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < MP / 16; ++mt) {
        mma16816<T>(acc[mt][2 * np], at[mt][kk], b0, b1);
        mma16816<T>(acc[mt][2 * np + 1], at[mt][kk], b2, b3);
      }
    }
  }
}

// out[i][n] += sum_k A[i][k] * B[k][n] with A given in accumulator layout (registers).
template <typename T, int MP, int BCH>
__device__ __forceinline__ void mm_rn64(float (&acc)[MP / 16][8][4], const float (&A)[MP / 16][MP / 8][4], const T* B,
                                        int bc0, int zr, int lane) {
#pragma unroll
  for (int kk = 0; kk < MP / 16; ++kk) {
    uint32_t a[MP / 16][4];
#pragma unroll
    for (int mt = 0; mt < MP / 16; ++mt) frag_from_acc<T, MP>(A, mt, kk, a[mt]);
    const int r = min(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), zr);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(B + swz<BCH>(r, bc0 + np * 2 + (lane >> 4))), b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < MP / 16; ++mt) {
        mma16816<T>(acc[mt][2 * np], a[mt], b0, b1);
        mma16816<T>(acc[mt][2 * np + 1], a[mt], b2, b3);
      }
    }
  }
}

template <int MP>
__device__ __forceinline__ void zero(float (&a)[MP / 16][8][4]) {
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int n = 0; n < 8; ++n) a[mt][n][0] = a[mt][n][1] = a[mt][n][2] = a[mt][n][3] = 0.f;
}

// 64 output columns (half of D = 128 or all of D = 64) of an accumulator -> swizzled staging rows.
template <typename T, int MP, int CH>
__device__ __forceinline__ void stage_rows64(T* S, int c0, const float (&v)[MP / 16][8][4], const float* rowscale,
                                             int m, int lane) {
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + (lane >> 2) + h * 8;
      if (r >= m) continue;  // tiles hold rows [0, m) and the zero row m
      const float s = rowscale ? rowscale[r] : 1.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int col = c0 * 8 + nt * 8 + (lane & 3) * 2;
        *reinterpret_cast<uint32_t*>(S + swz<CH>(r, col >> 3) + (col & 7)) =
            Elem<T>::pack(v[mt][nt][2 * h] * s, v[mt][nt][2 * h + 1] * s);
      }
    }
}

// stage_rows64 for the dout tile, which is written over the out tile: before each pair is
// overwritten, its out values are multiplied with the bf16-rounded dout values that replace them,
// and the products are summed per row (this lane's share of sum_c out[c] dout[c]).
template <typename T, int MP, int CH>
__device__ __forceinline__ void stage_rows64_dot(T* S, int c0, const float (&v)[MP / 16][8][4],
                                                 float (&dot)[MP / 16][2], int m, int lane) {
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + (lane >> 2) + h * 8;
      if (r >= m) continue;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int col = c0 * 8 + nt * 8 + (lane & 3) * 2;
        uint32_t* p = reinterpret_cast<uint32_t*>(S + swz<CH>(r, col >> 3) + (col & 7));
        const uint32_t w = Elem<T>::pack(v[mt][nt][2 * h], v[mt][nt][2 * h + 1]);
        const float2 o = Elem<T>::unpack(*p), g = Elem<T>::unpack(w);
        dot[mt][h] = fmaf(o.x, g.x, fmaf(o.y, g.y, dot[mt][h]));
        *p = w;
      }
    }
}

// Offset (elements) of head hb of a [bh][N][cols] view split (n1, 1): (hb % n1) s1 + (hb / n1) s3.
__device__ __forceinline__ int64_t head_off(const View& v, int n1, int64_t hb) {
  const int64_t c3 = hb / n1;
  return (hb - c3 * n1) * v.s1 + c3 * v.s3;
}

// Gathers rows i < m (token i*b + j) of a [N][W] tensor, columns [c0*8, (c0+nch)*8), into a
// swizzled [m + 1][CH] tile; rows whose token < skip are zero-filled. Row m is the tile's zero row
// (zero_row), which the MMA loaders read for every row index >= m.

template <typename T, int CH>
__device__ __forceinline__ void gather(T* dst, const T* src, int64_t W, int c0, int nch, int m, int64_t b, int j,
                                       int64_t skip, int lane, int nthr = 32) {
  for (int c = lane; c < m * nch; c += nthr) {
    const int i = c / nch, ch = c % nch;
    const int64_t tok = (int64_t)i * b + j;
    const bool ok = tok >= skip;
    cp_async16(smem_u32(dst + swz<CH>(i, c0 + ch)), src + (ok ? tok : 0) * W + (c0 + ch) * 8, ok ? 16 : 0);
  }
}
template <typename T, int CH>
__device__ __forceinline__ void zero_row(T* dst, int m, int lane, int nthr = 32) {
  for (int ch = lane; ch < CH; ch += nthr) *reinterpret_cast<uint4*>(dst + m * CH * 8 + ch * 8) = make_uint4(0, 0, 0, 0);
}

// Per-warp shared memory (bytes) of the L-step kernels: gathered tiles of m + 1 rows (the last one
// zero); the forward adds an m x m staging tile of MP rows and MP column scales. The layout below
// follows the same order.
template <int MP>
__host__ __device__ __forceinline__ size_t lstep_warp_bytes(int m, int D, int OW, bool bwd, int esize) {
  const size_t rows = (size_t)m + 1;
  return bwd ? rows * (2 * D + OW) * esize
             : (rows * (D + OW) + (size_t)MP * (MP + 8)) * esize + MP * sizeof(float);
}

// Writes rows r < m of a swizzled [MP][CH] staging tile to token r*b + j of a [N][W] tensor.
template <typename T, int CH>
__device__ __forceinline__ void scatter(T* dst, const T* S, int64_t W, int c0, int nch, int m, int64_t b, int j,
                                        int64_t skip, int MP, int lane, int nthr = 32) {
  for (int c = lane; c < MP * nch; c += nthr) {
    const int r = c / nch, ch = c % nch;
    const int64_t tok = (int64_t)r * b + j;
    if (r < m && tok >= skip)
      *reinterpret_cast<uint4*>(dst + tok * W + (c0 + ch) * 8) = *reinterpret_cast<const uint4*>(S + swz<CH>(r, c0 + ch));
  }
}

// logits -> a = softmax over valid k of (scale * logit + ent_k); padded rows / columns become 0.
template <int MP>
__device__ __forceinline__ void softmax_rows(float (&acc)[MP / 16][MP / 8][4], const float (&ent)[MP / 8][2],
                                             float scale, int m, int lane) {
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int k = nt * 8 + (lane & 3) * 2 + e;
          const float x = k < m ? (acc[mt][nt][2 * h + e] * scale + ent[nt][e]) * kLog2e : -INFINITY;
          acc[mt][nt][2 * h + e] = x;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float s = 0.f;
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = exp2f(acc[mt][nt][2 * h + e] - mx);
          acc[mt][nt][2 * h + e] = pv;
          s += pv;
        }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      const bool row_ok = mt * 16 + (lane >> 2) + h * 8 < m;
      const float inv = row_ok ? 1.f / s : 0.f;
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) acc[mt][nt][2 * h + e] *= inv;
    }
}

// Column sums over all rows: result for this thread's columns (nt, e), replicated across lane>>2.
template <int MP>
__device__ __forceinline__ void col_sums(const float (&v)[MP / 16][MP / 8][4], float (&cs)[MP / 8][2]) {
#pragma unroll
  for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float s = 0.f;
#pragma unroll
      for (int mt = 0; mt < MP / 16; ++mt) s += v[mt][nt][e] + v[mt][nt][2 + e];
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 8);
      s += __shfl_xor_sync(0xffffffffu, s, 16);
      cs[nt][e] = s;
    }
}

template <typename T, int MP>
__device__ __forceinline__ void load_ent(float (&ent)[MP / 8][2], const float* e, int64_t b, int j, int m, int lane) {
#pragma unroll
  for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      const int k = nt * 8 + (lane & 3) * 2 + x;
      ent[nt][x] = k < m ? e[(int64_t)k * b + j] : 0.f;
    }
}

// ============================================================================ forward
template <typename T, int MP, int D, bool LAST>
__global__ void __launch_bounds__(kWarpsFwd * 32) lstep_fwd_mma_kernel(const LstepParams p) {
  constexpr int DCH = D / 8, OW = LAST ? 2 * D : D, OCH = OW / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = (int)p.m;
  T* sq = reinterpret_cast<T*>(smem_raw + warp * lstep_warp_bytes<MP>(m, D, OW, false, sizeof(T)));
  T* so = sq + (m + 1) * D;
  T* sa = so + (m + 1) * OW;
  float* svec = reinterpret_cast<float*>(sa + MP * Tile<MP>::SA);

  const int64_t col = (int64_t)blockIdx.x * kWarpsFwd + warp;
  if (col >= p.bh * p.b) return;  // no block-level barrier below: each warp is independent
  const int64_t bh = col / p.b;
  const int j = (int)(col % p.b);
  const int64_t N = p.m * p.b;
  const T* gq = static_cast<const T*>(p.q) + head_off(p.qv, p.n1, bh);
  const T* go = static_cast<const T*>(p.out) + head_off(p.outv, p.n1, bh);
  gather<T, DCH>(sq, gq, p.qv.rs, 0, DCH, m, p.b, j, 0, lane);
  gather<T, OCH>(so, go, p.outv.rs, 0, OCH, m, p.b, j, 0, lane);
  cp_async_commit();
  zero_row<T, DCH>(sq, m, lane);
  zero_row<T, OCH>(so, m, lane);
  float ent[MP / 8][2];
  load_ent<T, MP>(ent, p.ent + bh * N, p.b, j, m, lane);
  cp_async_wait<0>();
  __syncwarp();

  float a[MP / 16][MP / 8][4];
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt) a[mt][nt][0] = a[mt][nt][1] = a[mt][nt][2] = a[mt][nt][3] = 0.f;
  mm_rows<T, MP, D, DCH, OCH>(a, sq, 0, so, 0, m, lane);
  softmax_rows<MP>(a, ent, p.scale, m, lane);

  if (LAST) {
    // z_i = sum_k a_ik y_k -> staged in sq (q no longer needed)
    __syncwarp();
    T* gz = static_cast<T*>(p.z) + head_off(p.zv, p.n1, bh);
#pragma unroll 1
    for (int half = 0; half < D / 64; ++half) {
      float z[MP / 16][8][4];
      zero<MP>(z);
      mm_rn64<T, MP, OCH>(z, a, so, DCH + half * 8, m, lane);
      stage_rows64<T, MP, DCH>(sq, half * 8, z, nullptr, m, lane);
    }
    __syncwarp();
    scatter<T, DCH>(gz, sq, p.zv.rs, 0, DCH, m, p.b, j, p.skip_rows, MP, lane);
  } else {
    float cs[MP / 8][2];
    col_sums<MP>(a, cs);
    if ((lane >> 2) == 0) {
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) svec[nt * 8 + lane * 2 + e] = p.scale / fmaxf(cs[nt][e], p.min_col_mass);
    }
    stage_mm<T, MP>(sa, a, lane);
    __syncwarp();
    T* gu = static_cast<T*>(p.u) + head_off(p.uv, p.n1, bh);
#pragma unroll 1
    for (int half = 0; half < D / 64; ++half) {
      float u[MP / 16][8][4];
      zero<MP>(u);
      mm_tn64<T, MP, DCH>(u, sa, sq, half * 8, m, lane);
      stage_rows64<T, MP, OCH>(so, half * 8, u, svec, m, lane);  // so (out_D) is free after the logits
    }
    __syncwarp();
    scatter<T, OCH>(gu, so, p.uv.rs, 0, DCH, m, p.b, j, 0, MP, lane);
  }
}

// ============================================================================ backward
template <typename T, int MP, int D, bool LAST>
__global__ void __launch_bounds__(kWarpsBwd * 32) lstep_bwd_mma_kernel(const LstepParams p) {
  constexpr int DCH = D / 8, OW = LAST ? 2 * D : D, OCH = OW / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = (int)p.m;
  T* sq = reinterpret_cast<T*>(smem_raw + warp * lstep_warp_bytes<MP>(m, D, OW, true, sizeof(T)));
  T* so = sq + (m + 1) * D;     // out rows (kr | y), later the dout staging
  T* sg = so + (m + 1) * OW;    // du (non-last) or dz (last), element dtype

  const int64_t col = (int64_t)blockIdx.x * kWarpsBwd + warp;
  if (col >= p.bh * p.b) return;
  const int64_t bh = col / p.b;
  const int j = (int)(col % p.b);
  const int64_t N = p.m * p.b;
  gather<T, DCH>(sq, static_cast<const T*>(p.q) + head_off(p.qv, p.n1, bh), p.qv.rs, 0, DCH, m, p.b, j, 0, lane);
  gather<T, OCH>(so, static_cast<const T*>(p.out) + head_off(p.outv, p.n1, bh), p.outv.rs, 0, OCH, m, p.b, j, 0, lane);
  if (LAST)
    gather<T, DCH>(sg, static_cast<const T*>(p.dz) + head_off(p.dzv, p.n1, bh), p.dzv.rs, 0, DCH, m, p.b, j,
                   p.skip_rows, lane);
  cp_async_commit();
  zero_row<T, DCH>(sq, m, lane);
  zero_row<T, OCH>(so, m, lane);
  zero_row<T, DCH>(sg, m, lane);
  if (!LAST) {  // du is fp32: convert while the other rows are in flight
    // four chunks' loads are issued before any is converted, so a warp waits for one memory round
    // trip per four chunks instead of one per chunk
    const float* du = p.du + head_off(p.duv, p.n1, bh);
    const int kChunks = (m * DCH + 31) / 32;  // per lane, rows < m
#pragma unroll 1
    for (int t0 = 0; t0 < kChunks; t0 += 4) {
      float4 v[4][2];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = lane + 32 * (t0 + u), k = c / DCH, ch = c % DCH;
        if (k < m) {
          const float4* src = reinterpret_cast<const float4*>(du + ((int64_t)k * p.b + j) * p.duv.rs + ch * 8);
          v[u][0] = src[0];
          v[u][1] = src[1];
        } else {
          v[u][0] = v[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = lane + 32 * (t0 + u), k = c / DCH, ch = c % DCH;
        if (k >= m) continue;
        uint4 w;
        w.x = Elem<T>::pack(v[u][0].x, v[u][0].y);
        w.y = Elem<T>::pack(v[u][0].z, v[u][0].w);
        w.z = Elem<T>::pack(v[u][1].x, v[u][1].y);
        w.w = Elem<T>::pack(v[u][1].z, v[u][1].w);
        *reinterpret_cast<uint4*>(sg + swz<DCH>(k, ch)) = w;
      }
    }
  }
  float ent[MP / 8][2];
  load_ent<T, MP>(ent, p.ent + bh * N, p.b, j, m, lane);
  cp_async_wait<0>();
  __syncwarp();

  float a[MP / 16][MP / 8][4], g[MP / 16][MP / 8][4], ac[MP / 16][MP / 8][4];
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) a[mt][nt][e] = g[mt][nt][e] = ac[mt][nt][e] = 0.f;
  mm_rows<T, MP, D, DCH, OCH>(a, sq, 0, so, 0, m, lane);
  softmax_rows<MP>(a, ent, p.scale, m, lane);

  if (LAST) {
    // dA = dz y^T
    mm_rows<T, MP, D, DCH, OCH>(g, sg, 0, so, DCH, m, lane);
  } else {
    // G = q du^T ; dc_k = sum_i a_ik G_ik ; dA = c_k G_ik + dcm_k ; ac = a * c for the dq term
    mm_rows<T, MP, D, DCH, DCH>(g, sq, 0, sg, 0, m, lane);
    float cs[MP / 8][2], dc[MP / 8][2];
    col_sums<MP>(a, cs);
#pragma unroll
    for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) ac[mt][nt][e] = a[mt][nt][e] * g[mt][nt][e];
    col_sums<MP>(ac, dc);
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float cm = fmaxf(cs[nt][e], p.min_col_mass);
        const float c = p.scale / cm;
        const float dcm = cs[nt][e] > p.min_col_mass ? -dc[nt][e] * c / cm : 0.f;
#pragma unroll
        for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            g[mt][nt][2 * h + e] = c * g[mt][nt][2 * h + e] + dcm;   // dA
            ac[mt][nt][2 * h + e] = a[mt][nt][2 * h + e] * c;        // a * c
          }
      }
  }
  // dlog = a (dA - rowsum(a dA)), computed in place in g and pre-multiplied by scale
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float rs = 0.f;
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
        rs += a[mt][nt][2 * h] * g[mt][nt][2 * h] + a[mt][nt][2 * h + 1] * g[mt][nt][2 * h + 1];
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) g[mt][nt][2 * h + e] = a[mt][nt][2 * h + e] * (g[mt][nt][2 * h + e] - rs) * p.scale;
    }
  // a^T (last) as transposed A fragments for dout[D:] = a^T dz; a is not needed after this
  uint32_t at[MP / 16][MP / 16][4];
  if (LAST) frag_t_from_acc<T, MP>(a, at);

  // dq_i += sum_k (scale dlog_ik) out_k  [non-last: + sum_k (a_ik c_k) du_k]
  float* gdq = p.dq + head_off(p.dqv, p.n1, bh);
#pragma unroll 1
  for (int half = 0; half < D / 64; ++half) {
    float acc[MP / 16][8][4];
    zero<MP>(acc);
    mm_rn64<T, MP, OCH>(acc, g, so, half * 8, m, lane);
    if (!LAST) mm_rn64<T, MP, DCH>(acc, ac, sg, half * 8, m, lane);
#pragma unroll
    for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = mt * 16 + (lane >> 2) + h * 8;
        if (i >= m) continue;
        float* dst = gdq + ((int64_t)i * p.b + j) * p.dqv.rs + half * 64 + (lane & 3) * 2;
        // fire-and-forget reductions (or plain stores in the store mode): this warp alone owns
        // these dq elements, so nothing waits for the old value
        if (p.dq_store) {
#pragma unroll
          for (int nt = 0; nt < 8; ++nt)
            *reinterpret_cast<float2*>(dst + nt * 8) = make_float2(acc[mt][nt][2 * h], acc[mt][nt][2 * h + 1]);
        } else {
#pragma unroll
          for (int nt = 0; nt < 8; ++nt)
            asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(dst + nt * 8), "f"(acc[mt][nt][2 * h]),
                         "f"(acc[mt][nt][2 * h + 1])
                         : "memory");
        }
      }
  }
  __syncwarp();
  // dout_k[:D] = sum_i (scale dlog_ik) q_i ; last: dout_k[D:] = sum_i a_ik dz_i   (staged in so,
  // over out; delta_k = sum_c out_k[c] dout_k[c] is summed on the way, the preprocessing of the
  // R step's attention backward)
  T* gdo = static_cast<T*>(p.dout) + head_off(p.doutv, p.n1, bh);
  uint32_t gt[MP / 16][MP / 16][4];  // (scale dlog)^T as transposed A fragments
  frag_t_from_acc<T, MP>(g, gt);
  float dot[MP / 16][2];
#pragma unroll
  for (int mt = 0; mt < MP / 16; ++mt) dot[mt][0] = dot[mt][1] = 0.f;
#pragma unroll 1
  for (int half = 0; half < D / 64; ++half) {
    float acc[MP / 16][8][4];
    zero<MP>(acc);
    mm_tn64_reg<T, MP, DCH>(acc, gt, sq, half * 8, m, lane);
    stage_rows64_dot<T, MP, OCH>(so, half * 8, acc, dot, m, lane);
  }
  if (LAST) {
#pragma unroll 1
    for (int half = 0; half < D / 64; ++half) {
      float acc[MP / 16][8][4];
      zero<MP>(acc);
      mm_tn64_reg<T, MP, DCH>(acc, at, sg, half * 8, m, lane);
      stage_rows64_dot<T, MP, OCH>(so, DCH + half * 8, acc, dot, m, lane);
    }
  }
  if (p.delta_out) {
#pragma unroll
    for (int mt = 0; mt < MP / 16; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float d = dot[mt][h];
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        const int r = mt * 16 + (lane >> 2) + h * 8;
        if ((lane & 3) == 0 && r < m) p.delta_out[bh * N + (int64_t)r * p.b + j] = d;
      }
  }
  __syncwarp();
  scatter<T, OCH>(gdo, so, p.doutv.rs, 0, OCH, m, p.b, j, 0, MP, lane);
}

// ============================================================================ several warps per column
// One CTA of NW = 4 (m <= 64) or 8 (m <= 128) warps per grid column, MP = 16 NW; also NW = 2 for
// the non-last steps with 16 < m <= 32. Warp w owns the logit rows [16 w, 16 w + 16):
// the row-local products (logits, softmax, z, G or dA, dlog, dq) stay in its registers, as in the
// one-warp kernels above; the products that sum over rows (column masses, u, dout) go through
// m x m staging tiles in shared memory, warp w producing their rows [16 w, 16 w + 16). The
// helpers below are the one-m-tile forms of the ones above.
constexpr int kMaxMP = 128;  // the largest grid (m) of the tensor-core L-step kernels

// acc[nt] (rows [r0, r0 + 16), all MP columns k) = sum_d X[r][d] * Y[k][d]
template <typename T, int MP, int D, int XCH, int YCH>
__device__ __forceinline__ void mm_rows_t(float (&acc)[MP / 8][4], const T* X, int xc0, const T* Y, int yc0, int r0,
                                          int zr, int lane) {
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a[4];
    ldsm_x4(smem_u32(X + swz<XCH>(min(r0 + (lane & 15), zr), xc0 + kk * 2 + (lane >> 4))), a[0], a[1], a[2], a[3]);
#pragma unroll
    for (int np = 0; np < MP / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(Y + swz<YCH>(min(np * 16 + (lane & 7) + ((lane >> 4) << 3), zr), yc0 + kk * 2 + ((lane >> 3) & 1))),
              b0, b1, b2, b3);
      mma16816<T>(acc[2 * np], a, b0, b1);
      mma16816<T>(acc[2 * np + 1], a, b2, b3);
    }
  }
}

__device__ __forceinline__ void zero_t(float (&a)[8][4]) {
#pragma unroll
  for (int n = 0; n < 8; ++n) a[n][0] = a[n][1] = a[n][2] = a[n][3] = 0.f;
}

// softmax_rows for the rows [r0, r0 + 16)
template <int MP>
__device__ __forceinline__ void softmax_t(float (&acc)[MP / 8][4], const float (&ent)[MP / 8][2], float scale, int m, int r0,
                                          int lane) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int k = nt * 8 + (lane & 3) * 2 + e;
        const float x = k < m ? (acc[nt][2 * h + e] * scale + ent[nt][e]) * kLog2e : -INFINITY;
        acc[nt][2 * h + e] = x;
        mx = fmaxf(mx, x);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    float s = 0.f;
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float pv = exp2f(acc[nt][2 * h + e] - mx);
        acc[nt][2 * h + e] = pv;
        s += pv;
      }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    const bool row_ok = r0 + (lane >> 2) + h * 8 < m;
    const float inv = row_ok ? 1.f / s : 0.f;
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) acc[nt][2 * h + e] *= inv;
  }
}

// Column sums over this warp's 16 rows: cs[nt][e] is column nt * 8 + 2 (lane & 3) + e (replicated
// over lane >> 2).
template <int MP>
__device__ __forceinline__ void col_sums_t(const float (&v)[MP / 8][4], float (&cs)[MP / 8][2]) {
#pragma unroll
  for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float s = v[nt][e] + v[nt][2 + e];
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 8);
      s += __shfl_xor_sync(0xffffffffu, s, 16);
      cs[nt][e] = s;
    }
}

// col_sums_t of the elementwise product u * v
template <int MP>
__device__ __forceinline__ void col_sums_prod_t(const float (&u)[MP / 8][4], const float (&v)[MP / 8][4],
                                                float (&cs)[MP / 8][2]) {
#pragma unroll
  for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float s = u[nt][e] * v[nt][e] + u[nt][2 + e] * v[nt][2 + e];
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 8);
      s += __shfl_xor_sync(0xffffffffu, s, 16);
      cs[nt][e] = s;
    }
}

// Rows [r0, r0 + 16) of an m x m matrix into the row-major [MP][SA] staging tile.
template <typename T, int MP>
__device__ __forceinline__ void stage_mm_t(T* S, const float (&v)[MP / 8][4], int r0, int lane) {
#pragma unroll
  for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = r0 + (lane >> 2) + h * 8, c = nt * 8 + (lane & 3) * 2;
      *reinterpret_cast<uint32_t*>(S + r * Tile<MP>::SA + c) = Elem<T>::pack(v[nt][2 * h], v[nt][2 * h + 1]);
    }
}

// out[k][n] for k in [r0, r0 + 16), 64 columns from chunk bc0 of B: sum_i S[i][k] * B[i][n]
// (the staging tile read transposed, B rows i).
template <typename T, int BCH, int MP>
__device__ __forceinline__ void mm_tn64_t(float (&acc)[8][4], const T* S, const T* B, int bc0, int r0, int zr, int lane) {
  const int mi = lane >> 3;
#pragma unroll
  for (int kk = 0; kk < MP / 16; ++kk) {
    uint32_t a[4];
    ldsm_x4_t(smem_u32(S + (kk * 16 + (lane & 7) + ((mi >> 1) << 3)) * Tile<MP>::SA + r0 + ((mi & 1) << 3)), a[0], a[1],
              a[2], a[3]);
    const int r = min(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), zr);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(B + swz<BCH>(r, bc0 + np * 2 + (lane >> 4))), b0, b1, b2, b3);
      mma16816<T>(acc[2 * np], a, b0, b1);
      mma16816<T>(acc[2 * np + 1], a, b2, b3);
    }
  }
}

// out[i][n] += sum_k A[i][k] * B[k][n] for this warp's 16 rows, A in accumulator layout.
template <typename T, int BCH, int MP>
__device__ __forceinline__ void mm_rn64_t(float (&acc)[8][4], const float (&A)[MP / 8][4], const T* B, int bc0, int zr,
                                          int lane) {
#pragma unroll
  for (int kk = 0; kk < MP / 16; ++kk) {
    uint32_t a[4];
    a[0] = Elem<T>::pack(A[2 * kk][0], A[2 * kk][1]);
    a[1] = Elem<T>::pack(A[2 * kk][2], A[2 * kk][3]);
    a[2] = Elem<T>::pack(A[2 * kk + 1][0], A[2 * kk + 1][1]);
    a[3] = Elem<T>::pack(A[2 * kk + 1][2], A[2 * kk + 1][3]);
    const int r = min(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), zr);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(B + swz<BCH>(r, bc0 + np * 2 + (lane >> 4))), b0, b1, b2, b3);
      mma16816<T>(acc[2 * np], a, b0, b1);
      mma16816<T>(acc[2 * np + 1], a, b2, b3);
    }
  }
}

// stage_rows64 / stage_rows64_dot for the rows [r0, r0 + 16)
template <typename T, int CH>
__device__ __forceinline__ void stage_rows64_t(T* S, int c0, const float (&v)[8][4], const float* rowscale, int m, int r0,
                                               int lane) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = r0 + (lane >> 2) + h * 8;
    if (r >= m) continue;
    const float s = rowscale ? rowscale[r] : 1.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = c0 * 8 + nt * 8 + (lane & 3) * 2;
      *reinterpret_cast<uint32_t*>(S + swz<CH>(r, col >> 3) + (col & 7)) = Elem<T>::pack(v[nt][2 * h] * s, v[nt][2 * h + 1] * s);
    }
  }
}
template <typename T, int CH>
__device__ __forceinline__ void stage_rows64_dot_t(T* S, int c0, const float (&v)[8][4], float (&dot)[2], int m, int r0,
                                                   int lane) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = r0 + (lane >> 2) + h * 8;
    if (r >= m) continue;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = c0 * 8 + nt * 8 + (lane & 3) * 2;
      uint32_t* q = reinterpret_cast<uint32_t*>(S + swz<CH>(r, col >> 3) + (col & 7));
      const uint32_t w = Elem<T>::pack(v[nt][2 * h], v[nt][2 * h + 1]);
      const float2 o = Elem<T>::unpack(*q), g = Elem<T>::unpack(w);
      dot[h] = fmaf(o.x, g.x, fmaf(o.y, g.y, dot[h]));
      *q = w;
    }
  }
}

// Shared memory (bytes) of one column's CTA: gathered tiles of m + 1 rows, the m x m staging
// tiles (the forward's a; the backward's dlog and a), then fp32 column partials and scales.
__host__ __device__ __forceinline__ size_t lstepw_bytes(int m, int D, int OW, bool bwd, int esize, int NW) {
  const size_t MP = 16 * (size_t)NW, rows = (size_t)m + 1;
  const size_t tiles = bwd ? rows * (2 * D + OW) : rows * (D + OW);
  const size_t stg = (bwd ? 2 : 1) * MP * (MP + 8);  // Tile<MP>::SA = MP + 8
  const size_t floats = bwd ? (2 * NW + 2) * MP : (NW + 1) * MP;
  return (tiles + stg) * esize + floats * sizeof(float);
}

template <typename T, int D, bool LAST, int NW>
__global__ void __launch_bounds__(NW * 32) lstep_fwd_mmaw_kernel(const LstepParams p) {
  constexpr int MP = 16 * NW, DCH = D / 8, OW = LAST ? 2 * D : D, OCH = OW / 8, NTH = NW * 32;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, r0 = 16 * warp;
  const int m = (int)p.m;
  T* sq = reinterpret_cast<T*>(smem_raw);
  T* so = sq + (m + 1) * D;
  T* sa = so + (m + 1) * OW;                                        // a, MP x SA
  float* part = reinterpret_cast<float*>(sa + MP * Tile<MP>::SA);  // [warp][k] column partials
  float* svec = part + NW * MP;                               // [k] c_k

  const int64_t bh = blockIdx.x / p.b;  // one CTA per grid column: bh * b CTAs
  const int j = (int)(blockIdx.x % p.b);
  const int64_t N = p.m * p.b;
  const T* gq = static_cast<const T*>(p.q) + head_off(p.qv, p.n1, bh);
  const T* go = static_cast<const T*>(p.out) + head_off(p.outv, p.n1, bh);
  gather<T, DCH>(sq, gq, p.qv.rs, 0, DCH, m, p.b, j, 0, tid, NTH);
  gather<T, OCH>(so, go, p.outv.rs, 0, OCH, m, p.b, j, 0, tid, NTH);
  cp_async_commit();
  zero_row<T, DCH>(sq, m, tid, NTH);
  zero_row<T, OCH>(so, m, tid, NTH);
  float ent[MP / 8][2];
  load_ent<T, MP>(ent, p.ent + bh * N, p.b, j, m, lane);
  cp_async_wait<0>();
  __syncthreads();

  float a[MP / 8][4];
#pragma unroll
  for (int nt = 0; nt < MP / 8; ++nt) a[nt][0] = a[nt][1] = a[nt][2] = a[nt][3] = 0.f;
  mm_rows_t<T, MP, D, DCH, OCH>(a, sq, 0, so, 0, r0, m, lane);
  softmax_t<MP>(a, ent, p.scale, m, r0, lane);

  if (LAST) {
    // z_i = sum_k a_ik y_k -> staged in sq once every warp's logits have read it
    __syncthreads();
    T* gz = static_cast<T*>(p.z) + head_off(p.zv, p.n1, bh);
#pragma unroll 1
    for (int half = 0; half < D / 64; ++half) {
      float z[8][4];
      zero_t(z);
      mm_rn64_t<T, OCH, MP>(z, a, so, DCH + half * 8, m, lane);
      stage_rows64_t<T, DCH>(sq, half * 8, z, nullptr, m, r0, lane);
    }
    __syncthreads();
    scatter<T, DCH>(gz, sq, p.zv.rs, 0, DCH, m, p.b, j, p.skip_rows, MP, tid, NTH);
  } else {
    float cs[MP / 8][2];
    col_sums_t<MP>(a, cs);
    if ((lane >> 2) == 0) {
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) part[warp * MP + nt * 8 + lane * 2 + e] = cs[nt][e];
    }
    stage_mm_t<T, MP>(sa, a, r0, lane);
    __syncthreads();
    if (tid < MP) {
      float c = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) c += part[w * MP + tid];
      svec[tid] = p.scale / fmaxf(c, p.min_col_mass);
    }
    __syncthreads();
    // u_k = c_k sum_i a_ik q_i for k in this warp's rows, staged over out_D (free after the logits)
    T* gu = static_cast<T*>(p.u) + head_off(p.uv, p.n1, bh);
#pragma unroll 1
    for (int half = 0; half < D / 64; ++half) {
      float u[8][4];
      zero_t(u);
      mm_tn64_t<T, DCH, MP>(u, sa, sq, half * 8, r0, m, lane);
      stage_rows64_t<T, OCH>(so, half * 8, u, svec, m, r0, lane);
    }
    __syncthreads();
    scatter<T, OCH>(gu, so, p.uv.rs, 0, DCH, m, p.b, j, 0, MP, tid, NTH);
  }
}

template <typename T, int D, bool LAST, int NW>
__global__ void __launch_bounds__(NW * 32) lstep_bwd_mmaw_kernel(const LstepParams p) {
  constexpr int MP = 16 * NW, DCH = D / 8, OW = LAST ? 2 * D : D, OCH = OW / 8, NTH = NW * 32;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, r0 = 16 * warp;
  const int m = (int)p.m;
  T* sq = reinterpret_cast<T*>(smem_raw);
  T* so = sq + (m + 1) * D;          // out rows (kr | y), later the dout staging
  T* sg = so + (m + 1) * OW;         // du (non-last) or dz (last), element dtype
  T* sd = sg + (m + 1) * D;          // dlog staging, MP x SA
  T* sa = sd + MP * Tile<MP>::SA;    // a staging (last), MP x SA
  float* part = reinterpret_cast<float*>(sa + MP * Tile<MP>::SA);  // [2][warp][k]: sums of a, of a G
  float* svec = part + 2 * NW * MP;                           // [2][k]: c_k, dcm_k

  const int64_t bh = blockIdx.x / p.b;
  const int j = (int)(blockIdx.x % p.b);
  const int64_t N = p.m * p.b;
  gather<T, DCH>(sq, static_cast<const T*>(p.q) + head_off(p.qv, p.n1, bh), p.qv.rs, 0, DCH, m, p.b, j, 0, tid, NTH);
  gather<T, OCH>(so, static_cast<const T*>(p.out) + head_off(p.outv, p.n1, bh), p.outv.rs, 0, OCH, m, p.b, j, 0, tid,
                 NTH);
  if (LAST)
    gather<T, DCH>(sg, static_cast<const T*>(p.dz) + head_off(p.dzv, p.n1, bh), p.dzv.rs, 0, DCH, m, p.b, j,
                   p.skip_rows, tid, NTH);
  cp_async_commit();
  zero_row<T, DCH>(sq, m, tid, NTH);
  zero_row<T, OCH>(so, m, tid, NTH);
  zero_row<T, DCH>(sg, m, tid, NTH);
  if (!LAST) {  // du is fp32: convert while the other rows are in flight, four chunks per round trip
    const float* du = p.du + head_off(p.duv, p.n1, bh);
    const int kChunks = (m * DCH + NTH - 1) / NTH;
#pragma unroll 1
    for (int t0 = 0; t0 < kChunks; t0 += 4) {
      float4 v[4][2];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = tid + NTH * (t0 + u), k = c / DCH, ch = c % DCH;
        if (k < m) {
          const float4* src = reinterpret_cast<const float4*>(du + ((int64_t)k * p.b + j) * p.duv.rs + ch * 8);
          v[u][0] = src[0];
          v[u][1] = src[1];
        } else {
          v[u][0] = v[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = tid + NTH * (t0 + u), k = c / DCH, ch = c % DCH;
        if (k >= m) continue;
        uint4 w;
        w.x = Elem<T>::pack(v[u][0].x, v[u][0].y);
        w.y = Elem<T>::pack(v[u][0].z, v[u][0].w);
        w.z = Elem<T>::pack(v[u][1].x, v[u][1].y);
        w.w = Elem<T>::pack(v[u][1].z, v[u][1].w);
        *reinterpret_cast<uint4*>(sg + swz<DCH>(k, ch)) = w;
      }
    }
  }
  float ent[MP / 8][2];
  load_ent<T, MP>(ent, p.ent + bh * N, p.b, j, m, lane);
  cp_async_wait<0>();
  __syncthreads();

  // a, then (non-last, once dlog is formed) a_ik c_k in place: two m x m arrays per thread
  float a[MP / 8][4], g[MP / 8][4];
#pragma unroll
  for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) a[nt][e] = g[nt][e] = 0.f;
  mm_rows_t<T, MP, D, DCH, OCH>(a, sq, 0, so, 0, r0, m, lane);
  softmax_t<MP>(a, ent, p.scale, m, r0, lane);
  if (LAST) {
    mm_rows_t<T, MP, D, DCH, OCH>(g, sg, 0, so, DCH, r0, m, lane);  // dA = dz y^T
  } else {
    // G = q du^T; column sums of a and of a G over all rows (every warp's partials)
    mm_rows_t<T, MP, D, DCH, DCH>(g, sq, 0, sg, 0, r0, m, lane);
    float cs[MP / 8][2], dc[MP / 8][2];
    col_sums_t<MP>(a, cs);
    col_sums_prod_t<MP>(a, g, dc);
    if ((lane >> 2) == 0) {
#pragma unroll
      for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          part[warp * MP + nt * 8 + lane * 2 + e] = cs[nt][e];
          part[(NW + warp) * MP + nt * 8 + lane * 2 + e] = dc[nt][e];
        }
    }
    __syncthreads();
    if (tid < MP) {
      float csum = 0.f, dsum = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        csum += part[w * MP + tid];
        dsum += part[(NW + w) * MP + tid];
      }
      const float cm = fmaxf(csum, p.min_col_mass);
      const float c = p.scale / cm;
      svec[tid] = c;
      svec[MP + tid] = csum > p.min_col_mass ? -dsum * c / cm : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int k = nt * 8 + (lane & 3) * 2 + e;
        const float c = svec[k], dcm = svec[MP + k];
#pragma unroll
        for (int h = 0; h < 2; ++h) g[nt][2 * h + e] = c * g[nt][2 * h + e] + dcm;  // dA
      }
  }
  // dlog = a (dA - rowsum(a dA)), in place in g and pre-multiplied by scale
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float rs = 0.f;
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt) rs += a[nt][2 * h] * g[nt][2 * h] + a[nt][2 * h + 1] * g[nt][2 * h + 1];
    rs += __shfl_xor_sync(0xffffffffu, rs, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) g[nt][2 * h + e] = a[nt][2 * h + e] * (g[nt][2 * h + e] - rs) * p.scale;
  }
  if (!LAST) {  // a -> a_ik c_k for the dq term
#pragma unroll
    for (int nt = 0; nt < MP / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float c = svec[nt * 8 + (lane & 3) * 2 + e];
        a[nt][e] *= c;
        a[nt][2 + e] *= c;
      }
  }

  // dq_i += sum_k (scale dlog_ik) out_k  [non-last: + sum_k (a_ik c_k) du_k] for this warp's rows
  float* gdq = p.dq + head_off(p.dqv, p.n1, bh);
#pragma unroll 1
  for (int half = 0; half < D / 64; ++half) {
    float acc[8][4];
    zero_t(acc);
    mm_rn64_t<T, OCH, MP>(acc, g, so, half * 8, m, lane);
    if (!LAST) mm_rn64_t<T, DCH, MP>(acc, a, sg, half * 8, m, lane);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = r0 + (lane >> 2) + h * 8;
      if (i >= m) continue;
      float* dst = gdq + ((int64_t)i * p.b + j) * p.dqv.rs + half * 64 + (lane & 3) * 2;
      if (p.dq_store) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<float2*>(dst + nt * 8) = make_float2(acc[nt][2 * h], acc[nt][2 * h + 1]);
      } else {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(dst + nt * 8), "f"(acc[nt][2 * h]),
                       "f"(acc[nt][2 * h + 1])
                       : "memory");
      }
    }
  }
  stage_mm_t<T, MP>(sd, g, r0, lane);
  if (LAST) stage_mm_t<T, MP>(sa, a, r0, lane);
  __syncthreads();  // dlog (and a) staged; every warp's dq products are done with the out rows

  // dout_k[:D] = sum_i (scale dlog_ik) q_i ; last: dout_k[D:] = sum_i a_ik dz_i, for k in this
  // warp's rows, staged over out with delta_k = sum_c out_k[c] dout_k[c] summed on the way
  T* gdo = static_cast<T*>(p.dout) + head_off(p.doutv, p.n1, bh);
  float dot[2] = {0.f, 0.f};
#pragma unroll 1
  for (int half = 0; half < D / 64; ++half) {
    float acc[8][4];
    zero_t(acc);
    mm_tn64_t<T, DCH, MP>(acc, sd, sq, half * 8, r0, m, lane);
    stage_rows64_dot_t<T, OCH>(so, half * 8, acc, dot, m, r0, lane);
  }
  if (LAST) {
#pragma unroll 1
    for (int half = 0; half < D / 64; ++half) {
      float acc[8][4];
      zero_t(acc);
      mm_tn64_t<T, DCH, MP>(acc, sa, sg, half * 8, r0, m, lane);
      stage_rows64_dot_t<T, OCH>(so, DCH + half * 8, acc, dot, m, r0, lane);
    }
  }
  if (p.delta_out) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float d = dot[h];
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      const int r = r0 + (lane >> 2) + h * 8;
      if ((lane & 3) == 0 && r < m) p.delta_out[bh * N + (int64_t)r * p.b + j] = d;
    }
  }
  __syncthreads();
  scatter<T, OCH>(gdo, so, p.doutv.rs, 0, OCH, m, p.b, j, 0, MP, tid, NTH);
}

template <typename T, int D, bool LAST, int NW>
cudaError_t launch_w(const LstepParams& p, bool bwd, cudaStream_t st) {
  constexpr int OW = LAST ? 2 * D : D;
  const size_t smem = lstepw_bytes((int)p.m, D, OW, bwd, sizeof(T), NW);
  auto kern = bwd ? lstep_bwd_mmaw_kernel<T, D, LAST, NW> : lstep_fwd_mmaw_kernel<T, D, LAST, NW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  const int64_t blocks = p.bh * p.b;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  if (blocks == 0) return cudaSuccess;
  kern<<<(unsigned)blocks, NW * 32, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T, int MP, int D, bool LAST>
cudaError_t launch(const LstepParams& p, bool bwd, cudaStream_t st) {
  constexpr int OW = LAST ? 2 * D : D;
  const size_t per_warp = lstep_warp_bytes<MP>((int)p.m, D, OW, bwd, sizeof(T));
  const int warps = bwd ? kWarpsBwd : kWarpsFwd;
  const size_t smem = per_warp * warps;
  auto kern = bwd ? lstep_bwd_mma_kernel<T, MP, D, LAST> : lstep_fwd_mma_kernel<T, MP, D, LAST>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // residency is bounded by shared memory: ask for the largest carveout
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (p.bh * p.b + warps - 1) / warps;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, warps * 32, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t dispatch_m(const LstepParams& p, bool last, bool bwd, cudaStream_t st) {
  if (p.m <= 16) return last ? launch<T, 16, D, true>(p, bwd, st) : launch<T, 16, D, false>(p, bwd, st);
  // 16 < m <= 32: the last step on one warp per column, the others on two (measured at m = 21:
  // 0.674 vs 0.70-0.73 ms for the last backward, 0.64 vs 0.686 ms for the non-last one)
  if (p.m <= 32) return last ? launch<T, 32, D, true>(p, bwd, st) : launch_w<T, D, false, 2>(p, bwd, st);
  if (p.m <= 64) return last ? launch_w<T, D, true, 4>(p, bwd, st) : launch_w<T, D, false, 4>(p, bwd, st);
  return last ? launch_w<T, D, true, 8>(p, bwd, st) : launch_w<T, D, false, 8>(p, bwd, st);
}

}  // namespace

bool lstep_mma_supported(const LstepParams& p, bool last) {
  return p.m <= kMaxMP && (p.d == 64 || p.d == 128) && p.dw == (last ? 2 * p.d : p.d);
}

cudaError_t lstep_mma_launch(const LstepParams& p, bool last, bool bwd, bool bf16, cudaStream_t st) {
  if (bf16) {
    return p.d == 64 ? dispatch_m<__nv_bfloat16, 64>(p, last, bwd, st) : dispatch_m<__nv_bfloat16, 128>(p, last, bwd, st);
  }
  return p.d == 64 ? dispatch_m<__half, 64>(p, last, bwd, st) : dispatch_m<__half, 128>(p, last, bwd, st);
}

}  // namespace vmb
