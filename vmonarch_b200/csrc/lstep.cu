// Monarch L step (the b dense m x m blocks), forward and backward.
//
// Reference: video_monarch_attention/vmonarch.py:51-63. For one (batch*head, grid column j),
// with q_i = q[i*b + j] (i = grid row / frame), kr_k = out[k*b + j, :D] * scale,
// y_k = out[k*b + j, D:] and ent_k = the R-step row entropy of token k*b + j:
//   logit_ik = q_i . kr_k                                (vmonarch.py:55)
//   a_ik     = softmax_k(logit_ik + ent_k)               (vmonarch.py:56, neg_ent = -ent)
//   last:     z_i = sum_k a_ik y_k                        (vmonarch.py:57-59)
//   non-last: cm_k = max(sum_i a_ik, min_col_mass)        (vmonarch.py:61)
//             u_k  = (sum_i a_ik q_i) * scale / cm_k      (vmonarch.py:62-63)
// The backward is the derivative of exactly these expressions; the entropy is detached in the
// reference (vmonarch.py:26), so no gradient flows into `ent`.
//
// One CTA handles one grid column: the m rows of q and out it needs are gathered with 16-byte
// loads (each row is a contiguous D- or Dw-wide slice), all contractions are m x m x D in fp32
// out of shared memory, and the CTA exclusively owns the rows it writes, so the fp32 dq
// accumulation needs no atomics.
#include "common.cuh"
#include "launch.h"

namespace vmb {

constexpr int kLstepThreads = 128;

struct LsSmem {
  float* q;   // [m][D+1]
  float* kr;  // [m][D+1]
  float* y;   // [m][DV+1]   (last)  or  du / dU'  [m][D+1] (non-last bwd)
  float* g;   // [m][DV+1]   dz (last bwd)  or  U' [m][D+1] (non-last bwd)
  float* a;   // [m][m+1]
  float* da;  // [m][m+1]
  float* vec; // [4][m]
};

template <typename T>
__device__ __forceinline__ void load_rows(float* dst, int ld, const T* base, int64_t row_elems, int col0,
                                          int ncols, int m, int64_t skip_before, int64_t b, int j) {
  // rows i = 0..m-1 at element offset (i*b + j) * row_elems + col0, ncols columns (multiple of 8)
  const int nch = ncols / 8;
  for (int c = threadIdx.x; c < m * nch; c += blockDim.x) {
    const int i = c / nch, ch = c % nch;
    const int64_t tok = (int64_t)i * b + j;
    float* d = dst + i * ld + ch * 8;
    if (tok < skip_before) {
#pragma unroll
      for (int e = 0; e < 8; ++e) d[e] = 0.f;
      continue;
    }
    const uint4 raw = *reinterpret_cast<const uint4*>(base + tok * row_elems + col0 + ch * 8);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Elem<T>::unpack(w[e]);
      d[2 * e] = f.x;
      d[2 * e + 1] = f.y;
    }
  }
}

// a[i][k] = softmax_k(q_i . kr_k + ent_k); warp w takes rows i = w, w+4, ..; lane takes k.
template <int D>
__device__ __forceinline__ void lstep_softmax(const LsSmem& s, const float* ent_s, int m) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < m; i += kLstepThreads / 32) {
    float lg[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = lane + 32 * h;
      float acc = -INFINITY;
      if (k < m) {
        acc = 0.f;
        const float* qi = s.q + i * (D + 1);
        const float* kk = s.kr + k * (D + 1);
#pragma unroll 8
        for (int d = 0; d < D; ++d) acc = fmaf(qi[d], kk[d], acc);
        acc += ent_s[k];
      }
      lg[h] = acc;
    }
    float mx = fmaxf(lg[0], lg[1]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float e0 = lane < m ? __expf(lg[0] - mx) : 0.f;
    float e1 = lane + 32 < m ? __expf(lg[1] - mx) : 0.f;
    float sum = e0 + e1;
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.f / sum;
    if (lane < m) s.a[i * (m + 1) + lane] = e0 * inv;
    if (lane + 32 < m) s.a[i * (m + 1) + lane + 32] = e1 * inv;
  }
}

template <typename T, int D>
__device__ __forceinline__ void lstep_load_common(const LstepParams& p, const LsSmem& s, int64_t bh, int j) {
  const int m = (int)p.m;
  const int64_t N = p.m * p.b;
  const T* q = static_cast<const T*>(p.q) + bh * N * D;
  const T* out = static_cast<const T*>(p.out) + bh * N * p.dw;
  load_rows<T>(s.q, D + 1, q, D, 0, D, m, 0, p.b, j);
  load_rows<T>(s.kr, D + 1, out, p.dw, 0, D, m, 0, p.b, j);
  for (int k = threadIdx.x; k < m; k += blockDim.x) s.vec[k] = p.ent[bh * N + (int64_t)k * p.b + j];
  __syncthreads();
  for (int c = threadIdx.x; c < m * D; c += blockDim.x) s.kr[(c / D) * (D + 1) + c % D] *= p.scale;
  __syncthreads();
}

template <typename T, int D, bool LAST>
__global__ void __launch_bounds__(kLstepThreads) lstep_fwd_kernel(const LstepParams p) {
  extern __shared__ float smf[];
  const int m = (int)p.m;
  const int dv = p.dw - D;
  const int64_t bh = blockIdx.x / p.b;
  const int j = (int)(blockIdx.x % p.b);
  const int64_t N = p.m * p.b;
  LsSmem s;
  s.q = smf;
  s.kr = s.q + m * (D + 1);
  s.y = s.kr + m * (D + 1);
  s.a = s.y + (LAST ? m * (dv + 1) : 0);
  s.vec = s.a + m * (m + 1);
  lstep_load_common<T, D>(p, s, bh, j);
  if (LAST) {
    load_rows<T>(s.y, dv + 1, static_cast<const T*>(p.out) + bh * N * p.dw, p.dw, D, dv, m, 0, p.b, j);
  }
  lstep_softmax<D>(s, s.vec, m);
  __syncthreads();

  if (LAST) {
    // z_i = sum_k a_ik y_k for tokens not covered by the exact recompute
    T* z = static_cast<T*>(p.z) + bh * N * dv;
    const int nch = dv / 8;
    for (int c = threadIdx.x; c < m * nch; c += blockDim.x) {
      const int i = c / nch, ch = c % nch;
      const int64_t tok = (int64_t)i * p.b + j;
      if (tok < p.skip_rows) continue;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int k = 0; k < m; ++k) {
        const float a = s.a[i * (m + 1) + k];
        const float* yk = s.y + k * (dv + 1) + ch * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(a, yk[e], acc[e]);
      }
      uint4 w;
      w.x = Elem<T>::pack(acc[0], acc[1]);
      w.y = Elem<T>::pack(acc[2], acc[3]);
      w.z = Elem<T>::pack(acc[4], acc[5]);
      w.w = Elem<T>::pack(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(z + tok * dv + ch * 8) = w;
    }
  } else {
    float* cscale = s.vec + m;  // scale / col_mass
    for (int k = threadIdx.x; k < m; k += blockDim.x) {
      float cs = 0.f;
      for (int i = 0; i < m; ++i) cs += s.a[i * (m + 1) + k];
      cscale[k] = p.scale / fmaxf(cs, p.min_col_mass);
    }
    __syncthreads();
    T* u = static_cast<T*>(p.u) + bh * N * D;
    constexpr int nch = D / 8;
    for (int c = threadIdx.x; c < m * nch; c += blockDim.x) {
      const int k = c / nch, ch = c % nch;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int i = 0; i < m; ++i) {
        const float a = s.a[i * (m + 1) + k];
        const float* qi = s.q + i * (D + 1) + ch * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(a, qi[e], acc[e]);
      }
      const float sc = cscale[k];
      uint4 w;
      w.x = Elem<T>::pack(acc[0] * sc, acc[1] * sc);
      w.y = Elem<T>::pack(acc[2] * sc, acc[3] * sc);
      w.z = Elem<T>::pack(acc[4] * sc, acc[5] * sc);
      w.w = Elem<T>::pack(acc[6] * sc, acc[7] * sc);
      *reinterpret_cast<uint4*>(u + ((int64_t)k * p.b + j) * D + ch * 8) = w;
    }
  }
}

// dlog_ik = a_ik (dA_ik - sum_k' a_ik' dA_ik') in place in s.da; warp per row.
__device__ __forceinline__ void softmax_bwd_rows(const LsSmem& s, int m) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < m; i += kLstepThreads / 32) {
    float a0 = 0.f, a1 = 0.f, g0 = 0.f, g1 = 0.f;
    if (lane < m) { a0 = s.a[i * (m + 1) + lane]; g0 = s.da[i * (m + 1) + lane]; }
    if (lane + 32 < m) { a1 = s.a[i * (m + 1) + lane + 32]; g1 = s.da[i * (m + 1) + lane + 32]; }
    float rs = a0 * g0 + a1 * g1;
#pragma unroll
    for (int o = 16; o; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
    if (lane < m) s.da[i * (m + 1) + lane] = a0 * (g0 - rs);
    if (lane + 32 < m) s.da[i * (m + 1) + lane + 32] = a1 * (g1 - rs);
  }
}

// dA_ik = sum_d X[i][d] * Y[k][d] (+ bias_k); warp per row i, lane per k.
__device__ __forceinline__ void rowdot(const float* X, int ldx, const float* Y, int ldy, int n, const float* bias,
                                       float* out, int m) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < m; i += kLstepThreads / 32) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = lane + 32 * h;
      if (k < m) {
        float acc = bias ? bias[k] : 0.f;
        const float* xi = X + i * ldx;
        const float* yk = Y + k * ldy;
        for (int d = 0; d < n; ++d) acc = fmaf(xi[d], yk[d], acc);
        out[i * (m + 1) + k] = acc;
      }
    }
  }
}

template <typename T, int D, bool LAST>
__global__ void __launch_bounds__(kLstepThreads) lstep_bwd_kernel(const LstepParams p) {
  extern __shared__ float smf[];
  const int m = (int)p.m;
  const int dv = LAST ? p.dw - D : D;
  const int64_t bh = blockIdx.x / p.b;
  const int j = (int)(blockIdx.x % p.b);
  const int64_t N = p.m * p.b;
  LsSmem s;
  s.q = smf;
  s.kr = s.q + m * (D + 1);
  s.y = s.kr + m * (D + 1);
  s.g = s.y + m * (dv + 1);
  s.a = s.g + m * (dv + 1);
  s.da = s.a + m * (m + 1);
  s.vec = s.da + m * (m + 1);
  lstep_load_common<T, D>(p, s, bh, j);
  if (LAST) {
    load_rows<T>(s.y, dv + 1, static_cast<const T*>(p.out) + bh * N * p.dw, p.dw, D, dv, m, 0, p.b, j);
    load_rows<T>(s.g, dv + 1, static_cast<const T*>(p.dz) + bh * N * dv, dv, 0, dv, m, p.skip_rows, p.b, j);
  } else {
    // du (fp32) -> s.y
    const float* du = p.du + bh * N * D;
    constexpr int nch = D / 4;
    for (int c = threadIdx.x; c < m * nch; c += blockDim.x) {
      const int k = c / nch, ch = c % nch;
      const float4 v = *reinterpret_cast<const float4*>(du + ((int64_t)k * p.b + j) * D + ch * 4);
      float* d = s.y + k * (D + 1) + ch * 4;
      d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
  }
  lstep_softmax<D>(s, s.vec, m);
  __syncthreads();

  T* dout = static_cast<T*>(p.dout) + bh * N * p.dw;
  float* dq = p.dq + bh * N * D;

  if (LAST) {
    // dA_ik = dz_i . y_k
    rowdot(s.g, dv + 1, s.y, dv + 1, dv, nullptr, s.da, m);
    __syncthreads();
    softmax_bwd_rows(s, m);
    __syncthreads();
    // dout[k, D:] = dy_k = sum_i a_ik dz_i
    for (int c = threadIdx.x; c < m * dv; c += blockDim.x) {
      const int k = c / dv, d = c % dv;
      float acc = 0.f;
      for (int i = 0; i < m; ++i) acc = fmaf(s.a[i * (m + 1) + k], s.g[i * (dv + 1) + d], acc);
      dout[((int64_t)k * p.b + j) * p.dw + D + d] = Elem<T>::from_f(acc);
    }
  } else {
    float* cs = s.vec + m;      // column sums
    float* cm = s.vec + 2 * m;  // clamped column mass
    float* dcm = s.vec + 3 * m;
    for (int k = threadIdx.x; k < m; k += blockDim.x) {
      float c = 0.f;
      for (int i = 0; i < m; ++i) c += s.a[i * (m + 1) + k];
      cs[k] = c;
      cm[k] = fmaxf(c, p.min_col_mass);
    }
    // U'_k = sum_i a_ik q_i  -> s.g
    for (int c = threadIdx.x; c < m * D; c += blockDim.x) {
      const int k = c / D, d = c % D;
      float acc = 0.f;
      for (int i = 0; i < m; ++i) acc = fmaf(s.a[i * (m + 1) + k], s.q[i * (D + 1) + d], acc);
      s.g[k * (D + 1) + d] = acc;
    }
    __syncthreads();
    // dc_k = du_k . U'_k ; dcm_k ; dU'_k = du_k * scale / cm_k (in place in s.y)
    {
      const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
      for (int k = warp; k < m; k += kLstepThreads / 32) {
        float acc = 0.f;
        for (int d = lane; d < D; d += 32) acc = fmaf(s.y[k * (D + 1) + d], s.g[k * (D + 1) + d], acc);
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        const float c = p.scale / cm[k];
        if (lane == 0) dcm[k] = cs[k] > p.min_col_mass ? -acc * c / cm[k] : 0.f;
        for (int d = lane; d < D; d += 32) s.y[k * (D + 1) + d] *= c;
      }
    }
    __syncthreads();
    // dA_ik = dU'_k . q_i + dcm_k
    rowdot(s.q, D + 1, s.y, D + 1, D, dcm, s.da, m);
    __syncthreads();
    softmax_bwd_rows(s, m);
    __syncthreads();
  }
  // dq_i += sum_k a_ik dU'_k (non-last) + sum_k dlog_ik kr_k
  for (int c = threadIdx.x; c < m * D; c += blockDim.x) {
    const int i = c / D, d = c % D;
    float acc = 0.f;
    for (int k = 0; k < m; ++k) {
      acc = fmaf(s.da[i * (m + 1) + k], s.kr[k * (D + 1) + d], acc);
      if (!LAST) acc = fmaf(s.a[i * (m + 1) + k], s.y[k * (D + 1) + d], acc);
    }
    float& dst = dq[((int64_t)i * p.b + j) * D + d];
    dst = p.dq_store ? acc : dst + acc;
  }
  // dout[k, :D] = scale * sum_i dlog_ik q_i
  for (int c = threadIdx.x; c < m * D; c += blockDim.x) {
    const int k = c / D, d = c % D;
    float acc = 0.f;
    for (int i = 0; i < m; ++i) acc = fmaf(s.da[i * (m + 1) + k], s.q[i * (D + 1) + d], acc);
    dout[((int64_t)k * p.b + j) * p.dw + d] = Elem<T>::from_f(acc * p.scale);
  }
}

size_t lstep_smem_bytes(int m, int d, int dw, bool last, bool bwd) {
  const int dv = last ? dw - d : d;
  size_t f = 2 * (size_t)m * (d + 1) + (size_t)m * (m + 1) + 4 * (size_t)m;
  if (!bwd) {
    if (last) f += (size_t)m * (dv + 1);
  } else {
    f += 2 * (size_t)m * (dv + 1) + (size_t)m * (m + 1);
  }
  return f * sizeof(float);
}

template <typename T, int D, bool LAST>
static cudaError_t launch_lstep_t(const LstepParams& p, bool bwd, cudaStream_t st) {
  const size_t smem = lstep_smem_bytes((int)p.m, D, p.dw, LAST, bwd);
  auto kern = bwd ? lstep_bwd_kernel<T, D, LAST> : lstep_fwd_kernel<T, D, LAST>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t blocks = p.bh * p.b;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, kLstepThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t dispatch_lstep(const LstepParams& p, bool last, bool bwd, cudaStream_t st) {
  if (p.d == 16) return last ? launch_lstep_t<T, 16, true>(p, bwd, st) : launch_lstep_t<T, 16, false>(p, bwd, st);
  if (p.d == 32) return last ? launch_lstep_t<T, 32, true>(p, bwd, st) : launch_lstep_t<T, 32, false>(p, bwd, st);
  if (p.d == 64) return last ? launch_lstep_t<T, 64, true>(p, bwd, st) : launch_lstep_t<T, 64, false>(p, bwd, st);
  if (p.d == 128) return last ? launch_lstep_t<T, 128, true>(p, bwd, st) : launch_lstep_t<T, 128, false>(p, bwd, st);
  return cudaErrorNotSupported;
}

cudaError_t lstep_launch(const LstepParams& p, bool last, bool bwd, bool bf16, cudaStream_t st) {
  return bf16 ? dispatch_lstep<__nv_bfloat16>(p, last, bwd, st) : dispatch_lstep<__half>(p, last, bwd, st);
}

}  // namespace vmb
