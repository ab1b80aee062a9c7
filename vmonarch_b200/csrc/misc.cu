// Small HBM-bound helpers of the FlashEntropyAttention backward.
//
// fea_bwd_pre replaces _attn_bwd_preprocess (video_monarch_attention/kernel.py:154-162) and also
// folds the entropy-gradient terms of kernel.py:202/241 into two per-row constants:
//   c_i = sum_d o_id dO_id + dE_i (E_i - LSE_i)     (LSE_i natural: LSE2_i * ln 2)
//   g_i = dE_i ln 2
// so the backward kernels compute dS = P (dP - c_i - g_i x_ij) with one extra FMA. For the tcgen05
// kernels the constants are folded once more (t = x - LSE2, P = 2^t):
//   nl_i = -LSE2_i,  nc_i = -sm_scale (c_i + g_i LSE2_i),  ng_i = -sm_scale g_i
// so that dS = P (sm_scale dP + nc + ng t), and written as three planes [batch][n_pad] with the
// rows past n_q set to (-1e30, 0, 0) (P = 0 and dS = 0 there): a query tile's statistics are
// then one aligned bulk copy per plane.
#include "common.cuh"
#include "launch.h"

namespace vmb {

// LPR lanes per row (dv / 32 of them: 2, 4 or 8), each loading four 16-byte chunks of o and of dO
// up front, so a warp has 32 / LPR rows and eight loads per lane in flight.
template <typename T, int LPR>
__global__ void __launch_bounds__(256) fea_bwd_pre_kernel(const T* o, int64_t o_bs, const T* dout, int64_t do_bs,
                                                          const float* lse, const float* ent, const float* dent,
                                                          float* cc, float* gg, int64_t rows, int n_q, int dv,
                                                          float* fold, int64_t n_pad, int64_t plane, float sm_scale,
                                                          const float* delta) {
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31, gl = lane % LPR;
  const int64_t row = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * RPW + lane / LPR;
  const int64_t rp = fold ? n_pad : n_q;  // rows are [batch][rp]
  const bool live = row < rows;
  const int64_t bi = live ? row / rp : 0, r = live ? row % rp : 0;
  const bool real = live && r < n_q;      // false: padding row of the folded planes
  float acc = 0.f;
  if (real && !delta) {
    const uint4* po = reinterpret_cast<const uint4*>(o + bi * o_bs + r * dv);
    const uint4* pd = reinterpret_cast<const uint4*>(dout + bi * do_bs + r * dv);
    uint4 va[4], vb[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      va[u] = po[gl + u * LPR];
      vb[u] = pd[gl + u * LPR];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t wa[4] = {va[u].x, va[u].y, va[u].z, va[u].w}, wb[4] = {vb[u].x, vb[u].y, vb[u].z, vb[u].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fa = Elem<T>::unpack(wa[e]), fb = Elem<T>::unpack(wb[e]);
        acc = fmaf(fa.x, fb.x, acc);
        acc = fmaf(fa.y, fb.y, acc);
      }
    }
  }
#pragma unroll
  for (int off = LPR / 2; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (!live || gl != 0) return;
  if (!real) {
    fold[row] = -1e30f;
    fold[plane + row] = 0.f;
    fold[2 * plane + row] = 0.f;
    return;
  }
  const int64_t src = bi * n_q + r;  // row of the [batch][n_q] inputs
  if (delta) acc = delta[src];       // sum o dO precomputed by the caller
  float c = acc, g = 0.f;
  if (dent) {
    const float de = dent[src];
    c = fmaf(de, ent[src] - lse[src] * kLn2, acc);
    g = de * kLn2;
  }
  if (fold) {
    const float l2 = lse[src];
    fold[row] = -l2;
    fold[plane + row] = -sm_scale * fmaf(g, l2, c);
    fold[2 * plane + row] = -sm_scale * g;
  } else {
    cc[src] = c;
    if (gg) gg[src] = g;
  }
}

template <typename T, int LPR>
void launch_pre(const void* o, int64_t o_bs, const void* dout, int64_t do_bs, const float* lse, const float* ent,
                const float* dent, float* cc, float* gg, int64_t rows, int n_q, int dv, float* fold, int64_t n_pad,
                int64_t plane, float sm_scale, const float* delta, cudaStream_t st) {
  const int64_t warps = (rows + 32 / LPR - 1) / (32 / LPR);
  fea_bwd_pre_kernel<T, LPR><<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
      static_cast<const T*>(o), o_bs, static_cast<const T*>(dout), do_bs, lse, ent, dent, cc, gg, rows, n_q, dv, fold,
      n_pad, plane, sm_scale, delta);
}

cudaError_t fea_bwd_pre(const void* o, int64_t o_bs, const void* dout, int64_t do_bs, const float* lse,
                        const float* ent, const float* dent, float* cc, float* gg, int64_t batch, int n_q, int dv,
                        float* fold, int64_t n_pad, float sm_scale, const float* delta, bool bf16, cudaStream_t st) {
  const int64_t rows = batch * (fold ? n_pad : n_q);
  const int64_t plane = batch * n_pad;
  if ((rows + 3) / 4 / 8 + 1 > 0x7fffffff) return cudaErrorInvalidConfiguration;
  if (dv != 64 && dv != 128 && dv != 256) return cudaErrorInvalidValue;
  const int lpr = dv / 32;
#define VMB_PRE(TT, L) launch_pre<TT, L>(o, o_bs, dout, do_bs, lse, ent, dent, cc, gg, rows, n_q, dv, fold, n_pad, plane, sm_scale, delta, st)
  if (bf16) {
    if (lpr == 2) VMB_PRE(__nv_bfloat16, 2); else if (lpr == 4) VMB_PRE(__nv_bfloat16, 4); else VMB_PRE(__nv_bfloat16, 8);
  } else {
    if (lpr == 2) VMB_PRE(__half, 2); else if (lpr == 4) VMB_PRE(__half, 4); else VMB_PRE(__half, 8);
  }
#undef VMB_PRE
  return cudaGetLastError();
}

// dst[b][i] = (T) src[b][i] for i < n, 4 elements per thread (n % 4 == 0, strides % 4 == 0)
template <typename T>
__global__ void cast_f32_kernel(const float* src, int64_t src_bs, T* dst, int64_t dst_bs, int64_t n4, int64_t total4) {
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total4; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bi = idx / n4, i = (idx % n4) * 4;
    const float4 v = *reinterpret_cast<const float4*>(src + bi * src_bs + i);
    uint2 w;
    w.x = Elem<T>::pack(v.x, v.y);
    w.y = Elem<T>::pack(v.z, v.w);
    *reinterpret_cast<uint2*>(dst + bi * dst_bs + i) = w;
  }
}

cudaError_t cast_f32(const float* src, int64_t src_bs, void* dst, int64_t dst_bs, int64_t batch, int64_t n, bool bf16,
                     cudaStream_t st) {
  const int64_t n4 = n / 4, total4 = batch * n4;
  if (total4 == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total4 + 255) / 256;
  const unsigned blocks = (unsigned)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  if (bf16)
    cast_f32_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(src, src_bs, static_cast<__nv_bfloat16*>(dst), dst_bs, n4, total4);
  else
    cast_f32_kernel<__half><<<blocks, 256, 0, st>>>(src, src_bs, static_cast<__half*>(dst), dst_bs, n4, total4);
  return cudaGetLastError();
}

}  // namespace vmb
