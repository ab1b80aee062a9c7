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

// LPR lanes per row, each loading CPL 16-byte chunks of o and of dO up front (dv = 8 CPL LPR: 16
// and 32 take one lane with two or four chunks, 64 / 128 / 256 take 2 / 4 / 8 lanes with four), so
// a warp has 32 / LPR rows and 2 CPL loads per lane in flight.
template <typename T, int LPR, int CPL>
__global__ void __launch_bounds__(256) fea_bwd_pre_kernel(const T* o, View ov, const T* dout, View dov, int n1, int n2,
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
    const uint4* po = reinterpret_cast<const uint4*>(o + view_offset(ov, n1, n2, bi, r));
    const uint4* pd = reinterpret_cast<const uint4*>(dout + view_offset(dov, n1, n2, bi, r));
    uint4 va[CPL], vb[CPL];
#pragma unroll
    for (int u = 0; u < CPL; ++u) {
      va[u] = po[gl + u * LPR];
      vb[u] = pd[gl + u * LPR];
    }
#pragma unroll
    for (int u = 0; u < CPL; ++u) {
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

template <typename T, int LPR, int CPL>
void launch_pre(const void* o, View ov, const void* dout, View dov, int n1, int n2, const float* lse, const float* ent,
                const float* dent, float* cc, float* gg, int64_t rows, int n_q, int dv, float* fold, int64_t n_pad,
                int64_t plane, float sm_scale, const float* delta, cudaStream_t st) {
  const int64_t warps = (rows + 32 / LPR - 1) / (32 / LPR);
  fea_bwd_pre_kernel<T, LPR, CPL><<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
      static_cast<const T*>(o), ov, static_cast<const T*>(dout), dov, n1, n2, lse, ent, dent, cc, gg, rows, n_q, dv, fold,
      n_pad, plane, sm_scale, delta);
}

cudaError_t fea_bwd_pre(const void* o, View ov, const void* dout, View dov, int n1, int n2, const float* lse,
                        const float* ent, const float* dent, float* cc, float* gg, int64_t batch, int n_q, int dv,
                        float* fold, int64_t n_pad, float sm_scale, const float* delta, bool bf16, cudaStream_t st) {
  const int64_t rows = batch * (fold ? n_pad : n_q);
  const int64_t plane = batch * n_pad;
  if ((rows + 3) / 4 / 8 + 1 > 0x7fffffff) return cudaErrorInvalidConfiguration;
#define VMB_PRE(TT, L, C) launch_pre<TT, L, C>(o, ov, dout, dov, n1, n2, lse, ent, dent, cc, gg, rows, n_q, dv, fold, n_pad, plane, sm_scale, delta, st)
#define VMB_PRE_ALL(TT)                          \
  switch (dv) {                                  \
    case 16: VMB_PRE(TT, 1, 2); break;           \
    case 32: VMB_PRE(TT, 1, 4); break;           \
    case 64: VMB_PRE(TT, 2, 4); break;           \
    case 128: VMB_PRE(TT, 4, 4); break;          \
    case 256: VMB_PRE(TT, 8, 4); break;          \
    default: return cudaErrorInvalidValue;       \
  }
  if (bf16) {
    VMB_PRE_ALL(__nv_bfloat16)
  } else {
    VMB_PRE_ALL(__half)
  }
#undef VMB_PRE_ALL
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

// dst(s, r, c) = (T) src(s, r, c) over [batch][rows][cols] views (cols % 4 == 0, 16-byte aligned
// rows): the fp32 accumulator of a strided (e.g. token-major) gradient converted in place of
// cast_f32's flat rows. Grid row y = batch entries y, y + gridDim.y, ...; one warp per four tensor
// rows, lane = 4 columns, so the view offsets are computed once per batch entry and there is no
// division per element.
template <typename T>
__global__ void __launch_bounds__(256) cast_f32_view_kernel(const float* src, View sv, T* dst, View dvw, int n1, int n2,
                                                            int64_t batch, int64_t rows, int c4n) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int64_t bi = blockIdx.y; bi < batch; bi += gridDim.y) {
    const float* s0 = src + view_offset(sv, n1, n2, bi, 0);
    T* d0 = dst + view_offset(dvw, n1, n2, bi, 0);
    // four rows per warp and pass: four 16-byte loads in flight per lane before the stores
    for (int64_t r0 = ((int64_t)blockIdx.x * warps + (threadIdx.x >> 5)) * 4; r0 < rows;
         r0 += (int64_t)gridDim.x * warps * 4) {
      const int nr = rows - r0 < 4 ? (int)(rows - r0) : 4;
      for (int c = lane; c < c4n; c += 32) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (u < nr) v[u] = *reinterpret_cast<const float4*>(s0 + (r0 + u) * sv.rs + 4 * c);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (u < nr) {
            uint2 w;
            w.x = Elem<T>::pack(v[u].x, v[u].y);
            w.y = Elem<T>::pack(v[u].z, v[u].w);
            *reinterpret_cast<uint2*>(d0 + (r0 + u) * dvw.rs + 4 * c) = w;
          }
        }
      }
    }
  }
}

cudaError_t cast_f32_view(const float* src, const View& sv, void* dst, const View& dvw, int n1, int n2, int64_t batch,
                          int64_t rows, int64_t cols, bool bf16, cudaStream_t st) {
  if (batch == 0 || rows == 0 || cols == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // about eight 256-thread blocks per SM over the whole grid
  const int64_t gy = batch < 65535 ? batch : 65535;
  int64_t gx = ((int64_t)sms * 8 + gy - 1) / gy;
  const int64_t need = (rows + 31) / 32;  // 8 warps x 4 rows per block and pass
  if (gx > need) gx = need;
  if (gx < 1) gx = 1;
  const dim3 grid((unsigned)gx, (unsigned)gy);
  const int c4n = (int)(cols / 4);
  if (bf16)
    cast_f32_view_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(src, sv, static_cast<__nv_bfloat16*>(dst), dvw, n1, n2,
                                                              batch, rows, c4n);
  else
    cast_f32_view_kernel<__half><<<grid, 256, 0, st>>>(src, sv, static_cast<__half*>(dst), dvw, n1, n2, batch, rows, c4n);
  return cudaGetLastError();
}

// e4m3 operands of the fp8 R step: dst(s, r, c) = e4m3(scale * src(s, r, c)), rounded to nearest,
// saturating. Same walk as cast_f32_view: one warp per four rows, lane = 8 columns (one 16-byte load,
// one 8-byte store), view offsets once per batch entry.
template <typename T>
__global__ void __launch_bounds__(256) quant_e4m3_kernel(const T* src, View sv, uint8_t* dst, View dvw, int n1, int n2,
                                                         int64_t batch, int64_t rows, int c8n, float scale) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int64_t bi = blockIdx.y; bi < batch; bi += gridDim.y) {
    const T* s0 = src + view_offset(sv, n1, n2, bi, 0);
    uint8_t* d0 = dst + view_offset(dvw, n1, n2, bi, 0);
    for (int64_t r0 = ((int64_t)blockIdx.x * warps + (threadIdx.x >> 5)) * 4; r0 < rows;
         r0 += (int64_t)gridDim.x * warps * 4) {
      const int nr = rows - r0 < 4 ? (int)(rows - r0) : 4;
      for (int c = lane; c < c8n; c += 32) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (u < nr) v[u] = *reinterpret_cast<const uint4*>(s0 + (r0 + u) * sv.rs + 8 * c);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (u < nr) {
            const uint32_t w4[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
            uint32_t q[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float2 a = Elem<T>::unpack(w4[2 * h]), b = Elem<T>::unpack(w4[2 * h + 1]);
              q[h] = pack_e4m3x2(a.x * scale, a.y * scale) | (pack_e4m3x2(b.x * scale, b.y * scale) << 16);
            }
            *reinterpret_cast<uint2*>(d0 + (r0 + u) * dvw.rs + 8 * c) = make_uint2(q[0], q[1]);
          }
        }
      }
    }
  }
}

cudaError_t quant_e4m3(const void* src, const View& sv, void* dst, const View& dvw, int n1, int n2, int64_t batch,
                       int64_t rows, int64_t cols, bool bf16, float scale, cudaStream_t st) {
  if (batch == 0 || rows == 0 || cols == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t gy = batch < 65535 ? batch : 65535;
  int64_t gx = ((int64_t)sms * 8 + gy - 1) / gy;
  const int64_t need = (rows + 31) / 32;  // 8 warps x 4 rows per block and pass
  if (gx > need) gx = need;
  if (gx < 1) gx = 1;
  const dim3 grid((unsigned)gx, (unsigned)gy);
  const int c8n = (int)(cols / 8);
  uint8_t* d = static_cast<uint8_t*>(dst);
  if (bf16)
    quant_e4m3_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(src), sv, d, dvw, n1, n2,
                                                           batch, rows, c8n, scale);
  else
    quant_e4m3_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(src), sv, d, dvw, n1, n2, batch, rows,
                                                    c8n, scale);
  return cudaGetLastError();
}

}  // namespace vmb
