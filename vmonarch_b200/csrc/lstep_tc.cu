// Monarch L step on tcgen05 / TMEM / TMA, D = 128, m <= 32 (reference: video_monarch_attention/
// vmonarch.py:51-63). For every grid column j of a head the L step is an m x m problem:
//   logits_ik = q_i . kr_k (kr = out[:, :D]),  a = softmax_k(scale logits + ent_k),
//   non-last:  u_k = scale / max(sum_i a_ik, min_col_mass) * sum_i a_ik q_i,
//   last:      z_i = sum_k a_ik y_k (y = out[:, D:2D]).
// Stacking. A CTA takes 4 consecutive columns j0 .. j0+3 of one head; column jj owns rows
// [32 jj, 32 jj + 32) of 128-row operand tiles (row 32 jj + i = token i b + j0 + jj), brought in by
// one TMA box {64 elements, 1 column, 32 rows} per column and 64-wide atom (128-byte swizzled
// K-major rows, each box on a 4 KB boundary); rows i >= m lie past the tensor's m rows, so the
// load zero-fills them and the store skips them.
//   L = Q O^T (M = N = 128, K = D) holds the four columns' logits as 32 x 32 diagonal blocks.
//   Warp jj = column jj and lane i = row i: the warp loads the 32 TMEM columns of its own block,
//   softmaxes row i over k < m, and sums the columns across its lanes (a 31-shuffle reduce-
//   scatter leaves sum_i a_ik in lane k). A (bf16, zero off the diagonal blocks) goes to shared
//   memory.
//   non-last: U = A^T Q (A read M-major): lane k of warp jj holds row 32 jj + k = u_k up to the
//             factor scale / max(mass_k, min_col_mass), which that lane already has.
//   last:     Z = A Y (Y read N-major).
// Outputs are staged in the same layout and written back by the same boxes (columns past b and
// rows past m are clipped). The CTAs are persistent (a few per SM, each walking column groups
// g, g + grid, ...): TMEM, barriers and tensor maps are set up once, and the next group's boxes
// are prefetched into L2 while the current one computes. Every wait is bounded.
#include <algorithm>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace vmb {

__device__ int g_lstep_err;

namespace {

using namespace sm100;

constexpr int kAtom = 128 * 128;  // one swizzle-atom column block: 128 rows x 128 B
constexpr int kCols = 4;          // grid columns per CTA (32 rows each)

struct LstepTcParams {
  CUtensorMap tm_q, tm_o, tm_y;  // q [m][b][D], out [m][b][DW], output u / z [m][b][D] per head
  const float* ent;              // [bh][N]
  int64_t b, n;                  // columns per head, tokens per head (m b)
  int m, nblk;                   // rows per column, column groups per head
  int n1;                        // head index split of the column maps (hb % n1, hb / n1)
  int64_t n_groups;              // bh * nblk
  float scale, min_col_mass;
};

// Column maps are rank 5: (element, grid column j, grid row i, c1, c3), the head index hb split as
// c1 = hb % n1 and c3 = hb / n1 (make_map_col); callers split hb once per column group.
__device__ __forceinline__ void tma_load_col(uint32_t dst, const CUtensorMap* map, int x, int j, int c1, int c3,
                                             uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(j), "r"(0), "r"(c1), "r"(c3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_store_col(const CUtensorMap* map, int x, int j, int c1, int c3, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4, %5}], [%6];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(j), "r"(0), "r"(c1), "r"(c3), "r"(src)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_col(const CUtensorMap* map, int x, int j, int c1, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(j), "r"(0), "r"(c1), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Lane l ends with sum over the warp's lanes of v[l] (31 shuffles: each round halves the vector,
// keeping the half whose index bit equals the lane's bit and adding the partner's copy of it).
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int half = 16; half >= 1; half >>= 1) {
    const bool up = lane & half;
#pragma unroll
    for (int t = 0; t < half; ++t) {
      const float send = up ? v[t] : v[t + half];
      const float keep = up ? v[t + half] : v[t];
      v[t] = keep + __shfl_xor_sync(0xffffffffu, send, half);
    }
  }
  return v[0];
}

template <bool LAST>
struct FwdCfg {
  static constexpr int OATOMS = LAST ? 4 : 2;  // out: kr (| y)
  static constexpr int SQ = 0;                 // Q: 2 atoms; later the output staging
  static constexpr int SO = 2 * kAtom;         // out atoms; A is written over kr
  static constexpr int SENT = SO + OATOMS * kAtom;
  static constexpr int SMEM = 1024 + SENT + kCols * 32 * 4;
};

// grid: bh * nblk CTAs of 128 threads (warp = grid column, lane = row of that column)
template <typename T, bool LAST>
__global__ void __launch_bounds__(128, 3) lstep_fwd_tc_kernel(const __grid_constant__ LstepTcParams p) {
  using C = FwdCfg<LAST>;
  constexpr bool kBf16 = Elem<T>::is_bf16;
  constexpr uint32_t IDESC_L = idesc_f16(kBf16, 128, 128, false, false);  // Q O^T
  constexpr uint32_t IDESC_U = idesc_f16(kBf16, 128, 128, true, true);    // A^T Q
  constexpr uint32_t IDESC_Z = idesc_f16(kBf16, 128, 128, false, true);   // A Y

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_sh;
  __shared__ int abort_sh;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = p.m;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sQ = base + C::SQ, sO = base + C::SO, sA = sO;
  float* sEnt = reinterpret_cast<float*>(smem_raw + (base - smem_u32(smem_raw)) + C::SENT);
  const uint32_t bar_ld = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);
  volatile int* abort = &abort_sh;
  constexpr uint32_t kLoadBytes = kCols * (2 + C::OATOMS) * 32 * 128;  // full boxes, zero-filled rows included

  if (tid == 0) {
    abort_sh = 0;
    mbar_init(bar_ld, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    prefetch_tmap(&p.tm_q);
    prefetch_tmap(&p.tm_o);
    prefetch_tmap(&p.tm_y);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_sh), 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const float sl2 = p.scale * kLog2e;

  auto load_group = [&](int64_t g) {  // thread 0
    const int hb = (int)(g / p.nblk), j0 = (int)(g % p.nblk) * kCols;
    const int c3 = hb / p.n1, c1 = hb - c3 * p.n1;
    mbar_expect_tx(bar_ld, kLoadBytes);
    for (int c = 0; c < kCols; ++c) {
      const uint32_t ro = c * 32 * 128;
      tma_load_col(sQ + ro, &p.tm_q, 0, j0 + c, c1, c3, bar_ld);
      tma_load_col(sQ + kAtom + ro, &p.tm_q, 64, j0 + c, c1, c3, bar_ld);
      for (int a = 0; a < C::OATOMS; ++a) tma_load_col(sO + a * kAtom + ro, &p.tm_o, 64 * a, j0 + c, c1, c3, bar_ld);
    }
  };
  auto prefetch_group = [&](int64_t g) {  // thread 0: the boxes of a later group into L2
    const int hb = (int)(g / p.nblk), j0 = (int)(g % p.nblk) * kCols;
    const int c3 = hb / p.n1, c1 = hb - c3 * p.n1;
    for (int c = 0; c < kCols; ++c) {
      tma_prefetch_col(&p.tm_q, 0, j0 + c, c1, c3);
      tma_prefetch_col(&p.tm_q, 64, j0 + c, c1, c3);
      for (int a = 0; a < C::OATOMS; ++a) tma_prefetch_col(&p.tm_o, 64 * a, j0 + c, c1, c3);
    }
  };

  bool ok = true;
  int it = 0;       // groups of this CTA so far: phase it & 1 of bar_ld, phases 2 it, 2 it + 1 of bar_mma
  int loaded = 0;   // loads issued on bar_ld (drained before exit)
  int mma_phases = 0;  // commits issued on bar_mma (drained before exit)
  if (tid == 0 && (int64_t)blockIdx.x < p.n_groups) {
    load_group(blockIdx.x);
    ++loaded;
  }
  for (int64_t g = blockIdx.x; g < p.n_groups && ok; g += gridDim.x, ++it) {
    const int hb = (int)(g / p.nblk), j0 = (int)(g % p.nblk) * kCols;
    if (tid == 0 && g + gridDim.x < p.n_groups) prefetch_group(g + gridDim.x);
    {  // entropies of this warp's column (lane k -> token k b + j), while the boxes are in flight
      const int64_t j = (int64_t)j0 + warp;
      sEnt[tid] = (lane < m && j < p.b) ? p.ent[(int64_t)hb * p.n + lane * p.b + j] : 0.f;
    }
    __syncwarp();
    ok = __all_sync(0xffffffffu, mbar_wait(bar_ld, it & 1, abort, &g_lstep_err, 1));
    tc_fence_after();
    if (warp == 0) {
      const uint32_t leader = (elect_one() && ok) ? 1u : 0u;
      mma_phases += ok ? 1 : 0;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // L = Q kr^T over D
        const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
        mma_ss_if(leader, tmem, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(sO + off, 16, 1024), IDESC_L, kk > 0);
      }
      mma_commit_if(leader, bar_mma);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_mma, 0, abort, &g_lstep_err, 2));
    tc_fence_after();

    // ---- softmax of row i = lane over k < m (the 32 TMEM columns of this warp's block)
    uint32_t raw[32];
    if (ok) {
      tmem_ld32(tmem + lane_off + 32 * warp, raw);
      tmem_wait_ld();
    }
    float a[32];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float x = (k < m) ? fmaf(__uint_as_float(raw[k]), sl2, sEnt[32 * warp + k] * kLog2e) : -INFINITY;
      a[k] = x;
      mx = fmaxf(mx, x);
    }
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float e = (k < m) ? fast_exp2(a[k] - mx) : 0.f;
      a[k] = e;
      sum += e;
    }
    const float inv = lane < m ? 1.f / sum : 0.f;
    {  // A row 32 warp + lane: this block's 32 columns, zeros in the other blocks (over kr, consumed)
      const int row = 32 * warp + lane;
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if ((ch >> 2) == warp) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = 8 * (ch & 3) + 2 * e;
            w[e] = Elem<T>::pack(a[k] * inv, a[k + 1] * inv);
          }
        }
        st_shared_v4(sA + (ch >> 3) * kAtom + row * 128 + (((ch & 7) ^ (row & 7)) << 4), w[0], w[1], w[2], w[3]);
      }
    }
    float colscale = 1.f;
    if (!LAST) {  // column masses of this block: lane k gets sum_i a_ik
#pragma unroll
      for (int k = 0; k < 32; ++k) a[k] *= inv;
      const float mass = warp_reduce_scatter32(a, lane);
      colscale = p.scale / fmaxf(mass, p.min_col_mass);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {
      const uint32_t leader = (elect_one() && ok) ? 1u : 0u;
      mma_phases += ok ? 1 : 0;
      if (!LAST) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // U = A^T Q over the 128 stacked rows
          mma_ss_if(leader, tmem, smem_desc_sw128(sA + kk * 2048, kAtom, 1024), smem_desc_sw128(sQ + kk * 2048, kAtom, 1024),
                    IDESC_U, kk > 0);
      } else {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // Z = A Y over the 128 stacked columns
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          mma_ss_if(leader, tmem, smem_desc_sw128(sA + off, 16, 1024),
                    smem_desc_sw128(sO + 2 * kAtom + kk * 2048, kAtom, 1024), IDESC_Z, kk > 0);
        }
      }
      mma_commit_if(leader, bar_mma);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_mma, 1, abort, &g_lstep_err, 4));
    tc_fence_after();

    // ---- epilogue: row 32 warp + lane of U (u_k, k = lane) or Z (z_i, i = lane) -> 16-bit into Q's atoms
    if (ok) {
      const int row = 32 * warp + lane;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {  // 32 columns at a time: 16-byte chunks 4c .. 4c + 3 of the row
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = 4 * c + q;
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = Elem<T>::pack(__uint_as_float(v[8 * q + 2 * e]) * colscale, __uint_as_float(v[8 * q + 2 * e + 1]) * colscale);
          st_shared_v4(sQ + (ch >> 3) * kAtom + row * 128 + (((ch & 7) ^ (row & 7)) << 4), w[0], w[1], w[2], w[3]);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok ? 1 : 0) != 0;
    tc_fence_after();
    if (tid == 0 && ok && !*abort) {
      const int c3 = hb / p.n1, c1 = hb - c3 * p.n1;
      for (int c = 0; c < kCols; ++c) {
        tma_store_col(&p.tm_y, 0, j0 + c, c1, c3, sQ + c * 32 * 128);
        tma_store_col(&p.tm_y, 64, j0 + c, c1, c3, sQ + kAtom + c * 32 * 128);
      }
      tma_store_commit_and_wait();  // the staging (Q's atoms) is read before the next group's load
      if (g + gridDim.x < p.n_groups) {
        load_group(g + gridDim.x);
        ++loaded;
      }
    }
    ok = __syncthreads_and(ok && !*abort ? 1 : 0) != 0;
  }
  if (tid == 0) {  // after a timed-out wait: let in-flight copies and MMAs land before exit
    if (loaded > 0) mbar_wait_drain(bar_ld, (loaded - 1) & 1);
    if (mma_phases > 0) mbar_wait_drain(bar_mma, (mma_phases - 1) & 1);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// 5-D map over the view `v` of one [bh][N][W] tensor of 16-bit elements (token i b + j of head hb
// at row i b + j): dims (W, b, m, n1, bh / n1), boxes {64 elements, 1 column, 32 rows, 1, 1},
// 128-byte swizzle. Rows past m are zero-filled on load and skipped on store. The view's split
// must have n2 = 1 (hb = c1 + n1 c3).
bool make_map_col(CUtensorMap* map, const void* ptr, bool bf16, int W, int64_t b, int64_t m, int64_t bh,
                  const View& v, int n1) {
  tma::EncodeTiledFn enc = tma::encode_fn();
  if (!enc || n1 < 1 || bh % n1) return false;
  const int64_t n3 = bh / n1;
  cuuint64_t dims[5] = {(cuuint64_t)W, (cuuint64_t)b, (cuuint64_t)m, (cuuint64_t)n1, (cuuint64_t)n3};
  int64_t st[4] = {v.rs * 2, v.rs * b * 2, v.s1 * 2, v.s3 * 2};
  const int64_t ext[4] = {b, m, n1, n3};
  for (int i = 0; i < 4; ++i) {
    if (ext[i] == 1 && (st[i] <= 0 || st[i] % 16)) st[i] = v.rs * b * m * 2;  // unused stride
    if (st[i] <= 0 || st[i] % 16) return false;
  }
  cuuint64_t strides[4] = {(cuuint64_t)st[0], (cuuint64_t)st[1], (cuuint64_t)st[2], (cuuint64_t)st[3]};
  cuuint32_t box[5] = {64, 1, 32, 1, 1};  // rows past m: zero-filled on load, skipped on store
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(ptr),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, bool LAST>
cudaError_t launch_fwd(const LstepParams& lp, cudaStream_t st) {
  constexpr bool bf16 = Elem<T>::is_bf16;
  LstepTcParams p{};
  p.m = (int)lp.m;
  p.b = lp.b;
  p.n = lp.m * lp.b;
  p.nblk = (int)((lp.b + kCols - 1) / kCols);
  p.n_groups = lp.bh * p.nblk;
  p.ent = lp.ent;
  p.scale = lp.scale;
  p.min_col_mass = lp.min_col_mass;
  p.n1 = lp.n1;
  if (!make_map_col(&p.tm_q, lp.q, bf16, 128, lp.b, lp.m, lp.bh, lp.qv, lp.n1)) return cudaErrorInvalidValue;
  if (!make_map_col(&p.tm_o, lp.out, bf16, lp.dw, lp.b, lp.m, lp.bh, lp.outv, lp.n1)) return cudaErrorInvalidValue;
  if (!make_map_col(&p.tm_y, LAST ? lp.z : lp.u, bf16, 128, lp.b, lp.m, lp.bh, LAST ? lp.zv : lp.uv, lp.n1))
    return cudaErrorInvalidValue;
  auto kern = lstep_fwd_tc_kernel<T, LAST>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdCfg<LAST>::SMEM);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148, smem_sm = 233472;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  }
  // resident CTAs per SM: shared memory (+1 KB reserved per CTA) bounds it; 128 registers x 128
  // threads allow four
  const int per_sm = std::max(1, std::min(4, smem_sm / (FwdCfg<LAST>::SMEM + 1024)));
  const int64_t blocks = std::min<int64_t>(p.n_groups, (int64_t)sms * per_sm);
  if (blocks < 1) return cudaSuccess;
  kern<<<(unsigned)blocks, 128, FwdCfg<LAST>::SMEM, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

bool lstep_tc_supported(const LstepParams& p, bool last, bool bwd) {
  if (bwd || p.d != 128 || p.m < 1 || p.m > 32) return false;
  if (p.dw != (last ? 256 : 128)) return false;
  return !last || p.skip_rows == 0;  // the stacked TMA store cannot leave tokens < skip_rows unwritten
}

cudaError_t lstep_tc_launch(const LstepParams& p, bool last, bool bwd, bool bf16, cudaStream_t st) {
  if (bwd) return cudaErrorInvalidValue;
  if (bf16) return last ? launch_fwd<__nv_bfloat16, true>(p, st) : launch_fwd<__nv_bfloat16, false>(p, st);
  return last ? launch_fwd<__half, true>(p, st) : launch_fwd<__half, false>(p, st);
}

cudaError_t lstep_tc_status(cudaStream_t st, int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_lstep_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && *out) e = cudaMemcpyToSymbolAsync(g_lstep_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e;
}

}  // namespace vmb
