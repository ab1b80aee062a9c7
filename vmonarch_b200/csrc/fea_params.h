// Kernel-side parameter blocks for the FlashEntropyAttention kernels. These are filled by the
// C-ABI layer (capi.cu) from the public argument structs declared in include/vmonarch_b200.h.
#pragma once
#include <stdint.h>

namespace vmb {

// A tensor seen as [batch][rows][cols] (16-bit or fp32 elements, contiguous columns). The batch
// index s of a call splits as c1 = s % n1, c2 = s / n1 % n2, c3 = s / (n1 * n2), with (n1, n2)
// shared by every tensor of the call, and element (s, r, c) lies at
//   c + r * rs + c1 * s1 + c2 * s2 + c3 * s3   (elements).
// A dense tensor with batch stride bs is dense_view(cols, bs, n1, n2); a token-major caller tensor
// (B, N, H, D) has rs = H * D and head stride D, so no transpose is ever made.
struct View {
  int64_t rs, s1, s2, s3;
};

inline View dense_view(int64_t cols, int64_t bs, int n1, int n2) {
  return View{cols, bs, bs * n1, bs * (int64_t)n1 * n2};
}

#ifdef __CUDACC__
__host__ __device__
#endif
inline int64_t view_offset(const View& v, int n1, int n2, int64_t s, int64_t r) {
  // batch indices fit 32 bits (the launch grids bound them), so the split is 32-bit arithmetic
  const int si = (int)s, t = si / n1, c1 = si - t * n1, c3 = t / n2, c2 = t - c3 * n2;
  return r * v.rs + c1 * v.s1 + c2 * v.s2 + c3 * v.s3;
}

struct FwdParams {
  const void* q;   // [batch][n_q][D]
  const void* k;   // [batch][n_kv][D]
  const void* v;   // [batch][n_kv][dv1]   -> o columns [0, dv1)
  const void* v2;  // [batch][n_kv][DV-dv1] -> o columns [dv1, DV)
  void* o;         // [batch][n_q][DV]
  float* lse;      // [batch][n_q]  log2-domain LSE of x = s * sm_scale * log2(e)
  float* ent;      // [batch][n_q]  natural-log row entropy
  int64_t q_bs, k_bs, v_bs, v2_bs, o_bs;  // batch strides in elements (dense layout)
  View qv, kv, vv, v2v, ov;                // the same tensors as strided views (tcgen05 kernels)
  int n1, n2;                              // batch split of the views
  int n_q, n_kv, dv1, n_qtiles;
  float scale_log2;  // sm_scale * log2(e)
  void* work;        // optional workspace (key-range split of the d = dv = 128 kernel), may be NULL
  int64_t work_bytes;
  long long wait_limit;  // tcgen05 kernels' pipeline wait limit in cycles (0: the default ~2 s)
  int hold_loads;        // test of the timeout path: the tcgen05 producers issue no load
  bool e4m3;             // q, k, v, v2 hold e4m3 bytes (dense, D = 128, V aliasing K); o stays 16-bit
};

struct BwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* v2;
  const void* dout;   // [batch][n_q][DV]
  const float* lse;   // [batch][n_q]
  const float* cc;    // [batch][n_q]  delta_i + dE_i * (E_i - LSE_i)
  const float* gg;    // [batch][n_q]  dE_i * ln(2)
  const float* fold;  // tcgen05 path: planes nl, nc, ng, each [batch][n_pad] (see fea_bwd_pre)
  int64_t n_pad;      // rows per sequence of the planes: n_q rounded up to 128
  float* dq_part;     // tcgen05 path, split key range: partial dQ tiles [split][batch][n_pad][D]
  void* ds;           // tcgen05 path, dQ from dS: dS^T [batch][round_up(n_kv, 128)][round_up(n_q, 64)] 16-bit
  float* dq;          // fp32 accumulator [batch][n_q][D] (batch stride dq_bs)
  void* dk;           // [batch][n_kv][D]      element type or fp32 (acc_kv)
  void* dv;           // [batch][n_kv][dv1]    unused when v aliases k
  void* dv2;          // [batch][n_kv][DV-dv1]
  int64_t q_bs, k_bs, v_bs, v2_bs, do_bs, dq_bs, dk_bs, dv_bs, dv2_bs;  // dense layout
  View qv, kv, vv, v2v, dov, dqv, dkv, dvv, dv2v;  // strided views (tcgen05 kernels)
  View finqv, finkv, finvv, finv2v;
  int n1, n2;                                      // batch split of the views
  int d;                                           // head dim of q / k (64 or 128 on the tcgen05 path)
  int n_q, n_kv, dv1, n_ktiles;
  int acc_kv;         // 1: dk/dv/dv2 are fp32 buffers that are added into
  int acc_q;          // 1: dq is an fp32 buffer that is added into (else element dtype)
  float scale_log2;   // sm_scale * log2(e)
  float sm_scale;
  bool deterministic;  // bitwise reproducible results (no concurrent fp32 reductions into dq)
  // grad_mode 3: fp32 accumulators whose values are added before the 16-bit gradients are written
  const float* fin_q;
  const float* fin_k;
  const float* fin_v;
  const float* fin_v2;
  int64_t fin_q_bs, fin_k_bs, fin_v_bs, fin_v2_bs;
};

}  // namespace vmb
