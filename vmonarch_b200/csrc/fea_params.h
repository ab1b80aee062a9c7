// Kernel-side parameter blocks for the FlashEntropyAttention kernels. These are filled by the
// C-ABI layer (capi.cu) from the public argument structs declared in include/vmonarch_b200.h.
#pragma once
#include <stdint.h>

namespace vmb {

struct FwdParams {
  const void* q;   // [batch][n_q][D]
  const void* k;   // [batch][n_kv][D]
  const void* v;   // [batch][n_kv][dv1]   -> o columns [0, dv1)
  const void* v2;  // [batch][n_kv][DV-dv1] -> o columns [dv1, DV)
  void* o;         // [batch][n_q][DV]
  float* lse;      // [batch][n_q]  log2-domain LSE of x = s * sm_scale * log2(e)
  float* ent;      // [batch][n_q]  natural-log row entropy
  int64_t q_bs, k_bs, v_bs, v2_bs, o_bs;  // batch strides in elements
  int n_q, n_kv, dv1, n_qtiles;
  float scale_log2;  // sm_scale * log2(e)
  void* work;        // optional workspace (key-range split of the d = dv = 128 kernel), may be NULL
  int64_t work_bytes;
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
  int64_t q_bs, k_bs, v_bs, v2_bs, do_bs, dq_bs, dk_bs, dv_bs, dv2_bs;
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
