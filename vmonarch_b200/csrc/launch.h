// Internal (C++) launch interface between the C-ABI layer (capi.cu) and the kernel files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "fea_params.h"

struct vmb_fea_bwd_args;

namespace vmb {

struct LstepParams {
  const void* q;      // [bh][N][D]
  const void* out;    // [bh][N][dw]   R-step output; cols [0,D) -> kr, [D,dw) -> y (last step)
  const float* ent;   // [bh][N]       R-step row entropy
  void* u;            // fwd, non-last: [bh][N][D]
  void* z;            // fwd, last:     [bh][N][dw-D]
  const float* du;    // bwd, non-last: [bh][N][D] fp32 gradient of u
  const void* dz;     // bwd, last:     [bh][N][dw-D]
  float* dq;          // bwd: [bh][N][D] fp32, added into (or written when dq_store)
  void* dout;         // bwd: [bh][N][dw] gradient of `out`
  int64_t bh, m, b;
  int d, dw;
  int64_t skip_rows;  // tokens [0, skip_rows) of every head are not produced / carry no gradient
  float scale, min_col_mass;
  int dq_store;
  float* delta_out;   // bwd, optional: [bh][N] fp32 sum_c out[c] dout[c] per token
  // The tensors above as [bh][N][cols] views (fea_params.h) with head split (n1, n2 = 1): token t
  // of head hb at t * rs + (hb % n1) * s1 + (hb / n1) * s3. ent and delta_out stay dense [bh][N].
  View qv, outv, uv, zv, duv, dzv, dqv, doutv;
  int n1;
};

cudaError_t fea_fwd_mma(const FwdParams& p, int64_t batch, int d, int dv, bool ent, bool bf16, cudaStream_t st);
bool fea_fwd_sm100_supported(int d, int dv, int dv1, bool vk);
bool fea_fwd_sm100_e4m3_supported(int d, int dv, int dv1, bool vk);
cudaError_t fea_fwd_sm100(const FwdParams& p, int64_t batch, int d, int dv, bool ent, bool bf16, bool vk,
                          cudaStream_t st);
cudaError_t fea_fwd_sm100_status(cudaStream_t st, int* out);
bool fea_bwd_sm100_supported(int d, int dv, int dv1, bool vk);
cudaError_t fea_bwd_sm100(const BwdParams& p, int64_t batch, int dv, bool vk, bool bf16, cudaStream_t st);
// Number of CTAs sharing one query tile's key range in the tcgen05 dQ kernel (1 = no split; only
// the accumulate mode splits). The partial tiles need split * batch * round_up(n_q, 128) * 128
// fp32 of workspace when the result is above 1.
int fea_bwd_dq_split(int64_t batch, int n_q, int n_kv, bool acc);
// True when the tcgen05 backward forms dQ inside the dK kernel (fp32 reductions, no dq kernel).
bool fea_bwd_fuses_dq(int n_kv, int d, int dv, bool vk, int acc_q, bool deterministic);
// True when the tcgen05 backward takes dQ from dS: the dK/dV kernel stores dS^T (16-bit) and a
// GEMM forms dQ = dS K, instead of a dq kernel recomputing S and dP.
bool fea_bwd_ds_gemm(int64_t batch, int n_q, int n_kv, int dv, bool vk, int acc_q);
// Bytes of that dS^T buffer.
int64_t fea_bwd_ds_bytes(int64_t batch, int n_q, int n_kv);
// Smallest workspace vmb_fea_bwd accepts for these arguments (vmb_fea_bwd_workspace_bytes
// reports the preferred size, which may add optional buffers such as dS^T).
int64_t fea_bwd_min_workspace_bytes(const vmb_fea_bwd_args* a);
// Workspace bytes that let the tcgen05 forward split long key ranges (0: it would not split).
int64_t fea_fwd_sm100_workspace_bytes(int64_t batch, int n_q, int n_kv, int d, int dv, int dv1, bool vk);
// Key-range split the tcgen05 forward will use with this workspace (1 = none).
int fea_fwd_sm100_split(int64_t batch, int n_q, int n_kv, int d, int dv, const void* work, int64_t work_bytes);
cudaError_t fea_bwd_sm100_status(cudaStream_t st, int* out);
cudaError_t fea_bwd_mma(const BwdParams& p, int64_t batch, int d, int dv, bool vk, bool bf16, cudaStream_t st);
cudaError_t fea_bwd_pre(const void* o, View ov, const void* dout, View dov, int n1, int n2, const float* lse,
                        const float* ent, const float* dent, float* cc, float* gg, int64_t batch, int n_q, int dv,
                        float* fold, int64_t n_pad, float sm_scale, const float* delta, bool bf16, cudaStream_t st);
// dst = e4m3(scale * src) over [batch][rows][cols] views (16-bit src); cols % 16 == 0.
cudaError_t quant_e4m3(const void* src, const View& sv, void* dst, const View& dvw, int n1, int n2, int64_t batch,
                       int64_t rows, int64_t cols, bool bf16, float scale, cudaStream_t st);
// dst = (16-bit) src over [batch][rows][cols] views with batch split (n1, n2); cols % 4 == 0.
cudaError_t cast_f32_view(const float* src, const View& sv, void* dst, const View& dvw, int n1, int n2, int64_t batch,
                          int64_t rows, int64_t cols, bool bf16, cudaStream_t st);
cudaError_t cast_f32(const float* src, int64_t src_bs, void* dst, int64_t dst_bs, int64_t batch, int64_t n,
                     bool bf16, cudaStream_t st);
bool lstep_mma_supported(const LstepParams& p, bool last);
cudaError_t lstep_mma_launch(const LstepParams& p, bool last, bool bwd, bool bf16, cudaStream_t st);
cudaError_t lstep_launch(const LstepParams& p, bool last, bool bwd, bool bf16, cudaStream_t st);
// tcgen05 / TMA L step (D = 128, stacked columns); forward only, and the last step only without
// skipped tokens.
bool lstep_tc_supported(const LstepParams& p, bool last, bool bwd);
cudaError_t lstep_tc_launch(const LstepParams& p, bool last, bool bwd, bool bf16, cudaStream_t st);
cudaError_t lstep_tc_status(cudaStream_t st, int* out);
size_t lstep_smem_bytes(int m, int d, int dw, bool last, bool bwd);

// Records `code` and a printf-style message as the calling thread's last error; returns `code`.
int set_error(int code, const char* fmt, ...);

}  // namespace vmb
