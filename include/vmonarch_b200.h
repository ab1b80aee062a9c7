/*
 * vmonarch_b200 — C ABI of the B200 (sm_100a) VMonarch attention hot path.
 *
 * The reference (EricLina/VMonarch) is a Python package whose hot path crosses from the host to
 * the GPU only at its Triton kernel launches and at a handful of torch ops. Each entry point
 * below replaces one of those crossings; the Python package `vmonarch_b200` binds them with
 * ctypes and mirrors the reference's Python API on top.
 *
 * Conventions
 *  - Every pointer is a device pointer; tensors are dense row-major with the batch stride given
 *    in ELEMENTS. Rows are contiguous (row stride = number of columns). Base pointers must be
 *    16-byte aligned and batch strides multiples of 8 elements.
 *  - dtype selects the 16-bit element type (VMB_DTYPE_BF16 or VMB_DTYPE_F16); all arithmetic
 *    accumulates in fp32. Statistics (lse, ent, dent) are fp32.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). Calls only enqueue work; they
 *    never synchronize and never allocate.
 *  - Return value: VMB_OK or an error code; vmb_last_error() describes the last failure of the
 *    calling thread.
 */
#ifndef VMONARCH_B200_H
#define VMONARCH_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VMB_ABI_VERSION 7

#define VMB_DTYPE_BF16 0
#define VMB_DTYPE_F16 1

#define VMB_OK 0
#define VMB_EINVAL 1   /* malformed argument: null pointer, bad size, misalignment */
#define VMB_ENOTSUP 2  /* head dimensions without a kernel, or a strided layout a kernel cannot take */
#define VMB_ECUDA 3    /* CUDA runtime error while launching */

/* ABI version (VMB_ABI_VERSION of the library that was loaded). */
int vmb_abi_version(void);

/* Human-readable description of the last error returned on the calling thread. */
const char* vmb_last_error(void);

/* Pipeline-timeout status of the tcgen05 kernels on the current device: synchronises `stream`,
 * stores into *out the OR of the error codes recorded since the last call (0 = none) and clears
 * them. A kernel whose pipeline wait exceeds its time limit (~2 s) records a code, drains its
 * in-flight copies and MMAs, frees its tensor memory and exits instead of hanging; its outputs
 * are then invalid. No counterpart in the reference (Triton kernels have no such check). */
int vmb_device_status(void* stream, int32_t* out);

/* Test hook of the pipeline-timeout path; no counterpart in the reference. wait_cycles > 0
 * shortens the tcgen05 forward kernels' pipeline wait limit to that many SM cycles; hold_loads != 0
 * (only with 0 < wait_cycles <= 1e8) makes their load producers issue no copy, so the consumers'
 * first waits run out: the kernels record their codes (vmb_device_status), drain, free their
 * tensor memory and exit with their outputs invalid. (0, 0) restores normal operation. The
 * setting is process-wide and read at each vmb_fea_fwd call; it exists for tests only. */
int vmb_test_pipeline_timeout(int64_t wait_cycles, int32_t hold_loads);

/* Number of kernels this library has launched in the process so far (all threads, all devices).
 * Diagnostic with no reference counterpart: the benchmark reports it as its launch count. */
uint64_t vmb_kernel_launches(void);

/*
 * Strided layouts (ABI version 6). By default every tensor is dense [batch][rows][cols] with the
 * batch stride given in its *_bs field. A call may instead pass a layout that gives each tensor a
 * view: element (s, r, c) of batch entry s, row r, column c lies at
 *     c + r * row + (s % n1) * s1 + (s / n1 % n2) * s2 + (s / (n1 * n2)) * s3
 * elements from the tensor's base, with (n1, n2) shared by the call's tensors (batch must be a
 * multiple of n1 * n2). This is how token-major callers are served without transposes: the
 * reference's Video-DiT caller holds tokens as (B, N, H, D) (README.md:74-76), whose head h of
 * batch b is rows of stride H * D starting at (b * N * H + h) * D, so FlashEntropyAttention over
 * its B * H sequences is the view {H * D, D, 0, N * H * D} with (n1, n2) = (H, 1), and the VMonarch
 * R step over its B * H * m grid rows of b tokens is {H * D, b * H * D, D, N * H * D} with
 * (n1, n2) = (m, H). Strides are in elements and multiples of 8 (4 for fp32 tensors); row >= cols.
 * Statistics (lse, ent, dent, delta) stay dense [batch][rows] in every layout. Only the D = 128
 * kernels take non-uniform views (a view is uniform when row == cols and entry s starts at s * X);
 * other head dimensions return VMB_ENOTSUP for them.
 */
typedef struct vmb_view {
  int64_t row, s1, s2, s3;
} vmb_view;

typedef struct vmb_fea_layout {
  int64_t n1, n2;
  vmb_view q, k, v, v2, o, dout, grad_q, grad_k, grad_v, grad_v2, fin_q, fin_k, fin_v, fin_v2;
} vmb_fea_layout;

/*
 * FlashEntropyAttention forward over `batch` independent sequences:
 *   o = softmax(sm_scale q k^T) [v | v2],  ent_i = -sum_j P_ij log P_ij,
 *   lse_i = log2 sum_j 2^(x_ij) with x = sm_scale q k^T log2(e)   (kept for the backward).
 * Replaces the `_attn_fwd` launch and the pad-row zeroing of _FlashEntropyAttention.forward
 * (video_monarch_attention/kernel.py:346-353) and the F.pad / slice of flash_entropy_attention
 * (kernel.py:399-402): sequences of any length are handled without padding. The optional second
 * value tensor replaces the torch.cat([kg, vg], -1) of the last R step (vmonarch.py:50).
 * Shapes: d, dv in {16, 32, 64, 128, 256} with dv a multiple of d (the reference requires
 * Dv % D == 0 for its backward, kernel.py:260). o may be a strided view (o_bs) into a larger
 * tensor, which is how the exact first-frame recompute writes straight into z.
 * workspace / workspace_bytes are optional (NULL / 0 is valid). With a workspace of
 * vmb_fea_fwd_workspace_bytes() bytes the d = dv = 128 kernel may split each sequence's key range
 * over several CTAs when the query tiles alone would fill the GPU poorly (few, long sequences, e.g.
 * the recompute's r queries over all N keys on a few heads); the partial results are merged
 * exactly by a second kernel. Without one, or when no split pays off, nothing changes. The
 * workspace contents need not be initialised; it is 256-byte aligned when obtained from a
 * caching allocator (16 bytes is required).
 */
typedef struct vmb_fea_fwd_args {
  const void* q;  int64_t q_bs;   /* [batch][n_q][d]                               */
  const void* k;  int64_t k_bs;   /* [batch][n_kv][d]                              */
  const void* v;  int64_t v_bs;   /* [batch][n_kv][dv1]  -> o columns [0, dv1)     */
  const void* v2; int64_t v2_bs;  /* [batch][n_kv][dv-dv1] -> o columns [dv1, dv); NULL if dv1 == dv */
  void* o;        int64_t o_bs;   /* [batch][n_q][dv]                              */
  float* lse;                     /* [batch][n_q] or NULL                          */
  float* ent;                     /* [batch][n_q] or NULL (entropy not computed)   */
  int64_t batch, n_q, n_kv;
  int32_t d, dv, dv1, dtype;
  float sm_scale;
  void* workspace;  int64_t workspace_bytes;  /* optional, see above (ABI version 2) */
  const vmb_fea_layout* layout;  /* optional strided layout of q, k, v, v2, o (ABI version 6);
                                    NULL: dense with the *_bs batch strides */
  int32_t qkv_e4m3;  /* ABI version 7. Nonzero: q, k, v and v2 hold e4m3 (fp8, one byte per
                        element; see vmb_quant_e4m3) and both products run on the fp8 tensor cores,
                        with P rounded to e4m3 as well; o, lse and ent are as usual (dtype gives o's
                        type). Only the VMonarch R-step forms: d = 128, v aliasing k (v == k, dv1 = d),
                        dv = 128 or dv = 256 with a 128-wide v2. Batch and layout strides are then
                        multiples of 16 elements (bytes). No reference counterpart: an opt-in
                        B200 extension of the R step (the reference computes it in bf16). */
} vmb_fea_fwd_args;

/* Workspace that lets vmb_fea_fwd split long key ranges (0 when it would not split). No
 * counterpart in the reference, whose forward launch allocates through torch. */
int64_t vmb_fea_fwd_workspace_bytes(const vmb_fea_fwd_args* a);
int vmb_fea_fwd(const vmb_fea_fwd_args* a, void* stream);

/*
 * FlashEntropyAttention backward. Replaces `_attn_bwd_preprocess` + `_attn_bwd`
 * (video_monarch_attention/kernel.py:360-381) including the entropy-gradient term
 * dS = P (dP - delta) + dE P (-E - log P) (kernel.py:165-167).
 * grad_mode 0: grad_q/grad_k/grad_v/grad_v2 are written in the element dtype (standalone op).
 * grad_mode 1: grad_* are fp32 buffers that the gradients are ADDED into (VMonarch chains
 *              several R steps and the recompute into one set of accumulators).
 * grad_mode 2: grad_* are fp32 buffers that are OVERWRITTEN (the first contribution to a set of
 *              accumulators, so they need no zero-fill).
 * grad_mode 3: the last contribution: grad_* are written in the element dtype as the sum of the
 *              fp32 accumulator fin_* (same shape, batch stride fin_*_bs) and this call's gradient,
 *              which saves a separate fp32 -> 16-bit pass. fin_q/fin_k (and fin_v / fin_v2 where
 *              grad_v / grad_v2 are given) are required; their contents are unspecified afterwards
 *              (shapes without a tcgen05 kernel add into them before converting).
 * v_is_k = 1: the value columns [0, dv1) are the key tensor itself (dv1 == d); their gradient is
 *              added into grad_k and grad_v must be NULL. This is the VMonarch R step
 *              (vmonarch.py:50).
 * dent may be NULL (dE = 0, e.g. the detached entropy of VMonarch, vmonarch.py:26); ent is then
 * not read either.
 * The caller provides a device workspace of vmb_fea_bwd_workspace_bytes() bytes (256-byte
 * aligned); its contents need not be initialised.
 */
typedef struct vmb_fea_bwd_args {
  const void* q;    int64_t q_bs;
  const void* k;    int64_t k_bs;
  const void* v;    int64_t v_bs;
  const void* v2;   int64_t v2_bs;
  const void* o;    int64_t o_bs;    /* forward output                         */
  const void* dout; int64_t do_bs;   /* gradient of o, [batch][n_q][dv]        */
  const float* lse;                  /* forward lse, [batch][n_q]              */
  const float* ent;                  /* forward entropy (read only with dent)  */
  const float* dent;                 /* gradient of ent or NULL                */
  void* grad_q;  int64_t grad_q_bs;   /* [batch][n_q][d]                        */
  void* grad_k;  int64_t grad_k_bs;   /* [batch][n_kv][d]                       */
  void* grad_v;  int64_t grad_v_bs;   /* [batch][n_kv][dv1]  (NULL if v_is_k)   */
  void* grad_v2; int64_t grad_v2_bs;  /* [batch][n_kv][dv-dv1] (NULL if no v2)  */
  void* workspace; int64_t workspace_bytes;
  int64_t batch, n_q, n_kv;
  int32_t d, dv, dv1, dtype;
  int32_t grad_mode, v_is_k;
  float sm_scale;
  const float* delta;  /* optional [batch][n_q] fp32: sum_c o[c] dout[c] per query row, precomputed
                          by the caller (vmb_lstep_bwd's delta_out); NULL: computed here (ABI 2) */
  int32_t deterministic; /* nonzero: bitwise reproducible gradients. Zero lets grad_mode 1 / 2 with
                            v_is_k, dv == d == 128 and n_kv <= 4096 form dQ with concurrent fp32
                            reductions (one kernel fewer; summation order varies) (ABI 3) */
  const float* fin_q;  int64_t fin_q_bs;   /* grad_mode 3 accumulators (ABI 4) */
  const float* fin_k;  int64_t fin_k_bs;
  const float* fin_v;  int64_t fin_v_bs;
  const float* fin_v2; int64_t fin_v2_bs;
  const vmb_fea_layout* layout;  /* optional strided layout of every tensor but the statistics
                                    (ABI version 6); NULL: dense with the *_bs batch strides */
} vmb_fea_bwd_args;

int64_t vmb_fea_bwd_workspace_bytes(const vmb_fea_bwd_args* a);
/* The smallest workspace vmb_fea_bwd accepts (ABI 5). vmb_fea_bwd_workspace_bytes reports the
 * preferred size, which for the last VMonarch R step (v_is_k, dv = 2 d, n_kv <= 4096) adds a dS^T
 * buffer (batch x round_up(n_kv, 128) x round_up(n_q, 64) 16-bit values) so that dQ comes from
 * dS by a GEMM instead of a kernel recomputing S and dP; a workspace between the two sizes runs
 * the latter. -1 for malformed sizes. */
int64_t vmb_fea_bwd_min_workspace_bytes(const vmb_fea_bwd_args* a);
int vmb_fea_bwd(const vmb_fea_bwd_args* a, void* stream);

/*
 * vmb_fea_bwd for callers that cannot allocate device memory. No counterpart in the reference.
 * Same arguments and results as vmb_fea_bwd, but `workspace` / `workspace_bytes` are ignored: the
 * scratch comes from a 32 MiB array compiled into the library (a static __device__ buffer that
 * every GPU holding the library's module keeps until the process exits). Meant for hosts that
 * cannot hand over a workspace: plugins whose enqueue hook must not allocate because the host
 * framework owns all device memory, foreign-language bindings that can only pass the user's
 * tensors, and pipelines that cannot afford cudaMalloc inside a step.
 *  - Calls whose minimal workspace (vmb_fea_bwd_min_workspace_bytes) exceeds 32 MiB return
 *    VMB_EINVAL. A call whose preferred workspace (vmb_fea_bwd_workspace_bytes, which adds the
 *    dS^T buffer of the dQ-from-dS route) also fits takes that route; otherwise it runs the dQ
 *    kernel that recomputes S and dP, with the same results.
 *  - The first call on a device looks the buffer's address up with that device current; make
 *    that first call before any stream capture begins. The address is kept for the process: after
 *    cudaDeviceReset (which unloads the library's module) or from a context other than the
 *    device's primary context this entry point must not be used.
 *  - All calls share the buffer, which keeps the previous call's contents (the backward clears
 *    what must start at zero). Calls that overlap on the GPU race on it: serialise them.
 *  - Calls no cudaMalloc, cudaFree or other allocating routine.
 */
int vmb_fea_bwd_noalloc(const vmb_fea_bwd_args* a, void* stream);

/*
 * Monarch L step (the b dense m x m blocks), forward and backward, for `bh` heads of
 * N = m * b tokens. Replaces the einsum / softmax / col_mass / scaling ops of
 * video_monarch_attention/vmonarch.py:51-63 (forward) and their autograd backward.
 *   q    [bh][N][d]   original queries        out [bh][N][dw] R-step output
 *   ent  [bh][N]      R-step row entropy (the reference's -neg_ent)
 * forward, last == 0: u  [bh][N][d]    next R-step queries (already scaled)
 * forward, last == 1: z  [bh][N][dw-d] Monarch output; tokens < skip_rows are left unwritten
 * backward, last == 0: du [bh][N][d] fp32 gradient of u
 * backward, last == 1: dz [bh][N][dw-d] gradient of z; tokens < skip_rows carry none
 * backward outputs: dq [bh][N][d] fp32 (ADDED into, or OVERWRITTEN when dq_store != 0),
 *   dout [bh][N][dw] gradient of out.
 * m <= 128 (m <= 64 unless d in {64, 128} with dw = d, or 2d when last), d in {16, 32, 64, 128},
 * dw - d in {16, ..., 256} and a multiple of d when last.
 */
/* Strided layout of an L-step call (ABI version 6): each tensor is a [bh][N][cols] view (rows =
 * tokens) whose head hb starts at (hb % n1) * s1 + (hb / n1) * s3 (s2 unused); a token-major
 * (B, N, H, D) tensor is {H * D, D, 0, N * H * D} with n1 = H. ent and delta_out stay dense. The
 * kernels for m <= 128 with d in {64, 128} take any view; other shapes need dense tensors. */
typedef struct vmb_lstep_layout {
  int64_t n1;
  vmb_view q, out, u, z, du, dz, dq, dout;
} vmb_lstep_layout;

typedef struct vmb_lstep_args {
  const void* q;
  const void* out;
  const float* ent;
  void* u;
  void* z;
  const float* du;
  const void* dz;
  float* dq;
  void* dout;
  int64_t bh, m, b;
  int32_t d, dw, dtype, last;
  int64_t skip_rows;
  float scale, min_col_mass;
  int32_t dq_store;  /* backward: 1 = write dq instead of adding into it (ABI version 2) */
  float* delta_out;  /* backward, optional [bh][N] fp32: sum_c out[c] dout[c] per token, the
                        preprocessing of the R step's attention backward (its `delta`) */
  const vmb_lstep_layout* layout;  /* optional (ABI version 6), see above; NULL: dense */
} vmb_lstep_args;


int vmb_lstep_fwd(const vmb_lstep_args* a, void* stream);
int vmb_lstep_bwd(const vmb_lstep_args* a, void* stream);

/* dst[b][i] = (dtype) src[b][i], i < n (n and both batch strides multiples of 4).
 * Converts the fp32 gradient accumulators of grad_mode 1 to the element dtype. */
int vmb_cast_f32(const float* src, int64_t src_bs, void* dst, int64_t dst_bs, int64_t batch, int64_t n,
                 int32_t dtype, void* stream);

/* dst(s, r, c) = e4m3(scale * src(s, r, c)) over [batch][rows][cols] views with batch split (n1, n2)
 * (ABI version 7): the operands of an e4m3 forward (vmb_fea_fwd_args.qkv_e4m3) from 16-bit tensors
 * of element type dtype. Rounded to nearest even, saturating at +-448 (the format's largest finite
 * value); NaN stays NaN. cols a multiple of 16; src rows 16-byte aligned (view strides multiples of
 * 8 elements), dst rows 16-byte aligned (multiples of 16). */
int vmb_quant_e4m3(const void* src, const vmb_view* src_view, void* dst, const vmb_view* dst_view, int64_t n1,
                   int64_t n2, int64_t batch, int64_t rows, int64_t cols, int32_t dtype, float scale, void* stream);

/* dst(s, r, c) = (dtype) src(s, r, c) over [batch][rows][cols] views with batch split (n1, n2)
 * (ABI version 6): the fp32 accumulator of a strided (e.g. token-major) gradient converted into
 * the caller's tensor. cols a multiple of 4; src rows 16-byte aligned, dst rows 8-byte aligned. */
int vmb_cast_f32_view(const float* src, const vmb_view* src_view, void* dst, const vmb_view* dst_view, int64_t n1,
                      int64_t n2, int64_t batch, int64_t rows, int64_t cols, int32_t dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VMONARCH_B200_H */
