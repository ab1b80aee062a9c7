// extern "C" entry points declared in include/vmonarch_b200.h: argument validation, workspace
// carving and dispatch to the kernel files.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/vmonarch_b200.h"
#include "launch.h"

static constexpr float kLog2eHost = 1.4426950408889634f;

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
// vmb_test_pipeline_timeout: shortened wait limit and load hold of the tcgen05 forward kernels
std::atomic<int64_t> g_test_wait_cycles{0};
std::atomic<int> g_test_hold_loads{0};

void count(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return VMB_OK;
  if (e == cudaErrorNotSupported) return fail(VMB_ENOTSUP, "%s: unsupported head dimensions", what);
  return fail(VMB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The head dims the reference accepts (video_monarch_attention/kernel.py:260, 324).
bool pow2_dim(int x) { return x == 16 || x == 32 || x == 64 || x == 128 || x == 256; }
bool fea_dims_ok(int d, int dv) { return pow2_dim(d) && pow2_dim(dv) && dv % d == 0; }

int check_common(const char* what, int64_t batch, int64_t n_q, int64_t n_kv, int d, int dv, int dv1, int dtype,
                 const void* v2) {
  if (dtype != VMB_DTYPE_BF16 && dtype != VMB_DTYPE_F16) return fail(VMB_EINVAL, "%s: unknown dtype %d", what, dtype);
  if (batch < 0 || n_q < 0 || n_kv < 1) return fail(VMB_EINVAL, "%s: bad sizes batch=%lld n_q=%lld n_kv=%lld", what,
                                                   (long long)batch, (long long)n_q, (long long)n_kv);
  if (n_q > 0x7fffffff || n_kv > 0x7fffffff) return fail(VMB_EINVAL, "%s: sequence longer than 2^31-1", what);
  if (!fea_dims_ok(d, dv)) return fail(VMB_ENOTSUP, "%s: no kernel for head dims d=%d dv=%d", what, d, dv);
  if (dv1 <= 0 || dv1 > dv || dv1 % 8) return fail(VMB_EINVAL, "%s: dv1=%d must be a multiple of 8 in (0, dv]", what, dv1);
  if ((dv1 < dv) != (v2 != nullptr)) return fail(VMB_EINVAL, "%s: v2 must be given exactly when dv1 < dv", what);
  return VMB_OK;
}

int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

vmb::View to_view(const vmb_view& v) { return vmb::View{v.row, v.s1, v.s2, v.s3}; }

// A view (or its absence: dense with batch stride bs) of a tensor with `cols` columns.
vmb::View view_or_dense(const vmb_view* v, int64_t cols, int64_t bs) {
  return v ? to_view(*v) : vmb::dense_view(cols, bs, 1, 1);
}

// Strides multiples of `align` elements, rows at least `cols` apart.
bool view_ok(const vmb::View& v, int64_t cols, int align) {
  return v.rs >= cols && v.rs % align == 0 && v.s1 % align == 0 && v.s2 % align == 0 && v.s3 % align == 0 &&
         v.s1 >= 0 && v.s2 >= 0 && v.s3 >= 0;
}

// True when entry s of the view starts at s * X with contiguous rows (the dense layout the
// non-tcgen05 kernels take); X is returned in *bs.
bool uniform(const vmb::View& v, int64_t cols, int64_t n1, int64_t n2, int64_t batch, int64_t* bs) {
  if (v.rs != cols) return false;
  const int64_t n3 = batch / (n1 * n2);
  const int64_t x = n1 > 1 ? v.s1 : (n2 > 1 ? v.s2 : v.s3);
  if ((n1 > 1 && v.s1 != x) || (n2 > 1 && v.s2 != n1 * x) || (n3 > 1 && v.s3 != n1 * n2 * x)) return false;
  *bs = x;
  return true;
}

int check_split(const char* what, int64_t n1, int64_t n2, int64_t batch) {
  if (n1 < 1 || n2 < 1 || n1 > 0x7fffffff || n2 > 0x7fffffff || (batch > 0 && batch % (n1 * n2)))
    return fail(VMB_EINVAL, "%s: layout split n1=%lld n2=%lld does not divide batch=%lld", what, (long long)n1,
                (long long)n2, (long long)batch);
  return VMB_OK;
}

}  // namespace

namespace vmb {
int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}
}  // namespace vmb

extern "C" {

int vmb_abi_version(void) { return VMB_ABI_VERSION; }

const char* vmb_last_error(void) { return g_last_error.c_str(); }

uint64_t vmb_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int vmb_test_pipeline_timeout(int64_t wait_cycles, int32_t hold_loads) {
  if (wait_cycles < 0 || (hold_loads && (wait_cycles == 0 || wait_cycles > 100000000)))
    return fail(VMB_EINVAL, "vmb_test_pipeline_timeout: hold_loads needs 0 < wait_cycles <= 1e8");
  g_test_wait_cycles.store(wait_cycles, std::memory_order_relaxed);
  g_test_hold_loads.store(hold_loads ? 1 : 0, std::memory_order_relaxed);
  return VMB_OK;
}

int vmb_device_status(void* stream, int32_t* out) {
  if (!out) return fail(VMB_EINVAL, "vmb_device_status: null output");
  int v = 0, w = 0, x = 0;
  cudaError_t e = vmb::fea_fwd_sm100_status(static_cast<cudaStream_t>(stream), &v);
  if (e == cudaSuccess) e = vmb::fea_bwd_sm100_status(static_cast<cudaStream_t>(stream), &w);
  if (e == cudaSuccess) e = vmb::lstep_tc_status(static_cast<cudaStream_t>(stream), &x);
  if (e != cudaSuccess) return cuda_status(e, "vmb_device_status");
  *out = v | (w << 8) | (x << 16);
  return VMB_OK;
}

static bool same_view(const vmb_view& a, const vmb_view& b) {
  return a.row == b.row && a.s1 == b.s1 && a.s2 == b.s2 && a.s3 == b.s3;
}

static bool fwd_v_is_k(const vmb_fea_fwd_args* a) {
  if (a->v != a->k || a->dv1 != a->d) return false;
  return a->layout ? same_view(a->layout->v, a->layout->k) : a->v_bs == a->k_bs;
}

int64_t vmb_fea_fwd_workspace_bytes(const vmb_fea_fwd_args* a) {
  if (!a || a->batch < 0 || a->n_q < 0 || a->n_kv < 1) return -1;
  if (a->batch == 0 || a->n_q == 0 || a->n_q > 0x7fffffff || a->n_kv > 0x7fffffff || a->qkv_e4m3) return 0;
  return vmb::fea_fwd_sm100_workspace_bytes(a->batch, (int)a->n_q, (int)a->n_kv, a->d, a->dv, a->dv1,
                                            fwd_v_is_k(a));
}

int vmb_fea_fwd(const vmb_fea_fwd_args* a, void* stream) {
  if (!a) return fail(VMB_EINVAL, "vmb_fea_fwd: null args");
  int rc = check_common("vmb_fea_fwd", a->batch, a->n_q, a->n_kv, a->d, a->dv, a->dv1, a->dtype, a->v2);
  if (rc) return rc;
  if (a->batch == 0 || a->n_q == 0) return VMB_OK;
  if (!a->q || !a->k || !a->v || !a->o) return fail(VMB_EINVAL, "vmb_fea_fwd: null tensor pointer");
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) || (a->v2 && !aligned16(a->v2)))
    return fail(VMB_EINVAL, "vmb_fea_fwd: tensors must be 16-byte aligned");
  if ((a->q_bs | a->k_bs | a->v_bs | a->o_bs | a->v2_bs) & 7)
    return fail(VMB_EINVAL, "vmb_fea_fwd: batch strides must be multiples of 8 elements");
  const bool e4m3 = a->qkv_e4m3 != 0;
  if (e4m3) {
    // fp8 operands: the VMonarch R-step forms only (one-byte elements, 16-byte aligned rows)
    if (!fwd_v_is_k(a) || !vmb::fea_fwd_sm100_e4m3_supported(a->d, a->dv, a->dv1, true))
      return fail(VMB_ENOTSUP,
                  "vmb_fea_fwd: e4m3 operands need d = 128 with v aliasing k and dv = 128, or dv = 256 with a "
                  "128-wide v2 (got d=%d dv=%d dv1=%d)", a->d, a->dv, a->dv1);
    if ((a->q_bs | a->k_bs | a->v2_bs) & 15)
      return fail(VMB_EINVAL, "vmb_fea_fwd: e4m3 batch strides must be multiples of 16 elements");
  }
  if (a->workspace && (!aligned16(a->workspace) || a->workspace_bytes < 0))
    return fail(VMB_EINVAL, "vmb_fea_fwd: workspace must be 16-byte aligned");
  vmb::FwdParams p{};
  p.q = a->q; p.k = a->k; p.v = a->v; p.v2 = a->v2; p.o = a->o; p.lse = a->lse; p.ent = a->ent;
  p.q_bs = a->q_bs; p.k_bs = a->k_bs; p.v_bs = a->v_bs; p.v2_bs = a->v2_bs; p.o_bs = a->o_bs;
  const vmb_fea_layout* L = a->layout;
  p.n1 = L ? (int)L->n1 : 1;
  p.n2 = L ? (int)L->n2 : 1;
  if (L && (rc = check_split("vmb_fea_fwd", L->n1, L->n2, a->batch))) return rc;
  p.qv = view_or_dense(L ? &L->q : nullptr, a->d, a->q_bs);
  p.kv = view_or_dense(L ? &L->k : nullptr, a->d, a->k_bs);
  p.vv = view_or_dense(L ? &L->v : nullptr, a->dv1, a->v_bs);
  p.v2v = view_or_dense(L ? &L->v2 : nullptr, a->dv - a->dv1, a->v2_bs);
  p.ov = view_or_dense(L ? &L->o : nullptr, a->dv, a->o_bs);
  if (L && (!view_ok(p.qv, a->d, 8) || !view_ok(p.kv, a->d, 8) || !view_ok(p.vv, a->dv1, 8) ||
            (a->v2 && !view_ok(p.v2v, a->dv - a->dv1, 8)) || !view_ok(p.ov, a->dv, 8)))
    return fail(VMB_EINVAL, "vmb_fea_fwd: layout strides must be multiples of 8 elements with rows >= cols");
  if (L && e4m3 && (!view_ok(p.qv, a->d, 16) || !view_ok(p.kv, a->d, 16) || (a->v2 && !view_ok(p.v2v, a->dv - a->dv1, 16))))
    return fail(VMB_EINVAL, "vmb_fea_fwd: e4m3 layout strides must be multiples of 16 elements");
  p.e4m3 = e4m3;
  p.n_q = (int)a->n_q; p.n_kv = (int)a->n_kv; p.dv1 = a->dv1;
  p.scale_log2 = a->sm_scale * kLog2eHost;
  p.wait_limit = g_test_wait_cycles.load(std::memory_order_relaxed);
  p.hold_loads = g_test_hold_loads.load(std::memory_order_relaxed);
  p.work = a->workspace;
  p.work_bytes = a->workspace ? a->workspace_bytes : 0;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = a->dtype == VMB_DTYPE_BF16;
  // V aliasing K (the VMonarch R step): the key tile in shared memory doubles as the value tile.
  // At d = 64 the separate-values kernel reads the same tensor twice instead (its only tcgen05 route).
  // d = 64: V aliasing K runs as such only with a second value tensor ([K | V2], dv = 128); V = K
  // alone takes the separate-values kernel over the same pointer
  const bool vk = fwd_v_is_k(a) && (a->d != 64 || a->dv == 128);
  if (e4m3) {
    count(1);
    return cuda_status(vmb::fea_fwd_sm100(p, a->batch, a->d, a->dv, a->ent != nullptr, bf16, true, st), "vmb_fea_fwd");
  }
  if (vmb::fea_fwd_sm100_supported(a->d, a->dv, a->dv1, vk)) {
    // a split key range adds the merge kernel
    count(vmb::fea_fwd_sm100_split(a->batch, p.n_q, p.n_kv, a->d, a->dv, p.work, p.work_bytes) > 1 ? 2 : 1);
    return cuda_status(vmb::fea_fwd_sm100(p, a->batch, a->d, a->dv, a->ent != nullptr, bf16, vk, st), "vmb_fea_fwd");
  }
  if (L) {
    // the mma.sync kernels take dense tensors: a layout must reduce to plain batch strides
    if (!uniform(p.qv, a->d, p.n1, p.n2, a->batch, &p.q_bs) || !uniform(p.kv, a->d, p.n1, p.n2, a->batch, &p.k_bs) ||
        !uniform(p.vv, a->dv1, p.n1, p.n2, a->batch, &p.v_bs) ||
        (a->v2 && !uniform(p.v2v, a->dv - a->dv1, p.n1, p.n2, a->batch, &p.v2_bs)) ||
        !uniform(p.ov, a->dv, p.n1, p.n2, a->batch, &p.o_bs))
      return fail(VMB_ENOTSUP, "vmb_fea_fwd: strided layouts need d = 128 (got d=%d dv=%d)", a->d, a->dv);
  }
  count(1);
  return cuda_status(vmb::fea_fwd_mma(p, a->batch, a->d, a->dv, a->ent != nullptr, bf16, st), "vmb_fea_fwd");
}

// Workspace: the tcgen05 path keeps three folded statistics planes [batch][round_up(n_q, 128)]
// and, when its dQ kernel splits the key range (long keys, few query tiles, grad_mode 1), the
// partial dQ tiles [split][batch][round_up(n_q, 128)][128]; the mma.sync path keeps c and g
// [batch][n_q] and, in grad_mode 0, an fp32 dQ accumulator.
static bool bwd_uses_sm100(const vmb_fea_bwd_args* a) {
  // d = 64 with [K | V2]: the dK tile's halves are dK and dV2, with no finalize (grad_mode 3) form
  if (a->d == 64 && a->v_is_k && a->dv == 128 && a->grad_mode == 3) return false;
  return vmb::fea_bwd_sm100_supported(a->d, a->dv, a->dv1, a->v_is_k != 0);
}

// Views of every tensor of a backward call (the layout's, or dense from the *_bs strides).
struct BwdViews {
  vmb::View q, k, v, v2, o, dout, gq, gk, gv, gv2, fq, fk, fv, fv2;
  int n1, n2;
};
static BwdViews bwd_views(const vmb_fea_bwd_args* a) {
  const vmb_fea_layout* L = a->layout;
  const int d = a->d, dv = a->dv, dv1 = a->dv1, dv2 = a->dv - a->dv1;
  BwdViews w;
  w.n1 = L ? (int)L->n1 : 1;
  w.n2 = L ? (int)L->n2 : 1;
  w.q = view_or_dense(L ? &L->q : nullptr, d, a->q_bs);
  w.k = view_or_dense(L ? &L->k : nullptr, d, a->k_bs);
  w.v = view_or_dense(L ? &L->v : nullptr, dv1, a->v_bs);
  w.v2 = view_or_dense(L ? &L->v2 : nullptr, dv2, a->v2_bs);
  w.o = view_or_dense(L ? &L->o : nullptr, dv, a->o_bs);
  w.dout = view_or_dense(L ? &L->dout : nullptr, dv, a->do_bs);
  w.gq = view_or_dense(L ? &L->grad_q : nullptr, d, a->grad_q_bs);
  w.gk = view_or_dense(L ? &L->grad_k : nullptr, d, a->grad_k_bs);
  w.gv = view_or_dense(L ? &L->grad_v : nullptr, dv1, a->grad_v_bs);
  w.gv2 = view_or_dense(L ? &L->grad_v2 : nullptr, dv2, a->grad_v2_bs);
  w.fq = view_or_dense(L ? &L->fin_q : nullptr, d, a->fin_q_bs);
  w.fk = view_or_dense(L ? &L->fin_k : nullptr, d, a->fin_k_bs);
  w.fv = view_or_dense(L ? &L->fin_v : nullptr, dv1, a->fin_v_bs);
  w.fv2 = view_or_dense(L ? &L->fin_v2 : nullptr, dv2, a->fin_v2_bs);
  return w;
}

// dQ's view is plain [batch][n_q][d] with one batch stride (the fused dQ path clears it with one
// 2-D memset in the overwrite mode)
static bool bwd_dq_uniform(const vmb_fea_bwd_args* a) {
  if (!a->layout) return true;
  int64_t bs;
  const BwdViews w = bwd_views(a);
  return uniform(w.gq, a->d, w.n1, w.n2, a->batch, &bs);
}

// tcgen05 path: dQ formed inside the dK kernel (no dq kernel, no split)
static bool bwd_fuses_dq(const vmb_fea_bwd_args* a) {
  return vmb::fea_bwd_fuses_dq((int)a->n_kv, a->d, a->dv, a->v_is_k != 0, a->grad_mode,
                               a->deterministic != 0 || !bwd_dq_uniform(a));
}

// tcgen05 path: dQ = dS K from the dS^T the dK/dV kernel stores (no dq kernel, no split)
static bool bwd_ds_gemm(const vmb_fea_bwd_args* a) {
  return vmb::fea_bwd_ds_gemm(a->batch, (int)a->n_q, (int)a->n_kv, a->dv, a->v_is_k != 0, a->grad_mode);
}

// tcgen05 path: CTAs sharing one query tile's key range in the dq kernel (1: no split)
static int bwd_dq_split(const vmb_fea_bwd_args* a, bool use_ds) {
  if (bwd_fuses_dq(a) || use_ds) return 1;
  return vmb::fea_bwd_dq_split(a->batch, (int)a->n_q, (int)a->n_kv, a->grad_mode != 0);
}

// tcgen05 workspace: three statistics planes, then either the split key range's partial dQ tiles
// (dq kernel) or the dS^T buffer (dQ from dS, taken when the workspace holds it)
static int64_t bwd_planes_bytes(const vmb_fea_bwd_args* a) {
  return 3 * round_up(a->batch * round_up(a->n_q, 128) * 4, 256);
}
static int64_t bwd_min_bytes(const vmb_fea_bwd_args* a) {
  const int split = bwd_dq_split(a, false);
  return bwd_planes_bytes(a) + (split > 1 ? round_up((int64_t)split * a->batch * round_up(a->n_q, 128) * 128 * 4, 256) : 0);
}
// + 256 bytes: dS^T starts at a 256-byte boundary (the dK/dV kernel stores it 32 bytes at a time)
static int64_t bwd_ds_need(const vmb_fea_bwd_args* a) {
  return bwd_planes_bytes(a) + round_up(vmb::fea_bwd_ds_bytes(a->batch, (int)a->n_q, (int)a->n_kv), 256) + 256;
}


int64_t vmb_fea_bwd_workspace_bytes(const vmb_fea_bwd_args* a) {
  if (!a || a->batch < 0 || a->n_q < 0) return -1;
  if (bwd_uses_sm100(a))  // the preferred size: room for dS^T where it is used
    return bwd_ds_gemm(a) ? std::max(bwd_min_bytes(a), bwd_ds_need(a)) : bwd_min_bytes(a);
  const int64_t rows = a->batch * a->n_q;
  int64_t bytes = 2 * round_up(rows * 4, 256);
  if (a->grad_mode == 0) bytes += round_up(rows * a->d * 4, 256);
  return bytes;
}

int64_t vmb_fea_bwd_min_workspace_bytes(const vmb_fea_bwd_args* a) {
  if (!a || a->batch < 0 || a->n_q < 0) return -1;
  if (!bwd_uses_sm100(a)) return vmb_fea_bwd_workspace_bytes(a);
  return bwd_min_bytes(a);
}

int vmb_fea_bwd(const vmb_fea_bwd_args* a, void* stream) {
  if (!a) return fail(VMB_EINVAL, "vmb_fea_bwd: null args");
  int rc = check_common("vmb_fea_bwd", a->batch, a->n_q, a->n_kv, a->d, a->dv, a->dv1, a->dtype, a->v2);
  if (rc) return rc;
  if (a->grad_mode < 0 || a->grad_mode > 3) return fail(VMB_EINVAL, "vmb_fea_bwd: grad_mode must be 0, 1, 2 or 3");
  if (a->grad_mode == 3) {
    if (!a->fin_q || !a->fin_k || (a->grad_v && !a->fin_v) || (a->grad_v2 && !a->fin_v2))
      return fail(VMB_EINVAL, "vmb_fea_bwd: grad_mode 3 needs an fp32 accumulator for every gradient");
    const void* fins[] = {a->fin_q, a->fin_k, a->fin_v, a->fin_v2};
    for (const void* ptr : fins)
      if (ptr && !aligned16(ptr)) return fail(VMB_EINVAL, "vmb_fea_bwd: accumulators must be 16-byte aligned");
    if ((a->fin_q_bs | a->fin_k_bs | a->fin_v_bs | a->fin_v2_bs) & 3)
      return fail(VMB_EINVAL, "vmb_fea_bwd: accumulator batch strides must be multiples of 4 elements");
  }
  if (a->v_is_k && (a->dv1 != a->d || a->grad_v != nullptr))
    return fail(VMB_EINVAL, "vmb_fea_bwd: v_is_k needs dv1 == d and grad_v == NULL");
  if (!a->v_is_k && !a->grad_v) return fail(VMB_EINVAL, "vmb_fea_bwd: grad_v is NULL");
  if ((a->dv1 < a->dv) != (a->grad_v2 != nullptr))
    return fail(VMB_EINVAL, "vmb_fea_bwd: grad_v2 must be given exactly when dv1 < dv");
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->grad_q || !a->grad_k)
    return fail(VMB_EINVAL, "vmb_fea_bwd: null tensor pointer");
  if (a->dent && !a->ent) return fail(VMB_EINVAL, "vmb_fea_bwd: dent given without ent");
  const void* ptrs[] = {a->q, a->k, a->v, a->v2, a->o, a->dout, a->grad_q, a->grad_k, a->grad_v, a->grad_v2,
                        a->workspace};
  for (const void* ptr : ptrs)
    if (ptr && !aligned16(ptr)) return fail(VMB_EINVAL, "vmb_fea_bwd: tensors must be 16-byte aligned");
  if ((a->q_bs | a->k_bs | a->v_bs | a->v2_bs | a->o_bs | a->do_bs | a->grad_q_bs | a->grad_k_bs | a->grad_v_bs |
       a->grad_v2_bs) & 7)
    return fail(VMB_EINVAL, "vmb_fea_bwd: batch strides must be multiples of 8 elements");
  const BwdViews w = bwd_views(a);
  if (a->layout) {
    if ((rc = check_split("vmb_fea_bwd", a->layout->n1, a->layout->n2, a->batch))) return rc;
    const int d = a->d, dv = a->dv, dv1 = a->dv1, dv2 = a->dv - a->dv1;
    const int ga = (a->grad_mode == 1 || a->grad_mode == 2) ? 4 : 8;  // fp32 gradients: 16-byte rows
    if (!view_ok(w.q, d, 8) || !view_ok(w.k, d, 8) || !view_ok(w.v, dv1, 8) || (a->v2 && !view_ok(w.v2, dv2, 8)) ||
        !view_ok(w.o, dv, 8) || !view_ok(w.dout, dv, 8) || !view_ok(w.gq, d, ga) || !view_ok(w.gk, d, ga) ||
        (a->grad_v && !view_ok(w.gv, dv1, ga)) || (a->grad_v2 && !view_ok(w.gv2, dv2, ga)) ||
        (a->grad_mode == 3 && (!view_ok(w.fq, d, 4) || !view_ok(w.fk, d, 4) || (a->fin_v && !view_ok(w.fv, dv1, 4)) ||
                               (a->fin_v2 && !view_ok(w.fv2, dv2, 4)))))
      return fail(VMB_EINVAL, "vmb_fea_bwd: layout strides must be multiples of 8 elements (4 for fp32) with rows >= cols");
  }
  if (a->batch == 0) return VMB_OK;
  // at least the minimal workspace; the tcgen05 path takes dQ from dS when the workspace also holds dS^T
  const int64_t need = bwd_uses_sm100(a) ? bwd_min_bytes(a) : vmb_fea_bwd_workspace_bytes(a);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(VMB_EINVAL, "vmb_fea_bwd: workspace of %lld bytes needed", (long long)need);
  const bool use_ds = bwd_uses_sm100(a) && bwd_ds_gemm(a) && a->workspace_bytes >= bwd_ds_need(a);
  if (a->n_q == 0) return VMB_OK;  // no query: no gradient contribution (grad_mode 1 adds nothing)
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = a->dtype == VMB_DTYPE_BF16;
  const int64_t rows = a->batch * a->n_q;
  char* ws = static_cast<char*>(a->workspace);
  const bool sm100 = bwd_uses_sm100(a);
  // tcgen05 path: folded planes (the dQ kernel writes grad_q directly in either grad mode)
  const int64_t n_pad = round_up(a->n_q, 128);
  float* fold = sm100 ? reinterpret_cast<float*>(ws) : nullptr;
  // mma.sync path: c, g and the fp32 dQ accumulator of grad_mode 0
  float* cc = sm100 ? nullptr : reinterpret_cast<float*>(ws);
  float* gg = sm100 ? nullptr : reinterpret_cast<float*>(ws + round_up(rows * 4, 256));
  float* dq_acc =
      (!sm100 && a->grad_mode == 0) ? reinterpret_cast<float*>(ws + 2 * round_up(rows * 4, 256)) : nullptr;
  count(sm100 ? (bwd_fuses_dq(a) ? 2 : (bwd_dq_split(a, use_ds) > 1 ? 4 : 3)) : (dq_acc ? 3 : 2));
  vmb::BwdParams p{};
  p.n1 = w.n1; p.n2 = w.n2;
  p.d = a->d;
  p.qv = w.q; p.kv = w.k; p.vv = w.v; p.v2v = w.v2; p.dov = w.dout;
  p.dqv = w.gq; p.dkv = w.gk; p.dvv = w.gv; p.dv2v = w.gv2;
  p.finqv = w.fq; p.finkv = w.fk; p.finvv = w.fv; p.finv2v = w.fv2;
  p.q_bs = a->q_bs; p.k_bs = a->k_bs; p.v_bs = a->v_bs; p.v2_bs = a->v2_bs; p.do_bs = a->do_bs;
  p.dk_bs = a->grad_k_bs; p.dv_bs = a->grad_v_bs; p.dv2_bs = a->grad_v2_bs;
  p.fin_q_bs = a->fin_q_bs; p.fin_k_bs = a->fin_k_bs; p.fin_v_bs = a->fin_v_bs; p.fin_v2_bs = a->fin_v2_bs;
  int64_t o_bs = a->o_bs, gq_bs = a->grad_q_bs;
  if (a->layout) uniform(w.gq, a->d, w.n1, w.n2, a->batch, &gq_bs);  // dQ's batch stride when it is plain
  if (!sm100 && a->layout) {
    // the mma.sync kernels take dense tensors: the layout must reduce to plain batch strides
    const int64_t B = a->batch;
    const int n1 = w.n1, n2 = w.n2;
    const bool ok = uniform(w.q, a->d, n1, n2, B, &p.q_bs) && uniform(w.k, a->d, n1, n2, B, &p.k_bs) &&
                    uniform(w.v, a->dv1, n1, n2, B, &p.v_bs) &&
                    (!a->v2 || uniform(w.v2, a->dv - a->dv1, n1, n2, B, &p.v2_bs)) &&
                    uniform(w.o, a->dv, n1, n2, B, &o_bs) && uniform(w.dout, a->dv, n1, n2, B, &p.do_bs) &&
                    uniform(w.gq, a->d, n1, n2, B, &gq_bs) && uniform(w.gk, a->d, n1, n2, B, &p.dk_bs) &&
                    (!a->grad_v || uniform(w.gv, a->dv1, n1, n2, B, &p.dv_bs)) &&
                    (!a->grad_v2 || uniform(w.gv2, a->dv - a->dv1, n1, n2, B, &p.dv2_bs)) &&
                    (a->grad_mode != 3 ||
                     (uniform(w.fq, a->d, n1, n2, B, &p.fin_q_bs) && uniform(w.fk, a->d, n1, n2, B, &p.fin_k_bs) &&
                      (!a->fin_v || uniform(w.fv, a->dv1, n1, n2, B, &p.fin_v_bs)) &&
                      (!a->fin_v2 || uniform(w.fv2, a->dv - a->dv1, n1, n2, B, &p.fin_v2_bs))));
    if (!ok) return fail(VMB_ENOTSUP, "vmb_fea_bwd: strided layouts need d = 128 (got d=%d dv=%d)", a->d, a->dv);
  }
  cudaError_t e = vmb::fea_bwd_pre(a->o, w.o, a->dout, w.dout, w.n1, w.n2, a->lse, a->ent, a->dent, cc, gg, a->batch,
                                   (int)a->n_q, a->dv, fold, n_pad, a->sm_scale, a->delta, bf16, st);
  if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(pre)");
  if (dq_acc) {
    e = cudaMemsetAsync(dq_acc, 0, rows * a->d * 4, st);
    if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(memset)");
  }
  p.q = a->q; p.k = a->k; p.v = a->v; p.v2 = a->v2; p.dout = a->dout; p.lse = a->lse; p.cc = cc; p.gg = gg;
  p.fold = fold; p.n_pad = n_pad;
  p.dq_part = nullptr;
  if (sm100 && bwd_dq_split(a, use_ds) > 1) p.dq_part = reinterpret_cast<float*>(ws + bwd_planes_bytes(a));
  p.ds = use_ds ? reinterpret_cast<void*>(round_up(reinterpret_cast<intptr_t>(ws + bwd_planes_bytes(a)), 256)) : nullptr;
  p.dq = dq_acc ? dq_acc : static_cast<float*>(a->grad_q);
  p.dk = a->grad_k; p.dv = a->grad_v; p.dv2 = a->grad_v2;
  p.dq_bs = dq_acc ? a->n_q * a->d : gq_bs;
  p.n_q = (int)a->n_q; p.n_kv = (int)a->n_kv; p.dv1 = a->dv1;
  p.acc_kv = a->grad_mode;
  p.acc_q = a->grad_mode;
  p.sm_scale = a->sm_scale;
  p.scale_log2 = a->sm_scale * kLog2eHost;
  p.deterministic = a->deterministic != 0 || !bwd_dq_uniform(a);  // fused dQ needs a plain dQ
  p.fin_q = a->fin_q; p.fin_k = a->fin_k; p.fin_v = a->fin_v; p.fin_v2 = a->fin_v2;
  if (sm100) return cuda_status(vmb::fea_bwd_sm100(p, a->batch, a->dv, a->v_is_k != 0, bf16, st), "vmb_fea_bwd");
  // batch strides of the dense (mma.sync) path: the *_bs fields, or those a uniform layout reduces to
  const int64_t gk_bs = p.dk_bs, gv_bs = p.dv_bs, gv2_bs = p.dv2_bs;
  const int64_t fq_bs = p.fin_q_bs, fk_bs = p.fin_k_bs, fv_bs = p.fin_v_bs, fv2_bs = p.fin_v2_bs;
  if (a->grad_mode == 3) {
    // the mma.sync kernels add into the fp32 accumulators, which are then converted to grad_*
    p.dq = const_cast<float*>(a->fin_q);
    p.dq_bs = fq_bs;
    p.dk = const_cast<float*>(a->fin_k);
    p.dv = const_cast<float*>(a->fin_v);
    p.dv2 = const_cast<float*>(a->fin_v2);
    p.dk_bs = fk_bs; p.dv_bs = fv_bs; p.dv2_bs = fv2_bs;
    p.acc_kv = p.acc_q = 1;
    e = vmb::fea_bwd_mma(p, a->batch, a->d, a->dv, a->v_is_k != 0, bf16, st);
    auto conv = [&](const float* src, int64_t sbs, void* dst, int64_t dbs, int64_t n) -> cudaError_t {
      if (!dst) return cudaSuccess;
      count(1);
      return vmb::cast_f32(src, sbs, dst, dbs, a->batch, n, bf16, st);
    };
    if (e == cudaSuccess) e = conv(a->fin_q, fq_bs, a->grad_q, gq_bs, a->n_q * a->d);
    if (e == cudaSuccess) e = conv(a->fin_k, fk_bs, a->grad_k, gk_bs, a->n_kv * a->d);
    if (e == cudaSuccess) e = conv(a->fin_v, fv_bs, a->grad_v, gv_bs, a->n_kv * a->dv1);
    if (e == cudaSuccess) e = conv(a->fin_v2, fv2_bs, a->grad_v2, gv2_bs, a->n_kv * (a->dv - a->dv1));
    return cuda_status(e, "vmb_fea_bwd");
  }
  if (a->grad_mode == 2) {
    // the mma.sync kernels only add: clear the fp32 gradients, then accumulate
    auto clear = [&](void* ptr, int64_t bs, int64_t rows, int cols) -> cudaError_t {
      return ptr ? cudaMemset2DAsync(ptr, bs * 4, 0, rows * cols * 4, a->batch, st) : cudaSuccess;
    };
    e = clear(a->grad_q, gq_bs, a->n_q, a->d);
    if (e == cudaSuccess) e = clear(a->grad_k, gk_bs, a->n_kv, a->d);
    if (e == cudaSuccess) e = clear(a->grad_v, gv_bs, a->n_kv, a->dv1);
    if (e == cudaSuccess) e = clear(a->grad_v2, gv2_bs, a->n_kv, a->dv - a->dv1);
    if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(clear)");
    p.acc_kv = p.acc_q = 1;
  }
  e = vmb::fea_bwd_mma(p, a->batch, a->d, a->dv, a->v_is_k != 0, bf16, st);
  if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd");
  if (dq_acc) {
    e = vmb::cast_f32(dq_acc, a->n_q * a->d, a->grad_q, gq_bs, a->batch, a->n_q * a->d, bf16, st);
    if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(dq cast)");
  }
  return VMB_OK;
}

static int lstep_check(const char* what, const vmb_lstep_args* a, bool bwd) {
  if (!a) return fail(VMB_EINVAL, "%s: null args", what);
  if (a->dtype != VMB_DTYPE_BF16 && a->dtype != VMB_DTYPE_F16) return fail(VMB_EINVAL, "%s: unknown dtype", what);
  if (a->d != 16 && a->d != 32 && a->d != 64 && a->d != 128) return fail(VMB_ENOTSUP, "%s: no kernel for d=%d", what, a->d);
  if (a->m < 1 || a->m > 128) return fail(VMB_ENOTSUP, "%s: num_blocks m=%lld outside [1, 128]", what, (long long)a->m);
  if (a->b < 1 || a->bh < 0) return fail(VMB_EINVAL, "%s: bad sizes", what);
  if (a->last) {
    const int dv = a->dw - a->d;
    if (!pow2_dim(dv) || dv % a->d) return fail(VMB_ENOTSUP, "%s: no kernel for value dim %d", what, dv);
  } else if (a->dw != a->d) {
    return fail(VMB_EINVAL, "%s: non-last step needs dw == d", what);
  }
  if (!a->q || !a->out || !a->ent) return fail(VMB_EINVAL, "%s: null tensor pointer", what);
  if (!bwd && !(a->last ? a->z : a->u)) return fail(VMB_EINVAL, "%s: null output pointer", what);
  if (bwd && (!a->dq || !a->dout || !(a->last ? (const void*)a->dz : (const void*)a->du)))
    return fail(VMB_EINVAL, "%s: null gradient pointer", what);
  if (bwd && a->delta_out && !pow2_dim(a->dw))
    return fail(VMB_ENOTSUP, "%s: delta_out needs an out width of 16, 32, 64, 128 or 256 (got %d)", what, a->dw);
  const void* ptrs[] = {a->q, a->out, a->u, a->z, a->du, a->dz, a->dq, a->dout};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return fail(VMB_EINVAL, "%s: tensors must be 16-byte aligned", what);
  if (const vmb_lstep_layout* L = a->layout) {
    if (L->n1 < 1 || L->n1 > 0x7fffffff || a->bh % L->n1)
      return fail(VMB_EINVAL, "%s: layout n1=%lld does not divide bh=%lld", what, (long long)L->n1, (long long)a->bh);
    const int d = a->d, dw = a->dw, dv = a->dw - a->d;
    const bool ok = view_ok(to_view(L->q), d, 8) && view_ok(to_view(L->out), dw, 8) &&
                    (!a->u || view_ok(to_view(L->u), d, 8)) && (!a->z || view_ok(to_view(L->z), dv, 8)) &&
                    (!bwd || ((!a->du || view_ok(to_view(L->du), d, 4)) && (!a->dz || view_ok(to_view(L->dz), dv, 8)) &&
                              view_ok(to_view(L->dq), d, 4) && view_ok(to_view(L->dout), dw, 8)));
    if (!ok) return fail(VMB_EINVAL, "%s: layout strides must be multiples of 8 elements (4 for fp32) with rows >= cols", what);
  }
  return VMB_OK;
}

static int lstep_run(const char* what, const vmb_lstep_args* a, bool bwd, void* stream) {
  int rc = lstep_check(what, a, bwd);
  if (rc) return rc;
  if (a->bh == 0) return VMB_OK;
  count(1);
  vmb::LstepParams p{};
  p.q = a->q; p.out = a->out; p.ent = a->ent; p.u = a->u; p.z = a->z; p.du = a->du; p.dz = a->dz;
  p.dq = a->dq; p.dout = a->dout;
  p.bh = a->bh; p.m = a->m; p.b = a->b; p.d = a->d; p.dw = a->dw; p.skip_rows = a->skip_rows;
  p.scale = a->scale; p.min_col_mass = a->min_col_mass;
  p.dq_store = a->dq_store != 0;
  p.delta_out = bwd ? a->delta_out : nullptr;
  const vmb_lstep_layout* L = a->layout;
  const int64_t N = p.m * p.b;
  const int dv = a->dw - a->d;
  p.n1 = L ? (int)L->n1 : 1;
  p.qv = view_or_dense(L ? &L->q : nullptr, a->d, N * a->d);
  p.outv = view_or_dense(L ? &L->out : nullptr, a->dw, N * a->dw);
  p.uv = view_or_dense(L ? &L->u : nullptr, a->d, N * a->d);
  p.zv = view_or_dense(L ? &L->z : nullptr, dv, N * dv);
  p.duv = view_or_dense(L ? &L->du : nullptr, a->d, N * a->d);
  p.dzv = view_or_dense(L ? &L->dz : nullptr, dv, N * dv);
  p.dqv = view_or_dense(L ? &L->dq : nullptr, a->d, N * a->d);
  p.doutv = view_or_dense(L ? &L->dout : nullptr, a->dw, N * a->dw);
  const bool bf16 = a->dtype == VMB_DTYPE_BF16;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vmb::lstep_tc_supported(p, a->last != 0, bwd))
    return cuda_status(vmb::lstep_tc_launch(p, a->last != 0, bwd, bf16, st), what);
  if (vmb::lstep_mma_supported(p, a->last != 0))
    return cuda_status(vmb::lstep_mma_launch(p, a->last != 0, bwd, bf16, st), what);
  // the generic kernel keeps the m rows of every operand in shared memory
  if (a->m > 64)
    return fail(VMB_ENOTSUP, "%s: num_blocks m=%lld > 64 needs d in {64, 128} with dw = d (2d when last)", what,
                (long long)a->m);
  if (L) {
    // the generic kernel takes dense [bh][N][cols] tensors only
    auto dense = [&](const vmb::View& v, int64_t cols, const void* ptr) {
      int64_t bs;
      return !ptr || (uniform(v, cols, p.n1, 1, a->bh, &bs) && bs == N * cols);
    };
    if (!dense(p.qv, a->d, a->q) || !dense(p.outv, a->dw, a->out) || !dense(p.uv, a->d, a->u) ||
        !dense(p.zv, dv, a->z) || (bwd && (!dense(p.duv, a->d, a->du) || !dense(p.dzv, dv, a->dz) ||
                                           !dense(p.dqv, a->d, a->dq) || !dense(p.doutv, a->dw, a->dout))))
      return fail(VMB_ENOTSUP, "%s: strided layouts need m <= 128 and d in {64, 128} (got m=%lld, d=%d)", what, (long long)a->m, a->d);
  }
  cudaError_t e = vmb::lstep_launch(p, a->last != 0, bwd, bf16, st);
  if (e == cudaSuccess && p.delta_out) {
    // the generic kernel does not fold delta in: sum out . dout per token, like the preprocess
    count(1);
    const vmb::View dense_out = vmb::dense_view(a->dw, N * a->dw, 1, 1);
    e = vmb::fea_bwd_pre(a->out, dense_out, a->dout, dense_out, 1, 1, nullptr, nullptr, nullptr, p.delta_out, nullptr,
                         a->bh, (int)N, a->dw, nullptr, 0, 0.f, nullptr, bf16, st);
  }
  return cuda_status(e, what);
}

int vmb_lstep_fwd(const vmb_lstep_args* a, void* stream) { return lstep_run("vmb_lstep_fwd", a, false, stream); }
int vmb_lstep_bwd(const vmb_lstep_args* a, void* stream) { return lstep_run("vmb_lstep_bwd", a, true, stream); }

int vmb_cast_f32(const float* src, int64_t src_bs, void* dst, int64_t dst_bs, int64_t batch, int64_t n, int32_t dtype,
                 void* stream) {
  if (dtype != VMB_DTYPE_BF16 && dtype != VMB_DTYPE_F16) return fail(VMB_EINVAL, "vmb_cast_f32: unknown dtype");
  if (batch < 0 || n < 0 || (n | src_bs | dst_bs) & 3) return fail(VMB_EINVAL, "vmb_cast_f32: sizes must be multiples of 4");
  if (batch == 0 || n == 0) return VMB_OK;
  if (!src || !dst || !aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7))
    return fail(VMB_EINVAL, "vmb_cast_f32: bad pointer");
  count(1);
  return cuda_status(vmb::cast_f32(src, src_bs, dst, dst_bs, batch, n, dtype == VMB_DTYPE_BF16, static_cast<cudaStream_t>(stream)),
                     "vmb_cast_f32");
}

int vmb_quant_e4m3(const void* src, const vmb_view* src_view, void* dst, const vmb_view* dst_view, int64_t n1,
                   int64_t n2, int64_t batch, int64_t rows, int64_t cols, int32_t dtype, float scale, void* stream) {
  if (dtype != VMB_DTYPE_BF16 && dtype != VMB_DTYPE_F16) return fail(VMB_EINVAL, "vmb_quant_e4m3: unknown dtype");
  if (!src_view || !dst_view || batch < 0 || rows < 0 || cols < 0 || cols % 16)
    return fail(VMB_EINVAL, "vmb_quant_e4m3: bad sizes or views (cols a multiple of 16)");
  int rc = check_split("vmb_quant_e4m3", n1, n2, batch);
  if (rc) return rc;
  if (batch == 0 || rows == 0 || cols == 0) return VMB_OK;
  const vmb::View sv = to_view(*src_view), dv = to_view(*dst_view);
  if (!src || !dst || !aligned16(src) || !aligned16(dst) || !view_ok(sv, cols, 8) || !view_ok(dv, cols, 16))
    return fail(VMB_EINVAL, "vmb_quant_e4m3: bad pointer or view");
  count(1);
  return cuda_status(vmb::quant_e4m3(src, sv, dst, dv, (int)n1, (int)n2, batch, rows, cols, dtype == VMB_DTYPE_BF16,
                                     scale, static_cast<cudaStream_t>(stream)),
                     "vmb_quant_e4m3");
}

int vmb_cast_f32_view(const float* src, const vmb_view* src_view, void* dst, const vmb_view* dst_view, int64_t n1,
                      int64_t n2, int64_t batch, int64_t rows, int64_t cols, int32_t dtype, void* stream) {
  if (dtype != VMB_DTYPE_BF16 && dtype != VMB_DTYPE_F16) return fail(VMB_EINVAL, "vmb_cast_f32_view: unknown dtype");
  if (!src_view || !dst_view || batch < 0 || rows < 0 || cols < 0 || cols % 4)
    return fail(VMB_EINVAL, "vmb_cast_f32_view: bad sizes or views");
  int rc = check_split("vmb_cast_f32_view", n1, n2, batch);
  if (rc) return rc;
  if (batch == 0 || rows == 0 || cols == 0) return VMB_OK;
  const vmb::View sv = to_view(*src_view), dv = to_view(*dst_view);
  if (!src || !dst || !aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7) || !view_ok(sv, cols, 4) ||
      !view_ok(dv, cols, 4))
    return fail(VMB_EINVAL, "vmb_cast_f32_view: bad pointer or view");
  count(1);
  return cuda_status(vmb::cast_f32_view(src, sv, dst, dv, (int)n1, (int)n2, batch, rows, cols, dtype == VMB_DTYPE_BF16,
                                        static_cast<cudaStream_t>(stream)),
                     "vmb_cast_f32_view");
}

}  // extern "C"

namespace vmb {
int64_t fea_bwd_min_workspace_bytes(const vmb_fea_bwd_args* a) { return vmb_fea_bwd_min_workspace_bytes(a); }
}  // namespace vmb
