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

bool fea_dims_ok(int d, int dv) {
  return (d == 64 || d == 128) && (dv == 64 || dv == 128 || dv == 256) && dv % d == 0;
}

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

static bool fwd_v_is_k(const vmb_fea_fwd_args* a) {
  return a->v == a->k && a->v_bs == a->k_bs && a->dv1 == a->d;
}

int64_t vmb_fea_fwd_workspace_bytes(const vmb_fea_fwd_args* a) {
  if (!a || a->batch < 0 || a->n_q < 0 || a->n_kv < 1) return -1;
  if (a->batch == 0 || a->n_q == 0 || a->n_q > 0x7fffffff || a->n_kv > 0x7fffffff) return 0;
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
  if (a->workspace && (!aligned16(a->workspace) || a->workspace_bytes < 0))
    return fail(VMB_EINVAL, "vmb_fea_fwd: workspace must be 16-byte aligned");
  vmb::FwdParams p{};
  p.q = a->q; p.k = a->k; p.v = a->v; p.v2 = a->v2; p.o = a->o; p.lse = a->lse; p.ent = a->ent;
  p.q_bs = a->q_bs; p.k_bs = a->k_bs; p.v_bs = a->v_bs; p.v2_bs = a->v2_bs; p.o_bs = a->o_bs;
  p.n_q = (int)a->n_q; p.n_kv = (int)a->n_kv; p.dv1 = a->dv1;
  p.scale_log2 = a->sm_scale * kLog2eHost;
  p.work = a->workspace;
  p.work_bytes = a->workspace ? a->workspace_bytes : 0;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = a->dtype == VMB_DTYPE_BF16;
  // V aliasing K (the VMonarch R step): the key tile in shared memory doubles as the value tile
  const bool vk = fwd_v_is_k(a);
  if (vmb::fea_fwd_sm100_supported(a->d, a->dv, a->dv1, vk)) {
    // a split key range adds the merge kernel
    count(vmb::fea_fwd_sm100_split(a->batch, p.n_q, p.n_kv, a->dv, p.work, p.work_bytes) > 1 ? 2 : 1);
    return cuda_status(vmb::fea_fwd_sm100(p, a->batch, a->d, a->dv, a->ent != nullptr, bf16, vk, st), "vmb_fea_fwd");
  }
  count(1);
  return cuda_status(vmb::fea_fwd_mma(p, a->batch, a->d, a->dv, a->ent != nullptr, bf16, st), "vmb_fea_fwd");
}

// Workspace: the tcgen05 path keeps three folded statistics planes [batch][round_up(n_q, 128)]
// and, when its dQ kernel splits the key range (long keys, few query tiles, grad_mode 1), the
// partial dQ tiles [split][batch][round_up(n_q, 128)][128]; the mma.sync path keeps c and g
// [batch][n_q] and, in grad_mode 0, an fp32 dQ accumulator.
static bool bwd_uses_sm100(const vmb_fea_bwd_args* a) {
  return vmb::fea_bwd_sm100_supported(a->d, a->dv, a->dv1, a->v_is_k != 0);
}

// tcgen05 path: dQ formed inside the dK kernel (no dq kernel, no split)
static bool bwd_fuses_dq(const vmb_fea_bwd_args* a) {
  return vmb::fea_bwd_fuses_dq((int)a->n_kv, a->dv, a->v_is_k != 0, a->grad_mode, a->deterministic != 0);
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
  cudaError_t e = vmb::fea_bwd_pre(a->o, a->o_bs, a->dout, a->do_bs, a->lse, a->ent, a->dent, cc, gg, a->batch,
                                   (int)a->n_q, a->dv, fold, n_pad, a->sm_scale, a->delta, bf16, st);
  if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(pre)");
  if (dq_acc) {
    e = cudaMemsetAsync(dq_acc, 0, rows * a->d * 4, st);
    if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(memset)");
  }
  vmb::BwdParams p{};
  p.q = a->q; p.k = a->k; p.v = a->v; p.v2 = a->v2; p.dout = a->dout; p.lse = a->lse; p.cc = cc; p.gg = gg;
  p.fold = fold; p.n_pad = n_pad;
  p.dq_part = nullptr;
  if (sm100 && bwd_dq_split(a, use_ds) > 1) p.dq_part = reinterpret_cast<float*>(ws + bwd_planes_bytes(a));
  p.ds = use_ds ? reinterpret_cast<void*>(round_up(reinterpret_cast<intptr_t>(ws + bwd_planes_bytes(a)), 256)) : nullptr;
  p.dq = dq_acc ? dq_acc : static_cast<float*>(a->grad_q);
  p.dk = a->grad_k; p.dv = a->grad_v; p.dv2 = a->grad_v2;
  p.q_bs = a->q_bs; p.k_bs = a->k_bs; p.v_bs = a->v_bs; p.v2_bs = a->v2_bs; p.do_bs = a->do_bs;
  p.dq_bs = dq_acc ? a->n_q * a->d : a->grad_q_bs;
  p.dk_bs = a->grad_k_bs; p.dv_bs = a->grad_v_bs; p.dv2_bs = a->grad_v2_bs;
  p.n_q = (int)a->n_q; p.n_kv = (int)a->n_kv; p.dv1 = a->dv1;
  p.acc_kv = a->grad_mode;
  p.acc_q = a->grad_mode;
  p.sm_scale = a->sm_scale;
  p.scale_log2 = a->sm_scale * kLog2eHost;
  p.deterministic = a->deterministic != 0;
  p.fin_q = a->fin_q; p.fin_k = a->fin_k; p.fin_v = a->fin_v; p.fin_v2 = a->fin_v2;
  p.fin_q_bs = a->fin_q_bs; p.fin_k_bs = a->fin_k_bs; p.fin_v_bs = a->fin_v_bs; p.fin_v2_bs = a->fin_v2_bs;
  if (sm100) return cuda_status(vmb::fea_bwd_sm100(p, a->batch, a->dv, a->v_is_k != 0, bf16, st), "vmb_fea_bwd");
  if (a->grad_mode == 3) {
    // the mma.sync kernels add into the fp32 accumulators, which are then converted to grad_*
    p.dq = const_cast<float*>(a->fin_q);
    p.dq_bs = a->fin_q_bs;
    p.dk = const_cast<float*>(a->fin_k);
    p.dv = const_cast<float*>(a->fin_v);
    p.dv2 = const_cast<float*>(a->fin_v2);
    p.dk_bs = a->fin_k_bs; p.dv_bs = a->fin_v_bs; p.dv2_bs = a->fin_v2_bs;
    p.acc_kv = p.acc_q = 1;
    e = vmb::fea_bwd_mma(p, a->batch, a->d, a->dv, a->v_is_k != 0, bf16, st);
    auto conv = [&](const float* src, int64_t sbs, void* dst, int64_t dbs, int64_t n) -> cudaError_t {
      if (!dst) return cudaSuccess;
      count(1);
      return vmb::cast_f32(src, sbs, dst, dbs, a->batch, n, bf16, st);
    };
    if (e == cudaSuccess) e = conv(a->fin_q, a->fin_q_bs, a->grad_q, a->grad_q_bs, a->n_q * a->d);
    if (e == cudaSuccess) e = conv(a->fin_k, a->fin_k_bs, a->grad_k, a->grad_k_bs, a->n_kv * a->d);
    if (e == cudaSuccess) e = conv(a->fin_v, a->fin_v_bs, a->grad_v, a->grad_v_bs, a->n_kv * a->dv1);
    if (e == cudaSuccess) e = conv(a->fin_v2, a->fin_v2_bs, a->grad_v2, a->grad_v2_bs, a->n_kv * (a->dv - a->dv1));
    return cuda_status(e, "vmb_fea_bwd");
  }
  if (a->grad_mode == 2) {
    // the mma.sync kernels only add: clear the fp32 gradients, then accumulate
    auto clear = [&](void* ptr, int64_t bs, int64_t rows, int cols) -> cudaError_t {
      return ptr ? cudaMemset2DAsync(ptr, bs * 4, 0, rows * cols * 4, a->batch, st) : cudaSuccess;
    };
    e = clear(a->grad_q, a->grad_q_bs, a->n_q, a->d);
    if (e == cudaSuccess) e = clear(a->grad_k, a->grad_k_bs, a->n_kv, a->d);
    if (e == cudaSuccess) e = clear(a->grad_v, a->grad_v_bs, a->n_kv, a->dv1);
    if (e == cudaSuccess) e = clear(a->grad_v2, a->grad_v2_bs, a->n_kv, a->dv - a->dv1);
    if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(clear)");
    p.acc_kv = p.acc_q = 1;
  }
  e = vmb::fea_bwd_mma(p, a->batch, a->d, a->dv, a->v_is_k != 0, bf16, st);
  if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd");
  if (dq_acc) {
    e = vmb::cast_f32(dq_acc, a->n_q * a->d, a->grad_q, a->grad_q_bs, a->batch, a->n_q * a->d, bf16, st);
    if (e != cudaSuccess) return cuda_status(e, "vmb_fea_bwd(dq cast)");
  }
  return VMB_OK;
}

static int lstep_check(const char* what, const vmb_lstep_args* a, bool bwd) {
  if (!a) return fail(VMB_EINVAL, "%s: null args", what);
  if (a->dtype != VMB_DTYPE_BF16 && a->dtype != VMB_DTYPE_F16) return fail(VMB_EINVAL, "%s: unknown dtype", what);
  if (a->d != 64 && a->d != 128) return fail(VMB_ENOTSUP, "%s: no kernel for d=%d", what, a->d);
  if (a->m < 1 || a->m > 64) return fail(VMB_ENOTSUP, "%s: num_blocks m=%lld outside [1, 64]", what, (long long)a->m);
  if (a->b < 1 || a->bh < 0) return fail(VMB_EINVAL, "%s: bad sizes", what);
  if (a->last) {
    const int dv = a->dw - a->d;
    if (dv != 64 && dv != 128 && dv != 256) return fail(VMB_ENOTSUP, "%s: no kernel for value dim %d", what, dv);
  } else if (a->dw != a->d) {
    return fail(VMB_EINVAL, "%s: non-last step needs dw == d", what);
  }
  if (!a->q || !a->out || !a->ent) return fail(VMB_EINVAL, "%s: null tensor pointer", what);
  if (!bwd && !(a->last ? a->z : a->u)) return fail(VMB_EINVAL, "%s: null output pointer", what);
  if (bwd && (!a->dq || !a->dout || !(a->last ? (const void*)a->dz : (const void*)a->du)))
    return fail(VMB_EINVAL, "%s: null gradient pointer", what);
  if (bwd && a->delta_out && a->dw != 64 && a->dw != 128 && a->dw != 256)
    return fail(VMB_ENOTSUP, "%s: delta_out needs an out width of 64, 128 or 256 (got %d)", what, a->dw);
  const void* ptrs[] = {a->q, a->out, a->u, a->z, a->du, a->dz, a->dq, a->dout};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return fail(VMB_EINVAL, "%s: tensors must be 16-byte aligned", what);
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
  const bool bf16 = a->dtype == VMB_DTYPE_BF16;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vmb::lstep_tc_supported(p, a->last != 0, bwd))
    return cuda_status(vmb::lstep_tc_launch(p, a->last != 0, bwd, bf16, st), what);
  if (vmb::lstep_mma_supported(p, a->last != 0))
    return cuda_status(vmb::lstep_mma_launch(p, a->last != 0, bwd, bf16, st), what);
  cudaError_t e = vmb::lstep_launch(p, a->last != 0, bwd, bf16, st);
  if (e == cudaSuccess && p.delta_out) {
    // the generic kernel does not fold delta in: sum out . dout per token, like the preprocess
    count(1);
    e = vmb::fea_bwd_pre(a->out, p.m * p.b * a->dw, a->dout, p.m * p.b * a->dw, nullptr, nullptr, nullptr,
                         p.delta_out, nullptr, a->bh, (int)(p.m * p.b), a->dw, nullptr, 0, 0.f, nullptr, bf16, st);
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

}  // extern "C"

namespace vmb {
int64_t fea_bwd_min_workspace_bytes(const vmb_fea_bwd_args* a) { return vmb_fea_bwd_min_workspace_bytes(a); }
}  // namespace vmb
