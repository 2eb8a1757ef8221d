// extern "C" boundary of libpolyattn.so: argument validation, kernel choice,
// thread-local error reporting. Declarations and the reference interfaces
// each entry point replaces are in include/poly_attention.h.
#include <atomic>
#include <cstdlib>
#include <string>

#include "common.cuh"

namespace poly {

static thread_local std::string g_error;

void set_error(const std::string& msg) { g_error = msg; }

static std::atomic<unsigned long long> g_launches{0};
void note_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

static int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

static int check_pass(const PolyPassArgs* a) {
  if (!a) return fail(POLY_EINVAL, "null args");
  if (a->batch <= 0 || a->heads <= 0 || a->kv_heads <= 0 || a->seq_q < 0 || a->seq_k <= 0 || a->head_dim <= 0)
    return fail(POLY_EINVAL, "batch, heads, kv_heads, seq_k and head_dim must be positive, seq_q non-negative");
  if (a->heads % a->kv_heads != 0) return fail(POLY_EINVAL, "heads must be divisible by kv_heads");
  if (a->dtype != POLY_F32 && a->dtype != POLY_F16 && a->dtype != POLY_BF16) return fail(POLY_EINVAL, "unknown dtype");
  if (a->head_dim > 128) return fail(POLY_EUNSUPPORTED, "head_dim > 128 is not supported");
  if (!a->q || !a->k || !a->v || !a->out) return fail(POLY_EINVAL, "q, k, v and out are required");
  if (a->epi_out && !a->epi_mul) return fail(POLY_EINVAL, "epi_out requires epi_mul");
  if (!(a->scale == a->scale)) return fail(POLY_EINVAL, "scale is NaN");
  if (a->causal_offset < 0) return fail(POLY_EINVAL, "causal_offset must be non-negative");
  return POLY_OK;
}

enum class FwdKind { kSimt, kTc, kDecode, kSmall, kF32 };

static FwdKind choose_fwd(const PolyPassArgs& a) {
  // a causal offset only on the tcgen05 forward (kSimt is then refused by the caller)
  if (a.causal_offset) return pass_fwd_tc_eligible(a) && pass_fwd_tc2_eligible(a) ? FwdKind::kTc : FwdKind::kSimt;
  if (pass_decode_eligible(a)) return FwdKind::kDecode;
  if (pass_small_eligible(a)) return FwdKind::kSmall;
  if (pass_f32_eligible(a)) return FwdKind::kF32;
  if (pass_fwd_tc_eligible(a)) return FwdKind::kTc;
  return FwdKind::kSimt;
}

static bool use_bwd_tc(const PolyPassBwdArgs& a) { return pass_bwd_tc_eligible(a); }

static size_t simt_bwd_workspace(const PolyPassBwdArgs& a) {
  return (size_t)a.fwd.batch * a.fwd.heads * (size_t)a.fwd.seq_q * (sizeof(float) + sizeof(int));
}

}  // namespace poly

using namespace poly;

extern "C" {

const char* poly_last_error(void) { return g_error.c_str(); }
unsigned long long poly_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int poly_device_error(int* out, int reset) {
  if (!out) return fail(POLY_EINVAL, "null out");
  int a = 0, b = 0, c = 0, d = 0, e = 0;
  int rc = read_device_error_fwd(&a, reset != 0);
  if (!rc) rc = read_device_error_fwd2(&c, reset != 0);
  if (!rc) rc = read_device_error_bwd(&b, reset != 0);
  if (!rc) rc = read_device_error_dec(&d, reset != 0);
  if (!rc) rc = read_device_error_bwd128(&e, reset != 0);
  *out = a ? a : (c ? c : (b ? b : (d ? d : e)));
  return rc;
}
int poly_selftest_wait_timeout(unsigned long long limit_ns, int* result, void* stream) {
  if (!result) return fail(POLY_EINVAL, "null result");
  if (limit_ns == 0 || limit_ns > 1000000000ull) return fail(POLY_EINVAL, "limit_ns must be in (0, 1e9]");
  return selftest_wait_timeout(limit_ns, result, (cudaStream_t)stream);
}
int poly_abi_version(void) { return POLY_ABI_VERSION; }
size_t poly_sizeof_pass_args(void) { return sizeof(PolyPassArgs); }
size_t poly_sizeof_pass_bwd_args(void) { return sizeof(PolyPassBwdArgs); }
size_t poly_sizeof_merge_args(void) { return sizeof(PolyMergeArgs); }

size_t poly_pass_fwd_workspace_size(const PolyPassArgs* a) {
  if (check_pass(a) != POLY_OK) return 0;
  switch (choose_fwd(*a)) {
    case FwdKind::kDecode: return pass_decode_workspace(*a);
    case FwdKind::kTc: return pass_fwd_tc_workspace(*a);
    default: return 0;
  }
}

const char* poly_pass_fwd_kernel_name(const PolyPassArgs* a) {
  if (check_pass(a) != POLY_OK) return "invalid";
  switch (choose_fwd(*a)) {
    case FwdKind::kDecode: return "decode";
    case FwdKind::kSmall: return "small";
    case FwdKind::kF32: return "tf32x3";
    case FwdKind::kTc: return "tc100";
    default: return "simt";
  }
}

int poly_pass_fwd(const PolyPassArgs* a, void* stream) {
  int rc = check_pass(a);
  if (rc) return rc;
  if (a->seq_q == 0) return POLY_OK;
  const FwdKind kind = choose_fwd(*a);
  if (a->causal_offset && (kind != FwdKind::kTc || !a->causal || (a->causal_offset % 128) != 0))
    return fail(POLY_EUNSUPPORTED, "causal_offset needs causal, a multiple of 128 and the tcgen05 forward "
                                   "(bf16 / fp16, head_dim 64 or 128, no masks, no softclamp)");
  size_t need = 0;
  if (kind == FwdKind::kDecode) need = pass_decode_workspace(*a);
  if (kind == FwdKind::kTc) need = pass_fwd_tc_workspace(*a);
  if (need && (!a->workspace || a->workspace_bytes < need))
    return fail(POLY_EINVAL, "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = (cudaStream_t)stream;
  switch (kind) {
    case FwdKind::kDecode: return launch_pass_decode(*a, s);
    case FwdKind::kSmall: return launch_pass_small(*a, s);
    case FwdKind::kF32: return launch_pass_f32(*a, s);
    case FwdKind::kTc: return launch_pass_fwd_tc(*a, s);
    default: return launch_pass_fwd_simt(*a, s);
  }
}

int poly_head_rmsnorm(const PolyHeadNorm* norms, int n, void* stream) {
  return head_rmsnorm(norms, n, (cudaStream_t)stream);
}

int poly_copy_rows(const PolyRowCopy* copies, int n, void* stream) {
  return copy_rows(copies, n, (cudaStream_t)stream);
}

int poly_decode_chain(const PolyPassArgs* passes, int n, void* stream) {
  if (!passes || n < 0) return fail(POLY_EINVAL, "poly_decode_chain: null passes or negative count");
  for (int i = 0; i < n; ++i) {
    const int rc = check_pass(&passes[i]);
    if (rc) return rc;
    if (passes[i].seq_q != 1 || choose_fwd(passes[i]) != FwdKind::kDecode)
      return fail(POLY_EUNSUPPORTED, "poly_decode_chain: pass " + std::to_string(i) + " does not take the decode kernel");
  }
  for (int i = 0; i < n; ++i) {
    const size_t need = pass_decode_workspace(passes[i]);
    if (need && (!passes[i].workspace || passes[i].workspace_bytes < need))
      return fail(POLY_EINVAL, "poly_decode_chain: pass " + std::to_string(i) + " needs a workspace of " +
                                   std::to_string(need) + " bytes");
  }
  cudaStream_t s = (cudaStream_t)stream;
  for (int i = 0; i < n; ++i) {
    const int rc = launch_pass_decode(passes[i], s, i > 0);
    if (rc) return rc;
  }
  return POLY_OK;
}

size_t poly_pass_bwd_workspace_size(const PolyPassBwdArgs* a) {
  if (!a || check_pass(&a->fwd) != POLY_OK) return 0;
  return use_bwd_tc(*a) ? pass_bwd_tc_workspace(*a) : simt_bwd_workspace(*a);
}

const char* poly_pass_bwd_kernel_name(const PolyPassBwdArgs* a) {
  if (!a || check_pass(&a->fwd) != POLY_OK) return "invalid";
  return use_bwd_tc(*a) ? "tc100" : "simt";
}

int poly_pass_bwd(const PolyPassBwdArgs* a, void* stream) {
  if (!a) return fail(POLY_EINVAL, "null args");
  int rc = check_pass(&a->fwd);
  if (rc) return rc;
  if (a->fwd.v_mul) return fail(POLY_EUNSUPPORTED, "v_mul is forward-only");
  if (a->fwd.causal_offset) return fail(POLY_EUNSUPPORTED, "causal_offset is forward-only");
  if (!a->fwd.lse || !a->dout || !a->dq || !a->dk || !a->dv)
    return fail(POLY_EINVAL, "backward needs fwd.out, fwd.lse, dout, dq, dk and dv");
  const bool tc = use_bwd_tc(*a);
  const size_t need = tc ? pass_bwd_tc_workspace(*a) : simt_bwd_workspace(*a);
  if (need && (!a->workspace || a->workspace_bytes < need))
    return fail(POLY_EINVAL, "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = (cudaStream_t)stream;
  if (a->fwd.seq_q == 0) {
    // no queries: dk, dv and dbias are zero
    const size_t es = a->fwd.dtype == POLY_F32 ? 4 : 2;
    for (int b = 0; b < a->fwd.batch; ++b)
      for (int h = 0; h < a->fwd.kv_heads; ++h) {
        char* dk = (char*)a->dk + (b * a->dk_stride[0] + h * a->dk_stride[1]) * es;
        char* dv = (char*)a->dv + (b * a->dv_stride[0] + h * a->dv_stride[1]) * es;
        rc = cuda_status(cudaMemset2DAsync(dk, a->dk_stride[2] * es, 0, a->fwd.head_dim * es, a->fwd.seq_k, s), "memset dk");
        if (rc) return rc;
        rc = cuda_status(cudaMemset2DAsync(dv, a->dv_stride[2] * es, 0, a->fwd.head_dim * es, a->fwd.seq_k, s), "memset dv");
        if (rc) return rc;
        if (a->dbias) {
          rc = cuda_status(cudaMemsetAsync(a->dbias + b * a->dbias_stride[0] + h * a->dbias_stride[1], 0,
                                           a->fwd.seq_k * sizeof(float), s), "memset dbias");
          if (rc) return rc;
        }
      }
    return POLY_OK;
  }
  return tc ? launch_pass_bwd_tc(*a, s) : launch_pass_bwd_simt(*a, s);
}

int poly_lse_merge(const PolyMergeArgs* a, void* stream) {
  if (!a) return fail(POLY_EINVAL, "null args");
  if (a->parts <= 0 || a->head_dim <= 0 || a->rows < 0) return fail(POLY_EINVAL, "bad merge sizes");
  if (!a->part_out || !a->part_lse || !a->out) return fail(POLY_EINVAL, "merge needs part_out, part_lse and out");
  if (a->dtype != POLY_F32 && a->dtype != POLY_F16 && a->dtype != POLY_BF16) return fail(POLY_EINVAL, "unknown dtype");
  if (a->rows == 0) return POLY_OK;
  return launch_lse_merge(*a, (cudaStream_t)stream);
}

}  // extern "C"
