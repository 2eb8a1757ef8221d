/*
 * poly_attention.h -- C ABI of libpolyattn.so, the B200 (sm_100a) poly-attention
 * hot path.
 *
 * Every entry point is stream-ordered (it only enqueues work on `stream`, a
 * cudaStream_t passed as void*), allocates no device memory, keeps no
 * per-call state, and returns one of the POLY_* status codes below. On a
 * non-zero status, poly_last_error() returns a message for the calling thread.
 *
 * Layout convention for every tensor argument: element strides are given for
 * the (batch, head, row) axes; the last (feature) axis is contiguous. Score
 * rows are queries i, columns are keys j. Grouped-query attention: query head
 * h reads key/value head h / (heads / kv_heads).
 *
 * Reference interfaces replaced (lucidrains/poly-attention 0.3.6):
 *   poly_pass_fwd  <- _poly_flash_fwd_kernel launch
 *                     (poly_attention/flash_poly_attention.py:21-154, launched
 *                     at :347-359 for pass 1 and :365-377 for pass 2), and the
 *                     materialised passes of reference_poly_attention
 *                     (poly_attention/poly_attention.py:63-114) incl. masks
 *   poly_pass_bwd  <- _poly_flash_bwd_kernel launch
 *                     (poly_attention/flash_poly_attention.py:164-316, launched
 *                     at :409-422 and :429-442) plus the dq2 sum at :444
 *   poly_lse_merge <- no counterpart: merges key-split partial passes (the
 *                     long-context sequence split across GPUs)
 *   poly_decode_chain <- the cached passes of one decoding step, run level
 *                     after level (poly_attention/n_poly_attention.py:263-313,
 *                     poly_attention/poly_attention.py:63-114 with cache)
 */
#ifndef POLY_ATTENTION_H_
#define POLY_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define POLY_ABI_VERSION 2

#if defined(__GNUC__)
#define POLY_API __attribute__((visibility("default")))
#else
#define POLY_API
#endif

/* status codes */
#define POLY_OK 0
#define POLY_EINVAL 1        /* bad shape, stride, dtype or pointer */
#define POLY_EUNSUPPORTED 2  /* valid request this build has no kernel for */
#define POLY_ECUDA 3         /* a CUDA call failed (launch, attribute, driver) */

/* element types */
#define POLY_F32 0
#define POLY_F16 1
#define POLY_BF16 2

/*
 * One attention pass with an additive per-key bias, emitting per-row
 * log-sum-exp. Both passes of order-2 poly attention and every level of the
 * order-n chain are instances of it:
 *
 *   s_ij  = scale * q_i . k_j ; if softclamp > 0: s_ij = c * tanh(s_ij / c)
 *   masked (causal j > i, key_mask[j] == 0, query_mask[i] == 0) -> excluded
 *   s_ij += bias_j
 *   out_i = softmax_j(s_ij) v_j ,  lse_i = logsumexp_j s_ij
 *
 * A row whose every entry is excluded gets the reference's value for it: the
 * uniform average of v over its keys (all keys except those both masked and
 * "dead", i.e. with bias <= -FLT_MAX/2, where the reference overflows to
 * -inf), lse = -FLT_MAX.
 *
 * Optional value multiplier (forward only): if v_mul != NULL the pass uses
 * v_j * v_mul_j as its values, so a decode step reads the order-n chain's
 * V' = v_k * msg (n_poly_attention.py:287) from the two cached tensors.
 *
 * Optional fused epilogue for the order-n chain (V' = v_k * msg,
 * n_poly_attention.py:287): if epi_out != NULL, epi_out_i = epi_mul_i * out_i is
 * written as well (same shape as out; epi_mul rows indexed like out rows).
 */
typedef struct PolyPassArgs {
  int32_t batch;
  int32_t heads;      /* query heads (q, out, lse, query-side) */
  int32_t kv_heads;   /* key/value heads (k, v, bias); divides heads */
  int32_t seq_q;
  int32_t seq_k;
  int32_t head_dim;   /* q/k/v/out feature size */
  int32_t dtype;      /* POLY_F32 / POLY_F16 / POLY_BF16 for q, k, v, out, epi_mul, epi_out */
  int32_t causal;     /* 1: key j visible to query i iff j <= i (top-left aligned) */
  float scale;        /* usually head_dim ** -0.5 */
  float softclamp;    /* > 0 enables c * tanh(s / c) */

  const void* q;        int64_t q_stride[3];     /* [batch, heads, seq_q, d]      */
  const void* k;        int64_t k_stride[3];     /* [batch, kv_heads, seq_k, d]   */
  const void* v;        int64_t v_stride[3];     /* [batch, kv_heads, seq_k, d]   */
  const void* v_mul;    int64_t v_mul_stride[3]; /* [batch, kv_heads, seq_k, d] | NULL: v_j *= v_mul_j */
  const float* bias;    int64_t bias_stride[2];  /* [batch, kv_heads, seq_k] | NULL */
  const uint8_t* key_mask;   int64_t key_mask_stride;    /* [batch, seq_k] | NULL, 0 = masked */
  const uint8_t* query_mask; int64_t query_mask_stride;  /* [batch, seq_q] | NULL, 0 = masked */
  void* out;            int64_t out_stride[3];   /* [batch, heads, seq_q, d]      */
  float* lse;           int64_t lse_stride[2];   /* [batch, heads, seq_q] | NULL  */
  const void* epi_mul;     int64_t epi_mul_stride[3];  /* [batch, heads, seq_q, d] | NULL */
  void* epi_out;           int64_t epi_out_stride[3];  /* [batch, heads, seq_q, d] | NULL */

  void* workspace;          /* device scratch, >= poly_pass_fwd_workspace_size() bytes */
  size_t workspace_bytes;

  /* With causal: key j visible to query i iff j <= i + causal_offset, i.e. the
   * queries are rows [causal_offset, causal_offset + seq_q) of a longer
   * sequence whose first seq_k keys are given (no counterpart in the
   * reference: it lets one launch cover a sequence shard's queries against
   * all earlier keys). 0 is the reference's top-left causal mask. Non-zero
   * values must be multiples of 128 and are taken by the tcgen05 forward only
   * (bf16 / fp16, head_dim 64 or 128, no masks, no softclamp); elsewhere
   * POLY_EUNSUPPORTED. Negative: POLY_EINVAL. */
  int32_t causal_offset;
  int32_t reserved_;
} PolyPassArgs;

/*
 * Backward of one pass (recomputes the scores from q, k and lse):
 *   dv_j   = sum_i p_ij dout_i
 *   ds_ij  = p_ij (dout_i . v_j - dout_i . out_i + dlse_i)
 *   dbias_j = sum_i ds_ij               (includes masked entries, as autograd does)
 *   dz_ij  = ds_ij (1 - tanh^2) on kept entries, 0 on masked ones
 *   dq_i   = scale sum_j dz_ij k_j ,   dk_j = scale sum_i dz_ij q_i
 * With GQA, dk / dv / dbias sum over the query heads of each group.
 * If dq_accumulate != 0, dq += result (used for dq2 = part1 + part2,
 * poly_attention/flash_poly_attention.py:444); otherwise dq = result.
 */
typedef struct PolyPassBwdArgs {
  PolyPassArgs fwd;         /* the forward's inputs; fwd.out and fwd.lse are required */
  const void* dout;     int64_t dout_stride[3];  /* [batch, heads, seq_q, d]    */
  const float* dlse;    int64_t dlse_stride[2];  /* [batch, heads, seq_q] | NULL */
  void* dq;             int64_t dq_stride[3];    /* [batch, heads, seq_q, d]    */
  void* dk;             int64_t dk_stride[3];    /* [batch, kv_heads, seq_k, d] */
  void* dv;             int64_t dv_stride[3];    /* [batch, kv_heads, seq_k, d] */
  float* dbias;         int64_t dbias_stride[2]; /* [batch, kv_heads, seq_k] | NULL */
  int32_t dq_accumulate;
  int32_t reserved;
  void* workspace;          /* >= poly_pass_bwd_workspace_size() bytes */
  size_t workspace_bytes;
} PolyPassBwdArgs;

/*
 * Merge P partial passes over disjoint key shards of the same queries:
 *   lse_i = logsumexp_p lse_p,i ;  out_i = sum_p exp(lse_p,i - lse_i) out_p,i
 * part_out: [P][rows][d] (dtype), part_lse: [P][rows] fp32, rows = batch*heads*seq_q
 * flattened contiguously; out: [rows][d] (dtype); lse: [rows] fp32 (may be NULL).
 */
typedef struct PolyMergeArgs {
  int32_t parts;
  int32_t head_dim;
  int32_t dtype;
  int32_t reserved;
  int64_t rows;
  const void* part_out;
  const float* part_lse;
  void* out;
  float* lse;
} PolyMergeArgs;

POLY_API int poly_pass_fwd(const PolyPassArgs* args, void* stream);
POLY_API size_t poly_pass_fwd_workspace_size(const PolyPassArgs* args);

POLY_API int poly_pass_bwd(const PolyPassBwdArgs* args, void* stream);
POLY_API size_t poly_pass_bwd_workspace_size(const PolyPassBwdArgs* args);

POLY_API int poly_lse_merge(const PolyMergeArgs* args, void* stream);

/*
 * The n passes of one KV-cache decoding step of the order-n chain, in order,
 * in one call. Contract: passes[i + 1] reads what passes[i] wrote only in the
 * LAST key row (row seq_k - 1, the row the step appended) of its v, v_mul and
 * bias; every other input is complete when the call is made (stream order);
 * no pass writes what an earlier pass of the list reads. Under it, each pass
 * after the first is launched as a programmatic dependent of the previous one:
 * its CTAs start while the previous pass drains, stream every key tile but the
 * last, and wait for the previous pass before loading the last. Every pass
 * must take the decode kernel (poly_pass_fwd_kernel_name() == "decode"), else
 * POLY_EUNSUPPORTED and nothing is launched. A pass with few (batch, kv head)
 * groups needs a workspace of poly_pass_fwd_workspace_size() bytes (0 otherwise);
 * a pass given too little gets POLY_EINVAL and nothing is launched.
 */
POLY_API int poly_decode_chain(const PolyPassArgs* passes, int n, void* stream);

/*
 * Row copies for KV-cache appends (replaces the reference's per-step
 * torch.cat cache growth, poly_attention/poly_attention.py:283-287 and
 * n_poly_attention.py:206-207, 281-302, by in-place writes of the new rows).
 * Copy i moves outer x inner rows of row_bytes bytes; row (o, i) starts at
 * src + o * src_stride[0] + i * src_stride[1] (same for dst). All n <= 16
 * copies run in ONE kernel launch. Pointers, strides and row_bytes must be
 * multiples of 16 bytes, else POLY_EINVAL.
 */
#define POLY_MAX_ROW_COPIES 16
typedef struct {
  const void* src;
  void* dst;
  int32_t outer;
  int32_t inner;
  int32_t row_bytes;
  int32_t reserved;
  int64_t src_stride[2]; /* bytes */
  int64_t dst_stride[2]; /* bytes */
} PolyRowCopy;

POLY_API int poly_copy_rows(const PolyRowCopy* copies, int n, void* stream);

/*
 * Per-head RMSNorm of query/key tensors straight from the head-split view of a
 * projection output (replaces q_norms, poly_attention/poly_attention.py:272,
 * n_poly_attention.py:186-187, and the contiguous copy torch makes of the
 * strided view first): dst = src * rsqrt(mean(src^2) + eps) * weight over the
 * last dim, fp32 arithmetic. src [batch, heads, rows, dim] with element
 * strides (batch, head, row), last dim contiguous; dst contiguous, in
 * dst_dtype (src's dtype, or F32 inside autocast). weight [dim] in
 * weight_dtype. dim <= 256, dim % 8 == 0, 16-byte aligned rows. All n <= 4
 * tensors are normalised in ONE kernel launch.
 */
#define POLY_MAX_NORMS 4
typedef struct {
  const void* src;
  void* dst;
  const void* weight;
  int32_t batch;
  int32_t heads;
  int32_t rows;
  int32_t dim;
  int64_t src_stride[3]; /* elements: batch, head, row */
  int32_t src_dtype;     /* POLY_F32 / POLY_F16 / POLY_BF16 */
  int32_t dst_dtype;
  int32_t weight_dtype;
  float eps;
} PolyHeadNorm;

POLY_API int poly_head_rmsnorm(const PolyHeadNorm* norms, int n, void* stream);

/*
 * poly_pass_bwd without a caller workspace. No counterpart in the reference:
 * it exists for callers that cannot allocate device memory (FFI hosts that
 * only pass existing buffers, processes whose device memory another
 * allocator has fully planned). Scratch comes from an 8 MiB array built into
 * the library (held per GPU until exit); larger problems get POLY_EINVAL.
 * All calls on a device share that array: calls overlapping on the GPU race.
 * Every call outside stream capture resolves the array's address afresh
 * (a device reset leaves no stale address); a call during capture reuses the
 * last one, so make the first call on a device before any stream capture.
 * args->workspace is ignored.
 */
POLY_API int poly_pass_bwd_noalloc(const PolyPassBwdArgs* args, void* stream);
POLY_API size_t poly_noalloc_scratch_bytes(void);

/* Name of the kernel family poly_pass_fwd / poly_pass_bwd would launch for
 * these arguments: forward "decode" (one query row against a cache), "small"
 * (short sequences, mma.sync), "tf32x3" (fp32 on tensor cores), "tc100"
 * (tcgen05) or "simt" (CUDA cores); backward "tc100" or "simt"; "invalid"
 * when the arguments fail validation. */
POLY_API const char* poly_pass_fwd_kernel_name(const PolyPassArgs* args);
POLY_API const char* poly_pass_bwd_kernel_name(const PolyPassBwdArgs* args);

/* Last error message of the calling thread ("" if none). */
POLY_API const char* poly_last_error(void);

/* Number of kernels this library has launched in this process. */
POLY_API unsigned long long poly_launch_count(void);

/* Device error word of the current device (synchronous read): non-zero if a
 * kernel's bounded wait gave up since the last reset: 1 | site << 8, the
 * first give-up wins. The launch that gave up freed its resources and
 * returned; the outputs of that call are undefined. Other CTAs of the same
 * launch give up at once; later launches run normally whether or not the
 * word has been reset. reset != 0 clears the word. */
POLY_API int poly_device_error(int* out, int reset);

/* Diagnostics, no counterpart in the reference: launches one CTA that holds
 * TMEM and waits on a barrier nothing arrives on, with a wait limit of
 * limit_ns (0 < limit_ns <= 1e9), so the bounded-wait give-up path runs:
 * *result (device int) becomes 2 once the wait gave up and the CTA freed its
 * TMEM and returned (1 if the wait wrongly succeeded); the device error word
 * then reads 1 | 99 << 8. */
POLY_API int poly_selftest_wait_timeout(unsigned long long limit_ns, int* result, void* stream);

/* ABI checks for bindings: POLY_ABI_VERSION and the struct sizes. */
POLY_API int poly_abi_version(void);
POLY_API size_t poly_sizeof_pass_args(void);
POLY_API size_t poly_sizeof_pass_bwd_args(void);
POLY_API size_t poly_sizeof_merge_args(void);

#ifdef __cplusplus
}
#endif

#endif /* POLY_ATTENTION_H_ */
