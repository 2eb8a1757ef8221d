// CUDA-core (FFMA) implementation of one poly-attention pass, forward and
// backward. It serves fp32 inputs (whose 1e-4 tolerance tcgen05's TF32 mode
// cannot meet), head sizes the tensor-core kernels do not take, and masked
// inputs. fp32 accumulation throughout.
//
// Follows the per-pass semantics of reference_poly_attention
// (poly_attention/poly_attention.py:63-114): softclamp, causal triu(1), key
// mask, query mask, then the additive per-key bias; a fully excluded row is the
// uniform average over all keys (the -finfo.max masking of :68).
#include "common.cuh"

namespace poly {
namespace {

constexpr int kWarps = 8;   // rows per CTA (one warp per row)
constexpr int kTile = 32;   // keys (or queries) per smem tile: one per lane

struct RowCtx {
  int b, h, kvh;
};

__device__ __forceinline__ RowCtx bh_ctx(int bh, int heads, int kv_heads) {
  RowCtx c;
  c.b = bh / heads;
  c.h = bh - c.b * heads;
  c.kvh = c.h / (heads / kv_heads);
  return c;
}

// Loads rows [r0, r0 + kTile) of a [rows, d] slice into smem as fp32 with a
// padded row stride (DMAX + 1) so lane-per-row dot products are conflict-free.
template <typename T, int DMAX>
__device__ __forceinline__ void load_tile(float (*dst)[DMAX + 1], const T* base, int64_t row_stride,
                                          int r0, int rows, int d) {
  for (int idx = threadIdx.x; idx < kTile * DMAX; idx += blockDim.x) {
    int r = idx / DMAX, c = idx - r * DMAX;
    float v = 0.f;
    if (r0 + r < rows && c < d) v = to_f32(base[(int64_t)(r0 + r) * row_stride + c]);
    dst[r][c] = v;
  }
}

// In a fully excluded row, does key j take part in the reference's uniform
// average? Yes unless it is masked (causal / key / query) and dead at once.
__device__ __forceinline__ bool fallback_key(const PolyPassArgs& a, int i, int j, bool q_masked,
                                             const uint8_t* km, const float* bias, int seq_k) {
  const bool masked = q_masked || (a.causal && j > i) || (km && km[j] == 0);
  const bool dead = bias && bias[j] <= kDeadBias;
  return !(masked && dead);
}

template <typename T, int DMAX>
__global__ void __launch_bounds__(kWarps * 32) pass_fwd_simt_kernel(const PolyPassArgs a) {
  constexpr int NT = DMAX / 32;
  __shared__ float Ks[kTile][DMAX + 1];
  __shared__ float Vs[kTile][DMAX + 1];
  __shared__ float Qs[kWarps][DMAX];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const RowCtx c = bh_ctx(blockIdx.y, a.heads, a.kv_heads);
  const int row0 = blockIdx.x * kWarps;
  const int i = row0 + warp;
  const int d = a.head_dim;
  const bool row_ok = i < a.seq_q;

  const T* q = (const T*)a.q + c.b * a.q_stride[0] + c.h * a.q_stride[1];
  const T* k = (const T*)a.k + c.b * a.k_stride[0] + c.kvh * a.k_stride[1];
  const T* v = (const T*)a.v + c.b * a.v_stride[0] + c.kvh * a.v_stride[1];
  const T* vmk = a.v_mul ? (const T*)a.v_mul + c.b * a.v_mul_stride[0] + c.kvh * a.v_mul_stride[1] : nullptr;
  const float* bias = a.bias ? a.bias + c.b * a.bias_stride[0] + c.kvh * a.bias_stride[1] : nullptr;
  const uint8_t* km = a.key_mask ? a.key_mask + c.b * a.key_mask_stride : nullptr;
  const bool q_masked = row_ok && a.query_mask && a.query_mask[c.b * a.query_mask_stride + i] == 0;

  for (int t = lane; t < DMAX; t += 32) Qs[warp][t] = (row_ok && t < d) ? to_f32(q[(int64_t)i * a.q_stride[2] + t]) : 0.f;

  float m = -INFINITY, l = 0.f, acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;

  const int kend = a.causal ? min(a.seq_k, row0 + kWarps) : a.seq_k;
  const float sl2 = a.scale;
  for (int j0 = 0; j0 < kend; j0 += kTile) {
    __syncthreads();
    load_tile<T, DMAX>(Ks, k, a.k_stride[2], j0, a.seq_k, d);
    load_tile<T, DMAX>(Vs, v, a.v_stride[2], j0, a.seq_k, d);
    if (vmk) {
      __syncthreads();
      for (int idx = threadIdx.x; idx < kTile * DMAX; idx += blockDim.x) {
        const int r = idx / DMAX, cc = idx - r * DMAX;
        if (j0 + r < a.seq_k && cc < d) Vs[r][cc] = to_f32(from_f32<T>(Vs[r][cc] * to_f32(vmk[(int64_t)(j0 + r) * a.v_mul_stride[2] + cc])));
      }
    }
    __syncthreads();
    if (!row_ok) continue;
    const int j = j0 + lane;
    float s = 0.f;
#pragma unroll 8
    for (int t = 0; t < DMAX; ++t) s = fmaf(Qs[warp][t], Ks[lane][t], s);
    s *= sl2;
    if (a.softclamp > 0.f) s = a.softclamp * tanhf(s / a.softclamp);
    bool keep = j < a.seq_k && !q_masked && (!a.causal || j <= i) && (!km || km[j] != 0);
    if (keep && bias) {
      float bj = bias[j];
      if (bj <= kDeadBias) keep = false;
      s += bj;
    }
    s = keep ? s : -INFINITY;
    const float mn = fmaxf(m, warp_max(s));
    if (mn == -INFINITY) continue;
    const float p = keep ? exp2f((s - mn) * kLog2e) : 0.f;
    const float alpha = exp2f((m - mn) * kLog2e);
    l = l * alpha + warp_sum(p);
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] *= alpha;
#pragma unroll 4
    for (int jj = 0; jj < kTile; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = fmaf(pj, Vs[jj][lane + 32 * t], acc[t]);
    }
    m = mn;
  }
  if (!row_ok) return;

  float lse;
  if (m == -INFINITY) {
    // Every entry excluded: the reference's -finfo.max fill makes the row a
    // uniform average over its keys, except keys that are both masked and
    // dead (-max + -max overflows to -inf there).
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    int count = 0;
    for (int j = 0; j < a.seq_k; ++j) {
      if (!fallback_key(a, i, j, q_masked, km, bias, a.seq_k)) continue;
      ++count;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int col = lane + 32 * t;
        if (col < d) {
          float vv = to_f32(v[(int64_t)j * a.v_stride[2] + col]);
          if (vmk) vv = to_f32(from_f32<T>(vv * to_f32(vmk[(int64_t)j * a.v_mul_stride[2] + col])));
          acc[t] += vv;
        }
      }
    }
    const float inv = count ? 1.f / (float)count : 0.f;
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] *= inv;
    lse = -FLT_MAX;
  } else {
    const float inv = 1.f / l;
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] *= inv;
    lse = m + logf(l);
  }

  T* out = (T*)a.out + c.b * a.out_stride[0] + c.h * a.out_stride[1] + (int64_t)i * a.out_stride[2];
  const T* vm = a.epi_out ? (const T*)a.epi_mul + c.b * a.epi_mul_stride[0] + c.h * a.epi_mul_stride[1] + (int64_t)i * a.epi_mul_stride[2] : nullptr;
  T* vo = a.epi_out ? (T*)a.epi_out + c.b * a.epi_out_stride[0] + c.h * a.epi_out_stride[1] + (int64_t)i * a.epi_out_stride[2] : nullptr;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int col = lane + 32 * t;
    if (col < d) {
      const T o = from_f32<T>(acc[t]);
      out[col] = o;
      if (vo) vo[col] = from_f32<T>(to_f32(vm[col]) * to_f32(o));
    }
  }
  if (a.lse && lane == 0) a.lse[c.b * a.lse_stride[0] + c.h * a.lse_stride[1] + i] = lse;
}

// delta_i = dout_i . out_i - dlse_i  (the row term of ds; dlse folds in the
// log-sum-exp gradient, poly_attention/flash_poly_attention.py:280-284)
template <typename T>
__global__ void bwd_delta_kernel(const PolyPassBwdArgs a, float* delta, int* fb_count) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int rows = a.fwd.batch * a.fwd.heads * a.fwd.seq_q;
  if (warp >= rows) return;
  const int i = warp % a.fwd.seq_q, bh = warp / a.fwd.seq_q;
  const int b = bh / a.fwd.heads, h = bh - b * a.fwd.heads;
  const T* o = (const T*)a.fwd.out + b * a.fwd.out_stride[0] + h * a.fwd.out_stride[1] + (int64_t)i * a.fwd.out_stride[2];
  const T* g = (const T*)a.dout + b * a.dout_stride[0] + h * a.dout_stride[1] + (int64_t)i * a.dout_stride[2];
  float s = 0.f;
  for (int t = lane; t < a.fwd.head_dim; t += 32) s += to_f32(o[t]) * to_f32(g[t]);
  s = warp_sum(s);
  const float lse_i = a.fwd.lse[b * a.fwd.lse_stride[0] + h * a.fwd.lse_stride[1] + i];
  int count = 0;
  if (lse_i <= kDeadBias) {
    const int kvh = h / (a.fwd.heads / a.fwd.kv_heads);
    const float* bias = a.fwd.bias ? a.fwd.bias + b * a.fwd.bias_stride[0] + kvh * a.fwd.bias_stride[1] : nullptr;
    const uint8_t* km = a.fwd.key_mask ? a.fwd.key_mask + b * a.fwd.key_mask_stride : nullptr;
    const bool qm = a.fwd.query_mask && a.fwd.query_mask[b * a.fwd.query_mask_stride + i] == 0;
    for (int j = lane; j < a.fwd.seq_k; j += 32) count += fallback_key(a.fwd, i, j, qm, km, bias, a.fwd.seq_k);
    for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xffffffffu, count, o);
  }
  if (lane == 0) {
    if (a.dlse) s -= a.dlse[b * a.dlse_stride[0] + h * a.dlse_stride[1] + i];
    delta[warp] = s;
    fb_count[warp] = count;
  }
}

// Entry term shared by both backward kernels. Returns p (probability) and the
// softclamp derivative factor; `keep` says whether the score itself is live.
struct Entry {
  float p, dfac;
  bool keep;
};

__device__ __forceinline__ Entry bwd_entry(const PolyPassArgs& a, float dot, int i, int j, bool q_masked,
                                           bool k_masked, const float* bias, float lse_i, int fb_count) {
  Entry e;
  float s = dot * a.scale;
  e.dfac = 1.f;
  if (a.softclamp > 0.f) {
    const float th = tanhf(s / a.softclamp);
    s = a.softclamp * th;
    e.dfac = 1.f - th * th;
  }
  e.keep = j < a.seq_k && i < a.seq_q && !q_masked && !k_masked && (!a.causal || j <= i);
  float bj = 0.f;
  if (e.keep && bias) {
    bj = bias[j];
    if (bj <= kDeadBias) e.keep = false;
  }
  if (i >= a.seq_q || j >= a.seq_k) {
    e.p = 0.f;
  } else if (lse_i <= kDeadBias) {
    // fully excluded row: the reference's uniform average (see fallback_key)
    const bool masked = q_masked || k_masked || (a.causal && j > i);
    const bool dead = bias && bias[j] <= kDeadBias;
    e.p = (!(masked && dead) && fb_count > 0) ? 1.f / (float)fb_count : 0.f;
    // unmasked entries (dead only) still pass gradient to their score, as
    // autograd through the reference's masked_fill + add does
    e.keep = !masked;
  } else {
    e.p = e.keep ? exp2f((s + bj - lse_i) * kLog2e) : 0.f;
  }
  return e;
}

template <typename T, int DMAX>
__global__ void __launch_bounds__(kWarps * 32) pass_bwd_dq_simt_kernel(const PolyPassBwdArgs ab, const float* delta, const int* fb_count) {
  constexpr int NT = DMAX / 32;
  const PolyPassArgs& a = ab.fwd;
  __shared__ float Ks[kTile][DMAX + 1];
  __shared__ float Vs[kTile][DMAX + 1];
  __shared__ float Qs[kWarps][DMAX];
  __shared__ float Gs[kWarps][DMAX];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const RowCtx c = bh_ctx(blockIdx.y, a.heads, a.kv_heads);
  const int row0 = blockIdx.x * kWarps, i = row0 + warp, d = a.head_dim;
  const bool row_ok = i < a.seq_q;
  const T* q = (const T*)a.q + c.b * a.q_stride[0] + c.h * a.q_stride[1];
  const T* g = (const T*)ab.dout + c.b * ab.dout_stride[0] + c.h * ab.dout_stride[1];
  const T* k = (const T*)a.k + c.b * a.k_stride[0] + c.kvh * a.k_stride[1];
  const T* v = (const T*)a.v + c.b * a.v_stride[0] + c.kvh * a.v_stride[1];
  const float* bias = a.bias ? a.bias + c.b * a.bias_stride[0] + c.kvh * a.bias_stride[1] : nullptr;
  const uint8_t* km = a.key_mask ? a.key_mask + c.b * a.key_mask_stride : nullptr;
  const bool q_masked = row_ok && a.query_mask && a.query_mask[c.b * a.query_mask_stride + i] == 0;
  for (int t = lane; t < DMAX; t += 32) {
    Qs[warp][t] = (row_ok && t < d) ? to_f32(q[(int64_t)i * a.q_stride[2] + t]) : 0.f;
    Gs[warp][t] = (row_ok && t < d) ? to_f32(g[(int64_t)i * ab.dout_stride[2] + t]) : 0.f;
  }
  const float lse_i = row_ok ? a.lse[c.b * a.lse_stride[0] + c.h * a.lse_stride[1] + i] : 0.f;
  const float del = row_ok ? delta[((int64_t)blockIdx.y * a.seq_q) + i] : 0.f;
  const int fbc = row_ok ? fb_count[((int64_t)blockIdx.y * a.seq_q) + i] : 0;
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  const int kend = a.causal ? min(a.seq_k, row0 + kWarps) : a.seq_k;
  for (int j0 = 0; j0 < kend; j0 += kTile) {
    __syncthreads();
    load_tile<T, DMAX>(Ks, k, a.k_stride[2], j0, a.seq_k, d);
    load_tile<T, DMAX>(Vs, v, a.v_stride[2], j0, a.seq_k, d);
    __syncthreads();
    if (!row_ok) continue;
    const int j = j0 + lane;
    float dot = 0.f, dp = 0.f;
#pragma unroll 8
    for (int t = 0; t < DMAX; ++t) {
      dot = fmaf(Qs[warp][t], Ks[lane][t], dot);
      dp = fmaf(Gs[warp][t], Vs[lane][t], dp);
    }
    const bool k_masked = km && j < a.seq_k && km[j] == 0;
    const Entry e = bwd_entry(a, dot, i, j, q_masked, k_masked, bias, lse_i, fbc);
    const float dz = e.keep ? e.p * (dp - del) * e.dfac : 0.f;
#pragma unroll 4
    for (int jj = 0; jj < kTile; ++jj) {
      const float z = __shfl_sync(0xffffffffu, dz, jj);
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = fmaf(z, Ks[jj][lane + 32 * t], acc[t]);
    }
  }
  if (!row_ok) return;
  T* dq = (T*)ab.dq + c.b * ab.dq_stride[0] + c.h * ab.dq_stride[1] + (int64_t)i * ab.dq_stride[2];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int col = lane + 32 * t;
    if (col < d) {
      float r = acc[t] * a.scale;
      if (ab.dq_accumulate) r += to_f32(dq[col]);
      dq[col] = from_f32<T>(r);
    }
  }
}

template <typename T, int DMAX>
__global__ void __launch_bounds__(kWarps * 32) pass_bwd_dkv_simt_kernel(const PolyPassBwdArgs ab, const float* delta, const int* fb_count) {
  constexpr int NT = DMAX / 32;
  const PolyPassArgs& a = ab.fwd;
  __shared__ float Qt[kTile][DMAX + 1];
  __shared__ float Gt[kTile][DMAX + 1];
  __shared__ float Kr[kWarps][DMAX];
  __shared__ float Vr[kWarps][DMAX];
  __shared__ float lse_t[kTile], del_t[kTile];
  __shared__ uint8_t qm_t[kTile];
  __shared__ int fb_t[kTile];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y / a.kv_heads, kvh = blockIdx.y - b * a.kv_heads;
  const int rep = a.heads / a.kv_heads;
  const int row0 = blockIdx.x * kWarps, j = row0 + warp, d = a.head_dim;
  const bool row_ok = j < a.seq_k;
  const T* k = (const T*)a.k + b * a.k_stride[0] + kvh * a.k_stride[1];
  const T* v = (const T*)a.v + b * a.v_stride[0] + kvh * a.v_stride[1];
  const float* bias = a.bias ? a.bias + b * a.bias_stride[0] + kvh * a.bias_stride[1] : nullptr;
  const bool k_masked = row_ok && a.key_mask && a.key_mask[b * a.key_mask_stride + j] == 0;
  for (int t = lane; t < DMAX; t += 32) {
    Kr[warp][t] = (row_ok && t < d) ? to_f32(k[(int64_t)j * a.k_stride[2] + t]) : 0.f;
    Vr[warp][t] = (row_ok && t < d) ? to_f32(v[(int64_t)j * a.v_stride[2] + t]) : 0.f;
  }
  float dk[NT], dv[NT], db = 0.f;
#pragma unroll
  for (int t = 0; t < NT; ++t) dk[t] = dv[t] = 0.f;
  const bool may_dead = a.key_mask || a.query_mask || a.bias;
  const int istart = (a.causal && !may_dead) ? row0 : 0;
  for (int hr = 0; hr < rep; ++hr) {
    const int h = kvh * rep + hr;
    const T* q = (const T*)a.q + b * a.q_stride[0] + h * a.q_stride[1];
    const T* g = (const T*)ab.dout + b * ab.dout_stride[0] + h * ab.dout_stride[1];
    for (int i0 = istart; i0 < a.seq_q; i0 += kTile) {
      __syncthreads();
      load_tile<T, DMAX>(Qt, q, a.q_stride[2], i0, a.seq_q, d);
      load_tile<T, DMAX>(Gt, g, ab.dout_stride[2], i0, a.seq_q, d);
      if (threadIdx.x < kTile) {
        const int ii = i0 + threadIdx.x;
        const bool ok = ii < a.seq_q;
        lse_t[threadIdx.x] = ok ? a.lse[b * a.lse_stride[0] + h * a.lse_stride[1] + ii] : 0.f;
        del_t[threadIdx.x] = ok ? delta[((int64_t)(b * a.heads + h) * a.seq_q) + ii] : 0.f;
        fb_t[threadIdx.x] = ok ? fb_count[((int64_t)(b * a.heads + h) * a.seq_q) + ii] : 0;
        qm_t[threadIdx.x] = (ok && a.query_mask) ? (a.query_mask[b * a.query_mask_stride + ii] == 0) : 0;
      }
      __syncthreads();
      if (!row_ok) continue;
      const int i = i0 + lane;
      float dot = 0.f, dp = 0.f;
#pragma unroll 8
      for (int t = 0; t < DMAX; ++t) {
        dot = fmaf(Qt[lane][t], Kr[warp][t], dot);
        dp = fmaf(Gt[lane][t], Vr[warp][t], dp);
      }
      const Entry e = bwd_entry(a, dot, i, j, qm_t[lane] != 0, k_masked, bias, lse_t[lane], fb_t[lane]);
      const float ds = e.p * (dp - del_t[lane]);
      db += (i < a.seq_q) ? ds : 0.f;
      const float dz = e.keep ? ds * e.dfac : 0.f;
#pragma unroll 4
      for (int ii = 0; ii < kTile; ++ii) {
        const float pz = __shfl_sync(0xffffffffu, e.p, ii);
        const float zz = __shfl_sync(0xffffffffu, dz, ii);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          dv[t] = fmaf(pz, Gt[ii][lane + 32 * t], dv[t]);
          dk[t] = fmaf(zz, Qt[ii][lane + 32 * t], dk[t]);
        }
      }
    }
  }
  if (!row_ok) return;
  db = warp_sum(db);
  T* dkp = (T*)ab.dk + b * ab.dk_stride[0] + kvh * ab.dk_stride[1] + (int64_t)j * ab.dk_stride[2];
  T* dvp = (T*)ab.dv + b * ab.dv_stride[0] + kvh * ab.dv_stride[1] + (int64_t)j * ab.dv_stride[2];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int col = lane + 32 * t;
    if (col < d) {
      dkp[col] = from_f32<T>(dk[t] * a.scale);
      dvp[col] = from_f32<T>(dv[t]);
    }
  }
  if (ab.dbias && lane == 0) ab.dbias[b * ab.dbias_stride[0] + kvh * ab.dbias_stride[1] + j] = db;
}

template <typename T, int DMAX>
int launch_fwd_t(const PolyPassArgs& a, cudaStream_t s) {
  dim3 grid((a.seq_q + kWarps - 1) / kWarps, a.batch * a.heads);
  pass_fwd_simt_kernel<T, DMAX><<<grid, kWarps * 32, 0, s>>>(a);
  note_launch(1);
  return cuda_status(cudaGetLastError(), "pass_fwd_simt launch");
}

template <typename T, int DMAX>
int launch_bwd_t(const PolyPassBwdArgs& a, cudaStream_t s) {
  const int rows = a.fwd.batch * a.fwd.heads * a.fwd.seq_q;
  float* delta = (float*)a.workspace;
  int* fb_count = (int*)(delta + rows);
  bwd_delta_kernel<T><<<(rows + 7) / 8, 256, 0, s>>>(a, delta, fb_count);
  dim3 gq((a.fwd.seq_q + kWarps - 1) / kWarps, a.fwd.batch * a.fwd.heads);
  pass_bwd_dq_simt_kernel<T, DMAX><<<gq, kWarps * 32, 0, s>>>(a, delta, fb_count);
  dim3 gk((a.fwd.seq_k + kWarps - 1) / kWarps, a.fwd.batch * a.fwd.kv_heads);
  pass_bwd_dkv_simt_kernel<T, DMAX><<<gk, kWarps * 32, 0, s>>>(a, delta, fb_count);
  note_launch(3);
  return cuda_status(cudaGetLastError(), "pass_bwd_simt launch");
}

template <int DMAX>
int fwd_by_dtype(const PolyPassArgs& a, cudaStream_t s) {
  switch (a.dtype) {
    case POLY_F32: return launch_fwd_t<float, DMAX>(a, s);
    case POLY_F16: return launch_fwd_t<__half, DMAX>(a, s);
    default: return launch_fwd_t<__nv_bfloat16, DMAX>(a, s);
  }
}

template <int DMAX>
int bwd_by_dtype(const PolyPassBwdArgs& a, cudaStream_t s) {
  switch (a.fwd.dtype) {
    case POLY_F32: return launch_bwd_t<float, DMAX>(a, s);
    case POLY_F16: return launch_bwd_t<__half, DMAX>(a, s);
    default: return launch_bwd_t<__nv_bfloat16, DMAX>(a, s);
  }
}

}  // namespace

int launch_pass_fwd_simt(const PolyPassArgs& a, cudaStream_t s) {
  if (a.head_dim <= 32) return fwd_by_dtype<32>(a, s);
  if (a.head_dim <= 64) return fwd_by_dtype<64>(a, s);
  return fwd_by_dtype<128>(a, s);
}

int launch_pass_bwd_simt(const PolyPassBwdArgs& a, cudaStream_t s) {
  if (a.fwd.head_dim <= 32) return bwd_by_dtype<32>(a, s);
  if (a.fwd.head_dim <= 64) return bwd_by_dtype<64>(a, s);
  return bwd_by_dtype<128>(a, s);
}

}  // namespace poly
