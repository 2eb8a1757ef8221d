// KV-cache decode pass: one new query row per head against a long cache
// (seq_q == 1), HBM-bound. Replaces the reference's per-step materialised
// passes over the concatenated cache (poly_attention/poly_attention.py:63-114
// with cache, n_poly_attention.py:263-313 with cache).
//
// Split-K: CTA (split, group) reads keys [split * kps, (split + 1) * kps) of
// one (batch, kv head) group once and serves all R = heads / kv_heads query
// heads of the group. A key row (D 16-bit values) is read by D / 8 lanes with
// 16-byte loads, so a warp covers 32 / (D / 8) keys per step, fully coalesced;
// values are multiplied by v_mul (the order-n chain's V' = v * msg) and the
// per-key bias (the previous level's lse) is added on the fly. Each lane group
// keeps its own running (max, sum, acc) with a lazy max (rescale only when the
// max grows by more than 2^8); warps write partials that a combine kernel
// merges, writing out, lse and the optional epilogue product.
#include "common.cuh"

namespace poly {
namespace {

constexpr int kWarps = 4;

template <typename T>
struct Vec8 {
  float f[8];
  __device__ __forceinline__ void load(const T* p) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = to_f32(t[e]);
  }
};

struct DecodeGeom {
  int splits, kps;  // key splits and keys per split
};

template <int D>
__host__ __device__ constexpr int keys_per_step() { return 32 / (D / 8); }

template <typename T, int D, int R, bool HAS_BIAS, bool HAS_VMUL, bool SOFTCLAMP>
__global__ void __launch_bounds__(kWarps * 32) decode_partial_kernel(const PolyPassArgs a, float* part, int kps) {
  constexpr int LPK = D / 8;            // lanes per key row
  constexpr int KPS = 32 / LPK;         // keys per warp step
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPK, li = lane % LPK;
  const int group = blockIdx.y;
  const int b = group / a.kv_heads, g = group - b * a.kv_heads;
  const int split = blockIdx.x;
  const int k0 = split * kps, k1 = min(a.seq_k, k0 + kps);

  const T* kp = (const T*)a.k + b * a.k_stride[0] + g * a.k_stride[1] + li * 8;
  const T* vp = (const T*)a.v + b * a.v_stride[0] + g * a.v_stride[1] + li * 8;
  const T* mp = HAS_VMUL ? (const T*)a.v_mul + b * a.v_mul_stride[0] + g * a.v_mul_stride[1] + li * 8 : nullptr;
  const float* bp = HAS_BIAS ? a.bias + b * a.bias_stride[0] + g * a.bias_stride[1] : nullptr;

  float q[R][8];
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    Vec8<T> qv;
    qv.load((const T*)a.q + b * a.q_stride[0] + (g * R + rr) * a.q_stride[1] + li * 8);
#pragma unroll
    for (int e = 0; e < 8; ++e) q[rr][e] = qv.f[e] * (SOFTCLAMP ? a.scale : a.scale * kLog2e);
  }
  float m[R], l[R], acc[R][8];
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    m[rr] = -INFINITY;
    l[rr] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[rr][e] = 0.f;
  }
  const float sc_in = SOFTCLAMP ? 1.f / a.softclamp : 0.f;
  const float sc_out = SOFTCLAMP ? a.softclamp * kLog2e : 0.f;

  // warp-uniform trip count: every lane runs every step (the shuffles below
  // need the whole warp); lanes whose key is past the split end skip the update
#pragma unroll 2
  for (int jb = k0 + warp * KPS; jb < k1; jb += kWarps * KPS) {
    const int j = jb + sub;
    const bool valid = j < k1;
    Vec8<T> kv, vv;
    if (valid) {
      kv.load(kp + (int64_t)j * a.k_stride[2]);
      vv.load(vp + (int64_t)j * a.v_stride[2]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) kv.f[e] = vv.f[e] = 0.f;
    }
    if (HAS_VMUL && valid) {
      Vec8<T> mv;
      mv.load(mp + (int64_t)j * a.v_mul_stride[2]);
#pragma unroll
      for (int e = 0; e < 8; ++e) vv.f[e] = to_f32(from_f32<T>(vv.f[e] * mv.f[e]));
    }
    float b2 = 0.f;
    if (HAS_BIAS && valid) {
      const float braw = bp[j];
      b2 = braw <= kDeadBias ? -INFINITY : braw * kLog2e;
    }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(q[rr][e], kv.f[e], s);
#pragma unroll
      for (int o = 1; o < LPK; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (SOFTCLAMP) s = tanhf(s * sc_in) * sc_out;
      s += b2;
      if (!valid) continue;
      if (s > m[rr] + 8.f) {                  // lazy max: rescale only on large growth
        const float alpha = exp2f(m[rr] - s);
        m[rr] = s;
        l[rr] *= alpha;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[rr][e] *= alpha;
      }
      const float pr = exp2f(s - m[rr]);
      l[rr] += pr;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[rr][e] = fmaf(pr, vv.f[e], acc[rr][e]);
    }
  }
  // merge the KPS lane groups of this warp (lanes li, li + LPK, ...)
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    float mm = m[rr];
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
    const float f = (mm == -INFINITY) ? 0.f : exp2f(m[rr] - mm);
    float ll = l[rr] * f;
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1) ll += __shfl_xor_sync(0xffffffffu, ll, o);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float x = acc[rr][e] * f;
#pragma unroll
      for (int o = LPK; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      acc[rr][e] = x;
    }
    // partial record: [m, l, acc[D]] per (group, split * kWarps + warp, rr)
    float* rec = part + (((int64_t)group * gridDim.x * kWarps + split * kWarps + warp) * R + rr) * (D + 2);
    if (sub == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) rec[2 + li * 8 + e] = acc[rr][e];
      if (li == 0) {
        rec[0] = mm;
        rec[1] = ll;
      }
    }
  }
}

// One warp per (group, head-in-group): merge all partials of the row.
template <typename T, int D, int R>
__global__ void decode_combine_kernel(const PolyPassArgs a, const float* part, int nparts) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int groups = a.batch * a.kv_heads;
  if (w >= groups * R) return;
  const int group = w / R, rr = w - group * R;
  const int b = group / a.kv_heads, g = group - b * a.kv_heads, h = g * R + rr;
  float M = -INFINITY;
  for (int pi = 0; pi < nparts; ++pi) M = fmaxf(M, part[(((int64_t)group * nparts + pi) * R + rr) * (D + 2)]);
  float L = 0.f;
  float o[D / 32];
#pragma unroll
  for (int t = 0; t < D / 32; ++t) o[t] = 0.f;
  for (int pi = 0; pi < nparts; ++pi) {
    const float* rec = part + (((int64_t)group * nparts + pi) * R + rr) * (D + 2);
    const float mv = rec[0];
    const float f = (mv == -INFINITY) ? 0.f : exp2f(mv - M);
    L += rec[1] * f;
#pragma unroll
    for (int t = 0; t < D / 32; ++t) o[t] += rec[2 + lane + 32 * t] * f;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* out = (T*)a.out + b * a.out_stride[0] + h * a.out_stride[1];
  const T* em = a.epi_out ? (const T*)a.epi_mul + b * a.epi_mul_stride[0] + h * a.epi_mul_stride[1] : nullptr;
  T* eo = a.epi_out ? (T*)a.epi_out + b * a.epi_out_stride[0] + h * a.epi_out_stride[1] : nullptr;
#pragma unroll
  for (int t = 0; t < D / 32; ++t) {
    const T ov = from_f32<T>(o[t] * inv);
    out[lane + 32 * t] = ov;
    if (eo) eo[lane + 32 * t] = from_f32<T>(to_f32(em[lane + 32 * t]) * to_f32(ov));
  }
  if (a.lse && lane == 0) a.lse[b * a.lse_stride[0] + h * a.lse_stride[1]] = (M + __log2f(L)) * kLn2;
}

DecodeGeom geometry(const PolyPassArgs& a, int keys_step) {
  const int groups = a.batch * a.kv_heads;
  const int step = keys_step * kWarps;
  int splits = (a.seq_k + step - 1) / step;                       // at most one warp-step of keys per warp
  const int want = (8 * 148 + groups - 1) / groups;               // ~8 CTAs per SM
  splits = max(1, min(splits, want));
  DecodeGeom gm;
  gm.kps = (a.seq_k + splits - 1) / splits;
  gm.kps = (gm.kps + step - 1) / step * step;
  gm.splits = (a.seq_k + gm.kps - 1) / gm.kps;
  return gm;
}

template <typename T, int D, int R>
int launch3(const PolyPassArgs& a, cudaStream_t s) {
  const DecodeGeom gm = geometry(a, keys_per_step<D>());
  float* part = (float*)a.workspace;
  dim3 grid(gm.splits, a.batch * a.kv_heads);
  const bool bias = a.bias != nullptr, vm = a.v_mul != nullptr, sc = a.softclamp > 0.f;
#define POLY_DEC(B, V, C) decode_partial_kernel<T, D, R, B, V, C><<<grid, kWarps * 32, 0, s>>>(a, part, gm.kps)
  if (sc) {
    if (bias) { if (vm) POLY_DEC(true, true, true); else POLY_DEC(true, false, true); }
    else { if (vm) POLY_DEC(false, true, true); else POLY_DEC(false, false, true); }
  } else {
    if (bias) { if (vm) POLY_DEC(true, true, false); else POLY_DEC(true, false, false); }
    else { if (vm) POLY_DEC(false, true, false); else POLY_DEC(false, false, false); }
  }
#undef POLY_DEC
  const int rows = a.batch * a.kv_heads * R;
  decode_combine_kernel<T, D, R><<<(rows * 32 + 255) / 256, 256, 0, s>>>(a, part, gm.splits * kWarps);
  note_launch(2);
  return cuda_status(cudaGetLastError(), "decode launch");
}

template <typename T, int D>
int launch2(const PolyPassArgs& a, cudaStream_t s) {
  switch (a.heads / a.kv_heads) {
    case 1: return launch3<T, D, 1>(a, s);
    case 2: return launch3<T, D, 2>(a, s);
    case 4: return launch3<T, D, 4>(a, s);
    default: return launch3<T, D, 8>(a, s);
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

bool pass_decode_eligible(const PolyPassArgs& a) {
  if (a.seq_q != 1 || a.causal || a.key_mask || a.query_mask) return false;
  if (a.dtype != POLY_BF16 && a.dtype != POLY_F16) return false;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  const int r = a.heads / a.kv_heads;
  if (r != 1 && r != 2 && r != 4 && r != 8) return false;
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v)) return false;
  if ((a.k_stride[2] & 7) || (a.v_stride[2] & 7) || (a.q_stride[1] & 7) || (a.q_stride[0] & 7)) return false;
  if ((a.k_stride[0] | a.k_stride[1] | a.v_stride[0] | a.v_stride[1]) & 7) return false;
  if (a.v_mul && (!aligned16(a.v_mul) || ((a.v_mul_stride[0] | a.v_mul_stride[1] | a.v_mul_stride[2]) & 7)))
    return false;
  return true;
}

size_t pass_decode_workspace(const PolyPassArgs& a) {
  const DecodeGeom gm = geometry(a, a.head_dim == 64 ? keys_per_step<64>() : keys_per_step<128>());
  return (size_t)a.batch * a.kv_heads * gm.splits * kWarps * (a.heads / a.kv_heads) * (a.head_dim + 2) * sizeof(float);
}

int launch_pass_decode(const PolyPassArgs& a, cudaStream_t s) {
  if (a.dtype == POLY_BF16)
    return a.head_dim == 64 ? launch2<__nv_bfloat16, 64>(a, s) : launch2<__nv_bfloat16, 128>(a, s);
  return a.head_dim == 64 ? launch2<__half, 64>(a, s) : launch2<__half, 128>(a, s);
}

}  // namespace poly
