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
#include <mutex>

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

constexpr int kTileKeys = 32;   // keys per pipeline stage
constexpr int kStages = 3;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = valid ? 16 : 0;   // zero-fill past the end
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename T, int D, int R, bool HAS_BIAS, bool HAS_VMUL, bool SOFTCLAMP>
__global__ void __launch_bounds__(kWarps * 32) decode_partial_kernel(const PolyPassArgs a, float* part, int kps) {
  constexpr int LPK = D / 8;            // lanes per key row (16-byte chunks per row)
  constexpr int KPS = 32 / LPK;         // keys per warp step
  constexpr int ROWB = D * 2;           // bytes per row
  constexpr int NARR = HAS_VMUL ? 3 : 2;
  extern __shared__ __align__(16) uint8_t dsm[];
  uint8_t* st_base = dsm;                                              // [stage][arr][key][ROWB]
  float* sbias = (float*)(dsm + kStages * NARR * kTileKeys * ROWB);   // [stage][key]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPK, li = lane % LPK;
  const int group = blockIdx.y;
  const int b = group / a.kv_heads, g = group - b * a.kv_heads;
  const int split = blockIdx.x;
  const int k0 = split * kps, k1 = min(a.seq_k, k0 + kps);
  const int ntile = (k1 - k0 + kTileKeys - 1) / kTileKeys;

  const T* kg = (const T*)a.k + b * a.k_stride[0] + g * a.k_stride[1];
  const T* vg = (const T*)a.v + b * a.v_stride[0] + g * a.v_stride[1];
  const T* mg = HAS_VMUL ? (const T*)a.v_mul + b * a.v_mul_stride[0] + g * a.v_mul_stride[1] : nullptr;
  const float* bg = HAS_BIAS ? a.bias + b * a.bias_stride[0] + g * a.bias_stride[1] : nullptr;

  auto issue = [&](int tile) {
    const int stg = tile % kStages;
    const int kb = k0 + tile * kTileKeys;
    uint8_t* dst = st_base + stg * NARR * kTileKeys * ROWB;
    for (int c = threadIdx.x; c < kTileKeys * LPK; c += kWarps * 32) {
      const int key = c / LPK, ch = c % LPK;
      const int j = kb + key;
      const bool ok = j < k1;
      const int jj = ok ? j : k0;
      cp_async16(dst + (0 * kTileKeys + key) * ROWB + ch * 16, kg + (int64_t)jj * a.k_stride[2] + ch * 8, ok);
      cp_async16(dst + (1 * kTileKeys + key) * ROWB + ch * 16, vg + (int64_t)jj * a.v_stride[2] + ch * 8, ok);
      if (HAS_VMUL)
        cp_async16(dst + (2 * kTileKeys + key) * ROWB + ch * 16, mg + (int64_t)jj * a.v_mul_stride[2] + ch * 8, ok);
    }
    if (HAS_BIAS && threadIdx.x < kTileKeys) {
      const int j = kb + threadIdx.x;
      sbias[stg * kTileKeys + threadIdx.x] = j < k1 ? bg[j] : 0.f;
    }
  };

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

#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) {
    if (t < ntile) issue(t);
    cp_async_commit();
  }
  for (int tile = 0; tile < ntile; ++tile) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    if (tile + kStages - 1 < ntile) issue(tile + kStages - 1);
    cp_async_commit();
    const int stg = tile % kStages;
    const uint8_t* src = st_base + stg * NARR * kTileKeys * ROWB;
    const int kb = k0 + tile * kTileKeys;
    // warp w takes keys [w * 8, w * 8 + 8) of the tile, KPS keys per step
#pragma unroll
    for (int st = 0; st < kTileKeys / kWarps / KPS; ++st) {
      const int key = warp * (kTileKeys / kWarps) + st * KPS + sub;
      const bool valid = kb + key < k1;
      Vec8<T> kv, vv;
      kv.load(reinterpret_cast<const T*>(src + (0 * kTileKeys + key) * ROWB + li * 16));
      vv.load(reinterpret_cast<const T*>(src + (1 * kTileKeys + key) * ROWB + li * 16));
      if (HAS_VMUL) {
        Vec8<T> mv;
        mv.load(reinterpret_cast<const T*>(src + (2 * kTileKeys + key) * ROWB + li * 16));
#pragma unroll
        for (int e = 0; e < 8; ++e) vv.f[e] = to_f32(from_f32<T>(vv.f[e] * mv.f[e]));
      }
      float b2 = 0.f;
      if (HAS_BIAS) {
        const float braw = sbias[stg * kTileKeys + key];
        b2 = braw <= kDeadBias ? -INFINITY : braw * kLog2e;
      }
#pragma unroll
      for (int rr = 0; rr < R; ++rr) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          s0 = fmaf(q[rr][e], kv.f[e], s0);
          s1 = fmaf(q[rr][e + 1], kv.f[e + 1], s1);
        }
        float s = s0 + s1;
#pragma unroll
        for (int o = 1; o < LPK; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (SOFTCLAMP) s = tanhf(s * sc_in) * sc_out;
        s = valid ? s + b2 : -INFINITY;
        if (s > m[rr] + 8.f) {                  // lazy max: rescale only on large growth
          const float alpha = exp2f(m[rr] - s);
          m[rr] = s;
          l[rr] *= alpha;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[rr][e] *= alpha;
        }
        const float pr = (s == -INFINITY) ? 0.f : exp2f(s - m[rr]);
        l[rr] += pr;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[rr][e] = fmaf(pr, vv.f[e], acc[rr][e]);
      }
    }
  }
  cp_async_wait<0>();
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

// One warp per (group, head-in-group): merge all partials of the row. Lanes
// read the (max, sum) of different partials in parallel; the accumulators are
// then summed with independent loads.
template <typename T, int D, int R>
__global__ void decode_combine_kernel(const PolyPassArgs a, const float* part, int nparts) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int groups = a.batch * a.kv_heads;
  if (w >= groups * R) return;
  const int group = w / R, rr = w - group * R;
  const int b = group / a.kv_heads, g = group - b * a.kv_heads, h = g * R + rr;
  auto rec = [&](int pi) { return part + (((int64_t)group * nparts + pi) * R + rr) * (D + 2); };
  // lane p owns partials p and p + 32 (nparts <= 64): their weights stay in
  // registers and are broadcast with shuffles, so every accumulator load below
  // is independent of the others
  float mv0 = -INFINITY, mv1 = -INFINITY, lv0 = 0.f, lv1 = 0.f;
  if (lane < nparts) { mv0 = rec(lane)[0]; lv0 = rec(lane)[1]; }
  if (lane + 32 < nparts) { mv1 = rec(lane + 32)[0]; lv1 = rec(lane + 32)[1]; }
  const float M = warp_max(fmaxf(mv0, mv1));
  const float w0 = (mv0 == -INFINITY) ? 0.f : exp2f(mv0 - M);
  const float w1 = (mv1 == -INFINITY) ? 0.f : exp2f(mv1 - M);
  const float L = warp_sum(lv0 * w0 + lv1 * w1);
  float o[D / 32];
#pragma unroll
  for (int t = 0; t < D / 32; ++t) o[t] = 0.f;
#pragma unroll 8
  for (int pi = 0; pi < nparts; ++pi) {
    const float f = __shfl_sync(0xffffffffu, pi < 32 ? w0 : w1, pi & 31);
    const float* r_ = rec(pi);
#pragma unroll
    for (int t = 0; t < D / 32; ++t) o[t] = fmaf(r_[2 + lane + 32 * t], f, o[t]);
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
  const int step = kTileKeys;                 // keys one CTA stages per pipeline step
  (void)keys_step;
  int splits = (a.seq_k + step - 1) / step;                       // at most one warp-step of keys per warp
  const int want = (8 * 148 + groups - 1) / groups;               // ~8 CTAs per SM
  splits = max(1, min(min(splits, want), 64 / kWarps));   // the combine holds <= 64 partials per row
  DecodeGeom gm;
  gm.kps = (a.seq_k + splits - 1) / splits;
  gm.kps = (gm.kps + step - 1) / step * step;
  gm.splits = (a.seq_k + gm.kps - 1) / gm.kps;
  return gm;
}

template <int D, bool V>
constexpr int smem_bytes() { return kStages * (V ? 3 : 2) * kTileKeys * D * 2 + kStages * kTileKeys * 4; }

template <typename T, int D, int R>
int launch3(const PolyPassArgs& a, cudaStream_t s) {
  const DecodeGeom gm = geometry(a, keys_per_step<D>());
  float* part = (float*)a.workspace;
  dim3 grid(gm.splits, a.batch * a.kv_heads);
  const bool bias = a.bias != nullptr, vm = a.v_mul != nullptr, sc = a.softclamp > 0.f;
#define POLY_DEC(B, V, C)                                                                                  \
  do {                                                                                                     \
    static std::once_flag once_;                                                                           \
    static cudaError_t err_ = cudaSuccess;                                                                 \
    std::call_once(once_, [] {                                                                             \
      err_ = cudaFuncSetAttribute(decode_partial_kernel<T, D, R, B, V, C>,                                 \
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes<D, V>());        \
    });                                                                                                    \
    if (err_ != cudaSuccess) return cuda_status(err_, "cudaFuncSetAttribute(decode)");                     \
    decode_partial_kernel<T, D, R, B, V, C><<<grid, kWarps * 32, smem_bytes<D, V>(), s>>>(a, part, gm.kps); \
  } while (0)
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
