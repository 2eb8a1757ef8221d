// Per-head RMSNorm of query / key tensors read straight from the strided
// head-split view of a projection output (q_norms of
// poly_attention/poly_attention.py:272 and n_poly_attention.py:186-187).
// The module path otherwise pays a contiguous copy of the view plus a
// layer-norm kernel built for long rows: at dim_head 64 the pair ran at
// ~0.35 TB/s. Here 8 lanes own one row (16-byte loads), the sum of squares is
// a 3-step shuffle, and up to POLY_MAX_NORMS tensors go in one launch.
#include <string>
#include <type_traits>

#include "common.cuh"

namespace poly {
namespace {

struct Norms {
  PolyHeadNorm d[POLY_MAX_NORMS];
  int64_t start[POLY_MAX_NORMS + 1];   // first global row of each tensor
  int n;
};

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, int i) { return to_f32(p[i]); }
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, int i) { return p[i]; }

template <typename T>
__device__ __forceinline__ T st_f(float x) { return from_f32<T>(x); }
template <>
__device__ __forceinline__ float st_f<float>(float x) { return x; }

template <typename TS, typename TD, typename TW, int NJ>
__global__ void __launch_bounds__(256) head_rmsnorm_kernel(const Norms P) {
  constexpr int VEC = 16 / sizeof(TS);   // elements per 16-byte chunk; a lane owns NJ chunks of a row
  constexpr int NR = 2;                  // rows per lane group per iteration (loads in flight)
  const int lane = threadIdx.x & 31, sub = lane >> 3, li = lane & 7;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = P.start[P.n];
  for (int64_t r0 = warp * 4 * NR; r0 < total; r0 += nwarps * 4 * NR) {
    float v[NR][NJ * VEC];
    float ss[NR];
    const TS* src[NR];
    int kd[NR];
    int64_t dst_row[NR];
#pragma unroll
    for (int u = 0; u < NR; ++u) {
      const int64_t r = r0 + u * 4 + sub;
      const bool ok = r < total;
      int k = 0;
      while (k + 1 < P.n && r >= P.start[k + 1]) ++k;
      const PolyHeadNorm& d = P.d[k];
      // row coordinates in 32-bit arithmetic (a tensor has < 2^31 rows)
      const int local = ok ? (int)(r - P.start[k]) : 0;
      const int t = local / d.rows, ni = local - t * d.rows;
      const int bi = t / d.heads, hi = t - bi * d.heads;
      kd[u] = ok ? k : -1;
      src[u] = (const TS*)d.src + (int64_t)bi * d.src_stride[0] + (int64_t)hi * d.src_stride[1] +
               (int64_t)ni * d.src_stride[2];
      dst_row[u] = (int64_t)local * d.dim;
    }
#pragma unroll
    for (int u = 0; u < NR; ++u) {
      const int chunks = kd[u] >= 0 ? P.d[kd[u]].dim / VEC : 0;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int c = li + 8 * j;
        if (c < chunks) {
          const uint4 q4 = *reinterpret_cast<const uint4*>(src[u] + c * VEC);
          const TS* e = reinterpret_cast<const TS*>(&q4);
#pragma unroll
          for (int q = 0; q < VEC; ++q) v[u][j * VEC + q] = ld_f<TS>(e, q);
        } else {
#pragma unroll
          for (int q = 0; q < VEC; ++q) v[u][j * VEC + q] = 0.f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < NR; ++u) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < NJ * VEC; ++i) a = fmaf(v[u][i], v[u][i], a);
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      a += __shfl_xor_sync(0xffffffffu, a, 2);
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      ss[u] = a;
    }
#pragma unroll
    for (int u = 0; u < NR; ++u) {
      if (kd[u] < 0) continue;
      const PolyHeadNorm& d = P.d[kd[u]];
      const float rs = rsqrtf(ss[u] / (float)d.dim + d.eps);
      const int chunks = d.dim / VEC;
      const TW* w = (const TW*)d.weight;
      TD* dst = (TD*)d.dst + dst_row[u];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int c = li + 8 * j;
        if (c < chunks) {
          // weights and outputs of the chunk as 16-byte vectors
          float wv[VEC];
#pragma unroll
          for (int q0 = 0; q0 < VEC; q0 += 16 / (int)sizeof(TW)) {
            const uint4 q4 = *reinterpret_cast<const uint4*>(w + c * VEC + q0);
            const TW* e = reinterpret_cast<const TW*>(&q4);
#pragma unroll
            for (int q = 0; q < 16 / (int)sizeof(TW); ++q) wv[q0 + q] = ld_f<TW>(e, q);
          }
          constexpr int OV = 16 / sizeof(TD);   // outputs per 16-byte store
#pragma unroll
          for (int q0 = 0; q0 < VEC; q0 += OV) {
            uint4 q4;
            TD* e = reinterpret_cast<TD*>(&q4);
#pragma unroll
            for (int q = 0; q < OV; ++q) e[q] = st_f<TD>(v[u][j * VEC + q0 + q] * rs * wv[q0 + q]);
            *reinterpret_cast<uint4*>(dst + c * VEC + q0) = q4;
          }
        }
      }
    }
  }
}

int bad(const std::string& m) {
  set_error(m);
  return POLY_EINVAL;
}

template <typename TS, typename TD, typename TW>
int launch(const Norms& P, cudaStream_t s) {
  const int64_t warps = (P.start[P.n] + 7) / 8;
  const int64_t blocks = (warps * 32 + 255) / 256;
  const unsigned grid = (unsigned)(blocks < 148 * 16 ? blocks : 148 * 16);
  constexpr int VEC = 16 / sizeof(TS);
  int maxdim = 0;
  for (int i = 0; i < P.n; ++i) maxdim = P.d[i].dim > maxdim ? P.d[i].dim : maxdim;
  const int nj = (maxdim / VEC + 7) / 8;   // chunks per lane for the widest row
  if (nj <= 1) head_rmsnorm_kernel<TS, TD, TW, 1><<<grid, 256, 0, s>>>(P);
  else if (nj <= 2) head_rmsnorm_kernel<TS, TD, TW, 2><<<grid, 256, 0, s>>>(P);
  else head_rmsnorm_kernel<TS, TD, TW, 32 / VEC><<<grid, 256, 0, s>>>(P);
  note_launch(1);
  return cuda_status(cudaGetLastError(), "head_rmsnorm launch");
}

template <typename TS>
int dispatch_dw(const Norms& P, cudaStream_t s) {
  const bool dst32 = P.d[0].dst_dtype == POLY_F32, w32 = P.d[0].weight_dtype == POLY_F32;
  if (std::is_same<TS, float>::value) return launch<float, float, float>(P, s);
  if (dst32) return w32 ? launch<TS, float, float>(P, s) : launch<TS, float, TS>(P, s);
  return w32 ? launch<TS, TS, float>(P, s) : launch<TS, TS, TS>(P, s);
}

}  // namespace

int head_rmsnorm(const PolyHeadNorm* norms, int n, cudaStream_t s) {
  if (n < 0 || n > POLY_MAX_NORMS || (n > 0 && !norms))
    return bad("poly_head_rmsnorm: n must be in [0, 4] with a norms array");
  if (n == 0) return POLY_OK;
  Norms P;
  P.n = n;
  P.start[0] = 0;
  const int sd = norms[0].src_dtype;
  for (int i = 0; i < n; ++i) {
    const PolyHeadNorm& d = norms[i];
    const std::string at = "poly_head_rmsnorm: tensor " + std::to_string(i) + ": ";
    if (d.src_dtype != sd || d.dst_dtype != norms[0].dst_dtype || d.weight_dtype != norms[0].weight_dtype)
      return bad(at + "all tensors of one call share their dtypes");
    if (d.src_dtype < POLY_F32 || d.src_dtype > POLY_BF16 || (d.dst_dtype != d.src_dtype && d.dst_dtype != POLY_F32) ||
        (d.weight_dtype != d.src_dtype && d.weight_dtype != POLY_F32))
      return bad(at + "dst / weight dtype must be the source dtype or F32");
    if (d.batch < 0 || d.heads < 0 || d.rows < 0) return bad(at + "negative extent");
    if ((int64_t)d.batch * d.heads * d.rows >= (int64_t)1 << 31) return bad(at + "more than 2^31 - 1 rows");
    const int esz = d.src_dtype == POLY_F32 ? 4 : 2;
    if (d.dim <= 0 || d.dim > 256 || d.dim % 8) return bad(at + "dim must be a multiple of 8 in [8, 256]");
    const int64_t cnt = (int64_t)d.batch * d.heads * d.rows;
    if (cnt && (!d.src || !d.dst || !d.weight || ((uintptr_t)d.src & 15) || ((uintptr_t)d.dst & 15) ||
                ((uintptr_t)d.weight & 15) ||
                ((d.src_stride[0] * esz) & 15) || ((d.src_stride[1] * esz) & 15) || ((d.src_stride[2] * esz) & 15)))
      return bad(at + "needs 16-byte aligned src rows (pointer and strides), dst and weight");
    P.d[i] = d;
    P.start[i + 1] = P.start[i] + cnt;
  }
  if (P.start[n] == 0) return POLY_OK;
  if (sd == POLY_F32) return dispatch_dw<float>(P, s);
  if (sd == POLY_F16) return dispatch_dw<__half>(P, s);
  return dispatch_dw<__nv_bfloat16>(P, s);
}

}  // namespace poly
