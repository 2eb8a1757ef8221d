// Attention pass for short sequences (seq_q, seq_k <= 128): one CTA per
// (batch, head), one warp per 16 query rows. PolyViT's 64-token images
// (poly_vit.py:42-101 calling poly_attention.py:63-114) are the case: there a
// 128 x 128 tcgen05 tile pair would be >85% padding. The whole key range fits
// in shared memory (cp.async, 16-byte chunks XOR-swizzled by row so ldmatrix
// is conflict-free), a row's scores stay in registers, so the softmax needs no
// running rescale: S = Q K^T and O = P V on mma.sync m16n8k16 (fp32
// accumulation), exact row max, one normalisation. Same semantics as the other
// pass kernels: scale, softclamp, causal (top-left aligned), per-key bias in
// the log2 domain with dead keys (bias <= -FLT_MAX / 2) dropped, lse in
// natural-log units.
#include <cfloat>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace poly {
namespace {

constexpr int kMaxN = 128;

__device__ __forceinline__ void cp16(uint32_t sa, const void* g, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(g), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
template <typename T>
__device__ __forceinline__ void mma(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                    uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ uint32_t pk2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return tc::pack_bf16(lo, hi);
  else return tc::pack_f16(lo, hi);
}

// byte offset of 16-byte chunk ch of row r in a [kMaxN][D] tile
template <int D>
__device__ __forceinline__ uint32_t soff(int r, int ch) {
  return (uint32_t)(r * (D * 2) + ((ch ^ (r & 7)) << 4));
}

template <typename T, int D, bool HAS_BIAS, bool SOFTCLAMP>
__global__ void __launch_bounds__(256) pass_small_kernel(const PolyPassArgs a) {
  constexpr int KS = D / 16, NB = D / 8, CH = D / 8;
  constexpr int KNB = kMaxN / 8;   // key n-blocks
  const int nq = a.seq_q, nk = a.seq_k;
  const int kp = (nk + 15) & ~15;   // keys padded to the P.V K step
  // shared memory sized to the keys present: K [kp][D], V [kp][D], bias [kp]
  extern __shared__ __align__(16) uint8_t sm[];
  const uint32_t sK = tc::smem_u32(sm), sV = sK + kp * D * 2;
  float* sB = reinterpret_cast<float*>(sm + 2 * kp * D * 2);

  const int bh = blockIdx.x;
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int g = h / (a.heads / a.kv_heads);
  const T* kg = (const T*)a.k + b * a.k_stride[0] + g * a.k_stride[1];
  const T* vg = (const T*)a.v + b * a.v_stride[0] + g * a.v_stride[1];
  for (int c = threadIdx.x; c < kp * CH; c += blockDim.x) {
    const int r = c / CH, ch = c - r * CH;
    const bool ok = r < nk;
    const int rr = ok ? r : 0;
    cp16(sK + soff<D>(r, ch), kg + (int64_t)rr * a.k_stride[2] + ch * 8, ok);
    cp16(sV + soff<D>(r, ch), vg + (int64_t)rr * a.v_stride[2] + ch * 8, ok);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if (HAS_BIAS)
    for (int j = threadIdx.x; j < kp; j += blockDim.x) {
      float x = -INFINITY;
      if (j < nk) {
        const float raw = a.bias[b * a.bias_stride[0] + g * a.bias_stride[1] + j];
        x = raw <= kDeadBias ? -INFINITY : raw * kLog2e;
      }
      sB[j] = x;
    }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int r0 = warp * 16 + gq, r1 = r0 + 8;   // this thread's two query rows
  // Q fragments (rows r0 / r1, K step ks): loaded while the keys stream in
  uint32_t qa[KS][4];
  {
    const T* qb = (const T*)a.q + b * a.q_stride[0] + h * a.q_stride[1];
    const T* q0 = qb + (int64_t)(r0 < nq ? r0 : 0) * a.q_stride[2];
    const T* q1 = qb + (int64_t)(r1 < nq ? r1 : 0) * a.q_stride[2];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int c0 = ks * 16 + 2 * tq;
      qa[ks][0] = r0 < nq ? *reinterpret_cast<const uint32_t*>(q0 + c0) : 0u;
      qa[ks][1] = r1 < nq ? *reinterpret_cast<const uint32_t*>(q1 + c0) : 0u;
      qa[ks][2] = r0 < nq ? *reinterpret_cast<const uint32_t*>(q0 + c0 + 8) : 0u;
      qa[ks][3] = r1 < nq ? *reinterpret_cast<const uint32_t*>(q1 + c0 + 8) : 0u;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (warp * 16 >= nq) return;

  // S = Q K^T over every key block; scores of rows r0 (e = 0, 1) and r1 (e = 2, 3)
  float s[KNB][4];
  const float qk = SOFTCLAMP ? a.scale / a.softclamp : a.scale * kLog2e;
  const float sc_out = SOFTCLAMP ? a.softclamp * kLog2e : 0.f;
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int nb = 0; nb < KNB; ++nb) {
    s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
    if (nb * 8 < kp) {
      const int key = nb * 8 + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm4(sK + soff<D>(key, ks * 2 + (lane >> 3)), b0, b1, b2, b3);
        mma<T>(s[nb], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma<T>(s[nb], qa[ks + 1][0], qa[ks + 1][1], qa[ks + 1][2], qa[ks + 1][3], b2, b3);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = nb * 8 + 2 * tq + (e & 1);
        const int row = e < 2 ? r0 : r1;
        float x = s[nb][e] * qk;
        if (SOFTCLAMP) x = tanhf(x) * sc_out;
        if (HAS_BIAS) x += sB[j];
        if (j >= nk || (a.causal && j > row)) x = -INFINITY;
        s[nb][e] = x;
      }
      m0 = fmaxf(m0, fmaxf(s[nb][0], s[nb][1]));
      m1 = fmaxf(m1, fmaxf(s[nb][2], s[nb][3]));
    }
  }
  m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
  m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int nb = 0; nb < KNB; ++nb) {
    if (nb * 8 < kp) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = e < 2 ? m0 : m1;
        const float p = s[nb][e] == -INFINITY ? 0.f : exp2f(s[nb][e] - m);
        s[nb][e] = p;
        if (e < 2) l0 += p; else l1 += p;
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // O = P V, K steps of 16 keys (P from the score registers, V via ldmatrix.trans)
  float o[NB][4];
#pragma unroll
  for (int n = 0; n < NB; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < kMaxN / 16; ++kk) {
    if (kk * 16 < kp) {
      const uint32_t pa0 = pk2<T>(s[2 * kk][0], s[2 * kk][1]), pa1 = pk2<T>(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t pa2 = pk2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t pa3 = pk2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      const int vkey = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int n2 = 0; n2 < NB / 2; ++n2) {
        uint32_t v0, v1, v2, v3;
        ldsm4t(sV + soff<D>(vkey, n2 * 2 + (lane >> 4)), v0, v1, v2, v3);
        mma<T>(o[2 * n2], pa0, pa1, pa2, pa3, v0, v1);
        mma<T>(o[2 * n2 + 1], pa0, pa1, pa2, pa3, v2, v3);
      }
    }
  }
  bool fb0 = false, fb1 = false;   // row took the fully-excluded result
  // A row whose every key is excluded (only dead keys can do that here) gets
  // the reference's -finfo.max result: the uniform average over the keys that
  // are not both causally masked and dead, lse = -FLT_MAX.
  if (HAS_BIAS && (m0 == -INFINITY || m1 == -INFINITY)) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = hf ? r1 : r0;
      if ((hf ? m1 : m0) != -INFINITY) continue;
      int count = 0;
#pragma unroll
      for (int n = 0; n < NB; ++n) o[n][2 * hf] = o[n][2 * hf + 1] = 0.f;
      for (int j = 0; j < nk; ++j) {
        if (a.causal && j > row && sB[j] == -INFINITY) continue;
        ++count;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(sm + kp * D * 2 + soff<D>(j, n) + 4 * tq);
          const T* e = reinterpret_cast<const T*>(&w);
          o[n][2 * hf] += to_f32(e[0]);
          o[n][2 * hf + 1] += to_f32(e[1]);
        }
      }
      if (hf) { l1 = (float)count; fb1 = true; } else { l0 = (float)count; fb0 = true; }
    }
  }
  const float j0 = l0 > 0.f ? 1.f / l0 : 0.f, j1 = l1 > 0.f ? 1.f / l1 : 0.f;
  T* ob = (T*)a.out + b * a.out_stride[0] + h * a.out_stride[1];
#pragma unroll
  for (int n = 0; n < NB; ++n) {
    const int c = n * 8 + 2 * tq;
    if (r0 < nq) *reinterpret_cast<uint32_t*>(ob + (int64_t)r0 * a.out_stride[2] + c) = pk2<T>(o[n][0] * j0, o[n][1] * j0);
    if (r1 < nq) *reinterpret_cast<uint32_t*>(ob + (int64_t)r1 * a.out_stride[2] + c) = pk2<T>(o[n][2] * j1, o[n][3] * j1);
  }
  if (a.lse && tq == 0) {
    float* lb = a.lse + b * a.lse_stride[0] + h * a.lse_stride[1];
    if (r0 < nq) lb[r0] = fb0 ? -FLT_MAX : (m0 + __log2f(l0)) * kLn2;
    if (r1 < nq) lb[r1] = fb1 ? -FLT_MAX : (m1 + __log2f(l1)) * kLn2;
  }
}

template <typename T, int D, bool B, bool C>
int launch_t(const PolyPassArgs& a, cudaStream_t s) {
  constexpr int smem = 2 * kMaxN * D * 2 + kMaxN * 4;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(pass_small_kernel<T, D, B, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (err != cudaSuccess) return cuda_status(err, "cudaFuncSetAttribute(small)");
  const int threads = 32 * ((a.seq_q + 15) / 16);
  const int kp = (a.seq_k + 15) & ~15;
  const int bytes = 2 * kp * D * 2 + kp * 4;   // <= smem (the attribute's maximum)
  pass_small_kernel<T, D, B, C><<<a.batch * a.heads, threads, bytes, s>>>(a);
  note_launch(1);
  return cuda_status(cudaGetLastError(), "pass_small launch");
}

template <typename T, int D>
int launch_d(const PolyPassArgs& a, cudaStream_t s) {
  const bool bias = a.bias != nullptr, sc = a.softclamp > 0.f;
  if (sc) return bias ? launch_t<T, D, true, true>(a, s) : launch_t<T, D, false, true>(a, s);
  return bias ? launch_t<T, D, true, false>(a, s) : launch_t<T, D, false, false>(a, s);
}

bool al(const void* p, int bytes) { return ((uintptr_t)p % bytes) == 0; }

}  // namespace

bool pass_small_eligible(const PolyPassArgs& a) {
  if (a.seq_q < 1 || a.seq_q > kMaxN || a.seq_k < 1 || a.seq_k > kMaxN) return false;
  if (a.dtype != POLY_BF16 && a.dtype != POLY_F16) return false;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  if (a.key_mask || a.query_mask || a.v_mul || a.epi_out) return false;
  if (!al(a.k, 16) || !al(a.v, 16) || !al(a.q, 4) || !al(a.out, 4)) return false;
  if ((a.k_stride[0] | a.k_stride[1] | a.k_stride[2] | a.v_stride[0] | a.v_stride[1] | a.v_stride[2]) & 7)
    return false;
  if ((a.q_stride[0] | a.q_stride[1] | a.q_stride[2] | a.out_stride[0] | a.out_stride[1] | a.out_stride[2]) & 1)
    return false;
  return true;
}

int launch_pass_small(const PolyPassArgs& a, cudaStream_t s) {
  if (a.dtype == POLY_BF16)
    return a.head_dim == 64 ? launch_d<__nv_bfloat16, 64>(a, s) : launch_d<__nv_bfloat16, 128>(a, s);
  return a.head_dim == 64 ? launch_d<__half, 64>(a, s) : launch_d<__half, 128>(a, s);
}

}  // namespace poly
