// fp32 attention pass on the tensor cores with 3xTF32 (config 1's fp32
// PolyAttention forward, poly_attention/poly_attention.py:63-114): every
// product a.b is formed as a_hi.b_hi + a_hi.b_lo + a_lo.b_hi from the TF32
// split x_hi = tf32(x), x_lo = tf32(x - x_hi), which keeps the error near fp32
// rounding (the fp32 parity bar is 1e-4; plain TF32 would miss it).
//
// CTA = 64 query rows of one (batch, head), 4 warps x 16 rows; key tiles of 64
// through a 2-stage cp.async ring (rows padded to 68 floats: the fragment
// loads below are bank-conflict free). mma.sync m16n8k8 tf32. The score
// accumulator pairs keys (2t, 2t + 1) per lane; P.V uses that pairing as its
// K order (V rows are read in the same order), so P never moves between lanes.
// Online softmax in the log2 domain. Rows whose every key is excluded get the
// reference's -finfo.max result: a uniform average over the keys that are not
// both masked (causal) and dead (bias <= -FLT_MAX / 2), lse = -FLT_MAX.
#include <cfloat>
#include <mutex>

#include "common.cuh"

namespace poly {
namespace {

constexpr int D = 64, BM = 64, BN = 64, LD = D + 4;   // padded row pitch (floats)

__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void split(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32(x);
  lo = tf32(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma8(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// c += a.b in 3xTF32
__device__ __forceinline__ void mma3(float* c, const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0,
                                     uint32_t bh1, uint32_t bl0, uint32_t bl1) {
  mma8(c, al[0], al[1], al[2], al[3], bh0, bh1);
  mma8(c, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
  mma8(c, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
}
__device__ __forceinline__ void cp16(uint32_t sa, const void* g, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(g), "r"(ok ? 16 : 0) : "memory");
}

template <bool HAS_BIAS, bool SOFTCLAMP>
__global__ void __launch_bounds__(128) pass_f32_kernel(const PolyPassArgs a) {
  extern __shared__ __align__(16) float smf[];
  float(*sK)[BN * LD] = reinterpret_cast<float(*)[BN * LD]>(smf);
  float(*sV)[BN * LD] = reinterpret_cast<float(*)[BN * LD]>(smf + 2 * BN * LD);
  float(*sB)[BN] = reinterpret_cast<float(*)[BN]>(smf + 4 * BN * LD);
  const int bh = blockIdx.y;
  const int b = bh / a.heads, h = bh - b * a.heads, g = h / (a.heads / a.kv_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  const int i0 = blockIdx.x * BM + warp * 16 + gq, i1 = i0 + 8;   // this thread's two rows
  const int nq = a.seq_q, nk = a.seq_k;
  const float* kg = (const float*)a.k + b * a.k_stride[0] + g * a.k_stride[1];
  const float* vg = (const float*)a.v + b * a.v_stride[0] + g * a.v_stride[1];
  const float* bg = HAS_BIAS ? a.bias + b * a.bias_stride[0] + g * a.bias_stride[1] : nullptr;
  const int kend = a.causal ? min(nk, (int)blockIdx.x * BM + BM) : nk;
  const int ntile = (kend + BN - 1) / BN;

  auto issue = [&](int t) {
    const int st = t & 1, j0 = t * BN;
    for (int c = threadIdx.x; c < BN * (D / 4); c += 128) {
      const int r = c / (D / 4), ch = c - r * (D / 4);
      const bool ok = j0 + r < nk;
      const int rr = ok ? j0 + r : 0;
      cp16((uint32_t)__cvta_generic_to_shared(&sK[st][r * LD + ch * 4]), kg + (int64_t)rr * a.k_stride[2] + ch * 4, ok);
      cp16((uint32_t)__cvta_generic_to_shared(&sV[st][r * LD + ch * 4]), vg + (int64_t)rr * a.v_stride[2] + ch * 4, ok);
    }
    if (threadIdx.x < BN) {
      const int j = j0 + threadIdx.x;
      float x = 0.f;
      if (HAS_BIAS && j < nk) {
        const float raw = bg[j];
        x = raw <= kDeadBias ? -INFINITY : raw * kLog2e;
      }
      sB[st][threadIdx.x] = x;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  // Q split into TF32 hi / lo A fragments (rows i0 / i1, K steps of 8)
  uint32_t qh[D / 8][4], ql[D / 8][4];
  {
    const float* qb = (const float*)a.q + b * a.q_stride[0] + h * a.q_stride[1];
    const float* q0 = qb + (int64_t)(i0 < nq ? i0 : 0) * a.q_stride[2];
    const float* q1 = qb + (int64_t)(i1 < nq ? i1 : 0) * a.q_stride[2];
#pragma unroll
    for (int ks = 0; ks < D / 8; ++ks) {
      const float x[4] = {i0 < nq ? q0[ks * 8 + tq] : 0.f, i1 < nq ? q1[ks * 8 + tq] : 0.f,
                          i0 < nq ? q0[ks * 8 + tq + 4] : 0.f, i1 < nq ? q1[ks * 8 + tq + 4] : 0.f};
#pragma unroll
      for (int e = 0; e < 4; ++e) split(x[e], qh[ks][e], ql[ks][e]);
    }
  }
  const float qk = SOFTCLAMP ? a.scale / a.softclamp : a.scale * kLog2e;
  const float sc_out = SOFTCLAMP ? a.softclamp * kLog2e : 0.f;
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  if (ntile > 0) issue(0);
  for (int t = 0; t < ntile; ++t) {
    if (t + 1 < ntile) {
      issue(t + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const int st = t & 1, j0 = t * BN;
    const float* K = sK[st];
    const float* V = sV[st];
    // S = Q K^T: n-block nb = keys j0 + 8 nb .. + 7
    float s[BN / 8][4];
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
      const float* kr = K + (nb * 8 + gq) * LD;
#pragma unroll
      for (int ks = 0; ks < D / 8; ++ks) {
        uint32_t bh0, bl0, bh1, bl1;
        split(kr[ks * 8 + tq], bh0, bl0);
        split(kr[ks * 8 + tq + 4], bh1, bl1);
        mma3(s[nb], qh[ks], ql[ks], bh0, bh1, bl0, bl1);
      }
    }
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int jl = nb * 8 + 2 * tq + (e & 1), j = j0 + jl;
        const int row = e < 2 ? i0 : i1;
        float x = s[nb][e] * qk;
        if (SOFTCLAMP) x = tanhf(x) * sc_out;
        if (HAS_BIAS) x += sB[st][jl];
        if (j >= nk || (a.causal && j > row)) x = -INFINITY;
        s[nb][e] = x;
        if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float a0 = mx0 == -INFINITY ? 1.f : exp2f(m0 - mx0), a1 = mx1 == -INFINITY ? 1.f : exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    l0 *= a0;
    l1 *= a1;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= a0;
      o[n][1] *= a0;
      o[n][2] *= a1;
      o[n][3] *= a1;
    }
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = e < 2 ? m0 : m1;
        const float p = s[nb][e] == -INFINITY ? 0.f : exp2f(s[nb][e] - m);
        s[nb][e] = p;
        if (e < 2) l0 += p; else l1 += p;
      }
    // O += P V: K step = n-block nb, element (row, t) <-> key 8 nb + 2t, (row, t + 4) <-> key 8 nb + 2t + 1
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb) {
      uint32_t ph[4], pl[4];
      split(s[nb][0], ph[0], pl[0]);
      split(s[nb][2], ph[1], pl[1]);
      split(s[nb][1], ph[2], pl[2]);
      split(s[nb][3], ph[3], pl[3]);
      const float* v0 = V + (nb * 8 + 2 * tq) * LD;
      const float* v1 = v0 + LD;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        uint32_t bh0, bl0, bh1, bl1;
        split(v0[n * 8 + gq], bh0, bl0);
        split(v1[n * 8 + gq], bh1, bl1);
        mma3(o[n], ph, pl, bh0, bh1, bl0, bl1);
      }
    }
    __syncthreads();   // the stage is refilled next iteration
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  float* ob = (float*)a.out + b * a.out_stride[0] + h * a.out_stride[1];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int row = hf ? i1 : i0;
    const float m = hf ? m1 : m0, l = hf ? l1 : l0;
    if (row >= nq) continue;
    float lse;
    float r[D / 8][2];
    if (m == -INFINITY) {
      // every key excluded: uniform average over keys not both masked and dead
      int count = 0;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) r[n][0] = r[n][1] = 0.f;
      for (int j = 0; j < nk; ++j) {
        const bool masked = a.causal && j > row;
        const bool dead = HAS_BIAS && bg[j] <= kDeadBias;
        if (masked && dead) continue;
        ++count;
        const float* vr = vg + (int64_t)j * a.v_stride[2];
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          r[n][0] += vr[n * 8 + 2 * tq];
          r[n][1] += vr[n * 8 + 2 * tq + 1];
        }
      }
      const float inv = count ? 1.f / (float)count : 0.f;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        r[n][0] *= inv;
        r[n][1] *= inv;
      }
      lse = -FLT_MAX;
    } else {
      const float inv = 1.f / l;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        r[n][0] = o[n][2 * hf] * inv;
        r[n][1] = o[n][2 * hf + 1] * inv;
      }
      lse = (m + __log2f(l)) * kLn2;
    }
    float* orow = ob + (int64_t)row * a.out_stride[2];
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<float2*>(orow + n * 8 + 2 * tq) = make_float2(r[n][0], r[n][1]);
    if (a.lse && tq == 0) a.lse[b * a.lse_stride[0] + h * a.lse_stride[1] + row] = lse;
  }
}

bool al(const void* p, int bytes) { return ((uintptr_t)p % bytes) == 0; }

}  // namespace

bool pass_f32_eligible(const PolyPassArgs& a) {
  if (a.dtype != POLY_F32 || a.head_dim != D || a.seq_q < 1 || a.seq_k < 1) return false;
  if (a.key_mask || a.query_mask || a.v_mul || a.epi_out) return false;
  if (!al(a.k, 16) || !al(a.v, 16) || !al(a.out, 8)) return false;
  if ((a.k_stride[0] | a.k_stride[1] | a.k_stride[2] | a.v_stride[0] | a.v_stride[1] | a.v_stride[2]) & 3) return false;
  if ((a.out_stride[0] | a.out_stride[1] | a.out_stride[2]) & 1) return false;
  return true;
}

namespace {
constexpr int kSmem = (4 * BN * LD + 2 * BN) * 4;

template <bool B, bool C>
int launch_t(const PolyPassArgs& a, cudaStream_t s) {
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(pass_f32_kernel<B, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (err != cudaSuccess) return cuda_status(err, "cudaFuncSetAttribute(f32)");
  const dim3 grid((a.seq_q + BM - 1) / BM, a.batch * a.heads);
  pass_f32_kernel<B, C><<<grid, 128, kSmem, s>>>(a);
  return POLY_OK;
}
}  // namespace

int launch_pass_f32(const PolyPassArgs& a, cudaStream_t s) {
  const bool bias = a.bias != nullptr, sc = a.softclamp > 0.f;
  int rc;
  if (sc) rc = bias ? launch_t<true, true>(a, s) : launch_t<false, true>(a, s);
  else rc = bias ? launch_t<true, false>(a, s) : launch_t<false, false>(a, s);
  if (rc) return rc;
  note_launch(1);
  return cuda_status(cudaGetLastError(), "pass_f32 launch");
}

}  // namespace poly
