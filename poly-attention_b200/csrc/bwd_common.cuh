// Pieces shared by the tcgen05 backward kernels (bwd_tc100.cu: head_dim 64,
// bwd_tc128.cu: head_dim 128): kernel parameters, the per-element softmax
// backward, the dS^T tile store, and the prep / dQ-convert kernels around
// them.
#pragma once

#include "common.cuh"
#include "tc_ptx.cuh"

namespace poly {
namespace bwdc {
using namespace tc;

struct BwdParams {
  int seq_q, seq_k, heads, kv_heads, nq_pad, q_tiles, k_tiles, causal;
  float scale, sl2, sc_in, sc_out;
  const float* bias; int64_t bias_stride[2];
  float* dq_acc;                 // [b*heads][seq_q][head_dim] fp32
  const float* lse2;             // [b*heads][nq_pad] log2-domain lse (+inf padding)
  const float* delta;            // [b*heads][nq_pad]
  void* dk; int64_t dk_stride[3];
  void* dv; int64_t dv_stride[3];
  float* dbias; int64_t dbias_stride[2];
};

template <typename T>
__device__ __forceinline__ uint32_t pk(float a, float b);
template <>
__device__ __forceinline__ uint32_t pk<__nv_bfloat16>(float a, float b) { return pack_bf16(a, b); }
template <>
__device__ __forceinline__ uint32_t pk<__half>(float a, float b) { return pack_f16(a, b); }

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitNs) return;
}

// Writes 32 consecutive 16-bit values (one 32-query chunk c of row r) into a
// [128 rows][128 cols] tile stored as two 128-byte-swizzled 64-column atoms.
__device__ __forceinline__ void store_chunk(uint8_t* tile, int r, int c, const uint32_t (&w)[16]) {
  const int atom = c >> 1;
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int idx = (c & 1) * 4 + q4;
    uint4 val = make_uint4(w[q4 * 4 + 0], w[q4 * 4 + 1], w[q4 * 4 + 2], w[q4 * 4 + 3]);
    *reinterpret_cast<uint4*>(tile + atom * (128 * 128) + r * 128 + ((idx ^ (r & 7)) << 4)) = val;
  }
}

// One 32-query chunk of the softmax backward for this thread's key row.
// x = s * scale * log2(e) + bias - lse (log2 domain), p = 2^x,
// ds = p (dp - delta), d-bias += ds, dS = ds * softclamp'(s). MASK adds the
// causal diagonal (queries il < diag_row) and invalid-key masks; the
// unmasked variant is the common case and carries no per-element selects.
template <typename T, bool SOFTCLAMP, bool HAS_BIAS, bool MASK, bool DB>
__device__ __forceinline__ void softmax_bwd_chunk(const uint32_t (&sv)[32], const uint32_t (&dv)[32],
                                                  const float* nl, const float* dl, float b2, const BwdParams& p,
                                                  bool key_ok, int il0, int diag_row, float& dbias,
                                                  uint32_t (&pw)[16], uint32_t (&dw)[16]) {
  const float4* l4 = reinterpret_cast<const float4*>(nl);
  const float4* d4 = reinterpret_cast<const float4*>(dl);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 lq = l4[q], dq = d4[q];
    const float lv[4] = {lq.x, lq.y, lq.z, lq.w};
    const float dd4[4] = {dq.x, dq.y, dq.z, dq.w};
    float pp[4], dd[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int u = q * 4 + e;
      const float sr = __uint_as_float(sv[u]);
      const float off = HAS_BIAS ? lv[e] + b2 : lv[e];
      float x, dfac = 1.f;
      if (SOFTCLAMP) {
        const float th = tanhf(sr * p.sc_in);
        dfac = 1.f - th * th;
        x = fmaf(th, p.sc_out, off);
      } else {
        x = fmaf(sr, p.sl2, off);
      }
      float pr = ex2(x);
      if (MASK && (!key_ok || il0 + u < diag_row)) pr = 0.f;
      const float ds = pr * (__uint_as_float(dv[u]) - dd4[e]);
      if (DB) dbias += ds;   // only when the caller wants the key-bias gradient
      pp[e] = pr;
      dd[e] = SOFTCLAMP ? ds * dfac : ds;
    }
    pw[2 * q] = pk<T>(pp[0], pp[1]);
    pw[2 * q + 1] = pk<T>(pp[2], pp[3]);
    dw[2 * q] = pk<T>(dd[0], dd[1]);
    dw[2 * q + 1] = pk<T>(dd[2], dd[3]);
  }
}

// delta_i = dout_i . out_i - dlse_i and nlse2_i = -lse_i * log2(e), padded to
// nq_pad rows per (batch, head) with (delta 0, nlse2 -inf) so padded queries
// get p = 0. Eight lanes per row, 16-byte loads (D / 64 per lane).
template <typename T, int D>
__global__ void bwd_prep_kernel(const PolyPassBwdArgs a, float* lse2, float* delta, int nq_pad) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  const int sub = threadIdx.x & 7;
  const int64_t rows = (int64_t)a.fwd.batch * a.fwd.heads * nq_pad;
  if (w >= rows) return;
  const int i = (int)(w % nq_pad);
  const int bh = (int)(w / nq_pad);
  const int b = bh / a.fwd.heads, h = bh - b * a.fwd.heads;
  float s = 0.f;
  if (i < a.fwd.seq_q) {
    const T* o = (const T*)a.fwd.out + b * a.fwd.out_stride[0] + h * a.fwd.out_stride[1] +
                 (int64_t)i * a.fwd.out_stride[2] + sub * (D / 8);
    const T* g = (const T*)a.dout + b * a.dout_stride[0] + h * a.dout_stride[1] + (int64_t)i * a.dout_stride[2] +
                 sub * (D / 8);
#pragma unroll
    for (int v8 = 0; v8 < D / 64; ++v8) {
      const uint4 ov = *reinterpret_cast<const uint4*>(o + v8 * 8);
      const uint4 gv = *reinterpret_cast<const uint4*>(g + v8 * 8);
      const T* op = reinterpret_cast<const T*>(&ov);
      const T* gp = reinterpret_cast<const T*>(&gv);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += to_f32(op[e]) * to_f32(gp[e]);
    }
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  if (sub == 0) {
    if (i >= a.fwd.seq_q) {
      lse2[w] = -INFINITY;      // stored negated: padded queries get p = 2^-inf = 0
      delta[w] = 0.f;
    } else {
      if (a.dlse) s -= a.dlse[b * a.dlse_stride[0] + h * a.dlse_stride[1] + i];
      delta[w] = s;
      lse2[w] = -a.fwd.lse[b * a.fwd.lse_stride[0] + h * a.fwd.lse_stride[1] + i] * kLog2e;
    }
  }
}

// dq = scale * dq_acc (+ dq when accumulating), 8 elements per thread.
template <typename T, int D>
__global__ void bwd_dq_convert_kernel(const PolyPassBwdArgs a, const float* dq_acc) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)a.fwd.batch * a.fwd.heads * a.fwd.seq_q * (D / 8);
  if (idx >= total) return;
  const int c8 = (int)(idx % (D / 8));
  const int64_t row = idx / (D / 8);
  const int i = (int)(row % a.fwd.seq_q);
  const int bh = (int)(row / a.fwd.seq_q);
  const int b = bh / a.fwd.heads, h = bh - b * a.fwd.heads;
  const float* src = dq_acc + row * D + c8 * 8;
  T* dst = (T*)a.dq + b * a.dq_stride[0] + h * a.dq_stride[1] + (int64_t)i * a.dq_stride[2] + c8 * 8;
  const float4 x0 = *reinterpret_cast<const float4*>(src);
  const float4 x1 = *reinterpret_cast<const float4*>(src + 4);
  float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  const float sc = a.fwd.scale;
  if (a.dq_accumulate) {
    const uint4 old = *reinterpret_cast<const uint4*>(dst);
    const uint32_t* ow = &old.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const T* pr = reinterpret_cast<const T*>(&ow[e]);
      v[2 * e] = v[2 * e] * sc + to_f32(pr[0]);
      v[2 * e + 1] = v[2 * e + 1] * sc + to_f32(pr[1]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] *= sc;
  }
  uint4 out;
  uint32_t* w = &out.x;
#pragma unroll
  for (int e = 0; e < 4; ++e) w[e] = pk<T>(v[2 * e], v[2 * e + 1]);
  *reinterpret_cast<uint4*>(dst) = out;
}

struct BwdWs {
  float* dq_acc;
  float* lse2;
  float* delta;
  int nq_pad;
  size_t bytes;
};

// Workspace: fp32 dQ accumulator [b * heads][seq_q][D], then the log2-domain
// lse and delta rows padded to the query tile BQ.
template <int D, int BQ>
BwdWs bwd_ws(const PolyPassBwdArgs& a) {
  BwdWs w{};
  w.nq_pad = (a.fwd.seq_q + BQ - 1) / BQ * BQ;
  const size_t bh = (size_t)a.fwd.batch * a.fwd.heads;
  const size_t acc = (bh * a.fwd.seq_q * D * 4 + 255) / 256 * 256;
  const size_t vec = (bh * w.nq_pad * 4 + 255) / 256 * 256;
  w.bytes = acc + 2 * vec;
  char* base = (char*)a.workspace;
  w.dq_acc = (float*)base;
  w.lse2 = (float*)(base + acc);
  w.delta = (float*)(base + acc + vec);
  return w;
}

}  // namespace bwdc
}  // namespace poly
