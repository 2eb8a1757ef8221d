// KV-cache decode pass: one new query row per head against a long cache
// (seq_q == 1), HBM-bound. Replaces the reference's per-step materialised
// passes over the concatenated cache (poly_attention/poly_attention.py:63-114
// with cache, n_poly_attention.py:263-313 with cache).
//
// One launch per pass. The grid is (splits, batch * kv_heads), launched as
// thread-block clusters of `splits` CTAs along x: the cluster owns one
// (batch, kv head) group and CTA `split` streams keys [split * kps,
// (split + 1) * kps) of it exactly once, serving all R = heads / kv_heads
// query heads of the group.
//
// Keys arrive in 64-key stages: a producer warp fills a ring of stages with TMA
// tensor loads (128-byte swizzle, so ldmatrix reads are free of bank
// conflicts; rows past seq_k read as zeros) and the 64 per-key bias values with
// 4-byte cp.async, all completing on the stage's mbarrier. Each of the 4
// consumer warps takes 16 keys of a stage and computes, on the tensor cores
// (mma.sync m16n8k16, fp32 accumulation):
//   S[16 x 16]  = Q[16 x D] . K^T      (rows 0..R-1 are the group's heads,
//                                       rows R..15 are zero padding)
//   O[16 x D]  += P[16 x 16] . V'      (P from S's registers, V' = v * v_mul
//                                       rounded to the storage type, as the
//                                       order-n chain's v * msg)
// with an online softmax in the log2 domain (the per-key bias, the previous
// level's lse, added on the fly; lazy rescale when the running max grows by
// more than 2^8). The padding rows cost tensor-core issue slots only: with at
// most 8 real rows per 16 the pass stays HBM-bound by a wide margin, and
// tcgen05's smallest tile (M = 64) would waste more while adding TMEM round
// trips. The four warp states are merged through shared memory, then the
// cluster's CTA records are merged through distributed shared memory, and the
// cluster writes out, lse and the optional epilogue product: no partials go
// through HBM and no second kernel runs. With few groups (one long sequence)
// a global-split mode runs up to 64 splits per group instead and merges their
// records with a small combine kernel (workspace, see global_splits).
#include <cooperative_groups.h>

#include <cfloat>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace cg = cooperative_groups;

namespace poly {
namespace {

constexpr int kWarps = 4;
constexpr int kWarpKeys = 16;                 // keys per warp per stage (one m16n8k16 K step of P.V)
constexpr int kTile = kWarps * kWarpKeys;     // keys per stage
constexpr int kMaxSplits = 8;                 // portable cluster size
constexpr int kMaxGlobalSplits = 64;          // splits per group in the global-split mode
constexpr int kMinGlobalTiles = 16;           // key tiles per split, at least, in that mode
constexpr int kThreads = (kWarps + 1) * 32;  // warps 0..3 consume, warp 4 produces

// Shared memory: ring [stage][array (k, v, v_mul)][64 keys x D] (1024-byte
// aligned swizzled tiles), bias [stage][64] fp32, full / empty mbarriers and
// the abort flag. After the key loop the ring holds the merge records.
template <int D, int NARR>
__host__ __device__ constexpr int stage_bytes() { return NARR * kTile * D * 2; }
// ~100 KB of ring per CTA: two CTAs per SM, each with >= one stage in flight
template <int D, int NARR>
__host__ __device__ constexpr int num_stages() {
  return (100 * 1024) / stage_bytes<D, NARR>() < 2   ? 2
         : (100 * 1024) / stage_bytes<D, NARR>() > 4 ? 4
                                                      : (100 * 1024) / stage_bytes<D, NARR>();
}
template <int D, int R>
__host__ __device__ constexpr int record_bytes() { return (kWarps + 1) * R * (D + 2) * 4; }
template <int D, int R, int NARR>
__host__ __device__ constexpr int ring_bytes() {
  return num_stages<D, NARR>() * stage_bytes<D, NARR>() > record_bytes<D, R>()
             ? num_stages<D, NARR>() * stage_bytes<D, NARR>()
             : record_bytes<D, R>();
}
template <int D, int R, int NARR>
__host__ __device__ constexpr int smem_bytes() {   // + bias, barriers, flag, alignment slack
  return ring_bytes<D, R, NARR>() + num_stages<D, NARR>() * (kTile * 4 + 16) + 16 + 1024;
}

static __device__ int g_decode_error[2] = {0, 0};

__device__ __forceinline__ void cp_async4(uint32_t sa, const void* gmem, bool valid) {
  const int n = valid ? 4 : 0;   // zero-fill past the end
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sa), "l"(gmem), "r"(n) : "memory");
}
// arrive on `bar` once this thread's earlier cp.async copies have landed
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = tc::globaltimer();
  while (!tc::mbar_try_wait(bar, parity))
    if (tc::globaltimer() - t0 > tc::kWaitNs) return;
}

__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}

// c[4] += A[16x16] . B[16x8]; A rows 8..15 are zero (a1 = a3 = 0)
template <typename T>
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return tc::pack_bf16(lo, hi);
  else return tc::pack_f16(lo, hi);
}

// elementwise product of two packed pairs, rounded once to T (the product of
// two 16-bit values is exact in fp32, so this equals fp32 multiply + round)
template <typename T>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 p = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                     *reinterpret_cast<const __nv_bfloat162*>(&b));
    r = *reinterpret_cast<const uint32_t*>(&p);
  } else {
    const __half2 p = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    r = *reinterpret_cast<const uint32_t*>(&p);
  }
  return r;
}

// byte offset of 16-byte chunk `ch` of key row `key` inside one stage array:
// TMA boxes of 64 keys x 64 features (128-byte rows, 128-byte swizzle: chunk
// c of row r sits at c ^ (r & 7)), one box per 64 features
__device__ __forceinline__ uint32_t swz(int key, int ch) {
  return (uint32_t)((ch >> 3) * (kTile * 128) + key * 128 + (((ch & 7) ^ (key & 7)) << 4));
}

template <typename T, int D, int R, bool HAS_BIAS, bool HAS_VMUL, bool SOFTCLAMP>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                               const __grid_constant__ CUtensorMap tm_v,
                                                               const __grid_constant__ CUtensorMap tm_m,
                                                               const PolyPassArgs a, int kps, float* part) {
  constexpr int NARR = HAS_VMUL ? 3 : 2;
  constexpr int NST = num_stages<D, NARR>();
  constexpr int SB = stage_bytes<D, NARR>();
  constexpr int AB = kTile * D * 2;     // bytes of one array of a stage
  constexpr int KS = D / 16;            // K steps of Q.K^T
  constexpr int NB = D / 8;             // n8 column blocks of O
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = dsm_raw + ((1024 - (tc::smem_u32(dsm_raw) & 1023)) & 1023);
  const uint32_t sbase = tc::smem_u32(dsm);
  float* sbias = reinterpret_cast<float*>(dsm + ring_bytes<D, R, NARR>());   // [NST][kTile]
  uint64_t* full = reinterpret_cast<uint64_t*>(sbias + NST * kTile);
  uint64_t* empty = full + NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NST);
  int* err = g_decode_error;

  cg::cluster_group cluster = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.y;
  const int b = group / a.kv_heads, g = group - b * a.kv_heads;
  const int split = blockIdx.x;
  const int k0 = split * kps, k1 = min(a.seq_k, k0 + kps);
  const int ntile = k1 > k0 ? (k1 - k0 + kTile - 1) / kTile : 0;

  // dependents (the next pass of a decode chain) may start as this grid
  // drains; they wait for this grid before reading anything it writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(&full[s], HAS_BIAS ? 33 : 1);   // producer lane 0 (+ tx), + 32 bias lanes
      tc::mbar_init(&empty[s], kWarps);
    }
    tc::abort_init(abort_flag, err);
    tc::fence_barrier_init();
  }
  __syncthreads();

  float m = -INFINITY, l = 0.f;   // consumer state of row gq (quad-uniform m)
  float o[NB][4];
#pragma unroll
  for (int n = 0; n < NB; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  if (warp == kWarps) {
    // ------------------------------------------------------------ producer
    const float* bg = HAS_BIAS ? a.bias + b * a.bias_stride[0] + g * a.bias_stride[1] : nullptr;
    if (lane == 0) {
      tc::tma_prefetch_desc(&tm_k);
      tc::tma_prefetch_desc(&tm_v);
      if (HAS_VMUL) tc::tma_prefetch_desc(&tm_m);
    }
    int issued = 0;
    for (int t = 0; t < ntile; ++t) {
      const int s = t % NST;
      if (t >= NST && !tc::mbar_wait_warp(&empty[s], ((t / NST) - 1) & 1, abort_flag, err, 61)) break;
      const int kb = k0 + t * kTile;
      // the last key row may come from the previous pass of a decode chain:
      // wait for that grid first (a no-op without a programmatic dependency)
      if (kb + kTile >= a.seq_k) asm volatile("griddepcontrol.wait;" ::: "memory");
      uint8_t* st = dsm + s * SB;
      if (lane == 0) {
        tc::mbar_arrive_expect_tx(&full[s], SB);
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf) {
          tc::tma_load_4d(st + hf * (kTile * 128), &tm_k, &full[s], hf * 64, kb, g, b);
          tc::tma_load_4d(st + AB + hf * (kTile * 128), &tm_v, &full[s], hf * 64, kb, g, b);
          if (HAS_VMUL) tc::tma_load_4d(st + 2 * AB + hf * (kTile * 128), &tm_m, &full[s], hf * 64, kb, g, b);
        }
      }
      if (HAS_BIAS) {
#pragma unroll
        for (int e = 0; e < kTile / 32; ++e) {
          const int kl = lane + 32 * e, j = kb + kl;
          cp_async4(tc::smem_u32(sbias + s * kTile + kl), bg + (j < k1 ? j : k0), j < k1);
        }
        cp_async_arrive_noinc(&full[s]);
      }
      issued = t + 1;
    }
    if (*abort_flag) {   // let every copy in flight land before the CTA moves on
      for (int t = max(0, issued - NST); t < issued; ++t) drain_wait(&full[t % NST], (t / NST) & 1);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int gq = lane >> 2, tq = lane & 3;   // mma fragment row group / thread in group
    // Q as the A operand: row gq (< R) = head g * R + gq, K step ks holds
    // dims 16 ks + {2 tq, 2 tq + 1} and 16 ks + 8 + {2 tq, 2 tq + 1}
    uint32_t qa[KS][2];
    {
      const T* qrow = (const T*)a.q + b * a.q_stride[0] + (int64_t)(g * R + (gq < R ? gq : 0)) * a.q_stride[1];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const uint32_t lo = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * tq);
        const uint32_t hi = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * tq);
        qa[ks][0] = gq < R ? lo : 0u;
        qa[ks][1] = gq < R ? hi : 0u;
      }
    }
    const float qk_scale = SOFTCLAMP ? a.scale / a.softclamp : a.scale * kLog2e;
    const float sc_out = SOFTCLAMP ? a.softclamp * kLog2e : 0.f;
    const int wk0 = warp * kWarpKeys;
    for (int tile = 0; tile < ntile; ++tile) {
      const int s = tile % NST;
      if (!tc::mbar_wait_warp(&full[s], (tile / NST) & 1, abort_flag, err, 62)) break;
      const uint32_t sK = sbase + s * SB, sV = sK + AB, sM = sV + AB;
      const int kb = k0 + tile * kTile;

      // S = Q . K^T for keys wk0 .. wk0 + 15 (two n8 blocks)
      float sc[2][4];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
        const int key = wk0 + nb * 8 + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < KS; ks += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sK + swz(key, ks * 2 + (lane >> 3)), b0, b1, b2, b3);
          mma16816<T>(sc[nb], qa[ks][0], qa[ks][1], b0, b1);
          mma16816<T>(sc[nb], qa[ks + 1][0], qa[ks + 1][1], b2, b3);
        }
      }
      // scores of row gq, keys wk0 + nb * 8 + 2 tq + e, in the log2 domain
      float x[4];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kl = wk0 + nb * 8 + 2 * tq + e;
          float v = sc[nb][e] * qk_scale;
          if (SOFTCLAMP) v = tanhf(v) * sc_out;
          if (HAS_BIAS) {
            const float braw = sbias[s * kTile + kl];
            v = braw <= kDeadBias ? -INFINITY : v + braw * kLog2e;
          }
          x[nb * 2 + e] = kb + kl < k1 ? v : -INFINITY;
        }
      }
      float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      if (mx > m + 8.f) {   // lazy max: rescale only on large growth (quad-uniform)
        const float alpha = m == -INFINITY ? 0.f : exp2f(m - mx);
        m = mx;
        l *= alpha;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          o[n][0] *= alpha;
          o[n][1] *= alpha;
        }
      }
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) p[e] = x[e] == -INFINITY ? 0.f : exp2f(x[e] - m);
      l += (p[0] + p[1]) + (p[2] + p[3]);
      const uint32_t pa0 = pack2<T>(p[0], p[1]), pa2 = pack2<T>(p[2], p[3]);

      // O += P . V' : ldmatrix.trans gives V' as the B operand (keys x dims)
      const int vkey = wk0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int n2 = 0; n2 < NB / 2; ++n2) {
        const uint32_t off = swz(vkey, n2 * 2 + (lane >> 4));
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(sV + off, v0, v1, v2, v3);
        if (HAS_VMUL) {
          uint32_t m0, m1, m2, m3;
          ldsm_x4_t(sM + off, m0, m1, m2, m3);
          v0 = mul2<T>(v0, m0);
          v1 = mul2<T>(v1, m1);
          v2 = mul2<T>(v2, m2);
          v3 = mul2<T>(v3, m3);
        }
        mma16816<T>(o[2 * n2], pa0, pa2, v0, v1);
        mma16816<T>(o[2 * n2 + 1], pa0, pa2, v2, v3);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
  }
  __syncthreads();   // the ring is idle (every issued stage consumed or drained): reuse it

  // warp records [warp][row][m, l, acc[D]], then the CTA record [row][...]
  float* wrec = reinterpret_cast<float*>(dsm);
  float* crec = wrec + kWarps * R * (D + 2);
  if (warp < kWarps && (lane >> 2) < R) {
    const int gq = lane >> 2, tq = lane & 3;
    float* r = wrec + (warp * R + gq) * (D + 2);
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      r[2 + n * 8 + 2 * tq] = o[n][0];
      r[2 + n * 8 + 2 * tq + 1] = o[n][1];
    }
    if (tq == 0) {
      r[0] = m;
      r[1] = l;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < R * D; idx += kThreads) {
    const int rr = idx / D, c = idx - rr * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wrec[(w * R + rr) * (D + 2)]);
    float acc = 0.f, ls = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float* r = wrec + (w * R + rr) * (D + 2);
      const float f = r[0] == -INFINITY ? 0.f : exp2f(r[0] - M);
      acc = fmaf(r[2 + c], f, acc);
      ls = fmaf(r[1], f, ls);
    }
    crec[rr * (D + 2) + 2 + c] = acc;
    if (c == 0) {
      crec[rr * (D + 2)] = M;
      crec[rr * (D + 2) + 1] = ls;
    }
  }
  if (part) {
    // global-split mode: the CTA record goes to the workspace for the combine kernel
    __syncthreads();
    float* dstp = part + ((int64_t)group * gridDim.x + split) * R * (D + 2);
    for (int i = threadIdx.x; i < R * (D + 2); i += kThreads) dstp[i] = crec[i];
    return;
  }
  cluster.sync();   // CTA records visible to the whole cluster

  // cluster merge: CTA `split` writes its share of the group's R x D outputs
  const int nsp = gridDim.x;
  for (int idx = split * kThreads + threadIdx.x; idx < R * D; idx += nsp * kThreads) {
    const int rr = idx / D, c = idx - rr * D;
    float M = -INFINITY;
    for (int sp = 0; sp < nsp; ++sp) M = fmaxf(M, cluster.map_shared_rank(crec, sp)[rr * (D + 2)]);
    float acc = 0.f, L = 0.f;
    for (int sp = 0; sp < nsp; ++sp) {
      const float* r = cluster.map_shared_rank(crec, sp) + rr * (D + 2);
      const float ms = r[0];
      const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
      acc = fmaf(r[2 + c], f, acc);
      L = fmaf(r[1], f, L);
    }
    const int h = g * R + rr;
    float lse_v = (M + __log2f(L)) * kLn2;
    if (M == -INFINITY) {
      // every key dead: the reference's -finfo.max arithmetic gives the
      // uniform average of the values (decode has no masks), lse = -FLT_MAX
      const T* vg = (const T*)a.v + b * a.v_stride[0] + g * a.v_stride[1];
      const T* mg = HAS_VMUL ? (const T*)a.v_mul + b * a.v_mul_stride[0] + g * a.v_mul_stride[1] : nullptr;
      acc = 0.f;
      for (int j = 0; j < a.seq_k; ++j) {
        float vv = to_f32(vg[(int64_t)j * a.v_stride[2] + c]);
        if (HAS_VMUL) vv = to_f32(from_f32<T>(vv * to_f32(mg[(int64_t)j * a.v_mul_stride[2] + c])));
        acc += vv;
      }
      L = (float)a.seq_k;
      lse_v = -FLT_MAX;
    }
    const T ov = from_f32<T>(L > 0.f ? acc / L : 0.f);
    ((T*)a.out)[b * a.out_stride[0] + h * a.out_stride[1] + c] = ov;
    if (a.epi_out) {
      const T em = ((const T*)a.epi_mul)[b * a.epi_mul_stride[0] + h * a.epi_mul_stride[1] + c];
      ((T*)a.epi_out)[b * a.epi_out_stride[0] + h * a.epi_out_stride[1] + c] = from_f32<T>(to_f32(em) * to_f32(ov));
    }
    if (a.lse && c == 0) a.lse[b * a.lse_stride[0] + h * a.lse_stride[1]] = lse_v;
  }
  cluster.sync();   // no CTA leaves while its record may still be read
}

}  // namespace

int read_device_error_dec(int* out, bool reset) {
  int rc = cuda_status(cudaMemcpyFromSymbol(out, g_decode_error, sizeof(int)), "read device error word");
  if (rc == POLY_OK && reset) {
    const int zero = 0;
    rc = cuda_status(cudaMemcpyToSymbol(g_decode_error, &zero, sizeof(int)), "reset device error word");
  }
  return rc;
}

namespace {

// Global-split mode: one CTA per (group, query head of the group) merges the
// `nsp` CTA records of the row. The records' weights go to shared memory
// first; then 8 slices of 32 threads each sum every 8th record over the
// features (independent loads, so the records stream in parallel rather than
// one L2 round trip per record), the slices add up in shared memory, and the
// CTA writes out, lse and the epilogue product as the cluster path does.
constexpr int kCombThreads = 256, kCombSlices = kCombThreads / 32;

template <typename T, int D, int R, bool HAS_VMUL>
__global__ void __launch_bounds__(kCombThreads) decode_combine_kernel(const PolyPassArgs a, const float* part,
                                                                       int nsp) {
  __shared__ float sf[kMaxGlobalSplits], sl[kMaxGlobalSplits];
  __shared__ float red[kCombSlices][D];
  __shared__ float sM, sL;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, slice = tid >> 5;
  const int group = row / R, rr = row - group * R;
  const int b = group / a.kv_heads, g = group - b * a.kv_heads, h = g * R + rr;
  auto rec = [&](int sp) { return part + (((int64_t)group * nsp + sp) * R + rr) * (D + 2); };
  // the split kernel's records are complete once the primary grid is
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid < nsp) {
    sf[tid] = rec(tid)[0];
    sl[tid] = rec(tid)[1];
  }
  __syncthreads();
  if (slice == 0) {
    float m = -INFINITY;
    for (int sp = lane; sp < nsp; sp += 32) m = fmaxf(m, sf[sp]);
    m = warp_max(m);
    float l = 0.f;
    for (int sp = lane; sp < nsp; sp += 32) l += sf[sp] == -INFINITY ? 0.f : sl[sp] * exp2f(sf[sp] - m);
    l = warp_sum(l);
    __syncwarp();
    for (int sp = lane; sp < nsp; sp += 32) sf[sp] = sf[sp] == -INFINITY ? 0.f : exp2f(sf[sp] - m);
    if (lane == 0) {
      sM = m;
      sL = l;
    }
  }
  __syncthreads();
  float o[D / 32];
#pragma unroll
  for (int t = 0; t < D / 32; ++t) o[t] = 0.f;
#pragma unroll 4
  for (int sp = slice; sp < nsp; sp += kCombSlices) {
    const float f = sf[sp];
    const float* r = rec(sp) + 2;
#pragma unroll
    for (int t = 0; t < D / 32; ++t) o[t] = fmaf(r[lane + 32 * t], f, o[t]);
  }
#pragma unroll
  for (int t = 0; t < D / 32; ++t) red[slice][lane + 32 * t] = o[t];
  __syncthreads();
  if (tid >= D) return;
  const int c = tid;
  const float M = sM, L = sL;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < kCombSlices; ++k) acc += red[k][c];
  float inv = L > 0.f ? 1.f / L : 0.f, lse_v = (M + __log2f(L)) * kLn2;
  if (M == -INFINITY) {
    // every key dead: the reference's uniform average of the values, lse = -FLT_MAX
    const T* vg = (const T*)a.v + b * a.v_stride[0] + g * a.v_stride[1];
    const T* mg = HAS_VMUL ? (const T*)a.v_mul + b * a.v_mul_stride[0] + g * a.v_mul_stride[1] : nullptr;
    acc = 0.f;
    for (int j = 0; j < a.seq_k; ++j) {
      float vv = to_f32(vg[(int64_t)j * a.v_stride[2] + c]);
      if (HAS_VMUL) vv = to_f32(from_f32<T>(vv * to_f32(mg[(int64_t)j * a.v_mul_stride[2] + c])));
      acc += vv;
    }
    inv = a.seq_k > 0 ? 1.f / (float)a.seq_k : 0.f;
    lse_v = -FLT_MAX;
  }
  const T ov = from_f32<T>(acc * inv);
  ((T*)a.out)[b * a.out_stride[0] + h * a.out_stride[1] + c] = ov;
  if (a.epi_out) {
    const T em = ((const T*)a.epi_mul)[b * a.epi_mul_stride[0] + h * a.epi_mul_stride[1] + c];
    ((T*)a.epi_out)[b * a.epi_out_stride[0] + h * a.epi_out_stride[1] + c] = from_f32<T>(to_f32(em) * to_f32(ov));
  }
  if (a.lse && c == 0) a.lse[b * a.lse_stride[0] + h * a.lse_stride[1]] = lse_v;
}

struct DecodeGeom {
  int splits, kps;  // key splits (cluster size) and keys per split
};

// Splits per group: the most (<= kMaxSplits) that still fit every CTA of the
// grid into one wave (`slots` = resident CTAs per SM x SMs), so that each CTA
// streams one long key range and pays its pipeline ramp-up and merge once;
// at least one 64-key tile per split.
DecodeGeom geometry(const PolyPassArgs& a, int slots) {
  const int groups = a.batch * a.kv_heads;
  const int ntiles = (a.seq_k + kTile - 1) / kTile;
  int splits = max(1, min(kMaxSplits, slots / max(groups, 1)));
  splits = max(1, min(splits, ntiles));
  DecodeGeom gm;
  gm.kps = max(kTile, ((a.seq_k + splits - 1) / splits + kTile - 1) / kTile * kTile);
  gm.splits = max(1, (a.seq_k + gm.kps - 1) / gm.kps);
  return gm;
}

// Global-split mode, for few (batch, kv head) groups (e.g. one long sequence):
// clusters of <= kMaxSplits CTAs cannot fill the GPU there, so up to
// kMaxGlobalSplits splits per group write their CTA records to the workspace
// and a combine kernel merges them. The choice and the split count depend on
// the SM count only, so the workspace size and the launch agree.

int sm_count() {
  static std::mutex mu;
  static int sms_dev[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lk(mu);
  if (!sms_dev[dev]) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sms_dev[dev] = max(1, sms);
  }
  return sms_dev[dev];
}

// splits of the global-split mode, or 0 when the cluster path is used: the
// mode is taken only where it gives more splits than a cluster can hold, with
// every split still streaming >= kMinGlobalTiles tiles (fewer, and the
// pipeline ramp-up of each CTA costs more than the extra CTAs gain) and the
// whole grid inside one wave of two CTAs per SM
int global_splits(const PolyPassArgs& a) {
  const int groups = max(1, a.batch * a.kv_heads);
  const int ntiles = (a.seq_k + kTile - 1) / kTile;
  const int target = 2 * sm_count();
  const int want = min(kMaxGlobalSplits, min(ntiles / kMinGlobalTiles, target / groups));
  if (want <= kMaxSplits) return 0;
  const int kps = ((a.seq_k + want - 1) / want + kTile - 1) / kTile * kTile;
  return (a.seq_k + kps - 1) / kps;
}

// (batch, kv head, row) strides for a tensor map: the stride of an extent-1
// dimension is never used, so it is replaced by one TMA accepts
void map_strides(const int64_t* st, const PolyPassArgs& a, int64_t* out) {
  out[2] = st[2] > 0 ? st[2] : a.head_dim;
  out[1] = (a.kv_heads == 1 || st[1] <= 0) ? out[2] * max(a.seq_k, 1) : st[1];
  out[0] = (a.batch == 1 || st[0] <= 0) ? out[1] * a.kv_heads : st[0];
}

template <typename T, int D, int R, bool B, bool V, bool C>
int launch_one(const PolyPassArgs& a, cudaStream_t s, bool dependent) {
  constexpr int smem = smem_bytes<D, R, V ? 3 : 2>();
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(decode_split_kernel<T, D, R, B, V, C>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (attr_err != cudaSuccess) return cuda_status(attr_err, "cudaFuncSetAttribute(decode)");
  // resident CTAs per SM x SMs of the current device (cached per device)
  static std::mutex mu;
  static int slots_dev[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  int slots;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!slots_dev[dev]) {
      int per_sm = 0, sms = 0;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_split_kernel<T, D, R, B, V, C>, kThreads, smem);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      slots_dev[dev] = max(1, per_sm) * max(1, sms);
    }
    slots = slots_dev[dev];
  }
  DecodeGeom gm = geometry(a, slots);
  const int gsp = global_splits(a);
  float* part = nullptr;
  if (gsp > 0) {
    gm.splits = gsp;
    gm.kps = ((a.seq_k + gsp - 1) / gsp + kTile - 1) / kTile * kTile;
    part = (float*)a.workspace;
  }
  CUtensorMap tk, tv, tm;
  const int rows = max(a.seq_k, 1);   // seq_k == 0 issues no load
  int64_t ks[3], vs[3], ms[3];
  map_strides(a.k_stride, a, ks);
  map_strides(a.v_stride, a, vs);
  int rc = make_map(&tk, a.k, a.dtype, D, rows, a.kv_heads, a.batch, ks, kTile);
  if (!rc) rc = make_map(&tv, a.v, a.dtype, D, rows, a.kv_heads, a.batch, vs, kTile);
  memset(&tm, 0, sizeof(tm));
  if (!rc && V) {
    map_strides(a.v_mul_stride, a, ms);
    rc = make_map(&tm, a.v_mul, a.dtype, D, rows, a.kv_heads, a.batch, ms, kTile);
  }
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gm.splits, a.batch * a.kv_heads);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = part ? 1 : gm.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_split_kernel<T, D, R, B, V, C>, tk, tv, tm, a, gm.kps, part);
  note_launch(1);
  if (e == cudaSuccess && part) {
    // programmatic dependent of the split kernel: it waits (griddepcontrol)
    // for the records, and lets the next pass of a chain start its prologue
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3(a.batch * a.kv_heads * R);
    cc.blockDim = dim3(kCombThreads);
    cc.stream = s;
    cc.attrs = &attr[1];
    cc.numAttrs = 1;
    e = cudaLaunchKernelEx(&cc, decode_combine_kernel<T, D, R, V>, a, (const float*)part, gm.splits);
    note_launch(1);
  }
  return cuda_status(e, "decode launch");
}

template <typename T, int D, int R>
int launch3(const PolyPassArgs& a, cudaStream_t s, bool dep) {
  const bool bias = a.bias != nullptr, vm = a.v_mul != nullptr, sc = a.softclamp > 0.f;
  if (sc) {
    if (bias) return vm ? launch_one<T, D, R, true, true, true>(a, s, dep) : launch_one<T, D, R, true, false, true>(a, s, dep);
    return vm ? launch_one<T, D, R, false, true, true>(a, s, dep) : launch_one<T, D, R, false, false, true>(a, s, dep);
  }
  if (bias) return vm ? launch_one<T, D, R, true, true, false>(a, s, dep) : launch_one<T, D, R, true, false, false>(a, s, dep);
  return vm ? launch_one<T, D, R, false, true, false>(a, s, dep) : launch_one<T, D, R, false, false, false>(a, s, dep);
}

template <typename T, int D>
int launch2(const PolyPassArgs& a, cudaStream_t s, bool dep) {
  switch (a.heads / a.kv_heads) {
    case 1: return launch3<T, D, 1>(a, s, dep);
    case 2: return launch3<T, D, 2>(a, s, dep);
    case 4: return launch3<T, D, 4>(a, s, dep);
    default: return launch3<T, D, 8>(a, s, dep);
  }
}

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
  // TMA needs positive strides wherever the extent exceeds one
  auto pos = [&](const int64_t* st) {
    return (a.seq_k <= 1 || st[2] > 0) && (a.kv_heads == 1 || st[1] > 0) && (a.batch == 1 || st[0] > 0);
  };
  if (!pos(a.k_stride) || !pos(a.v_stride) || (a.v_mul && !pos(a.v_mul_stride))) return false;
  return true;
}

// partials never leave the cluster: no workspace
// partials go through the workspace only in the global-split mode
size_t pass_decode_workspace(const PolyPassArgs& a) {
  // A fixed bound (the most splits any length can take) rather than this
  // length's split count: once a cache is long enough for the global mode it
  // stays there as it grows, so a workspace sized at the cache's capacity
  // covers every shorter length too.
  if (!global_splits(a)) return 0;
  return (size_t)a.batch * a.kv_heads * kMaxGlobalSplits * (a.heads / a.kv_heads) * (a.head_dim + 2) * sizeof(float);
}

int launch_pass_decode(const PolyPassArgs& a, cudaStream_t s, bool dependent) {
  if (a.dtype == POLY_BF16)
    return a.head_dim == 64 ? launch2<__nv_bfloat16, 64>(a, s, dependent)
                            : launch2<__nv_bfloat16, 128>(a, s, dependent);
  return a.head_dim == 64 ? launch2<__half, 64>(a, s, dependent) : launch2<__half, 128>(a, s, dependent);
}

}  // namespace poly
