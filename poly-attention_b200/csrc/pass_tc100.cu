// tcgen05 / TMEM / TMA forward kernel for one poly-attention pass (sm_100a).
//
// One CTA computes a 128-query tile of one (batch, head) against all visible
// 128-key tiles (flash-style online softmax), replacing the Triton forward
// kernel (poly_attention/flash_poly_attention.py:21-154) used for both passes.
//
// Warp roles (256 threads):
//   warp 0      TMA producer: Q once, then K / V tiles through a ring of stages
//   warp 1      TMEM allocator + MMA issuer (one thread):
//                 S[j%2] = Q K_j^T   (M=128, N=128, K=D, both K-major, fp32 in TMEM)
//                 O     += P_j V_j   (M=128, N=D,  K=128, P K-major, V MN-major)
//   warps 4-7   softmax / correction / epilogue: thread t owns query row t,
//               i.e. TMEM lane t. Reads S with tcgen05.ld, adds the per-key
//               bias (pass 2's lse23, poly_attention/poly_attention.py:109),
//               online softmax in the log2 domain, rescales O in TMEM when the
//               row max grows, writes P (bf16/fp16, 128B-swizzled) to smem.
//
// Shared memory tiles are 128-byte swizzled (one 64-element atom per row
// chunk); TMEM holds two S buffers (2 x 128 columns) and O (D columns).
#include <cstdlib>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "tc_ptx.cuh"
#include "tc_host.cuh"

namespace poly {

// Device error word of this file's kernels: set by bounded waits that gave up.
// (Without relocatable device code every .cu file has its own; the host
// combines them in poly_device_error.)
static __device__ int g_poly_device_error[2] = {0, 0};

int read_device_error_fwd(int* out, bool reset) {
  int rc = cuda_status(cudaMemcpyFromSymbol(out, g_poly_device_error, sizeof(int)), "read device error word");
  if (rc == POLY_OK && reset) {
    const int zero = 0;
    rc = cuda_status(cudaMemcpyToSymbol(g_poly_device_error, &zero, sizeof(int)), "reset device error word");
  }
  return rc;
}

namespace {
using namespace tc;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int kFwdThreads = 256;
constexpr int kSoftmaxWarp0 = 4;

template <int D>
struct FwdLayout {
  static constexpr int kStages = (D == 64) ? 3 : 2;
  static constexpr int kQBytes = BM * D * 2;
  static constexpr int kKVBytes = BN * D * 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;
  static constexpr int kV = kK + kStages * kKVBytes;
  static constexpr int kP = kV + kStages * kKVBytes;
  static constexpr int kBias = kP + BM * BN * 2;        // 2 x BN floats
  static constexpr int kBar = kBias + 2 * BN * 4;       // mbarriers
  static constexpr int kNumBars = 1 + 3 * kStages + 2 + 3 + 2;
  static constexpr int kMisc = kBar + kNumBars * 8;     // tmem slot + abort flag
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;          // slack for 1024-byte alignment
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kTmemS = 0;                 // two S buffers: columns [0, 256)
  static constexpr uint32_t kTmemO = 256;               // O: columns [256, 256 + D)
};

struct FwdParams {
  int seq_q, seq_k, heads, kv_heads, m_tiles, causal;
  float sl2;          // scale * log2(e)
  float softclamp;    // > 0: c * tanh(s / c)
  float sc_in;        // scale / c
  float sc_out;       // c * log2(e)
  const float* bias; int64_t bias_stride[2];
  void* out; int64_t out_stride[3];
  float* lse; int64_t lse_stride[2];
  const void* epi_mul; int64_t epi_mul_stride[3];
  void* epi_out; int64_t epi_out_stride[3];
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) { return pack_bf16(a, b); }
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) { return pack_f16(a, b); }

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<__half2*>(&u));
}

// Bounded wait that ignores the abort flag: used only to drain copies and
// MMAs already in flight before the CTA exits.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitNs) return;
}

template <int D, typename T, bool HAS_BIAS, bool SOFTCLAMP>
__global__ void __launch_bounds__(kFwdThreads, 1)
    pass_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using L = FwdLayout<D>;
  constexpr int S = L::kStages;
  constexpr int ND = D / 64;               // 64-element (128-byte) swizzle atoms per row
  constexpr int kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint8_t* sP = smem + L::kP;
  float* sBias = (float*)(smem + L::kBias);
  uint64_t* bars = (uint64_t*)(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 1 + S;
  uint64_t* kv_empty = bars + 1 + 2 * S;
  uint64_t* s_full = bars + 1 + 3 * S;
  uint64_t* p_full = bars + 3 + 3 * S;
  uint64_t* o_done = bars + 4 + 3 * S;
  uint64_t* drain = bars + 5 + 3 * S;
  uint64_t* bias_ready = bars + 6 + 3 * S;   // [2]
  uint32_t* tmem_slot = (uint32_t*)(smem + L::kMisc);
  volatile int* abort_flag = (volatile int*)(smem + L::kMisc + 4);
  int* err = g_poly_device_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid: x = (batch, head), y = query tile, heaviest first (longest-first dispatch)
  const int b = blockIdx.x / p.heads, h = blockIdx.x - b * p.heads;
  const int kvh = h / (p.heads / p.kv_heads);
  const int mt = p.causal ? (p.m_tiles - 1 - (int)blockIdx.y) : (int)blockIdx.y;
  const int row0 = mt * BM;
  const int kt_total = (p.seq_k + BN - 1) / BN;
  const int nt = p.causal ? min(kt_total, mt + 1) : kt_total;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    mbar_init(&bias_ready[0], 128);
    mbar_init(&bias_ready[1], 128);
    tc::abort_init(abort_flag, err);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(q_full, L::kQBytes);
      for (int c = 0; c < ND; ++c) tma_load_4d(sQ + c * BM * 128, &tm_q, q_full, c * 64, row0, h, b);
      int issued = 0;
      for (int j = 0; j < nt; ++j) {
        const int s = j % S;
        if (j >= S && !mbar_wait(&kv_empty[s], ((j / S) - 1) & 1, abort_flag, err, 21)) break;
        mbar_arrive_expect_tx(&k_full[s], L::kKVBytes);
        for (int c = 0; c < ND; ++c)
          tma_load_4d(sK + s * L::kKVBytes + c * BN * 128, &tm_k, &k_full[s], c * 64, j * BN, kvh, b);
        mbar_arrive_expect_tx(&v_full[s], L::kKVBytes);
        for (int c = 0; c < ND; ++c)
          tma_load_4d(sV + s * L::kKVBytes + c * BN * 128, &tm_v, &v_full[s], c * 64, j * BN, kvh, b);
        issued = j + 1;
      }
      if (*abort_flag) {
        drain_wait(q_full, 0);
        for (int j = max(0, issued - S); j < issued; ++j) {
          drain_wait(&k_full[j % S], (j / S) & 1);
          drain_wait(&v_full[j % S], (j / S) & 1);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idS = idesc_f16(BM, BN, kIsBf16, 0, 0);
      constexpr uint32_t idO = idesc_f16(BM, D, kIsBf16, 0, 1);
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK), va = smem_u32(sV), pa = smem_u32(sP);
      auto issue_s = [&](int j) -> bool {
        const int s = j % S;
        if (!mbar_wait(&k_full[s], (j / S) & 1, abort_flag, err, 22)) return false;
        tc_fence_after();
        const uint32_t d_t = tmem + L::kTmemS + (uint32_t)(j & 1) * BN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * (BM * 128) + (uint32_t)(kk & 3) * 32;
          mma_f16_ss(d_t, smem_desc_sw128(qa + off, 16, 1024),
                     smem_desc_sw128(ka + s * L::kKVBytes + off, 16, 1024), idS, kk > 0);
        }
        mma_commit(&s_full[j & 1]);
        return true;
      };
      if (mbar_wait(q_full, 0, abort_flag, err, 23) && issue_s(0)) {
        for (int j = 0; j < nt; ++j) {
          if (j + 1 < nt && !issue_s(j + 1)) break;
          if (!mbar_wait(p_full, j & 1, abort_flag, err, 24)) break;
          const int s = j % S;
          if (!mbar_wait(&v_full[s], (j / S) & 1, abort_flag, err, 25)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint32_t aoff = (uint32_t)(kk >> 2) * (BM * 128) + (uint32_t)(kk & 3) * 32;
            mma_f16_ss(tmem + L::kTmemO, smem_desc_sw128(pa + aoff, 16, 1024),
                       smem_desc_sw128(va + s * L::kKVBytes + kk * 2048, BN * 128, 1024), idO, (j > 0 || kk > 0));
          }
          mma_commit(&kv_empty[s]);
          mma_commit(o_done);
        }
      }
      mma_commit(drain);
      drain_wait(drain, 0);
    }
  } else if (warp >= kSoftmaxWarp0) {
    // -------------------------------------------------- softmax / epilogue
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int tid = threadIdx.x - kSoftmaxWarp0 * 32;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const float* bias = HAS_BIAS ? p.bias + b * p.bias_stride[0] + kvh * p.bias_stride[1] : nullptr;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    int nbias = 0;
    for (int j = 0; j < nt && ok; ++j) {
      const bool tail = (j == kt_total - 1) && (p.seq_k % BN) != 0;
      const bool use_bias = HAS_BIAS || tail;
      if (use_bias) {
        const int key = j * BN + tid;
        float bv = -INFINITY;
        if (key < p.seq_k) {
          bv = 0.f;
          if (HAS_BIAS) {
            const float braw = bias[key];
            bv = braw <= kDeadBias ? -INFINITY : braw * kLog2e;
          }
        }
        // bias tiles are counted separately: without a bias only the tail tile uses one
        sBias[(nbias & 1) * BN + tid] = bv;
        mbar_arrive(&bias_ready[nbias & 1]);
        if (!mbar_wait_warp(&bias_ready[nbias & 1], (nbias >> 1) & 1, abort_flag, err, 26)) { ok = false; break; }
      }
      if (!mbar_wait_warp(&s_full[j & 1], (j >> 1) & 1, abort_flag, err, 27)) { ok = false; break; }
      tc_fence_after();
      uint32_t v[BN];
      const uint32_t s_addr = tmem + lane_base + L::kTmemS + (uint32_t)(j & 1) * BN;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tmem_wait_ld();
      const float* bt = sBias + (nbias & 1) * BN;
      if (use_bias) ++nbias;
      const bool diag = p.causal && (j == mt);
      float tmax = -INFINITY;
      // without softclamp or bias the scale is folded into the exponent's FFMA
      const bool fold = !SOFTCLAMP && !use_bias;
      if (SOFTCLAMP) {
#pragma unroll
        for (int c = 0; c < BN; ++c) v[c] = __float_as_uint(tanhf(__uint_as_float(v[c]) * p.sc_in) * p.sc_out);
        if (use_bias) {
#pragma unroll
          for (int c = 0; c < BN; ++c) v[c] = __float_as_uint(__uint_as_float(v[c]) + bt[c]);
        }
      } else if (use_bias) {
#pragma unroll
        for (int c = 0; c < BN; ++c) v[c] = __float_as_uint(fmaf(__uint_as_float(v[c]), p.sl2, bt[c]));
      }
      if (diag) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c > r) v[c] = __float_as_uint(-INFINITY);
      }
#pragma unroll
      for (int c = 0; c < BN; ++c) tmax = fmaxf(tmax, __uint_as_float(v[c]));
      if (fold) tmax *= p.sl2;
      // lazy max: the running max (and O in TMEM) moves only when a row's max
      // grows by more than 2^8; exponentials stay <= 2^8, exact in fp32 sums
      float alpha = 1.f;
      if (tmax > m_run + 8.f) {
        alpha = ex2(m_run - tmax);
        m_run = tmax;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      float sum = 0.f;
      if (fold) {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const float e = ex2(fmaf(__uint_as_float(v[c]), p.sl2, -m_use));
          sum += e;
          v[c] = __float_as_uint(e);
        }
      } else {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const float e = ex2(__uint_as_float(v[c]) - m_use);
          sum += e;
          v[c] = __float_as_uint(e);
        }
      }
      l_run = l_run * alpha + sum;
      if (j > 0) {
        // PV_{j-1} must be complete before O is rescaled and P is overwritten
        if (!mbar_wait_warp(o_done, (j - 1) & 1, abort_flag, err, 28)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
          const uint32_t o_addr = tmem + lane_base + L::kTmemO;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(o_addr + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
            tmem_st32(o_addr + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      // P row -> smem, 128-byte swizzled K-major (two 64-key atoms)
#pragma unroll
      for (int c = 0; c < BN / 8; ++c) {
        const int atom = c >> 3, cc = c & 7;
        uint4 val;
        val.x = pack2<T>(__uint_as_float(v[c * 8 + 0]), __uint_as_float(v[c * 8 + 1]));
        val.y = pack2<T>(__uint_as_float(v[c * 8 + 2]), __uint_as_float(v[c * 8 + 3]));
        val.z = pack2<T>(__uint_as_float(v[c * 8 + 4]), __uint_as_float(v[c * 8 + 5]));
        val.w = pack2<T>(__uint_as_float(v[c * 8 + 6]), __uint_as_float(v[c * 8 + 7]));
        *reinterpret_cast<uint4*>(sP + atom * (BM * 128) + r * 128 + ((cc ^ (r & 7)) << 4)) = val;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait_warp(o_done, (nt - 1) & 1, abort_flag, err, 29)) {
      tc_fence_after();
      const int row = row0 + r;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T* out = (T*)p.out + b * p.out_stride[0] + h * p.out_stride[1] + (int64_t)row * p.out_stride[2];
      const T* em = p.epi_out ? (const T*)p.epi_mul + b * p.epi_mul_stride[0] + h * p.epi_mul_stride[1] +
                                    (int64_t)row * p.epi_mul_stride[2]
                              : nullptr;
      T* eo = p.epi_out ? (T*)p.epi_out + b * p.epi_out_stride[0] + h * p.epi_out_stride[1] +
                              (int64_t)row * p.epi_out_stride[2]
                        : nullptr;
      const uint32_t o_addr = tmem + lane_base + L::kTmemO;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_addr + c * 32, o);
        tmem_wait_ld();
        if (row < p.seq_q) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 val;
            uint32_t* w = &val.x;
#pragma unroll
            for (int t = 0; t < 4; ++t)
              w[t] = pack2<T>(__uint_as_float(o[q4 * 8 + 2 * t]) * inv, __uint_as_float(o[q4 * 8 + 2 * t + 1]) * inv);
            *reinterpret_cast<uint4*>(out + c * 32 + q4 * 8) = val;
            if (eo) {
              const uint4 mv = *reinterpret_cast<const uint4*>(em + c * 32 + q4 * 8);
              const uint32_t* mw = &mv.x;
              uint4 ev;
              uint32_t* ew = &ev.x;
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const float2 a = unpack2<T>(w[t]), m2 = unpack2<T>(mw[t]);
                ew[t] = pack2<T>(a.x * m2.x, a.y * m2.y);
              }
              *reinterpret_cast<uint4*>(eo + c * 32 + q4 * 8) = ev;
            }
          }
        }
      }
      if (p.lse && row < p.seq_q)
        p.lse[b * p.lse_stride[0] + h * p.lse_stride[1] + row] = (m_run + __log2f(l_run)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, L::kTmemCols);
}

// ---------------------------------------------------------------- host side

template <int D, typename T, bool HAS_BIAS, bool SOFTCLAMP>
int launch_fwd_tc_t(const PolyPassArgs& a, cudaStream_t s) {
  using L = FwdLayout<D>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(pass_fwd_tc_kernel<D, T, HAS_BIAS, SOFTCLAMP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    L::kAlloc);
  });
  if (attr_err != cudaSuccess) return cuda_status(attr_err, "cudaFuncSetAttribute(fwd tc)");
  CUtensorMap tq, tk, tv;
  int rc = make_map(&tq, a.q, a.dtype, D, a.seq_q, a.heads, a.batch, a.q_stride, BM);
  if (!rc) rc = make_map(&tk, a.k, a.dtype, D, a.seq_k, a.kv_heads, a.batch, a.k_stride, BN);
  if (!rc) rc = make_map(&tv, a.v, a.dtype, D, a.seq_k, a.kv_heads, a.batch, a.v_stride, BN);
  if (rc) return rc;
  FwdParams p{};
  p.seq_q = a.seq_q;
  p.seq_k = a.seq_k;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.m_tiles = (a.seq_q + BM - 1) / BM;
  p.causal = a.causal;
  p.sl2 = a.scale * kLog2e;
  p.softclamp = a.softclamp;
  p.sc_in = a.softclamp > 0.f ? a.scale / a.softclamp : 0.f;
  p.sc_out = a.softclamp * kLog2e;
  p.bias = a.bias;
  p.bias_stride[0] = a.bias_stride[0];
  p.bias_stride[1] = a.bias_stride[1];
  p.out = a.out;
  for (int i = 0; i < 3; ++i) {
    p.out_stride[i] = a.out_stride[i];
    p.epi_mul_stride[i] = a.epi_mul_stride[i];
    p.epi_out_stride[i] = a.epi_out_stride[i];
  }
  p.lse = a.lse;
  p.lse_stride[0] = a.lse_stride[0];
  p.lse_stride[1] = a.lse_stride[1];
  p.epi_mul = a.epi_mul;
  p.epi_out = a.epi_out;
  dim3 grid(a.batch * a.heads, p.m_tiles);
  pass_fwd_tc_kernel<D, T, HAS_BIAS, SOFTCLAMP><<<grid, kFwdThreads, L::kAlloc, s>>>(tq, tk, tv, p);
  note_launch(1);
  return cuda_status(cudaGetLastError(), "pass_fwd_tc launch");
}

template <int D, typename T>
int fwd_bias(const PolyPassArgs& a, cudaStream_t s) {
  if (a.softclamp > 0.f)
    return a.bias ? launch_fwd_tc_t<D, T, true, true>(a, s) : launch_fwd_tc_t<D, T, false, true>(a, s);
  return a.bias ? launch_fwd_tc_t<D, T, true, false>(a, s) : launch_fwd_tc_t<D, T, false, false>(a, s);
}

}  // namespace

bool pass_fwd_tc_eligible(const PolyPassArgs& a) {
  if (a.dtype != POLY_BF16 && a.dtype != POLY_F16) return false;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  if (a.key_mask || a.query_mask || a.v_mul) return false;
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.out)) return false;
  if (!strides_ok(a.q_stride, 3) || !strides_ok(a.k_stride, 3) || !strides_ok(a.v_stride, 3) ||
      !strides_ok(a.out_stride, 3))
    return false;
  if (a.epi_out && (!aligned16(a.epi_out) || !aligned16(a.epi_mul) || !strides_ok(a.epi_out_stride, 3) ||
                    !strides_ok(a.epi_mul_stride, 3)))
    return false;
  return true;
}

size_t pass_fwd_tc_workspace(const PolyPassArgs&) { return 0; }

int launch_pass_fwd_tc(const PolyPassArgs& a, cudaStream_t s) {
  if (pass_fwd_tc2_eligible(a)) return launch_pass_fwd_tc2(a, s);
  if (a.dtype == POLY_BF16)
    return a.head_dim == 64 ? fwd_bias<64, __nv_bfloat16>(a, s) : fwd_bias<128, __nv_bfloat16>(a, s);
  return a.head_dim == 64 ? fwd_bias<64, __half>(a, s) : fwd_bias<128, __half>(a, s);
}


}  // namespace poly
