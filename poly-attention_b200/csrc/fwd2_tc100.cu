// tcgen05 forward pass, head_dim 64 or 128, two 128-query tiles per CTA (sm_100a).
//
// Same maths as pass_fwd_tc_kernel (pass_tc100.cu), organised so the tensor
// core never waits on one softmax warpgroup: a CTA owns query rows
// [256 m, 256 m + 256) of one (batch, head) as tiles A and B, each with its own
// softmax warpgroup, S buffer, P buffer and O accumulator, sharing the K / V
// (and per-key bias) stages. Each warpgroup releases its S buffer as soon as
// the tile is in registers, so S(j+1) is computed while it exponentiates S(j).
//
// Warps: 0 TMA producer, 1 TMEM allocator + MMA issuer, 4-7 softmax A,
// 8-11 softmax B. TMEM columns: S_A [0,128), S_B [128,256), O_A [256,320),
// O_B [320,384), P_A [384,448), P_B [448,512). P (16-bit, two per column)
// stays in TMEM and is the A operand of the P V MMA, so no probability tile
// crosses shared memory (shared-memory operand bandwidth bounds SS MMAs).
#include <algorithm>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace poly {

static __device__ int g_poly_device_error[2] = {0, 0};

int read_device_error_fwd2(int* out, bool reset) {
  int rc = cuda_status(cudaMemcpyFromSymbol(out, g_poly_device_error, sizeof(int)), "read device error word");
  if (rc == POLY_OK && reset) {
    const int zero = 0;
    rc = cuda_status(cudaMemcpyToSymbol(g_poly_device_error, &zero, sizeof(int)), "reset device error word");
  }
  return rc;
}

namespace {
using namespace tc;

constexpr int BM = 128;   // rows per tile (two tiles per CTA)
constexpr int BN = 128;   // keys per stage
constexpr int kThreads = 384;

// D = 64: 3 K / V stages, P in its own TMEM columns. D = 128: 2 stages, P
// written over the first 64 columns of its own S buffer (TMEM holds S_A, S_B,
// O_A, O_B at 128 columns each), so S(j + 1) is issued after P V(j).
template <int D>
struct L2T {
  static constexpr int S = D == 64 ? 3 : 2;
  static constexpr int kTile = 128 * D * 2;   // one [128][D] 16-bit tile (D / 64 swizzle atoms)
  static constexpr int kQ = 0;                // 2 tiles
  static constexpr int kK = kQ + 2 * kTile;   // S stages
  static constexpr int kV = kK + S * kTile;
  static constexpr int kB = kV + S * kTile;   // S x 128 fp32 bias
  static constexpr int kBar = kB + S * BN * 4;
  static constexpr int kNumBars = 1 + 3 * S + 2 * 4 + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
};

struct Fwd2Params {
  int seq_q, seq_k, heads, kv_heads, m_tiles, causal;
  int off_tiles;      // causal offset in 128-key tiles
  int n_bh, grp_bh;   // batch * heads; (batch, head) units per dispatch group
  float sl2, scale;
  void* out; int64_t out_stride[3];
  float* lse; int64_t lse_stride[2];
  const void* epi_mul; int64_t epi_mul_stride[3];
  void* epi_out; int64_t epi_out_stride[3];
};

template <typename T>
__device__ __forceinline__ uint32_t pk2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pk2<__nv_bfloat16>(float a, float b) { return pack_bf16(a, b); }
template <>
__device__ __forceinline__ uint32_t pk2<__half>(float a, float b) { return pack_f16(a, b); }

template <typename T>
__device__ __forceinline__ float2 up2(uint32_t u);
template <>
__device__ __forceinline__ float2 up2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}
template <>
__device__ __forceinline__ float2 up2<__half>(uint32_t u) { return __half22float2(*reinterpret_cast<__half2*>(&u)); }

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitNs) return;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

template <typename T, bool HAS_BIAS, int D>
__global__ void __launch_bounds__(kThreads, 1)
    pass_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_b,
                        const Fwd2Params p) {
  using L2 = L2T<D>;
  constexpr int S = L2::S;
  constexpr bool kAlias = D == 128;   // P over the first half of its S buffer
  constexpr int kAtom = 128 * 128;     // bytes of one 64-column swizzle atom of a 128-row tile
  constexpr int kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem + L2::kQ;
  uint8_t* sK = smem + L2::kK;
  uint8_t* sV = smem + L2::kV;
  float* sB = (float*)(smem + L2::kB);
  uint64_t* bars = (uint64_t*)(smem + L2::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 1 + S;
  uint64_t* kv_empty = bars + 1 + 2 * S;
  uint64_t* s_full = bars + 1 + 3 * S;    // [2]
  uint64_t* s_free = bars + 3 + 3 * S;    // [2]
  uint64_t* p_full = bars + 5 + 3 * S;    // [2]
  uint64_t* o_done = bars + 7 + 3 * S;    // [2]
  uint64_t* drain = bars + 9 + 3 * S;
  uint32_t* tmem_slot = (uint32_t*)(smem + L2::kMisc);
  volatile int* abort_flag = (volatile int*)(smem + L2::kMisc + 4);
  int* err = g_poly_device_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid over groups of grp_bh consecutive (batch, head) units (whole GQA
  // groups, sized so their K / V stay in L2 together); inside a group the
  // query-tile pairs go heaviest (most key tiles) first, every unit of the
  // group at one pair index before the next, so the dispatch is
  // longest-first while the CTAs in flight share few K / V streams
  int bh, yi;
  {
    const int lin = blockIdx.x;
    const int grp = lin / (p.grp_bh * p.m_tiles);
    const int gsz = min(p.grp_bh, p.n_bh - grp * p.grp_bh);
    const int rem = lin - grp * p.grp_bh * p.m_tiles;
    yi = rem / gsz;
    bh = grp * p.grp_bh + (rem - yi * gsz);
  }
  const int b = bh / p.heads, h = bh - b * p.heads;
  const int kvh = h / (p.heads / p.kv_heads);
  const int mt = p.causal ? (p.m_tiles - 1 - yi) : yi;
  const int row0 = mt * 2 * BM;
  const int kt_total = (p.seq_k + BN - 1) / BN;
  // key tiles seen by tile A (rows row0..) and tile B (rows row0 + 128..)
  const int ntA = p.causal ? min(kt_total, 2 * mt + 1 + p.off_tiles) : kt_total;
  const int ntB = p.causal ? min(kt_total, 2 * mt + 2 + p.off_tiles) : kt_total;
  const int ntMax = ntB;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], 128);
      mbar_init(&p_full[x], 128);
      mbar_init(&o_done[x], 1);
    }
    mbar_init(drain, 1);
    tc::abort_init(abort_flag, err);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, L2::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      mbar_arrive_expect_tx(q_full, 2 * L2::kTile);
#pragma unroll
      for (int hf = 0; hf < D / 64; ++hf) {
        tma_load_4d(sQ + hf * kAtom, &tm_q, q_full, hf * 64, row0, h, b);
        tma_load_4d(sQ + L2::kTile + hf * kAtom, &tm_q, q_full, hf * 64, row0 + BM, h, b);
      }
      int issued = 0;
      for (int j = 0; j < ntMax; ++j) {
        const int s = j % S;
        if (j >= S && !mbar_wait(&kv_empty[s], ((j / S) - 1) & 1, abort_flag, err, 41)) break;
        mbar_arrive_expect_tx(&k_full[s], L2::kTile + (HAS_BIAS ? BN * 4 : 0));
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf)
          tma_load_4d(sK + s * L2::kTile + hf * kAtom, &tm_k, &k_full[s], hf * 64, j * BN, kvh, b);
        if (HAS_BIAS) tma_load_3d(sB + s * BN, &tm_b, &k_full[s], j * BN, kvh, b);
        mbar_arrive_expect_tx(&v_full[s], L2::kTile);
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf)
          tma_load_4d(sV + s * L2::kTile + hf * kAtom, &tm_v, &v_full[s], hf * 64, j * BN, kvh, b);
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
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK), va = smem_u32(sV);
      auto issue_s = [&](int x, int j) {
        const int s = j % S;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (uint32_t)(kk >> 2) * kAtom + (uint32_t)(kk & 3) * 32;
          mma_f16_ss(tmem + x * BN, smem_desc_sw128(qa + x * L2::kTile + koff, 16, 1024),
                     smem_desc_sw128(ka + s * L2::kTile + koff, 16, 1024), idS, kk > 0);
        }
        mma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {
        const int s = j % S;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_f16_ts(tmem + 256 + x * D, tmem + (kAlias ? x * BN : 384 + x * 64) + kk * 8,
                     smem_desc_sw128(va + s * L2::kTile + kk * 2048, BN * 128, 1024), idO, (j > 0 || kk > 0));
        mma_commit(&o_done[x]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, err, 42) && mbar_wait(&k_full[0], 0, abort_flag, err, 43);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int j = 0; ok && j < ntMax; ++j) {
        const int s = j % S;
        const bool next_k = j + 1 < ntMax;
        if (next_k) {
          ok = mbar_wait(&k_full[(j + 1) % S], ((j + 1) / S) & 1, abort_flag, err, 44);
          if (!ok) break;
        }
        bool v_ok = false;
        for (int x = 0; x < 2; ++x) {
          const int nt = x == 0 ? ntA : ntB;
          if (j >= nt) continue;
          if (!kAlias && j + 1 < nt) {
            if (!(ok = mbar_wait(&s_free[x], j & 1, abort_flag, err, 45))) break;
            tc_fence_after();
            issue_s(x, j + 1);
          }
          if (!(ok = mbar_wait(&p_full[x], j & 1, abort_flag, err, 46))) break;
          if (!v_ok) {
            if (!(ok = mbar_wait(&v_full[s], (j / S) & 1, abort_flag, err, 47))) break;
            v_ok = true;
          }
          tc_fence_after();
          issue_pv(x, j);
          // aliased P: S(j + 1) overwrites P(j); MMAs of one issuer run in order,
          // so P V(j) has read P before S(j + 1) writes those columns
          if (kAlias && j + 1 < nt) issue_s(x, j + 1);
        }
        if (!ok) break;
        mma_commit(&kv_empty[s]);
      }
      mma_commit(drain);
      drain_wait(drain, 0);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------- softmax (thread = query row)
    const int x = (warp - 4) >> 2;                // tile A or B
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int nt = x == 0 ? ntA : ntB;
    const int diag_tile = 2 * mt + x + p.off_tiles;  // causal: the key tile on this tile's diagonal
    const uint32_t s_addr = tmem + lane_base + x * BN;
    const uint32_t o_addr = tmem + lane_base + 256 + x * D;
    const uint32_t p_addr = tmem + lane_base + (kAlias ? x * BN : 384 + x * 64);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int s = j % S;
      if (HAS_BIAS && !mbar_wait_warp(&k_full[s], (j / S) & 1, abort_flag, err, 48)) { ok = false; break; }
      if (!mbar_wait_warp(&s_full[x], j & 1, abort_flag, err, 49)) { ok = false; break; }
      tc_fence_after();
      uint32_t v[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tmem_wait_ld();
      if (!kAlias) {
        tc_fence_before();
        mbar_arrive(&s_free[x]);                // S is in registers: the MMA may overwrite it
      }
      const bool tail = (j == kt_total - 1) && (p.seq_k % BN) != 0;
      const bool diag = p.causal && (j == diag_tile);
      float tmax = -INFINITY;
      // Without a bias the row max is taken on the raw scores and the scale is
      // folded into the exponent's FFMA; with a bias x = s * scale + b (natural
      // units, one FFMA) is formed first and log2(e) folded into the exponent's
      // FFMA instead. Both end with v[] holding values whose 2^(v*mul - m) is
      // the unnormalised probability.
      float mul = p.sl2;
      if (HAS_BIAS) {
        mul = kLog2e;
        const float4* b4 = reinterpret_cast<const float4*>(sB + s * BN);
#pragma unroll
        for (int q = 0; q < BN / 4; ++q) {
          const float4 bb = b4[q];
          v[4 * q + 0] = __float_as_uint(fmaf(__uint_as_float(v[4 * q + 0]), p.scale, bb.x));
          v[4 * q + 1] = __float_as_uint(fmaf(__uint_as_float(v[4 * q + 1]), p.scale, bb.y));
          v[4 * q + 2] = __float_as_uint(fmaf(__uint_as_float(v[4 * q + 2]), p.scale, bb.z));
          v[4 * q + 3] = __float_as_uint(fmaf(__uint_as_float(v[4 * q + 3]), p.scale, bb.w));
        }
      }
      if (tail) {
        const int kvalid = p.seq_k - j * BN;
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c >= kvalid) v[c] = __float_as_uint(-INFINITY);
      }
      if (diag) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c > r) v[c] = __float_as_uint(-INFINITY);
      }
      {
        float mx[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) mx[u] = __uint_as_float(v[u]);
#pragma unroll
        for (int c = 4; c < BN; ++c) mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(v[c]));
        tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * mul;
      }
      // Lazy rescaling: the reference max only moves when the row max grows
      // by more than 2^8 (log2 domain), so P <= 256 and O is rarely rescaled;
      // lse = m_run + log2(l) stays exact.
      const bool grow = tmax > m_run + 8.f;
      const float m_new = grow ? tmax : m_run;
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2(m_run - m_use);
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float e0 = ex2(fmaf(__uint_as_float(v[c]), mul, -m_use));
        const float e1 = ex2(fmaf(__uint_as_float(v[c + 1]), mul, -m_use));
        sum0 += e0;
        sum1 += e1;
        v[c >> 1] = pk2<T>(e0, e1);              // packed P overwrites the consumed half
      }
      l_run = l_run * alpha + (sum0 + sum1);
      m_run = m_new;
      if (j > 0) {
        if (!mbar_wait_warp(&o_done[x], (j - 1) & 1, abort_flag, err, 50)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
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
      // packed P (64 columns of bf16x2) -> TMEM, the A operand of P V
      tmem_st32(p_addr, *reinterpret_cast<const uint32_t(*)[32]>(&v[0]));
      tmem_st32(p_addr + 32, *reinterpret_cast<const uint32_t(*)[32]>(&v[32]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    if (ok && nt > 0 && mbar_wait_warp(&o_done[x], (nt - 1) & 1, abort_flag, err, 51)) {
      tc_fence_after();
      const int row = row0 + x * BM + r;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T* out = (T*)p.out + b * p.out_stride[0] + h * p.out_stride[1] + (int64_t)row * p.out_stride[2];
      const T* em = p.epi_out ? (const T*)p.epi_mul + b * p.epi_mul_stride[0] + h * p.epi_mul_stride[1] +
                                    (int64_t)row * p.epi_mul_stride[2]
                              : nullptr;
      T* eo = p.epi_out ? (T*)p.epi_out + b * p.epi_out_stride[0] + h * p.epi_out_stride[1] +
                              (int64_t)row * p.epi_out_stride[2]
                        : nullptr;
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
              w[t] = pk2<T>(__uint_as_float(o[q4 * 8 + 2 * t]) * inv, __uint_as_float(o[q4 * 8 + 2 * t + 1]) * inv);
            *reinterpret_cast<uint4*>(out + c * 32 + q4 * 8) = val;
            if (eo) {
              const uint4 mv = *reinterpret_cast<const uint4*>(em + c * 32 + q4 * 8);
              const uint32_t* mw = &mv.x;
              uint4 ev;
              uint32_t* ew = &ev.x;
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const float2 a2 = up2<T>(w[t]), m2 = up2<T>(mw[t]);
                ew[t] = pk2<T>(a2.x * m2.x, a2.y * m2.y);
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
  if (warp == 1) tmem_dealloc(tmem, L2::kTmemCols);
}

template <typename T, bool HAS_BIAS, int D>
int launch_t(const PolyPassArgs& a, cudaStream_t st) {
  using L2 = L2T<D>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(pass_fwd_tc2_kernel<T, HAS_BIAS, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    L2::kAlloc);
  });
  if (attr_err != cudaSuccess) return cuda_status(attr_err, "cudaFuncSetAttribute(fwd tc2)");
  CUtensorMap tq, tk, tv, tb;
  int rc = make_map(&tq, a.q, a.dtype, D, a.seq_q, a.heads, a.batch, a.q_stride, BM);
  if (!rc) rc = make_map(&tk, a.k, a.dtype, D, a.seq_k, a.kv_heads, a.batch, a.k_stride, BN);
  if (!rc) rc = make_map(&tv, a.v, a.dtype, D, a.seq_k, a.kv_heads, a.batch, a.v_stride, BN);
  if (rc) return rc;
  memset(&tb, 0, sizeof(tb));
  if (HAS_BIAS) {
    EncodeTiledFn fn = encode_fn();
    const cuuint64_t dims[3] = {(cuuint64_t)a.seq_k, (cuuint64_t)a.kv_heads, (cuuint64_t)a.batch};
    const cuuint64_t strides[2] = {(cuuint64_t)a.bias_stride[1] * 4, (cuuint64_t)a.bias_stride[0] * 4};
    const cuuint32_t box[3] = {BN, 1, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(a.bias), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled (bias) failed (" + std::to_string((int)r) + ")");
      return POLY_ECUDA;
    }
  }
  Fwd2Params p{};
  p.seq_q = a.seq_q;
  p.seq_k = a.seq_k;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.m_tiles = (a.seq_q + 2 * BM - 1) / (2 * BM);
  p.causal = a.causal;
  p.off_tiles = a.causal ? a.causal_offset / BN : 0;
  p.sl2 = a.scale * kLog2e;
  p.scale = a.scale;
  p.out = a.out;
  p.lse = a.lse;
  p.epi_mul = a.epi_mul;
  p.epi_out = a.epi_out;
  for (int i = 0; i < 3; ++i) {
    p.out_stride[i] = a.out_stride[i];
    p.epi_mul_stride[i] = a.epi_mul_stride[i];
    p.epi_out_stride[i] = a.epi_out_stride[i];
  }
  p.lse_stride[0] = a.lse_stride[0];
  p.lse_stride[1] = a.lse_stride[1];
  // dispatch groups: whole GQA groups whose K / V (2 x seq_k x D x 2 bytes per
  // kv head) fit in ~32 MB of L2
  const int rep_h = a.heads / a.kv_heads;
  const size_t kv_bytes = (size_t)a.seq_k * D * 4;
  const int grp_kv = (int)std::max<size_t>(1, (32u << 20) / std::max<size_t>(kv_bytes, 1));
  p.n_bh = a.batch * a.heads;
  p.grp_bh = std::min(p.n_bh, grp_kv * rep_h);
  dim3 grid((unsigned)(p.n_bh * p.m_tiles));
  pass_fwd_tc2_kernel<T, HAS_BIAS, D><<<grid, kThreads, L2::kAlloc, st>>>(tq, tk, tv, tb, p);
  note_launch(1);
  return cuda_status(cudaGetLastError(), "pass_fwd_tc2 launch");
}

}  // namespace

// d = 64 or 128, no softclamp (the two-tile kernel keeps 128 scores per
// thread in registers; softclamp's tanh goes to the one-tile kernel), bias
// rows usable by TMA (16-byte aligned base and strides).
bool pass_fwd_tc2_eligible(const PolyPassArgs& a) {
  if ((a.head_dim != 64 && a.head_dim != 128) || a.softclamp > 0.f) return false;
  if (a.bias && (!aligned16(a.bias) || (a.bias_stride[0] & 3) || (a.bias_stride[1] & 3) || a.bias_stride[0] <= 0 ||
                 a.bias_stride[1] <= 0))
    return false;
  return true;
}

namespace {
template <int D>
int launch_d(const PolyPassArgs& a, cudaStream_t s) {
  if (a.dtype == POLY_BF16)
    return a.bias ? launch_t<__nv_bfloat16, true, D>(a, s) : launch_t<__nv_bfloat16, false, D>(a, s);
  return a.bias ? launch_t<__half, true, D>(a, s) : launch_t<__half, false, D>(a, s);
}
}  // namespace

int launch_pass_fwd_tc2(const PolyPassArgs& a, cudaStream_t s) {
  return a.head_dim == 128 ? launch_d<128>(a, s) : launch_d<64>(a, s);
}

}  // namespace poly
