// tcgen05 / TMEM / TMA backward kernel for one poly-attention pass (sm_100a),
// head_dim 128, bf16 / fp16 (the order-n modules' head size at config 4).
// Replaces the Triton backward (poly_attention/flash_poly_attention.py:164-316)
// for d = 128, where the head_dim-64 kernel's TMEM layout does not fit.
//
// Key-stationary like bwd_tc100.cu: one CTA owns 128 keys of one (batch, kv
// head) and walks the query tiles, here 64 queries each. Per tile t:
//   S^T  = K Q_t^T   (M 128 keys, N 64 queries, K 128)        -> TMEM
//   dP^T = V dO_t^T                                           -> TMEM
//   two softmax warpgroups (thread = key row, warpgroup hw takes queries
//   [32 hw, 32 hw + 32)) load their slice into registers and release both
//   TMEM buffers at once, so S^T / dP^T of tile t + 1 run while they work:
//     P^T -> TMEM (16-bit), dS^T -> 128B-swizzled smem, d-bias in a register
//   dV += P^T dO_t   (TS MMA, N = 128)     dK += dS^T Q_t   (SS, N = 128)
//   dQ_t^T = K^T dS^T (M = d = 128 feature rows, N = 64 queries): the dQ
//   accumulator is transposed in TMEM (thread = feature) because a 64-row
//   M would need a different TMEM lane layout; warpgroup 0 writes it to a
//   swizzled fp32 smem tile in the accumulator's [query][feature] layout and
//   reduces it with four 32-feature TMA reduce-adds.
// TMEM (512 columns): S^T 0, dP^T 64, dV 128, dK 256, dQ^T 384, P^T 448.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>
#include <type_traits>

#include "bwd_common.cuh"
#include "common.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace poly {

// Device error record of this file's kernel (reported with the backward's).
static __device__ int g_poly_device_error[2] = {0, 0};

int read_device_error_bwd128(int* out, bool reset) {
  int rc = cuda_status(cudaMemcpyFromSymbol(out, g_poly_device_error, sizeof(int)), "read device error word");
  if (rc == POLY_OK && reset) {
    const int zero = 0;
    rc = cuda_status(cudaMemcpyToSymbol(g_poly_device_error, &zero, sizeof(int)), "reset device error word");
  }
  return rc;
}

namespace {
using namespace tc;
using namespace bwdc;

constexpr int D = 128;
constexpr int BK = 128;   // keys per CTA
constexpr int BQ = 64;    // queries per tile
constexpr int kThreads = 384;
constexpr int kHeadGroup = 8;

struct Layout {
  static constexpr int kKTile = BK * D * 2;       // 32 KB: [128 keys][128 d], two 64-feature atoms
  static constexpr int kKAtom = BK * 128;         // 16 KB
  static constexpr int kQTile = BQ * D * 2;       // 16 KB: [64 queries][128 d], two atoms
  static constexpr int kQAtom = BQ * 128;         // 8 KB
  static constexpr int kStages = 3;               // Q / dO / lse / delta stages
  static constexpr int kK = 0;
  static constexpr int kV = kK + kKTile;
  static constexpr int kQ = kV + kKTile;
  static constexpr int kDO = kQ + kStages * kQTile;
  static constexpr int kDST = kDO + kStages * kQTile;   // dS^T [128 keys][64 queries], one atom
  static constexpr int kDQS = kDST + BK * 128;           // dQ staging: 4 x [64 queries][32 fp32]
  static constexpr int kDQBox = BQ * 128;                 // 8 KB per 32-feature box
  static constexpr int kLse = kDQS + 4 * kDQBox;
  static constexpr int kDel = kLse + kStages * BQ * 4;
  static constexpr int kDb = kDel + kStages * BQ * 4;
  static constexpr int kBar = kDb + BK * 4;
  static constexpr int kNumBars = 16;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kS = 0, kDP = 64, kDV = 128, kDK = 256, kDQT = 384, kPT = 448;
};

template <typename T, bool SOFTCLAMP, bool HAS_BIAS, bool DB>
__global__ void __launch_bounds__(kThreads, 1)
    pass_bwd_tc128_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_dq, const BwdParams p) {
  using L = Layout;
  constexpr int kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr int QS = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sDO = smem + L::kDO;
  uint8_t* sDST = smem + L::kDST;
  uint8_t* sDQ = smem + L::kDQS;
  float* sLse = (float*)(smem + L::kLse);
  float* sDel = (float*)(smem + L::kDel);
  float* sDb = (float*)(smem + L::kDb);
  float dbias_part = 0.f;
  uint64_t* bars = (uint64_t*)(smem + L::kBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;     // [QS]
  uint64_t* q_empty = bars + 4;    // [QS]
  uint64_t* sdp_full = bars + 7;
  uint64_t* sdp_free = bars + 8;
  uint64_t* p_ready = bars + 9;
  uint64_t* mma_done = bars + 10;
  uint64_t* dq_full = bars + 11;
  uint64_t* dq_free = bars + 12;
  uint64_t* dkv_done = bars + 13;
  uint64_t* drain = bars + 14;
  uint32_t* tmem_slot = (uint32_t*)(smem + L::kMisc);
  volatile int* abort_flag = (volatile int*)(smem + L::kMisc + 4);
  int* err = g_poly_device_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid over (head group of kHeadGroup (batch, kv head)s, key tile,
  // head in group): heaviest key tiles first within a group.
  int kt, bh;
  {
    const int nkt = p.k_tiles, nbh = gridDim.x / p.k_tiles;
    const int lin = blockIdx.x;
    const int grp = lin / (kHeadGroup * nkt);
    const int gsz = min(kHeadGroup, nbh - grp * kHeadGroup);
    const int rem = lin - grp * kHeadGroup * nkt;
    kt = rem / gsz;
    bh = grp * kHeadGroup + (rem - kt * gsz);
  }
  const int b = bh / p.kv_heads, kvh = bh - b * p.kv_heads;
  const int rep = p.heads / p.kv_heads;
  const int qt0 = p.causal ? kt * (BK / BQ) : 0;     // the first query tile that sees these keys
  const int nqt = max(0, p.q_tiles - qt0);
  const int NT = rep * nqt;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < QS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(sdp_full, 1);
    mbar_init(sdp_free, 256);
    mbar_init(p_ready, 256);
    mbar_init(mma_done, 1);
    mbar_init(dkv_done, 1);
    mbar_init(drain, 1);
    tc::abort_init(abort_flag, err);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto tile_of = [&](int t, int& h, int& qt) {
    const int hr = t / max(nqt, 1);
    qt = qt0 + (t - hr * nqt);
    h = kvh * rep + hr;
  };

  // dQ of tile t: TMEM (transposed: lane = feature, column = query) ->
  // swizzled fp32 smem in the accumulator's [query][feature] layout, four
  // boxes of 32 features -> four TMA reduce-adds. Run by softmax warpgroup 0
  // after it has handed tile t + 1 to the MMA. Returns false if a wait gave
  // up; the decision is shared by the warpgroup.
  auto stage_dq = [&](int t) -> bool {
    int h, qt;
    tile_of(t, h, qt);
    const int f = (warp & 3) * 32 + lane;                  // this thread's feature
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    if (!named_bar_and(3, 128, mbar_wait_warp(dq_full, t & 1, abort_flag, err, 10))) return false;
    tc_fence_after();
    uint32_t a[32], c2[32];
    tmem_ld32(tmem + lane_base + L::kDQT, a);
    tmem_ld32(tmem + lane_base + L::kDQT + 32, c2);
    tmem_wait_ld();
    tc_fence_before();
    mbar_arrive(dq_free);
    if (lane == 0 && warp == 4 && t > 0) bulk_wait_group_read0();
    named_bar_sync(2, 128);
    // feature f lives in box f / 32, float column f % 32 of each query row;
    // one warp writes one 128-byte row per store (conflict-free)
    uint8_t* box = sDQ + (f >> 5) * L::kDQBox;
    const int col = f & 31, chunk = col >> 2, within = (col & 3) * 4;
#pragma unroll
    for (int q = 0; q < BQ; ++q) {
      const uint32_t v = q < 32 ? a[q] : c2[q - 32];
      *reinterpret_cast<uint32_t*>(box + q * 128 + ((chunk ^ (q & 7)) << 4) + within) = v;
    }
    fence_proxy_async_smem();
    named_bar_sync(2, 128);
    if (lane == 0 && warp == 4) {
      const int plane = b * p.heads + h;
#pragma unroll
      for (int bx = 0; bx < 4; ++bx) tma_reduce_add_3d(&tm_dq, sDQ + bx * L::kDQBox, bx * 32, qt * BQ, plane);
      bulk_commit_group();
    }
    return true;
  };

  if (warp == 0) {
    if (lane == 0 && NT > 0) {
      // ------------------------------------------------ TMA producer
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(kv_full, 2 * L::kKTile);
#pragma unroll
      for (int at = 0; at < 2; ++at) {
        tma_load_4d(sK + at * L::kKAtom, &tm_k, kv_full, at * 64, kt * BK, kvh, b);
        tma_load_4d(sV + at * L::kKAtom, &tm_v, kv_full, at * 64, kt * BK, kvh, b);
      }
      int issued = 0;
      for (int t = 0; t < NT; ++t) {
        const int s = t % QS;
        if (t >= QS && !mbar_wait(&q_empty[s], ((t / QS) - 1) & 1, abort_flag, err, 1)) break;
        int h, qt;
        tile_of(t, h, qt);
        const int64_t row = (int64_t)(b * p.heads + h) * p.nq_pad + qt * BQ;
        mbar_arrive_expect_tx(&q_full[s], 2 * L::kQTile + 2 * BQ * 4);
#pragma unroll
        for (int at = 0; at < 2; ++at) {
          tma_load_4d(sQ + s * L::kQTile + at * L::kQAtom, &tm_q, &q_full[s], at * 64, qt * BQ, h, b);
          tma_load_4d(sDO + s * L::kQTile + at * L::kQAtom, &tm_do, &q_full[s], at * 64, qt * BQ, h, b);
        }
        bulk_load(sLse + s * BQ, p.lse2 + row, BQ * 4, &q_full[s]);
        bulk_load(sDel + s * BQ, p.delta + row, BQ * 4, &q_full[s]);
        issued = t + 1;
      }
      if (*abort_flag) {
        drain_wait(kv_full, 0);
        for (int t = max(0, issued - QS); t < issued; ++t) drain_wait(&q_full[t % QS], (t / QS) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && NT > 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idSD = idesc_f16(128, BQ, kIsBf16, 0, 0);    // K x Q^T, both K-major
      constexpr uint32_t idKV = idesc_f16(128, D, kIsBf16, 0, 1);     // P^T / dS^T x dO / Q (MN)
      constexpr uint32_t idQT = idesc_f16(128, BQ, kIsBf16, 1, 1);    // K^T (MN) x dS^T (MN)
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV), qa = smem_u32(sQ), doa = smem_u32(sDO);
      const uint32_t dsa = smem_u32(sDST);
      auto issue_sdp = [&](int s) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t ko = (uint32_t)(kk >> 2) * L::kKAtom + (uint32_t)(kk & 3) * 32;
          const uint32_t qo = (uint32_t)(s * L::kQTile) + (uint32_t)(kk >> 2) * L::kQAtom + (uint32_t)(kk & 3) * 32;
          mma_f16_ss(tmem + L::kS, smem_desc_sw128(ka + ko, 16, 1024), smem_desc_sw128(qa + qo, 16, 1024), idSD,
                     kk > 0);
          mma_f16_ss(tmem + L::kDP, smem_desc_sw128(va + ko, 16, 1024), smem_desc_sw128(doa + qo, 16, 1024), idSD,
                     kk > 0);
        }
        mma_commit(sdp_full);
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, err, 2) && mbar_wait(&q_full[0], 0, abort_flag, err, 3);
      if (ok) {
        tc_fence_after();
        issue_sdp(0);
      }
      for (int t = 0; ok && t < NT; ++t) {
        const int s = t % QS;
        if (t + 1 < NT) {
          if (!mbar_wait(sdp_free, t & 1, abort_flag, err, 11)) break;
          if (!mbar_wait(&q_full[(t + 1) % QS], ((t + 1) / QS) & 1, abort_flag, err, 5)) break;
          tc_fence_after();
          issue_sdp((t + 1) % QS);
        }
        if (!mbar_wait(p_ready, t & 1, abort_flag, err, 4)) break;
        tc_fence_after();
        // dV += P^T dO, dK += dS^T Q: K = 64 queries in 4 steps; dO / Q are
        // the MN-major B operand, N = 128 features over two 8 KB atoms
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t acc = (t > 0 || kk > 0);
          const uint32_t bo = (uint32_t)(s * L::kQTile) + (uint32_t)kk * 2048;
          mma_f16_ts(tmem + L::kDV, tmem + L::kPT + kk * 8, smem_desc_sw128(doa + bo, L::kQAtom, 1024), idKV, acc);
          mma_f16_ss(tmem + L::kDK, smem_desc_sw128(dsa + kk * 32, 16, 1024), smem_desc_sw128(qa + bo, L::kQAtom, 1024),
                     idKV, acc);
        }
        if (t >= 1 && !mbar_wait(dq_free, (t - 1) & 1, abort_flag, err, 6)) break;
        tc_fence_after();
        // dQ^T = K^T dS^T: M = 128 features (MN-major K, two 16 KB atoms), K =
        // 128 keys in 8 steps, N = 64 queries (dS^T read MN-major)
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          mma_f16_ss(tmem + L::kDQT, smem_desc_sw128(ka + kk * 2048, L::kKAtom, 1024),
                     smem_desc_sw128(dsa + kk * 2048, L::kKAtom, 1024), idQT, kk > 0);
        }
        mma_commit(&q_empty[s]);
        mma_commit(mma_done);
        mma_commit(dq_full);
      }
      mma_commit(dkv_done);
      mma_commit(drain);
      drain_wait(drain, 0);
    }
  } else if (warp >= 4 && warp < 12) {
    // -------------------------------------------------- softmax-backward
    const int hw = (warp - 4) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const int j = kt * BK + r;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const bool key_ok = j < p.seq_k;
    const bool key_ok_warp = __all_sync(0xffffffffu, key_ok);
    float b2 = 0.f;
    if (HAS_BIAS && key_ok) {
      const float braw = p.bias[b * p.bias_stride[0] + kvh * p.bias_stride[1] + j];
      b2 = braw <= kDeadBias ? -INFINITY : braw * kLog2e;
    }
    float dbias = 0.f;
    bool ok = true;
    for (int t = 0; t < NT && ok; ++t) {
      const int s = t % QS;
      int h, qt;
      tile_of(t, h, qt);
      if (!mbar_wait_warp(sdp_full, t & 1, abort_flag, err, 7)) { ok = false; break; }
      tc_fence_after();
      // causal: query il of this tile sees key j iff qt * 64 + il >= j
      const int diag_row = p.causal ? kt * BK + r - qt * BQ : -1;
      const bool mask = (p.causal && qt * BQ < kt * BK + BK) || !key_ok_warp;
      uint32_t sv[32], dv[32];
      tmem_ld32(tmem + lane_base + L::kS + hw * 32, sv);
      tmem_ld32(tmem + lane_base + L::kDP + hw * 32, dv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(sdp_free);
      uint32_t pw[16], dw[16];
      const float* nl = sLse + s * BQ + hw * 32;
      const float* dl = sDel + s * BQ + hw * 32;
      if (mask)
        softmax_bwd_chunk<T, SOFTCLAMP, HAS_BIAS, true, DB>(sv, dv, nl, dl, b2, p, key_ok, hw * 32, diag_row, dbias,
                                                        pw, dw);
      else
        softmax_bwd_chunk<T, SOFTCLAMP, HAS_BIAS, false, DB>(sv, dv, nl, dl, b2, p, key_ok, hw * 32, -1, dbias, pw,
                                                         dw);
      if (t > 0 && !mbar_wait_warp(mma_done, (t - 1) & 1, abort_flag, err, 8)) { ok = false; break; }
      tmem_st16(tmem + lane_base + L::kPT + hw * 16, pw);
      store_chunk(sDST, r, hw, dw);
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_ready);
      if (hw == 0 && t > 0 && !stage_dq(t - 1)) { ok = false; break; }
    }
    if (hw == 0 && ok && NT > 0 && !stage_dq(NT - 1)) ok = false;
    if (hw == 0 && lane == 0 && warp == 4) bulk_wait_group0();
    // dK (warpgroup 0) or dV (warpgroup 1): 128 feature columns of this key row
    bool have = ok && NT > 0 && mbar_wait_warp(dkv_done, 0, abort_flag, err, 9);
    if (have) tc_fence_after();
    if (have || NT == 0) {
      T* dst = hw == 0 ? (T*)p.dk + b * p.dk_stride[0] + kvh * p.dk_stride[1] + (int64_t)j * p.dk_stride[2]
                       : (T*)p.dv + b * p.dv_stride[0] + kvh * p.dv_stride[1] + (int64_t)j * p.dv_stride[2];
      const float mul = hw == 0 ? p.scale : 1.f;
      const uint32_t col = hw == 0 ? L::kDK : L::kDV;
#pragma unroll 1
      for (int part = 0; part < D / 32; ++part) {
        uint32_t a[32];
        if (have) {
          tmem_ld32(tmem + lane_base + col + part * 32, a);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int u = 0; u < 32; ++u) a[u] = 0u;
        }
        if (key_ok) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 w4;
            uint32_t* wp = &w4.x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int u = q8 * 8 + 2 * e;
              wp[e] = pk<T>(__uint_as_float(a[u]) * mul, __uint_as_float(a[u + 1]) * mul);
            }
            *reinterpret_cast<uint4*>(dst + part * 32 + q8 * 8) = w4;
          }
        }
      }
    }
    if (hw == 1) sDb[r] = dbias;
    dbias_part = dbias;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, L::kTmemCols);
  if (warp >= 4 && warp < 8 && p.dbias) {
    const int r = (warp & 3) * 32 + lane;
    const int j = kt * BK + r;
    if (j < p.seq_k) p.dbias[b * p.dbias_stride[0] + kvh * p.dbias_stride[1] + j] = dbias_part + sDb[r];
  }
}

template <typename T, bool SOFTCLAMP, bool HAS_BIAS, bool DB>
int launch_t(const PolyPassBwdArgs& a, cudaStream_t s) {
  using L = Layout;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(pass_bwd_tc128_kernel<T, SOFTCLAMP, HAS_BIAS, DB>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  });
  if (attr_err != cudaSuccess) return cuda_status(attr_err, "cudaFuncSetAttribute(bwd tc128)");
  const PolyPassArgs& f = a.fwd;
  BwdWs w = bwd_ws<D, BQ>(a);
  CUtensorMap tq, tdo, tk, tv, tdq;
  int rc = make_map(&tq, f.q, f.dtype, D, f.seq_q, f.heads, f.batch, f.q_stride, BQ);
  if (!rc) rc = make_map(&tdo, a.dout, f.dtype, D, f.seq_q, f.heads, f.batch, a.dout_stride, BQ);
  if (!rc) rc = make_map(&tk, f.k, f.dtype, D, f.seq_k, f.kv_heads, f.batch, f.k_stride, BK);
  if (!rc) rc = make_map(&tv, f.v, f.dtype, D, f.seq_k, f.kv_heads, f.batch, f.v_stride, BK);
  if (!rc) rc = make_map_f32_acc(&tdq, w.dq_acc, f.seq_q, f.batch * f.heads, D, BQ);
  if (rc) return rc;
  rc = cuda_status(cudaMemsetAsync(w.dq_acc, 0, (size_t)f.batch * f.heads * f.seq_q * D * 4, s), "memset dq acc");
  if (rc) return rc;
  const int64_t prow = (int64_t)f.batch * f.heads * w.nq_pad;
  bwd_prep_kernel<T, D><<<(unsigned)((prow * 8 + 255) / 256), 256, 0, s>>>(a, w.lse2, w.delta, w.nq_pad);
  BwdParams p{};
  p.seq_q = f.seq_q;
  p.seq_k = f.seq_k;
  p.heads = f.heads;
  p.kv_heads = f.kv_heads;
  p.nq_pad = w.nq_pad;
  p.q_tiles = w.nq_pad / BQ;
  p.causal = f.causal;
  p.scale = f.scale;
  p.sl2 = f.scale * kLog2e;
  p.sc_in = f.softclamp > 0.f ? f.scale / f.softclamp : 0.f;
  p.sc_out = f.softclamp * kLog2e;
  p.bias = f.bias;
  p.bias_stride[0] = f.bias_stride[0];
  p.bias_stride[1] = f.bias_stride[1];
  p.dq_acc = w.dq_acc;
  p.lse2 = w.lse2;
  p.delta = w.delta;
  p.dk = a.dk;
  p.dv = a.dv;
  for (int i = 0; i < 3; ++i) {
    p.dk_stride[i] = a.dk_stride[i];
    p.dv_stride[i] = a.dv_stride[i];
  }
  p.dbias = a.dbias;
  p.dbias_stride[0] = a.dbias_stride[0];
  p.dbias_stride[1] = a.dbias_stride[1];
  p.k_tiles = (f.seq_k + BK - 1) / BK;
  dim3 grid(p.k_tiles * f.batch * f.kv_heads);
  pass_bwd_tc128_kernel<T, SOFTCLAMP, HAS_BIAS, DB><<<grid, kThreads, L::kAlloc, s>>>(tq, tdo, tk, tv, tdq, p);
  const int64_t cthreads = (int64_t)f.batch * f.heads * f.seq_q * (D / 8);
  bwd_dq_convert_kernel<T, D><<<(unsigned)((cthreads + 255) / 256), 256, 0, s>>>(a, w.dq_acc);
  note_launch(3);
  return cuda_status(cudaGetLastError(), "pass_bwd_tc128 launch");
}

template <typename T>
int dispatch(const PolyPassBwdArgs& a, cudaStream_t s) {
  const bool sc = a.fwd.softclamp > 0.f, bias = a.fwd.bias != nullptr, db = a.dbias != nullptr;
  if (db) {
    if (sc) return bias ? launch_t<T, true, true, true>(a, s) : launch_t<T, true, false, true>(a, s);
    return bias ? launch_t<T, false, true, true>(a, s) : launch_t<T, false, false, true>(a, s);
  }
  if (sc) return bias ? launch_t<T, true, true, false>(a, s) : launch_t<T, true, false, false>(a, s);
  return bias ? launch_t<T, false, true, false>(a, s) : launch_t<T, false, false, false>(a, s);
}

}  // namespace

size_t pass_bwd_tc128_workspace(const PolyPassBwdArgs& a) { return bwd_ws<D, BQ>(a).bytes; }

int launch_pass_bwd_tc128(const PolyPassBwdArgs& a, cudaStream_t s) {
  return a.fwd.dtype == POLY_BF16 ? dispatch<__nv_bfloat16>(a, s) : dispatch<__half>(a, s);
}

}  // namespace poly
