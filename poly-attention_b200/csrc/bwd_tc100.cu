// tcgen05 / TMEM / TMA backward kernel for one poly-attention pass (sm_100a),
// head_dim 64, bf16 / fp16. Replaces the Triton backward
// (poly_attention/flash_poly_attention.py:164-316), without its dQ atomics
// into the input dtype: dQ is reduced in fp32 and converted once.
//
// Key-stationary: one CTA owns 128 keys of one (batch, kv head) and walks
// every 128-query tile (of every query head of its GQA group) that sees them.
// Per query tile t:
//   S^T  = K Q_t^T        (M=128 keys, N=128 queries, K=64)   -> TMEM
//   dP^T = V dO_t^T                                          -> TMEM
//   two softmax warpgroups (thread = key row j, warpgroup hw takes query
//   columns [64 hw, 64 hw + 64)) load their whole slice of S^T and dP^T into
//   registers and release the two TMEM buffers at once, so S^T / dP^T of
//   tile t + 1 are computed while they work on tile t:
//     p = exp2(s*log2e*scale + bias_j - lse2_i), ds = p (dp - delta_i),
//     dbias_j += ds (a register: the column sum of dS needs no reduction),
//     P^T -> TMEM (16-bit), dS^T (x softclamp factor) -> 128B-swizzled smem
//   dV += P^T dO_t (TS MMA, A from TMEM), dK += dS^T Q_t  (TMEM accumulators)
//   dQ_t = dS K  (A = the same dS^T tile read MN-major)    -> TMEM
//   dQ_t staging by warpgroup 0 once it has handed tile t + 1 to the MMA:
//   TMEM -> swizzled fp32 smem -> TMA reduce-add into the fp32 accumulator
// A preprocessing kernel forms delta_i = dout_i . out_i - dlse_i and the
// log2-domain lse; a final kernel converts the fp32 dq accumulator.
#include <cstdlib>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"
#include "bwd_common.cuh"

namespace poly {

// Device error word of this file's kernels (see read_device_error_bwd).
static __device__ int g_poly_device_error[2] = {0, 0};

int read_device_error_bwd(int* out, bool reset) {
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

constexpr int D = 64;
constexpr int BK = 128;   // keys per CTA
constexpr int BQ = 128;   // queries per tile
constexpr int kThreads = 384;
constexpr int kHeadGroup = 8;
constexpr int kSelftestSite = 99;   // error-record site of wait_selftest_kernel

struct BwdLayout {
  static constexpr int kTile = 128 * D * 2;  // 16 KB: one [128][64] 16-bit tile
  static constexpr int kK = 0;
  static constexpr int kV = kK + kTile;
  static constexpr int kStages = 3;              // Q / dO / lse / delta stages
  static constexpr int kQ = kV + kTile;
  static constexpr int kDO = kQ + kStages * kTile;
  static constexpr int kDST = kDO + kStages * kTile;  // dS^T [128 keys][128 queries], read MN-major by dQ
  static constexpr int kDQS = kDST + 2 * kTile;  // dQ staging: 2 x [128 rows][32 fp32], swizzled
  static constexpr int kLse = kDQS + 2 * kTile;  // kStages x 128 floats
  static constexpr int kDel = kLse + kStages * BQ * 4;
  static constexpr int kDb = kDel + kStages * BQ * 4;   // d-bias partials of warpgroup 1
  static constexpr int kBar = kDb + BK * 4;
  static constexpr int kNumBars = 16;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  // P^T (16-bit, two queries per column) lives in TMEM as the A operand of dV += P^T dO
  static constexpr uint32_t kS = 0, kDP = 128, kDV = 256, kDK = 320, kDQ = 384, kPT = 448;
};

template <typename T, bool SOFTCLAMP, bool HAS_BIAS, bool DB>
__global__ void __launch_bounds__(kThreads, 1)
    pass_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_dq, const BwdParams p) {
  using L = BwdLayout;
  constexpr int kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
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
  constexpr int QS = L::kStages;
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;     // [QS]
  uint64_t* q_empty = bars + 4;    // [QS]
  uint64_t* sdp_full = bars + 7;   // S^T / dP^T of the tile are in TMEM
  uint64_t* sdp_free = bars + 8;   // ... and in the softmax threads' registers
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
  // head in group): heaviest key tiles first within a group (longest-first
  // dispatch), while the CTAs running together cover only a few heads, whose
  // Q / dO streams stay in L2.
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
  const int qt0 = p.causal ? kt : 0;
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

  // dQ of tile t: TMEM -> swizzled fp32 smem tile -> one TMA reduce-add into
  // the accumulator. Run by softmax warpgroup 0 (warps 4-7, all four TMEM lane
  // quarters) right after it has handed tile t + 1 to the MMA. Its cost is
  // latency (barriers, shared-memory stores competing with the MMAs' operand
  // reads, the TMA issue), not volume: splitting it over both warpgroups
  // measured slower. Returns false if a wait gave up; the decision is shared
  // by the warpgroup.
  auto stage_dq = [&](int t) -> bool {
    int h, qt;
    tile_of(t, h, qt);
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    if (!named_bar_and(3, 128, mbar_wait_warp(dq_full, t & 1, abort_flag, err, 10))) return false;
    tc_fence_after();
    uint32_t a[32], c2[32];
    tmem_ld32(tmem + lane_base + L::kDQ, a);
    tmem_ld32(tmem + lane_base + L::kDQ + 32, c2);
    tmem_wait_ld();
    tc_fence_before();
    mbar_arrive(dq_free);
    if (lane == 0 && warp == 4 && t > 0) bulk_wait_group_read0();
    named_bar_sync(2, 128);
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      const uint32_t* src = hb == 0 ? a : c2;
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4) {
        const uint4 val = make_uint4(src[q4 * 4], src[q4 * 4 + 1], src[q4 * 4 + 2], src[q4 * 4 + 3]);
        *reinterpret_cast<uint4*>(sDQ + hb * (128 * 128) + r * 128 + ((q4 ^ (r & 7)) << 4)) = val;
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(2, 128);
    if (lane == 0 && warp == 4) {
      const int plane = b * p.heads + h;
      tma_reduce_add_3d(&tm_dq, sDQ, 0, qt * BQ, plane);
      tma_reduce_add_3d(&tm_dq, sDQ + 128 * 128, 32, qt * BQ, plane);
      bulk_commit_group();
    }
    return true;
  };

  if (warp == 0) {
    if (lane == 0 && NT > 0) {
      // ------------------------------------------------ TMA producer
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(kv_full, 2 * L::kTile);
      tma_load_4d(sK, &tm_k, kv_full, 0, kt * BK, kvh, b);
      tma_load_4d(sV, &tm_v, kv_full, 0, kt * BK, kvh, b);
      int issued = 0;
      for (int t = 0; t < NT; ++t) {
        const int s = t % QS;
        if (t >= QS && !mbar_wait(&q_empty[s], ((t / QS) - 1) & 1, abort_flag, err, 1)) break;
        int h, qt;
        tile_of(t, h, qt);
        const int64_t row = (int64_t)(b * p.heads + h) * p.nq_pad + qt * BQ;
        mbar_arrive_expect_tx(&q_full[s], 2 * L::kTile + 2 * BQ * 4);
        tma_load_4d(sQ + s * L::kTile, &tm_q, &q_full[s], 0, qt * BQ, h, b);
        tma_load_4d(sDO + s * L::kTile, &tm_do, &q_full[s], 0, qt * BQ, h, b);
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
      constexpr uint32_t idSD = idesc_f16(128, 128, kIsBf16, 0, 0);   // K-major x K-major
      constexpr uint32_t idKV = idesc_f16(128, D, kIsBf16, 0, 1);     // P^T / dS^T  x  dO / Q (MN)
      constexpr uint32_t idQ = idesc_f16(128, D, kIsBf16, 1, 1);      // dS (MN view) x K (MN)
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV), qa = smem_u32(sQ), doa = smem_u32(sDO);
      const uint32_t dsa = smem_u32(sDST);
      auto issue_sdp = [&](int s) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          mma_f16_ss(tmem + L::kS, smem_desc_sw128(ka + kk * 32, 16, 1024),
                     smem_desc_sw128(qa + s * L::kTile + kk * 32, 16, 1024), idSD, kk > 0);
          mma_f16_ss(tmem + L::kDP, smem_desc_sw128(va + kk * 32, 16, 1024),
                     smem_desc_sw128(doa + s * L::kTile + kk * 32, 16, 1024), idSD, kk > 0);
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
          // S^T / dP^T of tile t are in the softmax threads' registers: the
          // buffers take tile t + 1 while the softmax still works on t
          if (!mbar_wait(sdp_free, t & 1, abort_flag, err, 11)) break;
          if (!mbar_wait(&q_full[(t + 1) % QS], ((t + 1) / QS) & 1, abort_flag, err, 5)) break;
          tc_fence_after();
          issue_sdp((t + 1) % QS);
        }
        if (!mbar_wait(p_ready, t & 1, abort_flag, err, 4)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t aoff = (uint32_t)(kk >> 2) * (128 * 128) + (uint32_t)(kk & 3) * 32;
          const uint32_t acc = (t > 0 || kk > 0);
          mma_f16_ts(tmem + L::kDV, tmem + L::kPT + kk * 8,
                     smem_desc_sw128(doa + s * L::kTile + kk * 2048, 128 * 128, 1024), idKV, acc);
          mma_f16_ss(tmem + L::kDK, smem_desc_sw128(dsa + aoff, 16, 1024),
                     smem_desc_sw128(qa + s * L::kTile + kk * 2048, 128 * 128, 1024), idKV, acc);
        }
        if (t >= 1 && !mbar_wait(dq_free, (t - 1) & 1, abort_flag, err, 6)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          mma_f16_ss(tmem + L::kDQ, smem_desc_sw128(dsa + kk * 2048, 128 * 128, 1024),
                     smem_desc_sw128(ka + kk * 2048, 128 * 128, 1024), idQ, kk > 0);
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
    // Two warpgroups: thread = key row r, warpgroup hw takes query columns
    // [64 hw, 64 hw + 64) of every tile.
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
      const bool diag = p.causal && qt == kt;
      // the whole 64-query slice of S^T and dP^T into registers, then the
      // TMEM buffers are released for tile t + 1
      uint32_t sv[2][32], dv[2][32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        tmem_ld32(tmem + lane_base + L::kS + (hw * 2 + cc) * 32, sv[cc]);
        tmem_ld32(tmem + lane_base + L::kDP + (hw * 2 + cc) * 32, dv[cc]);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(sdp_free);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = hw * 2 + cc;
        uint32_t pw[16], dw[16];
        const float* nl = sLse + s * BQ + c * 32;       // -lse2 of the chunk's queries
        const float* dl = sDel + s * BQ + c * 32;
        if (diag || !key_ok_warp)
          softmax_bwd_chunk<T, SOFTCLAMP, HAS_BIAS, true, DB>(sv[cc], dv[cc], nl, dl, b2, p, key_ok, c * 32,
                                                          diag ? r : -1, dbias, pw, dw);
        else
          softmax_bwd_chunk<T, SOFTCLAMP, HAS_BIAS, false, DB>(sv[cc], dv[cc], nl, dl, b2, p, key_ok, c * 32, -1,
                                                           dbias, pw, dw);
        // P^T (TMEM) / dS^T (smem) are free once the previous tile's MMAs completed
        if (cc == 0 && t > 0 && !mbar_wait_warp(mma_done, (t - 1) & 1, abort_flag, err, 8)) {
          ok = false;
          break;
        }
        tmem_st16(tmem + lane_base + L::kPT + c * 16, pw);   // queries c*32.. -> 16 packed columns
        store_chunk(sDST, r, c, dw);
      }
      if (!ok) break;
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_ready);
      if (hw == 0 && t > 0 && !stage_dq(t - 1)) { ok = false; break; }
    }
    if (hw == 0 && ok && NT > 0 && !stage_dq(NT - 1)) ok = false;
    if (hw == 0 && lane == 0 && warp == 4) bulk_wait_group0();
    // dK (warpgroup 0) or dV (warpgroup 1) for this key row. tcgen05.ld is
    // warp-collective: every lane runs it; only the stores depend on key_ok.
    bool have = ok && NT > 0 && mbar_wait_warp(dkv_done, 0, abort_flag, err, 9);
    if (have) tc_fence_after();
    if (have || NT == 0) {
      T* dst = hw == 0 ? (T*)p.dk + b * p.dk_stride[0] + kvh * p.dk_stride[1] + (int64_t)j * p.dk_stride[2]
                       : (T*)p.dv + b * p.dv_stride[0] + kvh * p.dv_stride[1] + (int64_t)j * p.dv_stride[2];
      const float mul = hw == 0 ? p.scale : 1.f;
      const uint32_t col = hw == 0 ? L::kDK : L::kDV;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t a[32];
        if (have) {
          tmem_ld32(tmem + lane_base + col + half * 32, a);
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
            *reinterpret_cast<uint4*>(dst + half * 32 + q8 * 8) = w4;
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
  // d-bias = sum of both warpgroups' partial column sums
  if (warp >= 4 && warp < 8 && p.dbias) {
    const int r = (warp & 3) * 32 + lane;
    const int j = kt * BK + r;
    if (j < p.seq_k) p.dbias[b * p.dbias_stride[0] + kvh * p.dbias_stride[1] + j] = dbias_part + sDb[r];
  }
}

template <typename T, bool SOFTCLAMP, bool HAS_BIAS, bool DB>
int launch_bwd_t(const PolyPassBwdArgs& a, cudaStream_t s) {
  using L = BwdLayout;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(pass_bwd_tc_kernel<T, SOFTCLAMP, HAS_BIAS, DB>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  });
  if (attr_err != cudaSuccess) return cuda_status(attr_err, "cudaFuncSetAttribute(bwd tc)");
  const PolyPassArgs& f = a.fwd;
  BwdWs w = bwd_ws<D, BQ>(a);
  CUtensorMap tq, tdo, tk, tv, tdq;
  int rc = make_map(&tq, f.q, f.dtype, D, f.seq_q, f.heads, f.batch, f.q_stride, BQ);
  if (!rc) rc = make_map(&tdo, a.dout, f.dtype, D, f.seq_q, f.heads, f.batch, a.dout_stride, BQ);
  if (!rc) rc = make_map(&tk, f.k, f.dtype, D, f.seq_k, f.kv_heads, f.batch, f.k_stride, BK);
  if (!rc) rc = make_map(&tv, f.v, f.dtype, D, f.seq_k, f.kv_heads, f.batch, f.v_stride, BK);
  if (!rc) rc = make_map_f32_acc(&tdq, w.dq_acc, f.seq_q, f.batch * f.heads);
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
  pass_bwd_tc_kernel<T, SOFTCLAMP, HAS_BIAS, DB><<<grid, kThreads, L::kAlloc, s>>>(tq, tdo, tk, tv, tdq, p);
  const int64_t cthreads = (int64_t)f.batch * f.heads * f.seq_q * (D / 8);
  bwd_dq_convert_kernel<T, D><<<(unsigned)((cthreads + 255) / 256), 256, 0, s>>>(a, w.dq_acc);
  note_launch(3);
  return cuda_status(cudaGetLastError(), "pass_bwd_tc launch");
}

template <typename T>
int bwd_dispatch(const PolyPassBwdArgs& a, cudaStream_t s) {
  const bool sc = a.fwd.softclamp > 0.f, bias = a.fwd.bias != nullptr, db = a.dbias != nullptr;
  if (db) {
    if (sc) return bias ? launch_bwd_t<T, true, true, true>(a, s) : launch_bwd_t<T, true, false, true>(a, s);
    return bias ? launch_bwd_t<T, false, true, true>(a, s) : launch_bwd_t<T, false, false, true>(a, s);
  }
  if (sc) return bias ? launch_bwd_t<T, true, true, false>(a, s) : launch_bwd_t<T, true, false, false>(a, s);
  return bias ? launch_bwd_t<T, false, true, false>(a, s) : launch_bwd_t<T, false, false, false>(a, s);
}

// Self-test of the bounded waits (poly_selftest_wait_timeout): one CTA holds
// TMEM like the pass kernels do, waits on an mbarrier that nothing arrives on,
// with a limit of limit_ns, and must give up through the same path as a real
// timeout: error record of this file, CTA abort flag, TMEM freed, return.
// result: 1 if the wait (wrongly) succeeded, 2 if it gave up.
__global__ void __launch_bounds__(64, 1) wait_selftest_kernel(uint64_t limit_ns, int* result) {
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  __shared__ int abort_state[2];
  int* err = g_poly_device_error;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_init(abort_state, err);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) tmem_alloc(&slot, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool ok = mbar_wait_warp(&bar, 0, abort_state, err, kSelftestSite, limit_ns);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(slot, 32);
  if (threadIdx.x == 0) *result = ok ? 1 : 2;
}

}  // namespace

int selftest_wait_timeout(uint64_t limit_ns, int* result, cudaStream_t s) {
  wait_selftest_kernel<<<1, 64, 0, s>>>(limit_ns, result);
  note_launch(1);
  return cuda_status(cudaGetLastError(), "wait_selftest_kernel launch");
}

bool pass_bwd_tc_eligible(const PolyPassBwdArgs& a) {
  const PolyPassArgs& f = a.fwd;
  if (f.dtype != POLY_BF16 && f.dtype != POLY_F16) return false;
  if (f.head_dim != D && f.head_dim != 128) return false;   // 128: bwd_tc128.cu
  if (f.key_mask || f.query_mask || f.v_mul) return false;
  if (!aligned16(f.q) || !aligned16(f.k) || !aligned16(f.v) || !aligned16(a.dout) || !aligned16(a.dq) ||
      !aligned16(a.dk) || !aligned16(a.dv) || !aligned16(f.out))
    return false;
  if (!strides_ok(f.q_stride, 3) || !strides_ok(f.k_stride, 3) || !strides_ok(f.v_stride, 3) ||
      !strides_ok(a.dout_stride, 3) || !strides_ok(a.dq_stride, 3) || !strides_ok(a.dk_stride, 3) ||
      !strides_ok(a.dv_stride, 3))
    return false;
  return true;
}

size_t pass_bwd_tc_workspace(const PolyPassBwdArgs& a) {
  return a.fwd.head_dim == 128 ? pass_bwd_tc128_workspace(a) : bwd_ws<D, BQ>(a).bytes;
}

int launch_pass_bwd_tc(const PolyPassBwdArgs& a, cudaStream_t s) {
  if (a.fwd.head_dim == 128) return launch_pass_bwd_tc128(a, s);
  return a.fwd.dtype == POLY_BF16 ? bwd_dispatch<__nv_bfloat16>(a, s) : bwd_dispatch<__half>(a, s);
}

}  // namespace poly
