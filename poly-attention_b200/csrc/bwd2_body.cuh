// Two-tile pipelined backward, opt-in with POLY_BWD_TWO_TILE=1 (included by
// bwd_tc100.cu inside its anonymous namespace; uses its BwdParams, helpers and
// error word). Measured slower than pass_bwd_tc_kernel at config 2: it exposes
// more TMEM-load latencies per tile with the same two softmax warps per
// scheduler; it is kept as the base for a version with more softmax warps.
//
// Same maths and grid as pass_bwd_tc_kernel, but two query tiles are in
// flight per CTA so that no hand-off is single-buffered. TMEM (512 columns):
//   R[x]  [128 x, +128)   S^T(t), then dP^T(t), of tile parity x = t & 1
//   PT[x] [256 + 64 x, +64) P^T(t) (16-bit pairs), then dQ(t) (fp32, lane = query)
//   dV [384, 448), dK [448, 512)
// MMA issuer, iteration t: S(t) -> R[t&1] once the softmax has taken dP(t-2)
// out of it; dP(t-1) -> R and dV += P^T(t-1) dO(t-1) once P^T(t-1) is
// written; dK += dS^T(t-2) Q(t-2) and dQ(t-2) -> PT once dS^T(t-2) is ready.
// Softmax step k (two warpgroups, 64 query columns each, thread = key row):
// S-phase(k): P(k) from S(k); stage dQ(k-2) out of PT (its own 32 columns,
// then TMA reduce-add); P^T(k) -> PT. dP-phase(k-1): dP(k-1) and P(k-1)
// (16-bit, re-read from PT) -> dS = P (dP - delta), d-bias, dS^T -> smem.
// Every wait then has about one softmax phase of slack. Q / lse2 / delta have
// 4 stages (a tile's Q is read by S(t) and dK(t), two iterations apart), dO 3.
// Softclamp (whose dS factor would have to cross phases) stays on
// pass_bwd_tc_kernel.

struct Bwd2Layout {
  static constexpr int kTile = 128 * D * 2;      // 16 KB: one [128][64] 16-bit tile
  static constexpr int kQS = 4, kDS = 3;         // Q (+ lse2, delta) stages, dO stages
  static constexpr int kK = 0;
  static constexpr int kV = kK + kTile;
  static constexpr int kQ = kV + kTile;
  static constexpr int kDO = kQ + kQS * kTile;
  static constexpr int kDST = kDO + kDS * kTile;  // dS^T [128 keys][128 queries], one buffer
  static constexpr int kDQS = kDST + 2 * kTile;   // dQ staging: 2 x [128 rows][32 fp32], swizzled
  static constexpr int kLse = kDQS + 2 * kTile;   // kQS x 128 floats
  static constexpr int kDel = kLse + kQS * BQ * 4;
  static constexpr int kDb = kDel + kQS * BQ * 4;  // d-bias partials of warpgroup 1
  static constexpr int kBar = kDb + BK * 4;
  static constexpr int kNumBars = 32;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kR = 0, kPT = 256, kDV = 384, kDK = 448;
};
static_assert(Bwd2Layout::kAlloc <= 232448, "two-tile backward exceeds shared memory");

// P of one 32-query chunk from S: p = 2^(s * scale * log2e + bias - lse2), 0
// where masked; packed 16-bit pairs (the P^T tile and the dP-phase input).
template <typename T, bool HAS_BIAS, bool MASK>
__device__ __forceinline__ void p_chunk(const uint32_t (&sv)[32], const float* nl, float b2, float sl2, bool key_ok,
                                        int il0, int diag_row, uint32_t (&pw)[16]) {
  const float4* l4 = reinterpret_cast<const float4*>(nl);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 lq = l4[q];
    const float lv[4] = {lq.x, lq.y, lq.z, lq.w};
    float pp[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int u = q * 4 + e;
      const float off = HAS_BIAS ? lv[e] + b2 : lv[e];
      float pr = ex2(fmaf(__uint_as_float(sv[u]), sl2, off));
      if (MASK && (!key_ok || il0 + u < diag_row)) pr = 0.f;
      pp[e] = pr;
    }
    pw[2 * q] = pk<T>(pp[0], pp[1]);
    pw[2 * q + 1] = pk<T>(pp[2], pp[3]);
  }
}

template <typename T>
__device__ __forceinline__ float2 unpk(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  else
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// dS of one 32-query chunk: ds = p (dp - delta), d-bias += ds, packed dS^T row.
template <typename T, bool DB>
__device__ __forceinline__ void ds_chunk(const uint32_t (&dv)[32], const uint32_t* pw, const float* dl,
                                         float& dbias, uint32_t (&dw)[16]) {
  const float4* d4 = reinterpret_cast<const float4*>(dl);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 dq = d4[q];
    const float2 p01 = unpk<T>(pw[2 * q]), p23 = unpk<T>(pw[2 * q + 1]);
    const float pp[4] = {p01.x, p01.y, p23.x, p23.y};
    const float dd[4] = {dq.x, dq.y, dq.z, dq.w};
    float ds[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ds[e] = pp[e] * (__uint_as_float(dv[q * 4 + e]) - dd[e]);
      if (DB) dbias += ds[e];
    }
    dw[2 * q] = pk<T>(ds[0], ds[1]);
    dw[2 * q + 1] = pk<T>(ds[2], ds[3]);
  }
}

__device__ __forceinline__ void tmem_ld16p(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <typename T, bool HAS_BIAS, bool DB>
__global__ void __launch_bounds__(kThreads, 1)
    pass_bwd_tc2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                        const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_dq, const BwdParams p) {
  using L = Bwd2Layout;
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
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;      // [kQS] Q, lse2, delta of a tile landed
  uint64_t* q_empty = bars + 5;     // [kQS] dK of that tile done (last reader)
  uint64_t* do_full = bars + 9;     // [kDS]
  uint64_t* do_empty = bars + 12;   // [kDS] dP and dV of that tile done
  uint64_t* s_full = bars + 15;     // [2] S(t) in R[x]
  uint64_t* s_taken = bars + 17;    // [2] softmax read S(t) and wrote P^T(t)        (256 arrivals)
  uint64_t* dp_full = bars + 19;    // [2] dP(t) in R[x], dV(t) done
  uint64_t* dp_taken = bars + 21;   // [2] softmax read dP(t) and P(t): R[x] free   (256 arrivals)
  uint64_t* ds_ready = bars + 23;   // dS^T(t) in smem                              (256 arrivals)
  uint64_t* dst_free = bars + 24;   // dK / dQ(t) done reading dS^T
  uint64_t* dq_full = bars + 25;    // [2] dQ(t) in PT[x]
  uint64_t* dkv_done = bars + 27;
  uint64_t* drain = bars + 28;
  uint32_t* tmem_slot = (uint32_t*)(smem + L::kMisc);
  volatile int* abort_flag = (volatile int*)(smem + L::kMisc + 4);
  int* err = &g_poly_device_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    for (int s = 0; s < L::kQS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int s = 0; s < L::kDS; ++s) {
      mbar_init(&do_full[s], 1);
      mbar_init(&do_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_taken[x], 256);
      mbar_init(&dp_full[x], 1);
      mbar_init(&dp_taken[x], 256);
      mbar_init(&dq_full[x], 1);
    }
    mbar_init(ds_ready, 256);
    mbar_init(dst_free, 1);
    mbar_init(dkv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
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

  if (warp == 0) {
    if (lane == 0 && NT > 0) {
      // ------------------------------------------------ TMA producer
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(kv_full, 2 * L::kTile);
      tma_load_4d(sK, &tm_k, kv_full, 0, kt * BK, kvh, b);
      tma_load_4d(sV, &tm_v, kv_full, 0, kt * BK, kvh, b);
      int issued_q = 0, issued_do = 0;
      for (int t = 0; t < NT; ++t) {
        int h, qt;
        tile_of(t, h, qt);
        const int qs = t % L::kQS, ds = t % L::kDS;
        if (t >= L::kQS && !mbar_wait(&q_empty[qs], ((t / L::kQS) - 1) & 1, abort_flag, err, 61)) break;
        const int64_t row = (int64_t)(b * p.heads + h) * p.nq_pad + qt * BQ;
        mbar_arrive_expect_tx(&q_full[qs], L::kTile + 2 * BQ * 4);
        tma_load_4d(sQ + qs * L::kTile, &tm_q, &q_full[qs], 0, qt * BQ, h, b);
        bulk_load(sLse + qs * BQ, p.lse2 + row, BQ * 4, &q_full[qs]);
        bulk_load(sDel + qs * BQ, p.delta + row, BQ * 4, &q_full[qs]);
        issued_q = t + 1;
        if (t >= L::kDS && !mbar_wait(&do_empty[ds], ((t / L::kDS) - 1) & 1, abort_flag, err, 62)) break;
        mbar_arrive_expect_tx(&do_full[ds], L::kTile);
        tma_load_4d(sDO + ds * L::kTile, &tm_do, &do_full[ds], 0, qt * BQ, h, b);
        issued_do = t + 1;
      }
      if (*abort_flag) {
        drain_wait(kv_full, 0);
        for (int t = max(0, issued_q - L::kQS); t < issued_q; ++t) drain_wait(&q_full[t % L::kQS], (t / L::kQS) & 1);
        for (int t = max(0, issued_do - L::kDS); t < issued_do; ++t)
          drain_wait(&do_full[t % L::kDS], (t / L::kDS) & 1);
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
      bool ok = mbar_wait(kv_full, 0, abort_flag, err, 63);
      for (int t = 0; ok && t < NT + 2; ++t) {
        if (t < NT) {   // S(t) -> R[t & 1]
          const int x = t & 1, qs = t % L::kQS;
          if (t >= 2 && !(ok = mbar_wait(&dp_taken[x], ((t - 2) >> 1) & 1, abort_flag, err, 64))) break;
          if (!(ok = mbar_wait(&q_full[qs], (t / L::kQS) & 1, abort_flag, err, 65))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_f16_ss(tmem + L::kR + x * 128, smem_desc_sw128(ka + kk * 32, 16, 1024),
                       smem_desc_sw128(qa + qs * L::kTile + kk * 32, 16, 1024), idSD, kk > 0);
          mma_commit(&s_full[x]);
        }
        if (t >= 1 && t - 1 < NT) {   // dP(u) -> R[u & 1], dV += P^T(u) dO(u)
          const int u = t - 1, x = u & 1, ds = u % L::kDS;
          if (!(ok = mbar_wait(&s_taken[x], (u >> 1) & 1, abort_flag, err, 66))) break;
          if (!(ok = mbar_wait(&do_full[ds], (u / L::kDS) & 1, abort_flag, err, 67))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_f16_ss(tmem + L::kR + x * 128, smem_desc_sw128(va + kk * 32, 16, 1024),
                       smem_desc_sw128(doa + ds * L::kTile + kk * 32, 16, 1024), idSD, kk > 0);
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            mma_f16_ts(tmem + L::kDV, tmem + L::kPT + x * 64 + kk * 8,
                       smem_desc_sw128(doa + ds * L::kTile + kk * 2048, 128 * 128, 1024), idKV, (u > 0 || kk > 0));
          mma_commit(&dp_full[x]);
          mma_commit(&do_empty[ds]);
        }
        if (t >= 2 && t - 2 < NT) {   // dK += dS^T(u) Q(u), dQ(u) -> PT[u & 1]
          const int u = t - 2, x = u & 1, qs = u % L::kQS;
          if (!(ok = mbar_wait(ds_ready, u & 1, abort_flag, err, 68))) break;
          // dV(u) read PT[x]; its completion is implied by dp_taken(u)
          if (!(ok = mbar_wait(&dp_taken[x], (u >> 1) & 1, abort_flag, err, 69))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {
            const uint32_t aoff = (uint32_t)(kk >> 2) * (128 * 128) + (uint32_t)(kk & 3) * 32;
            mma_f16_ss(tmem + L::kDK, smem_desc_sw128(dsa + aoff, 16, 1024),
                       smem_desc_sw128(qa + qs * L::kTile + kk * 2048, 128 * 128, 1024), idKV, (u > 0 || kk > 0));
          }
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16_ss(tmem + L::kPT + x * 64, smem_desc_sw128(dsa + kk * 2048, 128 * 128, 1024),
                       smem_desc_sw128(ka + kk * 2048, 128 * 128, 1024), idQ, kk > 0);
          mma_commit(&dq_full[x]);
          mma_commit(&q_empty[qs]);
          mma_commit(dst_free);
        }
      }
      mma_commit(dkv_done);
      mma_commit(drain);
      drain_wait(drain, 0);
    }
  } else if (warp >= 4 && warp < 12) {
    // -------------------------------------------------- softmax-backward
    const int hw = (warp - 4) >> 2;              // query columns [64 hw, 64 hw + 64)
    const int r = (warp & 3) * 32 + lane;         // key row / TMEM lane
    const int j = kt * BK + r;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const bool key_ok = j < p.seq_k;
    const bool key_ok_warp = __all_sync(0xffffffffu, key_ok);
    const bool leader = lane == 0 && (warp & 3) == 0;
    const int bar_and = 3 + 2 * hw, bar_sync = 2 + 2 * hw;   // named barriers of this warpgroup
    float b2 = 0.f;
    if (HAS_BIAS && key_ok) {
      const float braw = p.bias[b * p.bias_stride[0] + kvh * p.bias_stride[1] + j];
      b2 = braw <= kDeadBias ? -INFINITY : braw * kLog2e;
    }
    float dbias = 0.f;
    bool ok = true;
    // dQ(u) in PT[u & 1] (lane = query row): this warpgroup's 32 columns ->
    // swizzled fp32 smem -> one TMA reduce-add into the accumulator
    auto stage_dq = [&](int u) -> bool {
      int h, qt;
      tile_of(u, h, qt);
      const int x = u & 1;
      if (!named_bar_and(bar_and, 128, mbar_wait_warp(&dq_full[x], (u >> 1) & 1, abort_flag, err, 70))) return false;
      tc_fence_after();
      uint32_t a[32];
      tmem_ld32(tmem + lane_base + L::kPT + x * 64 + hw * 32, a);
      tmem_wait_ld();
      if (leader) bulk_wait_group_read0();      // this warpgroup's previous reduce has read its buffer
      named_bar_sync(bar_sync, 128);
      uint8_t* dst = sDQ + hw * (128 * 128);
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4) {
        const uint4 val = make_uint4(a[q4 * 4], a[q4 * 4 + 1], a[q4 * 4 + 2], a[q4 * 4 + 3]);
        *reinterpret_cast<uint4*>(dst + r * 128 + ((q4 ^ (r & 7)) << 4)) = val;
      }
      fence_proxy_async_smem();
      named_bar_sync(bar_sync, 128);
      if (leader) {
        tma_reduce_add_3d(&tm_dq, dst, hw * 32, qt * BQ, b * p.heads + h);
        bulk_commit_group();
      }
      return true;
    };

    for (int k = 0; k < NT + 1 && ok; ++k) {
      // ---------------- S-phase(k): P(k), stage dQ(k-2), P^T(k) -> PT
      if (k < NT) {
        const int x = k & 1, qs = k % L::kQS;
        int h, qt;
        tile_of(k, h, qt);
        const bool diag = p.causal && qt == kt;
        if (!mbar_wait_warp(&s_full[x], (k >> 1) & 1, abort_flag, err, 71)) { ok = false; break; }
        tc_fence_after();
        uint32_t pw[2][16];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = hw * 2 + cc;               // 32-query chunk
          uint32_t sv[32];
          tmem_ld32(tmem + lane_base + L::kR + x * 128 + c * 32, sv);
          tmem_wait_ld();
          const float* nl = sLse + qs * BQ + c * 32;
          if (diag || !key_ok_warp)
            p_chunk<T, HAS_BIAS, true>(sv, nl, b2, p.sl2, key_ok, c * 32, diag ? r : -1, pw[cc]);
          else
            p_chunk<T, HAS_BIAS, false>(sv, nl, b2, p.sl2, key_ok, c * 32, -1, pw[cc]);
        }
        if (k >= 2 && !stage_dq(k - 2)) { ok = false; break; }
        tmem_st16(tmem + lane_base + L::kPT + x * 64 + (hw * 2) * 16, pw[0]);
        tmem_st16(tmem + lane_base + L::kPT + x * 64 + (hw * 2 + 1) * 16, pw[1]);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&s_taken[x]);
      }
      // ---------------- dP-phase(k-1): dS = P (dP - delta) -> dS^T smem
      if (k >= 1 && k - 1 < NT) {
        const int u = k - 1, x = u & 1, qs = u % L::kQS;
        if (!mbar_wait_warp(&dp_full[x], (u >> 1) & 1, abort_flag, err, 72)) { ok = false; break; }
        tc_fence_after();
        uint32_t dv[2][32], pr[32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) tmem_ld32(tmem + lane_base + L::kR + x * 128 + (hw * 2 + cc) * 32, dv[cc]);
        tmem_ld32(tmem + lane_base + L::kPT + x * 64 + hw * 32, pr);   // P(u), 16-bit pairs
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&dp_taken[x]);
        uint32_t dw[2][16];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc)
          ds_chunk<T, DB>(dv[cc], pr + cc * 16, sDel + qs * BQ + (hw * 2 + cc) * 32, dbias, dw[cc]);
        if (u >= 1 && !mbar_wait_warp(dst_free, (u - 1) & 1, abort_flag, err, 73)) { ok = false; break; }
        store_chunk(sDST, r, hw * 2, dw[0]);
        store_chunk(sDST, r, hw * 2 + 1, dw[1]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(ds_ready);
      }
    }
    // the last two tiles' dQ
    for (int u = max(0, NT - 2); ok && u < NT; ++u)
      if (!stage_dq(u)) ok = false;
    if (leader) bulk_wait_group0();
    // dK (warpgroup 0) or dV (warpgroup 1) for this key row
    bool have = ok && NT > 0 && mbar_wait_warp(dkv_done, 0, abort_flag, err, 74);
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
  if (warp >= 4 && warp < 8 && p.dbias) {
    const int r = (warp & 3) * 32 + lane;
    const int j = kt * BK + r;
    if (j < p.seq_k) p.dbias[b * p.dbias_stride[0] + kvh * p.dbias_stride[1] + j] = dbias_part + sDb[r];
  }
}
