// Shared helpers for the poly-attention kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cfloat>
#include <string>

#include "poly_attention.h"

namespace poly {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// A key whose additive bias is at or below this is "dead": the reference adds
// a -finfo.max log-sum-exp there, which no finite score can lift back.
constexpr float kDeadBias = -FLT_MAX * 0.5f;

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Thread-local error message for poly_last_error().
void set_error(const std::string& msg);

// Counts kernel launches made by this library (poly_launch_count()).
void note_launch(int n = 1);

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return POLY_OK;
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return POLY_ECUDA;
}

// Launchers implemented in the individual .cu files.
int launch_pass_fwd_simt(const PolyPassArgs& a, cudaStream_t s);
int launch_pass_bwd_simt(const PolyPassBwdArgs& a, cudaStream_t s);
int launch_lse_merge(const PolyMergeArgs& a, cudaStream_t s);

bool pass_fwd_tc_eligible(const PolyPassArgs& a);
int launch_pass_fwd_tc(const PolyPassArgs& a, cudaStream_t s);
size_t pass_fwd_tc_workspace(const PolyPassArgs& a);

bool pass_bwd_tc_eligible(const PolyPassBwdArgs& a);
int launch_pass_bwd_tc(const PolyPassBwdArgs& a, cudaStream_t s);
size_t pass_bwd_tc_workspace(const PolyPassBwdArgs& a);

int read_device_error_fwd(int* out, bool reset);
int read_device_error_bwd(int* out, bool reset);
int read_device_error_fwd2(int* out, bool reset);
int read_device_error_dec(int* out, bool reset);
int read_device_error_bwd128(int* out, bool reset);
size_t pass_bwd_tc128_workspace(const PolyPassBwdArgs& a);
int launch_pass_bwd_tc128(const PolyPassBwdArgs& a, cudaStream_t s);
int selftest_wait_timeout(uint64_t limit_ns, int* result, cudaStream_t s);
bool pass_fwd_tc2_eligible(const PolyPassArgs& a);
int launch_pass_fwd_tc2(const PolyPassArgs& a, cudaStream_t s);

bool pass_f32_eligible(const PolyPassArgs& a);
int launch_pass_f32(const PolyPassArgs& a, cudaStream_t s);
bool pass_small_eligible(const PolyPassArgs& a);
int launch_pass_small(const PolyPassArgs& a, cudaStream_t s);
bool pass_decode_eligible(const PolyPassArgs& a);
int launch_pass_decode(const PolyPassArgs& a, cudaStream_t s, bool dependent = false);
size_t pass_decode_workspace(const PolyPassArgs& a);
int copy_rows(const PolyRowCopy* copies, int n, cudaStream_t s);
int head_rmsnorm(const PolyHeadNorm* norms, int n, cudaStream_t s);

}  // namespace poly
