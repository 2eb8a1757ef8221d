// Merge of key-split partial passes: the exchange step of the long-context
// sequence split. Each partial p holds (out_p, lse_p) for the same query rows
// over a disjoint key shard; the merged row is the softmax-weighted sum.
#include "common.cuh"

namespace poly {
namespace {

template <typename T>
__global__ void lse_merge_kernel(const PolyMergeArgs a) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.rows) return;
  float m = -INFINITY;
  for (int p = 0; p < a.parts; ++p) m = fmaxf(m, a.part_lse[(int64_t)p * a.rows + row]);
  float w_sum = 0.f;
  for (int p = 0; p < a.parts; ++p) {
    const float l = a.part_lse[(int64_t)p * a.rows + row];
    w_sum += (m == -INFINITY) ? 0.f : exp2f((l - m) * kLog2e);
  }
  const T* po = (const T*)a.part_out;
  for (int c = lane; c < a.head_dim; c += 32) {
    float acc = 0.f;
    for (int p = 0; p < a.parts; ++p) {
      const float l = a.part_lse[(int64_t)p * a.rows + row];
      const float w = (m == -INFINITY) ? 0.f : exp2f((l - m) * kLog2e);
      acc += w * to_f32(po[((int64_t)p * a.rows + row) * a.head_dim + c]);
    }
    ((T*)a.out)[row * a.head_dim + c] = from_f32<T>(w_sum > 0.f ? acc / w_sum : 0.f);
  }
  if (a.lse && lane == 0) a.lse[row] = (w_sum > 0.f) ? m + logf(w_sum) : -INFINITY;
}

}  // namespace

int launch_lse_merge(const PolyMergeArgs& a, cudaStream_t s) {
  const int warps = 8;
  const unsigned grid = (unsigned)((a.rows + warps - 1) / warps);
  switch (a.dtype) {
    case POLY_F32: lse_merge_kernel<float><<<grid, warps * 32, 0, s>>>(a); break;
    case POLY_F16: lse_merge_kernel<__half><<<grid, warps * 32, 0, s>>>(a); break;
    default: lse_merge_kernel<__nv_bfloat16><<<grid, warps * 32, 0, s>>>(a); break;
  }
  note_launch();
  return cuda_status(cudaGetLastError(), "lse_merge launch");
}

}  // namespace poly
