// KV-cache append: up to POLY_MAX_ROW_COPIES strided row copies in one launch
// (16-byte vector moves). A decoding step appends one row to every key /
// value cache of the chain; one launch instead of one per cache.
#include <string>

#include "common.cuh"

namespace poly {
namespace {

struct RowCopies {
  PolyRowCopy c[POLY_MAX_ROW_COPIES];
};

__global__ void __launch_bounds__(256) copy_rows_kernel(const RowCopies rc) {
  const PolyRowCopy& c = rc.c[blockIdx.y];
  const int vec = c.row_bytes >> 4;                      // 16-byte chunks per row
  const int64_t total = (int64_t)c.outer * c.inner * vec;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / vec;
    const int v = (int)(e - row * vec);
    const int64_t o = row / c.inner, i = row - o * c.inner;
    const uint4* s = reinterpret_cast<const uint4*>((const char*)c.src + o * c.src_stride[0] + i * c.src_stride[1]);
    uint4* d = reinterpret_cast<uint4*>((char*)c.dst + o * c.dst_stride[0] + i * c.dst_stride[1]);
    d[v] = s[v];
  }
}

bool al16(int64_t x) { return (x & 15) == 0; }

int bad(const std::string& msg) {
  set_error(msg);
  return POLY_EINVAL;
}

}  // namespace

int copy_rows(const PolyRowCopy* copies, int n, cudaStream_t s) {
  if (n < 0 || n > POLY_MAX_ROW_COPIES || (n > 0 && !copies))
    return bad("poly_copy_rows: n must be in [0, 16] with a copies array");
  RowCopies rc;
  int64_t most = 0;
  for (int i = 0; i < n; ++i) {
    const PolyRowCopy& c = copies[i];
    if (c.outer < 0 || c.inner < 0 || c.row_bytes < 0)
      return bad("poly_copy_rows: negative extent in copy " + std::to_string(i));
    const int64_t rows = (int64_t)c.outer * c.inner;
    if (rows && c.row_bytes &&
        (!c.src || !c.dst || !al16((int64_t)(uintptr_t)c.src) || !al16((int64_t)(uintptr_t)c.dst) ||
         !al16(c.row_bytes) || !al16(c.src_stride[0]) || !al16(c.src_stride[1]) || !al16(c.dst_stride[0]) ||
         !al16(c.dst_stride[1])))
      return bad("poly_copy_rows: copy " + std::to_string(i) + " needs 16-byte aligned pointers, strides and row_bytes");
    rc.c[i] = c;
    const int64_t chunks = rows * (c.row_bytes / 16);
    if (chunks > most) most = chunks;
  }
  if (n == 0 || most == 0) return POLY_OK;
  const int64_t want = (most + 255) / 256;
  const int blocks = (int)(want < 1184 ? want : 1184);
  copy_rows_kernel<<<dim3(blocks, n), 256, 0, s>>>(rc);
  note_launch(1);
  return cuda_status(cudaGetLastError(), "copy_rows launch");
}

}  // namespace poly
